/*
 * qwen_tts_cuda_b200.h -- the drop-in replacement surface for the reference's
 * GPU-resident decode path.
 *
 * Every function below keeps the exact name and signature of the reference's
 * extern "C" entry point it replaces (file:line of the reference given per
 * declaration), so a reference build links this library instead of
 * qwen_tts_cuda_talker.cu without touching its callers
 * (qwen_tts_talker.c:531-565, qwen_tts_code_predictor.c:725-761, qwen_tts.c:
 * 1460-1475 / 2423-2731, main.c:1568-1594).
 *
 * Conventions kept from the reference:
 *   - ownership: a single-stream state owns its device weights; batch states
 *     share them and never free them (qwen_tts_cuda_talker.cu:601-605, 647);
 *   - the step functions return void; a failure is printed to stderr (as the
 *     reference's CK() does, qwen_tts_cuda_talker.cu:36) and additionally
 *     recorded for qwen_cuda_last_error();
 *   - precision is chosen per state from the non-NULL quantized pointers,
 *     q4_0 > int8 > bf16 (qwen_tts_cuda_talker.cu:308-311).
 *
 * Additions (no counterpart in the reference's CUDA TU): qwen_cuda_last_error,
 * qwen_cuda_cp_frame (the device-resident code-predictor frame modelled on the
 * reference's Metal qwen_metal_cp_frame, qwen_tts_code_predictor.c:931-940),
 * and qwen_cuda_talker_batch_set_pages (paged KV for the batched state).
 *
 * The ctx-reading entry points (qwen_cuda_talker_init, qwen_cuda_cp_init,
 * qwen_cuda_talker_upload_kv, qwen_cuda_batch_selftest) live in
 * libqwen_tts_cuda_b200.so, which is compiled against the reference's own
 * qwen_tts.h; everything else lives in libqwen3tts_b200.so.
 */
#ifndef QWEN_TTS_CUDA_B200_H
#define QWEN_TTS_CUDA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct qwen_tts_ctx;

/* ---- talker, single stream ---------------------------------------------- */
/* replaces qwen_tts_cuda_talker.cu:313 (decl qwen_tts_cuda.h:144) */
void *qwen_cuda_talker_init(struct qwen_tts_ctx *ctx);
/* replaces qwen_tts_cuda_talker.cu:395 (decl qwen_tts_cuda.h:145) */
void  qwen_cuda_talker_step(void *state, const float *embed, float *hidden_out, int pos);
/* replaces qwen_tts_cuda_talker.cu:419 */
void  qwen_cuda_talker_get_dec_x(void *state, float *out);
/* replaces qwen_tts_cuda_talker.cu:424 */
void  qwen_cuda_talker_upload_kv(void *state, struct qwen_tts_ctx *ctx, int prefill_len);
/* replaces qwen_tts_cuda_talker.cu:933 (decl qwen_tts_cuda.h:146) */
void  qwen_cuda_talker_free(void *state);

/* ---- talker, batched (the reference caps B at 8; this library at 64) ------ */
/* replaces qwen_tts_cuda_talker.cu:595 */
void *qwen_cuda_talker_batch_init(void *single, int B);
/* replaces qwen_tts_cuda_talker.cu:618 */
void  qwen_cuda_talker_batch_step(void *state, const float *embeds, const int *pos_arr, float *hidden_out);
/* replaces qwen_tts_cuda_talker.cu:629 */
void  qwen_cuda_talker_batch_upload_slot(void *state, int b, const uint16_t *kv_k, const uint16_t *kv_v,
                                         int src_kv_max, int prefill_len);
/* replaces qwen_tts_cuda_talker.cu:643 */
void  qwen_cuda_talker_batch_free(void *state);

/* ---- code predictor ------------------------------------------------------- */
/* replaces qwen_tts_cuda_talker.cu:751 */
void *qwen_cuda_cp_init(struct qwen_tts_ctx *ctx);
/* replaces qwen_tts_cuda_talker.cu:824 */
void  qwen_cuda_cp_step(void *state, float *x, int pos);
/* replaces qwen_tts_cuda_talker.cu:917 */
void  qwen_cuda_cp_free(void *state);
/* replaces qwen_tts_cuda_talker.cu:879 */
void *qwen_cuda_cp_batch_init(void *single, int B);
/* replaces qwen_tts_cuda_talker.cu:902 */
void  qwen_cuda_cp_batch_step(void *state, float *x, const int *pos_arr);
/* replaces qwen_tts_cuda_talker.cu:910 */
void  qwen_cuda_cp_batch_free(void *state);

/* replaces qwen_tts_cuda_talker.cu:657 */
int   qwen_cuda_batch_selftest(struct qwen_tts_ctx *ctx, int B, int frames);

/* ---- per-op backend (the CUDA entries of the backend vtable,
 * qwen_tts_backend.h:34-49): host bf16 W [rows][cols], host f32 x [cols] /
 * X [cols][B] (row-major), y [rows] / Y [rows][B]; B <= 64.  Each weight is
 * uploaded once and kept resident, cached by its host pointer (as in the
 * reference); the device is QWEN_CUDA_DEVICE (default 0). */
/* replaces qwen_tts_cuda.c:67 (decl qwen_tts_cuda.h:23) */
int   qwen_cuda_available(void);
/* replaces qwen_tts_cuda.c:73 (decl qwen_tts_cuda.h:24) */
void *qwen_cuda_init(void);
/* replaces qwen_tts_cuda.c:84 (decl qwen_tts_cuda.h:25) */
void  qwen_cuda_free(void *ctx);
/* replaces qwen_tts_cuda.c:138 (decl qwen_tts_cuda.h:28) */
void  qwen_cuda_matvec_bf16(void *ctx, float *y, const uint16_t *W, const float *x, int rows, int cols);
/* replaces qwen_tts_cuda.c:119 (decl qwen_tts_cuda.h:33) */
void  qwen_cuda_matmat_bf16(void *ctx, float *Y, const uint16_t *W, const float *X, int rows, int cols, int B);

/* ---- additions -------------------------------------------------------------- */
/* Last failure of any entry point above on this thread: 0 or a QTB_E_* code;
 * qtb_last_error() (qwen3tts_b200.h) has the message. */
int   qwen_cuda_last_error(void);
/* Whole code-predictor frame on the device (16 passes, 15 greedy lm_heads, the
 * embedding feedback): talker_hidden [hidden], code0, out_codes [15].  Same
 * result contract as qwen_cp_predict (qwen_tts_code_predictor.c:926-1045) with
 * greedy heads.  Works on single (B=1) and batched CP states (then
 * talker_hidden is [B][hidden], code0/out_codes point at B / B*15 ints).
 * Returns 0 or a QTB_E_* code. */
int   qwen_cuda_cp_frame(void *state, const float *talker_hidden, const int *code0, int *out_codes);
/* Page table for slot b of a batched talker state (pages of 16 positions from
 * the state's pool).  Returns 0 or a QTB_E_* code. */
int   qwen_cuda_talker_batch_set_pages(void *state, int b, const int32_t *pages, int n);

/* ---- glue used by libqwen_tts_cuda_b200.so ----------------------------------- */
struct qtb_engine;
struct qtb_session;
/* Wrap an engine + session as a reference-compatible state.  kind: 0 talker,
 * 1 code predictor.  owns_engine: free the engine with the state. */
void *qtb_ref_wrap(struct qtb_engine *e, struct qtb_session *s, int kind, int owns_engine);
struct qtb_session *qtb_ref_session(void *state);
void  qtb_ref_set_error(int code);

#ifdef __cplusplus
}
#endif
#endif
