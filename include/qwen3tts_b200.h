/*
 * qwen3tts_b200.h -- C ABI of the B200 (sm_100a) decode engine for the
 * Qwen3-TTS talker and code predictor.
 *
 * Plain pointers and sizes only.  Host pointers are read during the call and
 * never retained; every weight is copied to the device (and repacked into the
 * engine's tensor-core fragment order) at create time.
 *
 * Two layers of entry points live in this library:
 *
 *  1. The drop-in symbols of the reference's GPU backend, with the reference's
 *     exact signatures (declared in qwen_tts_cuda_b200.h, which replaces the
 *     extern "C" surface of qwen_tts_cuda_talker.cu / qwen_tts_cuda.h).
 *  2. The engine API below (qtb_*), which those symbols are built on and which
 *     a host that does not link the reference's qwen_tts_ctx_t can call
 *     directly.
 *
 * Every qtb_* function returns 0 on success or a negative QTB_E_* code and
 * records a message retrievable with qtb_last_error() (thread-local).
 */
#ifndef QWEN3TTS_B200_H
#define QWEN3TTS_B200_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    QTB_OK = 0,
    QTB_E_INVALID = -1,   /* bad argument / shape / position out of range */
    QTB_E_CUDA = -2,      /* a CUDA runtime call failed */
    QTB_E_OOM = -3,       /* device allocation failed */
    QTB_E_DEVICE = -4,    /* the decode kernel raised its error flag (bounded wait
                             expired or an index failed its device-side check) */
    QTB_E_UNSUPPORTED = -5
};

/* Weight storage formats.  One format per transformer (the reference picks one
 * precision per state, qwen_tts_cuda_talker.cu:308-311). */
enum {
    QTB_FMT_BF16 = 0,   /* uint16 bf16 bits [rows][cols]                                 */
    QTB_FMT_INT8 = 1,   /* int8 [rows][cols] + f32 row_scale[rows] (qwen_tts_kernels.c:2143) */
    QTB_FMT_Q4_0 = 2,   /* the reference's q4_0 blocks, 18 B / 32 weights
                           (qwen_tts_kernels.h:207-210)                                 */
    QTB_FMT_INT4G32 = 3 /* asymmetric int4, group 32 along cols: codes [rows][cols/2]
                           (low nibble = even col), fp16 scale and fp16 zero
                           [rows][cols/32]; w = (q - zero) * scale                      */
};

/* One weight matrix as the host holds it (row-major, rows x cols). */
typedef struct {
    const void *data;            /* format-dependent, see QTB_FMT_*         */
    const float *row_scale;      /* QTB_FMT_INT8 only                       */
    const uint16_t *group_scale; /* QTB_FMT_INT4G32 only (fp16 bits)        */
    const uint16_t *group_zero;  /* QTB_FMT_INT4G32 only (fp16 bits)        */
} qtb_matrix_t;

/* One decoder layer.  gate_up is the reference's row-interleaved fused matrix
 * (rows g0,u0,g1,u1,...; qwen_tts_talker.c:378-388). */
typedef struct {
    qtb_matrix_t wq, wk, wv, wo, gate_up, down;
    const float *input_norm, *post_attn_norm, *q_norm, *k_norm;
} qtb_layer_t;

/* A Qwen3 decoder stack (the talker or the code predictor). */
typedef struct {
    int hidden, n_layers, n_heads, n_kv_heads, head_dim, inter;
    float eps;
    int fmt;                      /* QTB_FMT_*                                  */
    const qtb_layer_t *layers;    /* [n_layers]                                 */
    const float *rope_cos;        /* [rope_len][head_dim/2]; the engine uses     */
    const float *rope_sin;        /*   these tables as given (bit-exact RoPE)    */
    int rope_len;
    float rope_theta;             /* used only when rope_cos == NULL            */
    const float *final_norm;      /* [hidden] or NULL (the CP has none in-step) */
} qtb_stack_desc_t;

/* Everything one decode engine serves: the talker and, optionally, the code
 * predictor with its heads and embeddings (qwen_tts.h:514-553). */
typedef struct {
    qtb_stack_desc_t talker;
    const uint16_t *codec_head;      /* bf16 [codec_vocab][hidden]              */
    const uint16_t *codec_embedding; /* bf16 [codec_vocab][hidden]              */
    int codec_vocab;
    int codebook;                    /* 2048: greedy code0 limit and CP vocab    */

    int has_cp;
    qtb_stack_desc_t cp;
    const float *cp_norm;            /* [cp_hidden]                               */
    qtb_matrix_t cp_lm_head[15];     /* [codebook][cp_hidden], format cp.fmt      */
    const uint16_t *cp_codec_emb[15];/* bf16 [codebook][cp_emb_dim]               */
    int cp_emb_dim;                  /* talker hidden (1.7B) or cp hidden (0.6B)  */
    qtb_matrix_t cp_mtp_proj;        /* [cp_hidden][cp_emb_dim] or data == NULL   */
    int cp_mtp_fmt;                  /* QTB_FMT_BF16 or QTB_FMT_INT8              */
    const float *cp_mtp_bias;        /* [cp_hidden] or NULL                       */
    /* The talker's layers in QTB_FMT_BF16 for qtb_prefill, or NULL (prefill
     * then uses the decode weights).  The reference prefills from its bf16
     * weights in every mode (qwen_talker_prefill, qwen_tts_talker.c:840-851,
     * 911-918, 940-981) and decodes from the quantized ones. */
    const qtb_layer_t *talker_prefill_layers;
} qtb_engine_desc_t;

typedef struct qtb_engine qtb_engine_t;
typedef struct qtb_session qtb_session_t;

const char *qtb_last_error(void);
int qtb_device_count(void);
/* How the per-head QK RMSNorm before the K/V append computes 1/sqrt:
 * 1 = as the reference's x86 build does (qwen_rms_norm_per_head,
 * qwen_tts_kernels.c:486-577, compiled with -ffast-math: this host CPU's
 * rsqrtss seed and one Newton step), so appended K bytes equal the
 * reference's on this host; 0 = IEEE 1/sqrtf (non-x86 hosts, a host whose
 * rsqrtss the engine cannot tabulate, or QTB_QK_NORM=ieee). */
int qtb_qk_norm_mode(void);

int  qtb_engine_create(const qtb_engine_desc_t *desc, int device, qtb_engine_t **out);
void qtb_engine_destroy(qtb_engine_t *e);
/* Bytes of weight data the engine streams per talker step / per CP pass
 * (algorithmic bytes: stored weights incl. scales and zeros). */
int64_t qtb_engine_talker_weight_bytes(const qtb_engine_t *e);
int64_t qtb_engine_cp_pass_weight_bytes(const qtb_engine_t *e);
int64_t qtb_engine_cp_head_weight_bytes(const qtb_engine_t *e);

/* A batch of `batch` decode slots sharing the engine's weights.  Each slot owns
 * a page table into a pool of `n_pages` KV pages of 16 positions (all layers);
 * max_ctx bounds the positions of one slot.  n_pages = 0 gives every slot
 * max_ctx/16 private pages (the reference's contiguous cache as an identity
 * page table). */
int  qtb_session_create(qtb_engine_t *e, int batch, int max_ctx, int n_pages, qtb_session_t **out);
void qtb_session_destroy(qtb_session_t *s);
int  qtb_session_batch(const qtb_session_t *s);
/* CTAs a session's program launches with: which = 0 talker step, 1 CP pass,
 * 2 CP frame, 3 whole frame, 4 prefill.  Negative: the program runs as one
 * cluster of that many CTAs (the single-cluster schedule of small batches,
 * opt-in with QTB_CL=1 in the environment at engine creation, used when the
 * device can co-schedule the cluster and every stage of the program fits it).
 * 0: no such program. */
int  qtb_session_program_grid(const qtb_session_t *s, int which);
/* The large-batch (tcgen05) GEMV plan of a rows x cols matrix at `batch` rows
 * over `grid` CTAs, for CTA `cta` (host arithmetic only, no device needed):
 * out[0] first 128-row tile, out[1] tile count, out[2] first 128-byte K chunk,
 * out[3] chunk count, out[4] k-slice, out[5] slices in the plan.  Returns 0,
 * or QTB_E_UNSUPPORTED when the shape does not take that path (format other
 * than bf16 / int8, rows % 128 != 0, batch outside 1..64).  Introspection for
 * tests and tuning; no reference counterpart. */
int  qtb_tc_plan(int fmt, int rows, int cols, int batch, int grid, int cta, int out[6]);
int  qtb_session_n_pages(const qtb_session_t *s);

int  qtb_session_max_ctx(const qtb_session_t *s);
qtb_engine_t *qtb_session_engine(qtb_session_t *s);
/* Pre-final-norm residual of the last talker step, host [batch][hidden]. */
int  qtb_session_get_dec_x(qtb_session_t *s, float *out);

/* Page table of slot b: pages[i] holds positions [16 i, 16 i + 16). */
int qtb_session_set_pages(qtb_session_t *s, int b, const int32_t *pages, int n);
/* Per-slot decode position of the next appended token (host copy -> device). */
int qtb_session_set_pos(qtb_session_t *s, const int32_t *pos /*[batch]*/);
int qtb_session_get_pos(qtb_session_t *s, int32_t *pos /*[batch]*/);

/* One talker decode step for all slots.  embeds: host [batch][hidden];
 * pos: host [batch] (NULL = use the device positions, which qtb_decode_frames
 * advances by one per frame);
 * hidden_out: host [batch][hidden] final-normed hidden, or NULL;
 * dec_x_out: host [batch][hidden] pre-final-norm residual, or NULL. */
int qtb_talker_step(qtb_session_t *s, const float *embeds, const int32_t *pos,
                    float *hidden_out, float *dec_x_out);
/* One code-predictor transformer pass for all slots (no final norm): x is
 * host [batch][cp_hidden], updated in place; pos host [batch]. */
int qtb_cp_pass(qtb_session_t *s, float *x, const int32_t *pos);
/* The whole code-predictor frame on the device (16 passes, 15 greedy heads and
 * the embedding feedback; qwen_tts_code_predictor.c:926-1045).  talker_hidden
 * host [batch][hidden], code0 host [batch], codes_out host [batch][15]. */
int qtb_cp_frame(qtb_session_t *s, const float *talker_hidden, const int32_t *code0,
                 int32_t *codes_out);
/* n_frames whole greedy frames on the device, starting from the next-input
 * embeddings `embeds` (host [batch][hidden]) at the device positions: talker
 * step, codec-head argmax over the first `codebook` rows (code0), the CP frame
 * (when the engine has a CP) and the next embedding
 *   codec_embedding[code0] + sum_g cp_codec_emb[g][code_{g+1}] + pad
 * (qwen_tts.c:1648-1816 with greedy sampling).  pad: host [hidden] or NULL.
 * codes_out: host [n_frames][batch][16] (code0 and the 15 CP codes). */
int qtb_decode_frames(qtb_session_t *s, const float *embeds, const float *pad, int n_frames,
                      int32_t *codes_out, float *last_hidden_out);

/* Talker prefill of n prompt tokens of slot b on the device (the reference's
 * qwen_talker_prefill, qwen_tts_talker.c:730-1038, which the reference runs
 * on the CPU and uploads with qwen_cuda_talker_upload_kv): embeds host
 * [n][hidden] at positions pos0 .. pos0 + n - 1, in chunks of up to 64 tokens
 * run as a batch on the large-batch tensor-core GEMVs (every token's K/V is
 * appended before any of them attends, causally).  As in the reference, the
 * prompt's tokens attend to the prompt's K/V in f32 (positions before pos0
 * come from the bf16 cache); the cache receives the bf16 K/V.  Fills the
 * slot's KV pages and sets its position to pos0 + n.  The f32 prompt K/V
 * buffer (layers x kv heads x 128 x 8 bytes per prompt token) is allocated on
 * the first call and grown to the longest prompt.  hidden_out: host [hidden] final-normed
 * hidden of the last token, or NULL; dec_x_out: its pre-norm residual, or
 * NULL.  The slot's pages must cover the positions. */
int qtb_prefill(qtb_session_t *s, int b, const float *embeds, int n, int pos0, float *hidden_out,
                float *dec_x_out);

/* The codec vocabulary's end-of-speech token (QWEN_TTS_CODEC_EOS, qwen_tts.h:49). */
#define QTB_CODEC_EOS 2150

/* Switch qtb_decode_frames' codec head to the reference's generation-loop
 * rules with greedy sampling (qwen_tts.c:1648-1720, qwen_tts_sampling.c:160-181):
 * logits clipped to +-100, special tokens >= codebook masked except EOS, EOS
 * masked for a slot's first 2 frames and boosted by min(0.5 (frame - 2 E), 10)
 * once frame > 2 E (E = expected_frames[b], 3 x the slot's text tokens in the
 * reference; <= 0 or expected_frames == NULL: no boost), the repetition penalty
 * rep_penalty over the slot's earlier code0 tokens (1 = off; the reference's
 * default is 1.05), then the first maximum.  Frame counters, repetition counts
 * and stop flags restart at zero.  A slot that samples EOS stops: its position
 * no longer advances; qtb_decode_frames reports code0 = QTB_CODEC_EOS with
 * codes 1..15 = -1 in that frame and -1 everywhere afterwards.  Without this
 * call the head is a plain greedy argmax over the first `codebook` rows. */
int qtb_session_begin_generation(qtb_session_t *s, const int32_t *expected_frames, float rep_penalty);
/* Per-slot stop flags of the generation (1 = sampled EOS), host [batch]. */
int qtb_session_get_done(qtb_session_t *s, int32_t *done);
/* Continuous batching (the reference's admit / evict loop, qwen_tts.c:
 * 2389-2740): restart slot b's generation state -- frame counter, repetition
 * counts, EOS boost start (2 x expected_frames, <= 0: none) -- as a running
 * slot (active = 1) or a parked one that neither advances nor reports codes
 * (active = 0).  Needs qtb_session_begin_generation first. */
int qtb_session_reset_slot(qtb_session_t *s, int b, int32_t expected_frames, int active);
/* Slot b's decode position alone (qtb_session_set_pos sets every slot). */
int qtb_session_set_slot_pos(qtb_session_t *s, int b, int32_t pos);
/* Slot b's next talker input (host [hidden]), as qtb_decode_frames with
 * embeds == NULL then consumes it: the embedding of an admitted request's last
 * prompt token, while the other slots keep the inputs their last frame made. */
int qtb_session_set_embed(qtb_session_t *s, int b, const float *embed);
/* Sampling of slot b's code0 (the reference's qwen_tts_sample,
 * qwen_tts_sampling.c:160-202, as its generation loop calls it at
 * qwen_tts.c:1694): temperature (< 1e-6: greedy, the default after
 * qtb_session_begin_generation / qtb_session_reset_slot), top-k (<= 0 or >=
 * the vocabulary: off), top-p (>= 1: off) and the seed of the reference's
 * per-slot LCG (qwen_set_seed; the engine keeps each slot's state across
 * frames, as the reference's batched loop does with qwen_get_seed, qwen_tts.c:
 * 2641-2643).  Softmax, top-k, top-p and the draw run on the device after the
 * codec head's rules (clip, mask, EOS, repetition penalty); sums run in another
 * order than the reference's loops, so a draw can differ from the reference's
 * only when its uniform falls within f32 rounding of a cumulative boundary.
 * The code predictor's heads stay greedy, as in the reference. */
int qtb_session_set_sampling(qtb_session_t *s, int b, float temperature, int32_t top_k, float top_p, uint32_t seed);
/* Every slot's LCG state, host [batch] (qwen_get_seed per slot). */
int qtb_session_get_rng(qtb_session_t *s, uint32_t *state);
/* The device sampler alone on host logits [batch][n] (n <= 2176; row n - 1
 * plays the EOS row): per row temperature, top_k, top_p and LCG state rng
 * (updated in place); out [batch] = the row drawn. */
int qtb_codec_sample_host(const float *logits, int batch, int n, const float *temperature, const int32_t *top_k,
                          const float *top_p, uint32_t *rng, int32_t *out);

/* KV pages <-> contiguous bf16 ([layer][len][kv_dim] with per-layer stride
 * layer_stride positions, the reference's host layout qwen_tts_talker.c:454-460). */
int qtb_session_upload_kv(qtb_session_t *s, int b, const uint16_t *k, const uint16_t *v,
                          int layer_stride, int len);
int qtb_session_download_kv(qtb_session_t *s, int b, uint16_t *k, uint16_t *v,
                            int layer_stride, int len);
int qtb_session_download_cp_kv(qtb_session_t *s, int b, uint16_t *k, uint16_t *v,
                               int layer_stride, int len);

/* Device-side timing of the last call (ms, CUDA events on the launch stream),
 * the number of decode-kernel launches it made, and the per-launch kernel time
 * of the last qtb_decode_frames call. */
double qtb_session_last_ms(const qtb_session_t *s);
/* Stage-level profile of one iteration of program `which` (0 talker step,
 * 1 CP pass, 2 CP frame, 3 whole frame): SM cycles per stage (between grid
 * barriers, measured on CTA 0), the stage kind (1 GEMV, 2 attention, 3 embed,
 * 4 norm, 5 position advance) and rows * 65536 + cols for GEMV stages.
 * Returns the number of stages (or a negative QTB_E_* code). */
int qtb_session_profile(qtb_session_t *s, int which, long long *cycles, int *kind, int64_t *shape, int max_stages);
/* Intra-stage checkpoints of the last qtb_session_profile call: 8 SM-clock
 * stamps per stage taken by CTA 0 (0 where a checkpoint was not reached). */
int qtb_session_profile_checkpoints(qtb_session_t *s, long long *out, int max_vals);
/* Per-CTA grid-barrier arrival times (global timer, ns) of the last
 * qtb_session_profile call, [stage][cta]. */
int qtb_session_profile_arrivals(qtb_session_t *s, long long *out, int max_vals);
int    qtb_session_last_launches(const qtb_session_t *s);

/* Host-side weight encoders (no device needed).  src is bf16 [rows][cols].
 *   int8:    per-row absmax int8 + f32 scale (qwen_quantize_bf16_to_int8,
 *            qwen_tts_kernels.c:2143-2238, nearest-even rounding)
 *   q4_0:    the reference's weighted-LSQ q4_0 blocks, 18 B / 32 weights
 *            (qwen_quantize_bf16_to_q4_0, qwen_tts_kernels.c:2662-2726)
 *   int4g32: asymmetric int4, group 32: codes [rows][cols/2] (low nibble = even
 *            col), fp16 scale and zero [rows][cols/32] (RNE); per group
 *            scale = (max - min) / 15, zero = -min / scale, q = clamp(rint(w /
 *            scale + zero), 0, 15) with the fp16-rounded scale and zero. */
int qtb_quantize_int8(const uint16_t *src_bf16, int rows, int cols, int8_t *dst, float *scale);
int qtb_quantize_q4_0(const uint16_t *src_bf16, int rows, int cols, uint8_t *dst_blocks);
int qtb_quantize_int4g32(const uint16_t *src_bf16, int rows, int cols,
                         uint8_t *codes, uint16_t *scale, uint16_t *zero);

/* Standalone kernels for per-kernel parity and profiling (device pointers are
 * allocated inside; all arguments are host memory).
 *   qtb_gemv_host: y[B][rows] = W x (+ the format's dequant), x [B][cols]. */
int qtb_gemv_host(int fmt, const qtb_matrix_t *w, int rows, int cols,
                  const float *x, int batch, float *y);
/* Fused QK-RMSNorm + RoPE + paged KV append followed by split-K GQA attention,
 * for one layer: qkv host [batch][q_dim + 2 kv_dim] (pre-norm, as the QKV GEMV
 * writes it); kv pages host [n_pages][n_kv][16][head_dim] (bf16, updated in
 * place with the appended token); page_table host [batch][pt_stride]; pos host
 * [batch]; out host [batch][q_dim]. */
int qtb_attention_host(const float *qkv, int batch, int n_heads, int n_kv, int head_dim,
                       const float *q_norm, const float *k_norm, float eps,
                       const float *rope_cos, const float *rope_sin, int rope_len,
                       uint16_t *kpages, uint16_t *vpages, int n_pages,
                       const int32_t *page_table, int pt_stride, const int32_t *pos,
                       int max_splits, float *out);

/* qtb_attention_noalloc: no counterpart in the reference.  The same stage as
 * qtb_attention_host, but every pointer is DEVICE memory owned by the caller
 * (same layouts), `stream` is a cudaStream_t (NULL = legacy default stream),
 * and the call allocates nothing: the launch's scratch lives in one fixed
 * file-scope device array (1,068,032 bytes, ~1.04 MB) that bounds batch <= 4, n_kv <= 16
 * and max_splits <= 16; larger requests return QTB_E_INVALID untouched.  For
 * callers that must not allocate device memory while they run -- code between
 * a pool's reservation and its release, or code whose memory budget is fixed
 * up front.  The array is shared: calls that overlap in time race on it.  The
 * first call on a device (with that device current) does one-time set-up, so
 * make it before any stream capture.  Returns after the stage has finished. */
int qtb_attention_noalloc(const float *qkv, int batch, int n_heads, int n_kv, int head_dim,
                          const float *q_norm, const float *k_norm, float eps,
                          const float *rope_cos, const float *rope_sin, int rope_len,
                          uint16_t *kpages, uint16_t *vpages, int n_pages,
                          const int32_t *page_table, int pt_stride, const int32_t *pos,
                          int max_splits, float *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif
