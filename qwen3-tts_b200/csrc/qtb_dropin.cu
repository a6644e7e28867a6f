// qtb_dropin.cu -- the reference-named entry points whose signatures carry
// only plain pointers (steps, frees, batch states).  Each one replaces the
// function of the same name in the reference's qwen_tts_cuda_talker.cu (see
// include/qwen_tts_cuda_b200.h for the file:line map) and runs on the engine
// in qtb_engine.cu.  The ctx-reading ones are in qtb_ctx_adapter.c.
#include "../../include/qwen3tts_b200.h"
#include "../../include/qwen_tts_cuda_b200.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace {
struct RefState {
  qtb_engine_t *e;
  qtb_session_t *s;
  int kind;          // 0 talker, 1 code predictor
  int owns_engine;
};
thread_local int g_last = 0;

void report(const char *fn, int rc) {
  g_last = rc;
  if (rc) fprintf(stderr, "qwen3tts_b200: %s failed (%d): %s\n", fn, rc, qtb_last_error());
}
}  // namespace

extern "C" void qtb_ref_set_error(int code) { g_last = code; }
extern "C" int qwen_cuda_last_error(void) { return g_last; }

extern "C" void *qtb_ref_wrap(struct qtb_engine *e, struct qtb_session *s, int kind, int owns_engine) {
  RefState *r = new RefState{e, s, kind, owns_engine};
  return r;
}
extern "C" struct qtb_session *qtb_ref_session(void *state) { return state ? ((RefState *)state)->s : nullptr; }

static void free_state(void *st) {
  RefState *r = (RefState *)st;
  if (!r) return;
  qtb_session_destroy(r->s);
  if (r->owns_engine) qtb_engine_destroy(r->e);
  delete r;
}

static void *batch_init(void *single, int B, int kind) {
  RefState *r = (RefState *)single;
  if (!r || B < 1 || B > 64) {
    report("batch_init", QTB_E_INVALID);
    return nullptr;
  }
  qtb_session_t *s = nullptr;
  int rc = qtb_session_create(r->e, B, qtb_session_max_ctx(r->s), 0, &s);
  if (rc) { report("batch_init", rc); return nullptr; }
  g_last = 0;
  return qtb_ref_wrap(r->e, s, kind, 0);
}

// ---------------------------------------------------------------- talker ----
extern "C" void qwen_cuda_talker_step(void *st, const float *embed, float *hidden_out, int pos) {
  RefState *r = (RefState *)st;
  if (!r) { report("qwen_cuda_talker_step", QTB_E_INVALID); return; }
  const int32_t p = pos;
  report("qwen_cuda_talker_step", qtb_talker_step(r->s, embed, &p, hidden_out, nullptr));
}

extern "C" void qwen_cuda_talker_get_dec_x(void *st, float *out) {
  RefState *r = (RefState *)st;
  if (!r || !out) return;
  report("qwen_cuda_talker_get_dec_x", qtb_session_get_dec_x(r->s, out));
}

extern "C" void qwen_cuda_talker_free(void *st) { free_state(st); }

extern "C" void *qwen_cuda_talker_batch_init(void *single, int B) { return batch_init(single, B, 0); }

extern "C" void qwen_cuda_talker_batch_step(void *st, const float *embeds, const int *pos_arr, float *hidden_out) {
  RefState *r = (RefState *)st;
  if (!r) { report("qwen_cuda_talker_batch_step", QTB_E_INVALID); return; }
  report("qwen_cuda_talker_batch_step", qtb_talker_step(r->s, embeds, pos_arr, hidden_out, nullptr));
}

extern "C" void qwen_cuda_talker_batch_upload_slot(void *st, int b, const uint16_t *kv_k, const uint16_t *kv_v,
                                                   int src_kv_max, int prefill_len) {
  RefState *r = (RefState *)st;
  if (!r || prefill_len <= 0) return;
  // source layout ((b * n_layers + l) * src_kv_max + pos) * kv_dim
  // (qwen_tts_cuda_talker.cu:626-642): slot b's block starts at b * n_layers * src_kv_max * kv_dim
  extern int qtb_engine_talker_layers(const qtb_engine_t *e);
  extern int qtb_engine_talker_kv_dim(const qtb_engine_t *e);
  const size_t blk = (size_t)qtb_engine_talker_layers(r->e) * src_kv_max * qtb_engine_talker_kv_dim(r->e);
  report("qwen_cuda_talker_batch_upload_slot",
         qtb_session_upload_kv(r->s, b, kv_k + (size_t)b * blk, kv_v + (size_t)b * blk, src_kv_max, prefill_len));
}

extern "C" void qwen_cuda_talker_batch_free(void *st) { free_state(st); }

extern "C" int qwen_cuda_talker_batch_set_pages(void *st, int b, const int32_t *pages, int n) {
  RefState *r = (RefState *)st;
  if (!r) return QTB_E_INVALID;
  int rc = qtb_session_set_pages(r->s, b, pages, n);
  g_last = rc;
  return rc;
}

// ------------------------------------------------------- code predictor -----
extern "C" void qwen_cuda_cp_step(void *st, float *x, int pos) {
  RefState *r = (RefState *)st;
  if (!r) { report("qwen_cuda_cp_step", QTB_E_INVALID); return; }
  const int32_t p = pos;
  report("qwen_cuda_cp_step", qtb_cp_pass(r->s, x, &p));
}

extern "C" void qwen_cuda_cp_free(void *st) { free_state(st); }

extern "C" void *qwen_cuda_cp_batch_init(void *single, int B) { return batch_init(single, B, 1); }

extern "C" void qwen_cuda_cp_batch_step(void *st, float *x, const int *pos_arr) {
  RefState *r = (RefState *)st;
  if (!r) { report("qwen_cuda_cp_batch_step", QTB_E_INVALID); return; }
  report("qwen_cuda_cp_batch_step", qtb_cp_pass(r->s, x, pos_arr));
}

extern "C" void qwen_cuda_cp_batch_free(void *st) { free_state(st); }

extern "C" int qwen_cuda_cp_frame(void *st, const float *talker_hidden, const int *code0, int *out_codes) {
  RefState *r = (RefState *)st;
  if (!r) return QTB_E_INVALID;
  int rc = qtb_cp_frame(r->s, talker_hidden, code0, out_codes);
  report("qwen_cuda_cp_frame", rc);
  return rc;
}
