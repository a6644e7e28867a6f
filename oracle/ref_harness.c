/*
 * ref_harness.c -- TEST INFRASTRUCTURE ONLY (the parity oracle's driver).
 *
 * This file is compiled together with the UNMODIFIED reference CPU sources
 * (qwen_tts_kernels.c, qwen_tts_thread.c, qwen_tts_talker.c,
 * qwen_tts_code_predictor.c and the vendored ingot safetensors reader) into
 * oracle/_ref/libqwen_ref_*.so by oracle/Makefile.  Nothing in the product
 * (qwen3-tts_b200/) links or loads it: only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg do, as the checker / the timed CPU reference.
 *
 * It plays the role of the reference's own generation loop for the decode
 * path (qwen_tts.c:632-660 load wiring, qwen_tts.c:1648-1816 frame loop):
 *   - opens a safetensors file with ingot (as qwen_tts_load_ex does),
 *   - fills qwen_tts_config_t by hand (qwen_tts.h:82-119),
 *   - calls qwen_talker_load / qwen_cp_load (qwen_tts_talker.c:319,
 *     qwen_tts_code_predictor.c:393) which quantize INT8 / q4_0 when asked,
 *   - steps qwen_talker_step (qwen_tts_talker.c:537) and qwen_cp_predict
 *     (qwen_tts_code_predictor.c:926),
 *   - exposes the KV cache and quantized weights for byte-level comparison.
 *
 * When built with -DQREF_DROPIN it also wires the reference's own GPU
 * delegation globals (g_cuda_talker_state, g_cuda_cp_state, g_gpu_fused_owner
 * from qwen_tts_talker.c:516-524, qwen_tts_code_predictor.c:725-731) exactly as
 * main.c:1568-1594 does, so that the reference's qwen_talker_step /
 * qwen_cp_predict delegate into a qwen_cuda_* implementation resolved at load
 * time (the drop-in library under test).
 */
#include "qwen_tts.h"
#include "qwen_tts_kernels.h"
#include "ingot/safetensors.h"

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

int qwen_talker_load(qwen_tts_ctx_t *ctx);
int qwen_cp_load(qwen_tts_ctx_t *ctx);
int qwen_talker_step(qwen_tts_ctx_t *ctx, float *embed, float *hidden_out);
int qwen_cp_predict(qwen_tts_ctx_t *ctx, float *talker_hidden, int code0, int *out_codes);

/* Plain-int model description handed in from Python (ctypes). */
typedef struct {
    int hidden, layers, heads, kv_heads, head_dim, inter;
    int codec_vocab, codebook;
    int cp_hidden, cp_layers, cp_heads, cp_kv_heads, cp_head_dim, cp_inter;
    float eps, theta;
} qref_cfg_t;

static int g_threads_started = 0;

void qref_set_threads(int n) {
    if (!g_threads_started) { qwen_init_threads(); g_threads_started = 1; }
    qwen_set_threads(n);
}

int qref_get_threads(void) { return qwen_get_threads(); }

/* Load the talker (+ code predictor when cfg->cp_layers > 0).
 * use_int8 / use_int4 follow qwen_tts_load_ex's flags (qwen_tts.h:663). */
void *qref_load(const char *st_path, const qref_cfg_t *cfg, int use_int8, int use_int4) {
    if (!g_threads_started) { qwen_init_threads(); g_threads_started = 1; }
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)calloc(1, sizeof(qwen_tts_ctx_t));
    if (!ctx) return NULL;
    char err[256] = {0};
    ingot_st *st = NULL;
    if (ingot_st_open(&st, st_path, err, sizeof err) != 0 || !st) {
        fprintf(stderr, "qref_load: %s\n", err);
        free(ctx);
        return NULL;
    }
    ctx->safetensors = st;
    ctx->silent = 1;
    ctx->use_int8 = use_int8;
    ctx->use_int4 = use_int4;
    qwen_tts_config_t *c = &ctx->config;
    c->hidden_size = cfg->hidden;
    c->text_hidden_size = 2048;
    c->num_layers = cfg->layers;
    c->num_heads = cfg->heads;
    c->num_kv_heads = cfg->kv_heads;
    c->head_dim = cfg->head_dim;
    c->intermediate_size = cfg->inter;
    c->codec_vocab_size = cfg->codec_vocab;
    c->codebook_size = cfg->codebook;
    c->rms_norm_eps = cfg->eps;
    c->rope_theta = cfg->theta;
    c->cp_hidden_size = cfg->cp_hidden;
    c->cp_num_layers = cfg->cp_layers;
    c->cp_num_heads = cfg->cp_heads;
    c->cp_num_kv_heads = cfg->cp_kv_heads;
    c->cp_head_dim = cfg->cp_head_dim;
    c->cp_intermediate_size = cfg->cp_inter;
    if (qwen_talker_load(ctx) != 0) { fprintf(stderr, "qref_load: talker load failed\n"); return NULL; }
    if (cfg->cp_layers > 0 && qwen_cp_load(ctx) != 0) { fprintf(stderr, "qref_load: cp load failed\n"); return NULL; }
    return ctx;
}

void *qref_ctx(void *h) { return h; }

int qref_talker_step(void *h, const float *embed, float *hidden_out) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    int H = ctx->config.hidden_size;
    float *e = (float *)malloc((size_t)H * sizeof(float));
    memcpy(e, embed, (size_t)H * sizeof(float));
    int rc = qwen_talker_step(ctx, e, hidden_out);
    free(e);
    return rc;
}

int qwen_talker_prefill(qwen_tts_ctx_t *ctx, float *input_embeds, int seq_len);

/* The reference's batched CPU prefill (qwen_tts_talker.c:730-1038) of n prompt
 * embeddings at positions 0..n-1: fills the host KV cache and dec_x. */
int qref_talker_prefill(void *h, const float *embeds, int n, float *dec_x_out) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    float *e = (float *)malloc((size_t)n * ctx->config.hidden_size * sizeof(float));
    memcpy(e, embeds, (size_t)n * ctx->config.hidden_size * sizeof(float));
    int rc = qwen_talker_prefill(ctx, e, n);
    free(e);
    if (dec_x_out) memcpy(dec_x_out, ctx->dec_x, (size_t)ctx->config.hidden_size * sizeof(float));
    return rc;
}

int qref_cp_predict(void *h, const float *talker_hidden, int code0, int *out_codes) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    int H = ctx->config.hidden_size;
    float *t = (float *)malloc((size_t)H * sizeof(float));
    memcpy(t, talker_hidden, (size_t)H * sizeof(float));
    int rc = qwen_cp_predict(ctx, t, code0, out_codes);
    free(t);
    return rc;
}

int qref_kv_len(void *h) { return ((qwen_tts_ctx_t *)h)->kv_len; }
int qref_kv_max(void *h) { return ((qwen_tts_ctx_t *)h)->kv_max; }
void qref_set_kv_len(void *h, int n) { ((qwen_tts_ctx_t *)h)->kv_len = n; }

/* Copy layer `l`'s first n positions of the contiguous bf16 KV
 * ([layer][kv_max][kv_dim], qwen_tts_talker.c:454-460) into dst_k/dst_v. */
void qref_copy_kv(void *h, int l, int n, uint16_t *dst_k, uint16_t *dst_v) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    int kvd = ctx->config.num_kv_heads * ctx->config.head_dim;
    size_t off = (size_t)l * ctx->kv_max * kvd;
    memcpy(dst_k, ctx->kv_cache_k + off, (size_t)n * kvd * sizeof(uint16_t));
    memcpy(dst_v, ctx->kv_cache_v + off, (size_t)n * kvd * sizeof(uint16_t));
}

/* The CP's own bf16 KV for the last predicted frame ([layer][64][kv_dim]). */
void qref_copy_cp_kv(void *h, int l, int n, uint16_t *dst_k, uint16_t *dst_v) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    int kvd = ctx->config.cp_num_kv_heads * ctx->config.cp_head_dim;
    size_t off = (size_t)l * ctx->cp_kv_max * kvd;
    memcpy(dst_k, ctx->cp_kv_k + off, (size_t)n * kvd * sizeof(uint16_t));
    memcpy(dst_v, ctx->cp_kv_v + off, (size_t)n * kvd * sizeof(uint16_t));
}

/* Greedy codec token of the harness frame loop: argmax over the first `limit`
 * rows of codec_head (qwen_tts.c:1650-1663 with the logit mask reduced to a
 * vocabulary limit), using the reference's own fused argmax matvec. */
int qref_codec_argmax(void *h, const float *hidden, int limit) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    return qwen_argmax_matvec_bf16(hidden, ctx->codec_head_bf16, ctx->config.hidden_size, limit);
}

int qwen_tts_sample(float *logits, int vocab_size, float temp, int top_k, float top_p,
                    float rep_penalty, int *prev_tokens, int n_prev);
void qwen_set_seed(uint32_t seed);
uint32_t qwen_get_seed(void);

/* code0 of one frame of the reference's generation loop with greedy sampling:
 * the codec-head logits over the whole vocabulary (qwen_tts.c:1650), the
 * clip / special-token mask / EOS rules of qwen_tts.c:1652-1676 (restated here:
 * qwen_tts_generate is not part of this harness), then the reference's own
 * qwen_tts_sample at temperature 0 with the repetition penalty over the
 * earlier code0 tokens (qwen_tts_sampling.c:160-181).  2150 = EOS. */
/* The same with the reference's sampling (temperature, top-k, top-p) and its
 * LCG state in and out (qwen_set_seed / qwen_get_seed around the draw, as its
 * batched loop does per slot, qwen_tts.c:2641-2643). */
int qref_codec_sample_t(void *h, const float *hidden, int frame, int expected_frames, float rep_penalty,
                        int *prev_tokens, int n_prev, float temp, int top_k, float top_p, uint32_t *seed) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    const int V = ctx->config.codec_vocab_size, H = ctx->config.hidden_size;
    float *logits = (float *)malloc((size_t)V * sizeof(float));
    qwen_matvec_bf16(logits, ctx->codec_head_bf16, hidden, V, H);
    for (int t = 0; t < V; t++) {
        if (logits[t] > 100.0f) logits[t] = 100.0f;
        if (logits[t] < -100.0f) logits[t] = -100.0f;
    }
    for (int t = 2048; t < V; t++)
        if (t != 2150) logits[t] = -1e30f;
    if (frame < 2) logits[2150] = -1e30f;
    {
        int boost_start = expected_frames * 2;
        if (expected_frames > 0 && frame > boost_start) {
            float boost = 0.5f * (frame - boost_start);
            if (boost > 10.0f) boost = 10.0f;
            logits[2150] += boost;
        }
    }
    qwen_set_seed(*seed);
    int c = qwen_tts_sample(logits, V, temp, top_k, top_p, rep_penalty, prev_tokens, n_prev);
    *seed = qwen_get_seed();
    free(logits);
    return c;
}

int qref_codec_sample(void *h, const float *hidden, int frame, int expected_frames, float rep_penalty,
                      int *prev_tokens, int n_prev) {
    uint32_t seed = 12345;
    return qref_codec_sample_t(h, hidden, frame, expected_frames, rep_penalty, prev_tokens, n_prev, 0.0f, 50, 1.0f,
                               &seed);
}

/* The reference's sampler alone on given logits (no repetition penalty). */
int qref_sample_logits(const float *logits_in, int n, float temp, int top_k, float top_p, uint32_t *seed) {
    float *logits = (float *)malloc((size_t)n * sizeof(float));
    memcpy(logits, logits_in, (size_t)n * sizeof(float));
    qwen_set_seed(*seed);
    int c = qwen_tts_sample(logits, n, temp, top_k, top_p, 1.0f, NULL, 0);
    *seed = qwen_get_seed();
    free(logits);
    return c;
}

/* Talker codec embedding row -> f32 (qwen_tts.c:1768-1778, first term). */
void qref_codec_embed(void *h, int code, float *out) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    int H = ctx->config.hidden_size;
    qwen_bf16_to_f32_vec(out, ctx->codec_embedding_bf16 + (size_t)code * H, H);
}

/* Accessors for the quantized weights the reference produced, so the GPU
 * library can be given byte-identical INT8 / q4_0 data.  which:
 * 0 wq 1 wk 2 wv 3 wo 4 gate_up_fused 5 down.  kind: 0 bf16 1 int8 2 int8-scale
 * 3 q4_0.  cp selects the code-predictor layer table. */
const void *qref_weight(void *h, int cp, int layer, int which, int kind) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
#define PICK(L) do { \
        switch (which) { \
        case 0: return kind==0?(const void*)(L)->wq_bf16:kind==1?(const void*)(L)->wq_int8:kind==2?(const void*)(L)->wq_scale:(const void*)(L)->wq_q4; \
        case 1: return kind==0?(const void*)(L)->wk_bf16:kind==1?(const void*)(L)->wk_int8:kind==2?(const void*)(L)->wk_scale:(const void*)(L)->wk_q4; \
        case 2: return kind==0?(const void*)(L)->wv_bf16:kind==1?(const void*)(L)->wv_int8:kind==2?(const void*)(L)->wv_scale:(const void*)(L)->wv_q4; \
        case 3: return kind==0?(const void*)(L)->wo_bf16:kind==1?(const void*)(L)->wo_int8:kind==2?(const void*)(L)->wo_scale:(const void*)(L)->wo_q4; \
        case 4: return kind==0?(const void*)(L)->gate_up_fused_bf16:kind==1?(const void*)(L)->gate_up_fused_int8:kind==2?(const void*)(L)->gate_up_fused_scale:(const void*)(L)->gate_up_fused_q4; \
        case 5: return kind==0?(const void*)(L)->down_bf16:kind==1?(const void*)(L)->down_int8:kind==2?(const void*)(L)->down_scale:(const void*)(L)->down_q4; \
        } } while (0)
    if (cp) { qwen_cp_layer_t *L = &ctx->cp_layers[layer]; PICK(L); }
    else    { qwen_talker_layer_t *L = &ctx->layers[layer]; PICK(L); }
#undef PICK
    return NULL;
}

/* lm_head g of the CP: kind 0 bf16, 1 int8, 2 int8 scale, 3 q4_0. */
const void *qref_cp_lm_head(void *h, int g, int kind) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    if (kind == 0) return ctx->cp_lm_head_bf16[g];
    if (kind == 1) return ctx->cp_lm_head_int8[g];
    if (kind == 2) return ctx->cp_lm_head_scale[g];
    return ctx->cp_lm_head_q4[g];
}

/* The code predictor's small_to_mtp_projection (qwen_tts_code_predictor.c:
 * 458-479): kind 0 bf16 weight, 1 its int8 twin, 2 the int8 row scales,
 * 3 the f32 bias (NULL when the talker and CP widths match). */
const void *qref_cp_mtp(void *h, int kind) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    if (kind == 0) return ctx->cp_mtp_proj_bf16;
    if (kind == 1) return ctx->cp_mtp_proj_int8;
    if (kind == 2) return ctx->cp_mtp_proj_scale;
    return ctx->cp_mtp_proj_bias;
}

/* RoPE tables the reference built at load (qwen_tts_talker.c:478-495,
 * qwen_tts_code_predictor.c:498-507): which 0 = cos, 1 = sin. */
const float *qref_rope(void *h, int cp, int which) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    if (cp) return which ? ctx->cp_rope_sin : ctx->cp_rope_cos;
    return which ? ctx->rope_sin : ctx->rope_cos;
}
int qref_rope_len(void *h, int cp) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    return cp ? ctx->cp_rope_cache_len : ctx->rope_cache_len;
}

/* The talker's K/V append for one token from its pre-norm q/k/v rows
 * (qwen_tts_talker.c:603-615): the reference's own qwen_rms_norm_per_head
 * (exported by qwen_tts_kernels.c) on q and k, then NeoX RoPE as
 * apply_rope_neox_inplace's AVX2 branch computes it (qwen_tts_talker.c:
 * 203-251, static there, so restated here: x1 c - (x2 s) and x2 c + (x1 s),
 * each one fused multiply-add over a rounded product), then bf16 truncation of
 * k and v (f32_to_bf16_vec, qwen_tts_talker.c:125-159).  q (in place), k (in
 * place) and the bf16 rows k_out / v_out. */
void qref_qk_norm_rope_append(float *q, float *k, const float *v, int n_heads, int n_kv, int head_dim,
                              const float *q_norm, const float *k_norm, float eps,
                              const float *cos_cache, const float *sin_cache, int pos,
                              uint16_t *k_out, uint16_t *v_out) {
    qwen_rms_norm_per_head(q, q_norm, 1, n_heads, head_dim, eps);
    qwen_rms_norm_per_head(k, k_norm, 1, n_kv, head_dim, eps);
    const int half = head_dim / 2;
    const float *c = cos_cache + (size_t)pos * half, *sn = sin_cache + (size_t)pos * half;
    for (int t = 0; t < 2; t++) {
        float *x = t ? k : q;
        const int nh = t ? n_kv : n_heads;
        for (int h = 0; h < nh; h++) {
            float *xh = x + (size_t)h * head_dim;
            for (int i = 0; i < half; i++) {
                const float x1 = xh[i], x2 = xh[i + half];
                volatile float p2s = x2 * sn[i], p1s = x1 * sn[i];   /* rounded products */
                xh[i] = fmaf(x1, c[i], -p2s);
                xh[i + half] = fmaf(x2, c[i], p1s);
            }
        }
    }
    const int kvd = n_kv * head_dim;
    for (int i = 0; i < kvd; i++) {
        uint32_t a, b;
        memcpy(&a, &k[i], 4);
        memcpy(&b, &v[i], 4);
        k_out[i] = (uint16_t)(a >> 16);
        v_out[i] = (uint16_t)(b >> 16);
    }
}

void qref_free(void *h) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    if (!ctx) return;
    /* Weights that were not mmapped (quantized copies, fused gate_up, norms)
     * leak here on purpose: the oracle process is short-lived and the
     * reference's own unload (qwen_tts.c) is not part of the linked sources. */
    if (ctx->safetensors) ingot_st_close((ingot_st *)ctx->safetensors);
    free(ctx->kv_cache_k); free(ctx->kv_cache_v);
    free(ctx->cp_kv_k); free(ctx->cp_kv_v);
    free(ctx);
}

#ifdef QREF_DROPIN
/* The reference's delegation globals (defined in the linked talker/CP TUs). */
extern void *g_cuda_talker_state;
extern void *g_cuda_cp_state;
extern void *g_gpu_fused_owner;
/* Resolved from the drop-in library at load time. */
void *qwen_cuda_talker_init(qwen_tts_ctx_t *ctx);
void  qwen_cuda_talker_free(void *st);
void *qwen_cuda_cp_init(qwen_tts_ctx_t *ctx);
void  qwen_cuda_cp_free(void *st);

/* Same wiring as main.c:1568-1594 (--backend cuda + QWEN_CUDA_FUSED_TALKER=1). */
int qref_dropin_attach(void *h, int talker, int cp) {
    qwen_tts_ctx_t *ctx = (qwen_tts_ctx_t *)h;
    if (talker) {
        g_cuda_talker_state = qwen_cuda_talker_init(ctx);
        if (!g_cuda_talker_state) return -1;
    }
    if (cp) {
        g_cuda_cp_state = qwen_cuda_cp_init(ctx);
        if (!g_cuda_cp_state) return -2;
    }
    g_gpu_fused_owner = ctx;
    return 0;
}

void qref_dropin_detach(void) {
    if (g_cuda_talker_state) qwen_cuda_talker_free(g_cuda_talker_state);
    if (g_cuda_cp_state) qwen_cuda_cp_free(g_cuda_cp_state);
    g_cuda_talker_state = NULL;
    g_cuda_cp_state = NULL;
    g_gpu_fused_owner = NULL;
}
#endif
