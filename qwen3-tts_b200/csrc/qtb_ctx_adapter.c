/*
 * qtb_ctx_adapter.c -- the drop-in entry points that read the reference's
 * qwen_tts_ctx_t.  Compiled against the reference's own public header
 * (qwen_tts.h, which defines the context layout these functions bind to) and
 * linked against libqwen3tts_b200.so; nothing here computes: it only maps the
 * context's weight pointers (qwen_tts.h:131-260, 478-546) onto the engine's
 * plain-pointer descriptors.
 *
 *   qwen_cuda_talker_init   replaces qwen_tts_cuda_talker.cu:313
 *   qwen_cuda_cp_init       replaces qwen_tts_cuda_talker.cu:751
 *   qwen_cuda_talker_upload_kv replaces qwen_tts_cuda_talker.cu:424
 *   qwen_cuda_batch_selftest   replaces qwen_tts_cuda_talker.cu:657
 */
#include "qwen_tts.h"
#include "qwen3tts_b200.h"
#include "qwen_tts_cuda_b200.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

/* One precision per state, q4_0 > int8 > bf16 (qwen_tts_cuda_talker.cu:308-311). */
#define PICK_FMT(L) ((L)->wq_q4 ? QTB_FMT_Q4_0 : (L)->wq_int8 ? QTB_FMT_INT8 : QTB_FMT_BF16)

static qtb_matrix_t mat(int fmt, const void *q4, const int8_t *i8, const float *sc, const uint16_t *bf) {
    qtb_matrix_t m;
    memset(&m, 0, sizeof m);
    if (fmt == QTB_FMT_Q4_0) m.data = q4;
    else if (fmt == QTB_FMT_INT8) { m.data = i8; m.row_scale = sc; }
    else m.data = bf;
    return m;
}

#define FILL_LAYER(dst, L, fmt) do { \
    (dst)->wq = mat(fmt, (L)->wq_q4, (L)->wq_int8, (L)->wq_scale, (L)->wq_bf16); \
    (dst)->wk = mat(fmt, (L)->wk_q4, (L)->wk_int8, (L)->wk_scale, (L)->wk_bf16); \
    (dst)->wv = mat(fmt, (L)->wv_q4, (L)->wv_int8, (L)->wv_scale, (L)->wv_bf16); \
    (dst)->wo = mat(fmt, (L)->wo_q4, (L)->wo_int8, (L)->wo_scale, (L)->wo_bf16); \
    (dst)->gate_up = mat(fmt, (L)->gate_up_fused_q4, (L)->gate_up_fused_int8, (L)->gate_up_fused_scale, (L)->gate_up_fused_bf16); \
    (dst)->down = mat(fmt, (L)->down_q4, (L)->down_int8, (L)->down_scale, (L)->down_bf16); \
    (dst)->input_norm = (L)->input_norm; (dst)->post_attn_norm = (L)->post_attn_norm; \
    (dst)->q_norm = (L)->q_norm; (dst)->k_norm = (L)->k_norm; } while (0)

static int env_device(void) {
    const char *e = getenv("QWEN_CUDA_DEVICE");
    return e ? atoi(e) : 0;
}

void *qwen_cuda_talker_init(qwen_tts_ctx_t *ctx) {
    if (!ctx) return NULL;
    qwen_tts_config_t *c = &ctx->config;
    const int L = c->num_layers;
    if (L <= 0 || L > QWEN_TTS_MAX_TALKER_LAYERS) return NULL;
    qtb_layer_t layers[QWEN_TTS_MAX_TALKER_LAYERS];
    const int fmt = PICK_FMT(&ctx->layers[0]);
    for (int l = 0; l < L; l++) {
        qwen_talker_layer_t *ly = &ctx->layers[l];
        if (!ly->wq_bf16 && !ly->wq_int8 && !ly->wq_q4) {
            fprintf(stderr, "qwen3tts_b200: talker layer %d has no weights\n", l);
            return NULL;
        }
        if (PICK_FMT(ly) != fmt) {
            fprintf(stderr, "qwen3tts_b200: mixed talker precisions are not supported\n");
            return NULL;
        }
        FILL_LAYER(&layers[l], ly, fmt);
    }
    qtb_engine_desc_t d;
    memset(&d, 0, sizeof d);
    d.talker.hidden = c->hidden_size;
    d.talker.n_layers = L;
    d.talker.n_heads = c->num_heads;
    d.talker.n_kv_heads = c->num_kv_heads;
    d.talker.head_dim = c->head_dim;
    d.talker.inter = c->intermediate_size;
    d.talker.eps = c->rms_norm_eps;
    d.talker.fmt = fmt;
    d.talker.layers = layers;
    d.talker.rope_cos = ctx->rope_cos;
    d.talker.rope_sin = ctx->rope_sin;
    d.talker.rope_len = ctx->rope_cache_len;
    d.talker.rope_theta = c->rope_theta;
    d.talker.final_norm = ctx->talker_norm;
    d.codec_head = ctx->codec_head_bf16;
    d.codec_embedding = ctx->codec_embedding_bf16;
    d.codec_vocab = c->codec_vocab_size;
    d.codebook = c->codebook_size;
    qtb_engine_t *e = NULL;
    int rc = qtb_engine_create(&d, env_device(), &e);
    if (rc) {
        fprintf(stderr, "qwen3tts_b200: talker init failed: %s\n", qtb_last_error());
        qtb_ref_set_error(rc);
        return NULL;
    }
    qtb_session_t *s = NULL;
    /* positions up to the RoPE table (8192), independent of the host kv_max */
    rc = qtb_session_create(e, 1, ctx->rope_cache_len, 0, &s);
    if (rc) {
        fprintf(stderr, "qwen3tts_b200: talker session failed: %s\n", qtb_last_error());
        qtb_engine_destroy(e);
        qtb_ref_set_error(rc);
        return NULL;
    }
    return qtb_ref_wrap(e, s, 0, 1);
}

void *qwen_cuda_cp_init(qwen_tts_ctx_t *ctx) {
    if (!ctx) return NULL;
    qwen_tts_config_t *c = &ctx->config;
    const int L = c->cp_num_layers;
    if (L <= 0 || L > QWEN_TTS_MAX_CP_LAYERS) return NULL;
    qtb_layer_t layers[QWEN_TTS_MAX_CP_LAYERS];
    const int fmt = PICK_FMT(&ctx->cp_layers[0]);
    for (int l = 0; l < L; l++) {
        qwen_cp_layer_t *ly = &ctx->cp_layers[l];
        if (!ly->wq_bf16 && !ly->wq_int8 && !ly->wq_q4) {
            fprintf(stderr, "qwen3tts_b200: CP layer %d has no weights\n", l);
            return NULL;
        }
        if (PICK_FMT(ly) != fmt || ly->gate_up_fused_q2 || ly->down_q2) {
            fprintf(stderr, "qwen3tts_b200: mixed / q2 CP precisions are not supported\n");
            return NULL;
        }
        FILL_LAYER(&layers[l], ly, fmt);
    }
    qtb_engine_desc_t d;
    memset(&d, 0, sizeof d);
    d.has_cp = 1;
    d.cp.hidden = c->cp_hidden_size;
    d.cp.n_layers = L;
    d.cp.n_heads = c->cp_num_heads;
    d.cp.n_kv_heads = c->cp_num_kv_heads;
    d.cp.head_dim = c->cp_head_dim;
    d.cp.inter = c->cp_intermediate_size;
    d.cp.eps = c->rms_norm_eps;
    d.cp.fmt = fmt;
    d.cp.layers = layers;
    d.cp.rope_cos = ctx->cp_rope_cos;
    d.cp.rope_sin = ctx->cp_rope_sin;
    d.cp.rope_len = ctx->cp_rope_cache_len;
    d.cp.rope_theta = c->rope_theta;
    d.cp_norm = ctx->cp_norm;
    d.codebook = c->codebook_size;
    d.codec_vocab = c->codec_vocab_size;
    d.codec_embedding = ctx->codec_embedding_bf16;
    d.cp_emb_dim = ctx->cp_emb_dim;
    for (int g = 0; g < 15; g++) {
        if (fmt == QTB_FMT_Q4_0 && ctx->cp_lm_head_q4[g]) d.cp_lm_head[g].data = ctx->cp_lm_head_q4[g];
        else if (fmt == QTB_FMT_INT8 && ctx->cp_lm_head_int8[g]) {
            d.cp_lm_head[g].data = ctx->cp_lm_head_int8[g];
            d.cp_lm_head[g].row_scale = ctx->cp_lm_head_scale[g];
        } else if (fmt == QTB_FMT_BF16) d.cp_lm_head[g].data = ctx->cp_lm_head_bf16[g];
        else {
            fprintf(stderr, "qwen3tts_b200: CP lm_head %d precision differs from the CP layers\n", g);
            return NULL;
        }
        d.cp_codec_emb[g] = ctx->cp_codec_emb_bf16[g];
    }
    if (ctx->cp_mtp_proj_int8) {
        d.cp_mtp_proj.data = ctx->cp_mtp_proj_int8;
        d.cp_mtp_proj.row_scale = ctx->cp_mtp_proj_scale;
        d.cp_mtp_fmt = QTB_FMT_INT8;
    } else if (ctx->cp_mtp_proj_bf16) {
        d.cp_mtp_proj.data = ctx->cp_mtp_proj_bf16;
        d.cp_mtp_fmt = QTB_FMT_BF16;
    }
    d.cp_mtp_bias = ctx->cp_mtp_proj_bias;
    qtb_engine_t *e = NULL;
    int rc = qtb_engine_create(&d, env_device(), &e);
    if (rc) {
        fprintf(stderr, "qwen3tts_b200: CP init failed: %s\n", qtb_last_error());
        qtb_ref_set_error(rc);
        return NULL;
    }
    qtb_session_t *s = NULL;
    rc = qtb_session_create(e, 1, ctx->cp_kv_max, 0, &s);
    if (rc) {
        fprintf(stderr, "qwen3tts_b200: CP session failed: %s\n", qtb_last_error());
        qtb_engine_destroy(e);
        qtb_ref_set_error(rc);
        return NULL;
    }
    return qtb_ref_wrap(e, s, 1, 1);
}

void qwen_cuda_talker_upload_kv(void *state, qwen_tts_ctx_t *ctx, int prefill_len) {
    if (!state || !ctx || prefill_len <= 0) return;
    /* host bf16 KV [layer][kv_max][kv_dim] (qwen_tts_talker.c:454-460) -> pages,
     * bit-exact (no f32 round trip) */
    int rc = qtb_session_upload_kv(qtb_ref_session(state), 0, ctx->kv_cache_k, ctx->kv_cache_v, ctx->kv_max, prefill_len);
    qtb_ref_set_error(rc);
    if (rc) fprintf(stderr, "qwen3tts_b200: upload_kv failed: %s\n", qtb_last_error());
}

static double now_ms(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec * 1e3 + t.tv_nsec / 1e6;
}

/* Same contract as the reference self-test: a batched row must equal the
 * single-stream run on the same embeds/positions (< 1e-3), then throughput of
 * single vs batched.  Returns 0 on PASS. */
int qwen_cuda_batch_selftest(qwen_tts_ctx_t *ctx, int B, int frames) {
    const int H = ctx->config.hidden_size;
    if (frames < 8) frames = 8;
    void *S = qwen_cuda_talker_init(ctx);
    if (!S) return -1;
    void *Bs = qwen_cuda_talker_batch_init(S, B);
    if (!Bs) { qwen_cuda_talker_free(S); return -1; }
    float *e1 = malloc((size_t)H * 4), *eB = malloc((size_t)B * H * 4);
    float *h1 = malloc((size_t)H * 4), *hB = malloc((size_t)B * H * 4);
    int *posB = malloc((size_t)B * 4);
    double maxdiff = 0;
    const int chk = frames < 32 ? frames : 32;
    for (int p = 0; p < chk; p++) {
        for (int i = 0; i < H; i++) e1[i] = 0.02f * sinf(0.11f * (i + 1) + 0.3f * p);
        for (int b = 0; b < B; b++) { memcpy(eB + (size_t)b * H, e1, (size_t)H * 4); posB[b] = p; }
        qwen_cuda_talker_step(S, e1, h1, p);
        qwen_cuda_talker_batch_step(Bs, eB, posB, hB);
        for (int b = 0; b < B; b++)
            for (int i = 0; i < H; i++) {
                double dd = fabs(hB[(size_t)b * H + i] - h1[i]);
                if (dd > maxdiff) maxdiff = dd;
            }
    }
    fprintf(stderr, "batch selftest: max|batched-single| = %.2e over %d steps (%s)\n", maxdiff, chk,
            maxdiff < 1e-3 ? "PASS" : "FAIL");
    double t0 = now_ms();
    for (int p = chk; p < chk + frames; p++) qwen_cuda_talker_step(S, e1, h1, p);
    const double ts = (now_ms() - t0) / frames;
    t0 = now_ms();
    for (int p = chk; p < chk + frames; p++) {
        for (int b = 0; b < B; b++) posB[b] = p;
        qwen_cuda_talker_batch_step(Bs, eB, posB, hB);
    }
    const double tb = (now_ms() - t0) / frames;
    fprintf(stderr, "batch talker throughput (B=%d): single %.3f ms/step | batched %.3f ms/step | gain %.2fx\n", B, ts,
            tb, B * ts / tb);
    free(e1); free(eB); free(h1); free(hB); free(posB);
    qwen_cuda_talker_batch_free(Bs);
    qwen_cuda_talker_free(S);
    return maxdiff < 1e-3 ? 0 : 1;
}
