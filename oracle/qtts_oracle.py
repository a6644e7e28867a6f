"""qtts_oracle -- TEST INFRASTRUCTURE ONLY: a numpy restatement of the
reference's CPU decode path (gabriele-mastrapasqua/qwen3-tts), used as the
parity checker for the CUDA engine.

Pinning: tests/test_oracle_pin.py checks every function here against the
compiled reference (oracle/_ref, built from the reference's own sources) and
tests/test_golden.py against the committed golden vectors in tests/golden/
(generated from the compiled reference by tests/golden/make_golden.py).  The
two formats the reference does not have -- paged KV and asymmetric int4 g32 --
are defined here and in the engine; their parity is "gather(pages) ==
contiguous cache" and "same codes + same dequant" (unpinned by the reference).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  Dot products accumulate in float64 (the reference accumulates in
f32 in a SIMD-dependent order; float64 is closer to the exact value than either
side, so the comparison tolerance covers both).
"""
from __future__ import annotations

import numpy as np


def f32_from_bf16(a):
    return (np.asarray(a).astype(np.uint32) << 16).view(np.float32)


def bf16_trunc(x):
    """f32 -> bf16 bits by truncation (qwen_tts_talker.c:98-103, :125-159)."""
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def f16_to_f32(h):
    return np.asarray(h, np.uint16).view(np.float16).astype(np.float32)


# --------------------------------------------------------------- matvecs ----
def matvec_bf16(W, x):
    """qwen_matvec_bf16 (qwen_tts_kernels.c:1091-1100): y = W x, W bf16."""
    return (f32_from_bf16(W).astype(np.float64) @ np.asarray(x, np.float64).T).T.astype(np.float32)


def matvec_int8(W, scale, x):
    """qwen_matvec_int8 f32-activation path (qwen_tts_kernels.c:2548-2599):
    y[r] = scale[r] * sum_k W[r,k] x[k]."""
    acc = (np.asarray(W, np.float64) @ np.asarray(x, np.float64).T).T
    return (acc * np.asarray(scale, np.float64)).astype(np.float32)


def q4_0_unpack(blocks, rows, cols):
    """q4_0 blocks (qwen_tts_kernels.h:207-210) -> (codes [rows][cols] in 0..15,
    scales [rows][cols/32] f32)."""
    b = np.asarray(blocks, np.uint8).reshape(rows, cols // 32, 18)
    sc = f16_to_f32(b[:, :, 0].astype(np.uint16) | (b[:, :, 1].astype(np.uint16) << 8))
    qs = b[:, :, 2:]
    codes = np.empty((rows, cols // 32, 32), np.uint8)
    codes[:, :, 0::2] = qs & 0xF
    codes[:, :, 1::2] = qs >> 4
    return codes.reshape(rows, cols), sc


def dequant_q4_0(blocks, rows, cols):
    """w = (nib - 8) * scale (q4_0_matvec_inner, qwen_tts_kernels.c:2810-2820)."""
    codes, sc = q4_0_unpack(blocks, rows, cols)
    return ((codes.astype(np.float32) - 8.0).reshape(rows, cols // 32, 32) * sc[:, :, None]).reshape(rows, cols)


def matvec_q4_0(blocks, rows, cols, x):
    codes, sc = q4_0_unpack(blocks, rows, cols)
    q = codes.astype(np.float64).reshape(rows, cols // 32, 32) - 8.0
    xx = np.asarray(x, np.float64).reshape(-1, cols // 32, 32)
    return np.einsum("rgk,bgk,rg->br", q, xx, sc.astype(np.float64)).astype(np.float32)


def int4g_unpack(codes, rows, cols):
    c = np.asarray(codes, np.uint8).reshape(rows, cols // 2)
    out = np.empty((rows, cols), np.uint8)
    out[:, 0::2] = c & 0xF
    out[:, 1::2] = c >> 4
    return out


def matvec_int4g(codes, scale, zero, rows, cols, x):
    """Asymmetric int4 g32: w = (q - zero) * scale (the engine's format)."""
    q = int4g_unpack(codes, rows, cols).astype(np.float64).reshape(rows, cols // 32, 32)
    s = f16_to_f32(scale).astype(np.float64).reshape(rows, cols // 32)
    z = f16_to_f32(zero).astype(np.float64).reshape(rows, cols // 32)
    xx = np.asarray(x, np.float64).reshape(-1, cols // 32, 32)
    return np.einsum("rgk,bgk,rg->br", q - z[:, :, None], xx, s).astype(np.float32)


# ------------------------------------------------------------- quantizers ---
def quantize_int8(W_bf16):
    """qwen_quantize_bf16_to_int8 (qwen_tts_kernels.c:2143-2238), x86 vector
    path: scale = amax/127, q = round-half-even(w * 127/amax)."""
    w = f32_from_bf16(W_bf16)
    amax = np.abs(w).max(axis=1).astype(np.float32)
    # built with -ffast-math: amax / 127.0f compiles to amax * (1/127.0f)
    s = (amax * np.float32(1.0 / 127.0)).astype(np.float32)
    inv = np.where(s > 0, np.float32(127.0) / np.where(amax > 0, amax, 1), 0).astype(np.float32)
    q = np.clip(np.rint(w * inv[:, None]), -128, 127).astype(np.int8)
    return q, s


def quantize_int4g32(W_bf16):
    """The engine's asymmetric int4 g32 encoder (qtb_quantize_int4g32)."""
    w = f32_from_bf16(W_bf16)
    rows, cols = w.shape
    g = w.reshape(rows, cols // 32, 32)
    mn, mx = g.min(axis=2), g.max(axis=2)
    sc = ((mx - mn) / np.float32(15.0)).astype(np.float32)
    flat = ~(sc > 0)
    z = np.where(flat, -mn, -mn / np.where(flat, 1, sc)).astype(np.float32)
    sc = np.where(flat, np.float32(1.0), sc).astype(np.float32)
    hs = sc.astype(np.float16)
    hz = z.astype(np.float16)
    s16, z16 = hs.astype(np.float32), hz.astype(np.float32)
    q = np.clip(np.rint((g / s16[:, :, None]).astype(np.float32) + z16[:, :, None]), 0, 15).astype(np.uint8)
    q = q.reshape(rows, cols)
    codes = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return codes, hs.view(np.uint16), hz.view(np.uint16)


# -------------------------------------------------------- norms / rope / act -
def rms_norm(x, w, eps):
    """qwen_rms_norm (qwen_tts_kernels.c:292-382): x * (1/sqrt(mean x^2 + eps)) * w."""
    x = np.asarray(x, np.float32)
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    inv = (1.0 / np.sqrt(ss / x.shape[-1] + eps)).astype(np.float32)
    return ((x * inv) * np.asarray(w, np.float32)).astype(np.float32)


def rms_norm_per_head(x, w, n_heads, head_dim, eps):
    """qwen_rms_norm_per_head (qwen_tts_kernels.c:486-577), shared w[head_dim]."""
    xh = np.asarray(x, np.float32).reshape(n_heads, head_dim)
    return rms_norm(xh, w, eps).reshape(-1)


def rope_neox(x, n_heads, head_dim, cos_t, sin_t, pos):
    """apply_rope_neox_inplace (qwen_tts_talker.c:203-251), x86 FMA form:
    x1' = fma(x1, c, -(x2*s)), x2' = fma(x2, c, x1*s).  The fused multiply-add
    is evaluated with the exact product in float64 and one final f32 rounding."""
    half = head_dim // 2
    xh = np.asarray(x, np.float32).reshape(n_heads, head_dim)
    c = cos_t[pos].astype(np.float32)
    s = sin_t[pos].astype(np.float32)
    x1, x2 = xh[:, :half], xh[:, half:]
    p2 = (x2 * s).astype(np.float32)
    p1 = (x1 * s).astype(np.float32)
    n1 = (x1.astype(np.float64) * c.astype(np.float64) - p2.astype(np.float64)).astype(np.float32)
    n2 = (x2.astype(np.float64) * c.astype(np.float64) + p1.astype(np.float64)).astype(np.float32)
    return np.concatenate([n1, n2], axis=1).reshape(-1)


def swiglu(gu):
    """qwen_swiglu_inplace (qwen_tts_kernels.c:3857-3878) on interleaved rows."""
    g = np.asarray(gu, np.float32)[..., 0::2]
    u = np.asarray(gu, np.float32)[..., 1::2]
    return (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)


def attention_bf16kv(q, K, V, n_heads, n_kv, head_dim, L):
    """qwen_causal_attention_bf16kv (qwen_tts_kernels.c:3704-3846) for one
    query at position L-1: K, V bf16 bits [L][n_kv*head_dim]."""
    scale = np.float32(1.0) / np.sqrt(np.float32(head_dim))
    qh = np.asarray(q, np.float64).reshape(n_heads, head_dim)
    Kf = f32_from_bf16(K[:L]).astype(np.float64).reshape(L, n_kv, head_dim)
    Vf = f32_from_bf16(V[:L]).astype(np.float64).reshape(L, n_kv, head_dim)
    grp = n_heads // n_kv
    out = np.empty((n_heads, head_dim), np.float64)
    for h in range(n_heads):
        g = h // grp
        s = (Kf[:, g, :] @ qh[h]).astype(np.float32) * scale
        s = s.astype(np.float64)
        p = np.exp(s - s.max())
        out[h] = (p @ Vf[:, g, :]) / p.sum()
    return out.reshape(-1).astype(np.float32)


# ------------------------------------------------------------- paged KV -----
def gather_pages(kpool, vpool, page_table, length):
    """Paged cache (pool [n_pages][n_kv][16][128]) -> contiguous [length][kv_dim]."""
    n_kv = kpool.shape[1]
    k = np.empty((length, n_kv * 128), np.uint16)
    v = np.empty_like(k)
    for p in range(length):
        pg = page_table[p // 16]
        k[p] = kpool[pg, :, p % 16, :].reshape(-1)
        v[p] = vpool[pg, :, p % 16, :].reshape(-1)
    return k, v


# -------------------------------------------------------------- the model ---
class Stack:
    """Dequantized f32 weights of one decoder stack (talker or CP)."""

    def __init__(self, layers, H, nh, nkv, hd, I, eps, rope_cos, rope_sin, final_norm=None, fmt="bf16", q=None):
        self.H, self.nh, self.nkv, self.hd, self.I, self.eps = H, nh, nkv, hd, I, eps
        self.cos, self.sin = rope_cos, rope_sin
        self.final_norm = final_norm
        self.layers = []
        for i, ly in enumerate(layers):
            d = {}
            for nm in ("wq", "wk", "wv", "wo", "gate_up", "down"):
                src = (q or {}).get(f"{i}.{nm}")
                d[nm] = dequant(fmt, getattr(ly, nm), src)
            d.update(input_norm=ly.input_norm, post_attn_norm=ly.post_attn_norm, q_norm=ly.q_norm, k_norm=ly.k_norm)
            self.layers.append(d)


def dequant(fmt, w_bf16, qdict=None):
    rows, cols = w_bf16.shape
    if fmt == "bf16":
        return f32_from_bf16(w_bf16)
    if fmt == "int8":
        q, s = (qdict["data"], qdict["row_scale"]) if qdict else quantize_int8(w_bf16)
        return (q.astype(np.float32) * s[:, None]).astype(np.float32)
    if fmt == "q4_0":
        return dequant_q4_0(qdict["data"], rows, cols)
    if fmt == "int4g32":
        c, s, z = (qdict["data"], qdict["group_scale"], qdict["group_zero"]) if qdict else quantize_int4g32(w_bf16)
        qv = int4g_unpack(c, rows, cols).astype(np.float32).reshape(rows, cols // 32, 32)
        return ((qv - f16_to_f32(z)[:, :, None]) * f16_to_f32(s)[:, :, None]).reshape(rows, cols)
    raise ValueError(fmt)


# float64 accumulation by default; the full-size (1.7B) restatement runs in
# f32 BLAS (set MV_F64 = False): ~1e-6 relative, still far inside the 1e-2 bar
MV_F64 = True


def mv(W, x):
    if not MV_F64:
        return (W @ np.asarray(x, np.float32)).astype(np.float32)
    return (W.astype(np.float64) @ np.asarray(x, np.float64)).astype(np.float32)


def layer_step(st: Stack, d, x, K, V, pos):
    """One decoder layer for one token (qwen_tts_talker.c:584-681 /
    cp_layer_body, qwen_tts_code_predictor.c:595-717).  K, V: contiguous bf16
    caches [max][kv_dim] of this layer, appended in place."""
    xn = rms_norm(x, d["input_norm"], st.eps)
    q = mv(d["wq"], xn)
    k = mv(d["wk"], xn)
    v = mv(d["wv"], xn)
    q = rms_norm_per_head(q, d["q_norm"], st.nh, st.hd, st.eps)
    k = rms_norm_per_head(k, d["k_norm"], st.nkv, st.hd, st.eps)
    q = rope_neox(q, st.nh, st.hd, st.cos, st.sin, pos)
    k = rope_neox(k, st.nkv, st.hd, st.cos, st.sin, pos)
    K[pos] = bf16_trunc(k)
    V[pos] = bf16_trunc(v)
    a = attention_bf16kv(q, K, V, st.nh, st.nkv, st.hd, pos + 1)
    x = (x + mv(d["wo"], a)).astype(np.float32)
    xn = rms_norm(x, d["post_attn_norm"], st.eps)
    h = swiglu(mv(d["gate_up"], xn))
    return (x + mv(d["down"], h)).astype(np.float32)


def stack_step(st: Stack, x, caches, pos):
    x = np.asarray(x, np.float32).copy()
    for i, d in enumerate(st.layers):
        x = layer_step(st, d, x, caches[i][0], caches[i][1], pos)
    return x


def new_caches(st: Stack, n):
    return [(np.zeros((n, st.nkv * st.hd), np.uint16), np.zeros((n, st.nkv * st.hd), np.uint16))
            for _ in st.layers]


def talker_step(st: Stack, embed, caches, pos):
    """qwen_talker_step (qwen_tts_talker.c:537-699) -> (hidden, dec_x)."""
    x = stack_step(st, embed, caches, pos)
    return rms_norm(x, st.final_norm, st.eps), x


def argmax_first(y):
    """First maximum wins (the reference scans with a strict '>')."""
    return int(np.argmax(y))


def cp_predict(cp: Stack, cp_norm, lm_heads, cp_emb, codec_emb, talker_hidden, code0, mtp=None, force=None,
               margins=None):
    """qwen_cp_predict (qwen_tts_code_predictor.c:926-1045), greedy heads.
    lm_heads: f32 [2048][cp_h] x 15; cp_emb / codec_emb: f32 tables;
    mtp: (W f32, b f32) or None.  force: codes to feed back instead of the
    argmax (teacher forcing); margins: list receiving (top1 - top2, logit std)
    per head."""
    def proj(v):
        if mtp is None:
            return np.asarray(v, np.float32)[: cp.H].copy()
        return (mv(mtp[0], v) + mtp[1]).astype(np.float32)

    caches = new_caches(cp, 64)
    x = stack_step(cp, proj(talker_hidden), caches, 0)
    x = stack_step(cp, proj(codec_emb[code0]), caches, 1)
    codes = []
    for g in range(15):
        logits = mv(lm_heads[g], rms_norm(x, cp_norm, cp.eps))
        c = argmax_first(logits)
        if margins is not None:
            top = np.sort(np.asarray(logits, np.float64))[-2:]
            margins.append((float(top[1] - top[0]), float(np.std(logits))))
        if force is not None:
            c = int(force[g])
        codes.append(c)
        if g == 14:
            break
        x = stack_step(cp, proj(cp_emb[g][c]), caches, g + 2)
    return np.array(codes, np.int32), caches


def lcg_next(state):
    """The reference's rand_uniform (qwen_tts_sampling.c:38-42): new state and draw."""
    state = (state * 1103515245 + 12345) & 0xFFFFFFFF
    return state, np.float32(((state >> 16) & 0x7FFF) / 32768.0)


def sample(logits, temp, top_k, top_p, seed):
    """qwen_tts_sample (qwen_tts_sampling.c:160-202) without the repetition
    penalty, in f32 with the reference's loop orders: softmax (max, exp of
    (x - max) * (1 / T), sequential sum, x * (1 / sum)), top-k (values below
    the k-th largest zeroed), top-p (descending until the running sum passes
    p), renormalisation, one LCG draw against the running sum in index order.
    Returns (token, LCG state, draw, the running sums) for boundary checks."""
    x = np.asarray(logits, np.float32).copy()
    n = x.shape[0]
    if temp < 1e-6:
        return int(np.argmax(x)), seed, None, None
    mx = np.float32(x.max())
    inv_t = np.float32(np.float32(1.0) / np.float32(temp))
    p = np.exp((x - mx) * inv_t).astype(np.float32)
    s = np.float32(0)
    for v in p:
        s = np.float32(s + v)
    p = (p * np.float32(np.float32(1.0) / s)).astype(np.float32)
    if 0 < top_k < n:
        thr = np.sort(p)[::-1][top_k - 1]
        p[p < thr] = 0
    if 0 < top_p < 1:
        order = sorted(range(n), key=lambda i: (-float(p[i]), i))
        cum = np.float32(0)
        keep = np.zeros(n, bool)
        for i in order:
            cum = np.float32(cum + p[i])
            keep[i] = True
            if cum > np.float32(top_p):
                break
        p[~keep] = 0
    s = np.float32(0)
    for v in p:
        s = np.float32(s + v)
    if s > 0:
        p = (p * np.float32(np.float32(1.0) / s)).astype(np.float32)
    seed, u = lcg_next(seed)
    cums = np.cumsum(p.astype(np.float64))
    run = np.float32(0)
    for i in range(n):
        run = np.float32(run + p[i])
        if u < run:
            return i, seed, float(u), cums
    return n - 1, seed, float(u), cums
