"""Pins the numpy oracle (oracle/qtts_oracle.py) against the reference itself
(oracle/_ref: the reference's CPU sources compiled unmodified), and the
engine's host-side encoders against the reference's quantizers.  CPU only."""
import numpy as np
import pytest

import qtts_b200 as Q
import qtts_oracle as O
import refbind
from models import build, kv_close, rel_l2, tiny_cfg

P = refbind.p


@pytest.fixture(scope="module")
def R():
    return refbind.ref_lib()


def rand_bf16(rng, rows, cols, std=0.02):
    return Q.bf16_from_f32(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std))


@pytest.mark.parametrize("rows,cols", [(256, 1024), (384, 3072), (128, 2048)])
def test_matvec_bf16_int8_q4_0_against_reference(R, rows, cols):
    rng = np.random.default_rng(rows + cols)
    W = rand_bf16(rng, rows, cols)
    x = rng.standard_normal(cols, dtype=np.float32)
    y = np.empty(rows, np.float32)
    R.qwen_matvec_bf16(P(y), P(W), P(x), rows, cols)
    assert rel_l2(O.matvec_bf16(W, x), y) < 1e-6
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.float32)
    R.qwen_quantize_bf16_to_int8(P(W), rows, cols, P(q), P(s))
    R.qwen_matvec_int8(P(y), P(q), P(s), P(x), rows, cols)
    assert rel_l2(O.matvec_int8(q, s, x), y) < 1e-6
    b = np.empty((rows, cols // 32 * 18), np.uint8)
    R.qwen_quantize_bf16_to_q4_0(P(W), rows, cols, P(b))
    R.qwen_matvec_q4_0(P(y), P(b), P(x), rows, cols)
    assert rel_l2(O.matvec_q4_0(b, rows, cols, x)[0], y) < 1e-6


@pytest.mark.parametrize("rows,cols", [(256, 1024), (200, 3072)])
def test_int8_encoder_bit_exact(R, rows, cols):
    rng = np.random.default_rng(7)
    W = rand_bf16(rng, rows, cols)
    W[3] = 0  # an all-zero row (scale 0)
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.float32)
    R.qwen_quantize_bf16_to_int8(P(W), rows, cols, P(q), P(s))
    mine = Q.quantize(W, Q.FMT_INT8)
    oq, os_ = O.quantize_int8(W)
    assert np.array_equal(mine["data"], q) and np.array_equal(mine["row_scale"], s)
    assert np.array_equal(oq, q) and np.array_equal(os_, s)


def test_q4_0_encoder_bit_exact(R):
    rng = np.random.default_rng(11)
    rows, cols = 256, 1024
    W = rand_bf16(rng, rows, cols)
    W[5, :32] = 0  # an all-zero block
    b = np.empty((rows, cols // 32 * 18), np.uint8)
    R.qwen_quantize_bf16_to_q4_0(P(W), rows, cols, P(b))
    mine = Q.quantize(W, Q.FMT_Q4_0)["data"]
    diff = np.any(mine.reshape(rows, -1, 18) != b.reshape(rows, -1, 18), axis=2)
    assert diff.sum() == 0, f"{diff.sum()} of {diff.size} q4_0 blocks differ"


def test_int4g32_encoder_matches_restatement():
    rng = np.random.default_rng(3)
    W = rand_bf16(rng, 256, 2048)
    W[0, :32] = W[0, 0]  # a flat group
    mine = Q.quantize(W, Q.FMT_INT4G32)
    c, s, z = O.quantize_int4g32(W)
    assert np.array_equal(mine["data"], c)
    assert np.array_equal(mine["group_scale"], s)
    assert np.array_equal(mine["group_zero"], z)
    # dequantization error of a 4-bit asymmetric code is at most half a step
    deq = O.dequant("int4g32", W, mine)
    step = O.f16_to_f32(s).repeat(32, axis=1)
    assert np.all(np.abs(deq - O.f32_from_bf16(W)) <= 0.5 * step + 1e-6)


def test_attention_norms_swiglu_against_reference(R):
    rng = np.random.default_rng(5)
    nh, nkv, hd, L = 16, 8, 128, 37
    q = rng.standard_normal(nh * hd, dtype=np.float32)
    K = Q.bf16_from_f32(rng.standard_normal((L, nkv * hd), dtype=np.float32))
    V = Q.bf16_from_f32(rng.standard_normal((L, nkv * hd), dtype=np.float32))
    out = np.empty(nh * hd, np.float32)
    R.qwen_causal_attention_bf16kv(P(out), P(q), P(K), P(V), 1, L, nh, nkv, hd, np.float32(1 / np.sqrt(128)), L - 1)
    assert rel_l2(O.attention_bf16kv(q, K, V, nh, nkv, hd, L), out) < 1e-5
    x = rng.standard_normal(1024, dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    y = np.empty(1024, np.float32)
    R.qwen_rms_norm(P(y), P(x), P(w), 1, 1024, np.float32(1e-6))
    assert rel_l2(O.rms_norm(x, w, 1e-6), y) < 1e-6
    xh = rng.standard_normal(nh * hd, dtype=np.float32)
    wh = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    yh = xh.copy()
    R.qwen_rms_norm_per_head(P(yh), P(wh), 1, nh, hd, np.float32(1e-6))
    assert rel_l2(O.rms_norm_per_head(xh, wh, nh, hd, 1e-6), yh) < 1e-6
    gu = rng.standard_normal(2 * 3072, dtype=np.float32)
    ref = gu.copy()
    tmp = np.empty(3072, np.float32)
    R.qwen_swiglu_inplace(P(ref), P(tmp), 3072)
    assert rel_l2(O.swiglu(gu), ref[:3072]) < 1e-6


@pytest.fixture(scope="module")
def tiny():
    cfg = tiny_cfg(layers=2, cp_layers=2)
    m, path = build(cfg)
    return cfg, m, path


def oracle_stacks(ref, cfg, m, fmt="bf16", q=None):
    cs, sn = ref.rope(False)
    ccs, csn = ref.rope(True)
    tk = O.Stack(m.talker.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.inter, cfg.eps, cs, sn,
                 m.talker.final_norm, fmt, q)
    cp = O.Stack(m.cp.layers, cfg.cp_hidden, cfg.cp_heads, cfg.cp_kv_heads, cfg.cp_head_dim, cfg.cp_inter, cfg.eps,
                 ccs, csn, None, fmt, None)
    return tk, cp


def test_talker_steps_match_reference(tiny):
    cfg, m, path = tiny
    ref = refbind.RefModel(path, cfg, threads=4)
    tk, _ = oracle_stacks(ref, cfg, m)
    caches = O.new_caches(tk, 64)
    rng = np.random.default_rng(1)
    for pos in range(20):
        e = (0.1 * rng.standard_normal(cfg.hidden)).astype(np.float32)
        h_ref = ref.talker_step(e)
        h_or, _ = O.talker_step(tk, e, caches, pos)
        assert rel_l2(h_or, h_ref) < 1e-4, pos
    for l in range(cfg.layers):
        k, v = ref.kv(l, 20)
        # bf16 truncation of nearly equal f32 values
        assert kv_close(caches[l][0][:20], k, 0.99) and kv_close(caches[l][1][:20], v, 0.99)
    ref.close()


def test_cp_predict_matches_reference(tiny):
    cfg, m, path = tiny
    ref = refbind.RefModel(path, cfg, threads=4)
    _, cp = oracle_stacks(ref, cfg, m)
    rng = np.random.default_rng(2)
    lm = [O.f32_from_bf16(w) for w in m.cp_lm_head]
    emb = [O.f32_from_bf16(w) for w in m.cp_codec_emb]
    cemb = O.f32_from_bf16(m.codec_embedding)
    for it in range(3):
        hidden = rng.standard_normal(cfg.hidden).astype(np.float32)
        code0 = int(rng.integers(0, 2048))
        codes_ref = ref.cp_predict(hidden, code0)
        codes_or, _ = O.cp_predict(cp, m.cp_norm, lm, emb, cemb, hidden, code0)
        assert np.array_equal(codes_ref, codes_or), (it, codes_ref, codes_or)
    ref.close()


def test_sampler_matches_reference():
    """The restated sampler (qtts_oracle.sample) draws the reference's
    qwen_tts_sample token and leaves its LCG in the same state, over random
    logits, temperatures, top-k and top-p settings."""
    rng = np.random.default_rng(1)
    for _ in range(120):
        lg = (rng.standard_normal(2049) * rng.uniform(0.5, 4)).astype(np.float32)
        temp = float(rng.choice([0.0, 0.5, 0.9, 1.3]))
        k = int(rng.choice([0, 1, 20, 50, 3000]))
        p = float(rng.choice([1.0, 0.9, 0.5]))
        seed = int(rng.integers(0, 2 ** 32))
        want = refbind.sample_logits(lg, temp, k, p, seed)
        got = O.sample(lg, temp, k, p, seed)
        assert (got[0], got[1]) == want, (temp, k, p, seed, got[:2], want)
