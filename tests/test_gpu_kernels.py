"""Per-kernel parity on the B200: the engine's tensor-core GEMV (all weight
formats, batch 1..64) and the fused QK-norm + RoPE + paged KV append + split-K
attention, against the numpy oracle (itself pinned to the reference in
test_oracle_pin.py).  Tolerances are far tighter than the 1e-2 relative L2
the reference's CPU kernels allow: f32 activations are carried as hi+lo
halves, so the GEMV error is ~1e-6 relative."""
import numpy as np
import pytest

import qtts_b200 as Q
import qtts_oracle as O
from models import rel_l2

pytestmark = pytest.mark.gpu

GEMV_TOL = 2e-5


def rand_w(rng, rows, cols):
    return Q.bf16_from_f32(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))


def oracle_gemv(fmt, q, W, x):
    rows, cols = W.shape
    if fmt == Q.FMT_BF16:
        return O.matvec_bf16(W, x)
    if fmt == Q.FMT_INT8:
        return O.matvec_int8(q["data"], q["row_scale"], x)
    if fmt == Q.FMT_Q4_0:
        return O.matvec_q4_0(q["data"], rows, cols, x)
    return O.matvec_int4g(q["data"], q["group_scale"], q["group_zero"], rows, cols, x)


@pytest.mark.parametrize("fmt", [Q.FMT_BF16, Q.FMT_INT8, Q.FMT_Q4_0, Q.FMT_INT4G32])
@pytest.mark.parametrize("rows,cols", [(256, 1024), (1024, 3072), (4096, 1024), (2048, 2048), (1024, 6144)])
@pytest.mark.parametrize("batch", [1, 2, 5, 8, 17, 64])
def test_gemv_matches_oracle(have_gpu, fmt, rows, cols, batch):
    rng = np.random.default_rng(rows * 7 + cols + batch + fmt)
    W = rand_w(rng, rows, cols)
    q = Q.quantize(W, fmt)
    x = rng.standard_normal((batch, cols), dtype=np.float32)
    y = Q.gemv(fmt, q, rows, cols, x)
    ref = oracle_gemv(fmt, q, W, x)
    for b in range(batch):
        assert rel_l2(y[b], ref[b]) < GEMV_TOL, (b, rel_l2(y[b], ref[b]))


def test_gemv_large_activations_and_zero_rows(have_gpu):
    rng = np.random.default_rng(9)
    W = rand_w(rng, 256, 1024)
    W[17] = 0
    x = (rng.standard_normal((3, 1024)) * 300).astype(np.float32)
    for fmt in (Q.FMT_BF16, Q.FMT_INT8, Q.FMT_Q4_0, Q.FMT_INT4G32):
        q = Q.quantize(W, fmt)
        y = Q.gemv(fmt, q, 256, 1024, x)
        ref = oracle_gemv(fmt, q, W, x)
        assert np.all(y[:, 17] == 0)
        assert rel_l2(y, ref) < GEMV_TOL


def make_attention_case(rng, B, pos, n_pages, nh=16, nkv=8, permute=True):
    hd = 128
    pt_stride = max(p // 16 + 1 for p in pos) + 2
    pool = rng.permutation(n_pages) if permute else np.arange(n_pages)
    pt = np.full((B, pt_stride), -1, np.int32)
    nxt = 0
    for b in range(B):
        for i in range(pos[b] // 16 + 1):
            pt[b, i] = pool[nxt]
            nxt += 1
    kp = Q.bf16_from_f32(rng.standard_normal((n_pages, nkv, 16, hd), dtype=np.float32))
    vp = Q.bf16_from_f32(rng.standard_normal((n_pages, nkv, 16, hd), dtype=np.float32))
    qkv = rng.standard_normal((B, (nh + 2 * nkv) * hd), dtype=np.float32)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    cs, sn = Q.rope_tables(1e6, hd, 8192)
    return qkv, kp, vp, pt, qn, kn, cs, sn


_MANY = [int(v) for v in np.random.default_rng(77).integers(0, 1500, 24)]


# the last two cases have more items than CTAs: CTAs take them in dynamic order
@pytest.mark.parametrize("pos,max_splits", [([0, 15, 16, 37], 4), ([200, 1, 513, 2047], 8), ([4095], 32),
                                            ([63, 64], 1), (_MANY, 1), (_MANY, 8)])
def test_attention_append_matches_oracle(have_gpu, pos, max_splits):
    rng = np.random.default_rng(sum(pos) + max_splits)
    B, nh, nkv, hd, eps = len(pos), 16, 8, 128, 1e-6
    n_pages = sum(p // 16 + 1 for p in pos) + 5
    qkv, kp, vp, pt, qn, kn, cs, sn = make_attention_case(rng, B, pos, n_pages)
    kp0, vp0 = kp.copy(), vp.copy()
    out = Q.attention(qkv, nh, nkv, qn, kn, eps, cs, sn, kp, vp, pt, np.array(pos, np.int32), max_splits)
    for b in range(B):
        p = pos[b]
        q = O.rope_neox(O.rms_norm_per_head(qkv[b, :nh * hd], qn, nh, hd, eps), nh, hd, cs, sn, p)
        k = O.rope_neox(O.rms_norm_per_head(qkv[b, nh * hd:(nh + nkv) * hd], kn, nkv, hd, eps), nkv, hd, cs, sn, p)
        v = qkv[b, (nh + nkv) * hd:]
        page, slot = pt[b, p // 16], p % 16
        got_k = kp[page, :, slot, :].reshape(-1)
        got_v = vp[page, :, slot, :].reshape(-1)
        # V append is a pure bf16 truncation: bit-exact
        assert np.array_equal(got_v, O.bf16_trunc(v))
        # K passes through QK-norm + RoPE first: equal up to one bf16 ulp
        dk = np.abs(got_k.astype(np.int32) - O.bf16_trunc(k).astype(np.int32))
        assert dk.max() <= 1 and np.mean(dk == 0) > 0.98
        K, V = O.gather_pages(kp, vp, pt[b], p + 1)
        ref = O.attention_bf16kv(q, K, V, nh, nkv, hd, p + 1)
        assert rel_l2(out[b], ref) < 1e-5, (b, rel_l2(out[b], ref))
    # nothing but the appended slots changed
    touched = np.zeros(kp.shape[:1] + kp.shape[2:3], bool)
    for b in range(B):
        touched[pt[b, pos[b] // 16], pos[b] % 16] = True
    for page in range(n_pages):
        for slot in range(16):
            if not touched[page, slot]:
                assert np.array_equal(kp[page, :, slot], kp0[page, :, slot])
                assert np.array_equal(vp[page, :, slot], vp0[page, :, slot])


def test_attention_tensor_cores_match_cuda_cores(have_gpu, monkeypatch):
    """With QTB_ATTN_TC=1 batch >= 8 decode attention runs its pages on the
    tensor cores (bf16 MMA, q and p as three bf16 parts, pages copied as
    swizzled TMA boxes); it gives the outputs of the CUDA-core page loop (the
    default) to f32 rounding and the same appended K/V bytes.  64 slots,
    lengths across page edges, splits in dynamic order."""
    rng = np.random.default_rng(91)
    pos = [15, 16, 17, 31, 32, 0, 1, 4095] + [int(v) for v in rng.integers(0, 3000, 56)]
    B, nh, nkv, hd, eps = len(pos), 16, 8, 128, 1e-6
    n_pages = sum(p // 16 + 1 for p in pos) + 3
    qkv, kp, vp, pt, qn, kn, cs, sn = make_attention_case(rng, B, pos, n_pages)
    outs, pools = {}, {}
    for mode in ("1", "0"):
        monkeypatch.setenv("QTB_ATTN_TC", mode)
        k2, v2 = kp.copy(), vp.copy()
        outs[mode] = Q.attention(qkv, nh, nkv, qn, kn, eps, cs, sn, k2, v2, pt, np.array(pos, np.int32), 16)
        pools[mode] = (k2, v2)
    assert np.array_equal(pools["1"][0], pools["0"][0]) and np.array_equal(pools["1"][1], pools["0"][1])
    for b in range(B):
        assert rel_l2(outs["1"][b], outs["0"][b]) < 1e-5, (b, pos[b], rel_l2(outs["1"][b], outs["0"][b]))
    # and against the restatement for a few slots
    for b in (0, 1, 7, 20):
        p = pos[b]
        q = O.rope_neox(O.rms_norm_per_head(qkv[b, :nh * hd], qn, nh, hd, eps), nh, hd, cs, sn, p)
        K, V = O.gather_pages(pools["1"][0], pools["1"][1], pt[b], p + 1)
        ref = O.attention_bf16kv(q, K, V, nh, nkv, hd, p + 1)
        assert rel_l2(outs["1"][b], ref) < 1e-5, (b, rel_l2(outs["1"][b], ref))


@pytest.mark.parametrize("scale", [1.0, 300.0, 1e-3])
def test_kv_append_bit_exact_vs_reference(have_gpu, scale):
    """Identical f32 q/k/v rows into the reference's own K/V append (its
    qwen_rms_norm_per_head from oracle/_ref, NeoX RoPE in its FMA order, bf16
    truncation: qwen_tts_talker.c:603-615) and into the engine's attention
    prologue: the appended K and V bytes must be identical, every element."""
    import platform
    import ctypes as C
    import refbind
    if platform.machine() in ("x86_64", "AMD64"):
        # the engine reproduces this host's rsqrtss (the reference's -ffast-math
        # 1/sqrtf) from a table it checks when it builds it
        assert Q.lib().qtb_qk_norm_mode() == 1
    L = refbind.ref_lib()
    rng = np.random.default_rng(int(scale * 1000) + 5)
    nh, nkv, hd, eps = 16, 8, 128, 1e-6
    pos = [int(p) for p in rng.integers(0, 4000, 64)]
    B = len(pos)
    n_pages = sum(p // 16 + 1 for p in pos) + 3
    qkv, kp, vp, pt, qn, kn, cs, sn = make_attention_case(rng, B, pos, n_pages)
    qkv = (qkv * np.float32(scale) * (1 + rng.random(qkv.shape[1], dtype=np.float32))).astype(np.float32)
    Q.attention(qkv, nh, nkv, qn, kn, eps, cs, sn, kp, vp, pt, np.array(pos, np.int32), 4)
    bad = 0
    for b in range(B):
        q = qkv[b, :nh * hd].copy()
        k = qkv[b, nh * hd:(nh + nkv) * hd].copy()
        v = qkv[b, (nh + nkv) * hd:].copy()
        k_ref = np.empty(nkv * hd, np.uint16)
        v_ref = np.empty(nkv * hd, np.uint16)
        L.qref_qk_norm_rope_append(refbind.p(q), refbind.p(k), refbind.p(v), nh, nkv, hd, refbind.p(qn),
                                   refbind.p(kn), C.c_float(eps), refbind.p(cs), refbind.p(sn), pos[b],
                                   refbind.p(k_ref), refbind.p(v_ref))
        page, slot = pt[b, pos[b] // 16], pos[b] % 16
        got_k = kp[page, :, slot, :].reshape(-1)
        got_v = vp[page, :, slot, :].reshape(-1)
        assert np.array_equal(got_v, v_ref), b
        bad += int(np.count_nonzero(got_k != k_ref))
    assert bad == 0, f"{bad} of {B * nkv * hd} K elements differ from the reference's bytes"


def test_attention_ignores_pool_slots_past_the_end(have_gpu):
    # slots after the newest token hold NaN in the pool: they must not reach
    # the output (neither through the scores nor through P.V)
    rng = np.random.default_rng(11)
    pos = [5, 37, 70]
    B, nh, nkv, hd, eps = len(pos), 16, 8, 128, 1e-6
    n_pages = sum(p // 16 + 1 for p in pos) + 2
    qkv, kp, vp, pt, qn, kn, cs, sn = make_attention_case(rng, B, pos, n_pages)
    nan = np.uint16(0x7FC0)
    for b in range(B):
        page = pt[b, pos[b] // 16]
        kp[page, :, pos[b] % 16 + 1:, :] = nan
        vp[page, :, pos[b] % 16 + 1:, :] = nan
    out = Q.attention(qkv, nh, nkv, qn, kn, eps, cs, sn, kp, vp, pt, np.array(pos, np.int32), 2)
    assert np.all(np.isfinite(out))
    for b in range(B):
        p = pos[b]
        q = O.rope_neox(O.rms_norm_per_head(qkv[b, :nh * hd], qn, nh, hd, eps), nh, hd, cs, sn, p)
        K, V = O.gather_pages(kp, vp, pt[b], p + 1)
        ref = O.attention_bf16kv(q, K, V, nh, nkv, hd, p + 1)
        assert rel_l2(out[b], ref) < 1e-5, (b, rel_l2(out[b], ref))


def test_attention_rejects_bad_page_table(have_gpu):
    rng = np.random.default_rng(4)
    qkv, kp, vp, pt, qn, kn, cs, sn = make_attention_case(rng, 1, [40], 8)
    pt[0, 1] = 99  # outside the pool: refused on the host before launch
    with pytest.raises(RuntimeError, match="page table"):
        Q.attention(qkv, 16, 8, qn, kn, 1e-6, cs, sn, kp, vp, pt, np.array([40], np.int32), 4)


def test_backend_vtable_matmat_bf16(have_gpu):
    """The reference's per-op backend entries (qwen_cuda_init / _matmat_bf16 /
    _matvec_bf16 / _free): row-major X [cols][B], Y [rows][B], shapes that are
    not multiples of the tile sizes, and a second call that hits the resident
    weight cache."""
    import ctypes as C
    L = Q.lib()
    L.qwen_cuda_init.restype = C.c_void_p
    L.qwen_cuda_free.argtypes = [C.c_void_p]
    L.qwen_cuda_matmat_bf16.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
    L.qwen_cuda_matvec_bf16.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]
    assert L.qwen_cuda_available() == 1
    ctx = L.qwen_cuda_init()
    assert ctx
    rng = np.random.default_rng(31)
    # the resident-weight cache is keyed by the host pointer, as in the
    # reference, whose weights live as long as the process: every matrix stays
    # alive here so no later one can reuse a freed address
    keep = []
    try:
        for rows, cols, B in [(100, 200, 1), (256, 1024, 3), (72, 640, 64)]:
            W = Q.bf16_from_f32(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
            keep.append(W)
            Wf = O.f32_from_bf16(W).astype(np.float64)
            for call in range(2):
                X = rng.standard_normal((cols, B), dtype=np.float32)
                Y = np.full((rows, B), np.nan, np.float32)
                L.qwen_cuda_matmat_bf16(ctx, Y.ctypes.data, W.ctypes.data, X.ctypes.data, rows, cols, B)
                assert L.qwen_cuda_last_error() == 0
                assert rel_l2(Y, Wf @ X.astype(np.float64)) < GEMV_TOL, (rows, cols, B, call)
        x = rng.standard_normal(200, dtype=np.float32)
        W = Q.bf16_from_f32(rng.standard_normal((100, 200), dtype=np.float32) * np.float32(0.02))
        keep.append(W)
        y = np.empty(100, np.float32)
        L.qwen_cuda_matvec_bf16(ctx, y.ctypes.data, W.ctypes.data, x.ctypes.data, 100, 200)
        assert rel_l2(y, O.f32_from_bf16(W).astype(np.float64) @ x) < GEMV_TOL
    finally:
        L.qwen_cuda_free(ctx)


def test_codec_sampler_matches_reference(have_gpu):
    """The device sampler of the codec head (softmax at a temperature, top-k,
    top-p, one draw of the reference's LCG) against the reference's
    qwen_tts_sample on the same logits: the LCG state always equal, the token
    equal except where the draw falls within f32 rounding (1e-5) of a
    cumulative-probability boundary (the sums run in another order)."""
    import refbind
    rng = np.random.default_rng(8)
    rows, n = 64, 2049
    for rep in range(4):
        lg = (rng.standard_normal((rows, n)) * rng.uniform(0.5, 4, (rows, 1))).astype(np.float32)
        lg[:, n - 1] = rng.choice([-1e30, 2.0], rows)          # the EOS row, masked or live
        temp = rng.choice([0.5, 0.9, 1.3], rows).astype(np.float32)
        top_k = rng.choice([0, 1, 20, 50, 5000], rows).astype(np.int32)
        top_p = rng.choice([1.0, 0.9, 0.5], rows).astype(np.float32)
        seed = rng.integers(0, 2 ** 32, rows, dtype=np.uint64).astype(np.uint32)
        got, st = Q.codec_sample(lg, temp, top_k, top_p, seed)
        near = 0
        for b in range(rows):
            want, wst = refbind.sample_logits(lg[b], float(temp[b]), int(top_k[b]), float(top_p[b]), int(seed[b]))
            assert int(st[b]) == wst, b
            if int(got[b]) != want:
                tok, _, u, cums = O.sample(lg[b], float(temp[b]), int(top_k[b]), float(top_p[b]), int(seed[b]))
                assert tok == want
                lo, hi = sorted((int(got[b]), want))
                assert np.min(np.abs(cums[lo:hi + 1] - u)) < 1e-5, (b, got[b], want)
                near += 1
        assert near <= 2, near
