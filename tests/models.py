"""Synthetic model fixtures shared by the CPU and GPU tests (seeded; the shapes
of the Qwen3-TTS 0.6B / 1.7B talker and code predictor, or smaller stacks)."""
import os
import tempfile

import numpy as np

import qtts_b200 as Q
import qtts_oracle as O
import refbind


def tiny_cfg(layers=2, cp_layers=2, hidden=1024, inter=3072):
    return Q.ModelCfg(hidden=hidden, layers=layers, inter=inter, cp_layers=cp_layers)


_cache = {}


def build(cfg, seed=0, norm_gain="random", with_cp=True, tmpdir=None):
    """(HostModel, safetensors path) for cfg; cached per process."""
    key = (tuple(sorted(cfg.__dict__.items())), seed, norm_gain, with_cp)
    if key in _cache:
        return _cache[key]
    m = Q.synth_model(cfg, seed=seed, with_cp=with_cp, norm_gain=norm_gain)
    d = tmpdir or tempfile.mkdtemp(prefix="qtb_st_")
    path = os.path.join(d, f"model_{abs(hash(key)) % 10**8}.safetensors")
    refbind.write_safetensors(path, refbind.model_tensors(m))
    _cache[key] = (m, path)
    return m, path


def ref_quantized(ref, cfg, fmt, cp=False, n_layers=None):
    """The reference's own quantized bytes for every matrix (so the engine is
    given byte-identical INT8 / q4_0 weights), keyed like Engine(quantized=)."""
    out = {}
    if fmt == "bf16":
        return out
    H = cfg.cp_hidden if cp else cfg.hidden
    I = cfg.cp_inter if cp else cfg.inter
    nh, nkv, hd = (cfg.cp_heads, cfg.cp_kv_heads, cfg.cp_head_dim) if cp else (cfg.heads, cfg.kv_heads, cfg.head_dim)
    L = n_layers if n_layers is not None else (cfg.cp_layers if cp else cfg.layers)
    shapes = {"wq": (nh * hd, H), "wk": (nkv * hd, H), "wv": (nkv * hd, H), "wo": (H, nh * hd),
              "gate_up": (2 * I, H), "down": (H, I)}
    which = {"wq": 0, "wk": 1, "wv": 2, "wo": 3, "gate_up": 4, "down": 5}
    pre = "c" if cp else "t"
    for l in range(L):
        for nm, (r, c) in shapes.items():
            if fmt == "int8":
                q = ref.weight(cp, l, which[nm], 1, r * c, np.int8).reshape(r, c)
                s = ref.weight(cp, l, which[nm], 2, r * 4, np.float32)
                out[f"{pre}{l}.{nm}"] = {"data": q, "row_scale": s}
            elif fmt == "q4_0":
                b = ref.weight(cp, l, which[nm], 3, r * (c // 32) * 18, np.uint8).reshape(r, c // 32 * 18)
                out[f"{pre}{l}.{nm}"] = {"data": b}
    if cp and cfg.hidden != cfg.cp_hidden and fmt in ("int8", "q4_0"):
        # the MTP projection's int8 twin (int8 under --int4 too)
        r, c = cfg.cp_hidden, cfg.hidden
        out["mtp"] = {"data": ref.cp_mtp(1, r * c, np.int8).reshape(r, c), "row_scale": ref.cp_mtp(2, r * 4, np.float32)}
    if cp:
        for g in range(15):
            r, c = cfg.codebook, cfg.cp_hidden
            if fmt == "int8":
                out[f"lm{g}"] = {"data": ref.lm_head(g, 1, r * c, np.int8).reshape(r, c),
                                 "row_scale": ref.lm_head(g, 2, r * 4, np.float32)}
            elif fmt == "q4_0":
                out[f"lm{g}"] = {"data": ref.lm_head(g, 3, r * (c // 32) * 18, np.uint8).reshape(r, c // 32 * 18)}
    return out


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def kv_close(a, b, min_equal=0.98):
    """bf16 KV caches computed from nearly equal f32 values: most bytes equal,
    and every element within one bf16 ulp of its magnitude or a tiny absolute
    floor (elements near zero after cancellation may differ by many ulps in bit
    pattern while differing by ~1e-7 absolute)."""
    fa = (np.asarray(a).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    fb = (np.asarray(b).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    rms = np.sqrt(np.mean(fb ** 2)) + 1e-30
    tol = 2.0 ** -6 * np.maximum(np.abs(fa), np.abs(fb)) + 2e-3 * rms
    ok = bool(np.all(np.abs(fa - fb) <= tol)) and float(np.mean(np.asarray(a) == np.asarray(b))) > min_equal
    if not ok:
        i = np.unravel_index(np.argmax(np.abs(fa - fb) - tol), fa.shape)
        print("kv_close: worst", i, fa[i], fb[i], "tol", tol[i], "equal", float(np.mean(np.asarray(a) == np.asarray(b))))
    return ok


def codec_margin(m, cfg, h):
    """(top1 - top2) / std of the codec-head logits on hidden h (float64)."""
    lg = O.f32_from_bf16(m.codec_head)[:cfg.codebook].astype(np.float64) @ np.asarray(h, np.float64)
    top = np.sort(lg)[-2:]
    return float((top[1] - top[0]) / lg.std())


def cp_margins(ref, m, cfg, fmt, h, code0, codes):
    """Relative top-2 margins ((top1 - top2) / std) of the 15 code-predictor
    heads for talker hidden h and code0, with the given codes fed back
    (float64 restatement on the reference's quantized bytes)."""
    q = ref_quantized(ref, cfg, fmt, cp=True)
    cq = {k[1:]: v for k, v in q.items() if k.startswith("c")}
    ccs, csn = ref.rope(True)
    cp = O.Stack(m.cp.layers, cfg.cp_hidden, cfg.cp_heads, cfg.cp_kv_heads, cfg.cp_head_dim, cfg.cp_inter, cfg.eps,
                 ccs, csn, None, fmt, cq or None)
    lm = [O.dequant(fmt, w, q.get(f"lm{g}")) for g, w in enumerate(m.cp_lm_head)]
    emb = [O.f32_from_bf16(w) for w in m.cp_codec_emb]
    margins = []
    O.cp_predict(cp, m.cp_norm, lm, emb, O.f32_from_bf16(m.codec_embedding), h, code0, force=codes, margins=margins)
    return [mg / sd for mg, sd in margins]


# A greedy fork between two implementations that agree to ~1e-4 is only
# acceptable at a near-tie: the reference's own top-2 logits closer than this
# fraction of the logit spread.
NEAR_TIE = 5e-3
