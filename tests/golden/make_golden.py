"""Generates the golden vectors in this folder from the reference itself.

Run where the reference's CPU sources are compiled (oracle/_ref, built by
`make -C oracle` from the reference tree):

    python tests/golden/make_golden.py

Every input is seeded; the outputs are the reference's own results
(oracle/_ref: qwen_tts_kernels.c, qwen_tts_talker.c, qwen_tts_code_predictor.c
compiled unmodified, with the f32-activation dispatch that the parity tests
use).  tests/test_golden.py checks the numpy restatement (oracle/) and the
library's host-side encoders against these files on any machine.
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "qwen3-tts_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
for _k in ("QWEN_NO_BF16DOT", "QWEN_NO_VNNI", "QWEN_NO_SDOT"):
    os.environ.setdefault(_k, "1")

import numpy as np  # noqa: E402

import qtts_b200 as Q  # noqa: E402
import refbind  # noqa: E402
from models import build, tiny_cfg  # noqa: E402

P = refbind.p


def kernels(R):
    rng = np.random.default_rng(1001)
    rows, cols = 64, 256
    W = Q.bf16_from_f32(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
    W[3] = 0            # an all-zero row (int8 scale 0)
    W[5, :32] = 0       # an all-zero q4_0 block
    x = rng.standard_normal(cols, dtype=np.float32)
    q8 = np.empty((rows, cols), np.int8)
    s8 = np.empty(rows, np.float32)
    R.qwen_quantize_bf16_to_int8(P(W), rows, cols, P(q8), P(s8))
    q4 = np.empty((rows, cols // 32 * 18), np.uint8)
    R.qwen_quantize_bf16_to_q4_0(P(W), rows, cols, P(q4))
    y_bf16 = np.empty(rows, np.float32)
    y_int8 = np.empty(rows, np.float32)
    y_q4 = np.empty(rows, np.float32)
    R.qwen_matvec_bf16(P(y_bf16), P(W), P(x), rows, cols)
    R.qwen_matvec_int8(P(y_int8), P(q8), P(s8), P(x), rows, cols)
    R.qwen_matvec_q4_0(P(y_q4), P(q4), P(x), rows, cols)
    # attention over a bf16 cache, norms, SwiGLU
    nh, nkv, hd, L = 4, 2, 128, 37
    q = rng.standard_normal(nh * hd, dtype=np.float32)
    K = Q.bf16_from_f32(rng.standard_normal((L, nkv * hd), dtype=np.float32))
    V = Q.bf16_from_f32(rng.standard_normal((L, nkv * hd), dtype=np.float32))
    att = np.empty(nh * hd, np.float32)
    R.qwen_causal_attention_bf16kv(P(att), P(q), P(K), P(V), 1, L, nh, nkv, hd, np.float32(1 / np.sqrt(128)), L - 1)
    xn = rng.standard_normal(1024, dtype=np.float32)
    wn = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    yn = np.empty(1024, np.float32)
    R.qwen_rms_norm(P(yn), P(xn), P(wn), 1, 1024, np.float32(1e-6))
    xh = rng.standard_normal(nh * hd, dtype=np.float32)
    wh = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    yh = xh.copy()
    R.qwen_rms_norm_per_head(P(yh), P(wh), 1, nh, hd, np.float32(1e-6))
    gu = rng.standard_normal(2 * 512, dtype=np.float32)
    sw = gu.copy()
    tmp = np.empty(512, np.float32)
    R.qwen_swiglu_inplace(P(sw), P(tmp), 512)
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), W=W, x=x, q8=q8, s8=s8, q4=q4, y_bf16=y_bf16,
                        y_int8=y_int8, y_q4_0=y_q4, att_q=q, att_K=K, att_V=V, att_out=att, att_shape=np.array(
                            [nh, nkv, hd, L]), xn=xn, wn=wn, yn=yn, xh=xh, wh=wh, yh=yh, gu=gu, swiglu=sw[:512])


def model():
    cfg = tiny_cfg(layers=2, cp_layers=2)
    m, path = build(cfg, seed=0, norm_gain="random")
    ref = refbind.RefModel(path, cfg, threads=4)
    rng = np.random.default_rng(1002)
    steps = 8
    E = (0.1 * rng.standard_normal((steps, cfg.hidden))).astype(np.float32)
    H = np.stack([ref.talker_step(E[i]) for i in range(steps)])
    Kc = np.stack([ref.kv(l, steps)[0] for l in range(cfg.layers)])
    Vc = np.stack([ref.kv(l, steps)[1] for l in range(cfg.layers)])
    cs, sn = ref.rope(False)
    ccs, csn = ref.rope(True)
    hid = rng.standard_normal((2, cfg.hidden)).astype(np.float32)
    code0 = rng.integers(0, 2048, 2).astype(np.int32)
    codes = np.stack([ref.cp_predict(hid[i], int(code0[i])) for i in range(2)])
    ref.close()
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), embeds=E, hidden=H, K=Kc, V=Vc,
                        rope_cos=cs[:64], rope_sin=sn[:64], cp_rope_cos=ccs[:32], cp_rope_sin=csn[:32],
                        cp_hidden=hid, cp_code0=code0, cp_codes=codes,
                        cfg=np.array([cfg.layers, cfg.cp_layers, cfg.hidden, cfg.inter]))


if __name__ == "__main__":
    kernels(refbind.ref_lib())
    model()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")
