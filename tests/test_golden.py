"""Pins the numpy restatement (oracle/) and the library's host encoders to
golden vectors produced by the reference itself (tests/golden/*.npz, made by
tests/golden/make_golden.py from oracle/_ref).  CPU only; needs neither the
reference tree nor a GPU."""
import os

import numpy as np
import pytest

import qtts_b200 as Q
import qtts_oracle as O
from models import kv_close, rel_l2, tiny_cfg

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def kern():
    return np.load(os.path.join(GOLD, "kernels.npz"))


def test_int8_and_q4_0_encoders_match_golden(kern):
    W = kern["W"]
    q, s = O.quantize_int8(W)
    assert np.array_equal(q, kern["q8"]) and np.array_equal(s, kern["s8"])
    lib8 = Q.quantize(W, Q.FMT_INT8)
    assert np.array_equal(lib8["data"], kern["q8"]) and np.array_equal(lib8["row_scale"], kern["s8"])
    lib4 = Q.quantize(W, Q.FMT_Q4_0)["data"]
    assert np.array_equal(lib4, kern["q4"])


def test_matvecs_match_golden(kern):
    W, x = kern["W"], kern["x"]
    rows, cols = W.shape
    assert rel_l2(O.matvec_bf16(W, x), kern["y_bf16"]) < 1e-6
    assert rel_l2(O.matvec_int8(kern["q8"], kern["s8"], x), kern["y_int8"]) < 1e-6
    assert rel_l2(O.matvec_q4_0(kern["q4"], rows, cols, x)[0], kern["y_q4_0"]) < 1e-6


def test_attention_norms_swiglu_match_golden(kern):
    nh, nkv, hd, L = (int(v) for v in kern["att_shape"])
    out = O.attention_bf16kv(kern["att_q"], kern["att_K"], kern["att_V"], nh, nkv, hd, L)
    assert rel_l2(out, kern["att_out"]) < 1e-5
    assert rel_l2(O.rms_norm(kern["xn"], kern["wn"], 1e-6), kern["yn"]) < 1e-6
    assert rel_l2(O.rms_norm_per_head(kern["xh"], kern["wh"], nh, hd, 1e-6), kern["yh"]) < 1e-6
    assert rel_l2(O.swiglu(kern["gu"]), kern["swiglu"]) < 1e-6


def test_tiny_model_steps_and_codes_match_golden():
    g = np.load(os.path.join(GOLD, "tiny_model.npz"))
    layers, cp_layers, hidden, inter = (int(v) for v in g["cfg"])
    cfg = tiny_cfg(layers=layers, cp_layers=cp_layers, hidden=hidden, inter=inter)
    m = Q.synth_model(cfg, seed=0, with_cp=True, norm_gain="random")
    tk = O.Stack(m.talker.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.inter, cfg.eps,
                 g["rope_cos"], g["rope_sin"], m.talker.final_norm)
    caches = O.new_caches(tk, 16)
    for pos, e in enumerate(g["embeds"]):
        h, _ = O.talker_step(tk, e, caches, pos)
        assert rel_l2(h, g["hidden"][pos]) < 1e-4, pos
    n = len(g["embeds"])
    for l in range(layers):
        assert kv_close(caches[l][0][:n], g["K"][l], 0.99) and kv_close(caches[l][1][:n], g["V"][l], 0.99), l
    cp = O.Stack(m.cp.layers, cfg.cp_hidden, cfg.cp_heads, cfg.cp_kv_heads, cfg.cp_head_dim, cfg.cp_inter, cfg.eps,
                 g["cp_rope_cos"], g["cp_rope_sin"])
    lm = [O.f32_from_bf16(w) for w in m.cp_lm_head]
    emb = [O.f32_from_bf16(w) for w in m.cp_codec_emb]
    cemb = O.f32_from_bf16(m.codec_embedding)
    for i in range(len(g["cp_code0"])):
        codes, _ = O.cp_predict(cp, m.cp_norm, lm, emb, cemb, g["cp_hidden"][i], int(g["cp_code0"][i]))
        assert np.array_equal(codes, g["cp_codes"][i]), i
