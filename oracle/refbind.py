"""refbind -- TEST INFRASTRUCTURE ONLY: ctypes access to the compiled reference.

Loads oracle/_ref/libqwen_ref_<isa>.so (the reference's own CPU decode path,
built from its unmodified sources by oracle/Makefile) and drives it the way the
reference's generation loop does (oracle/ref_harness.c).  Also writes the
synthetic safetensors file the reference loader reads (tensor names from
qwen_tts_talker.c:330-376 and qwen_tts_code_predictor.c:403-468).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module.  Nothing in the product imports it.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

F32_ACT_ENV = {"QWEN_NO_BF16DOT": "1", "QWEN_NO_VNNI": "1", "QWEN_NO_SDOT": "1"}


def cpu_flags() -> set:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def isa() -> str:
    fl = cpu_flags()
    need = {"avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512_vnni", "avx512_bf16"}
    return "avx512" if need <= fl else "avx2"


class Cfg(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("inter", C.c_int), ("codec_vocab", C.c_int), ("codebook", C.c_int),
                ("cp_hidden", C.c_int), ("cp_layers", C.c_int), ("cp_heads", C.c_int), ("cp_kv_heads", C.c_int),
                ("cp_head_dim", C.c_int), ("cp_inter", C.c_int), ("eps", C.c_float), ("theta", C.c_float)]


_libs = {}


def ref_lib(flavour: str | None = None, dropin: bool = False, refcuda: bool = False):
    """refcuda: the drop-in flavour linked with the reference's own CUDA
    talker / code predictor (qwen_tts_cuda_talker.cu built for sm_100a)."""
    flavour = flavour or isa()
    name = f"libqwen_ref_{'refcuda_' if refcuda else ('dropin_' if dropin else '')}{flavour}.so"
    if name in _libs:
        return _libs[name]
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        raise RuntimeError(f"oracle library missing: {path} (build with make -C oracle)")
    L = C.CDLL(path, mode=C.RTLD_GLOBAL if (dropin and not refcuda) else C.RTLD_LOCAL)
    vp = C.c_void_p
    L.qref_load.restype = vp
    L.qref_load.argtypes = [C.c_char_p, C.POINTER(Cfg), C.c_int, C.c_int]
    L.qref_talker_step.argtypes = [vp, vp, vp]
    L.qref_cp_predict.argtypes = [vp, vp, C.c_int, vp]
    L.qref_kv_len.argtypes = [vp]
    L.qref_kv_max.argtypes = [vp]
    L.qref_set_kv_len.argtypes = [vp, C.c_int]
    L.qref_copy_kv.argtypes = [vp, C.c_int, C.c_int, vp, vp]
    L.qref_copy_cp_kv.argtypes = [vp, C.c_int, C.c_int, vp, vp]
    L.qref_codec_argmax.argtypes = [vp, vp, C.c_int]
    L.qref_codec_embed.argtypes = [vp, C.c_int, vp]
    L.qref_codec_sample.argtypes = [vp, vp, C.c_int, C.c_int, C.c_float, vp, C.c_int]
    L.qref_codec_sample_t.argtypes = [vp, vp, C.c_int, C.c_int, C.c_float, vp, C.c_int, C.c_float, C.c_int,
                                      C.c_float, vp]
    L.qref_sample_logits.argtypes = [vp, C.c_int, C.c_float, C.c_int, C.c_float, vp]
    L.qref_talker_prefill.argtypes = [vp, vp, C.c_int, vp]
    L.qref_weight.restype = vp
    L.qref_weight.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int]
    L.qref_cp_mtp.restype = vp
    L.qref_cp_mtp.argtypes = [vp, C.c_int]
    L.qref_cp_lm_head.restype = vp
    L.qref_cp_lm_head.argtypes = [vp, C.c_int, C.c_int]
    L.qref_free.argtypes = [vp]
    L.qref_rope.restype = vp
    L.qref_rope.argtypes = [vp, C.c_int, C.c_int]
    L.qref_rope_len.argtypes = [vp, C.c_int]
    L.qref_set_threads.argtypes = [C.c_int]
    L.qref_qk_norm_rope_append.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, C.c_float, vp, vp, C.c_int,
                                           vp, vp]
    L.qref_ctx.restype = vp
    L.qref_ctx.argtypes = [vp]
    # the reference's own kernels, exported by the same library
    L.qwen_matvec_bf16.argtypes = [vp, vp, vp, C.c_int, C.c_int]
    L.qwen_matvec_int8.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int]
    L.qwen_matvec_q4_0.argtypes = [vp, vp, vp, C.c_int, C.c_int]
    L.qwen_quantize_bf16_to_int8.argtypes = [vp, C.c_int, C.c_int, vp, vp]
    L.qwen_quantize_bf16_to_q4_0.argtypes = [vp, C.c_int, C.c_int, vp]
    L.qwen_causal_attention_bf16kv.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                               C.c_float, C.c_int]
    L.qwen_rms_norm.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_float]
    L.qwen_rms_norm_per_head.argtypes = [vp, vp, C.c_int, C.c_int, C.c_int, C.c_float]
    L.qwen_swiglu_inplace.argtypes = [vp, vp, C.c_int]
    L.qwen_argmax_matvec_bf16.argtypes = [vp, vp, C.c_int, C.c_int]
    if dropin or refcuda:
        L.qref_dropin_attach.argtypes = [vp, C.c_int, C.c_int]
    _libs[name] = L
    return L


def p(a):
    return a.ctypes.data_as(C.c_void_p)


# ------------------------------------------------------- safetensors writer --
def write_safetensors(path: str, tensors: dict):
    """tensors: name -> (dtype_str, shape, ndarray) with dtype 'BF16' (uint16
    bits) or 'F32'."""
    header = {}
    off = 0
    items = []
    for name, (dt, shape, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        items.append(b)
        off += len(b)
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in items:
            f.write(b)


def model_tensors(m) -> dict:
    """Reference tensor names for a qtts_b200.HostModel (bf16 weights)."""
    t = {}
    cfg = m.cfg
    t["talker.model.text_embedding.weight"] = ("BF16", (1, 2048), np.zeros((1, 2048), np.uint16))

    def layer(prefix, ly):
        t[f"{prefix}.self_attn.q_proj.weight"] = ("BF16", ly.wq.shape, ly.wq)
        t[f"{prefix}.self_attn.k_proj.weight"] = ("BF16", ly.wk.shape, ly.wk)
        t[f"{prefix}.self_attn.v_proj.weight"] = ("BF16", ly.wv.shape, ly.wv)
        t[f"{prefix}.self_attn.o_proj.weight"] = ("BF16", ly.wo.shape, ly.wo)
        t[f"{prefix}.self_attn.q_norm.weight"] = ("F32", ly.q_norm.shape, ly.q_norm)
        t[f"{prefix}.self_attn.k_norm.weight"] = ("F32", ly.k_norm.shape, ly.k_norm)
        t[f"{prefix}.input_layernorm.weight"] = ("F32", ly.input_norm.shape, ly.input_norm)
        t[f"{prefix}.post_attention_layernorm.weight"] = ("F32", ly.post_attn_norm.shape, ly.post_attn_norm)
        gate = np.ascontiguousarray(ly.gate_up[0::2])
        up = np.ascontiguousarray(ly.gate_up[1::2])
        t[f"{prefix}.mlp.gate_proj.weight"] = ("BF16", gate.shape, gate)
        t[f"{prefix}.mlp.up_proj.weight"] = ("BF16", up.shape, up)
        t[f"{prefix}.mlp.down_proj.weight"] = ("BF16", ly.down.shape, ly.down)

    for i, ly in enumerate(m.talker.layers):
        layer(f"talker.model.layers.{i}", ly)
    t["talker.model.norm.weight"] = ("F32", m.talker.final_norm.shape, m.talker.final_norm)
    t["talker.codec_head.weight"] = ("BF16", m.codec_head.shape, m.codec_head)
    t["talker.model.codec_embedding.weight"] = ("BF16", m.codec_embedding.shape, m.codec_embedding)
    if m.cp is not None:
        for i, ly in enumerate(m.cp.layers):
            layer(f"talker.code_predictor.model.layers.{i}", ly)
        t["talker.code_predictor.model.norm.weight"] = ("F32", m.cp_norm.shape, m.cp_norm)
        for g in range(15):
            t[f"talker.code_predictor.lm_head.{g}.weight"] = ("BF16", m.cp_lm_head[g].shape, m.cp_lm_head[g])
            t[f"talker.code_predictor.model.codec_embedding.{g}.weight"] = ("BF16", m.cp_codec_emb[g].shape,
                                                                            m.cp_codec_emb[g])
        if m.mtp_w is not None:
            t["talker.code_predictor.small_to_mtp_projection.weight"] = ("BF16", m.mtp_w.shape, m.mtp_w)
            t["talker.code_predictor.small_to_mtp_projection.bias"] = ("BF16", m.mtp_b.shape, m.mtp_b)
    return t


class RefModel:
    """The reference's talker + CP loaded from a synthetic safetensors file."""

    def __init__(self, st_path: str, cfg, use_int8=False, use_int4=False, threads=None, flavour=None,
                 dropin=False, cp=True, refcuda=False):
        self.L = ref_lib(flavour, dropin=dropin, refcuda=refcuda)
        self.cfg = cfg
        c = Cfg(cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.inter, cfg.codec_vocab,
                cfg.codebook, cfg.cp_hidden, cfg.cp_layers if cp else 0, cfg.cp_heads, cfg.cp_kv_heads,
                cfg.cp_head_dim, cfg.cp_inter, cfg.eps, cfg.theta)
        if threads is not None:
            self.L.qref_set_threads(int(threads))
        h = self.L.qref_load(st_path.encode(), C.byref(c), int(use_int8), int(use_int4))
        if not h:
            raise RuntimeError("reference load failed")
        self.h = h

    def close(self):
        if self.h:
            self.L.qref_free(self.h)
            self.h = None

    def talker_step(self, embed):
        out = np.empty(self.cfg.hidden, np.float32)
        e = np.ascontiguousarray(embed, np.float32)
        rc = self.L.qref_talker_step(self.h, p(e), p(out))
        if rc:
            raise RuntimeError("qwen_talker_step failed")
        return out

    def cp_predict(self, hidden, code0):
        out = np.empty(15, np.int32)
        hh = np.ascontiguousarray(hidden, np.float32)
        if self.L.qref_cp_predict(self.h, p(hh), int(code0), p(out)):
            raise RuntimeError("qwen_cp_predict failed")
        return out

    @property
    def kv_len(self):
        return self.L.qref_kv_len(self.h)

    def set_kv_len(self, n):
        self.L.qref_set_kv_len(self.h, n)

    def kv(self, layer, n):
        kvd = self.cfg.kv_heads * self.cfg.head_dim
        k = np.empty((n, kvd), np.uint16)
        v = np.empty((n, kvd), np.uint16)
        self.L.qref_copy_kv(self.h, layer, n, p(k), p(v))
        return k, v

    def cp_kv(self, layer, n):
        kvd = self.cfg.cp_kv_heads * self.cfg.cp_head_dim
        k = np.empty((n, kvd), np.uint16)
        v = np.empty((n, kvd), np.uint16)
        self.L.qref_copy_cp_kv(self.h, layer, n, p(k), p(v))
        return k, v

    def codec_argmax(self, hidden, limit=None):
        hh = np.ascontiguousarray(hidden, np.float32)
        return self.L.qref_codec_argmax(self.h, p(hh), int(limit or self.cfg.codebook))

    def talker_prefill(self, embeds):
        """The reference's CPU prefill of embeds [n][hidden] at positions 0..n-1;
        returns dec_x (the last token's pre-norm residual)."""
        e = np.ascontiguousarray(embeds, np.float32)
        dx = np.empty(self.cfg.hidden, np.float32)
        if self.L.qref_talker_prefill(self.h, p(e), e.shape[0], p(dx)) != 0:
            raise RuntimeError("reference prefill failed")
        return dx

    def codec_sample(self, hidden, frame, expected_frames, rep_penalty, prev_tokens):
        """code0 under the reference's generation-loop rules (qref_codec_sample)."""
        hh = np.ascontiguousarray(hidden, np.float32)
        prev = np.ascontiguousarray(prev_tokens if len(prev_tokens) else [0], np.int32)
        return self.L.qref_codec_sample(self.h, p(hh), int(frame), int(expected_frames), C.c_float(rep_penalty),
                                        p(prev), len(prev_tokens))

    def codec_sample_t(self, hidden, frame, expected_frames, rep_penalty, prev_tokens, temp, top_k, top_p, seed):
        """code0 with the reference's sampling; returns (code, LCG state after the draw)."""
        hh = np.ascontiguousarray(hidden, np.float32)
        prev = np.ascontiguousarray(prev_tokens if len(prev_tokens) else [0], np.int32)
        st = np.array([seed], np.uint32)
        c = self.L.qref_codec_sample_t(self.h, p(hh), int(frame), int(expected_frames), C.c_float(rep_penalty),
                                       p(prev), len(prev_tokens), C.c_float(temp), int(top_k), C.c_float(top_p),
                                       p(st))
        return c, int(st[0])

    def codec_embed(self, code):
        out = np.empty(self.cfg.hidden, np.float32)
        self.L.qref_codec_embed(self.h, int(code), p(out))
        return out

    def weight(self, cp, layer, which, kind, nbytes, dtype):
        addr = self.L.qref_weight(self.h, int(cp), int(layer), int(which), int(kind))
        if not addr:
            return None
        return np.ctypeslib.as_array((C.c_uint8 * nbytes).from_address(addr)).view(dtype).copy()

    def lm_head(self, g, kind, nbytes, dtype):
        addr = self.L.qref_cp_lm_head(self.h, int(g), int(kind))
        if not addr:
            return None
        return np.ctypeslib.as_array((C.c_uint8 * nbytes).from_address(addr)).view(dtype).copy()

    def cp_mtp(self, kind, nbytes, dtype):
        """The reference's MTP projection pieces (qref_cp_mtp kinds), or None."""
        addr = self.L.qref_cp_mtp(self.h, int(kind))
        if not addr:
            return None
        return np.frombuffer((C.c_char * nbytes).from_address(addr), dtype=dtype).copy()

    def rope(self, cp=False):
        n = self.L.qref_rope_len(self.h, int(cp))
        hd = self.cfg.cp_head_dim if cp else self.cfg.head_dim
        out = []
        for which in (0, 1):
            addr = self.L.qref_rope(self.h, int(cp), which)
            out.append(np.ctypeslib.as_array((C.c_float * (n * hd // 2)).from_address(addr)).reshape(n, hd // 2).copy())
        return out[0], out[1]

    def ctx(self):
        return self.L.qref_ctx(self.h)


def sample_logits(logits, temp, top_k, top_p, seed, flavour=None):
    """The reference's qwen_tts_sample on given logits (no repetition
    penalty); returns (token, LCG state after the draw)."""
    L = ref_lib(flavour)
    lg = np.ascontiguousarray(logits, np.float32)
    st = np.array([seed], np.uint32)
    c = L.qref_sample_logits(p(lg), lg.shape[0], C.c_float(temp), int(top_k), C.c_float(top_p), p(st))
    return c, int(st[0])
