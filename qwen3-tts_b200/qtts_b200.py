"""qtts_b200 -- Python host bindings (ctypes) of the B200 decode engine.

The engine is the C ABI in include/qwen3tts_b200.h, implemented by
lib/libqwen3tts_b200.so (CUDA, sm_100a).  This module only marshals numpy
arrays into the C descriptors and provides the synthetic model builder used by
bench.py and the tests (random-init weights of the Qwen3-TTS shapes, since no
checkpoint is available).  It never computes anything itself and it raises if
the native library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(HERE, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libqwen3tts_b200.so")
DROPIN_PATH = os.path.join(LIB_DIR, "libqwen_tts_cuda_b200.so")

FMT_BF16, FMT_INT8, FMT_Q4_0, FMT_INT4G32 = 0, 1, 2, 3
FMT_NAMES = {"bf16": FMT_BF16, "int8": FMT_INT8, "q4_0": FMT_Q4_0, "int4g32": FMT_INT4G32}

_vp = C.c_void_p
_fp = C.POINTER(C.c_float)


class Matrix(C.Structure):
    _fields_ = [("data", _vp), ("row_scale", _vp), ("group_scale", _vp), ("group_zero", _vp)]


class Layer(C.Structure):
    _fields_ = [("wq", Matrix), ("wk", Matrix), ("wv", Matrix), ("wo", Matrix), ("gate_up", Matrix),
                ("down", Matrix), ("input_norm", _vp), ("post_attn_norm", _vp), ("q_norm", _vp), ("k_norm", _vp)]


class StackDesc(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("inter", C.c_int), ("eps", C.c_float), ("fmt", C.c_int),
                ("layers", C.POINTER(Layer)), ("rope_cos", _vp), ("rope_sin", _vp), ("rope_len", C.c_int),
                ("rope_theta", C.c_float), ("final_norm", _vp)]


class EngineDesc(C.Structure):
    _fields_ = [("talker", StackDesc), ("codec_head", _vp), ("codec_embedding", _vp), ("codec_vocab", C.c_int),
                ("codebook", C.c_int), ("has_cp", C.c_int), ("cp", StackDesc), ("cp_norm", _vp),
                ("cp_lm_head", Matrix * 15), ("cp_codec_emb", _vp * 15), ("cp_emb_dim", C.c_int),
                ("cp_mtp_proj", Matrix), ("cp_mtp_fmt", C.c_int), ("cp_mtp_bias", _vp),
                ("talker_prefill_layers", C.POINTER(Layer))]


_lib = None


CODEC_EOS = 2150   # QWEN_TTS_CODEC_EOS (qwen_tts.h:49)
NCKPT = 32   # intra-stage profiling checkpoints per stage (kernel constant)


def lib():
    """Load libqwen3tts_b200.so (raises when it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"native engine not built: {LIB_PATH} missing (run __graft_entry__.build())")
    L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
    L.qtb_last_error.restype = C.c_char_p
    L.qtb_engine_create.argtypes = [C.POINTER(EngineDesc), C.c_int, C.POINTER(_vp)]
    L.qtb_engine_destroy.argtypes = [_vp]
    for n in ("qtb_engine_talker_weight_bytes", "qtb_engine_cp_pass_weight_bytes", "qtb_engine_cp_head_weight_bytes"):
        getattr(L, n).argtypes = [_vp]
        getattr(L, n).restype = C.c_int64
    L.qtb_session_create.argtypes = [_vp, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
    L.qtb_session_destroy.argtypes = [_vp]
    L.qtb_session_last_ms.argtypes = [_vp]
    L.qtb_session_last_ms.restype = C.c_double
    L.qtb_session_last_launches.argtypes = [_vp]
    for n in ("qtb_session_batch", "qtb_session_n_pages", "qtb_session_max_ctx"):
        getattr(L, n).argtypes = [_vp]
    L.qtb_session_set_pages.argtypes = [_vp, C.c_int, _vp, C.c_int]
    L.qtb_session_set_pos.argtypes = [_vp, _vp]
    L.qtb_session_get_pos.argtypes = [_vp, _vp]
    L.qtb_session_get_dec_x.argtypes = [_vp, _vp]
    L.qtb_talker_step.argtypes = [_vp, _vp, _vp, _vp, _vp]
    L.qtb_cp_pass.argtypes = [_vp, _vp, _vp]
    L.qtb_cp_frame.argtypes = [_vp, _vp, _vp, _vp]
    L.qtb_decode_frames.argtypes = [_vp, _vp, _vp, C.c_int, _vp, _vp]
    L.qtb_session_begin_generation.argtypes = [_vp, _vp, C.c_float]
    L.qtb_prefill.argtypes = [_vp, C.c_int, _vp, C.c_int, C.c_int, _vp, _vp]
    L.qtb_session_program_grid.argtypes = [_vp, C.c_int]
    L.qtb_tc_plan.argtypes = [C.c_int] * 6 + [_vp]
    L.qtb_session_set_sampling.argtypes = [_vp, C.c_int, C.c_float, C.c_int, C.c_float, C.c_uint32]
    L.qtb_session_get_rng.argtypes = [_vp, _vp]
    L.qtb_codec_sample_host.argtypes = [_vp, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp]
    L.qtb_session_reset_slot.argtypes = [_vp, C.c_int, C.c_int, C.c_int]
    L.qtb_session_set_slot_pos.argtypes = [_vp, C.c_int, C.c_int]
    L.qtb_session_set_embed.argtypes = [_vp, C.c_int, _vp]
    L.qtb_session_get_done.argtypes = [_vp, _vp]
    for n in ("qtb_session_upload_kv", "qtb_session_download_kv", "qtb_session_download_cp_kv"):
        getattr(L, n).argtypes = [_vp, C.c_int, _vp, _vp, C.c_int, C.c_int]
    L.qtb_session_profile.argtypes = [_vp, C.c_int, _vp, _vp, _vp, C.c_int]
    L.qtb_session_profile_checkpoints.argtypes = [_vp, _vp, C.c_int]
    L.qtb_session_profile_arrivals.argtypes = [_vp, _vp, C.c_int]
    L.qtb_quantize_int8.argtypes = [_vp, C.c_int, C.c_int, _vp, _vp]
    L.qtb_quantize_q4_0.argtypes = [_vp, C.c_int, C.c_int, _vp]
    L.qtb_quantize_int4g32.argtypes = [_vp, C.c_int, C.c_int, _vp, _vp, _vp]
    L.qtb_gemv_host.argtypes = [C.c_int, C.POINTER(Matrix), C.c_int, C.c_int, _vp, C.c_int, _vp]
    L.qtb_attention_host.argtypes = [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, C.c_float, _vp, _vp,
                                     C.c_int, _vp, _vp, C.c_int, _vp, C.c_int, _vp, C.c_int, _vp]
    _lib = L
    return L


def check(rc):
    if rc != 0:
        raise RuntimeError(f"qwen3tts_b200 error {rc}: {lib().qtb_last_error().decode()}")


def ptr(a):
    return None if a is None else a.ctypes.data_as(_vp)


# ------------------------------------------------------------ model config --
@dataclass
class ModelCfg:
    hidden: int = 1024
    layers: int = 28
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 3072
    codec_vocab: int = 3072
    codebook: int = 2048
    cp_hidden: int = 1024
    cp_layers: int = 5
    cp_heads: int = 16
    cp_kv_heads: int = 8
    cp_head_dim: int = 128
    cp_inter: int = 3072
    eps: float = 1e-6
    theta: float = 1e6

    @property
    def cp_emb_dim(self):
        return self.hidden


CFG_06B = ModelCfg()
CFG_17B = ModelCfg(hidden=2048, inter=6144)


def bf16_from_f32(a: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bits by truncation (the synthetic weights' rounding rule)."""
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def f32_from_bf16(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


@dataclass
class HostLayer:
    wq: np.ndarray
    wk: np.ndarray
    wv: np.ndarray
    wo: np.ndarray
    gate_up: np.ndarray          # row-interleaved g0,u0,g1,u1,...
    down: np.ndarray
    input_norm: np.ndarray
    post_attn_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray


@dataclass
class HostStack:
    layers: list
    final_norm: np.ndarray | None = None


@dataclass
class HostModel:
    cfg: ModelCfg
    talker: HostStack
    codec_head: np.ndarray
    codec_embedding: np.ndarray
    cp: HostStack | None = None
    cp_norm: np.ndarray | None = None
    cp_lm_head: list = field(default_factory=list)
    cp_codec_emb: list = field(default_factory=list)
    mtp_w: np.ndarray | None = None
    mtp_b: np.ndarray | None = None


def synth_model(cfg: ModelCfg, seed: int = 0, with_cp: bool = True, norm_gain: str = "ones",
                std: float = 0.02) -> HostModel:
    """Random-init weights of the Qwen3-TTS shapes: N(0, std) f32 truncated to
    bf16, norm gains 1 (or 1 + N(0, 0.1) with norm_gain='random')."""
    rng = np.random.default_rng(seed)

    def w(rows, cols):
        return bf16_from_f32(rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std))

    def g(n):
        if norm_gain == "ones":
            return np.ones(n, np.float32)
        return (1.0 + 0.1 * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)

    def stack(H, L, nh, nkv, hd, I):
        layers = []
        for _ in range(L):
            gate, up = w(I, H), w(I, H)
            gu = np.empty((2 * I, H), np.uint16)
            gu[0::2] = gate
            gu[1::2] = up
            layers.append(HostLayer(w(nh * hd, H), w(nkv * hd, H), w(nkv * hd, H), w(H, nh * hd), gu, w(H, I),
                                    g(H), g(H), g(hd), g(hd)))
        return layers

    talker = HostStack(stack(cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.inter), g(cfg.hidden))
    m = HostModel(cfg, talker, w(cfg.codec_vocab, cfg.hidden), w(cfg.codec_vocab, cfg.hidden))
    if with_cp:
        m.cp = HostStack(stack(cfg.cp_hidden, cfg.cp_layers, cfg.cp_heads, cfg.cp_kv_heads, cfg.cp_head_dim,
                               cfg.cp_inter))
        m.cp_norm = g(cfg.cp_hidden)
        m.cp_lm_head = [w(cfg.codebook, cfg.cp_hidden) for _ in range(15)]
        m.cp_codec_emb = [w(cfg.codebook, cfg.cp_emb_dim) for _ in range(15)]
        if cfg.hidden != cfg.cp_hidden:
            m.mtp_w = w(cfg.cp_hidden, cfg.hidden)
            m.mtp_b = bf16_from_f32(rng.standard_normal(cfg.cp_hidden, dtype=np.float32) * np.float32(std))
    return m


# ------------------------------------------------------- quantized storage --
def quantize(w_bf16: np.ndarray, fmt: int) -> dict:
    """Encode a bf16 matrix in an engine format with the library's encoders."""
    L = lib()
    rows, cols = w_bf16.shape
    src = np.ascontiguousarray(w_bf16)
    if fmt == FMT_BF16:
        return {"data": src}
    if fmt == FMT_INT8:
        q = np.empty((rows, cols), np.int8)
        s = np.empty(rows, np.float32)
        check(L.qtb_quantize_int8(ptr(src), rows, cols, ptr(q), ptr(s)))
        return {"data": q, "row_scale": s}
    if fmt == FMT_Q4_0:
        b = np.empty((rows, cols // 32 * 18), np.uint8)
        check(L.qtb_quantize_q4_0(ptr(src), rows, cols, ptr(b)))
        return {"data": b}
    if fmt == FMT_INT4G32:
        c = np.empty((rows, cols // 2), np.uint8)
        s = np.empty((rows, cols // 32), np.uint16)
        z = np.empty((rows, cols // 32), np.uint16)
        check(L.qtb_quantize_int4g32(ptr(src), rows, cols, ptr(c), ptr(s), ptr(z)))
        return {"data": c, "group_scale": s, "group_zero": z}
    raise ValueError(fmt)


def matrix(q: dict) -> Matrix:
    return Matrix(ptr(q.get("data")), ptr(q.get("row_scale")), ptr(q.get("group_scale")), ptr(q.get("group_zero")))


def rope_tables(theta: float, head_dim: int, n: int):
    """cos/sin [n][head_dim/2] f32 (qwen_tts_talker.c:478-495 formula)."""
    half = head_dim // 2
    inv = (1.0 / np.power(np.float32(theta), (np.arange(half, dtype=np.float32) * 2) / np.float32(head_dim))).astype(np.float32)
    ang = np.arange(n, dtype=np.float32)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


class Engine:
    """Weights of the talker (+ code predictor) resident on one device."""

    def __init__(self, model: HostModel, talker_fmt: int = FMT_BF16, cp_fmt: int | None = None, device: int = 0,
                 rope=None, cp_rope=None, quantized=None, prefill_bf16=True):
        """prefill_bf16: with a quantized talker, also keep its bf16 weights for
        qtb_prefill, as the reference prefills from bf16 in every mode."""
        L = lib()
        cfg = model.cfg
        self.cfg = cfg
        self._keep = []
        quantized = quantized or {}

        def enc(key, w, fmt):
            q = quantized.get(key) or quantize(w, fmt)
            self._keep.append(q)
            return matrix(q)

        def stack_desc(st: HostStack, prefix, H, L_, nh, nkv, hd, I, fmt, rope_t, theta):
            arr = (Layer * L_)()
            for i, ly in enumerate(st.layers):
                for nm in ("input_norm", "post_attn_norm", "q_norm", "k_norm"):
                    self._keep.append(getattr(ly, nm))
                arr[i] = Layer(enc(f"{prefix}{i}.wq", ly.wq, fmt), enc(f"{prefix}{i}.wk", ly.wk, fmt),
                               enc(f"{prefix}{i}.wv", ly.wv, fmt), enc(f"{prefix}{i}.wo", ly.wo, fmt),
                               enc(f"{prefix}{i}.gate_up", ly.gate_up, fmt), enc(f"{prefix}{i}.down", ly.down, fmt),
                               ptr(ly.input_norm), ptr(ly.post_attn_norm), ptr(ly.q_norm), ptr(ly.k_norm))
            self._keep.append(arr)
            cs, sn = rope_t if rope_t is not None else rope_tables(theta, hd, 8192 if prefix == "t" else 64)
            self._keep += [cs, sn]
            if st.final_norm is not None:
                self._keep.append(st.final_norm)
            return StackDesc(H, L_, nh, nkv, hd, I, cfg.eps, fmt, arr, ptr(cs), ptr(sn), cs.shape[0], cfg.theta,
                             ptr(st.final_norm))

        d = EngineDesc()
        if model.talker is not None and len(model.talker.layers) > 0:
            d.talker = stack_desc(model.talker, "t", cfg.hidden, len(model.talker.layers), cfg.heads, cfg.kv_heads,
                                  cfg.head_dim, cfg.inter, talker_fmt, rope, cfg.theta)
            d.codec_head = ptr(model.codec_head)
            if prefill_bf16 and talker_fmt != FMT_BF16:
                pf = stack_desc(model.talker, "pf", cfg.hidden, len(model.talker.layers), cfg.heads, cfg.kv_heads,
                                cfg.head_dim, cfg.inter, FMT_BF16, rope, cfg.theta)
                d.talker_prefill_layers = pf.layers
        d.codec_embedding = ptr(model.codec_embedding)
        self._keep += [model.codec_head, model.codec_embedding]
        d.codec_vocab = cfg.codec_vocab
        d.codebook = cfg.codebook
        if model.cp is not None:
            cf = talker_fmt if cp_fmt is None else cp_fmt
            d.has_cp = 1
            d.cp = stack_desc(model.cp, "c", cfg.cp_hidden, len(model.cp.layers), cfg.cp_heads, cfg.cp_kv_heads,
                              cfg.cp_head_dim, cfg.cp_inter, cf, cp_rope, cfg.theta)
            d.cp_norm = ptr(model.cp_norm)
            self._keep.append(model.cp_norm)
            for gi in range(15):
                d.cp_lm_head[gi] = enc(f"lm{gi}", model.cp_lm_head[gi], cf)
                d.cp_codec_emb[gi] = ptr(model.cp_codec_emb[gi])
                self._keep.append(model.cp_codec_emb[gi])
            d.cp_emb_dim = cfg.cp_emb_dim
            if model.mtp_w is not None:
                mf = FMT_INT8 if cf != FMT_BF16 else FMT_BF16
                d.cp_mtp_proj = enc("mtp", model.mtp_w, mf)
                d.cp_mtp_fmt = mf
                bias = f32_from_bf16(model.mtp_b)
                self._keep.append(bias)
                d.cp_mtp_bias = ptr(bias)
        self.desc = d
        h = _vp()
        check(L.qtb_engine_create(C.byref(d), device, C.byref(h)))
        self.h = h
        self._keep = None  # the engine copied everything

    def talker_weight_bytes(self):
        return lib().qtb_engine_talker_weight_bytes(self.h)

    def cp_pass_weight_bytes(self):
        return lib().qtb_engine_cp_pass_weight_bytes(self.h)

    def cp_head_weight_bytes(self):
        return lib().qtb_engine_cp_head_weight_bytes(self.h)

    def close(self):
        if self.h:
            lib().qtb_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """B decode slots with paged KV, sharing an Engine's weights."""

    def __init__(self, eng: Engine, batch: int = 1, max_ctx: int = 0, n_pages: int = 0):
        self.eng = eng
        self.B = batch
        h = _vp()
        check(lib().qtb_session_create(eng.h, batch, max_ctx, n_pages, C.byref(h)))
        self.h = h
        self.max_ctx = lib().qtb_session_max_ctx(h)

    def close(self):
        if self.h:
            lib().qtb_session_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def n_pages(self):
        """KV pages in the session's pool (qtb_session_n_pages)."""
        return lib().qtb_session_n_pages(self.h)

    def set_pages(self, b, pages):
        p = np.ascontiguousarray(pages, np.int32)
        check(lib().qtb_session_set_pages(self.h, b, ptr(p), len(p)))

    def set_pos(self, pos):
        p = np.ascontiguousarray(pos, np.int32)
        check(lib().qtb_session_set_pos(self.h, ptr(p)))

    def get_pos(self):
        p = np.empty(self.B, np.int32)
        check(lib().qtb_session_get_pos(self.h, ptr(p)))
        return p

    def talker_step(self, embeds, pos=None, want_dec_x=False):
        cfg = self.eng.cfg
        e = np.ascontiguousarray(embeds, np.float32).reshape(self.B, cfg.hidden)
        out = np.empty((self.B, cfg.hidden), np.float32)
        dx = np.empty((self.B, cfg.hidden), np.float32) if want_dec_x else None
        p = None if pos is None else np.ascontiguousarray(np.broadcast_to(pos, (self.B,)), np.int32)
        check(lib().qtb_talker_step(self.h, ptr(e), ptr(p), ptr(out), ptr(dx)))
        return (out, dx) if want_dec_x else out

    def cp_pass(self, x, pos):
        cfg = self.eng.cfg
        xx = np.ascontiguousarray(x, np.float32).reshape(self.B, cfg.cp_hidden).copy()
        p = np.ascontiguousarray(np.broadcast_to(pos, (self.B,)), np.int32)
        check(lib().qtb_cp_pass(self.h, ptr(xx), ptr(p)))
        return xx

    def cp_frame(self, talker_hidden, code0):
        cfg = self.eng.cfg
        th = np.ascontiguousarray(talker_hidden, np.float32).reshape(self.B, cfg.hidden)
        c0 = np.ascontiguousarray(np.broadcast_to(code0, (self.B,)), np.int32)
        out = np.empty((self.B, 15), np.int32)
        check(lib().qtb_cp_frame(self.h, ptr(th), ptr(c0), ptr(out)))
        return out

    def decode_frames(self, embeds, n_frames, pad=None, want_codes=True):
        cfg = self.eng.cfg
        e = None if embeds is None else np.ascontiguousarray(embeds, np.float32).reshape(self.B, cfg.hidden)
        pd = None if pad is None else np.ascontiguousarray(pad, np.float32)
        codes = np.empty((n_frames, self.B, 16), np.int32) if want_codes else None
        hid = np.empty((self.B, cfg.hidden), np.float32)
        check(lib().qtb_decode_frames(self.h, ptr(e), ptr(pd), n_frames, ptr(codes), ptr(hid)))
        return codes, hid

    def set_sampling(self, b, temperature, top_k=50, top_p=1.0, seed=12345):
        """Slot b samples code0 (qtb_session_set_sampling); temperature 0 = greedy."""
        check(lib().qtb_session_set_sampling(self.h, int(b), float(temperature), int(top_k), float(top_p),
                                             int(seed) & 0xffffffff))

    def get_rng(self):
        st = np.zeros(self.B, np.uint32)
        check(lib().qtb_session_get_rng(self.h, ptr(st)))
        return st

    def program_grid(self, which):
        """CTAs of program `which` (0 talker, 1 CP pass, 2 CP frame, 3 frame,
        4 prefill); negative = one cluster of that many CTAs."""
        return lib().qtb_session_program_grid(self.h, int(which))

    def prefill(self, b, embeds, pos0=0):
        """Device prefill of slot b (qtb_prefill): embeds [n][hidden] at
        positions pos0.. ; returns (last hidden, last pre-norm residual)."""
        cfg = self.eng.cfg
        e = np.ascontiguousarray(embeds, np.float32).reshape(-1, cfg.hidden)
        h = np.empty(cfg.hidden, np.float32)
        dx = np.empty(cfg.hidden, np.float32)
        check(lib().qtb_prefill(self.h, int(b), ptr(e), e.shape[0], int(pos0), ptr(h), ptr(dx)))
        return h, dx

    def begin_generation(self, expected_frames=None, rep_penalty=1.0):
        """The reference's generation-loop codec head for decode_frames
        (qtb_session_begin_generation): EOS rules, repetition penalty, stops."""
        ef = None if expected_frames is None else np.ascontiguousarray(np.broadcast_to(expected_frames, (self.B,)),
                                                                       np.int32)
        check(lib().qtb_session_begin_generation(self.h, ptr(ef), C.c_float(rep_penalty)))

    def reset_slot(self, b, expected_frames=0, active=True):
        check(lib().qtb_session_reset_slot(self.h, int(b), int(expected_frames), int(bool(active))))

    def set_slot_pos(self, b, pos):
        check(lib().qtb_session_set_slot_pos(self.h, int(b), int(pos)))

    def set_embed(self, b, embed):
        e = np.ascontiguousarray(embed, np.float32)
        check(lib().qtb_session_set_embed(self.h, int(b), ptr(e)))

    def get_done(self):
        d = np.zeros(self.B, np.int32)
        check(lib().qtb_session_get_done(self.h, ptr(d)))
        return d

    def profile(self, which=3, max_stages=4096):
        """Per-stage SM cycles of one iteration of a program (see
        qtb_session_profile); returns (cycles, kind, shape) arrays."""
        cyc = np.zeros(max_stages, np.int64)
        kind = np.zeros(max_stages, np.int32)
        shape = np.zeros(max_stages, np.int64)
        n = lib().qtb_session_profile(self.h, which, ptr(cyc), ptr(kind), ptr(shape), max_stages)
        if n < 0:
            check(n)
        ck = np.zeros(n * NCKPT, np.int64)
        lib().qtb_session_profile_checkpoints(self.h, ptr(ck), n * NCKPT)
        self.checkpoints = ck.reshape(n, NCKPT)
        return cyc[:n], kind[:n], shape[:n]

    def last_ms(self):
        return lib().qtb_session_last_ms(self.h)

    def last_launches(self):
        return lib().qtb_session_last_launches(self.h)

    def upload_kv(self, b, k, v, layer_stride, length):
        check(lib().qtb_session_upload_kv(self.h, b, ptr(np.ascontiguousarray(k)), ptr(np.ascontiguousarray(v)),
                                          layer_stride, length))

    def download_kv(self, b, n_layers, kv_dim, length, cp=False):
        k = np.zeros((n_layers, length, kv_dim), np.uint16)
        v = np.zeros((n_layers, length, kv_dim), np.uint16)
        fn = lib().qtb_session_download_cp_kv if cp else lib().qtb_session_download_kv
        check(fn(self.h, b, ptr(k), ptr(v), length, length))
        return k, v


def tc_plan(fmt: int, rows: int, cols: int, batch: int, grid: int, cta: int):
    """qtb_tc_plan: (first tile, tiles, first chunk, chunks, slice, slices) of
    one CTA in the large-batch GEMV plan, or None when the shape does not take
    that path."""
    out = np.zeros(6, np.int32)
    rc = lib().qtb_tc_plan(int(fmt), int(rows), int(cols), int(batch), int(grid), int(cta), ptr(out))
    if rc == -5:   # QTB_E_UNSUPPORTED
        return None
    check(rc)
    return tuple(int(v) for v in out)


def gemv(fmt: int, q: dict, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    """Standalone tensor-core GEMV y[B][rows] = W x (the engine's GEMV stage)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    y = np.empty((x.shape[0], rows), np.float32)
    m = matrix(q)
    check(lib().qtb_gemv_host(fmt, C.byref(m), rows, cols, ptr(x), x.shape[0], ptr(y)))
    return y


def attention(qkv, n_heads, n_kv, q_norm, k_norm, eps, rope_cos, rope_sin, kpages, vpages, page_table, pos,
              max_splits=4):
    """Standalone fused QK-norm + RoPE + paged append + split-K attention."""
    qkv = np.ascontiguousarray(qkv, np.float32)
    B = qkv.shape[0]
    out = np.empty((B, n_heads * 128), np.float32)
    pt = np.ascontiguousarray(page_table, np.int32)
    check(lib().qtb_attention_host(ptr(qkv), B, n_heads, n_kv, 128, ptr(np.ascontiguousarray(q_norm, np.float32)),
                                   ptr(np.ascontiguousarray(k_norm, np.float32)), eps, ptr(rope_cos), ptr(rope_sin),
                                   rope_cos.shape[0], ptr(kpages), ptr(vpages), kpages.shape[0], ptr(pt), pt.shape[1],
                                   ptr(np.ascontiguousarray(pos, np.int32)), max_splits, ptr(out)))
    return out


def codec_sample(logits, temperature, top_k, top_p, rng):
    """The device sampler on host logits [batch][n] (qtb_codec_sample_host);
    returns (rows drawn, updated LCG states)."""
    lg = np.ascontiguousarray(logits, np.float32)
    B, n = lg.shape
    t = np.ascontiguousarray(np.broadcast_to(temperature, (B,)), np.float32)
    k = np.ascontiguousarray(np.broadcast_to(top_k, (B,)), np.int32)
    p = np.ascontiguousarray(np.broadcast_to(top_p, (B,)), np.float32)
    st = np.array(np.broadcast_to(rng, (B,)), np.uint32)
    out = np.zeros(B, np.int32)
    check(lib().qtb_codec_sample_host(ptr(lg), B, n, ptr(t), ptr(k), ptr(p), ptr(st), ptr(out)))
    return out, st
