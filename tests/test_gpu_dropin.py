"""The reference's batched GPU entry points called through the C ABI, as the
reference's own generation loop and batch self-test call them
(qwen_tts_cuda_talker.cu:595-730, qwen_tts.c:1469-1475 / 2431-2731):

- qwen_cuda_talker_init(ctx) + qwen_cuda_talker_upload_kv(ctx, prefill_len):
  the GPU continues a sequence the reference prefilled on the CPU;
- qwen_cuda_talker_batch_init / _upload_slot / _step / _free: slots seeded from
  the batch engine's host KV layout ((b * L + l) * src_kv_max + pos) * kv_dim,
  a slot's row equal to the single-state step and to the reference's CPU step;
- qwen_cuda_cp_init / qwen_cuda_cp_batch_init / _step / _free in lockstep
  against the single-state qwen_cuda_cp_step (the reference's criterion: max
  |batched - single| < 1e-3);
- qwen_cuda_batch_selftest(ctx, B, frames) returns 0.

Runs in a child process: the drop-in flavour of the reference resolves its
qwen_cuda_* symbols from this library at load time."""
import os
import subprocess
import sys

import pytest

from models import build, tiny_cfg

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import sys, ctypes as C, numpy as np
sys.path[:0] = __PATHS__
import qtts_b200 as Q
eng_lib = C.CDLL(Q.LIB_PATH, mode=C.RTLD_GLOBAL)
ad_lib = C.CDLL(Q.DROPIN_PATH, mode=C.RTLD_GLOBAL)
import refbind
from models import tiny_cfg
vp = C.c_void_p
f = lambda v: v.ctypes.data_as(vp)
for name, res, args in [
        ("qwen_cuda_talker_init", vp, [vp]), ("qwen_cuda_talker_upload_kv", None, [vp, vp, C.c_int]),
        ("qwen_cuda_talker_step", None, [vp, vp, vp, C.c_int]), ("qwen_cuda_talker_free", None, [vp]),
        ("qwen_cuda_talker_batch_init", vp, [vp, C.c_int]),
        ("qwen_cuda_talker_batch_upload_slot", None, [vp, C.c_int, vp, vp, C.c_int, C.c_int]),
        ("qwen_cuda_talker_batch_step", None, [vp, vp, vp, vp]), ("qwen_cuda_talker_batch_free", None, [vp]),
        ("qwen_cuda_cp_init", vp, [vp]), ("qwen_cuda_cp_step", None, [vp, vp, C.c_int]),
        ("qwen_cuda_cp_free", None, [vp]), ("qwen_cuda_cp_batch_init", vp, [vp, C.c_int]),
        ("qwen_cuda_cp_batch_step", None, [vp, vp, vp]), ("qwen_cuda_cp_batch_free", None, [vp]),
        ("qwen_cuda_batch_selftest", C.c_int, [vp, C.c_int, C.c_int]), ("qwen_cuda_last_error", C.c_int, [])]:
    fn = getattr(ad_lib, name)
    fn.restype = res
    fn.argtypes = args
    globals()[name] = fn

def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))

cfg = tiny_cfg(layers=3, cp_layers=2)
ref = refbind.RefModel(__MODEL__, cfg, threads=8, dropin=True)
ctx = ref.ctx()
H, L, kvd = cfg.hidden, cfg.layers, cfg.kv_heads * 128
rng = np.random.default_rng(13)
P = 20
for _ in range(P):                       # CPU prefill (the reference's own path)
    ref.talker_step((0.1 * rng.standard_normal(H)).astype(np.float32))

# single state continuing the CPU-prefilled sequence
S = qwen_cuda_talker_init(ctx)
assert S and qwen_cuda_last_error() == 0
qwen_cuda_talker_upload_kv(S, ctx, P)
assert qwen_cuda_last_error() == 0
e = (0.1 * rng.standard_normal(H)).astype(np.float32)
h_gpu = np.empty(H, np.float32)
qwen_cuda_talker_step(S, f(e), f(h_gpu), P)
h_cpu = ref.talker_step(e)
r1 = rel(h_gpu, h_cpu)
assert r1 < 1e-3, ("single after upload_kv", r1)

# batched state: slot 1 holds this sequence (P + 1 positions), slots 0 and 2 other KV
B, src_kv_max = 3, 64
kk = np.zeros((B, L, src_kv_max, kvd), np.uint16)
vv = np.zeros((B, L, src_kv_max, kvd), np.uint16)
for l in range(L):
    k, v = ref.kv(l, P + 1)
    kk[1, l, :P + 1], vv[1, l, :P + 1] = k, v
for b in (0, 2):
    kk[b, :, :P + 1] = Q.bf16_from_f32(rng.standard_normal((L, P + 1, kvd), dtype=np.float32))
    vv[b, :, :P + 1] = Q.bf16_from_f32(rng.standard_normal((L, P + 1, kvd), dtype=np.float32))
Bs = qwen_cuda_talker_batch_init(S, B)
assert Bs and qwen_cuda_last_error() == 0
for b in range(B):
    qwen_cuda_talker_batch_upload_slot(Bs, b, f(kk), f(vv), src_kv_max, P + 1)
    assert qwen_cuda_last_error() == 0
e2 = (0.1 * rng.standard_normal((B, H))).astype(np.float32)
pos = np.full(B, P + 1, np.int32)
hB = np.empty((B, H), np.float32)
qwen_cuda_talker_batch_step(Bs, f(e2), f(pos), f(hB))
assert qwen_cuda_last_error() == 0
qwen_cuda_talker_step(S, f(np.ascontiguousarray(e2[1])), f(h_gpu), P + 1)
h_cpu = ref.talker_step(e2[1])
r2, r3 = rel(hB[1], h_gpu), rel(hB[1], h_cpu)
assert r2 < 1e-3 and r3 < 1e-3, ("batched slot vs single / CPU", r2, r3)
assert np.all(np.isfinite(hB))
qwen_cuda_talker_batch_free(Bs)
qwen_cuda_talker_free(S)

# code predictor: batched passes in lockstep against the single state
CS = qwen_cuda_cp_init(ctx)
CB = qwen_cuda_cp_batch_init(CS, B)
assert CS and CB and qwen_cuda_last_error() == 0
cdiff = 0.0
for p in range(16):
    x1 = (0.02 * np.sin(0.13 * (np.arange(cfg.cp_hidden) + 1) + 0.2 * p)).astype(np.float32)
    xB = np.ascontiguousarray(np.broadcast_to(x1, (B, cfg.cp_hidden)))
    qwen_cuda_cp_step(CS, f(x1), p)
    qwen_cuda_cp_batch_step(CB, f(xB), f(np.full(B, p, np.int32)))
    cdiff = max(cdiff, float(np.max(np.abs(xB - x1[None]))))
assert qwen_cuda_last_error() == 0
assert cdiff < 1e-3, ("CP batched vs single", cdiff)
qwen_cuda_cp_batch_free(CB)
qwen_cuda_cp_free(CS)

rc = qwen_cuda_batch_selftest(ctx, 4, 8)
assert rc == 0, ("qwen_cuda_batch_selftest", rc)
print("DROPIN_OK", r1, r2, r3, cdiff)
"""


def test_batched_dropin_entry_points(have_gpu, tmp_path):
    cfg = tiny_cfg(layers=3, cp_layers=2)
    m, path = build(cfg)
    script = tmp_path / "batched_dropin.py"
    paths = [os.path.join(ROOT, "qwen3-tts_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
    script.write_text(SCRIPT.replace("__PATHS__", repr(paths)).replace("__MODEL__", repr(path)))
    r = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    assert "DROPIN_OK" in r.stdout, r.stdout[-2000:]
