"""The reference's default x86 dispatch against the engine: a reported gap,
not an equality.

The parity tests run the reference with its f32-activation kernels
(QWEN_NO_BF16DOT / QWEN_NO_VNNI / QWEN_NO_SDOT = 1): they compute what the
reference's portable C code computes, and what this engine computes.  On a CPU
with AVX-512 VNNI and BF16 the reference's default build instead quantizes the
activation of every INT8 matvec to 8 bits (qwen_tts_kernels.c:2445-2568) and
takes bf16 dot products with VDPBF16PS, which round the activation to bf16
(qwen_tts_kernels.c:758-856).  The dispatch switches are read once per process,
so the default-dispatch reference runs in a child process.

For the full-size 0.6B talker (INT8 and BF16; 8 steps, then 16 measured) the
test prints the rel L2 of the last hidden state between
  - the reference's default dispatch and its f32-activation kernels,
  - the engine and the f32-activation reference (~1e-3: the parity contract),
  - the engine and the default dispatch,
and requires the engine to be no further from the default dispatch than the
reference's own f32-activation path is, plus 10 % (the default dispatch's
activation rounding is nearly the whole gap: 3.4e-2 at INT8 on this host).
"""
import json
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

import qtts_b200 as Q
import refbind
from models import build, rel_l2
from test_gpu_model import engine_from_ref

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
THREADS = os.cpu_count()
PREFIX, STEPS = 8, 16

_CHILD = r"""
import json, sys
import numpy as np
sys.path[:0] = [sys.argv[1], sys.argv[2], sys.argv[3]]
import qtts_b200 as Q
import refbind
path, fmt, out = sys.argv[4], sys.argv[5], sys.argv[6]
cfg = Q.CFG_06B
ref = refbind.RefModel(path, cfg, use_int8=(fmt == "int8"), threads=int(sys.argv[7]), cp=False)
rng = np.random.default_rng(41)
hs = []
for pos in range(%d):
    e = (0.1 * rng.standard_normal(cfg.hidden)).astype(np.float32)
    hs.append(ref.talker_step(e))
np.save(out, np.stack(hs))
ref.close()
""" % (PREFIX + STEPS)


def _default_dispatch_steps(path, fmt):
    env = dict(os.environ)
    for k in refbind.F32_ACT_ENV:
        env[k] = "0"
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "h.npy")
        subprocess.run([sys.executable, "-c", _CHILD, os.path.join(ROOT, "qwen3-tts_b200"),
                        os.path.join(ROOT, "oracle"), HERE, path, fmt, out, str(THREADS)],
                       env=env, check=True, timeout=900)
        return np.load(out)


@pytest.mark.parametrize("fmt", ["int8", "bf16"])
def test_default_dispatch_gap(have_gpu, fmt):
    cfg = Q.CFG_06B
    m, path = build(cfg, seed=0, norm_gain="ones", with_cp=False)
    ref = refbind.RefModel(path, cfg, use_int8=(fmt == "int8"), threads=THREADS, cp=False)
    eng = engine_from_ref(ref, m, cfg, fmt, with_cp=False)
    ses = Q.Session(eng, 1, 256)
    rng = np.random.default_rng(41)
    f32_ref, gpu = [], []
    for pos in range(PREFIX + STEPS):
        e = (0.1 * rng.standard_normal(cfg.hidden)).astype(np.float32)
        f32_ref.append(ref.talker_step(e))
        gpu.append(ses.talker_step(e, pos)[0])
    ref.close()
    dflt = _default_dispatch_steps(path, fmt)
    rows = []
    for pos in range(PREFIX, PREFIX + STEPS):
        rows.append((rel_l2(dflt[pos], f32_ref[pos]), rel_l2(gpu[pos], f32_ref[pos]), rel_l2(gpu[pos], dflt[pos])))
    worst = np.max(np.array(rows), axis=0)
    print(json.dumps({"fmt": fmt, "flags": sorted(refbind.cpu_flags() & {"avx512_vnni", "avx512_bf16"}),
                      "ref_default_vs_ref_f32": float(worst[0]), "engine_vs_ref_f32": float(worst[1]),
                      "engine_vs_ref_default": float(worst[2])}))
    # the parity contract itself is tested elsewhere (1e-3 over 64 steps at
    # full size); here it only has to stay far inside the dispatch gap
    assert worst[1] < 2e-3, worst
    assert worst[2] <= 1.1 * worst[0] + 2e-3, worst
