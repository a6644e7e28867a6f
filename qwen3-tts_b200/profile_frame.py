"""Profiling driver: single-frame decode launches of a BASELINE workload, for
capturing one `decode_kernel` launch under a profiler.

    python qwen3-tts_b200/profile_frame.py [--config c2] [--frames 3] [--pos 64]

Builds the same synthetic engine as bench.py (seeded random weights of the
config's shapes), places the session at context position --pos (KV contents
are whatever the fresh pool holds: timing and traffic do not depend on them)
and runs --frames launches of one frame each.  Launch 0 is the cold first
launch; capture launch 1 (`ncu -k regex:decode_kernel -s 1 -c 1 ...`).
"""
import argparse
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import qtts_b200 as Q  # noqa: E402

CFG = {"c1": ("0.6B", "bf16", False), "c2": ("0.6B", "int8", True), "c3": ("1.7B", "int4g32", False)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c2", choices=sorted(CFG))
    ap.add_argument("--frames", type=int, default=3)
    ap.add_argument("--pos", type=int, default=64)
    args = ap.parse_args()
    model, fmt, with_cp = CFG[args.config]
    mcfg = Q.CFG_06B if model == "0.6B" else Q.CFG_17B
    m = Q.synth_model(mcfg, seed=0, with_cp=with_cp, norm_gain="ones")
    f = Q.FMT_NAMES[fmt]
    eng = Q.Engine(m, f, f if with_cp else None)
    ses = Q.Session(eng, 1, max(1024, args.pos + args.frames + 16))
    ses.set_pos([args.pos])
    e = (0.1 * np.random.default_rng(0).standard_normal(mcfg.hidden)).astype(np.float32)
    for i in range(args.frames):
        ses.decode_frames(e if i == 0 else None, 1, want_codes=False)
        print(f"frame {i}: {ses.last_ms():.3f} ms", flush=True)


if __name__ == "__main__":
    main()
