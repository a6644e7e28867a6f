"""Profiling driver: single-frame decode launches of a BASELINE workload, for
capturing one `decode_kernel` launch under a profiler.

    python qwen3-tts_b200/profile_frame.py [--config c2] [--frames 3] [--pos 64] [--trace]
    python qwen3-tts_b200/profile_frame.py --stage gemv [--rows 1024 --cols 2048 --batch 64 --fmt bf16]
    python qwen3-tts_b200/profile_frame.py --stage attn [--batch 64] [--pos P]

Builds the same synthetic engine as bench.py (seeded random weights of the
config's shapes), places the session at context position --pos (KV contents
are whatever the fresh pool holds: timing and traffic do not depend on them)
and runs --frames launches of one frame each.  Launch 0 is the cold first
launch; capture launch 1 (`ncu -k regex:decode_kernel -s 1 -c 1 ...`).

--stage runs one stage kind alone, three launches of one stage each (capture
launch 2): a GEMV stage (bf16 or int8) of the given shape and batch, or a
paged decode attention stage with its K/V append (16 query / 8 KV heads) of
--batch slots at context lengths drawn from U[128, 2048), the config-4 mix, or
all at position --pos.
"""
import argparse
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import qtts_b200 as Q  # noqa: E402

CFG = {"c1": ("0.6B", "bf16", False), "c2": ("0.6B", "int8", True), "c3": ("1.7B", "int4g32", False),
       "c4": ("0.6B", "bf16", False), "c5": ("1.7B", "int8", True)}
KIND = {1: "gemv", 2: "attention", 3: "embed", 4: "norm", 5: "pos_inc"}


def stage_trace(ses, which, frame_ms):
    """Per-stage table of one program iteration (qtb_session_profile): count,
    mean and total time per (stage kind, GEMV shape), and the busiest CTA's
    time between its barriers (the rest of a stage is waiting at the grid
    barrier).  SM cycles are turned into microseconds with the clock implied
    by the plain frame time."""
    cyc, kind, shape = ses.profile(which)
    n = len(cyc)
    arr = np.zeros(2 * n * 1024, np.int64)
    got = Q.lib().qtb_session_profile_arrivals(ses.h, Q.ptr(arr), arr.size)
    grid = got // (2 * n)
    busy = (arr[n * grid:2 * n * grid].reshape(n, grid) & ((1 << 48) - 1)).astype(np.float64)
    ghz = cyc.sum() / (frame_ms * 1e6)
    groups = {}
    for i in range(n):
        key = (int(kind[i]), int(shape[i]) >> 16, int(shape[i]) & 0xffff)
        groups.setdefault(key, []).append(i)
    print(f"{n} stages, {grid} CTAs, {cyc.sum() / ghz / 1e3:.1f} us in all (scale {ghz:.3f} cycles per ns)")
    print()
    print("| stage | rows x K | count | mean us | busiest CTA us | total us |")
    print("|---|---|---|---|---|---|")
    for key, idx in sorted(groups.items(), key=lambda kv: -cyc[kv[1]].sum()):
        c = cyc[idx] / ghz / 1e3
        mb = busy[idx].max(axis=1) / ghz / 1e3
        shp = f"{key[1]} x {key[2]}" if key[0] == 1 else "-"
        print(f"| {KIND.get(key[0], key[0])} | {shp} | {len(idx)} | {c.mean():.2f} | {mb.mean():.2f} | {c.sum():.1f} |")



def one_stage(args):
    rng = np.random.default_rng(0)
    if args.stage == "gemv":
        rows, K, B = args.rows, args.cols, args.batch
        W = Q.bf16_from_f32(rng.standard_normal((rows, K), dtype=np.float32) * np.float32(0.02))
        fmt = Q.FMT_NAMES[args.fmt]
        q = Q.quantize(W, fmt)
        x = rng.standard_normal((B, K), dtype=np.float32)
        for _ in range(3):
            y = Q.gemv(fmt, q, rows, K, x)
        ref = Q.f32_from_bf16(W).astype(np.float64) @ x.T.astype(np.float64)
        print("gemv", y.shape, "rel err %.2e" % (np.linalg.norm(y - ref.T) / np.linalg.norm(ref)))
        return
    B = args.batch
    pos = np.full(B, args.pos) if args.pos_given else rng.integers(128, 2048, B)
    nkv, nh, hd = 8, 16, 128
    pt_stride = int(max(pos)) // 16 + 2
    n_pages = int(sum(p // 16 + 1 for p in pos)) + 4
    pt = np.full((B, pt_stride), -1, np.int32)
    perm = rng.permutation(n_pages)
    nxt = 0
    for b in range(B):
        for i in range(int(pos[b]) // 16 + 1):
            pt[b, i] = perm[nxt]
            nxt += 1
    kp = np.full((n_pages, nkv, 16, hd), 0x3F80, np.uint16)
    vp = np.full((n_pages, nkv, 16, hd), 0x3F00, np.uint16)
    qkv = rng.standard_normal((B, (nh + 2 * nkv) * hd), dtype=np.float32)
    ones = np.ones(hd, np.float32)
    cs, sn = Q.rope_tables(1e6, hd, 8192)
    for _ in range(3):
        out = Q.attention(qkv, nh, nkv, ones, ones, 1e-6, cs, sn, kp, vp, pt, pos.astype(np.int32), 16)
    print("attention", out.shape, "finite", bool(np.isfinite(out).all()))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c2", choices=sorted(CFG))
    ap.add_argument("--frames", type=int, default=3)
    ap.add_argument("--pos", type=int, default=64)
    ap.add_argument("--stage", choices=["gemv", "attn"])
    ap.add_argument("--rows", type=int, default=1024)
    ap.add_argument("--cols", type=int, default=2048)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--fmt", default="bf16", choices=["bf16", "int8"])
    ap.add_argument("--trace", action="store_true",
                    help="after the frames, print the stage table of one more frame (c4 / c5: 64 slots at --pos)")
    args = ap.parse_args()
    args.pos_given = "--pos" in sys.argv
    if args.stage:
        one_stage(args)
        return
    model, fmt, with_cp = CFG[args.config]
    mcfg = Q.CFG_06B if model == "0.6B" else Q.CFG_17B
    m = Q.synth_model(mcfg, seed=0, with_cp=with_cp, norm_gain="ones")
    f = Q.FMT_NAMES[fmt]
    eng = Q.Engine(m, f, f if with_cp else None)
    B = 64 if args.config in ("c4", "c5") else 1
    ses = Q.Session(eng, B, max(1024, args.pos + args.frames + 16))
    ses.set_pos([args.pos] * B)
    e = (0.1 * np.random.default_rng(0).standard_normal((B, mcfg.hidden))).astype(np.float32)
    for i in range(args.frames):
        ses.decode_frames(e if i == 0 else None, 1, want_codes=False)
        print(f"frame {i}: {ses.last_ms():.3f} ms", flush=True)
    if args.trace:
        stage_trace(ses, 3 if with_cp else 0, ses.last_ms())


if __name__ == "__main__":
    main()
