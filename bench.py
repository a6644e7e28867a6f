#!/usr/bin/env python3
"""bench.py -- decode throughput of the B200 engine on BASELINE.json's
headline workload (config 2: 0.6B-shaped talker + code predictor, INT8
per-row weights, batch 1; one unit = one codec frame = 1 talker step + 16
code-predictor passes + 15 greedy lm_heads + the codec-head argmax and the
next-embedding sum, all inside one persistent kernel launch).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config c1|c2|c3|c4|c5]

Multi-GPU (torchrun, one process per GPU): every rank serves its own
independent request stream on its own weight replica and KV pool (request
sharding, no collective on the data path); rank 0 prints the aggregate.

Synthetic data: random N(0, 0.02) weights of the 0.6B / 1.7B shapes (no
checkpoint is available offline), random N(0,1)*0.1 prefill embeddings.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen3-tts_b200"))

KV_BYTES_PER_POS = 28 * 1024 * 2 * 2   # layers x kv_dim x (K,V) x bf16


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


CONFIGS = {
    # name: (model, talker fmt, cp?, batch, prefill, description)
    "c1": ("0.6B", "bf16", False, 1, 64, "0.6B talker BF16, B=1, 64-token prefill, greedy decode"),
    "c2": ("0.6B", "int8", True, 1, 64, "0.6B talker + code predictor, INT8 per-row, B=1, 64-token prefill"),
    "c2t": ("0.6B", "int8", False, 1, 64, "0.6B talker alone, INT8 per-row, B=1, 64-token prefill (talker step + "
                                          "codec-head argmax + next embedding per frame)"),
    "c3": ("1.7B", "int4g32", False, 1, 128, "1.7B talker INT4 g32 asymmetric, B=1, context from 128"),
    "c4": ("0.6B", "bf16", False, 64, None, "0.6B talker BF16, 64 requests, paged KV L~U[128,2048]"),
    "c5": ("1.7B", "int8", True, 64, None, "1.7B talker + CP INT8, 64 requests/GPU, paged KV L~U[256,4096]"),
}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, device):
        self.device = device
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms",
                                          "200", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            try:
                sm.append(float(s[1]))
                mx = float(s[2])
                for i, n in enumerate(names):
                    if s[5 + i].lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_engine(cfg_name, device, seed=0):
    import qtts_b200 as Q
    model_name, fmt, with_cp, B, prefill, _ = CONFIGS[cfg_name]
    mcfg = Q.CFG_06B if model_name == "0.6B" else Q.CFG_17B
    m = Q.synth_model(mcfg, seed=seed, with_cp=with_cp, norm_gain="ones")
    f = Q.FMT_NAMES[fmt]
    eng = Q.Engine(m, f, f if with_cp else None, device=device)
    return Q, mcfg, m, eng


def frame_bytes(eng, with_cp, kv_positions, batch, pages_appended=1):
    """Algorithmic HBM bytes of one step: the talker's stored weights (incl.
    scales/zeros) once, the code predictor's weights and heads once (its 16
    passes re-read them from L2, where they stay resident by design), the
    talker KV read (positions 0..pos, all 28 layers) and the KV appended.  The
    code predictor's own per-frame KV (at most 16 positions) lives in L2."""
    w = eng.talker_weight_bytes()
    if with_cp:
        w += eng.cp_pass_weight_bytes() + 15 * eng.cp_head_weight_bytes()
    return w + KV_BYTES_PER_POS * (kv_positions + batch * pages_appended)


def run_b200(args, rank, world, local_rank):
    import qtts_b200 as Q
    cfg_name = args.config
    model_name, fmt, with_cp, B, prefill, desc = CONFIGS[cfg_name]
    Q, mcfg, m, eng = build_engine(cfg_name, local_rank, seed=0)
    rng = np.random.default_rng(1234 + rank)
    H = mcfg.hidden
    K, W = args.steps, args.warmup
    if B == 1:
        ses = Q.Session(eng, 1, 8192)
        for pos in range(prefill):
            ses.talker_step((0.1 * rng.standard_normal(H)).astype(np.float32), pos)
        ses.set_pos([prefill])
        e0 = (0.1 * rng.standard_normal(H)).astype(np.float32)
        ses.decode_frames(e0, W, want_codes=False)           # warm-up frames
        start_pos = int(ses.get_pos()[0])
    else:
        # the global request set (B per GPU), partitioned over the ranks by KV
        # bytes (qtb_shard.partition): this rank serves its share
        import qtb_shard
        lo, hi = (128, 2048) if cfg_name == "c4" else (256, 4096)
        all_lens = np.random.default_rng(0).integers(lo, hi + 1, B * world)
        reqs = [qtb_shard.Request(i, int(all_lens[i]), W + K) for i in range(B * world)]
        mine = qtb_shard.partition(reqs, list(range(world)))[rank]
        lens = np.array([q.kv_len for q in mine][:B] + [int(all_lens[0])] * max(0, B - len(mine)), np.int64)
        grow = W + K + max(4, min(K, 64))   # positions appended: warm-up, timed and end-to-end frames
        per = [(int(L) + grow + 15) // 16 + 1 for L in lens]
        n_pages = sum(per)
        ses = Q.Session(eng, B, int(max(lens)) + grow + 32, n_pages=n_pages)
        perm = np.random.default_rng(0).permutation(n_pages)
        off = 0
        for b in range(B):
            ses.set_pages(b, perm[off:off + per[b]])
            off += per[b]
        # KV contents N(0,1) truncated to bf16, uploaded per slot
        for b in range(B):
            L = int(lens[b])
            kv = Q.bf16_from_f32(np.random.default_rng(b).standard_normal((mcfg.layers, L, 1024), dtype=np.float32))
            ses.upload_kv(b, kv, kv, L, L)
        ses.set_pos(lens.astype(np.int32))
        e0 = (0.1 * rng.standard_normal((B, H))).astype(np.float32)
        ses.decode_frames(e0, W, want_codes=False)
        start_pos = ses.get_pos()
    # ---- timed region: K frames in one persistent launch ----
    dist_barrier()
    with ClockSampler(local_rank) as clk:
        ses.decode_frames(None, K, want_codes=False)
        ms = ses.last_ms()
        launches = ses.last_launches()
    dist_barrier()
    ms_max = dist_max(ms)
    # ---- end-to-end through the public API with host buffers ----
    e2e_frames = max(4, min(K, 64))
    hid = np.zeros((B, H), np.float32)
    pin_embed = (0.1 * rng.standard_normal((B, H))).astype(np.float32)
    cpe = [Q.f32_from_bf16(t) for t in m.cp_codec_emb] if with_cp else None
    cemb = Q.f32_from_bf16(m.codec_embedding)
    dist_barrier()
    t0 = time.perf_counter()
    for f in range(e2e_frames):
        codes, hid = ses.decode_frames(pin_embed, 1, want_codes=True)
        c = codes[0]
        nxt = cemb[c[:, 0]]
        if with_cp:
            for g in range(15):
                nxt = nxt + cpe[g][c[:, 1 + g]]
        pin_embed = nxt.astype(np.float32)
    e2e_s = time.perf_counter() - t0
    e2e_s = dist_max(e2e_s * 1e3) / 1e3
    # ---- algorithmic bytes of the timed frames ----
    if B == 1:
        kv_read = sum(start_pos + i + 1 for i in range(K))
    else:
        kv_read = sum(int(sum(start_pos + i + 1)) for i in range(K))
    total_bytes = 0
    wbytes = frame_bytes(eng, with_cp, 0, B, 0)
    total_bytes = K * wbytes + KV_BYTES_PER_POS * (kv_read + K * B)
    per_frame_bytes = total_bytes / K
    peak, peak_kind = load_peaks()
    achieved_gbs = total_bytes / (ms * 1e-3) / 1e9
    value = world * K * B / (ms_max * 1e-3)
    traffic = measured_traffic(cfg_name, per_frame_bytes * K, K)
    out = {
        "metric": "talker decode steps/s",
        "value": round(value, 2),
        "unit": "steps/s",
        "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms_max / K, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": fmt,
        "data": "synthetic (random N(0,0.02) weights of the Qwen3-TTS shapes, seeded)",
        "config": config_dict(cfg_name, world),
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved_gbs / peak, 4), "traffic": traffic,
                     "peak_source": peak_kind, "algorithmic_bytes_per_step": int(per_frame_bytes)},
        # qtb_decode_frames(embeds, n_frames=1): embeddings in, codes and the
        # last hidden state out, through the session's pinned staging buffers
        "e2e": {"value": round(world * e2e_frames * B / e2e_s, 2), "unit": "steps/s",
                "h2d_bytes_per_step": B * H * 4,
                "d2h_bytes_per_step": B * 16 * 4 + B * H * 4},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    # which schedule the timed program ran (qtb_session_program_grid: negative
    # = one cluster of that many CTAs, the small-batch single-cluster schedule)
    g = ses.program_grid(3)
    out["config"]["schedule"] = (f"one cluster of {-g} CTAs (cluster barriers)" if g < 0
                                 else f"{g} CTAs, grid barrier")
    return out


def config_dict(cfg_name, world):
    model_name, fmt, with_cp, B, prefill, desc = CONFIGS[cfg_name]
    return {"workload": f"BASELINE config {cfg_name[1]}: {desc}"
                        + ("; every step is a whole codec frame: 1 talker step + 16 code-predictor passes "
                           "+ 15 greedy heads + codec-head argmax + next embedding" if with_cp else ""),
            "batch_per_gpu": B,
            "parallelism": f"request-sharded replicas x{world}, no collectives",
            "l2": "inputs larger than L2: the talker weights (0.44-1.4 GB) exceed the 126 MB L2 and stream from "
                  "HBM every step; the code-predictor weights stay L2-resident across its 16 passes by design",
            "start_positions": f"{prefill}-token prefill" if B == 1 else "U[128,2048]/U[256,4096] paged"}


def measured_traffic(cfg_name, algorithmic_bytes, steps):
    """DRAM bytes (read + write) of one timed launch, from the committed ncu
    capture of the same kernel and workload (profiles/decode_kernel_<cfg>.json:
    bytes per frame measured on a short launch, scaled to `steps` frames)."""
    try:
        with open(os.path.join(ROOT, "profiles", f"decode_kernel_{cfg_name}.json")) as f:
            d = json.load(f)
        return int(d["dram_bytes_per_frame"] * steps)
    except Exception:
        return None


def cpu_baseline_sample(cfg_name, frames=None, threads=None):
    """The reference's own AVX-512 CPU path (oracle/_ref, default dispatch)
    timed on this host's cores on a bounded sample of the same workload."""
    code = f"""
import os, sys, time, json, tempfile
sys.path[:0] = [{os.path.join(ROOT, 'qwen3-tts_b200')!r}, {os.path.join(ROOT, 'oracle')!r}]
import numpy as np, qtts_b200 as Q, refbind
model_name, fmt, with_cp = {CONFIGS[cfg_name][0]!r}, {CONFIGS[cfg_name][1]!r}, {CONFIGS[cfg_name][2]!r}
cfg = Q.CFG_06B if model_name == '0.6B' else Q.CFG_17B
m = Q.synth_model(cfg, seed=0, with_cp=with_cp, norm_gain='ones')
d = tempfile.mkdtemp()
path = os.path.join(d, 'm.safetensors')
refbind.write_safetensors(path, refbind.model_tensors(m))
threads = {threads!r} or os.cpu_count()
ref = refbind.RefModel(path, cfg, use_int8=(fmt == 'int8'), use_int4=(fmt in ('q4_0', 'int4g32')), threads=threads,
                       cp=with_cp)
rng = np.random.default_rng(0)
for p in range({CONFIGS[cfg_name][4] or 64}):   # the same prefill length as the GPU arm
    h = ref.talker_step((0.1 * rng.standard_normal(cfg.hidden)).astype(np.float32))
n = {frames!r}
e = (0.1 * rng.standard_normal(cfg.hidden)).astype(np.float32)
t0 = time.perf_counter(); done = 0
while True:
    h = ref.talker_step(e)
    c0 = ref.codec_argmax(h, cfg.codebook)
    if with_cp:
        ref.cp_predict(h, c0)
    e = ref.codec_embed(c0)
    done += 1
    el = time.perf_counter() - t0
    if (n and done >= n) or (not n and el > 12.0):
        break
print(json.dumps({{"value": done / el, "cores": threads, "frames": done, "seconds": el, "isa": refbind.isa()}}))
"""
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=900)
    if r.returncode != 0:
        return {"error": r.stderr[-400:]}
    return json.loads(r.stdout.strip().splitlines()[-1])


# ------------------------------------------------------------ dist plumbing --
_dist = None


def dist_init():
    global _dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return 0, 1, int(os.environ.get("LOCAL_RANK", "0"))
    import datetime
    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device(f"cuda:{local}"))
    _dist = (torch, dist)
    return dist.get_rank(), world, local


def dist_barrier():
    if _dist:
        _dist[1].barrier()


def dist_max(v):
    if not _dist:
        return v
    torch, dist = _dist
    t = torch.tensor([float(v)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=512)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank, world, local = dist_init()
    if args.gpus != world:
        sys.exit(f"bench.py: --gpus {args.gpus} but WORLD_SIZE is {world}; launch N>1 GPUs with "
                 f"torchrun --nproc-per-node {args.gpus} (one process per GPU)")
    if args.impl == "reference":
        if rank == 0:
            cb = cpu_baseline_sample(args.config)   # a ~12 s sample of the same workload
            unit = "steps/s"
            line = {"impl": "reference", "metric": "talker decode steps/s", "value": round(cb.get("value", 0.0), 3),
                    "unit": unit,
                    "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                    "config": config_dict(args.config, world),
                    "cpu_baseline": {"value": cb.get("value"), "unit": unit, "cores": cb.get("cores"),
                                     "kind": "reference", "sample": f"{cb.get('frames')} steps (~12 s) after a "
                                     f"{CONFIGS[args.config][4] or 64}-step prefill, default dispatch ({cb.get('isa')}), all host threads"},
                    "e2e": {"value": round(cb.get("value", 0.0), 3), "unit": unit, "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0}}
            if "error" in cb:
                line = {"impl": "reference", "unavailable": cb["error"].splitlines()[-1] if cb["error"] else "failed"}
            print(json.dumps(line), flush=True)
        if _dist:
            _dist[1].destroy_process_group()
        return
    out = run_b200(args, rank, world, local)
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            cb = cpu_baseline_sample(args.config)
            out["cpu_baseline"] = {"value": round(cb.get("value", 0.0), 3), "unit": out["unit"],
                                   "cores": cb.get("cores"), "kind": "reference",
                                   "sample": f"{cb.get('frames')} frames (~12 s) of the same workload on the "
                                             f"reference's CPU path (oracle/_ref, default dispatch, {cb.get('isa')})"}
        print(json.dumps(out), flush=True)
    if _dist:
        _dist[1].destroy_process_group()


if __name__ == "__main__":
    main()
