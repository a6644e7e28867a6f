"""Request sharding across ranks (host logic of the multi-GPU path), on CPU:
world-size-2 process groups over gloo (127.0.0.1), a tiny talker restated in
numpy (the oracle) standing in for each rank's GPU engine.

- partition() covers every request exactly once, deterministically, with
  balanced KV bytes per rank;
- two ranks serving a request set return exactly the results of one rank
  serving all of it;
- a rank whose serve call fails with DeviceError (injected on the host) drops
  out; its requests are re-queued onto the surviving rank and the union of
  results is still exactly the single-rank one.
"""
import os
import socket

import numpy as np
import pytest

import qtb_shard as S


def _tiny_serve_factory():
    import qtts_oracle as O
    rng = np.random.default_rng(3)
    H, nh, nkv, hd, I, L = 256, 2, 1, 128, 512, 2

    class Ly:
        pass

    layers = []
    for _ in range(L):
        ly = Ly()
        for nm, shp in (("wq", (nh * hd, H)), ("wk", (nkv * hd, H)), ("wv", (nkv * hd, H)), ("wo", (H, nh * hd)),
                        ("gate_up", (2 * I, H)), ("down", (H, I))):
            setattr(ly, nm, (rng.standard_normal(shp, dtype=np.float32) * 0.05).view(np.uint32) >> 16)
            setattr(ly, nm, getattr(ly, nm).astype(np.uint16))
        ly.input_norm = np.ones(H, np.float32)
        ly.post_attn_norm = np.ones(H, np.float32)
        ly.q_norm = np.ones(hd, np.float32)
        ly.k_norm = np.ones(hd, np.float32)
        layers.append(ly)
    cs = np.cos(np.arange(256)[:, None] * (1e6 ** (-np.arange(64) / 64.0))).astype(np.float32)
    sn = np.sin(np.arange(256)[:, None] * (1e6 ** (-np.arange(64) / 64.0))).astype(np.float32)
    st = O.Stack(layers, H, nh, nkv, hd, I, 1e-6, cs, sn, np.ones(H, np.float32))

    def serve(rank, reqs):
        out = {}
        for q in reqs:
            r = np.random.default_rng(1000 + q.rid)
            caches = O.new_caches(st, q.kv_len + q.n_frames + 1)
            h = None
            for p in range(q.kv_len + q.n_frames):
                h, _ = O.talker_step(st, (0.1 * r.standard_normal(H)).astype(np.float32), caches, p)
            out[q.rid] = h
        return out
    return serve


def _requests():
    rng = np.random.default_rng(11)
    return [S.Request(i, int(rng.integers(1, 6)), int(rng.integers(1, 4))) for i in range(10)]


def test_partition_covers_each_request_once_and_balances():
    rng = np.random.default_rng(5)
    reqs = [S.Request(i, int(rng.integers(128, 4097)), 256) for i in range(512)]
    for world in (1, 2, 4, 8):
        share = S.partition(reqs, list(range(world)))
        ids = sorted(q.rid for v in share.values() for q in v)
        assert ids == list(range(512))
        loads = [sum(S.request_cost(q) for q in share[r]) for r in range(world)]
        assert max(loads) - min(loads) <= max(S.request_cost(q) for q in reqs)
        assert share == S.partition(list(reversed(reqs)), list(range(world)))   # order-independent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fail_rank, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [os.path.join(root, "qwen3-tts_b200"), os.path.join(root, "oracle"), here]
    import datetime
    import torch.distributed as dist
    import qtb_shard as SS
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    serve = _tiny_serve_factory()
    calls = {"n": 0}

    def maybe_failing(r, reqs):
        calls["n"] += 1
        if r == fail_rank and calls["n"] == 1:
            raise SS.DeviceError("injected: decode kernel error (bounded wait expired)")
        return serve(r, reqs)

    runner = SS.ShardedRunner(dist)
    res = runner.run(_requests(), maybe_failing)
    q.put((rank, {k: v.tolist() for k, v in res.items()}, list(runner.failed)))
    dist.destroy_process_group()


def _run_group(world, fail_rank):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(outs)


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_two_ranks_equal_one_rank(fail_rank):
    single = _tiny_serve_factory()(0, _requests())
    outs = _run_group(2, fail_rank)
    for rank, res, failed in outs:
        assert failed == ([] if fail_rank < 0 else [fail_rank])
        assert sorted(res) == sorted(single)
        for rid, v in res.items():
            assert np.array_equal(np.asarray(v, np.float32), single[rid]), rid
