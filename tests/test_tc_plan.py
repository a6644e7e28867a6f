"""Host-side checks of the large-batch (tcgen05) GEMV plan, through qtb_tc_plan
(host arithmetic only, no GPU): for the model shapes at several batch sizes,
the CTAs' shares cover every (128-row tile, 128-byte K chunk) exactly once,
each slice is one contiguous chunk range, the slices of a tile are the same
for every row group, and wide stages run without split-K."""
import numpy as np
import pytest

import qtts_b200 as Q

G = 148   # B200 SMs
SHAPES = [(4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (2048, 1024), (2176, 1024),
          (4096, 2048), (2048, 2048), (12288, 2048), (2048, 6144), (2176, 2048)]


@pytest.mark.parametrize("fmt", [Q.FMT_BF16, Q.FMT_INT8])
@pytest.mark.parametrize("batch", [5, 17, 64])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_plan_covers_every_tile_chunk_once(fmt, batch, rows, cols):
    kchunk = 128 if fmt == Q.FMT_INT8 else 64
    T, NKC = rows // 128, cols // kchunk
    seen = np.zeros((T, NKC), np.int32)
    slices = set()
    for cta in range(G):
        t0, nt, kb, kc, sl, S = Q.tc_plan(fmt, rows, cols, batch, G, cta)
        assert 1 <= S <= min(NKC, G)
        if nt == 0:
            continue
        assert 0 <= t0 and t0 + nt <= T and 0 <= kb and kb + kc <= NKC and kc >= 1
        assert 0 <= sl < S
        slices.add((sl, kb, kc))
        seen[t0:t0 + nt, kb:kb + kc] += 1
    assert (seen == 1).all(), np.argwhere(seen != 1)[:4]
    # one chunk range per slice, in order, covering K
    ranges = sorted(slices)
    assert [r[0] for r in ranges] == list(range(len(ranges)))
    assert ranges[0][1] == 0 and ranges[-1][1] + ranges[-1][2] == NKC
    for (s0, b0, c0), (s1, b1, c1) in zip(ranges, ranges[1:]):
        assert b1 == b0 + c0


def test_wide_stages_need_no_split_k():
    # the 1.7B gate/up (96 tiles) fills the grid with one slice per tile
    assert Q.tc_plan(Q.FMT_INT8, 12288, 2048, 64, G, 0)[5] == 1


def test_other_shapes_are_not_planned():
    assert Q.tc_plan(Q.FMT_Q4_0, 1024, 1024, 64, G, 0) is None
    assert Q.tc_plan(Q.FMT_INT8, 1000, 1024, 64, G, 0) is None
    assert Q.tc_plan(Q.FMT_INT8, 1024, 1024, 65, G, 0) is None
