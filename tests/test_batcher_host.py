"""Host-side checks of the continuous batcher (qtb_batcher.ContinuousBatcher)
against a fake session that keeps the device's slot semantics on the host: a
running slot produces one frame per step and stops at EOS (the frame at which
its request's script says so), a parked slot produces nothing.  No GPU.

Checked: every request is served once, its codes are its own script's (in
order, the EOS frame last, or cut at max_frames), no KV page is ever held by
two running slots, pages return to the pool at retirement, every running slot
owns enough pages for its prompt and frames, sampling is set only for
requests with a temperature, and prefill covers all prompt tokens but the
last."""
import numpy as np
import pytest

import qtb_batcher as QB
import qtts_b200 as Q

HIDDEN = 8


class FakeSession:
    def __init__(self, B, n_pages, scripts):
        self.B, self._n_pages = B, n_pages
        self.scripts = scripts          # rid -> list of code0 per frame (CODEC_EOS ends)
        self.pages = [[] for _ in range(B)]
        self.active = [False] * B
        self.rid_of = [None] * B
        self.frame = [0] * B
        self.pos = [0] * B
        self.sampling_seeds = []
        self.prefilled = {}
        self.log = []

    def n_pages(self):
        return self._n_pages

    def begin_generation(self, expected, rep):
        self.log.append(("begin", rep))

    def set_pages(self, b, pages):
        self.pages[b] = list(pages)

    def set_slot_pos(self, b, pos):
        self.pos[b] = pos

    def reset_slot(self, b, expected, active=True):
        self.active[b] = active
        self.frame[b] = 0

    def prefill(self, b, embeds, pos0):
        assert pos0 == 0
        self.prefilled[b] = np.array(embeds)

    def set_sampling(self, b, t, k, p, seed):
        assert t > 0
        self.sampling_seeds.append(seed)

    def set_embed(self, b, e):
        # the batcher admits a request right after set_embed: the embedding
        # carries the request id in this fake
        self.rid_of[b] = int(e[0])

    def decode_frames(self, embeds, n, want_codes=True):
        assert embeds is None and n == 1
        running = [b for b in range(self.B) if self.active[b]]
        held = [p for b in running for p in self.pages[b]]
        assert len(held) == len(set(held)), "a page is held by two running slots"
        codes = np.full((1, self.B, 16), -1, np.int32)
        for b in running:
            script = self.scripts[self.rid_of[b]]
            assert len(self.pages[b]) * QB.PAGE >= self.pos[b] + self.frame[b] + 1
            c0 = script[self.frame[b]]
            codes[0, b, 0] = c0
            if c0 != Q.CODEC_EOS:
                codes[0, b, 1:] = c0 % 2048
                self.frame[b] += 1
            else:
                self.active[b] = False
        return codes, None


def make_requests(rng, n, temp_every=3):
    reqs, scripts = [], {}
    for rid in range(n):
        n_prompt = int(rng.integers(1, 40))
        frames = int(rng.integers(1, 30))
        max_frames = int(rng.integers(5, 40))
        script = [int(c) for c in rng.integers(0, 2048, frames)] + [Q.CODEC_EOS]
        scripts[rid] = script + [0] * 64
        prompt = np.zeros((n_prompt, HIDDEN), np.float32)
        prompt[:, 0] = rid
        t = 0.8 if rid % temp_every == 0 else 0.0
        reqs.append(QB.GenRequest(rid, prompt, max_frames, expected_frames=frames, temperature=t, seed=1000 + rid))
    return reqs, scripts


@pytest.mark.parametrize("B,n_pages,n_req", [(1, 8, 5), (4, 40, 17), (8, 30, 40)])
def test_batcher_serves_every_request_with_its_own_codes(B, n_pages, n_req):
    rng = np.random.default_rng(B * 100 + n_req)
    reqs, scripts = make_requests(rng, n_req)
    ses = FakeSession(B, n_pages, scripts)
    out = QB.ContinuousBatcher(ses, rep_penalty=1.05).run(reqs)
    assert sorted(out) == list(range(n_req))
    for r in reqs:
        got = out[r.rid]
        script = scripts[r.rid]
        eos_at = script.index(Q.CODEC_EOS)
        want_len = min(eos_at + 1, r.max_frames)
        assert len(got) == want_len, (r.rid, len(got), want_len)
        assert list(got[:, 0]) == script[:want_len]
        if got[-1, 0] == Q.CODEC_EOS:
            assert (got[-1, 1:] == -1).all()
    assert not any(ses.active)
    assert ses.log == [("begin", 1.05)]
    # sampling set once for each request with a temperature, with its seed
    assert sorted(ses.sampling_seeds) == sorted(1000 + r.rid for r in reqs if r.temperature > 0)


def test_pages_return_to_the_pool():
    rng = np.random.default_rng(7)
    reqs, scripts = make_requests(rng, 12)
    ses = FakeSession(3, 24, scripts)
    bat = QB.ContinuousBatcher(ses)
    bat.run(reqs)
    assert sorted(bat.free) == list(range(3, 24))


def test_prefill_covers_all_but_the_last_prompt_token():
    rng = np.random.default_rng(3)
    reqs, scripts = make_requests(rng, 1)
    reqs[0].prompt = np.zeros((5, HIDDEN), np.float32)
    ses = FakeSession(1, 8, scripts)
    QB.ContinuousBatcher(ses).run(reqs)
    assert ses.prefilled[0].shape == (4, HIDDEN)


def test_request_larger_than_the_pool_is_refused():
    rng = np.random.default_rng(5)
    reqs, scripts = make_requests(rng, 1)
    reqs[0].max_frames = 10_000
    ses = FakeSession(2, 6, scripts)
    with pytest.raises(RuntimeError, match="more KV pages"):
        QB.ContinuousBatcher(ses).run(reqs)
