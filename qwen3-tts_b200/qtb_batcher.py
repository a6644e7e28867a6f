"""Continuous batching on one engine session (host side).

The reference's server admits requests into a fixed set of batch slots, steps
them together and retires each one at EOS (qwen_tts_serve_continuous,
qwen_tts.c:2389-2740, B <= 8 on its GPU path).  This is that loop over a
paged session of up to 64 slots:

- admit: a free slot takes the next request; its KV pages come from a host
  free list of the session's page pool; the prompt (all tokens but the last)
  is prefilled on the device (qtb_prefill); the slot's generation state is
  reset and the last prompt token's embedding becomes its next input;
- step: one frame for every slot on the device (qtb_decode_frames: talker
  step, codec head under the reference's rules, code predictor, next
  embedding); running slots advance, parked slots do not;
- retire: a slot whose frame sampled EOS (or reached its frame limit) returns
  its pages and is parked on its own scratch page, so its idle talker step
  never touches pages that another request now owns.

Each request decodes greedily or samples its code0 with its own temperature,
top-k, top-p and seed (the device sampler, qtb_session_set_sampling); every
code of a request equals the codes of the same request run alone in a session
of the same batch width.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional

import numpy as np

import qtts_b200 as Q

PAGE = 16


@dataclasses.dataclass
class GenRequest:
    rid: int
    prompt: np.ndarray          # [n][hidden] prompt embeddings (n >= 1)
    max_frames: int
    expected_frames: int = 0    # 3 x text tokens in the reference (EOS boost); 0 = none
    temperature: float = 0.0    # code0 sampling (qtb_session_set_sampling); 0 = greedy
    top_k: int = 50
    top_p: float = 1.0
    seed: int = 12345           # the request's own LCG seed, as the reference's per-slot seed


class ContinuousBatcher:
    def __init__(self, session: "Q.Session", rep_penalty: float = 1.05):
        self.s = session
        self.B = session.B
        self.n_pages = session.n_pages()
        # one scratch page per slot for parking, the rest shared
        self.scratch = list(range(self.B))
        self.free = list(range(self.B, self.n_pages))
        self.rep_penalty = rep_penalty

    def _alloc(self, n: int) -> Optional[List[int]]:
        if n > len(self.free):
            return None
        pages, self.free = self.free[:n], self.free[n:]
        return pages

    def _park(self, b: int):
        self.s.set_pages(b, [self.scratch[b]])
        self.s.set_slot_pos(b, 0)
        self.s.reset_slot(b, 0, active=False)

    def run(self, requests: List[GenRequest]) -> Dict[int, np.ndarray]:
        """Serve every request; returns rid -> codes [frames][16] (the EOS
        frame last, as (2150, -1, ...), when the request stopped at EOS)."""
        s = self.s
        pending = list(requests)
        slot_req: List[Optional[GenRequest]] = [None] * self.B
        slot_pages: List[List[int]] = [[] for _ in range(self.B)]
        out: Dict[int, list] = {}
        s.begin_generation(None, self.rep_penalty)
        for b in range(self.B):
            self._park(b)
        while pending or any(r is not None for r in slot_req):
            # admit into free slots while pages last
            for b in range(self.B):
                if slot_req[b] is not None or not pending:
                    continue
                r = pending[0]
                n = r.prompt.shape[0]
                pages = self._alloc((n + r.max_frames + PAGE - 1) // PAGE + 1)
                if pages is None:
                    break
                pending.pop(0)
                s.set_pages(b, pages)
                if n > 1:
                    s.prefill(b, r.prompt[:n - 1], 0)
                s.set_slot_pos(b, n - 1)
                s.reset_slot(b, r.expected_frames, active=True)
                if r.temperature > 0.0:
                    s.set_sampling(b, r.temperature, r.top_k, r.top_p, r.seed)
                s.set_embed(b, r.prompt[n - 1])
                slot_req[b], slot_pages[b] = r, pages
                out[r.rid] = []
            if not any(r is not None for r in slot_req):
                raise RuntimeError("a request needs more KV pages than the pool holds")
            codes, _ = s.decode_frames(None, 1, want_codes=True)
            for b in range(self.B):
                r = slot_req[b]
                if r is None:
                    continue
                c = codes[0, b]
                out[r.rid].append(c.copy())
                if c[0] == Q.CODEC_EOS or len(out[r.rid]) >= r.max_frames:
                    self.free += slot_pages[b]
                    slot_req[b], slot_pages[b] = None, []
                    self._park(b)
        return {rid: np.array(v, np.int32) for rid, v in out.items()}
