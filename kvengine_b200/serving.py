"""Continuous-batching greedy speculative decoding.

The reference's continuous-batching `Engine` (kvengine/engine.py:182-501) keeps a
waiting queue and a running set, admits requests while the block pool has room
above a watermark (`_admit`, engine.py:284-324), preempts the most recently
admitted request by recompute when the pool runs dry (`_preempt`,
engine.py:425-440; resume recomputes from the tokens, engine.py:137-146) and
retires finished requests every step. It does not speculate. `SpecServer`
applies the same policy to the speculative path: every step is one batched
draft/verify/accept iteration (`SpecEngine.step`) over the running set, where a
newly admitted (or resumed) request's prompt rides in the same ragged verify
pass as the other requests' k+1 rows, and finished requests free their blocks
before the next admission.

Prefix sharing (the reference engine's `share_prefixes`, engine.py:204-207,
312-318, 362-369, 413-419): an admitted request adopts the longest run of
published full blocks matching its tokens in both the target and the draft pool
(`PagedSequenceCache.adopt_prefix`), so its first ragged pass computes only the
rest; after every step each running request publishes its newly full blocks of
verified tokens (`register_prefix_blocks`). Rollback never reaches a published
block: both caches are truncated only past len(tokens) - 1, and only blocks below
that are published.

Greedy output depends only on a request's own tokens, so every request's tokens
equal `speculative_greedy` on that request alone, whatever the admission order,
batch composition, preemptions or shared prefixes.
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass

from .blocks import OutOfBlocks
from .decode import AUTO_EOS, _resolve_eos, _sync
from .speculative import SpecDecodeResult, SpecEngine, _Request


@dataclass
class ServeStats:
    steps: int = 0
    admitted: int = 0
    preempted: int = 0
    finished: int = 0
    peak_running: int = 0
    new_tokens: int = 0
    prefix_tokens_reused: int = 0  # prompt tokens whose target K/V came from shared blocks


class SpecServer:
    """Waiting queue + running set over one SpecEngine.

    max_batch caps the running set; watermark is the fraction of each pool kept
    free at admission (headroom for running requests' growth, as the reference's
    engine does); share_prefixes adopts and publishes full blocks of common
    prefixes. `engine` may be given (tests inject a host-only fake)."""

    def __init__(self, target=None, draft=None, target_pool=None, draft_pool=None, k: int = 4,
                 max_batch: int = 64, watermark: float = 0.02, eos_token_id=AUTO_EOS,
                 engine: SpecEngine | None = None, share_prefixes: bool = True):
        if max_batch < 1:
            raise ValueError("max_batch must be at least 1")
        self.eng = engine or SpecEngine(target, draft, target_pool, draft_pool, k)
        self.k = self.eng.k
        self.t_pool, self.d_pool = self.eng.t_pool, self.eng.d_pool
        self.eos = _resolve_eos(self.eng.target, eos_token_id)
        self.max_batch = max_batch
        self.watermark = watermark
        self.share_prefixes = share_prefixes
        self.waiting: deque[_Request] = deque()
        self.running: list[_Request] = []
        self.results: dict[object, SpecDecodeResult] = {}
        self.stats = ServeStats()
        self._ids: dict[int, object] = {}
        self._t_submit: dict[int, float] = {}
        self._order = 0

    # ---------------------------------------------------------- requests
    def add_request(self, prompt: list[int], max_new_tokens: int, request_id=None):
        rid = request_id if request_id is not None else self._order
        self._order += 1
        r = _Request(list(prompt), None, None, max_new_tokens)
        self._ids[id(r)] = rid
        self._t_submit[id(r)] = time.perf_counter()
        if r.done:  # zero budget: finished on arrival
            self._finish(r)
        else:
            self.waiting.append(r)
        return rid

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    # --------------------------------------------------------- scheduling
    def _blocks_for_next_step(self, r: _Request, pool) -> int:
        # a fresh sequence holds every token but the last after a step: worst case
        # len(tokens) + k + 1 slots in its first iteration
        return pool.manager.blocks_needed(len(r.tokens) + self.k + 1)

    def _fits(self, r: _Request) -> bool:
        for pool in (self.t_pool, self.d_pool):
            m = pool.manager
            headroom = int(self.watermark * m.num_blocks)
            if self._blocks_for_next_step(r, pool) + headroom > m.num_free:
                return False
        return True

    def _admit(self) -> None:
        while self.waiting and len(self.running) < self.max_batch:
            r = self.waiting[0]
            if not self._fits(r):
                if not self.running:
                    raise OutOfBlocks(self._blocks_for_next_step(r, self.t_pool), self.t_pool.manager.num_free)
                break
            self.waiting.popleft()
            rid = self._ids[id(r)]
            r.t_seq = self.t_pool.new_sequence(("t", rid))
            r.d_seq = self.d_pool.new_sequence(("d", rid))
            if self.share_prefixes:
                # The step's ragged pass then feeds only tokens[seq.length:].
                self.stats.prefix_tokens_reused += r.t_seq.adopt_prefix(r.tokens)
                r.d_seq.adopt_prefix(r.tokens)
            self.running.append(r)
            self.stats.admitted += 1
        self.stats.peak_running = max(self.stats.peak_running, len(self.running))

    def _preempt_newest(self) -> None:
        """Free the most recently admitted request's blocks and queue it first;
        on resume its whole token list is recomputed as a prompt."""
        r = self.running.pop()
        r.t_seq.free()
        r.d_seq.free()
        r.t_seq = r.d_seq = None
        self.waiting.appendleft(r)
        self.stats.preempted += 1

    def _finish(self, r: _Request) -> None:
        res = r.res
        if len(res.new_token_ids) > r.max_new:
            res.new_token_ids = res.new_token_ids[: r.max_new]
            res.stopped_on_eos = bool(res.new_token_ids) and res.new_token_ids[-1] in self.eos
        res.elapsed_s = time.perf_counter() - self._t_submit.pop(id(r))
        if r.t_seq is not None:
            r.t_seq.free()
            r.d_seq.free()
        self.results[self._ids.pop(id(r))] = res
        self.stats.finished += 1
        self.stats.new_tokens += len(res.new_token_ids)

    def step(self) -> None:
        """Admit, run one draft/verify/accept iteration over the running set
        (preempting the newest requests while the pools cannot hold it), retire."""
        self._admit()
        if not self.running:
            return
        while True:
            try:
                self.eng.step(self.running, self.eos)
                break
            except OutOfBlocks:
                if len(self.running) == 1:
                    raise
                self._preempt_newest()
        self.stats.steps += 1
        still = []
        for r in self.running:
            if r.done:
                self._finish(r)
            else:
                if self.share_prefixes:
                    # Both caches hold len(tokens) - 1 verified tokens: publish their full blocks.
                    r.t_seq.register_prefix_blocks(r.tokens)
                    r.d_seq.register_prefix_blocks(r.tokens)
                still.append(r)
        self.running = still

    def run(self) -> dict[object, SpecDecodeResult]:
        """Step until every submitted request has finished; returns results by id."""
        while self.has_work():
            self.step()
        if hasattr(self.eng, "check"):
            self.eng.check()
        if hasattr(self.eng, "device"):
            _sync(self.eng.device)
        return self.results
