"""SpecServer scheduling (admission, retire-and-refill, preemption by
recompute) on the host with a fake engine: every step emits one token per
running request, the next token being a function of the request's own tokens,
so the output of each request must not depend on the schedule."""

import pytest
import torch

from kvengine_b200.blocks import OutOfBlocks
from kvengine_b200.paged import PagedKVCache
from kvengine_b200.serving import SpecServer


class _Cfg:
    num_layers, num_kv_heads, head_dim = 1, 1, 8


class FakeEngine:
    """Reserves and commits like SpecEngine.step (draft u_d + k - 1, target u_t + k,
    then truncate both caches to len(tokens) - 1) and emits next = f(tokens)."""

    def __init__(self, t_pool, d_pool, k):
        self.t_pool, self.d_pool, self.k = t_pool, d_pool, k
        self.target = object()
        self.steps = 0

    def step(self, reqs, eos):
        k = self.k
        for r in reqs:
            r.u_d = len(r.tokens) - r.d_seq.length
            r.u_t = len(r.tokens) - r.t_seq.length
            r.d_seq.reserve(r.u_d + k - 1)
        for r in reqs:
            r.t_seq.reserve(r.u_t + k)
        self.steps += 1
        for r in reqs:
            r.d_seq.commit(r.u_d + k - 1)
            r.t_seq.commit(r.u_t + k)
            nxt = (sum(r.tokens) * 31 + len(r.tokens)) % 1000
            r.tokens.append(nxt)
            r.res.new_token_ids.append(nxt)
            r.res.iterations += 1
            keep = len(r.tokens) - 1
            r.t_seq.truncate(min(r.t_seq.length, keep))
            r.d_seq.truncate(min(r.d_seq.length, keep))
            if len(r.res.new_token_ids) >= r.max_new:
                r.done = True


def _expected(prompt, n):
    toks, out = list(prompt), []
    for _ in range(n):
        nxt = (sum(toks) * 31 + len(toks)) % 1000
        toks.append(nxt)
        out.append(nxt)
    return out


def _pools(n_blocks, bs=4):
    def mk():
        return PagedKVCache(_Cfg.num_layers, _Cfg.num_kv_heads, _Cfg.head_dim, n_blocks, bs, torch.float32, "cpu")
    return mk(), mk()


def _requests():
    return [([i + 1] * (3 + (i * 5) % 11), 2 + (i * 3) % 7) for i in range(12)]


@pytest.mark.parametrize("max_batch", [1, 3, 64])
def test_outputs_do_not_depend_on_schedule(max_batch):
    t_pool, d_pool = _pools(256)
    srv = SpecServer(engine=FakeEngine(t_pool, d_pool, 4), max_batch=max_batch, eos_token_id=None)
    ids = [srv.add_request(p, n) for p, n in _requests()]
    res = srv.run()
    for rid, (p, n) in zip(ids, _requests()):
        assert res[rid].new_token_ids == _expected(p, n)
    assert srv.stats.finished == len(ids) and srv.stats.peak_running <= max_batch
    assert t_pool.manager.num_free == 256 and d_pool.manager.num_free == 256


def test_small_pool_preempts_and_recomputes():
    t_pool, d_pool = _pools(14)  # 56 slots: a few requests at a time
    srv = SpecServer(engine=FakeEngine(t_pool, d_pool, 4), max_batch=8, watermark=0.0, eos_token_id=None)
    ids = [srv.add_request(p, n) for p, n in _requests()]
    res = srv.run()
    for rid, (p, n) in zip(ids, _requests()):
        assert res[rid].new_token_ids == _expected(p, n)
    assert t_pool.manager.num_free == 14 and d_pool.manager.num_free == 14


def test_preemption_happens_when_running_requests_outgrow_the_pool():
    t_pool, d_pool = _pools(10)
    eng = FakeEngine(t_pool, d_pool, 2)
    srv = SpecServer(engine=eng, max_batch=4, watermark=0.0, eos_token_id=None)
    ids = [srv.add_request([7] * 4, 12) for _ in range(4)]
    res = srv.run()
    assert srv.stats.preempted > 0
    for rid in ids:
        assert res[rid].new_token_ids == _expected([7] * 4, 12)


def test_a_request_larger_than_the_pool_is_refused():
    t_pool, d_pool = _pools(2)
    srv = SpecServer(engine=FakeEngine(t_pool, d_pool, 4), max_batch=2, eos_token_id=None)
    srv.add_request([1] * 40, 3)
    with pytest.raises(OutOfBlocks):
        srv.run()


def test_zero_budget_finishes_on_arrival():
    t_pool, d_pool = _pools(8)
    srv = SpecServer(engine=FakeEngine(t_pool, d_pool, 4), eos_token_id=None)
    rid = srv.add_request([1, 2, 3], 0)
    assert srv.run()[rid].new_token_ids == []


def test_shared_prefixes_are_adopted_and_outputs_unchanged():
    """Requests repeating a common prompt prefix adopt its published blocks in both
    pools (reference engine.py:312-318, 362-369): the first ragged pass feeds only
    the rest, outputs equal the unshared run, and every block comes back."""
    common = [7] * 13 + [9] * 6                      # 19 tokens: 4 full blocks of 4
    reqs = [(common + [i + 1] * (2 + i % 3), 3 + i % 4) for i in range(8)]
    outs = {}
    for share in (False, True):
        t_pool, d_pool = _pools(128)
        eng = FakeEngine(t_pool, d_pool, 4)
        fed = []
        orig = eng.step

        def step(rs, eos, orig=orig, fed=fed):
            fed.append(sum(len(r.tokens) - r.t_seq.length for r in rs))
            orig(rs, eos)
        eng.step = step
        srv = SpecServer(engine=eng, max_batch=2, eos_token_id=None, share_prefixes=share)
        ids = [srv.add_request(p, n) for p, n in reqs]
        res = srv.run()
        outs[share] = ([res[i].new_token_ids for i in ids], sum(fed), srv.stats.prefix_tokens_reused)
        for rid, (p, n) in zip(ids, reqs):
            assert res[rid].new_token_ids == _expected(p, n)
        assert t_pool.manager.num_free == 128 and d_pool.manager.num_free == 128
        t_pool.manager.check_invariants()
        d_pool.manager.check_invariants()
    assert outs[True][0] == outs[False][0]
    assert outs[False][2] == 0
    # Requests admitted after the first step find the common prefix published.
    assert outs[True][2] >= 6 * 16 and outs[True][1] == outs[False][1] - outs[True][2]
