"""Continuous-batching spec decoding on the GPU, checked against the CPU oracle.

Every request served by `SpecServer` (admission limits, a pool small enough to
force preemption by recompute, prefix sharing) must emit exactly the tokens the
oracle's single-request `speculative_greedy` (a restatement of
kvengine/speculative.py:111-216, pinned to the reference's own outputs by
tests/test_oracle_golden.py) emits for that request on the same weights. In
bf16 a divergence at a step whose oracle top-2 logit margin is below 2e-2 is
reported as a near-tie instead of failed.
"""

import pytest
import torch

from conftest import first_divergence, top2_margins
from kvengine_b200 import Model, PagedKVCache
from kvengine_b200.serving import SpecServer
from oracle.model import OracleModel
from oracle.paged import OraclePool
from oracle.spec import oracle_speculative_greedy, verify_log_margins

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-3, torch.bfloat16: 2e-2}


def _oracle_runs(target_om, draft_om, reqs, k=4):
    """(tokens, margins) of the oracle's single-request spec decode for each (prompt, budget)."""
    out = []
    for p, b in reqs:
        tc, dc = target_om.cfg, draft_om.cfg
        tp = OraclePool(tc.num_layers, tc.num_kv_heads, tc.head_dim, 64, 16, target_om.dtype)
        dp = OraclePool(dc.num_layers, dc.num_kv_heads, dc.head_dim, 64, 16, draft_om.dtype)
        log = []
        r = oracle_speculative_greedy(target_om, draft_om, p, tp.new_sequence(), dp.new_sequence(), k=k,
                                      max_new_tokens=b, verify_log=log)
        out.append((r["new_token_ids"], top2_margins(verify_log_margins(log))))
    return out


def _check(res, ids, want, tol, label):
    near = []
    for rid, (tokens, margins) in zip(ids, want):
        d = first_divergence(res[rid].new_token_ids, tokens, margins, tol)
        if d is not None:
            assert d["near_tie"], (label, rid, d)
            near.append((label, rid, d))
    return near


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_server_tokens_equal_oracle(cuda_device, tiny_state_dicts, dtype):
    cfg, sd = tiny_state_dicts["tiny"]
    target = Model(cfg, sd, dtype, cuda_device)
    draft = Model(cfg, sd, dtype, cuda_device, roll_lm_head=1)
    g = torch.Generator().manual_seed(7)
    reqs = [(torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist(), int(b))
            for n, b in zip(torch.randint(3, 40, (10,), generator=g), torch.randint(1, 24, (10,), generator=g))]
    want = _oracle_runs(OracleModel(cfg, sd, dtype), OracleModel(cfg, sd, dtype, roll_head=1), reqs)
    near = []
    for blocks, max_batch in ((256, 4), (12, 8)):
        t_pool = PagedKVCache.for_model(target, num_blocks=blocks, block_size=16)
        d_pool = PagedKVCache.for_model(draft, num_blocks=blocks, block_size=16)
        srv = SpecServer(target, draft, t_pool, d_pool, k=4, max_batch=max_batch, watermark=0.0, eos_token_id=None)
        ids = [srv.add_request(p, b) for p, b in reqs]
        res = srv.run()
        near += _check(res, ids, want, TOL[dtype], (blocks, max_batch))
        for rid, (p, b) in zip(ids, reqs):
            assert len(res[rid].new_token_ids) == b
        assert t_pool.manager.num_free == blocks and d_pool.manager.num_free == blocks
        if blocks == 12:
            assert srv.stats.preempted > 0
    print("near-ties (reported, not failed):", near)


def test_server_3b_shape_bf16_equals_oracle(cuda_device, shape3b_state_dicts):
    """The same check at the benchmark's layer shapes (two layers, bf16, head_dim 128
    target, 0.5B-shape draft, full vocabulary) with preemption: 6 requests, at most 3
    running, a pool that cannot hold them all."""
    (t_cfg, t_sd), (d_cfg, d_sd) = shape3b_state_dicts["target"], shape3b_state_dicts["draft"]
    target = Model(t_cfg, t_sd, torch.bfloat16, cuda_device)
    draft = Model(d_cfg, d_sd, torch.bfloat16, cuda_device)
    g = torch.Generator().manual_seed(17)
    reqs = [(torch.randint(0, t_cfg.vocab_size, (int(n),), generator=g).tolist(), int(b))
            for n, b in zip((9, 40, 23, 70, 3, 33), (12, 5, 16, 9, 14, 7))]
    want = _oracle_runs(OracleModel(t_cfg, t_sd, torch.bfloat16), OracleModel(d_cfg, d_sd, torch.bfloat16), reqs)
    t_pool = PagedKVCache.for_model(target, num_blocks=14, block_size=16)
    d_pool = PagedKVCache.for_model(draft, num_blocks=14, block_size=16)
    srv = SpecServer(target, draft, t_pool, d_pool, k=4, max_batch=3, watermark=0.0, eos_token_id=None)
    ids = [srv.add_request(p, b) for p, b in reqs]
    res = srv.run()
    print("near-ties (reported, not failed):", _check(res, ids, want, 2e-2, "3b-shape"))
    assert t_pool.manager.num_free == 14 and d_pool.manager.num_free == 14


def test_self_draft_is_fully_accepted_with_prompt_sized_batches(cuda_device, tiny_state_dicts):
    """Draft = target in bf16 under continuous batching: the first iteration's
    passes carry whole prompts (over 2048 rows) next to one-token rows, yet every
    draft token is accepted - the GEMMs' reduction order does not depend on the
    batch."""
    cfg, sd = tiny_state_dicts["tiny"]
    model = Model(cfg, sd, torch.bfloat16, cuda_device)
    g = torch.Generator().manual_seed(11)
    t_pool = PagedKVCache.for_model(model, num_blocks=512, block_size=16)
    d_pool = PagedKVCache.for_model(model, num_blocks=512, block_size=16)
    srv = SpecServer(model, model, t_pool, d_pool, k=4, max_batch=12, eos_token_id=None)
    for i in range(12):
        srv.add_request(torch.randint(0, cfg.vocab_size, (300 - 7 * i,), generator=g).tolist(), 9 + i)
    res = srv.run()
    assert len(res) == 12
    for r in res.values():
        assert r.tokens_drafted > 0 and r.tokens_accepted == r.tokens_drafted


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_shared_prefixes_give_oracle_tokens(cuda_device, tiny_state_dicts, dtype):
    """Requests with a common 70-token prefix adopt each other's published blocks
    (target and draft pools): the later ones prefill only their own suffix, and every
    request's tokens still equal the oracle's single-request spec decode."""
    cfg, sd = tiny_state_dicts["tiny"]
    target = Model(cfg, sd, dtype, cuda_device)
    draft = Model(cfg, sd, dtype, cuda_device, roll_lm_head=1)
    g = torch.Generator().manual_seed(13)
    common = torch.randint(0, cfg.vocab_size, (70,), generator=g).tolist()
    reqs = [(common + torch.randint(0, cfg.vocab_size, (3 + 5 * i,), generator=g).tolist(), 6 + 3 * i)
            for i in range(6)]
    want = _oracle_runs(OracleModel(cfg, sd, dtype), OracleModel(cfg, sd, dtype, roll_head=1), reqs)
    t_pool = PagedKVCache.for_model(target, num_blocks=128, block_size=16)
    d_pool = PagedKVCache.for_model(draft, num_blocks=128, block_size=16)
    srv = SpecServer(target, draft, t_pool, d_pool, k=4, max_batch=2, watermark=0.0, eos_token_id=None)
    ids = [srv.add_request(p, b) for p, b in reqs]
    res = srv.run()
    print("near-ties (reported, not failed):", _check(res, ids, want, TOL[dtype], "prefix"))
    assert srv.stats.prefix_tokens_reused >= 4 * 64  # four later requests adopt the 4 common full blocks
    assert t_pool.manager.num_free == 128 and d_pool.manager.num_free == 128


def test_rollback_into_a_shared_block_is_refused(cuda_device, tiny_state_dicts):
    """kvengine tests/test_phase6.py:366-390 on the GPU path: a sequence whose full
    blocks were published and adopted by another cannot be truncated into them
    (ValueError naming the sharing), and nothing leaks."""
    from kvengine_b200 import forward_with_own_cache

    cfg, sd = tiny_state_dicts["tiny"]
    model = Model(cfg, sd, torch.bfloat16, cuda_device)
    pool = PagedKVCache.for_model(model, num_blocks=64, block_size=4)
    toks = torch.randint(0, cfg.vocab_size, (16,), generator=torch.Generator().manual_seed(23)).tolist()
    a = pool.new_sequence("a")
    forward_with_own_cache(model, torch.tensor([toks], device=cuda_device), a)
    a.register_prefix_blocks(toks)
    b = pool.new_sequence("b")
    assert b.adopt_prefix(toks) > 0
    with pytest.raises(ValueError, match="shared"):
        a.truncate(2)
    a.free()
    b.free()
    assert pool.manager.num_allocated == 0
    pool.manager.check_invariants()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rollback_beside_shared_blocks_under_serving(cuda_device, tiny_state_dicts, dtype):
    """Two requests with the same 64-token prompt: the second adopts the first's
    published prompt blocks while a hostile draft (k = 8) makes every iteration roll
    back both requests' caches. Rollback stops at len(tokens) - 1, past every
    published block, so both requests emit the oracle's tokens and the shared blocks
    end cached, not reused."""
    cfg, sd = tiny_state_dicts["tiny"]
    target = Model(cfg, sd, dtype, cuda_device)
    draft = Model(cfg, sd, dtype, cuda_device, roll_lm_head=1)
    g = torch.Generator().manual_seed(19)
    prompt = torch.randint(0, cfg.vocab_size, (64,), generator=g).tolist()
    reqs = [(prompt, 20), (prompt, 11)]
    want = _oracle_runs(OracleModel(cfg, sd, dtype), OracleModel(cfg, sd, dtype, roll_head=1), reqs, k=8)
    t_pool = PagedKVCache.for_model(target, num_blocks=64, block_size=16)
    d_pool = PagedKVCache.for_model(draft, num_blocks=64, block_size=16)
    srv = SpecServer(target, draft, t_pool, d_pool, k=8, max_batch=1, watermark=0.0, eos_token_id=None)
    ids = [srv.add_request(p, b) for p, b in reqs]
    res = srv.run()
    print("near-ties (reported, not failed):", _check(res, ids, want, TOL[dtype], "beside-shared"))
    assert srv.stats.prefix_tokens_reused >= 48
    t_pool.manager.check_invariants()
    d_pool.manager.check_invariants()
    assert t_pool.manager.num_reclaimable >= 3 and t_pool.manager.num_free == 64
