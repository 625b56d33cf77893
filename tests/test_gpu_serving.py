"""Continuous-batching spec decoding on the GPU: every request's tokens equal
speculative_greedy on that request alone, with admission limits and a pool small
enough to force preemption by recompute."""

import pytest
import torch

from kvengine_b200 import Model, PagedKVCache, speculative_greedy
from kvengine_b200.serving import SpecServer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_server_tokens_equal_single_request_spec(cuda_device, tiny_state_dicts, dtype):
    cfg, sd = tiny_state_dicts["tiny"]
    target = Model(cfg, sd, dtype, cuda_device)
    draft = Model(cfg, sd, dtype, cuda_device, roll_lm_head=1)
    g = torch.Generator().manual_seed(7)
    reqs = [(torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist(), int(b))
            for n, b in zip(torch.randint(3, 40, (10,), generator=g), torch.randint(1, 24, (10,), generator=g))]
    want = []
    for p, b in reqs:
        pool = PagedKVCache.for_model(target, num_blocks=64, block_size=16)
        s = speculative_greedy(target, draft, torch.tensor([p], device=cuda_device), pool.new_sequence("t"),
                               pool.new_sequence("d"), k=4, max_new_tokens=b, eos_token_id=None)
        want.append(s.new_token_ids)
    for blocks, max_batch in ((256, 4), (12, 8)):
        t_pool = PagedKVCache.for_model(target, num_blocks=blocks, block_size=16)
        d_pool = PagedKVCache.for_model(draft, num_blocks=blocks, block_size=16)
        srv = SpecServer(target, draft, t_pool, d_pool, k=4, max_batch=max_batch, watermark=0.0, eos_token_id=None)
        ids = [srv.add_request(p, b) for p, b in reqs]
        res = srv.run()
        for rid, w in zip(ids, want):
            assert res[rid].new_token_ids == w, (blocks, max_batch, rid)
        assert t_pool.manager.num_free == blocks and d_pool.manager.num_free == blocks
        if blocks == 12:
            assert srv.stats.preempted > 0


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
def test_shared_prefixes_give_single_request_tokens(cuda_device, tiny_state_dicts, dtype):
    """Requests with a common 70-token prefix adopt each other's published blocks
    (target and draft pools): the later ones prefill only their own suffix, and every
    request's tokens still equal speculative_greedy on it alone."""
    cfg, sd = tiny_state_dicts["tiny"]
    target = Model(cfg, sd, dtype, cuda_device)
    draft = Model(cfg, sd, dtype, cuda_device, roll_lm_head=1)
    g = torch.Generator().manual_seed(13)
    common = torch.randint(0, cfg.vocab_size, (70,), generator=g).tolist()
    reqs = [(common + torch.randint(0, cfg.vocab_size, (3 + 5 * i,), generator=g).tolist(), 6 + 3 * i)
            for i in range(6)]
    want = []
    for p, b in reqs:
        pool = PagedKVCache.for_model(target, num_blocks=64, block_size=16)
        s = speculative_greedy(target, draft, torch.tensor([p], device=cuda_device), pool.new_sequence("t"),
                               pool.new_sequence("d"), k=4, max_new_tokens=b, eos_token_id=None)
        want.append(s.new_token_ids)
    t_pool = PagedKVCache.for_model(target, num_blocks=128, block_size=16)
    d_pool = PagedKVCache.for_model(draft, num_blocks=128, block_size=16)
    srv = SpecServer(target, draft, t_pool, d_pool, k=4, max_batch=2, watermark=0.0, eos_token_id=None)
    ids = [srv.add_request(p, b) for p, b in reqs]
    res = srv.run()
    for rid, w in zip(ids, want):
        assert res[rid].new_token_ids == w, rid
    assert srv.stats.prefix_tokens_reused >= 4 * 64  # four later requests adopt the 4 common full blocks
    assert t_pool.manager.num_free == 128 and d_pool.manager.num_free == 128
