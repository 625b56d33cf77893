"""End-to-end parity on the GPU: model passes, plain greedy and speculative
decoding through the sm_100a path against the reference's golden outputs and
the CPU oracle. Tolerances: logits within 1e-3 (fp32) / 2e-2 (bf16); token
sequences identical, with argmax near-ties (top-2 margin below the tolerance
in the oracle) reported rather than failed."""

import pytest
import torch

from conftest import load_golden
from kvengine_b200 import (Model, PagedKVCache, forward_with_own_cache, greedy_batch, greedy_paged,
                           speculative_greedy, speculative_greedy_batch)
from oracle.model import OracleModel, oracle_forward
from oracle.paged import OraclePool

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-3, torch.bfloat16: 2e-2}


@pytest.fixture(scope="module")
def tiny_golden():
    return load_golden("tiny")


def _models(tiny_state_dicts, name, dtype, dev):
    cfg, sd = tiny_state_dicts[name]
    return cfg, Model(cfg, sd, dtype, dev), Model(cfg, sd, dtype, dev, roll_lm_head=1)


@pytest.mark.parametrize("name,dtype", [("tiny", torch.float32), ("tiny", torch.bfloat16),
                                        ("tiny_hd128", torch.float32)])
def test_forward_logits_match_oracle(cuda_device, tiny_state_dicts, name, dtype):
    cfg, m, _ = _models(tiny_state_dicts, name, dtype, cuda_device)
    om = OracleModel(cfg, tiny_state_dicts[name][1], dtype)
    g = torch.Generator().manual_seed(3)
    pool = PagedKVCache.for_model(m, num_blocks=64, block_size=16)
    opool = OraclePool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 64, 16, dtype)
    seq, oseq = pool.new_sequence("a"), opool.new_sequence()
    for T in (37, 1, 5, 16, 2):  # prefill, decode, verify-sized chunks
        ids = torch.randint(0, cfg.vocab_size, (1, T), generator=g)
        got = forward_with_own_cache(m, ids.to(cuda_device), seq, all_logits=True)[0].float().cpu()
        ref = oracle_forward(om, ids[0].tolist(), oseq, all_logits=True).float()
        err = (got - ref).abs().max().item()
        assert err <= TOL[dtype], (T, err)
    assert seq.blocks == oseq.blocks and seq.length == oseq.length


@pytest.mark.parametrize("name,dt_name,dtype", [("tiny", "f32", torch.float32), ("tiny", "bf16", torch.bfloat16),
                                                ("tiny_hd128", "f32", torch.float32)])
def test_spec_and_greedy_match_reference_tokens(cuda_device, tiny_state_dicts, tiny_golden, name, dt_name, dtype):
    rec = tiny_golden[f"{name}_{dt_name}"]
    cfg, m, hostile = _models(tiny_state_dicts, name, dtype, cuda_device)
    for i, p in enumerate(rec["prompts"]):
        pool = PagedKVCache.for_model(m, num_blocks=256, block_size=16)
        g = greedy_paged(m, torch.tensor([p], device=cuda_device), pool, max_new_tokens=20, eos_token_id=None)
        assert g.new_token_ids == rec["greedy"][i]
        assert pool.manager.num_allocated == 0
    for k in (1, 2, 4, 8):
        for i, p in enumerate(rec["prompts"]):
            for draft, key in ((m, "spec_self"), (hostile, "spec_hostile")):
                pool = PagedKVCache.for_model(m, num_blocks=256, block_size=16)
                s = speculative_greedy(m, draft, torch.tensor([p], device=cuda_device), pool.new_sequence("t"),
                                       pool.new_sequence("d"), k=k, max_new_tokens=20, eos_token_id=None)
                want = rec[key][str(k)][i]
                assert s.new_token_ids == want["tokens"], (key, k, i)
                assert s.accepted_per_iter == want["accepted_per_iter"], (key, k, i)
                assert (s.target_forwards, s.draft_forwards) == (want["target_forwards"], want["draft_forwards"])


def test_budgets_eos_block_sizes_and_rollback_tables(cuda_device, tiny_state_dicts, tiny_golden):
    rec = tiny_golden["tiny_f32"]
    cfg, m, hostile = _models(tiny_state_dicts, "tiny", torch.float32, cuda_device)
    p = torch.tensor([rec["prompts"][1]], device=cuda_device)
    for budget, want in rec["budgets"].items():
        pool = PagedKVCache.for_model(m, num_blocks=256, block_size=16)
        s = speculative_greedy(m, m, p, pool.new_sequence("t"), pool.new_sequence("d"), k=4,
                               max_new_tokens=int(budget), eos_token_id=None)
        assert s.new_token_ids == want and len(s.new_token_ids) == int(budget)
    for bs, want in rec["block_sizes"].items():
        pool = PagedKVCache.for_model(m, num_blocks=512, block_size=int(bs))
        assert greedy_paged(m, p, pool, max_new_tokens=16, eos_token_id=None).new_token_ids == want
    e = rec["eos"]
    pool = PagedKVCache.for_model(m, num_blocks=256, block_size=16)
    s = speculative_greedy(m, m, p, pool.new_sequence("t"), pool.new_sequence("d"), k=4, max_new_tokens=20,
                           eos_token_id=e["eos_id"])
    assert s.new_token_ids == e["tokens"] and s.stopped_on_eos == e["stopped"]
    assert s.new_token_ids.count(e["eos_id"]) == 1
    rb = rec["rollback"]
    pool = PagedKVCache.for_model(m, num_blocks=64, block_size=4)
    t_seq, d_seq = pool.new_sequence("target"), pool.new_sequence("draft")
    s = speculative_greedy(m, hostile, p, t_seq, d_seq, k=8, max_new_tokens=16, eos_token_id=None)
    assert s.new_token_ids == rb["tokens"]
    assert (t_seq.blocks, d_seq.blocks, t_seq.length, d_seq.length) == (
        rb["t_blocks"], rb["d_blocks"], rb["t_len"], rb["d_len"])
    assert pool.manager.free_list == rb["free_list"]
    assert len(t_seq.blocks) == pool.manager.blocks_needed(t_seq.length)
    t_seq.free()
    d_seq.free()
    assert pool.manager.num_allocated == 0
    pool.manager.check_invariants()


def test_truncate_then_continue_matches_uninterrupted(cuda_device, tiny_state_dicts):
    """kvengine tests/test_phase5.py:240-265: junk K/V written then rolled back leaves no trace."""
    cfg, m, _ = _models(tiny_state_dicts, "tiny", torch.float32, cuda_device)
    ids = torch.randint(0, cfg.vocab_size, (1, 9), generator=torch.Generator().manual_seed(0)).to(cuda_device)
    pool = PagedKVCache.for_model(m, num_blocks=64, block_size=4)
    straight = greedy_paged(m, ids, pool, max_new_tokens=12, eos_token_id=None).new_token_ids
    cache = pool.new_sequence("x")
    logits = forward_with_own_cache(m, ids, cache)
    produced = []
    for step in range(12):
        tok = int(torch.argmax(logits[0, -1]))
        produced.append(tok)
        if step == 5:
            mark = cache.length
            forward_with_own_cache(m, torch.tensor([[tok, tok, tok]], device=cuda_device), cache)
            cache.truncate(mark)
        logits = forward_with_own_cache(m, torch.tensor([[tok]], device=cuda_device), cache)
    assert produced == straight


def test_batched_spec_equals_per_request(cuda_device, tiny_state_dicts, tiny_golden):
    rec = tiny_golden["tiny_bf16"]
    cfg, m, hostile = _models(tiny_state_dicts, "tiny", torch.bfloat16, cuda_device)
    prompts = rec["prompts"]
    for draft, key in ((m, "spec_self"), (hostile, "spec_hostile")):
        tp = PagedKVCache.for_model(m, num_blocks=512, block_size=16)
        dp = PagedKVCache.for_model(m, num_blocks=512, block_size=16)
        res, _ = speculative_greedy_batch(m, draft, prompts, tp, dp, k=4, max_new_tokens=[20, 13, 20],
                                          eos_token_id=None)
        for i, r in enumerate(res):
            want = rec[key]["4"][i]["tokens"]
            assert r.new_token_ids == want[: len(r.new_token_ids)]
            assert len(r.new_token_ids) == (13 if i == 1 else 20)
        assert tp.manager.num_allocated == 0 and dp.manager.num_allocated == 0


@pytest.fixture(scope="module")
def cfg1_model(cuda_device):
    from kvengine_b200.config import QWEN2_0_5B

    return Model.random_init(QWEN2_0_5B, seed=0, dtype=torch.float32, device=cuda_device, init_device="cpu")


def test_config1_self_spec_full_acceptance_and_greedy_identity(cuda_device, cfg1_model):
    """Config 1: 0.5B arch, seed 0, fp32, 4 requests x 64 random ids, 64 new tokens, k=4, bs=16:
    acceptance exactly 100% and tokens identical to the reference's spec and greedy output."""
    g = load_golden("cfg1")
    m = cfg1_model
    tp = PagedKVCache.for_model(m, num_blocks=512, block_size=16)
    dp = PagedKVCache.for_model(m, num_blocks=512, block_size=16)
    res, _ = speculative_greedy_batch(m, m, g["prompts"], tp, dp, k=4, max_new_tokens=64, eos_token_id=None)
    for i, r in enumerate(res):
        assert r.acceptance_rate == 1.0, (i, r.accepted_per_iter)
        assert r.new_token_ids == g["spec"][i]["tokens"] == g["greedy"][i]
    pool = PagedKVCache.for_model(m, num_blocks=512, block_size=16)
    gr = greedy_batch(m, g["prompts"], pool, 64, eos_token_id=None, collect_logits=True)
    for i, r in enumerate(gr):
        assert r.new_token_ids == g["greedy"][i]
        top = torch.tensor(g["greedy_top2"][i]["values"])
        got = r.step_logits.topk(2, dim=-1).values
        assert (got - top).abs().max().item() <= 1e-3


def test_config1_logits_within_1e3_of_oracle(cuda_device, cfg1_model):
    """Teacher-forced prompt + generated tokens: every row of our fp32 logits within 1e-3 of the oracle."""
    from kvengine_b200.config import QWEN2_0_5B
    from kvengine_b200.weights import init_state_dict

    g = load_golden("cfg1")
    seqv = g["prompts"][0] + g["greedy"][0][:20]
    om = OracleModel(QWEN2_0_5B, init_state_dict(QWEN2_0_5B, seed=0), torch.float32)
    opool = OraclePool(24, 2, 64, 64, 16, torch.float32)
    ref = oracle_forward(om, seqv, opool.new_sequence(), all_logits=True)
    pool = PagedKVCache.for_model(cfg1_model, num_blocks=64, block_size=16)
    got = forward_with_own_cache(cfg1_model, torch.tensor([seqv], device=cuda_device), pool.new_sequence("x"),
                                 all_logits=True)[0].cpu()
    assert (got - ref).abs().max().item() <= 1e-3


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_layer_ranges_and_graphs_compose_bit_identically(cuda_device, dtype):
    """A pass split into stream-launched layers [0, e) and a graph-launched rest
    [e, n) (kve_forward_layers + kve_forward_layers_graphed, the spec engine's first
    draft pass) computes exactly what one kve_forward call computes, for e = 0, 1,
    n/2 and n, with one graph slot reused across every split and pass shape (the
    executable graph is updated in place or rebuilt): logits and the K/V pool are
    bit-identical."""
    from dataclasses import replace

    from kvengine_b200.config import TINY
    from kvengine_b200.forward import runner_for
    from kvengine_b200.model import ForwardPlan, SeqSpec
    from kvengine_b200.weights import init_state_dict

    cfg = replace(TINY, num_layers=6)
    m = Model(cfg, init_state_dict(cfg, seed=9, bias_std=0.02, norm_jitter=0.1), dtype, cuda_device)
    pool = PagedKVCache.for_model(m, num_blocks=32, block_size=16)
    runner = runner_for(m, pool)
    g = torch.Generator().manual_seed(5)
    chunks = [torch.randint(0, cfg.vocab_size, (T,), generator=g).to(torch.int32) for T in (37, 5, 1)]
    stream = torch.cuda.Stream(device=cuda_device)

    def run(graph, eager):
        pool.manager.reset()            # same blocks, same slots, every run
        pool.k.zero_()
        pool.v.zero_()
        seq = pool.new_sequence("x")
        outs = []
        with torch.cuda.stream(stream):
            for ids in chunks:
                T = ids.numel()
                start = seq.length
                seq.reserve(T)
                plan = ForwardPlan([SeqSpec(start, T, list(seq.blocks), n_out=T)], pool.block_size)
                logits = torch.empty(T, cfg.vocab_size, dtype=dtype, device=cuda_device)
                runner.forward(plan, ids.to(cuda_device), logits, graph=graph, eager_layers=eager)
                seq.commit(T)
                outs.append(logits)
        stream.synchronize()
        state = ([o.cpu() for o in outs], pool.k.cpu().clone(), pool.v.cpu().clone())
        seq.free()
        return state

    ref = run(None, 0)
    for e in (0, 1, cfg.num_layers // 2, cfg.num_layers):
        got = run("split", e)
        for a, b in zip(got[0], ref[0]):
            assert torch.equal(a, b), e
        assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2]), e
    assert runner.graph_fallbacks == []
    runner.check_status()


def test_spec_next_draft_plan_matches_host_plan(cuda_device):
    """kve_spec_next_draft_plan writes, on the device, the plan the host builds for
    the next step's first draft pass (ForwardPlan.from_arrays over the same tables):
    one row (position T0 + n, bonus token) or two rows (T0 + n - 1 with the token
    there, then the bonus) per sequence, for every accepted count n in 0..k; rows
    past a sequence's blocks read and write the dump block."""
    import numpy as np

    from kvengine_b200 import ops
    from kvengine_b200.model import ForwardPlan

    rng = np.random.default_rng(5)
    S, k, bs, dump = 13, 4, 16, 4095
    start = rng.integers(1, 300, S)
    start[:3] = [16 - k + 1, 32 - k, 48 - k - 1]          # rows landing at a block boundary
    nb = (start + k - 2) // bs + 1                         # the draft's reservation: up to T0 + k - 2
    width = int(nb.max()) + 2
    ids = rng.permutation(4000)[: int(nb.sum())]
    tables = np.zeros((S, width), dtype=np.int64)
    tables[np.arange(width) < nb[:, None]] = ids
    n_acc = np.concatenate([[k - 1, k, k - 1, 0, k], rng.integers(0, k + 1, S - 5)])
    emitted = np.full((S, k + 1), -1, dtype=np.int64)
    for s in range(S):
        emitted[s, : n_acc[s] + 1] = rng.integers(0, 151936, n_acc[s] + 1)
    last = rng.integers(0, 151936, S)

    def dev(a):
        return torch.tensor(np.ascontiguousarray(a), dtype=torch.int32, device=cuda_device).reshape(-1)

    full = np.where(np.arange(width) < nb[:, None], tables, dump)   # the table the plan uses
    for rows in (1, 2):
        desc = ForwardPlan.device_built(S, rows, width, int(start.max()) + k + 1, bs)
        plan = torch.full((desc.size + 8,), -99, dtype=torch.int32, device=cuda_device)
        out_ids = torch.full((2 * S,), -99, dtype=torch.int32, device=cuda_device)
        vids = torch.full((S * (k + 1),), -99, dtype=torch.int32, device=cuda_device)
        status = ops.status_tensor(cuda_device)
        ops.spec_next_draft_plan(dev(start), dev(last), dev(nb), dev(tables), bs, k, rows, dump, dev(n_acc),
                                 dev(emitted), plan, out_ids, vids, status=status)
        ops.check_status(status)
        if rows == 1:
            first = start + np.minimum(n_acc, k - 1)
            want_ids = emitted[np.arange(S), n_acc]
        else:
            first = start + n_acc - 1
            prev = np.where(n_acc > 0, emitted[np.arange(S), np.maximum(n_acc - 1, 0)], last)
            want_ids = np.stack([prev, emitted[np.arange(S), n_acc]], 1).reshape(-1)
        host = ForwardPlan.from_arrays(first, np.full(S, rows), np.ones(S, dtype=np.int64), full,
                                       np.full(S, width), bs)
        assert host.offsets == desc.offsets and host.n_tokens == desc.n_tokens and host.width == desc.width
        assert plan[: desc.size].cpu().numpy().tolist() == host.host.tolist(), rows
        assert plan[desc.size:].cpu().tolist() == [-99] * 8
        assert out_ids[: rows * S].cpu().numpy().tolist() == want_ids.tolist()
        v = vids.view(S, k + 1).cpu().numpy()
        assert v[:, 0].tolist() == emitted[np.arange(S), n_acc].tolist()
        assert (v[:, 1:] == -99).all()
        # rows past a sequence's blocks (set up at the block boundaries above) hit the dump block
        pos_last = first + rows - 1
        slots = plan[desc.offsets["slots"][0]: desc.offsets["slots"][0] + rows * S].cpu().numpy()
        hit = pos_last >= nb * bs
        assert hit[0] and (rows == 1 or hit[1])
        assert ((slots.reshape(S, rows)[:, -1] // bs == dump) == hit).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_speculated_first_draft_pass_changes_no_token(cuda_device, tiny_state_dicts, dtype):
    """The first draft pass of each step queued before the accept readback (planned
    on the device) gives exactly the tokens, acceptances and final free lists of the
    host-planned pass: with a hostile draft (one-row plans, used) and a self draft
    (two-row plans after the first full acceptance), ragged prompts and budgets
    (the request list shrinks, so some queued passes are discarded)."""
    from kvengine_b200 import SpecEngine

    cfg, m, hostile = _models(tiny_state_dicts, "tiny", dtype, cuda_device)
    g = torch.Generator().manual_seed(17)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 23, 40, 9, 17, 31)]
    ragged = [20, 13, 26, 31, 8, 24]
    for draft, k, budgets in ((hostile, 4, ragged), (hostile, 1, ragged), (m, 3, ragged), (m, 3, [40] * 6),
                              (m, 4, [33] * 6)):
        outs = []
        for spec in (False, True):
            tp = PagedKVCache.for_model(m, num_blocks=256, block_size=16)
            dp = PagedKVCache.for_model(m, num_blocks=256, block_size=16)
            eng = SpecEngine(m, draft, tp, dp, k, speculate=spec)
            res, _ = speculative_greedy_batch(m, draft, prompts, tp, dp, k=k, max_new_tokens=budgets,
                                              eos_token_id=None, engine=eng)
            eng.check()
            outs.append(([r.new_token_ids for r in res], [r.accepted_per_iter for r in res],
                         list(tp.manager._stack), list(dp.manager._stack)))
            if spec and (draft is hostile or budgets != ragged):
                assert eng.spec_stats["used"] > 0, (k, eng.spec_stats)
            assert tp.manager.num_allocated == 0 and dp.manager.num_allocated == 0
        assert outs[0] == outs[1], (k, draft is m)
