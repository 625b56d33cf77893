"""Pin the CPU oracle to the reference: every golden vector the reference
produced (tests/golden/make_golden.py ran kvengine itself) must come out of
the oracle restatement unchanged. CPU only."""

import hashlib

import numpy as np
import pytest
import torch

from conftest import load_golden, load_golden_arrays
from kvengine_b200 import workloads
from oracle.accept import oracle_accept, oracle_accept_tables
from oracle.attention import oracle_paged_attention
from oracle.model import OracleModel
from oracle.paged import OraclePool
from oracle.spec import oracle_greedy_paged, oracle_speculative_greedy


def _sha(t: torch.Tensor) -> str:
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


@pytest.fixture(scope="module")
def tiny_golden():
    return load_golden("tiny"), load_golden_arrays("tiny")


CASES = [("tiny", "f32", torch.float32), ("tiny", "bf16", torch.bfloat16), ("tiny_hd128", "f32", torch.float32)]


@pytest.mark.parametrize("cfg_name,dt_name,dtype", CASES)
def test_oracle_greedy_matches_reference(tiny_golden, tiny_state_dicts, cfg_name, dt_name, dtype):
    g, arr = tiny_golden
    rec = g[f"{cfg_name}_{dt_name}"]
    cfg, sd = tiny_state_dicts[cfg_name]
    m = OracleModel(cfg, sd, dtype)
    for i, p in enumerate(rec["prompts"]):
        pool = OraclePool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 256, 16, dtype)
        log = []
        out = oracle_greedy_paged(m, p, pool.new_sequence(), 20, logits_log=log)
        assert out["new_token_ids"] == rec["greedy"][i]
        ref = torch.from_numpy(arr[f"{cfg_name}_{dt_name}_greedy_logits_{i}"])
        assert (torch.stack(log) - ref).abs().max().item() == 0.0


@pytest.mark.parametrize("cfg_name,dt_name,dtype", CASES)
def test_oracle_spec_matches_reference(tiny_golden, tiny_state_dicts, cfg_name, dt_name, dtype):
    g, _ = tiny_golden
    rec = g[f"{cfg_name}_{dt_name}"]
    cfg, sd = tiny_state_dicts[cfg_name]
    m = OracleModel(cfg, sd, dtype)
    hostile = OracleModel(cfg, sd, dtype, roll_head=1)
    for k in (1, 2, 4, 8):
        for i, p in enumerate(rec["prompts"]):
            for draft, key in ((m, "spec_self"), (hostile, "spec_hostile")):
                pool = OraclePool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 256, 16, dtype)
                out = oracle_speculative_greedy(m, draft, p, pool.new_sequence(), pool.new_sequence(), k=k,
                                                max_new_tokens=20)
                want = rec[key][str(k)][i]
                assert out["new_token_ids"] == want["tokens"], (key, k, i)
                assert out["accepted_per_iter"] == want["accepted_per_iter"]
                assert out["target_forwards"] == want["target_forwards"]
                assert out["draft_forwards"] == want["draft_forwards"]


def test_oracle_budgets_eos_blocksizes_rollback(tiny_golden, tiny_state_dicts):
    g, _ = tiny_golden
    rec = g["tiny_f32"]
    cfg, sd = tiny_state_dicts["tiny"]
    m = OracleModel(cfg, sd, torch.float32)
    p = rec["prompts"][1]

    def pool(n=256, bs=16):
        return OraclePool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, n, bs, torch.float32)

    for budget, want in rec["budgets"].items():
        pl = pool()
        out = oracle_speculative_greedy(m, m, p, pl.new_sequence(), pl.new_sequence(), k=4,
                                        max_new_tokens=int(budget))
        assert out["new_token_ids"] == want
    for bs, want in rec["block_sizes"].items():
        pl = pool(512, int(bs))
        assert oracle_greedy_paged(m, p, pl.new_sequence(), 16)["new_token_ids"] == want
    e = rec["eos"]
    pl = pool()
    out = oracle_speculative_greedy(m, m, p, pl.new_sequence(), pl.new_sequence(), k=4, max_new_tokens=20,
                                    eos_ids={e["eos_id"]})
    assert out["new_token_ids"] == e["tokens"] and out["stopped_on_eos"] == e["stopped"]
    rb = rec["rollback"]
    pl = pool(64, 4)
    t, d = pl.new_sequence(), pl.new_sequence()
    hostile = OracleModel(cfg, sd, torch.float32, roll_head=1)
    out = oracle_speculative_greedy(m, hostile, p, t, d, k=8, max_new_tokens=16)
    assert out["new_token_ids"] == rb["tokens"]
    assert (t.blocks, d.blocks, t.length, d.length) == (rb["t_blocks"], rb["d_blocks"], rb["t_len"], rb["d_len"])
    assert pl.alloc.free_list == rb["free_list"]


@pytest.mark.parametrize("k", [1, 2, 4, 8])
def test_oracle_accept_matches_reference(k):
    g = load_golden("accept")[str(k)]
    arr = load_golden_arrays("accept")
    w = workloads.accept_workload(k)
    n, emitted, preds = oracle_accept(w.logits.numpy(), w.drafts.numpy())
    assert n.tolist() == g["n_accepted"]
    assert [list(e[: nn + 1]) for e, nn in zip(emitted.tolist(), n.tolist())] == g["emitted"]
    assert _sha(torch.from_numpy(preds.astype(np.int64))) == g["preds_sha"]
    tables, free_list, lens = oracle_accept_tables(w.pre_len, k, n.tolist(), num_blocks=32768, block_size=16)
    flat = np.array([x for t in tables for x in t], dtype=np.int32)
    assert np.array_equal(flat, arr[f"k{k}_tables_flat"])
    assert np.array_equal(np.array([len(t) for t in tables], np.int32), arr[f"k{k}_tables_len"])
    assert np.array_equal(np.array(free_list, np.int32), arr[f"k{k}_free_list"])
    assert lens == g["seq_len_after"]


def test_oracle_attention_matches_reference():
    g = load_golden("attention")
    arr = load_golden_arrays("attention")
    w = workloads.attention_workload()
    assert w.ctx_lens == g["ctx_lens"]
    out, pool_k, _, gathered = oracle_paged_attention(w, return_gathered=True)
    for b, (kk, vv) in enumerate(gathered):
        assert _sha(kk[None]) == g["k_gather_sha"][b]
        assert _sha(vv[None]) == g["v_gather_sha"][b]
    used = torch.tensor([x for t in w.tables for x in t])
    assert _sha(pool_k[used]) == g["pool_k_used_sha"]
    ref = torch.from_numpy(arr["attn_out_bf16"]).view(torch.bfloat16)
    assert torch.equal(out, ref)


def test_oracle_cfg1_request0_matches_reference():
    """Config 1 (0.5B arch, seed 0, fp32): request 0, greedy and self-spec k=4, 64 tokens."""
    from kvengine_b200.config import QWEN2_0_5B
    from kvengine_b200.weights import init_state_dict

    torch.set_num_threads(max(1, torch.get_num_threads()))
    g = load_golden("cfg1")
    sd = init_state_dict(QWEN2_0_5B, seed=0)
    m = OracleModel(QWEN2_0_5B, sd, torch.float32)
    p = g["prompts"][0]
    cfg = QWEN2_0_5B
    pool = OraclePool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 512, 16, torch.float32)
    out = oracle_speculative_greedy(m, m, p, pool.new_sequence(), pool.new_sequence(), k=4, max_new_tokens=64)
    assert out["new_token_ids"] == g["spec"][0]["tokens"] == g["greedy"][0] == g["hf_greedy_0"]
    assert out["accepted_per_iter"] == g["spec"][0]["accepted_per_iter"]


# ------------------------------------------------ benchmark layer shapes (two layers, bf16)
@pytest.fixture(scope="module")
def shape3b_oracles(shape3b_state_dicts):
    (t_cfg, t_sd), (d_cfg, d_sd) = shape3b_state_dicts["target"], shape3b_state_dicts["draft"]
    return {"target": OracleModel(t_cfg, t_sd, torch.bfloat16), "small": OracleModel(d_cfg, d_sd, torch.bfloat16),
            "hostile": OracleModel(t_cfg, t_sd, torch.bfloat16, roll_head=1)}


def _pool_for(m, n=256, bs=16):
    c = m.cfg
    return OraclePool(c.num_layers, c.num_kv_heads, c.head_dim, n, bs, torch.bfloat16)


def test_oracle_shape3b_greedy_matches_reference(shape3b_oracles):
    """3B-shape target, bf16: greedy tokens and the bit pattern of every step's logits."""
    g = load_golden("shape3b")
    tm = shape3b_oracles["target"]
    for i, p in enumerate(g["prompts"]):
        log = []
        out = oracle_greedy_paged(tm, p, _pool_for(tm).new_sequence(), g["new_tokens"], logits_log=log)
        assert out["new_token_ids"] == g["greedy"][i]
        assert _sha(torch.stack(log)) == g["greedy_logits_sha"][i]


@pytest.mark.parametrize("name", ["self", "small", "hostile"])
def test_oracle_shape3b_spec_matches_reference(shape3b_oracles, name):
    g = load_golden("shape3b")
    tm = shape3b_oracles["target"]
    dm = shape3b_oracles["target" if name == "self" else name]
    for k in (1, 2, 4, 8):
        for i, p in enumerate(g["prompts"]):
            out = oracle_speculative_greedy(tm, dm, p, _pool_for(tm).new_sequence(), _pool_for(dm).new_sequence(),
                                            k=k, max_new_tokens=g["new_tokens"])
            want = g["spec"][name][str(k)][i]
            assert out["new_token_ids"] == want["tokens"], (name, k, i)
            assert out["accepted_per_iter"] == want["accepted_per_iter"]
            assert (out["target_forwards"], out["draft_forwards"]) == (want["target_forwards"],
                                                                       want["draft_forwards"])


def test_oracle_shape3b_rollback_tables_match_reference(shape3b_oracles):
    g = load_golden("shape3b")
    rb = g["rollback"]
    tm, dm = shape3b_oracles["target"], shape3b_oracles["small"]
    tp, dp = _pool_for(tm, 512, 4), _pool_for(dm, 512, 4)
    t, d = tp.new_sequence(), dp.new_sequence()
    out = oracle_speculative_greedy(tm, dm, g["prompts"][1], t, d, k=8, max_new_tokens=g["new_tokens"])
    assert out["new_token_ids"] == rb["tokens"]
    assert (t.blocks, d.blocks, t.length, d.length) == (rb["t_blocks"], rb["d_blocks"], rb["t_len"], rb["d_len"])
    assert tp.alloc.free_list == rb["t_free"] and dp.alloc.free_list == rb["d_free"]


@pytest.mark.parametrize("name", ["config4", "lognormal"])
def test_oracle_attention_hd128_matches_reference(name):
    """The 3B target's verify attention (16/2 heads, head_dim 128): gather hashes and
    the bf16 output bit for bit."""
    g = load_golden("attention_hd128")[name]
    arr = load_golden_arrays("attention_hd128")
    kw = {} if name == "lognormal" else {"median_ctx": 165.0, "sigma": 0.1, "ctx_clip": (133, 197)}
    w = workloads.attention_workload(seed=7, num_heads=16, num_kv_heads=2, head_dim=128, **kw)
    assert w.ctx_lens == g["ctx_lens"]
    out, _, _, gathered = oracle_paged_attention(w, return_gathered=True)
    for b, (kk, _) in enumerate(gathered):
        assert _sha(kk[None]) == g["k_gather_sha"][b]
    ref = torch.from_numpy(arr[f"{name}_attn_out_bf16"]).view(torch.bfloat16)
    assert torch.equal(out, ref.view_as(out))
