"""Kernel parity on the GPU, each entry point through the C ABI against the CPU oracle.

Bit-exact for integer/copy work (accept, argmax, append, gather, embed, RoPE);
fp32 kernels within 1e-5 relative of an fp64/fp32 reference; bf16 attention
within the 2e-2 absolute tolerance the task states for bf16 logits.
"""

import ctypes
import hashlib
import time

import numpy as np
import pytest
import torch

from conftest import load_golden, load_golden_arrays
from kvengine_b200 import _lib as L
from kvengine_b200 import ops, workloads
from oracle.accept import oracle_accept, oracle_accept_tables
from oracle.attention import build_pool, gather, oracle_paged_attention

pytestmark = pytest.mark.gpu


def _sha(t):
    t = t.contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


# ------------------------------------------------------------------ accept
@pytest.mark.parametrize("k", [1, 2, 4, 8])
def test_accept_config3_bit_exact(cuda_device, k):
    """Config 3: [256, k+1, 151936] fp32 -> accepted length, emitted tokens,
    truncated block tables and free list, all against the reference's outputs."""
    from kvengine_b200.paged import PagedKVCache

    g = load_golden("accept")[str(k)]
    arr = load_golden_arrays("accept")
    w = workloads.accept_workload(k)
    logits = w.logits.to(cuda_device)
    drafts = w.drafts.to(torch.int32).to(cuda_device)
    preds, n_acc, emitted = ops.greedy_accept(logits, drafts)
    n = n_acc.cpu().tolist()
    assert n == g["n_accepted"]
    em = emitted.cpu().tolist()
    assert [e[: nn + 1] for e, nn in zip(em, n)] == g["emitted"]
    assert all(x == -1 for e, nn in zip(em, n) for x in e[nn + 1:])
    assert _sha(preds.cpu().to(torch.int64)) == g["preds_sha"]
    # block tables through kvengine_b200's own PagedSequenceCache/BlockManager
    pool = PagedKVCache(1, 1, 8, 32768, 16, torch.float32, "cpu")
    seqs = [pool.new_sequence(b) for b in range(w.logits.shape[0])]
    for b, s in enumerate(seqs):
        s.reserve(w.pre_len[b])
        s.commit(w.pre_len[b])
    for s in seqs:
        s.reserve(k + 1)
        s.commit(k + 1)
    for b, s in enumerate(seqs):
        s.truncate(min(s.length, w.pre_len[b] + n[b] + 1))
    flat = np.array([x for s in seqs for x in s.blocks], dtype=np.int32)
    assert np.array_equal(flat, arr[f"k{k}_tables_flat"])
    assert np.array_equal(np.array(pool.manager.free_list, np.int32), arr[f"k{k}_free_list"])


def test_accept_bf16_ties_nan_and_k31(cuda_device):
    g = torch.Generator().manual_seed(5)
    B, k, V = 9, 31, 1000
    logits = torch.randn(B, k + 1, V, generator=g).to(torch.bfloat16)
    drafts = torch.randint(0, V, (B, k), generator=g)
    # plant matches, an exact tie (lower index must win) and a NaN (counts as max)
    for b in range(B):
        for j in range(b * 3):
            if j < k:
                logits[b, j, drafts[b, j]] = 30.0
    logits[1, 3, 10] = 40.0
    logits[1, 3, 5] = 40.0
    logits[2, 0, 7] = float("nan")
    logits[2, 0, 900] = float("nan")
    ref_n, ref_em, ref_p = oracle_accept(logits.float().numpy(), drafts.numpy())
    assert ref_p[1, 3] == 5 and ref_p[2, 0] == 7
    preds, n_acc, emitted = ops.greedy_accept(logits.to(cuda_device), drafts.to(torch.int32).to(cuda_device))
    assert np.array_equal(preds.cpu().numpy(), ref_p)
    assert np.array_equal(n_acc.cpu().numpy(), ref_n)
    assert np.array_equal(emitted.cpu().numpy(), ref_em)


def test_accept_workspace_stays_zero_and_repeats(cuda_device):
    w = workloads.accept_workload(4, batch=16, vocab=4096, seed=9)
    ws = ops.Workspace(cuda_device)
    lg, dr = w.logits.to(cuda_device), w.drafts.to(torch.int32).to(cuda_device)
    a = ops.greedy_accept(lg, dr, ws)
    assert int(ws.buf.abs().sum()) == 0
    b = ops.greedy_accept(lg, dr, ws)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    # results written into views of one caller buffer (emitted, then n_accepted)
    B, kp1 = dr.shape[0], dr.shape[1] + 1
    buf = torch.full((B * (kp1 + 1),), -7, dtype=torch.int32, device=cuda_device)
    preds = torch.empty(B, kp1, dtype=torch.int32, device=cuda_device)
    c = ops.greedy_accept(lg, dr, ws, out=(preds, buf[B * kp1:], buf[:B * kp1].view(B, kp1)))
    for x, y in zip(a, c):
        assert torch.equal(x, y)


def test_argmax_rows(cuda_device):
    g = torch.Generator().manual_seed(1)
    for dt in (torch.float32, torch.bfloat16):
        x = torch.randn(37, 151936, generator=g).to(dt)
        x[3, 100] = x[3, 200] = 1e4
        got = ops.argmax_rows(x.to(cuda_device)).cpu()
        assert torch.equal(got.long(), torch.argmax(x.float(), -1))
    x = torch.randn(5, 1001, generator=g)  # unaligned rows take the scalar path
    assert torch.equal(ops.argmax_rows(x.to(cuda_device)).cpu().long(), x.argmax(-1))


def test_argmax_rows_split_over_parts(cuda_device):
    """Few long rows split each row over a cluster of CTAs (8 parts of 18,992 columns
    here): a tie across a part boundary resolves to the lower index, the first NaN is
    the maximum, an all -inf row gives 0 - every row equal to torch.argmax."""
    g = torch.Generator().manual_seed(9)
    for dt in (torch.float32, torch.bfloat16):
        x = torch.randn(8, 151936, generator=g).to(dt)
        x[0, 18991] = x[0, 18992] = 100.0                 # the two sides of the first part boundary
        x[1, 18992 * 3 + 5] = x[1, 18992 * 7 + 1] = 100.0
        x[2, 100000] = x[2, 150000] = float("nan")
        x[3, :] = float("-inf")
        x[4, 151935] = 100.0                              # the last column
        got = ops.argmax_rows(x.to(cuda_device)).cpu().long()
        assert torch.equal(got, torch.argmax(x.float(), -1)), (dt, got)
        assert got[:5].tolist() == [18991, 18992 * 3 + 5, 100000, 0, 151935]


def test_argmax_rows_scatter_places_drafts_in_the_verify_feed(cuda_device):
    """The draft loop's argmax writes each row's token both to the drafts buffer and
    to its slot of the verify pass's token ids (kvengine speculative.py:160-162:
    unseen tokens followed by the drafts); an index outside the feed is skipped and
    reported as KVE_ERR_BOUNDS."""
    g = torch.Generator().manual_seed(4)
    x = torch.randn(6, 151936, generator=g).to(torch.bfloat16)
    x[2, 7] = x[2, 9] = 50.0                                     # tie: the lower index wins
    feed = torch.full((40,), -5, dtype=torch.int32)
    idx = torch.tensor([3, 11, 12, 20, 39, 0], dtype=torch.int32)
    status = ops.status_tensor(cuda_device)
    feed_d = feed.to(cuda_device)
    got = ops.argmax_rows(x.to(cuda_device), scatter_index=idx.to(cuda_device), scatter_out=feed_d,
                          status=status).cpu()
    want = torch.argmax(x.float(), -1).to(torch.int32)
    assert torch.equal(got, want) and int(got[2]) == 7
    feed[idx.long()] = want
    assert torch.equal(feed_d.cpu(), feed)
    assert int(status.item()) == 0
    bad = torch.tensor([0, 1, 2, 3, 40, 5], dtype=torch.int32, device=cuda_device)
    ops.argmax_rows(x.to(cuda_device), scatter_index=bad, scatter_out=feed_d, status=status)
    assert int(status.item()) == -7  # KVE_ERR_BOUNDS; the other rows were still written


# ------------------------------------------------------------------ append / gather / rope
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_kv_append_matches_index_copy(cuda_device, dtype):
    g = torch.Generator().manual_seed(2)
    nb, bs, nkv, hd, n = 64, 16, 2, 64, 37
    pk = torch.randn(nb, bs, nkv, hd, generator=g).to(dtype)
    pv = torch.randn(nb, bs, nkv, hd, generator=g).to(dtype)
    kn = torch.randn(n, nkv, hd, generator=g).to(dtype)
    vn = torch.randn(n, nkv, hd, generator=g).to(dtype)
    slots = torch.randperm(nb * bs, generator=g)[:n]
    ref_k, ref_v = pk.clone(), pv.clone()
    ref_k.view(-1, nkv, hd).index_copy_(0, slots, kn)
    ref_v.view(-1, nkv, hd).index_copy_(0, slots, vn)
    dk, dv = pk.to(cuda_device), pv.to(cuda_device)
    ops.kv_append(kn.to(cuda_device), vn.to(cuda_device), slots.to(cuda_device), dk, dv)
    assert torch.equal(dk.cpu(), ref_k) and torch.equal(dv.cpu(), ref_v)


def test_kv_append_rejects_out_of_range_slot(cuda_device):
    nb, bs, nkv, hd = 4, 16, 2, 64
    dk = torch.zeros(nb, bs, nkv, hd, device=cuda_device)
    dv = torch.zeros_like(dk)
    kn = torch.ones(2, nkv, hd, device=cuda_device)
    status = ops.status_tensor(cuda_device)
    slots = torch.tensor([3, nb * bs], device=cuda_device)
    ops.kv_append(kn, kn, slots, dk, dv, status=status)
    assert int(status.item()) == -7  # KVE_ERR_BOUNDS
    assert dk.view(-1, nkv, hd)[3].eq(1).all() and int(dk.ne(0).sum()) == nkv * hd


@pytest.mark.parametrize("bs", [1, 3, 16, 17])
def test_gather_kv_in_table_order(cuda_device, bs):
    g = torch.Generator().manual_seed(bs)
    nb, nkv, hd = 40, 2, 128
    pool = torch.randn(nb, bs, nkv, hd, generator=g).to(torch.bfloat16)
    table = torch.randperm(nb, generator=g)[:9].tolist()[::-1]
    length = min(len(table) * bs, 5 * bs + 2)
    ref = gather(pool, table, length, bs)
    got = ops.gather_kv(pool.to(cuda_device), torch.tensor(table, dtype=torch.int32, device=cuda_device), length)
    assert torch.equal(got.cpu(), ref)


@pytest.mark.parametrize("dtype,hd", [(torch.float32, 64), (torch.bfloat16, 64), (torch.float32, 128),
                                      (torch.bfloat16, 128)])
def test_qkv_rope_append_bit_exact(cuda_device, dtype, hd):
    from kvengine_b200.config import ModelConfig
    from kvengine_b200.weights import rope_tables
    from oracle.model import OracleModel, _rotate_half

    nq, nkv, n = 4, 2, 11
    cfg = ModelConfig(num_layers=1, hidden_size=nq * hd, num_heads=nq, num_kv_heads=nkv, head_dim=hd,
                      intermediate_size=64, vocab_size=16)
    om = OracleModel(cfg, {}, dtype)
    g = torch.Generator().manual_seed(4)
    qkv = torch.randn(n, (nq + 2 * nkv) * hd, generator=g).to(dtype)
    pos = torch.tensor([0, 1, 2, 15, 16, 17, 100, 511, 512, 4000, 4095])
    nb, bs = 8, 16
    slots = torch.randperm(nb * bs, generator=g)[:n]
    cos, sin = om.rope(pos)
    q = qkv[:, : nq * hd].view(n, nq, hd)
    k = qkv[:, nq * hd:(nq + nkv) * hd].view(n, nkv, hd)
    v = qkv[:, (nq + nkv) * hd:].view(n, nkv, hd)
    q_ref = q * cos[:, None] + _rotate_half(q) * sin[:, None]
    k_ref = k * cos[:, None] + _rotate_half(k) * sin[:, None]
    tc, ts = rope_tables(cfg, 4096)
    dk = torch.zeros(nb, bs, nkv, hd, dtype=dtype, device=cuda_device)
    dv = torch.zeros_like(dk)
    q_out = torch.empty(n, nq, hd, dtype=dtype, device=cuda_device)
    ops.qkv_rope_append(qkv.to(cuda_device), pos.to(torch.int32).to(cuda_device),
                        slots.to(torch.int32).to(cuda_device), tc.to(cuda_device), ts.to(cuda_device), q_out, dk,
                        dv, nq, nkv, hd)
    assert torch.equal(q_out.cpu(), q_ref)
    assert torch.equal(dk.cpu().view(-1, nkv, hd)[slots], k_ref)
    assert torch.equal(dv.cpu().view(-1, nkv, hd)[slots], v)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rmsnorm_and_embed(cuda_device, dtype):
    from kvengine_b200.config import TINY
    from oracle.model import OracleModel

    g = torch.Generator().manual_seed(6)
    x = torch.randn(13, 896, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(896, generator=g)).to(dtype)
    om = OracleModel(TINY, {}, dtype)
    ref = om.rmsnorm(x, w)
    rows = torch.tensor([12, 0, 5], dtype=torch.int32)
    got = ops.rmsnorm(x.to(cuda_device), w.float().to(cuda_device), 1e-6, row_index=rows.to(cuda_device)).cpu()
    if dtype == torch.float32:
        torch.testing.assert_close(got, ref[rows.long()], rtol=2e-6, atol=1e-6)
    else:  # at most one bf16 ulp from a different sum order of mean(x^2)
        assert ((got.float() - ref[rows.long()].float()).abs() <= ref[rows.long()].float().abs() / 128 + 1e-6).all()
    table = torch.randn(50, 256, generator=g).to(dtype)
    ids = torch.tensor([3, 49, 0, 3], dtype=torch.int32)
    assert torch.equal(ops.embed(ids.to(cuda_device), table.to(cuda_device)).cpu(), table[ids.long()])


# ------------------------------------------------------------------ attention
def _attn_inputs(w, device, pool_k=None, pool_v=None):
    B = w.num_seqs
    width = max(len(t) for t in w.tables)
    tables = torch.zeros(B, width, dtype=torch.int32)
    for b, t in enumerate(w.tables):
        tables[b, : len(t)] = torch.tensor(t, dtype=torch.int32)
    ctx = torch.tensor(w.ctx_lens, dtype=torch.int32)
    ql = torch.full((B,), w.q_len, dtype=torch.int32)
    qo = torch.arange(B + 1, dtype=torch.int32) * w.q_len
    return [t.to(device) for t in (tables, ctx, ql, qo)]


def test_attention_config2_layout_and_output(cuda_device):
    """Config 2: 64 seqs x 5 queries, 14/2 heads, hd 64, bf16, lognormal ctx up to 4096."""
    g = load_golden("attention")
    arr = load_golden_arrays("attention")
    w = workloads.attention_workload()
    nkv, hd = w.k_new.shape[1], w.k_new.shape[2]
    # Build the pool on the device with the append kernel: history, then the q_len new rows.
    dk = torch.zeros(w.num_blocks, w.block_size, nkv, hd, dtype=torch.bfloat16, device=cuda_device)
    dv = torch.zeros_like(dk)
    bs = w.block_size
    for b, ctx in enumerate(w.ctx_lens):
        ids = torch.tensor(w.tables[b])
        pos = torch.arange(ctx)
        slots = (ids[pos // bs] * bs + pos % bs).to(cuda_device)
        rows = slice(b * w.q_len, (b + 1) * w.q_len)
        hist = ctx - w.q_len
        ops.kv_append(w.k_hist[b].to(cuda_device), w.v_hist[b].to(cuda_device), slots[:hist], dk, dv)
        ops.kv_append(w.k_new[rows].contiguous().to(cuda_device), w.v_new[rows].contiguous().to(cuda_device),
                      slots[hist:], dk, dv)
    used = torch.tensor([x for t in w.tables for x in t])
    assert _sha(dk.cpu()[used]) == g["pool_k_used_sha"]
    for b in (0, 17, 63):
        table = torch.tensor(w.tables[b], dtype=torch.int32, device=cuda_device)
        assert _sha(ops.gather_kv(dk, table, w.ctx_lens[b])[None]) == g["k_gather_sha"][b]
        assert _sha(ops.gather_kv(dv, table, w.ctx_lens[b])[None]) == g["v_gather_sha"][b]
    tables, ctx, ql, qo = _attn_inputs(w, cuda_device)
    status = ops.status_tensor(cuda_device)
    out = ops.paged_attention(w.q.to(cuda_device), dk, dv, tables, ctx, ql, qo, w.q_len, max(w.ctx_lens),
                              w.scale, status=status)
    assert int(status.item()) == 0
    ref = torch.from_numpy(arr["attn_out_bf16"]).view(torch.bfloat16).float()
    err = (out.float().cpu() - ref).abs().max().item()
    assert err <= 2e-2, err
    ref32, _, _ = oracle_paged_attention(w, compute_dtype=torch.float32)
    err32 = (out.float().cpu() - ref32).abs().max().item()
    assert err32 <= 1e-2, err32


@pytest.mark.parametrize("bs,hd,nq,nkv", [(16, 64, 14, 2), (1, 128, 16, 2), (3, 64, 4, 2), (17, 128, 8, 1)])
def test_attention_fp32_ragged(cuda_device, bs, hd, nq, nkv):
    """fp32, ragged q_lens (1, 2, 5, 9, 40), contexts at block edges and past one chunk."""
    g = torch.Generator().manual_seed(bs + hd)
    q_lens = [1, 2, 5, 9, 40, 5]
    ctx = [1, bs * 4, bs * 4 + 1, 600, 1100, 513]
    num_blocks = sum(-(-c // bs) for c in ctx) + 10
    perm = torch.randperm(num_blocks, generator=g).tolist()
    tables, off = [], 0
    for c in ctx:
        nb = -(-c // bs)
        tables.append(perm[off:off + nb])
        off += nb
    rows = sum(q_lens)
    q = torch.randn(rows, nq, hd, generator=g)
    outs = []
    # oracle per sequence with its own q_len (reusing the config-2 oracle one sequence at a time)
    pool_k = torch.randn(num_blocks, bs, nkv, hd, generator=g)
    pool_v = torch.randn(num_blocks, bs, nkv, hd, generator=g)
    from oracle.model import attend, causal_mask

    start = 0
    for b, c in enumerate(ctx):
        ql = q_lens[b]
        kk = gather(pool_k, tables[b], c, bs)
        vv = gather(pool_v, tables[b], c, bs)
        qq = q[start:start + ql].transpose(0, 1)[None]
        o = attend(qq, kk[None], vv[None], causal_mask(ql, c, torch.float32), hd ** -0.5, nq // nkv, use_sdpa=False)
        outs.append(o[0])
        start += ql
    ref = torch.cat(outs, 0)
    width = max(len(t) for t in tables)
    tt = torch.zeros(len(ctx), width, dtype=torch.int32)
    for b, t in enumerate(tables):
        tt[b, : len(t)] = torch.tensor(t, dtype=torch.int32)
    qo = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32)
    dev = cuda_device
    status = ops.status_tensor(dev)
    got = ops.paged_attention(q.to(dev), pool_k.to(dev), pool_v.to(dev), tt.to(dev),
                              torch.tensor(ctx, dtype=torch.int32, device=dev),
                              torch.tensor(q_lens, dtype=torch.int32, device=dev), qo.to(dev), max(q_lens), max(ctx),
                              hd ** -0.5, status=status)
    assert int(status.item()) == 0
    torch.testing.assert_close(got.cpu(), ref, rtol=1e-5, atol=1e-5)


def test_attention_row_result_is_batch_invariant(cuda_device):
    """A query's output is identical whether it is scored alone (draft pass) or
    as the first of k+1 rows (verify pass), including across chunk boundaries."""
    g = torch.Generator().manual_seed(8)
    nb, bs, nkv, hd, nq = 100, 16, 2, 64, 14
    dev = cuda_device
    pk = torch.randn(nb, bs, nkv, hd, generator=g).to(dev)
    pv = torch.randn(nb, bs, nkv, hd, generator=g).to(dev)
    table = torch.randperm(nb, generator=g)[:80].to(torch.int32).to(dev)[None]
    for pos in (0, 15, 511, 512, 700, 1024):
        q5 = torch.randn(5, nq, hd, generator=g).to(dev)
        one = ops.paged_attention(q5[:1].contiguous(), pk, pv, table, torch.tensor([pos + 1], dtype=torch.int32, device=dev),
                                  torch.tensor([1], dtype=torch.int32, device=dev),
                                  torch.tensor([0, 1], dtype=torch.int32, device=dev), 1, pos + 1, hd ** -0.5)
        five = ops.paged_attention(q5, pk, pv, table, torch.tensor([pos + 5], dtype=torch.int32, device=dev),
                                   torch.tensor([5], dtype=torch.int32, device=dev),
                                   torch.tensor([0, 5], dtype=torch.int32, device=dev), 5, pos + 5, hd ** -0.5)
        assert torch.equal(one[0], five[0]), pos


# ------------------------------------------------------------------ GEMM
SHAPES = [(1, 256, 256), (5, 384, 512), (20, 1152, 896), (64, 896, 4864), (320, 2560, 2048), (300, 200, 136),
          (600, 512, 1024), (17, 1000, 64)]


def _ref_gemm(x, w):
    return (x.double() @ w.double().t()).float()


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_simt_fp32(cuda_device, m, n, k):
    g = torch.Generator().manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g)
    w = torch.randn(n, k, generator=g) * 0.05
    got = ops.gemm(x.to(cuda_device), w.to(cuda_device)).cpu()
    torch.testing.assert_close(got, _ref_gemm(x, w), rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_tcgen05_bf16(cuda_device, m, n, k):
    g = torch.Generator().manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
    status = ops.status_tensor(cuda_device)
    got = ops.gemm(x.to(cuda_device), w.to(cuda_device), out_dtype=torch.float32, status=status).cpu()
    assert int(status.item()) == 0
    ref = _ref_gemm(x.float(), w.float())
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4 * (k ** 0.5))


@pytest.mark.parametrize("algo", [L.GEMM_SIMT, L.GEMM_TCGEN05])
@pytest.mark.parametrize("m,n,k", [(33, 512, 256), (40, 19200, 256), (320, 2560, 2048), (7, 1000, 136),
                                   (330, 40000, 128)])
def test_gemm_epilogues(cuda_device, algo, m, n, k):
    """BIAS / RESIDUAL (in place) / SILU_MUL on split-K (cluster) and unsplit tilings,
    and on persistent launches (more tiles than SMs: 150 and 939 tiles)."""
    dt = torch.bfloat16 if algo == L.GEMM_TCGEN05 else torch.float32
    g = torch.Generator().manual_seed(11)
    x = torch.randn(m, k, generator=g).to(dt)
    w = (torch.randn(n, k, generator=g) * 0.1).to(dt)
    bias = (torch.randn(n, generator=g) * 0.1).to(dt).float()
    res = torch.randn(m, n, generator=g).to(dt)
    acc = _ref_gemm(x.float(), w.float())

    def rnd(t):
        return t.to(dt).float()

    dev = cuda_device
    tol = dict(rtol=1e-2, atol=2e-2 * max(1.0, (k / 256) ** 0.5))
    got = ops.gemm(x.to(dev), w.to(dev), L.EPI_BIAS, bias=bias.to(dev), algo=algo).cpu().float()
    torch.testing.assert_close(got, rnd(acc + bias), **tol)
    r = res.to(dev)
    ops.gemm(x.to(dev), w.to(dev), L.EPI_RESIDUAL, residual=r, out=r, algo=algo)
    torch.testing.assert_close(r.cpu().float(), rnd(res.float() + rnd(acc)), **tol)
    got = ops.gemm(x.to(dev), w.to(dev), L.EPI_SILU_MUL, algo=algo).cpu().float()
    gate, up = rnd(acc[:, 0::2]), rnd(acc[:, 1::2])
    torch.testing.assert_close(got, rnd(rnd(torch.nn.functional.silu(gate)) * up), **tol)
    got = ops.gemm(x.to(dev), w.to(dev), out_dtype=torch.float32, algo=algo).cpu()
    torch.testing.assert_close(got, acc, rtol=1e-4, atol=1e-4 * (k ** 0.5))


@pytest.mark.parametrize("algo,dt", [(L.GEMM_SIMT, torch.float32), (L.GEMM_TCGEN05, torch.bfloat16)])
def test_gemm_rows_are_batch_invariant(cuda_device, algo, dt):
    """Row r of x @ w^T is bit-identical for m = 1, 5, 64, 320, 600 (with split-K shapes too)."""
    g = torch.Generator().manual_seed(12)
    for n, k in ((2560, 2048), (896, 4864), (1024, 256), (19200, 256)):
        x = torch.randn(600, k, generator=g).to(dt).to(cuda_device)
        w = (torch.randn(n, k, generator=g) * 0.05).to(dt).to(cuda_device)
        full = ops.gemm(x, w, out_dtype=torch.float32, algo=algo)
        for m in (1, 5, 64, 320):
            part = ops.gemm(x[:m].contiguous(), w, out_dtype=torch.float32, algo=algo)
            assert torch.equal(part, full[:m]), (n, k, m)
        shifted = ops.gemm(x[3:8].contiguous(), w, out_dtype=torch.float32, algo=algo)
        assert torch.equal(shifted, full[3:8])


@pytest.mark.gpu
def test_gemm_launch_shapes_give_identical_bits(cuda_device):
    """Token tiles, weight halves per CTA, k-chunks per pipeline stage, CTA
    pairs (2-CTA MMA) and 64-row MMA tiles change speed only: every forced shape
    reproduces the model-chosen result exactly (cases 8-10 run persistent CTAs,
    with one or two TMEM accumulators; the last two are the draft's decode
    projections, which pick 64-row tiles)."""
    lib = L.load()
    g = torch.Generator(device=cuda_device).manual_seed(11)
    cases = [(320, 2560, 2048, L.EPI_BIAS), (64, 9728, 896, L.EPI_SILU_MUL), (320, 4096, 2048, L.EPI_SILU_MUL),
             (300, 1000, 136, L.EPI_STORE), (64, 896, 4864, L.EPI_RESIDUAL), (17, 512, 256, L.EPI_STORE),
             (160, 1024, 512, L.EPI_RESIDUAL), (330, 40000, 128, L.EPI_STORE), (64, 19200, 256, L.EPI_RESIDUAL),
             (300, 20000, 192, L.EPI_SILU_MUL), (64, 1152, 896, L.EPI_BIAS), (64, 896, 896, L.EPI_RESIDUAL)]
    shapes = [(1, 1, 1), (1, 2, 1), (2, 2, 2), (4, 1, 4), (3, 2, 4), (7, 1, 2), (2, 1, 2)]
    try:
        for m, n, k, epi in cases:
            x = torch.randn(m, k, device=cuda_device, generator=g).to(torch.bfloat16)
            w = (torch.randn(n, k, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
            n_out = n // 2 if epi == L.EPI_SILU_MUL else n
            bias = torch.randn(n, device=cuda_device, generator=g) if epi == L.EPI_BIAS else None
            res0 = torch.randn(m, n_out, device=cuda_device, generator=g).to(torch.bfloat16)

            def run():
                out = res0.clone() if epi == L.EPI_RESIDUAL else None
                return ops.gemm(x, w, epilogue=epi, bias=bias, residual=out, out=out)

            L.check(lib.kve_gemm_force_shape(0, 0, 0))
            L.check(lib.kve_gemm_force_pair(0))
            ref = run()
            for pair in (1, 2):  # one-CTA tiles only / CTA pairs wherever valid
                L.check(lib.kve_gemm_force_pair(pair))
                for t, mh, kc in [(0, 0, 0)] + shapes:
                    L.check(lib.kve_gemm_force_shape(t, mh, kc))
                    got = run()
                    assert torch.equal(got, ref), (m, n, k, epi, pair, t, mh, kc)
                L.check(lib.kve_gemm_force_shape(0, 0, 0))
            L.check(lib.kve_gemm_force_pair(0))
            for rows in (128, 64):  # 128-row MMA tiles only / 64-row tiles wherever valid
                L.check(lib.kve_gemm_force_rows(rows))
                for t, mh, kc in [(0, 0, 0), (1, 0, 0), (4, 0, 4), (2, 0, 2)]:
                    L.check(lib.kve_gemm_force_shape(t, mh, kc))
                    got = run()
                    assert torch.equal(got, ref), (m, n, k, epi, rows, t, kc)
                L.check(lib.kve_gemm_force_shape(0, 0, 0))
            L.check(lib.kve_gemm_force_rows(0))
    finally:
        L.check(lib.kve_gemm_force_shape(0, 0, 0))
        L.check(lib.kve_gemm_force_pair(0))
        L.check(lib.kve_gemm_force_rows(0))


def test_gemm_split_k_inside_one_cta_gives_identical_bits(cuda_device):
    """Split-K computed inside one CTA or one CTA pair (one TMEM accumulator per
    k-range, summed in the epilogue; the default for prompt-sized batches)
    reproduces the cluster reduction bit for bit, for every epilogue and both
    output types, and a prompt-sized batch's rows equal the same rows computed in a
    decode-sized batch (which splits over a cluster)."""
    lib = L.load()
    g = torch.Generator(device=cuda_device).manual_seed(21)
    # (m, n, k, epilogue, forced split factor or 0 for the (n, k) rule)
    cases = [(64, 896, 4864, L.EPI_RESIDUAL, 0), (300, 2048, 11008, L.EPI_RESIDUAL, 0),
             (2100, 896, 4864, L.EPI_RESIDUAL, 0), (2100, 2048, 11008, L.EPI_STORE, 0),
             (17, 1000, 2048, L.EPI_BIAS, 3), (200, 1024, 1024, L.EPI_SILU_MUL, 4),
             (100, 512, 4096, L.EPI_STORE, 8), (130, 768, 1536, L.EPI_RESIDUAL, 5)]
    try:
        for m, n, k, epi, fs in cases:
            x = torch.randn(m, k, device=cuda_device, generator=g).to(torch.bfloat16)
            w = (torch.randn(n, k, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
            n_out = n // 2 if epi == L.EPI_SILU_MUL else n
            bias = torch.randn(n, device=cuda_device, generator=g) if epi == L.EPI_BIAS else None
            res0 = torch.randn(m, n_out, device=cuda_device, generator=g).to(torch.bfloat16)
            L.check(lib.kve_gemm_force_splits(fs))
            info = (ctypes.c_int * 13)()
            L.check(lib.kve_gemm_plan_info(m, n, k, info))
            assert info[0] > 1, (m, n, k, "expected a split-K plan")
            for out_dtype in (torch.bfloat16, torch.float32):
                if epi == L.EPI_RESIDUAL and out_dtype != torch.bfloat16:
                    continue

                def run():
                    out = res0.clone() if epi == L.EPI_RESIDUAL else None
                    return ops.gemm(x, w, epilogue=epi, bias=bias, residual=out, out=out, out_dtype=out_dtype)

                L.check(lib.kve_gemm_force_local_split(1))  # over a cluster
                ref = run()
                L.check(lib.kve_gemm_force_local_split(2))  # inside one CTA / one CTA pair
                for pair in (1, 2):  # one-CTA tiles only / CTA pairs wherever valid
                    L.check(lib.kve_gemm_force_pair(pair))
                    got = run()
                    assert torch.equal(got, ref), (m, n, k, epi, fs, out_dtype, pair)
                L.check(lib.kve_gemm_force_local_split(0))  # the rule (inside one CTA from m = 2048)
                assert torch.equal(run(), ref), (m, n, k, epi, fs, out_dtype)
                if m >= 2048 and out_dtype == torch.bfloat16:
                    full = ops.gemm(x, w, epilogue=L.EPI_STORE, out_dtype=torch.float32)
                    for lo, hi in ((0, 64), (1000, 1320), (2093, 2100)):
                        part = ops.gemm(x[lo:hi].contiguous(), w, epilogue=L.EPI_STORE, out_dtype=torch.float32)
                        assert torch.equal(part, full[lo:hi]), (m, n, k, lo, hi)
    finally:
        L.check(lib.kve_gemm_force_local_split(0))
        L.check(lib.kve_gemm_force_splits(0))
        L.check(lib.kve_gemm_force_pair(0))


def test_bounded_wait_gives_up_and_context_survives(cuda_device):
    """The device-side timeout path. A wait that can never complete (an mbarrier that
    nothing arrives at, through the library's bounded wait with its limit cut to 50
    ms) gives up, records KVE_ERR_TIMEOUT in the status word and lets its kernel
    return; the context stays usable. GEMMs launched while the status word already
    holds KVE_ERR_TIMEOUT (one-CTA tiles, a split-K cluster, CTA pairs) skip their
    work and return at once instead of each waiting out the limit; their outputs
    are not meaningful, and the status word keeps the first error."""
    lib = L.load()
    timeout = next(c for c, name in L.KVE_ERR.items() if name == "KVE_ERR_TIMEOUT")
    stream = L.stream_handle(cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    L.check(lib.kve_selftest_mbar_timeout(status.data_ptr(), 50_000_000, stream))
    torch.cuda.synchronize()
    assert int(status.item()) == timeout
    assert time.perf_counter() - t0 < 1.5  # the 50 ms limit, not the library's 2 s

    g = torch.Generator(device=cuda_device).manual_seed(5)

    def check_gemm():
        x = torch.randn(64, 896, device=cuda_device, generator=g).to(torch.bfloat16)
        w = (torch.randn(1152, 896, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
        got = ops.gemm(x, w, out_dtype=torch.float32)
        torch.testing.assert_close(got, x.float() @ w.float().t(), rtol=1e-4, atol=1e-3)

    check_gemm()  # the context still computes correctly
    flagged = torch.full((1,), timeout, dtype=torch.int32, device=cuda_device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for m, n, k, epi in ((64, 1152, 896, L.EPI_BIAS), (64, 896, 4864, L.EPI_RESIDUAL),
                         (320, 22016, 2048, L.EPI_SILU_MUL), (2100, 2048, 11008, L.EPI_RESIDUAL)):
        x = torch.randn(m, k, device=cuda_device, generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, device=cuda_device, generator=g) * 0.05).to(torch.bfloat16)
        bias = torch.zeros(n, device=cuda_device) if epi == L.EPI_BIAS else None
        res = torch.zeros(m, n, dtype=torch.bfloat16, device=cuda_device) if epi == L.EPI_RESIDUAL else None
        ops.gemm(x, w, epilogue=epi, bias=bias, residual=res, out=res, status=flagged)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.5
    assert int(flagged.item()) == timeout
    check_gemm()


def test_gemm_repeatable_and_no_workspace(cuda_device):
    """Split-K partials are reduced in cluster shared memory: no workspace, identical repeats."""
    x = torch.randn(320, 2048, device=cuda_device).to(torch.bfloat16)
    w = torch.randn(2560, 2048, device=cuda_device).to(torch.bfloat16)
    assert L.load().kve_gemm_workspace_bytes(320, 2560, 2048, L.KVE_BF16) == 0
    a = ops.gemm(x, w)
    b = ops.gemm(x, w)
    assert torch.equal(a, b)
