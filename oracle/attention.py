"""Oracle: paged verify attention for one layer. TEST INFRASTRUCTURE ONLY.

Restates what the reference does per sequence for the config-2 workload:
scatter the history and the q_len new K/V rows into the pool through the
block table (kvengine/paged.py:288-313, index_copy_ on the flat view),
gather the whole history back in table order (paged.py:315-331), and run
`attend` with the causal mask (kvengine/forward.py:85-144: repeat_kv, SDPA,
additive finfo.min mask, scale hd^-0.5).
"""

from __future__ import annotations

import torch

from .model import attend, causal_mask


def build_pool(w, dtype=None):
    """Pool tensors [num_blocks, bs, nkv, hd] holding the workload's history + new rows."""
    dtype = dtype or w.q.dtype
    nkv, hd = w.k_new.shape[1], w.k_new.shape[2]
    shape = (w.num_blocks, w.block_size, nkv, hd)
    pool_k = torch.zeros(shape, dtype=dtype)
    pool_v = torch.zeros(shape, dtype=dtype)
    kf = pool_k.view(-1, nkv, hd)
    vf = pool_v.view(-1, nkv, hd)
    bs = w.block_size
    for b, ctx in enumerate(w.ctx_lens):
        ids = torch.tensor(w.tables[b], dtype=torch.long)
        pos = torch.arange(ctx)
        slots = ids[pos // bs] * bs + pos % bs
        rows = slice(b * w.q_len, (b + 1) * w.q_len)
        k_all = torch.cat([w.k_hist[b], w.k_new[rows]], 0).to(dtype)
        v_all = torch.cat([w.v_hist[b], w.v_new[rows]], 0).to(dtype)
        kf.index_copy_(0, slots, k_all)
        vf.index_copy_(0, slots, v_all)
    return pool_k, pool_v


def gather(pool, table, end, bs):
    nb = -(-end // bs)
    ids = torch.tensor(table[:nb], dtype=torch.long)
    nkv, hd = pool.shape[2], pool.shape[3]
    return pool[ids].reshape(nb * bs, nkv, hd)[:end].transpose(0, 1).contiguous()


def oracle_paged_attention(w, compute_dtype=None, return_gathered=False):
    """Returns (out [B*q_len, nq, hd], pool_k, pool_v[, gathered list])."""
    pool_k, pool_v = build_pool(w)
    cd = compute_dtype or w.q.dtype
    nq = w.q.shape[1]
    nkv = w.k_new.shape[1]
    outs, gathered = [], []
    for b, ctx in enumerate(w.ctx_lens):
        k_all = gather(pool_k, w.tables[b], ctx, w.block_size)
        v_all = gather(pool_v, w.tables[b], ctx, w.block_size)
        gathered.append((k_all, v_all))
        rows = slice(b * w.q_len, (b + 1) * w.q_len)
        q = w.q[rows].transpose(0, 1)[None].to(cd)
        mask = causal_mask(w.q_len, ctx, cd)
        o = attend(q, k_all[None].to(cd), v_all[None].to(cd), mask, w.scale, nq // nkv, use_sdpa=True)
        outs.append(o[0])
    out = torch.cat(outs, 0)
    if return_gathered:
        return out, pool_k, pool_v, gathered
    return out, pool_k, pool_v
