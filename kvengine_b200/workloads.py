"""Seeded synthetic workloads for the five benchmark configurations.

There is no public dataset for this path: the reference measures on its own
prompts and random token ids (kvengine/bench.py:84-115 for the lognormal
request mix). Every generator here is deterministic in its seed and uses only
torch's CPU generator and Python's `random`, so the same inputs come out on any
machine with the same torch version.
"""

from __future__ import annotations

import math
import random
from dataclasses import dataclass

import torch

from .config import VOCAB_QWEN2


def random_prompts(n: int, length: int, seed: int, vocab: int = VOCAB_QWEN2) -> torch.Tensor:
    """[n, length] int64 uniform in [0, vocab) (config 1: n=4, length=64, seed 0)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n, length), generator=g)


def lognormal_length(rng: random.Random, mean: float, sigma: float, lo: int, hi: int) -> int:
    """exp(N(log(mean), sigma)) rounded and clamped to [lo, hi].

    Same parameterisation as the reference's `_lognormal_length`
    (kvengine/bench.py:73-81): `mean` is used as the median, mu = log(mean).
    """
    mu = math.log(max(mean, 1.0))
    return max(lo, min(hi, int(round(math.exp(rng.gauss(mu, sigma))))))


def lognormal_requests(n: int, seed: int, prompt_mean=128.0, output_mean=64.0, sigma=0.7,
                       prompt_clip=(8, 512), output_clip=(4, 256), vocab: int = VOCAB_QWEN2):
    """Config 5 request mix: lognormal prompt and output lengths, uniform tokens."""
    rng = random.Random(seed)
    g = torch.Generator().manual_seed(seed)
    reqs = []
    for _ in range(n):
        p = lognormal_length(rng, prompt_mean, sigma, *prompt_clip)
        o = lognormal_length(rng, output_mean, sigma, *output_clip)
        reqs.append((torch.randint(0, vocab, (p,), generator=g).tolist(), o))
    return reqs


@dataclass
class AttentionWorkload:
    """Config 2: paged GQA verify attention for one layer."""
    ctx_lens: list[int]
    q_len: int
    tables: list[list[int]]
    num_blocks: int
    block_size: int
    q: torch.Tensor          # [B*q_len, nq, hd]
    k_hist: list[torch.Tensor]  # per seq [ctx-q_len, nkv, hd]
    v_hist: list[torch.Tensor]
    k_new: torch.Tensor      # [B*q_len, nkv, hd]
    v_new: torch.Tensor
    scale: float

    @property
    def num_seqs(self) -> int:
        return len(self.ctx_lens)


def attention_workload(seed: int = 2, num_seqs: int = 64, q_len: int = 5, num_heads: int = 14,
                       num_kv_heads: int = 2, head_dim: int = 64, num_blocks: int = 65536,
                       block_size: int = 16, median_ctx: float = 512.0, sigma: float = 0.8,
                       ctx_clip=(16, 4096), dtype=torch.bfloat16) -> AttentionWorkload:
    """Context ~ lognormal(median, sigma) clipped; block tables sliced from a
    seeded permutation of the pool; q/k/v ~ N(0,1) in `dtype`."""
    rng = random.Random(seed)
    ctx = [max(q_len, lognormal_length(rng, median_ctx, sigma, *ctx_clip)) for _ in range(num_seqs)]
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g).tolist()
    tables, off = [], 0
    for c in ctx:
        nb = (c + block_size - 1) // block_size
        if off + nb > num_blocks:
            raise ValueError("pool too small for the sampled contexts")
        tables.append(perm[off:off + nb])
        off += nb
    q = torch.randn(num_seqs * q_len, num_heads, head_dim, generator=g).to(dtype)
    k_new = torch.randn(num_seqs * q_len, num_kv_heads, head_dim, generator=g).to(dtype)
    v_new = torch.randn(num_seqs * q_len, num_kv_heads, head_dim, generator=g).to(dtype)
    k_hist = [torch.randn(c - q_len, num_kv_heads, head_dim, generator=g).to(dtype) for c in ctx]
    v_hist = [torch.randn(c - q_len, num_kv_heads, head_dim, generator=g).to(dtype) for c in ctx]
    return AttentionWorkload(ctx, q_len, tables, num_blocks, block_size, q, k_hist, v_hist,
                             k_new, v_new, head_dim ** -0.5)


@dataclass
class AcceptWorkload:
    """Config 3: greedy acceptance over [B, k+1, V] target logits."""
    logits: torch.Tensor    # [B, k+1, V]
    drafts: torch.Tensor    # [B, k] int64
    pre_len: list[int]      # Lt per sequence: cache length before the verify
    k: int


def accept_workload(k: int, batch: int = 256, vocab: int = VOCAB_QWEN2, seed: int | None = None,
                    p_match: float = 0.75, boost: float = 10.0, dtype=torch.float32,
                    len_range=(16, 1024)) -> AcceptWorkload:
    """Logits ~ N(0,1); drafts uniform; with probability p_match (independent,
    per position j<k) the draft token's logit is raised by `boost`."""
    seed = 1000 + k if seed is None else seed
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(batch, k + 1, vocab, generator=g)
    drafts = torch.randint(0, vocab, (batch, k), generator=g)
    hit = torch.rand(batch, k, generator=g) < p_match
    b_idx, j_idx = hit.nonzero(as_tuple=True)
    logits[b_idx, j_idx, drafts[b_idx, j_idx]] += boost
    pre = torch.randint(len_range[0], len_range[1], (batch,), generator=g).tolist()
    return AcceptWorkload(logits.to(dtype), drafts, pre, k)
