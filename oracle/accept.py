"""Oracle: greedy acceptance and the rollback of block tables. TEST INFRASTRUCTURE ONLY.

`oracle_accept` restates kvengine/speculative.py:167-182 in numpy: per
sequence, preds = argmax over each of the k+1 verify rows (first maximum
wins; NaN counts as the maximum, like torch.argmax), n = length of the
matching prefix of drafts, emitted = drafts[:n] + [preds[n]].

`oracle_accept_tables` restates the block bookkeeping of the config-3
microbenchmark through the allocator rules of kvengine/blocks.py:85-213 and
kvengine/paged.py:179-195,344-380: sequences reserve their pre-verify length
in order, then k+1 verify slots each, then truncate to pre_len + n + 1
(keep = len(tokens) - 1, speculative.py:190-197).
"""

from __future__ import annotations

import numpy as np

from .paged import OracleAllocator


def oracle_accept(logits: np.ndarray, drafts: np.ndarray):
    B, kp1, _ = logits.shape
    k = kp1 - 1
    preds = np.argmax(logits, axis=-1).astype(np.int64)
    n = np.full(B, k, dtype=np.int64)
    emitted = np.full((B, kp1), -1, dtype=np.int64)
    for b in range(B):
        for j in range(k):
            if preds[b, j] != drafts[b, j]:
                n[b] = j
                break
        nb = int(n[b])
        emitted[b, :nb] = drafts[b, :nb]
        emitted[b, nb] = preds[b, nb]
    return n, emitted, preds


def oracle_accept_tables(pre_len, k: int, n_accepted, num_blocks: int, block_size: int):
    alloc = OracleAllocator(num_blocks, block_size)
    tables = [[] for _ in pre_len]
    lens = [0] * len(pre_len)

    def reserve(b, n):
        need = alloc.blocks_needed(lens[b] + n) - len(tables[b])
        if need > 0:
            tables[b].extend(alloc.allocate(need))
        lens[b] += n

    for b, L in enumerate(pre_len):
        reserve(b, L)
    for b in range(len(pre_len)):
        reserve(b, k + 1)
    for b, L in enumerate(pre_len):
        keep_len = min(lens[b], L + n_accepted[b] + 1)
        keep = alloc.blocks_needed(keep_len)
        if keep < len(tables[b]):
            alloc.free(tables[b][keep:])
            tables[b] = tables[b][:keep]
        lens[b] = keep_len
    return tables, list(alloc.free_list), lens
