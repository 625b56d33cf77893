"""Oracle: block allocator and paged KV cache. TEST INFRASTRUCTURE ONLY.

Restates, for checking:
  * the allocator's free-list discipline, kvengine/blocks.py:85-106 (free list
    initialised `reversed(range(N))` so the first pop hands out block 0),
    `blocks_needed` :144-146, atomic `allocate` :150-174 (pop from the end),
    atomic `free` :194-213 (append in argument order);
  * the paged sequence cache, kvengine/paged.py: pool layout
    `[L, N, bs, n_kv, hd]` with flat `[L, N*bs, n_kv, hd]` views :59-67,
    `reserve` :179-195, `slot_indices` :197-205, `write` :288-313
    (index_copy_ into the flat view, then `_gather`), `_gather` :315-331
    (whole blocks in table order, trimmed), `commit` :333-342, `truncate`
    :344-380 (free blocks[keep:] in table order, no data movement), `free`
    :384-398.
Prefix sharing (registry, refcounts > 1) is out of this path and not restated.
"""

from __future__ import annotations

import torch


class OracleOutOfBlocks(RuntimeError):
    def __init__(self, requested: int, available: int):
        super().__init__(f"requested {requested} blocks, only {available} available")
        self.requested = requested
        self.available = available


class OracleAllocator:
    def __init__(self, num_blocks: int, block_size: int):
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("num_blocks and block_size must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.free_list = list(reversed(range(num_blocks)))
        self.live: set[int] = set()

    @property
    def num_free(self) -> int:
        return len(self.free_list)

    def blocks_needed(self, n_tokens: int) -> int:
        return (n_tokens + self.block_size - 1) // self.block_size

    def allocate(self, n: int) -> list[int]:
        if n < 0:
            raise ValueError("n_blocks must be non-negative")
        if n > len(self.free_list):
            raise OracleOutOfBlocks(n, len(self.free_list))
        taken = [self.free_list.pop() for _ in range(n)]
        self.live.update(taken)
        return taken

    def free(self, ids) -> None:
        ids = list(ids)
        for b in ids:
            if b not in self.live:
                raise RuntimeError(f"block {b} is not referenced")
        for b in ids:
            self.live.discard(b)
            self.free_list.append(b)


class OraclePool:
    def __init__(self, num_layers, num_kv_heads, head_dim, num_blocks, block_size, dtype):
        shape = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        self.k = torch.zeros(shape, dtype=dtype)
        self.v = torch.zeros(shape, dtype=dtype)
        flat = (num_layers, num_blocks * block_size, num_kv_heads, head_dim)
        self.k_flat = self.k.view(flat)
        self.v_flat = self.v.view(flat)
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.alloc = OracleAllocator(num_blocks, block_size)

    def new_sequence(self) -> "OracleSeq":
        return OracleSeq(self)


class OracleSeq:
    def __init__(self, pool: OraclePool):
        self.pool = pool
        self.blocks: list[int] = []
        self.length = 0
        self._pending: torch.Tensor | None = None
        self._pending_n = 0

    def reserve(self, n_tokens: int) -> None:
        need = self.pool.alloc.blocks_needed(self.length + n_tokens)
        extra = need - len(self.blocks)
        if extra > 0:
            self.blocks.extend(self.pool.alloc.allocate(extra))
        self._pending = self.slot_indices(self.length, n_tokens)
        self._pending_n = n_tokens

    def slot_indices(self, start: int, n_tokens: int) -> torch.Tensor:
        bs = self.pool.block_size
        ids = torch.tensor(self.blocks, dtype=torch.long)
        pos = torch.arange(start, start + n_tokens)
        return ids[pos // bs] * bs + (pos % bs)

    def write(self, layer: int, k: torch.Tensor, v: torch.Tensor, start: int):
        """k, v: [n_kv, T, hd]. Returns the gathered history [n_kv, start+T, hd]."""
        n = k.shape[1]
        assert start == self.length and self._pending_n == n
        self.pool.k_flat[layer].index_copy_(0, self._pending, k.transpose(0, 1).contiguous())
        self.pool.v_flat[layer].index_copy_(0, self._pending, v.transpose(0, 1).contiguous())
        return self.gather(layer, start + n)

    def gather(self, layer: int, end: int):
        bs = self.pool.block_size
        nb = self.pool.alloc.blocks_needed(end)
        ids = torch.tensor(self.blocks[:nb], dtype=torch.long)
        shape = (nb * bs, self.pool.num_kv_heads, self.pool.head_dim)
        k_all = self.pool.k[layer][ids].reshape(shape)[:end].transpose(0, 1)
        v_all = self.pool.v[layer][ids].reshape(shape)[:end].transpose(0, 1)
        return k_all.contiguous(), v_all.contiguous()

    def commit(self, n_tokens: int) -> None:
        self.length += n_tokens
        self._pending = None
        self._pending_n = 0

    def truncate(self, n_tokens: int) -> None:
        if not 0 <= n_tokens <= self.length:
            raise ValueError(f"cannot truncate to {n_tokens}, length is {self.length}")
        keep = self.pool.alloc.blocks_needed(n_tokens)
        if keep < len(self.blocks):
            self.pool.alloc.free(self.blocks[keep:])
            self.blocks = self.blocks[:keep]
        self.length = n_tokens
        self._pending = None
        self._pending_n = 0

    def free(self) -> None:
        if self.blocks:
            self.pool.alloc.free(self.blocks)
            self.blocks = []
        self.length = 0
