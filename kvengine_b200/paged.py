"""Paged KV pool on the GPU and the per-sequence block table.

Mirrors kvengine/paged.py (`PagedKVCache` :38-119, `PagedSequenceCache`
:122-404) with the same layout, names and error behaviour:

  pool tensors k, v: [num_layers, num_blocks, block_size, num_kv_heads, head_dim]
  flat slot of logical position p: block_table[p // bs] * bs + p % bs

What changes is where the work runs: `write` appends through the
`kve_kv_append` kernel, and the forward pass never gathers the history —
attention reads blocks in place (`kve_paged_verify_attn`). `write` still
returns the gathered history for callers of the KVCacheLike protocol.
`truncate` is pure block-table bookkeeping, exactly like the reference: no
data moves, whole trailing blocks go back to the allocator.
"""

from __future__ import annotations

import torch

from .blocks import ROOT_DIGEST, BlockManager, OutOfBlocks, chain_digest

DEFAULT_BLOCK_SIZE = 16


class PagedKVCache:
    """The shared pool: device K/V tensors plus the allocator that owns the blocks."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, num_blocks: int,
                 block_size: int, dtype: torch.dtype, device: torch.device | str):
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.dtype = dtype
        self.device = torch.device(device)
        shape = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v = torch.zeros(shape, dtype=dtype, device=self.device)
        flat = (num_layers, num_blocks * block_size, num_kv_heads, head_dim)
        self.k_flat = self.k.view(flat)
        self.v_flat = self.v.view(flat)
        self.manager = BlockManager(num_blocks, block_size)

    @classmethod
    def for_model(cls, model, num_blocks: int, block_size: int = DEFAULT_BLOCK_SIZE) -> "PagedKVCache":
        """`model` is a kvengine_b200 `Model` (or anything `as_model` accepts)."""
        from .model import as_model

        m = as_model(model)
        c = m.cfg
        return cls(c.num_layers, c.num_kv_heads, c.head_dim, num_blocks, block_size, m.dtype, m.device)

    def nbytes(self) -> int:
        return self.k.numel() * self.k.element_size() * 2

    def bytes_per_block(self) -> int:
        return self.nbytes() // self.num_blocks

    @property
    def total_slots(self) -> int:
        return self.num_blocks * self.block_size

    def new_sequence(self, request_id: object) -> "PagedSequenceCache":
        return PagedSequenceCache(self, request_id)

    def stats(self) -> dict:
        return {
            "num_blocks": self.num_blocks,
            "block_size": self.block_size,
            "blocks_allocated": self.manager.num_allocated,
            "blocks_free": self.manager.num_free,
            "pool_utilization": self.manager.pool_utilization(),
            "mib": self.nbytes() / 2**20,
        }

    def __repr__(self) -> str:
        return (f"PagedKVCache(blocks={self.num_blocks}x{self.block_size}, "
                f"free={self.manager.num_free}, {self.nbytes() / 2**20:.1f} MiB)")


class PagedSequenceCache:
    """One request's block table and length (the KVCacheLike protocol of
    kvengine/forward.py:30-46 plus `truncate`)."""

    def __init__(self, pool: PagedKVCache, request_id: object):
        self.pool = pool
        self.request_id = request_id
        self.blocks: list[int] = []
        self._length = 0
        self._pending_n = 0
        self._pending_start: int | None = None  # first position of the reserved, uncommitted tokens
        self._digest_chain: list[bytes] = []
        self._registered = 0
        self.tokens_reused = 0

    # ------------------------------------------------------------ state
    @property
    def length(self) -> int:
        return self._length

    @property
    def block_size(self) -> int:
        return self.pool.block_size

    @property
    def capacity(self) -> int:
        return len(self.blocks) * self.block_size

    def free_slots(self) -> int:
        return self.capacity - self._length

    def utilization(self) -> float:
        return self._length / self.capacity if self.blocks else 0.0

    def nbytes(self) -> int:
        return len(self.blocks) * self.pool.bytes_per_block()

    # ------------------------------------------------------- allocation
    def reserve(self, n_tokens: int) -> None:
        """Grow the table to cover length + n_tokens (atomic: OutOfBlocks leaves it untouched)."""
        extra = -(-(self._length + n_tokens) // self.pool.block_size) - len(self.blocks)
        if extra > 0:
            self.blocks.extend(self.pool.manager.allocate(extra, owner=self.request_id))
        self._pending_start = self._length  # slots are listed only if write() needs them
        self._pending_n = n_tokens

    def slot_list(self, start: int, n_tokens: int) -> list[int]:
        bs = self.block_size
        blocks = self.blocks
        return [blocks[p // bs] * bs + p % bs for p in range(start, start + n_tokens)]

    def slot_indices(self, start: int, n_tokens: int) -> torch.Tensor:
        """Flat slot index per logical position in [start, start+n) (paged.py:197-205)."""
        return torch.tensor(self.slot_list(start, n_tokens), dtype=torch.long, device=self.pool.device)

    def block_table_tensor(self, width: int | None = None) -> torch.Tensor:
        width = len(self.blocks) if width is None else width
        t = torch.zeros(max(width, 1), dtype=torch.int32)
        t[: len(self.blocks)] = torch.tensor(self.blocks, dtype=torch.int32)
        return t.to(self.pool.device)

    # ------------------------------------------------------ write/gather
    def write(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor, start: int):
        """Append this layer's K/V ([1, nkv, T, hd]) and return the history [1, nkv, start+T, hd]."""
        from . import ops

        assert k.shape == v.shape, f"k/v shape mismatch: {k.shape} vs {v.shape}"
        assert k.shape[0] == 1, "one request per sequence cache"
        n = k.shape[2]
        assert start == self._length, f"write at {start} but sequence length is {self._length}"
        assert self._pending_start == start and self._pending_n == n, (
            "reserve() must be called with this pass's token count before write()")
        slots = torch.tensor(self.slot_list(start, n), dtype=torch.long, device=self.pool.device)
        k_src = k[0].transpose(0, 1).contiguous()
        v_src = v[0].transpose(0, 1).contiguous()
        ops.kv_append(k_src, v_src, slots, self.pool.k[layer_idx], self.pool.v[layer_idx])
        return self._gather(layer_idx, start + n)

    def _gather(self, layer_idx: int, end: int):
        from . import ops

        table = self.block_table_tensor()
        k_all = ops.gather_kv(self.pool.k[layer_idx], table, end)[None]
        v_all = ops.gather_kv(self.pool.v[layer_idx], table, end)[None]
        return k_all, v_all

    def commit(self, n_tokens: int) -> None:
        if self._length + n_tokens > self.capacity:
            raise OutOfBlocks(self.pool.manager.blocks_needed(self._length + n_tokens) - len(self.blocks),
                              self.pool.manager.num_free)
        self._length += n_tokens
        self._pending_start = None
        self._pending_n = 0

    def commit_and_keep(self, n_tokens: int, keep: int) -> None:
        """commit(n_tokens) followed by truncate(min(length, keep)) - the per-iteration
        bookkeeping of the spec loop in one call."""
        new_len = self._length + n_tokens
        bs = self.pool.block_size
        blocks = self.blocks
        if new_len > len(blocks) * bs:
            raise OutOfBlocks(self.pool.manager.blocks_needed(new_len) - len(blocks),
                              self.pool.manager.num_free)
        self._pending_start = None
        self._pending_n = 0
        if keep >= new_len:
            self._length = new_len
        elif 0 <= keep and self._registered <= keep // bs:
            # the spec loop's rollback: no published block is touched, so this is
            # truncate(keep) without its unregister walk
            need = -(-keep // bs)
            if need < len(blocks):
                self.pool.manager.free(blocks[need:])
                del blocks[need:]
            if len(self._digest_chain) > keep // bs:
                del self._digest_chain[keep // bs:]
            self._length = keep
        else:
            self._length = new_len
            self.truncate(keep)

    def truncate(self, n_tokens: int) -> None:
        """Roll back to n_tokens, freeing whole trailing blocks; no data moves (paged.py:344-380)."""
        if not 0 <= n_tokens <= self._length:
            raise ValueError(f"cannot truncate to {n_tokens}, length is {self._length}")
        bs = self.block_size
        mgr = self.pool.manager
        first_invalid = n_tokens // bs
        for i in range(first_invalid, min(self._registered, len(self.blocks))):
            b = self.blocks[i]
            if mgr.refcount(b) > 1:
                raise ValueError(f"block {b} is shared by another sequence; cannot roll back into it")
            mgr.unregister_prefix(b)
        keep = mgr.blocks_needed(n_tokens)
        if keep < len(self.blocks):
            mgr.free(self.blocks[keep:])
            del self.blocks[keep:]
        self._registered = min(self._registered, first_invalid)
        del self._digest_chain[first_invalid:]
        self._length = n_tokens
        self._pending_start = None
        self._pending_n = 0

    # ------------------------------------------------- prefix sharing
    def adopt_prefix(self, token_ids: list[int]) -> int:
        """Reuse published blocks for the longest shared prefix (paged.py:209-249)."""
        assert self._length == 0 and not self.blocks, "adopt_prefix needs a fresh sequence"
        bs = self.block_size
        reusable = max(len(token_ids) - 1, 0)
        parent, adopted, chain = ROOT_DIGEST, [], []
        for i in range(reusable // bs):
            chunk = token_ids[i * bs:(i + 1) * bs]
            digest = chain_digest(parent, chunk)
            b = self.pool.manager.lookup_prefix(digest, chunk)
            if b is None:
                break
            adopted.append(b)
            chain.append(digest)
            parent = digest
        if adopted:
            self.pool.manager.incref(adopted)
            self.blocks.extend(adopted)
            self._digest_chain = chain
            self._registered = len(adopted)
            self._length = len(adopted) * bs
        self.tokens_reused = self._length
        return self._length

    def register_prefix_blocks(self, token_ids: list[int]) -> int:
        """Publish every full block so others can share it (paged.py:251-279)."""
        bs = self.block_size
        full = min(self._length // bs, len(token_ids) // bs, len(self.blocks))
        while len(self._digest_chain) < full:
            i = len(self._digest_chain)
            parent = self._digest_chain[-1] if self._digest_chain else ROOT_DIGEST
            self._digest_chain.append(chain_digest(parent, token_ids[i * bs:(i + 1) * bs]))
        published = 0
        for i in range(self._registered, full):
            if self.pool.manager.register_prefix(self.blocks[i], self._digest_chain[i],
                                                 token_ids[i * bs:(i + 1) * bs]):
                published += 1
        self._registered = max(self._registered, full)
        return published

    # -------------------------------------------------------- teardown
    def free(self) -> None:
        """Return every block to the pool. Idempotent."""
        if self.blocks:
            self.pool.manager.free(self.blocks)
            self.blocks = []
        self._length = 0
        self._pending_start = None
        self._pending_n = 0
        self._digest_chain = []
        self._registered = 0
        self.tokens_reused = 0

    def __repr__(self) -> str:
        return (f"PagedSequenceCache(req={self.request_id!r}, len={self._length}, "
                f"blocks={len(self.blocks)}, util={self.utilization():.1%})")
