"""Host-side block allocator for the paged KV pool.

Same contract as the reference's `BlockManager` (kvengine/blocks.py:70-353), so
block tables come out identical for the same sequence of calls:

* the free list starts as [N-1, ..., 1, 0] and hands out from its end, so the
  first allocation gets block 0 (blocks.py:91-93);
* `allocate(n)` is atomic: it checks capacity before taking anything and raises
  `OutOfBlocks(requested, available)` (blocks.py:150-174), spending truly free
  blocks before evicting least-recently-released cached ones;
* `free(ids)` is atomic across the batch, raises `DoubleFree` for an
  unreferenced id, and appends released blocks in argument order
  (blocks.py:194-213), which makes reuse LIFO;
* reference counts and the content-addressed prefix registry (blake2b chain,
  blocks.py:42-50, 217-310) are kept so `PagedSequenceCache.truncate` can apply
  the reference's shared-block guard.

Tensor-free: the device pool lives in `kvengine_b200.paged`.
"""

from __future__ import annotations

import hashlib
import struct
from collections import OrderedDict
from collections.abc import Sequence

ROOT_DIGEST = bytes(16)


def chain_digest(parent: bytes, token_ids: Sequence[int]) -> bytes:
    """Content address of a block: its int32 little-endian tokens chained on the parent digest."""
    h = hashlib.blake2b(parent, digest_size=16)
    h.update(struct.pack(f"<{len(token_ids)}i", *token_ids))
    return h.digest()


class OutOfBlocks(RuntimeError):
    """Not enough allocatable blocks; carries what was asked for and what was left."""

    def __init__(self, requested: int, available: int):
        super().__init__(f"requested {requested} blocks, only {available} available")
        self.requested = requested
        self.available = available


class DoubleFree(RuntimeError):
    """A block was released (or increfed) while nothing referenced it."""


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("num_blocks and block_size must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._free: list[int] = list(range(num_blocks - 1, -1, -1))
        self._refcount: dict[int, int] = {}
        self._owner: dict[int, object] = {}
        self._reclaimable: OrderedDict[int, None] = OrderedDict()
        self._by_digest: dict[bytes, int] = {}
        self._digest_of: dict[int, bytes] = {}
        self._tokens_of: dict[int, tuple[int, ...]] = {}
        self.prefix_hits = 0
        self.prefix_misses = 0
        self.evictions = 0

    # ------------------------------------------------------------- state
    @property
    def num_free(self) -> int:
        return len(self._free) + len(self._reclaimable)

    @property
    def num_unused(self) -> int:
        return len(self._free)

    @property
    def num_reclaimable(self) -> int:
        return len(self._reclaimable)

    @property
    def num_allocated(self) -> int:
        return len(self._refcount)

    @property
    def total_slots(self) -> int:
        return self.num_blocks * self.block_size

    def pool_utilization(self) -> float:
        return self.num_allocated / self.num_blocks

    def owner_of(self, block_id: int):
        return self._owner.get(block_id)

    def refcount(self, block_id: int) -> int:
        return self._refcount.get(block_id, 0)

    def blocks_needed(self, n_tokens: int) -> int:
        return -(-n_tokens // self.block_size)

    # -------------------------------------------------------- alloc/free
    def allocate(self, n_blocks: int, owner: object = None) -> list[int]:
        if n_blocks < 0:
            raise ValueError("n_blocks must be non-negative")
        available = self.num_free
        if n_blocks > available:
            raise OutOfBlocks(n_blocks, available)
        taken = []
        for _ in range(n_blocks):
            taken.append(self._free.pop() if self._free else self._evict_lru())
        for b in taken:
            self._refcount[b] = 1
            self._owner[b] = owner
        return taken

    def incref(self, block_ids: Sequence[int]) -> None:
        ids = list(block_ids)
        bad = [b for b in ids if b not in self._refcount and b not in self._reclaimable]
        if bad:
            raise DoubleFree(f"block {bad[0]} is neither referenced nor reclaimable")
        for b in ids:
            if b in self._reclaimable:
                del self._reclaimable[b]
                self._refcount[b] = 1
            else:
                self._refcount[b] += 1

    def free(self, block_ids) -> None:
        ids = list(block_ids)
        # Validate the whole batch first (counting repeats) so a bad id frees nothing.
        pending: dict[int, int] = {}
        for b in ids:
            pending[b] = pending.get(b, 0) + 1
            if self._refcount.get(b, 0) < pending[b]:
                raise DoubleFree(f"block {b} is not referenced")
        for b in ids:
            c = self._refcount[b] - 1
            if c:
                self._refcount[b] = c
                continue
            del self._refcount[b]
            if b in self._digest_of:
                self._reclaimable[b] = None
            else:
                self._owner.pop(b, None)
                self._free.append(b)

    def free_owner(self, owner: object) -> list[int]:
        ids = [b for b, o in self._owner.items() if o == owner and b in self._refcount]
        self.free(ids)
        return ids

    def reset(self) -> None:
        self._free = list(range(self.num_blocks - 1, -1, -1))
        for d in (self._refcount, self._owner, self._reclaimable, self._by_digest, self._digest_of,
                  self._tokens_of):
            d.clear()

    # -------------------------------------------------- prefix registry
    def register_prefix(self, block_id: int, digest: bytes, token_ids: Sequence[int]) -> bool:
        if len(token_ids) != self.block_size:
            raise ValueError(
                f"only full blocks are shareable: got {len(token_ids)} tokens, block_size is {self.block_size}")
        if digest in self._by_digest:
            return self._by_digest[digest] == block_id
        if self.refcount(block_id) <= 0:
            raise ValueError(f"cannot register unreferenced block {block_id}")
        self._by_digest[digest] = block_id
        self._digest_of[block_id] = digest
        self._tokens_of[block_id] = tuple(token_ids)
        return True

    def lookup_prefix(self, digest: bytes, token_ids: Sequence[int]) -> int | None:
        b = self._by_digest.get(digest)
        if b is None or self._tokens_of.get(b) != tuple(token_ids):
            self.prefix_misses += 1
            return None
        self.prefix_hits += 1
        if b in self._reclaimable:
            self._reclaimable.move_to_end(b)
        return b

    def unregister_prefix(self, block_id: int) -> bool:
        digest = self._digest_of.pop(block_id, None)
        if digest is None:
            return False
        if self._by_digest.get(digest) == block_id:
            del self._by_digest[digest]
        self._tokens_of.pop(block_id, None)
        if block_id in self._reclaimable:
            del self._reclaimable[block_id]
            self._owner.pop(block_id, None)
            self._free.append(block_id)
        return True

    def _evict_lru(self) -> int:
        b, _ = self._reclaimable.popitem(last=False)
        digest = self._digest_of.pop(b, None)
        if digest is not None:
            self._by_digest.pop(digest, None)
        self._tokens_of.pop(b, None)
        self._owner.pop(b, None)
        self.evictions += 1
        return b

    def prefix_hit_rate(self) -> float:
        total = self.prefix_hits + self.prefix_misses
        return self.prefix_hits / total if total else 0.0

    # -------------------------------------------------------- invariants
    def check_invariants(self) -> None:
        free_set = set(self._free)
        assert len(free_set) == len(self._free), "duplicate block in free list"
        reclaim = set(self._reclaimable)
        live = set(self._refcount)
        assert not free_set & live, f"blocks both free and referenced: {sorted(free_set & live)}"
        assert not free_set & reclaim, f"blocks both free and reclaimable: {sorted(free_set & reclaim)}"
        assert not reclaim & live, f"blocks both reclaimable and referenced: {sorted(reclaim & live)}"
        assert free_set | reclaim | live == set(range(self.num_blocks)), "blocks leaked"
        assert all(c > 0 for c in self._refcount.values()), "non-positive refcount"
        for digest, b in self._by_digest.items():
            assert self._digest_of.get(b) == digest, f"prefix registry disagrees for block {b}"
        for b in reclaim:
            assert b in self._digest_of, f"reclaimable block {b} holds no registered prefix"

    def __repr__(self) -> str:
        return (f"BlockManager(num_blocks={self.num_blocks}, block_size={self.block_size}, "
                f"unused={self.num_unused}, reclaimable={self.num_reclaimable}, "
                f"referenced={self.num_allocated})")
