"""Host-side block allocator for the paged KV pool.

Observable contract shared with the reference's `BlockManager`
(kvengine/blocks.py:70-353), which block tables depend on, so the same call
sequence yields the same tables:

* the first allocation of a fresh pool gets block 0, then 1, 2, ... (blocks.py:91-93);
* released blocks are reused last-released-first, and one `free(ids)` call
  releases in argument order (blocks.py:194-213);
* `allocate(n)` changes nothing unless all n blocks can be handed out, else it
  raises `OutOfBlocks(requested, available)` (blocks.py:150-174); blocks that
  were never cached go first, then cached prefix blocks, least recently
  released or looked up first;
* a block whose reference count drops to zero while it holds a registered
  prefix stays cached (findable by `lookup_prefix`) instead of becoming free.

Design (not the reference's): every per-block fact lives in a flat list indexed
by block id - reference count, owner, allocation serial, registered digest and
tokens, and the links of an intrusive doubly linked LRU list threaded through
the cached blocks (sentinel node at index `num_blocks`). Never-cached free
blocks sit on a plain stack. Every operation is O(blocks touched); there are
no per-block dict entries to create or delete on the spec loop's per-step
allocate/free traffic.

Tensor-free: the device pool lives in `kvengine_b200.paged`.
"""

from __future__ import annotations

import hashlib
import struct
from collections.abc import Iterable, Sequence

ROOT_DIGEST = bytes(16)


def chain_digest(parent: bytes, token_ids: Sequence[int]) -> bytes:
    """Content address of a full block: blake2b-128 over the parent block's
    address followed by the block's token ids as int32 little-endian, so a
    block's address depends on every token before it (kvengine/blocks.py:42-50)."""
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
    """Reference-counted fixed-size blocks with an LRU cache of released prefix blocks."""

    def __init__(self, num_blocks: int, block_size: int):
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("num_blocks and block_size must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.prefix_hits = 0
        self.prefix_misses = 0
        self.evictions = 0
        self.reset()

    def reset(self) -> None:
        """Every block free and uncached, as after construction."""
        n = self.num_blocks
        self._stack: list[int] = list(range(n - 1, -1, -1))   # never-cached free blocks; pop() hands out
        self._refs = [0] * n                                   # > 0: referenced by that many sequences
        self._owner: list[object] = [None] * n
        self._serial = [0] * n                                 # allocation order, for free_owner
        self._next_serial = 0
        self._key: list[bytes | None] = [None] * n             # registered digest
        self._toks: list[tuple | None] = [None] * n            # its tokens
        self._where: dict[bytes, int] = {}                     # digest -> block
        self._cached = bytearray(n)                            # 1: unreferenced, kept for its prefix
        self._lru_prev = list(range(n + 1))                    # LRU links, sentinel at index n
        self._lru_next = list(range(n + 1))
        self._live = 0
        self._n_cached = 0

    # ------------------------------------------------------------- counts
    @property
    def num_free(self) -> int:
        """Blocks `allocate` can hand out: never-cached free ones plus cached ones."""
        return len(self._stack) + self._n_cached

    @property
    def num_unused(self) -> int:
        return len(self._stack)

    @property
    def num_reclaimable(self) -> int:
        return self._n_cached

    @property
    def num_allocated(self) -> int:
        return self._live

    @property
    def total_slots(self) -> int:
        return self.num_blocks * self.block_size

    def pool_utilization(self) -> float:
        return self._live / self.num_blocks

    def owner_of(self, block_id: int):
        return self._owner[block_id] if 0 <= block_id < self.num_blocks else None

    def refcount(self, block_id: int) -> int:
        return self._refs[block_id] if 0 <= block_id < self.num_blocks else 0

    def blocks_needed(self, n_tokens: int) -> int:
        return -(-n_tokens // self.block_size)

    def unused_block(self) -> int | None:
        """A never-cached free block (the last one `allocate` would hand out), without
        allocating it, or None: scratch space for device work that must touch no
        sequence's blocks (whoever allocates it later writes it after that work)."""
        return self._stack[0] if self._stack else None

    @property
    def free_list(self) -> list[int]:
        """The never-cached free blocks, next to be handed out LAST (a copy)."""
        return list(self._stack)

    def reclaimable_order(self) -> list[int]:
        """Cached blocks from the next to be evicted to the most recently used."""
        out, nxt, end = [], self._lru_next, self.num_blocks
        b = nxt[end]
        while b != end:
            out.append(b)
            b = nxt[b]
        return out

    # ----------------------------------------------------- LRU list links
    def _lru_push(self, b: int) -> None:
        end = self.num_blocks
        last = self._lru_prev[end]
        self._lru_next[last] = b
        self._lru_prev[b] = last
        self._lru_next[b] = end
        self._lru_prev[end] = b
        self._cached[b] = 1
        self._n_cached += 1

    def _lru_unlink(self, b: int) -> None:
        p, n = self._lru_prev[b], self._lru_next[b]
        self._lru_next[p] = n
        self._lru_prev[n] = p
        self._cached[b] = 0
        self._n_cached -= 1

    def _forget_prefix(self, b: int) -> None:
        key = self._key[b]
        if key is not None and self._where.get(key) == b:
            del self._where[key]
        self._key[b] = None
        self._toks[b] = None

    # --------------------------------------------------------- alloc/free
    def _check_ids(self, ids: Iterable[int]) -> None:
        for b in ids:
            if not 0 <= b < self.num_blocks:
                raise DoubleFree(f"block {b} is not referenced")

    def allocate(self, n_blocks: int, owner: object = None) -> list[int]:
        if n_blocks < 0:
            raise ValueError("n_blocks must be non-negative")
        available = len(self._stack) + self._n_cached
        if n_blocks > available:
            raise OutOfBlocks(n_blocks, available)
        from_stack = min(n_blocks, len(self._stack))
        taken = self._stack[len(self._stack) - from_stack:][::-1]
        del self._stack[len(self._stack) - from_stack:]
        end = self.num_blocks
        for _ in range(n_blocks - from_stack):
            b = self._lru_next[end]         # least recently used cached block
            self._lru_unlink(b)
            self._forget_prefix(b)
            self.evictions += 1
            taken.append(b)
        refs, own, serial = self._refs, self._owner, self._serial
        for b in taken:
            refs[b] = 1
            own[b] = owner
            serial[b] = self._next_serial
            self._next_serial += 1
        self._live += n_blocks
        return taken

    def incref(self, block_ids: Sequence[int]) -> None:
        """One more reference on each id (prefix sharing); cached blocks come back into use."""
        ids = list(block_ids)
        self._check_ids(ids)
        for b in ids:
            if self._refs[b] == 0 and not self._cached[b]:
                raise DoubleFree(f"block {b} is neither referenced nor reclaimable")
        for b in ids:
            if self._cached[b]:
                self._lru_unlink(b)
                self._refs[b] = 1
                self._live += 1
            else:
                self._refs[b] += 1

    def free(self, block_ids) -> None:
        """Drop one reference per id, in argument order; nothing changes if any id
        (counting repeats) has no reference left to drop."""
        ids = list(block_ids)
        self._check_ids(ids)
        refs = self._refs
        if len(ids) == len(set(ids)):
            for b in ids:
                if refs[b] <= 0:
                    raise DoubleFree(f"block {b} is not referenced")
        else:
            need: dict[int, int] = {}
            for b in ids:
                need[b] = need.get(b, 0) + 1
            for b, c in need.items():
                if refs[b] < c:
                    raise DoubleFree(f"block {b} is not referenced")
        for b in ids:
            refs[b] -= 1
            if refs[b]:
                continue
            self._live -= 1
            if self._key[b] is not None:
                self._lru_push(b)           # stays findable until evicted
            else:
                self._owner[b] = None
                self._stack.append(b)

    def free_owner(self, owner: object) -> list[int]:
        """Release every referenced block of `owner`, in the order they were allocated."""
        ids = [b for b in range(self.num_blocks) if self._refs[b] > 0 and self._owner[b] == owner]
        ids.sort(key=self._serial.__getitem__)
        self.free(ids)
        return ids

    # --------------------------------------------------- prefix registry
    def register_prefix(self, block_id: int, digest: bytes, token_ids: Sequence[int]) -> bool:
        """Publish a full, referenced block under its chain digest. Returns False when
        the digest already names a different block (the caller keeps its own copy)."""
        if len(token_ids) != self.block_size:
            raise ValueError(f"a shared block must be full: {len(token_ids)} of {self.block_size} tokens")
        holder = self._where.get(digest)
        if holder is not None:
            return holder == block_id
        if self.refcount(block_id) <= 0:
            raise ValueError(f"block {block_id} is not referenced and cannot be published")
        self._forget_prefix(block_id)
        self._where[digest] = block_id
        self._key[block_id] = digest
        self._toks[block_id] = tuple(token_ids)
        return True

    def lookup_prefix(self, digest: bytes, token_ids: Sequence[int]) -> int | None:
        """The published block for `digest` holding exactly `token_ids`, or None;
        a cached hit becomes the most recently used."""
        b = self._where.get(digest)
        if b is None or self._toks[b] != tuple(token_ids):
            self.prefix_misses += 1
            return None
        self.prefix_hits += 1
        if self._cached[b]:
            self._lru_unlink(b)
            self._lru_push(b)
        return b

    def unregister_prefix(self, block_id: int) -> bool:
        """Withdraw a block's published prefix; a cached block becomes plainly free."""
        if not 0 <= block_id < self.num_blocks or self._key[block_id] is None:
            return False
        self._forget_prefix(block_id)
        if self._cached[block_id]:
            self._lru_unlink(block_id)
            self._owner[block_id] = None
            self._stack.append(block_id)
        return True

    def prefix_hit_rate(self) -> float:
        total = self.prefix_hits + self.prefix_misses
        return self.prefix_hits / total if total else 0.0

    # -------------------------------------------------------- invariants
    def check_invariants(self) -> None:
        """Each block is in exactly one state (referenced, cached, stacked free), the
        counters agree with the per-block facts, and the registry maps both ways."""
        n = self.num_blocks
        on_stack = bytearray(n)
        for b in self._stack:
            if on_stack[b]:
                raise AssertionError(f"free stack holds block {b} twice")
            on_stack[b] = 1
        lru = self.reclaimable_order()
        if len(lru) != self._n_cached or sum(self._cached) != self._n_cached:
            raise AssertionError("cached-block count disagrees with the LRU list")
        live = 0
        for b in range(n):
            states = (self._refs[b] > 0) + bool(self._cached[b]) + on_stack[b]
            if states != 1:
                raise AssertionError(f"block {b}: refcount {self._refs[b]}, cached {self._cached[b]}, "
                                     f"stacked {on_stack[b]}")
            if self._refs[b] < 0:
                raise AssertionError(f"block {b} has a negative refcount")
            live += self._refs[b] > 0
            if self._cached[b] and self._key[b] is None:
                raise AssertionError(f"cached block {b} has no published prefix")
        if live != self._live:
            raise AssertionError(f"live-block count {self._live}, counted {live}")
        for key, b in self._where.items():
            if self._key[b] != key:
                raise AssertionError(f"registry maps a digest to block {b}, which holds another")

    def __repr__(self) -> str:
        return (f"<BlockManager {self.num_blocks} x {self.block_size} tokens: {self._live} live, "
                f"{self._n_cached} cached, {len(self._stack)} free>")
