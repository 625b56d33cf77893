"""Block allocator: the reference's allocator tests (kvengine tests/test_blocks.py)
restated against kvengine_b200.BlockManager, plus the reference's own churn
allocation sequence (golden `blocks.json`, seed 1234) reproduced id for id."""

import random

import pytest

from conftest import load_golden
from kvengine_b200 import BlockManager, DoubleFree, OutOfBlocks


def test_starts_fully_free():
    m = BlockManager(num_blocks=8, block_size=16)
    assert m.num_free == 8 and m.num_allocated == 0 and m.total_slots == 128
    m.check_invariants()


def test_allocate_and_free_roundtrip():
    m = BlockManager(4, 16)
    blocks = m.allocate(3, owner="a")
    assert len(set(blocks)) == 3 and m.num_free == 1
    m.free(blocks)
    assert m.num_free == 4 and m.num_allocated == 0
    m.check_invariants()


def test_first_allocation_is_block_zero_and_ascending():
    m = BlockManager(8, 4)
    assert m.allocate(3) == [0, 1, 2]


def test_blocks_needed_rounds_up():
    m = BlockManager(100, 16)
    assert [m.blocks_needed(n) for n in (0, 1, 16, 17, 32)] == [0, 1, 1, 2, 2]


def test_a_block_is_never_owned_twice():
    m = BlockManager(16, 8)
    a, b = m.allocate(6, owner="a"), m.allocate(6, owner="b")
    assert not set(a) & set(b)
    assert all(m.owner_of(x) == "a" for x in a) and all(m.owner_of(x) == "b" for x in b)


def test_oom_raises_and_changes_nothing():
    m = BlockManager(4, 16)
    held = m.allocate(3, owner="a")
    with pytest.raises(OutOfBlocks) as exc:
        m.allocate(2, owner="b")
    assert exc.value.requested == 2 and exc.value.available == 1
    assert m.num_free == 1 and m.num_allocated == len(held)
    assert len(m.allocate(1, owner="c")) == 1
    m.check_invariants()


def test_zero_block_allocation_is_a_noop():
    m = BlockManager(4, 16)
    assert m.allocate(0) == [] and m.num_free == 4


def test_double_free_is_rejected_and_atomic():
    m = BlockManager(8, 16)
    good = m.allocate(3)
    with pytest.raises(DoubleFree):
        m.free(good + [7])
    assert m.num_allocated == 3
    m.free(good)
    with pytest.raises(DoubleFree):
        m.free(good)
    one = m.allocate(1)
    with pytest.raises(DoubleFree):
        m.free(one + one)  # the same id twice in one call frees nothing
    assert m.num_allocated == 1
    m.check_invariants()


def test_lifo_reuse_returns_the_hottest_block():
    m = BlockManager(8, 16)
    first = m.allocate(1)
    m.free(first)
    assert m.allocate(1) == first


def test_free_appends_in_argument_order():
    m = BlockManager(8, 16)
    held = m.allocate(4)          # [0, 1, 2, 3]
    m.free(held[1:])              # free list tail: ..., 1, 2, 3
    assert m.allocate(3) == [3, 2, 1]


def test_reset_and_free_owner():
    m = BlockManager(16, 8)
    m.allocate(4, owner="a")
    b = m.allocate(4, owner="b")
    assert len(m.free_owner("a")) == 4 and m.num_allocated == 4
    assert all(m.owner_of(x) == "b" for x in b)
    m.reset()
    assert m.num_free == 16
    m.check_invariants()


def test_rejects_nonsense_construction():
    with pytest.raises(ValueError):
        BlockManager(0, 16)
    with pytest.raises(ValueError):
        BlockManager(16, 0)


def test_churn_matches_reference_allocation_sequence():
    """Replays the reference churn test's RNG and compares every block id handed out."""
    g = load_golden("blocks")
    rng = random.Random(1234)
    m = BlockManager(num_blocks=64, block_size=8)
    live, next_id, ops = {}, 0, []
    for _ in range(4000):
        if live and rng.random() < 0.45:
            owner = rng.choice(list(live))
            m.free(live.pop(owner))
            ops.append(["free", owner])
        else:
            owner = f"r{next_id}"
            next_id += 1
            want = rng.randint(1, 12)
            try:
                live[owner] = m.allocate(want, owner=owner)
                ops.append(["alloc", owner, want, live[owner]])
            except OutOfBlocks as e:
                ops.append(["oom", owner, want, e.available])
        m.check_invariants()
    assert ops == g["ops"]
    assert m.free_list == g["final_free"]


def test_prefix_registry_and_shared_truncate_guard():
    """Registered blocks become reclaimable, are found again, and shared ones block rollback
    (kvengine tests/test_phase6.py:366-390)."""
    import torch

    from kvengine_b200.paged import PagedKVCache

    pool = PagedKVCache(1, 1, 8, 16, 4, torch.float32, "cpu")
    a = pool.new_sequence("a")
    toks = list(range(12))
    a.reserve(12)
    a.commit(12)
    assert a.register_prefix_blocks(toks) == 3
    b = pool.new_sequence("b")
    assert b.adopt_prefix(toks + [99]) == 12
    assert b.blocks == a.blocks
    with pytest.raises(ValueError, match="shared"):
        a.truncate(5)
    b.free()
    a.free()
    assert pool.manager.num_reclaimable == 3
    pool.manager.check_invariants()


def test_commit_and_keep_matches_commit_then_truncate():
    """`commit_and_keep` (the spec loop's per-iteration commit + rollback, with a fast path
    when no published block is rolled back) leaves the same table, free list, length and
    prefix chain as `commit` followed by `truncate` (kvengine paged.py:344-380), including
    rollbacks into published blocks."""
    import random

    import torch

    from kvengine_b200.paged import PagedKVCache

    rng = random.Random(7)
    for bs in (1, 3, 4, 16):
        pools = [PagedKVCache(1, 1, 8, 96, bs, torch.float32, "cpu") for _ in range(2)]
        seqs = [[p.new_sequence(i) for i in range(4)] for p in pools]
        toks = [[rng.randrange(50) for _ in range(400)] for _ in range(4)]
        for _ in range(300):
            i = rng.randrange(4)
            fast, slow = seqs[0][i], seqs[1][i]
            op = rng.random()
            if op < 0.1:
                fast.free()
                slow.free()
                continue
            n = rng.randint(1, 6)
            try:
                fast.reserve(n)
            except Exception as e:       # out of blocks: both must refuse
                with pytest.raises(type(e)):
                    slow.reserve(n)
                continue
            slow.reserve(n)
            keep = rng.randint(max(0, fast.length - 2), fast.length + n)
            errs = []
            for s, f in ((fast, lambda s: s.commit_and_keep(n, keep)),
                         (slow, lambda s: (s.commit(n), s.truncate(keep) if keep < s.length else None))):
                try:
                    f(s)
                    errs.append(None)
                except ValueError as e:
                    errs.append(str(e))
            assert errs[0] == errs[1]
            if op < 0.5 and errs[0] is None:
                for s in (fast, slow):
                    s.register_prefix_blocks(toks[i][: s.length])
            if errs[0] is not None:      # a refused rollback leaves the committed length
                for s in (fast, slow):
                    s.free()
            for s in (fast, slow):
                s.pool.manager.check_invariants()
            assert (fast.blocks, fast.length, fast._digest_chain, fast._registered) == \
                (slow.blocks, slow.length, slow._digest_chain, slow._registered)
            assert pools[0].manager.free_list == pools[1].manager.free_list
            assert pools[0].manager.reclaimable_order() == pools[1].manager.reclaimable_order()
