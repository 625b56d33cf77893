"""The C-ABI library loads without a GPU and exports every function the header
declares (no compute calls here), and the host-side plan/bookkeeping logic."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT
from kvengine_b200 import _lib as L
from kvengine_b200.model import ForwardPlan, SeqSpec
from kvengine_b200.paged import PagedKVCache


def _declared():
    names = set()
    inc = os.path.join(ROOT, "include")
    for fn in os.listdir(inc):
        if fn.endswith(".h"):
            text = open(os.path.join(inc, fn)).read()
            names.update(re.findall(r"\b(kve_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = L.load()
    declared = _declared()
    assert "kve_greedy_accept" in declared and "kve_forward" in declared
    raw = ctypes.CDLL(L.lib_path())
    for name in sorted(declared):
        assert hasattr(raw, name), f"{name} declared in include/ but not exported"
    assert declared <= set(L.EXPORTED), "ctypes signatures missing for " + str(declared - set(L.EXPORTED))
    assert lib.kve_version() >= 1


def test_workspace_queries_without_gpu():
    lib = L.load()
    assert lib.kve_greedy_accept_workspace_bytes(256) == 1024
    # split-K partials live in the cluster's shared memory: no GEMM workspace
    assert lib.kve_gemm_workspace_bytes(320, 2560, 2048, L.KVE_BF16) == 0
    # contexts past one 512-key chunk split across CTAs: 64 KiB of chunk counters + fp32 partials
    # (64 rows x (hd + 2) floats per sequence, kv head, query tile and chunk); at head_dim 64 a
    # query tile holds two 16-row blocks, 4 of the 5 tokens of a 7-head group: 2 query tiles
    assert lib.kve_paged_attn_workspace_bytes(64, 5, 4096, 14, 2, 64) == 65536 + 64 * 2 * 2 * 8 * 64 * 66 * 4
    assert lib.kve_paged_attn_workspace_bytes(64, 5, 4096, 16, 2, 128) == 65536 + 64 * 2 * 1 * 8 * 64 * 130 * 4
    assert lib.kve_paged_attn_workspace_bytes(64, 5, 512, 14, 2, 64) == 0


def test_forward_plan_layout():
    bs = 4
    seqs = [SeqSpec(start=5, q_len=3, blocks=[7, 2], n_out=1), SeqSpec(start=0, q_len=2, blocks=[9], n_out=2)]
    p = ForwardPlan(seqs, bs)
    h = p.host

    def part(name):
        o, n = p.offsets[name]
        return h[o:o + n].tolist()

    assert part("positions") == [5, 6, 7, 0, 1]
    assert part("slots") == [2 * 4 + 1, 2 * 4 + 2, 2 * 4 + 3, 9 * 4 + 0, 9 * 4 + 1]
    assert part("q_offsets") == [0, 3, 5] and part("ctx_lens") == [8, 2]
    assert part("out_rows") == [2, 3, 4]
    assert part("tables") == [7, 2, 9, 0]
    assert p.n_tokens == 5 and p.n_out == 3 and p.max_q_len == 3 and p.max_ctx == 8
    with pytest.raises(ValueError):
        ForwardPlan([SeqSpec(start=8, q_len=1, blocks=[1, 2], n_out=1)], bs)


def test_sequence_cache_bookkeeping_matches_reference_rules():
    """Truncate frees whole blocks only (kvengine tests/test_phase5.py:220-237)."""
    pool = PagedKVCache(1, 1, 8, 32, 4, torch.float32, "cpu")
    seq = pool.new_sequence("t")
    seq.reserve(16)
    seq.commit(16)
    assert len(seq.blocks) == 4
    seq.truncate(9)
    assert seq.length == 9 and len(seq.blocks) == 3 and pool.manager.num_free == 29
    seq.truncate(8)
    assert len(seq.blocks) == 2
    with pytest.raises(ValueError):
        seq.truncate(9)
    with pytest.raises(ValueError):
        seq.truncate(-1)
    seq.truncate(0)
    assert seq.blocks == []
    pool.manager.check_invariants()
    assert seq.slot_list(0, 0) == []


def test_reserve_is_atomic_on_out_of_blocks():
    from kvengine_b200 import OutOfBlocks

    pool = PagedKVCache(1, 1, 8, 4, 4, torch.float32, "cpu")
    a = pool.new_sequence("a")
    a.reserve(12)
    a.commit(12)
    b = pool.new_sequence("b")
    with pytest.raises(OutOfBlocks) as e:
        b.reserve(5)
    assert (e.value.requested, e.value.available) == (2, 1)
    assert b.blocks == [] and pool.manager.num_free == 1


def test_product_path_has_no_cpu_fallback():
    """Models refuse a CPU device; ops refuse CPU tensors."""
    from kvengine_b200 import Model, ops
    from kvengine_b200.config import TINY
    from kvengine_b200.weights import init_state_dict

    with pytest.raises(ValueError):
        Model(TINY, init_state_dict(TINY, 0), torch.float32, "cpu")
    with pytest.raises(ValueError):
        ops.gemm(torch.zeros(2, 8), torch.zeros(4, 8))
    with pytest.raises(ValueError):
        ops.argmax_rows(torch.zeros(2, 8))


def test_oracle_not_imported_by_product():
    pkg = os.path.join(ROOT, "kvengine_b200")
    for dirpath, _, files in os.walk(pkg):
        for fn in files:
            if fn.endswith(".py"):
                src = open(os.path.join(dirpath, fn)).read()
                assert not re.search(r"^\s*(from|import)\s+oracle", src, re.M), fn
