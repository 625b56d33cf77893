"""kve_greedy_accept_noalloc: the allocation-free accept entry point.

Called through the C ABI (ctypes) and compared with kve_greedy_accept, which
takes a caller-provided workspace, on two calls in a row: the second call only
matches if the first left the built-in counters at zero. The file name sorts
last so the test also runs after every other test in the session.
"""

import ctypes

import pytest
import torch

from kvengine_b200 import _lib as L
from kvengine_b200 import workloads


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _with_workspace(lib, logits, drafts, k, dev):
    b, vocab = drafts.shape[0], logits.shape[-1]
    preds = torch.full((b, k + 1), -7, dtype=torch.int32, device=dev)
    n_acc = torch.full((b,), -7, dtype=torch.int32, device=dev)
    emitted = torch.full((b, k + 1), -7, dtype=torch.int32, device=dev)
    ws = torch.zeros(lib.kve_greedy_accept_workspace_bytes(b), dtype=torch.uint8, device=dev)
    rc = lib.kve_greedy_accept(logits.data_ptr(), L.dtype_code(logits.dtype), vocab, drafts.data_ptr(), k, 1, b, k,
                               vocab, preds.data_ptr(), n_acc.data_ptr(), emitted.data_ptr(), ws.data_ptr(),
                               ws.numel(), None, _stream(dev))
    assert rc == 0, lib.kve_last_error()
    return preds, n_acc, emitted


def _noalloc(lib, logits, drafts, k, dev):
    b, vocab = drafts.shape[0], logits.shape[-1]
    preds = torch.full((b, k + 1), -7, dtype=torch.int32, device=dev)
    n_acc = torch.full((b,), -7, dtype=torch.int32, device=dev)
    emitted = torch.full((b, k + 1), -7, dtype=torch.int32, device=dev)
    rc = lib.kve_greedy_accept_noalloc(logits.data_ptr(), L.dtype_code(logits.dtype), vocab, drafts.data_ptr(), k,
                                       1, b, k, vocab, preds.data_ptr(), n_acc.data_ptr(), emitted.data_ptr(),
                                       _stream(dev))
    assert rc == 0, lib.kve_last_error()
    return preds, n_acc, emitted


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_accept_matches_workspace_accept_twice(cuda_device, dtype):
    lib = L.load()
    dev = cuda_device
    for k, batch in ((4, 256), (8, 64), (1, 300)):
        w = workloads.accept_workload(k, batch=batch, vocab=32000, dtype=dtype)
        logits = w.logits.to(dev)
        drafts = w.drafts.to(torch.int32).to(dev).contiguous()
        want = _with_workspace(lib, logits, drafts, k, dev)
        first = _noalloc(lib, logits, drafts, k, dev)
        second = _noalloc(lib, logits, drafts, k, dev)
        torch.cuda.synchronize(dev)
        for got in (first, second):
            for a, b in zip(got, want):
                assert torch.equal(a, b)


@pytest.mark.gpu
def test_noalloc_accept_full_size_batch(cuda_device):
    """The largest batch the built-in counters allow, on tiny rows, twice."""
    lib = L.load()
    dev = cuda_device
    k, batch = 3, lib.kve_greedy_accept_noalloc_max_batch()
    w = workloads.accept_workload(k, batch=batch, vocab=64)
    logits = w.logits.to(dev)
    drafts = w.drafts.to(torch.int32).to(dev).contiguous()
    want = _with_workspace(lib, logits, drafts, k, dev)
    for _ in range(2):
        got = _noalloc(lib, logits, drafts, k, dev)
        torch.cuda.synchronize(dev)
        for a, b in zip(got, want):
            assert torch.equal(a, b)


def test_noalloc_accept_rejects_batches_over_the_maximum():
    """Rejected on the host, before any device work."""
    lib = L.load()
    cap = lib.kve_greedy_accept_noalloc_max_batch()
    assert cap == 4096
    fake = ctypes.c_void_p(16)
    rc = lib.kve_greedy_accept_noalloc(fake, L.KVE_F32, 100, fake, 4, 1, cap + 1, 4, 100, fake, fake, fake, None)
    assert L.KVE_ERR.get(rc) == "KVE_ERR_ARG"
    assert b"exceeds the built-in maximum" in lib.kve_last_error()
