"""Torch-tensor wrappers over the C ABI, one per kernel entry point.

Each wrapper checks shapes, dtypes and devices on the host, then launches on
the current CUDA stream. Workspaces are plain zero-filled uint8 tensors the
caller keeps (the kernels leave them zeroed).
"""

from __future__ import annotations

import torch

from . import _lib as L


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def status_tensor(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def check_status(status: torch.Tensor) -> None:
    """Raise if a kernel recorded a device-side error (syncs on `status`)."""
    code = int(status.item())
    if code != 0:
        status.zero_()
        raise L.KveError(code, "device-side check failed (see the op that wrote dev_status)")


class Workspace:
    """A grow-only zero-filled device scratch buffer."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.buf = _ws(256, self.device)

    def get(self, nbytes: int) -> torch.Tensor:
        if nbytes > self.buf.numel():
            self.buf = _ws(int(nbytes * 1.25) + 4096, self.device)
        return self.buf


def greedy_accept(logits: torch.Tensor, drafts: torch.Tensor, workspace: Workspace | None = None,
                  status: torch.Tensor | None = None, out=None):
    """logits [B, k+1, V] (fp32/bf16), drafts [B, k] (any int strides) ->
    (preds [B, k+1], n_accepted [B], emitted [B, k+1]) int32. `out` may give
    the three contiguous int32 result tensors (they may be views of one buffer,
    so that a single copy reads n_accepted and emitted back)."""
    lib = L.load()
    L.require_cuda(logits, drafts)
    B, kp1, V = logits.shape
    k = kp1 - 1
    if drafts.dtype != torch.int32 or tuple(drafts.shape) != (B, k):
        raise ValueError("drafts must be int32 [B, k]")
    if logits.stride(2) != 1 or logits.stride(0) != kp1 * logits.stride(1):
        raise ValueError("logits rows must be evenly strided with unit column stride")
    dev = logits.device
    if out is None:
        preds = torch.empty(B, kp1, dtype=torch.int32, device=dev)
        n_acc = torch.empty(B, dtype=torch.int32, device=dev)
        emitted = torch.empty(B, kp1, dtype=torch.int32, device=dev)
    else:
        preds, n_acc, emitted = out
        for t, shape in ((preds, (B, kp1)), (n_acc, (B,)), (emitted, (B, kp1))):
            if t.dtype != torch.int32 or tuple(t.shape) != shape or not t.is_contiguous() or t.device != dev:
                raise ValueError("greedy_accept out tensors must be contiguous int32 on the logits' device")
    ws = (workspace or Workspace(dev)).get(lib.kve_greedy_accept_workspace_bytes(B))
    L.check(lib.kve_greedy_accept(
        logits.data_ptr(), L.dtype_code(logits.dtype), logits.stride(1), drafts.data_ptr(),
        drafts.stride(0), drafts.stride(1), B, k, V, preds.data_ptr(), n_acc.data_ptr(),
        emitted.data_ptr(), ws.data_ptr(), ws.numel(), L.ptr(status), L.stream_handle(dev)))
    return preds, n_acc, emitted


def argmax_rows(x: torch.Tensor, out: torch.Tensor | None = None, scatter_index: torch.Tensor | None = None,
                scatter_out: torch.Tensor | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    """int32 argmax of every row (first index on ties, NaN largest). With
    `scatter_index` / `scatter_out` (contiguous int32), row i's result is also
    written to scatter_out[scatter_index[i]]."""
    lib = L.load()
    L.require_cuda(x)
    rows, cols = x.shape
    if x.stride(1) != 1:
        raise ValueError("argmax_rows needs unit column stride")
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=x.device)
    if scatter_out is None:
        L.check(lib.kve_argmax_rows(x.data_ptr(), L.dtype_code(x.dtype), rows, cols, x.stride(0),
                                    out.data_ptr(), L.stream_handle(x.device)))
        return out
    for t in (scatter_index, scatter_out):
        if t.dtype != torch.int32 or not t.is_contiguous() or not t.is_cuda:
            raise ValueError("argmax_rows: scatter_index and scatter_out must be contiguous int32 CUDA tensors")
    if scatter_index.numel() != rows:
        raise ValueError("argmax_rows: one scatter index per row")
    L.check(lib.kve_argmax_rows_scatter(x.data_ptr(), L.dtype_code(x.dtype), rows, cols, x.stride(0),
                                        out.data_ptr(), scatter_index.data_ptr(), scatter_out.data_ptr(),
                                        scatter_out.numel(), L.ptr(status), L.stream_handle(x.device)))
    return out


def kv_append(k_new, v_new, slot_ids, pool_k_layer, pool_v_layer, status=None) -> None:
    """pool[slot] = new rows; pool_*_layer: [num_blocks, bs, nkv, hd] (one layer)."""
    lib = L.load()
    L.require_cuda(k_new, v_new, slot_ids, pool_k_layer, pool_v_layer)
    n, nkv, hd = k_new.shape
    num_slots = pool_k_layer.shape[0] * pool_k_layer.shape[1]
    for t in (k_new, v_new, pool_k_layer, pool_v_layer):
        if not t.is_contiguous() or t.dtype != k_new.dtype:
            raise ValueError("kv_append operands must be contiguous and share a dtype")
    if slot_ids.dtype != torch.int64:
        raise ValueError("slot_ids must be int64 (as index_copy_ takes)")
    L.check(lib.kve_kv_append(k_new.data_ptr(), v_new.data_ptr(), L.dtype_code(k_new.dtype),
                              slot_ids.data_ptr(), n, nkv, hd, pool_k_layer.data_ptr(),
                              pool_v_layer.data_ptr(), num_slots, L.ptr(status),
                              L.stream_handle(k_new.device)))


def qkv_rope_append(qkv, positions, slots, rope_cos, rope_sin, q_out, pool_k_layer, pool_v_layer,
                    num_heads, num_kv_heads, head_dim, status=None) -> None:
    lib = L.load()
    n = qkv.shape[0]
    num_slots = pool_k_layer.shape[0] * pool_k_layer.shape[1]
    L.check(lib.kve_qkv_rope_append(qkv.data_ptr(), L.dtype_code(qkv.dtype), n, num_heads, num_kv_heads,
                                    head_dim, positions.data_ptr(), slots.data_ptr(), rope_cos.data_ptr(),
                                    rope_sin.data_ptr(), rope_cos.shape[0], q_out.data_ptr(),
                                    pool_k_layer.data_ptr(), pool_v_layer.data_ptr(), num_slots,
                                    L.ptr(status), L.stream_handle(qkv.device)))


def paged_attention(q, pool_k_layer, pool_v_layer, block_tables, ctx_lens, q_lens, q_offsets,
                    max_q_len: int, max_ctx: int, scale: float, out=None, workspace: Workspace | None = None,
                    status=None) -> torch.Tensor:
    """q [sum q_lens, nq, hd]; pools [num_blocks, bs, nkv, hd]; int32 tables/lengths."""
    lib = L.load()
    L.require_cuda(q, pool_k_layer, pool_v_layer, block_tables, ctx_lens, q_lens, q_offsets)
    _, nq, hd = q.shape
    num_blocks, bs, nkv, _ = pool_k_layer.shape
    B = ctx_lens.shape[0]
    for t in (block_tables, ctx_lens, q_lens, q_offsets):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("tables and lengths must be contiguous int32")
    if out is None:
        out = torch.empty_like(q)
    need = lib.kve_paged_attn_workspace_bytes(B, max_q_len, max_ctx, nq, nkv, hd)
    ws = (workspace or Workspace(q.device)).get(need) if need else None
    L.check(lib.kve_paged_verify_attn(
        q.data_ptr(), L.dtype_code(q.dtype), pool_k_layer.data_ptr(), pool_v_layer.data_ptr(),
        block_tables.data_ptr(), block_tables.shape[1], ctx_lens.data_ptr(), q_lens.data_ptr(),
        q_offsets.data_ptr(), B, max_q_len, max_ctx, nq, nkv, hd, bs, num_blocks, scale, out.data_ptr(),
        L.ptr(ws), 0 if ws is None else ws.numel(), L.ptr(status), L.stream_handle(q.device)))
    return out


def gather_kv(pool_layer, block_table, length: int, status=None) -> torch.Tensor:
    """[nkv, length, hd] history of one sequence (pool_layer [num_blocks, bs, nkv, hd])."""
    lib = L.load()
    num_blocks, bs, nkv, hd = pool_layer.shape
    out = torch.empty(nkv, length, hd, dtype=pool_layer.dtype, device=pool_layer.device)
    L.check(lib.kve_gather_kv(pool_layer.data_ptr(), L.dtype_code(pool_layer.dtype), block_table.data_ptr(),
                              length, nkv, hd, bs, num_blocks, out.data_ptr(), L.ptr(status),
                              L.stream_handle(pool_layer.device)))
    return out


def embed(ids, table, out=None, status=None):
    lib = L.load()
    n = ids.shape[0]
    vocab, hidden = table.shape
    if out is None:
        out = torch.empty(n, hidden, dtype=table.dtype, device=table.device)
    L.check(lib.kve_embed(ids.data_ptr(), n, table.data_ptr(), L.dtype_code(table.dtype), hidden, vocab,
                          out.data_ptr(), L.ptr(status), L.stream_handle(table.device)))
    return out


def rmsnorm(x, weight, eps: float, row_index=None, out=None):
    lib = L.load()
    rows = x.shape[0] if row_index is None else row_index.shape[0]
    hidden = x.shape[1]
    if out is None:
        out = torch.empty(rows, hidden, dtype=x.dtype, device=x.device)
    L.check(lib.kve_rmsnorm(x.data_ptr(), L.dtype_code(x.dtype), weight.data_ptr(), rows, hidden, eps,
                            L.ptr(row_index), out.data_ptr(), L.stream_handle(x.device)))
    return out


def gemm(x, w, epilogue: int = L.EPI_STORE, bias=None, residual=None, out=None, out_dtype=None,
         workspace: Workspace | None = None, status=None, algo: int = L.GEMM_AUTO) -> torch.Tensor:
    lib = L.load()
    L.require_cuda(x, w)
    m, k = x.shape
    n = w.shape[0]
    if w.shape[1] != k or x.dtype != w.dtype or not x.is_contiguous() or not w.is_contiguous():
        raise ValueError("gemm: x [m,k] and w [n,k] must be contiguous and share a dtype")
    out_dtype = out_dtype or x.dtype
    n_out = n // 2 if epilogue == L.EPI_SILU_MUL else n
    if out is None:
        out = torch.empty(m, n_out, dtype=out_dtype, device=x.device)
    dc = L.dtype_code(x.dtype)
    need = lib.kve_gemm_workspace_bytes(m, n, k, dc)
    ws = (workspace or Workspace(x.device)).get(need) if need else None
    L.check(lib.kve_gemm_ex(x.data_ptr(), w.data_ptr(), dc, m, n, k, epilogue, L.ptr(bias), L.ptr(residual),
                            out.data_ptr(), L.dtype_code(out_dtype), L.ptr(ws), 0 if ws is None else ws.numel(),
                            L.ptr(status), algo, L.stream_handle(x.device)))
    return out


def spec_next_draft_plan(start_lens: torch.Tensor, last_tokens: torch.Tensor, n_blocks: torch.Tensor,
                         tables: torch.Tensor, block_size: int, k: int, rows: int, dump_block: int,
                         n_accepted: torch.Tensor, emitted: torch.Tensor, plan_out: torch.Tensor,
                         ids_out: torch.Tensor, verify_ids_out: torch.Tensor, status: torch.Tensor | None = None):
    """The next step's first draft pass planned on the device (kve_spec_next_draft_plan).
    start_lens, last_tokens, n_blocks [S], tables [S, width], n_accepted [S],
    emitted [S, k+1] (contiguous int32); writes plan_out (the packed ForwardPlan
    layout of `ForwardPlan.device_built(S, rows, width, ...)`), ids_out [rows * S]
    and verify_ids_out[s * (k+1)]."""
    lib = L.load()
    S = start_lens.numel()
    tensors = (start_lens, last_tokens, n_blocks, tables, n_accepted, emitted, plan_out, ids_out, verify_ids_out)
    L.require_cuda(*tensors)
    for t in tensors:
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("spec_next_draft_plan takes contiguous int32 tensors")
    width = tables.numel() // max(S, 1)
    if tables.numel() != S * width or n_blocks.numel() != S or n_accepted.numel() < S or \
            emitted.numel() < S * (k + 1) or ids_out.numel() < rows * S or verify_ids_out.numel() < S * (k + 1) or \
            plan_out.numel() < 2 * rows * S + 4 * S + 1 + S * width:
        raise ValueError("spec_next_draft_plan: buffer sizes do not match")
    L.check(lib.kve_spec_next_draft_plan(start_lens.data_ptr(), last_tokens.data_ptr(), n_blocks.data_ptr(),
                                         tables.data_ptr(), S, width, block_size, k, rows, dump_block,
                                         n_accepted.data_ptr(), emitted.data_ptr(), plan_out.data_ptr(),
                                         ids_out.data_ptr(), verify_ids_out.data_ptr(), L.ptr(status),
                                         L.stream_handle(start_lens.device)))
