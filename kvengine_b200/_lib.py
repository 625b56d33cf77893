"""ctypes binding of the sm_100a C-ABI library (`libkvengine_b200.so`, include/kvengine_b200.h).

The library is built in-tree by `kvengine_b200/build.py` (or `make -C
kvengine_b200/csrc`). There is no CPU fallback: if the library is missing, or
CUDA is unavailable, every op raises.
"""

from __future__ import annotations

import ctypes as C
import os

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libkvengine_b200.so")

KVE_OK = 0
KVE_ERR = {
    -1: "KVE_ERR_ARG", -2: "KVE_ERR_SHAPE", -3: "KVE_ERR_DTYPE", -4: "KVE_ERR_CUDA",
    -5: "KVE_ERR_TIMEOUT", -6: "KVE_ERR_WORKSPACE", -7: "KVE_ERR_BOUNDS",
}
KVE_F32, KVE_BF16 = 0, 1
EPI_STORE, EPI_BIAS, EPI_RESIDUAL, EPI_SILU_MUL = 0, 1, 2, 3
GEMM_AUTO, GEMM_SIMT, GEMM_TCGEN05 = 0, 1, 2

vp, i32, i64, f32, sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t


class KveError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{KVE_ERR.get(code, code)}: {message}")
        self.code = code


class LayerT(C.Structure):
    _fields_ = [("w_qkv", vp), ("b_qkv", vp), ("w_o", vp), ("w_gu", vp), ("w_down", vp),
                ("ln1", vp), ("ln2", vp), ("pool_k", vp), ("pool_v", vp)]


class ModelT(C.Structure):
    _fields_ = [("dtype", i32), ("num_layers", i32), ("hidden", i32), ("num_heads", i32),
                ("num_kv_heads", i32), ("head_dim", i32), ("intermediate", i32), ("vocab", i32),
                ("rms_eps", f32), ("layers", C.POINTER(LayerT)), ("embed", vp), ("lm_head", vp),
                ("final_norm", vp), ("rope_cos", vp), ("rope_sin", vp), ("rope_len", i32),
                ("num_blocks", i64), ("block_size", i32)]


class BatchT(C.Structure):
    _fields_ = [("n_tokens", i32), ("n_seqs", i32), ("max_q_len", i32), ("max_ctx", i32),
                ("ids", vp), ("positions", vp), ("slots", vp), ("q_lens", vp), ("q_offsets", vp),
                ("ctx_lens", vp), ("block_tables", vp), ("table_stride", i32), ("n_out", i32),
                ("out_rows", vp), ("logits", vp), ("logits_dtype", i32)]


class ScratchT(C.Structure):
    _fields_ = [("hidden", vp), ("normed", vp), ("qkv", vp), ("q", vp), ("attn", vp), ("act", vp),
                ("out_normed", vp), ("gemm_ws", vp), ("gemm_ws_bytes", sz), ("attn_ws", vp),
                ("attn_ws_bytes", sz), ("dev_status", vp)]


_SIGNATURES = {
    "kve_version": (i32, []),
    "kve_last_error": (C.c_char_p, []),
    "kve_launch_count": (C.c_ulonglong, []),
    "kve_greedy_accept_workspace_bytes": (sz, [i32]),
    "kve_greedy_accept": (i32, [vp, i32, i64, vp, i64, i64, i32, i32, i32, vp, vp, vp, vp, sz, vp, vp]),
    "kve_greedy_accept_noalloc_max_batch": (i32, []),
    "kve_greedy_accept_noalloc": (i32, [vp, i32, i64, vp, i64, i64, i32, i32, i32, vp, vp, vp, vp]),
    "kve_argmax_rows": (i32, [vp, i32, i32, i32, i64, vp, vp]),
    "kve_argmax_rows_scatter": (i32, [vp, i32, i32, i32, i64, vp, vp, vp, i64, vp, vp]),
    "kve_kv_append": (i32, [vp, vp, i32, vp, i32, i32, i32, vp, vp, i64, vp, vp]),
    "kve_qkv_rope_append": (i32, [vp, i32, i32, i32, i32, i32, vp, vp, vp, vp, i32, vp, vp, vp, i64, vp, vp]),
    "kve_paged_attn_workspace_bytes": (sz, [i32, i32, i32, i32, i32, i32]),
    "kve_paged_verify_attn": (i32, [vp, i32, vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32,
                                    i64, f32, vp, vp, sz, vp, vp]),
    "kve_gather_kv": (i32, [vp, i32, vp, i32, i32, i32, i32, i64, vp, vp, vp]),
    "kve_embed": (i32, [vp, i32, vp, i32, i32, i32, vp, vp, vp]),
    "kve_rmsnorm": (i32, [vp, i32, vp, i32, i32, f32, vp, vp, vp]),
    "kve_gemm_workspace_bytes": (sz, [i32, i32, i32, i32]),
    "kve_gemm": (i32, [vp, vp, i32, i32, i32, i32, i32, vp, vp, vp, i32, vp, sz, vp, vp]),
    "kve_gemm_force_shape": (i32, [i32, i32, i32]),
    "kve_gemm_force_pair": (i32, [i32]),
    "kve_gemm_force_splits": (i32, [i32]),
    "kve_gemm_force_rows": (i32, [i32]),
    "kve_gemm_force_local_split": (i32, [i32]),
    "kve_selftest_mbar_timeout": (i32, [vp, i64, vp]),
    "kve_gemm_plan_info": (i32, [i32, i32, i32, vp]),
    "kve_gemm_ex": (i32, [vp, vp, i32, i32, i32, i32, i32, vp, vp, vp, i32, vp, sz, vp, i32, vp]),
    "kve_forward_gemm_ws_bytes": (sz, [C.POINTER(ModelT), i32, i32]),
    "kve_forward_attn_ws_bytes": (sz, [C.POINTER(ModelT), i32, i32, i32]),
    "kve_forward": (i32, [C.POINTER(ModelT), C.POINTER(BatchT), C.POINTER(ScratchT), vp]),
    "kve_forward_graphed": (i32, [C.POINTER(ModelT), C.POINTER(BatchT), C.POINTER(ScratchT),
                                  C.POINTER(C.c_void_p), vp]),
    "kve_forward_graph_free": (i32, [vp]),
    "kve_forward_layers": (i32, [C.POINTER(ModelT), C.POINTER(BatchT), C.POINTER(ScratchT), i32, i32, vp]),
    "kve_forward_layers_graphed": (i32, [C.POINTER(ModelT), C.POINTER(BatchT), C.POINTER(ScratchT), i32, i32,
                                         C.POINTER(C.c_void_p), vp]),
    "kve_spec_next_draft_plan": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


def lib_path() -> str:
    return _LIB_PATH


def load() -> C.CDLL:
    """Load the library (once). Raises ImportError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise ImportError(
            f"{_LIB_PATH} is missing: build it with `python -m kvengine_b200.build` "
            "(there is no CPU fallback for the kvengine_b200 kernels)"
        )
    lib = C.CDLL(_LIB_PATH)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != KVE_OK:
        msg = load().kve_last_error().decode(errors="replace")
        raise KveError(rc, msg)


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return KVE_F32
    if dtype == torch.bfloat16:
        return KVE_BF16
    raise TypeError(f"unsupported dtype {dtype} (kvengine_b200 runs fp32 or bf16)")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("kvengine_b200 ops take CUDA tensors (no CPU fallback)")
