"""Models on the device and the per-(model, pool) forward runner.

`Model` owns device weights in the layout `weights.DeviceWeights` describes;
it can be built from a HuggingFace Qwen2 model (the reference's model type,
kvengine/loader.py:35-52) or from a seeded random init. `Runner` binds a model
to a `PagedKVCache` and executes `kve_forward` (one C call per model pass) on
a `ForwardPlan`: the ragged batch description the forward kernels read.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from itertools import chain
from types import SimpleNamespace

import numpy as np
import torch

from . import _lib as L
from .config import ModelConfig
from .weights import DeviceWeights, init_state_dict, state_dict_from_hf


class Model:
    def __init__(self, cfg: ModelConfig, state_dict: dict, dtype: torch.dtype = torch.bfloat16,
                 device: str | torch.device = "cuda", eos_token_id=None, roll_lm_head: int = 0):
        L.dtype_code(dtype)
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("kvengine_b200 models live on a CUDA device (no CPU fallback)")
        self.weights = DeviceWeights(cfg, state_dict, dtype, self.device, roll_lm_head=roll_lm_head)
        self.generation_config = SimpleNamespace(eos_token_id=eos_token_id)
        self.config = cfg

    @classmethod
    def from_hf(cls, hf_model, dtype: torch.dtype | None = None, device="cuda", roll_lm_head: int = 0):
        cfg = ModelConfig.from_hf(hf_model.config)
        dtype = dtype or next(hf_model.parameters()).dtype
        eos = getattr(getattr(hf_model, "generation_config", None), "eos_token_id", None)
        return cls(cfg, state_dict_from_hf(hf_model), dtype, device, eos, roll_lm_head)

    @classmethod
    def random_init(cls, cfg: ModelConfig, seed: int, dtype=torch.bfloat16, device="cuda",
                    init_device: str = "cpu", eos_token_id=None, roll_lm_head: int = 0, **init_kw):
        """Seeded N(0, 0.02) init. `init_device="cpu"` reproduces the CPU
        oracle's weights exactly; "cuda" is much faster for large models."""
        sd = init_state_dict(cfg, seed, dtype=dtype, device=init_device, **init_kw)
        return cls(cfg, sd, dtype, device, eos_token_id, roll_lm_head)

    def parameters(self):
        yield self.weights.embed


def as_model(m) -> Model:
    """Accept a kvengine_b200 Model or a HuggingFace model (converted once and cached on it)."""
    if isinstance(m, Model):
        return m
    cached = getattr(m, "_kvengine_b200_model", None)
    if cached is not None:
        return cached
    if hasattr(m, "model") and hasattr(m, "lm_head"):
        dev = "cuda"
        roll = 1 if type(m).__name__ == "HostileDraft" else 0
        base = m if roll == 0 else SimpleNamespace(model=m.model, lm_head=m._head, config=m.config,
                                                   generation_config=m.generation_config,
                                                   parameters=lambda: iter([m._head.weight]))
        conv = Model.from_hf(base, device=dev, roll_lm_head=roll)
        try:
            m._kvengine_b200_model = conv
        except AttributeError:
            pass
        return conv
    raise TypeError(f"cannot use {type(m).__name__} as a kvengine_b200 model")


# ---------------------------------------------------------------- plans
@dataclass
class SeqSpec:
    """One sequence of a ragged batch: `q_len` new tokens at positions [start, start+q_len)."""
    start: int
    q_len: int
    blocks: list[int]
    n_out: int = 1          # logits for the last n_out rows of this sequence


@dataclass
class ForwardPlan:
    """The ragged batch of one model pass, as the int32 arrays the forward kernels
    read (packed into `host` in one buffer, so one copy uploads it): per token its
    position and pool slot, per sequence its query length, row offset, context
    length and block-table row, and the rows whose logits are wanted."""

    seqs: list[SeqSpec] | None
    block_size: int
    host: np.ndarray = field(init=False)
    n_seqs: int = field(init=False)
    n_tokens: int = field(init=False)
    n_out: int = field(init=False)
    max_q_len: int = field(init=False)
    max_ctx: int = field(init=False)
    width: int = field(init=False)
    offsets: dict = field(init=False)

    def __post_init__(self):
        if self.seqs is None:  # filled in by from_arrays
            return
        seqs = self.seqs
        S = len(seqs)
        nb = [len(s.blocks) for s in seqs]
        width = max(1, max(nb) if S else 1)
        tables = np.zeros((S, width), dtype=np.int64)
        if S:
            nblk = np.array(nb, dtype=np.int64)
            tables[np.arange(width) < nblk[:, None]] = list(chain.from_iterable(s.blocks for s in seqs))
        else:
            nblk = np.zeros(0, dtype=np.int64)
        self._build(np.array([s.start for s in seqs], dtype=np.int64),
                    np.array([s.q_len for s in seqs], dtype=np.int64),
                    np.array([s.n_out for s in seqs], dtype=np.int64), tables, nblk)

    @classmethod
    def from_arrays(cls, start: np.ndarray, q_len: np.ndarray, n_out: np.ndarray, tables: np.ndarray,
                    n_blocks: np.ndarray, block_size: int) -> "ForwardPlan":
        """The same plan from per-sequence arrays: start positions, query lengths and
        output-row counts [S], the zero-padded block tables [S, width] and each row's
        block count [S] (a caller that keeps these arrays builds several plans over
        one table without going back to the per-sequence lists)."""
        plan = cls(None, block_size)
        plan._build(np.asarray(start, dtype=np.int64), np.asarray(q_len, dtype=np.int64),
                    np.asarray(n_out, dtype=np.int64), tables, np.asarray(n_blocks, dtype=np.int64))
        return plan

    @classmethod
    def device_built(cls, n_seqs: int, rows: int, width: int, max_ctx: int, block_size: int) -> "ForwardPlan":
        """The shape of a plan whose arrays a kernel writes on the device (no host
        copy): `rows` rows per sequence, the last one's logits wanted, tables of
        `width` blocks, contexts up to `max_ctx`. Same packed layout as _build."""
        plan = cls(None, block_size)
        S, M = n_seqs, rows * n_seqs
        plan.host = None
        plan.n_seqs, plan.n_tokens, plan.n_out = S, M, S
        plan.max_q_len, plan.max_ctx, plan.width = rows, max_ctx, width
        plan.offsets = {}
        off = 0
        for name, n in (("positions", M), ("slots", M), ("q_lens", S), ("q_offsets", S + 1), ("ctx_lens", S),
                        ("out_rows", S), ("tables", S * width)):
            plan.offsets[name] = (off, n)
            off += n
        plan.size = off
        return plan

    def _build(self, start, q, n_out, tables, nblk):
        S = q.shape[0]
        bs = self.block_size
        M = int(q.sum())
        self.n_seqs = S
        self.n_tokens = M
        self.max_q_len = int(q.max()) if S else 0
        ctx = start + q
        self.max_ctx = int(ctx.max()) if S else 0
        if S and bool((nblk * bs < ctx).any()):
            raise ValueError("block table does not cover the sequence (reserve first)")
        self.width = tables.shape[1]
        q_off = np.zeros(S + 1, dtype=np.int64)
        np.cumsum(q, out=q_off[1:])
        if M == S and bool((q == 1).all()):      # one row per sequence (decode passes)
            seq_of_tok, pos = np.arange(S), start
        else:
            seq_of_tok = np.repeat(np.arange(S), q)
            pos = (np.arange(M) - q_off[:-1][seq_of_tok]) + start[seq_of_tok]
        slots = tables[seq_of_tok, pos // bs] * bs + pos % bs
        # logits rows: the last n_out rows of every sequence
        n_tot = int(n_out.sum())
        if n_tot == S and bool((n_out == 1).all()):
            out_rows = q_off[1:] - 1
        else:
            out_rows = (np.repeat(q_off[1:] - n_out, n_out)
                        + (np.arange(n_tot) - np.repeat(np.cumsum(n_out) - n_out, n_out)))
        self.n_out = n_tot
        parts = (("positions", pos), ("slots", slots), ("q_lens", q), ("q_offsets", q_off), ("ctx_lens", ctx),
                 ("out_rows", out_rows), ("tables", tables.reshape(-1)))
        host = np.empty(sum(arr.shape[0] for _, arr in parts), dtype=np.int32)
        self.offsets = {}
        off = 0
        for name, arr in parts:
            n = arr.shape[0]
            self.offsets[name] = (off, n)
            host[off:off + n] = arr
            off += n
        self.host = host


def block_tables(seqs, min_width: int = 1) -> tuple[np.ndarray, np.ndarray]:
    """Zero-padded [len(seqs), width] int64 table of the sequences' block lists and
    the block count of each row."""
    nb = np.fromiter((len(s.blocks) for s in seqs), dtype=np.int64, count=len(seqs))
    width = max(min_width, int(nb.max()) if len(seqs) else 1)
    tables = np.zeros((len(seqs), width), dtype=np.int64)
    if len(seqs):
        tables[np.arange(width) < nb[:, None]] = np.fromiter(chain.from_iterable(s.blocks for s in seqs),
                                                             dtype=np.int64, count=int(nb.sum()))
    return tables, nb


class Runner:
    """Executes forward passes of `model` against `pool` with preallocated scratch."""

    def __init__(self, model: Model, pool):
        self.model = model
        self.pool = pool
        cfg = model.cfg
        if pool.num_layers != cfg.num_layers or pool.head_dim != cfg.head_dim or \
                pool.num_kv_heads != cfg.num_kv_heads or pool.dtype != model.dtype:
            raise ValueError("pool shape/dtype does not match the model")
        self.device = model.device
        self.dt = L.dtype_code(model.dtype)
        w = model.weights
        self._layers = (L.LayerT * cfg.num_layers)()
        for i, lw in enumerate(w.layers):
            self._layers[i] = L.LayerT(lw["w_qkv"].data_ptr(), lw["b_qkv"].data_ptr(), lw["w_o"].data_ptr(),
                                       lw["w_gu"].data_ptr(), lw["w_down"].data_ptr(), lw["ln1"].data_ptr(),
                                       lw["ln2"].data_ptr(), pool.k[i].data_ptr(), pool.v[i].data_ptr())
        self._model_c = L.ModelT(self.dt, cfg.num_layers, cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads,
                                 cfg.head_dim, cfg.intermediate_size, cfg.vocab_size, cfg.rms_norm_eps,
                                 self._layers, w.embed.data_ptr(), w.lm_head.data_ptr(), w.norm.data_ptr(),
                                 w.rope_cos.data_ptr(), w.rope_sin.data_ptr(), w.rope_cos.shape[0],
                                 pool.num_blocks, pool.block_size)
        self._cap_tokens = 0
        self._cap_out = 0
        self._bufs: dict[str, torch.Tensor] = {}
        self.gemm_ws = torch.zeros(256, dtype=torch.uint8, device=self.device)
        self.attn_ws = torch.zeros(256, dtype=torch.uint8, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.plan_dev = torch.zeros(1024, dtype=torch.int32, device=self.device)
        self._graphs: dict[str, C.c_void_p] = {}  # executable graphs of kve_forward_graphed, by slot name
        self.graph_fallbacks: list[str] = []  # errors of graph-launched ranges that ran as stream launches

    def __del__(self):
        graphs = getattr(self, "_graphs", None)
        if graphs and L._lib is not None:
            for h in graphs.values():
                if h.value:
                    L._lib.kve_forward_graph_free(h)
            graphs.clear()

    def _refresh_rope(self, max_pos: int):
        w = self.model.weights
        if max_pos > w.rope_cos.shape[0]:
            w.ensure_rope(max_pos)
            self._model_c.rope_cos = w.rope_cos.data_ptr()
            self._model_c.rope_sin = w.rope_sin.data_ptr()
            self._model_c.rope_len = w.rope_cos.shape[0]

    def ensure(self, n_tokens: int, n_out: int, n_seqs: int, max_q_len: int, max_ctx: int):
        cfg, dev, dt = self.model.cfg, self.device, self.model.dtype
        if n_tokens > self._cap_tokens:
            cap = max(n_tokens, 64)
            self._bufs.update({
                "hidden": torch.empty(cap, cfg.hidden_size, dtype=dt, device=dev),
                "normed": torch.empty(cap, cfg.hidden_size, dtype=dt, device=dev),
                "qkv": torch.empty(cap, cfg.qkv_size, dtype=dt, device=dev),
                "q": torch.empty(cap, cfg.q_size, dtype=dt, device=dev),
                "attn": torch.empty(cap, cfg.q_size, dtype=dt, device=dev),
                "act": torch.empty(cap, cfg.intermediate_size, dtype=dt, device=dev),
            })
            self._cap_tokens = cap
        if n_out > self._cap_out:
            cap = max(n_out, 16)
            self._bufs["out_normed"] = torch.empty(cap, cfg.hidden_size, dtype=dt, device=dev)
            self._cap_out = cap
        need = L.load().kve_forward_gemm_ws_bytes(C.byref(self._model_c), n_tokens, n_out)
        if need > self.gemm_ws.numel():
            self.gemm_ws = torch.zeros(int(need * 1.25) + 4096, dtype=torch.uint8, device=dev)
        need = L.load().kve_forward_attn_ws_bytes(C.byref(self._model_c), n_seqs, max_q_len, max_ctx)
        if need > self.attn_ws.numel():
            self.attn_ws = torch.zeros(int(need * 1.25) + 4096, dtype=torch.uint8, device=dev)
        self._refresh_rope(max_ctx)

    def scratch(self) -> L.ScratchT:
        b = self._bufs
        return L.ScratchT(b["hidden"].data_ptr(), b["normed"].data_ptr(), b["qkv"].data_ptr(), b["q"].data_ptr(),
                          b["attn"].data_ptr(), b["act"].data_ptr(), b["out_normed"].data_ptr(),
                          self.gemm_ws.data_ptr(), self.gemm_ws.numel(), self.attn_ws.data_ptr(),
                          self.attn_ws.numel(), self.status.data_ptr())

    def upload(self, plan: ForwardPlan, dst: torch.Tensor | None = None) -> torch.Tensor:
        """Copy the plan's int32 arrays to the device (one H2D copy)."""
        host = torch.from_numpy(plan.host)
        if dst is None:
            if plan.host.shape[0] > self.plan_dev.numel():
                self.plan_dev = torch.zeros(int(plan.host.shape[0] * 1.5), dtype=torch.int32, device=self.device)
            dst = self.plan_dev
        dst[: host.shape[0]].copy_(host, non_blocking=False)
        return dst

    def batch_struct(self, plan: ForwardPlan, plan_dev: torch.Tensor, ids: torch.Tensor,
                     logits: torch.Tensor | None) -> L.BatchT:
        base = plan_dev.data_ptr()

        def p(name):
            return base + plan.offsets[name][0] * 4

        logits_ptr = logits.data_ptr() if logits is not None else None
        ldt = L.dtype_code(logits.dtype) if logits is not None else self.dt
        return L.BatchT(plan.n_tokens, plan.n_seqs, plan.max_q_len, plan.max_ctx, ids.data_ptr(),
                        p("positions"), p("slots"), p("q_lens"), p("q_offsets"), p("ctx_lens"), p("tables"),
                        plan.width, plan.n_out if logits is not None else 0, p("out_rows"), logits_ptr, ldt)

    def forward(self, plan: ForwardPlan, ids: torch.Tensor, logits: torch.Tensor | None,
                plan_dev: torch.Tensor | None = None, graph: str | None = None, eager_layers: int = 0) -> None:
        """Launch one model pass. `ids`: int32 device [n_tokens]; logits: [n_out, V] or None.
        With `graph` (a slot name) the pass is recorded into that slot's CUDA graph and
        launched as one graph (the current stream must not be the legacy default stream);
        `eager_layers` > 0 launches that many first layers as stream launches before
        recording the rest, so the GPU starts at once."""
        if plan.n_tokens == 0:
            return
        self.ensure(plan.n_tokens, plan.n_out, plan.n_seqs, plan.max_q_len, plan.max_ctx)
        if plan_dev is None:
            plan_dev = self.upload(plan)
        batch = self.batch_struct(plan, plan_dev, ids, logits)
        scratch = self.scratch()
        lib = L.load()
        if graph is None:
            L.check(lib.kve_forward(C.byref(self._model_c), C.byref(batch), C.byref(scratch),
                                    L.stream_handle(self.device)))
        else:
            slot = self._graphs.setdefault(graph, C.c_void_p())
            n_layers = self.model.cfg.num_layers
            e = min(max(eager_layers, 0), n_layers)
            stream = L.stream_handle(self.device)
            if e:
                L.check(lib.kve_forward_layers(C.byref(self._model_c), C.byref(batch), C.byref(scratch), 0, e,
                                               stream))
            rc = lib.kve_forward_layers_graphed(C.byref(self._model_c), C.byref(batch), C.byref(scratch), e,
                                                n_layers, C.byref(slot), stream)
            if rc != L.KVE_OK:
                # Recording or launching the graph failed (the stream is out of capture
                # again and nothing of the range ran): finish the pass with stream
                # launches, so a pass whose first layers already ran still completes.
                msg = lib.kve_last_error().decode(errors="replace")
                if slot.value:
                    lib.kve_forward_graph_free(slot)
                    slot.value = None
                self.graph_fallbacks.append(msg)
                L.check(lib.kve_forward_layers(C.byref(self._model_c), C.byref(batch), C.byref(scratch), e,
                                               n_layers, stream))

    def check_status(self) -> None:
        code = int(self.status.item())
        if code:
            self.status.zero_()
            raise L.KveError(code, "device-side check failed during a forward pass")
