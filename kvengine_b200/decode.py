"""Plain greedy decoding on the device path (the spec path's correctness anchor).

`greedy_paged` mirrors kvengine/decode.py:261-332 (prefill through
`forward_with_own_cache`, then one token per pass, argmax each step, blocks
freed at the end unless `free_on_finish=False`). `greedy_batch` runs many
requests together with one ragged forward per step.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from . import ops
from .forward import forward_with_own_cache, runner_for
from .model import ForwardPlan, SeqSpec, as_model

AUTO_EOS = "auto"


def _normalize_eos(eos_token_id) -> set[int]:
    if eos_token_id is None:
        return set()
    if isinstance(eos_token_id, int):
        return {eos_token_id}
    return set(eos_token_id)


def _resolve_eos(model, eos_token_id) -> set[int]:
    """kvengine/decode.py:60-71: AUTO_EOS takes the model's own generation config."""
    if eos_token_id == AUTO_EOS:
        eos_token_id = getattr(getattr(model, "generation_config", None), "eos_token_id", None)
    return _normalize_eos(eos_token_id)


def _sync(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


@dataclass
class GenerationResult:
    prompt_token_ids: list[int]
    new_token_ids: list[int]
    elapsed_s: float
    stopped_on_eos: bool
    step_logits: torch.Tensor | None = field(default=None, repr=False)
    cache_utilization: float | None = None
    blocks_held: int | None = None
    sequence: object | None = field(default=None, repr=False)

    @property
    def all_token_ids(self) -> list[int]:
        return self.prompt_token_ids + self.new_token_ids

    @property
    def tokens_per_s(self) -> float:
        return len(self.new_token_ids) / self.elapsed_s if self.elapsed_s else 0.0


@torch.no_grad()
def greedy_paged(model, input_ids: torch.Tensor, pool, max_new_tokens: int = 32, eos_token_id=AUTO_EOS,
                 collect_logits: bool = False, request_id: object = "req",
                 free_on_finish: bool = True) -> GenerationResult:
    assert input_ids.dim() == 2 and input_ids.shape[0] == 1, "one request at a time"
    m = as_model(model)
    eos = _resolve_eos(model, eos_token_id)
    prompt = input_ids[0].tolist()
    seq = pool.new_sequence(request_id)
    new, logs, stopped = [], [], False
    _sync(m.device)
    t0 = time.perf_counter()
    try:
        logits = forward_with_own_cache(m, input_ids, seq)
        nxt = logits[0, -1]
        for _ in range(max_new_tokens):
            if collect_logits:
                logs.append(nxt.detach().float().cpu())
            tok = int(ops.argmax_rows(nxt[None])[0])
            new.append(tok)
            if tok in eos:
                stopped = True
                break
            nxt = forward_with_own_cache(m, torch.tensor([[tok]], device=m.device), seq)[0, -1]
        _sync(m.device)
        elapsed = time.perf_counter() - t0
        util, held = seq.utilization(), len(seq.blocks)
    finally:
        if free_on_finish:
            seq.free()
    return GenerationResult(prompt, new, elapsed, stopped, torch.stack(logs) if logs else None, util, held,
                            None if free_on_finish else seq)


@torch.no_grad()
def greedy_batch(model, prompts: list[list[int]], pool, max_new_tokens, eos_token_id=AUTO_EOS,
                 collect_logits: bool = False) -> list[GenerationResult]:
    """Greedy decode of many requests with one ragged forward per step."""
    m = as_model(model)
    eos = _resolve_eos(model, eos_token_id)
    budgets = max_new_tokens if isinstance(max_new_tokens, (list, tuple)) else [max_new_tokens] * len(prompts)
    runner = runner_for(m, pool)
    seqs = [pool.new_sequence(f"greedy{i}") for i in range(len(prompts))]
    out = [[] for _ in prompts]
    logs = [[] for _ in prompts]
    stopped = [False] * len(prompts)
    active = [i for i in range(len(prompts)) if budgets[i] > 0]
    pending = {i: list(prompts[i]) for i in active}
    V = m.cfg.vocab_size
    _sync(m.device)
    t0 = time.perf_counter()
    try:
        while active:
            specs = []
            for i in active:
                seqs[i].reserve(len(pending[i]))
                specs.append(SeqSpec(seqs[i].length, len(pending[i]), list(seqs[i].blocks), 1))
            plan = ForwardPlan(specs, pool.block_size)
            ids = torch.tensor([t for i in active for t in pending[i]], dtype=torch.int32).to(m.device)
            logits = torch.empty(len(active), V, dtype=m.dtype, device=m.device)
            runner.forward(plan, ids, logits)
            toks = ops.argmax_rows(logits).tolist()
            if collect_logits:
                lf = logits.float().cpu()
            nxt_active = []
            for row, i in enumerate(active):
                seqs[i].commit(len(pending[i]))
                if collect_logits:
                    logs[i].append(lf[row])
                out[i].append(toks[row])
                if toks[row] in eos:
                    stopped[i] = True
                elif len(out[i]) < budgets[i]:
                    pending[i] = [toks[row]]
                    nxt_active.append(i)
            active = nxt_active
        runner.check_status()
        _sync(m.device)
        elapsed = time.perf_counter() - t0
    finally:
        for s in seqs:
            s.free()
    return [GenerationResult(list(prompts[i]), out[i], elapsed, stopped[i],
                             torch.stack(logs[i]) if logs[i] else None) for i in range(len(prompts))]
