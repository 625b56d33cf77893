"""Drop-in `forward_with_own_cache` (kvengine/forward.py:147-215) on the sm_100a kernels.

Same signature and contract as the reference: one pass over `input_ids`
[1, T] appending to `cache` (reserve once, every layer writes at the same
start, commit once); returns logits [1, T, V] if `all_logits` else [1, 1, V].
The whole pass is one `kve_forward` call; K/V is appended in place and
attention reads the paged blocks directly, so nothing is gathered.
"""

from __future__ import annotations

import torch

from .model import ForwardPlan, Model, Runner, SeqSpec, as_model


def runner_for(model: Model, pool) -> Runner:
    runners = pool.__dict__.setdefault("_runners", {})
    r = runners.get(id(model))
    if r is None:
        r = Runner(model, pool)
        runners[id(model)] = r
    return r


@torch.no_grad()
def forward_with_own_cache(model, input_ids: torch.Tensor, cache, all_logits: bool = False) -> torch.Tensor:
    assert input_ids.dim() == 2 and input_ids.shape[0] == 1, "one request at a time"
    m = as_model(model)
    runner = runner_for(m, cache.pool)
    T = input_ids.shape[1]
    start = cache.length
    cache.reserve(T)
    plan = ForwardPlan([SeqSpec(start, T, list(cache.blocks), n_out=T if all_logits else 1)],
                       cache.pool.block_size)
    ids = input_ids[0].to(device=m.device, dtype=torch.int32)
    logits = torch.empty(plan.n_out, m.cfg.vocab_size, dtype=m.dtype, device=m.device)
    runner.forward(plan, ids, logits)
    cache.commit(T)
    return logits[None]
