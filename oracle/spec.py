"""Oracle: greedy speculative decoding and plain greedy. TEST INFRASTRUCTURE ONLY.

`oracle_speculative_greedy` restates kvengine/speculative.py:111-216 step for
step (draft k tokens with one forward each, verify u+k in one target forward,
accept the longest matching prefix plus the bonus/correction token, truncate
both caches to len(tokens)-1, trim at EOS and at the budget).
`oracle_greedy_paged` restates kvengine/decode.py:261-332 (prefill, then one
token per forward; blocks freed at the end).

Both take an optional `logits_log` list that receives, per emitted decision,
the fp32 logits row the argmax was taken over, so tests can compare logits and
measure top-1/top-2 margins (near-tie reporting).
"""

from __future__ import annotations

import torch

from .model import OracleModel, oracle_forward


def oracle_speculative_greedy(target: OracleModel, draft: OracleModel, prompt: list[int],
                              t_cache, d_cache, k: int = 4, max_new_tokens: int = 32,
                              eos_ids=(), use_sdpa: bool = True, verify_log: list | None = None):
    assert k >= 1
    assert t_cache.length == 0 and d_cache.length == 0
    eos_ids = set(eos_ids or ())
    tokens = list(prompt)
    res = {"new_token_ids": [], "stopped_on_eos": False, "iterations": 0,
           "tokens_drafted": 0, "tokens_accepted": 0, "accepted_per_iter": [],
           "target_forwards": 0, "draft_forwards": 0}

    def feed(model, cache, ids):
        return oracle_forward(model, ids, cache, all_logits=True, use_sdpa=use_sdpa)

    while len(res["new_token_ids"]) < max_new_tokens:
        unseen = tokens[d_cache.length:]
        logits = feed(draft, d_cache, unseen)
        res["draft_forwards"] += 1
        drafts = []
        for j in range(k):
            drafts.append(int(torch.argmax(logits[-1])))
            if j < k - 1:
                logits = feed(draft, d_cache, [drafts[-1]])
                res["draft_forwards"] += 1
        unseen_t = tokens[t_cache.length:]
        u = len(unseen_t)
        t_logits = feed(target, t_cache, unseen_t + drafts)
        res["target_forwards"] += 1
        rows = t_logits[u - 1:]
        if verify_log is not None:
            verify_log.append({"drafts": list(drafts), "rows": rows.float().clone(),
                               "position": len(tokens)})
        preds = torch.argmax(rows, dim=-1).tolist()
        n = 0
        for j in range(k):
            if preds[j] != drafts[j]:
                break
            n += 1
        emitted = drafts + [preds[k]] if n == k else drafts[:n] + [preds[n]]
        res["iterations"] += 1
        res["tokens_drafted"] += k
        res["tokens_accepted"] += n
        res["accepted_per_iter"].append(n)
        tokens.extend(emitted)
        res["new_token_ids"].extend(emitted)
        keep = len(tokens) - 1
        t_cache.truncate(min(t_cache.length, keep))
        d_cache.truncate(min(d_cache.length, keep))
        if any(t in eos_ids for t in emitted):
            first = next(i for i, t in enumerate(emitted) if t in eos_ids)
            trim = len(emitted) - (first + 1)
            if trim:
                res["new_token_ids"] = res["new_token_ids"][:-trim]
            res["stopped_on_eos"] = True
            break
    if len(res["new_token_ids"]) > max_new_tokens:
        res["new_token_ids"] = res["new_token_ids"][:max_new_tokens]
        res["stopped_on_eos"] = res["new_token_ids"][-1] in eos_ids
    return res


def oracle_greedy_paged(model: OracleModel, prompt: list[int], cache, max_new_tokens: int = 32,
                        eos_ids=(), use_sdpa: bool = True, logits_log: list | None = None):
    eos_ids = set(eos_ids or ())
    new = []
    stopped = False
    logits = oracle_forward(model, list(prompt), cache, use_sdpa=use_sdpa)
    nxt = logits[-1]
    for _ in range(max_new_tokens):
        if logits_log is not None:
            logits_log.append(nxt.float().clone())
        tok = int(torch.argmax(nxt))
        new.append(tok)
        if tok in eos_ids:
            stopped = True
            break
        nxt = oracle_forward(model, [tok], cache, use_sdpa=use_sdpa)[-1]
    return {"new_token_ids": new, "stopped_on_eos": stopped, "blocks_held": len(cache.blocks)}


def top2_margin(row: torch.Tensor) -> float:
    v = row.float().topk(2).values
    return float(v[0] - v[1])


def verify_log_margins(verify_log: list) -> dict:
    """Top-2 logits of the target row behind every emitted token of an
    `oracle_speculative_greedy` run that was given `verify_log`: per iteration
    the rows u-1 .. u-1+n decided the n accepted drafts and the bonus or
    correction token (kvengine/speculative.py:167-182). Same layout as a greedy
    run's per-step top-2 record ({"values": [[v0, v1], ...]}), so token-identity
    checks can tell near-ties from real differences."""
    values = []
    for it in verify_log:
        rows = it["rows"]
        drafts = it["drafts"]
        preds = torch.argmax(rows, dim=-1).tolist()
        n = 0
        while n < len(drafts) and preds[n] == drafts[n]:
            n += 1
        top = rows[: n + 1].float().topk(2, dim=-1).values
        values.extend(top.tolist())
    return {"values": values}


def config4_oracle_models(target, draft):
    """Oracle copies (CPU, bf16) of the benchmark's device-resident 3B target and
    0.5B draft."""
    from .model import state_dict_from_device

    return (OracleModel(target.cfg, state_dict_from_device(target), torch.bfloat16),
            OracleModel(draft.cfg, state_dict_from_device(draft), torch.bfloat16))


@torch.no_grad()
def teacher_forced_check(model: OracleModel, prompt: list[int], tokens: list[int], tol: float,
                         model_fp32: OracleModel | None = None) -> dict:
    """Check a generated sequence token by token against the oracle's logits.

    One oracle pass over prompt + tokens[:-1] gives the logits row that predicts
    every generated token along the sequence's OWN history, so a near-tie early
    on does not end the comparison. `exact` counts tokens that are the (bf16)
    oracle's argmax outright (first index on ties, as torch.argmax).

    Without `model_fp32`, token j passes when its oracle logit is within `tol`
    of the row maximum. With it (the same weights evaluated in fp32: the exact
    answer bf16 arithmetic approximates), token j passes when its fp32 logit is
    within max(tol, 2 * eps_j) of the fp32 row maximum, where eps_j is the
    largest |bf16 - fp32| logit difference of the oracle - i.e. of the
    reference, which the oracle reproduces bit for bit - on that row: a choice
    the reference's own rounding could have made. `near_ties` lists the passing
    tokens that are not the bf16 oracle's argmax; `worst` is the largest
    (fp32 max - token logit) / allowed ratio (<= 1 passes)."""
    from .paged import OraclePool

    if not tokens:
        return {"ok": True, "checked": 0, "exact": 0, "near_ties": [], "worst": 0.0}

    def rows_of(m):
        cfg = m.cfg
        seq = OraclePool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim,
                         -(-(len(prompt) + len(tokens)) // 16) + 1, 16, m.dtype).new_sequence()
        logits = oracle_forward(m, list(prompt) + list(tokens[:-1]), seq, all_logits=True).float()
        return logits[len(prompt) - 1:]

    tok = torch.tensor(tokens, dtype=torch.long)
    rows = rows_of(model)
    arg = rows.argmax(dim=-1)
    exact = int((arg == tok).sum())
    if model_fp32 is None:
        ref, allow = rows, torch.full((len(tokens),), float(tol))
    else:
        ref = rows_of(model_fp32)
        eps = (rows - ref).abs().max(dim=-1).values
        allow = torch.clamp(2 * eps, min=tol)
    gap = ref.max(dim=-1).values - ref.gather(1, tok[:, None])[:, 0]
    ratio = gap / allow
    near = [{"position": j, "gap": round(float(gap[j]), 5), "allowed": round(float(allow[j]), 5)}
            for j in range(len(tokens)) if int(arg[j]) != tokens[j] and float(ratio[j]) <= 1.0]
    return {"ok": bool((ratio <= 1.0).all()), "checked": len(tokens), "exact": exact, "near_ties": near,
            "worst": round(float(ratio.max()), 4), "max_allowed": round(float(allow.max()), 5)}
