"""Generate the golden fixtures by running the REFERENCE itself (kvengine + transformers).

Run in a container where the reference source tree is present:

    python tests/golden/make_golden.py --reference /path/to/kvengine-checkout

It imports the reference's own `speculative_greedy`, `greedy_paged`,
`hf_greedy`, `PagedKVCache`, `BlockManager` and `attend` on CPU, feeds them the
seeded synthetic inputs from `kvengine_b200.workloads` / weights from
`kvengine_b200.weights.init_state_dict` (loaded into a stock
`transformers.Qwen2ForCausalLM`), and writes small JSON/NPZ fixtures next to
this script. The GPU box never runs this file; tests only read its outputs.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from kvengine_b200.config import QWEN2_0_5B, TINY, TINY_HD128  # noqa: E402
from kvengine_b200.weights import init_state_dict  # noqa: E402
from kvengine_b200 import workloads  # noqa: E402


def sha(t) -> str:
    if isinstance(t, torch.Tensor):
        t = t.contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        b = t.numpy().tobytes()
    elif isinstance(t, np.ndarray):
        b = t.tobytes()
    else:
        b = json.dumps(t).encode()
    return hashlib.sha256(b).hexdigest()


def hf_model(cfg, sd, dtype):
    from transformers import Qwen2ForCausalLM

    m = Qwen2ForCausalLM(cfg.to_hf()).eval()
    m.load_state_dict(sd, strict=True)
    # Cast parameters only: `from_pretrained(dtype=...)` (how the reference loads
    # models, kvengine/loader.py:48) keeps the rotary inv_freq buffer in fp32,
    # whereas `.to(dtype)` would round it to the model dtype.
    for p in m.parameters():
        p.data = p.data.to(dtype)
    return m


class Hostile:
    """Same construction as the reference tests' HostileDraft (tests/test_phase5.py:35-50)."""

    def __init__(self, base):
        self.model = base.model
        self.config = base.config
        self.generation_config = base.generation_config
        self._head = base.lm_head

    def lm_head(self, hidden):
        return self._head(hidden).roll(shifts=1, dims=-1)


class Recording:
    """Pass-through view of a model whose lm_head keeps every output it returns,
    so the verify rows of a reference spec run can be read back afterwards."""

    def __init__(self, base):
        self.model = base.model
        self.config = base.config
        self.generation_config = base.generation_config
        self._head = base.lm_head
        self.outputs = []

    def lm_head(self, hidden):
        out = self._head(hidden)
        self.outputs.append(out.detach().float())
        return out


def spec_margins(outputs, k, accepted_per_iter):
    """Top-2 logit margin of the target row behind every emitted token: the verify
    pass of iteration i fed u + k rows; rows u-1 .. u-1+n decided the n accepted
    drafts and the bonus or correction (kvengine/speculative.py:160-182)."""
    margins = []
    for logits, n in zip(outputs, accepted_per_iter):
        rows = logits[0, logits.shape[1] - k - 1:]
        top = rows[: n + 1].topk(2, dim=-1).values
        margins.extend((top[:, 0] - top[:, 1]).tolist())
    return margins


def tiny_fixtures(kv):
    """Spec/greedy sweeps on the two-layer models, fp32 and bf16, with full logits."""
    out = {}
    arrays = {}
    for cfg_name, cfg in (("tiny", TINY), ("tiny_hd128", TINY_HD128)):
        for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            if cfg_name == "tiny_hd128" and dt_name == "bf16":
                continue
            sd = init_state_dict(cfg, seed=3, bias_std=0.02, norm_jitter=0.1)
            m = hf_model(cfg, sd, dt)
            prompts = [workloads.random_prompts(1, n, seed=10 + n, vocab=cfg.vocab_size)[0].tolist()
                       for n in (5, 16, 33)]
            key = f"{cfg_name}_{dt_name}"
            rec = {"prompts": prompts, "greedy": [], "spec_self": {}, "spec_hostile": {},
                   "budgets": {}, "block_sizes": {}}
            for pi, p in enumerate(prompts):
                pool = kv.PagedKVCache.for_model(m, num_blocks=256, block_size=16)
                ids = torch.tensor([p])
                g = kv.greedy_paged(m, ids, pool, max_new_tokens=20, eos_token_id=None,
                                    collect_logits=True)
                rec["greedy"].append(g.new_token_ids)
                arrays[f"{key}_greedy_logits_{pi}"] = g.step_logits.float().numpy()
                hf = kv.hf_greedy(m, ids, max_new_tokens=20, eos_token_id=None)
                assert hf.new_token_ids == g.new_token_ids, "reference greedy_paged != hf_greedy"
            for k in (1, 2, 4, 8):
                rec["spec_self"][k] = []
                rec["spec_hostile"][k] = []
                for p in prompts:
                    pool = kv.PagedKVCache.for_model(m, num_blocks=256, block_size=16)
                    s = kv.speculative_greedy(m, m, torch.tensor([p]), pool.new_sequence("t"),
                                              pool.new_sequence("d"), k=k, max_new_tokens=20,
                                              eos_token_id=None)
                    rec["spec_self"][k].append({"tokens": s.new_token_ids,
                                                "accepted_per_iter": s.accepted_per_iter,
                                                "target_forwards": s.target_forwards,
                                                "draft_forwards": s.draft_forwards})
                    pool = kv.PagedKVCache.for_model(m, num_blocks=256, block_size=16)
                    s = kv.speculative_greedy(m, Hostile(m), torch.tensor([p]), pool.new_sequence("t"),
                                              pool.new_sequence("d"), k=k, max_new_tokens=20,
                                              eos_token_id=None)
                    rec["spec_hostile"][k].append({"tokens": s.new_token_ids,
                                                   "accepted_per_iter": s.accepted_per_iter,
                                                   "target_forwards": s.target_forwards,
                                                   "draft_forwards": s.draft_forwards})
            p = prompts[1]
            for budget in (1, 3, 7, 10):
                pool = kv.PagedKVCache.for_model(m, num_blocks=256, block_size=16)
                s = kv.speculative_greedy(m, m, torch.tensor([p]), pool.new_sequence("t"),
                                          pool.new_sequence("d"), k=4, max_new_tokens=budget,
                                          eos_token_id=None)
                rec["budgets"][budget] = s.new_token_ids
            for bs in (1, 3, 7, 16, 17, 64):
                pool = kv.PagedKVCache.for_model(m, num_blocks=512, block_size=bs)
                g = kv.greedy_paged(m, torch.tensor([p]), pool, max_new_tokens=16, eos_token_id=None)
                rec["block_sizes"][bs] = g.new_token_ids
            # EOS: pick the 6th greedy token of prompt 1 as the stop id.
            eos = rec["greedy"][1][5]
            pool = kv.PagedKVCache.for_model(m, num_blocks=256, block_size=16)
            s = kv.speculative_greedy(m, m, torch.tensor([p]), pool.new_sequence("t"),
                                      pool.new_sequence("d"), k=4, max_new_tokens=20, eos_token_id=eos)
            rec["eos"] = {"eos_id": eos, "tokens": s.new_token_ids, "stopped": s.stopped_on_eos}
            # Rollback: hostile draft, block size 4, k=8 (tests/test_phase5.py:178-201).
            pool = kv.PagedKVCache.for_model(m, num_blocks=64, block_size=4)
            t_seq, d_seq = pool.new_sequence("target"), pool.new_sequence("draft")
            s = kv.speculative_greedy(m, Hostile(m), torch.tensor([p]), t_seq, d_seq, k=8,
                                      max_new_tokens=16, eos_token_id=None)
            rec["rollback"] = {"tokens": s.new_token_ids, "t_blocks": list(t_seq.blocks),
                               "d_blocks": list(d_seq.blocks), "t_len": t_seq.length,
                               "d_len": d_seq.length, "free_list": list(pool.manager._free)}
            out[key] = rec
            print(f"  {key} done", flush=True)
    return out, arrays


SHAPE3B_PROMPT_LENS = (5, 40, 130, 600)
SHAPE3B_NEW = 16


def shape3b_models():
    """The two-layer models with the benchmark's layer shapes, bf16: target of the
    3B architecture (seed 5) and draft of the 0.5B architecture (seed 6), both with
    non-trivial biases and norm weights so a dropped bias or norm weight shows."""
    from kvengine_b200.config import QWEN2_0_5B_L2, QWEN2_3B_L2

    t_sd = init_state_dict(QWEN2_3B_L2, seed=5, bias_std=0.02, norm_jitter=0.1)
    d_sd = init_state_dict(QWEN2_0_5B_L2, seed=6, bias_std=0.02, norm_jitter=0.1)
    return (QWEN2_3B_L2, t_sd), (QWEN2_0_5B_L2, d_sd)


def shape3b_prompts():
    return [workloads.random_prompts(1, n, seed=50 + n)[0].tolist() for n in SHAPE3B_PROMPT_LENS]


def shape3b_fixture(kv):
    """bf16 greedy and speculative decoding at the benchmark's layer shapes (head_dim
    128 / 16-2 heads target, head_dim 64 / 14-2 heads draft, full vocabulary), prompts
    of 5, 40, 130 and 600 ids (the last spans two 512-key attention chunks): greedy
    tokens with the top-2 logits of every step and a hash of the step logits, spec
    tokens for k = 1, 2, 4, 8 with the target itself, the 0.5B-shape model and the
    rolled-head target as drafts, and the rollback tables of one hostile run."""
    (t_cfg, t_sd), (d_cfg, d_sd) = shape3b_models()
    tm = hf_model(t_cfg, t_sd, torch.bfloat16)
    dm = hf_model(d_cfg, d_sd, torch.bfloat16)
    prompts = shape3b_prompts()
    rec = {"prompts": prompts, "new_tokens": SHAPE3B_NEW, "greedy": [], "greedy_top2": [],
           "greedy_logits_sha": [], "spec": {"self": {}, "small": {}, "hostile": {}}}
    for p in prompts:
        pool = kv.PagedKVCache.for_model(tm, num_blocks=256, block_size=16)
        g = kv.greedy_paged(tm, torch.tensor([p]), pool, max_new_tokens=SHAPE3B_NEW, eos_token_id=None,
                            collect_logits=True)
        top = g.step_logits.float().topk(2, dim=-1)
        rec["greedy"].append(g.new_token_ids)
        rec["greedy_top2"].append({"values": top.values.tolist(), "indices": top.indices.tolist()})
        rec["greedy_logits_sha"].append(sha(g.step_logits))
    drafts = {"self": tm, "small": dm, "hostile": Hostile(tm)}
    for name, draft in drafts.items():
        for k in (1, 2, 4, 8):
            rec["spec"][name][k] = []
            for p in prompts:
                t_pool = kv.PagedKVCache.for_model(tm, num_blocks=256, block_size=16)
                d_pool = kv.PagedKVCache.for_model(draft if name != "hostile" else tm, num_blocks=256,
                                                   block_size=16)
                target = Recording(tm)
                s = kv.speculative_greedy(target, draft, torch.tensor([p]), t_pool.new_sequence("t"),
                                          d_pool.new_sequence("d"), k=k, max_new_tokens=SHAPE3B_NEW,
                                          eos_token_id=None)
                rec["spec"][name][k].append({"tokens": s.new_token_ids, "accepted_per_iter": s.accepted_per_iter,
                                             "target_forwards": s.target_forwards,
                                             "draft_forwards": s.draft_forwards,
                                             "margins": spec_margins(target.outputs, k, s.accepted_per_iter)})
        print(f"  shape3b spec {name} done", flush=True)
    # Rollback: 0.5B-shape draft, k = 8, block size 4 (every iteration frees blocks).
    t_pool = kv.PagedKVCache.for_model(tm, num_blocks=512, block_size=4)
    d_pool = kv.PagedKVCache.for_model(dm, num_blocks=512, block_size=4)
    t_seq, d_seq = t_pool.new_sequence("target"), d_pool.new_sequence("draft")
    target = Recording(tm)
    s = kv.speculative_greedy(target, dm, torch.tensor([prompts[1]]), t_seq, d_seq, k=8,
                              max_new_tokens=SHAPE3B_NEW, eos_token_id=None)
    rec["rollback"] = {"tokens": s.new_token_ids, "margins": spec_margins(target.outputs, 8, s.accepted_per_iter), "t_blocks": list(t_seq.blocks), "d_blocks": list(d_seq.blocks),
                       "t_len": t_seq.length, "d_len": d_seq.length, "t_free": list(t_pool.manager._free),
                       "d_free": list(d_pool.manager._free)}
    return rec


def attention_hd128_fixture(kv):
    """The verify attention of the 3B target through the reference's
    PagedSequenceCache.write/_gather and attend(): 16 query / 2 kv heads,
    head_dim 128, 64 sequences x 5 query rows, bf16, block size 16, contexts
    (a) as config 2 draws them (lognormal, median 512) and (b) as config 4's
    decode has them (133..197)."""
    out, arrays = {}, {}
    for name, kw in (("lognormal", {}), ("config4", {"median_ctx": 165.0, "sigma": 0.1,
                                                      "ctx_clip": (133, 197)})):
        w = workloads.attention_workload(seed=7, num_heads=16, num_kv_heads=2, head_dim=128, **kw)
        rec, arr = _attention_reference(kv, w)
        out[name] = rec
        arrays[f"{name}_attn_out_bf16"] = arr
    return out, arrays


def _attention_reference(kv, w):
    from kvengine.forward import attend, causal_mask

    nq, hd = w.q.shape[1], w.q.shape[2]
    nkv = w.k_new.shape[1]

    class A:
        num_key_value_groups = nq // nkv
        scaling = w.scale

    pool = kv.PagedKVCache(num_layers=1, num_kv_heads=nkv, head_dim=hd, num_blocks=w.num_blocks,
                           block_size=w.block_size, dtype=torch.bfloat16, device="cpu")
    outs, k_sha = [], []
    for b, ctx in enumerate(w.ctx_lens):
        s = pool.new_sequence(b)
        s.blocks = list(w.tables[b])
        s._refresh_block_ids()
        hist = ctx - w.q_len
        if hist:
            s.reserve(hist)
            s.write(0, w.k_hist[b].transpose(0, 1)[None], w.v_hist[b].transpose(0, 1)[None], 0)
            s.commit(hist)
        s.reserve(w.q_len)
        rows = slice(b * w.q_len, (b + 1) * w.q_len)
        k_all, v_all = s.write(0, w.k_new[rows].transpose(0, 1)[None], w.v_new[rows].transpose(0, 1)[None], hist)
        s.commit(w.q_len)
        k_sha.append(sha(k_all))
        q = w.q[rows].transpose(0, 1)[None]
        mask = causal_mask(w.q_len, ctx, torch.bfloat16, torch.device("cpu"))
        outs.append(attend(A, q, k_all, v_all, mask, use_sdpa=True)[0])
    out = torch.cat(outs, 0)
    return {"ctx_lens": w.ctx_lens, "k_gather_sha": k_sha}, out.view(torch.int16).numpy()


def cfg1_fixture(kv):
    """Config 1: 0.5B arch, seed 0, fp32, 4 prompts x 64 ids, 64 new tokens, k=4, bs=16."""
    cfg = QWEN2_0_5B
    sd = init_state_dict(cfg, seed=0)
    m = hf_model(cfg, sd, torch.float32)
    prompts = workloads.random_prompts(4, 64, seed=0)
    rec = {"prompts": prompts.tolist(), "spec": [], "greedy": [], "greedy_top2": [], "hf_greedy_0": None}
    for i in range(4):
        ids = prompts[i:i + 1]
        pool = kv.PagedKVCache.for_model(m, num_blocks=512, block_size=16)
        g = kv.greedy_paged(m, ids, pool, max_new_tokens=64, eos_token_id=None, collect_logits=True)
        top = g.step_logits.topk(2, dim=-1)
        rec["greedy"].append(g.new_token_ids)
        rec["greedy_top2"].append({"values": top.values.tolist(), "indices": top.indices.tolist()})
        s = kv.speculative_greedy(m, m, ids, pool.new_sequence("t"), pool.new_sequence("d"), k=4,
                                  max_new_tokens=64, eos_token_id=None)
        rec["spec"].append({"tokens": s.new_token_ids, "accepted_per_iter": s.accepted_per_iter,
                            "target_forwards": s.target_forwards, "draft_forwards": s.draft_forwards,
                            "acceptance_rate": s.acceptance_rate})
        print(f"  cfg1 request {i}: spec==greedy {s.new_token_ids == g.new_token_ids} "
              f"acceptance {s.acceptance_rate:.3f}", flush=True)
    rec["hf_greedy_0"] = kv.hf_greedy(m, prompts[0:1], max_new_tokens=64, eos_token_id=None).new_token_ids
    return rec


def accept_fixture(kv):
    """Config 3 outputs for k in {1,2,4,8}: accepted length, emitted tokens,
    truncated block tables and the free list, through the reference's own
    PagedKVCache / BlockManager and the accept rule of speculative.py:167-197."""
    out = {}
    arrays = {}
    for k in (1, 2, 4, 8):
        w = workloads.accept_workload(k)
        B = w.logits.shape[0]
        pool = kv.PagedKVCache(num_layers=1, num_kv_heads=1, head_dim=1, num_blocks=32768,
                               block_size=16, dtype=torch.float32, device="cpu")
        seqs = [pool.new_sequence(b) for b in range(B)]
        for b, s in enumerate(seqs):
            s.reserve(w.pre_len[b])
            s.commit(w.pre_len[b])
        for b, s in enumerate(seqs):
            s.reserve(k + 1)
            s.commit(k + 1)
        preds = torch.argmax(w.logits, dim=-1)
        n_acc, emitted = [], []
        for b in range(B):
            p = preds[b].tolist()
            d = w.drafts[b].tolist()
            n = 0
            for j in range(k):
                if p[j] != d[j]:
                    break
                n += 1
            em = d + [p[k]] if n == k else d[:n] + [p[n]]
            n_acc.append(n)
            emitted.append(em)
        for b, s in enumerate(seqs):
            keep = w.pre_len[b] + n_acc[b] + 1
            s.truncate(min(s.length, keep))
        tables = [list(s.blocks) for s in seqs]
        flat = np.array([x for t in tables for x in t], dtype=np.int32)
        lens = np.array([len(t) for t in tables], dtype=np.int32)
        arrays[f"k{k}_tables_flat"] = flat
        arrays[f"k{k}_tables_len"] = lens
        arrays[f"k{k}_free_list"] = np.array(pool.manager._free, dtype=np.int32)
        out[k] = {"n_accepted": n_acc, "emitted": emitted, "preds_sha": sha(preds),
                  "seq_len_after": [s.length for s in seqs]}
        print(f"  accept k={k}: mean accepted {np.mean(n_acc):.3f}", flush=True)
    return out, arrays


def attention_fixture(kv):
    """Config 2 through the reference's PagedSequenceCache.write/_gather and attend()."""
    from kvengine.forward import attend, causal_mask

    w = workloads.attention_workload()
    nq, hd = w.q.shape[1], w.q.shape[2]
    nkv = w.k_new.shape[1]

    class A:
        num_key_value_groups = nq // nkv
        scaling = w.scale

    pool = kv.PagedKVCache(num_layers=1, num_kv_heads=nkv, head_dim=hd, num_blocks=w.num_blocks,
                           block_size=w.block_size, dtype=torch.bfloat16, device="cpu")
    outs, k_sha, v_sha = [], [], []
    for b, ctx in enumerate(w.ctx_lens):
        s = pool.new_sequence(b)
        s.blocks = list(w.tables[b])
        s._refresh_block_ids()
        hist = ctx - w.q_len
        if hist:
            s.reserve(hist)
            kh = w.k_hist[b].transpose(0, 1)[None]
            vh = w.v_hist[b].transpose(0, 1)[None]
            s.write(0, kh, vh, 0)
            s.commit(hist)
        s.reserve(w.q_len)
        rows = slice(b * w.q_len, (b + 1) * w.q_len)
        k_all, v_all = s.write(0, w.k_new[rows].transpose(0, 1)[None], w.v_new[rows].transpose(0, 1)[None], hist)
        s.commit(w.q_len)
        k_sha.append(sha(k_all))
        v_sha.append(sha(v_all))
        q = w.q[rows].transpose(0, 1)[None]
        mask = causal_mask(w.q_len, ctx, torch.bfloat16, torch.device("cpu"))
        o = attend(A, q, k_all, v_all, mask, use_sdpa=True)  # [1, T, nq, hd]
        outs.append(o[0])
    out = torch.cat(outs, 0)  # [B*q_len, nq, hd]
    pool_k_used = pool.k[0][torch.tensor([x for t in w.tables for x in t])]
    return ({"ctx_lens": w.ctx_lens, "k_gather_sha": k_sha, "v_gather_sha": v_sha,
             "pool_k_used_sha": sha(pool_k_used)},
            {"attn_out_bf16": out.view(torch.int16).numpy()})


def blocks_fixture(kv):
    """Allocation sequence of the reference's churn test (tests/test_blocks.py:152-192, seed 1234)."""
    import random

    rng = random.Random(1234)
    m = kv.BlockManager(num_blocks=64, block_size=8)
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
            except kv.OutOfBlocks as e:
                ops.append(["oom", owner, want, e.available])
    return {"ops": ops, "final_free": list(m._free)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the kvengine source tree")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import kvengine as kv
    import transformers

    torch.set_num_threads(os.cpu_count() or 1)
    meta = {"torch": torch.__version__, "transformers": transformers.__version__,
            "generated_by": "tests/golden/make_golden.py (reference kvengine on CPU)"}
    jobs = ["blocks", "accept", "attention", "attention_hd128", "tiny", "shape3b", "cfg1"]
    if args.only:
        jobs = args.only.split(",")
    for job in jobs:
        t0 = time.time()
        print(f"[{job}]", flush=True)
        if job == "blocks":
            rec, arr = blocks_fixture(kv), None
        elif job == "accept":
            rec, arr = accept_fixture(kv)
        elif job == "attention":
            rec, arr = attention_fixture(kv)
        elif job == "tiny":
            rec, arr = tiny_fixtures(kv)
        elif job == "attention_hd128":
            rec, arr = attention_hd128_fixture(kv)
        elif job == "shape3b":
            rec, arr = shape3b_fixture(kv), None
        elif job == "cfg1":
            rec, arr = cfg1_fixture(kv), None
        rec = {"meta": meta, "data": rec}
        with open(os.path.join(HERE, f"{job}.json"), "w") as f:
            json.dump(rec, f, separators=(",", ":"))
        if arr:
            np.savez_compressed(os.path.join(HERE, f"{job}.npz"), **arr)
        print(f"[{job}] {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    main()
