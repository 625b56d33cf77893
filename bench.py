"""Benchmark: accepted tokens/s of greedy speculative decoding, 0.5B-arch draft -> 3B-arch target, k=4.

Workload (benchmark config 4 at k=4): draft Qwen2.5-0.5B architecture (seed 1),
target Qwen2.5-3B architecture (seed 2), random-init bf16, 64 requests per
GPU with 128 uniform-random prompt ids each, 64 new tokens per request, KV
block size 16. One step = one full batched speculative decode of those
requests (prefill fused into the first verify pass, as the reference does).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

`value`: accepted (emitted) tokens/s over all ranks with the weights and the
request token lists resident before the timed region; `e2e`: the same through
the public API `speculative_greedy_batch` from a pinned host prompt tensor,
with every host<->device copy inside the timed region. `roofline`: the verify
step (one target pass over B*(k+1) rows), timed with CUDA events on its
stream during the timed steps. `--impl reference` times the CPU oracle port
of the reference's path on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K_SPEC = 4
N_REQ = 64
PROMPT = 128
NEW = 64
BLOCK = 16


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p["bf16_tflops_sustained"], "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def verify_algorithmic(plans, target_cfg, weight_bytes: int):
    """Bytes and FLOPs one verify pass must move/do (per launch, averaged)."""
    kv_tok = target_cfg.kv_bytes_per_token(2)
    V, H = target_cfg.vocab_size, target_cfg.hidden_size
    L, nq, hd = target_cfg.num_layers, target_cfg.num_heads, target_cfg.head_dim
    tot_b = tot_f = 0.0
    for plan in plans:
        rows = plan.n_tokens
        off = plan.offsets
        q = plan.host[off["q_lens"][0]: off["q_lens"][0] + off["q_lens"][1]]
        ctx = plan.host[off["ctx_lens"][0]: off["ctx_lens"][0] + off["ctx_lens"][1]]
        hist = float((ctx - q).sum())
        n_out = plan.n_out
        b = weight_bytes + hist * kv_tok + rows * kv_tok + n_out * V * 2 + rows * H * 2
        params = weight_bytes / 2
        attn = 4.0 * float((q.astype("float64") * ctx).sum()) * nq * hd * L
        f = 2.0 * rows * (params - V * H) + 2.0 * n_out * V * H + attn
        tot_b += b
        tot_f += f
    n = max(1, len(plans))
    return tot_b / n, tot_f / n


def run_gpu(args):
    import torch.distributed as dist

    from kvengine_b200 import Model, PagedKVCache, SpecEngine, speculative_greedy_batch
    from kvengine_b200 import _lib as L
    from kvengine_b200.config import QWEN2_0_5B, QWEN2_3B
    from kvengine_b200.speculative import _Request
    from kvengine_b200.workloads import random_prompts

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=600))
    draft = Model.random_init(QWEN2_0_5B, seed=1, dtype=torch.bfloat16, device=dev, init_device=dev)
    target = Model.random_init(QWEN2_3B, seed=2, dtype=torch.bfloat16, device=dev, init_device=dev)
    # Requests are sharded by rank: rank r decodes requests [r*64, (r+1)*64) of a seeded set.
    prompts_all = random_prompts(N_REQ * world, PROMPT, seed=4)
    prompts = prompts_all[rank * N_REQ:(rank + 1) * N_REQ].tolist()
    blocks_per_seq = -(-(PROMPT + NEW + 2 * K_SPEC + 2) // BLOCK)
    t_pool = PagedKVCache.for_model(target, num_blocks=N_REQ * blocks_per_seq + 64, block_size=BLOCK)
    d_pool = PagedKVCache.for_model(draft, num_blocks=N_REQ * blocks_per_seq + 64, block_size=BLOCK)
    eng = SpecEngine(target, draft, t_pool, d_pool, K_SPEC)
    lib = L.load()

    def one_step(collect=None):
        reqs = [_Request(p, t_pool.new_sequence(f"t{i}"), d_pool.new_sequence(f"d{i}"), NEW)
                for i, p in enumerate(prompts)]
        eng.run(reqs, set())
        toks = sum(len(r.res.new_token_ids) for r in reqs)
        if collect is not None:
            collect.append(reqs)
        for r in reqs:
            r.t_seq.free()
            r.d_seq.free()
        return toks

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()

    # ---------------------------------------------------------------- value
    props = torch.cuda.get_device_properties(dev)
    bus = getattr(props, "pci_bus_id", None)
    smi_id = f"{getattr(props, 'pci_domain_id', 0):08x}:{bus:02x}:{getattr(props, 'pci_device_id', 0):02x}.0" \
        if bus is not None else str(local)
    sampler = ClockSampler(smi_id)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    eng.verify_events = []
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = lib.kve_launch_count()
    stats0 = dict(eng.stats)
    spec0 = dict(eng.spec_stats)
    collected = []
    ev0.record()
    tokens = 0
    for _ in range(args.steps):
        tokens += one_step(collected)
    ev1.record()
    torch.cuda.synchronize()
    launches = lib.kve_launch_count() - launches0
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    verify_ev = eng.verify_events
    eng.verify_events = None
    t = torch.tensor([ms], device=dev)
    tok_t = torch.tensor([float(tokens)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(tok_t, op=dist.ReduceOp.SUM)
    ms_max = float(t.item())
    total_tokens = float(tok_t.item())
    value = total_tokens / (ms_max / 1e3)
    accepted = sum(r.res.tokens_accepted for reqs in collected for r in reqs)
    drafted = sum(r.res.tokens_drafted for reqs in collected for r in reqs)
    iters = eng.stats["iterations"] - stats0["iterations"]
    spec_first = {key: eng.spec_stats[key] - spec0[key] for key in spec0}

    # ------------------------------------------------------------ roofline
    steady = [(a, b, p) for a, b, p in verify_ev if p.max_q_len == K_SPEC + 1]
    prefill = [(a, b, p) for a, b, p in verify_ev if p.max_q_len != K_SPEC + 1]
    v_ms = statistics.mean(a.elapsed_time(b) for a, b, _ in steady) if steady else float("nan")
    wb = target.weights.weight_bytes()
    alg_b, alg_f = verify_algorithmic([p for _, _, p in steady], QWEN2_3B, wb)
    ctx_sum = statistics.mean(float(p.host[p.offsets["ctx_lens"][0]: p.offsets["ctx_lens"][0] + p.offsets["ctx_lens"][1]]
                                    .sum()) for _, _, p in steady) if steady else float(VERIFY_KERNEL_DRAM_CTX)
    traffic = verify_pass_traffic(QWEN2_3B.num_layers, ctx_sum)
    pk = peaks()
    t_hbm = alg_b / (pk["hbm_gbs"] * 1e9)
    t_tc = alg_f / (pk["bf16_tflops_sustained"] * 1e12)
    bound = "tensor" if t_tc > t_hbm else "hbm"
    if bound == "tensor":
        achieved = alg_f / (v_ms / 1e3) / 1e12
        peak = pk["bf16_tflops_sustained"]
        unit = "TFLOP/s"
    else:
        achieved = alg_b / (v_ms / 1e3) / 1e9
        peak = pk["hbm_gbs"]
        unit = "GB/s"
    roofline = {
        "kernel": "verify step: kve_forward of the 3B target over B*(k+1)=320 rows (36 layers + lm_head)",
        "bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
        "frac": round(achieved / peak, 4), "peak_src": pk["src"] + (" sustained" if bound == "tensor" else ""),
        "traffic": traffic, "traffic_src": "per-kernel ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch "
        "each (profiles/verify_pass_dram_config4.md) x launches per 36-layer pass; attention scaled by context",
        "verify_ms": round(v_ms, 4), "verify_passes_timed": len(steady),
        "alg_bytes_per_launch": round(alg_b), "alg_flops_per_launch": round(alg_f),
        "hbm_gbs_achieved": round(alg_b / (v_ms / 1e3) / 1e9, 1),
        "hbm_frac": round(alg_b / (v_ms / 1e3) / 1e9 / pk["hbm_gbs"], 4),
        "roofline_ms": round(max(t_hbm, t_tc) * 1e3, 4),
        "frac_of_roofline_time": round(max(t_hbm, t_tc) * 1e3 / v_ms, 4),
        "prefill_verify_ms": round(statistics.mean(a.elapsed_time(b) for a, b, _ in prefill), 3) if prefill else None,
    }

    # ----------------------------------------------------------------- e2e
    pinned = torch.tensor(prompts, dtype=torch.int64).pin_memory()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h2d0, d2h0 = eng.stats["h2d_bytes"], eng.stats["d2h_bytes"]
    e_tokens = 0
    out_bytes = 0
    e0.record()
    for _ in range(args.steps):
        res, _wall = speculative_greedy_batch(target, draft, pinned, t_pool, d_pool, k=K_SPEC,
                                              max_new_tokens=NEW, eos_token_id=None, engine=eng)
        out = torch.tensor([r.new_token_ids for r in res], dtype=torch.int32)
        out_bytes += out.numel() * 4
        e_tokens += int(out.numel())
    e1.record()
    torch.cuda.synchronize()
    e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    e_tok = torch.tensor([float(e_tokens)], device=dev)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(e_tok, op=dist.ReduceOp.SUM)
    h2d = (eng.stats["h2d_bytes"] - h2d0) / args.steps
    d2h = (eng.stats["d2h_bytes"] - d2h0) / args.steps
    e2e = {"value": round(float(e_tok.item()) / (float(e_ms.item()) / 1e3), 2), "unit": "accepted tokens/s",
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
           "api": "kvengine_b200.speculative_greedy_batch(pinned host prompt tensor) -> host token lists; "
                  "counted bytes = every plan/token upload and every accept readback"}

    # ------------------------------------------------- results to every rank (NCCL, untimed)
    if world > 1:
        from kvengine_b200.distributed import gather_tokens

        local = {rank * N_REQ + i: r.res.new_token_ids for i, r in enumerate(collected[-1])}
        everything = gather_tokens(local, device=dev)
        assert len(everything) == N_REQ * world
        dist.barrier()
        dist.destroy_process_group()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gpu_tokens = [r.res.new_token_ids for r in collected[-1]]
        cpu = cpu_baseline(oracle_models(target, draft), prompts, gpu_tokens)

    if rank == 0:
        line = {
            "metric": f"accepted tokens/s (0.5B->3B, k={K_SPEC})",
            "value": round(value, 2), "unit": "accepted tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random ids, random-init weights)",
            "config": {"workload": f"config 4 at k={K_SPEC}: 0.5B-arch draft (seed 1) -> 3B-arch target (seed 2), bf16",
                       "requests_per_gpu": N_REQ, "prompt_len": PROMPT, "new_tokens": NEW, "k": K_SPEC,
                       "block_size": BLOCK, "global_requests": N_REQ * world, "parallelism": f"dp{world} (requests sharded)",
                       "l2": "inputs larger than L2 (6.2 GB target + 1.0 GB draft weights streamed per pass)"},
            "acceptance_rate": round(accepted / drafted, 4) if drafted else None,
            "iterations_per_step": iters / args.steps,
            "first_draft_pass_planned_on_device": spec_first,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "roofline": roofline,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if cpu is not None and "tokens_match" in cpu:
            line["tokens_match"] = cpu["tokens_match"]
            line["tokens_checked"] = cpu["tokens_checked"]
            line["near_ties"] = len(cpu["near_ties"])
        print(json.dumps(line), flush=True)


CPU_SAMPLE_TOKENS = 24
CPU_SAMPLES = 5


def oracle_models(target=None, draft=None):
    """CPU oracle models holding the benchmark's weights: copied from the GPU
    models when given, else the same seeded init generated on the GPU if one is
    present, else on the CPU."""
    from kvengine_b200.config import QWEN2_0_5B, QWEN2_3B
    from kvengine_b200.weights import init_state_dict
    from oracle.model import OracleModel
    from oracle.spec import config4_oracle_models

    if target is not None:
        return config4_oracle_models(target, draft)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    t_sd = {k: v.cpu() for k, v in init_state_dict(QWEN2_3B, 2, dtype=torch.bfloat16, device=dev).items()}
    d_sd = {k: v.cpu() for k, v in init_state_dict(QWEN2_0_5B, 1, dtype=torch.bfloat16, device=dev).items()}
    return OracleModel(QWEN2_3B, t_sd, torch.bfloat16), OracleModel(QWEN2_0_5B, d_sd, torch.bfloat16)


def cpu_sample(models, prompt, verify_log=None):
    """One bounded CPU sample: the oracle (a port of the reference's
    speculative_greedy path) decodes one request of the benchmark - the
    prefill-fused first verify, then spec iterations - until CPU_SAMPLE_TOKENS
    new tokens, bf16, on every host thread. Returns (result, seconds)."""
    from oracle.paged import OraclePool
    from oracle.spec import oracle_speculative_greedy

    torch.set_num_threads(len(os.sched_getaffinity(0)))
    tm, dm = models
    tp = OraclePool(36, 2, 128, 64, BLOCK, torch.bfloat16)
    dp = OraclePool(24, 2, 64, 64, BLOCK, torch.bfloat16)
    t0 = time.perf_counter()
    res = oracle_speculative_greedy(tm, dm, prompt, tp.new_sequence(), dp.new_sequence(), k=K_SPEC,
                                    max_new_tokens=CPU_SAMPLE_TOKENS, verify_log=verify_log)
    return res, time.perf_counter() - t0


def _sample_text(n, iters, secs):
    return (f"median of {CPU_SAMPLES} samples, each 1 request (prompt {PROMPT} ids, requests 0-{CPU_SAMPLES - 1} of "
            f"the benchmark), k={K_SPEC}, {n} new tokens in {iters} iterations incl. the prefill-fused first "
            f"verify; CPU oracle port of kvengine's speculative_greedy in bf16; {secs:.1f} s in all")


def cpu_baseline(models, prompts, gpu_tokens=None):
    """The CPU baseline on CPU_SAMPLES bounded samples (requests 0 .. CPU_SAMPLES-1
    of the workload, one each), reported as the median. With `gpu_tokens` (the
    GPU's new tokens per request), every GPU token of those requests is also
    checked against the oracle teacher-forced along the GPU's own sequence (one
    bf16 and one fp32 oracle pass of the full-depth target per request):
    `tokens_match` is true when every token is a choice the reference's own bf16
    rounding could make (its fp32 logit within max(2e-2, twice the bf16 oracle's
    deviation from fp32 on that row) of the fp32 maximum, oracle.spec.
    teacher_forced_check); `tokens_exact` counts the tokens that are the bf16
    oracle's argmax outright and `near_ties` lists the others."""
    from oracle.spec import teacher_forced_check

    target32 = models[0].as_fp32() if gpu_tokens is not None else None
    vals, total, n, iters = [], 0.0, 0, 0
    checked = exact = 0
    ok, near_ties, worst = True, [], 0.0
    for i in range(CPU_SAMPLES):
        res, dt = cpu_sample(models, prompts[i])
        n, iters = len(res["new_token_ids"]), res["iterations"]
        vals.append(n / dt)
        total += dt
        if gpu_tokens is not None:
            tf = teacher_forced_check(models[0], prompts[i], list(gpu_tokens[i]), 2e-2, model_fp32=target32)
            ok = ok and tf["ok"]
            checked += tf["checked"]
            exact += tf["exact"]
            worst = max(worst, tf["worst"])
            near_ties += [dict(request=i, **t) for t in tf["near_ties"]]
    out = {"value": round(statistics.median(vals), 3), "unit": "accepted tokens/s",
           "cores": len(os.sched_getaffinity(0)), "kind": "port", "sample": _sample_text(n, iters, total),
           "samples": [round(v, 3) for v in vals]}
    if gpu_tokens is not None:
        out["tokens_match"] = ok
        out["tokens_checked"] = checked
        out["tokens_exact"] = exact
        out["near_ties"] = near_ties
        out["worst_gap_ratio"] = worst
        out["token_rule"] = ("every GPU token of requests 0-%d teacher-forced along the GPU's sequence through the "
                             "full-depth 3B oracle: fp32 logit within max(2e-2, 2 x the bf16 oracle's deviation from "
                             "fp32 on the row) of the fp32 max" % (CPU_SAMPLES - 1))
    return out


def run_reference(args):
    from kvengine_b200.workloads import random_prompts

    rank, world, _ = dist_env()
    if rank != 0:
        return
    models = oracle_models()
    prompts = random_prompts(N_REQ, PROMPT, seed=4).tolist()
    vals, secs, n, iters = [], 0.0, 0, 0
    for i in range(args.warmup + args.steps):
        res, dt = cpu_sample(models, prompts[i % CPU_SAMPLES])
        if i >= args.warmup:
            n, iters = len(res["new_token_ids"]), res["iterations"]
            vals.append(n / dt)
            secs += dt
    v = statistics.median(vals)
    sample = (f"median of {args.steps} steps, each 1 request (prompt {PROMPT} ids, requests 0-{CPU_SAMPLES - 1} of "
              f"the benchmark in turn), k={K_SPEC}, {n} new tokens in {iters} iterations incl. the prefill-fused "
              f"first verify; CPU oracle port of kvengine's speculative_greedy in bf16; {secs:.1f} s timed")
    line = {"impl": "reference", "metric": f"accepted tokens/s (0.5B->3B, k={K_SPEC})", "value": round(v, 3),
            "unit": "accepted tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random ids, random-init weights)",
            "config": {"workload": f"config 4 at k={K_SPEC}: 0.5B-arch draft (seed 1) -> 3B-arch target (seed 2), bf16",
                       "sample_per_step": sample},
            "cpu_baseline": {"value": round(v, 3), "unit": "accepted tokens/s",
                             "cores": len(os.sched_getaffinity(0)), "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 3), "unit": "accepted tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _time_launches(fns, iters: int) -> float:
    """Mean GPU ms per kernel call. `fns` is a list of zero-argument launches over
    disjoint inputs whose total size exceeds the L2 (so every call reads from
    HBM); they are captured once into a CUDA graph and the graph is replayed
    between CUDA events, which keeps host launch overhead out of the number."""
    for f in fns:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for f in fns:
                f()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (iters * len(fns))
    del g
    return ms


L2_BYTES = 126 * 2**20

# DRAM bytes (read + write) per launch of each kernel of a steady verify pass, from
# single-kernel ncu captures (dram__bytes_read.sum + dram__bytes_write.sum, one launch
# each, --cache-control none) of `bench.py --profile-verify-small`: the config-4 batch
# (64 requests, k = 4, block size 16) on two-layer models with the benchmark's layer
# shapes, whose per-layer kernels have the 36-layer pass's grids and shapes. Summary and
# commands: profiles/verify_pass_dram_config4.md. The attention kernel's traffic is its
# K/V reads; it is scaled by the timed plans' context sum over the captured case's
# (64 sequences at context 136).
VERIFY_KERNEL_DRAM = {
    "embed": 1_047_808, "rmsnorm": 31_744, "qkv_rope_append_gemm": 10_690_000, "attention": 9_312_512,
    "o_proj": 8_610_000, "gate_up_swiglu": 107_810_000, "down": 52_750_000, "lm_head": 721_610_000,
}
VERIFY_KERNEL_DRAM_CTX = 64 * 136


def verify_pass_traffic(n_layers: int, ctx_sum: float) -> int:
    k = VERIFY_KERNEL_DRAM
    per_layer = (k["qkv_rope_append_gemm"] + k["o_proj"] + k["gate_up_swiglu"] + k["down"] + 2 * k["rmsnorm"]
                 + k["attention"] * ctx_sum / VERIFY_KERNEL_DRAM_CTX)
    return int(n_layers * per_layer + k["embed"] + k["rmsnorm"] + k["lm_head"])


def run_micro(args):
    """Per-kernel microbenchmarks (one JSON line each) on the benchmark configurations
    2 (attention), 3 (accept) and the verify GEMM shapes, timed with CUDA events."""
    from kvengine_b200 import ops, workloads

    dev = torch.device("cuda", 0)
    pk = peaks()
    out = []
    which = args.micro.split(",")
    if "accept" in which:
        for k in (1, 2, 4, 8):
            w = workloads.accept_workload(k)
            lg, dr = w.logits.to(dev), w.drafts.to(torch.int32).to(dev)
            ws = ops.Workspace(dev)
            ms = _time_launches([lambda: ops.greedy_accept(lg, dr, ws)], args.steps)
            nbytes = lg.numel() * 4
            out.append({"micro": "greedy_accept (config 3)", "k": k, "batch": 256, "ms": round(ms, 4),
                        "alg_bytes": nbytes, "gbs": round(nbytes / ms / 1e6, 1),
                        "frac_hbm": round(nbytes / ms / 1e6 / pk["hbm_gbs"], 4)})
            del lg
    if "attention" in which:
        w = workloads.attention_workload()
        shape = (w.num_blocks, w.block_size, w.k_new.shape[1], w.k_new.shape[2])
        dk = torch.randn(shape, device=dev).to(torch.bfloat16)  # timing only: any finite contents
        dv = torch.randn(shape, device=dev).to(torch.bfloat16)
        B = w.num_seqs
        width = max(len(t) for t in w.tables)
        tables = torch.zeros(B, width, dtype=torch.int32)
        for b, t in enumerate(w.tables):
            tables[b, : len(t)] = torch.tensor(t, dtype=torch.int32)
        tables = tables.to(dev)
        ctx = torch.tensor(w.ctx_lens, dtype=torch.int32, device=dev)
        ql = torch.full((B,), w.q_len, dtype=torch.int32, device=dev)
        qo = (torch.arange(B + 1, dtype=torch.int32) * w.q_len).to(dev)
        q = w.q.to(dev)
        o = torch.empty_like(q)
        ws = ops.Workspace(dev)
        mc = max(w.ctx_lens)
        # 8 block-id shifts of the same tables: each call reads (mostly) different blocks, 8x the K/V > L2
        shifted = [((tables + r * 8192) % w.num_blocks).to(torch.int32) for r in range(8)]
        ms = _time_launches([(lambda tb=tb: ops.paged_attention(q, dk, dv, tb, ctx, ql, qo, w.q_len, mc, w.scale, out=o,
                                                                workspace=ws)) for tb in shifted], args.steps)
        kvb = sum(w.ctx_lens) * 2 * 64 * 2 * 2
        qob = q.numel() * 2 * 2
        out.append({"micro": "paged_verify_attention (config 2)", "seqs": B, "q_len": w.q_len,
                    "mean_ctx": round(sum(w.ctx_lens) / B, 1), "ms": round(ms, 4), "alg_bytes": kvb + qob,
                    "gbs": round((kvb + qob) / ms / 1e6, 1), "frac_hbm": round((kvb + qob) / ms / 1e6 / pk["hbm_gbs"], 4)})
    if "attention_decode" in which:
        # Config 4's decode attention: the draft pass (0.5B: 14 query / 2 kv heads, hd 64,
        # one row per sequence) and the verify pass (3B: 16 / 2 heads, hd 128, k + 1 = 5 rows),
        # 64 sequences at context 190, block size 16; 8 disjoint block sets, cycled.
        # Also the prompt pass (fused into the first verify: 128 prompt ids + k + 1 = 132 rows
        # per sequence on the 3B; 128 on the draft), causal over its own rows.
        for name, nq, nkv, hd, qlen, ctx_len in (("draft", 14, 2, 64, 1, 190), ("verify", 16, 2, 128, 5, 190),
                                                  ("draft prompt", 14, 2, 64, 128, 128),
                                                  ("verify prompt", 16, 2, 128, 132, 132)):
            B, bs = 64, 16
            nbs = -(-ctx_len // bs)
            shape = (B * nbs * 8, bs, nkv, hd)
            dk = torch.randn(shape, device=dev).to(torch.bfloat16)  # timing only: any finite contents
            dv = torch.randn(shape, device=dev).to(torch.bfloat16)
            tables = torch.arange(B * nbs, dtype=torch.int32, device=dev).view(B, nbs)
            shifted = [(tables + r * B * nbs).to(torch.int32) for r in range(8)]
            ctx = torch.full((B,), ctx_len, dtype=torch.int32, device=dev)
            ql = torch.full((B,), qlen, dtype=torch.int32, device=dev)
            qo = (torch.arange(B + 1, dtype=torch.int32) * qlen).to(dev)
            q = torch.randn(B * qlen, nq, hd, device=dev).to(torch.bfloat16)
            o = torch.empty_like(q)
            ws = ops.Workspace(dev)
            ms = _time_launches([(lambda tb=tb: ops.paged_attention(q, dk, dv, tb, ctx, ql, qo, qlen, ctx_len,
                                                                    hd ** -0.5, out=o, workspace=ws))
                                 for tb in shifted], args.steps)
            kvb = B * ctx_len * nkv * hd * 2 * 2
            out.append({"micro": f"paged_verify_attention decode (config 4 {name})", "seqs": B, "q_len": qlen,
                        "ctx": ctx_len, "heads": [nq, nkv, hd], "ms": round(ms, 4), "alg_bytes": kvb + 2 * q.numel() * 2,
                        "gbs": round((kvb + 2 * q.numel() * 2) / ms / 1e6, 1)})
            del dk, dv
    if "gemm" in which:
        g = torch.Generator(device=dev).manual_seed(0)
        from kvengine_b200 import _lib as L

        # Each shape with the epilogue the forward pass uses on it (verify pass of
        # 64 requests x 5 rows on the 3B target; one-token draft pass on the 0.5B).
        cases = (("qkv", 320, 2560, 2048, L.EPI_BIAS), ("o_proj", 320, 2048, 2048, L.EPI_RESIDUAL),
                 ("gate_up", 320, 22016, 2048, L.EPI_SILU_MUL), ("down", 320, 2048, 11008, L.EPI_RESIDUAL),
                 ("lm_head", 320, 151936, 2048, L.EPI_STORE),
                 ("draft_qkv", 64, 1152, 896, L.EPI_BIAS), ("draft_o_proj", 64, 896, 896, L.EPI_RESIDUAL),
                 ("draft_gate_up", 64, 9728, 896, L.EPI_SILU_MUL), ("draft_down", 64, 896, 4864, L.EPI_RESIDUAL),
                 ("draft_lm_head", 64, 151936, 896, L.EPI_STORE),
                 # the prompt pass fused into the first verify (64 requests x 132 rows)
                 ("prefill_qkv", 8448, 2560, 2048, L.EPI_BIAS), ("prefill_o_proj", 8448, 2048, 2048, L.EPI_RESIDUAL),
                 ("prefill_gate_up", 8448, 22016, 2048, L.EPI_SILU_MUL),
                 ("prefill_down", 8448, 2048, 11008, L.EPI_RESIDUAL),
                 # the draft's prompt pass (64 requests x 128 rows)
                 ("prefill_draft_down", 8192, 896, 4864, L.EPI_RESIDUAL))
        for name, m, n, k, epi in cases:
            if args.gemm_case and name not in args.gemm_case.split(","):
                continue
            x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            copies = max(1, -(-2 * L2_BYTES // (n * k * 2)))  # cold weights on every call
            wts = [(torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16) for _ in range(copies)]
            n_out = n // 2 if epi == L.EPI_SILU_MUL else n
            y = torch.randn(m, n_out, device=dev, generator=g).to(torch.bfloat16)
            bias = torch.randn(n, device=dev, generator=g) if epi == L.EPI_BIAS else None
            res = y if epi == L.EPI_RESIDUAL else None  # in place, as the forward pass does
            ms = _time_launches([(lambda wt=wt: ops.gemm(x, wt, epilogue=epi, bias=bias, residual=res, out=y))
                                 for wt in wts], args.steps)
            bts = (n * k + m * k + m * n_out * (2 if res is not None else 1)) * 2
            fl = 2.0 * m * n * k
            out.append({"micro": f"gemm_tcgen05 {name}", "m": m, "n": n, "k": k, "ms": round(ms, 4),
                        "weight_copies": copies,
                        "gbs": round(bts / ms / 1e6, 1), "frac_hbm": round(bts / ms / 1e6 / pk["hbm_gbs"], 4),
                        "tflops": round(fl / ms / 1e9, 1), "frac_tensor": round(fl / ms / 1e9 / pk["bf16_tflops"], 4)})
            del wts
    for line in out:
        print(json.dumps(line), flush=True)


def run_profile_iteration(args):
    """Warm up on the benchmark workload, then run exactly one steady-state spec
    iteration between cudaProfilerStart/Stop (for `ncu --profile-from-start off`)."""
    from kvengine_b200 import Model, PagedKVCache, SpecEngine
    from kvengine_b200.config import QWEN2_0_5B, QWEN2_3B
    from kvengine_b200.speculative import _Request
    from kvengine_b200.workloads import random_prompts

    dev = torch.device("cuda", 0)
    draft = Model.random_init(QWEN2_0_5B, seed=1, dtype=torch.bfloat16, device=dev, init_device=dev)
    target = Model.random_init(QWEN2_3B, seed=2, dtype=torch.bfloat16, device=dev, init_device=dev)
    prompts = random_prompts(N_REQ, PROMPT, seed=4).tolist()
    nb = N_REQ * (-(-(PROMPT + NEW + 2 * K_SPEC + 2) // BLOCK)) + 64
    t_pool = PagedKVCache.for_model(target, num_blocks=nb, block_size=BLOCK)
    d_pool = PagedKVCache.for_model(draft, num_blocks=nb, block_size=BLOCK)
    eng = SpecEngine(target, draft, t_pool, d_pool, K_SPEC)
    reqs = [_Request(p, t_pool.new_sequence(f"t{i}"), d_pool.new_sequence(f"d{i}"), NEW)
            for i, p in enumerate(prompts)]
    for _ in range(4):  # prefill-fused first iteration + 3 steady iterations
        eng.step(reqs, set())
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    eng.step(reqs, set())
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"profiled": "one steady-state spec iteration", "requests": N_REQ, "k": K_SPEC}))


def run_profile_verify_small(args):
    """A small case of the verify pass for per-kernel DRAM counter captures: the two-layer
    models with the benchmark's layer shapes (3B-shape target, 0.5B-shape draft, bf16,
    full vocabulary; about 1.2 GB on the device), the benchmark's batch (64 requests x 128
    prompt ids, k = 4, block size 16); after the prefill-fused first iteration and 3
    steady ones, exactly one steady verify pass runs between cudaProfilerStart/Stop.
    Every per-layer kernel of the 36-layer pass appears here with the same grid and
    shape, so its per-launch traffic scales to the full pass by the layer count."""
    from kvengine_b200 import Model, PagedKVCache, SpecEngine
    from kvengine_b200.config import QWEN2_0_5B_L2, QWEN2_3B_L2
    from kvengine_b200.speculative import _Request
    from kvengine_b200.workloads import random_prompts

    dev = torch.device("cuda", 0)
    draft = Model.random_init(QWEN2_0_5B_L2, seed=1, dtype=torch.bfloat16, device=dev, init_device=dev)
    target = Model.random_init(QWEN2_3B_L2, seed=2, dtype=torch.bfloat16, device=dev, init_device=dev)
    prompts = random_prompts(N_REQ, PROMPT, seed=4).tolist()
    nb = N_REQ * (-(-(PROMPT + NEW + 2 * K_SPEC + 2) // BLOCK)) + 64
    t_pool = PagedKVCache.for_model(target, num_blocks=nb, block_size=BLOCK)
    d_pool = PagedKVCache.for_model(draft, num_blocks=nb, block_size=BLOCK)
    eng = SpecEngine(target, draft, t_pool, d_pool, K_SPEC)
    reqs = [_Request(p, t_pool.new_sequence(f"t{i}"), d_pool.new_sequence(f"d{i}"), NEW)
            for i, p in enumerate(prompts)]
    for _ in range(4):
        eng.step(reqs, set())
    torch.cuda.synchronize()
    orig = eng.tr.forward

    def profiled(*a, **kw):
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        orig(*a, **kw)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()

    eng.tr.forward = profiled
    eng.step(reqs, set())
    torch.cuda.synchronize()
    print(json.dumps({"profiled": "one steady verify pass, two-layer 3B-shape target", "requests": N_REQ,
                      "k": K_SPEC}))


def run_serve(args):
    """Config 5: continuous-batching spec decode over a lognormal request mix
    (prompt mean 128, output mean 64, sigma 0.7, uniform tokens), requests sharded
    over the ranks in longest-processing-time order by prompt + output length
    (`kvengine_b200.distributed.shard_requests`), `--serve N` requests
    in total. 0.5B-arch draft -> 3B-arch target, or with --self-draft the 3B target
    as its own draft (full acceptance). One timed pass over the whole mix."""
    import torch.distributed as dist

    from kvengine_b200 import Model, PagedKVCache, SpecServer
    from kvengine_b200.config import QWEN2_0_5B, QWEN2_3B
    from kvengine_b200.workloads import lognormal_requests

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=600))
    target = Model.random_init(QWEN2_3B, seed=2, dtype=torch.bfloat16, device=dev, init_device=dev)
    draft = target if args.self_draft else Model.random_init(QWEN2_0_5B, seed=1, dtype=torch.bfloat16, device=dev,
                                                             init_device=dev)
    from kvengine_b200.distributed import shard_requests

    everything = lognormal_requests(args.serve, seed=5)
    mine = shard_requests([len(p) + o for p, o in everything], world)[rank]
    mix = [everything[i] for i in mine]
    blocks = args.serve_blocks
    t_pool = PagedKVCache.for_model(target, num_blocks=blocks, block_size=BLOCK)
    d_pool = PagedKVCache.for_model(draft, num_blocks=blocks, block_size=BLOCK)

    def serve(reqs):
        srv = SpecServer(target, draft, t_pool, d_pool, k=K_SPEC, max_batch=args.serve_batch, eos_token_id=None)
        for p, n in reqs:
            srv.add_request(p, n)
        srv.run()
        return srv

    serve(mix[: min(len(mix), 2 * args.serve_batch)])  # warm-up: kernels, plans, allocator caches
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    srv = serve(mix)
    ev1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([ev0.elapsed_time(ev1)], device=dev)
    tok = torch.tensor([float(srv.stats.new_tokens)], device=dev)
    drafted = sum(r.tokens_drafted for r in srv.results.values())
    accepted = sum(r.tokens_accepted for r in srv.results.values())
    acc = torch.tensor([float(drafted), float(accepted)], device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(tok, op=dist.ReduceOp.SUM)
        dist.all_reduce(acc, op=dist.ReduceOp.SUM)
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": f"accepted tokens/s (config 5, continuous batching, k={K_SPEC})",
            "value": round(float(tok.item()) / (float(ms.item()) / 1e3), 2), "unit": "accepted tokens/s",
            "n_gpus": world, "higher_is_better": True, "scaling": "strong",
            "ms_total": round(float(ms.item()), 1), "new_tokens": int(tok.item()),
            "acceptance_rate": round(float(acc[1].item() / acc[0].item()), 4) if acc[0].item() else None,
            "config": {"workload": "config 5: lognormal prompts (mean 128) and outputs (mean 64), sigma 0.7",
                       "requests": args.serve, "draft": "3B target (self)" if args.self_draft else "0.5B-arch seed 1",
                       "target": "3B-arch seed 2", "max_batch_per_gpu": args.serve_batch,
                       "kv_blocks_per_pool": blocks, "block_size": BLOCK},
            "server": {"steps": srv.stats.steps, "admitted": srv.stats.admitted, "preempted": srv.stats.preempted,
                       "peak_running": srv.stats.peak_running,
                       "prefix_tokens_reused": srv.stats.prefix_tokens_reused},
            "dtype": "bf16", "data": "synthetic (seeded random ids, random-init weights)"}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="kvengine_b200", choices=["kvengine_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--micro", default=None, help="comma list of accept,attention,attention_decode,gemm microbenchmarks")
    ap.add_argument("--gemm-case", default=None, help="restrict --micro gemm to these shapes (comma list)")
    ap.add_argument("--profile-iteration", action="store_true")
    ap.add_argument("--profile-verify-small", action="store_true",
                    help="one steady verify pass of two-layer benchmark-shape models (for counter captures)")
    ap.add_argument("--serve", type=int, default=0, help="config 5: continuous batching over this many requests")
    ap.add_argument("--serve-batch", type=int, default=128, help="running requests per GPU (--serve)")
    ap.add_argument("--serve-blocks", type=int, default=8192, help="KV blocks per pool (--serve)")
    ap.add_argument("--self-draft", action="store_true", help="--serve with the target as its own draft")
    ap.add_argument("--k", type=int, default=4, help="draft tokens per iteration (config 4 sweeps 1, 2, 4, 8)")
    args = ap.parse_args()
    global K_SPEC
    K_SPEC = args.k
    if args.warmup < 3:
        args.warmup = 3
    if args.micro:
        run_micro(args)
    elif args.profile_iteration:
        run_profile_iteration(args)
    elif args.profile_verify_small:
        run_profile_verify_small(args)
    elif args.serve:
        run_serve(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
