"""Greedy speculative decoding with draft, verify and accept on the device.

Same API and result type as kvengine/speculative.py:53-216:
`speculative_greedy(target_model, draft_model, input_ids, target_cache,
draft_cache, k=4, max_new_tokens=32, eos_token_id=AUTO_EOS) -> SpecDecodeResult`,
with identical bookkeeping (u unseen target tokens + k drafts fed in one
verify pass, rows u-1 .. u-1+k predict drafts[0..k-1] and the bonus, the
longest matching prefix is accepted and the first disagreement resolved in
the target's favour, both caches truncated to len(tokens)-1, trims at EOS and
at the budget).

What differs is where it runs. `speculative_greedy_batch` advances many
requests together: per iteration one ragged draft pass (each request's unseen
tokens), k-1 one-token draft passes whose inputs are the previous argmax
kernel's outputs (no host sync between draft tokens), one verify pass over
B*(u+k) rows, and the fused accept kernel. The host sees one small
device->host copy per iteration (accepted counts and emitted tokens) and
does the block-table bookkeeping. `speculative_greedy` is the batch of one.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from itertools import chain

import numpy as np
import torch

from . import ops
from .decode import AUTO_EOS, _resolve_eos, _sync
from .forward import runner_for
from .model import ForwardPlan, as_model, block_tables


@dataclass
class SpecDecodeResult:
    prompt_token_ids: list[int]
    new_token_ids: list[int]
    elapsed_s: float
    stopped_on_eos: bool
    iterations: int = 0
    tokens_drafted: int = 0
    tokens_accepted: int = 0
    accepted_per_iter: list[int] = field(default_factory=list)
    target_forwards: int = 0
    draft_forwards: int = 0

    @property
    def tokens_per_s(self) -> float:
        return len(self.new_token_ids) / self.elapsed_s if self.elapsed_s else 0.0

    @property
    def acceptance_rate(self) -> float:
        return self.tokens_accepted / self.tokens_drafted if self.tokens_drafted else 0.0

    @property
    def tokens_per_target_forward(self) -> float:
        return len(self.new_token_ids) / self.target_forwards if self.target_forwards else 0.0

    def summary(self) -> dict:
        return {
            "new_tokens": len(self.new_token_ids),
            "elapsed_s": round(self.elapsed_s, 3),
            "tokens_per_s": round(self.tokens_per_s, 2),
            "iterations": self.iterations,
            "tokens_drafted": self.tokens_drafted,
            "tokens_accepted": self.tokens_accepted,
            "acceptance_rate": round(self.acceptance_rate, 4),
            "tokens_per_target_forward": round(self.tokens_per_target_forward, 3),
            "target_forwards": self.target_forwards,
            "draft_forwards": self.draft_forwards,
            "stopped_on_eos": self.stopped_on_eos,
        }


class _Request:
    __slots__ = ("tokens", "t_seq", "d_seq", "res", "max_new", "done", "u_d", "u_t")

    def __init__(self, prompt, t_seq, d_seq, max_new):
        self.tokens = list(prompt)
        self.t_seq = t_seq
        self.d_seq = d_seq
        self.res = SpecDecodeResult(list(prompt), [], 0.0, False)
        self.max_new = max_new
        self.done = max_new <= 0
        self.u_d = self.u_t = 0


def verify_feed(token_lists: list[list[int]], u_t: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """The verify pass's token ids and where the drafts go in them.

    Request i feeds its last u_t[i] tokens (the ones the target has not seen)
    followed by its k drafts, as kvengine/speculative.py:160-162 builds
    `unseen + drafts`. Returns the int32 ids with zeros in the draft slots and
    dst [k, S] int32: draft j of request i goes to ids[dst[j, i]]."""
    S = len(token_lists)
    u_t = np.asarray(u_t, dtype=np.int64)
    v_len = u_t + k
    v_off = np.zeros(S + 1, dtype=np.int64)
    np.cumsum(v_len, out=v_off[1:])
    seq_of = np.repeat(np.arange(S), v_len)
    unseen = (np.arange(int(v_off[-1])) - v_off[:-1][seq_of]) < u_t[seq_of]
    v_ids = np.zeros(int(v_off[-1]), dtype=np.int32)
    v_ids[unseen] = np.fromiter(chain.from_iterable(t[len(t) - u:] for t, u in zip(token_lists, u_t.tolist())),
                                dtype=np.int32, count=int(u_t.sum()))
    dst = ((v_off[:-1] + u_t)[None, :] + np.arange(k)[:, None]).astype(np.int32)
    return v_ids, dst


class SpecEngine:
    """Batched draft/verify/accept loop over one target and one draft model."""

    def __init__(self, target, draft, target_pool, draft_pool, k: int, graphs: bool = True,
                 eager_layers: int | None = None, speculate: bool = True):
        assert k >= 1, "k must be at least 1"
        self.target = as_model(target)
        self.draft = as_model(draft)
        if self.target.cfg.vocab_size != self.draft.cfg.vocab_size:
            raise ValueError("draft and target must share a vocabulary")
        self.k = k
        self.t_pool, self.d_pool = target_pool, draft_pool
        self.tr = runner_for(self.target, target_pool)
        self.dr = runner_for(self.draft, draft_pool)
        self.device = self.target.device
        self.V = self.target.cfg.vocab_size
        self._cap = 0
        self.stats = {"iterations": 0, "verify_rows": 0, "h2d_bytes": 0, "d2h_bytes": 0}
        self._pinned: list[torch.Tensor | None] = []
        # When a list, every verify pass appends (start_event, end_event, plan) so a
        # caller can time the verify step on the stream it runs on.
        self.verify_events: list | None = None
        # Steps run on the engine's own stream (ordered after, and followed by, the
        # caller's current stream), so that the draft passes and the verify pass can be
        # launched as CUDA graphs (the first layers of the first draft pass of a step stay
        # stream launches: the GPU waits on them, and recording would delay its first kernel).
        self.graphs = graphs
        self.stream = torch.cuda.Stream(device=self.device)
        # Layers of draft pass 0 launched before the rest is recorded: enough that
        # recording the rest ends before the GPU has run them (a quarter of the layers
        # measured best on config 4: 6 of 24; 7, 8, 10 and 12 were 0.2-0.5 % slower).
        # `eager_layers` overrides it: 0 records the whole pass, num_layers launches it all.
        n_layers = self.draft.cfg.num_layers
        self.eager0 = max(1, n_layers // 4) if eager_layers is None else min(max(int(eager_layers), 0), n_layers)
        # Speculative planning of the next step's first draft pass: after the accept
        # kernel the engine queues a device-side plan (kve_spec_next_draft_plan) and that
        # pass, so the GPU runs it while the host reads the accept result back and does
        # its bookkeeping. One row per sequence (exact unless a sequence accepted all k
        # drafts) while the previous step saw no full acceptance, two rows (exact for
        # every outcome) otherwise. The next step uses the pass if its request list is
        # the one planned for and every request's draft feed matches; else it is
        # discarded (its K/V writes land only past each draft's committed prefix).
        self.speculate = speculate
        self._spec = None
        self._saw_full_accept = False
        self.spec_stats = {"planned": 0, "used": 0, "discarded": 0}

    def _ensure(self, S: int):
        if S <= self._cap:
            return
        dev, k = self.device, self.k
        self._cap = S
        self.dlog = torch.empty(S, self.V, dtype=self.draft.dtype, device=dev)
        self.tlog = torch.empty(S * (k + 1), self.V, dtype=self.target.dtype, device=dev)
        self.drafts = torch.empty(k, S, dtype=torch.int32, device=dev)
        self.accept_ws = ops.Workspace(dev)
        self.preds = torch.empty(S * (k + 1), dtype=torch.int32, device=dev)
        # emitted [S, k+1] then n_accepted [S]: read back by one copy
        self.accepted = torch.empty(S * (k + 2), dtype=torch.int32, device=dev)
        self.accepted_host = torch.empty(S * (k + 2), dtype=torch.int32, pin_memory=True)
        self.accepted_ready = torch.cuda.Event()
        # speculated first draft pass: its token ids (up to 2 rows per sequence), the
        # next verify feed (bonus + k drafts per sequence) and where draft j goes in it
        self.spec_ids = torch.empty(2 * S, dtype=torch.int32, device=dev)
        self.spec_vids = torch.zeros(S * (k + 1), dtype=torch.int32, device=dev)
        self.spec_dst = (torch.arange(S, dtype=torch.int32)[None, :] * (k + 1) + 1
                         + torch.arange(k, dtype=torch.int32)[:, None]).to(dev).contiguous()
        self.spec_plans = [torch.empty(0, dtype=torch.int32, device=dev) for _ in range(2)]
        self._spec_flip = 0

    def _upload(self, slot: int, arrays: list[np.ndarray]) -> list[torch.Tensor]:
        """Copy int32 host arrays to the device in one transfer through pinned
        staging buffer `slot` (the next iteration reuses it only after this one's
        readback, by which time the copy has run); returns device views."""
        offs = np.cumsum([0] + [a.shape[0] for a in arrays])
        n = int(offs[-1])
        buf = self._pinned[slot] if slot < len(self._pinned) else None
        if buf is None or buf.numel() < n:
            buf = torch.empty(max(n, 4096) * 2, dtype=torch.int32, pin_memory=True)
            while len(self._pinned) <= slot:
                self._pinned.append(None)
            self._pinned[slot] = buf
        host = buf.numpy()
        for a, lo in zip(arrays, offs[:-1]):
            host[lo:lo + a.shape[0]] = a
        dev = buf[:n].to(self.device, non_blocking=True)
        self.stats["h2d_bytes"] += n * 4
        return [dev[offs[i]:offs[i + 1]] for i in range(len(arrays))]

    def step(self, reqs: list[_Request], eos: set[int]) -> None:
        """One draft/verify/accept iteration for every request in `reqs`."""
        caller = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(caller)
        with torch.cuda.stream(self.stream):
            self._step(reqs, eos)
        caller.wait_stream(self.stream)

    def _step(self, reqs: list[_Request], eos: set[int]) -> None:
        k, S = self.k, len(reqs)
        self._ensure(S)
        spec, self._spec = self._spec, None
        # --- block reservation, in the reference's order: draft feeds, then the verify feed.
        lens = []
        for r in reqs:
            n = len(r.tokens)
            dl, tl = r.d_seq.length, r.t_seq.length
            r.u_d, r.u_t = n - dl, n - tl
            lens.append((dl, tl, n))
            r.d_seq.reserve(r.u_d + k - 1)
        d_len, t_len, n_tok = np.array(lens, dtype=np.int64).T
        u_d, u_t = n_tok - d_len, n_tok - t_len
        bs_d, bs_t = self.d_pool.block_size, self.t_pool.block_size
        ones = np.ones(S, dtype=np.int64)
        # One draft block table serves all k draft passes of the step (every slot they
        # write was reserved above).
        t_d, nb_d = block_tables([r.d_seq for r in reqs])
        # The first draft pass was queued by the previous step (planned on the device)
        # when it fed what this step's feed is: the same requests, every target feed the
        # bonus alone and every draft feed covered by the planned rows.
        use_spec = spec is not None and len(spec["reqs"]) == S and all(a is b for a, b in zip(spec["reqs"], reqs)) \
            and bool((u_t == 1).all()) and bool((u_d <= spec["rows"]).all()) and bool((n_tok - 1 < spec["cover"]).all())
        if spec is not None:
            self.spec_stats["used" if use_spec else "discarded"] += 1
        status = self.tr.status
        if use_spec:
            plan0 = spec["plan"]
            v_ids_dev = self.spec_vids[: S * (k + 1)]
            dst_dev = self.spec_dst[:, :S]
        else:
            plan0 = ForwardPlan.from_arrays(d_len, u_d, ones, t_d, nb_d, bs_d)
            # --- upload 1: the first draft pass's plan and ids, and the verify pass's token
            # ids with a slot per draft (the draft argmax kernels write the drafts there),
            # so the GPU starts while the host builds the other plans (the later uploads
            # queue behind that pass).
            d_ids = np.fromiter(chain.from_iterable(r.tokens[len(r.tokens) - r.u_d:] for r in reqs),
                                dtype=np.int32, count=int(u_d.sum()))
            v_ids, dst = verify_feed([r.tokens for r in reqs], u_t, k)
            (plan0_dev, d_ids_dev, v_ids_dev, dst_dev) = self._upload(0, [plan0.host, d_ids, v_ids,
                                                                           dst.reshape(-1)])
            dst_dev = dst_dev.view(k, S)
            # --- draft: k passes, argmax feeding the next pass on the device
            # Pass 0: the first draft layers as stream launches (the GPU is idle until they
            # arrive), the rest recorded into a graph while those run.
            self.dr.forward(plan0, d_ids_dev, self.dlog[:S], plan_dev=plan0_dev,
                            graph="draft0" if self.graphs else None, eager_layers=self.eager0)
            ops.argmax_rows(self.dlog[:S], out=self.drafts[0, :S], scatter_index=dst_dev[0], scatter_out=v_ids_dev,
                            status=status)
        v_len = u_t + k
        # The target reservations follow the draft ones with no allocator call in
        # between, as in the reference's order, while the first draft pass runs.
        for r in reqs:
            r.t_seq.reserve(r.u_t + k)
        gd = "draft" if self.graphs else None
        plans = [plan0]
        # Pass 1 goes first, with its own upload, so that it is recorded and launched
        # while the GPU still runs pass 0; the other plans are built while pass 1 runs.
        if k > 1:
            plans.append(ForwardPlan.from_arrays(d_len + u_d, ones, ones, t_d, nb_d, bs_d))
            (plan1_dev,) = self._upload(1, [plans[1].host])
            self.dr.forward(plans[1], self.drafts[0, :S], self.dlog[:S], plan_dev=plan1_dev, graph=gd)
            ops.argmax_rows(self.dlog[:S], out=self.drafts[1, :S], scatter_index=dst_dev[1], scatter_out=v_ids_dev,
                            status=status)
        for j in range(2, k):
            plans.append(ForwardPlan.from_arrays(d_len + u_d + j - 1, ones, ones, t_d, nb_d, bs_d))
        t_t, nb_t = block_tables([r.t_seq for r in reqs])
        vplan = ForwardPlan.from_arrays(t_len, v_len, np.full(S, k + 1, dtype=np.int64), t_t, nb_t, bs_t)
        # What the device needs to plan the next step's first draft pass: each request's
        # token count and last token at the start of this step, and its draft blocks (the
        # table two entries wider: a planned row may land up to two positions past them).
        last_tok = np.fromiter((r.tokens[-1] for r in reqs), dtype=np.int32, count=S)
        t_d2 = np.zeros((S, t_d.shape[1] + 2), dtype=np.int32)
        t_d2[:, : t_d.shape[1]] = t_d
        views = self._upload(2, [p.host for p in plans[2:]] + [vplan.host, n_tok.astype(np.int32), last_tok,
                                                               nb_d.astype(np.int32), t_d2.reshape(-1)])
        nv = len(plans) - 2 if k > 1 else 0
        vplan_dev = views[nv]
        spec_src = views[nv + 1:]
        for j in range(2, k):
            self.dr.forward(plans[j], self.drafts[j - 1, :S], self.dlog[:S], plan_dev=views[j - 2], graph=gd)
            ops.argmax_rows(self.dlog[:S], out=self.drafts[j, :S], scatter_index=dst_dev[j],
                            scatter_out=v_ids_dev, status=status)
        # --- verify: one target pass over every request's u+k rows
        drafts = self.drafts[:, :S]
        tlog = self.tlog[: S * (k + 1)]
        if self.verify_events is not None:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        self.tr.forward(vplan, v_ids_dev, tlog, plan_dev=vplan_dev, graph="verify" if self.graphs else None)
        if self.verify_events is not None:
            ev1.record()
            self.verify_events.append((ev0, ev1, vplan))
        # --- accept (fused argmax + prefix match + bonus)
        ne = S * (k + 1)
        out = (self.preds[:ne].view(S, k + 1), self.accepted[ne:ne + S], self.accepted[:ne].view(S, k + 1))
        ops.greedy_accept(tlog.view(S, k + 1, self.V), drafts.t(), self.accept_ws, out=out)
        # pinned readback, waited on by an event (no pageable staging, no device-wide sync)
        back_t = self.accepted_host[:ne + S]
        back_t.copy_(self.accepted[:ne + S], non_blocking=True)
        self.accepted_ready.record()
        if self.speculate:
            self._queue_next_draft_pass(reqs, n_tok, nb_d, t_d2.shape[1], spec_src, ne)
        self.accepted_ready.synchronize()
        back = back_t.numpy()
        n_host = back[ne:].tolist()
        em_host = back[:ne].reshape(S, k + 1).tolist()
        self._saw_full_accept = k in n_host
        self.stats["d2h_bytes"] += back.nbytes
        self.stats["iterations"] += 1
        self.stats["verify_rows"] += vplan.n_tokens
        for r, n, row in zip(reqs, n_host, em_host):
            em = row[: n + 1]
            res = r.res
            res.iterations += 1
            res.tokens_drafted += k
            res.tokens_accepted += n
            res.accepted_per_iter.append(n)
            res.draft_forwards += k
            res.target_forwards += 1
            r.tokens.extend(em)
            res.new_token_ids.extend(em)
            keep = len(r.tokens) - 1
            # target before draft: the order rejected blocks return to the free list
            r.t_seq.commit_and_keep(r.u_t + k, keep)
            r.d_seq.commit_and_keep(r.u_d + k - 1, keep)
            if eos and any(t in eos for t in em):
                first = next(j for j, t in enumerate(em) if t in eos)
                trim = len(em) - (first + 1)
                if trim:
                    res.new_token_ids = res.new_token_ids[:-trim]
                res.stopped_on_eos = True
                r.done = True
            elif len(res.new_token_ids) >= r.max_new:
                r.done = True

    def _queue_next_draft_pass(self, reqs, n_tok, nb_d, width, spec_src, ne) -> None:
        """Plan the next step's first draft pass on the device from this step's accept
        result and queue it (with its argmax) behind the accept readback. Skipped when
        a request is expected to finish (the next step's request list would differ)
        or the draft pool has no unused block for rows past a sequence's blocks."""
        k, S = self.k, len(reqs)
        rows = 2 if self._saw_full_accept else 1
        # A request expected to finish this step (it emits its previous step's accepted
        # count + 1 tokens, 1 on its first step) would change the next request list.
        if any(len(r.res.new_token_ids) + 1 + (r.res.accepted_per_iter[-1] if r.res.accepted_per_iter else 0)
               >= r.max_new for r in reqs):
            return
        dump = self.d_pool.manager.unused_block()
        if dump is None:
            return
        bs = self.d_pool.block_size
        desc = ForwardPlan.device_built(S, rows, width, int(n_tok.max()) + k + 1, bs)
        self._spec_flip ^= 1
        buf = self.spec_plans[self._spec_flip]
        if buf.numel() < desc.size:
            buf = self.spec_plans[self._spec_flip] = torch.empty(int(desc.size * 1.5) + 256, dtype=torch.int32,
                                                                 device=self.device)
        start, last, nblk, tables = spec_src
        ops.spec_next_draft_plan(start, last, nblk, tables, bs, k, rows, dump, self.accepted[ne:ne + S],
                                 self.accepted[:ne], buf, self.spec_ids, self.spec_vids[: S * (k + 1)],
                                 status=self.tr.status)
        self.dr.forward(desc, self.spec_ids[: rows * S], self.dlog[:S], plan_dev=buf,
                        graph="draft_spec" if self.graphs else None)
        ops.argmax_rows(self.dlog[:S], out=self.drafts[0, :S], scatter_index=self.spec_dst[0, :S],
                        scatter_out=self.spec_vids[: S * (k + 1)], status=self.tr.status)
        # the next step's last row must lie in the blocks this plan used
        self._spec = {"reqs": list(reqs), "rows": rows, "plan": desc, "cover": nb_d * bs}
        self.spec_stats["planned"] += 1

    def check(self) -> None:
        self.tr.check_status()
        self.dr.check_status()

    def run(self, reqs: list[_Request], eos: set[int], t0: float | None = None) -> None:
        t0 = time.perf_counter() if t0 is None else t0
        active = [r for r in reqs if not r.done]
        while active:
            self.step(active, eos)
            now = None
            for r in active:
                if r.done:
                    now = now or time.perf_counter()
                    r.res.elapsed_s = now - t0
            active = [r for r in active if not r.done]
        self.check()
        _sync(self.device)
        end = time.perf_counter()
        for r in reqs:
            if r.res.elapsed_s == 0.0:
                r.res.elapsed_s = end - t0
            new = r.res.new_token_ids
            if len(new) > r.max_new:
                r.res.new_token_ids = new[: r.max_new]
                r.res.stopped_on_eos = r.res.new_token_ids[-1] in eos if r.res.new_token_ids else False


@torch.no_grad()
def speculative_greedy(target_model, draft_model, input_ids: torch.Tensor, target_cache, draft_cache,
                       k: int = 4, max_new_tokens: int = 32, eos_token_id=AUTO_EOS) -> SpecDecodeResult:
    """Greedy speculative decoding of one request; output equals greedy decoding of the target."""
    assert input_ids.dim() == 2 and input_ids.shape[0] == 1, "one request at a time"
    assert k >= 1, "k must be at least 1"
    assert target_cache.length == 0 and draft_cache.length == 0, "caches must be empty"
    eos = _resolve_eos(target_model, eos_token_id)
    eng = SpecEngine(target_model, draft_model, target_cache.pool, draft_cache.pool, k)
    req = _Request(input_ids[0].tolist(), target_cache, draft_cache, max_new_tokens)
    _sync(eng.device)
    t0 = time.perf_counter()
    req.done = False
    if max_new_tokens <= 0:
        req.done = True
    eng.run([req], eos, t0)
    req.res.elapsed_s = time.perf_counter() - t0
    return req.res


@torch.no_grad()
def speculative_greedy_batch(target_model, draft_model, prompts: list[list[int]], target_pool, draft_pool,
                             k: int = 4, max_new_tokens=32, eos_token_id=AUTO_EOS,
                             free_on_finish: bool = True, engine: SpecEngine | None = None):
    """Batched greedy speculative decoding. `prompts`: list of token lists or a host
    int tensor [B, P]; `max_new_tokens`: an int or a per-request list.

    Returns (results, wall_seconds). Token output per request is identical to
    `speculative_greedy` on that request alone (greedy output depends only on
    the request's own tokens)."""
    eos = _resolve_eos(target_model, eos_token_id)
    if isinstance(prompts, torch.Tensor):
        prompts = prompts.tolist()
    eng = engine or SpecEngine(target_model, draft_model, target_pool, draft_pool, k)
    budgets = max_new_tokens if isinstance(max_new_tokens, (list, tuple)) else [max_new_tokens] * len(prompts)
    reqs = [_Request(p, target_pool.new_sequence(f"t{i}"), draft_pool.new_sequence(f"d{i}"), budgets[i])
            for i, p in enumerate(prompts)]
    _sync(eng.device)
    t0 = time.perf_counter()
    try:
        eng.run(reqs, eos, t0)
    finally:
        if free_on_finish:
            for r in reqs:
                r.t_seq.free()
                r.d_seq.free()
    wall = time.perf_counter() - t0
    return [r.res for r in reqs], wall
