"""Host-side pass plans (CPU): the vectorised plan builder and the verify feed
layout the spec engine uploads, against direct per-sequence constructions."""

import random

import numpy as np

from kvengine_b200.model import ForwardPlan, SeqSpec, block_tables
from kvengine_b200.speculative import verify_feed


class _Seq:
    def __init__(self, blocks):
        self.blocks = blocks


def test_from_arrays_equals_per_sequence_plan():
    rng = random.Random(3)
    for bs in (1, 4, 16):
        for _ in range(40):
            S = rng.randint(1, 9)
            specs = []
            for _ in range(S):
                start = rng.randint(0, 300)
                q = rng.choice([1, 1, 2, 5, rng.randint(1, 40)])
                nb = -(-(start + q) // bs) + rng.randint(0, 2)
                specs.append(SeqSpec(start, q, [rng.randrange(5000) for _ in range(nb)], rng.randint(1, q)))
            ref = ForwardPlan(specs, bs)
            tables, nb = block_tables([_Seq(s.blocks) for s in specs])
            got = ForwardPlan.from_arrays(np.array([s.start for s in specs]), np.array([s.q_len for s in specs]),
                                          np.array([s.n_out for s in specs]), tables, nb, bs)
            assert np.array_equal(got.host, ref.host) and got.offsets == ref.offsets
            assert (got.n_seqs, got.n_tokens, got.n_out, got.max_q_len, got.max_ctx, got.width) == \
                (ref.n_seqs, ref.n_tokens, ref.n_out, ref.max_q_len, ref.max_ctx, ref.width)


def test_verify_feed_layout():
    """Unseen tokens then k draft slots per request (kvengine speculative.py:160-162)."""
    rng = random.Random(5)
    for k in (1, 2, 4, 8):
        toks = [[rng.randrange(100) for _ in range(rng.randint(1, 30))] for _ in range(7)]
        u_t = np.array([rng.randint(1, len(t)) for t in toks])
        ids, dst = verify_feed(toks, u_t, k)
        want, slots = [], []
        for t, u in zip(toks, u_t.tolist()):
            want.extend(t[len(t) - u:])
            slots.append(list(range(len(want), len(want) + k)))
            want.extend([0] * k)
        assert ids.tolist() == want
        assert dst.shape == (k, len(toks)) and dst.T.tolist() == slots


def test_device_built_plan_layout_equals_host_layout():
    """The packed layout a device-side planner writes (ForwardPlan.device_built) is
    the one the host builder gives a pass of `rows` rows per sequence with the last
    row's logits wanted: same offsets, sizes and shape fields."""
    rng = random.Random(11)
    for rows in (1, 2):
        for _ in range(20):
            S, bs = rng.randint(1, 70), rng.choice([1, 3, 16])
            start = np.array([rng.randint(rows, 400) for _ in range(S)]) - (rows - 1)
            nb = (start + rows + bs - 1) // bs + np.array([rng.randint(0, 2) for _ in range(S)])
            width = int(nb.max())
            tables = np.zeros((S, width), dtype=np.int64)
            tables[np.arange(width) < nb[:, None]] = [rng.randrange(9000) for _ in range(int(nb.sum()))]
            host = ForwardPlan.from_arrays(start, np.full(S, rows), np.ones(S, dtype=np.int64), tables, nb, bs)
            dev = ForwardPlan.device_built(S, rows, width, host.max_ctx, bs)
            assert dev.offsets == host.offsets and dev.size == host.host.shape[0]
            assert (dev.n_seqs, dev.n_tokens, dev.n_out, dev.max_q_len, dev.max_ctx, dev.width) == \
                (host.n_seqs, host.n_tokens, host.n_out, host.max_q_len, host.max_ctx, host.width)
