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
