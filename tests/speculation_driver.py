"""A seeded decode session driving a speculation policy, for parity of the
adaptive-depth policy with the reference (moe_prefetch/speculative.py:39-77).

Used by tests/golden/make_golden.py on the reference's AdaptiveSpeculationPolicy
and by tests/test_speculation_golden.py on yanah_b200.speculation's. Step
times follow a simple cost model (a plain step costs ~1; a draft round of depth
d costs ~1 + 0.35 d and emits 1 + the accepted drafts), with noise, so the
policy calibrates, halves its depth and, in some sessions, stops.
"""
from __future__ import annotations

import numpy as np


def drive_policy(policy_cls, seed: int, max_depth: int, accept_p: float, draft_cost: float, rounds: int = 400):
    rng = np.random.default_rng(seed)
    pol = policy_cls(max_depth)
    ctx, log = 10, []
    for _ in range(rounds):
        act = pol.action(ctx)
        if act in ("calibrate", "plain"):
            t = 1.0 + 0.05 * rng.standard_normal()
            pol.observe_plain(t, ctx)
            ctx += 1
            log.append([str(act), round(t, 12), 1, pol.depth, int(pol.stopped)])
        else:
            d = int(act)
            acc = 0
            while acc < d and rng.random() < accept_p:
                acc += 1
            emitted = acc + 1
            t = 1.0 + draft_cost * d + 0.05 * rng.standard_normal()
            pol.observe_draft(t, emitted)
            ctx += emitted
            log.append([d, round(t, 12), emitted, pol.depth, int(pol.stopped)])
    return log
