"""Routing traces and an orchestrator-like driver for slot-pool parity.

Used twice with the same inputs: by tests/golden/make_golden.py on the
reference's SlotPool / cache_sim (to write the fixtures) and by
tests/test_pool_golden.py on yanah_b200.pool (to compare).
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import numpy as np


def make_trace(rng, S: int, L: int, E: int, k: int, zipf: float = 1.1, p_repeat: float = 0.6,
               n_cand: int = 16, lookahead: int = 2):
    """Routed ids (S, L, k) with Zipf(zipf) popularity per layer (popularity
    ranks permuted per layer) where each of the k slots repeats the previous
    token's expert with probability p_repeat; per (step, layer) forecast
    candidates for the next `lookahead` layers: the top n_cand of a noisy
    softmax that favours the experts that layer will route."""
    pop = 1.0 / np.arange(1, E + 1) ** zipf
    pop /= pop.sum()
    perms = [rng.permutation(E) for _ in range(L)]
    routed = np.zeros((S, L, k), np.int64)
    for s in range(S):
        for l in range(L):
            chosen: List[int] = []
            for j in range(k):
                prev = int(routed[s - 1, l, j]) if s else -1
                if prev >= 0 and prev not in chosen and rng.random() < p_repeat:
                    chosen.append(prev)
                    continue
                while True:
                    e = int(perms[l][rng.choice(E, p=pop)])
                    if e not in chosen:
                        chosen.append(e)
                        break
            routed[s, l] = chosen
    fc: List[List[Dict[int, List[Tuple[int, float]]]]] = [[{} for _ in range(L)] for _ in range(S)]
    for s in range(S):
        for l in range(L):
            for t in range(l + 1, min(L, l + 1 + lookahead)):
                logit = np.log(pop[np.argsort(perms[t])]) + rng.normal(0.0, 1.0, E)
                logit[routed[s, t]] += 2.0
                p = np.exp(logit - logit.max())
                p = (p / p.sum()).astype(np.float32)
                top = np.argsort(-p, kind="stable")[:n_cand]
                fc[s][l][t] = [(int(e), float(p[e])) for e in top]
    return routed, fc


def fc_to_arrays(fc):
    rows = [(s, l, t, e, p) for s, per in enumerate(fc) for l, d in enumerate(per) for t, c in d.items() for e, p in c]
    a = np.array(rows, dtype=np.float64) if rows else np.zeros((0, 5))
    return {"fc_step": a[:, 0].astype(np.int32), "fc_layer": a[:, 1].astype(np.int16),
            "fc_target": a[:, 2].astype(np.int16), "fc_expert": a[:, 3].astype(np.int16),
            "fc_prob": a[:, 4].astype(np.float32)}


def fc_from_arrays(z, S: int, L: int):
    fc = [[{} for _ in range(L)] for _ in range(S)]
    for s, l, t, e, p in zip(z["fc_step"], z["fc_layer"], z["fc_target"], z["fc_expert"], z["fc_prob"]):
        fc[int(s)][int(l)].setdefault(int(t), []).append((int(e), float(p)))
    return fc


class NullMemory:
    def views(self, i):
        return []

    def close(self):
        pass


def drive_slot_pool(pool, routed, fc, threshold: float = 0.062, issue_cap: int = 32):
    """Orchestrator-like use of a SlotPool: per (step, layer) the routed
    experts are hit, adopted (a completed forecast) or claimed and published,
    then unpinned; forecasts are reserved for the target layers and returned
    when their target layer has passed; every forecast is returned at the end
    of a token. Returns the log of slot decisions (encoded ints)."""
    S, L = routed.shape[0], routed.shape[1]
    log: List[int] = []
    tickets: Dict[Tuple[int, int], int] = {}
    for s in range(S):
        for l in range(L):
            pool.drain_returned()
            out, misses = {}, []
            for e in sorted({int(x) for x in routed[s, l]}):
                key = (l, e)
                slot = pool.hit(key)
                if slot is not None:
                    out[e] = slot
                    log.append(slot)
                    continue
                t = tickets.pop(key, None)
                if t is not None:
                    pool.adopt(t, key)
                    out[e] = t
                    log.append(1_000_000 + t)
                    continue
                slot = pool.claim_for_demand(key)
                out[e] = slot
                misses.append(e)
                log.append(2_000_000 + slot)
            for e in misses:
                pool.publish(out[e], (l, e))
            for slot in out.values():
                pool.unpin(slot)
            for target, cands in fc[s][l].items():
                n = 0
                for e, p in sorted(cands, key=lambda c: -c[1]):
                    if p < threshold or (target, e) in tickets:
                        continue
                    if n >= issue_cap:
                        break
                    r = pool.reserve_speculative((target, e))
                    if r is None:
                        log.append(-1)
                        continue
                    tickets[(target, e)] = r
                    log.append(3_000_000 + r)
                    n += 1
            for key in [kk for kk in tickets if kk[0] <= l]:
                pool.return_speculative(tickets.pop(key))
        for key in list(tickets):
            pool.return_speculative(tickets.pop(key))
    pool.drain_returned()
    return log


def stats_tuple(st) -> List[int]:
    return [st.hits, st.misses, st.evictions, st.adopted, st.spec_reserved, st.spec_discarded, st.spec_refused,
            st.adopt_evictions, st.admitted]
