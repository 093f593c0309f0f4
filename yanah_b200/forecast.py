"""Lookahead candidate selection (host side of the two-layer forecast).

The device computes, in the same pass as routing, each target layer's
probabilities softmax(router_t(RMSNorm_t(h))) taken as a max over rows
(``yn_post_attention`` with targets). This class turns those (E,) vectors
into the candidate list the prefetcher issues, and keeps recall statistics,
as ``RouterForecast`` in backend mode does in moe_prefetch/predictor.py:49-125
(``select`` :100-111, ``observe`` :113-118, stats :37-47).

Selection order: the `top` largest probabilities by numpy's introselect
(`argpartition`), then ordered by descending probability with numpy's
default sort. Equal probabilities are common (router logits are bf16 before
the softmax), and these two calls fix their order exactly as the reference's
selection does, so the candidate lists match element for element.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Set, Tuple

import numpy as np


@dataclass
class ForecastStats:
    forecasts: int = 0
    candidates: int = 0
    actual: int = 0
    covered: int = 0   # routed experts that had been forecast for their layer

    @property
    def recall(self) -> float:
        return self.covered / max(1, self.actual)


class RouterForecast:
    def __init__(self, geometry=None):
        self.g = geometry
        self._pending: Dict[int, Set[int]] = {}
        self.stats = ForecastStats()

    def select(self, target_layer: int, score: np.ndarray, top: int = 24) -> List[Tuple[int, float]]:
        """The `top` most probable experts of `target_layer` as (id, prob).

        Every forecast made for a layer before it is routed joins one pending
        set (a layer is forecast from two layers back and again from one)."""
        score = np.asarray(score)
        k = min(int(top), score.shape[0])
        if k <= 0:
            return []
        neg = -score
        # numpy's argpartition (introselect) and default argsort, as the array methods the module functions call
        part = neg.argpartition(k - 1)[:k]              # the k most probable, in no particular order
        order = part[neg[part].argsort()]               # most probable first; ties as numpy's sort leaves them
        ids = order.tolist()
        out = list(zip(ids, score[order].astype(np.float64).tolist()))
        self._pending.setdefault(target_layer, set()).update(ids)
        self.stats.forecasts += 1
        self.stats.candidates += len(out)
        return out

    def observe(self, layer: int, routed: np.ndarray) -> None:
        """Score the pending forecast of `layer` against the experts it routed."""
        actual = set(np.asarray(routed).ravel().tolist())
        pred = self._pending.pop(layer, None)
        if pred is None:
            return
        self.stats.actual += len(actual)
        self.stats.covered += len(actual & pred)

    def reset(self) -> None:
        self._pending.clear()
