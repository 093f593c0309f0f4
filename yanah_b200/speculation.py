"""Adaptive draft depth for self-speculative decoding
(moe_prefetch/speculative.py:39-77 `AdaptiveSpeculationPolicy`).

The policy decides, before each decode round, whether to run a plain
single-token step (to calibrate, or because speculation was switched off) or a
draft round of `depth` tokens, whose verify pass is the 1 + depth row batch
this library runs on the batch path (`ExpertParallelStack` with
`batch = 1 + depth`; `bench.py --workload verify` measures 1 + 4):

* calibrate on three plain steps (their step times);
* afterwards compare the median cost per emitted token of the last three
  draft rounds with the median of the three plain steps; when drafting is more
  than 5% slower, halve the depth (its draft history restarts), and at depth 1
  stop drafting for good;
* recalibrate (forget both histories) after 16 draft rounds or 256 tokens of
  context growth since the last plain step.

Depth starts at the requested maximum, clamped to [1, 16].
"""
from __future__ import annotations

from typing import List, Union

CALIBRATE = "calibrate"
PLAIN = "plain"


def _median3(v: List[float]) -> float:
    return sorted(v)[1]


class AdaptiveSpeculationPolicy:
    CALIBRATE, PLAIN = CALIBRATE, PLAIN

    def __init__(self, maximum_depth: int):
        self.depth = max(1, min(16, int(maximum_depth)))
        self.plain: List[float] = []     # the last (up to) three plain step times
        self.draft: List[float] = []     # the last (up to) three draft-round costs per emitted token
        self.stopped = False
        self.baseline_ctx = 0            # context length at the last plain step
        self.rounds_since = 0            # draft rounds since the last recalibration

    def action(self, ctx: int) -> Union[str, int]:
        """PLAIN, CALIBRATE, or the draft depth for a round at context length `ctx`."""
        if self.stopped:
            return PLAIN
        calibrated = len(self.plain) == 3
        if calibrated and (self.rounds_since >= 16 or ctx - self.baseline_ctx >= 256):
            self.plain, self.draft, self.rounds_since = [], [], 0
            calibrated = False
        return self.depth if calibrated else CALIBRATE

    def observe_plain(self, seconds: float, ctx: int) -> None:
        self.plain = (self.plain + [seconds])[-3:]
        self.baseline_ctx = ctx

    def observe_draft(self, seconds: float, emitted: int) -> None:
        """A draft round took `seconds` and emitted `emitted` tokens (>= 1)."""
        self.rounds_since += 1
        self.draft = (self.draft + [seconds / emitted])[-3:]
        if len(self.draft) < 3 or len(self.plain) < 3:
            return
        if _median3(self.draft) > _median3(self.plain) * 1.05:
            if self.depth == 1:
                self.stopped = True
            else:
                self.depth = max(1, self.depth // 2)
                self.draft = []
