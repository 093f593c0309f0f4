"""Adaptive speculation depth against the reference's own policy.

Fixture (tests/golden/speculation.json, written by tests/golden/make_golden.py):
the reference AdaptiveSpeculationPolicy (moe_prefetch/speculative.py:39-77)
driven through seeded decode sessions by tests/speculation_driver.py. The same
driver runs yanah_b200.speculation's policy; every action, depth and stop flag
must match.
"""
from __future__ import annotations

import json
from pathlib import Path

import pytest

from tests.speculation_driver import drive_policy
from yanah_b200.speculation import CALIBRATE, PLAIN, AdaptiveSpeculationPolicy

SESSIONS = json.loads((Path(__file__).resolve().parent / "golden" / "speculation.json").read_text())["sessions"]


@pytest.mark.parametrize("i", range(len(SESSIONS)))
def test_policy_matches_reference(i):
    s = SESSIONS[i]
    log = drive_policy(AdaptiveSpeculationPolicy, *s["args"])
    assert log == s["log"]


def test_policy_paths_covered():
    kinds = set()
    for s in SESSIONS:
        depths = [r[3] for r in s["log"]]
        if any(b < a for a, b in zip(depths, depths[1:])):
            kinds.add("halved")
        if s["log"][-1][4]:
            kinds.add("stopped")
        else:
            kinds.add("kept drafting")
        if sum(r[0] == "calibrate" for r in s["log"]) > 3:
            kinds.add("recalibrated")
    assert kinds == {"halved", "stopped", "kept drafting", "recalibrated"}


def test_depth_clamp_and_constants():
    assert AdaptiveSpeculationPolicy(0).depth == 1
    assert AdaptiveSpeculationPolicy(40).depth == 16
    assert (CALIBRATE, PLAIN) == ("calibrate", "plain")
