"""Record writer against the reference's own output.

Fixture (tests/golden/repack.json, written by tests/golden/make_golden.py):
the reference repack (moe_prefetch/repack.py) run on the tiny seeded
checkpoints of tests/repack_driver.py. For uniform stacks the experts.bin
written here must have the same SHA-256 and experts.json the same text. The
mixed-bit checkpoint, which the reference rejects, is checked record by record
against the shards themselves.
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import numpy as np
import pytest

from tests.repack_driver import CASES, expected_records, write_checkpoint
from yanah_b200.formats import PAGE
from yanah_b200.repack import FileHostTier, read_specs, repack

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "repack.json").read_text())


@pytest.mark.parametrize("case", ["uniform4_mtp", "uniform2_g32"])
def test_uniform_stack_matches_reference(case, tmp_path):
    model, out = str(tmp_path / "model"), str(tmp_path / "out")
    write_checkpoint(model, case)
    repack(model, out)
    data = (tmp_path / "out" / "experts.bin").read_bytes()
    ref = GOLDEN[case]
    assert len(data) == ref["bytes"]
    assert hashlib.sha256(data).hexdigest() == ref["sha256"]
    assert (tmp_path / "out" / "experts.json").read_text() == ref["json"]


def test_mixed_bit_stack(tmp_path):
    assert GOLDEN["mixed42"]["error"] == "ValueError"   # the reference's writer stops here
    case = "mixed42"
    bits, gs, H, I, E, mtp, _ = CASES[case]
    model, out = str(tmp_path / "model"), str(tmp_path / "out")
    write_checkpoint(model, case)
    specs = repack(model, out)
    assert [s.bits for s in specs] == list(bits)
    specs2, slot = read_specs(out)
    assert [s.to_json() for s in specs2] == [s.to_json() for s in specs]
    assert slot == max(s.slot_bytes for s in specs) and slot % PAGE == 0
    data = (tmp_path / "out" / "experts.bin").read_bytes()
    assert len(data) == len(bits) * E * slot
    want = expected_records(model, range(len(bits)), len(bits), E)
    for (l, e), rec in want.items():
        o = (l * E + e) * slot
        assert data[o:o + len(rec)] == rec, (l, e)
        assert not any(data[o + len(rec):o + slot]), (l, e)   # zero padding
    meta = json.loads((tmp_path / "out" / "experts.json").read_text())
    assert len(meta["layers"]) == len(bits) and meta["stack_slot_bytes"] == slot


def test_file_host_tier(tmp_path):
    case = "uniform4_mtp"
    bits, gs, H, I, E, mtp, _ = CASES[case]
    model, out = str(tmp_path / "model"), str(tmp_path / "out")
    write_checkpoint(model, case)
    repack(model, out)
    tier = FileHostTier(out, layers=[0, 2], pin=False)   # layer 2 is the MTP layer
    want = expected_records(model, [0, 2], len(bits) - 1, E)
    for (l, e), rec in want.items():
        o = e * tier.rec[l]
        assert tier.buf[l][o:o + len(rec)].numpy().tobytes() == rec, (l, e)
    assert tier.nbytes == 2 * E * tier.slot
