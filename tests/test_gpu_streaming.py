"""Streaming decode (HBM slot pool + pinned host tier + forecast-driven
copies) against the all-resident decode: identical outputs, bit for bit, on
the same tokens (the same kernels run; only where the records sit and when
they arrive differs), with the pool and copy statistics consistent."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.gpu_helpers import bf16_dev, bf16_np, hidden_rows, small_config
from yanah_b200.stack import ResidentStack
from yanah_b200.streaming import StreamingDecoder

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("frac,spec", [(0.3, 8), (0.6, 16)])
def test_streaming_equals_resident(frac, spec):
    cfg = small_config(bits=(4, 2, 2, 4), seed=23, zipf=1.1)
    N = 6
    x = bf16_dev(hidden_rows(cfg, N, stream=4))
    ref = torch.empty_like(x)
    ResidentStack(cfg, "cuda").run(x, ref)
    torch.cuda.synchronize()
    dec = StreamingDecoder(cfg, slot_fraction=frac, spec_slot_cap=spec, device="cuda")
    got = torch.empty_like(x)
    dec.decode(x, got)
    torch.cuda.synchronize()
    assert np.array_equal(bf16_np(got), bf16_np(ref))
    assert dec.be.check_error() == 0
    r = dec.report(1.0)
    assert r["tokens"] == N
    assert r["hits"] + r["misses"] > 0 and r["misses"] == r["demand_records"]
    assert r["h2d_gb"] > 0 and 0.0 <= r["hit_rate"] <= 1.0 and r["hidden_fraction"] <= 1.0
    # every routed (layer, expert) of a token was resident, adopted or demanded
    assert r["hits"] + r["misses"] >= N * cfg.n_layers
