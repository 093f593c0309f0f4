"""Record format, packing and workload byte counts (host only)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import cpu
from yanah_b200.formats import dequantize_np, pack, unpack
from yanah_b200.synthetic import qwen3_next_block, qwen3_next_stack


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_pack_unpack_roundtrip_and_word_order(bits):
    rng = np.random.default_rng(bits)
    codes = rng.integers(0, 2 ** bits, (7, 64))
    w = pack(codes, bits)
    assert w.shape == (7, 64 * bits // 32) and w.dtype == np.uint32
    assert np.array_equal(unpack(w, bits), codes)
    # code k sits at bit bits*(k % (32/bits)) of word k // (32/bits), little-endian
    one = np.zeros((1, 32 // bits * 2), np.int64)
    one[0, 1] = 1
    assert pack(one, bits)[0, 0] == 1 << bits


@pytest.mark.parametrize("bits,gs", [(2, 32), (2, 64), (4, 64), (4, 128), (8, 64)])
def test_oracle_dequantize_equals_affine_formula(bits, gs):
    rng = np.random.default_rng(bits * gs)
    rows, cols = 16, 256
    codes = rng.integers(0, 2 ** bits, (rows, cols))
    w = pack(codes, bits)
    s = np.abs(rng.standard_normal((rows, cols // gs)) * 0.02).astype(np.float16)
    b = (rng.standard_normal((rows, cols // gs)) * 0.01).astype(np.float16)
    got = cpu.dequantize(w, s, b, cols, bits, gs)
    # scale*q is exact in fp32 for fp16 scales and small codes, so one rounding either way
    assert np.array_equal(got.view(np.uint32), dequantize_np(w, s, b, bits, gs).view(np.uint32))


def test_workload_byte_counts():
    cfg = qwen3_next_stack(seed=0)
    assert cfg.record_spec(0).record_bytes == 1_769_472
    assert cfg.record_spec(4).record_bytes == 983_040
    assert cfg.record_spec(47).record_bytes == 1_769_472
    assert cfg.dense_bytes_per_layer() == 4_458_624
    assert cfg.bytes_per_token() == 748_787_712
    blk = qwen3_next_block(seed=0)
    assert blk.n_layers == 1 and blk.record_spec(0).bits == 4
