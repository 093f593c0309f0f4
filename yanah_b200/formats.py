"""Expert geometry, record format and MLX affine packing.

Mirrors the reference's on-disk contract so records and traces interchange:

* ``ModelGeometry`` / ``ExpertLayout`` follow ``moe_prefetch/layout.py:28-119``
  (record size formula, 16 KiB slot alignment, row-major (layer, expert)).
* ``Piece`` / ``RecordSpec`` follow ``moe_prefetch/repack.py:27-63``: nine
  pieces per expert in the order gate/up/down x weight/scales/biases.
* ``pack`` / ``unpack`` implement MLX's affine format: ``32/bits`` codes per
  little-endian uint32 word, code k of a row at bit ``bits*(k % (32/bits))``
  of word ``k // (32/bits)``; ``w = scale*q + bias`` per group along the row.
"""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

PAGE = 16 * 1024
ExpertKey = Tuple[int, int]  # (layer, expert id)

PROJS = ("gate_proj", "up_proj", "down_proj")
PARTS = ("weight", "scales", "biases")
PIECES = [f"{p}.{q}" for p in PROJS for q in PARTS]


def align_up(n: int, a: int = PAGE) -> int:
    return (n + a - 1) // a * a


@dataclass(frozen=True)
class ModelGeometry:
    """Expert geometry (defaults: Qwen3-Next-80B-A3B), as moe_prefetch/layout.py:28-68."""
    n_layers: int = 48
    n_mtp_layers: int = 1
    n_experts: int = 512
    top_k: int = 10
    hidden: int = 2048
    moe_inter: int = 512
    bits: int = 4
    group_size: int = 64
    scale_bytes: int = 2
    record_bytes: int = 0

    @property
    def total_moe_layers(self) -> int:
        return self.n_layers + self.n_mtp_layers

    @property
    def expert_param_count(self) -> int:
        return 3 * self.hidden * self.moe_inter

    @property
    def expert_nbytes(self) -> int:
        if self.record_bytes:
            return self.record_bytes
        p = self.expert_param_count
        return p * self.bits // 8 + (p // self.group_size) * self.scale_bytes * 2

    @property
    def slot_nbytes(self) -> int:
        return align_up(self.expert_nbytes)


@dataclass(frozen=True)
class ExpertLocation:
    file_idx: int
    offset: int
    nbytes: int


class ExpertLayout:
    """(layer, expert) -> location of its contiguous record (layout.py:78-119)."""

    def __init__(self, geometry: ModelGeometry, files: List[str], locations: Dict[ExpertKey, ExpertLocation]):
        self.geometry, self.files, self.locations = geometry, files, locations

    def __getitem__(self, key: ExpertKey) -> ExpertLocation:
        return self.locations[key]

    def keys_for_layer(self, layer: int) -> Iterable[ExpertKey]:
        return ((layer, e) for e in range(self.geometry.n_experts))

    @classmethod
    def contiguous(cls, geometry: ModelGeometry, path: str) -> "ExpertLayout":
        stride = geometry.slot_nbytes
        locs = {(l, e): ExpertLocation(0, (l * geometry.n_experts + e) * stride, geometry.expert_nbytes)
                for l in range(geometry.total_moe_layers) for e in range(geometry.n_experts)}
        return cls(geometry, [path], locs)


@dataclass
class Piece:
    name: str
    dtype: str          # "U32" | "F16" | "BF16"
    shape: List[int]    # per-expert shape
    nbytes: int


@dataclass
class RecordSpec:
    """One record per expert, pieces back to back (repack.py:40-63)."""
    pieces: List[Piece]
    group_size: int
    bits: int
    n_layers: int
    n_mtp_layers: int
    n_experts: int

    @property
    def record_bytes(self) -> int:
        return sum(p.nbytes for p in self.pieces)

    @property
    def slot_bytes(self) -> int:
        return align_up(self.record_bytes, PAGE)

    @property
    def offsets(self) -> List[int]:
        out, o = [], 0
        for p in self.pieces:
            out.append(o)
            o += p.nbytes
        return out

    def to_json(self) -> dict:
        return {**asdict(self), "record_bytes": self.record_bytes, "slot_bytes": self.slot_bytes}

    @classmethod
    def from_json(cls, d: dict) -> "RecordSpec":
        return cls([Piece(**p) for p in d["pieces"]], d["group_size"], d["bits"], d["n_layers"],
                   d["n_mtp_layers"], d["n_experts"])


def expert_record_spec(hidden: int, inter: int, bits: int, group_size: int, n_layers: int = 1,
                       n_experts: int = 1, n_mtp_layers: int = 0) -> RecordSpec:
    """Record of one SwiGLU expert: gate/up (inter, hidden), down (hidden, inter)."""
    if bits not in (2, 4, 8):
        raise ValueError("bits must be 2, 4 or 8")
    pieces = []
    for proj in PROJS:
        rows, cols = (hidden, inter) if proj == "down_proj" else (inter, hidden)
        if cols % group_size or (cols * bits) % 32:
            raise ValueError(f"{proj}: {cols} columns do not fit group {group_size} / {bits}-bit words")
        ng = cols // group_size
        pieces += [Piece(f"{proj}.weight", "U32", [rows, cols * bits // 32], rows * cols * bits // 8),
                   Piece(f"{proj}.scales", "F16", [rows, ng], rows * ng * 2),
                   Piece(f"{proj}.biases", "F16", [rows, ng], rows * ng * 2)]
    return RecordSpec(pieces, group_size, bits, n_layers, n_mtp_layers, n_experts)


# ----------------------------------------------------------------- packing
def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """(rows, cols) integer codes -> (rows, cols*bits/32) uint32 words."""
    codes = np.asarray(codes, dtype=np.uint64)
    rows, cols = codes.shape
    cpw = 32 // bits
    if cols % cpw:
        raise ValueError("cols must be a multiple of 32/bits")
    if codes.size and int(codes.max()) >= (1 << bits):
        raise ValueError("code out of range")
    c = codes.reshape(rows, cols // cpw, cpw)
    shifts = (np.arange(cpw, dtype=np.uint64) * bits)[None, None, :]
    return (c << shifts).sum(axis=-1).astype(np.uint32)


def unpack(words: np.ndarray, bits: int, cols: Optional[int] = None) -> np.ndarray:
    """(rows, n_words) uint32 -> (rows, n_words*32/bits) codes (uint8)."""
    words = np.asarray(words, dtype=np.uint32)
    cpw = 32 // bits
    shifts = (np.arange(cpw, dtype=np.uint32) * bits)[None, None, :]
    c = (words[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    out = c.reshape(words.shape[0], -1).astype(np.uint8)
    return out if cols is None else out[:, :cols]


def dequantize_np(words: np.ndarray, scales: np.ndarray, biases: np.ndarray, bits: int, group_size: int) -> np.ndarray:
    """Reference-style dequantisation in numpy (fp32 multiply-add per element)."""
    q = unpack(words, bits).astype(np.float32)
    s = np.repeat(scales.astype(np.float32), group_size, axis=1)
    b = np.repeat(biases.astype(np.float32), group_size, axis=1)
    return s * q + b


# ----------------------------------------------------------------- bf16 bits
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    r = (u + np.uint32(0x7FFF) + lsb) >> np.uint32(16)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    r = np.where(nan, (u >> np.uint32(16)) | np.uint32(0x40), r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)
