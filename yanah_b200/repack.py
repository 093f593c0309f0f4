"""Record writer: the routed experts of an MLX-quantised checkpoint -> one
record per (layer, expert) in experts.bin, plus experts.json
(moe_prefetch/repack.py:66-126), and the reader that loads such a file into
pinned host memory as the streaming path's host tier.

Format (uniform stacks, byte-identical to the reference's files): records in
(layer, expert) order, MTP layers after the main ones; a record is the nine
pieces gate/up/down x weight/scales/biases back to back, padded with zeros to
a 16 KiB slot; experts.json is the record spec (pieces, group size, bits,
layer and expert counts, record and slot bytes).

Mixed-bit stacks (the reference rejects a layer whose pieces differ from layer
0's): every layer keeps its own pieces, every record is padded to the largest
layer's slot, and experts.json adds "layers" (one spec per layer) and
"stack_slot_bytes"; its top-level keys stay layer 0's.

Only the safetensors headers are parsed (8-byte little-endian header length,
JSON header, raw data); record bytes are copied by offset, so no tensor is
materialised.
"""
from __future__ import annotations

import glob
import json
import os
import struct
from typing import Dict, List, Optional, Sequence, Tuple

from .formats import PIECES, Piece, RecordSpec

Headers = Dict[str, Tuple[str, dict, int]]


def read_headers(model_dir: str) -> Headers:
    """tensor name -> (file, header entry, absolute offset of the file's data)."""
    out: Headers = {}
    for path in sorted(glob.glob(os.path.join(model_dir, "*.safetensors"))):
        with open(path, "rb") as fh:
            n = struct.unpack("<Q", fh.read(8))[0]
            header = json.loads(fh.read(n))
        for name, entry in header.items():
            if name != "__metadata__":
                out[name] = (path, entry, 8 + n)
    return out


def layer_prefix(layer: int, n_layers: int) -> str:
    """Tensor-name prefix of MoE layer `layer` (MTP layers follow the main ones)."""
    if layer < n_layers:
        return f"model.layers.{layer}.mlp.switch_mlp"
    return f"mtp.layers.{layer - n_layers}.mlp.switch_mlp"


def _layer_spec(hdrs: Headers, layer: int, n_layers: int, n_mtp: int, E: int, cfg: dict) -> RecordSpec:
    pieces = []
    for name in PIECES:
        key = f"{layer_prefix(layer, n_layers)}.{name}"
        if key not in hdrs:
            raise KeyError(f"missing tensor {key}")
        _, ent, _ = hdrs[key]
        b, e = ent["data_offsets"]
        if ent["shape"][0] != E or (e - b) % E:
            raise ValueError(f"{key}: leading dimension is not the {E} experts")
        pieces.append(Piece(name, ent["dtype"], list(ent["shape"][1:]), (e - b) // E))
    q = cfg.get("quantization", {})
    bits, gs = q.get("bits", 4), q.get("group_size", 64)
    H = cfg.get("hidden_size")
    if H:  # the layer's own format, from its gate_proj shapes (mixed-bit stacks)
        words, ng = pieces[0].shape[1], pieces[1].shape[1]
        if (words * 32) % H == 0 and ng and H % ng == 0:
            bits, gs = words * 32 // H, H // ng
    return RecordSpec(pieces, gs, bits, n_layers, n_mtp, E)


def build_specs(model_dir: str) -> Tuple[List[RecordSpec], Headers]:
    """One record spec per MoE layer (main layers, then MTP)."""
    with open(os.path.join(model_dir, "config.json")) as fh:
        cfg = json.load(fh)
    hdrs = read_headers(model_dir)
    n_layers, E = cfg["num_hidden_layers"], cfg["num_experts"]
    n_mtp = 1 if any(k.startswith("mtp.layers.0.mlp.switch_mlp.") for k in hdrs) else 0
    specs = [_layer_spec(hdrs, l, n_layers, n_mtp, E, cfg) for l in range(n_layers + n_mtp)]
    return specs, hdrs


def _uniform(specs: Sequence[RecordSpec]) -> bool:
    return all(s.pieces == specs[0].pieces for s in specs)


def repack(model_dir: str, out_dir: str) -> List[RecordSpec]:
    """Write out_dir/experts.bin and out_dir/experts.json; returns the per-layer specs."""
    specs, hdrs = build_specs(model_dir)
    slot = max(s.slot_bytes for s in specs)
    os.makedirs(out_dir, exist_ok=True)
    fds: Dict[str, int] = {}
    try:
        with open(os.path.join(out_dir, "experts.bin"), "wb") as out:
            for layer, spec in enumerate(specs):
                srcs = []
                for p in spec.pieces:
                    path, ent, base = hdrs[f"{layer_prefix(layer, spec.n_layers)}.{p.name}"]
                    if path not in fds:
                        fds[path] = os.open(path, os.O_RDONLY)
                    srcs.append((fds[path], base + ent["data_offsets"][0], p.nbytes))
                pad = b"\0" * (slot - spec.record_bytes)
                for e in range(spec.n_experts):
                    for fd, off, nb in srcs:
                        chunk = os.pread(fd, nb, off + e * nb)
                        if len(chunk) != nb:
                            raise IOError(f"short read in layer {layer}, expert {e}")
                        out.write(chunk)
                    out.write(pad)
    finally:
        for fd in fds.values():
            os.close(fd)
    meta = specs[0].to_json()
    if not _uniform(specs):
        meta["layers"] = [s.to_json() for s in specs]
        meta["stack_slot_bytes"] = slot
    with open(os.path.join(out_dir, "experts.json"), "w") as fh:
        json.dump(meta, fh, indent=1)
    return specs


def read_specs(out_dir: str) -> Tuple[List[RecordSpec], int]:
    """Per-layer specs and the slot stride of an experts.json."""
    with open(os.path.join(out_dir, "experts.json")) as fh:
        meta = json.load(fh)
    if "layers" in meta:
        return [RecordSpec.from_json(d) for d in meta["layers"]], int(meta["stack_slot_bytes"])
    spec = RecordSpec.from_json(meta)
    return [spec] * (spec.n_layers + spec.n_mtp_layers), spec.slot_bytes


class FileHostTier:
    """The records of an experts.bin in pinned host memory, one buffer per
    layer (records at the file's slot stride), for the streaming path and the
    prefill sweep (the same attributes as `streaming.HostTier`: `buf`, `rec`,
    `layers`, `record_ptr`)."""

    def __init__(self, out_dir: str, layers: Optional[Sequence[int]] = None, pin: bool = True):
        import numpy as np
        import torch
        self.specs, self.slot = read_specs(out_dir)
        self.layers = list(range(len(self.specs))) if layers is None else list(layers)
        path = os.path.join(out_dir, "experts.bin")
        self.buf: Dict[int, "torch.Tensor"] = {}
        self.rec: Dict[int, int] = {}
        E = self.specs[0].n_experts
        for l in self.layers:
            a = np.fromfile(path, dtype=np.uint8, count=E * self.slot, offset=l * E * self.slot)
            if a.size != E * self.slot:
                raise IOError(f"{path}: layer {l} is truncated")
            t = torch.from_numpy(a)
            self.buf[l] = t.pin_memory() if pin else t
            self.rec[l] = self.slot

    def record_ptr(self, layer: int, expert: int) -> int:
        return self.buf[layer].data_ptr() + expert * self.rec[layer]

    @property
    def nbytes(self) -> int:
        return sum(b.numel() for b in self.buf.values())
