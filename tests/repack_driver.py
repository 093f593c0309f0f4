"""Tiny seeded MLX-format checkpoints (safetensors shards + config.json) for
the record-writer parity tests.

Used twice with the same inputs: by tests/golden/make_golden.py, which runs
the reference's repack (moe_prefetch/repack.py) on them and records its
output, and by tests/test_repack_golden.py, which runs yanah_b200.repack on
the same checkpoints and compares. The tensor bytes are random: the writer
copies bytes and never interprets them. tests/test_gpu_sweep.py also writes a
checkpoint from a synthetic host tier (write_checkpoint_from_tier) to run the
prefill sweep from a repacked experts.bin.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Sequence

import numpy as np

PIECE_ORDER = [f"{p}.{q}" for p in ("gate_proj", "up_proj", "down_proj") for q in ("weight", "scales", "biases")]

# name -> (layer bits, group size, hidden, inter, experts, mtp layer, shards)
CASES = {
    "uniform4_mtp": ((4, 4, 4), 64, 256, 128, 8, True, 2),
    "uniform2_g32": ((2, 2), 32, 256, 64, 6, False, 1),
    "mixed42": ((4, 2, 4), 64, 256, 128, 4, False, 3),
}


def _write_safetensors(path: str, tensors) -> None:
    """tensors: list of (name, dtype, shape, raw bytes)."""
    header, off = {}, 0
    for name, dtype, shape, raw in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * (-len(hb) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(hb)))
        fh.write(hb)
        for _, _, _, raw in tensors:
            fh.write(raw)


def write_checkpoint(model_dir: str, case: str, seed: int = 7) -> None:
    layer_bits, gs, H, I, E, mtp, shards = CASES[case]
    rng = np.random.default_rng(seed)
    os.makedirs(model_dir, exist_ok=True)
    n_main = len(layer_bits) - (1 if mtp else 0)
    tensors = []
    for layer, bits in enumerate(layer_bits):
        prefix = (f"model.layers.{layer}.mlp.switch_mlp" if layer < n_main
                  else f"mtp.layers.{layer - n_main}.mlp.switch_mlp")
        for piece in PIECE_ORDER:
            proj, part = piece.split(".")
            rows, cols = (H, I) if proj == "down_proj" else (I, H)
            if part == "weight":
                dtype, shape, nb = "U32", (E, rows, cols * bits // 32), E * rows * cols * bits // 8
            else:
                dtype, shape, nb = "F16", (E, rows, cols // gs), E * rows * (cols // gs) * 2
            tensors.append((f"{prefix}.{piece}", dtype, shape, rng.integers(0, 256, nb, dtype=np.uint8).tobytes()))
        # a non-expert tensor of the layer, which the writer must skip
        tensors.append((f"model.layers.{layer}.input_layernorm.weight", "F16", (H,),
                        rng.integers(0, 256, 2 * H, dtype=np.uint8).tobytes()))
    per = -(-len(tensors) // shards)
    for s in range(shards):
        _write_safetensors(os.path.join(model_dir, f"model-{s + 1:05d}-of-{shards:05d}.safetensors"),
                           tensors[s * per:(s + 1) * per])
    cfg = {"num_hidden_layers": n_main, "num_experts": E, "hidden_size": H, "moe_intermediate_size": I,
           "quantization": {"group_size": gs, "bits": layer_bits[0]}}
    with open(os.path.join(model_dir, "config.json"), "w") as fh:
        json.dump(cfg, fh)


def expected_records(model_dir: str, layers: Sequence[int], n_main: int, E: int):
    """Per (layer, expert) the concatenated piece bytes, read straight from the shards."""
    import glob
    hdrs = {}
    for path in sorted(glob.glob(os.path.join(model_dir, "*.safetensors"))):
        with open(path, "rb") as fh:
            n = struct.unpack("<Q", fh.read(8))[0]
            for name, ent in json.loads(fh.read(n)).items():
                hdrs[name] = (path, ent, 8 + n)
    out = {}
    for layer in layers:
        prefix = (f"model.layers.{layer}.mlp.switch_mlp" if layer < n_main
                  else f"mtp.layers.{layer - n_main}.mlp.switch_mlp")
        for e in range(E):
            rec = b""
            for piece in PIECE_ORDER:
                path, ent, base = hdrs[f"{prefix}.{piece}"]
                b0, b1 = ent["data_offsets"]
                nb = (b1 - b0) // E
                with open(path, "rb") as fh:
                    fh.seek(base + b0 + e * nb)
                    rec += fh.read(nb)
            out[(layer, e)] = rec
    return out


def write_checkpoint_from_tier(model_dir: str, cfg, tier, layers: Sequence[int]) -> None:
    """An MLX-format checkpoint holding the routed experts of a host tier
    (records of `cfg`'s format): per layer and piece, the experts' piece bytes
    stacked along a leading expert dimension."""
    os.makedirs(model_dir, exist_ok=True)
    tensors = []
    for layer in layers:
        spec = cfg.record_spec(layer)
        host = tier.buf[layer].numpy()
        rb = tier.rec[layer]
        E = cfg.n_experts
        for off, p in zip(spec.offsets, spec.pieces):
            raw = b"".join(host[e * rb + off:e * rb + off + p.nbytes].tobytes() for e in range(E))
            tensors.append((f"model.layers.{layer}.mlp.switch_mlp.{p.name}", p.dtype, (E, *p.shape), raw))
    _write_safetensors(os.path.join(model_dir, "model-00001-of-00001.safetensors"), tensors)
    spec0 = cfg.record_spec(layers[0])
    with open(os.path.join(model_dir, "config.json"), "w") as fh:
        json.dump({"num_hidden_layers": len(layers), "num_experts": cfg.n_experts, "hidden_size": cfg.hidden,
                   "quantization": {"group_size": spec0.group_size, "bits": spec0.bits}}, fh)
