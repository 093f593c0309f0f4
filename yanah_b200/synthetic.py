"""Seeded synthetic Qwen3-Next-shaped MoE stacks.

There is no checkpoint or recorded routing trace to load, so the workloads
are generated from a seed with the shapes and value distributions of the
benchmark configurations:

* routed experts: codes uniform in [0, 2^bits) (uniform uint32 words), fp16
  scales |N(0, 0.02)|, fp16 biases N(0, 0.01), MLX affine packing, group 64;
* routers and the shared expert: 8-bit, group 64, centred (bias = -127.5 *
  scale) so that outputs have unit-scale variance;
* router logits carry a per-layer offset log p_e with p Zipf(s) over a
  per-layer permutation of the experts, so expert popularity is Zipf-skewed;
* hidden inputs: bf16 N(0, 1).

Routed expert pieces (27 GB for the 48-layer stack) are produced on the GPU
by a counter-based generator: element i of piece p of layer l is a pure
function of (seed, layer, p, i), so any record can be regenerated on the CPU
bit for bit. Dense weights (routers, shared expert, norms: ~4.5 MB a layer)
are generated on the host with numpy.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

from .formats import RecordSpec, expert_record_spec, f32_to_bf16_bits

TAG_EXPERT = 1
TAG_HIDDEN = 2


def expert_stream_id(layer: int, piece: int) -> int:
    """Generator stream of piece `piece` (0..8, record order) of layer `layer`."""
    return (TAG_EXPERT << 48) | (layer << 8) | piece


def hidden_stream_id(stream: int) -> int:
    return (TAG_HIDDEN << 48) | stream


EXPERT_SCALE_STD = 0.02
EXPERT_BIAS_STD = 0.01


@dataclass
class StackConfig:
    name: str
    n_layers: int
    expert_bits: Tuple[int, ...]
    hidden: int = 2048
    n_experts: int = 512
    top_k: int = 10
    moe_inter: int = 512
    shared_inter: int = 512
    group_size: int = 64
    dense_group: int = 64
    zipf_s: float = 1.1
    router_noise: float = 1.3
    seed: int = 0
    norm_topk: bool = True
    eps: float = 1e-6

    def __post_init__(self):
        if len(self.expert_bits) != self.n_layers:
            raise ValueError("expert_bits needs one entry per layer")

    def record_spec(self, layer: int) -> RecordSpec:
        return expert_record_spec(self.hidden, self.moe_inter, self.expert_bits[layer], self.group_size,
                                  n_layers=self.n_layers, n_experts=self.n_experts)

    @property
    def slot_bytes(self) -> int:
        """Uniform slot size: the largest record, 16 KiB aligned (mixed-bit stacks)."""
        return max(self.record_spec(l).slot_bytes for l in range(self.n_layers))

    def routed_bytes_per_token(self) -> int:
        return sum(self.top_k * self.record_spec(l).record_bytes for l in range(self.n_layers))

    def dense_bytes_per_layer(self) -> int:
        H, E, Ish, g = self.hidden, self.n_experts, self.shared_inter, self.dense_group
        q = lambda r, c: r * c + 2 * r * (c // g) * 2
        return q(E, H) + (q(Ish, H) * 2 + q(H, Ish) + q(1, H) if Ish else 0)

    def bytes_per_token(self) -> int:
        """Algorithmic HBM bytes of one bs1 decode token (weights read once)."""
        return self.routed_bytes_per_token() + self.n_layers * self.dense_bytes_per_layer()


def qwen3_next_block(seed: int = 0) -> StackConfig:
    """One Qwen3-Next-shaped MoE block, 4-bit routed experts (the bs1 block workload)."""
    return StackConfig("qwen3next_block_bs1", 1, (4,), seed=seed)


def qwen3_next_stack(seed: int = 0, n_layers: int = 48) -> StackConfig:
    """48-layer Qwen3-Next-80B-A3B-shaped stack: experts 4-bit in the first and
    last 4 layers, 2-bit elsewhere; router/shared 8-bit."""
    bits = tuple(4 if (l < 4 or l >= n_layers - 4) else 2 for l in range(n_layers))
    return StackConfig("qwen3next_80b_a3b_stack48", n_layers, bits, seed=seed)


def lfm2_stack(seed: int = 0, n_layers: int = 40) -> StackConfig:
    """40-layer LFM2-24B-A2B-shaped MoE stack for the tensor-core prefill path:
    64 experts, top-4, SwiGLU intermediate 1536, 4-bit g64 experts, 8-bit
    router, no shared expert."""
    return StackConfig("lfm2_24b_a2b_stack40", n_layers, (4,) * n_layers, hidden=2048, n_experts=64, top_k=4,
                       moe_inter=1536, shared_inter=0, seed=seed)


# ------------------------------------------------------------ dense weights
@dataclass
class DenseLayer:
    """Host copies of one layer's resident weights (numpy)."""
    norm: np.ndarray                    # (H,) uint16 bf16 bits
    router: Tuple[np.ndarray, np.ndarray, np.ndarray]
    router_bias: np.ndarray             # (E,) float32
    shared_gate: Optional[Tuple[np.ndarray, np.ndarray, np.ndarray]] = None
    shared_up: Optional[Tuple[np.ndarray, np.ndarray, np.ndarray]] = None
    shared_down: Optional[Tuple[np.ndarray, np.ndarray, np.ndarray]] = None
    shared_expert_gate: Optional[Tuple[np.ndarray, np.ndarray, np.ndarray]] = None


def _centred_q8(rng, rows: int, cols: int, gs: int, out_std: float):
    """8-bit matrix whose dequantised weights are ~zero-mean with std out_std."""
    w = rng.integers(0, 2**32, size=(rows, cols // 4), dtype=np.uint32)
    s = (out_std / 73.9) * (1.0 + 0.1 * rng.standard_normal((rows, cols // gs)))
    s = np.abs(s).astype(np.float16)
    b = (-127.5 * s.astype(np.float32)).astype(np.float16)
    return w, s, b


def zipf_bias(rng, n_experts: int, s: float) -> np.ndarray:
    p = 1.0 / np.arange(1, n_experts + 1, dtype=np.float64) ** s
    p /= p.sum()
    perm = rng.permutation(n_experts)
    bias = np.empty(n_experts, np.float64)
    bias[perm] = np.log(p)
    return (bias - bias.mean()).astype(np.float32)


def dense_layer(cfg: StackConfig, layer: int) -> DenseLayer:
    rng = np.random.default_rng([cfg.seed, 1000 + layer])
    H, E, Ish, g = cfg.hidden, cfg.n_experts, cfg.shared_inter, cfg.dense_group
    norm = f32_to_bf16_bits(1.0 + 0.1 * rng.standard_normal(H).astype(np.float32))
    router = _centred_q8(rng, E, H, g, cfg.router_noise / np.sqrt(H))
    bias = zipf_bias(rng, E, cfg.zipf_s) if cfg.zipf_s > 0 else np.zeros(E, np.float32)
    d = DenseLayer(norm, router, bias)
    if Ish:
        d.shared_gate = _centred_q8(rng, Ish, H, g, 1.0 / np.sqrt(H))
        d.shared_up = _centred_q8(rng, Ish, H, g, 1.0 / np.sqrt(H))
        d.shared_down = _centred_q8(rng, H, Ish, g, 1.0 / np.sqrt(Ish))
        d.shared_expert_gate = _centred_q8(rng, 1, H, g, 1.0 / np.sqrt(H))
    return d


def piece_kind(piece: int) -> str:
    return ("weight", "scales", "biases")[piece % 3]


def piece_elements(spec: RecordSpec, piece: int) -> int:
    p = spec.pieces[piece]
    return p.nbytes // (4 if p.dtype == "U32" else 2)
