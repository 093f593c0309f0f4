"""Shared helpers for the GPU parity tests (device side vs the CPU oracle)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from oracle import cpu
from yanah_b200 import _lib
from yanah_b200.device import DeviceLayer, ExpertArena, Workspace, dims_struct, fill_synthetic_experts, stream_ptr
from yanah_b200.synthetic import StackConfig, dense_layer

REL_L2_TOL = 1e-2  # bf16 layer outputs vs the oracle (relative L2)


def small_config(bits=(4,), gs=64, seed=3, hidden=1024, n_experts=64, top_k=4, inter=256, shared=256,
                 zipf=1.1) -> StackConfig:
    return StackConfig("small", len(bits), tuple(bits), hidden=hidden, n_experts=n_experts, top_k=top_k,
                       moe_inter=inter, shared_inter=shared, group_size=gs, zipf_s=zipf, seed=seed)


def bf16_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def bf16_dev(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).to(device).view(torch.bfloat16)


def rel_l2(a_bf16: np.ndarray, b_bf16: np.ndarray) -> float:
    a = cpu.bf16_to_f32(a_bf16).astype(np.float64)
    b = cpu.bf16_to_f32(b_bf16).astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class DeviceModel:
    """Device layers of a seeded config, one arena per layer (slot = expert id)."""

    def __init__(self, cfg: StackConfig, device="cuda"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dims = dims_struct(cfg)
        self.arenas, self.layers = [], []
        for l in range(cfg.n_layers):
            spec = cfg.record_spec(l)
            a = ExpertArena(cfg.n_experts, spec.slot_bytes, self.device)
            fill_synthetic_experts(a, cfg, l)
            self.arenas.append(a)
            self.layers.append(DeviceLayer(cfg, l, dense_layer(cfg, l), a, 0, None, self.device))
        self.structs = [L.struct() for L in self.layers]
        self.ws = Workspace(self.dims, self.device)

    def post_attention(self, layer: int, h1: torch.Tensor, targets=()):
        T = h1.shape[0]
        tg = (_lib.Layer * max(1, len(targets)))(*[self.structs[t] for t in targets]) if targets else None
        _lib.check(_lib.lib().yn_post_attention(C.byref(self.dims), C.byref(self.structs[layer]), h1.data_ptr(), T,
                                                tg, len(targets), self.ws.ptr, stream_ptr()))

    def layer(self, layer: int, h_in: torch.Tensor, h_out: torch.Tensor):
        _lib.check(_lib.lib().yn_moe_layer(C.byref(self.dims), C.byref(self.structs[layer]), h_in.data_ptr(),
                                           h_in.shape[0], None, 0, h_out.data_ptr(), self.ws.ptr, stream_ptr()))

    def ws_out(self, T: int, n_targets: int = 0):
        cfg = self.cfg
        ws = self.ws
        K, H, E = cfg.top_k, cfg.hidden, cfg.n_experts
        out = dict(
            x=bf16_np(ws.tensor("x", (T, H), torch.bfloat16)),
            logits=ws.tensor("logits", (T, E), torch.float32).cpu().numpy(),
            ids=ws.tensor("ids", (T, K), torch.int32).cpu().numpy(),
            w=ws.tensor("weights", (T, K), torch.float32).cpu().numpy(),
            act=bf16_np(ws.tensor("act", (T, K, cfg.moe_inter), torch.bfloat16)),
            y=bf16_np(ws.tensor("y", (T, K, H), torch.bfloat16)),
        )
        if cfg.shared_inter:
            out["act_sh"] = bf16_np(ws.tensor("act_sh", (T, cfg.shared_inter), torch.bfloat16))
            out["sgate"] = ws.tensor("sgate", (T,), torch.float32).cpu().numpy()
            out["ysh"] = bf16_np(ws.tensor("y_shared", (T, H), torch.bfloat16))
        if n_targets:
            out["fprobs"] = ws.tensor("fprobs", (n_targets, E), torch.float32).cpu().numpy()
        return out


def hidden_rows(cfg: StackConfig, T: int, stream: int = 0) -> np.ndarray:
    from yanah_b200.synthetic import hidden_stream_id
    return cpu.synth_bf16(T * cfg.hidden, cfg.seed, hidden_stream_id(stream), 1.0).reshape(T, cfg.hidden)
