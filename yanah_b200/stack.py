"""All-resident MoE stack decode (every routed expert in HBM).

One decode token walks the layers; each layer is one ``yn_moe_layer`` call
(post-attention + routing kernel, routed gate/up kernel, down + combine
kernel). The host never syncs inside a token: routing stays on the device.
A whole decode of N tokens is captured once into a CUDA graph and replayed,
so per-kernel launch cost leaves the critical path.

This is the reference's pool-path layer loop (orchestrator.py:308-343 with
_pool_layer :226-300) for the case where the pool holds every expert.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional

import numpy as np
import torch

from . import _lib
from .device import DeviceLayer, ExpertArena, Workspace, dims_struct, fill_synthetic_experts, stream_ptr
from .synthetic import StackConfig, dense_layer


class ResidentStack:
    def __init__(self, cfg: StackConfig, device: str = "cuda", layers: Optional[List[int]] = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.layer_ids = list(range(cfg.n_layers)) if layers is None else list(layers)
        self.dims = dims_struct(cfg)
        self.arenas: List[ExpertArena] = []
        self.layers: List[DeviceLayer] = []
        for l in self.layer_ids:
            spec = cfg.record_spec(l)
            arena = ExpertArena(cfg.n_experts, spec.slot_bytes, self.device)
            fill_synthetic_experts(arena, cfg, l)
            self.arenas.append(arena)
            self.layers.append(DeviceLayer(cfg, l, dense_layer(cfg, l), arena, 0, None, self.device))
        self.structs = [L.struct() for L in self.layers]
        self.ws = Workspace(self.dims, self.device)
        H = cfg.hidden
        self._ping = torch.empty((2, 1, H), dtype=torch.bfloat16, device=self.device)
        torch.cuda.synchronize(self.device)

    @property
    def expert_bytes(self) -> int:
        return sum(a.nbytes for a in self.arenas)

    def run_token(self, h_in: torch.Tensor, h_out: torch.Tensor, stream=None) -> None:
        """One bs1 token through every layer: h_in (1,H) bf16 -> h_out (1,H)."""
        lib = _lib.lib()
        st = stream_ptr(stream)
        n = len(self.structs)
        src = h_in.data_ptr()
        for i, L in enumerate(self.structs):
            dst = h_out.data_ptr() if i == n - 1 else self._ping[i % 2].data_ptr()
            _lib.check(lib.yn_moe_layer(C.byref(self.dims), C.byref(L), src, 1, None, 0, dst, self.ws.ptr, st))
            src = dst

    def run(self, inputs: torch.Tensor, outputs: torch.Tensor, stream=None) -> None:
        """Sequential bs1 decode of inputs (N,H) -> outputs (N,H)."""
        for t in range(inputs.shape[0]):
            self.run_token(inputs[t:t + 1], outputs[t:t + 1], stream)

    def capture(self, inputs: torch.Tensor, outputs: torch.Tensor) -> torch.cuda.CUDAGraph:
        """Capture `run(inputs, outputs)` as one CUDA graph (call run once first)."""
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.run(inputs, outputs, s)
        torch.cuda.current_stream(self.device).wait_stream(s)
        return g

    def kernel_launches_per_token(self) -> int:
        return 3 * len(self.structs)
