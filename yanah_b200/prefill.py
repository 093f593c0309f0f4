"""Prompt prefill of a ragged batch through the routed experts on the tcgen05
tensor cores (the LFM2-24B-A2B-shaped configuration).

Per layer: post-attention and routing of every prompt row (`yn_rows_route`,
bit-identical to the single-row path); the rows' fp16 K-permuted copy
(`yn_gather_f16_kperm`, in pair order); the grouping of the (row, column) pairs by expert, as
the reference's prefill sweep plans its staging groups (sweep.py:80-138); the grouped gate/up + SwiGLU and down GEMMs
(`yn_tc_experts`, 128 weight rows x up to 256 rows per tile); the combine in
column order plus the residual (`yn_pairs_combine`). The grouping runs on the
device (`yn_prefill_plan`); `plan_prefill` is its host restatement.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from .device import DeviceLayer, ExpertArena, dims_struct, fill_synthetic_experts, stream_ptr
from .synthetic import StackConfig, dense_layer

TILE_ROWS = 256      # token rows per tile
UP_UNITS = 64        # gate/up units per tile (128 weight rows)
DOWN_ROWS = 128      # down output rows per tile


class TcTile(C.Structure):
    _fields_ = [("e", C.c_int32), ("p0", C.c_int32), ("n", C.c_int32), ("u0", C.c_int32)]


def plan_prefill(ids: np.ndarray, n_experts: int, inter: int, hidden: int):
    """Pairs grouped by expert (ascending id, rows in order inside an expert).
    Returns pair_row (P,), pair_of (T, K), gate/up tiles and down tiles as
    int32 arrays of (e, p0, n, u0)."""
    ids = np.asarray(ids)
    T, K = ids.shape
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind="stable")          # pair p -> flat index t * K + j
    pair_row = (order // K).astype(np.int32)
    pair_of = np.empty(T * K, np.int32)
    pair_of[order] = np.arange(T * K, dtype=np.int32)
    experts, starts, counts = np.unique(flat[order], return_index=True, return_counts=True)
    up, down = [], []
    for e, p0, n in zip(experts.tolist(), starts.tolist(), counts.tolist()):
        for c0 in range(0, n, TILE_ROWS):
            m = min(TILE_ROWS, n - c0)
            up += [(e, p0 + c0, m, u) for u in range(0, inter, UP_UNITS)]
            down += [(e, p0 + c0, m, r) for r in range(0, hidden, DOWN_ROWS)]
    return (pair_row, pair_of.reshape(T, K), np.array(up, np.int32).reshape(-1, 4),
            np.array(down, np.int32).reshape(-1, 4))


class PrefillStack:
    """Resident experts and dense weights of `layers` of `cfg`, and the
    buffers for prompts of up to `max_rows` rows in total. A layer runs
    entirely on the device (routing, grouping, GEMMs, combine): no host
    synchronisation."""

    def __init__(self, cfg: StackConfig, max_rows: int, device: str = "cuda",
                 layers: Optional[Sequence[int]] = None):
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
        lib = _lib.lib()
        H, K, I = cfg.hidden, cfg.top_k, cfg.moe_inter
        T, P = max_rows, max_rows * K
        dev = self.device
        self.max_rows = max_rows
        nb = int(lib.yn_rows_route_bytes(C.byref(self.dims), max_rows))
        if not nb:
            raise ValueError("max_rows outside what the routing workspace supports")
        self.route_ws = torch.zeros(nb, dtype=torch.uint8, device=dev)
        mu, md = C.c_int32(0), C.c_int32(0)
        _lib.check(lib.yn_prefill_max_tiles(C.byref(self.dims), max_rows, C.byref(mu), C.byref(md)))
        self.max_up, self.max_dn = mu.value, md.value
        self.tiles_up = torch.empty((self.max_up, 4), dtype=torch.int32, device=dev)
        self.tiles_dn = torch.empty((self.max_dn, 4), dtype=torch.int32, device=dev)
        self.n_tiles = torch.zeros(2, dtype=torch.int32, device=dev)
        self.pair_row = torch.empty(P, dtype=torch.int32, device=dev)
        self.pair_of = torch.empty(P, dtype=torch.int32, device=dev)
        self.x = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        self.x16 = torch.empty((P, H), dtype=torch.float16, device=dev)  # rows in pair order
        self.ids = torch.empty((T, K), dtype=torch.int32, device=dev)
        self.w = torch.empty((T, K), dtype=torch.float32, device=dev)
        self.act = torch.empty((P, I), dtype=torch.bfloat16, device=dev)
        self.y = torch.empty((P, H), dtype=torch.bfloat16, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ping = torch.empty((2, T, H), dtype=torch.bfloat16, device=dev)

    def layer(self, i: int, h: torch.Tensor, out: torch.Tensor, stream=None, gemm_events=None) -> None:
        """Layer i (index into `layer_ids`) of T = h.shape[0] rows. gemm_events:
        optional list that receives (start, end) CUDA events around the two
        grouped GEMM launches."""
        lib, cfg = _lib.lib(), self.cfg
        T, H = h.shape[0], cfg.hidden
        if T > self.max_rows:
            raise ValueError("more rows than the buffers hold")
        st = stream_ptr(stream)
        D, L = C.byref(self.dims), C.byref(self.structs[i])
        _lib.check(lib.yn_rows_route(D, L, h.data_ptr(), T, self.x.data_ptr(), self.ids.data_ptr(), self.w.data_ptr(),
                                     self.route_ws.data_ptr(), self.route_ws.numel(), st))
        _lib.check(lib.yn_prefill_plan(D, self.ids.data_ptr(), T, self.pair_row.data_ptr(), self.pair_of.data_ptr(),
                                       self.tiles_up.data_ptr(), self.max_up, self.tiles_dn.data_ptr(), self.max_dn,
                                       self.n_tiles.data_ptr(), self.err.data_ptr(), st))
        P = T * cfg.top_k
        _lib.check(lib.yn_gather_f16_kperm(self.x.data_ptr(), self.pair_row.data_ptr(), P, H, self.x16.data_ptr(), st))
        if gemm_events is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        nt = self.n_tiles.data_ptr()
        _lib.check(lib.yn_tc_experts(D, L, 0, self.tiles_up.data_ptr(), self.max_up, nt, self.x16.data_ptr(), P,
                                     self.act.data_ptr(), None, self.err.data_ptr(), st))
        _lib.check(lib.yn_tc_experts(D, L, 1, self.tiles_dn.data_ptr(), self.max_dn, nt + 4, self.act.data_ptr(), P,
                                     None, self.y.data_ptr(), self.err.data_ptr(), st))
        if gemm_events is not None:
            e1.record(stream)
            gemm_events.append((e0, e1))
        _lib.check(lib.yn_pairs_combine(D, self.y.data_ptr(), self.pair_of.data_ptr(), self.w.data_ptr(), None,
                                        h.data_ptr(), T, out.data_ptr(), st))

    def plan(self, T: int):
        """Host copies of the last layer's ids, pair -> row and (row, column) -> pair."""
        K = self.cfg.top_k
        return (self.ids[:T].cpu().numpy(), self.pair_row[:T * K].cpu().numpy(),
                self.pair_of[:T * K].cpu().numpy().reshape(T, K))

    def prefill(self, h: torch.Tensor, stream=None, gemm_events=None) -> torch.Tensor:
        """Every layer for the rows h (T, H) bf16; returns the last layer's output."""
        T = h.shape[0]
        self.ping[0, :T].copy_(h)
        for i in range(len(self.layer_ids)):
            self.layer(i, self.ping[i % 2, :T], self.ping[(i + 1) % 2, :T], stream, gemm_events)
        return self.ping[len(self.layer_ids) % 2, :T]

    def check_error(self) -> int:
        torch.cuda.synchronize(self.device)
        code = int(self.err.item())
        rc = C.c_int32(0)
        _lib.check(_lib.lib().yn_route_error(self.route_ws.data_ptr(), C.byref(self.dims), stream_ptr(),
                                             C.byref(rc)))
        self.err.zero_()
        return code or rc.value


def kperm_inverse(a: np.ndarray) -> np.ndarray:
    """Natural column order of a K-permuted (…, cols) array."""
    cols = a.shape[-1]
    k = np.arange(cols)
    p = k & 7
    pos = (k & ~7) | np.where(p < 4, 2 * p, 2 * (p - 4) + 1)
    return a[..., pos]
