"""Device-resident weights, expert slot arenas and workspaces.

PyTorch is used only to allocate device memory and to name streams; all
compute goes through libyanah_b200.so. Each holder keeps its tensors alive
and builds the C structs (``_lib.QMat`` / ``_lib.Layer``) that point at them.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from . import _lib
from .formats import RecordSpec
from .synthetic import (EXPERT_BIAS_STD, EXPERT_SCALE_STD, DenseLayer, StackConfig, expert_stream_id,
                        piece_elements)


def stream_ptr(stream: Optional[torch.cuda.Stream] = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _u32_tensor(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(device)


def _u16_tensor(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device)


class DeviceQMat:
    """One MLX-affine matrix on the device: words (int32 view of uint32), fp16 scales/biases."""

    def __init__(self, w: np.ndarray, s: np.ndarray, b: np.ndarray, cols: int, bits: int, group_size: int, device):
        self.w = _u32_tensor(w, device)
        self.s = _u16_tensor(np.asarray(s, np.float16).view(np.uint16), device)
        self.b = _u16_tensor(np.asarray(b, np.float16).view(np.uint16), device)
        self.rows, self.cols, self.bits, self.group_size = int(w.shape[0]), cols, bits, group_size

    def struct(self) -> _lib.QMat:
        return _lib.QMat(self.w.data_ptr(), self.s.data_ptr(), self.b.data_ptr(), self.rows, self.cols, self.bits,
                         self.group_size)


def record_struct(spec: RecordSpec) -> _lib.Record:
    r = _lib.Record()
    r.bits, r.group_size = spec.bits, spec.group_size
    for i, o in enumerate(spec.offsets):
        r.piece_offset[i] = o
    r.record_bytes = spec.record_bytes
    return r


class ExpertArena:
    """Slot arena: `n_slots` records of `slot_bytes` each, one per slot.

    The arena is the HBM counterpart of the reference's per-piece slot
    memory (mlx_backend.py:79-108): a record keeps the on-disk piece order,
    so a slot is filled by one contiguous copy."""

    def __init__(self, n_slots: int, slot_bytes: int, device):
        self.n_slots, self.slot_bytes = n_slots, slot_bytes
        self.buf = torch.empty(n_slots * slot_bytes, dtype=torch.uint8, device=device)

    @property
    def base(self) -> int:
        return self.buf.data_ptr()

    @property
    def nbytes(self) -> int:
        return self.buf.numel()

    def slot_view(self, slot: int) -> torch.Tensor:
        return self.buf[slot * self.slot_bytes:(slot + 1) * self.slot_bytes]


def fill_synthetic_experts(arena: ExpertArena, cfg: StackConfig, layer: int, first_slot: int = 0,
                           experts: Optional[Sequence[int]] = None, stream=None) -> None:
    """Write the seeded records of `layer` into consecutive slots from `first_slot`.
    experts: which expert ids (default all, in order)."""
    lib = _lib.lib()
    spec = cfg.record_spec(layer)
    ids = list(range(cfg.n_experts)) if experts is None else list(experts)
    n = len(ids)
    st = stream_ptr(stream)
    view = arena.buf.view(arena.n_slots, arena.slot_bytes)[first_slot:first_slot + n]
    contiguous = ids == list(range(ids[0], ids[0] + n)) if n else True
    for p, (off, piece) in enumerate(zip(spec.offsets, spec.pieces)):
        ne = piece_elements(spec, p)
        total = cfg.n_experts * ne
        elem = 4 if piece.dtype == "U32" else 2
        tmp = torch.empty(total * elem, dtype=torch.uint8, device=arena.buf.device)
        sid = expert_stream_id(layer, p)
        if piece.dtype == "U32":
            _lib.check(lib.yn_synth_u32(tmp.data_ptr(), total, cfg.seed, sid, st))
        else:
            std = EXPERT_SCALE_STD if p % 3 == 1 else EXPERT_BIAS_STD
            _lib.check(lib.yn_synth_f16(tmp.data_ptr(), total, cfg.seed, sid, std, 1 if p % 3 == 1 else 0, st))
        tv = tmp.view(cfg.n_experts, piece.nbytes)
        if contiguous:
            view[:, off:off + piece.nbytes].copy_(tv[ids[0]:ids[0] + n])
        else:
            idx = torch.tensor(ids, dtype=torch.long, device=arena.buf.device)
            view[:, off:off + piece.nbytes].copy_(tv.index_select(0, idx))
        del tmp


class DeviceLayer:
    """Resident weights of one MoE layer plus where its routed experts live."""

    def __init__(self, cfg: StackConfig, layer: int, dense: DenseLayer, arena: ExpertArena, first_slot: int,
                 slot_map: Optional[torch.Tensor], device):
        H, g = cfg.hidden, cfg.dense_group
        self.cfg, self.layer = cfg, layer
        self.norm = _u16_tensor(dense.norm, device)
        self.router = DeviceQMat(*dense.router, H, 8, g, device)
        self.router_bias = torch.from_numpy(dense.router_bias).to(device) if dense.router_bias is not None else None
        self.shared = None
        if cfg.shared_inter:
            self.shared = [DeviceQMat(*dense.shared_gate, H, 8, g, device),
                           DeviceQMat(*dense.shared_up, H, 8, g, device),
                           DeviceQMat(*dense.shared_down, cfg.shared_inter, 8, g, device),
                           DeviceQMat(*dense.shared_expert_gate, H, 8, g, device)]
        self.arena = arena
        self.first_slot = first_slot
        self.slot_map = slot_map  # (E,) int32 device tensor or None: slot = first_slot + id
        self.spec = cfg.record_spec(layer)
        self._struct = None

    def struct(self) -> _lib.Layer:
        L = _lib.Layer()
        L.post_norm = self.norm.data_ptr()
        L.router = self.router.struct()
        L.router_bias = self.router_bias.data_ptr() if self.router_bias is not None else None
        if self.shared is not None:
            L.shared_gate, L.shared_up, L.shared_down, L.shared_expert_gate = [m.struct() for m in self.shared]
        if self.slot_map is None:
            L.expert_base = self.arena.base + self.first_slot * self.arena.slot_bytes
            L.n_slots = self.arena.n_slots - self.first_slot
            L.expert_slot = None
        else:
            L.expert_base = self.arena.base
            L.n_slots = self.arena.n_slots
            L.expert_slot = self.slot_map.data_ptr()
        L.slot_stride = self.arena.slot_bytes
        L.record = record_struct(self.spec)
        self._struct = L
        return L


def dims_struct(cfg: StackConfig) -> _lib.Dims:
    return _lib.Dims(cfg.hidden, cfg.n_experts, cfg.top_k, cfg.moe_inter, cfg.shared_inter, int(cfg.norm_topk),
                     cfg.eps)


class Workspace:
    """Scratch for the layer kernels (sized for any row count up to YN_MAX_ROWS)."""

    def __init__(self, dims: _lib.Dims, device, stream=None):
        lib = _lib.lib()
        self.dims = dims
        self.nbytes = int(lib.yn_workspace_bytes(C.byref(dims)))
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        _lib.check(lib.yn_workspace_init(self.buf.data_ptr(), self.nbytes, C.byref(dims), stream_ptr(stream)))
        self.view = _lib.WsView()
        _lib.check(lib.yn_workspace_view(self.buf.data_ptr(), C.byref(dims), C.byref(self.view)))
        self._views: Dict[tuple, torch.Tensor] = {}

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    def tensor(self, name: str, shape, dtype) -> torch.Tensor:
        """A torch view of a named workspace region (see _lib.WsView)."""
        key = (name, tuple(shape), dtype)
        t = self._views.get(key)
        if t is None:
            off = getattr(self.view, name) - self.ptr
            elem = torch.empty((), dtype=dtype).element_size()
            n = int(np.prod(shape))
            t = self._views[key] = self.buf[off:off + n * elem].view(dtype).view(*shape)
        return t

    def check_error(self, stream=None) -> int:
        code = C.c_int32(0)
        rc = _lib.lib().yn_workspace_error(self.ptr, C.byref(self.dims), stream_ptr(stream), C.byref(code))
        if rc != _lib.YN_OK and code.value == 0:
            _lib.check(rc)
        return code.value
