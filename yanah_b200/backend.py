"""CUDA backend for the MoE part of the reference's ModelBackend interface.

Mirrors the hooks `moe_prefetch/orchestrator.py` calls on
`moe_prefetch/mlx_backend.py` (see INTEGRATION.md for the table):

    pre_moe(layer, h1) -> (h_res, x, logits)          mlx_backend.py:290-306
    route(logits) -> (ids np (T,k), w)                :308-316
    route_and_forecast(logits, h_res, targets)        :326-348
    moe_ready(layer, x, ids, memory, ready) -> handle :376-391
    moe_rest(layer, x, ids, w, memory, rows, handle)  :393-409
    moe(layer, x, ids, w, memory, rows, sync=True)    :411-436 (pool path)
    moe_finalize(layer, routed)                       :438-440
    launch(h), fence()                                :365-374
    make_expert_memory(n), layout()                   :239-243

Differences from the MLX backend, all outside the MoE path:
* attention is not part of this path: `pre_moe` takes the post-attention
  residual h1 (T, H) bf16 on the device (the synthetic workloads use the
  residual identity for attention);
* tensors are torch device tensors; routed ids come back as numpy, like the
  reference's `np.array(inds)` sync;
* the shared expert is added in the same kernel as the weighted sum over the
  k columns (same bf16 rounding order as `routed + shared`), so
  `moe_finalize` returns its input;
* `moe` with experts missing from `rows` (the prefill sweep's staging groups,
  mlx_backend.py:421-433) is not built yet and raises.

Every call is asynchronous on the backend's stream; `fence()` blocks until the
work that reads pool slots has finished.
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from . import _lib
from .device import DeviceLayer, ExpertArena, Workspace, dims_struct, record_struct, stream_ptr
from .formats import ExpertLayout, ModelGeometry, RecordSpec
from .synthetic import StackConfig, dense_layer


class CudaExpertMemory:
    """Pool or staging slots in HBM (mlx_backend.py:79-108): n slots of
    `slot_bytes`, each holding one record in the on-disk piece order."""

    def __init__(self, n: int, spec: RecordSpec, device, slot_bytes: Optional[int] = None):
        self.n, self.spec = n, spec
        self.arena = ExpertArena(n, slot_bytes or spec.slot_bytes, device)
        # typed per-piece views (n, *shape) over the slot-major arena
        self.arrays: Dict[str, torch.Tensor] = {}
        rows = self.arena.buf.view(n, self.arena.slot_bytes)
        for off, p in zip(spec.offsets, spec.pieces):
            dt = torch.int32 if p.dtype == "U32" else torch.float16
            self.arrays[p.name] = rows[:, off:off + p.nbytes].view(dt).view(n, *p.shape)

    def views(self, i: int) -> List[torch.Tensor]:
        """Device byte views of slot i, one per piece (the reference returns
        host memoryviews for its file reader; device slots are written with
        `load`)."""
        s = self.arena.slot_view(i)
        return [s[o:o + p.nbytes] for o, p in zip(self.spec.offsets, self.spec.pieces)]

    def load(self, slots: Sequence[int], host_records: Sequence[torch.Tensor], record_bytes: int,
             stream=None) -> None:
        """Copy pinned host records into slots (one cudaMemcpyAsync each)."""
        n = len(slots)
        if n == 0:
            return
        sl = (C.c_int32 * n)(*[int(s) for s in slots])
        src = (C.c_void_p * n)(*[int(r.data_ptr()) for r in host_records])
        _lib.check(_lib.lib().yn_slot_copy(self.arena.base, self.arena.slot_bytes, sl, src, n, int(record_bytes),
                                           stream_ptr(stream)))

    @property
    def nbytes(self) -> int:
        return self.arena.nbytes

    def close(self) -> None:
        self.arrays = {}
        self.arena = None


class CudaMoEBackend:
    supports_lazy_moe = True

    def __init__(self, cfg: StackConfig, device="cuda", lookahead: int = 2, stream: Optional[torch.cuda.Stream] = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.stream = stream or torch.cuda.current_stream(self.device)
        self.geometry = ModelGeometry(n_layers=cfg.n_layers, n_mtp_layers=0, n_experts=cfg.n_experts,
                                      top_k=cfg.top_k, hidden=cfg.hidden, moe_inter=cfg.moe_inter,
                                      bits=max(cfg.record_spec(l).bits for l in range(cfg.n_layers)),
                                      group_size=cfg.group_size,
                                      record_bytes=max(cfg.record_spec(l).record_bytes for l in range(cfg.n_layers)))
        self.lookahead = lookahead
        self.dims = dims_struct(cfg)
        self._dummy = ExpertArena(1, 16, self.device)
        self.layers = [DeviceLayer(cfg, l, dense_layer(cfg, l), self._dummy, 0, None, self.device)
                       for l in range(cfg.n_layers)]
        self.ws = Workspace(self.dims, self.device, self.stream)
        self._lut = torch.zeros(cfg.n_experts, dtype=torch.int32, device=self.device)
        # expert -> slot tables go up through a ring of pinned buffers (no host sync)
        self._lut_host = [torch.empty(cfg.n_experts, dtype=torch.int32, pin_memory=True) for _ in range(8)]
        self._lut_ev: List[Optional[torch.cuda.Event]] = [None] * len(self._lut_host)
        self._lut_i = 0
        self._pre: Dict[int, dict] = {}
        self._unfenced: Optional[torch.cuda.Event] = None

    # -------------------------------------------------------------- helpers
    def _st(self) -> int:
        return stream_ptr(self.stream)

    def _targets(self, layer: int) -> List[int]:
        return [t for t in range(layer + 1, layer + 1 + self.lookahead) if t < self.cfg.n_layers]

    def _layer_struct(self, layer: int, memory: CudaExpertMemory, rows: Dict[int, int]) -> _lib.Layer:
        """Layer descriptor whose routed experts live in `memory` at `rows`."""
        i = self._lut_i
        self._lut_i = (i + 1) % len(self._lut_host)
        if self._lut_ev[i] is not None:
            self._lut_ev[i].synchronize()        # the copy out of this buffer has run
        lut = self._lut_host[i].numpy()
        lut[:] = 0
        if rows:
            lut[np.fromiter(rows.keys(), dtype=np.int64)] = np.fromiter(rows.values(), dtype=np.int64)
        with torch.cuda.stream(self.stream):
            dev = torch.empty(self.cfg.n_experts, dtype=torch.int32, device=self.device)
            dev.copy_(self._lut_host[i], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(self.stream)
        self._lut_ev[i] = ev
        self._lut = dev   # freed tensors are reused in stream order by the caching allocator
        L = self.layers[layer].struct()
        L.expert_base = memory.arena.base
        L.slot_stride = memory.arena.slot_bytes
        L.n_slots = memory.n
        L.expert_slot = self._lut.data_ptr()
        L.record = record_struct(self.cfg.record_spec(layer))
        return L

    def layout(self) -> ExpertLayout:
        return ExpertLayout.contiguous(self.geometry, "experts.bin")

    def make_expert_memory(self, n: int) -> CudaExpertMemory:
        spec = max((self.cfg.record_spec(l) for l in range(self.cfg.n_layers)), key=lambda s: s.slot_bytes)
        return CudaExpertMemory(n, spec, self.device)

    # --------------------------------------------------------------- routing
    def pre_moe(self, layer: int, h1: torch.Tensor):
        """Post-attention half of the layer on the residual h1 (T, H) bf16:
        x = RMSNorm(h1), shared-expert activations and gate, router logits,
        and the lookahead probabilities of the next `lookahead` layers."""
        T = h1.shape[0]
        targets = self._targets(layer)
        tg = (_lib.Layer * max(len(targets), 1))(*[self.layers[t].struct() for t in targets]) if targets else None
        _lib.check(_lib.lib().yn_post_attention(C.byref(self.dims), C.byref(self.layers[layer].struct()),
                                                h1.data_ptr(), T, tg, len(targets), self.ws.ptr, self._st()))
        x = self.ws.tensor("x", (T, self.cfg.hidden), torch.bfloat16)
        logits = self.ws.tensor("logits", (T, self.cfg.n_experts), torch.float32)
        self._pre = {"layer": layer, "T": T, "targets": targets}
        return h1, x, logits

    def _ids_w(self):
        T, K = self._pre["T"], self.cfg.top_k
        ids = self.ws.tensor("ids", (T, K), torch.int32)
        with torch.cuda.stream(self.stream):
            ids_np = ids.cpu().numpy().astype(np.int64)          # the routing sync
        return ids_np, self.ws.tensor("weights", (T, K), torch.float32)

    def route(self, logits):
        """Routing of the last `pre_moe` (computed there on the device)."""
        return self._ids_w()

    def route_and_forecast(self, logits, h_res, targets: Sequence[int]):
        ids, w = self._ids_w()
        have = self._pre["targets"]
        fp = self.ws.tensor("fprobs", (max(len(have), 1), self.cfg.n_experts), torch.float32)
        with torch.cuda.stream(self.stream):
            fp_np = fp.cpu().numpy()
        return ids, w, {t: fp_np[have.index(t)].copy() for t in targets if t in have}

    # ---------------------------------------------------------------- experts
    def moe_ready(self, layer: int, x, ids: np.ndarray, memory: CudaExpertMemory, ready: Dict[int, int]):
        """Start the routed columns whose experts are already in memory."""
        cols = [j for j in range(ids.shape[1]) if int(ids[0, j]) in ready]
        if cols:
            L = self._layer_struct(layer, memory, ready)
            cc = (C.c_int32 * len(cols))(*cols)
            _lib.check(_lib.lib().yn_moe_up(C.byref(self.dims), C.byref(L), None, None, ids.shape[0], cc, len(cols),
                                            self.ws.ptr, self._st()))
        return cols

    def moe_rest(self, layer: int, x, ids: np.ndarray, w, memory: CudaExpertMemory, rows: Dict[int, int],
                 handle) -> torch.Tensor:
        """The remaining columns, then the weighted sum over all k columns in
        column order plus the gated shared expert."""
        cols = set(handle or [])
        rest = [j for j in range(ids.shape[1]) if j not in cols]
        L = self._layer_struct(layer, memory, rows)
        if rest:
            cc = (C.c_int32 * len(rest))(*rest)
            _lib.check(_lib.lib().yn_moe_up(C.byref(self.dims), C.byref(L), None, None, ids.shape[0], cc, len(rest),
                                            self.ws.ptr, self._st()))
        return self._down(L, ids.shape[0])

    def moe(self, layer: int, x, ids: np.ndarray, w, memory: CudaExpertMemory, rows: Dict[int, int],
            sync: bool = True) -> torch.Tensor:
        if not np.isin(ids, np.fromiter(rows.keys(), dtype=np.int64)).all():
            raise NotImplementedError("moe over a partial staging group (prefill sweep) is not built yet")
        L = self._layer_struct(layer, memory, rows)
        _lib.check(_lib.lib().yn_moe_up(C.byref(self.dims), C.byref(L), None, None, ids.shape[0], None, 0,
                                        self.ws.ptr, self._st()))
        out = self._down(L, ids.shape[0])
        if sync:
            self.stream.synchronize()   # slots may be overwritten once this returns
        return out

    def _down(self, L, T: int) -> torch.Tensor:
        out = torch.empty((T, self.cfg.hidden), dtype=torch.bfloat16, device=self.device)
        mode = 1 if self.cfg.shared_inter else 0
        _lib.check(_lib.lib().yn_moe_down(C.byref(self.dims), C.byref(L), None, None, T, None, mode, out.data_ptr(),
                                          self.ws.ptr, self._st()))
        return out

    def moe_finalize(self, layer: int, routed: torch.Tensor) -> torch.Tensor:
        """routed + shared: the shared expert was added with the weighted sum."""
        return routed

    # ------------------------------------------------------ lazy + write fence
    def launch(self, h) -> None:
        ev = torch.cuda.Event()
        ev.record(self.stream)
        self._unfenced = ev

    def fence(self) -> None:
        """Block until every submitted kernel that reads pool slots has finished."""
        if self._unfenced is not None:
            self._unfenced.synchronize()
            self._unfenced = None

    def check_error(self) -> int:
        """Read and clear the device error word (synchronises the stream)."""
        return self.ws.check_error(self.stream)

    def reset(self) -> None:
        self._pre = {}
        self._unfenced = None
