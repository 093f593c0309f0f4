"""CUDA backend for the MoE part of the reference's ModelBackend interface.

Mirrors the hooks `moe_prefetch/orchestrator.py` calls on
`moe_prefetch/mlx_backend.py`:

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
* prompt passes of more than 8 rows route with `yn_rows_route` (bit-identical
  to the single-row routing, row by row; no lookahead routers) and run their
  routed experts as grouped GEMMs on the tensor cores (`yn_tc_experts`), as
  does `moe` with experts missing from `rows` (the prefill sweep's staging
  groups, mlx_backend.py:421-433): the group's (row, column) pairs sorted by
  slot, the contribution of those pairs only. The grouped path takes 4-bit g64
  and 2-bit g64 / g32 routed records; the shared expert of such a pass (its
  activations and gates come from the row routing) runs as one more grouped
  GEMM over every row in `moe_finalize`.

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
        # constant per layer: the dense pointers and record layout of each layer's descriptor
        self._structs = [L.struct() for L in self.layers]
        self._records = [record_struct(cfg.record_spec(l)) for l in range(cfg.n_layers)]
        self._tg: Dict[int, tuple] = {}
        # expert -> slot tables go up through a ring of pinned host rows into a ring of device rows,
        # one row per kernel launch that reads a table; a row is rewritten only after the event
        # recorded behind its last copy has completed (no host sync on the common path)
        n_lut = 8
        E = cfg.n_experts
        self._lut_host = torch.zeros((n_lut, E), dtype=torch.int32, pin_memory=True)
        self._lut_np = self._lut_host.numpy()
        self._lut_dev = torch.zeros((n_lut, E), dtype=torch.int32, device=self.device)
        self._lut_ev = [torch.cuda.Event() for _ in range(n_lut)]
        self._lut_used = [False] * n_lut
        self._lut_i = 0
        self._lut_last = None        # (memory, rows, ring row) of the last table written
        # layer descriptors over (layer, table row, memory), built once: the launches only read them
        self._desc: Dict[tuple, _lib.Layer] = {}
        self._desc_mem: Dict[tuple, object] = {}
        # pinned landing rows for the routing readback (ids, then lookahead probabilities)
        self._ids_host = torch.empty(_lib.YN_MAX_ROWS * cfg.top_k, dtype=torch.int32, pin_memory=True)
        self._fp_host = torch.empty(max(lookahead, 1) * E, dtype=torch.float32, pin_memory=True)
        self._ids_np, self._fp_np = self._ids_host.numpy(), self._fp_host.numpy()
        self._pre: Dict[int, dict] = {}
        self._unfenced: Optional[torch.cuda.Event] = None
        self._route_ws: Optional[torch.Tensor] = None     # yn_rows_route workspace (prompt passes)
        self._route_rows = 0
        self._tc_err = torch.zeros(1, dtype=torch.int32, device=self.device)

    # -------------------------------------------------------------- helpers
    def _st(self) -> int:
        return stream_ptr(self.stream)

    def _targets(self, layer: int) -> List[int]:
        return [t for t in range(layer + 1, layer + 1 + self.lookahead) if t < self.cfg.n_layers]

    def _layer_struct(self, layer: int, memory: CudaExpertMemory, rows: Dict[int, int]) -> _lib.Layer:
        """Layer descriptor whose routed experts live in `memory` at `rows`.
        A table equal to the previous one (moe_rest after a moe_ready that
        had every expert) reuses that device row."""
        last = self._lut_last
        if last is not None and last[0] is memory and last[1] == rows:
            i = last[2]
        else:
            i = self._lut_i
            self._lut_i = (i + 1) % len(self._lut_ev)
            if self._lut_used[i]:
                self._lut_ev[i].synchronize()        # the copy out of this row has run
            lut = self._lut_np[i]
            if rows:   # only the entries of `rows`: a launch reads the table at its routed experts, all in `rows`
                lut[list(rows.keys())] = list(rows.values())
            _lib.check(_lib.lib().yn_memcpy_async(self._lut_dev[i].data_ptr(), self._lut_host[i].data_ptr(),
                                                  lut.nbytes, self._st()))
            self._lut_ev[i].record(self.stream)
            self._lut_used[i] = True
            self._lut_last = (memory, dict(rows), i)
        key = (layer, i, id(memory))
        L = self._desc.get(key)
        if L is None or self._desc_mem.get(key) is not memory:
            L = _lib.Layer.from_buffer_copy(self._structs[layer])
            L.expert_base = memory.arena.base
            L.slot_stride = memory.arena.slot_bytes
            L.n_slots = memory.n
            L.expert_slot = self._lut_dev[i].data_ptr()
            L.record = self._records[layer]
            self._desc[key], self._desc_mem[key] = L, memory
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
        if T > _lib.YN_MAX_ROWS:
            return self._pre_rows(layer, h1)
        if layer not in self._tg:
            t = self._targets(layer)
            self._tg[layer] = (t, (_lib.Layer * len(t))(*[self._structs[j] for j in t]) if t else None)
        targets, tg = self._tg[layer]
        _lib.check(_lib.lib().yn_post_attention(C.byref(self.dims), C.byref(self._structs[layer]),
                                                h1.data_ptr(), T, tg, len(targets), self.ws.ptr, self._st()))
        x = self.ws.tensor("x", (T, self.cfg.hidden), torch.bfloat16)
        logits = self.ws.tensor("logits", (T, self.cfg.n_experts), torch.float32)
        self._pre = {"layer": layer, "T": T, "targets": targets}
        return h1, x, logits

    def _grouped_supported(self, layer: int) -> Optional[str]:
        spec = self.cfg.record_spec(layer)
        if (spec.bits, spec.group_size) not in ((4, 64), (2, 64), (2, 32)):
            return "the grouped expert path needs 4-bit g64 or 2-bit g64 / g32 routed experts"
        if self.cfg.shared_inter and self.cfg.shared_inter != self.cfg.moe_inter:
            return "the grouped path runs the shared expert with shared_inter == moe_inter"
        return None

    def _pre_rows(self, layer: int, h1: torch.Tensor):
        """Prompt pass of T > 8 rows: RMSNorm, router logits, top-k ids and
        weights of every row (`yn_rows_route`). The logits stay in the routing
        workspace (None is returned in their place)."""
        why = self._grouped_supported(layer)
        if why:
            raise NotImplementedError(f"prompt pass of {h1.shape[0]} rows: {why}")
        lib, cfg = _lib.lib(), self.cfg
        T, H, K = h1.shape[0], cfg.hidden, cfg.top_k
        with torch.cuda.stream(self.stream):
            if self._route_ws is None or T > self._route_rows:
                nb = int(lib.yn_rows_route_bytes(C.byref(self.dims), T))
                if not nb:
                    raise ValueError(f"{T} rows: more than the routing workspace supports")
                self._route_ws = torch.zeros(nb, dtype=torch.uint8, device=self.device)
                self._route_rows = T
            x = torch.empty((T, H), dtype=torch.bfloat16, device=self.device)
            ids = torch.empty((T, K), dtype=torch.int32, device=self.device)
            w = torch.empty((T, K), dtype=torch.float32, device=self.device)
        _lib.check(lib.yn_rows_route(C.byref(self.dims), C.byref(self._structs[layer]), h1.data_ptr(), T,
                                     x.data_ptr(), ids.data_ptr(), w.data_ptr(), self._route_ws.data_ptr(),
                                     self._route_ws.numel(), self._st()))
        self._pre = {"layer": layer, "T": T, "targets": [], "rows": (ids, w)}
        return h1, x, None

    def _ids_w(self, fprobs: bool = False):
        T, K = self._pre["T"], self.cfg.top_k
        if "rows" in self._pre:
            ids, w = self._pre["rows"]
            with torch.cuda.stream(self.stream):
                ids_np = ids.cpu().numpy().astype(np.int64)      # the routing sync
            return ids_np, w, None
        lib, st = _lib.lib(), self._st()
        ids = self.ws.tensor("ids", (T, K), torch.int32)
        _lib.check(lib.yn_memcpy_async(self._ids_host.data_ptr(), ids.data_ptr(), T * K * 4, st))
        n_fp = len(self._pre["targets"]) if fprobs else 0
        if n_fp:
            fp = self.ws.tensor("fprobs", (n_fp, self.cfg.n_experts), torch.float32)
            _lib.check(lib.yn_memcpy_async(self._fp_host.data_ptr(), fp.data_ptr(), fp.numel() * 4, st))
        self.stream.synchronize()                                 # the routing sync
        ids_np = self._ids_np[:T * K].reshape(T, K).astype(np.int64)
        fp_np = self._fp_np[:n_fp * self.cfg.n_experts].reshape(n_fp, -1) if n_fp else None
        return ids_np, self.ws.tensor("weights", (T, K), torch.float32), fp_np

    def route(self, logits):
        """Routing of the last `pre_moe` (computed there on the device)."""
        ids, w, _ = self._ids_w()
        return ids, w

    def route_and_forecast(self, logits, h_res, targets: Sequence[int]):
        have = self._pre["targets"]
        ids, w, fp_np = self._ids_w(fprobs=True)
        if fp_np is None:
            return ids, w, {}
        return ids, w, {t: fp_np[have.index(t)].copy() for t in targets if t in have}

    # ---------------------------------------------------------------- experts
    def moe_ready(self, layer: int, x, ids: np.ndarray, memory: CudaExpertMemory, ready: Dict[int, int]):
        """Start the routed columns whose experts are already in memory."""
        cols = [j for j, e in enumerate(ids[0].tolist()) if e in ready]
        if cols:
            L = self._layer_struct(layer, memory, ready)
            cc = (C.c_int32 * len(cols))(*cols)
            _lib.check(_lib.lib().yn_moe_up(C.byref(self.dims), C.byref(L), None, None, ids.shape[0], cc, len(cols),
                                            self.ws.ptr, self._st()))
        return cols

    def moe_rest(self, layer: int, x, ids: np.ndarray, w, memory: CudaExpertMemory, rows: Dict[int, int],
                 handle, h_res: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The remaining columns, then the weighted sum over all k columns in
        column order plus the gated shared expert. With `h_res` (a caller of
        its own, not the reference's orchestrator, whose `moe_finalize` result
        it adds itself) the residual is added in the same kernel, with the
        same rounding as bf16(h_res + moe_finalize(...))."""
        cols = set(handle or [])
        rest = [j for j in range(ids.shape[1]) if j not in cols]
        L = self._layer_struct(layer, memory, rows)
        if rest:
            cc = (C.c_int32 * len(rest))(*rest)
            _lib.check(_lib.lib().yn_moe_up(C.byref(self.dims), C.byref(L), None, None, ids.shape[0], cc, len(rest),
                                            self.ws.ptr, self._st()))
        return self._down(L, ids.shape[0], h_res)

    def moe(self, layer: int, x, ids: np.ndarray, w, memory: CudaExpertMemory, rows: Dict[int, int],
            sync: bool = True) -> torch.Tensor:
        if ids.shape[0] > _lib.YN_MAX_ROWS or not np.isin(ids, np.fromiter(rows.keys(), dtype=np.int64)).all():
            out = self._moe_grouped(layer, x, ids, w, memory, rows)
            if sync:
                self.stream.synchronize()
            return out
        L = self._layer_struct(layer, memory, rows)
        _lib.check(_lib.lib().yn_moe_up(C.byref(self.dims), C.byref(L), None, None, ids.shape[0], None, 0,
                                        self.ws.ptr, self._st()))
        out = self._down(L, ids.shape[0])
        if sync:
            self.stream.synchronize()   # slots may be overwritten once this returns
        return out

    def _moe_grouped(self, layer: int, x, ids: np.ndarray, w, memory: CudaExpertMemory,
                     rows: Dict[int, int]) -> torch.Tensor:
        """Sum over the (row, column) pairs whose expert is in `rows` of
        w * expert(x_row), as one grouped GEMM (mlx_backend.py:421-433): the
        pairs sorted by slot (stable in row-major order), gate/up + SwiGLU and
        down on the tensor cores, then per row the sum over its present
        columns in column order (fp32, one bf16 rounding). Rows without a
        present pair are zero."""
        why = self._grouped_supported(layer)
        if why:
            raise NotImplementedError(why)
        lib, cfg = _lib.lib(), self.cfg
        T, K = ids.shape
        H, I = cfg.hidden, cfg.moe_inter
        keys = np.fromiter(rows.keys(), dtype=np.int64, count=len(rows))
        lut = np.full(cfg.n_experts, -1, np.int64)
        lut[keys] = np.fromiter(rows.values(), dtype=np.int64, count=len(rows))
        t_idx, j_idx = np.nonzero(np.isin(ids, keys))
        with torch.cuda.stream(self.stream):
            out = torch.zeros((T, H), dtype=torch.bfloat16, device=self.device)
        n = len(t_idx)
        if n == 0:
            return out
        order = np.argsort(lut[ids[t_idx, j_idx]], kind="stable")
        t_idx, j_idx = t_idx[order], j_idx[order]
        e_of = ids[t_idx, j_idx]
        pair_of = np.full((T, K), -1, np.int64)
        pair_of[t_idx, j_idx] = np.arange(n)
        from .prefill import DOWN_ROWS, TILE_ROWS, UP_UNITS
        # chunks of at most TILE_ROWS pairs of one expert, then per chunk the gate/up and down tiles
        starts = np.flatnonzero(np.r_[True, e_of[1:] != e_of[:-1]])
        ends = np.r_[starts[1:], n]
        nch = (ends - starts + TILE_ROWS - 1) // TILE_ROWS
        run = np.repeat(np.arange(len(starts)), nch)
        p0 = starts[run] + (np.arange(len(run)) - np.repeat(np.cumsum(nch) - nch, nch)) * TILE_ROWS
        chunk = np.stack([e_of[starts][run], p0, np.minimum(TILE_ROWS, ends[run] - p0)], axis=1)

        def tiles(step_units, total):
            offs = np.arange(0, total, step_units)
            return np.concatenate([np.repeat(chunk, len(offs), axis=0),
                                   np.tile(offs, len(chunk))[:, None]], axis=1)
        up, dn = tiles(UP_UNITS, I), tiles(DOWN_ROWS, H)
        pad4 = lambda a: np.r_[a, np.zeros(-len(a) % 4, np.int64)]     # 16-byte aligned sections
        sec = [pad4(t_idx), pad4(pair_of.reshape(-1)), up.reshape(-1), dn.reshape(-1)]
        plan = np.concatenate(sec).astype(np.int32)
        L = self._layer_struct(layer, memory, rows)
        D, st = C.byref(self.dims), self._st()
        with torch.cuda.stream(self.stream):
            dev = torch.from_numpy(plan).pin_memory().to(self.device, non_blocking=True)
            x16 = torch.empty((n, H), dtype=torch.float16, device=self.device)
            act = torch.empty((n, I), dtype=torch.bfloat16, device=self.device)
            y = torch.empty((n, H), dtype=torch.bfloat16, device=self.device)
        p_row = dev.data_ptr()
        p_of = p_row + 4 * len(sec[0])
        p_up = p_of + 4 * len(sec[1])
        p_dn = p_up + 4 * len(sec[2])
        err = self._tc_err.data_ptr()
        bits = cfg.record_spec(layer).bits
        _lib.check(lib.yn_gather_kperm(x.data_ptr(), p_row, n, H, bits, 1, x16.data_ptr(), st))
        _lib.check(lib.yn_tc_experts(D, C.byref(L), 0, p_up, len(up), None, x16.data_ptr(), n, act.data_ptr(), None,
                                     err, st))
        _lib.check(lib.yn_tc_experts(D, C.byref(L), 1, p_dn, len(dn), None, act.data_ptr(), n, None, y.data_ptr(),
                                     err, st))
        _lib.check(lib.yn_pairs_combine(D, y.data_ptr(), p_of, w.data_ptr(), None, None, T, out.data_ptr(), st))
        return out

    def _down(self, L, T: int, h_res: Optional[torch.Tensor] = None) -> torch.Tensor:
        out = torch.empty((T, self.cfg.hidden), dtype=torch.bfloat16, device=self.device)
        mode = 2 if h_res is not None else (1 if self.cfg.shared_inter else 0)
        _lib.check(_lib.lib().yn_moe_down(C.byref(self.dims), C.byref(L), None, None, T,
                                          h_res.data_ptr() if h_res is not None else None, mode, out.data_ptr(),
                                          self.ws.ptr, self._st()))
        return out

    def moe_finalize(self, layer: int, routed: torch.Tensor) -> torch.Tensor:
        """routed + shared. Passes of at most 8 rows added the shared expert
        with the weighted sum (yn_moe_down); a prompt pass of more rows adds it
        here: bf16(routed + bf16(sigmoid(g) * shared(x)))."""
        if "rows" not in self._pre or not self.cfg.shared_inter:
            return routed
        return self._shared_rows(self._pre["layer"], routed)

    def _shared_layer(self, layer: int) -> _lib.Layer:
        """The shared expert's down matrix as a one-slot 'expert' of 8-bit
        records for the grouped down GEMM (pieces at their own addresses)."""
        L = _lib.Layer.from_buffer_copy(self._structs[layer])
        m = self.layers[layer].shared[2]
        L.expert_base = m.w.data_ptr()
        L.slot_stride = 16
        L.n_slots = 1
        L.expert_slot = None
        r = _lib.Record()
        r.bits, r.group_size = 8, self.cfg.dense_group
        r.piece_offset[6] = 0
        r.piece_offset[7] = m.s.data_ptr() - m.w.data_ptr()
        r.piece_offset[8] = m.b.data_ptr() - m.w.data_ptr()
        r.record_bytes = m.w.numel() * 4
        L.record = r
        return L

    def _shared_rows(self, layer: int, routed: torch.Tensor) -> torch.Tensor:
        lib, cfg = _lib.lib(), self.cfg
        T, H, K, I = routed.shape[0], cfg.hidden, cfg.top_k, cfg.shared_inter
        D, st = C.byref(self.dims), self._st()
        act_p, sg_p = C.c_void_p(), C.c_void_p()
        _lib.check(lib.yn_rows_route_shared(D, T, self._route_ws.data_ptr(), C.byref(act_p), C.byref(sg_p)))
        from .prefill import DOWN_ROWS, TILE_ROWS
        tiles = np.array([(0, p0, min(TILE_ROWS, T - p0), u0) for p0 in range(0, T, TILE_ROWS)
                          for u0 in range(0, H, DOWN_ROWS)], np.int32)
        with torch.cuda.stream(self.stream):
            dev_tiles = torch.from_numpy(tiles).pin_memory().to(self.device, non_blocking=True)
            act = torch.empty((T, I), dtype=torch.bfloat16, device=self.device)
            y = torch.empty((T, H), dtype=torch.bfloat16, device=self.device)
            term = torch.empty_like(y)
            out = torch.empty_like(routed)
            none = torch.full((T, K), -1, dtype=torch.int32, device=self.device)
        _lib.check(lib.yn_gather_kperm(act_p.value, None, T, I, 8, 0, act.data_ptr(), st))
        L = self._shared_layer(layer)
        _lib.check(lib.yn_tc_experts(D, C.byref(L), 1, dev_tiles.data_ptr(), len(tiles), None, act.data_ptr(), T, None,
                                     y.data_ptr(), self._tc_err.data_ptr(), st))
        _lib.check(lib.yn_scale_rows(y.data_ptr(), sg_p.value, T, H, term.data_ptr(), st))
        _ids, w = self._pre["rows"]
        _lib.check(lib.yn_pairs_combine(D, y.data_ptr(), none.data_ptr(), w.data_ptr(), term.data_ptr(),
                                        routed.data_ptr(), T, out.data_ptr(), st))
        return out

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
        """Read and clear the device error words (synchronises the stream)."""
        code = self.ws.check_error(self.stream)
        self.stream.synchronize()
        tc = int(self._tc_err.item())
        self._tc_err.zero_()
        rc = 0
        if self._route_ws is not None:
            v = C.c_int32(0)
            _lib.check(_lib.lib().yn_route_error(self._route_ws.data_ptr(), C.byref(self.dims), self._st(),
                                                 C.byref(v)))
            rc = v.value
        return code or tc or rc

    def reset(self) -> None:
        self._pre = {}
        self._unfenced = None
