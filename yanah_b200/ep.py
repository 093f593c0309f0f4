"""Batch decode with the routed experts grouped by expert, and expert
parallelism over peer memory (one process per GPU).

A decode step moves a batch of B token rows (at most 64) through every layer.
With `world` ranks, rank r holds the routed experts [r*E/world,
(r+1)*E/world) of every layer (their records only) plus all dense weights, and
owns B/world "home" rows. Per layer (``yn_ep_layer``): post-attention and
routing of the home rows; the rows and their ids go to every rank's gather
buffer (peer stores); each rank computes the pairs of its experts for every
row, reading each expert record once (union of experts); each output row is
stored into its home rank's buffer; the home rank combines in column order.
Outputs are bit-identical for every `world` (the same arithmetic per pair,
the same combine order), so routing stays identical across GPU counts.

The reference runs one MLX device and has no expert parallelism; the batch
path mirrors its union-of-experts batch decode (orchestrator.py:361-405
`generate_batch`, mlx_backend.py:411-436 `moe` with :111-123 `_gather_sort`).
Peer buffers are plain cudaMalloc memory shared with CUDA IPC handles; the
handles travel through ``torch.distributed`` (any backend).
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from .device import DeviceLayer, ExpertArena, dims_struct, fill_synthetic_experts, stream_ptr
from .synthetic import StackConfig, dense_layer

MAX_BATCH_ROWS = 64
MAX_RANKS = 8


def expert_range(n_experts: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous expert ids held by `rank` (the remainder goes to the last ranks)."""
    return rank * n_experts // world, (rank + 1) * n_experts // world


def home_rows(batch: int, rank: int, world: int) -> Tuple[int, int]:
    if batch % world:
        raise ValueError(f"batch {batch} is not a multiple of world {world}")
    per = batch // world
    return rank * per, (rank + 1) * per


def plan_pairs(ids: np.ndarray, e_lo: int, e_hi: int):
    """The segment plan the device builds per layer (k_batch_frags, block 0):
    the (row, column) pairs whose expert is in [e_lo, e_hi), grouped by
    expert in ascending id order, pairs of one expert in (row, column) order.
    Returns (experts, offsets, pairs) with pairs as row * K + column."""
    ids = np.asarray(ids)
    K = ids.shape[1]
    flat = ids.reshape(-1)
    sel = np.nonzero((flat >= e_lo) & (flat < e_hi))[0]
    order = sel[np.argsort(flat[sel], kind="stable")]
    experts, counts = np.unique(flat[order], return_counts=True)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    return experts.astype(np.int64), offsets, order.astype(np.int64)


def _exchange_handles(handle: bytes, world: int, group=None) -> List[bytes]:
    import torch.distributed as dist
    out: List[Optional[bytes]] = [None] * world
    dist.all_gather_object(out, handle, group=group)
    return [bytes(h) for h in out]


class ExpertParallelStack:
    """One rank of the batch / expert-parallel decode of a synthetic stack.

    batch: total rows of a step (all ranks); layers: which layers of `cfg`
    (default all). With world > 1, torch.distributed must be initialised and
    every rank constructs its stack collectively (the IPC handle exchange)."""

    def __init__(self, cfg: StackConfig, batch: int = 64, rank: int = 0, world: int = 1, device: str = "cuda",
                 layers: Optional[Sequence[int]] = None, group=None):
        if not 1 <= world <= MAX_RANKS:
            raise ValueError("world must be in [1, 8]")
        if not 1 <= batch <= MAX_BATCH_ROWS:
            raise ValueError("batch must be in [1, 64]")
        self.cfg, self.rank, self.world, self.batch = cfg, rank, world, batch
        self.group = group
        self.sym = None
        self._imported: List[int] = []
        self.device = torch.device(device)
        self.rows = home_rows(batch, rank, world)
        self.rows_per_rank = batch // world
        self.e_lo, self.e_hi = expert_range(cfg.n_experts, rank, world)
        self.layer_ids = list(range(cfg.n_layers)) if layers is None else list(layers)
        self.dims = dims_struct(cfg)
        self.ep = _lib.EpConfig(rank, world, self.rows_per_rank, self.e_lo, self.e_hi, len(self.layer_ids))
        lib = _lib.lib()
        self.arenas: List[ExpertArena] = []
        self.layers: List[DeviceLayer] = []
        local_ids = list(range(self.e_lo, self.e_hi))
        for l in self.layer_ids:
            spec = cfg.record_spec(l)
            arena = ExpertArena(len(local_ids), spec.slot_bytes, self.device)
            fill_synthetic_experts(arena, cfg, l, experts=local_ids)
            self.arenas.append(arena)
            self.layers.append(DeviceLayer(cfg, l, dense_layer(cfg, l), arena, 0, None, self.device))
        self.structs = [L.struct() for L in self.layers]
        # buffers: peer-visible (cudaMalloc for IPC) and private
        self.sym_bytes = int(lib.yn_ep_sym_bytes(C.byref(self.dims), C.byref(self.ep)))
        self.local_bytes = int(lib.yn_ep_local_bytes(C.byref(self.dims), C.byref(self.ep)))
        if not self.sym_bytes or not self.local_bytes:
            _lib.check(_lib.YN_E_INVALID)
        ptr = C.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(lib.yn_device_alloc(self.sym_bytes, C.byref(ptr)))
        self.sym = ptr.value
        self.local = torch.empty(self.local_bytes, dtype=torch.uint8, device=self.device)
        _lib.check(lib.yn_ep_init(self.sym, self.local.data_ptr(), C.byref(self.dims), C.byref(self.ep),
                                  stream_ptr()))
        torch.cuda.synchronize(self.device)
        if world > 1:
            h = (C.c_uint8 * _lib.YN_IPC_HANDLE_BYTES)()
            _lib.check(lib.yn_ipc_export(self.sym, h))
            handles = _exchange_handles(bytes(h), world, group)
            peers = []
            for r, hb in enumerate(handles):
                if r == rank:
                    peers.append(self.sym)
                    continue
                p = C.c_void_p()
                _lib.check(lib.yn_ipc_import((C.c_uint8 * len(hb)).from_buffer_copy(hb), C.byref(p)))
                peers.append(p.value)
                self._imported.append(p.value)
            import torch.distributed as dist
            dist.barrier(group=group)  # every rank's buffers are zeroed and mapped before any peer store
        else:
            peers = [self.sym]
        self.peers = (C.c_void_p * world)(*peers)
        H, T = cfg.hidden, self.rows_per_rank
        self._ping = torch.empty((2, T, H), dtype=torch.bfloat16, device=self.device)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.lview = _lib.EpLocalPtrs()
        _lib.check(lib.yn_ep_view(self.local.data_ptr(), C.byref(self.dims), C.byref(self.ep), C.byref(self.lview)))
        self.sview = _lib.EpSymPtrs()
        _lib.check(lib.yn_ep_sym_view(self.sym, C.byref(self.dims), C.byref(self.ep), C.byref(self.sview)))

    # ------------------------------------------------------------ launches
    def layer(self, i: int, h_in: torch.Tensor, h_out: torch.Tensor, stream=None) -> None:
        """Layer i (index into `layer_ids`) for the home rows."""
        _lib.check(_lib.lib().yn_ep_layer(C.byref(self.dims), C.byref(self.structs[i]), i, C.byref(self.ep),
                                          h_in.data_ptr(), h_out.data_ptr(), self.peers, self.local.data_ptr(),
                                          stream_ptr(stream)))

    def step_end(self, stream=None) -> None:
        _lib.check(_lib.lib().yn_ep_step_end(self.local.data_ptr(), C.byref(self.dims), C.byref(self.ep),
                                             stream_ptr(stream)))

    def _launch_step(self, stream=None) -> None:
        for i in range(len(self.layer_ids)):
            self.layer(i, self._ping[i % 2], self._ping[(i + 1) % 2], stream)
        self.step_end(stream)

    @property
    def out_slot(self) -> int:
        return len(self.layer_ids) % 2

    def step(self, h_home: torch.Tensor, stream=None) -> torch.Tensor:
        """One step of the home rows (rows_per_rank, H) bf16 -> (rows_per_rank, H) bf16."""
        self._ping[0].copy_(h_home)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._launch_step(stream)
        return self._ping[self.out_slot]

    def capture(self) -> None:
        """Capture one whole step (every layer, every kernel) into a CUDA graph."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._launch_step(s)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.graph = g

    # ------------------------------------------------------------ readback
    def check_error(self, stream=None) -> int:
        code = C.c_int32(0)
        _lib.check(_lib.lib().yn_ep_error(self.local.data_ptr(), C.byref(self.dims), C.byref(self.ep),
                                          stream_ptr(stream), C.byref(code)))
        return code.value

    def _tensor(self, addr: int, shape, dtype) -> torch.Tensor:
        n = int(np.prod(shape))
        storage_base = self.local.data_ptr()
        if storage_base <= addr < storage_base + self.local_bytes:
            off = addr - storage_base
            elem = torch.empty((), dtype=dtype).element_size()
            return self.local[off:off + n * elem].view(dtype).view(*shape)
        raise ValueError("address outside the private buffer")

    def home_outputs(self) -> dict:
        """Copies (numpy) of the last layer's home-row intermediates."""
        cfg, T, K, H = self.cfg, self.rows_per_rank, self.cfg.top_k, self.cfg.hidden
        v = self.lview
        out = {
            "x": self._tensor(v.x, (T, H), torch.int16).cpu().numpy().view(np.uint16),
            "ids": self._tensor(v.ids, (T, K), torch.int32).cpu().numpy(),
            "w": self._tensor(v.weights, (T, K), torch.float32).cpu().numpy(),
            "sgate": self._tensor(v.sgate, (T,), torch.float32).cpu().numpy(),
            "ysh": self._tensor(v.y_shared, (T, H), torch.int16).cpu().numpy().view(np.uint16),
        }
        y = np.empty((T, K, H), np.uint16)
        torch.cuda.synchronize(self.device)
        _copy_device_to_host(self.sview.y, y)
        out["y"] = y
        return out

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's peer-visible one.

        With world > 1 this is collective: every rank calls it after its
        last step. Peers store into this rank's buffer during a step, so it
        is freed only after a barrier over the group has shown that every
        rank has finished (its own steps synchronised first). If the process
        group is already gone the peers cannot be waited for, and the buffer
        is left mapped until the process exits rather than freed under them."""
        if self.sym is None and not self._imported:
            return
        lib = _lib.lib()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            import torch.distributed as dist
            if not (dist.is_available() and dist.is_initialized()):
                self._imported, self.sym = [], None
                return
            dist.barrier(group=self.group)
        for p in self._imported:
            lib.yn_ipc_close(p)
        self._imported = []
        if self.sym:
            lib.yn_device_free(self.sym)
            self.sym = None

    def __del__(self):
        # A collective cannot run from the garbage collector (ranks collect at
        # different times), so a multi-rank stack that was not closed keeps its
        # buffer until the process exits.
        if self.world > 1:
            return
        try:
            self.close()
        except Exception:
            pass


def _copy_device_to_host(addr: int, out: np.ndarray) -> None:
    """Copy raw device bytes (outside torch's allocator) into a numpy array."""
    _lib.check(_lib.lib().yn_memcpy(out.ctypes.data, addr, out.nbytes, None))
