"""Scan-resistant prefill sweep over the HBM slot pool (moe_prefetch/sweep.py:80-138).

A prompt pass of `min_tokens` rows or more does not go through the pool's
demand path (orchestrator.py:322-337). Per MoE layer:

1. the layer's routed experts, sorted by id, are cut into staging groups of
   `group` (32);
2. for each group, the experts resident in the pool are copied out of it
   (reference bits untouched: a prompt says nothing about decode locality) and
   the rest are read from the host tier, one read per run of consecutive ids;
3. the group runs as one grouped GEMM over its (row, column) pairs sorted by
   expert (`CudaMoEBackend.moe` with a partial `rows`: the tensor-core kernel);
4. the reads of group g+1 overlap the GEMM of group g: two staging buffers.

The sweep never writes the pool except on the final prompt pass, which admits
each layer's fair share (slots // layers) of its most frequently routed
experts from staging (`SlotPool.admit`). Group composition depends on routing
alone, never on residency, so the arithmetic is identical on a cold and a warm
pool.

On the device (`streams` given) host-tier reads and admissions run on a copy
stream, pool -> staging copies and the GEMMs on the compute stream, ordered by
events instead of host waits:

* at the start of a layer the copy stream waits for the compute stream (the
  pool slots and the layer's rows are final; an admitted record may replace a
  slot an earlier layer read);
* a group's reads are issued before its pool copies, so the host link starts
  at once; the group's `futures` are events on the copy stream, and `result()`
  makes the compute stream wait for them on the device;
* before a staging buffer is refilled (group g+2) the copy stream waits for the
  GEMM of group g, which read it (the compute stream's own copies follow it
  in stream order);
* admitted records are copied staging -> pool slot on the copy stream after it
  has waited for the compute stream (pool copies queued there read their slots
  first), and the compute stream waits for the copy stream at the end of the
  layer.

Without `streams` (host memory, the reference's arrangement) copies are
synchronous and futures are whatever the reader returns.
"""
from __future__ import annotations

import contextlib
import time
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np

GROUP = 32


@dataclass
class SweepStats:
    """Counters of the sweeps run so far. `passes` is advanced by the caller
    after a whole prompt pass (the reference's orchestrator does the same)."""
    passes: int = 0
    layers: int = 0
    pool_copies: int = 0        # staged records copied out of the pool
    host_records: int = 0       # staged records read from the host tier
    admitted: int = 0           # records written into the pool by final passes
    read_wait_s: float = 0.0    # host time spent waiting for staged records


@dataclass
class SweepPlan:
    """What the sweep does for one layer, decided from its routing alone:
    `experts`, the distinct routed experts in ascending id order, cut into
    consecutive `groups` of at most the staging size; `admit`, the experts a
    final pass writes into the pool: the layer's fair share of its most used
    experts (routing count descending, lower id first on equal counts)."""
    layer: int
    experts: List[int]
    groups: List[List[int]]
    admit: frozenset

    @classmethod
    def build(cls, layer: int, ids: np.ndarray, group: int, share: int, admit: bool) -> "SweepPlan":
        experts, counts = np.unique(np.asarray(ids), return_counts=True)
        chosen = experts[np.argsort(-counts, kind="stable")[:share]] if admit else experts[:0]
        ex = experts.tolist()
        return cls(layer, ex, [ex[i:i + group] for i in range(0, len(ex), group)],
                   frozenset(int(e) for e in chosen))


def _is_torch(v) -> bool:
    return hasattr(v, "data_ptr") and hasattr(v, "copy_")


def copy_record(dst: Sequence, src: Sequence) -> None:
    """Copy one record given as lists of piece buffers (pool.py:85-87).
    Device tensors (uint8 views of one slot, in record order): one
    asynchronous copy on the current stream of the span from the first piece's
    start to the end of the last (a slot holds the record's bytes in their
    on-disk layout, padding included); a record of a smaller layer format
    (mixed-bit stacks) fills the front of a larger slot. Host buffers: slice
    assignment."""
    if dst and _is_torch(dst[0]):
        def flat(parts):
            p0 = parts[0].data_ptr()
            span = max(t.data_ptr() + t.numel() * t.element_size() for t in parts) - p0
            return parts[0].as_strided((span,), (1,))
        d, s = flat(dst), flat(src)
        m = min(d.numel(), s.numel())
        d[:m].copy_(s[:m], non_blocking=True)
        return
    for a, b in zip(dst, src):
        a[:] = b


class DeviceFuture:
    """Completion of copies enqueued on a copy stream. `result()` makes the
    compute stream wait for them on the device (no host wait); `done()`
    polls."""

    def __init__(self, event, compute_stream):
        self.event, self.compute = event, compute_stream

    def result(self, timeout=None):
        self.compute.wait_event(self.event)

    def done(self) -> bool:
        return self.event.query()


class SweepStreams:
    """Copy and compute streams of a device sweep."""

    def __init__(self, compute=None, copy=None, device="cuda"):
        import torch
        self.compute = compute or torch.cuda.current_stream(device)
        self.copy = copy or torch.cuda.Stream(device)

    def event(self, stream):
        import torch
        ev = torch.cuda.Event()
        ev.record(stream)
        return ev


class HostSlabMemory:
    """n host slots of `slot_bytes` holding one record each (pool.py:66-82)."""

    def __init__(self, n: int, record_bytes: int, slot_bytes: int):
        self.n, self.record_bytes, self.slot_bytes = n, record_bytes, slot_bytes
        self._buf = bytearray(max(1, n * slot_bytes))
        self._view = memoryview(self._buf)

    def views(self, i: int) -> List[memoryview]:
        s = i * self.slot_bytes
        return [self._view[s:s + self.record_bytes]]

    def close(self) -> None:
        self._view.release()


class StagingBuffer:
    """One of the two staging buffers: `memory` is laid out like pool memory,
    so the backend's `moe` runs on it as on the pool, with staging slot i
    holding `experts[i]` of the group it was filled with."""

    def __init__(self, memory):
        self.memory = memory
        self.slot_of: Dict[int, int] = {}
        self.pending: List = []          # futures of the records still arriving
        self.gemm_done = None            # device event after the GEMM that last read it

    def fill_order(self, experts: List[int]) -> None:
        self.slot_of = {e: i for i, e in enumerate(experts)}

    def views(self, e: int):
        return self.memory.views(self.slot_of[e])


class HostTierReader:
    """Reads routed records from the pinned host tier into staging slots on
    the copy stream (the sweep half of io_lanes.py:145-173 `runs` /
    `submit_runs`): runs of consecutive expert ids, one asynchronous copy per
    record, one future per run."""

    def __init__(self, tier, streams: SweepStreams):
        self.tier, self.streams = tier, streams
        self.sweep_runs = 0
        self.sweep_records = 0

    @staticmethod
    def runs(experts: Sequence[int]) -> List[List[int]]:
        """Sorted ids split into runs of consecutive ids (records contiguous in the tier)."""
        out: List[List[int]] = []
        for e in experts:
            if out and e == out[-1][-1] + 1:
                out[-1].append(e)
            else:
                out.append([e])
        return out

    def submit_runs(self, layer: int, experts: Sequence[int], dst_for: Callable[[int], List]) -> List[DeviceFuture]:
        import torch
        futs = []
        rb = self.tier.rec[layer]
        host = self.tier.buf[layer]
        with torch.cuda.stream(self.streams.copy):
            for run in self.runs(list(experts)):
                for e in run:
                    copy_record(dst_for(e), [host[e * rb:(e + 1) * rb]])
                futs.append(DeviceFuture(self.streams.event(self.streams.copy), self.streams.compute))
                self.sweep_runs += 1
                self.sweep_records += len(run)
        return futs


class PrefillSweep:
    """Prompt-pass sweep of `pool` (a `SlotPool`). reader: `submit_runs(layer,
    experts, dst_for)` -> futures; make_memory(n): staging memory of n slots
    laid out like the pool's (default: host slabs); streams: `SweepStreams`
    for device memory, None for host memory. The constructor and `run_layer`
    are the surface the reference's orchestrator calls
    (orchestrator.py:322-337)."""

    def __init__(self, pool, reader, min_tokens: int = 16, group: int = GROUP,
                 make_memory: Optional[Callable[[int], object]] = None, streams: Optional[SweepStreams] = None):
        self.pool, self.reader = pool, reader
        self.min_tokens, self.group = min_tokens, group
        if make_memory is None:
            g = pool.g
            make_memory = lambda n: HostSlabMemory(n, g.expert_nbytes, g.slot_nbytes)
        self.streams = streams
        self.ring = [StagingBuffer(make_memory(group)) for _ in range(2)]
        self.stats = SweepStats()

    def fair_share(self) -> int:
        """Pool slots a final pass may fill per layer."""
        return self.pool.slots // self.pool.g.total_moe_layers

    def plan(self, layer: int, ids: np.ndarray, admit: bool) -> SweepPlan:
        return SweepPlan.build(layer, ids, self.group, self.fair_share(), admit)

    # ----------------------------------------------------------- staging
    def stage(self, buf: StagingBuffer, layer: int, experts: List[int]) -> None:
        """Fill `buf` with `experts`: the host-tier reads of those not in the
        pool are started first, then the resident ones are copied out of the
        pool (their reference bits are left alone: a prompt says nothing
        about what decode will reuse). On the device the reads go on the copy
        stream after the GEMM that last read this buffer, the pool copies on
        the compute stream."""
        dev = self.streams
        if dev is not None and buf.gemm_done is not None:
            dev.copy.wait_event(buf.gemm_done)
        buf.fill_order(experts)
        resident = [(e, self.pool.lookup((layer, e))) for e in experts]
        from_host = [e for e, s in resident if s is None]
        buf.pending = list(self.reader.submit_runs(layer, from_host, buf.views))
        if dev is not None:
            buf.pending.append(DeviceFuture(dev.event(dev.copy), dev.compute))
        self.stats.host_records += len(from_host)
        for e, s in resident:
            if s is not None:
                copy_record(buf.views(e), self.pool.views(s))
                self.stats.pool_copies += 1

    def _admit(self, buf: StagingBuffer, layer: int, members: List[int]) -> None:
        """Write `members` from staging into the pool (CLOCK victims). On the
        device: on the copy stream, after the compute stream (whose queued
        pool copies read the victims' old records first)."""
        dev = self.streams
        if dev is not None:
            dev.copy.wait_stream(dev.compute)
        ctx = contextlib.nullcontext()
        if dev is not None:
            import torch
            ctx = torch.cuda.stream(dev.copy)
        with ctx:
            self.stats.admitted += self.pool.admit(layer, members, len(members),
                                                   lambda e, dst: copy_record(dst, buf.views(e)))

    # ----------------------------------------------------------- execution
    def run_layer(self, layer: int, x, ids: np.ndarray, w, moe: Callable, admit: bool):
        """The routed contribution of every (row, column) of `ids`, one grouped
        `moe(layer, x, ids, w, staging_memory, {expert: staging slot})` per
        staging group, group g+1 staged while group g computes; a final pass
        (`admit`) also writes the plan's admitted experts into the pool."""
        dev = self.streams
        if dev is not None:
            dev.copy.wait_stream(dev.compute)     # pool contents and this layer's rows are final
        plan = self.plan(layer, ids, admit)
        self.stage(self.ring[0], layer, plan.groups[0])
        total = None
        for gi, experts in enumerate(plan.groups):
            buf = self.ring[gi % 2]
            if gi + 1 < len(plan.groups):
                self.stage(self.ring[(gi + 1) % 2], layer, plan.groups[gi + 1])
            t0 = time.perf_counter()
            for f in buf.pending:
                f.result()
            self.stats.read_wait_s += time.perf_counter() - t0
            part = moe(layer, x, ids, w, buf.memory, dict(buf.slot_of))
            if dev is not None:
                buf.gemm_done = dev.event(dev.compute)
            total = part if total is None else total + part
            if plan.admit:
                self._admit(buf, layer, [e for e in experts if e in plan.admit])
        if dev is not None:
            dev.compute.wait_stream(dev.copy)
        self.stats.layers += 1
        return total

    def close(self):
        for buf in self.ring:
            buf.memory.close()


def prompt_pass(backend, sweep: PrefillSweep, h, admit: bool = True, layers: Optional[Sequence[int]] = None):
    """The sweep branch of the orchestrator's forward (orchestrator.py:322-337)
    over the MoE half of each layer: `pre_moe`, routing (one host sync for the
    ids), the sweep, `moe_finalize`, residual. Staging reuse is ordered on the
    device, so the backend's `moe` runs without its host synchronisation."""
    import functools
    moe = functools.partial(backend.moe, sync=False)
    for layer in (range(backend.cfg.n_layers) if layers is None else layers):
        h_res, x, logits = backend.pre_moe(layer, h)
        ids, w = backend.route(logits)
        h = h_res + backend.moe_finalize(layer, sweep.run_layer(layer, x, ids, w, moe, admit))
    sweep.stats.passes += 1
    return h
