"""Streaming decode: an HBM slot pool in front of a pinned host tier.

The pool path of moe_prefetch/orchestrator.py:158-300 on CUDA streams:

* every routed expert record lives in pinned host memory (the host tier,
  standing in for the reference's SSD records, io_lanes.py:121-139);
* the HBM pool (`SlotPool` over `CudaExpertMemory`) holds a fraction of them;
* per layer: routing on the device (`pre_moe` + `route_and_forecast`, one host
  sync for the ids), then the pool classifies each routed expert as a hit, an
  adopted forecast or a demand miss; misses are copied host -> slot on the copy
  stream (one cudaMemcpyAsync per record) and the compute stream waits for
  them on the device (an event), not on the host;
* resident experts start first (`moe_ready`) while the misses are in flight;
* the lookahead probabilities of layers l+1, l+2 select candidates
  (`RouterForecast.select`, probability >= threshold, at most `issue_cap` per
  target) that are reserved in the speculative partition and copied on a
  second stream (io_lanes.py:271-362 `SpeculativeScheduler`); a forecast that
  is demanded is adopted in place and the compute stream waits for its copy
  if it is still in flight; unused forecasts go back to the partition once
  their target layer has passed;
* before a copy into a slot that compute may have read, the copy stream waits
  for the compute stream's last layer (slot reuse is ordered on the device).

Statistics: pool hit rate, bytes copied, device time the compute stream spent
waiting for demand copies (stall) and the time the copy streams were busy.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib
from .backend import CudaMoEBackend
from .device import ExpertArena, fill_synthetic_experts, stream_ptr
from .forecast import RouterForecast
from .pool import SlotPool
from .synthetic import StackConfig


class HostTier:
    """Every routed record of every layer in pinned host memory:
    layer l's records at base_l + e * record_bytes_l."""

    def __init__(self, cfg: StackConfig, device, layers: Optional[List[int]] = None):
        self.cfg = cfg
        self.layers = list(range(cfg.n_layers)) if layers is None else list(layers)
        self.buf: Dict[int, torch.Tensor] = {}
        self.rec: Dict[int, int] = {}
        for l in self.layers:
            spec = cfg.record_spec(l)
            rb = spec.record_bytes
            arena = ExpertArena(cfg.n_experts, rb, device)        # seeded records generated on the device
            fill_synthetic_experts(arena, cfg, l)
            host = torch.empty(cfg.n_experts * rb, dtype=torch.uint8, pin_memory=True)
            host.copy_(arena.buf)
            del arena
            self.buf[l], self.rec[l] = host, rb

    def record_ptr(self, layer: int, expert: int) -> int:
        return self.buf[layer].data_ptr() + expert * self.rec[layer]

    @property
    def nbytes(self) -> int:
        return sum(b.numel() for b in self.buf.values())


@dataclass
class StreamStats:
    tokens: int = 0
    layers: int = 0
    demand_records: int = 0
    spec_records: int = 0
    bytes_copied: int = 0
    stall_ms: float = 0.0          # compute stream waiting for demand copies (device time)
    copy_busy_ms: float = 0.0      # demand + speculative copy time on the copy streams (device time)
    _pending: list = field(default_factory=list)


class StreamingDecoder:
    def __init__(self, cfg: StackConfig, slot_fraction: float = 0.2, spec_slot_cap: int = 64, lookahead: int = 2,
                 threshold: float = 0.062, issue_cap: int = 32, top: int = 24, device="cuda",
                 host: Optional[HostTier] = None, measure: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        self.compute = torch.cuda.Stream(self.device)
        self.copy = torch.cuda.Stream(self.device)
        self.spec = torch.cuda.Stream(self.device)
        self.be = CudaMoEBackend(cfg, self.device, lookahead=lookahead, stream=self.compute)
        slots = max(int(round(slot_fraction * cfg.n_experts * cfg.n_layers)), 3 * cfg.top_k + spec_slot_cap)
        self.pool = SlotPool(self.be.geometry, slots, spec_slot_cap=spec_slot_cap,
                             memory=self.be.make_expert_memory(slots))
        self.fc = RouterForecast(self.be.geometry)
        self.host = host if host is not None else HostTier(cfg, self.device)
        self.threshold, self.cap, self.top = threshold, issue_cap, top
        self.tickets: Dict[Tuple[int, int], Tuple[int, torch.cuda.Event]] = {}
        self.ev_compute: Optional[torch.cuda.Event] = None
        self.stats = StreamStats()
        self.measure = measure
        self.trace: Optional[List[np.ndarray]] = None   # routed ids per layer, when set to a list

    # ------------------------------------------------------------- copies
    def _copy(self, stream, pairs: List[Tuple[int, int]], layer: int) -> Optional[torch.cuda.Event]:
        """Host records of `layer` -> slots, on `stream` after the last compute."""
        if not pairs:
            return None
        if self.ev_compute is not None:
            stream.wait_event(self.ev_compute)
        ev0 = torch.cuda.Event(enable_timing=True) if self.measure else None
        ev1 = torch.cuda.Event(enable_timing=True)
        if ev0 is not None:
            ev0.record(stream)
        n = len(pairs)
        sl = (C.c_int32 * n)(*[s for _, s in pairs])
        src = (C.c_void_p * n)(*[self.host.record_ptr(layer, e) for e, _ in pairs])
        mem = self.pool.memory
        _lib.check(_lib.lib().yn_slot_copy(mem.arena.base, mem.arena.slot_bytes, sl, src, n, self.host.rec[layer],
                                           stream_ptr(stream)))
        ev1.record(stream)
        self.stats.bytes_copied += n * self.host.rec[layer]
        if ev0 is not None:
            self.stats._pending.append(("busy", ev0, ev1))
        return ev1

    # -------------------------------------------------------------- layers
    def layer(self, l: int, h: torch.Tensor) -> torch.Tensor:
        be, pool = self.be, self.pool
        h_res, x, logits = be.pre_moe(l, h)
        targets = [t for t in (l + 1, l + 2) if t < self.cfg.n_layers]
        ids, w, probs = be.route_and_forecast(logits, h_res, targets)
        if self.trace is not None:
            self.trace.append(ids[0].copy())
        self.fc.observe(l, ids)
        pool.drain_returned()
        out: Dict[int, int] = {}
        ready: Dict[int, int] = {}
        misses: List[Tuple[int, int]] = []
        waits: List[torch.cuda.Event] = []
        for e in sorted({int(v) for v in ids.reshape(-1)}):
            key = (l, e)
            s = pool.hit(key)
            if s is not None:
                out[e] = ready[e] = s
                continue
            t = self.tickets.pop(key, None)
            if t is not None:
                s, ev = t
                pool.adopt(s, key)
                out[e] = s
                if ev.query():
                    ready[e] = s
                else:
                    waits.append(ev)
                continue
            s = pool.claim_for_demand(key)
            out[e] = s
            misses.append((e, s))
        ev_demand = self._copy(self.copy, misses, l)
        self.stats.demand_records += len(misses)
        handle = be.moe_ready(l, x, ids, pool.memory, ready)
        ev_ready = None
        if ev_demand is not None or waits:
            if self.measure and ev_demand is not None:
                ev_ready = torch.cuda.Event(enable_timing=True)
                ev_ready.record(self.compute)
            if ev_demand is not None:
                self.compute.wait_event(ev_demand)
            for ev in waits:
                self.compute.wait_event(ev)
        routed = be.moe_rest(l, x, ids, w, pool.memory, out, handle)
        with torch.cuda.stream(self.compute):
            h_next = h_res + be.moe_finalize(l, routed)
        if ev_ready is not None:
            self.stats._pending.append(("stall", ev_ready, ev_demand))
        self.ev_compute = torch.cuda.Event()
        self.ev_compute.record(self.compute)
        for e, s in misses:
            pool.publish(s, (l, e))
        for s in out.values():
            pool.unpin(s)
        # forecasts for the next layers, copied while this layer computes
        for t in targets:
            if t not in probs:
                continue
            cands = self.fc.select(t, probs[t], self.top)
            issued, pairs = 0, []
            for e, p in cands:
                if p < self.threshold or (t, e) in self.tickets or pool.is_resident((t, e)):
                    continue
                if issued >= self.cap:
                    break
                s = pool.reserve_speculative((t, e))
                if s is None:
                    break
                pairs.append((e, s))
                issued += 1
            ev = self._copy(self.spec, pairs, t)
            for e, s in pairs:
                self.tickets[(t, e)] = (s, ev)
            self.stats.spec_records += len(pairs)
        for key in [k for k in self.tickets if k[0] <= l]:
            pool.return_speculative(self.tickets.pop(key)[0])
        self.stats.layers += 1
        return h_next

    def token(self, h: torch.Tensor) -> torch.Tensor:
        for l in range(self.cfg.n_layers):
            h = self.layer(l, h)
        for key in list(self.tickets):
            self.pool.return_speculative(self.tickets.pop(key)[0])
        self.stats.tokens += 1
        return h

    def decode(self, inputs: torch.Tensor, outputs: torch.Tensor) -> None:
        """Sequential bs1 decode of inputs (N, H) -> outputs (N, H)."""
        self.compute.wait_stream(torch.cuda.current_stream(self.device))
        for t in range(inputs.shape[0]):
            out = self.token(inputs[t:t + 1])
            with torch.cuda.stream(self.compute):
                outputs[t:t + 1].copy_(out)
        torch.cuda.current_stream(self.device).wait_stream(self.compute)

    def collect(self) -> StreamStats:
        """Synchronise and turn recorded events into device times."""
        torch.cuda.synchronize(self.device)
        for kind, a, b in self.stats._pending:
            ms = a.elapsed_time(b)
            if kind == "busy":
                self.stats.copy_busy_ms += ms
            else:
                self.stats.stall_ms += max(0.0, ms)
        self.stats._pending = []
        return self.stats

    def reset_stats(self) -> None:
        """Start counting afresh (after a warm-up that filled the pool)."""
        self.collect()
        self.stats = StreamStats()
        self.pool.stats = type(self.pool.stats)()
        self.fc.stats = type(self.fc.stats)()

    def report(self, seconds: float) -> dict:
        st = self.collect()
        ps = self.pool.stats
        hidden = 1.0 - st.stall_ms / st.copy_busy_ms if st.copy_busy_ms > 0 else 1.0
        return {"tokens": st.tokens, "tok_s": st.tokens / seconds if seconds > 0 else 0.0,
                "pool_slots": self.pool.slots, "spec_slots": self.pool.spec_slot_cap,
                "hit_rate": ps.hit_rate, "hits": ps.hits, "misses": ps.misses, "adopted": ps.adopted,
                "spec_reserved": ps.spec_reserved, "spec_discarded": ps.spec_discarded,
                "forecast_recall": self.fc.stats.recall,
                "demand_records": st.demand_records, "spec_records": st.spec_records,
                "h2d_gb": st.bytes_copied / 1e9, "h2d_gbs": st.bytes_copied / 1e9 / seconds if seconds > 0 else 0.0,
                "stall_ms": st.stall_ms, "copy_busy_ms": st.copy_busy_ms, "hidden_fraction": hidden}
