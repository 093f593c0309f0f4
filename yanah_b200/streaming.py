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


class PoolPolicy:
    """Host bookkeeping of one pool-path layer, in the order of the reference's
    engine (orchestrator.py:158-214 `_submit_demand` / `_finish_demand`,
    :226-300 `_pool_layer`; io_lanes.py:271-362 `SpeculativeScheduler`), so that
    every slot decision equals the reference's on the same routing:

    1. `classify`: returned forecasts drained; the layer's distinct experts in
       ascending id order are hits (pinned) or forecasts taken into the cache
       (`adopt`); only then are the misses claimed (CLOCK victims, pinned), in
       the same order;
    2. `issue`: per target layer, the selected candidates in descending
       probability: below `threshold` skipped, at most `issue_cap` reserved,
       candidates already forecast or resident skipped, the first refusal of
       the partition ends that target; made while this layer's slots are
       still pinned;
    3. `publish` the misses; 4. `expire` forecasts whose target layer has
       passed (they go back to the partition); 5. `release` (unpin).

    Speculative reads are logically complete when their layer classifies
    (the device waits for a copy still in flight), which is the deterministic
    reading of the reference's engine that cache_sim also assumes."""

    def __init__(self, pool: SlotPool, forecast: RouterForecast, threshold: float = 0.062, issue_cap: int = 32,
                 top: int = 24):
        self.pool, self.fc = pool, forecast
        self.threshold, self.cap, self.top = threshold, issue_cap, top
        self.tickets: Dict[Tuple[int, int], int] = {}   # (target layer, expert) -> partition slot, in issue order

    def classify(self, l: int, ids: np.ndarray):
        """-> (out {expert: slot}, ready {expert: slot} (hits + adopted),
        misses [expert], adopted [expert]). Every slot in `out` is pinned."""
        pool = self.pool
        pool.drain_returned()
        out: Dict[int, int] = {}
        ready: Dict[int, int] = {}
        misses: List[int] = []
        adopted: List[int] = []
        for e in sorted(set(np.asarray(ids).ravel().tolist())):
            key = (l, e)
            s = pool.hit(key)
            if s is None:
                s = self.tickets.pop(key, None)
                if s is None:
                    misses.append(e)
                    continue
                pool.adopt(s, key)
                adopted.append(e)
            out[e] = ready[e] = s
        for e in misses:
            out[e] = pool.claim_for_demand((l, e))
        return out, ready, misses, adopted

    def issue(self, targets: List[int], probs: Dict[int, np.ndarray]):
        """-> ({target: [(expert, slot)] reserved}, {target: candidates})."""
        pool = self.pool
        reserved: Dict[int, List[Tuple[int, int]]] = {}
        cands_of: Dict[int, list] = {}
        for t in targets:
            if t not in probs:
                continue
            cands = self.fc.select(t, probs[t], self.top)
            cands_of[t] = cands
            n, pairs = 0, []
            for e, p in cands[:self.top]:
                if p < self.threshold:
                    continue
                if n >= self.cap:
                    break
                key = (t, e)
                if key in self.tickets or pool.is_resident(key):
                    continue
                s = pool.reserve_speculative(key)
                if s is None:
                    break
                self.tickets[key] = s
                pairs.append((e, s))
                n += 1
            reserved[t] = pairs
        return reserved, cands_of

    def publish(self, l: int, misses: List[int], out: Dict[int, int]) -> None:
        for e in misses:
            self.pool.publish(out[e], (l, e))

    def expire(self, l: int) -> List[Tuple[int, int]]:
        """Forecasts for layers <= l go back unused (in issue order)."""
        dead = [k for k in self.tickets if k[0] <= l]
        for k in dead:
            self.pool.return_speculative(self.tickets.pop(k))
        return dead

    def release(self, out: Dict[int, int]) -> None:
        for s in out.values():
            self.pool.unpin(s)

    def end_token(self) -> None:
        """A new token starts: every outstanding forecast goes back."""
        for k in list(self.tickets):
            self.pool.return_speculative(self.tickets.pop(k))


class StreamingDecoder:
    def __init__(self, cfg: StackConfig, slot_fraction: float = 0.2, spec_slot_cap: int = 64, lookahead: int = 2,
                 threshold: float = 0.062, issue_cap: int = 32, top: int = 24, device="cuda",
                 host: Optional[HostTier] = None, measure: bool = True, slots: Optional[int] = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.compute = torch.cuda.Stream(self.device)
        self.copy = torch.cuda.Stream(self.device)
        self.spec = torch.cuda.Stream(self.device)
        self.be = CudaMoEBackend(cfg, self.device, lookahead=lookahead, stream=self.compute)
        if slots is None:
            slots = max(int(round(slot_fraction * cfg.n_experts * cfg.n_layers)), 3 * cfg.top_k + spec_slot_cap)
        self.pool = SlotPool(self.be.geometry, slots, spec_slot_cap=spec_slot_cap,
                             memory=self.be.make_expert_memory(slots))
        self.fc = RouterForecast(self.be.geometry)
        self.policy = PoolPolicy(self.pool, self.fc, threshold, issue_cap, top)
        self.host = host if host is not None else HostTier(cfg, self.device)
        self.events: Dict[Tuple[int, int], torch.cuda.Event] = {}   # forecast copies in flight
        self.ev_compute: Optional[torch.cuda.Event] = None          # the last layer's kernels
        self._ev_layer = [torch.cuda.Event(), torch.cuda.Event()]   # alternate: the previous layer's stays valid
        self._ev_i = 0
        self.stats = StreamStats()
        self.measure = measure
        self.generation = 0
        # routing trace in the reference's format (orchestrator.py:268-270), when set to a list:
        # (generation, layer, routed experts, {target layer: [(expert, p)]})
        self.trace: Optional[list] = None

    # ------------------------------------------------------------- copies
    def _copy(self, stream, pairs: List[Tuple[int, int]], layer: int,
              after: Optional[torch.cuda.Event]) -> Optional[torch.cuda.Event]:
        """Host records of `layer` -> slots, on `stream` after the compute event `after`."""
        if not pairs:
            return None
        if after is not None:
            stream.wait_event(after)
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
        """One pool-path layer. The pool's steps run in the reference engine's
        order (classify, issue, publish, expire, release); the expert kernels are
        launched before the forecast bookkeeping, so the device computes while
        the host selects and reserves the next layers' candidates."""
        be, pool, pol = self.be, self.pool, self.policy
        h_res, x, logits = be.pre_moe(l, h)
        targets = [t for t in (l + 1, l + 2) if t < self.cfg.n_layers]
        ids, w, probs = be.route_and_forecast(logits, h_res, targets)
        self.fc.observe(l, ids)
        out, ready, misses, adopted = pol.classify(l, ids)
        waits: List[torch.cuda.Event] = []
        for e in adopted:
            ev = self.events.pop((l, e), None)
            if ev is not None and not ev.query():
                waits.append(ev)
                del ready[e]
        # copies into slots the last layer's kernels may have read wait for those kernels
        ev_prev = self.ev_compute
        ev_demand = self._copy(self.copy, [(e, out[e]) for e in misses], l, ev_prev)
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
        # routed + shared + residual in the down kernel: bf16(h_res + moe_finalize(...)) of orchestrator.py:287
        h_next = be.moe_rest(l, x, ids, w, pool.memory, out, handle, h_res=h_res)
        if ev_ready is not None:
            self.stats._pending.append(("stall", ev_ready, ev_demand))
        self._ev_i ^= 1
        self.ev_compute = self._ev_layer[self._ev_i]
        self.ev_compute.record(self.compute)     # copies queued from the next layer on wait for this layer's kernels
        # forecasts for the next layers, copied while this layer computes (into partition slots, which this
        # layer's kernels do not read: its slots are pinned)
        reserved, cands = pol.issue(targets, probs)
        for t, pairs in reserved.items():
            ev = self._copy(self.spec, pairs, t, ev_prev)
            for e, _ in pairs:
                self.events[(t, e)] = ev
            self.stats.spec_records += len(pairs)
        if self.trace is not None and ids.shape[0] == 1:
            self.trace.append((self.generation, l, [int(e) for e in ids[0]], cands))
        pol.publish(l, misses, out)
        for k in pol.expire(l):
            self.events.pop(k, None)
        pol.release(out)
        self.stats.layers += 1
        return h_next

    def begin_token(self) -> None:
        """Start of a token (a forward pass): forecasts left from the last
        token go back to the partition."""
        self.generation += 1
        self.policy.end_token()
        self.events.clear()

    def token(self, h: torch.Tensor) -> torch.Tensor:
        self.begin_token()
        for l in range(self.cfg.n_layers):
            h = self.layer(l, h)
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
