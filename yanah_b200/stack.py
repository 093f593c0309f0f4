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

# Stamp slots of the persistent decode kernel (16 per layer; phase i runs from
# slot i to slot i+1). Grid barriers end phases 4 (bar1) and 9 (bar2); bar3
# runs from slot 15 of a layer to slot 0 of the next.
DECODE_STAMPS = 16
DECODE_PHASES = ["loads", "wait_p1_tile", "norm_frags", "p1_rows", "bar1", "route", "issue_c", "p2_tiles",
                 "swiglu_issue_d", "bar2", "p3_frags", "wait_d", "p3_tiles", "combine", "end"]
# Data-flow form (yn_stack_flow_decode): the same 16 stamps per layer; phases 12-14 are empty.
FLOW_PHASES = ["h_in", "wait_p1_tile", "norm", "p1_rows_frags", "route", "issue", "gate_up_act_out",
               "act_in_frags_down", "y_out_next_issue", "y_in", "combine_h_out", "-", "-", "-", "-"]


def flow_phase_report(timing: np.ndarray) -> dict:
    """Per-phase means (over layers of the mean and of the max over CTAs, us)
    of the data-flow decode's stamps; `layer_us` as in decode_phase_report."""
    t = np.asarray(timing, dtype=np.float64) / 1e3
    d = np.diff(t, axis=1)
    out = {"phases_mean_us": {n: round(float(d[:, i].mean()), 3) for i, n in enumerate(FLOW_PHASES) if n != "-"},
           "phases_max_us": {n: round(float(d[:, i].max(axis=1).mean()), 3) for i, n in enumerate(FLOW_PHASES)
                             if n != "-"}}
    if t.shape[0] > 1:
        out["layer_us"] = round(float(np.diff(t[:, 0].min(1)).mean()), 3)
    return out


def decode_phase_report(timing: np.ndarray) -> dict:
    """Summarise (L, 16, G) global-timer stamps (ns) of one decoded token.

    Per phase: mean over layers of the mean and of the max over CTAs (us).
    Per grid barrier: the arrival skew (last arrival - first arrival) and the
    release latency (first CTA through - last arrival). `layer_us`: mean
    time from one layer's first stamp to the next layer's."""
    t = np.asarray(timing, dtype=np.float64) / 1e3
    L, S, G = t.shape
    d = np.diff(t, axis=1)                       # (L, S-1, G)
    out = {"phases_mean_us": {n: round(float(d[:, i].mean()), 3) for i, n in enumerate(DECODE_PHASES)},
           "phases_max_us": {n: round(float(d[:, i].max(axis=1).mean()), 3) for i, n in enumerate(DECODE_PHASES)}}
    bars = {}
    for name, arr_slot, exit_slot in (("bar1", 4, 5), ("bar2", 9, 10)):
        arr, ext = t[:, arr_slot], t[:, exit_slot]
        bars[name] = {"skew_us": round(float((arr.max(1) - arr.min(1)).mean()), 3),
                      "release_us": round(float((ext.min(1) - arr.max(1)).mean()), 3)}
    if L > 1:
        arr, ext = t[:-1, 15], t[1:, 0]
        bars["bar3"] = {"skew_us": round(float((arr.max(1) - arr.min(1)).mean()), 3),
                        "release_us": round(float((ext.min(1) - arr.max(1)).mean()), 3)}
        out["layer_us"] = round(float(np.diff(t[:, 0].min(1)).mean()), 3)
    out["barriers"] = bars
    return out


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
        # persistent decode: device layer table + scratch
        lib = _lib.lib()
        n = len(self.structs)
        tb = int(lib.yn_stack_table_bytes(n))
        self.table = torch.empty(tb, dtype=torch.uint8, device=self.device)
        arr = (_lib.Layer * n)(*self.structs)
        _lib.check(lib.yn_stack_prepare(C.byref(self.dims), arr, n, self.table.data_ptr(), tb))
        sb = max(int(lib.yn_stack_scratch_bytes(C.byref(self.dims))),
                 int(lib.yn_stack_flow_scratch_bytes(C.byref(self.dims))))
        self.scratch = torch.zeros(sb, dtype=torch.uint8, device=self.device)
        self._rows_scratch: Optional[torch.Tensor] = None
        self.layer_array = arr
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

    # ------------------------------------------------- persistent decode
    def decode(self, inputs: torch.Tensor, outputs: torch.Tensor, trace: Optional[torch.Tensor] = None,
               timing: Optional[torch.Tensor] = None, stream=None, trace_hidden: Optional[torch.Tensor] = None,
               trace_weights: Optional[torch.Tensor] = None, kernel: str = "flow") -> None:
        """Sequential bs1 decode of inputs (N,H) -> outputs (N,H) in ONE
        persistent cooperative launch. trace: (N, L, k) int32 routed ids;
        trace_hidden: (N, L, H) bf16 input row of every layer; trace_weights:
        (N, L, k) fp32 routed weights; timing: (L, 16, n_SM) int64
        global-timer stamps (ns) of every CTA for the last token. kernel:
        "flow" (data-flow form, yn_stack_flow_decode) or "barrier"
        (yn_stack_decode); both give the same outputs bit for bit."""
        lib = _lib.lib()
        n = len(self.structs)
        ptr = lambda t: t.data_ptr() if t is not None else None
        fn = {"flow": lib.yn_stack_flow_decode, "barrier": lib.yn_stack_decode}[kernel]
        _lib.check(fn(C.byref(self.dims), self.table.data_ptr(), self.layer_array, n,
                                       inputs.data_ptr(), inputs.shape[0], outputs.data_ptr(), self.scratch.data_ptr(),
                                       self.scratch.numel(), ptr(trace), ptr(trace_hidden), ptr(trace_weights),
                                       ptr(timing), stream_ptr(stream)))

    ROWS_MAX = 8

    def rows_decode(self, inputs: torch.Tensor, outputs: torch.Tensor, trace: Optional[torch.Tensor] = None,
                    trace_hidden: Optional[torch.Tensor] = None, trace_weights: Optional[torch.Tensor] = None,
                    timing: Optional[torch.Tensor] = None, stream=None) -> None:
        """A batch of T <= 8 rows (inputs (T,H) -> outputs (T,H)) through every
        layer in ONE persistent launch (yn_rows_flow_decode): the MoE forward
        of a speculative-verify pass. trace: (L, T, k) int32 routed ids;
        trace_hidden: (L, T, H) bf16 input rows of every layer;
        trace_weights: (L, T, k) fp32; timing: (L, 16, n_SM) int64 stamps.
        Errors land in the stack scratch's error word (decode_error)."""
        lib = _lib.lib()
        if self._rows_scratch is None:
            nb = int(lib.yn_rows_flow_scratch_bytes(C.byref(self.dims), self.ROWS_MAX))
            self._rows_scratch = torch.zeros(nb, dtype=torch.uint8, device=self.device)
        n = len(self.structs)
        ptr = lambda t: t.data_ptr() if t is not None else None
        _lib.check(lib.yn_rows_flow_decode(C.byref(self.dims), self.table.data_ptr(), self.layer_array, n,
                                           inputs.data_ptr(), inputs.shape[0], outputs.data_ptr(),
                                           self._rows_scratch.data_ptr(), self._rows_scratch.numel(), ptr(trace),
                                           ptr(trace_hidden), ptr(trace_weights), ptr(timing), stream_ptr(stream)))

    def rows_error(self, stream=None) -> int:
        """Read and clear the error word of the batch decode (synchronises)."""
        if self._rows_scratch is None:
            return 0
        code = C.c_int32(0)
        rc = _lib.lib().yn_stack_error(self._rows_scratch.data_ptr(), C.byref(self.dims), stream_ptr(stream),
                                       C.byref(code))
        if rc != _lib.YN_OK and code.value == 0:
            _lib.check(rc)
        return code.value

    def decode_error(self, stream=None) -> int:
        code = C.c_int32(0)
        rc = _lib.lib().yn_stack_error(self.scratch.data_ptr(), C.byref(self.dims), stream_ptr(stream), C.byref(code))
        if rc != _lib.YN_OK and code.value == 0:
            _lib.check(rc)
        return code.value

    def decode_host(self, host_inputs: torch.Tensor, host_outputs: torch.Tensor, dev_in: torch.Tensor,
                    dev_out: torch.Tensor, stream=None, kernel: str = "flow") -> None:
        """End-to-end call with host buffers: copy pinned inputs in, decode,
        copy outputs back (all on `stream`, asynchronous)."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        with torch.cuda.stream(s):
            dev_in.copy_(host_inputs, non_blocking=True)
            self.decode(dev_in, dev_out, stream=s, kernel=kernel)
            host_outputs.copy_(dev_out, non_blocking=True)

    # ------------------------------------------------------ kernel timing
    def run_token_timed(self, h_in: torch.Tensor, h_out: torch.Tensor, events: List[int], stream=None) -> None:
        """run_token with an event recorded before the first kernel and after
        every kernel (4 events per layer boundary set: pre, post_attention,
        expert_up, expert_down), so each kernel's duration can be read."""
        lib = _lib.lib()
        st = stream_ptr(stream)
        n = len(self.structs)
        src = h_in.data_ptr()
        d = C.byref(self.dims)
        _lib.check(lib.yn_record_event(events[0], st))
        for i, L in enumerate(self.structs):
            dst = h_out.data_ptr() if i == n - 1 else self._ping[i % 2].data_ptr()
            Lr = C.byref(L)
            _lib.check(lib.yn_post_attention(d, Lr, src, 1, None, 0, self.ws.ptr, st))
            _lib.check(lib.yn_record_event(events[3 * i + 1], st))
            _lib.check(lib.yn_moe_up(d, Lr, None, None, 1, None, 0, self.ws.ptr, st))
            _lib.check(lib.yn_record_event(events[3 * i + 2], st))
            _lib.check(lib.yn_moe_down(d, Lr, None, None, 1, src, 2, dst, self.ws.ptr, st))
            _lib.check(lib.yn_record_event(events[3 * i + 3], st))
            src = dst

    def profile_kernels(self, inputs: torch.Tensor, outputs: torch.Tensor, replays: int = 3):
        """Per-kernel device durations (ms) of a graph-captured decode of
        inputs, with external event nodes between kernels. Returns
        {"post_attention": [...], "expert_up": [...], "expert_down": [...]}
        with one entry per (replay, token, layer)."""
        lib = _lib.lib()
        n_ev = 3 * len(self.structs) + 1
        T = inputs.shape[0]
        evs = []
        for _ in range(T * n_ev):
            e = C.c_void_p()
            _lib.check(lib.yn_event_create(C.byref(e)))
            evs.append(e.value)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))

        def body(stream):
            for t in range(T):
                self.run_token_timed(inputs[t:t + 1], outputs[t:t + 1], evs[t * n_ev:(t + 1) * n_ev], stream)

        with torch.cuda.stream(s):
            body(s)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                body(s)
        out = {"post_attention": [], "expert_up": [], "expert_down": []}
        names = list(out)
        ms = C.c_float()
        for _ in range(replays):
            g.replay()
            torch.cuda.synchronize(self.device)
            for t in range(T):
                base = t * n_ev
                for i in range(len(self.structs)):
                    for k in range(3):
                        _lib.check(lib.yn_event_elapsed_ms(evs[base + 3 * i + k], evs[base + 3 * i + k + 1],
                                                           C.byref(ms)))
                        out[names[k]].append((self.layer_ids[i], ms.value))
        del g
        for e in evs:
            lib.yn_event_destroy(e)
        return out
