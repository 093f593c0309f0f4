"""Decode benchmark: bs1 tok/s of the 48-layer Qwen3-Next-80B-A3B-shaped MoE stack.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (all experts resident in HBM, seeded synthetic weights): 48 MoE
layers, hidden 2048, 512 experts, top-10, SwiGLU intermediate 512 plus a
shared expert (512) behind a sigmoid gate; experts 4-bit g64 in the first and
last 4 layers and 2-bit g64 elsewhere; router and shared expert 8-bit g64;
Zipf(1.1) expert popularity; attention replaced by the residual identity.
One step = sequential bs1 decode of 256 tokens (each token through all 48
layers), replayed from one CUDA graph. Inputs are bf16 N(0,1) rows.

--impl ours (default): the CUDA path. `value` = tokens/s with inputs resident;
`e2e` = same through ResidentStack.decode_host (pinned host inputs copied in
and outputs copied out inside the timed region); `roofline` = the dominant
kernel's algorithmic bytes per launch over its live CUDA-event duration;
`cpu_baseline` = the C oracle timed on the host cores on a bounded sample.
For N > 1 (torchrun) every rank decodes its own sequences (replicas: the
resident stack does not shard), and the slowest rank's time is reported; the
line also carries an `ep` object, the sharded path at the same N: the 64-row
batch decode with the experts split over the ranks (as --workload ep).

--impl reference: the reference's MLX path is unavailable on this box (MLX is
not installed), so this times the CPU restatement of that path (oracle/, a C
port using every host core) on one token per step.

Other workloads (--workload), each printing one JSON line of its own metric:
  streaming  the same stack with the HBM slot pool at 20% of the experts and a
             pinned host tier (hit rate, host-link GB/s, hidden copy fraction);
  ep         a batch of 64 rows, experts sharded over the torchrun ranks with
             dispatch/combine over NVLink peer memory (HBM and NVLink rooflines);
  prefill    8 ragged prompts through 40 LFM2-24B-A2B-shaped layers on the
             tcgen05 grouped expert GEMM (tensor-pipe roofline);
  verify     1 + 4-row speculative-verify batches through the same 40 layers;
  sweep      the same 8 prompts through the prefill sweep: staging groups of 32
             over an HBM slot pool at 20% of the experts, the rest read from
             the pinned host tier (host-link roofline).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s (bs1) Qwen3-Next-80B-A3B-shaped MoE; expert GEMV HBM GB/s vs peak"
TOKENS = 256
FALLBACK_HBM_GBS = 6650.0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def sub_label(name: str, args, n_total: int) -> str:
    """Workload name of a run over a layer sub-range (--layers/--first-layer):
    the full stack's name only when every layer runs."""
    n = args.layers or n_total
    if n == n_total and args.first_layer == 0:
        return name
    return f"{name}_sub{n}_from{args.first_layer}"


def line_kernel(kern: str) -> str:
    return "k_stack_flow" if kern == "flow" else "k_stack_decode"


def workload_config(cfg, tokens):
    return {
        "workload": "qwen3_next_80b_a3b_moe_stack48_bs1_decode",
        "layers": cfg.n_layers, "hidden": cfg.hidden, "experts": cfg.n_experts, "top_k": cfg.top_k,
        "moe_inter": cfg.moe_inter, "shared_inter": cfg.shared_inter,
        "expert_bits": "4-bit g64 layers 0-3 and 44-47, 2-bit g64 layers 4-43",
        "router_shared_bits": 8, "tokens_per_step": tokens, "batch": 1,
        "bytes_per_token": cfg.bytes_per_token(),
        "l2": "no flush: each token streams 749 MB of distinct weights (> 126 MB L2); 27.6 GB resident",
    }


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", self.gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def gpu_uuid(dev_index: int) -> str:
    import torch
    try:
        u = torch.cuda.get_device_properties(dev_index).uuid
        s = str(u)
        return s if s.startswith("GPU-") else "GPU-" + s
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        return vis.split(",")[dev_index] if vis else str(dev_index)


# ------------------------------------------------------------ CPU baseline
def cpu_sample(cfg, n_tokens: int, threads: int):
    """Time the C oracle on `n_tokens` sequential bs1 tokens through every
    layer (records regenerated and cached by an untimed first pass)."""
    import numpy as np
    from oracle import cpu
    from yanah_b200.synthetic import hidden_stream_id

    o = cpu.OracleStack(cfg, threads=threads)
    xs = cpu.synth_bf16(n_tokens * cfg.hidden, cfg.seed, hidden_stream_id(0), 1.0).reshape(n_tokens, cfg.hidden)

    def run():
        for t in range(n_tokens):
            h = xs[t:t + 1]
            for l in range(cfg.n_layers):
                h = o.layer(l, h)["out"]
    run()  # untimed: generates and caches the records this sample touches
    t0 = time.perf_counter()
    run()
    return time.perf_counter() - t0, cpu.lib().yo_num_threads()


# ------------------------------------------------------------- reference arm
def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    from yanah_b200.synthetic import qwen3_next_stack
    cfg = qwen3_next_stack(seed=0)
    threads = len(os.sched_getaffinity(0))
    from oracle import cpu
    import numpy as np
    from yanah_b200.synthetic import hidden_stream_id
    o = cpu.OracleStack(cfg, threads=threads)
    x = cpu.synth_bf16(cfg.hidden, cfg.seed, hidden_stream_id(0), 1.0).reshape(1, cfg.hidden)

    def step():
        h = x
        for l in range(cfg.n_layers):
            h = o.layer(l, h)["out"]
    step()  # record generation (not timed)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    tps = args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tps, 4), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": workload_config(cfg, 1),
        "cpu_baseline": {"value": round(tps, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": "1 token (48 layers) per step; MLX unavailable on this box, C port of the path"},
        "e2e": {"value": round(tps, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference MLX CPU path not installable here (no mlx/mlx-lm, no network); oracle C port timed",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- streaming leg
STREAM_METRIC = "decode tok/s (bs1) streaming: 20% HBM slot pool + pinned host tier, Qwen3-Next-80B-A3B-shaped"


def host_link_gbs(dev, nbytes: int = 1 << 30) -> float:
    """Pinned host -> device copy bandwidth (one large cudaMemcpyAsync, events)."""
    import torch
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        d.copy_(h, non_blocking=True)
        e1.record()
        torch.cuda.synchronize(dev)
        best = max(best, nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9)
    return best


def run_streaming(args, rank: int, world: int):
    """Streaming decode: the 48-layer stack with the slot pool at 20% of the experts;
    the rest in pinned host memory; lookahead-2 forecasts (threshold 0.062,
    at most 32 per target, top 24) copy on a side stream. Input rows follow
    an AR(1) process (rho = args.rho) so consecutive tokens route alike."""
    import numpy as np
    import torch
    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    from yanah_b200.streaming import HostTier, StreamingDecoder
    from yanah_b200.synthetic import hidden_stream_id, qwen3_next_stack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = qwen3_next_stack(seed=0)
    link = host_link_gbs(dev)
    host = HostTier(cfg, dev)
    dec = StreamingDecoder(cfg, slot_fraction=0.2, spec_slot_cap=64, lookahead=2, threshold=0.062, issue_cap=32,
                           top=24, device=dev, host=host)
    H, N = cfg.hidden, args.stream_tokens
    total = N * (args.warmup + args.steps)
    noise = torch.empty((total, H), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().yn_synth_bf16(noise.data_ptr(), total * H, cfg.seed, hidden_stream_id(100 + rank), 1.0, 0.0,
                                        stream_ptr()))
    x = noise.float()
    rho = args.rho
    for t in range(1, total):
        x[t] = rho * x[t - 1] + (1 - rho * rho) ** 0.5 * x[t]
    inputs = x.to(torch.bfloat16)
    outputs = torch.empty_like(inputs)
    for w in range(args.warmup):
        dec.decode(inputs[w * N:(w + 1) * N], outputs[w * N:(w + 1) * N])
    torch.cuda.synchronize(dev)
    dec.reset_stats()
    dec.trace = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    off = args.warmup * N
    for k in range(args.steps):
        dec.decode(inputs[off + k * N:off + (k + 1) * N], outputs[off + k * N:off + (k + 1) * N])
    e1.record()
    torch.cuda.synchronize(dev)
    secs = e0.elapsed_time(e1) / 1e3
    r = dec.report(secs)
    if dec.be.check_error():
        raise RuntimeError("device error in the streaming decode")
    tr = np.array([ids for _, _, ids, _ in dec.trace]).reshape(-1, cfg.n_layers, cfg.top_k)
    rep = float(np.mean([len(set(tr[t, l]) & set(tr[t - 1, l])) / cfg.top_k
                         for t in range(1, tr.shape[0]) for l in range(cfg.n_layers)])) if tr.shape[0] > 1 else 0.0
    tokens = N * args.steps
    line = {
        "metric": STREAM_METRIC, "value": round(tokens / secs, 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "qwen3_next_80b_a3b_moe_stack48_bs1_streaming", "pool_slots": r["pool_slots"],
                   "pool_fraction": 0.2, "spec_slots": r["spec_slots"], "lookahead": 2, "threshold": 0.062,
                   "issue_cap": 32, "forecast_top": 24, "tokens_per_step": N, "input_ar1_rho": rho,
                   "host_tier_gb": round(host.nbytes / 1e9, 2)},
        "streaming": {"hit_rate": round(r["hit_rate"], 4), "adopted": r["adopted"],
                      "forecast_recall": round(r["forecast_recall"], 4),
                      "demand_records_per_token": round(r["demand_records"] / tokens, 2),
                      "spec_records_per_token": round(r["spec_records"] / tokens, 2),
                      "h2d_gbs": round(r["h2d_gbs"], 2), "stall_ms_per_token": round(r["stall_ms"] / tokens, 3),
                      "copy_busy_ms_per_token": round(r["copy_busy_ms"] / tokens, 3),
                      "hidden_fraction": round(r["hidden_fraction"], 4),
                      "measured_repeat_rate": round(rep, 4), "target_repeat_rate": 0.6},
        "roofline": {"bound": "host-link", "achieved": round(r["h2d_gbs"], 2), "peak": round(link, 2),
                     "unit": "GB/s", "frac": round(r["h2d_gbs"] / link, 4),
                     "peak_source": "pinned host->device cudaMemcpyAsync of 1 GiB, measured in this run"},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------- expert-parallel leg
EP_METRIC = "decode tok/s, batch of 64 rows, experts sharded over GPUs (Qwen3-Next-80B-A3B-shaped, 48 layers)"


def run_ep(args, rank: int, world: int, emit: bool = True):
    """Expert-parallel batch decode: 64 rows (one token each per step) through
    the 48-layer stack, experts sharded 512/world per GPU, per-layer dispatch
    and combine over peer memory (yn_ep_layer). One step = one CUDA graph
    replay. Inputs differ every step (the previous step's outputs)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    from yanah_b200.ep import ExpertParallelStack, expert_range
    from yanah_b200.synthetic import hidden_stream_id, qwen3_next_stack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = qwen3_next_stack(seed=0)
    B = args.batch
    layer_ids = list(range(args.first_layer, args.first_layer + (args.layers or cfg.n_layers)))
    stack = ExpertParallelStack(cfg, batch=B, rank=rank, world=world, device=dev, layers=layer_ids)
    H, K, L = cfg.hidden, cfg.top_k, len(layer_ids)
    T_h = B // world
    rows = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().yn_synth_bf16(rows.data_ptr(), B * H, cfg.seed, hidden_stream_id(500), 1.0, 0.0,
                                        stream_ptr()))
    home = rows[rank * T_h:(rank + 1) * T_h].contiguous()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # untimed pass, layer by layer: which experts and pairs each layer touches
    lo, hi = stack.e_lo, stack.e_hi
    n_local, pairs_out, pairs_in = [], 0, 0
    ids_all = torch.empty((B, K), dtype=torch.int32)
    ping = [home.clone(), torch.empty_like(home)]
    for i in range(L):
        stack.layer(i, ping[i % 2], ping[(i + 1) % 2])
        torch.cuda.synchronize(dev)
        _lib.check(_lib.lib().yn_memcpy(ids_all.data_ptr(), stack.sview.ids_all, B * K * 4, None))
        ids = ids_all.numpy()
        local = (ids >= lo) & (ids < hi)
        n_local.append(len(np.unique(ids[local])))
        t_home = np.arange(B)[:, None] // T_h
        pairs_out += int((local & (t_home != rank)).sum())
        pairs_in += int(((~local) & (t_home == rank)).sum())
    stack.step_end()
    barrier()
    if stack.check_error():
        raise RuntimeError("device error in the first step")
    # graph of one step; warm-up replays
    stack.capture()
    h = home
    for _ in range(args.warmup):
        h = stack.step(h).clone()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid(dev.index)) as clk:
        start.record()
        for _ in range(args.steps):
            stack._ping[0].copy_(stack._ping[stack.out_slot])
            stack.graph.replay()
        end.record()
        torch.cuda.synchronize(dev)
    barrier()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    if stack.check_error():
        raise RuntimeError("device error during the timed steps")
    value = B * args.steps / (ms_max / 1e3)

    # e2e: pinned host rows in, outputs out, every step
    h_in = torch.empty((T_h, H), dtype=torch.bfloat16, pin_memory=True)
    h_in.copy_(home)
    h_out = torch.empty_like(h_in, pin_memory=True)
    for _ in range(2):
        stack._ping[0].copy_(h_in, non_blocking=True)
        stack.graph.replay()
        h_out.copy_(stack._ping[stack.out_slot], non_blocking=True)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        stack._ping[0].copy_(h_in, non_blocking=True)
        stack.graph.replay()
        h_out.copy_(stack._ping[stack.out_slot], non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    barrier()
    t2 = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e = B * args.steps / (float(t2.item()) / 1e3)

    # rooflines of this rank's step: HBM (each local expert record of a layer
    # once, the dense weights once) and NVLink (rows out, output rows back)
    rec = [cfg.record_spec(l).record_bytes for l in layer_ids]
    hbm_bytes = sum(n * r for n, r in zip(n_local, rec)) + L * cfg.dense_bytes_per_layer()
    link_bytes = L * T_h * (H * 2 + K * 4) * (world - 1) + pairs_out * H * 2
    hbm, src = peaks()
    step_s = ms_max / args.steps / 1e3
    achieved = hbm_bytes / step_s / 1e9
    line = {
        "metric": EP_METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": sub_label("qwen3_next_80b_a3b_moe_stack48_ep_batch64_decode", args, cfg.n_layers), "layers": L, "batch": B,
                   "rows_per_gpu": T_h, "experts_per_gpu": hi - lo, "hidden": H, "experts": cfg.n_experts,
                   "top_k": K, "expert_bits": "4-bit g64 layers 0-3 and 44-47, 2-bit g64 layers 4-43",
                   "parallelism": f"ep{world}",
                   "l2": "no flush: a step reads every local expert record a layer routes to once (~100 of "
                         "512 per layer, ~4.6 GB per step at one GPU) and all dense weights (>126 MB L2)"},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": T_h * H * 2,
                "d2h_bytes_per_step": T_h * H * 2},
        "gpu_launches": args.steps * (L * (9 + (T_h - 1) // 8) + 1),
        "clocks": clk.summary(),
        "roofline": {"bound": "hbm", "kernel": "whole step (every kernel of yn_ep_layer)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_source": src, "bytes_per_step": hbm_bytes, "traffic": None,
                     "local_experts_per_layer_mean": round(float(np.mean(n_local)), 1)},
        "nvlink": {"bytes_per_step": link_bytes, "achieved_gbs": round(link_bytes / step_s / 1e9, 2),
                   "peak_gbs": 770.0, "frac": round(link_bytes / step_s / 1e9 / 770.0, 4),
                   "pairs_sent_back_per_step": pairs_out},
    }
    if rank == 0 and emit:
        print(json.dumps(line), flush=True)
    stack.graph = None
    barrier()
    stack.close()
    return line


# ------------------------------------------------------------- prefill leg
PREFILL_METRIC = "prefill tok/s, ragged batch of 8 prompts (LFM2-24B-A2B-shaped, 40 layers), tensor-core expert GEMM"


def run_prefill(args, rank: int, world: int):
    """Tensor-core prefill: a ragged batch of 8 prompts with lengths uniform in
    1-512 (seeded) through the 40-layer LFM2-shaped stack: routing of every
    row, the host plan of the expert groups, the tcgen05 grouped gate/up +
    SwiGLU and down GEMMs, the combine. One step = the whole batch through
    every layer."""
    import numpy as np
    import torch

    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    from yanah_b200.prefill import PrefillStack
    from yanah_b200.synthetic import hidden_stream_id, lfm2_stack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = lfm2_stack(seed=0)
    lens = np.random.default_rng(3).integers(1, 513, size=8)
    T = int(lens.sum())
    layer_ids = list(range(args.first_layer, args.first_layer + (args.layers or cfg.n_layers)))
    stack = PrefillStack(cfg, max_rows=T, device=dev, layers=layer_ids)
    H, K, I = cfg.hidden, cfg.top_k, cfg.moe_inter
    h = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().yn_synth_bf16(h.data_ptr(), T * H, cfg.seed, hidden_stream_id(600 + rank), 1.0, 0.0,
                                        stream_ptr()))
    for _ in range(args.warmup):
        stack.prefill(h)
    torch.cuda.synchronize(dev)
    if stack.check_error():
        raise RuntimeError("device error in the prefill warm-up")
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid(dev.index)) as clk:
        start.record()
        for _ in range(args.steps):
            stack.prefill(h)
        end.record()
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(end)
    value = T * args.steps / (ms / 1e3)
    # grouped GEMM time (untimed pass with events around the two GEMM launches of every layer)
    ev = []
    stack.prefill(h, gemm_events=ev)
    torch.cuda.synchronize(dev)
    gemm_ms = sum(a.elapsed_time(b) for a, b in ev)
    L = len(layer_ids)
    flops = L * T * K * 6.0 * H * I
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tf_peak = float(peak.get("bf16_tflops", 1590.0))
    achieved = flops / (gemm_ms / 1e3) / 1e12
    # e2e: pinned host rows in, outputs back, every step
    h_in = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
    h_in.copy_(h)
    h_out = torch.empty_like(h_in, pin_memory=True)
    d_in = torch.empty_like(h)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        d_in.copy_(h_in, non_blocking=True)
        h_out.copy_(stack.prefill(d_in), non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    e2e = T * args.steps / (e0.elapsed_time(e1) / 1e3)
    if stack.check_error():
        raise RuntimeError("device error during the timed prefill")
    line = {
        "metric": PREFILL_METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": sub_label("lfm2_24b_a2b_moe_stack40_prefill", args, cfg.n_layers), "layers": L, "prompts": 8,
                   "prompt_lengths": lens.tolist(), "rows": T, "hidden": H, "experts": cfg.n_experts, "top_k": K,
                   "moe_inter": I, "expert_bits": "4-bit g64", "router_bits": 8,
                   "gemm_operands": "gate/up fp16, down bf16 (dequantised weights and activations), fp32 accumulate in TMEM",
                   "l2": "no flush: a step reads every routed expert of 40 layers (13.6 GB > 126 MB L2)"},
        "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2},
        "gpu_launches": args.steps * L * 7,  # rmsnorm, router dots, f16 copy, plan, 2 grouped GEMMs, combine
        "clocks": clk.summary(),
        "roofline": {"bound": "tensor", "kernel": "k_tc_experts (gate/up + down, every layer)",
                     "achieved": round(achieved, 1), "peak": tf_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / tf_peak, 4),
                     "peak_source": "measured (cuBLAS bf16 burst)" if peak else "fallback",
                     "flops_per_step": flops, "gemm_ms_per_step": round(gemm_ms, 3), "traffic": None},
    }
    if not args.no_cpu:
        from oracle import cpu
        threads = len(os.sched_getaffinity(0))
        o = cpu.OracleStack(cfg, threads=threads)
        rows = h[:16].view(torch.int16).cpu().numpy().view(np.uint16)
        o.layer(layer_ids[0], rows)  # record generation (not timed)
        t0 = time.perf_counter()
        o.layer(layer_ids[0], rows)
        secs = (time.perf_counter() - t0) * L
        line["cpu_baseline"] = {"value": round(16 / secs, 3), "unit": "tok/s", "cores": cpu.lib().yo_num_threads(),
                                "kind": "port",
                                "sample": "16 prompt rows through one layer with the C oracle, scaled to 40 layers"}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- sweep leg
SWEEP_METRIC = ("prefill tok/s through the prefill sweep, 8 prompts (LFM2-24B-A2B-shaped, 40 layers), "
                "20% HBM slot pool + pinned host tier")


def run_sweep(args, rank: int, world: int):
    """Prefill sweep: the prefill workload's 8 ragged prompts through the
    40-layer LFM2-shaped stack, every routed record held in pinned host
    memory and an HBM slot pool at 20% of the experts (512 slots). Per layer:
    routing of every row, then the routed experts in staging groups of 32
    (residents copied out of the pool, the rest read from the host tier on a
    copy stream, two staging buffers), each group one grouped tcgen05 GEMM.
    A warm-up pass admits each layer's fair share into the pool; the timed
    passes do not admit, so every step sees the same pool."""
    import numpy as np
    import torch

    from yanah_b200 import _lib
    from yanah_b200.backend import CudaMoEBackend
    from yanah_b200.device import stream_ptr
    from yanah_b200.pool import SlotPool
    from yanah_b200.streaming import HostTier
    from yanah_b200.sweep import HostTierReader, PrefillSweep, SweepStreams, prompt_pass
    from yanah_b200.synthetic import hidden_stream_id, lfm2_stack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = lfm2_stack(seed=0)
    lens = np.random.default_rng(3).integers(1, 513, size=8)
    T = int(lens.sum())
    link = host_link_gbs(dev)
    tier = HostTier(cfg, dev)
    be = CudaMoEBackend(cfg, device=dev)
    slots = int(0.2 * cfg.n_experts * cfg.n_layers)
    pool = SlotPool(be.geometry, slots, spec_slot_cap=0, memory=be.make_expert_memory(slots))
    streams = SweepStreams(device=dev)
    reader = HostTierReader(tier, streams)
    sweep = PrefillSweep(pool, reader, group=32, make_memory=be.make_expert_memory, streams=streams)
    H = cfg.hidden
    h = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().yn_synth_bf16(h.data_ptr(), T * H, cfg.seed, hidden_stream_id(600 + rank), 1.0, 0.0,
                                        stream_ptr()))
    for w in range(args.warmup):
        prompt_pass(be, sweep, h, admit=(w == 0))
    torch.cuda.synchronize(dev)
    if be.check_error():
        raise RuntimeError("device error in the sweep warm-up")
    st0 = (sweep.stats.pool_copies, sweep.stats.host_records, reader.sweep_runs)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid(dev.index)) as clk:
        start.record()
        for _ in range(args.steps):
            prompt_pass(be, sweep, h, admit=False)
        end.record()
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(end)
    value = T * args.steps / (ms / 1e3)
    res = (sweep.stats.pool_copies - st0[0]) / args.steps
    disk = (sweep.stats.host_records - st0[1]) / args.steps
    runs = (reader.sweep_runs - st0[2]) / args.steps
    rec = cfg.record_spec(0).record_bytes
    h2d = disk * rec / (ms / args.steps / 1e3) / 1e9
    # e2e: pinned host rows in, outputs back, every step
    h_in = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
    h_in.copy_(h)
    h_out = torch.empty_like(h_in, pin_memory=True)
    d_in = torch.empty_like(h)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        d_in.copy_(h_in, non_blocking=True)
        h_out.copy_(prompt_pass(be, sweep, d_in, admit=False), non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    e2e = T * args.steps / (e0.elapsed_time(e1) / 1e3)
    if be.check_error():
        raise RuntimeError("device error during the timed sweep")
    per_layer = (res + disk) / cfg.n_layers
    n_groups = int(np.ceil(per_layer / 32)) * cfg.n_layers
    line = {
        "metric": SWEEP_METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "lfm2_24b_a2b_moe_stack40_prefill_sweep", "layers": cfg.n_layers, "prompts": 8,
                   "prompt_lengths": lens.tolist(), "rows": T, "pool_slots": slots, "pool_fraction": 0.2,
                   "staging_group": 32, "host_tier_gb": round(tier.nbytes / 1e9, 2),
                   "admission": "warm-up pass admits each layer's fair share; timed passes do not admit",
                   "l2": "no flush: a step moves 13.6 GB of expert records (> 126 MB L2)"},
        "sweep": {"resident_copies_per_step": res, "host_records_per_step": disk, "host_runs_per_step": runs,
                  "distinct_experts_per_layer": round(per_layer, 2), "h2d_gbs": round(h2d, 2)},
        "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2},
        # per layer: row norm + router/routing; per staging group: row gather, two grouped GEMMs, combine
        "gpu_launches": args.steps * (cfg.n_layers * 2 + n_groups * 4),
        "clocks": clk.summary(),
        "roofline": {"bound": "host-link", "kernel": "host tier -> staging copies (cudaMemcpyAsync per record)",
                     "achieved": round(h2d, 2), "peak": round(link, 2), "unit": "GB/s",
                     "frac": round(h2d / link, 4),
                     "peak_source": "pinned host->device cudaMemcpyAsync of 1 GiB, measured in this run",
                     "traffic": None},
    }
    sweep.close()
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- verify leg
VERIFY_METRIC = "speculative-verify tok/s, 1+4 rows per step (LFM2-24B-A2B-shaped, 40 layers), union-of-experts batch"


def run_verify_tc(args, rank: int, world: int):
    """Speculative verify: 1 + 4 draft rows per step through the 40
    LFM2-shaped layers on the tcgen05 grouped expert GEMM (the prefill path:
    routing, device-side grouping by expert, gate/up + SwiGLU and down GEMMs
    that read each routed expert record once for all the rows that chose it,
    combine), one CUDA graph per step. HBM-bound: the roofline counts each
    distinct expert record a layer routes to once."""
    import numpy as np
    import torch

    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    from yanah_b200.prefill import PrefillStack
    from yanah_b200.synthetic import hidden_stream_id, lfm2_stack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = lfm2_stack(seed=0)
    B = 5
    layer_ids = list(range(args.first_layer, args.first_layer + (args.layers or cfg.n_layers)))
    stack = PrefillStack(cfg, max_rows=B, device=dev, layers=layer_ids)
    H, K, L = cfg.hidden, cfg.top_k, len(layer_ids)
    rows = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().yn_synth_bf16(rows.data_ptr(), B * H, cfg.seed, hidden_stream_id(700), 1.0, 0.0,
                                        stream_ptr()))
    # untimed pass: distinct experts per layer (the algorithmic bytes)
    n_distinct = []
    ping = [rows.clone(), torch.empty_like(rows)]
    for i in range(L):
        stack.layer(i, ping[i % 2], ping[(i + 1) % 2])
        n_distinct.append(len(np.unique(stack.ids[:B].cpu().numpy())))
    if stack.check_error():
        raise RuntimeError("device error in the first verify step")
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        stack.prefill(rows, stream=s)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            out = stack.prefill(rows, stream=s)
    torch.cuda.current_stream(dev).wait_stream(s)
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid(dev.index)) as clk:
        start.record()
        for _ in range(args.steps):
            g.replay()
        end.record()
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(end)
    if stack.check_error():
        raise RuntimeError("device error during the timed verify steps")
    value = B * args.steps / (ms / 1e3)
    h_in = torch.empty((B, H), dtype=torch.bfloat16, pin_memory=True)
    h_in.copy_(rows)
    h_out = torch.empty_like(h_in, pin_memory=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        rows.copy_(h_in, non_blocking=True)
        g.replay()
        h_out.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    e2e = B * args.steps / (e0.elapsed_time(e1) / 1e3)
    rec = [cfg.record_spec(l).record_bytes for l in layer_ids]
    hbm_bytes = sum(n * r for n, r in zip(n_distinct, rec)) + L * cfg.dense_bytes_per_layer()
    hbm, src = peaks()
    step_s = ms / args.steps / 1e3
    achieved = hbm_bytes / step_s / 1e9
    line = {
        "metric": VERIFY_METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": sub_label("lfm2_24b_a2b_moe_stack40_verify_1p4", args, cfg.n_layers), "layers": L,
                   "rows_per_step": B, "hidden": H, "experts": cfg.n_experts, "top_k": K, "moe_inter": cfg.moe_inter,
                   "expert_bits": "4-bit g64", "path": "tcgen05 grouped GEMM (yn_tc_experts)",
                   "l2": "no flush: a step reads the routed records of 40 layers (~1 GB > 126 MB L2)"},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": B * H * 2, "d2h_bytes_per_step": B * H * 2},
        "gpu_launches": args.steps * L * 7,
        "clocks": clk.summary(),
        "roofline": {"bound": "hbm", "kernel": "whole step (7 kernels per layer)", "achieved": round(achieved, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_source": src,
                     "bytes_per_step": hbm_bytes, "distinct_experts_per_layer_mean": round(float(np.mean(n_distinct)), 2),
                     "traffic": None},
    }
    print(json.dumps(line), flush=True)
    del g


def run_verify_flow(args, rank: int, world: int):
    """Speculative verify: 1 + 4 draft rows per step through the 40
    LFM2-shaped layers in ONE persistent launch per step
    (yn_rows_flow_decode): per layer each distinct routed expert of the 5 rows
    is read from HBM once by a group of CTAs, with the rows as the GEMV's MMA
    columns, and every exchange between CTAs is a flagged word. HBM-bound:
    the roofline counts each distinct expert record a layer routes to once,
    plus the router and norm."""
    import numpy as np
    import torch

    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    from yanah_b200.stack import ResidentStack
    from yanah_b200.synthetic import hidden_stream_id, lfm2_stack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = lfm2_stack(seed=0)
    B = 5
    layer_ids = list(range(args.first_layer, args.first_layer + (args.layers or cfg.n_layers)))
    stack = ResidentStack(cfg, device=dev, layers=layer_ids)
    H, K, L = cfg.hidden, cfg.top_k, len(layer_ids)
    rows = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().yn_synth_bf16(rows.data_ptr(), B * H, cfg.seed, hidden_stream_id(700), 1.0, 0.0,
                                        stream_ptr()))
    out = torch.empty_like(rows)
    # untimed traced pass: distinct experts per layer (the algorithmic bytes)
    trace = torch.full((L, B, K), -1, dtype=torch.int32, device=dev)
    stack.rows_decode(rows, out, trace=trace)
    torch.cuda.synchronize(dev)
    if stack.rows_error():
        raise RuntimeError("device error in the first verify step")
    tr = trace.cpu().numpy()
    n_distinct = [len(np.unique(tr[l])) for l in range(L)]
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            stack.rows_decode(rows, out, stream=s)
    s.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid(dev.index)) as clk:
        with torch.cuda.stream(s):
            start.record(s)
            for _ in range(args.steps):
                stack.rows_decode(rows, out, stream=s)
            end.record(s)
        s.synchronize()
    ms = start.elapsed_time(end)
    if stack.rows_error():
        raise RuntimeError("device error during the timed verify steps")
    value = B * args.steps / (ms / 1e3)
    h_in = torch.empty((B, H), dtype=torch.bfloat16, pin_memory=True)
    h_in.copy_(rows)
    h_out = torch.empty_like(h_in, pin_memory=True)
    with torch.cuda.stream(s):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(args.steps):
            rows.copy_(h_in, non_blocking=True)
            stack.rows_decode(rows, out, stream=s)
            h_out.copy_(out, non_blocking=True)
        e1.record(s)
    s.synchronize()
    e2e = B * args.steps / (e0.elapsed_time(e1) / 1e3)
    timing = None
    if args.phases:
        G = torch.cuda.get_device_properties(dev).multi_processor_count
        tm = torch.zeros((L, 16, G), dtype=torch.int64, device=dev)
        with torch.cuda.stream(s):
            stack.rows_decode(rows, out, timing=tm, stream=s)
        s.synchronize()
        t = tm.cpu().numpy().astype(np.float64)
        names = ["h_in", "norm", "router_rows", "logits_in_route", "plan_issue", "gate_up_frags", "gate_up_groups",
                 "act_in", "down_frags", "down_groups", "combine_h_out"]
        d = np.diff(t[:, :12, :], axis=1) / 1e3          # (L, 11, G) us
        timing = {"phases_mean_us": {n: round(float(d[:, i].mean()), 3) for i, n in enumerate(names)},
                  "phases_max_us": {n: round(float(d[:, i].max(axis=1).mean()), 3) for i, n in enumerate(names)},
                  "layer_us": round(float((t[-1, 11] - t[0, 0]).max() / 1e3 / L), 3),
                  "warp0_stage_wait_gate_up_us": round(float(t[:, 12].mean() / 1e3), 3),
                  "warp0_stage_wait_down_us": round(float(t[:, 13].mean() / 1e3), 3),
                  "groups_per_cta_mean": {"gate_up_8_units": round(float((t[:, 14] // 1000).mean()), 2),
                                          "down_16_rows": round(float((t[:, 14] % 1000).mean()), 2)}}
    rec = [cfg.record_spec(l).record_bytes for l in layer_ids]
    hbm_bytes = sum(n * r for n, r in zip(n_distinct, rec)) + L * cfg.dense_bytes_per_layer()
    hbm, src = peaks()
    step_s = ms / args.steps / 1e3
    achieved = hbm_bytes / step_s / 1e9
    traffic = None   # DRAM bytes per step: the ratio of a small ncu capture, applied to this step's bytes
    tf = ROOT / "profiles" / "kernel_traffic.json"
    if tf.exists() and not args.layers:
        try:
            ratio = json.loads(tf.read_text()).get("k_rows_flow_ratio_dram_to_algorithmic")
            traffic = int(ratio * hbm_bytes) if ratio else None
        except (ValueError, AttributeError, TypeError):
            traffic = None
    line = {
        "metric": VERIFY_METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": sub_label("lfm2_24b_a2b_moe_stack40_verify_1p4", args, cfg.n_layers), "layers": L,
                   "rows_per_step": B, "hidden": H, "experts": cfg.n_experts, "top_k": K, "moe_inter": cfg.moe_inter,
                   "expert_bits": "4-bit g64",
                   "path": "persistent multi-row data-flow decode (yn_rows_flow_decode), one launch per step",
                   "l2": "no flush: a step reads the routed records of 40 layers (~1.7 GB > 126 MB L2)"},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": B * H * 2, "d2h_bytes_per_step": B * H * 2},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
        "roofline": {"bound": "hbm", "kernel": "k_rows_flow", "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_source": src,
                     "bytes_per_step": hbm_bytes, "distinct_experts_per_layer_mean": round(float(np.mean(n_distinct)), 2),
                     "traffic": traffic},
    }
    if timing:
        line["phases"] = timing
    print(json.dumps(line), flush=True)


def run_verify(args, rank: int, world: int):
    """Speculative verify: 1 + 4 draft rows per step through the 40
    LFM2-shaped layers on the batch path (each routed expert record read
    once per layer however many of the 5 rows chose it). HBM-bound: the
    roofline counts each distinct expert record a layer routes to once."""
    import numpy as np
    import torch

    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    from yanah_b200.ep import ExpertParallelStack
    from yanah_b200.synthetic import hidden_stream_id, lfm2_stack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = lfm2_stack(seed=0)
    B = 5
    layer_ids = list(range(args.first_layer, args.first_layer + (args.layers or cfg.n_layers)))
    stack = ExpertParallelStack(cfg, batch=B, device=dev, layers=layer_ids)
    H, K, L = cfg.hidden, cfg.top_k, len(layer_ids)
    rows = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().yn_synth_bf16(rows.data_ptr(), B * H, cfg.seed, hidden_stream_id(700), 1.0, 0.0,
                                        stream_ptr()))
    # untimed pass: distinct experts per layer (the algorithmic bytes)
    n_distinct = []
    ids = torch.empty((B, K), dtype=torch.int32)
    ping = [rows.clone(), torch.empty_like(rows)]
    for i in range(L):
        stack.layer(i, ping[i % 2], ping[(i + 1) % 2])
        torch.cuda.synchronize(dev)
        _lib.check(_lib.lib().yn_memcpy(ids.data_ptr(), stack.sview.ids_all, B * K * 4, None))
        n_distinct.append(len(np.unique(ids.numpy())))
    stack.step_end()
    torch.cuda.synchronize(dev)
    if stack.check_error():
        raise RuntimeError("device error in the first verify step")
    stack.capture()
    for _ in range(args.warmup):
        stack.step(rows)
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid(dev.index)) as clk:
        start.record()
        for _ in range(args.steps):
            stack._ping[0].copy_(rows)
            stack.graph.replay()
        end.record()
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(end)
    if stack.check_error():
        raise RuntimeError("device error during the timed verify steps")
    value = B * args.steps / (ms / 1e3)
    h_in = torch.empty((B, H), dtype=torch.bfloat16, pin_memory=True)
    h_in.copy_(rows)
    h_out = torch.empty_like(h_in, pin_memory=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        stack._ping[0].copy_(h_in, non_blocking=True)
        stack.graph.replay()
        h_out.copy_(stack._ping[stack.out_slot], non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    e2e = B * args.steps / (e0.elapsed_time(e1) / 1e3)
    rec = [cfg.record_spec(l).record_bytes for l in layer_ids]
    hbm_bytes = sum(n * r for n, r in zip(n_distinct, rec)) + L * cfg.dense_bytes_per_layer()
    hbm, src = peaks()
    step_s = ms / args.steps / 1e3
    achieved = hbm_bytes / step_s / 1e9
    line = {
        "metric": VERIFY_METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": sub_label("lfm2_24b_a2b_moe_stack40_verify_1p4", args, cfg.n_layers), "layers": L, "rows_per_step": B,
                   "hidden": H, "experts": cfg.n_experts, "top_k": K, "moe_inter": cfg.moe_inter,
                   "expert_bits": "4-bit g64",
                   "l2": "no flush: a step reads the routed records of 40 layers (~1 GB > 126 MB L2)"},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": B * H * 2, "d2h_bytes_per_step": B * H * 2},
        "gpu_launches": args.steps * (L * 9 + 1),
        "clocks": clk.summary(),
        "roofline": {"bound": "hbm", "kernel": "whole step (every kernel of yn_ep_layer)", "achieved": round(achieved, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_source": src,
                     "bytes_per_step": hbm_bytes, "distinct_experts_per_layer_mean": round(float(np.mean(n_distinct)), 2),
                     "traffic": None},
    }
    print(json.dumps(line), flush=True)
    stack.graph = None
    stack.close()


def hooks_sample(cfg, dev, inputs, n_tok: int, layers=None, warm: int = 1) -> dict:
    """The same decode through the per-layer hook sequence the reference's
    orchestrator calls on a backend (orchestrator.py:226-300, every routed
    expert a pool hit): pre_moe -> route (the routed ids come to the host: the
    reference's routing sync) -> moe_ready -> moe_rest -> h_res +
    moe_finalize, on CudaMoEBackend with every expert of every layer in
    `layers` (default: all) resident in one CudaExpertMemory (slot = i * E +
    expert for the i-th of those layers)."""
    import numpy as np
    import torch

    from yanah_b200.backend import CudaMoEBackend
    from yanah_b200.device import fill_synthetic_experts

    E = cfg.n_experts
    layer_ids = list(range(cfg.n_layers)) if layers is None else list(layers)
    be = CudaMoEBackend(cfg, dev, lookahead=0)
    mem = be.make_expert_memory(len(layer_ids) * E)
    for i, l in enumerate(layer_ids):
        fill_synthetic_experts(mem.arena, cfg, l, first_slot=i * E)
    torch.cuda.synchronize(dev)

    def token(h):
        for i, l in enumerate(layer_ids):
            h_res, x, logits = be.pre_moe(l, h)
            ids, w = be.route(logits)
            rows = {e: i * E + e for e in set(ids.ravel().tolist())}
            handle = be.moe_ready(l, x, ids, mem, rows)
            out = be.moe_rest(l, x, ids, w, mem, rows, handle)
            h = h_res + be.moe_finalize(l, out)
        return h

    for t in range(warm):
        token(inputs[t % inputs.shape[0]:t % inputs.shape[0] + 1])
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for t in range(n_tok):
        token(inputs[t % inputs.shape[0]:t % inputs.shape[0] + 1])
    torch.cuda.synchronize(dev)
    secs = time.perf_counter() - t0
    if be.check_error():
        raise RuntimeError("device error in the hook-sequence decode")
    del mem
    return {"value": round(n_tok / secs, 2), "unit": "tok/s", "tokens": n_tok, "layers": len(layer_ids),
            "us_per_layer": round(secs / n_tok / len(layer_ids) * 1e6, 2),
            "path": "CudaMoEBackend hooks per layer: pre_moe, route (host routing sync), moe_ready, moe_rest, "
                    "moe_finalize; every expert resident"}


HOOKS_METRIC = "decode tok/s through the per-layer backend hooks, bs1 (Qwen3-Next-80B-A3B-shaped)"


def run_hooks(args, rank: int, world: int):
    """bs1 decode through the per-layer hook sequence (pre_moe, route,
    moe_ready, moe_rest, moe_finalize on CudaMoEBackend; the per-layer
    kernels k_post_attention, k_expert_up, k_expert_down) over the stack or a
    sub-stack (--layers): one step = --hook-tokens tokens, host loop and
    routing syncs included, wall clock around the steps."""
    import torch

    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    from yanah_b200.synthetic import hidden_stream_id, qwen3_next_stack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = qwen3_next_stack(seed=0)
    layer_ids = list(range(args.first_layer, args.first_layer + (args.layers or cfg.n_layers)))
    N = args.hook_tokens
    inputs = torch.empty((N, cfg.hidden), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().yn_synth_bf16(inputs.data_ptr(), N * cfg.hidden, cfg.seed, hidden_stream_id(rank), 1.0, 0.0,
                                        stream_ptr()))
    r = hooks_sample(cfg, dev, inputs, N * args.steps, layers=layer_ids, warm=N * args.warmup)
    secs = N * args.steps / r["value"]
    line = {
        "metric": HOOKS_METRIC, "value": r["value"], "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": sub_label("qwen3_next_80b_a3b_moe_stack48_bs1_hooks", args, cfg.n_layers),
                   "layers": len(layer_ids), "tokens_per_step": N},
        "hooks": {"us_per_layer": r["us_per_layer"], "path": r["path"]},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def run_ours(args, rank: int, world: int):
    import numpy as np
    import torch
    import torch.distributed as dist

    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    from yanah_b200.stack import DECODE_STAMPS, ResidentStack, decode_phase_report, flow_phase_report
    from yanah_b200.synthetic import hidden_stream_id, qwen3_next_stack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = qwen3_next_stack(seed=0)
    layers = list(range(args.first_layer, args.first_layer + (args.layers or cfg.n_layers)))
    stack = ResidentStack(cfg, dev, layers=layers)
    H, N = cfg.hidden, args.tokens
    lib = _lib.lib()
    inputs = torch.empty((N, H), dtype=torch.bfloat16, device=dev)
    _lib.check(lib.yn_synth_bf16(inputs.data_ptr(), N * H, cfg.seed, hidden_stream_id(rank), 1.0, 0.0,
                                 stream_ptr()))
    outputs = torch.empty_like(inputs)
    kern = args.decode_kernel
    stack.decode(inputs[:2], outputs[:2], kernel=kern)
    torch.cuda.synchronize(dev)
    if stack.decode_error():
        raise RuntimeError("device error in the first decode")
    # per-layer phase breakdown from global-timer stamps of every CTA (one
    # extra untimed launch)
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    timing = torch.zeros((len(layers), DECODE_STAMPS, n_sm), dtype=torch.int64, device=dev)
    stack.decode(inputs[:2], outputs[:2], timing=timing, kernel=kern)
    torch.cuda.synchronize(dev)
    phases = (flow_phase_report if kern == "flow" else decode_phase_report)(timing.cpu().numpy())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        stack.decode(inputs, outputs, kernel=kern)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid(dev.index)) as clk:
        start.record()
        for _ in range(args.steps):
            stack.decode(inputs, outputs, kernel=kern)
        end.record()
        torch.cuda.synchronize(dev)
    barrier()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    if stack.decode_error():
        raise RuntimeError("device error during the timed decode")
    value = world * N * args.steps / (ms_max / 1e3)

    # e2e through the host-buffer API: pinned inputs in, outputs back, every step.
    h_in = torch.empty((N, H), dtype=torch.bfloat16, pin_memory=True)
    h_in.copy_(inputs)
    h_out = torch.empty_like(h_in, pin_memory=True)
    d_in, d_out = torch.empty_like(inputs), torch.empty_like(outputs)
    for _ in range(2):
        stack.decode_host(h_in, h_out, d_in, d_out, kernel=kern)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        stack.decode_host(h_in, h_out, d_in, d_out, kernel=kern)
    e1.record()
    torch.cuda.synchronize(dev)
    barrier()
    t2 = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e = world * N * args.steps / (float(t2.item()) / 1e3)

    # The timed region runs one kernel per step: the persistent decode, which
    # moves N tokens x bytes_per_token of weights.
    bytes_tok = sum(cfg.top_k * cfg.record_spec(l).record_bytes + cfg.dense_bytes_per_layer() for l in layers)
    hbm, src = peaks()
    launch_ms = ms_max / args.steps
    achieved = bytes_tok * N / (launch_ms / 1e3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "kernel_traffic.json"
    if tf.exists() and not args.layers:
        try:
            per_tok = json.loads(tf.read_text()).get(f"{line_kernel(kern)}_bytes_per_token")
            traffic = int(per_tok * N) if per_tok else None
        except (ValueError, AttributeError, TypeError):
            traffic = None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {**workload_config(cfg, N), "parallelism": f"replicas{world}" if world > 1 else "single"},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": N * H * 2,
                "d2h_bytes_per_step": N * H * 2},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
        "roofline": {"bound": "hbm", "kernel": "k_stack_flow" if kern == "flow" else "k_stack_decode",
                     "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_source": src,
                     "bytes_per_launch": bytes_tok * N, "avg_launch_us": round(launch_ms * 1e3, 1),
                     "traffic": traffic},
        "phases": phases,
    }
    if args.layers or args.first_layer:
        line["config"]["workload"] = sub_label(line["config"]["workload"], args, cfg.n_layers)
        line["config"]["layers"] = len(layers)
        line["config"]["bytes_per_token"] = bytes_tok
    if rank == 0 and world == 1 and not args.no_cpu and not args.layers:
        threads = len(os.sched_getaffinity(0))
        secs, used = cpu_sample(cfg, args.cpu_tokens, threads)
        line["cpu_baseline"] = {"value": round(args.cpu_tokens / secs, 4), "unit": "tok/s", "cores": used,
                                "kind": "port",
                                "sample": f"{args.cpu_tokens} sequential bs1 token(s) through all 48 layers, "
                                          f"C oracle, {used} OpenMP threads"}
    if world == 1 and not args.no_hooks and not args.layers:
        line["e2e_hooks"] = hooks_sample(cfg, dev, inputs, 16)
    if world > 1 and not args.no_ep:
        # the sharded path at the same GPU count: config 4's 64-row batch decode with the experts split
        # over the ranks (its own line from `--workload ep`, reported here beside the replicas)
        ep = run_ep(args, rank, world, emit=False)
        line["ep"] = {k: ep[k] for k in ("metric", "value", "unit", "ms_per_step", "scaling", "config", "e2e",
                                         "gpu_launches", "clocks", "roofline", "nvlink")}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=TOKENS)
    ap.add_argument("--cpu-tokens", type=int, default=12)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ep", action="store_true", help="with --gpus N > 1: skip the expert-parallel leg")
    ap.add_argument("--no-hooks", action="store_true", help="skip the per-layer hook-sequence (e2e_hooks) sample")
    ap.add_argument("--layers", type=int, default=0, help="profile a sub-stack of this many layers (0: all 48)")
    ap.add_argument("--first-layer", type=int, default=0)
    ap.add_argument("--workload", choices=["resident", "streaming", "ep", "prefill", "verify", "sweep", "hooks"],
                    default="resident",
                    help="resident: the 48-layer all-in-HBM decode (default); streaming: 20%% slot pool + host tier; "
                         "ep: batch of 64 rows, experts sharded over the GPUs; prefill: tensor-core prefill; "
                         "verify: 1+4-row speculative-verify batches; sweep: prefill through the prefill sweep; "
                         "hooks: bs1 decode through the per-layer backend hooks")
    ap.add_argument("--batch", type=int, default=64, help="rows per step of the ep workload")
    ap.add_argument("--decode-kernel", choices=["flow", "barrier"], default="flow",
                    help="resident workload: the data-flow persistent decode (default) or the grid-barrier form")
    ap.add_argument("--verify-path", choices=["flow", "tc", "batch"], default="flow",
                    help="verify workload: the persistent multi-row decode (default), the tcgen05 grouped GEMM "
                         "(the prefill sequence) or the union-of-experts batch path")
    ap.add_argument("--phases", action="store_true",
                    help="verify workload (flow path): also report per-phase times from one stamped launch")
    ap.add_argument("--stream-tokens", type=int, default=32, help="tokens per step of the streaming workload")
    ap.add_argument("--rho", type=float, default=0.0, help="AR(1) correlation of consecutive streaming inputs")
    ap.add_argument("--hook-tokens", type=int, default=16, help="tokens per step of the hooks workload")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.workload == "streaming":
            if rank == 0:
                run_streaming(args, rank, world)
        elif args.workload == "ep":
            run_ep(args, rank, world)
        elif args.workload == "prefill":
            if rank == 0:
                run_prefill(args, rank, world)
        elif args.workload == "verify":
            if rank == 0:
                {"flow": run_verify_flow, "batch": run_verify, "tc": run_verify_tc}[args.verify_path](args, rank, world)
        elif args.workload == "sweep":
            if rank == 0:
                run_sweep(args, rank, world)
        elif args.workload == "hooks":
            if rank == 0:
                run_hooks(args, rank, world)
        else:
            run_ours(args, rank, world)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
