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
resident stack does not shard), and the slowest rank's time is reported.

--impl reference: the reference's MLX path is unavailable on this box (MLX is
not installed), so this times the CPU restatement of that path (oracle/, a C
port using every host core) on one token per step.
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


# ------------------------------------------------------------------ our arm
def run_ours(args, rank: int, world: int):
    import numpy as np
    import torch
    import torch.distributed as dist

    from yanah_b200 import _lib
    from yanah_b200.device import stream_ptr
    from yanah_b200.stack import DECODE_STAMPS, ResidentStack, decode_phase_report
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
    stack.decode(inputs[:2], outputs[:2])
    torch.cuda.synchronize(dev)
    if stack.decode_error():
        raise RuntimeError("device error in the first decode")
    # per-layer phase breakdown from global-timer stamps of every CTA (one
    # extra untimed launch)
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    timing = torch.zeros((len(layers), DECODE_STAMPS, n_sm), dtype=torch.int64, device=dev)
    stack.decode(inputs[:2], outputs[:2], timing=timing)
    torch.cuda.synchronize(dev)
    phases = decode_phase_report(timing.cpu().numpy())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        stack.decode(inputs, outputs)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid(dev.index)) as clk:
        start.record()
        for _ in range(args.steps):
            stack.decode(inputs, outputs)
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
        stack.decode_host(h_in, h_out, d_in, d_out)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        stack.decode_host(h_in, h_out, d_in, d_out)
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
            per_tok = json.loads(tf.read_text()).get("k_stack_decode_bytes_per_token")
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
        "roofline": {"bound": "hbm", "kernel": "k_stack_decode", "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_source": src,
                     "bytes_per_launch": bytes_tok * N, "avg_launch_us": round(launch_ms * 1e3, 1),
                     "traffic": traffic},
        "phases": phases,
    }
    if args.layers:
        line["config"]["layers"] = len(layers)
        line["config"]["bytes_per_token"] = bytes_tok
    if rank == 0 and world == 1 and not args.no_cpu and not args.layers:
        threads = len(os.sched_getaffinity(0))
        secs, used = cpu_sample(cfg, args.cpu_tokens, threads)
        line["cpu_baseline"] = {"value": round(args.cpu_tokens / secs, 4), "unit": "tok/s", "cores": used,
                                "kind": "port",
                                "sample": f"{args.cpu_tokens} sequential bs1 token(s) through all 48 layers, "
                                          f"C oracle, {used} OpenMP threads"}
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
    ap.add_argument("--layers", type=int, default=0, help="profile a sub-stack of this many layers (0: all 48)")
    ap.add_argument("--first-layer", type=int, default=0)
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
        else:
            run_ours(args, rank, world)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
