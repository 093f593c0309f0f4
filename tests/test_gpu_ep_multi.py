"""Expert parallelism on 2 GPUs (one process per GPU, peer memory over
NVLink): every rank's home rows come out bit-identical to the one-GPU batch
path, eagerly and from a replayed CUDA graph, and no wait runs out.

Skipped when fewer than 2 GPUs are visible.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

LAYERS = [0, 4, 5]   # a 4-bit layer and two 2-bit layers
BATCH = 16


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rows(cfg):
    from tests.gpu_helpers import hidden_rows
    return hidden_rows(cfg, BATCH, stream=21)


def _worker(rank: int, world: int, port: int, out_q):
    import datetime

    import torch.distributed as dist

    from tests.gpu_helpers import bf16_dev, bf16_np
    from yanah_b200.ep import ExpertParallelStack
    from yanah_b200.synthetic import qwen3_next_stack
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = qwen3_next_stack(n_layers=48)
        h = _rows(cfg)
        T = BATCH // world
        ep = ExpertParallelStack(cfg, batch=BATCH, rank=rank, world=world, device=f"cuda:{rank}", layers=LAYERS)
        mine = bf16_dev(h[rank * T:(rank + 1) * T], f"cuda:{rank}")
        eager = bf16_np(ep.step(mine))
        torch.cuda.synchronize()
        err1 = ep.check_error()
        dist.barrier()
        ep.capture()
        dist.barrier()
        graph = bf16_np(ep.step(mine))
        torch.cuda.synchronize()
        err2 = ep.check_error()
        dist.barrier()
        ep.graph = None
        ep.close()
        out_q.put((rank, eager, graph, err1, err2, None))
    except Exception as e:  # report instead of leaving the parent waiting
        out_q.put((rank, None, None, -1, -1, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_expert_parallel_matches_one_gpu():
    import torch.multiprocessing as mp

    from tests.gpu_helpers import bf16_dev, bf16_np
    from yanah_b200.ep import ExpertParallelStack
    from yanah_b200.synthetic import qwen3_next_stack
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    for rank, _, _, e1, e2, exc in res:
        assert exc is None, f"rank {rank}: {exc}"
        assert e1 == 0 and e2 == 0, (rank, e1, e2)
    assert all(p.exitcode == 0 for p in procs)
    # the same batch on one GPU (this process)
    cfg = qwen3_next_stack(n_layers=48)
    one = ExpertParallelStack(cfg, batch=BATCH, layers=LAYERS, device="cuda:0")
    ref = bf16_np(one.step(bf16_dev(_rows(cfg), "cuda:0")))
    torch.cuda.synchronize()
    assert one.check_error() == 0
    one.close()
    T = BATCH // world
    for rank, eager, graph, _, _, _ in res:
        assert np.array_equal(eager, ref[rank * T:(rank + 1) * T]), f"rank {rank} eager differs"
        assert np.array_equal(graph, ref[rank * T:(rank + 1) * T]), f"rank {rank} graph differs"
