"""Multi-rank host logic of bench.py on CPU (gloo, world size 2).

The kernels shard by token with no collective on the data path, so what runs
across ranks is the bench's own plumbing: the max-over-ranks reduction of the
step time, the barriers, and the reference arm that only rank 0 runs.
"""

import json
import os
import socket
import subprocess
import sys
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        import bench

        # Each rank's step time differs; every rank must see the slowest.
        slowest = bench.max_over_ranks(1.5 + rank, world, torch.device("cpu"))
        every = bench.gather_ranks(1.5 + rank, world, torch.device("cpu"))
        bench.barrier(world)
        q.put((rank, slowest, every, bench.dist_env()))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, slowest, every, env in got:
        assert slowest == 1.5 + (world - 1)
        assert every == [1.5 + r for r in range(world)]
        assert env == (world, rank, rank)


def test_reference_arm_runs_on_rank0_only():
    """torchrun with two CPU ranks: exactly one JSON line, from rank 0."""
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
           "--gpus", "2", "--steps", "1", "--warmup", "3"]
    env = dict(os.environ, OMP_NUM_THREADS="2")
    out = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["value"] == line["value"]


def test_algorithmic_bytes():
    """The bytes each rank's step counts (every tensor once) at 16x1024 tokens, n=4, D=768."""
    sys.path.insert(0, ROOT)
    import bench

    fb, bb = bench.fused_bytes(bench.TOKENS, bench.N_STREAMS, bench.BLOCK)
    assert (fb, bb) == (253_231_104, 380_633_088)
