"""Multi-process paths of bench.py on CPU (gloo, world size 2).

Requests shard across ranks with no collective on the data path; the only
collectives are the barrier around the timed region and the max-over-ranks
reduction of the timing, which run here on the gloo backend.
"""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        dist.barrier()
        got = bench.max_over_ranks(10.0 + rank * 5.0, torch.device("cpu"), world)
        out[rank] = got
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo():
    port = _free_port()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    assert dict(out) == {0: 15.0, 1: 15.0}


def test_max_over_ranks_single_process():
    import bench
    assert bench.max_over_ranks(3.5, torch.device("cpu"), 1) == 3.5


def test_reference_arm_two_ranks_prints_once():
    """Under torchrun with two ranks, rank 0 alone times the reference and prints one line."""
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), str(ROOT / "bench.py"),
           "--impl", "reference", "--workload", "cpu_verify_0p6b", "--steps", "1", "--warmup", "1", "--gpus", "2"]
    env = dict(os.environ, OMP_NUM_THREADS="2")
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=str(ROOT), env=env)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, res.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0
