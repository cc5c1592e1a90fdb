"""Multi-process (gloo, world_size 2, CPU) tests of the session data-parallel
harness: sharding, max-over-ranks timing, and bench.py's N>1 launch contract."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import __graft_entry__

__graft_entry__.load_package()  # spawned workers import this module without conftest
from oasis_b200 import parallel as PAR  # noqa: E402
from tests.helpers import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_sessions():
    assert [PAR.shard_sessions(64, 8, r) for r in range(8)] == [(8 * r, 8) for r in range(8)]
    assert PAR.shard_sessions(64, 1, 0) == (0, 64)
    covered = sorted(s for r in range(4) for s in range(*(lambda a, n: (a, a + n))(*PAR.shard_sessions(64, 4, r))))
    assert covered == list(range(64))
    with pytest.raises(ValueError):
        PAR.shard_sessions(64, 3, 0)
    with pytest.raises(ValueError):
        PAR.shard_sessions(64, 2, 2)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    r, w, _ = PAR.init_from_env("gloo")
    try:
        PAR.barrier()
        mx = PAR.max_over_ranks(10.0 + r)
        sm = PAR.sum_over_ranks(1.0)
        first, n = PAR.shard_sessions(64, w, r)
        q.put((r, w, mx, sm, first, n))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_reductions():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == [(0, 2, 11.0, 2.0, 0, 32), (1, 2, 11.0, 2.0, 32, 32)]


def test_bench_reference_arm_under_torchrun_world2():
    """bench.py --impl reference launched like the driver's N=2 run: rank 0 prints
    exactly one JSON line, the other rank exits 0 without output."""
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "bench.py"), "--gpus", "2",
           "--impl", "reference", "--steps", "1", "--warmup", "0", "--frames", "2"]
    env = dict(os.environ, OMP_NUM_THREADS="2")
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"
