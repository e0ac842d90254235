"""CPU: the multi-rank plumbing of bench.py under a world_size-2 gloo group.

The batch shards with no data-path collective; ranks only agree on the slowest
rank's time (MAX all-reduce), and the whole-job value is all ranks' matrices over it.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        ms_local = 1.0 + rank * 0.5                       # rank 1 is the slow one
        ms = bench.reduce_max(dist, ms_local, torch.device("cpu"))
        batch = 4096
        value = world * batch / (ms / 1e3)
        q.put((rank, ms, value))
    finally:
        dist.destroy_process_group()


def test_two_ranks_take_the_slowest_time():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [1.5, 1.5]
    assert res[0][2] == pytest.approx(2 * 4096 / 1.5e-3)


def test_bench_accounting():
    import bench
    assert bench.bytes_per_matrix(64) == 12 * 64 * 64 + 4 * 64
    assert bench.flops_per_matrix(3) == pytest.approx(72.0)
    assert bench.kernel_launches(64) == 1
    # n = 256: 8 panels, 7 trailing updates, 8 orgqr blocks
    # one row chunk for m <= 512: wpart (with W2) + update per tensor-core update
    assert bench.kernel_launches(256) == 8 + (7 + 8) * 2
    assert bench.kernel_launches(256, 4096) == 8 + (7 + 8) * 2
    # n = 2048 at batch 32: tall blocks split the W^T reduction and add the w2 sum
    assert 64 + 127 * 2 < bench.kernel_launches(2048, 32) <= 64 + 127 * 3
    assert bench.kernel_launches(258) == 9 + (8 + 9)              # n % 4 != 0: one SIMT launch per update


def test_reference_arm_under_torchrun_prints_once():
    """`bench.py --impl reference` launched by torchrun with two ranks: rank 0 times the CPU
    reference and prints one JSON line, the other rank exits 0 without work (no GPU needed)."""
    import json
    import socket
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), str(root / "bench.py"),
           "--impl", "reference", "--gpus", "2", "--config", "b64_n32", "--steps", "1", "--warmup", "1"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = lines[0]
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "reference"
