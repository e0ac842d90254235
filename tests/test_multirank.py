"""CPU: the multi-rank plumbing of bench.py under a world_size-2 gloo group.

One batch is split into contiguous slices, one per rank, with no data-path
collective; ranks only agree on the slowest rank's time (MAX all-reduce), and the
whole-job value is the batch over it.
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
        batch = 4097                                       # uneven: one rank gets the extra matrix
        lo, hi = bench.shard(batch, rank, world)
        ms_local = 1.0 + rank * 0.5                       # rank 1 is the slow one
        ms = bench.reduce_max(dist, ms_local, torch.device("cpu"))
        # every rank learns every slice size through the group as well
        sizes = torch.zeros(world, dtype=torch.int64)
        sizes[rank] = hi - lo
        dist.all_reduce(sizes)
        value = batch / (ms / 1e3)
        q.put((rank, ms, value, lo, hi, sizes.tolist()))
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
    assert res[0][2] == pytest.approx(4097 / 1.5e-3)
    # the slices tile the batch exactly, in rank order
    assert [(r[3], r[4]) for r in res] == [(0, 2048), (2048, 4097)]
    assert res[0][5] == res[1][5] == [2048, 2049]


@pytest.mark.parametrize("batch", [1, 7, 32, 4096, 4097])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_arithmetic(batch, world):
    import bench
    slices = [bench.shard(batch, r, world) for r in range(world)]
    assert slices[0][0] == 0 and slices[-1][1] == batch
    for (a, b), (c, d) in zip(slices, slices[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in slices]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes)                  # the larger slices go last


def kernel_launches(n, batch=1):
    import qr_b200
    return int(qr_b200.lib().qrb_kernel_launches(batch, n, 1))


def test_bench_accounting():
    import bench
    assert bench.bytes_per_matrix(64) == 12 * 64 * 64 + 4 * 64
    assert bench.flops_per_matrix(3) == pytest.approx(72.0)
    assert kernel_launches(64) == 1
    # n = 256: 8 panels, 7 trailing updates, 8 orgqr blocks
    # one row chunk for m <= 512: wpart (with W2) + update per tensor-core update
    assert kernel_launches(256) == 8 + (7 + 8) * 2
    assert kernel_launches(256, 4096) == 8 + (7 + 8) * 2
    # n = 2048 at batch 32: tall blocks split the W^T reduction and add the w2 sum
    assert 64 + 127 * 2 < kernel_launches(2048, 32) <= 64 + 127 * 3
    assert kernel_launches(258) == 9 + (8 + 9)              # n % 4 != 0: one SIMT launch per update


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


def test_reference_arm_loads_no_repo_library():
    """The reference arm imports only the seeded generators from the package: neither the
    ops module nor libqrb200 / the compiled call path may be mapped in its process."""
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    code = (
        "import sys, json; sys.argv=['bench.py']; import bench\n"
        "class A: config='b64_n32'; seed=1; steps=1; warmup=1; gpus=1\n"
        "out = bench.run_reference(A())\n"
        "maps = open('/proc/self/maps').read()\n"
        "print(json.dumps({'ok': out is not None, 'lib': 'libqrb200' in maps, '_entry': '_entry' in maps,\n"
        "  'ops': 'qr_b200.ops' in sys.modules, 'same': out['config']['sample_matrices'] == out['config']['batch']}))\n"
    )
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    import json
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d == {"ok": True, "lib": False, "_entry": False, "ops": False, "same": True}


def test_roofline_traffic_from_committed_profiles():
    """The roofline's DRAM traffic comes from the committed ncu summaries: a per-launch
    figure, or DRAM bytes per algorithmic byte scaled by the run's bytes per launch; a
    kernel without a capture reports None rather than another kernel's figure."""
    import bench
    t = bench.load_traffic("b32_n2048")
    assert set(t) >= {"wupdate_kernel", "ygemm_kernel"}
    r = t["wupdate_kernel"]["dram_per_algorithmic"]
    assert 0 < r <= 1
    assert bench.traffic_for(t, "wupdate_kernel", 1e9) == r * 1e9
    assert bench.traffic_for(t, "panel_kernel", 1e9) is None
    s = bench.load_traffic("b4096_n64")
    assert bench.traffic_for(s, "small_qr_kernel", 123.0) == s["small_qr_kernel"]["dram_bytes_per_launch"]
    assert bench.load_traffic("no_such_config") == {}
