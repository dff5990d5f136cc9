"""The benchmark's multi-rank logic on CPU: world size 2 over gloo (127.0.0.1). Each rank contributes its own timed
region; both must see the max over ranks, and the value must count every rank's rows (weak scaling). Also: under
torchrun only rank 0 runs the reference arm."""

import os
import socket
import subprocess
import sys

import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, REPO)
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    local_ms = [1000.0, 1250.0][rank]  # rank 1 is slower
    value, max_ms = bench.reduce_timing(local_ms, 256, 10, dist, None)
    q.put((rank, value, max_ms))
    dist.barrier()
    dist.destroy_process_group()


def test_reduce_timing_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get() for _ in range(2))
    for rank, value, max_ms in res:
        assert max_ms == 1250.0
        assert abs(value - 2 * 256 * 10 / 1.25) < 1e-6


def test_reference_arm_nonzero_rank_exits_quietly():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0
    assert r.stdout.strip() == ""
