"""bench.py's multi-rank rules on the CPU, as world-size-2 process groups
over gloo (no GPU): every multi-GPU figure is the slowest rank's (one
all-reduce MAX, the same on every rank), and under torchrun the reference
arm runs on rank 0 alone, which prints the one JSON line while the other
ranks exit 0 without work."""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, values, q):
    try:
        import datetime

        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        sys.path.insert(0, ROOT)
        import bench
        got = [bench.max_over_ranks(v, world, device="cpu") for v in values[rank]]
        dist.destroy_process_group()
        q.put((rank, got))
    except Exception as e:  # report, never hang the parent
        q.put((rank, repr(e)))


def test_max_over_ranks_gloo():
    """Two ranks report different durations; both get the larger, for
    every timing in order (the ranks take the same collectives in the same
    order)."""
    import torch.multiprocessing as mp
    values = {0: [1.5, 7.0, 0.25], 1: [2.5, 3.0, 0.125]}
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, values, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, got = q.get(timeout=120)
            res[rank] = got
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res[0] == res[1] == [2.5, 7.0, 0.25], res


def test_max_over_ranks_one_rank_needs_no_group():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks(3.25, 1) == 3.25


def test_reference_arm_under_torchrun():
    """`torchrun --nproc-per-node 2 bench.py --impl reference`, the way the
    scaling run launches it: exit 0, exactly one JSON line, from rank 0."""
    import oracle
    if not oracle.reference_available():
        pytest.skip("oracle/_ref is not built")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1"]
    # its own session, so that a timeout ends torchrun and its workers together
    proc = subprocess.Popen(cmd, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                            start_new_session=True)
    try:
        stdout, stderr = proc.communicate(timeout=600)
    except subprocess.TimeoutExpired:
        os.killpg(proc.pid, 9)
        proc.communicate()
        raise
    assert proc.returncode == 0, stderr[-2000:]
    lines = [ln for ln in stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
