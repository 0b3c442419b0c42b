"""The N > 1 path of bench.py on CPU: one process per rank over gloo, replicas
with no data-path collective -- only the barrier and the max-over-ranks of the
device time.  The reference arm runs on rank 0 alone; the other ranks exit 0."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


PORT = _free_port()


def _rank_main(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import bench
    r, w, local = bench.dist_setup(world)
    bench.barrier(w)
    # each replica reports its own time; the job's time is the slowest rank's
    q.put((r, bench.allmax(1.0 + r, w)))
    bench.barrier(w)
    import torch.distributed as dist
    dist.destroy_process_group()


def test_gloo_two_ranks_take_the_max_time():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, PORT, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got == {0: 2.0, 1: 2.0}



def test_reference_arm_under_torchrun_two_ranks(tmp_path):
    env = dict(os.environ, KIB_BENCH_DIR=str(tmp_path), CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "bench.py"), "--impl", "reference",
           "--gpus", "2", "--steps", "1", "--warmup", "3", "--layers", "1", "--vocab", "2048"]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1  # rank 0 alone prints
    line = lines[0]
    assert line["impl"] == "reference" and line["value"] > 0 and line["n_gpus"] == 2
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["config"]["reduced_model_for_profiling"] is True
