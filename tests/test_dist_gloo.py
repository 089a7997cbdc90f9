"""Data-parallel host logic (k-mamba_b200/kmb_dist.py) with world_size 2 over
gloo on CPU: each rank computes the 1D-scan gradient of its own shard with
the CPU oracle, the parameter gradient dA is summed over ranks, timing is
the max over ranks, and a rank that leaves before a collective is detected
by its peer as an error within the process-group timeout (no hang)."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard(seed, L=48, D=8, N=4):
    rng = np.random.default_rng(seed)
    f = np.float32
    x = rng.standard_normal((L, D)).astype(f)
    dt = np.log1p(np.exp(rng.standard_normal((L, D)) - 2)).astype(f)
    A = (-np.exp(rng.uniform(0, np.log(16), (D, N)))).astype(f)
    B = rng.standard_normal((L, N)).astype(f)
    C = rng.standard_normal((L, N)).astype(f)
    dy = rng.standard_normal((L, D)).astype(f)
    return x, dt, A, B, C, dy


def _shard_dA(oracle, seed):
    x, dt, A, B, C, dy = _shard(seed)
    _, _, hall = oracle.scan1d_fwd(x, dt, A, B, C, shared=True, want_h_all=True)
    _, _, dA, _, _ = oracle.scan1d_bwd(x, dt, A, B, C, hall, dy, shared=True)
    return dA


def _worker(rank, world, port, outdir, mode):
    sys.path.insert(0, os.path.join(ROOT, "k-mamba_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    import torch
    import kmb_dist
    import oracle
    r, w = kmb_dist.env_rank()
    assert (r, w) == (rank, world)
    dist = kmb_dist.init("gloo", timeout_s=10)
    try:
        if mode == "leave" and rank == 1:
            os._exit(0)  # leaves between steps, before the next collective
        dA = torch.from_numpy(_shard_dA(oracle, kmb_dist.shard_seed(1000, rank)))
        try:
            kmb_dist.sum_grads([dA], world)
        except Exception as e:  # noqa: BLE001 - the peer is gone
            with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
                f.write(f"detected {type(e).__name__}")
            return
        want = sum(_shard_dA(oracle, kmb_dist.shard_seed(1000, q)) for q in range(world))
        ok = np.allclose(dA.numpy(), want, rtol=1e-6, atol=1e-7)
        tmax = kmb_dist.max_over_ranks(1.5 + rank, world)
        with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{int(ok)} {tmax}")
    finally:
        if mode != "leave":
            dist.barrier()
            dist.destroy_process_group()


@pytest.fixture(scope="module")
def oracle_built(oracle):
    return oracle


def test_gradient_sum_and_timing_over_two_ranks(oracle_built, tmp_path):
    port = _free_port()
    mp.spawn(_worker, args=(2, port, str(tmp_path), "sum"), nprocs=2, join=True)
    for rank in range(2):
        ok, tmax = open(tmp_path / f"rank{rank}.txt").read().split()
        assert ok == "1"
        assert float(tmax) == pytest.approx(2.5)


def test_weak_scaling_rate():
    sys.path.insert(0, os.path.join(ROOT, "k-mamba_b200"))
    import kmb_dist
    # 2 ranks, 3 steps of 1.6235 GB each, slowest rank 0.012 s
    assert kmb_dist.weak_scaling_rate(1.6235e9, 2, 3, 0.012) == pytest.approx(811.75)
    assert kmb_dist.sum_grads(["unchanged"], 1) == ["unchanged"]
    assert kmb_dist.max_over_ranks(3.25, 1) == 3.25


@pytest.mark.timeout(120)
def test_rank_leaving_is_detected(oracle_built, tmp_path):
    port = _free_port()
    import time
    ctx = mp.spawn(_worker, args=(2, port, str(tmp_path), "leave"), nprocs=2, join=False)
    deadline = time.time() + 90
    # join() returns whenever one process ends: wait for both (bounded)
    while not ctx.join(timeout=max(1.0, deadline - time.time())):
        if time.time() > deadline:
            break
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    msg = open(tmp_path / "rank0.txt").read()
    assert msg.startswith("detected")
