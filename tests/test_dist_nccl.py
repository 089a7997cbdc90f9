"""The NCCL data-parallel layer of libkmamba_b200.so (kmamba_distributed.h;
reference cuda/kmamba_distributed.cu:22-138, src/kmamba_distributed.c:
19-158).

CPU tests: the batch / layer split arithmetic against a restatement of the
reference rule, the rendezvous file that carries rank 0's NCCL id to the
other ranks (two spawned processes; a timeout when no rank 0 writes), and
the reference's NULL / -1 conventions.  GPU tests: a one-rank communicator
(all-reduce and broadcast are identities, bucket coalescing counted by the
context's statistics) and, with two or more GPUs, real ranks through
tests/dist_worker.py."""
import ctypes as C
import multiprocessing as mp
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

import kmamba_b200 as kb

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref_share(count, parts, rank):
    """src/kmamba_distributed.c:118-137: earlier ranks take the extra items."""
    per, rem = count // parts, count % parts
    if rank < rem:
        return rank * (per + 1), rank * (per + 1) + per + 1
    return rank * per + rem, rank * per + rem + per


def test_split_batch_and_layers(lib):
    for count in (0, 1, 7, 8, 64, 65, 1000):
        for parts in (1, 2, 3, 4, 8):
            for rank in range(parts):
                cfg = kb.KMambaDistributedConfig()
                cfg.rank = rank
                lib.kmamba_distributed_split_batch(C.byref(cfg), count, parts)
                assert (cfg.batch_start, cfg.batch_end) == _ref_share(count, parts, rank)
                assert cfg.world_size == parts
                lib.kmamba_distributed_split_layers(C.byref(cfg), count, parts)
                assert (cfg.layer_start, cfg.layer_end) == _ref_share(count, parts, rank)
    cfg = kb.KMambaDistributedConfig()
    lib.kmamba_distributed_split_batch(C.byref(cfg), 8, 0)   # ignored, as the reference
    assert cfg.world_size == 0 and cfg.batch_end == 0


def _rendezvous_child(path, rank, blob, q):
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "k-mamba_b200"))
    import kmamba_b200 as kbc
    lib = kbc.load()
    buf = C.create_string_buffer(bytes(blob) if rank == 0 else bytes(128), 128)
    rc = lib.kmb_dist_rendezvous_file(path.encode(), rank, buf, 128, 20.0)
    q.put((rank, rc, buf.raw))


def test_rendezvous_file_between_processes(lib, tmp_path):
    path = str(tmp_path / "nccl.id")
    blob = np.random.default_rng(3).integers(0, 256, 128, dtype=np.uint8).tobytes()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    readers = [ctx.Process(target=_rendezvous_child, args=(path, r, blob, q)) for r in (1, 2)]
    for p in readers:
        p.start()
    writer = ctx.Process(target=_rendezvous_child, args=(path, 0, blob, q))
    writer.start()
    got = [q.get(timeout=60) for _ in range(3)]
    for p in readers + [writer]:
        p.join(timeout=60)
    for rank, rc, raw in got:
        assert rc == kb.KMB_OK, rank
        assert raw == blob, rank
    assert not [f for f in os.listdir(tmp_path) if ".tmp." in f]   # published by rename


def test_rendezvous_timeout_and_reference_conventions(lib, tmp_path):
    buf = C.create_string_buffer(128)
    rc = lib.kmb_dist_rendezvous_file(str(tmp_path / "never").encode(), 1, buf, 128, 0.2)
    assert rc == kb.KMB_ETIMEOUT
    assert b"no id" in lib.kmb_last_error()
    # world_size <= 1 has no communicator (NULL), as the reference
    assert not lib.kmamba_distributed_init_nccl(1, 0)
    old = os.environ.pop("KMAMBA_NCCL_ID_FILE", None)
    try:
        assert not lib.kmamba_distributed_init_nccl(2, 0)
        assert b"KMAMBA_NCCL_ID_FILE" in lib.kmb_last_error()
    finally:
        if old is not None:
            os.environ["KMAMBA_NCCL_ID_FILE"] = old
    # NULL contexts and buffers: -1, as the reference
    assert lib.kmamba_allreduce_gradients_nccl(None, None, 4) == -1
    assert lib.kmamba_broadcast_params_nccl(None, None, 4) == -1
    pc = lib.kmamba_distributed_init_pipeline(2)
    assert pc and pc.contents.config.world_size == 2
    assert lib.kmamba_pipeline_send_recv(pc, None, None, 4, 1, 0) == -1
    assert lib.kmamba_allreduce_gradients_nccl(pc, None, 4) == -1
    lib.kmamba_distributed_fini_pipeline(pc)


@pytest.mark.gpu
def test_one_rank_communicator_and_buckets(lib, cuda):
    import torch
    uid = C.create_string_buffer(128)
    assert lib.kmb_dist_get_unique_id(uid) == kb.KMB_OK
    ctx = lib.kmb_dist_init_with_id(1, 0, torch.cuda.current_device(), uid)
    assert ctx, kb.last_error(lib)
    x = torch.randn(10000, device="cuda")
    want = x.clone()
    assert lib.kmamba_allreduce_gradients_nccl(ctx, x.data_ptr(), x.numel()) == 0
    assert lib.kmamba_broadcast_params_nccl(ctx, x.data_ptr(), x.numel()) == 0
    assert torch.equal(x, want)
    # coalescing: adjacent ranges below the bucket size make one collective;
    # a gap or the size limit starts another
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    n0 = C.c_ulonglong()
    lib.kmb_dist_stats(ctx, C.byref(n0), None)
    assert lib.kmb_dist_set_bucket_bytes(ctx, 4 * 2500) == 0
    base = x.data_ptr()
    for off, n in ((0, 1000), (1000, 1000), (2000, 1000),    # reaches 3000 floats: flush
                   (5000, 100), (7000, 100)):                 # gap: two more
        assert lib.kmb_dist_bucket_add(ctx, base + 4 * off, n, 0, sp) == 0
    assert lib.kmb_dist_bucket_flush(ctx, sp) == 0
    assert lib.kmb_dist_wait(ctx, sp) == 0
    torch.cuda.synchronize()
    n1, nb = C.c_ulonglong(), C.c_ulonglong()
    lib.kmb_dist_stats(ctx, C.byref(n1), C.byref(nb))
    assert n1.value - n0.value == 3
    assert torch.equal(x, want)
    host = np.zeros(16, np.float32)
    assert lib.kmb_dist_bucket_add(ctx, host.ctypes.data, 16, 0, sp) == kb.KMB_EINVAL
    lib.kmamba_distributed_fini_nccl(ctx)


@pytest.mark.gpu
def test_two_or_more_ranks(lib, cuda):
    import torch
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two GPUs")
    with tempfile.TemporaryDirectory() as d:
        env = dict(os.environ, WORLD_SIZE=str(world), KMAMBA_NCCL_ID_FILE=os.path.join(d, "id"),
                   KMAMBA_NCCL_TIMEOUT_S="60", NCCL_NVLS_ENABLE="0")
        procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "dist_worker.py")],
                                  env=dict(env, RANK=str(r), LOCAL_RANK=str(r)),
                                  stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
                 for r in range(world)]
        outs = []
        for p in procs:
            try:
                out, _ = p.communicate(timeout=240)
            except subprocess.TimeoutExpired:
                for q in procs:
                    q.kill()
                raise
            outs.append((p.returncode, out))
    for r, (rc, out) in enumerate(outs):
        assert rc == 0 and f"RANK_OK {r}" in out, out[-2000:]
