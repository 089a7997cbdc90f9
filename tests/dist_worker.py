"""One rank of the multi-GPU NCCL test (tests/test_dist_nccl.py): meets the
other ranks through kmamba_distributed_init_nccl's rendezvous file and
checks the collectives of libkmamba_b200.so on its own GPU.  Prints
RANK_OK on success."""
import ctypes as C
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "k-mamba_b200"))


def main():
    import numpy as np
    import torch
    import kmamba_b200 as kb
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    lib = kb.load()
    ctx = lib.kmamba_distributed_init_nccl(world, rank)
    assert ctx, kb.last_error(lib)
    cfg = ctx.contents.config
    assert (cfg.world_size, cfg.rank, cfg.use_nccl) == (world, rank, 1)
    # synchronous all-reduce (sum): rank r contributes r + 1
    n = 1 << 20
    g = torch.full((n,), float(rank + 1), device="cuda")
    assert lib.kmamba_allreduce_gradients_nccl(ctx, g.data_ptr(), n) == 0, kb.last_error(lib)
    assert torch.all(g == world * (world + 1) / 2).item()
    # broadcast from rank 0
    p = torch.arange(4096, dtype=torch.float32, device="cuda") * (rank + 1)
    assert lib.kmamba_broadcast_params_nccl(ctx, p.data_ptr(), 4096) == 0
    assert torch.equal(p, torch.arange(4096, dtype=torch.float32, device="cuda"))
    # buckets on a side stream: three adjacent ranges become one collective,
    # a separate tensor another; the caller's stream waits at the end
    s = torch.cuda.Stream()
    flat = torch.full((3 * 1000,), float(rank), device="cuda")
    other = torch.full((777,), float(2 * rank), device="cuda")
    c0 = C.c_ulonglong()
    lib.kmb_dist_stats(ctx, C.byref(c0), None)
    with torch.cuda.stream(s):
        sp = C.c_void_p(s.cuda_stream)
        for i in range(3):
            flat[i * 1000:(i + 1) * 1000].add_(1.0)  # the "gradient" kernel on s
            assert lib.kmb_dist_bucket_add(ctx, flat.data_ptr() + 4000 * i, 1000, 1, sp) == 0
        assert lib.kmb_dist_bucket_add(ctx, other.data_ptr(), 777, 0, sp) == 0
        assert lib.kmb_dist_bucket_flush(ctx, sp) == 0
        assert lib.kmb_dist_wait(ctx, sp) == 0
    s.synchronize()
    c1 = C.c_ulonglong()
    lib.kmb_dist_stats(ctx, C.byref(c1), None)
    assert c1.value - c0.value == 2, (c0.value, c1.value)
    mean = sum(r + 1 for r in range(world)) / world
    assert torch.allclose(flat, torch.full_like(flat, mean))
    assert torch.all(other == sum(2 * r for r in range(world))).item()
    lib.kmamba_distributed_fini_nccl(ctx)
    del np
    print("RANK_OK", rank, flush=True)


if __name__ == "__main__":
    main()
