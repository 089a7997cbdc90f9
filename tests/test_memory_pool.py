"""km_memory_pool.h over device memory (reference src/km_memory_pool.c:28-178).

CPU tests cover the bookkeeping that needs no device (create / destroy,
invalid arguments, thread-local identity per host thread).  The GPU test
checks the reference's reuse rules on real device chunks: first fit among
free chunks, free / clear keep the capacity, and chunks go back to the
library's device pool (no new cudaMalloc) when a pool is destroyed."""
import ctypes as C
import threading

import pytest

import kmamba_b200 as kb


def test_pool_bookkeeping_without_device(lib):
    p = lib.km_memory_pool_create()
    assert p
    assert lib.km_pool_alloc(p, 0) is None          # size 0 -> NULL, as the reference
    assert lib.km_pool_alloc(None, 64) is None      # NULL pool -> NULL
    lib.km_pool_free(p, None)
    lib.km_pool_free(None, None)
    lib.km_pool_clear(None)
    lib.km_pool_clear(p)
    lib.km_memory_pool_destroy(p)
    lib.km_memory_pool_destroy(None)


def test_threadlocal_pool_is_per_host_thread(lib):
    main = lib.km_memory_pool_threadlocal()
    assert main and lib.km_memory_pool_threadlocal() == main
    seen = []

    def worker():
        a = lib.km_memory_pool_threadlocal()
        seen.append((a, lib.km_memory_pool_threadlocal()))

    ts = [threading.Thread(target=worker) for _ in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    pools = {a for a, _ in seen}
    assert all(a == b for a, b in seen)
    # plain threads get pools of their own (the reference's OpenMP keying
    # gives every non-OpenMP thread pool 0)
    assert len(pools) == 4 and main not in pools
    lib.km_memory_pool_destroy_all_threadlocal()
    fresh = lib.km_memory_pool_threadlocal()
    assert fresh
    lib.km_memory_pool_destroy_all_threadlocal()


class _PtrAttr(C.Structure):
    _fields_ = [("type", C.c_int), ("device", C.c_int), ("devicePointer", C.c_void_p),
                ("hostPointer", C.c_void_p)]


@pytest.mark.gpu
def test_pool_chunks_are_device_memory_and_reused(lib, cuda):
    import torch
    torch.cuda.synchronize()
    rt = C.CDLL("libcudart.so.12")
    rt.cudaPointerGetAttributes.argtypes = [C.POINTER(_PtrAttr), C.c_void_p]
    rt.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    p = lib.km_memory_pool_create()
    a = lib.km_pool_alloc(p, 1 << 20)
    b = lib.km_pool_alloc(p, 4096)
    assert a and b and a != b
    assert a % 256 == 0 and b % 256 == 0
    at = _PtrAttr()
    assert rt.cudaPointerGetAttributes(C.byref(at), a) == 0
    assert at.type == 2 and at.device == torch.cuda.current_device()  # cudaMemoryTypeDevice
    # device memory round trip through the chunk
    src = (C.c_float * 1024)(*range(1024))
    dst = (C.c_float * 1024)()
    assert rt.cudaMemcpy(a, C.addressof(src), 4096, 4) == 0  # cudaMemcpyDefault
    assert rt.cudaMemcpy(C.addressof(dst), a, 4096, 4) == 0
    assert list(dst) == list(src)
    # first fit among free chunks: a freed 1 MiB chunk serves a smaller request
    lib.km_pool_free(p, a)
    assert lib.km_pool_alloc(p, 1000) == a
    # a request larger than every free chunk grows the pool
    c = lib.km_pool_alloc(p, 2 << 20)
    assert c not in (a, b)
    # clear marks everything free; the capacity stays
    lib.km_pool_clear(p)
    assert lib.km_pool_alloc(p, 4096) in (a, b, c)
    held = lib.kmb_pool_bytes_held()
    lib.km_memory_pool_destroy(p)
    assert lib.kmb_pool_bytes_held() == held   # blocks cached, not freed
    q = lib.km_memory_pool_create()
    assert lib.km_pool_alloc(q, 2 << 20)      # served from the library cache
    assert lib.kmb_pool_bytes_held() == held
    lib.km_memory_pool_destroy(q)
