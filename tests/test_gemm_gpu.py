"""GPU parity of the tcgen05 bf16 GEMM (kmb_gemm_bf16) that replaces the
reference's cuBLAS SGEMM projections (cuda/mamba_block.cu:54-72).

The reference computes the projections in fp32 (kernels/gemm_f32.c on the
CPU path).  The tensor-core path rounds its operands to bf16 and
accumulates in fp32, so the exact product of the bf16-rounded operands is
the target: fp32 outputs are held to the 1e-4 parity bar against it
(float64 numpy, and the reference's own gemm_f32 from oracle/_ref on the
same rounded operands), bf16 outputs to one bf16 rounding (2^-8
relative)."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

import kmamba_b200 as kb

pytestmark = pytest.mark.gpu
TOL = 1e-4
BF16_TOL = 2.0 ** -8


def bf16_round(a):
    """float32 -> nearest-even bf16 value, returned as float32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def run(lib, A, B, a_mn=False, b_mn=False, c_bf16=False, bias=None, residual=None, act=0,
        c_init=None):
    """A [M, K], B [N, K] float32 values (already bf16-representable); the
    operands are stored K-major or, with a_mn / b_mn, transposed."""
    import torch
    M, K = A.shape
    N = B.shape[0]
    ta = torch.from_numpy(np.ascontiguousarray(A.T if a_mn else A)).to(torch.bfloat16).cuda()
    tb = torch.from_numpy(np.ascontiguousarray(B.T if b_mn else B)).to(torch.bfloat16).cuda()
    dt = torch.bfloat16 if c_bf16 else torch.float32
    tc = (torch.from_numpy(c_init).to(dt).cuda() if c_init is not None
          else torch.full((M, N), float("nan"), dtype=dt, device="cuda"))
    g = kb.KmbGemm()
    g.A, g.B, g.C = ta.data_ptr(), tb.data_ptr(), tc.data_ptr()
    tbias = torch.from_numpy(bias).cuda() if bias is not None else None
    tres = torch.from_numpy(residual).cuda() if residual is not None else None
    g.bias = tbias.data_ptr() if tbias is not None else None
    g.residual = tres.data_ptr() if tres is not None else None
    g.M, g.N, g.K = M, N, K
    g.lda, g.ldb = ta.shape[1], tb.shape[1]
    g.ldc, g.ldr = N, N
    g.a_mn_major, g.b_mn_major, g.c_bf16, g.act = int(a_mn), int(b_mn), int(c_bf16), act
    g.accumulate = int(c_init is not None)
    kb.check(lib, lib.kmb_gemm_bf16(C.byref(g)))
    torch.cuda.synchronize()
    return tc.float().cpu().numpy()


def problem(seed, M, N, K):
    rng = np.random.default_rng(seed)
    A = bf16_round(rng.standard_normal((M, K), dtype=np.float32))
    B = bf16_round(rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K))
    return A, B


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 256, 128), (200, 136, 72),
                                   (130, 300, 520), (1024, 512, 1024), (64, 16, 8),
                                   (385, 1000, 264)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False),
                                       (True, True)])
def test_gemm_fp32_out(lib, cuda, M, N, K, a_mn, b_mn):
    if (a_mn and M % 8) or (b_mn and N % 8):
        pytest.skip("MN-major storage needs the leading dimension a multiple of 8")
    A, B = problem(M * 7 + N + K, M, N, K)
    got = run(lib, A, B, a_mn, b_mn)
    want = A.astype(np.float64) @ B.astype(np.float64).T
    assert rel_err(got, want) <= TOL


def test_gemm_epilogue_and_bf16_out(lib, cuda):
    M, N, K = 300, 264, 192
    A, B = problem(5, M, N, K)
    rng = np.random.default_rng(6)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    z = A.astype(np.float64) @ B.astype(np.float64).T + bias
    silu = z / (1 + np.exp(-z))
    got = run(lib, A, B, bias=bias, residual=res, act=1)
    assert rel_err(got, silu + res) <= TOL
    got16 = run(lib, A, B, c_bf16=True, bias=bias)
    assert rel_err(got16, z) <= BF16_TOL
    # accumulate into an existing fp32 C
    c0 = rng.standard_normal((M, N)).astype(np.float32)
    got_acc = run(lib, A, B, c_init=c0)
    assert rel_err(got_acc, c0 + A.astype(np.float64) @ B.astype(np.float64).T) <= TOL


def test_gemm_vs_reference_gemm_f32(lib, cuda, oracle):
    """The reference's own fp32 GEMM (kernels/gemm_f32.c: C[M,N] = A[M,K]
    B[K,N]) on the same bf16-representable operands."""
    if not oracle.has_ref():
        pytest.skip("oracle/_ref (the reference's own C build) is not present")
    ref = oracle.ref_lib()
    ref.gemm_f32.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
    M, N, K = 384, 256, 384
    A, B = problem(9, M, N, K)
    Bt = np.ascontiguousarray(B.T)
    want = np.zeros((M, N), np.float32)
    ref.gemm_f32(A.ctypes.data, Bt.ctypes.data, want.ctypes.data, M, K, N)
    got = run(lib, A, B)
    exact = A.astype(np.float64) @ B.astype(np.float64).T
    assert rel_err(got, exact) <= TOL
    assert rel_err(got, want) <= TOL + rel_err(want, exact)


def test_gemm_rejects_bad_layouts(lib, cuda):
    import torch
    a = torch.zeros((16, 12), dtype=torch.bfloat16, device="cuda")
    g = kb.KmbGemm()
    g.A = g.B = g.C = a.data_ptr()
    g.M, g.N, g.K, g.lda, g.ldb, g.ldc = 16, 16, 12, 12, 12, 16
    assert lib.kmb_gemm_bf16(C.byref(g)) == kb.KMB_EUNSUPPORTED   # lda not a multiple of 8
    host = np.zeros((16, 16), np.float32)
    g.lda = g.ldb = 16
    g.K = 16
    g.C = host.ctypes.data
    assert lib.kmb_gemm_bf16(C.byref(g)) == kb.KMB_EINVAL        # host C
    assert lib.kmb_gemm_check_error() == 0


@pytest.mark.parametrize("M,N,K", [(256, 512, 16384), (136, 264, 8192), (128, 1024, 4096)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, True), (False, True)])
def test_gemm_split_k(lib, cuda, M, N, K, a_mn, b_mn):
    """Few M x N tiles and a long K (the weight-gradient shape d x d x
    tokens): the k-blocks are split over CTAs whose fp32 tiles are added
    atomically; bias and residual are added once, and an accumulating call
    keeps C."""
    A, B = problem(M + N + K, M, N, K)
    exact = A.astype(np.float64) @ B.astype(np.float64).T
    assert rel_err(run(lib, A, B, a_mn, b_mn), exact) <= TOL
    rng = np.random.default_rng(K)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    assert rel_err(run(lib, A, B, a_mn, b_mn, bias=bias, residual=res), exact + bias + res) <= TOL
    c0 = rng.standard_normal((M, N)).astype(np.float32)
    assert rel_err(run(lib, A, B, a_mn, b_mn, c_init=c0), exact + c0) <= TOL


def test_gemm_split_k_padded_mn_major(lib, cuda):
    """The dt-projection weight gradient of the ND model: A^T is [K, 40]
    with 35 live columns (M = 35, lda = 40), B MN-major, K = tokens."""
    import torch
    M, N, K, lda = 35, 512, 8192, 40
    A, B = problem(35, M, N, K)
    at = np.zeros((K, lda), np.float32)
    at[:, :M] = A.T
    ta = torch.from_numpy(at).to(torch.bfloat16).cuda()
    tb = torch.from_numpy(np.ascontiguousarray(B.T)).to(torch.bfloat16).cuda()
    tc = torch.full((M, N), float("nan"), device="cuda")
    g = kb.KmbGemm()
    g.A, g.B, g.C = ta.data_ptr(), tb.data_ptr(), tc.data_ptr()
    g.M, g.N, g.K, g.lda, g.ldb, g.ldc, g.ldr = M, N, K, lda, N, N, N
    g.a_mn_major, g.b_mn_major = 1, 1
    kb.check(lib, lib.kmb_gemm_bf16(C.byref(g)))
    torch.cuda.synchronize()
    assert rel_err(tc.cpu().numpy(), A.astype(np.float64) @ B.astype(np.float64).T) <= TOL
