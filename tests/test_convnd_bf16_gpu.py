"""GPU parity of the bf16-activation ConvND entry points (kmb_convnd_fwd_bf16,
kmb_convnd_bwd_bf16) against the CPU oracle, through the C ABI.

Inputs are rounded to bf16 once; the oracle runs in fp32 on those rounded
values, so the only differences left are the GPU's fp32 summation order and
the rounding of output / dinput to bf16 (round to nearest even, at most half
a bf16 ulp: 2^-9 relative).  Tolerances: output and dinput to 2e-2 (the bar
BASELINE sets for bf16 I/O; measured <= 4e-3 on the parity metric), dkernel
and dbias, which stay fp32, to 1e-4 against float64 sums of the same
rounded values (the fp32 bar of the fp32 entry points)."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err
from test_convnd_gpu import dkernel_f64, kb_conv

import kmamba_b200 as kb

pytestmark = pytest.mark.gpu
f32 = np.float32
TOL_BF16 = 2e-2
TOL_F32 = 1e-4


def bf16_round(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, f32)).to(torch.bfloat16).float().numpy()


@pytest.mark.parametrize("dims,D,K,bias", [
    # streamed 2D kernels (D a multiple of 64): ragged strips and column tiles
    ([70, 40], 64, 3, True), ([33, 17], 128, 2, False), ([130, 20], 64, 1, True),
    ([260, 33], 64, 3, True),
    # 3D kernels (D a multiple of 8): partial 64-channel tiles, K 1..3
    ([9, 10, 11], 64, 3, True), ([5, 7, 6], 72, 2, False), ([4, 4, 33], 8, 1, True),
    ([12, 13, 14], 128, 3, True), ([3, 1, 40], 24, 3, True)])
def test_convnd_bf16_vs_oracle(lib, cuda, oracle, dims, D, K, bias):
    import torch
    rng = np.random.default_rng(sum(dims) * 7 + D + K)
    batch = 2
    Pn = int(np.prod(dims))
    KV = K ** len(dims)
    inp = bf16_round(rng.normal(0, 1, (batch, Pn, D)))
    dy = bf16_round(rng.normal(0, 1, (batch, Pn, D)))
    ker = rng.normal(0, 1 / 3, (KV, D)).astype(f32)
    b = rng.normal(0, 0.1, (D,)).astype(f32) if bias else None
    t16 = lambda a: torch.from_numpy(a).cuda().to(torch.bfloat16)  # noqa: E731
    t32 = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa
    ti, tdy, tk, tb = t16(inp), t16(dy), t32(ker), t32(b)
    out = torch.full(ti.shape, float("nan"), device="cuda", dtype=torch.bfloat16)
    din = torch.full(ti.shape, float("nan"), device="cuda", dtype=torch.bfloat16)
    dk = torch.full(ker.shape, float("nan"), device="cuda")
    db = torch.full((D,), float("nan"), device="cuda") if bias else None
    a = kb_conv(dims, batch, D, K, ti, tk, tb, out, tdy, din, dk, db)
    kb.check(lib, lib.kmb_convnd_fwd_bf16(C.byref(a)))
    kb.check(lib, lib.kmb_convnd_bwd_bf16(C.byref(a)))
    out, din = out.float().cpu().numpy(), din.float().cpu().numpy()
    for i in range(batch):
        o = oracle.convnd_fwd(dims, K, inp[i], ker, b)
        di, _, _ = oracle.convnd_bwd(dims, K, inp[i], ker, dy[i], with_bias=True)
        assert rel_err(out[i], o) <= TOL_BF16, (i, rel_err(out[i], o))
        assert rel_err(din[i], di) <= TOL_BF16, (i, rel_err(din[i], di))
        # the rounding to bf16 is the only change: within half a bf16 ulp
        # of the fp32 result (plus fp32 reordering)
        assert np.all(np.abs(out[i] - o) <= np.abs(o) * 2.0 ** -8 + 1e-5)
    dk64, db64 = dkernel_f64(dims, K, inp, dy)
    assert rel_err(dk.cpu().numpy(), dk64) <= TOL_F32
    if bias:
        assert rel_err(db.cpu().numpy(), db64) <= TOL_F32


def test_convnd_bf16_rejects_unsupported(lib, cuda):
    import torch
    x = torch.zeros((1, 16 * 16, 32), device="cuda", dtype=torch.bfloat16)
    k = torch.zeros((9, 32), device="cuda")
    y = torch.empty_like(x)
    a = kb_conv([16, 16], 1, 32, 3, x, k, None, y, None, None, None, None)
    assert lib.kmb_convnd_fwd_bf16(C.byref(a)) == kb.KMB_EUNSUPPORTED  # D not a multiple of 64
    assert b"bf16" in lib.kmb_last_error()
    xh = np.zeros((1, 16 * 16, 64), np.uint16)
    kh = np.zeros((9, 64), f32)
    yh = np.zeros_like(xh)
    a = kb.KmbConvND()
    a.input, a.kernel, a.output = xh.ctypes.data, kh.ctypes.data, yh.ctypes.data
    a.dims[0] = a.dims[1] = 16
    a.ndims, a.batch, a.D, a.K = 2, 1, 64, 3
    assert lib.kmb_convnd_fwd_bf16(C.byref(a)) == kb.KMB_EINVAL      # host memory
