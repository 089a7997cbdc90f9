"""GPU parity of the causal depthwise ConvND (forward and backward) against
the CPU oracle and the reference's golden outputs, through the C ABI."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

import kmamba_b200 as kb

pytestmark = pytest.mark.gpu
f32 = np.float32
TOL = 1e-4
P_ = lambda a: None if a is None else a.ctypes.data  # noqa: E731


def params(dims, D, K, inp, ker, bias, out=None, dy=None, din=None, dk=None, db=None):
    dims = np.ascontiguousarray(dims, dtype=np.int64)
    p = kb.ConvNDParams(P_(inp), P_(ker), P_(bias), P_(out), P_(dy), P_(din), P_(dk), P_(db),
                        P_(dims), len(dims), D, K)
    return p, dims


def test_convnd_golden_host_pointers(lib, cuda, golden):
    """convnd(p, CONVND_COMPLETE) on host buffers vs the reference C outputs."""
    for tag, c in golden("convnd.npz").items():
        K = int(tag.split("_K")[1])
        Pn, D = c["input"].shape
        inp, ker, bias, dy = (np.ascontiguousarray(c[k]) for k in ("input", "kernel", "bias", "dy"))
        out = np.full((Pn, D), np.nan, f32)
        din = np.full((Pn, D), np.nan, f32)
        dk = np.full(ker.shape, np.nan, f32)
        db = np.full((D,), np.nan, f32)
        p, keep = params(c["dims"], D, K, inp, ker, bias, out, dy, din, dk, db)
        lib.convnd.argtypes = [C.POINTER(kb.ConvNDParams), C.c_int]
        lib.convnd(C.byref(p), 3)
        assert lib.kmb_last_status() == 0, kb.last_error(lib)
        assert rel_err(out, c["output"]) <= TOL, tag
        assert rel_err(din, c["dinput"]) <= TOL, tag
        assert rel_err(dk, c["dkernel"]) <= TOL, tag
        assert rel_err(db, c["dbias"]) <= TOL, tag


def test_convnd_known_answer(lib, cuda):
    # tests/unit/test_convnd_full.c:14-55
    inp = np.array([[1], [2], [3], [4]], f32)
    ker = np.array([[1], [2], [3], [4]], f32)
    bias = np.array([0.5], f32)
    out = np.zeros((4, 1), f32)
    p, keep = params([2, 2], 1, 2, inp, ker, bias, out)
    lib.convnd.argtypes = [C.POINTER(kb.ConvNDParams), C.c_int]
    lib.convnd(C.byref(p), 1)
    np.testing.assert_allclose(out[:, 0], [4.5, 11.5, 14.5, 30.5], atol=1e-5)
    assert lib.convnd_kernel_volume(2, 2) == 4


def run_batched(lib, dims, D, K, inp, ker, bias, dy):
    import torch
    batch = inp.shape[0]
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa
    ti, tk, tb, tdy = t(inp), t(ker), t(bias), t(dy)
    out = torch.full(inp.shape, float("nan"), device="cuda")
    din = torch.full(inp.shape, float("nan"), device="cuda")
    dk = torch.full(ker.shape, float("nan"), device="cuda")
    db = torch.full((D,), float("nan"), device="cuda") if bias is not None else None
    a = kb_conv(dims, batch, D, K, ti, tk, tb, out, tdy, din, dk, db)
    kb.check(lib, lib.kmb_convnd_fwd(C.byref(a)))
    kb.check(lib, lib.kmb_convnd_bwd(C.byref(a)))
    h = lambda x: None if x is None else x.cpu().numpy()  # noqa: E731
    return h(out), h(din), h(dk), h(db)


def kb_conv(dims, batch, D, K, ti, tk, tb, out, tdy, din, dk, db):
    a = kb.KmbConvND()
    ptr = lambda x: None if x is None else x.data_ptr()  # noqa: E731
    a.input, a.kernel, a.bias, a.output = ptr(ti), ptr(tk), ptr(tb), ptr(out)
    a.dy, a.dinput, a.dkernel, a.dbias = ptr(tdy), ptr(din), ptr(dk), ptr(db)
    for i, v in enumerate(dims):
        a.dims[i] = v
    a.ndims, a.batch, a.D, a.K = len(dims), batch, D, K
    return a


def dkernel_f64(dims, K, inp, dy):
    """float64 dkernel / dbias of the reference's definition
    (src/convnd.c): dker[k, d] = sum_p dy(p, d) in(p - (K-1-k_axis), d),
    k row-major over axes, zero outside the grid; summed over the batch."""
    nd = len(dims)
    x = inp.astype(np.float64).reshape((inp.shape[0], *dims, -1))
    g = dy.astype(np.float64).reshape((dy.shape[0], *dims, -1))
    pad = [(0, 0)] + [(K - 1, 0)] * nd + [(0, 0)]
    xp = np.pad(x, pad)
    out = []
    for k in np.ndindex(*([K] * nd)):
        sl = (slice(None),) + tuple(slice(ka, ka + n) for ka, n in zip(k, dims)) + (slice(None),)
        out.append((g * xp[sl]).sum(axis=tuple(range(nd + 1))))
    return np.stack(out), g.sum(axis=tuple(range(nd + 1)))


@pytest.mark.parametrize("dims,D,K,bias", [
    ([33, 17], 64, 3, True), ([20, 70], 8, 2, True), ([9, 11], 5, 3, True),
    ([16, 16], 12, 4, False), ([5, 40], 4, 5, True), ([1, 64], 16, 3, True),
    ([3, 300], 64, 1, True), ([13], 7, 3, True), ([6, 5, 7], 4, 3, True),
    ([3, 4, 2, 5], 3, 2, False), ([60], 64, 4, True),
    # streamed-row backward (D % 64 == 0, K <= 3): several strips, ragged
    # strips and column tiles
    ([260, 33], 64, 3, True), ([150, 40], 128, 2, False), ([129, 16], 64, 3, True),
    # 3D kernels (D % 4 == 0, K <= 3): partial 64-channel tiles, K 1..3,
    # edges on every axis
    ([9, 10, 11], 64, 3, True), ([5, 7, 6], 68, 2, False), ([4, 4, 33], 8, 1, True),
    ([12, 13, 14], 128, 3, True), ([3, 1, 40], 20, 3, True), ([16, 20, 24], 192, 3, True)])
def test_batched_vs_oracle(lib, cuda, oracle, dims, D, K, bias):
    rng = np.random.default_rng(sum(dims) * 13 + D + K)
    batch = 3
    Pn = int(np.prod(dims))
    KV = K ** len(dims)
    inp = rng.normal(0, 1, (batch, Pn, D)).astype(f32)
    ker = rng.normal(0, 1 / 3, (KV, D)).astype(f32)
    b = rng.normal(0, 0.1, (D,)).astype(f32) if bias else None
    dy = rng.normal(0, 1, (batch, Pn, D)).astype(f32)
    out, din, dk, db = run_batched(lib, dims, D, K, inp, ker, b, dy)
    dk_ref = np.zeros_like(ker)
    db_ref = np.zeros((D,), f32)
    for i in range(batch):
        o = oracle.convnd_fwd(dims, K, inp[i], ker, b)
        di, dki, dbi = oracle.convnd_bwd(dims, K, inp[i], ker, dy[i], with_bias=True)
        assert rel_err(out[i], o) <= TOL
        assert rel_err(din[i], di) <= TOL
        dk_ref += dki
        db_ref += dbi
    # dkernel / dbias are sums over batch * P points: held to the 1e-4 bar
    # against float64, and to the fp32 oracle within that oracle's own
    # rounding (its sequential fp32 sums drift ~1e-4 on 2.5e4 points)
    dk64, db64 = dkernel_f64(dims, K, inp, dy)
    assert rel_err(dk, dk64) <= TOL
    assert rel_err(dk, dk_ref) <= TOL + rel_err(dk_ref, dk64)
    if bias:
        assert rel_err(db, db64) <= TOL
        assert rel_err(db, db_ref) <= TOL + rel_err(db_ref, db64)


def test_config3_full_size(lib, cuda, oracle):
    """BASELINE config 3 (512x512, D 64, K 3, batch 16): every output of
    two batch items vs the oracle; dkernel / dbias checked through their
    linearity in dy (the sum over the batch of per-item gradients)."""
    import torch
    rng = np.random.default_rng(3)
    dims, D, K, batch = [512, 512], 64, 3, 16
    Pn = 512 * 512
    inp = rng.standard_normal((batch, Pn, D), dtype=f32)
    ker = (rng.standard_normal((9, D), dtype=f32) / 3).astype(f32)
    bias = (rng.standard_normal((D,), dtype=f32) * 0.1).astype(f32)
    dy = rng.standard_normal((batch, Pn, D), dtype=f32)
    out, din, dk, db = run_batched(lib, dims, D, K, inp, ker, bias, dy)
    for i in (0, 11):
        o = oracle.convnd_fwd(dims, K, inp[i], ker, bias)
        di, _, _ = oracle.convnd_bwd(dims, K, inp[i], ker, dy[i])
        assert rel_err(out[i], o) <= TOL
        assert rel_err(din[i], di) <= TOL
    # dbias = sum of dy; dkernel[k] = sum_p dy(p) in(p - off_k): fp64 numpy
    np.testing.assert_allclose(db, dy.sum(axis=(0, 1), dtype=np.float64), rtol=1e-4, atol=1e-2)
    ref = np.zeros((9, D))
    for bi in range(batch):
        x4 = inp[bi].reshape(512, 512, D).astype(np.float64)
        g4 = dy[bi].reshape(512, 512, D).astype(np.float64)
        for k0 in range(3):
            for k1 in range(3):
                s0, s1 = 2 - k0, 2 - k1
                ref[k0 * 3 + k1] += np.einsum("ijd,ijd->d", g4[s0:, s1:],
                                              x4[:512 - s0, :512 - s1])
    assert rel_err(dk, ref) <= TOL
    torch.cuda.empty_cache()


@pytest.mark.gpu
def test_3d_dkernel_dbias_4byte_aligned(lib, cuda):
    """dkernel / dbias at addresses that are 4- but not 8-byte aligned: the
    3D backward folds them with scalar atomics there, and must give the
    same values as with aligned outputs."""
    import torch
    dims, D, K, batch = [6, 7, 9], 64, 3, 2
    rng = np.random.default_rng(77)
    Pn = int(np.prod(dims))
    inp = rng.normal(0, 1, (batch, Pn, D)).astype(f32)
    ker = rng.normal(0, 1 / 3, (K ** 3, D)).astype(f32)
    b = rng.normal(0, 0.1, (D,)).astype(f32)
    dy = rng.normal(0, 1, (batch, Pn, D)).astype(f32)
    _, _, dk_ref, db_ref = run_batched(lib, dims, D, K, inp, ker, b, dy)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    ti, tk, tb, tdy = t(inp), t(ker), t(b), t(dy)
    out, din = torch.empty_like(ti), torch.empty_like(ti)
    buf_k = torch.full((ker.size + 1,), float("nan"), device="cuda")
    buf_b = torch.full((D + 1,), float("nan"), device="cuda")
    a = kb_conv(dims, batch, D, K, ti, tk, tb, out, tdy, din, None, None)
    a.dkernel, a.dbias = buf_k.data_ptr() + 4, buf_b.data_ptr() + 4
    assert a.dkernel % 8 == 4 and a.dbias % 8 == 4
    kb.check(lib, lib.kmb_convnd_bwd(C.byref(a)))
    dk = buf_k[1:].reshape(ker.shape).cpu().numpy()
    db = buf_b[1:].cpu().numpy()
    # the same sums in the same order per CTA; only the atomics' order across CTAs differs
    assert rel_err(dk, dk_ref) <= TOL
    assert rel_err(db, db_ref) <= TOL
