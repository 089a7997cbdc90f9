"""GPU parity of the Mamba-ND model (kmamba_ndmodel.h)
against its float64 torch restatement (oracle/ndmodel_ref.py), at a small
volume: the loss of a forward, every parameter gradient of a backward
(torch autograd of the restatement, with the same bf16 rounding of every
GEMM operand), and one AdamW step; also with the batch run as micro-batches
whose gradients accumulate.

Tolerances: the loss to 1e-4 relative (measured <= 6e-8).  Gradients to
5e-3 in norm (norm_err), with a loose elementwise guard (rel_err <= 0.2)
against errors confined to a few rows or tiles: the GPU rounds fp32
operands to bf16 and the restatement rounds float64 ones, so an operand
within fp32 noise of a rounding boundary goes to neighbouring bf16 values
on the two sides, and each such flip moves single gradient entries by up to
~1e-2 of the tensor's peak.  Measured: norm_err 2e-7 where no operand flips
(the d = 32 cases with one volume), 1.4e-4 at d = 64 with one layer, 1.2e-3
at d = 64 with two layers (6^3 volume); elementwise rel_err up to 7e-2
there.  The AdamW
update to 1e-4 of the step size."""
import ctypes as C

import numpy as np
import pytest

from conftest import norm_err, rel_err

import kmamba_b200 as kb

pytestmark = pytest.mark.gpu
N_STATE, QC = 16, 35


def split(flat, dims_d, L, V):
    """Flat layout of kmamba_ndmodel.h -> dict of float64 torch tensors."""
    import torch
    d = dims_d
    t = lambda a, shape: torch.tensor(a.reshape(shape), dtype=torch.float64)  # noqa: E731
    o = 0

    def take(n, shape):
        nonlocal o
        v = t(flat[o:o + n], shape)
        o += n
        return v
    out = {"embedding": take(V * d, (V, d)), "head": take(V * d, (V, d)), "layers": []}
    for _ in range(L):
        out["layers"].append({
            "W_a": take(d * d, (d, d)), "W_z": take(d * d, (d, d)), "W_out": take(d * d, (d, d)),
            "W_p": take(QC * d, (QC, d)), "dt_bias": take(3 * d, (3, d)),
            "A_log": take(3 * d * N_STATE, (3, d, N_STATE)),
            "conv_kernel": take(27 * d, (27, d)), "conv_bias": take(d, (d,))})
    assert o == flat.size
    return out


def flatten(tree):
    parts = [tree["embedding"], tree["head"]]
    for layer in tree["layers"]:
        parts += [layer[k] for k in ("W_a", "W_z", "W_out", "W_p", "dt_bias", "A_log",
                                     "conv_kernel", "conv_bias")]
    return parts


def device_array(ptr, n):
    import torch
    buf = torch.empty(n, dtype=torch.float32, device="cuda")
    rt = C.CDLL("libcudart.so.12")
    rt.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    assert rt.cudaMemcpy(buf.data_ptr(), ptr, 4 * n, 3) == 0   # device to device
    return buf.cpu().numpy()


@pytest.mark.parametrize("dims,d,L,batch,micro", [([3, 4, 5], 32, 2, 2, 0), ([4, 4, 4], 64, 1, 1, 0),
                                                  # T = batch * points above one 128-row
                                                  # GEMM tile, d = 64, two layers
                                                  ([6, 6, 6], 64, 2, 1, 0),
                                                  ([4, 4, 4], 64, 1, 3, 0),
                                                  # a batch of 3 run as passes of 1 and 2
                                                  # volumes whose gradients accumulate
                                                  ([4, 5, 3], 32, 2, 3, 1),
                                                  ([4, 5, 3], 32, 2, 3, 2),
                                                  ([4, 4, 4], 64, 2, 3, 2)])
def test_ndmodel_loss_gradients_and_step(lib, cuda, dims, d, L, batch, micro):
    import torch
    import ndmodel_ref as ref
    V = 256
    cfg = kb.KmbNDModelConfig()
    for i in range(3):
        cfg.dims[i] = dims[i]
    cfg.dim, cfg.n_layers, cfg.vocab, cfg.seed, cfg.micro_batch = d, L, V, 1234, micro
    m = lib.kmb_ndmodel_create(C.byref(cfg))
    assert m, kb.last_error(lib)
    try:
        n = lib.kmb_ndmodel_param_count(m)
        P = int(np.prod(dims))
        rng = np.random.default_rng(sum(dims) + d)
        tok = rng.integers(0, V, (batch, P), dtype=np.uint32)
        ttok = torch.from_numpy(tok.astype(np.int32)).cuda()
        loss = C.c_float()
        kb.check(lib, lib.kmb_ndmodel_backward(m, ttok.data_ptr(), batch, C.byref(loss)))
        flat = device_array(lib.kmb_ndmodel_params(m), n)
        grads = device_array(lib.kmb_ndmodel_grads(m), n)
        assert np.all(np.isfinite(grads))

        tree = split(flat, d, L, V)
        leaves = flatten(tree)
        for t in leaves:
            t.requires_grad_(True)
        want = ref.forward_loss(tree, torch.from_numpy(tok.astype(np.int64)), dims)
        want.backward()
        assert abs(loss.value - want.item()) <= 1e-4 * abs(want.item()), (loss.value, want.item())
        o = 0
        names = ["embedding", "head"] + [f"L{i}.{k}" for i in range(L) for k in (
            "W_a", "W_z", "W_out", "W_p", "dt_bias", "A_log", "conv_kernel", "conv_bias")]
        for name, t in zip(names, leaves):
            g_ref = t.grad.numpy().ravel()
            g = grads[o:o + g_ref.size]
            o += g_ref.size
            if name == "embedding":   # only the rows of tokens present have gradients
                g_ref, g = g_ref.reshape(V, d), g.reshape(V, d)
            assert norm_err(g, g_ref) <= 5e-3, (name, norm_err(g, g_ref))
            assert rel_err(g, g_ref) <= 0.2, (name, rel_err(g, g_ref))

        # one AdamW step: p - lr * (g / (|g| + eps)) on step 1, with decay
        lr, wd = 1e-3, 0.01
        kb.check(lib, lib.kmb_ndmodel_step(m, lr, wd))
        new = device_array(lib.kmb_ndmodel_params(m), n)
        mh = grads.astype(np.float64)
        vh = mh * mh
        upd = flat * (1 - lr * wd) - lr * mh / (np.sqrt(vh) + 1e-8)
        assert np.max(np.abs(new - upd)) <= 1e-4 * lr + 1e-6 * np.max(np.abs(flat))
        # the loss after the step goes down
        l2 = C.c_float()
        kb.check(lib, lib.kmb_ndmodel_forward(m, ttok.data_ptr(), batch, C.byref(l2)))
        assert l2.value < loss.value
    finally:
        lib.kmb_ndmodel_free(m)


def test_ndmodel_rejects_bad_config(lib):
    cfg = kb.KmbNDModelConfig()
    cfg.dims[0] = cfg.dims[1] = cfg.dims[2] = 4
    cfg.dim, cfg.n_layers, cfg.vocab = 48, 1, 256     # dim not a multiple of 32
    assert not lib.kmb_ndmodel_create(C.byref(cfg))
    assert b"multiple of 32" in lib.kmb_last_error()

