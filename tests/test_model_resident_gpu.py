"""Device-resident KMamba models (kmamba_resident.h): the same steps as the
host-array API, with the weights, gradients and moments kept on the GPU
between calls.

A resident model and a host-staged model built from the same seed take the
same forward / training steps through the same kernels: their first loss
is identical, and later losses, logits and weights agree to the rounding
of the gradient kernels' atomic sums (the embedding gradient is a
scatter-add), held to 1e-5.  The host arrays of the resident model stay
at their old values until synced; kmamba_save of a resident model writes
its current (device) values; kmamba_set_device_resident(m, 0) copies back
and releases the copies."""
import ctypes as C

import numpy as np
import pytest

import kmamba_b200 as kb
import model_util as mu

pytestmark = pytest.mark.gpu

CFG = dict(vocab_size=48, dim=32, state_size=16, seq_len=24, n_layers=2, dt_min=1e-3, dt_max=0.2)


def _close(a, b, what):
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6, err_msg=what)


def _pair(lib):
    a = mu.new_model(lib, seed=7, **CFG)
    b = mu.new_model(lib, seed=7, **CFG)
    o = mu.opt(lr=1e-3, eps=1e-6)
    for m in (a, b):
        assert lib.kmamba_enable_training(m, C.byref(o), 1e-3, 1e-5) == 0
    return a, b


def test_resident_steps_match_host_staged(lib, cuda, tmp_path):
    a, b = _pair(lib)
    rng = np.random.default_rng(1)
    V, L = CFG["vocab_size"], CFG["seq_len"]
    try:
        before = {k: v.copy() for k, v in mu.model_arrays(b).items()}
        assert lib.kmamba_set_device_resident(b, 1) == 0, kb.last_error(lib)
        for step in range(3):
            toks = rng.integers(0, V, L + 1).astype(np.uint32)
            la = lib.kmamba_train_step(a, toks.ctypes.data)
            lb = lib.kmamba_train_step(b, toks.ctypes.data)
            assert np.isfinite(la), kb.last_error(lib)
            if step == 0:
                assert la == lb
            assert lb == pytest.approx(la, rel=1e-5), (step, la, lb)
        # the resident model's host arrays still hold the initial values
        for k, v in mu.model_arrays(b).items():
            np.testing.assert_array_equal(v, before[k], err_msg=k)
        ya, yb = np.zeros(L * V, np.float32), np.zeros(L * V, np.float32)
        assert lib.kmamba_forward(a, toks.ctypes.data, ya.ctypes.data) == 0
        assert lib.kmamba_forward(b, toks.ctypes.data, yb.ctypes.data) == 0
        _close(yb, ya, "logits")
        # save writes the device values
        pa, pb = str(tmp_path / "a.kmamba"), str(tmp_path / "b.kmamba")
        assert lib.kmamba_save(a, pa.encode()) == 0
        assert lib.kmamba_save(b, pb.encode()) == 0
        ma = lib.kmamba_load(pa.encode(), 0, None, 0.0, 0.0)
        mb = lib.kmamba_load(pb.encode(), 0, None, 0.0, 0.0)
        assert ma and mb
        try:
            fa, fb = mu.model_arrays(ma), mu.model_arrays(mb)
            for k in fa:
                _close(fb[k], fa[k], k)
            assert not np.array_equal(fb["embedding"], before["embedding"])
        finally:
            lib.kmamba_free(ma)
            lib.kmamba_free(mb)
        # leaving resident mode copies back; both models then agree
        assert lib.kmamba_set_device_resident(b, 0) == 0
        wa, wb = mu.model_arrays(a), mu.model_arrays(b)
        for k in wa:
            _close(wb[k], wa[k], k)
        # and a further step on the now host-staged model still matches
        toks = rng.integers(0, V, L + 1).astype(np.uint32)
        la = lib.kmamba_train_step(a, toks.ctypes.data)
        assert lib.kmamba_train_step(b, toks.ctypes.data) == pytest.approx(la, rel=1e-5)
    finally:
        lib.kmamba_free(a)
        lib.kmamba_free(b)


def test_resident_init_reupload_and_free(lib, cuda):
    a, b = _pair(lib)
    V, L = CFG["vocab_size"], CFG["seq_len"]
    toks = np.random.default_rng(2).integers(0, V, L + 1).astype(np.uint32)
    try:
        assert lib.kmamba_set_device_resident(b, 1) == 0
        lib.kmamba_train_step(b, toks.ctypes.data)
        # kmamba_init rewrites the weights: the resident copies follow
        assert lib.kmamba_init(a, 11) == 0 and lib.kmamba_init(b, 11) == 0
        ya, yb = np.zeros(L * V, np.float32), np.zeros(L * V, np.float32)
        assert lib.kmamba_forward(a, toks.ctypes.data, ya.ctypes.data) == 0
        assert lib.kmamba_forward(b, toks.ctypes.data, yb.ctypes.data) == 0
        np.testing.assert_array_equal(ya, yb)  # same weights, deterministic forward
        assert lib.kmamba_sync_to_host(b) == 0
    finally:
        lib.kmamba_free(a)
        lib.kmamba_free(b)
    # a model created after the resident one was freed is host-staged again
    c = mu.new_model(lib, seed=7, **CFG)
    try:
        y = np.zeros(L * V, np.float32)
        assert lib.kmamba_forward(c, toks.ctypes.data, y.ctypes.data) == 0
        assert np.all(np.isfinite(y))
    finally:
        lib.kmamba_free(c)
