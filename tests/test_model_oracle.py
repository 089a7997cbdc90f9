"""CPU tests of the model API: struct layout and checkpoint format against
the reference, seeded initialisation, and the float64 block restatement
(oracle/block_ref.py) pinned against the reference's own CPU forward
(oracle/_ref).  No GPU: every call here is host-only in our library
(create / init / save / load) or runs the reference."""
import ctypes as C
import json
import os
import sys

import numpy as np
import pytest

import kmamba_b200 as kb
import model_util as mu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))


@pytest.fixture(scope="module")
def ref(oracle):
    if not oracle.has_ref():
        pytest.skip("reference library (oracle/_ref) not built")
    return mu.declare_ref(oracle.ref_lib())


def test_struct_layout_matches_reference():
    import layout_probe
    ours = layout_probe.probe([os.path.join(os.path.dirname(HERE), "include")])
    want = json.load(open(os.path.join(HERE, "golden", "kmamba_layout.json")))
    assert ours == want
    assert C.sizeof(kb.MambaBlock) == want["MambaBlock"]["sizeof"]
    assert C.sizeof(kb.KMamba) == want["KMamba"]["sizeof"]
    assert C.sizeof(kb.MBOptimState) == want["MBOptimState"]["sizeof"]
    assert C.sizeof(kb.MBConfig) == want["MBConfig"]["sizeof"]


def test_init_is_bit_exact_with_reference(lib, ref):
    cfg = dict(vocab_size=64, dim=24, state_size=10, seq_len=12, n_layers=2, mimo_rank=2)
    a = mu.new_model(lib, **cfg)
    b = mu.new_model(ref, **cfg)
    try:
        A, B = mu.model_arrays(a), mu.model_arrays(b)
        assert A.keys() == B.keys()
        for k in A:
            assert np.array_equal(A[k], B[k]), k
    finally:
        lib.kmamba_free(a)
        ref.kmamba_free(b)


def test_checkpoint_bytes_match_reference(lib, ref, tmp_path):
    cfg = dict(vocab_size=32, dim=16, state_size=6, seq_len=8, n_layers=2, mimo_rank=1,
               dt_scale=0.5, dt_min=1e-3, dt_max=0.2)
    a = mu.new_model(lib, seed=7, **cfg)
    b = mu.new_model(ref, seed=7, **cfg)
    pa, pb = str(tmp_path / "a.kmamba"), str(tmp_path / "b.kmamba")
    try:
        assert lib.kmamba_save(a, pa.encode()) == 0
        assert ref.kmamba_save(b, pb.encode()) == 0
        assert open(pa, "rb").read() == open(pb, "rb").read()
        # ours loads the reference's file; the reference loads ours
        for loader, path in ((lib, pb), (ref, pa)):
            m = loader.kmamba_load(path.encode(), 0, None, 0.0, 0.0)
            assert m
            got = mu.model_arrays(m)
            for k, v in mu.model_arrays(a).items():
                assert np.array_equal(got[k], v), k
            assert m.contents.cfg.dt_max == pytest.approx(0.2)
            loader.kmamba_free(m)
    finally:
        lib.kmamba_free(a)
        ref.kmamba_free(b)


def test_load_rejects_bad_header(lib, tmp_path):
    p = tmp_path / "bad"
    p.write_bytes(b"NOTKMAMBA" + bytes(100))
    assert not lib.kmamba_load(str(p).encode(), 0, None, 0.0, 0.0)
    assert not lib.kmamba_load(str(tmp_path / "missing").encode(), 0, None, 0.0, 0.0)


def test_reference_config1_values(ref):
    """Pins oracle/_ref on config 1 against the values the reference's own
    build gives (Σlogits, first train_step loss)."""
    m = mu.new_model(ref, **mu.CFG1)
    toks = mu.libc_tokens(mu.CFG1["seq_len"] + 1, seed=0)
    logits = np.zeros(mu.CFG1["seq_len"] * mu.CFG1["vocab_size"], np.float32)
    try:
        assert ref.kmamba_forward(m, toks.ctypes.data, logits.ctypes.data) == 0
        assert float(logits.astype(np.float64).sum()) == pytest.approx(mu.CFG1_SUM_LOGITS,
                                                                       rel=1e-6)
        assert ref.kmamba_enable_training(m, C.byref(mu.opt(**mu.CFG1_OPT)), 1e-3, 1e-5) == 0
        loss = ref.kmamba_train_step(m, toks.ctypes.data)
        assert loss == pytest.approx(mu.CFG1_LOSS, rel=1e-6)
    finally:
        ref.kmamba_free(m)


BLOCK_CASES = [
    dict(dim=16, state=8, seq_len=10, rank=1, batch=2),
    dict(dim=12, state=7, seq_len=9, rank=3, batch=1),
    dict(dim=20, state=1, seq_len=6, rank=2, batch=2),
]


@pytest.mark.parametrize("case", BLOCK_CASES, ids=lambda c: f"D{c['dim']}N{c['state']}R{c['rank']}")
def test_block_restatement_matches_reference(ref, case):
    """oracle/block_ref.block_forward (float64) against the reference's
    mamba_block_forward, with every parameter perturbed away from its
    initial value so all terms are exercised."""
    import torch
    import block_ref
    rng = np.random.default_rng(11)
    cfg = mu.mbconfig(case["dim"], case["state"], case["seq_len"], case["rank"])
    b = ref.mamba_block_create(C.byref(cfg))
    try:
        mu._libc.srand(3)
        ref.mamba_block_init(b)
        mu.perturb_block(b, rng)
        B, L, D = case["batch"], case["seq_len"], case["dim"]
        x = rng.standard_normal((B, L, D)).astype(np.float32)
        out = np.zeros_like(x)
        ref.mamba_block_forward(b, out.ctypes.data, x.ctypes.data, B)
        P = mu.block_params_torch(b, torch)
        want = block_ref.block_forward(torch.tensor(x, dtype=torch.float64), P, cfg.dt_min,
                                       cfg.dt_max, case["state"], case["rank"]).numpy()
        d = out - x  # compare the block's own contribution
        dw = want - x
        assert np.max(np.abs(d - dw)) <= 2e-5 * max(np.max(np.abs(dw)), 1e-3)
    finally:
        ref.mamba_block_free(b)


def test_model_restatement_matches_reference(ref):
    """Model forward and first-step loss of the float64 restatement against
    the reference, on a config-1-shaped model with a live dt range."""
    import torch
    import block_ref
    cfg = dict(vocab_size=64, dim=32, state_size=16, seq_len=20, n_layers=2, mimo_rank=1,
               dt_min=1e-3, dt_max=0.2)
    m = mu.new_model(ref, seed=5, **cfg)
    try:
        toks = mu.libc_tokens(cfg["seq_len"] + 1, seed=2, vocab=cfg["vocab_size"])
        logits = np.zeros(cfg["seq_len"] * cfg["vocab_size"], np.float32)
        assert ref.kmamba_forward(m, toks.ctypes.data, logits.ctypes.data) == 0
        arr = mu.model_arrays(m)
        emb = torch.tensor(arr["embedding"].reshape(64, 32), dtype=torch.float64)
        head = torch.tensor(arr["head"].reshape(32, 64), dtype=torch.float64)
        blocks = [{n: torch.tensor(arr[f"{i}.{n}"], dtype=torch.float64).reshape(
            block_ref.shapes(32, 16, 1)[n]) for n in kb.BLOCK_PARAMS} for i in range(2)]
        loss, lg = block_ref.model_loss(torch.tensor(toks.astype(np.int64))[None], emb, head,
                                        blocks, 1e-3, 0.2, 16, 1)
        want = lg[0].numpy().reshape(-1)
        assert np.max(np.abs(logits - want)) <= 1e-5 * np.max(np.abs(want))
        assert ref.kmamba_enable_training(m, C.byref(mu.opt(lr=1e-3, eps=1e-8)), 1e-3, 0.0) == 0
        l_ref = ref.kmamba_train_step(m, toks.ctypes.data)
        assert l_ref == pytest.approx(float(loss), rel=1e-5)
    finally:
        ref.kmamba_free(m)
