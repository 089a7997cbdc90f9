"""Helpers shared by the model tests: building KMamba / MambaBlock objects
through a library (ours or the reference's, same C API and struct
layout), reading their host arrays, and the seeded inputs of config 1."""
from __future__ import annotations

import ctypes as C

import numpy as np

import kmamba_b200 as kb

# the README model (reference README.md:163-180)
CFG1 = dict(vocab_size=256, dim=384, state_size=1024, seq_len=128, n_layers=1)
CFG1_SEED = 1234
CFG1_OPT = dict(lr=1e-3, clip_norm=1.0)
# values of the reference itself on config 1 (kmamba_init(1234), tokens
# srand(0), rand() % 256), observed with its own CPU build
CFG1_SUM_LOGITS = 4.14126587
CFG1_LOSS = 5.55145502

_libc = C.CDLL(None)
_libc.rand.restype = C.c_int
_libc.srand.argtypes = [C.c_uint]


def libc_tokens(n, seed=0, vocab=256):
    """srand(seed); rand() % vocab, n times (the reference test inputs)."""
    _libc.srand(seed)
    return np.array([_libc.rand() % vocab for _ in range(n)], dtype=np.uint32)


def kcfg(**kw):
    c = kb.KMambaConfig()
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def opt(**kw):
    o = kb.MBOptimConfig()
    for k, v in kw.items():
        setattr(o, k, v)
    return o


def declare_ref(ref):
    kb.declare(ref, kb.MODEL_PROTOTYPES)
    return ref


def new_model(lib, seed=CFG1_SEED, **cfg):
    m = lib.kmamba_create(C.byref(kcfg(**cfg)))
    assert m, "kmamba_create failed"
    assert lib.kmamba_init(m, seed) == 0
    return m


def model_arrays(m):
    """numpy views of embedding, head and every block parameter."""
    k = m.contents
    V, D = k.cfg.vocab_size, k.cfg.dim
    out = {"embedding": kb.as_array(k.embedding, V * D), "head": kb.as_array(k.head, D * V)}
    for i in range(k.cfg.n_layers):
        b = k.layers[i]
        for n in kb.BLOCK_PARAMS:
            out[f"{i}.{n}"] = kb.block_tensor(b, n)
    return out


def block_params_torch(block, torch, requires_grad=False):
    """float64 torch copies of a block's parameters, in block_ref shapes."""
    import block_ref
    c = (block.contents if hasattr(block, "contents") else block).config
    shp = block_ref.shapes(int(c.dim), int(c.state_size), max(int(c.mimo_rank), 1))
    return {n: torch.tensor(kb.block_tensor(block, n).astype(np.float64)).reshape(shp[n])
            .requires_grad_(requires_grad) for n in kb.BLOCK_PARAMS}


def mbconfig(dim, state, seq_len, rank=1, dt_min=1e-3, dt_max=0.1, dt_scale=1.0):
    c = kb.MBConfig()
    c.dim, c.state_size, c.seq_len, c.mimo_rank = dim, state, seq_len, rank
    c.dt_min, c.dt_max, c.dt_scale = dt_min, dt_max, dt_scale
    return c


def perturb_block(block, rng, scale=0.3):
    """Gives every parameter non-trivial values (b_B, b_C, A spread), so the
    gradient checks see every term."""
    for n in kb.BLOCK_PARAMS:
        a = kb.block_tensor(block, n)
        if n == "A_log":
            a[:] = -np.exp(rng.uniform(-1.0, 1.5, a.size)).astype(np.float32)
        elif n in ("b_B", "b_C"):
            a[:] = (scale * rng.standard_normal(a.size)).astype(np.float32)
        elif n == "theta":
            a[:] = rng.uniform(0.0, 1.0, a.size).astype(np.float32)
        elif n in ("delta_proj", "lambda_proj"):
            a[:] = (0.3 * rng.standard_normal(a.size)).astype(np.float32)
