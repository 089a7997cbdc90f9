"""CPU ORACLE — test infrastructure only.

Float64 torch restatement of the reference k-mamba block and LM step, used
by tests/ as the checker of the GPU block / model path (never by the
product).  torch autograd of this forward is the gradient oracle: the
reference's CPU block backward is an empty stub (src/mamba_block.c:834-836),
so its forward is the pinned part (checked against oracle/_ref in the CPU
tests) and the gradients follow from it exactly.

Block (src/mamba_block.c:89-120 controller, :413-465 scan, :471-502 block):
    u_t    = silu(W_in x_t)                                  [R]
    dt_t   = clamp(softplus(delta_proj . x_t), dt_min, dt_max)
    lam_t  = sigmoid(lambda_proj . x_t)
    B_t    = W_B x_t + b_B,   C_t = W_C x_t + b_C            [R*N], r*N + n
    Bu_t   = sum_r B_t[r, :] u_t[r]
    h_t    = e^{dt A} R(theta) h_{t-1} + (1 - lam) dt e^{dt A} Bu_{t-1}
             + lam dt Bu_t              (pairs (2i, 2i+1) rotated by theta[i])
    y_t[r] = C_t[r, :] . h_t,   out_t = x_t + W_out y_t
Model (src/kmamba.c:344-466): embedding gather, blocks, logits = h @ head,
mean token cross-entropy per sequence, mean over sequences.
"""
from __future__ import annotations

import torch

PARAMS = ("W_in", "W_out", "A_log", "W_B", "W_C", "b_B", "b_C", "delta_proj", "theta",
          "lambda_proj")


def shapes(D, N, R):
    return {"W_in": (R, D), "W_out": (D, R), "A_log": (N,), "W_B": (N * R, D),
            "W_C": (N * R, D), "b_B": (N * R,), "b_C": (N * R,), "delta_proj": (D,),
            "theta": (max(N // 2, 1),), "lambda_proj": (D,)}


def rotate(h, theta, N):
    """R(theta) h for pairs (2i, 2i+1), i < N // 2; an odd last state stays."""
    npair = N // 2
    if npair == 0:
        return h
    c, s = torch.cos(theta[:npair]), torch.sin(theta[:npair])
    he, ho = h[..., 0:2 * npair:2], h[..., 1:2 * npair:2]
    r = torch.stack([c * he - s * ho, s * he + c * ho], dim=-1).reshape(*h.shape[:-1], 2 * npair)
    return torch.cat([r, h[..., 2 * npair:]], dim=-1) if N % 2 else r


def block_forward(x, P, dt_min, dt_max, N, R):
    """x [B, L, D] float64; P: dict of float64 tensors (shapes()).  Returns
    out [B, L, D]."""
    Bsz, L, D = x.shape
    u = torch.nn.functional.silu(x @ P["W_in"].T)                      # [B, L, R]
    dt = torch.clamp(torch.nn.functional.softplus(x @ P["delta_proj"]), dt_min, dt_max)
    lam = torch.sigmoid(x @ P["lambda_proj"])                          # [B, L]
    Bm = (x @ P["W_B"].T + P["b_B"]).reshape(Bsz, L, R, N)
    Cm = (x @ P["W_C"].T + P["b_C"]).reshape(Bsz, L, R, N)
    bu_all = (Bm * u[..., None]).sum(2)                                # [B, L, N]
    h = x.new_zeros(Bsz, N)
    pb = x.new_zeros(Bsz, N)
    ys = []
    for t in range(L):
        dtt, lt = dt[:, t, None], lam[:, t, None]
        al = torch.exp(dtt * P["A_log"][None, :])
        bu = bu_all[:, t]
        h = al * rotate(h, P["theta"], N) + (1 - lt) * dtt * al * pb + lt * dtt * bu
        ys.append((Cm[:, t] * h[:, None, :]).sum(-1))                  # [B, R]
        pb = bu
    y = torch.stack(ys, 1)                                             # [B, L, R]
    return x + y @ P["W_out"].T


def model_loss(tokens, emb, head, blocks, dt_min, dt_max, N, R):
    """tokens [B, L+1] int64.  Mean over sequences of the mean token
    cross-entropy (train_step for B=1, train_batch otherwise), and logits."""
    tin, tgt = tokens[:, :-1], tokens[:, 1:]
    h = emb[tin]
    for P in blocks:
        h = block_forward(h, P, dt_min, dt_max, N, R)
    logits = h @ head
    lp = torch.log_softmax(logits, -1)
    nll = -lp.gather(-1, tgt[..., None])[..., 0]                       # [B, L]
    return nll.mean(1).mean(0), logits


def adamw(p, g, m, v, step, lr, eps, wd, b1=0.9, b2=0.999):
    """kernels/optimizer_f32.c:82-103; returns (p, m, v)."""
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    bc1 = 1 - b1 ** step
    bc2 = 1 - b2 ** step
    p = p * (1 - lr * wd) - lr * (m / bc1) / (torch.sqrt(v / bc2) + eps)
    return p, m, v


def newton_schulz(G, steps=5):
    """G <- 1.5 G - 0.5 G G^T G, `steps` times (kernels/optimizer_f32.c:31-80)."""
    for _ in range(steps):
        G = 1.5 * G - 0.5 * (G @ G.T) @ G
    return G


def muon(p, g, m, mu, lr, clip, rows=None, cols=None):
    """MUON update (kernels/optimizer_f32.c:110-161); a matrix when rows
    and cols are given.  Returns (p, m)."""
    m = mu * m + g
    G = newton_schulz(m.reshape(rows, cols)).reshape(-1) if rows else m
    norm = torch.sqrt((G * G).sum())
    scale = clip / norm if norm > clip else 1.0
    return p - lr * G * scale, m
