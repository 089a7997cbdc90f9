"""CPU ORACLE — test infrastructure only.

float64 torch restatement of the Mamba-ND model that libkmamba_b200's
kmb_ndmodel_* entry points train (a stack of ND blocks
over a 3D volume of byte tokens).  The reference has no working ND model
(kmamba_create with use_convnd overruns its heap, src/mamba_block.c:
223-234), so this file is the definition the GPU model is checked against;
its pieces follow the reference's operators:

  ConvND  causal depthwise K^3 stencil, src/convnd.c:67-129
  ScanND  h(n) = sum_k exp(delta_k A_k) h(n - e_k) + mean_k(delta_k) B x,
          y = sum_m C h, src/scan_nd.c:173-185 (channel-shared B / C)

Model (dims d = dim, N = 16 states, K = 3, 3 axes, P points per volume):

  x0 = E[tok]                                            [P, d]
  per layer (weights W_a, W_z, W_out [d, d]; W_p [35, d]; dt_bias [3, d];
             A_log [3, d, N]; conv kernel [K^3, d], conv bias [d]):
    a  = bf(x) bf(W_a)^T          z = bf(x) bf(W_z)^T    (bf16 GEMMs)
    v  = ConvND(a) + conv_bias
    c  = silu(v)
    q  = bf(c) bf(W_p)^T                                  [P, 35] (bf16 GEMM)
    delta_k = ln 3 + softplus(q[:, k] + dt_bias[k])       k = 0, 1, 2
    B  = q[:, 3:19],  C = q[:, 19:35]
    y  = ScanND(c, delta, A = -1 - exp(A_log), B, C)
         (|A| >= 1 and delta >= ln 3 keep every axis' decay <= 1/3, so the
         three decays of a point sum to <= 1: the recurrence stays bounded
         over the 190 wavefront levels of a 64^3 volume)
    g  = y * silu(z)
    x' = x + bf(g) bf(W_out)^T
  logits = bf(x_L) bf(H)^T                                [P, 256]
  loss = mean over positions of CE(logits[i], tok[(i + 1) mod P])

bf(.) is round-to-nearest-even to bf16 of a GEMM operand, in the forward
and in both gradient GEMMs (the GPU's tensor-core GEMMs take bf16
operands); every other operation is float64 here and fp32 on the GPU.
"""
from __future__ import annotations

import numpy as np
import torch

N_STATE = 16
P_COLS = 35
LN3 = float(np.log(3.0))


def bf(t):
    """Round to the nearest bf16 value (ties to even), kept in float64."""
    return t.to(torch.float32).to(torch.bfloat16).to(t.dtype)


class Bf16Linear(torch.autograd.Function):
    """y = bf(x) bf(W)^T with the gradient GEMMs on bf16-rounded operands."""

    @staticmethod
    def forward(ctx, x, W):
        ctx.save_for_backward(x, W)
        return bf(x) @ bf(W).T

    @staticmethod
    def backward(ctx, g):
        x, W = ctx.saved_tensors
        return bf(g) @ bf(W), bf(g).T @ bf(x)


def conv3d_causal(a, kern, bias, dims, K):
    """src/convnd.c:67-129 on one item: a [P, d] -> [P, d]."""
    d = a.shape[1]
    v = a.reshape(*dims, d)
    pad = torch.nn.functional.pad(v.permute(3, 0, 1, 2), (K - 1, 0, K - 1, 0, K - 1, 0))
    out = bias.reshape(1, 1, 1, d).expand(*dims, d).clone()
    for k0 in range(K):
        for k1 in range(K):
            for k2 in range(K):
                w = kern[(k0 * K + k1) * K + k2]
                sl = pad[:, k0:k0 + dims[0], k1:k1 + dims[1], k2:k2 + dims[2]].permute(1, 2, 3, 0)
                out = out + sl * w
    return out.reshape(-1, d)


def scan_nd(c, delta, A, B, C, dims):
    """src/scan_nd.c:173-185 with channel-shared B / C, one item.
    c [P, d]; delta [3, P, d]; A [3, d, N]; B, C [P, N] -> y [P, d]."""
    P, d = c.shape
    st = [dims[1] * dims[2], dims[2], 1]
    co = np.indices(dims).reshape(3, P)
    lvl = co.sum(0)
    order = np.argsort(lvl, kind="stable")
    bounds = np.searchsorted(lvl[order], np.arange(lvl.max() + 2))
    h = [None] * P
    dtbar = delta.mean(0)                                   # [P, d]
    for li in range(len(bounds) - 1):
        for p in order[bounds[li]:bounds[li + 1]]:
            hn = (dtbar[p] * c[p])[:, None] * B[p][None, :]  # [d, N]
            for k in range(3):
                if co[k, p] > 0:
                    hn = hn + torch.exp(delta[k, p][:, None] * A[k]) * h[p - st[k]]
            h[p] = hn
    return torch.stack([(h[p] * C[p][None, :]).sum(1) for p in range(P)])


def forward_loss(params, tokens, dims, K=3):
    """params: dict of float64 tensors (requires_grad as the caller wants);
    tokens: int64 [batch, P].  Returns the mean next-token loss."""
    batch, P = tokens.shape
    E = params["embedding"]
    total = 0.0
    for b in range(batch):
        x = E[tokens[b]]
        for layer in params["layers"]:
            a = Bf16Linear.apply(x, layer["W_a"])
            z = Bf16Linear.apply(x, layer["W_z"])
            v = conv3d_causal(a, layer["conv_kernel"], layer["conv_bias"], dims, K)
            c = v * torch.sigmoid(v)
            q = Bf16Linear.apply(c, layer["W_p"])
            delta = torch.stack([LN3 + torch.nn.functional.softplus(q[:, k][:, None] +
                                                                    layer["dt_bias"][k])
                                 for k in range(3)])
            Bm, Cm = q[:, 3:3 + N_STATE], q[:, 3 + N_STATE:3 + 2 * N_STATE]
            y = scan_nd(c, delta, -1.0 - torch.exp(layer["A_log"]), Bm, Cm, dims)
            g = y * (z * torch.sigmoid(z))
            x = x + Bf16Linear.apply(g, layer["W_out"])
        logits = Bf16Linear.apply(x, params["head"])
        tgt = torch.roll(tokens[b], -1)
        total = total + torch.nn.functional.cross_entropy(logits, tgt, reduction="sum")
    return total / (batch * P)
