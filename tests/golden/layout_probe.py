"""Struct-layout probe of the k-mamba model API.

Compiles a small C program against a kmamba.h (this repository's include/
or the reference's include/) that prints sizeof and offsetof of every
field of the structs callers allocate or read (MBMatrix, MBConfig,
MBOptimState, MambaBlockWorkspace, MambaBlock, KMambaConfig, KMamba,
MBOptimConfig).  `python tests/golden/layout_probe.py <include dir>` writes
the reference fixture tests/golden/kmamba_layout.json; tests compare the
repository header against it.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

FIELDS = {
    "MBMatrix": ["data", "rows", "cols"],
    "MBOptimConfig": ["lr", "mu", "beta2", "eps", "clip_norm", "weight_decay"],
    "MBConfig": ["dim", "state_size", "seq_len", "mimo_rank", "dt_scale", "dt_min", "dt_max",
                 "use_fp16", "use_bf16", "loss_scale", "spatial_ndims", "spatial_dims",
                 "use_convnd", "convnd_K", "convnd_ndims"],
    "MBOptimState": ["type", "step"] + [f"g_{n}" for n in (
        "W_in", "W_out", "A_log", "W_B", "W_C", "b_B", "b_C", "delta_proj", "theta",
        "lambda_proj")] + [f"{k}_{n}" for n in (
            "W_in", "W_out", "A_log", "W_B", "W_C", "b_B", "b_C", "delta_proj", "theta",
            "lambda_proj") for k in ("m", "v")],
    "MambaBlockWorkspace": ["hidden", "delta", "scan_B", "scan_C", "scan_delta", "scan_h"],
    "MambaBlock": ["config", "W_in", "W_out", "A_log", "W_B", "W_C", "delta_proj", "b_B",
                   "b_C", "theta", "lambda_proj", "wavefront_plan", "convnd_kernel",
                   "convnd_bias", "hidden", "delta", "scan_B", "scan_C", "scan_delta",
                   "scan_h", "opt_state"],
    "KMambaConfig": ["vocab_size", "dim", "state_size", "seq_len", "n_layers", "mimo_rank",
                     "dt_scale", "dt_min", "dt_max", "spatial_ndims", "spatial_dims",
                     "use_convnd", "convnd_K", "convnd_ndims", "weight_tying"],
    "KMamba": ["cfg", "embedding", "head", "layers", "for_training", "opt_blocks",
               "lr_embed_head", "weight_decay", "m_embedding", "v_embedding", "m_head",
               "v_head", "step_embed_head", "last_grad_norm", "last_grad_over_clip",
               "last_grad_would_clip"],
}


def probe(include_dirs: list[str]) -> dict:
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "kmamba.h"',
             'int main(void) {']
    for s, fs in FIELDS.items():
        lines.append(f'  printf("%s sizeof %zu\\n", "{s}", sizeof({s}));')
        for f in fs:
            lines.append(f'  printf("%s %s %zu\\n", "{s}", "{f}", offsetof({s}, {f}));')
    lines += ['  return 0;', '}']
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "p.c"), os.path.join(d, "p")
        open(src, "w").write("\n".join(lines))
        cmd = ["gcc", "-o", exe, src] + [f"-I{i}" for i in include_dirs]
        subprocess.run(cmd, check=True, capture_output=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    res: dict = {}
    for ln in out.splitlines():
        s, f, v = ln.split()
        res.setdefault(s, {})[f] = int(v)
    return res


if __name__ == "__main__":
    inc = sys.argv[1]
    extra = [os.path.join(os.path.dirname(inc.rstrip("/")), "cpu", "include")]
    lay = probe([inc] + extra)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kmamba_layout.json")
    json.dump(lay, open(out, "w"), indent=1, sort_keys=True)
    print("wrote", out)
