#!/usr/bin/env python3
"""Generate the golden fixture that pins the oracle's DFlash draft network to
the reference's own draft graph.

Runs ``DFlashExportWrapper`` from export/dflash_export.py (the graph the
reference exports to ncnn and runs in DFlashDraftRuntime::run,
src/dflash_runtime.cpp:213-290) on CPU fp32 over a draft module tree with the
attribute names the wrapper reads (fc, hidden_norm, layers[i].self_attn.*,
layers[i].mlp, norm, config), loaded with the seeded synthetic draft weights
(oracle/hy_oracle.py::make_draft_weights, 2 layers). Inputs: 16 noise rows and
4 aux hidden-state blocks of 24 context rows from numpy's default_rng; RoPE
tables from the oracle's build_dflash_rope (positions 0..39, theta 10000); the
all-zero draft mask (src/dflash_runtime.cpp:50-58). The fixture keeps the seeds,
checksums of the inputs and the wrapper's output.

Usage: python tests/golden/make_dflash_draft_golden.py [--reference /path/to/HunyuanOCR-ncnn]
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "oracle"))

SEED, NORM_STD, LAYERS, CTX = 17, 0.1, 2, 24
INPUT_SEED = 4242


class RMSNorm(nn.Module):
    def __init__(self, weight: np.ndarray, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.from_numpy(np.asarray(weight, np.float32).copy()))
        self.eps = eps

    def forward(self, x):
        return self.weight * (x * torch.rsqrt(x.square().mean(-1, keepdim=True) + self.eps))


def linear(w: np.ndarray) -> nn.Linear:
    lin = nn.Linear(w.shape[1], w.shape[0], bias=False)
    lin.weight = nn.Parameter(torch.from_numpy(np.asarray(w, np.float32).copy()))
    return lin


class MLP(nn.Module):
    def __init__(self, lw):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = linear(lw.gate), linear(lw.up), linear(lw.down)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


def build_draft(O, dw):
    eps = O.RMS_EPS
    layers = nn.ModuleList()
    for lw in dw.layers:
        layer = nn.Module()
        attn = nn.Module()
        attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj = linear(lw.q), linear(lw.k), linear(lw.v), linear(lw.o)
        attn.q_norm, attn.k_norm = RMSNorm(lw.q_norm, eps), RMSNorm(lw.k_norm, eps)
        layer.self_attn = attn
        layer.mlp = MLP(lw)
        layer.input_layernorm = RMSNorm(lw.input_norm, eps)
        layer.post_attention_layernorm = RMSNorm(lw.post_norm, eps)
        layers.append(layer)
    draft = nn.Module()
    draft.config = SimpleNamespace(hidden_size=O.HIDDEN, num_attention_heads=O.NUM_Q_HEADS,
                                   num_key_value_heads=O.NUM_KV_HEADS, head_dim=O.HEAD_DIM)
    draft.target_layer_ids = list(O.DFLASH_TARGET_LAYER_IDS)
    draft.block_size = O.DFLASH_BLOCK
    draft.fc = linear(dw.fc)
    draft.hidden_norm = RMSNorm(dw.hidden_norm, eps)
    draft.layers = layers
    draft.norm = RMSNorm(dw.norm, eps)
    return draft


def inputs(O):
    rng = np.random.default_rng(INPUT_SEED)
    noise = rng.standard_normal((O.DFLASH_BLOCK, O.HIDDEN)).astype(np.float32)
    aux = [rng.standard_normal((CTX, O.HIDDEN)).astype(np.float32) for _ in range(4)]
    return noise, aux


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of the HunyuanOCR-ncnn source tree (its export/ directory is imported)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "export"))
    from dflash_export import DFlashExportWrapper
    import hy_oracle as O

    dw = O.make_draft_weights(LAYERS, SEED, 0.02, NORM_STD)
    wrapper = DFlashExportWrapper.from_draft(build_draft(O, dw)).eval()
    noise, aux = inputs(O)
    total = CTX + O.DFLASH_BLOCK
    cos = torch.from_numpy(O.build_dflash_rope(0, total, True)).reshape(1, 1, total, O.HEAD_DIM)
    sin = torch.from_numpy(O.build_dflash_rope(0, total, False)).reshape(1, 1, total, O.HEAD_DIM)
    mask = torch.zeros(1, 1, O.DFLASH_BLOCK, total)
    with torch.no_grad():
        out = wrapper(torch.from_numpy(noise)[None], *[torch.from_numpy(a)[None] for a in aux], cos, sin, mask)
    np.savez_compressed(HERE / "dflash_draft_2l.npz", seed=SEED, norm_std=NORM_STD, layers=LAYERS, ctx=CTX,
                        input_seed=INPUT_SEED, noise_sum=np.float64(noise.astype(np.float64).sum()),
                        aux_sum=np.float64(sum(a.astype(np.float64).sum() for a in aux)),
                        out=out[0].numpy().astype(np.float32))
    print("wrote", HERE / "dflash_draft_2l.npz", out.shape)


if __name__ == "__main__":
    main()
