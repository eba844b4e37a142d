"""Seeded weights and inputs, drawn in the reference's RNG order.  TEST INFRASTRUCTURE ONLY.

The reference harness seeds, builds the module with default init and then draws
x (kernel/eval_checkpoint_kernel.py:58-70).  Module parameters are created in
the order qkv, out, gqproj, gkproj, edge_mlp.0, edge_mlp.2
(core/attention_fast_chunked.py:51-59), so default init consumes the CPU RNG in
that order; this helper repeats it with plain nn.Linear layers.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from .holonomy_oracle import Params, round_bf16


def seeded_state_dict(D: int, H: int, seed: int):
    torch.manual_seed(seed)
    d = D // H
    m = d * (d - 1) // 2
    qkv = nn.Linear(D, 3 * D, bias=False)
    out = nn.Linear(D, D, bias=False)
    gq = nn.Linear(D, m * H, bias=False)
    gk = nn.Linear(D, m * H, bias=False)
    e0 = nn.Linear(2 * D, 4 * D)
    e2 = nn.Linear(4 * D, m * H)
    return {
        "qkv.weight": qkv.weight.data, "out.weight": out.weight.data,
        "gqproj.weight": gq.weight.data, "gkproj.weight": gk.weight.data,
        "edge_mlp.0.weight": e0.weight.data, "edge_mlp.0.bias": e0.bias.data,
        "edge_mlp.2.weight": e2.weight.data, "edge_mlp.2.bias": e2.bias.data,
    }


def seeded_case(D: int, H: int, seed: int, B: int, L: int, bf16_round: bool = False):
    """(state_dict, x) exactly as the golden generator draws them."""
    sd = seeded_state_dict(D, H, seed)
    x = torch.randn(B, L, D)
    if bf16_round:
        sd = {k: v.to(torch.bfloat16).float() for k, v in sd.items()}
        x = x.to(torch.bfloat16).float()
    return sd, x


def checksums(sd):
    out = {}
    for k, t in sd.items():
        a = t.detach().double().cpu().numpy().ravel()
        out[k] = np.array([a.sum(), (a * a).sum(), *a[:4]], dtype=np.float64)
    return out


def params_of(sd, dtype=np.float64) -> Params:
    return Params.from_state_dict(sd, dtype=dtype)


__all__ = ["seeded_state_dict", "seeded_case", "checksums", "params_of", "round_bf16"]
