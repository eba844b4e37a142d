"""PyTorch restatement of the reference forward for full-size checks.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  It restates the chunked
reference (core/attention_fast_chunked.py:63-173, with core/utils.py:4-52)
in torch so that it runs on the GPU box at BASELINE sizes, one batch row at a
time to bound memory.  It is pinned against the numpy oracle and the golden
fixtures by tests/test_torch_ref.py.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F


def skew_from_vec(v: torch.Tensor, d: int) -> torch.Tensor:
    """core/utils.py:4-27, vectorised (row-major strict upper triangle)."""
    iu = torch.triu_indices(d, d, offset=1, device=v.device)
    A = v.new_zeros(*v.shape[:-1], d, d)
    A[..., iu[0], iu[1]] = v
    A[..., iu[1], iu[0]] = -v
    return A


def core_forward(a_all: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 edge_scale: float, scale: float, block_k: int = 64, return_P: bool = False):
    """(a_all (B,H,L,m) unscaled, q,k,v (B,H,L,d)) -> heads (B,H,L,d) in a_all's dtype.

    core/attention_fast_chunked.py:77 (scale), :86-94 (expm, prefix),
    :108-110 (transport), :119-171 (causal fold, out = P o).
    """
    dt = a_all.dtype
    B, H, L, m = a_all.shape
    d = q.shape[-1]
    a_all = a_all * edge_scale
    q, k, v = q.to(dt), k.to(dt), v.to(dt)
    # expm in batches of at most 4096 matrices: keeps every library call small
    a_adj = a_all[:, :, :-1].reshape(-1, m)
    G = torch.empty(a_adj.shape[0], d, d, dtype=dt, device=a_all.device)
    for i0 in range(0, a_adj.shape[0], 4096):
        G[i0:i0 + 4096] = torch.matrix_exp(skew_from_vec(a_adj[i0:i0 + 4096], d))
    G = G.view(B, H, L - 1, d, d)
    P = torch.empty(B, H, L, d, d, dtype=dt, device=a_all.device)
    Pt = torch.eye(d, dtype=dt, device=a_all.device).expand(B, H, d, d).clone()
    P[:, :, 0] = Pt
    for t in range(L - 1):
        Pt = G[:, :, t] @ Pt
        P[:, :, t + 1] = Pt
    del G
    qh = torch.einsum("bhide,bhid->bhie", P, q)
    kh = torch.einsum("bhjde,bhjd->bhje", P, k)
    vh = torch.einsum("bhjde,bhjd->bhje", P, v)
    neg = torch.finfo(dt).min
    m_run = torch.full((B, H, L), neg, dtype=dt, device=a_all.device)
    l_run = torch.zeros((B, H, L), dtype=dt, device=a_all.device)
    o_run = torch.zeros((B, H, L, d), dtype=dt, device=a_all.device)
    idx = torch.arange(L, device=a_all.device)
    for k0 in range(0, L, block_k):
        k1 = min(k0 + block_k, L)
        s = torch.einsum("bhie,bhje->bhij", qh, kh[:, :, k0:k1]) * scale
        allowed = idx.view(L, 1) >= idx[k0:k1].view(1, -1)
        s = s.masked_fill(~allowed.view(1, 1, L, -1), neg)
        m_new = torch.maximum(m_run, s.max(dim=-1).values)
        corr = torch.exp(m_run - m_new)
        p = torch.exp(s - m_new.unsqueeze(-1))
        l_run = l_run * corr + p.sum(dim=-1)
        o_run = o_run * corr.unsqueeze(-1) + torch.einsum("bhij,bhje->bhie", p, vh[:, :, k0:k1])
        m_run = m_new
    o_run = o_run / l_run.clamp_min(1e-20).unsqueeze(-1)
    heads = torch.einsum("bhide,bhie->bhid", P, o_run)
    return (heads, P) if return_P else heads


def module_forward(sd: dict, x: torch.Tensor, n_heads: int, edge_scale: float,
                   dtype=torch.float32, batch_slice: int = 1,
                   head_group: Optional[int] = None) -> torch.Tensor:
    """Whole reference forward (causal, tril) in ``dtype`` on x's device, batch rows in slices.

    ``head_group``: run the core region (expm, prefix, transport, attention)
    over groups of this many heads at a time.  Heads never mix between the qkv
    split and the out projection (core/attention_fast_chunked.py:69-171 works
    per (b, h) throughout), so the result is the same; only the memory of P
    (B, H, L, d, d) shrinks to that of one group."""
    dev = x.device
    W = {k: v.to(device=dev, dtype=dtype) for k, v in sd.items()
         if not k.startswith(("gqproj", "gkproj"))}
    B, L, D = x.shape
    H = n_heads
    d = D // H
    m = d * (d - 1) // 2
    ys = []
    for b0 in range(0, B, batch_slice):
        xb = x[b0:b0 + batch_slice].to(dtype)
        Bb = xb.shape[0]
        qkv = F.linear(xb, W["qkv.weight"]).view(Bb, L, H, 3 * d)
        q, k, v = (t.transpose(1, 2) for t in qkv.chunk(3, dim=-1))
        pair = torch.cat([xb, torch.roll(xb, -1, dims=1)], dim=-1)
        h = F.gelu(F.linear(pair, W["edge_mlp.0.weight"], W["edge_mlp.0.bias"]))
        a = F.linear(h, W["edge_mlp.2.weight"], W["edge_mlp.2.bias"])
        a = a.view(Bb, L, H, m).transpose(1, 2)
        hg = head_group or H
        heads = torch.cat([core_forward(a[:, h0:h0 + hg], q[:, h0:h0 + hg], k[:, h0:h0 + hg],
                                        v[:, h0:h0 + hg], edge_scale, 1.0 / math.sqrt(d))
                           for h0 in range(0, H, hg)], dim=1)
        del a, h
        ys.append(F.linear(heads.transpose(1, 2).reshape(Bb, L, D), W["out.weight"]))
    return torch.cat(ys, 0)
