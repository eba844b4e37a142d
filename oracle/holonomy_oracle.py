"""CPU oracle for the causal forward of path-ordered geometric attention.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference
leg of ``bench.py`` may use it, and only as the checker (or the timed CPU
baseline), never as the thing that is measured or shipped.

This is a plain-numpy restatement of the reference's forward, written from the
reference's behaviour (SiddhiMali/HolonomyAwareAttention):

* module constructor / parameter shapes      core/attention_fast_chunked.py:37-60
* q/k/v split per head ([q_h | k_h | v_h])    core/attention_fast_chunked.py:69-71
* edge MLP on (x_t, x_{t+1}), roll wraps      core/attention_fast_chunked.py:73-79
* skew_from_vec (row-major upper triangle)    core/utils.py:4-27
* so_exp = torch.matrix_exp                   core/utils.py:30-52
* prefix products P_0 = I, P_{t+1} = G_t P_t  core/attention_fast_chunked.py:89-94
* holonomy Hol = G_close P_{L-1}              core/attention_fast_chunked.py:95
* transport q^ = P^T q etc.                   core/attention_fast_chunked.py:108-110
* causal softmax fold, finfo.min masking,
  l.clamp_min(1e-20), out = P o               core/attention_fast_chunked.py:119-171
* output projection                           core/attention_fast_chunked.py:172-173
* any mask, the wrap pairs through Hol, the
  inert ablation, the additive link           core/attention.py:69-195 (forward_general)

The reference's causal+tril result equals core/attention.py:156-195 (its O(L^3)
arc walk); the golden fixtures under tests/golden pin both.

Matrix exponential.  The reference calls ``torch.matrix_exp`` (PyTorch, the
image's torch 2.11.0; the reference pins no version).  Its published method is
a truncated Taylor series with scaling and squaring (Bader, Blanes & Casas,
"Computing the matrix exponential with an optimized Taylor polynomial
approximation", Mathematics 7 (2019) 1174).  ``expm`` below restates that
method class: a Taylor polynomial (degree 8 in float32, 13 in float64)
evaluated by Horner's rule after scaling A by 2^-s so that ||A||_1 2^-s <= 1/2,
followed by s squarings.  The truncation error is below half an ulp in the
working precision, so the oracle's expm differs from torch's only by
rounding.

The softmax fold is evaluated in one pass over the causal row (a full row
softmax with the same ``finfo.min`` masking) instead of the reference's
64-key blocks; both are the same function and differ only by rounding.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional

import numpy as np

try:  # exact-erf GELU, as nn.GELU() (core/attention_fast_chunked.py:56-59)
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover - scipy is in the image
    _erf = np.vectorize(math.erf)


# ---------------------------------------------------------------------------
# parameters
# ---------------------------------------------------------------------------
@dataclass
class Params:
    """Weights of PathOrderedGeometricMHA, named as in its state_dict."""

    qkv: np.ndarray          # (3D, D)           qkv.weight
    out: np.ndarray          # (D, D)            out.weight
    w1: np.ndarray           # (4D, 2D)          edge_mlp.0.weight
    b1: np.ndarray           # (4D,)             edge_mlp.0.bias
    w2: np.ndarray           # (m*H, 4D)         edge_mlp.2.weight
    b2: np.ndarray           # (m*H,)            edge_mlp.2.bias
    gq: Optional[np.ndarray] = None   # (m*H, D)  gqproj.weight (link_mode "additive")
    gk: Optional[np.ndarray] = None   # (m*H, D)  gkproj.weight

    @staticmethod
    def from_state_dict(sd, dtype=np.float64) -> "Params":
        def g(k):
            if k not in sd:
                return None
            t = sd[k]
            if hasattr(t, "detach"):
                t = t.detach().float().cpu().numpy() if str(t.dtype) == "torch.bfloat16" \
                    else t.detach().cpu().numpy()
            return np.asarray(t, dtype=dtype)

        return Params(g("qkv.weight"), g("out.weight"), g("edge_mlp.0.weight"),
                      g("edge_mlp.0.bias"), g("edge_mlp.2.weight"), g("edge_mlp.2.bias"),
                      g("gqproj.weight"), g("gkproj.weight"))

    def astype(self, dtype) -> "Params":
        return Params(*(None if a is None else np.asarray(a, dtype=dtype) for a in
                        (self.qkv, self.out, self.w1, self.b1, self.w2, self.b2, self.gq, self.gk)))


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round float32/64 values to bfloat16 (round-to-nearest-even), returned as float32."""
    f = np.asarray(a, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(f), f, out)


# ---------------------------------------------------------------------------
# elementary pieces
# ---------------------------------------------------------------------------
def gelu(x: np.ndarray) -> np.ndarray:
    """nn.GELU() (exact erf form)."""
    return (0.5 * x * (1.0 + _erf(x / math.sqrt(2.0)))).astype(x.dtype)


def triu_index(d: int):
    """Row-major strict upper triangle order used by skew_from_vec (core/utils.py:20-26)."""
    return np.triu_indices(d, k=1)


def skew_from_vec(v: np.ndarray, d: int) -> np.ndarray:
    """A[i,j] = v[idx], A[j,i] = -v[idx] for i<j, idx row-major (core/utils.py:4-27)."""
    m = v.shape[-1]
    if m != d * (d - 1) // 2:
        raise ValueError(f"Expected last dim {d * (d - 1) // 2}, got {m}")
    A = np.zeros(v.shape[:-1] + (d, d), dtype=v.dtype)
    iu, ju = triu_index(d)
    A[..., iu, ju] = v
    A[..., ju, iu] = -v
    return A


def expm(A: np.ndarray) -> np.ndarray:
    """Batched matrix exponential in A's dtype (Taylor + scaling/squaring).

    Restates the published method behind torch.matrix_exp (core/utils.py:52);
    see the module docstring.
    """
    dt = A.dtype
    d = A.shape[-1]
    flat = A.reshape(-1, d, d)
    out = np.empty_like(flat)
    norms = np.abs(flat).sum(axis=-2).max(axis=-1)          # 1-norm per matrix
    s_all = np.maximum(0, np.ceil(np.log2(np.maximum(norms, 1e-300) / 0.5))).astype(int)
    eye = np.eye(d, dtype=dt)
    # ||X||_1 <= 1/2 after scaling: the remainder of the degree-q Taylor
    # polynomial is below 0.5^(q+1)/(q+1)!, i.e. 5e-9 for q=8 (float32) and
    # 7e-16 for q=13 (float64), under half an ulp of the result.
    q = 8 if dt == np.float32 else 13
    for s in np.unique(s_all):
        sel = np.nonzero(s_all == s)[0]
        X = flat[sel] * dt.type(2.0 ** -int(s))
        # Horner: T = I + X(I + X/2(I + X/3(...)))
        T = eye + X / dt.type(q)
        for k in range(q - 1, 0, -1):
            T = eye + (X @ T) / dt.type(k)
        for _ in range(int(s)):
            T = T @ T
        out[sel] = T
    return out.reshape(A.shape)


# ---------------------------------------------------------------------------
# forward
# ---------------------------------------------------------------------------
def project_qkv(p: Params, x: np.ndarray, n_heads: int):
    """qkv(x).view(B,L,H,3d).chunk(3) -> (B,H,L,d) each (core/attention_fast_chunked.py:69-71)."""
    B, L, D = x.shape
    d = D // n_heads
    qkv = (x @ p.qkv.T).reshape(B, L, n_heads, 3 * d)
    q, k, v = qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:]
    return (q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3))


def edge_generators(p: Params, x: np.ndarray, n_heads: int, edge_scale: float) -> np.ndarray:
    """a_all (B,H,L,m) = edge_scale * edge_mlp([x_t, x_{t+1 mod L}]) (core/attention_fast_chunked.py:73-77)."""
    B, L, D = x.shape
    d = D // n_heads
    m = d * (d - 1) // 2
    pair = np.concatenate([x, np.roll(x, -1, axis=1)], axis=-1)
    h = gelu(pair @ p.w1.T + p.b1)
    a = (h @ p.w2.T + p.b2).reshape(B, L, n_heads, m).transpose(0, 2, 1, 3)
    return a * x.dtype.type(edge_scale)


def edge_generators_additive(p: Params, x: np.ndarray, n_heads: int, edge_scale: float) -> np.ndarray:
    """link_mode "additive": a_t = edge_scale * (gq(x_t) + gk(x_{t+1 mod L})), (B,H,L,m)
    (core/attention.py:98-101: edges t < L-1 pair gq_t with gk_{t+1}, the closing
    edge gq_{L-1} with gk_0)."""
    B, L, D = x.shape
    d = D // n_heads
    m = d * (d - 1) // 2
    a = x @ p.gq.T + np.roll(x @ p.gk.T, -1, axis=1)
    return a.reshape(B, L, n_heads, m).transpose(0, 2, 1, 3) * x.dtype.type(edge_scale)


def prefix_products(G_adj: np.ndarray) -> np.ndarray:
    """P_0 = I, P_{t+1} = G_t P_t (core/attention_fast_chunked.py:89-94). G_adj (...,L-1,d,d)."""
    *lead, Lm1, d, _ = G_adj.shape
    L = Lm1 + 1
    P = np.empty(tuple(lead) + (L, d, d), dtype=G_adj.dtype)
    Pt = np.broadcast_to(np.eye(d, dtype=G_adj.dtype), tuple(lead) + (d, d)).copy()
    P[..., 0, :, :] = Pt
    for t in range(L - 1):
        Pt = G_adj[..., t, :, :] @ Pt
        P[..., t + 1, :, :] = Pt
    return P


def causal_attention(qh: np.ndarray, kh: np.ndarray, vh: np.ndarray, scale: float) -> np.ndarray:
    """Causal softmax(q^ k^T * scale) v^ with finfo.min masking and l.clamp_min(1e-20)
    (core/attention_fast_chunked.py:119-168, tril mask)."""
    dt = qh.dtype
    L = qh.shape[-2]
    s = (qh @ np.swapaxes(kh, -1, -2)) * dt.type(scale)
    allowed = np.tril(np.ones((L, L), dtype=bool))
    s = np.where(allowed, s, np.finfo(dt).min)
    mx = s.max(axis=-1, keepdims=True)
    e = np.exp(s - mx)
    l = np.maximum(e.sum(axis=-1, keepdims=True), dt.type(1e-20))
    return (e @ vh) / l


def forward(p: Params, x: np.ndarray, n_heads: int, edge_scale: float,
            dtype=np.float64, return_intermediates: bool = False):
    """y = PathOrderedGeometricMHA.forward(x, attn_mask=tril(L)) in ``dtype``.

    Returns y (B,L,D), or (y, dict) with q,k,v,P,Hol,qh,kh,vh,o,heads when
    ``return_intermediates``.
    """
    p = p.astype(dtype)
    x = np.asarray(x, dtype=dtype)
    B, L, D = x.shape
    H = n_heads
    d = D // H
    q, k, v = project_qkv(p, x, H)
    a_all = edge_generators(p, x, H, edge_scale)
    G_adj = expm(skew_from_vec(a_all[:, :, :-1], d))
    G_close = expm(skew_from_vec(a_all[:, :, -1], d))
    P = prefix_products(G_adj)
    Hol = G_close @ P[:, :, L - 1]
    PT = np.swapaxes(P, -1, -2)
    qh = (PT @ q[..., None])[..., 0]
    kh = (PT @ k[..., None])[..., 0]
    vh = (PT @ v[..., None])[..., 0]
    o = causal_attention(qh, kh, vh, 1.0 / math.sqrt(d))
    heads = (P @ o[..., None])[..., 0]                       # out_i = P_i o_i
    y = heads.transpose(0, 2, 1, 3).reshape(B, L, D) @ p.out.T
    if not return_intermediates:
        return y
    return y, dict(q=q, k=k, v=v, a_all=a_all, P=P, Hol=Hol, qh=qh, kh=kh, vh=vh, o=o,
                   heads=heads)


def masked_attention(qh, kh, vh, scale, mask=None, kw=None, vw=None):
    """softmax_j(q_i . key_ij * scale) over ALL keys, masked entries at finfo.min (so a
    fully masked row averages uniformly, as core/attention_fast_chunked.py:142-148 does),
    the sum divided by l.clamp_min(1e-20).  key_ij / value_ij are kh_j / vh_j for j <= i
    and, when kw / vw are given, kw_j / vw_j for the wrap pairs j > i."""
    L = qh.shape[-2]
    s = (qh @ np.swapaxes(kh, -1, -2)) * scale
    base = np.tril(np.ones((L, L), dtype=bool))
    if kw is not None:
        s = np.where(base, s, (qh @ np.swapaxes(kw, -1, -2)) * scale)
    if mask is not None:
        s = np.where(np.asarray(mask, dtype=bool), s, np.finfo(qh.dtype).min)
    mx = s.max(axis=-1, keepdims=True)
    pr = np.exp(s - mx)
    l = pr.sum(axis=-1, keepdims=True)
    if kw is None:
        o = pr @ vh
    else:
        o = (pr * base) @ vh + (pr * ~base) @ vw
    return o / np.maximum(l, 1e-20)


def forward_general(p: Params, x: np.ndarray, n_heads: int, edge_scale: float, mask=None,
                    mode: str = "causal", link_mode: str = "interaction", dtype=np.float64,
                    return_intermediates: bool = False):
    """core/attention.py:69-195 for any mask (None = all allowed), both modes and
    both link forms, in the P / Hol form of core/attention_fast_chunked.py:98-171.

    "causal" (arc transport, core/attention.py:156-165): the transport j -> i walks
    the ring, G_arc[i][j] = P_i P_j^T for j <= i and P_i Hol P_j^T for the wrap
    pairs j > i, so with q^ = P^T q etc. the wrap pairs see Hol k^_j and Hol v^_j.
    (core/attention_fast_chunked.py:116-117 applies Hol^T there; under the tril
    mask those pairs never count.)  "inert" (:166-169): G_arc[i][j] = P_i^T P_j, so
    q~ = P q, k~ = P k, v~ = P v and out_i = P_i^T o_i."""
    p = p.astype(dtype)
    x = np.asarray(x, dtype=dtype)
    B, L, D = x.shape
    H = n_heads
    d = D // H
    q, k, v = project_qkv(p, x, H)
    if link_mode == "interaction":
        a_all = edge_generators(p, x, H, edge_scale)
    elif link_mode == "additive":
        a_all = edge_generators_additive(p, x, H, edge_scale)
    else:
        raise ValueError(link_mode)
    G_adj = expm(skew_from_vec(a_all[:, :, :-1], d))
    G_close = expm(skew_from_vec(a_all[:, :, -1], d))
    P = prefix_products(G_adj)
    Hol = G_close @ P[:, :, L - 1]
    scale = 1.0 / math.sqrt(d)
    if mode == "causal":
        PT = np.swapaxes(P, -1, -2)
        qh, kh, vh = ((PT @ t[..., None])[..., 0] for t in (q, k, v))
        kw = (Hol[:, :, None] @ kh[..., None])[..., 0]
        vw = (Hol[:, :, None] @ vh[..., None])[..., 0]
        o = masked_attention(qh, kh, vh, scale, mask, kw, vw)
        heads = (P @ o[..., None])[..., 0]
    elif mode == "inert":
        qh, kh, vh = ((P @ t[..., None])[..., 0] for t in (q, k, v))
        o = masked_attention(qh, kh, vh, scale, mask)
        heads = (np.swapaxes(P, -1, -2) @ o[..., None])[..., 0]
    else:
        raise ValueError(mode)
    y = heads.transpose(0, 2, 1, 3).reshape(B, L, D) @ p.out.T
    if not return_intermediates:
        return y
    return y, dict(P=P, Hol=Hol, a_all=a_all, o=o, heads=heads)


def core_forward(a_all: np.ndarray, q: np.ndarray, k: np.ndarray, v: np.ndarray,
                 scale: float, edge_scale: float = 1.0, dtype=np.float64) -> np.ndarray:
    """The core region alone: (a_all (B,H,L,m), q,k,v (B,H,L,d)) -> heads (B,H,L,d).

    ``a_all`` is the unscaled edge-MLP output; it is multiplied by edge_scale
    first, as core/attention_fast_chunked.py:77 does.
    """
    a_all = np.asarray(a_all, dtype=dtype) * np.dtype(dtype).type(edge_scale)
    q, k, v = (np.asarray(t, dtype=dtype) for t in (q, k, v))
    d = q.shape[-1]
    P = prefix_products(expm(skew_from_vec(a_all[:, :, :-1], d)))
    PT = np.swapaxes(P, -1, -2)
    qh = (PT @ q[..., None])[..., 0]
    kh = (PT @ k[..., None])[..., 0]
    vh = (PT @ v[..., None])[..., 0]
    o = causal_attention(qh, kh, vh, scale)
    return (P @ o[..., None])[..., 0]


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))
