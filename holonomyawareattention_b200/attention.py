"""Drop-in PathOrderedGeometricMHA backed by the sm_100a kernels of libhoa.so.

Same constructor arguments, attributes, submodules (in the same creation
order, so seeded default init and state_dict keys match) and forward
signature as the reference module (core/attention.py:27-74,
core/attention_fast_chunked.py:37-60, 98).  The reference's experiments pick
the module by import path (`--attn-module`, experiments/session_cherry.py:278,
445), so `--attn-module holonomyawareattention_b200` selects this one.

The hot path is the reference kernel drop-in's case (kernel/attention_kernel.py:
193-208): mode "causal" with attn_mask exactly tril(L).  Every other input of
core/attention.py also runs on libhoa, through a general fp32 path: no mask or
any (L, L) bool mask (the wrap pairs j > i transported through the closing
edge by Hol, core/attention.py:156-165), mode "inert" (:166-169), link_mode
"additive" (:98-101).  return_geometry=True also returns {"C": P, "H": Hol} as
core/attention_fast_chunked.py:175-177 does.  Dropout must be inactive and the
input on CUDA; anything else raises NotImplementedError: there is no CPU or
PyTorch fallback.

Forward only.  The projections (qkv, edge_mlp, out) run as PyTorch GEMMs;
everything between them — link rotations, prefix composition, transport,
causal attention and the inverse transport — runs in libhoa.
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops


def _is_exact_tril(mask: Optional[torch.Tensor], L: int) -> bool:
    """Same rule as kernel/attention_kernel.py:193-199."""
    if mask is None or tuple(mask.shape) != (L, L):
        return False
    tril = torch.ones(L, L, dtype=torch.bool, device=mask.device).tril()
    return bool(torch.equal(mask.bool(), tril))


class PathOrderedGeometricMHA(nn.Module):
    """Path-ordered geometric multi-head attention (causal forward on B200).

    Attributes mirror the reference: h, d, m_dim, edge_scale, scale, mode,
    link_mode, qkv, out, dropout, gqproj, gkproj, edge_mlp.

    ``generator_precision`` (not in the reference) controls how the edge
    generators are produced when the module runs in bfloat16:
      * "bf16": the hidden activations are rounded to bf16 and the second GEMM
        accumulates and writes fp32 (the reference's own bf16 module also
        rounds the generators themselves and composes the rotations in bf16);
        about 1e-3 relative error per generator entry, whose effect on the
        output grows as sqrt(T) along the path product (measured at d_model
        1536, H 16: output rel-L2 4.5e-3 at T = 4096, 1.5e-2 over the last
        quarter of T = 16384);
      * "split": the hidden layer is kept in fp32 and the second GEMM runs over
        its high and low bf16 halves ([h_hi | h_lo] against [W2^T ; W2^T], fp32
        output), so the generators carry ~16 bits (3.7e-3 at both lengths) at
        twice the GEMM cost;
      * "split8": the high half as in "split", the low half (at most 2^-9 of
        the high one) in e4m3 against W2 in e4m3 in an fp8 GEMM that adds into
        the bf16 GEMM's fp32 output: ~13-bit generators at 1.5 times the
        bf16 GEMM's cost;
      * "auto" (default): "bf16" for sequences of up to 8192 positions, "split8"
        beyond ("split" where the fp8 GEMM does not take the shapes).
    In float32 the edge MLP runs in fp32, exactly as the reference.
    """

    def __init__(self, d_model: int, n_heads: int = 4, dropout: float = 0.0,
                 edge_scale: float = 0.1, mode: str = "causal"):
        super().__init__()
        if d_model % n_heads != 0:
            raise ValueError("d_model must be divisible by n_heads")
        if mode not in ("causal", "inert"):
            raise ValueError("mode must be 'causal' or 'inert'")
        self.h = n_heads
        self.d = d_model // n_heads
        self.m_dim = self.d * (self.d - 1) // 2
        self.edge_scale = edge_scale
        self.scale = 1.0 / math.sqrt(self.d)
        self.mode = mode

        # creation order matches core/attention_fast_chunked.py:51-59
        self.qkv = nn.Linear(d_model, 3 * d_model, bias=False)
        self.out = nn.Linear(d_model, d_model, bias=False)
        self.dropout = nn.Dropout(dropout)
        self.gqproj = nn.Linear(d_model, self.m_dim * n_heads, bias=False)
        self.gkproj = nn.Linear(d_model, self.m_dim * n_heads, bias=False)
        self.edge_mlp = nn.Sequential(
            nn.Linear(2 * d_model, 4 * d_model), nn.GELU(),
            nn.Linear(4 * d_model, self.m_dim * n_heads),
        )
        self.link_mode = "interaction"
        self.generator_precision = "auto"
        self.chunk: Optional[int] = None          # None: hoa_plan_chunk decides
        self._tril_ok: Dict[Tuple, bool] = {}

    # ------------------------------------------------------------------
    def _check_supported(self, x: torch.Tensor, attn_mask, return_geometry: bool) -> None:
        why = None
        if self.mode not in ("causal", "inert"):
            why = "mode must be 'causal' or 'inert'"
        elif self.link_mode not in ("interaction", "additive"):
            why = "link_mode must be 'interaction' or 'additive'"
        elif not x.is_cuda:
            why = "input must be a CUDA tensor"
        elif self.training and self.dropout.p != 0.0:
            why = "dropout must be 0 or the module in eval mode"
        elif x.dim() != 3 or x.shape[-1] != self.h * self.d:
            why = f"x must be (B, L, {self.h * self.d})"
        elif torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters())):
            why = "forward-only kernels: call under torch.no_grad() / torch.inference_mode()"
        elif attn_mask is not None and (tuple(attn_mask.shape) != (x.shape[1], x.shape[1])
                                        or attn_mask.dtype != torch.bool):
            why = "attn_mask must be None or an (L, L) bool tensor (True = allowed)"
        if why is not None:
            raise NotImplementedError(f"PathOrderedGeometricMHA (B200): {why}")

    def _mask_is_tril(self, mask, L: int) -> bool:
        if mask is None:
            return False
        key = (mask.data_ptr(), tuple(mask.shape), mask.dtype, mask._version, str(mask.device))
        ok = self._tril_ok.get(key)
        if ok is None:
            ok = _is_exact_tril(mask, L)
            if len(self._tril_ok) > 64:
                self._tril_ok.clear()
            self._tril_ok[key] = ok
        return ok

    def edge_generators(self, x: torch.Tensor) -> torch.Tensor:
        """a_all (B, L, H*m) in fp32, unscaled: edge_mlp([x_t, x_{t+1 mod L}]), in the
        reference's packed order.

        core/attention_fast_chunked.py:73-76 (the edge_scale multiply happens in
        the link kernel).
        """
        a, bias, layout = self._edge_generators_nobias(x)
        if bias is not None:
            a = a + bias
        return ops.gen_from_banked(a, self.h, self.d) if layout == "banked" else a

    def _gen_layout(self) -> str:
        """Generator layout handed to the link kernel: "banked" where the head dim
        allows it (d % 32 == 0), else the reference's packed upper triangle.  The
        banked layout costs nothing here: the projection's output rows are
        permuted once (and padded with a few zero rows), see _w2_rows."""
        return "banked" if self.d % 32 == 0 else "packed"

    def _w2_rows(self, w: torch.Tensor, b: torch.Tensor):
        """The output projection's weight (H*m x F) and bias with rows in the
        generator layout (zero rows at the banked layout's unused slots)."""
        if self._gen_layout() == "packed":
            return w, b
        idx = ops.gen_banked_index(self.d, self.h, w.device)
        width = self.h * ops.gen_stride(self.d, "banked")
        wb = w.new_zeros(width, w.shape[1])
        wb[idx] = w
        bb = b.new_zeros(width)
        bb[idx] = b
        return wb, bb

    def _edge_generators_nobias(self, x: torch.Tensor, x_next: Optional[torch.Tensor] = None,
                                seq_len: Optional[int] = None):
        """(a_all, bias or None, layout) with a_all (B, L, H*width) fp32, unscaled,
        in the generator layout ``layout`` (_gen_layout).

        In bfloat16 the second GEMM (hoa_edge_gemm, cuBLASLt) adds the MLP's fp32
        output bias in its epilogue, so a_all already carries it and the bias
        returned is None; the large fp32 output is written once by the GEMM and
        read once by the link kernel.  In float32 nn.Linear adds it.

        ``x_next`` (B, 1, D), for a sequence shard: the token that follows the
        shard (the next shard's first token; the whole sequence's first token
        for the last shard, as the reference's roll wraps).  None: ``x`` is the
        whole sequence and the pair partner is roll(x, -1).  ``seq_len``: the
        whole sequence's length when ``x`` is a shard (it selects the precision
        under "auto")."""
        B, L, D = x.shape
        if x_next is None:
            partner = torch.roll(x, shifts=-1, dims=1)
        else:
            partner = torch.cat([x[:, 1:], x_next.to(x.dtype)], dim=1)
        if self.link_mode == "additive":
            # a_t = gq(x_t) + gk(x_{t+1}) (core/attention.py:98-101), summed in fp32
            a = self.gqproj(x).float() + self.gkproj(partner).float()
            return a.contiguous(), None, "packed"
        pair = torch.cat([x, partner], dim=-1)
        lin0 = self.edge_mlp[0]
        layout = self._gen_layout()
        if x.dtype == torch.float32:
            if layout == "packed":
                return self.edge_mlp(pair), None, layout
            w2, b2 = self._w2f32()
            return F.linear(self.edge_mlp[1](lin0(pair)), w2, b2), None, layout
        if x.dtype != torch.bfloat16:
            raise NotImplementedError(f"dtype {x.dtype} is not supported (float32 or bfloat16)")
        mode = self._generator_mode(seq_len if seq_len is not None else
                                    (L if x_next is None else None))
        p2 = pair.reshape(B * L, 2 * D)
        w1t, b1 = self._w1t()
        h = ops.edge_gemm(p2, w1t, b1)            # fp32 out, the bias added in the epilogue
        if mode == "split8" and not self._fp8_shape_ok(B * L, h.shape[1]):
            mode = "split"                        # shapes the fp8 GEMM does not take
        if mode == "split8":
            # W2 g_hi in bf16 (the bias in the epilogue), then += W2 g_lo with both operands in
            # e4m3 (hoa_edge_gelu_split8, hoa_edge_gemm_fp8_acc)
            hi, lo = ops.edge_gelu_split8(h)
            del h
            wt, bias = self._stacked_w2t(False)
            a = ops.edge_gemm(hi, wt, bias)
            del hi
            w8, alpha = self._w2_fp8()
            ops.edge_gemm_fp8_acc(lo, w8, a, alpha)
            return a.view(B, L, -1), None, layout
        split = mode != "bf16"
        # GEMM operand [g_hi | g_lo] ("bf16": g_hi), g = GELU(h), in one pass (hoa_edge_gelu_split),
        # against [W2^T ; W2^T] (W2^T): W2 g_hi + W2 g_lo in fp32, the bias added in the GEMM's
        # epilogue (hoa_edge_gemm, cuBLASLt)
        lhs = ops.edge_gelu_split(h, split)
        del h
        wt, bias = self._stacked_w2t(split)
        a = ops.edge_gemm(lhs, wt, bias)
        return a.view(B, L, -1), None, layout

    # sequences longer than this use the split generators under "auto"
    AUTO_SPLIT_ABOVE = 8192

    def _generator_mode(self, L: Optional[int]) -> str:
        """The bf16 edge MLP's form for a sequence of L positions: "bf16", "split" or "split8"
        (None: a shard of a longer sequence, always a split form under "auto")."""
        p = self.generator_precision
        if p not in ("auto", "split", "split8", "bf16"):
            raise ValueError("generator_precision must be 'auto', 'split', 'split8' or 'bf16'")
        if p == "auto":
            return self.AUTO_LONG if (L is None or L > self.AUTO_SPLIT_ABOVE) else "bf16"
        return p

    # the split form "auto" uses beyond AUTO_SPLIT_ABOVE (same accuracy as "split", measured
    # at T = 65536, with the low half's GEMM in fp8)
    AUTO_LONG = "split8"

    def _fp8_shape_ok(self, M: int, K: int) -> bool:
        """Whether the fp8 GEMM of "split8" takes M rows x K hidden x the generator width
        (multiples of 16); otherwise "split" runs."""
        N = self.h * ops.gen_stride(self.d, self._gen_layout())
        return M % 16 == 0 and K % 16 == 0 and N % 16 == 0

    def _split_generators(self, L: Optional[int]) -> bool:
        """Whether the bf16 edge MLP runs a split form (the hidden layer's low half kept) for a
        sequence of L positions (None: a shard of a longer sequence)."""
        return self._generator_mode(L) != "bf16"

    def _w2_fp8(self):
        """(W2 in e4m3 (rows in the generator layout) times a power-of-two scale s, and
        alpha = 1 / (s * ops.SPLIT8_LO_SCALE)), cached until edge_mlp.2 changes."""
        w = self.edge_mlp[2].weight
        key = (w.data_ptr(), w._version, w.dtype, str(w.device))
        if getattr(self, "_w2fp8_key", None) != key:
            wr, _ = self._w2_rows(w.detach(), self.edge_mlp[2].bias.detach())
            wf = wr.float()
            amax = float(wf.abs().max())
            s = 2.0 ** math.floor(math.log2(448.0 / amax)) if amax > 0 else 1.0
            self._w2fp8 = ((wf * s).to(torch.float8_e4m3fn).contiguous(), 1.0 / (s * ops.SPLIT8_LO_SCALE))
            self._w2fp8_key = key
        return self._w2fp8

    def _stacked_w2t(self, split: bool = True):
        """([W2^T ; W2^T] (8D x m*H; W2^T alone for split=False) in bf16, the output bias in
        fp32), cached until edge_mlp.2 changes."""
        lin2 = self.edge_mlp[2]
        w, b = lin2.weight, lin2.bias
        key = (w.data_ptr(), w._version, b.data_ptr(), b._version, w.dtype, str(w.device), split)
        if getattr(self, "_w2cat_key", None) != key:
            wr, br = self._w2_rows(w.detach(), b.detach())
            wt = wr.t().to(torch.bfloat16)
            self._w2cat = (torch.cat([wt, wt], dim=0) if split else wt).contiguous()
            self._b2f = br.float().contiguous()
            self._w2cat_key = key
        return self._w2cat, self._b2f

    def _w1t(self):
        """(W1^T (2D x 4D) in bf16, b1 in fp32) of the edge MLP's first layer, cached until
        edge_mlp.0 changes."""
        lin0 = self.edge_mlp[0]
        w, b = lin0.weight, lin0.bias
        key = (w.data_ptr(), w._version, b.data_ptr(), b._version, w.dtype, str(w.device))
        if getattr(self, "_w1t_key", None) != key:
            self._w1t_cache = (w.detach().t().to(torch.bfloat16).contiguous(), b.detach().float().contiguous())
            self._w1t_key = key
        return self._w1t_cache

    def _w2f32(self):
        """(W2, b2) in fp32 with rows in the banked layout, cached until edge_mlp.2 changes."""
        lin2 = self.edge_mlp[2]
        w, b = lin2.weight, lin2.bias
        key = (w.data_ptr(), w._version, b.data_ptr(), b._version, str(w.device))
        if getattr(self, "_w2f_key", None) != key:
            wr, br = self._w2_rows(w.detach().float(), b.detach().float())
            self._w2f = (wr.contiguous(), br.contiguous())
            self._w2f_key = key
        return self._w2f

    # Batch rows are independent: the forward runs over pieces of about this many
    # tokens (whole rows).  The edge-MLP GEMM and the link kernel then alternate in
    # shorter bursts (measured at configs[2]: 4 pieces of 4 rows are ~5% faster
    # than one pass, the GPU spending less time at power-capped clocks), and the
    # per-piece generators and path products take a quarter of the memory.
    PIECE_TOKENS = 16384

    def forward(self, x: torch.Tensor, attn_mask: Optional[torch.Tensor] = None,
                return_geometry: bool = False):
        self._check_supported(x, attn_mask, return_geometry)
        # an earlier launch on this device whose device-side wait gave up raises here
        # (ops.check_status() waits for the launches still running and raises too)
        ops.poll_status(x.device)
        B, L, D = x.shape
        rows = max(1, self.PIECE_TOKENS // L)
        # the hot path: causal mode under exactly tril(L); everything else (no mask,
        # any other mask, the inert ablation) takes the general fp32 path
        general = not (self.mode == "causal" and self._mask_is_tril(attn_mask, L))
        mask = attn_mask.to(x.device) if (general and attn_mask is not None) else None
        if return_geometry:
            # {"C": P (B,H,L,d,d), "H": Hol (B,H,d,d)} in x's dtype, as
            # core/attention_fast_chunked.py:175-177 returns them
            y = torch.empty(B, L, D, dtype=x.dtype, device=x.device)
            P = torch.empty(B, self.h, L, self.d, self.d, dtype=x.dtype, device=x.device)
            Hol = torch.empty(B, self.h, self.d, self.d, dtype=x.dtype, device=x.device)
            for b0 in range(0, B, rows):
                sl = slice(b0, min(B, b0 + rows))
                y[sl], P[sl], Hol[sl] = self._forward_rows(x[sl], True, general, mask)
            return y, {"C": P, "H": Hol}
        if rows >= B:
            return self._forward_rows(x, False, general, mask), None
        y = torch.empty(B, L, D, dtype=x.dtype, device=x.device)
        for b0 in range(0, B, rows):
            y[b0:b0 + rows] = self._forward_rows(x[b0:b0 + rows], False, general, mask)
        return y, None

    def _forward_rows(self, x: torch.Tensor, geometry: bool = False, general: bool = False,
                      mask: Optional[torch.Tensor] = None):
        qkv = self.qkv(x)
        if not qkv.is_contiguous():
            qkv = qkv.contiguous()
        a_all, a_bias, layout = self._edge_generators_nobias(x)
        if geometry or general:
            B, L, _ = x.shape
            chunk = self.chunk or ops.plan_chunk(B, self.h, L, self.d, x.device)
        if general:
            r = ops.core_general(a_all, qkv, self.h, self.edge_scale, self.scale, x.dtype, chunk,
                                 self.mode, mask, a_bias, layout, geometry)
            if geometry:
                heads, P, Hol = r
                return self.out(heads), P, Hol
            return self.out(r)
        if geometry:
            heads, P, Hol = ops.core_geometry(a_all, qkv, self.h, self.edge_scale, self.scale,
                                              x.dtype, x.dtype, chunk, a_bias, layout)
            return self.out(heads), P, Hol
        heads = ops.core_forward(a_all, qkv, self.h, self.edge_scale, self.scale,
                                 out_dtype=x.dtype, hat_dtype=x.dtype, chunk=self.chunk,
                                 a_bias=a_bias, gen_layout=layout)
        return self.out(heads)
