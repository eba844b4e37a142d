"""Stage-level GPU tests: each kernel of the core region against a float64 torch reference.

Kernel (3) has two variants: fp32 SIMT (hoa_attn_fwd) and bf16 tcgen05
(hoa_attn_tc_fwd, v^ transposed); kernel (4) is hoa_out_transport.
"""
import math

import numpy as np
import pytest
import torch

from holonomyawareattention_b200 import ops
from oracle.holonomy_oracle import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


def causal_ref(qh, kh, vh, scale):
    q, k, v = (t.double() for t in (qh, kh, vh))
    T = q.shape[1]
    s = (q @ k.transpose(1, 2)) * scale
    s = s.masked_fill(~torch.tril(torch.ones(T, T, dtype=torch.bool, device=q.device)), float("-inf"))
    return torch.softmax(s, -1) @ v


@pytest.mark.parametrize("T", [1, 70, 150])
@pytest.mark.parametrize("d", [8, 48, 96, 120])
def test_attn_simt_fp32(T, d):
    torch.manual_seed(T + d)
    BH = 3
    qh, kh, vh = (torch.randn(BH, T, d, device=DEV) for _ in range(3))
    o = ops.attn_fwd(qh, kh, vh, 1 / math.sqrt(d))
    assert rel_l2(o.cpu().numpy(), causal_ref(qh, kh, vh, 1 / math.sqrt(d)).cpu().numpy()) < 1e-6


@pytest.mark.parametrize("T", [1, 100, 128, 129, 300])
@pytest.mark.parametrize("d", [16, 48, 64, 96, 120, 128])
def test_attn_tc_bf16(T, d):
    """tcgen05 attention vs float64 softmax on the same bf16 inputs (P is rounded to bf16)."""
    torch.manual_seed(1000 + T + d)
    BH = 3
    qh, kh, vh = (torch.randn(BH, T, d, device=DEV).to(torch.bfloat16) for _ in range(3))
    vt = torch.zeros(BH, d, ops.vt_stride(T), dtype=torch.bfloat16, device=DEV)
    vt[:, :, :T] = vh.transpose(1, 2)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(d)
    o = ops.attn_tc_fwd(qh, kh, vt, scale, status)
    ref = causal_ref(qh, kh, vh, scale)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    err = rel_l2(o.cpu().numpy(), ref.cpu().numpy())
    assert err < 1e-2, err


def test_attn_tc_large_scores():
    """Peaked softmax (large logits) exercises the running-max correction."""
    torch.manual_seed(7)
    BH, T, d = 2, 384, 96
    qh = (4 * torch.randn(BH, T, d, device=DEV)).to(torch.bfloat16)
    kh = (4 * torch.randn(BH, T, d, device=DEV)).to(torch.bfloat16)
    vh = torch.randn(BH, T, d, device=DEV).to(torch.bfloat16)
    vt = torch.zeros(BH, d, ops.vt_stride(T), dtype=torch.bfloat16, device=DEV)
    vt[:, :, :T] = vh.transpose(1, 2)
    o = ops.attn_tc_fwd(qh, kh, vt, 1 / math.sqrt(d))
    ref = causal_ref(qh, kh, vh, 1 / math.sqrt(d))
    assert rel_l2(o.cpu().numpy(), ref.cpu().numpy()) < 1e-2


@pytest.mark.parametrize("d", [6, 8, 48, 96, 120])
def test_out_transport(d):
    torch.manual_seed(d)
    B, H, T, chunk = 2, 3, 50, 16
    K = (T + chunk - 1) // chunk
    o = torch.randn(B * H, T, d, device=DEV)
    R = torch.randn(B * H, T, d, d, device=DEV)
    C = torch.randn(B * H, K, d, d, device=DEV)
    for dt in (torch.float32, torch.bfloat16):
        out = ops.out_transport(o, R, C, chunk, B, H, dt)
        kidx = torch.arange(T, device=DEV) // chunk
        w = torch.einsum("ntef,ntf->nte", C[:, kidx].double(), o.double())
        ref = torch.einsum("ntef,ntf->nte", R.double(), w).view(B, H, T, d).transpose(1, 2).reshape(B, T, H * d)
        tol = 1e-6 if dt == torch.float32 else 1e-2
        assert rel_l2(out.float().cpu().numpy(), ref.cpu().numpy()) < tol


def test_carry_apply_transposed_matches():
    torch.manual_seed(3)
    BH, T, d, chunk = 4, 77, 48, 16
    K = (T + chunk - 1) // chunk
    U = torch.randn(BH, T, 3, d, device=DEV)
    C = torch.randn(BH, K, d, d, device=DEV)
    q1, k1, v1 = ops.carry_apply(U, C, chunk, torch.bfloat16, v_transposed=False)
    q2, k2, vt = ops.carry_apply(U, C, chunk, torch.bfloat16, v_transposed=True)
    assert torch.equal(q1, q2) and torch.equal(k1, k2)
    assert torch.equal(v1, vt[:, :, :T].transpose(1, 2))
    kidx = torch.arange(T, device=DEV) // chunk
    ref = torch.einsum("ntfe,ntf->nte", C[:, kidx].double(), U[:, :, 0].double())
    assert rel_l2(q1.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2
    q3, _, _ = ops.carry_apply(U, C, chunk, torch.float32)
    assert rel_l2(q3.cpu().numpy(), ref.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_stages_equal_core_forward(dtype):
    """The one-call hoa_core_forward equals the stage-by-stage calls."""
    torch.manual_seed(11)
    B, T, H, d = 2, 90, 3, 48
    m = d * (d - 1) // 2
    a = (0.02 * torch.randn(B, T, H * m, device=DEV)).float()
    qkv = torch.randn(B, T, 3 * H * d, device=DEV).to(dtype)
    chunk = 32
    y1 = ops.core_forward(a, qkv, H, 0.5, chunk=chunk)
    y2 = ops.core_stages(a, qkv, H, 0.5, 1 / math.sqrt(d), dtype, dtype, chunk)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("d", [8, 32, 48, 64, 96, 120])
@pytest.mark.parametrize("scale", [0.01, 0.4])
def test_link_local_vs_oracle(d, scale):
    """Kernels (1)+(2): P_t = R_t C_k, the transports and the total against float64.

    scale 0.4 per generator entry makes ||A|| large, so the exponential takes
    the scaling-and-squaring branch (both the SIMT and the tensor-core kernel)."""
    from oracle import holonomy_oracle as O
    torch.manual_seed(d)
    B, H, T, chunk = 1, 2, 19, 8
    m = d * (d - 1) // 2
    a = (scale * torch.randn(B, T, H * m)).float()
    qkv = torch.randn(B, T, 3 * H * d).float()
    R, U, M = ops.link_local(a.to(DEV), qkv.to(DEV), H, 1.0, chunk)
    C, total = ops.carry_scan(M, want_total=True)
    kidx = torch.arange(T, device=DEV) // chunk
    P = torch.einsum("ntij,ntjk->ntik", R.double(), C[:, kidx].double()).cpu().numpy()
    a64 = a.double().numpy().reshape(B, T, H, m).transpose(0, 2, 1, 3)          # (B,H,T,m)
    G = O.expm(O.skew_from_vec(a64, d))                                          # (B,H,T,d,d)
    Pref = O.prefix_products(G[:, :, :-1]).reshape(B * H, T, d, d)
    tol = 1e-5 if scale < 0.1 else 1e-4
    assert O.rel_l2(P, Pref) < tol
    tot_ref = (G[:, :, -1] @ O.prefix_products(G[:, :, :-1])[:, :, -1]).reshape(B * H, d, d)
    assert O.rel_l2(total.cpu().numpy(), tot_ref) < tol
    q = qkv.double().numpy().reshape(B, T, H, 3 * d).transpose(0, 2, 1, 3).reshape(B * H, T, 3 * d)[..., :d]
    qhat = torch.einsum("ntfe,ntf->nte", C[:, kidx].double(), U[:, :, 0].double()).cpu().numpy()
    qref = np.einsum("ntde,ntd->nte", Pref, q)
    assert O.rel_l2(qhat, qref) < tol


def _offset_copy(t):
    """A copy of t whose data starts 4 bytes past a 16-byte boundary (the
    tensor-core link kernel declines it, so the SIMT kernel runs)."""
    buf = torch.empty(t.numel() + 4, dtype=t.dtype, device=t.device)
    v = buf[1:1 + t.numel()].view(t.shape)
    v.copy_(t)
    assert v.data_ptr() % 16 == 4
    return v


@pytest.mark.parametrize("d", [32, 64, 96])
@pytest.mark.parametrize("qdtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("with_bias", [False, True])
@pytest.mark.parametrize("simt", [False, True])
def test_link_banked_equals_packed(d, qdtype, with_bias, simt):
    """The banked generator layout (HOA_GEN_BANKED) gives bit-identical R, U, M
    to the packed one, on the tensor-core and on the SIMT kernel.  Generator
    entries of 0.3 make some positions take the squaring branch."""
    torch.manual_seed(d + 7 * with_bias)
    B, H, T, chunk = 2, 2, 37, 16
    m = d * (d - 1) // 2
    a = 0.3 * torch.randn(B, T, H * m, device=DEV)
    bias = 0.1 * torch.randn(H * m, device=DEV) if with_bias else None
    qkv = torch.randn(B, T, 3 * H * d, device=DEV).to(qdtype)
    ab = ops.gen_to_banked(a, H, d)
    bias_b = ops.gen_to_banked(bias, H, d) if with_bias else None
    if simt:
        a, ab = _offset_copy(a), _offset_copy(ab)
    R1, U1, M1 = ops.link_local(a, qkv, H, 0.7, chunk, bias)
    R2, U2, M2 = ops.link_local(ab, qkv, H, 0.7, chunk, bias_b, gen_layout="banked")
    torch.cuda.synchronize()
    assert torch.equal(R1, R2) and torch.equal(U1, U2) and torch.equal(M1, M2)
    assert torch.isfinite(R1).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_core_forward_banked_equals_packed(dtype):
    torch.manual_seed(5)
    B, T, H, d = 2, 70, 2, 96
    m = d * (d - 1) // 2
    a = 0.02 * torch.randn(B, T, H * m, device=DEV)
    qkv = torch.randn(B, T, 3 * H * d, device=DEV).to(dtype)
    y1 = ops.core_forward(a, qkv, H, 0.5, chunk=32)
    y2 = ops.core_forward(ops.gen_to_banked(a, H, d), qkv, H, 0.5, chunk=32, gen_layout="banked")
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("M,N,K", [(64, 48, 32), (1000, 1128, 768), (130, 77, 24)])
@pytest.mark.parametrize("with_bias", [True, False])
def test_edge_gemm_matches_torch(M, N, K, with_bias):
    """hoa_edge_gemm (cuBLASLt, bias in the epilogue) against an fp64 product of the same bf16 values."""
    torch.manual_seed(M + N + K)
    h = torch.randn(M, K, device=DEV).bfloat16()
    wt = torch.randn(K, N, device=DEV).bfloat16()
    b = torch.randn(N, device=DEV) if with_bias else None
    out = ops.edge_gemm(h, wt, b)
    ref = h.double() @ wt.double() + (b.double() if with_bias else 0.0)
    assert out.dtype == torch.float32 and out.shape == (M, N)
    assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("rows,cols", [(1, 4), (37, 96), (300, 6144)])
@pytest.mark.parametrize("split", [False, True])
def test_edge_gelu_split_matches_torch(rows, cols, split):
    """hoa_edge_gelu_split = F.gelu (exact erf) then the bf16 split, bit for bit."""
    torch.manual_seed(rows + cols)
    h = 3 * torch.randn(rows, cols, device=DEV)
    out = ops.edge_gelu_split(h, split)
    g = torch.nn.functional.gelu(h)
    hi = g.to(torch.bfloat16)
    assert torch.equal(out[:, :cols], hi)
    if split:
        assert out.shape == (rows, 2 * cols)
        assert torch.equal(out[:, cols:], (g - hi.float()).to(torch.bfloat16))
    else:
        assert out.shape == (rows, cols)


@pytest.mark.parametrize("rows,cols", [(1, 4), (37, 96), (300, 6144)])
def test_edge_gelu_split8_matches_torch(rows, cols):
    """hoa_edge_gelu_split8: the high half is bf16(F.gelu(h)) bit for bit; the low half is
    SPLIT8_LO_SCALE * (g - bf16(g)) rounded to e4m3 (within half an e4m3 step: 2^-4 relative,
    or the subnormal spacing 2^-9 absolute)."""
    torch.manual_seed(rows + cols)
    h = 3 * torch.randn(rows, cols, device=DEV)
    hi, lo = ops.edge_gelu_split8(h)
    g = torch.nn.functional.gelu(h)
    ref_hi = g.to(torch.bfloat16)
    assert torch.equal(hi, ref_hi)
    r = (g - ref_hi.float()) * ops.SPLIT8_LO_SCALE
    assert float(r.abs().max()) <= 448.0                       # |h| <= 3 * 6: no saturation here
    err = (lo.float() - r).abs()
    assert bool((err <= r.abs() * 2.0 ** -4 + 2.0 ** -10).all())


@pytest.mark.parametrize("M,N,K", [(64, 48, 32), (1024, 1152, 768)])
def test_edge_gemm_fp8_acc_matches_torch(M, N, K):
    """hoa_edge_gemm_fp8_acc adds alpha * lo @ w^T (e4m3 operands, fp32 accumulation) into out,
    against an fp64 product of the same e4m3 values."""
    torch.manual_seed(M + N + K)
    lo = (4 * torch.randn(M, K, device=DEV)).to(torch.float8_e4m3fn)
    w = (4 * torch.randn(N, K, device=DEV)).to(torch.float8_e4m3fn)
    out0 = torch.randn(M, N, device=DEV)
    out = out0.clone()
    alpha = 2.0 ** -7
    ops.edge_gemm_fp8_acc(lo, w, out, alpha)
    ref = out0.double() + alpha * (lo.double() @ w.double().t())
    assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) < 1e-6
