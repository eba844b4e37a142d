"""GPU parity of the sm_100a path against the oracle and the reference's golden vectors.

Bars (from the task): rel-L2 <= 1e-5 for fp32 inputs, <= 2e-2 for bf16 inputs,
against the reference PyTorch path on identical seeded inputs and weights.
Everything here calls the CUDA library through the C ABI (ops / module).
"""
import math
import os

import numpy as np
import pytest
import torch

from holonomyawareattention_b200 import PathOrderedGeometricMHA, ops
from oracle import holonomy_oracle as O
from oracle import torch_ref
from oracle.seeded import params_of, seeded_case

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
FP32_TOL = 1e-5
BF16_TOL = 2e-2
DEV = "cuda"


def load(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


def fixture_module(z, dtype=torch.float32):
    D, H, seed, B, L = (int(z[k]) for k in ("D", "H", "seed", "B", "L"))
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=float(z["edge_scale"]))
    if "w:qkv.weight" in z.files:
        m.load_state_dict({k[2:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("w:")})
    else:
        sd, _ = seeded_case(D, H, seed, B, L, bool(int(z["bf16_round"])))
        m.load_state_dict(sd)
    return m.to(device=DEV, dtype=dtype).eval()


def tril(L):
    return torch.tril(torch.ones(L, L, dtype=torch.bool, device=DEV))


def run(m, x):
    with torch.no_grad():
        y, geom = m(x, attn_mask=tril(x.shape[1]))
    assert geom is None
    return y.float().cpu().numpy()


@pytest.mark.parametrize("name", ["tiny_es01", "tiny_es15", "d48_L40", "d96_L32", "d120_L24", "c1"])
def test_golden_fp32(name):
    z = load(name)
    m = fixture_module(z)
    y = run(m, torch.from_numpy(z["x"]).to(DEV))
    assert O.rel_l2(y, z["y_chunked_f64"]) <= FP32_TOL
    assert O.rel_l2(y, z["y_chunked_f32"]) <= FP32_TOL
    if "y_orig_f32" in z.files:     # core/attention.py, the O(L^3) original
        assert O.rel_l2(y, z["y_orig_f32"]) <= FP32_TOL


def test_golden_bf16():
    z = load("bf16_d48_L64")
    m = fixture_module(z, torch.bfloat16)
    y = run(m, torch.from_numpy(z["x"]).to(DEV, torch.bfloat16))
    assert O.rel_l2(y, z["y_chunked_f64"]) <= BF16_TOL


@pytest.mark.parametrize("chunk", [1, 5, 16, 40])
def test_chunking_invariance(chunk):
    z = load("d48_L40")
    m = fixture_module(z)
    x = torch.from_numpy(z["x"]).to(DEV)
    m.chunk = None
    y0 = run(m, x)
    m.chunk = chunk
    y1 = run(m, x)
    assert O.rel_l2(y1, y0) < 2e-6
    assert O.rel_l2(y1, z["y_chunked_f64"]) <= FP32_TOL


@pytest.mark.parametrize("d", [8, 16, 32, 48, 64, 96, 120])
@pytest.mark.parametrize("L", [1, 2, 17, 65])
def test_lengths_and_head_dims(d, L):
    H = 3                                   # odd B*H
    D = d * H
    sd, x = seeded_case(D, H, seed=100 + d + L, B=1, L=L)
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=0.3)
    m.load_state_dict(sd)
    m = m.to(DEV).eval()
    y = run(m, x.to(DEV))
    ref = O.forward(params_of(sd), x.numpy().astype(np.float64), H, 0.3, np.float64)
    assert np.isfinite(y).all()
    assert O.rel_l2(y, ref) <= FP32_TOL


def test_link_stage_geometry_vs_oracle():
    """P_t = R_t C_k and the holonomy against the float64 oracle (kernels 1+2)."""
    z = load("tiny_es15")
    sd = {k[2:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("w:")}
    H, es = int(z["H"]), float(z["edge_scale"])
    x = torch.from_numpy(z["x"])
    p = params_of(sd)
    a_unscaled = O.edge_generators(p, x.numpy().astype(np.float64), H, 1.0)   # (B,H,L,m)
    B, _, L, mm = a_unscaled.shape
    d = x.shape[-1] // H
    a_dev = torch.from_numpy(a_unscaled.transpose(0, 2, 1, 3).reshape(B, L, H * mm)).float().to(DEV)
    qkv = torch.from_numpy((x.numpy().astype(np.float64) @ p.qkv.T)).float().to(DEV).contiguous()
    for chunk in (1, 4, L):
        R, U, M = ops.link_local(a_dev, qkv, H, es, chunk)
        C, total = ops.carry_scan(M, want_total=True)
        k_of_t = torch.arange(L, device=DEV) // chunk
        P = torch.einsum("ntij,ntjk->ntik", R, C[:, k_of_t]).view(B, H, L, d, d).cpu().numpy()
        assert O.rel_l2(P, z["P_f64"]) < 2e-6
        assert O.rel_l2(total.view(B, H, d, d).cpu().numpy(), z["Hol_f64"]) < 2e-6
        I = np.eye(d)
        assert np.abs(np.swapaxes(P, -1, -2) @ P - I).max() < 1e-5


def run_geometry(m, x):
    with torch.no_grad():
        y, geom = m(x, attn_mask=tril(x.shape[1]), return_geometry=True)
    return y, geom


@pytest.mark.parametrize("name", ["tiny_es01", "tiny_es15"])
def test_return_geometry_vs_golden(name):
    """forward(..., return_geometry=True): {"C": P, "H": Hol} against the reference's own
    float64 geometry (core/attention_fast_chunked.py:175-177); y unchanged bit for bit."""
    z = load(name)
    m = fixture_module(z)
    x = torch.from_numpy(z["x"]).to(DEV)
    B, L, _ = x.shape
    y, g = run_geometry(m, x)
    assert set(g) == {"C", "H"}
    assert g["C"].shape == (B, m.h, L, m.d, m.d) and g["H"].shape == (B, m.h, m.d, m.d)
    assert g["C"].dtype == torch.float32 and g["H"].dtype == torch.float32
    assert np.array_equal(y.cpu().numpy(), run(m, x))
    assert O.rel_l2(g["C"].cpu().numpy(), z["P_f64"]) < 2e-6
    assert O.rel_l2(g["H"].cpu().numpy(), z["Hol_f64"]) < 2e-6


@pytest.mark.parametrize("name", ["c1", "d48_L40", "d96_L32", "d120_L24"])
def test_return_geometry_samples(name):
    """P at the fixture's sampled positions (batch row 0, every head) against the reference's
    float64 P, at d = 48 (tensor-core link), 96 (banked generators) and 120 (SIMT link)."""
    z = load(name)
    m = fixture_module(z)
    x = torch.from_numpy(z["x"]).to(DEV)
    y, g = run_geometry(m, x)
    ts = [int(t) for t in z["P_sample_t"]]
    P = g["C"][0][:, ts].transpose(0, 1).cpu().numpy()
    assert O.rel_l2(P, z["P_sample_b0"]) < FP32_TOL
    assert np.array_equal(y.cpu().numpy(), run(m, x))
    Pf = g["C"].double()
    eye = torch.eye(m.d, dtype=torch.float64, device=DEV)
    assert (Pf.transpose(-1, -2) @ Pf - eye).abs().max().item() < 1e-5


def test_return_geometry_bf16_in_pieces():
    """bf16 module, forward split into one-row batch pieces: P and Hol come back in bf16,
    y equals the forward without geometry, P matches the float64 samples within the bf16 bar."""
    z = load("bf16_d48_L64")
    m = fixture_module(z, torch.bfloat16)
    m.PIECE_TOKENS = int(z["L"])                       # one batch row per piece
    x = torch.from_numpy(z["x"]).to(DEV, torch.bfloat16)
    y, g = run_geometry(m, x)
    assert g["C"].dtype == torch.bfloat16 and g["H"].dtype == torch.bfloat16
    ts = [int(t) for t in z["P_sample_t"]]
    P = g["C"][0][:, ts].transpose(0, 1).float().cpu().numpy()
    assert O.rel_l2(P, z["P_sample_b0"]) < BF16_TOL
    with torch.no_grad():
        y0, _ = m(x, attn_mask=tril(x.shape[1]))
    assert torch.equal(y, y0)


@pytest.mark.parametrize("d,T,chunk", [(8, 37, 16), (48, 100, 32), (96, 33, 16), (120, 20, 8)])
@pytest.mark.parametrize("p_dtype", [torch.float32, torch.bfloat16])
def test_compose_paths_kernel(d, T, chunk, p_dtype):
    """hoa_compose_paths: P_t = R_t C_{t/chunk} against a float64 product, ragged last chunk."""
    torch.manual_seed(d + T)
    BH = 3
    K = (T + chunk - 1) // chunk
    R = torch.randn(BH, T, d, d, device=DEV)
    C = torch.randn(BH, K, d, d, device=DEV)
    P = ops.compose_paths(R, C, chunk, p_dtype)
    kidx = torch.arange(T, device=DEV) // chunk
    ref = torch.einsum("ntij,ntjk->ntik", R.double(), C[:, kidx].double())
    tol = 1e-6 if p_dtype == torch.float32 else 5e-3
    assert O.rel_l2(P.double().cpu().numpy(), ref.cpu().numpy()) < tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_config2_full_size(dtype):
    """B=64, T=512, d_model=192, H=4 against the torch restatement (fp32)."""
    B, T, D, H, es = 64, 512, 192, 4, 0.05
    sd, x = seeded_case(D, H, seed=0, B=B, L=T, bf16_round=dtype == torch.bfloat16)
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=es)
    m.load_state_dict(sd)
    m = m.to(DEV, dtype).eval()
    y = run(m, x.to(DEV, dtype))
    ref = torch_ref.module_forward(sd, x.to(DEV), H, es, torch.float32, batch_slice=16).cpu().numpy()
    assert O.rel_l2(y, ref) <= (FP32_TOL if dtype == torch.float32 else BF16_TOL)


@pytest.mark.parametrize("precision", ["auto", "split", "split8"])
def test_config3_slice_bf16(precision):
    """configs[2] shape (T=4096, d_model=1536, H=16, bf16) on two batch rows vs fp32 torch
    restatement, with the default generator precision (bf16 at this length) and the split ones."""
    B, T, D, H, es = 2, 4096, 1536, 16, 0.05
    sd, x = seeded_case(D, H, seed=0, B=B, L=T, bf16_round=True)
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=es)
    m.load_state_dict(sd)
    m = m.to(DEV, torch.bfloat16).eval()
    m.generator_precision = precision
    y = run(m, x.to(DEV, torch.bfloat16))
    ref = torch_ref.module_forward(sd, x.to(DEV), H, es, torch.float32, batch_slice=1).cpu().numpy()
    err = O.rel_l2(y, ref)
    print(f"c3 slice bf16 ({precision}) rel-L2 {err:.3e}")
    assert err <= BF16_TOL


def rel_l2_whole_and_last_quarter(y, ref):
    """rel-L2 over the whole sequence and over its last quarter, where the drift of the
    long rotation products would show first."""
    T = y.shape[1]
    return O.rel_l2(y, ref), O.rel_l2(y[:, 3 * T // 4:], ref[:, 3 * T // 4:])


def test_config3_full_batch_bf16():
    """configs[2] at full size: all 16 batch rows (the module's forward runs them in 4 batch
    pieces of 16K tokens) against the fp32 torch restatement on bf16-rounded inputs and weights."""
    B, T, D, H, es = 16, 4096, 1536, 16, 0.05
    sd, x = seeded_case(D, H, seed=0, B=B, L=T, bf16_round=True)
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=es)
    m.load_state_dict(sd)
    m = m.to(DEV, torch.bfloat16).eval()
    assert B * T > m.PIECE_TOKENS                      # the batch-piece loop is exercised
    y = run(m, x.to(DEV, torch.bfloat16))
    del m
    torch.cuda.empty_cache()
    ref = torch_ref.module_forward(sd, x.to(DEV), H, es, torch.float32, batch_slice=1).cpu().numpy()
    err, err_q = rel_l2_whole_and_last_quarter(y, ref)
    print(f"configs[2] full batch bf16: rel-L2 {err:.3e}, last quarter {err_q:.3e}")
    assert err <= BF16_TOL and err_q <= BF16_TOL


@pytest.mark.parametrize("precision", ["auto", "split"])
def test_config5_long_sequence_bf16(precision):
    """one sequence of T = 65536 (d_model 1536, H 16, head_dim 96, bf16) on one GPU
    against the fp32 torch restatement (core/attention_fast_chunked.py:89-94: the sequential
    product over 65535 edges, the drift stress of this config), run two heads at a time to
    bound its memory.  "auto" selects a split form of the generators at this length."""
    B, T, D, H, es = 1, 65536, 1536, 16, 0.05
    sd, x = seeded_case(D, H, seed=0, B=B, L=T, bf16_round=True)
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=es)
    m.load_state_dict(sd)
    m = m.to(DEV, torch.bfloat16).eval()
    m.generator_precision = precision
    assert m._split_generators(T)
    y = run(m, x.to(DEV, torch.bfloat16))
    del m
    torch.cuda.empty_cache()
    ref = torch_ref.module_forward(sd, x.to(DEV), H, es, torch.float32, batch_slice=1,
                                   head_group=2).cpu().numpy()
    err, err_q = rel_l2_whole_and_last_quarter(y, ref)
    print(f"configs[4] T=65536 bf16 ({precision}): rel-L2 {err:.3e}, last quarter {err_q:.3e}")
    assert err <= BF16_TOL and err_q <= BF16_TOL


def test_config4_slice_bf16():
    """configs[3] shape (T=2048, d_model=2880, H=24, head_dim 120, bf16) on one batch row vs the
    fp32 torch restatement (head_dim 120 runs the FFMA link kernel)."""
    B, T, D, H, es = 1, 2048, 2880, 24, 0.05
    sd, x = seeded_case(D, H, seed=0, B=B, L=T, bf16_round=True)
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=es)
    m.load_state_dict(sd)
    m = m.to(DEV, torch.bfloat16).eval()
    y = run(m, x.to(DEV, torch.bfloat16))
    ref = torch_ref.module_forward(sd, x.to(DEV), H, es, torch.float32, batch_slice=1).cpu().numpy()
    err = O.rel_l2(y, ref)
    print(f"c4 slice bf16 rel-L2 {err:.3e}")
    assert err <= BF16_TOL


def test_deterministic_and_rejects():
    z = load("d96_L32")
    m = fixture_module(z)
    x = torch.from_numpy(z["x"]).to(DEV)
    assert np.array_equal(run(m, x), run(m, x))
    L = x.shape[1]
    with torch.no_grad():
        # other masks (and none) take the general path: they run and change the result
        y_t = run(m, x)
        other = tril(L).clone()
        other[5, 0] = False
        y_o, _ = m(x, attn_mask=other)
        y_n, _ = m(x, attn_mask=None)
        assert np.isfinite(y_o.cpu().numpy()).all() and np.isfinite(y_n.cpu().numpy()).all()
        assert not np.array_equal(y_o.cpu().numpy(), y_t)
        assert not np.array_equal(y_n.cpu().numpy(), y_t)
        with pytest.raises(NotImplementedError):
            m(x, attn_mask=tril(L).float())


@pytest.mark.parametrize("precision,tol", [("split", 3e-5), ("bf16", 6e-3)])
def test_edge_generators_bf16_precision(precision, tol):
    """bf16 module: generators (edge MLP output) against the fp32 MLP on the same bf16 values."""
    B, T, D, H = 2, 64, 192, 4
    sd, x = seeded_case(D, H, seed=7, B=B, L=T, bf16_round=True)
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=0.05)
    m.load_state_dict(sd)
    m = m.to(DEV, torch.bfloat16).eval()
    m.generator_precision = precision
    with torch.no_grad():
        a = m.edge_generators(x.to(DEV, torch.bfloat16)).float().cpu().numpy()
    p = params_of(sd, np.float64)
    ref = O.edge_generators(p, x.numpy().astype(np.float64), H, 1.0)        # (B,H,T,m)
    ref = ref.transpose(0, 2, 1, 3).reshape(B, T, -1)
    assert O.rel_l2(a, ref) < tol
