"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures in tests/golden were written by tests/golden/make_golden.py, which
ran the reference's core/attention.py (the O(L^3) original) and
core/attention_fast_chunked.py (the chunked drop-in) on seeded inputs.
"""
import os

import numpy as np
import pytest
import torch

from oracle import holonomy_oracle as O
from oracle.seeded import checksums, params_of, seeded_case

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


def case_inputs(z):
    """Weights and x of a fixture: stored weights, or regenerated from the seed."""
    D, H, seed, B, L = (int(z[k]) for k in ("D", "H", "seed", "B", "L"))
    if "w:qkv.weight" in z.files:
        sd = {k[2:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("w:")}
    else:
        sd, _ = seeded_case(D, H, seed, B, L, bool(int(z["bf16_round"])))
        cs = checksums(sd)
        for k, v in cs.items():
            np.testing.assert_allclose(v, z["cs:" + k], rtol=1e-9, atol=1e-12,
                                       err_msg=f"seeded weights differ from fixture: {k}")
    return sd, z["x"], H, float(z["edge_scale"])


def test_skew_from_vec_order():
    d = 5
    v = np.arange(1, d * (d - 1) // 2 + 1, dtype=np.float64)
    A = O.skew_from_vec(v, d)
    idx = 0
    for i in range(d):
        for j in range(i + 1, d):
            assert A[i, j] == v[idx] and A[j, i] == -v[idx]
            idx += 1
    assert np.all(np.diag(A) == 0)
    with pytest.raises(ValueError):
        O.skew_from_vec(np.zeros(7), 5)


@pytest.mark.parametrize("d", [8, 48, 96, 120])
@pytest.mark.parametrize("nrm", [0.2, 1.0, 7.0])
def test_expm_vs_torch_matrix_exp_golden(d, nrm):
    z = load("expm")
    seed = {8: 10, 48: 11, 96: 12, 120: 13}[d]
    rng = np.random.default_rng(seed)
    M = rng.standard_normal((d, d))
    S = M - M.T
    S /= np.linalg.norm(S, 2)
    A = (S * nrm).astype(np.float32)
    G_ref = z[f"G32_d{d}_n{nrm}"]
    G64 = O.expm(A.astype(np.float64))
    G32 = O.expm(A)
    # torch's fp32 result vs exact: a few ulp, growing with the squarings at large norm
    tol = 5e-7 * (1.0 + nrm)
    assert O.rel_l2(G64, G_ref) < tol
    assert O.rel_l2(G32, G_ref) < 2 * tol
    assert np.abs(G64.T @ G64 - np.eye(d)).max() < 1e-12


@pytest.mark.parametrize("name", ["tiny_es01", "tiny_es15"])
def test_oracle_tiny_full_geometry(name):
    z = load(name)
    sd, x, H, es = case_inputs(z)
    p = params_of(sd)
    y64, inter = O.forward(p, x.astype(np.float64), H, es, np.float64, return_intermediates=True)
    assert O.rel_l2(y64, z["y_chunked_f64"]) < 1e-11
    assert O.rel_l2(inter["P"], z["P_f64"]) < 1e-11
    assert O.rel_l2(inter["Hol"], z["Hol_f64"]) < 1e-11
    # the O(L^3) original agrees under the tril mask (fp32 run of core/attention.py)
    assert O.rel_l2(y64, z["y_orig_f32"]) < 1e-5
    y32 = O.forward(p, x, H, es, np.float32)
    assert O.rel_l2(y32, z["y_chunked_f32"]) < 1e-5


@pytest.mark.parametrize("name", ["d48_L40", "d96_L32", "d120_L24", "bf16_d48_L64", "c1"])
def test_oracle_vs_reference_golden(name):
    z = load(name)
    sd, x, H, es = case_inputs(z)
    p = params_of(sd)
    y64, inter = O.forward(p, x.astype(np.float64), H, es, np.float64, return_intermediates=True)
    assert O.rel_l2(y64, z["y_chunked_f64"]) < 1e-10
    ts = list(z["P_sample_t"])
    assert O.rel_l2(inter["P"][0][:, ts].transpose(1, 0, 2, 3), z["P_sample_b0"]) < 1e-6
    assert O.rel_l2(y64, z["y_chunked_f32"]) < 1e-5
    if "y_orig_f32" in z.files:
        assert O.rel_l2(y64, z["y_orig_f32"]) < 1e-5


def test_core_forward_matches_module_forward():
    z = load("tiny_es01")
    sd, x, H, es = case_inputs(z)
    p = params_of(sd)
    x = x.astype(np.float64)
    _, inter = O.forward(p, x, H, es, np.float64, return_intermediates=True)
    a_unscaled = O.edge_generators(p, x, H, 1.0)
    heads = O.core_forward(a_unscaled, inter["q"], inter["k"], inter["v"],
                           1.0 / np.sqrt(x.shape[-1] // H), es)
    assert O.rel_l2(heads, inter["heads"]) < 1e-12


def test_round_bf16():
    v = np.array([1.0, 1.00390625, 1.001953125, 3.14159, -2.5e-3], dtype=np.float32)
    r = O.round_bf16(v)
    t = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(r, t)


GENERAL = ["gen_none_es15", "gen_rand_es15", "gen_band_d48", "gen_inert_rand", "gen_additive_none"]


def general_case(name):
    """(params, x, mask, fixture) of a core/attention.py case (masks, wrap, inert, additive)."""
    z = np.load(os.path.join(GOLD, name + ".npz"))
    D, H, seed, B, L = (int(z[k]) for k in ("D", "H", "seed", "B", "L"))
    if "w:qkv.weight" in z.files:
        sd = {k[2:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("w:")}
    else:
        sd, _ = seeded_case(D, H, seed, B, L)
        cs = checksums(sd)
        for k in cs:
            assert np.allclose(cs[k], z["cs:" + k]), k
    mask = z["mask"] if "mask" in z.files else None
    return params_of(sd), z["x"], mask, z


@pytest.mark.parametrize("name", GENERAL)
def test_forward_general_vs_original(name):
    """forward_general against core/attention.py itself (the O(L^3) arc walk) in float64:
    any mask, wrap pairs through the closing edge, the inert ablation, the additive link."""
    p, x, mask, z = general_case(name)
    y, inter = O.forward_general(p, x, int(z["H"]), float(z["edge_scale"]), mask, str(z["mode"]),
                                 str(z["link_mode"]), np.float64, return_intermediates=True)
    assert O.rel_l2(y, z["y_orig_f64"]) < 1e-12
    assert O.rel_l2(inter["P"], z["P_f64"]) < 1e-12
    assert O.rel_l2(inter["Hol"], z["Hol_f64"]) < 1e-12
    y32 = O.forward_general(p, x, int(z["H"]), float(z["edge_scale"]), mask, str(z["mode"]),
                            str(z["link_mode"]), np.float32)
    assert O.rel_l2(y32, z["y_orig_f64"]) < 1e-5


def test_wrap_pairs_need_hol_not_its_transpose():
    """With the wrap pairs live (no mask), transporting them by Hol^T (as the chunked
    module's dead branch does) is far from core/attention.py: the fixtures tell the two apart."""
    p, x, mask, z = general_case("gen_none_es15")
    H, es = int(z["H"]), float(z["edge_scale"])
    _, inter = O.forward_general(p, x, H, es, mask, "causal", "interaction", np.float64,
                                 return_intermediates=True)
    P, Hol = inter["P"], inter["Hol"]
    q, k, v = O.project_qkv(p, x, H)
    PT = np.swapaxes(P, -1, -2)
    qh, kh, vh = ((PT @ t[..., None])[..., 0] for t in (q, k, v))
    HolT = np.swapaxes(Hol, -1, -2)[:, :, None]
    o = O.masked_attention(qh, kh, vh, 1 / np.sqrt(x.shape[-1] // H), None,
                           (HolT @ kh[..., None])[..., 0], (HolT @ vh[..., None])[..., 0])
    heads = (P @ o[..., None])[..., 0]
    y_t = heads.transpose(0, 2, 1, 3).reshape(x.shape) @ p.out.T
    assert O.rel_l2(y_t, z["y_orig_f64"]) > 0.05
