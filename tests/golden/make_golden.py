"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Run once, in a container where the reference checkout is present:

    python tests/golden/make_golden.py --ref /path/to/HolonomyAwareAttention

It imports the reference's ``core/attention.py`` (the O(L^3) original),
``core/attention_fast_chunked.py`` (the chunked drop-in) and ``core/utils.py``
and records their outputs on seeded inputs.  Nothing at test time reads the
reference; the tests read only the ``.npz`` files written here.

Seeding follows the reference's own harness (kernel/eval_checkpoint_kernel.py:58-70):
``torch.manual_seed(seed)``, build the module with default init, then draw
``x = torch.randn(B, L, D)``.  Large weight sets are not stored: they are
regenerated at test time from the seed by constructing a module with the
same parameter creation order, and checked against the checksums stored here.
"""
from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def checksums(sd):
    out = {}
    for k, t in sd.items():
        a = t.detach().double().cpu().numpy().ravel()
        out[k] = np.array([a.sum(), (a * a).sum(), *a[:4]], dtype=np.float64)
    return out


def build(ref_mod, D, H, es, seed, B, L, bf16_round=False):
    torch.manual_seed(seed)
    m = ref_mod.PathOrderedGeometricMHA(D, n_heads=H, edge_scale=es, mode="causal").eval()
    x = torch.randn(B, L, D)
    if bf16_round:
        with torch.no_grad():
            for p in m.parameters():
                p.copy_(p.to(torch.bfloat16).float())
        x = x.to(torch.bfloat16).float()
    return m, x


def run(mod, x, dtype):
    L = x.shape[1]
    mask = torch.tril(torch.ones(L, L, dtype=torch.bool))
    m = mod.to(dtype)
    with torch.no_grad():
        y, _ = m(x.to(dtype), attn_mask=mask)
    m.float()
    return y.numpy()


def geometry(mod, x, dtype):
    m = mod.to(dtype)
    with torch.no_grad():
        q, k, v, P, Hol = m._geometry(x.to(dtype))
    m.float()
    return P.numpy(), Hol.numpy()


def case(name, core, chunk, D, H, es, seed, B, L, *, store_weights, use_orig, bf16_round=False,
         P_samples=None):
    t0 = time.time()
    m, x = build(chunk, D, H, es, seed, B, L, bf16_round)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    rec = dict(B=B, L=L, D=D, H=H, edge_scale=es, seed=seed, bf16_round=int(bf16_round),
               x=x.numpy().astype(np.float32))
    rec["y_chunked_f32"] = run(m, x, torch.float32).astype(np.float32)
    rec["y_chunked_f64"] = run(m, x, torch.float64)
    if use_orig:
        o = core.PathOrderedGeometricMHA(D, n_heads=H, edge_scale=es, mode="causal").eval()
        o.load_state_dict(sd)
        rec["y_orig_f32"] = run(o, x, torch.float32).astype(np.float32)
    P64, Hol64 = geometry(m, x, torch.float64)
    if P_samples is None:
        rec["P_f64"] = P64
        rec["Hol_f64"] = Hol64
    else:
        rec["P_sample_t"] = np.array(P_samples)
        rec["P_sample_b0"] = P64[0, :, P_samples].astype(np.float32)
    cs = checksums(sd)
    for k, v in cs.items():
        rec["cs:" + k] = v
    if store_weights:
        for k, v in sd.items():
            rec["w:" + k] = v.numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
    print(f"{name}: {time.time() - t0:.1f}s", flush=True)


def make_mask(kind, L, seed):
    """(L, L) bool, True = allowed: None (no mask), a seeded random mask with the
    diagonal allowed, or a band |i - j| <= L // 4 (both wrap pairs and blocked pairs)."""
    if kind == "none":
        return None
    if kind == "random":
        g = torch.Generator().manual_seed(seed + 100)
        m = torch.rand(L, L, generator=g) < 0.6
        return m | torch.eye(L, dtype=torch.bool)
    if kind == "band":
        i = torch.arange(L)
        return (i.view(L, 1) - i.view(1, L)).abs() <= L // 4
    raise ValueError(kind)


def general_case(name, core, D, H, es, seed, B, L, mask_kind, mode, link_mode):
    """core/attention.py (the O(L^3) original: arc transport through the closing
    edge, any mask, the inert ablation, the additive link) on seeded inputs."""
    t0 = time.time()
    torch.manual_seed(seed)
    m = core.PathOrderedGeometricMHA(D, n_heads=H, edge_scale=es, mode=mode).eval()
    m.link_mode = link_mode
    x = torch.randn(B, L, D)
    mask = make_mask(mask_kind, L, seed)
    rec = dict(B=B, L=L, D=D, H=H, edge_scale=es, seed=seed, mode=mode, link_mode=link_mode,
               mask_kind=mask_kind, x=x.numpy())
    if mask is not None:
        rec["mask"] = mask.numpy()
    for dt, tag in ((torch.float32, "f32"), (torch.float64, "f64")):
        mm = m.to(dt)
        with torch.no_grad():
            y, g = mm(x.to(dt), attn_mask=mask, return_geometry=True)
        rec["y_orig_" + tag] = y.numpy()
        if dt == torch.float64:
            rec["Hol_f64"] = g["H"].numpy()
            rec["P_f64"] = g["C"].numpy()
    m.float()
    sd = m.state_dict()
    if D <= 32:
        for k, v in sd.items():
            rec["w:" + k] = v.numpy().astype(np.float32)
    else:                                          # regenerated from the seed at test time
        for k, v in checksums(sd).items():
            rec["cs:" + k] = v
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
    print(f"{name}: {time.time() - t0:.1f}s", flush=True)


def general_cases(core):
    # causal arc transport with the wrap pairs live (no mask, random, band), large rotations
    general_case("gen_none_es15", core, 32, 4, 1.5, 7, 2, 12, "none", "causal", "interaction")
    general_case("gen_rand_es15", core, 32, 4, 1.5, 8, 2, 12, "random", "causal", "interaction")
    general_case("gen_band_d48", core, 96, 2, 0.5, 9, 1, 16, "band", "causal", "interaction")
    # the inert ablation (endpoint transport P_i^T P_j) and the additive link
    general_case("gen_inert_rand", core, 32, 4, 1.5, 10, 2, 12, "random", "inert", "interaction")
    general_case("gen_additive_none", core, 32, 4, 1.5, 11, 2, 12, "none", "causal", "additive")


def expm_case():
    rec = {}
    for d, seed in ((8, 10), (48, 11), (96, 12), (120, 13)):
        rng = np.random.default_rng(seed)
        M = rng.standard_normal((d, d))
        S = M - M.T
        S /= np.linalg.norm(S, 2)
        for nrm in (0.2, 1.0, 7.0):
            A = (S * nrm).astype(np.float32)
            G32 = torch.matrix_exp(torch.from_numpy(A)).numpy()
            rec[f"G32_d{d}_n{nrm}"] = G32
    np.savez_compressed(os.path.join(HERE, "expm.npz"), **rec)
    print("expm fixtures written", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference checkout (folder holding core/)")
    ap.add_argument("--skip-c1", action="store_true")
    ap.add_argument("--only-general", action="store_true",
                    help="write only the core/attention.py cases (masks, wrap, inert, additive)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.ref, "core"))
    torch.set_num_threads(os.cpu_count())
    import attention as core                      # core/attention.py
    import attention_fast_chunked as chunk        # core/attention_fast_chunked.py

    general_cases(core)
    if args.only_general:
        return
    expm_case()
    # the reference self-test shape (core/attention_fast_chunked.py:214-236), default edge_scale
    case("tiny_es01", core, chunk, 32, 4, 0.1, 0, 2, 12, store_weights=True, use_orig=True)
    # the kernel self-test's large rotations (kernel/attention_kernel.py:224-240, edge_scale 1.5)
    case("tiny_es15", core, chunk, 32, 4, 1.5, 0, 2, 12, store_weights=True, use_orig=True)
    # head dims of the benchmark configs at short L
    case("d48_L40", core, chunk, 192, 4, 0.05, 5, 2, 40, store_weights=False, use_orig=True,
         P_samples=[0, 1, 20, 39])
    case("d96_L32", core, chunk, 384, 4, 0.05, 1, 1, 32, store_weights=False, use_orig=False,
         P_samples=[0, 1, 31])
    case("d120_L24", core, chunk, 480, 4, 0.05, 2, 1, 24, store_weights=False, use_orig=False,
         P_samples=[0, 1, 23])
    # bf16-valued inputs and weights (the oracle rule for bf16 configs)
    case("bf16_d48_L64", core, chunk, 192, 4, 0.05, 3, 2, 64, store_weights=False, use_orig=False,
         bf16_round=True, P_samples=[0, 63])
    if not args.skip_c1:
        # B=2, T=128, d_model=192, H=4, edge_scale 0.05, via core/attention.py
        case("c1", core, chunk, 192, 4, 0.05, 0, 2, 128, store_weights=False, use_orig=True,
             P_samples=[0, 1, 64, 127])


if __name__ == "__main__":
    main()
