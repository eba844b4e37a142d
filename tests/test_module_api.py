"""Drop-in API of PathOrderedGeometricMHA (CPU: construction, parameters, gating)."""
import os

import numpy as np
import pytest
import torch

from holonomyawareattention_b200 import PathOrderedGeometricMHA
from oracle.seeded import checksums

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_constructor_errors():
    with pytest.raises(ValueError):
        PathOrderedGeometricMHA(30, n_heads=4)
    with pytest.raises(ValueError):
        PathOrderedGeometricMHA(32, n_heads=4, mode="ring")


def test_attributes_and_state_dict():
    m = PathOrderedGeometricMHA(192, n_heads=4, edge_scale=0.05)
    assert (m.h, m.d, m.m_dim, m.edge_scale, m.mode, m.link_mode) == (4, 48, 1128, 0.05, "causal",
                                                                        "interaction")
    assert abs(m.scale - 48 ** -0.5) < 1e-12
    shapes = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    assert list(shapes) == ["qkv.weight", "out.weight", "gqproj.weight", "gkproj.weight",
                            "edge_mlp.0.weight", "edge_mlp.0.bias", "edge_mlp.2.weight",
                            "edge_mlp.2.bias"]
    assert shapes["edge_mlp.2.weight"] == (1128 * 4, 768)
    assert shapes["qkv.weight"] == (576, 192)


@pytest.mark.parametrize("name", ["tiny_es01", "d48_L40", "d96_L32"])
def test_seeded_init_matches_reference(name):
    """Same creation order as the reference => identical seeded default init."""
    z = np.load(os.path.join(GOLD, name + ".npz"))
    torch.manual_seed(int(z["seed"]))
    m = PathOrderedGeometricMHA(int(z["D"]), n_heads=int(z["H"]), edge_scale=float(z["edge_scale"]))
    for k, v in checksums(m.state_dict()).items():
        np.testing.assert_allclose(v, z["cs:" + k], rtol=1e-9, atol=1e-12)
    x = torch.randn(int(z["B"]), int(z["L"]), int(z["D"]))
    np.testing.assert_array_equal(x.numpy(), z["x"])


def test_unsupported_inputs_raise():
    m = PathOrderedGeometricMHA(32, n_heads=4).eval()
    x = torch.randn(2, 12, 32)
    tril = torch.tril(torch.ones(12, 12, dtype=torch.bool))
    with torch.no_grad():
        with pytest.raises(NotImplementedError, match="CUDA"):
            m(x, attn_mask=tril)
    # the inert ablation is supported; a CPU input is still refused
    inert = PathOrderedGeometricMHA(32, n_heads=4, mode="inert").eval()
    with torch.no_grad(), pytest.raises(NotImplementedError, match="CUDA"):
        inert(x, attn_mask=tril)
    # masks must be (L, L) bool; an unknown link form is refused
    m.link_mode = "other"
    with torch.no_grad(), pytest.raises(NotImplementedError, match="link_mode"):
        m(x, attn_mask=tril)
    m.link_mode = "interaction"
    # return_geometry=True is supported, but the CPU input is still refused
    with torch.no_grad(), pytest.raises(NotImplementedError, match="CUDA"):
        m(x, attn_mask=tril, return_geometry=True)


def test_generator_precision_policy():
    """"auto" runs the bf16 edge MLP unsplit up to 8192 positions and split beyond;
    shards of a longer sequence follow the whole sequence's length."""
    m = PathOrderedGeometricMHA(192, n_heads=4)
    assert m.generator_precision == "auto"
    assert not m._split_generators(4096)
    assert not m._split_generators(m.AUTO_SPLIT_ABOVE)
    assert m._split_generators(m.AUTO_SPLIT_ABOVE + 1)
    assert m._split_generators(None)
    m.generator_precision = "split"
    assert m._split_generators(128)
    m.generator_precision = "bf16"
    assert not m._split_generators(65536)
    m.generator_precision = "split8"
    assert m._split_generators(128) and m._generator_mode(128) == "split8"
    m.generator_precision = "auto"
    assert m._generator_mode(4096) == "bf16" and m._generator_mode(None) == m.AUTO_LONG
    m.generator_precision = "fp8"
    with pytest.raises(ValueError):
        m._split_generators(128)


def test_split8_shape_rule():
    """"split8" runs its fp8 GEMM only where rows, hidden width and generator width are
    multiples of 16 (cuBLASLt's fp8 shapes); elsewhere the forward takes "split"."""
    m = PathOrderedGeometricMHA(1536, n_heads=16)          # banked layout, 16 x 4608 generators
    assert m._fp8_shape_ok(16384, 6144)
    assert not m._fp8_shape_ok(16383, 6144)
    assert not m._fp8_shape_ok(16384, 6140)
    small = PathOrderedGeometricMHA(20, n_heads=4)          # d = 5: 4 x 10 packed generators
    assert not small._fp8_shape_ok(16384, 80)
