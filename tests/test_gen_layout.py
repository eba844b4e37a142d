"""The banked generator layout (HOA_GEN_BANKED): host-side facts, no GPU.

The layout is a permutation of the reference's packed upper triangle
(core/utils.py skew_from_vec order) into d(d-1)/2 of hoa_gen_stride(d, 1)
slots, with bank (i + j) mod 32 for entry {i, j}, so that a warp reading one
column of the skew matrix for 32 consecutive rows meets no bank conflict.
"""
import ctypes

import pytest
import torch

from holonomyawareattention_b200 import _lib, ops


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def packed_pairs(d):
    return [(i, j) for i in range(d) for j in range(i + 1, d)]


@pytest.mark.parametrize("d", [32, 64, 96])
def test_banked_map_is_a_bijection_with_conflict_free_reads(d):
    """The map is a bijection into the stride, and each read pattern of the link
    kernel's expansion (32 consecutive rows per warp, one block of columns) is
    free of shared-memory bank conflicts."""
    S = ops.gen_stride(d, "banked")
    nb = d // 32
    assert S == 1024 * (nb * (nb - 1) // 2) + 512 * nb
    assert ops.gen_stride(d, "packed") == d * (d - 1) // 2
    slots = ops.gen_banked_map(d).tolist()
    assert len(slots) == d * (d - 1) // 2
    assert len(set(slots)) == len(slots) and min(slots) >= 0 and max(slots) < S
    slot_of = {}
    for (i, j), s in zip(packed_pairs(d), slots):
        slot_of[(i, j)] = slot_of[(j, i)] = s
    for g in range(nb):                 # warp rows 32g .. 32g+31
        for bc in range(nb):            # its column block
            cols = range(32 * bc, 32 * bc + 32)
            if g > bc:
                # lower rows: one 4-byte access per column, 32 distinct banks
                for c in cols:
                    banks = [slot_of[(32 * g + l, c)] % 32 for l in range(32)]
                    assert len(set(banks)) == 32
            elif g < bc:
                # upper rows: each lane reads its own 32-slot line as 16-byte quads;
                # quad q of the columns sits at quad q ^ (l mod 8) of the line, in order
                for l in range(32):
                    line = [slot_of[(32 * g + l, c)] for c in cols]
                    base = min(line)
                    assert base % 32 == 0 and sorted(line) == list(range(base, base + 32))
                    for q in range(8):
                        quad = line[4 * q:4 * q + 4]
                        assert quad == list(range(quad[0], quad[0] + 4))
                        assert (quad[0] - base) // 4 == q ^ (l % 8)
                # 8 lanes of a phase read 8 distinct 16-byte bank groups
                for q in range(8):
                    for ph in range(4):
                        groups = [(slot_of[(32 * g + l, 32 * bc + 4 * q)] // 4) % 8
                                  for l in range(8 * ph, 8 * ph + 8)]
                        assert len(set(groups)) == 8
            else:
                # diagonal block: bank (i + j) mod 32, one access per column
                for c in cols:
                    rows = [32 * g + l for l in range(32) if 32 * g + l != c]
                    banks = [slot_of[(r, c)] % 32 for r in rows]
                    assert all(slot_of[(r, c)] % 32 == (r + c) % 32 for r in rows)
                    assert len(set(banks)) == len(banks)


def test_banked_layout_needs_d_multiple_of_32(lib):
    assert ops.gen_stride(48, "banked") == 0 and ops.gen_stride(120, "banked") == 0
    buf = (ctypes.c_int * 1128)()
    assert lib.hoa_gen_banked_map(48, buf) == _lib.HOA_ERR_UNSUPPORTED
    assert lib.hoa_gen_banked_map(96, None) == _lib.HOA_ERR_INVALID_ARG
    dummy = ctypes.c_void_p(16)
    banked_f32 = _lib.HOA_F32 | _lib.HOA_GEN_BANKED
    banked_bf16 = _lib.HOA_BF16 | _lib.HOA_GEN_BANKED
    # d = 48: no banked layout; bf16 generators: no banked layout -> HOA_ERR_UNSUPPORTED
    assert lib.hoa_link_local(dummy, banked_f32, None, 1.0, dummy, 0, dummy, dummy, dummy, None,
                              1, 1, 4, 48, 4, None) == _lib.HOA_ERR_UNSUPPORTED
    assert lib.hoa_link_local(dummy, banked_bf16, None, 1.0, dummy, 0, dummy, dummy, dummy, None,
                              1, 1, 4, 96, 4, None) == _lib.HOA_ERR_UNSUPPORTED


@pytest.mark.parametrize("d,H", [(32, 3), (96, 2)])
def test_to_and_from_banked_round_trip(d, H):
    m = d * (d - 1) // 2
    a = torch.randn(2, 5, H * m)
    b = ops.gen_to_banked(a, H, d)
    S = ops.gen_stride(d, "banked")
    assert b.shape == (2, 5, H * S)
    assert torch.equal(ops.gen_from_banked(b, H, d), a)
    # unused slots are zero, every value appears once
    assert int((b != 0).sum()) == int((a != 0).sum())
    # head h's entries stay inside head h's row segment
    heads = b.view(2, 5, H, S)
    for h in range(H):
        assert torch.equal(ops.gen_from_banked(heads[:, :, h], 1, d), a.view(2, 5, H, m)[:, :, h])


def test_module_weight_rows_follow_the_layout():
    from holonomyawareattention_b200 import PathOrderedGeometricMHA
    torch.manual_seed(0)
    mod = PathOrderedGeometricMHA(d_model=64, n_heads=2)        # d = 32: banked
    assert mod._gen_layout() == "banked"
    w, b = mod.edge_mlp[2].weight.detach(), mod.edge_mlp[2].bias.detach()
    wb, bb = mod._w2_rows(w, b)
    h = torch.randn(7, w.shape[1])
    packed = h @ w.t() + b
    banked = h @ wb.t() + bb
    assert torch.allclose(ops.gen_from_banked(banked, 2, 32), packed, atol=1e-5, rtol=1e-5)
    assert PathOrderedGeometricMHA(d_model=96, n_heads=2)._gen_layout() == "packed"   # d = 48
