"""The C-ABI library: it loads, exports every symbol include/hoa.h declares,
and rejects bad arguments before touching the GPU (no compute calls here)."""
import ctypes
import os
import re

import pytest

from holonomyawareattention_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hoa.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(hoa_[a-z_0-9]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from holonomyawareattention_b200 import _build
    _build.build()
    return _lib.load()


def test_header_symbols_exported(lib):
    syms = declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in hoa.h but not exported"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"


def test_debug_library_exports_the_same_abi():
    """libhoa_debug.so (device-side index checks compiled in) exports every entry point too;
    the product library answers hoa_debug_bounds with HOA_ERR_UNSUPPORTED (no GPU touched)."""
    from holonomyawareattention_b200 import _build
    _build.build(debug_bounds=True)
    dbg = _lib.load_debug()
    for s in declared_symbols():
        assert hasattr(dbg, s), f"{s} missing from libhoa_debug.so"
    st = ctypes.c_int(7)
    assert _lib.load().hoa_debug_bounds(0, ctypes.byref(st)) == _lib.HOA_ERR_UNSUPPORTED
    assert st.value == 0
    assert dbg.hoa_debug_bounds(-1, ctypes.byref(st)) == _lib.HOA_ERR_INVALID_ARG
    assert dbg.hoa_debug_bounds(0, None) == _lib.HOA_ERR_INVALID_ARG
    assert b"index" in dbg.hoa_status_string(_lib.HOA_ERR_BOUNDS)


def test_library_facts(lib):
    assert lib.hoa_abi_version() == 2
    assert lib.hoa_max_head_dim() == 120
    assert lib.hoa_status_string(0) == b"ok"
    assert b"workspace" in lib.hoa_status_string(4)


@pytest.mark.parametrize("B,H,T,d,sms", [(16, 16, 4096, 96, 148), (64, 4, 512, 48, 148),
                                          (128, 24, 2048, 120, 148), (1, 16, 65536, 96, 148),
                                          (2, 4, 12, 8, 148), (1, 1, 1, 8, 148)])
def test_plan_chunk(lib, B, H, T, d, sms):
    """The chunk minimises ceil(units / slots) * (chunk + 2) over chunks of >= 16 positions
    (units = B*H*ceil(T/chunk), slots = SMs x link CTAs per SM): the last wave stays full."""
    c = lib.hoa_plan_chunk(B, H, T, d, sms)
    assert 1 <= c <= max(T, 1)
    if T < 16:
        assert c == T
        return
    per_sm = 512 // (128 if 5 * d <= 128 else (256 if 5 * d <= 256 else 512)) \
        if d in (48, 64, 96) else (1 if d == 32 else None)

    def cost(chunk, slots):
        units = B * H * (-(-T // chunk))
        return -(-units // slots) * (chunk + 2)

    if per_sm is not None:
        slots = sms * per_sm
        best = min(cost(-(-T // K), slots) for K in range(1, T // 16 + 1))
        assert c >= 16 and cost(c, slots) == best
        if B * H * T >= 100 * slots:          # large problems: within 5% of a perfect split
            assert cost(c, slots) <= 1.05 * (B * H * T / slots) + 2 * -(-B * H * T // (slots * c))


def test_workspace_bytes(lib):
    n = lib.hoa_core_workspace_bytes(16, 16, 4096, 96, 832, _lib.HOA_BF16)
    # R dominates: B*H*T*d*d*4 bytes
    assert n >= 16 * 16 * 4096 * 96 * 96 * 4
    assert lib.hoa_core_workspace_bytes(0, 16, 4096, 96, 832, 1) == 0


def test_invalid_arguments_rejected_without_gpu(lib):
    null = None
    # null pointers -> HOA_ERR_INVALID_ARG (1) before any CUDA call
    assert lib.hoa_link_local(null, 0, null, 1.0, null, 0, null, null, null, null, 1, 1, 4, 8, 4, null) == 1
    assert lib.hoa_attn_fwd(null, null, null, 0, null, 1.0, 1, 4, 4, 0, 8, null) == 1
    assert lib.hoa_attn_tc_fwd(null, null, null, null, null, 1.0, 1, 4, 4, 0, 8, null) == 1
    assert lib.hoa_out_transport(null, null, null, 4, null, 0, 1, 1, 4, 8, null) == 1
    assert lib.hoa_carry_scan(null, null, null, null, 1, 1, 8, null) == 1
    # unsupported head dim -> HOA_ERR_UNSUPPORTED (2)
    dummy = ctypes.c_void_p(16)
    assert lib.hoa_link_local(dummy, 0, null, 1.0, dummy, 0, dummy, dummy, dummy, null, 1, 1, 4, 200, 4, null) == 2
    # bad dtype code
    assert lib.hoa_link_local(dummy, 7, null, 1.0, dummy, 0, dummy, dummy, dummy, null, 1, 1, 4, 8, 4, null) == 2
    # tensor-core attention needs d % 8 == 0 and d <= 128
    assert lib.hoa_attn_tc_fwd(dummy, dummy, dummy, dummy, null, 1.0, 1, 4, 4, 0, 12, null) == 2
    assert lib.hoa_attn_tc_fwd(dummy, dummy, dummy, dummy, null, 1.0, 1, 4, 4, 0, 136, null) == 2
    # a query shard must lie inside the key range
    assert lib.hoa_attn_tc_fwd(dummy, dummy, dummy, dummy, null, 1.0, 1, 4, 8, 6, 16, null) == 1
    assert lib.hoa_vt_stride(4093) == 4096 and lib.hoa_vt_stride(8) == 8
    # workspace too small -> HOA_ERR_WORKSPACE (4)
    assert lib.hoa_core_forward(dummy, 0, null, 1.0, dummy, 0, dummy, 0, 0, 1.0, null, null,
                                1, 1, 4, 8, 4, dummy, 16, null) == 4
    # the wait-bound diagnostic takes 0 (default) .. 4e9 cycles
    assert lib.hoa_set_wait_bound(-1) == 1
    assert lib.hoa_set_wait_bound(4_000_000_001) == 1
    assert lib.hoa_set_wait_bound(0) == 0
    assert lib.hoa_noalloc_status_word(null) == 1
    with pytest.raises(_lib.HoaError):
        _lib.check("hoa_link_local", 2)
