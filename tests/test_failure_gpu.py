"""Failure detection on the GPU without a fault: the bounded mbarrier waits that
every kernel of the library uses give up after their limit, raise the CTA's abort
flag so that the other waiters leave promptly, and report HOA_ERR_TIMEOUT to the
host; the context stays usable afterwards."""
import pytest
import torch

from holonomyawareattention_b200 import PathOrderedGeometricMHA, ops, _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_aborts_peers():
    max_cycles = 200_000
    status, peer_aborted, peer_kcycles, both = ops.selftest_wait(max_cycles)
    assert status == _lib.HOA_ERR_TIMEOUT
    assert peer_aborted == 1 and both == 1
    # the second waiter's own bound is 4e9 cycles; it must have left on the flag,
    # within a small multiple of the first waiter's bound
    assert peer_kcycles * 1024 < 100 * max_cycles


def test_context_usable_after_timeout():
    ops.selftest_wait(50_000)
    torch.cuda.synchronize()
    a = torch.randn(1, 8, 2 * 28, device="cuda") * 0.1
    qkv = torch.randn(1, 8, 2 * 3 * 8, device="cuda")
    out = ops.core_forward(a, qkv, 2, 1.0, 8 ** -0.5, out_dtype=torch.float32, hat_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()


def test_selftest_rejects_bad_bounds():
    with pytest.raises(_lib.HoaError):
        ops.selftest_wait(0)


def test_real_forward_surfaces_a_timed_out_wait():
    """A real forward whose bounded waits give up: with a wait bound of a few hundred SM
    cycles (hoa_set_wait_bound) the tensor-core link and attention kernels give up on waits
    that TMA copies and products normally satisfy within microseconds, leave early (after
    their copies and products in flight have landed) and set HOA_ERR_TIMEOUT.  The module
    must raise that status instead of returning the invalid output as valid; with the
    default bound restored, the same forward runs again and gives the first result."""
    D, H, L = 384, 4, 512
    torch.manual_seed(3)
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=0.05).to("cuda", torch.bfloat16).eval()
    x = torch.randn(1, L, D, device="cuda").to(torch.bfloat16)
    mask = torch.tril(torch.ones(L, L, dtype=torch.bool, device="cuda"))
    with torch.no_grad():
        y0, _ = m(x, attn_mask=mask)
        ops.check_status()
        ops.set_wait_bound(256)
        try:
            m(x, attn_mask=mask)
            torch.cuda.synchronize()
            with pytest.raises(_lib.HoaError) as e:
                ops.check_status()
            assert e.value.status == _lib.HOA_ERR_TIMEOUT
        finally:
            ops.set_wait_bound(0)
        y1, _ = m(x, attn_mask=mask)
        ops.check_status()
    assert torch.equal(y0, y1)


def test_stage_calls_surface_a_timed_out_wait():
    """The stage entry points (hoa_link_local, hoa_attn_tc_fwd, used by the sequence-sharded
    path) report through the shared status word: a forward in stages with a short wait bound
    raises HOA_ERR_TIMEOUT; the next poll after that is clean."""
    B, T, H, d = 1, 256, 2, 96
    g = torch.Generator(device="cuda").manual_seed(4)
    a = (0.02 * torch.randn(B, T, H * d * (d - 1) // 2, device="cuda", generator=g)).contiguous()
    qkv = torch.randn(B, T, 3 * H * d, device="cuda", generator=g).to(torch.bfloat16)
    ops.set_wait_bound(256)
    try:
        ops.core_stages(a, qkv, H, 0.5, d ** -0.5, torch.bfloat16, torch.bfloat16, 64)
        torch.cuda.synchronize()
        with pytest.raises(_lib.HoaError) as e:
            ops.check_status()
        assert e.value.status == _lib.HOA_ERR_TIMEOUT
    finally:
        ops.set_wait_bound(0)
    ops.core_stages(a, qkv, H, 0.5, d ** -0.5, torch.bfloat16, torch.bfloat16, 64)
    ops.check_status()


def test_status_watch_across_inference_mode():
    """The status words of a device are first watched under inference mode, then outside it
    (a module used for serving and for evaluation in one process)."""
    ops._WATCH.clear()
    B, T, H, d = 1, 64, 2, 32
    a = (0.02 * torch.randn(B, T, H * d * (d - 1) // 2, device="cuda")).contiguous()
    qkv = torch.randn(B, T, 3 * H * d, device="cuda").to(torch.bfloat16)
    with torch.inference_mode():
        ops.core_forward(a, qkv, H, 0.5)
    with torch.no_grad():
        ops.core_forward(a, qkv, H, 0.5)
        ops.core_stages(a, qkv, H, 0.5, d ** -0.5, torch.bfloat16, torch.bfloat16, 16)
    ops.check_status()
