"""Failure detection on the GPU without a fault: the bounded mbarrier waits that
every kernel of the library uses give up after their limit, raise the CTA's abort
flag so that the other waiters leave promptly, and report HOA_ERR_TIMEOUT to the
host; the context stays usable afterwards."""
import pytest
import torch

from holonomyawareattention_b200 import ops, _lib

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
