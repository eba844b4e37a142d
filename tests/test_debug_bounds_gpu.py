"""Device-side index checks of the debug build (libhoa_debug.so, -DHOA_DEBUG_BOUNDS).

compute-sanitizer is not available on the GPUs this library is tested on, so the
debug build carries its own checks: every kernel of the core path (link, carry
scan, carry apply, attention, inverse transport) checks the element range of each
global access against the extent its buffer has for the launch's shape, records
HOA_ERR_BOUNDS when a range falls outside and skips that access.  These tests run
the core forward through the debug library's C ABI:
  * with the true extents no check fires and the output equals the product
    library's bit for bit (the checks change nothing);
  * with the extents halved (hoa_debug_bounds' test hook) the checks fire on the
    upper half of every buffer, which the shape allows, and report HOA_ERR_BOUNDS;
    the skipped accesses were in bounds in reality, so nothing faults, and the
    context then runs the true-extent forward again with the first result.
"""
import ctypes
import math

import pytest
import torch

from holonomyawareattention_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
_DT = {torch.float32: _lib.HOA_F32, torch.bfloat16: _lib.HOA_BF16}


def _inputs(seed, B, T, H, d, dtype):
    g = torch.Generator(device=DEV).manual_seed(seed)
    m = d * (d - 1) // 2
    a = (0.02 * torch.randn(B, T, H * m, device=DEV, generator=g)).contiguous()
    qkv = torch.randn(B, T, 3 * H * d, device=DEV, generator=g).to(dtype).contiguous()
    return a, qkv


def _core(lib, a, qkv, H, d, es, chunk):
    """hoa_core_forward of `lib` (packed fp32 generators), workspace from torch."""
    B, T, _ = qkv.shape
    code = _DT[qkv.dtype]
    n = lib.hoa_core_workspace_bytes(B, H, T, d, chunk, code)
    ws = torch.empty(n, dtype=torch.uint8, device=DEV)
    out = torch.zeros(B, T, H * d, dtype=qkv.dtype, device=DEV)
    st = lib.hoa_core_forward(a.data_ptr(), _lib.HOA_F32, None, es, qkv.data_ptr(), code, out.data_ptr(),
                              code, code, 1.0 / math.sqrt(d), None, None, B, H, T, d, chunk,
                              ws.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    return out


def _debug_status(dbg, shift):
    """Waits for the device, returns the code recorded since the last call, sets the shift."""
    st = ctypes.c_int(-1)
    assert dbg.hoa_debug_bounds(shift, ctypes.byref(st)) == 0
    return st.value


@pytest.mark.parametrize("B,T,H,d,dtype,chunk", [
    (1, 200, 2, 96, torch.bfloat16, 64),     # tensor-core link and attention
    (2, 100, 3, 48, torch.bfloat16, 32),
    (1, 70, 2, 120, torch.float32, 16),      # SIMT link (head dim 120) and fp32 attention
])
def test_debug_checks_quiet_then_firing(B, T, H, d, dtype, chunk):
    dbg = _lib.load_debug()
    a, qkv = _inputs(B + T + d, B, T, H, d, dtype)
    ref = ops.core_forward(a, qkv, H, 0.3, chunk=chunk)        # product library
    torch.cuda.synchronize()
    _debug_status(dbg, 0)                                      # clear, true extents
    out = _core(dbg, a, qkv, H, d, 0.3, chunk)
    assert _debug_status(dbg, 1) == 0                          # quiet; now halve the extents
    assert torch.equal(out, ref)
    _core(dbg, a, qkv, H, d, 0.3, chunk)
    assert _debug_status(dbg, 0) == _lib.HOA_ERR_BOUNDS        # fired; true extents again
    out2 = _core(dbg, a, qkv, H, d, 0.3, chunk)
    assert _debug_status(dbg, 0) == 0
    assert torch.equal(out2, ref)
