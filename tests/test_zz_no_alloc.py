"""hoa_core_forward_noalloc: the entry point for callers that cannot allocate.

Some callers cannot call cudaMalloc when they invoke the forward (for example
an inference-engine plugin's enqueue callback, or a process whose device
memory is held by another allocator).  hoa_core_forward_noalloc serves them
from a 16 MiB static device array inside the library.  This test calls it
through the C ABI and checks it against the existing entry point
(hoa_core_forward, scratch allocated by the caller) on the same inputs, for two
calls in a row with different inputs (the shared array keeps the previous
call's contents, which must not leak into the next result), and checks that a
problem too large for the array is refused.  The file is named so that pytest
collects it last.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from holonomyawareattention_b200 import _lib, ops
from oracle.holonomy_oracle import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _inputs(seed, B, T, H, d, dtype):
    g = torch.Generator(device=DEV).manual_seed(seed)
    m = d * (d - 1) // 2
    a = (0.02 * torch.randn(B, T, H * m, device=DEV, generator=g)).float().contiguous()
    qkv = torch.randn(B, T, 3 * H * d, device=DEV, generator=g).to(dtype).contiguous()
    return a, qkv


def _noalloc_status(lib):
    """The device status word of the last hoa_core_forward_noalloc call on this device
    (hoa_noalloc_status_word), read after the stream has completed."""
    ptr = ctypes.c_void_p()
    assert lib.hoa_noalloc_status_word(ctypes.byref(ptr)) == 0 and ptr.value
    torch.cuda.synchronize()

    class _Word:
        __cuda_array_interface__ = {"shape": (1,), "typestr": "<i4", "data": (ptr.value, False),
                                    "version": 3}
    return int(torch.as_tensor(_Word(), device=DEV).cpu()[0])


def _noalloc(lib, a, qkv, H, d, es, chunk, dtype, out):
    B, T, _ = qkv.shape
    code = 0 if dtype == torch.float32 else 1
    return lib.hoa_core_forward_noalloc(a.data_ptr(), 0, None, es, qkv.data_ptr(), code, out.data_ptr(),
                                        code, code, 1.0 / math.sqrt(d), None, None, B, H, T, d,
                                        chunk, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_core_forward(dtype):
    lib = _lib.load()
    B, T, H, d, es, chunk = 2, 96, 4, 48, 0.3, 32
    need = lib.hoa_core_workspace_bytes(B, H, T, d, chunk, 0 if dtype == torch.float32 else 1)
    assert need <= 16 * 1024 * 1024
    for seed in (1, 2):                      # two calls in a row, different inputs
        a, qkv = _inputs(seed, B, T, H, d, dtype)
        ref = ops.core_forward(a, qkv, H, es, chunk=chunk)
        out = torch.full((B, T, H * d), float("nan"), dtype=dtype, device=DEV)
        assert _noalloc(lib, a, qkv, H, d, es, chunk, dtype, out) == 0
        torch.cuda.synchronize()
        assert _noalloc_status(lib) == 0           # no device-side wait gave up
        assert torch.isfinite(out).all()
        assert rel_l2(out.float().cpu().numpy(), ref.float().cpu().numpy()) <= TOL[dtype]


def test_noalloc_rejects_problems_beyond_its_scratch():
    lib = _lib.load()
    B, T, H, d, chunk = 8, 1024, 4, 48, 64
    assert lib.hoa_core_workspace_bytes(B, H, T, d, chunk, 0) > 16 * 1024 * 1024
    a, qkv = _inputs(3, 1, 4, H, d, torch.float32)      # pointers only; nothing is launched
    out = torch.empty(1, dtype=torch.float32, device=DEV)
    st = lib.hoa_core_forward_noalloc(a.data_ptr(), 0, None, 0.3, qkv.data_ptr(), 0, out.data_ptr(), 0, 0,
                                      0.1, None, None, B, H, T, d, chunk,
                                      torch.cuda.current_stream().cuda_stream)
    assert st == 4                                       # HOA_ERR_WORKSPACE
    assert b"workspace" in lib.hoa_status_string(st)
