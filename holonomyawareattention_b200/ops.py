"""Tensor-level wrappers over the libhoa C ABI (include/hoa.h).

Each function validates shapes/dtypes/devices, allocates outputs and scratch
with PyTorch (the C ABI never allocates), and enqueues the kernels on the
current CUDA stream.  There is no fallback path: a missing library, a CPU
tensor or an unsupported shape raises.
"""
from __future__ import annotations

import collections
import math
import threading
from typing import Optional, Tuple

import torch

from . import _lib

_DT = {torch.float32: _lib.HOA_F32, torch.bfloat16: _lib.HOA_BF16}


def _dtype_code(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError:
        raise NotImplementedError(f"dtype {t} is not supported (float32 or bfloat16)") from None


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise NotImplementedError("the B200 kernels need CUDA tensors (there is no CPU path)")


def _contig(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


# ---------------------------------------------------------------------------
# device status words.  The tensor-core kernels bound every wait on the GPU; a
# wait that gives up makes its kernel leave early and set HOA_ERR_TIMEOUT in a
# status word, and the output of that launch is not valid.  The word is known
# only once the stream has run, so every op here queues a 4-byte copy of it to
# pinned host memory behind its kernels: poll_status() raises for the copies
# that have landed (the module calls it at every forward), check_status() waits
# for all of them first (call it after synchronising, e.g. at the end of a run).
# ---------------------------------------------------------------------------
class _StatusWatch:
    RING = 256

    def __init__(self, dev: torch.device):
        self.dev = dev
        # normal tensors even when the first call comes under inference mode, so that
        # later calls outside it may update them
        with torch.inference_mode(False):
            # the word the stage entry points share: set by a kernel, cleared here
            self.sticky = torch.zeros(1, dtype=torch.int32, device=dev)
            self.host = torch.zeros(self.RING, dtype=torch.int32).pin_memory()
        self.pending = collections.deque()        # (slot, event, what)
        self.next = 0
        self.lock = threading.Lock()

    def watch(self, word: torch.Tensor, what: str) -> None:
        """Queue a copy of the device int32 ``word`` behind the current stream's work."""
        if torch.cuda.is_current_stream_capturing():
            return
        with self.lock:
            if len(self.pending) == self.RING:
                self.pending[0][1].synchronize()
                self._poll_locked()
            slot = self.next
            self.next = (self.next + 1) % self.RING
            self.host[slot:slot + 1].copy_(word.view(torch.int32)[:1], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.dev))
            self.pending.append((slot, ev, what))

    def _poll_locked(self) -> None:
        while self.pending and self.pending[0][1].query():
            slot, _, what = self.pending.popleft()
            st = int(self.host[slot])
            if st != 0:
                # report once: forget the other copies in flight and clear the shared word
                for _, ev, _ in self.pending:
                    ev.synchronize()
                self.pending.clear()
                self.sticky.zero_()
                _lib.check(what, st)

    def poll(self) -> None:
        with self.lock:
            self._poll_locked()

    def check(self) -> None:
        with self.lock:
            for _, ev, _ in self.pending:
                ev.synchronize()
            self._poll_locked()


_WATCH = {}


def _watch(dev: torch.device) -> _StatusWatch:
    dev = torch.device(dev)
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    w = _WATCH.get(dev)
    if w is None:
        w = _WATCH[dev] = _StatusWatch(dev)
    return w


def poll_status(device=None) -> None:
    """Raise HoaError for any finished launch on ``device`` whose device-side wait
    gave up (HOA_ERR_TIMEOUT).  Does not wait for launches still running."""
    _watch(device if device is not None else "cuda").poll()


def check_status(device=None) -> None:
    """Wait for every launch queued so far on ``device`` and raise HoaError if any
    of them reported HOA_ERR_TIMEOUT."""
    _watch(device if device is not None else "cuda").check()


def set_wait_bound(max_cycles: int) -> None:
    """Bound (SM cycles) of the device-side waits of the kernels launched from now
    on, process-wide; 0 restores the default.  A diagnostic: a short bound makes
    real kernels give up and report HOA_ERR_TIMEOUT (hoa_set_wait_bound)."""
    _lib.call("hoa_set_wait_bound", int(max_cycles))


def plan_chunk(B: int, H: int, T: int, d: int, device=None) -> int:
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    return int(_lib.load().hoa_plan_chunk(B, H, T, d, sms))


# ---------------------------------------------------------------------------
# generator layouts: "packed" (the reference's upper triangle, d(d-1)/2 floats
# per head) and "banked" (HOA_GEN_BANKED: the same values permuted, and a few
# unused slots, so that the link kernel reads rows without bank conflicts)
# ---------------------------------------------------------------------------
_BANKED_MAPS = {}


def gen_stride(d: int, layout: str = "packed") -> int:
    """Floats per head of a generator row in ``layout`` (0: not available for d)."""
    if layout not in ("packed", "banked"):
        raise ValueError("layout must be 'packed' or 'banked'")
    return int(_lib.load().hoa_gen_stride(d, 1 if layout == "banked" else 0))


def gen_banked_map(d: int) -> torch.Tensor:
    """(d(d-1)/2,) int64 on the CPU: the banked slot of every packed (reference-order) entry."""
    if d not in _BANKED_MAPS:
        m = d * (d - 1) // 2
        out = torch.empty(m, dtype=torch.int32)
        _lib.call("hoa_gen_banked_map", d, out.data_ptr())
        _BANKED_MAPS[d] = out.long()
    return _BANKED_MAPS[d]


def gen_banked_index(d: int, n_heads: int, device=None) -> torch.Tensor:
    """(H*m,) int64: the banked position (h*stride + slot) of packed entry h*m + i."""
    S = gen_stride(d, "banked")
    slots = gen_banked_map(d)
    idx = (torch.arange(n_heads).unsqueeze(1) * S + slots.unsqueeze(0)).reshape(-1)
    return idx if device is None else idx.to(device)


def gen_to_banked(a: torch.Tensor, n_heads: int, d: int) -> torch.Tensor:
    """(..., H*m) packed generators -> (..., H*stride) banked (zeros at unused slots)."""
    S = gen_stride(d, "banked")
    out = a.new_zeros(*a.shape[:-1], n_heads * S)
    out[..., gen_banked_index(d, n_heads, a.device)] = a
    return out


def gen_from_banked(a: torch.Tensor, n_heads: int, d: int) -> torch.Tensor:
    """(..., H*stride) banked generators -> (..., H*m) packed."""
    return a[..., gen_banked_index(d, n_heads, a.device)]


def _gen_code(a_all: torch.Tensor, layout: str) -> int:
    code = _dtype_code(a_all.dtype)
    if layout == "banked":
        if a_all.dtype != torch.float32:
            raise NotImplementedError("banked generators are fp32")
        code |= _lib.HOA_GEN_BANKED
    elif layout != "packed":
        raise ValueError("gen_layout must be 'packed' or 'banked'")
    return code


def _gen_width(n_heads: int, d: int, layout: str) -> int:
    S = gen_stride(d, layout)
    if S == 0:
        raise NotImplementedError(f"the {layout} generator layout needs d % 32 == 0 (d = {d})")
    return n_heads * S


def core_forward(a_all: torch.Tensor, qkv: torch.Tensor, n_heads: int, edge_scale: float,
                 softmax_scale: Optional[float] = None, out_dtype: Optional[torch.dtype] = None,
                 hat_dtype: Optional[torch.dtype] = None, chunk: Optional[int] = None,
                 carry_in: Optional[torch.Tensor] = None,
                 total_out: Optional[torch.Tensor] = None,
                 a_bias: Optional[torch.Tensor] = None,
                 gen_layout: str = "packed") -> torch.Tensor:
    """Core region (kernels 1-4): a_all (B,T,H*m) and qkv (B,T,3D) -> heads (B,T,D).

    ``a_all`` is the raw edge-MLP output (edge_scale is applied in the kernel,
    as core/attention_fast_chunked.py:77 does); ``a_bias`` (one generator row,
    fp32) is the MLP's output bias when the GEMM left it out.  ``gen_layout``
    "banked": a_all (B,T,H*stride) and a_bias in the banked layout
    (gen_to_banked).  ``carry_in`` / ``total_out`` are optional (B*H, d, d) fp32
    tensors (see hoa_core_forward).
    """
    _need_cuda(a_all, qkv, carry_in, total_out, a_bias)
    B, T, threeD = qkv.shape
    D = threeD // 3
    H = n_heads
    d = D // H
    a_code = _gen_code(a_all, gen_layout)
    width = _gen_width(H, d, gen_layout)
    if a_all.shape != (B, T, width):
        raise ValueError(f"a_all must be (B,T,{width}) for the {gen_layout} layout, got {tuple(a_all.shape)}")
    _contig(a_all, "a_all"); _contig(qkv, "qkv")
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(d)
    _check_bias(a_bias, width)
    out_dtype = out_dtype or qkv.dtype
    hat_dtype = hat_dtype or qkv.dtype
    if chunk is None:
        chunk = plan_chunk(B, H, T, d, qkv.device)
    for t, nm in ((carry_in, "carry_in"), (total_out, "total_out")):
        if t is not None and (t.dtype != torch.float32 or t.shape != (B * H, d, d) or not t.is_contiguous()):
            raise ValueError(f"{nm} must be a contiguous fp32 ({B * H},{d},{d}) tensor")
    lib = _lib.load()
    hat_code = _dtype_code(hat_dtype)
    ws_bytes = int(lib.hoa_core_workspace_bytes(B, H, T, d, chunk, hat_code))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=qkv.device)
    out = torch.empty(B, T, D, dtype=out_dtype, device=qkv.device)
    _lib.call("hoa_core_forward", _ptr(a_all), a_code, _ptr(a_bias), float(edge_scale),
              _ptr(qkv), _dtype_code(qkv.dtype), _ptr(out), _dtype_code(out_dtype), hat_code,
              float(softmax_scale), _ptr(carry_in), _ptr(total_out), B, H, T, d, int(chunk),
              _ptr(ws), ws_bytes, _stream(qkv.device))
    # the status word is the workspace's first 4 bytes (hoa_core_workspace_bytes)
    _watch(qkv.device).watch(ws[:4], "hoa_core_forward")
    return out


# ---------------------------------------------------------------------------
# individual stages (used by the tests and by the sequence-sharded path)
# ---------------------------------------------------------------------------
def _check_bias(a_bias, n):
    if a_bias is not None and (a_bias.dtype != torch.float32 or a_bias.numel() != n
                               or not a_bias.is_contiguous()):
        raise ValueError(f"a_bias must be a contiguous fp32 tensor of {n} elements")


def link_local(a_all: torch.Tensor, qkv: torch.Tensor, n_heads: int, edge_scale: float,
               chunk: int, a_bias: Optional[torch.Tensor] = None, gen_layout: str = "packed"
               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Kernel (1)+(2) local part -> (R (BH,T,d,d), U (BH,T,3,d), M (BH,K,d,d)), all fp32."""
    _need_cuda(a_all, qkv, a_bias)
    B, T, threeD = qkv.shape
    H = n_heads
    d = threeD // 3 // H
    K = (T + chunk - 1) // chunk
    a_code = _gen_code(a_all, gen_layout)
    width = _gen_width(H, d, gen_layout)
    if a_all.shape[-1] != width or a_all.numel() != B * T * width:
        raise ValueError(f"a_all must be (B,T,{width}) for the {gen_layout} layout, got {tuple(a_all.shape)}")
    _contig(a_all, "a_all"); _contig(qkv, "qkv")
    _check_bias(a_bias, width)
    dev = qkv.device
    R = torch.empty(B * H, T, d, d, dtype=torch.float32, device=dev)
    U = torch.empty(B * H, T, 3, d, dtype=torch.float32, device=dev)
    M = torch.empty(B * H, K, d, d, dtype=torch.float32, device=dev)
    w = _watch(dev)
    _lib.call("hoa_link_local", _ptr(a_all), a_code, _ptr(a_bias), float(edge_scale), _ptr(qkv),
              _dtype_code(qkv.dtype), _ptr(R), _ptr(U), _ptr(M), _ptr(w.sticky), B, H, T, d,
              int(chunk), _stream(dev))
    w.watch(w.sticky, "hoa_link_local")
    return R, U, M


def carry_scan(M: torch.Tensor, carry_in: Optional[torch.Tensor] = None,
               want_total: bool = False):
    """C_0 = carry_in (or I), C_{k+1} = M_k C_k -> (C (BH,K,d,d), total (BH,d,d) or None)."""
    _need_cuda(M, carry_in)
    BH, K, d, _ = M.shape
    _contig(M, "M")
    C = torch.empty_like(M)
    total = torch.empty(BH, d, d, dtype=torch.float32, device=M.device) if want_total else None
    _lib.call("hoa_carry_scan", _ptr(M), _ptr(carry_in), _ptr(C), _ptr(total), BH, K, d,
              _stream(M.device))
    return C, total


def vt_stride(T: int) -> int:
    return int(_lib.load().hoa_vt_stride(T))


def carry_apply(U: torch.Tensor, C: torch.Tensor, chunk: int, hat_dtype: torch.dtype,
                v_transposed: bool = False):
    """q^, k^ (BH,T,d) and v^ (BH,T,d), or v^T (BH,d,vt_stride(T)) if v_transposed."""
    _need_cuda(U, C)
    BH, T, _, d = U.shape
    dev = U.device
    qh = torch.empty(BH, T, d, dtype=hat_dtype, device=dev)
    kh = torch.empty(BH, T, d, dtype=hat_dtype, device=dev)
    vs = vt_stride(T) if v_transposed else 0
    vh = (torch.empty(BH, d, vs, dtype=hat_dtype, device=dev) if v_transposed
          else torch.empty(BH, T, d, dtype=hat_dtype, device=dev))
    _lib.call("hoa_carry_apply", _ptr(U), _ptr(C), _ptr(qh), _ptr(kh), _ptr(vh),
              _dtype_code(hat_dtype), vs, BH, T, d, int(chunk), _stream(dev))
    return qh, kh, vh


def attn_fwd(qh: torch.Tensor, kh: torch.Tensor, vh: torch.Tensor,
             softmax_scale: float, q_offset: int = 0) -> torch.Tensor:
    """Kernel (3), fp32 SIMT path: o = softmax(q^ k^T * scale, causal) v^ -> (BH,Tq,d) fp32.

    q^ (BH,Tq,d) holds global positions q_offset.., k^/v^ (BH,Tk,d) positions 0..Tk-1."""
    _need_cuda(qh, kh, vh)
    BH, Tq, d = qh.shape
    Tk = kh.shape[1]
    o = torch.empty(BH, Tq, d, dtype=torch.float32, device=qh.device)
    _lib.call("hoa_attn_fwd", _ptr(qh), _ptr(kh), _ptr(vh), _dtype_code(qh.dtype), _ptr(o),
              float(softmax_scale), BH, Tq, Tk, int(q_offset), d, _stream(qh.device))
    return o


def attn_tc_fwd(qh: torch.Tensor, kh: torch.Tensor, vhT: torch.Tensor, softmax_scale: float,
                status: Optional[torch.Tensor] = None, q_offset: int = 0) -> torch.Tensor:
    """Kernel (3), tcgen05 bf16 path (v^ transposed) -> o (BH,Tq,d) fp32.

    q^ (BH,Tq,d) holds global positions q_offset.., k^ (BH,Tk,d) and
    v^T (BH,d,vt_stride(Tk)) positions 0..Tk-1."""
    _need_cuda(qh, kh, vhT)
    BH, Tq, d = qh.shape
    Tk = kh.shape[1]
    if qh.dtype != torch.bfloat16:
        raise NotImplementedError("the tensor-core attention takes bf16 q^/k^/v^")
    if vhT.shape != (BH, d, vt_stride(Tk)):
        raise ValueError(f"v^T must be (BH, d, vt_stride(Tk)) = ({BH}, {d}, {vt_stride(Tk)})")
    o = torch.empty(BH, Tq, d, dtype=torch.float32, device=qh.device)
    w = _watch(qh.device) if status is None else None
    _lib.call("hoa_attn_tc_fwd", _ptr(qh), _ptr(kh), _ptr(vhT), _ptr(o),
              _ptr(status) if w is None else _ptr(w.sticky),
              float(softmax_scale), BH, Tq, Tk, int(q_offset), d, _stream(qh.device))
    if w is not None:
        w.watch(w.sticky, "hoa_attn_tc_fwd")
    return o


def out_transport(o: torch.Tensor, R: torch.Tensor, C: torch.Tensor, chunk: int, B: int, H: int,
                  out_dtype: torch.dtype) -> torch.Tensor:
    """Kernel (4): out_t = R_t C_k o_t -> (B,T,H*d) in out_dtype."""
    _need_cuda(o, R, C)
    BH, T, d = o.shape
    out = torch.empty(B, T, H * d, dtype=out_dtype, device=o.device)
    _lib.call("hoa_out_transport", _ptr(o), _ptr(R), _ptr(C), int(chunk), _ptr(out),
              _dtype_code(out_dtype), B, H, T, d, _stream(o.device))
    return out


def compose_paths(R: torch.Tensor, C: torch.Tensor, chunk: int, p_dtype: torch.dtype = torch.float32
                  ) -> torch.Tensor:
    """P_t = R_t C_{t/chunk} -> (BH, T, d, d) in p_dtype (the path products of return_geometry)."""
    _need_cuda(R, C)
    BH, T, d, _ = R.shape
    _contig(R, "R"); _contig(C, "C")
    if C.shape != (BH, (T + chunk - 1) // chunk, d, d):
        raise ValueError("C must be (BH, ceil(T/chunk), d, d)")
    P = torch.empty(BH, T, d, d, dtype=p_dtype, device=R.device)
    _lib.call("hoa_compose_paths", _ptr(R), _ptr(C), _ptr(P), _dtype_code(p_dtype), BH, T, d,
              int(chunk), _stream(R.device))
    return P


def core_geometry(a_all, qkv, n_heads, edge_scale, softmax_scale, out_dtype, hat_dtype, chunk,
                  a_bias=None, gen_layout="packed", geo_dtype=None):
    """The core region with the geometry kept: (heads (B,T,D), P (B,H,T,d,d), Hol (B,H,d,d)).

    Same kernels as core_forward, run stage by stage so that the local products
    R and the carries C survive: P_t = R_t C_{t/chunk} (hoa_compose_paths) and
    Hol = the carry scan's total through the closing edge t = T-1
    (core/attention_fast_chunked.py:95, 175-177).  P and Hol come in geo_dtype
    (default: out_dtype), as the reference returns them in x's dtype."""
    B, T, threeD = qkv.shape
    H = n_heads
    d = threeD // 3 // H
    geo_dtype = geo_dtype or out_dtype
    R, U, M = link_local(a_all, qkv, H, edge_scale, chunk, a_bias, gen_layout)
    C, total = carry_scan(M, want_total=True)
    tc = uses_tensor_cores(hat_dtype, d)
    qh, kh, vh = carry_apply(U, C, chunk, hat_dtype, v_transposed=tc)
    o = attn_tc_fwd(qh, kh, vh, softmax_scale) if tc else attn_fwd(qh, kh, vh, softmax_scale)
    heads = out_transport(o, R, C, chunk, B, H, out_dtype)
    del qh, kh, vh, o, U, M
    P = compose_paths(R, C, chunk, geo_dtype).view(B, H, T, d, d)
    return heads, P, total.view(B, H, d, d).to(geo_dtype)


# ---------------------------------------------------------------------------
# the general forms (any mask, wrap pairs, inert ablation), core/attention.py
# ---------------------------------------------------------------------------
def attn_general_fwd(qh: torch.Tensor, kh: torch.Tensor, vh: torch.Tensor, softmax_scale: float,
                     kw: Optional[torch.Tensor] = None, vw: Optional[torch.Tensor] = None,
                     mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention over all keys (fp32, (BH,T,d)): wrap pairs j > i use kw/vw when given;
    mask (T,T) bool/uint8, True = allowed, None = all allowed."""
    _need_cuda(qh, kh, vh, kw, vw, mask)
    BH, T, d = qh.shape
    for t, nm in ((qh, "qh"), (kh, "kh"), (vh, "vh"), (kw, "kw"), (vw, "vw")):
        if t is not None and (t.dtype != torch.float32 or t.shape != (BH, T, d) or not t.is_contiguous()):
            raise ValueError(f"{nm} must be a contiguous fp32 ({BH},{T},{d}) tensor")
    if (kw is None) != (vw is None):
        raise ValueError("kw and vw go together")
    m8 = None
    if mask is not None:
        if tuple(mask.shape) != (T, T):
            raise ValueError(f"mask must be ({T},{T})")
        m8 = mask.to(device=qh.device, dtype=torch.uint8).contiguous()
    o = torch.empty(BH, T, d, dtype=torch.float32, device=qh.device)
    _lib.call("hoa_attn_general_fwd", _ptr(qh), _ptr(kh), _ptr(vh), _ptr(kw), _ptr(vw), _ptr(m8),
              _ptr(o), float(softmax_scale), BH, T, d, _stream(qh.device))
    return o


def chain_matvec(x: torch.Tensor, M: torch.Tensor, transpose: bool = False) -> torch.Tensor:
    """y_t = M x_t (or M^T x_t), x (BH,T,d) fp32, M (BH,d,d) fp32."""
    _need_cuda(x, M)
    BH, T, d = x.shape
    _contig(x, "x"); _contig(M, "M")
    y = torch.empty_like(x)
    _lib.call("hoa_chain_matvec", _ptr(x), _ptr(M), _ptr(y), int(transpose), BH, T, d, _stream(x.device))
    return y


def apply_paths(x: torch.Tensor, R: torch.Tensor, C: torch.Tensor, chunk: int,
                transpose: bool = False) -> torch.Tensor:
    """y_t = P_t x_t (or P_t^T x_t) with P_t = R_t C_{t/chunk}; x (BH,T,d) fp32."""
    _need_cuda(x, R, C)
    BH, T, d = x.shape
    _contig(x, "x")
    y = torch.empty_like(x)
    _lib.call("hoa_apply_paths", _ptr(x), _ptr(R), _ptr(C), int(chunk), _ptr(y), int(transpose),
              BH, T, d, _stream(x.device))
    return y


def core_general(a_all, qkv, n_heads, edge_scale, softmax_scale, out_dtype, chunk, mode="causal",
                 mask=None, a_bias=None, gen_layout="packed", geometry=False, geo_dtype=None):
    """The core region for any mask and both modes of core/attention.py (fp32 throughout).

    "causal": q^ = P^T q etc.; the wrap pairs j > i (live when the mask allows any)
    see Hol k^_j and Hol v^_j (core/attention.py:156-165); out = P o.
    "inert": q~ = P q etc., no wrap pairs, out = P^T o (:166-169).
    Returns heads (B,T,D) in out_dtype, and with ``geometry`` also P (B,H,T,d,d) and
    Hol (B,H,d,d) in geo_dtype (default out_dtype)."""
    B, T, threeD = qkv.shape
    H = n_heads
    D = threeD // 3
    d = D // H
    R, U, M = link_local(a_all, qkv, H, edge_scale, chunk, a_bias, gen_layout)
    C, total = carry_scan(M, want_total=True)
    if mode == "causal":
        qh, kh, vh = carry_apply(U, C, chunk, torch.float32)
        wrap = mask is None or bool(torch.triu(mask.bool(), 1).any())
        kw = chain_matvec(kh, total) if wrap else None
        vw = chain_matvec(vh, total) if wrap else None
        o = attn_general_fwd(qh, kh, vh, softmax_scale, kw, vw, mask)
        heads = out_transport(o, R, C, chunk, B, H, out_dtype)
    elif mode == "inert":
        parts = qkv.view(B, T, H, 3, d).permute(3, 0, 2, 1, 4).float()        # (3,B,H,T,d)
        qt, kt, vt = (apply_paths(parts[i].reshape(B * H, T, d).contiguous(), R, C, chunk)
                      for i in range(3))
        o = attn_general_fwd(qt, kt, vt, softmax_scale, None, None, mask)
        heads = (apply_paths(o, R, C, chunk, transpose=True).view(B, H, T, d).permute(0, 2, 1, 3)
                 .reshape(B, T, D).to(out_dtype))
    else:
        raise ValueError("mode must be 'causal' or 'inert'")
    if not geometry:
        return heads
    geo_dtype = geo_dtype or out_dtype
    P = compose_paths(R, C, chunk, geo_dtype).view(B, H, T, d, d)
    return heads, P, total.view(B, H, d, d).to(geo_dtype)


def edge_gelu_split(h: torch.Tensor, split: bool) -> torch.Tensor:
    """GELU(h) (exact erf) of the fp32 hidden layer as the bf16 GEMM operand:
    (rows, cols) = bf16(g), or with ``split`` (rows, 2 cols) = [bf16(g) | bf16(g - bf16(g))]."""
    _need_cuda(h)
    if h.dtype != torch.float32 or h.dim() != 2 or not h.is_contiguous():
        raise ValueError("h must be a contiguous 2-D fp32 tensor")
    rows, cols = h.shape
    out = torch.empty(rows, (2 if split else 1) * cols, dtype=torch.bfloat16, device=h.device)
    _lib.call("hoa_edge_gelu_split", _ptr(h), _ptr(out), rows, cols, 1 if split else 0, _stream(h.device))
    return out


# fixed scale of the fp8 low half: g - bf16(g) is at most 2^-9 |g|, so 2^12 maps |g| up to 56
# onto e4m3's largest value (448, saturating beyond) and keeps remainders down to 2^-18 normal
SPLIT8_LO_SCALE = 4096.0


def edge_gelu_split8(h: torch.Tensor):
    """GELU(h) (exact erf) of the fp32 hidden layer as (bf16(g), e4m3(SPLIT8_LO_SCALE * (g - bf16(g))))
    (hoa_edge_gelu_split8), both (rows, cols)."""
    _need_cuda(h)
    if h.dtype != torch.float32 or h.dim() != 2 or not h.is_contiguous():
        raise ValueError("h must be a contiguous 2-D fp32 tensor")
    rows, cols = h.shape
    hi = torch.empty(rows, cols, dtype=torch.bfloat16, device=h.device)
    lo = torch.empty(rows, cols, dtype=torch.float8_e4m3fn, device=h.device)
    _lib.call("hoa_edge_gelu_split8", _ptr(h), _ptr(hi), _ptr(lo), rows, cols, SPLIT8_LO_SCALE,
              _stream(h.device))
    return hi, lo


_GEMM_WS = {}
_GEMM_WS_BYTES = 32 << 20


def _gemm_ws(dev):
    ws = _GEMM_WS.get(dev)
    if ws is None:
        ws = _GEMM_WS[dev] = torch.empty(_GEMM_WS_BYTES, dtype=torch.uint8, device=dev)
    return ws


def edge_gemm_fp8_acc(lo: torch.Tensor, w: torch.Tensor, out: torch.Tensor, alpha: float) -> torch.Tensor:
    """out (M,N) fp32 += alpha * lo (M,K) e4m3 @ w (N,K) e4m3 ^T (hoa_edge_gemm_fp8_acc), in place."""
    _need_cuda(lo, w, out)
    if lo.dtype != torch.float8_e4m3fn or w.dtype != torch.float8_e4m3fn or out.dtype != torch.float32:
        raise ValueError("lo and w must be float8_e4m3fn, out float32")
    lo = _contig(lo, "lo")
    w = _contig(w, "w")
    out = _contig(out, "out")
    M, K = lo.shape
    N = w.shape[0]
    if w.shape[1] != K or out.shape != (M, N):
        raise ValueError(f"shapes: lo {tuple(lo.shape)}, w {tuple(w.shape)}, out {tuple(out.shape)}")
    dev = lo.device
    _lib.call("hoa_edge_gemm_fp8_acc", _ptr(lo), _ptr(w), _ptr(out), float(alpha), M, N, K, _ptr(_gemm_ws(dev)),
              _GEMM_WS_BYTES, _stream(dev))
    return out


def edge_gemm(hidden: torch.Tensor, wt: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """hidden (M,K) bf16 @ wt (K,N) bf16 + bias (N,) fp32 -> (M,N) fp32 (hoa_edge_gemm: one
    cuBLASLt GEMM with the bias in its epilogue)."""
    _need_cuda(hidden, wt)
    if hidden.dtype != torch.bfloat16 or wt.dtype != torch.bfloat16:
        raise NotImplementedError("hoa_edge_gemm takes bf16 operands")
    hidden = _contig(hidden, "hidden")
    wt = _contig(wt, "wt")
    M, K = hidden.shape
    if wt.shape[0] != K:
        raise ValueError(f"wt must be (K={K}, N), got {tuple(wt.shape)}")
    N = wt.shape[1]
    if bias is not None:
        if bias.dtype != torch.float32 or bias.numel() != N:
            raise ValueError("bias must be float32 with N elements")
        bias = bias.contiguous()
    dev = hidden.device
    ws = _GEMM_WS.get(dev)
    if ws is None:
        ws = _GEMM_WS[dev] = torch.empty(_GEMM_WS_BYTES, dtype=torch.uint8, device=dev)
    out = torch.empty(M, N, dtype=torch.float32, device=dev)
    try:
        _lib.call("hoa_edge_gemm", _ptr(hidden), _ptr(wt), _ptr(bias), _ptr(out), M, N, K, _ptr(ws),
                  _GEMM_WS_BYTES, _stream(dev))
    except _lib.HoaError as e:
        if e.status != _lib.HOA_ERR_UNSUPPORTED:
            raise
        # no cuBLASLt algorithm for this shape (e.g. rows not 16-byte aligned): torch's GEMM
        torch.mm(hidden, wt, out_dtype=torch.float32, out=out)
        if bias is not None:
            out += bias
    return out


def selftest_wait(max_cycles: int, device=None) -> Tuple[int, int, int, int]:
    """Diagnostic of the bounded device-side waits (hoa_selftest_wait): returns
    (status of the bounded wait, 1 if the second waiter left on the abort flag,
    the second waiter's wait in units of 1024 cycles, 1 if both waits gave up)."""
    dev = torch.device(device if device is not None else "cuda")
    out = torch.zeros(4, dtype=torch.int32, device=dev)
    _lib.call("hoa_selftest_wait", _ptr(out), int(max_cycles), _stream(dev))
    r = out.cpu().tolist()
    return r[0], r[1], r[2], r[3]


def uses_tensor_cores(hat_dtype: torch.dtype, d: int) -> bool:
    """Same rule as the library: bf16 hats with d % 8 == 0 and d <= 128."""
    return hat_dtype == torch.bfloat16 and d % 8 == 0 and d <= 128


def core_stages(a_all, qkv, n_heads, edge_scale, softmax_scale, out_dtype, hat_dtype, chunk,
                a_bias=None, gen_layout="packed"):
    """The core region as separate stage calls (same kernels as core_forward)."""
    B, T, threeD = qkv.shape
    H = n_heads
    d = threeD // 3 // H
    R, U, M = link_local(a_all, qkv, H, edge_scale, chunk, a_bias, gen_layout)
    C, _ = carry_scan(M)
    tc = uses_tensor_cores(hat_dtype, d)
    qh, kh, vh = carry_apply(U, C, chunk, hat_dtype, v_transposed=tc)
    o = attn_tc_fwd(qh, kh, vh, softmax_scale) if tc else attn_fwd(qh, kh, vh, softmax_scale)
    return out_transport(o, R, C, chunk, B, H, out_dtype)
