"""Sequence-sharded causal forward for long sequences (one process per GPU).

Each rank holds a contiguous shard of one long sequence (positions
[r*S, (r+1)*S)).  The reference is single-device; this is the multi-GPU form
of the same computation (core/attention_fast_chunked.py:63-177):

1. halo: the token after the shard (the next shard's first token; the last
   shard takes the sequence's first token, as the reference's roll wraps) so
   that the shard's last edge generator can be formed;
2. local: link rotations and chunked local products on the shard
   (hoa_link_local), joined into the shard's total product (hoa_carry_scan);
3. carry: all-gather of the per-shard totals (B*H, d, d) and an exclusive
   product across shards (the carry-scan kernel again) gives P at the start
   of this shard; the chunk carries are recomputed from it;
4. attention: q^ of the shard against k^/v^ gathered from all shards (causal
   with the shard's query offset; the later shards use more of it);
5. inverse transport and the out projection on the shard.

The collectives go through torch.distributed (NCCL over NVLink for CUDA
tensors).  The pieces that only move data — the halo, the carry exchange, the
K/V gather — are separate functions so that they can be exercised on CPU
ranks (gloo).
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import ops


def shard_range(T: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous shard [start, stop) of a length-T sequence; T must divide evenly."""
    if T % world != 0:
        raise ValueError(f"sequence length {T} does not split into {world} equal shards")
    S = T // world
    return rank * S, (rank + 1) * S


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def next_shard_first_token(x_shard: torch.Tensor, group=None) -> torch.Tensor:
    """(B, 1, D): the first token of the next shard; the last shard receives
    shard 0's first token (the closing edge of the ring)."""
    world, rank = _world(group)
    first = x_shard[:, :1].contiguous()
    parts = [torch.empty_like(first) for _ in range(world)]
    dist.all_gather(parts, first, group=group)
    return parts[(rank + 1) % world]


def _carry_scan_compose(M: torch.Tensor) -> torch.Tensor:
    C, _ = ops.carry_scan(M.contiguous())
    return C


def shard_carry_in(total_local: torch.Tensor, group=None,
                   compose: Optional[Callable[[torch.Tensor], torch.Tensor]] = None) -> torch.Tensor:
    """P at the start of this shard, (B*H, d, d) fp32.

    Gathers every shard's total product M_r (through the boundary edge) and
    takes the exclusive product M_{r-1} ... M_0.  ``compose`` maps the stacked
    totals (B*H, N, d, d) to their exclusive products; by default the
    carry-scan kernel (fp32)."""
    world, rank = _world(group)
    total_local = total_local.contiguous()
    parts = [torch.empty_like(total_local) for _ in range(world)]
    dist.all_gather(parts, total_local, group=group)
    stacked = torch.stack(parts, dim=1)                       # (BH, N, d, d)
    C = (compose or _carry_scan_compose)(stacked)
    return C[:, rank].contiguous()


def gather_kv(kh: torch.Tensor, vh: torch.Tensor, S: int, v_transposed: bool, group=None):
    """All shards' k^ (BH, T, d) and v^: (BH, T, d), or transposed (BH, d, vt_stride(T))."""
    world, _ = _world(group)
    BH, _, d = kh.shape
    T = S * world
    parts = [torch.empty_like(kh) for _ in range(world)]
    dist.all_gather(parts, kh.contiguous(), group=group)
    kh_all = torch.cat(parts, dim=1)
    if not v_transposed:
        vparts = [torch.empty_like(vh) for _ in range(world)]
        dist.all_gather(vparts, vh.contiguous(), group=group)
        return kh_all, torch.cat(vparts, dim=1)
    v_local = vh[:, :, :S].contiguous()
    vparts = [torch.empty_like(v_local) for _ in range(world)]
    dist.all_gather(vparts, v_local, group=group)
    vt_all = torch.zeros(BH, d, ops.vt_stride(T), dtype=vh.dtype, device=vh.device)
    vt_all[:, :, :T] = torch.cat(vparts, dim=2)
    return kh_all, vt_all


def sequence_sharded_forward(mod, x_shard: torch.Tensor, group=None) -> torch.Tensor:
    """y for this rank's shard of the sequence: the causal forward of
    PathOrderedGeometricMHA (attn_mask = tril(T)) over the whole sequence,
    computed with the sequence split across the ranks of ``group``."""
    if mod.mode != "causal" or mod.link_mode != "interaction":
        raise NotImplementedError("sequence sharding serves mode='causal', link_mode='interaction'")
    if not x_shard.is_cuda:
        raise NotImplementedError("the B200 kernels need CUDA tensors (there is no CPU path)")
    world, rank = _world(group)
    B, S, D = x_shard.shape
    H, d = mod.h, mod.d
    dtype = x_shard.dtype
    x_next = next_shard_first_token(x_shard, group)
    qkv = mod.qkv(x_shard).contiguous()
    a, a_bias = mod._edge_generators_nobias(x_shard, x_next, seq_len=world * S)
    chunk = mod.chunk or ops.plan_chunk(B, H, S, d, x_shard.device)
    R, U, M = ops.link_local(a.contiguous(), qkv, H, mod.edge_scale, chunk, a_bias)
    del a
    _, total = ops.carry_scan(M, want_total=True)
    carry_in = shard_carry_in(total, group)
    C, _ = ops.carry_scan(M, carry_in=carry_in)
    tc = ops.uses_tensor_cores(dtype, d)
    qh, kh, vh = ops.carry_apply(U, C, chunk, dtype, v_transposed=tc)
    del U
    kh_all, vh_all = gather_kv(kh, vh, S, tc, group)
    if tc:
        o = ops.attn_tc_fwd(qh, kh_all, vh_all, mod.scale, q_offset=rank * S)
    else:
        o = ops.attn_fwd(qh, kh_all, vh_all, mod.scale, q_offset=rank * S)
    out = ops.out_transport(o, R, C, chunk, B, H, dtype)
    return mod.out(out)
