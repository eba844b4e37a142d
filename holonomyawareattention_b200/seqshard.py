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

from typing import Callable, List, Optional, Tuple

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


def segments_of(layout: str, world: int, rank: int) -> Tuple[List[int], int]:
    """(this rank's segments in the order its local tensor holds them, number of segments).

    "contiguous": N segments, rank r holds segment r.
    "zigzag": 2N segments, rank r holds segments r and 2N-1-r, so that every rank
    does the same causal attention work (early and late queries paired)."""
    if layout == "contiguous":
        return [rank], world
    if layout == "zigzag":
        return [rank, 2 * world - 1 - rank], 2 * world
    raise ValueError("layout must be 'contiguous' or 'zigzag'")


def shard_sequence(x: torch.Tensor, world: int, rank: int, layout: str = "contiguous") -> torch.Tensor:
    """This rank's local tensor (B, n_local * S, D) of a whole sequence x (B, T, D)."""
    segs, n = segments_of(layout, world, rank)
    T = x.shape[1]
    if T % n != 0:
        raise ValueError(f"sequence length {T} does not split into {n} equal segments")
    S = T // n
    return torch.cat([x[:, s * S:(s + 1) * S] for s in segs], dim=1)


def unshard_sequence(parts: List[torch.Tensor], layout: str = "contiguous") -> torch.Tensor:
    """Whole-sequence tensor from every rank's local tensor (rank order)."""
    world = len(parts)
    _, n = segments_of(layout, world, 0)
    S = parts[0].shape[1] // (n // world)
    by_seg = {}
    for r, part in enumerate(parts):
        segs, _ = segments_of(layout, world, r)
        for i, sg in enumerate(segs):
            by_seg[sg] = part[:, i * S:(i + 1) * S]
    return torch.cat([by_seg[sg] for sg in range(n)], dim=1)


def _gather_segments(t: torch.Tensor, layout: str, group) -> torch.Tensor:
    """All ranks' per-segment slices stacked in segment order.  ``t`` is
    (n_local, ...) for this rank; returns (n_segments, ...)."""
    world, _ = _world(group)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous(), group=group)
    _, n = segments_of(layout, world, 0)
    out = [None] * n
    for r, part in enumerate(parts):
        segs, _ = segments_of(layout, world, r)
        for i, sg in enumerate(segs):
            out[sg] = part[i]
    return torch.stack(out, dim=0)


def segment_halos(x_local: torch.Tensor, layout: str, group=None) -> torch.Tensor:
    """(n_local, B, 1, D): for each local segment the token that follows it (the
    next segment's first token; the last segment takes the sequence's first
    token, as the reference's roll wraps)."""
    world, rank = _world(group)
    segs, n = segments_of(layout, world, rank)
    B, L, D = x_local.shape
    S = L // len(segs)
    firsts = torch.stack([x_local[:, i * S:i * S + 1] for i in range(len(segs))], dim=0)
    table = _gather_segments(firsts, layout, group)                 # (n, B, 1, D)
    return torch.stack([table[(sg + 1) % n] for sg in segs], dim=0)


def segment_carries(total_local: torch.Tensor, layout: str, group=None,
                    compose: Optional[Callable[[torch.Tensor], torch.Tensor]] = None) -> torch.Tensor:
    """P at the start of each local segment, (n_local, BH, d, d) fp32.

    ``total_local`` (n_local, BH, d, d): each local segment's product through its
    boundary edge.  The totals of all segments are gathered in sequence order
    and their exclusive products taken (by default with the carry-scan kernel)."""
    world, rank = _world(group)
    segs, n = segments_of(layout, world, rank)
    table = _gather_segments(total_local, layout, group)            # (n, BH, d, d)
    C = (compose or _carry_scan_compose)(table.transpose(0, 1).contiguous())   # (BH, n, d, d)
    return torch.stack([C[:, sg] for sg in segs], dim=0).contiguous()


def gather_kv_segments(kh: torch.Tensor, vh: torch.Tensor, S: int, v_transposed: bool, layout: str,
                       group=None):
    """All segments' k^ (BH, T, d) and v^ ((BH, T, d), or transposed (BH, d, vt_stride(T))),
    from this rank's local segments kh (n_local, BH, S, d) and vh ((n_local, BH, S, d) or
    (n_local, BH, d, S))."""
    world, _ = _world(group)
    _, n = segments_of(layout, world, 0)
    T = n * S
    k_tab = _gather_segments(kh, layout, group)                     # (n, BH, S, d)
    kh_all = torch.cat(list(k_tab), dim=1)
    v_tab = _gather_segments(vh, layout, group)
    if not v_transposed:
        return kh_all, torch.cat(list(v_tab), dim=1)
    BH, d = kh.shape[1], kh.shape[3]
    vt_all = torch.zeros(BH, d, ops.vt_stride(T), dtype=vh.dtype, device=vh.device)
    vt_all[:, :, :T] = torch.cat(list(v_tab), dim=2)
    return kh_all, vt_all


def sequence_sharded_forward(mod, x_shard: torch.Tensor, group=None,
                             layout: str = "contiguous") -> torch.Tensor:
    """y for this rank's part of the sequence: the causal forward of
    PathOrderedGeometricMHA (attn_mask = tril(T)) over the whole sequence,
    computed with the sequence split across the ranks of ``group``.

    ``x_shard`` is this rank's local tensor in ``layout`` (see shard_sequence);
    the result has the same layout.  The local segments run through the link,
    carry and transport kernels as extra batch rows; attention runs once per
    local segment, at that segment's query offset."""
    if mod.mode != "causal" or mod.link_mode != "interaction":
        raise NotImplementedError("sequence sharding serves mode='causal', link_mode='interaction'")
    if not x_shard.is_cuda:
        raise NotImplementedError("the B200 kernels need CUDA tensors (there is no CPU path)")
    world, rank = _world(group)
    segs, n = segments_of(layout, world, rank)
    nl = len(segs)
    B, L, D = x_shard.shape
    if L % nl != 0:
        raise ValueError("the local tensor does not hold whole segments")
    S = L // nl
    H, d = mod.h, mod.d
    dtype = x_shard.dtype
    halos = segment_halos(x_shard, layout, group)                   # (nl, B, 1, D)
    # local segments as batch rows: row i*B + b is segment segs[i] of batch row b
    xs = x_shard.view(B, nl, S, D).transpose(0, 1).reshape(nl * B, S, D)
    x_next = halos.reshape(nl * B, 1, D)
    qkv = mod.qkv(xs).contiguous()
    a, a_bias, gen_layout = mod._edge_generators_nobias(xs, x_next, seq_len=n * S)
    chunk = mod.chunk or ops.plan_chunk(nl * B, H, S, d, x_shard.device)
    R, U, M = ops.link_local(a.contiguous(), qkv, H, mod.edge_scale, chunk, a_bias, gen_layout)
    del a
    _, total = ops.carry_scan(M, want_total=True)                   # (nl*B*H, d, d)
    BH = B * H
    carry_in = segment_carries(total.view(nl, BH, d, d), layout, group).view(nl * BH, d, d)
    C, _ = ops.carry_scan(M, carry_in=carry_in)
    tc = ops.uses_tensor_cores(dtype, d)
    qh, kh, vh = ops.carry_apply(U, C, chunk, dtype, v_transposed=tc)
    del U
    kh_seg = kh.view(nl, BH, S, d)
    vh_seg = vh[:, :, :S].reshape(nl, BH, d, S) if tc else vh.view(nl, BH, S, d)
    kh_all, vh_all = gather_kv_segments(kh_seg, vh_seg, S, tc, layout, group)
    o = torch.empty(nl * BH, S, d, dtype=torch.float32, device=x_shard.device)
    for i, sg in enumerate(segs):
        q_i = qh[i * BH:(i + 1) * BH]
        if tc:
            o[i * BH:(i + 1) * BH] = ops.attn_tc_fwd(q_i, kh_all, vh_all, mod.scale, q_offset=sg * S)
        else:
            o[i * BH:(i + 1) * BH] = ops.attn_fwd(q_i, kh_all, vh_all, mod.scale, q_offset=sg * S)
    out = ops.out_transport(o, R, C, chunk, nl * B, H, dtype)       # (nl*B, S, D)
    y = mod.out(out)
    return y.view(nl, B, S, D).transpose(0, 1).reshape(B, L, D)
