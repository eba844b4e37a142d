"""Host logic of the sequence-sharded path on CPU ranks (gloo, world_size 2 and 3).

Each rank runs in its own process; the results are compared with a
single-process computation of the same quantities in float64.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from holonomyawareattention_b200 import seqshard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exclusive_products(M):            # (BH, N, d, d) -> exclusive products, float64 on CPU
    BH, N, d, _ = M.shape
    out = torch.empty_like(M)
    acc = torch.eye(d, dtype=M.dtype).expand(BH, d, d).clone()
    for k in range(N):
        out[:, k] = acc
        acc = M[:, k] @ acc
    return out


def _by_value(*ts):
    """numpy copies for the result queue: a tensor put on a torch multiprocessing queue is
    shared through a file descriptor of the sending process, which may have exited by the
    time the parent reads it."""
    return tuple(t.detach().cpu().numpy().copy() for t in ts)


def _received(vals):
    return [torch.from_numpy(v) for v in vals]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        B, T, D, BH, d = 2, 12, 5, 3, 4
        x = torch.randn(B, T, D, generator=g, dtype=torch.float64)
        totals = torch.randn(world, BH, d, d, generator=g, dtype=torch.float64)
        kh = torch.randn(BH, T, d, generator=g, dtype=torch.float64)
        s0, s1 = seqshard.shard_range(T, world, rank)
        S = s1 - s0
        nxt = seqshard.next_shard_first_token(x[:, s0:s1], None)
        carry = seqshard.shard_carry_in(totals[rank], None, compose=_exclusive_products)
        k_all, v_all = seqshard.gather_kv(kh[:, s0:s1], kh[:, s0:s1], S, False, None)
        from holonomyawareattention_b200 import ops
        vt = torch.zeros(BH, d, ops.vt_stride(S), dtype=kh.dtype)
        vt[:, :, :S] = kh[:, s0:s1].transpose(1, 2)
        _, vt_all = seqshard.gather_kv(kh[:, s0:s1], vt, S, True, None)
        q.put((rank, *_by_value(nxt, carry, k_all, v_all, vt_all)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sequence_shard_collectives(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, *vals = q.get(timeout=120)
        res[r] = _received(vals)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(0)
    B, T, D, BH, d = 2, 12, 5, 3, 4
    x = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    totals = torch.randn(world, BH, d, d, generator=g, dtype=torch.float64)
    kh = torch.randn(BH, T, d, generator=g, dtype=torch.float64)
    excl = _exclusive_products(totals.permute(1, 0, 2, 3))
    S = T // world
    for r in range(world):
        nxt, carry, k_all, v_all, vt_all = res[r]
        # the token after the shard, wrapping to the first token (roll(x, -1) at the boundary)
        assert torch.equal(nxt, x[:, ((r + 1) * S) % T:((r + 1) * S) % T + 1])
        assert torch.allclose(carry, excl[:, r])
        assert torch.equal(k_all, kh) and torch.equal(v_all, kh)
        assert torch.equal(vt_all[:, :, :T], kh.transpose(1, 2))


def test_shard_range():
    assert seqshard.shard_range(65536, 8, 3) == (24576, 32768)
    with pytest.raises(ValueError):
        seqshard.shard_range(100, 8, 0)


def test_shard_unshard_round_trip():
    x = torch.arange(2 * 24 * 3, dtype=torch.float64).view(2, 24, 3)
    for layout in ("contiguous", "zigzag"):
        for world in (1, 2, 3):
            parts = [seqshard.shard_sequence(x, world, r, layout) for r in range(world)]
            assert all(p.shape == (2, 24 // world, 3) for p in parts)
            assert torch.equal(seqshard.unshard_sequence(parts, layout), x)
    # zig-zag pairs an early and a late segment on every rank
    assert seqshard.segments_of("zigzag", 3, 0) == ([0, 5], 6)
    assert seqshard.segments_of("zigzag", 3, 2) == ([2, 3], 6)


def _seg_worker(rank, world, port, q, layout):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(1)
        B, T, D, BH, d = 2, 24, 5, 3, 4
        segs, n = seqshard.segments_of(layout, world, rank)
        S = T // n
        x = torch.randn(B, T, D, generator=g, dtype=torch.float64)
        totals = torch.randn(n, BH, d, d, generator=g, dtype=torch.float64)
        kh = torch.randn(BH, T, d, generator=g, dtype=torch.float64)
        x_local = seqshard.shard_sequence(x, world, rank, layout)
        halos = seqshard.segment_halos(x_local, layout, None)
        carries = seqshard.segment_carries(torch.stack([totals[s] for s in segs]), layout, None,
                                           compose=_exclusive_products)
        k_loc = torch.stack([kh[:, s * S:(s + 1) * S] for s in segs])          # (nl, BH, S, d)
        v_loc = torch.stack([kh[:, s * S:(s + 1) * S].transpose(1, 2) for s in segs])
        k_all, v_all = seqshard.gather_kv_segments(k_loc, k_loc, S, False, layout, None)
        _, vt_all = seqshard.gather_kv_segments(k_loc, v_loc, S, True, layout, None)
        q.put((rank, *_by_value(halos, carries, k_all, v_all, vt_all)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
@pytest.mark.parametrize("world", [2, 3])
def test_segment_collectives(world, layout):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_seg_worker, args=(r, world, port, q, layout)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, *vals = q.get(timeout=120)
        res[r] = _received(vals)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(1)
    B, T, D, BH, d = 2, 24, 5, 3, 4
    _, n = seqshard.segments_of(layout, world, 0)
    S = T // n
    x = torch.randn(B, T, D, generator=g, dtype=torch.float64)
    totals = torch.randn(n, BH, d, d, generator=g, dtype=torch.float64)
    kh = torch.randn(BH, T, d, generator=g, dtype=torch.float64)
    excl = _exclusive_products(totals.permute(1, 0, 2, 3))                    # (BH, n, d, d)
    from holonomyawareattention_b200 import ops
    for r in range(world):
        halos, carries, k_all, v_all, vt_all = res[r]
        segs, _ = seqshard.segments_of(layout, world, r)
        for i, s in enumerate(segs):
            nxt = ((s + 1) % n) * S
            assert torch.equal(halos[i], x[:, nxt:nxt + 1])
            assert torch.allclose(carries[i], excl[:, s])
        assert torch.equal(k_all, kh) and torch.equal(v_all, kh)
        assert vt_all.shape == (BH, d, ops.vt_stride(T))
        assert torch.equal(vt_all[:, :, :T], kh.transpose(1, 2))
