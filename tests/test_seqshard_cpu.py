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
        q.put((rank, nxt, carry, k_all, v_all, vt_all))
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
        res[r] = vals
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
