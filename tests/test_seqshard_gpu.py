"""Sequence-sharded forward on GPUs: query-offset attention, and the sharded
forward against the unsharded one (1 rank in-process; 2 ranks when 2 GPUs)."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from holonomyawareattention_b200 import PathOrderedGeometricMHA, ops, seqshard
from oracle import torch_ref
from oracle.holonomy_oracle import rel_l2
from oracle.seeded import seeded_case

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("tc", [True, False])
def test_attention_query_offset_shards(tc):
    """Attention of query shards (with offsets) against all keys == whole attention."""
    torch.manual_seed(5)
    BH, T, d, S = 3, 300, 96, 100
    dt = torch.bfloat16 if tc else torch.float32
    qh, kh, vh = (torch.randn(BH, T, d, device=DEV).to(dt) for _ in range(3))
    scale = 1 / math.sqrt(d)
    if tc:
        vt = torch.zeros(BH, d, ops.vt_stride(T), dtype=dt, device=DEV)
        vt[:, :, :T] = vh.transpose(1, 2)
        full = ops.attn_tc_fwd(qh, kh, vt, scale)
        parts = [ops.attn_tc_fwd(qh[:, s:s + S].contiguous(), kh, vt, scale, q_offset=s)
                 for s in range(0, T, S)]
    else:
        full = ops.attn_fwd(qh, kh, vh, scale)
        parts = [ops.attn_fwd(qh[:, s:s + S].contiguous(), kh, vh, scale, q_offset=s)
                 for s in range(0, T, S)]
    assert rel_l2(torch.cat(parts, 1).cpu().numpy(), full.cpu().numpy()) < 1e-6


def _module(D, H, dtype, seed=0):
    sd, _ = seeded_case(D, H, seed=seed, B=1, L=2)
    m = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=0.05)
    m.load_state_dict(sd)
    return m.to(DEV, dtype).eval()


@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
def test_single_rank_sharded_equals_forward(layout):
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ["MASTER_PORT"] = str(_port())
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device(DEV, 0))
    try:
        D, H, T = 384, 4, 1000
        m = _module(D, H, torch.bfloat16)
        x = torch.randn(1, T, D, device=DEV).to(torch.bfloat16)
        mask = torch.tril(torch.ones(T, T, dtype=torch.bool, device=DEV))
        with torch.no_grad():
            y_ref, _ = m(x, attn_mask=mask)
            x_local = seqshard.shard_sequence(x, 1, 0, layout)
            y = seqshard.unshard_sequence([seqshard.sequence_sharded_forward(m, x_local, layout=layout)],
                                          layout)
        # contiguous: the same computation; zig-zag: two segments with their own
        # chunking and a carry between them (association and bf16 rounding differ)
        tol = 1e-6 if layout == "contiguous" else 5e-3
        assert rel_l2(y.float().cpu().numpy(), y_ref.float().cpu().numpy()) < tol
    finally:
        dist.destroy_process_group()


def _two_rank_worker(rank, port, T, D, H, layout, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=torch.device("cuda", rank))
    try:
        m = _module(D, H, torch.bfloat16).to(f"cuda:{rank}")
        g = torch.Generator().manual_seed(11)
        x = torch.randn(1, T, D, generator=g).to(f"cuda:{rank}", torch.bfloat16)
        x_local = seqshard.shard_sequence(x, 2, rank, layout).contiguous()
        del x
        with torch.no_grad():
            y = seqshard.sequence_sharded_forward(m, x_local, layout=layout)
        torch.save(y.float().cpu(), os.path.join(out_dir, f"y{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _run_two_ranks(T, D, H, layout, tmp_path):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, port, T, D, H, layout, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=900)
        assert p.exitcode == 0
    ys = [torch.load(os.path.join(tmp_path, f"y{r}.pt")) for r in range(2)]
    return seqshard.unshard_sequence(ys, layout).numpy()


def _oracle(T, D, H, head_group=None):
    """The fp32 torch restatement of the reference on the bf16-rounded weights and input
    that the sharded bf16 module sees."""
    sd, _ = seeded_case(D, H, seed=0, B=1, L=2, bf16_round=True)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(1, T, D, generator=g).to(torch.bfloat16).float()
    return torch_ref.module_forward(sd, x.to(DEV), H, 0.05, torch.float32, batch_slice=1,
                                    head_group=head_group).cpu().numpy()


def _errs(y, ref):
    T = y.shape[1]
    return rel_l2(y, ref), rel_l2(y[:, 3 * T // 4:], ref[:, 3 * T // 4:])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
def test_two_rank_sharded_vs_oracle_and_unsharded(layout, tmp_path):
    D, H, T = 384, 4, 4096
    y_sh = _run_two_ranks(T, D, H, layout, tmp_path)
    err, err_q = _errs(y_sh, _oracle(T, D, H))
    print(f"2 ranks, {layout}, T={T}: rel-L2 vs oracle {err:.3e}, last quarter {err_q:.3e}")
    assert err <= 2e-2 and err_q <= 2e-2
    m = _module(D, H, torch.bfloat16)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(1, T, D, generator=g).to(DEV, torch.bfloat16)
    mask = torch.tril(torch.ones(T, T, dtype=torch.bool, device=DEV))
    with torch.no_grad():
        y_ref, _ = m(x, attn_mask=mask)
    # same kernels; only the association of the rotation products and the
    # bf16 rounding of q^/k^/v^ that follows can differ
    assert rel_l2(y_sh, y_ref.float().cpu().numpy()) < 5e-3


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_sharded_config5_vs_oracle(tmp_path):
    """configs[4] (T = 65536, d_model 1536, H 16, bf16) sequence-sharded over 2 ranks in the
    zig-zag layout (four segments joined by the cross-rank boundary-rotation scan) against the
    fp32 torch restatement of the reference, two heads at a time."""
    D, H, T = 1536, 16, 65536
    y_sh = _run_two_ranks(T, D, H, "zigzag", tmp_path)
    err, err_q = _errs(y_sh, _oracle(T, D, H, head_group=2))
    print(f"configs[4], 2 ranks, zigzag: rel-L2 vs oracle {err:.3e}, last quarter {err_q:.3e}")
    assert err <= 2e-2 and err_q <= 2e-2
