#!/usr/bin/env python
"""Benchmark of the B200 causal forward of path-ordered geometric attention.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference]

One step = one forward of PathOrderedGeometricMHA (qkv / edge-MLP / out GEMMs
in PyTorch, the core region in libhoa) over a batch of synthetic inputs
already resident in HBM.  Default workload: configs[2] of the baseline
(B=16, T=4096, d_model=1536, H=16, head_dim=96, bf16 activations, fp32
rotations, edge_scale 0.05), the configuration the metric is quoted on.
With N GPUs every rank runs its own batch (batch sharding, no data-path
collective: weak scaling); rank 0 prints one JSON line.

`--impl reference` times the reference forward on the host's CPU cores (its
torch restatement in oracle/torch_ref.py, float32, all host threads; the
reference's own Python cannot travel to the GPU box) on a bounded sample of
the same workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd tokens/s/GPU at T=4096 H=16 d=96 bf16; % roofline; 1/2/4/8-GPU scaling"
CONFIGS = {
    # name: (B per GPU, T, d_model, H, dtype)
    "c2": (64, 512, 192, 4, "bf16"),
    "c2f32": (64, 512, 192, 4, "fp32"),
    "c3": (16, 4096, 1536, 16, "bf16"),
    "c4slice": (16, 2048, 2880, 24, "bf16"),
    # small case of the c3 kernels for ncu captures (inputs still larger than L2)
    "c3prof": (1, 512, 1536, 16, "bf16"),
    # one batch row of c3 (same T, so the same attention shape), ~5 GB on the device:
    # the case the full ncu captures run on
    "c3b1": (1, 4096, 1536, 16, "bf16"),
    # one batch row of configs[3] (head dim 120, the SIMT link kernel): the case its ncu
    # captures run on
    "c4b1": (1, 2048, 2880, 24, "bf16"),
    # one sequence of T=65536 split across the ranks (sequence sharding)
    "c5": (1, 65536, 1536, 16, "bf16"),
}
SEQ_SHARDED = {"c5"}
EDGE_SCALE = 0.05
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    except Exception:
        return dict(PEAKS_FALLBACK)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: str):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def _rows(self):
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [s.strip() for s in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
        except OSError:
            pass
        return rows

    def start(self):
        """Starts nvidia-smi (50 ms period) and returns once it has written its first
        sample (at most 3 s), so that a short timed region that begins right after
        still falls inside the sampling."""
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.n0 = 0
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while not self._rows() and time.time() - t0 < 3.0 and self.proc.poll() is None:
            time.sleep(0.01)

    def region_start(self):
        """Marks the start of the timed region: samples written before it are dropped."""
        if self.proc is not None:
            self.n0 = len(self._rows())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = self._rows()[self.n0:]
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "samples": len(rows), "reasons": reasons}


def physical_gpu_index(local_rank: int) -> str:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [s.strip() for s in vis.split(",") if s.strip()]
        if local_rank < len(ids):
            return ids[local_rank]
    return str(local_rank)


# ---------------------------------------------------------------------------
# CPU baseline: the reference forward restated in torch (oracle/torch_ref.py,
# the same torch operations as core/attention_fast_chunked.py, bit-identical
# output; the reference's own Python cannot travel to the GPU box), fp32, on all
# host cores
# ---------------------------------------------------------------------------
def cpu_threads():
    import torch
    return torch.get_num_threads()


def cpu_sample_setup(D, H):
    """(weights, input) of the CPU sample: seeded default init and x ~ N(0,1), both
    bf16-rounded (the values of the bf16 workload), as fp32 CPU tensors."""
    import torch
    from oracle.seeded import seeded_state_dict
    torch.set_num_threads(os.cpu_count() or 1)
    sd = seeded_state_dict(D, H, 0)
    return {k: v.to(torch.bfloat16).float() for k, v in sd.items() if not k.startswith(("gq", "gk"))}


def cpu_sample_forward(sd, D, H, T_sample):
    """Seconds for one reference forward of one sequence of T_sample positions."""
    import torch
    from oracle import torch_ref
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, T_sample, D, generator=g).to(torch.bfloat16).float()
    with torch.inference_mode():
        t0 = time.perf_counter()
        torch_ref.module_forward(sd, x, H, EDGE_SCALE, torch.float32)
        return time.perf_counter() - t0


def cpu_sample_len(T):
    """Positions of the CPU sample: one sequence of up to 1024 positions (a few seconds on
    the GPU host's cores at the c3 width; the cost grows with T like the full workload's)."""
    return min(T, 1024)


def cpu_sample_desc(D, H, Ts):
    return (f"1 sequence of T={Ts} at d_model={D}, H={H} per step: the reference forward "
            "(core/attention_fast_chunked.py) restated in torch (oracle/torch_ref.py, output "
            "bit-identical to the reference's on the same CPU), fp32, bf16-valued inputs and "
            "weights")


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    B, T, D, H, dt = CONFIGS[args.config]
    Ts = cpu_sample_len(T)
    p = cpu_sample_setup(D, H)
    times = []
    for i in range(args.warmup + args.steps):
        s = cpu_sample_forward(p, D, H, Ts)
        if i >= args.warmup:
            times.append(s)
    sec = statistics.mean(times)
    val = Ts / sec
    cores = cpu_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_obj(args.config, args.gpus),
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": cpu_sample_desc(D, H, Ts), "sample_tokens_per_step": Ts},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def config_obj(name, n, layout="zigzag"):
    B, T, D, H, dt = CONFIGS[name]
    if name in SEQ_SHARDED:
        segs = f"{2 * n} zig-zag segments" if layout == "zigzag" else f"{n} contiguous shards"
        return {"workload": f"{name}: B={B}, T={T} split into {segs} over {n} ranks, d_model={D}, "
                            f"H={H}, head_dim={D // H}, {dt} activations, fp32 rotations, "
                            f"edge_scale {EDGE_SCALE}",
                "global_batch": B, "seq_len": T, "d_model": D, "heads": H, "head_dim": D // H,
                "parallelism": f"sequence-sharded x{n}, {layout} (NCCL all-gather of halos, segment "
                               f"totals and K/V)",
                "l2": "inputs and workspace (tens of GB) far exceed the 126 MB L2"}
    return {"workload": f"{name}: B={B}/GPU, T={T}, d_model={D}, H={H}, head_dim={D // H}, {dt} "
                        f"activations, fp32 rotations, edge_scale {EDGE_SCALE}",
            "global_batch": B * n, "seq_len": T, "d_model": D, "heads": H, "head_dim": D // H,
            "parallelism": f"batch-sharded x{n} (no collective)",
            "l2": "inputs and workspace (tens of GB) far exceed the 126 MB L2"}


def cpu_baseline_leg(D, H, T):
    """The cpu_baseline object of our arm: one warm-up and two timed samples."""
    p = cpu_sample_setup(D, H)
    Ts = cpu_sample_len(T)
    cpu_sample_forward(p, D, H, min(Ts, 64))
    sec = min(cpu_sample_forward(p, D, H, Ts) for _ in range(2))
    return {"value": Ts / sec, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
            "sample": cpu_sample_desc(D, H, Ts), "sample_tokens_per_step": Ts}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def measure_tf32_peak(dev):
    """Dense tf32 tensor throughput of this GPU, TFLOP/s: cuBLAS fp32 GEMM 8192^3 with
    tf32 allowed, best of 10 (CUDA events)."""
    import torch
    n = 8192
    a = torch.randn(n, n, device=dev)
    b = torch.randn(n, n, device=dev)
    prev = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("high")
    try:
        for _ in range(3):
            a @ b
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            a @ b
            e1.record()
            torch.cuda.synchronize(dev)
            best = min(best, e0.elapsed_time(e1))
    finally:
        torch.set_float32_matmul_precision(prev)
    del a, b
    return 2.0 * n ** 3 / (best / 1e3) / 1e12


def precision_vs_fp32(mod, x1, mask):
    """rel-L2 of the benchmarked bf16 forward against the fp32 forward of the same weights
    on the same (bf16-valued) input, batch row 0: what the bf16 arithmetic and the generator
    precision cost.  The fp32 path matches the reference within 1e-5 (parity tests)."""
    import copy
    import torch
    # outside inference mode: the copy's weight caches track tensor versions
    with torch.inference_mode(False), torch.no_grad():
        m32 = copy.deepcopy(mod).float()
        y = mod(x1, attn_mask=mask)[0].float()
        y32 = m32(x1.float(), attn_mask=mask)[0]
        del m32
    q = 3 * y.shape[1] // 4

    def rel(a, b):
        return float((a - b).norm() / b.norm())
    return {"against": "fp32 forward of the same weights and input (batch row 0)",
            "rel_l2": rel(y, y32), "rel_l2_last_quarter": rel(y[:, q:], y32[:, q:]),
            "bar": 2e-2}


def generator_precision_label(mod, T, dtype):
    """The edge-MLP precision the timed forward used ("fp32" for a float32
    module; T None: a sequence shard)."""
    import torch
    if dtype == torch.float32:
        return "fp32"
    eff = mod._generator_mode(T)
    return f"{eff} (auto)" if mod.generator_precision == "auto" else eff


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    from holonomyawareattention_b200 import PathOrderedGeometricMHA, ops

    B, T, D, H, dtn = CONFIGS[args.config]
    dtype = torch.bfloat16 if dtn == "bf16" else torch.float32
    d = D // H
    m_dim = d * (d - 1) // 2
    torch.manual_seed(0)
    with torch.device(dev):
        mod = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=EDGE_SCALE)
    mod = mod.to(dtype).eval()
    if args.generator_precision:
        mod.generator_precision = args.generator_precision
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(B, T, D, device=dev, generator=g).to(dtype)
    mask = torch.tril(torch.ones(T, T, dtype=torch.bool, device=dev))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream(dev)
    clocks = ClockSampler(physical_gpu_index(local))
    with torch.inference_mode():
        for _ in range(args.warmup):
            mod(x, attn_mask=mask)
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        clocks.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.region_start()
        e0.record(stream)
        for _ in range(args.steps):
            y, _ = mod(x, attn_mask=mask)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        clk = clocks.stop()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        y_check = y
        value = world * B * T / (ms / 1e3)

        # ---- core region and per-kernel timing (events on the launching stream)
        qkv = mod.qkv(x).contiguous()
        a_all, a_bias, gen_layout = mod._edge_generators_nobias(x)
        chunk = ops.plan_chunk(B, H, T, d, dev)
        torch.cuda.empty_cache()
        tc = ops.uses_tensor_cores(dtype, d)
        names = ["link_local", "carry_scan", "carry_apply", "attn_tc_fwd" if tc else "attn_fwd",
                 "out_transport"]
        stage_ms = {k: [] for k in names}
        core_ms = []
        for it in range(args.warmup + args.steps):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            ev[0].record(stream)
            R, U, M = ops.link_local(a_all, qkv, H, EDGE_SCALE, chunk, a_bias, gen_layout)
            ev[1].record(stream)
            C, _ = ops.carry_scan(M)
            ev[2].record(stream)
            qh, kh, vh = ops.carry_apply(U, C, chunk, dtype, v_transposed=tc)
            ev[3].record(stream)
            o = (ops.attn_tc_fwd(qh, kh, vh, mod.scale) if tc else ops.attn_fwd(qh, kh, vh, mod.scale))
            ev[4].record(stream)
            out = ops.out_transport(o, R, C, chunk, B, H, dtype)
            ev[5].record(stream)
            torch.cuda.synchronize(dev)
            if it >= args.warmup:
                for i, k in enumerate(names):
                    stage_ms[k].append(ev[i].elapsed_time(ev[i + 1]))
                core_ms.append(ev[0].elapsed_time(ev[5]))
            del R, U, M, C, qh, kh, vh, o, out
        stage = {k: statistics.mean(v) for k, v in stage_ms.items()}
        core = statistics.mean(core_ms)
        del qkv, a_all
        torch.cuda.empty_cache()

        # ---- end to end through the public API with host buffers: every step copies
        # x from pinned host memory and y back.  The batch goes through the module in
        # the pieces it uses internally, with the copies on two copy streams, so the
        # host->device copy of piece i+1 and the device->host copy of piece i-1
        # overlap the forward of piece i (a piece's input buffer is refilled only
        # after the previous step's forward of that piece has finished).
        xh = x.cpu().pin_memory()
        yh = torch.empty(B, T, D, dtype=dtype).pin_memory()
        xd = torch.empty_like(x)
        rows_e = max(1, mod.PIECE_TOKENS // T)
        slices = [slice(i, min(B, i + rows_e)) for i in range(0, B, rows_e)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        done = [None] * len(slices)

        def e2e_step():
            for i, sl in enumerate(slices):
                with torch.cuda.stream(s_in):
                    if done[i] is not None:
                        s_in.wait_event(done[i])
                    xd[sl].copy_(xh[sl], non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(s_in)
                stream.wait_event(ready)
                yy, _ = mod(xd[sl], attn_mask=mask)
                done[i] = torch.cuda.Event()
                done[i].record(stream)
                s_out.wait_event(done[i])
                with torch.cuda.stream(s_out):
                    yh[sl].copy_(yy, non_blocking=True)
                    yy.record_stream(s_out)
            stream.wait_stream(s_out)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps)
        if not torch.equal(yh, y_check.cpu()):
            raise RuntimeError("end-to-end output differs from the device-resident forward")
        nbytes = x.numel() * x.element_size()
        # every launch above finished without a device-side wait giving up
        ops.check_status(dev)
        precision = precision_vs_fp32(mod, x[:1], mask) if dtype == torch.bfloat16 else None
    tf32_peak = measure_tf32_peak(dev)

    # our kernels per forward: link, carry scan, carry apply, attention, inverse
    # transport, once per batch piece of the module's forward
    rows = max(1, mod.PIECE_TOKENS // T)
    pieces = -(-B // rows)

    # ---- roofline of the dominant kernel (link_local) and the BASELINE formula
    peaks = load_peaks()
    s_x = 2 if dtype == torch.bfloat16 else 4
    n_pos = B * H * T
    link_bytes = n_pos * (m_dim * 4 + 3 * d * s_x + d * d * 4 + 3 * d * 4)   # a, q,k,v in; R, U out
    core_bytes = n_pos * (m_dim * 4 + 4 * d * s_x)                 # + o
    f_attn = 4.0 * B * H * d * T * (T + 1) / 2
    # F_rot: 3 d^3 products per position for the expm (A^2, A^4, the T8 product) and one for
    # the composition, each fp32-accurate (2 d^3 flops)
    f_rot = n_pos * 4 * 2.0 * d ** 3
    link_s = stage["link_local"] / 1e3
    attn_s = stage[names[3]] / 1e3
    hbm = peaks["hbm_gbs"]
    bf16_burst = peaks["bf16_tflops"]
    bf16_peak = peaks.get("bf16_tflops_sustained", bf16_burst)
    baseline_roof_s = max(f_attn / (bf16_peak * 1e12), core_bytes / (hbm * 1e9))
    sm_mhz = clk.get("sm_mhz") or 1965.0
    tc_link = d in (32, 48, 64, 96)
    if tc_link:
        # fp32-accurate products as 3xTF32: the bound is the tf32 tensor peak / 3
        fp32acc_peak = tf32_peak / 3
        peak_source = (f"tf32 dense peak measured in this run ({tf32_peak:.1f} TFLOP/s: cuBLAS TF32 "
                       "GEMM 8192^3, best of 10) / 3, the 3 tf32 passes of a 3xTF32 product")
        kname = "link_tc_kernel (hoa_link_local: kernels 1+2, tcgen05 3xTF32)"
    else:
        fp32acc_peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12
        peak_source = (f"nominal FFMA peak at the median SM clock ({sm_mhz:.0f} MHz): "
                       "148 SMs x 128 lanes x 2 flops")
        kname = "link_local_kernel (hoa_link_local: kernels 1+2, FFMA)"
    # DRAM traffic per launch: dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture of
    # the link kernel on c3b1 (65,536 positions, d 96, bf16 q/k/v, banked generators): 3.707e9
    # bytes, equal to its algorithmic bytes; traffic grows in proportion to the positions, so it is scaled by them.
    traffic = args.traffic
    if traffic is None and d == 96 and dtype == torch.bfloat16:
        traffic = 3.707e9 * n_pos / 65536
    rot_tflops = f_rot / link_s / 1e12
    roofline = {"bound": "tensor", "kernel": kname,
                "achieved": rot_tflops, "peak": fp32acc_peak, "unit": "TFLOP/s",
                "frac": rot_tflops / fp32acc_peak, "traffic": traffic,
                "traffic_unit": "bytes per launch (DRAM read + write)",
                "peak_source": peak_source,
                "algorithmic_flops_per_launch": f_rot,
                "definition": "F_rot = N_pos x 4 x 2 d^3 (three expm products + the composition, "
                              "fp32-accurate) / the kernel's CUDA-event time, against the "
                              "fp32-accurate peak"}
    extra = {
        "tf32_tflops_measured": tf32_peak,
        "roofline_attention": {
            "kernel": "attn_tc_kernel (hoa_attn_tc_fwd)" if tc else "attn_kernel (hoa_attn_fwd, fp32)",
            "definition": "F_attn = 4 B H d T(T+1)/2 (causal QK^T + PV) / the kernel's time, against "
                          "the measured bf16 burst peak",
            "achieved_tflops": f_attn / attn_s / 1e12, "peak_tflops": bf16_burst,
            "frac": f_attn / attn_s / 1e12 / bf16_burst},
        "roofline_link_hbm": {
            "achieved_gbs": link_bytes / link_s / 1e9, "peak_gbs": hbm,
            "frac": link_bytes / link_s / 1e9 / hbm, "algorithmic_bytes_per_launch": link_bytes},
        "core_ms_per_step": core, "stage_ms": stage, "chunk": chunk,
        "roofline_baseline_formula": {
            "definition": "max(F_attn / bf16 peak (sustained), (a_all fp32 + q,k,v,o) bytes / HBM BW) "
                          "over the core region",
            "target_ms": baseline_roof_s * 1e3, "core_ms": core, "frac": baseline_roof_s * 1e3 / core},
        "roofline_extended": {
            "definition": "max(that, F_rot / fp32-accurate peak) over the core region",
            "target_ms": max(baseline_roof_s, f_rot / (fp32acc_peak * 1e12)) * 1e3,
            "core_ms": core,
            "frac": max(baseline_roof_s, f_rot / (fp32acc_peak * 1e12)) * 1e3 / core},
    }
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_leg(D, H, T)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16" if dtype == torch.bfloat16 else "f32",
        "data": "synthetic (x ~ N(0,1), seeded default-init weights)",
        "config": config_obj(args.config, world),
        "per_gpu_tokens_s": value / world,
        "roofline": roofline, "cpu_baseline": cpu,
        "e2e": {"value": world * B * T / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes},
        # per batch piece: link, carry scan, carry apply, attention, inverse transport, and the
        # fused GELU of the edge MLP in bf16 (the GEMMs are cuBLAS / cuBLASLt kernels)
        "gpu_launches": (5 + (dtype == torch.bfloat16)) * pieces * args.steps, "clocks": clk,
        "generator_precision": generator_precision_label(mod, T, dtype),
        "precision_rel_l2": precision,
        **extra,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_seq_sharded(args):
    """one long sequence split across the ranks (sequence sharding:
    NCCL all-gathers of the halo tokens, the segment totals and K/V), in the
    zig-zag layout by default (rank r holds segments r and 2N-1-r of 2N, which
    balances the causal attention).  Strong scaling: the total work is fixed;
    value = B*T / time."""
    import socket
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    if world == 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if "MASTER_PORT" not in os.environ:
            with socket.socket() as s:
                s.bind(("127.0.0.1", 0))
                os.environ["MASTER_PORT"] = str(s.getsockname()[1])
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=600),
                                device_id=dev)
    else:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    from holonomyawareattention_b200 import PathOrderedGeometricMHA, ops, seqshard

    B, T, D, H, dtn = CONFIGS[args.config]
    dtype = torch.bfloat16 if dtn == "bf16" else torch.float32
    d = D // H
    torch.manual_seed(0)
    with torch.device(dev):
        mod = PathOrderedGeometricMHA(D, n_heads=H, edge_scale=EDGE_SCALE)
    mod = mod.to(dtype).eval()
    if args.generator_precision:
        mod.generator_precision = args.generator_precision
    g = torch.Generator(device=dev).manual_seed(1000)
    x = torch.randn(B, T, D, device=dev, generator=g).to(dtype)       # same sequence on every rank
    layout = args.seq_layout
    xs = seqshard.shard_sequence(x, world, rank, layout).contiguous()
    del x
    stream = torch.cuda.current_stream(dev)
    clocks = ClockSampler(physical_gpu_index(local))
    with torch.inference_mode():
        for _ in range(args.warmup):
            seqshard.sequence_sharded_forward(mod, xs, layout=layout)
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        clocks.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.region_start()
        e0.record(stream)
        for _ in range(args.steps):
            y = seqshard.sequence_sharded_forward(mod, xs, layout=layout)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        clk = clocks.stop()
        dist.barrier()
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        # end to end: the shard's input from pinned host memory, its output back
        xh = xs.cpu().pin_memory()
        yh = torch.empty(tuple(y.shape), dtype=y.dtype).pin_memory()
        xd = torch.empty_like(xs)
        dist.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            xd.copy_(xh, non_blocking=True)
            yy = seqshard.sequence_sharded_forward(mod, xd, layout=layout)
            yh.copy_(yy, non_blocking=True)
        f1.record(stream)
        torch.cuda.synchronize(dev)
        t2 = torch.tensor([f0.elapsed_time(f1) / args.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        e2e_ms = float(t2.item())
        ops.check_status(dev)
    peaks = load_peaks()
    n_pos = B * H * T
    m_dim = d * (d - 1) // 2
    core_bytes = n_pos * (m_dim * 4 + 4 * d * 2)
    f_attn = 4.0 * B * H * d * T * (T + 1) / 2
    bf16_peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    roof_s = max(f_attn / (bf16_peak * 1e12 * world), core_bytes / (peaks["hbm_gbs"] * 1e9 * world))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_leg(D, H, T)
    line = {
        "metric": METRIC, "value": B * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if dtype == torch.bfloat16 else "f32",
        "data": "synthetic (x ~ N(0,1), seeded default-init weights)",
        "config": config_obj(args.config, world, args.seq_layout),
        "per_gpu_tokens_s": B * T / (ms / 1e3) / world,
        "roofline": {"bound": "hbm", "kernel": "whole sharded forward",
                     "achieved": core_bytes / world / (ms / 1e3) / 1e9, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": core_bytes / world / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                     "traffic": None, "peak_source": f"{peaks['source']} hbm_gbs (of {peaks['source']})"},
        "roofline_baseline_formula": {"target_ms": roof_s * 1e3, "ms": ms, "frac": roof_s * 1e3 / ms},
        "cpu_baseline": cpu,
        "e2e": {"value": B * T / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": xs.numel() * xs.element_size(),
                "d2h_bytes_per_step": xs.numel() * xs.element_size()},
        # per step: link, two carry scans, carry apply, one attention per local segment,
        # inverse transport, and the fused GELU of the edge MLP in bf16
        "gpu_launches": (5 + len(seqshard.segments_of(layout, world, rank)[0])
                         + (dtype == torch.bfloat16)) * args.steps, "clocks": clk,
        "generator_precision": generator_precision_label(mod, T, dtype),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c3", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--generator-precision", default=None, choices=[None, "auto", "split", "split8", "bf16"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seq-layout", default="zigzag", choices=["zigzag", "contiguous"],
                    help="shard layout of the sequence-sharded configs")
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu dram bytes per link_local launch, from a capture (scaled), if known")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.config in SEQ_SHARDED:
        return run_seq_sharded(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
