#!/usr/bin/env python
"""Benchmark of the quantized MoE W13 grouped GEMM hot path (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload ep_prefill] [--no-extras]

One step = one pass of the W13 path over one batch: routing ids -> expert
permutation -> per-token FP8 quantization -> FP8 block-scaled grouped GEMM
(bf16 out).  Default workload: benchmark configuration 5, the DeepSeek-V3
prefill W13 batch the metric's 1/2/4/8-GPU sweep is defined on (E=256, top-8
Zipf(1.1), 32,768 tokens, K=7168, N=4096), seeded synthetic data and
random-init weights.  With N>1 GPUs the same global batch runs
expert-parallel (E/N experts per GPU, balanced placement, peer-memory
dispatch/combine over NVLink): strong scaling.  At N=1, with no --workload,
the line also carries configurations 2, 3 and 4 (decode, 8,192-token prefill,
INT4 decode) under "extra_workloads", each timed in the same run with its own
roofline.

Prints one JSON line on rank 0.  Timing: W untimed warm-up steps, then K
steps, each bracketed by CUDA events on the launching stream with a 256 MB
L2 flush between steps (outside the events); barrier + synchronize around the
timed region; max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FLUSH_BYTES = 256 << 20
DEFAULT_WORKLOAD = "ep_prefill"                  # configuration 5 (the 1/2/4/8-GPU sweep)
EXTRA_WORKLOADS = ("dsv3_decode", "dsv3_prefill", "kimi_int4_decode")   # configurations 2, 3, 4
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=None,
                    help=f"workload name (default {DEFAULT_WORKLOAD}, plus the extra workloads at N=1)")
    ap.add_argument("--no-extras", action="store_true",
                    help="N=1 default run: skip the extra workloads")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--placement", choices=["contiguous", "balanced"], default="balanced",
                    help="expert placement for N>1 (balanced = greedy LPT on the routing histogram)")
    ap.add_argument("--ep-mode", choices=["p2p", "gather", "a2a", "auto"], default="p2p",
                    help="N>1 exchange: p2p = peer-memory kernels (library ferret_ep_*); "
                         "gather / a2a / auto = torch.distributed NCCL collectives")
    ap.add_argument("--suite", choices=["", "v007-configs"], default="",
                    help="v007-configs: the reference kernel's own 8 benchmark shapes "
                         "(E=32 experts, gate_up and down, 1-16 rows per expert); with --impl "
                         "reference, the reference's own GPU kernel compiled unmodified")
    ap.add_argument("--scales", choices=["fp32", "ue8m0"], default="fp32",
                    help="FP8 block scales: fp32 (exact, the reference contract) or ue8m0 "
                         "(power-of-two weights and activations; the 128-row-tile GEMM applies "
                         "them inside the MMA, kind::mxf8f6f4.block_scale)")
    ap.add_argument("--prefill-pairs", action="store_true",
                    help="128-token-tile launches put each expert's whole 256-row chunks on CTA "
                         "pairs (tcgen05.mma.cta_group::2)")
    ap.add_argument("--gemm-only", type=int, default=0,
                    help="profiling aid: run N bare GEMM launches and exit")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
            "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class Clocks:
    """nvidia-smi sampler (a separate process, 100 ms interval) running during the
    timed region.  An in-process NVML polling thread was tried and dropped: with
    it the timed GEMMs read 2-13 % slower than the same launches timed without
    it (cause not isolated)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for _, _, fl in rows for n, v in zip(names, fl) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows), "sampler": "nvidia-smi 100 ms"}


def fp8_algorithmic(cfg, counts):
    """Algorithmic bytes and FLOPs of the FP8 W13 GEMM: every active expert's
    weights and block scales read once, activations and their scales read once,
    outputs written once; FLOPs 2*R*N*K over real rows (decode.yaml:100)."""
    R = int(sum(counts))
    active = sum(1 for c in counts if c > 0)
    n_out = cfg.N // 2 if cfg.silu else cfg.N
    nk = cfg.K // 128
    wbytes = active * (cfg.N * cfg.K + (cfg.N // 128) * nk * 4)
    byts = wbytes + R * cfg.K + R * nk * 4 + R * n_out * 2
    flops = 2.0 * R * cfg.N * cfg.K
    return byts, flops, active


def int4_algorithmic(cfg, counts):
    """Algorithmic bytes and FLOPs of the INT4 W13 GEMM (packed weights and
    group scales of every active expert once, activations once, outputs once),
    and the reference's narrower INT4 weight bytes (baseline_marlin.py:204-206)."""
    R = int(sum(counts))
    active = sum(1 for c in counts if c > 0)
    n_out = cfg.N // 2 if cfg.silu else cfg.N
    wbytes = active * (cfg.N * cfg.K // 2)
    byts = wbytes + active * cfg.N * (cfg.K // 32) * 2 + cfg.T * cfg.K * 2 + R * n_out * 2
    return byts, 2.0 * R * cfg.N * cfg.K, active, wbytes


def roofline(byts, flops, kernel_ms, pk, kernel):
    """Roofline of one kernel launch: the bound is whichever of HBM bytes or
    tensor FLOPs needs longer at peak.  The FP8 tensor peak is twice the
    measured bf16 cuBLAS burst figure (dense FP8 runs at twice the bf16 rate
    on B200)."""
    fp8_peak = 2.0 * pk["bf16_tflops"]
    t_hbm = byts / (pk["hbm_gbs"] * 1e9)
    t_tc = flops / (fp8_peak * 1e12)
    s = kernel_ms * 1e-3
    gbs, tfl = byts / s / 1e9, flops / s / 1e12
    if t_hbm >= t_tc:
        out = {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
               "frac": round(gbs / pk["hbm_gbs"], 4),
               "peak_source": pk["source"] + " hbm_gbs"}
    else:
        out = {"bound": "tensor", "achieved": round(tfl, 1), "peak": fp8_peak, "unit": "TFLOP/s",
               "frac": round(tfl / fp8_peak, 4),
               "peak_source": pk["source"] + " bf16_tflops x2 (fp8)"}
    out.update({"kernel": kernel, "kernel_ms": round(kernel_ms, 4), "algorithmic_bytes": byts,
                "hbm_frac": round(gbs / pk["hbm_gbs"], 4),
                "tensor_frac_fp8": round(tfl / fp8_peak, 4), "kernel_tflops": round(tfl, 2),
                "roofline_frac": round(max(t_hbm, t_tc) / s, 4)})
    return out


def graph_of(fn):
    """fn's launches captured once as a CUDA graph: timing its replays measures
    device time without the Python/ctypes launch overhead, which would
    otherwise dominate microsecond-sized steps."""
    import torch
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    return g


def read_traffic(kernel_tag):
    """dram bytes per launch recorded from an ncu capture in profiles/<tag>.md."""
    path = os.path.join(ROOT, "profiles", f"{kernel_tag}.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def cpu_baseline(a_q, a_scale, W, W_s, offsets, cfg, budget_s=12.0, max_experts=64):
    """The torch CPU fp32 dequantize-then-matmul path on a bounded sample of
    the same workload: whole experts in order until ~budget_s of CPU work."""
    import torch
    from oracle import oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    counts = (offsets[1:] - offsets[:-1]).tolist()
    experts = [e for e, c in enumerate(counts) if c > 0][:max_experts]
    flops = 0.0
    done = []
    t0 = time.perf_counter()
    for e in experts:
        r0, r1 = int(offsets[e]), int(offsets[e + 1])
        w_e = W[e:e + 1].cpu()
        ws_e = W_s[e:e + 1].cpu()
        off = torch.tensor([0, r1 - r0])
        t1 = time.perf_counter()
        O.fp8_w13_torch_cpu(a_q[r0:r1], a_scale[r0:r1], w_e, ws_e, off, [0], silu=cfg.silu)
        flops += 2.0 * (r1 - r0) * cfg.N * cfg.K
        done.append((e, time.perf_counter() - t1))
        if time.perf_counter() - t0 > budget_s:
            break
    compute_s = sum(t for _, t in done)
    rows = sum(int(offsets[e + 1] - offsets[e]) for e, _ in done)
    return {"value": flops / compute_s / 1e12, "unit": "TFLOPS", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{len(done)} of {sum(1 for c in counts if c > 0)} active experts "
                      f"({rows} routed rows), torch fp32 dequantize-then-matmul per expert, "
                      f"{compute_s:.1f} s"}


# ---------------------------------------------------------------------------
# our arm, one GPU
# ---------------------------------------------------------------------------

def int4_cpu_baseline(hidden, ids, samples, cfg, budget_s=12.0):
    """The torch CPU fp32 INT4 path (dequantize-then-matmul) on a bounded
    sample: the experts in `samples` ({expert: (raw, scales)} host copies) with
    all their routed rows, until ~budget_s of CPU work."""
    import torch
    from oracle import oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    flat = ids.reshape(-1).cpu()
    h = hidden.cpu()
    flops, t_sum, rows_done, n = 0.0, 0.0, 0, 0
    for e, (raw_e, sc_e) in samples.items():
        rows = torch.nonzero(flat == e).flatten() // cfg.topk
        t1 = time.perf_counter()
        O.int4_w13_torch_cpu(h[rows], raw_e, sc_e, silu=cfg.silu)
        t_sum += time.perf_counter() - t1
        flops += 2.0 * len(rows) * cfg.N * cfg.K
        rows_done += len(rows)
        n += 1
        if t_sum > budget_s:
            break
    return {"value": flops / t_sum / 1e12, "unit": "TFLOPS", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} active experts ({rows_done} routed rows), torch fp32 INT4 "
                      f"dequantize-then-matmul per expert, {t_sum:.1f} s"}


def run_single(args, cfg):
    import torch
    from ferret_b200 import build, data, ops
    build.build()
    if cfg.quant == "int4":
        return run_single_int4(args, cfg)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ue8m0 = getattr(args, "scales", "fp32") == "ue8m0"
    pairs = bool(getattr(args, "prefill_pairs", False))
    W, W_s = data.fp8_weights(cfg.E, cfg.N, cfg.K, device=dev, use_ue8m0=ue8m0)
    hidden = data.activations(cfg.T, cfg.K).to(dev)
    ids = data.routing(cfg.T, cfg.E, cfg.topk, cfg.routing, cfg.zipf_s).to(dev)
    n_out = cfg.N // 2 if cfg.silu else cfg.N
    bufs = ops.W13Buffers(cfg.T, cfg.topk, cfg.K, n_out, cfg.E, dev)

    def step():
        ops.fp8_moe_w13(hidden, ids, W, W_s, silu=cfg.silu, bufs=bufs, use_ue8m0=ue8m0,
                        prefill_pairs=pairs)

    def gemm():
        ops.m_grouped_fp8_gemm_nt_contiguous((bufs.a, bufs.a_scale), (W, W_s), bufs.out, None,
                                             disable_ue8m0_cast=not ue8m0,
                                             expert_offsets=bufs.offsets, silu=cfg.silu,
                                             prefill_pairs=pairs)

    if args.gemm_only:
        step()
        for _ in range(args.gemm_only):
            gemm()
        torch.cuda.synchronize()
        return None

    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if ops.last_device_status() != 0:
        raise RuntimeError("device status error after warm-up")

    def timed(fn, k):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(k)]
        for i in range(k):
            flush.zero_()
            evs[i][0].record(stream)
            fn()
            evs[i][1].record(stream)
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in evs]

    # each timed step replays the step's launches as one CUDA graph
    step_graph = graph_of(step)
    clocks = Clocks(torch.cuda.current_device())
    torch.cuda.synchronize()
    clocks.start()
    step_ms = timed(step_graph.replay, args.steps)
    clk = clocks.stop()
    torch.cuda.synchronize()

    # dominant kernel alone (same stream, same flush discipline)
    gemm_ms = timed(graph_of(gemm).replay, args.steps)

    # end to end through the public API with host buffers
    h_hidden = hidden.cpu().pin_memory()
    h_ids = ids.cpu().pin_memory()
    h_out = torch.empty(bufs.out.shape, dtype=bufs.out.dtype).pin_memory()
    d_hidden = torch.empty_like(hidden)
    d_ids = torch.empty_like(ids)

    def e2e():
        d_hidden.copy_(h_hidden, non_blocking=True)
        d_ids.copy_(h_ids, non_blocking=True)
        out, _, _ = ops.fp8_moe_w13(d_hidden, d_ids, W, W_s, silu=cfg.silu, bufs=bufs,
                                    use_ue8m0=ue8m0, prefill_pairs=pairs)
        h_out.copy_(out, non_blocking=True)
    e2e()
    e2e_ms = timed(e2e, args.steps)
    if ops.last_device_status() != 0:
        raise RuntimeError("device status error after timing")
    out_ok = bool(torch.isfinite(bufs.out[: int(bufs.offsets[-1])].float()).all())

    offsets = bufs.offsets.cpu()
    counts = (offsets[1:] - offsets[:-1]).tolist()
    byts, flops, active = fp8_algorithmic(cfg, counts)
    ms = sum(step_ms) / len(step_ms)
    ms_med = statistics.median(step_ms)
    g_ms = sum(gemm_ms) / len(gemm_ms)
    e_ms = sum(e2e_ms) / len(e2e_ms)
    pk = peaks()
    # the library runs the prefill kernel when experts average more than 48 rows
    prefill = (cfg.R + cfg.E - 1) // cfg.E > 48 and cfg.N % 256 == 0
    kname = (("fp8_w13_prefill_mx_kernel" if ue8m0 and not cfg.silu
              else "fp8_w13_prefill_pair_kernel" if pairs else "fp8_w13_prefill_kernel") if prefill
             else "fp8_w13_grouped_kernel")
    rl = roofline(byts, flops, g_ms, pk, kname)
    res = {
        "metric": "grouped W13 GEMM TFLOPS & HBM GB/s vs roofline",
        "value": round(flops / (ms * 1e-3) / 1e12, 3),
        "unit": "TFLOPS",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "ms_per_step_median": round(ms_med, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> f32 accumulate, bf16 out",
        "data": "synthetic (seeded), random-init weights",
        "config": {"workload": cfg.name, "E": cfg.E, "topk": cfg.topk, "tokens": cfg.T,
                   "routed_rows": cfg.R, "active_experts": active, "K": cfg.K, "N": cfg.N,
                   "silu": cfg.silu, "routing": cfg.routing, "parallelism": "single GPU",
                   "scales": "ue8m0 (powers of two)" if ue8m0 else "fp32 (exact)",
                   "prefill_pairs": pairs,
                   "l2": "256 MB flush between timed steps; weights (GBs) exceed L2"},
        "hbm_gbs_step": round(byts / (ms * 1e-3) / 1e9, 1),
        "roofline": dict(rl, traffic=read_traffic(f"{rl['kernel'].removesuffix('_kernel')}_{cfg.name}")),
        "e2e": {"value": round(flops / (e_ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
                "ms_per_step": round(e_ms, 4),
                "h2d_bytes_per_step": h_hidden.numel() * 2 + h_ids.numel() * 4,
                "d2h_bytes_per_step": h_out.numel() * 2},
        # permute (1, or count/scan/scatter), quant (1, or quant-once + gather), GEMM
        "gpu_launches": ((3 if bufs.perm_ws_bytes else 1) + (2 if bufs.quant_once else 1)
                         + (2 if pairs and prefill else 1)) * args.steps,
        "clocks": clk,
        "output_finite": out_ok,
    }
    if not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(bufs.a.cpu(), bufs.a_scale.cpu(), W, W_s, offsets, cfg)
    return res


def run_single_int4(args, cfg):
    """Kimi-style INT4 W4A16 W13 on one GPU: permute + INT4 grouped GEMM."""
    import torch
    from ferret_b200 import data, ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    raw, scales = data.int4_weights(cfg.E, cfg.N, cfg.K, device=dev)
    packed = ops.Int4W13Weights(raw, scales)
    hidden = data.activations(cfg.T, cfg.K).to(dev)
    ids = data.routing(cfg.T, cfg.E, cfg.topk, cfg.routing, cfg.zipf_s).to(dev)
    samples = {}
    if not args.no_cpu_baseline and not args.gemm_only:
        # host copies of the first active experts for the CPU baseline
        act = torch.nonzero(torch.bincount(ids.reshape(-1).long(), minlength=cfg.E)).flatten()
        samples = {int(e): (raw[e].cpu(), scales[e].cpu()) for e in act[:32]}
    del raw, scales
    n_out = cfg.N // 2 if cfg.silu else cfg.N
    out = torch.zeros(cfg.R, n_out, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(ops.lib().ferret_int4_moe_w13_workspace_size(cfg.T, cfg.topk, cfg.K),
                     dtype=torch.uint8, device=dev)

    def step():
        ops.moe_wna16_w13(hidden, packed, ids, silu=cfg.silu, out=out, workspace=ws)

    if args.gemm_only:
        perm = ops.moe_permute(ids, cfg.E)
        for _ in range(args.gemm_only):
            ops.moe_wna16_w13(hidden, packed, ids, silu=cfg.silu, out=out, perm=perm, workspace=ws)
        torch.cuda.synchronize()
        return None
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def timed(fn, k):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(k)]
        for i in range(k):
            flush.zero_()
            evs[i][0].record(stream)
            fn()
            evs[i][1].record(stream)
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in evs]

    step_graph = graph_of(step)
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    step_ms = timed(step_graph.replay, args.steps)
    clk = clocks.stop()
    perm = ops.moe_permute(ids, cfg.E)
    gemm_ms = timed(graph_of(lambda: ops.moe_wna16_w13(hidden, packed, ids, silu=cfg.silu, out=out,
                                                       perm=perm, workspace=ws)).replay,
                    args.steps)
    h_hidden, h_ids = hidden.cpu().pin_memory(), ids.cpu().pin_memory()
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    d_hidden, d_ids = torch.empty_like(hidden), torch.empty_like(ids)

    def e2e():
        d_hidden.copy_(h_hidden, non_blocking=True)
        d_ids.copy_(h_ids, non_blocking=True)
        ops.moe_wna16_w13(d_hidden, packed, d_ids, silu=cfg.silu, out=out, workspace=ws)
        h_out.copy_(out, non_blocking=True)
    e2e_ms = timed(e2e, args.steps)
    if ops.last_device_status() != 0:
        raise RuntimeError("device status error after timing")
    counts = torch.bincount(ids.reshape(-1).cpu().long(), minlength=cfg.E).tolist()
    byts, flops, active, wbytes = int4_algorithmic(cfg, counts)
    ms = sum(step_ms) / len(step_ms)
    ms_med = statistics.median(step_ms)
    g_ms = sum(gemm_ms) / len(gemm_ms)
    e_ms = sum(e2e_ms) / len(e2e_ms)
    pk = peaks()
    achieved = byts / (g_ms * 1e-3) / 1e9
    # the library's choice (ferret_int4_moe_w13): the register-dequant decode
    # kernel for more than 64 routed rows averaging at most 4 per possible expert
    i4_kernel = ("int4_w13_decode_kernel" if 64 < cfg.R <= 4 * min(cfg.R, cfg.E)
                 else "int4_w13_grouped_kernel")
    res = {
        "metric": "grouped W13 GEMM TFLOPS & HBM GB/s vs roofline",
        "value": round(flops / (ms * 1e-3) / 1e12, 3), "unit": "TFLOPS", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "ms_per_step_median": round(ms_med, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 weights dequantized to bf16 x bf16 -> f32 accumulate, bf16 out",
        "data": "synthetic (seeded), random-init weights",
        "config": {"workload": cfg.name, "E": cfg.E, "topk": cfg.topk, "tokens": cfg.T,
                   "routed_rows": cfg.R, "active_experts": active, "K": cfg.K, "N": cfg.N,
                   "silu": cfg.silu, "routing": cfg.routing, "parallelism": "single GPU",
                   "l2": "256 MB flush between timed steps; weights (GBs) exceed L2"},
        "int4_weight_tbs": round(wbytes / (g_ms * 1e-3) / 1e12, 3),
        "roofline": {"bound": "hbm", "kernel": i4_kernel,
                     "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4),
                     "peak_source": pk["source"] + " (hbm_gbs)", "algorithmic_bytes": byts,
                     "kernel_ms": round(g_ms, 4),
                     "kernel_tflops": round(flops / (g_ms * 1e-3) / 1e12, 3),
                     "traffic": read_traffic(f"{i4_kernel.removesuffix('_kernel')}_{cfg.name}")},
        "e2e": {"value": round(flops / (e_ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
                "ms_per_step": round(e_ms, 4),
                "h2d_bytes_per_step": h_hidden.numel() * 2 + h_ids.numel() * 4,
                "d2h_bytes_per_step": h_out.numel() * 2},
        "gpu_launches": 3 * args.steps,   # permute, row gather, INT4 GEMM
        "clocks": clk,
    }
    if samples:
        res["cpu_baseline"] = int4_cpu_baseline(hidden, ids, samples, cfg)
    return res


def run_extra(args, cfg):
    """One more single-GPU workload in the same run: its step time (mean and
    median), value, dominant-kernel roofline and end-to-end figure."""
    import copy
    import gc
    import torch
    a = copy.copy(args)
    a.no_cpu_baseline = True
    gc.collect()
    torch.cuda.empty_cache()
    r = run_single(a, cfg)
    keep = ("value", "unit", "ms_per_step", "ms_per_step_median", "roofline", "e2e", "clocks",
            "int4_weight_tbs", "hbm_gbs_step")
    out = {k: r[k] for k in keep if k in r}
    out["config"] = {k: r["config"][k] for k in ("E", "topk", "tokens", "routed_rows", "K", "N",
                                                  "silu", "routing") if k in r["config"]}
    gc.collect()
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU fp32 path on the host cores
# ---------------------------------------------------------------------------

def run_reference(args, cfg):
    import torch
    from ferret_b200 import data
    from oracle import oracle as O
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    ids = data.routing(cfg.T, cfg.E, cfg.topk, cfg.routing, cfg.zipf_s)
    flat = ids.reshape(-1)
    counts = torch.bincount(flat, minlength=cfg.E)
    experts = [int(e) for e in torch.nonzero(counts).flatten()]
    hidden = data.activations(cfg.T, cfg.K)
    # one step = a bounded sample: SAMPLE experts (all their routed rows)
    SAMPLE = 4
    g = torch.Generator().manual_seed(0)

    def expert_inputs(e):
        rows = torch.nonzero(flat == e).flatten() // cfg.topk
        w = torch.randn(1, cfg.N, cfg.K, generator=g) * 0.02
        wq, ws = data.per_block_cast_to_fp8(w)
        x = hidden[rows].float().view(len(rows), cfg.K // 128, 128)
        amax = x.abs().amax(dim=2).clamp(min=1e-4)
        aq = (x * (448.0 / amax.unsqueeze(2))).to(torch.float8_e4m3fn).view(len(rows), cfg.K)
        return aq, amax / 448.0, wq, ws

    samples = [expert_inputs(e) for e in experts[: SAMPLE * 2]]
    times, flops = [], []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        f = 0.0
        for j in range(SAMPLE):
            aq, as_, wq, ws = samples[(i * SAMPLE + j) % len(samples)]
            O.fp8_w13_torch_cpu(aq, as_, wq, ws, torch.tensor([0, aq.shape[0]]), [0], silu=cfg.silu)
            f += 2.0 * aq.shape[0] * cfg.N * cfg.K
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
            flops.append(f)
    tf = sum(flops) / sum(times) / 1e12
    ms = 1e3 * sum(times) / len(times)
    cores = torch.get_num_threads()
    sample = (f"{SAMPLE} experts per step (all their routed rows) of {len(experts)} active; "
              "torch fp32 dequantize-then-matmul (correctness/compare_marlin_vs_ref.py:44-100 "
              "restated for FP8 block scales)")
    return {
        "impl": "reference",
        "metric": "grouped W13 GEMM TFLOPS & HBM GB/s vs roofline",
        "value": round(tf, 5), "unit": "TFLOPS", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": cfg.name, "E": cfg.E, "topk": cfg.topk, "tokens": cfg.T,
                   "K": cfg.K, "N": cfg.N, "silu": cfg.silu, "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(tf, 5), "unit": "TFLOPS", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(tf, 5), "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# the reference kernel's own benchmark shapes
# (tasks/fp8-group-gemm-dsv3-decode.yaml:45-86, v007_dsv3_decode_verified_105.cu:473-478)
# ---------------------------------------------------------------------------

V007_CONFIGS = [("gate_up_M1", 1, 32, 7168, 4096), ("gate_up_M4", 4, 32, 7168, 4096),
                ("gate_up_M8", 8, 32, 7168, 4096), ("gate_up_M16", 16, 32, 7168, 4096),
                ("down_M1", 1, 32, 2048, 7168), ("down_M4", 4, 32, 2048, 7168),
                ("down_M8", 8, 32, 2048, 7168), ("down_M16", 16, 32, 2048, 7168)]


def run_v007_suite(args):
    """Our grouped GEMM through the DeepGEMM-style call (m_indices, segments
    derived on the device) at the reference kernel's 8 shapes: random e4m3
    operands (NaN codes skipped), scales in [0.5, 1), median of 100 launches,
    256 MB L2 flush before each."""
    import torch
    from ferret_b200 import build, ops
    build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(42)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def e4m3_bytes(*shape):
        b = torch.randint(0, 254, shape, generator=g, device=dev, dtype=torch.int32)
        return (b + (b >= 0x7F).int()).to(torch.uint8)

    res, us, res_tile, us_tile = {}, {}, {}, {}
    for name, mpe, E, K, N in V007_CONFIGS:
        M = mpe * E
        A, W = e4m3_bytes(M, K), e4m3_bytes(E, N, K)
        As = torch.rand(M, K // 128, generator=g, device=dev) * 0.5 + 0.5
        Ws = torch.rand(E, N // 128, K // 128, generator=g, device=dev) * 0.5 + 0.5
        mi = (torch.arange(M, device=dev) // mpe).to(torch.int32)
        # the work the reference kernel does: every 128-row tile takes the
        # expert of its first row (v007:162,286), so only 1-4 experts stream
        mi_tile = mi[(torch.arange(M, device=dev) // 128) * 128].contiguous()
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        for m_ind, rd, ud in ((mi, res, us), (mi_tile, res_tile, us_tile)):
            call = lambda: ops.m_grouped_fp8_gemm_nt_contiguous((A, As), (W, Ws), out, m_ind)
            run = graph_of(call).replay
            for _ in range(20):
                run()
            torch.cuda.synchronize()
            times = []
            for _ in range(100):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                run()
                b.record()
                b.synchronize()
                times.append(a.elapsed_time(b))
            times.sort()
            med = times[50]
            rd[name] = round(2.0 * M * N * K / (med * 1e-3) / 1e12, 4)
            ud[name] = round(med * 1e3, 2)
    if ops.last_device_status() != 0:
        raise RuntimeError("device status error")
    return {"suite": "v007-configs", "impl": "ours", "unit": "TFLOPS", "results": res, "us": us,
            "results_tile_expert": res_tile, "us_tile_expert": us_tile,
            "timing": "median of 100, 256 MB flush before each, CUDA events around a CUDA-graph "
                      "replay of the call",
            "numerics": "exact fp32 block scales, per-row experts; *_tile_expert: the same call "
                        "with m_indices set to each 128-row tile's first expert (the work the "
                        "reference kernel does)"}


def run_v007_suite_reference(args):
    """The reference's own kernel and benchmark main (v007, compiled unmodified
    into oracle/_ref by `make -C oracle ref`)."""
    import re
    import subprocess
    exe = os.path.join(ROOT, "oracle", "_ref", "v007_bench")
    if not os.path.exists(exe):
        return {"suite": "v007-configs", "impl": "reference",
                "unavailable": "oracle/_ref/v007_bench not built (needs the reference tree)"}
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    m = re.search(r"KERNEL_RESULT (\{.*?\})", r.stdout)
    if r.returncode != 0 or not m:
        return {"suite": "v007-configs", "impl": "reference",
                "unavailable": f"v007_bench exited {r.returncode}"}
    per_us = dict(re.findall(r"(\w+): [0-9.]+ TFLOPS, ([0-9.]+) us", r.stderr))
    return {"suite": "v007-configs", "impl": "reference", "unit": "TFLOPS",
            "results": json.loads(m.group(1)), "us": {k: float(v) for k, v in per_us.items()},
            "timing": "its own: median of 100, 128 MB flush before each, CUDA events",
            "numerics": "UE8M0-rounded scales, first-row-of-tile experts (its own check: 32 rows)"}


def main():
    args = parse_args()
    if args.suite == "v007-configs":
        res = run_v007_suite_reference(args) if args.impl == "reference" else run_v007_suite(args)
        print(json.dumps(res), flush=True)
        return
    from ferret_b200.data import CONFIGS
    cfg = CONFIGS[args.workload or DEFAULT_WORKLOAD]
    if args.impl == "reference":
        res = run_reference(args, cfg)
    elif args.gpus > 1 or int(os.environ.get("WORLD_SIZE", "1")) > 1:
        from ferret_b200 import ep_bench
        res = ep_bench.run(args, cfg)
    else:
        res = run_single(args, cfg)
        if res is not None and args.workload is None and not args.no_extras:
            res["extra_workloads"] = {name: run_extra(args, CONFIGS[name]) for name in EXTRA_WORKLOADS}
    if res is not None and int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
