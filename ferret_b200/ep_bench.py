"""Multi-GPU leg of bench.py: the same global W13 batch run expert-parallel.

Launched by torchrun (one process per GPU).  Rank r owns E/G experts
(contiguous ids, or the balanced placement with --placement balanced) and
T/G of the tokens; one step = ExpertParallelW13.forward.  The default
exchange (--ep-mode p2p) is the library's peer-memory path: own-token FP8
quantization, device flag barriers, routed FP8 rows pulled from the source
ranks, grouped GEMM storing its rows into the source ranks' outputs over
NVLink.  --ep-mode gather / a2a / auto use torch.distributed NCCL collectives
instead.  Strong scaling: the global batch is fixed as G grows.
Modes without a host synchronisation (p2p, gather) run each step as one CUDA
graph replay; "a2a" (one host sync per step for the splits) runs eagerly.
Timing: CUDA events per step on each rank's stream, 256 MB L2 flush between
steps, barrier + synchronize around the timed region, max over ranks.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

FLUSH_BYTES = 256 << 20


def _max(x: float, dev) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum(x: float, dev) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def run(args, cfg):
    import bench  # contract helpers (peaks, clocks, algorithmic bytes)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    ep = graph = None
    try:
        from . import build
        if local == 0:
            build.build()
        dist.barrier()
        from . import data
        from .ep import ExpertParallelW13, StepTimers, balanced_placement

        G = world
        if cfg.E % G or cfg.T % G:
            raise ValueError(f"E={cfg.E} and T={cfg.T} must divide by {G}")
        El, Tl = cfg.E // G, cfg.T // G
        ids_g = data.routing(cfg.T, cfg.E, cfg.topk, cfg.routing, cfg.zipf_s)
        hidden_g = data.activations(cfg.T, cfg.K)
        placement = None
        if getattr(args, "placement", "contiguous") == "balanced":
            placement = balanced_placement(torch.bincount(ids_g.reshape(-1), minlength=cfg.E), G)
        table = placement if placement is not None else torch.arange(cfg.E, dtype=torch.int32)
        mine = table[rank * El:(rank + 1) * El]
        W, Ws = data.fp8_weights(El, cfg.N, cfg.K, seed=1000 + rank, device=dev)
        ids = ids_g[rank * Tl:(rank + 1) * Tl].contiguous().to(dev)
        hidden = hidden_g[rank * Tl:(rank + 1) * Tl].contiguous().to(dev)
        mode = getattr(args, "ep_mode", "p2p")
        ep = ExpertParallelW13(W, Ws, cfg.E, silu=cfg.silu, placement=placement, mode=mode)
        n_out = cfg.N // 2 if cfg.silu else cfg.N
        if mode == "auto":
            mode = "gather" if ep.G * Tl * cfg.topk * n_out * 2 <= ep.GATHER_BYTES else "a2a"
        graphed = mode in ("p2p", "gather")      # no host synchronisation inside a step

        flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        for _ in range(args.warmup):
            ep.forward(hidden, ids)
        torch.cuda.synchronize()
        dist.barrier()
        graph = None
        if graphed:
            # the whole step -- collectives included -- as one CUDA graph; every
            # rank captures the same sequence of collectives
            # external events become record nodes of the graph, so the local
            # GEMM stays timed on replay
            tm_g = StepTimers(torch.cuda.Event(enable_timing=True, external=True),
                              torch.cuda.Event(enable_timing=True, external=True))
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=side):
                    out_static = ep.forward(hidden, ids, timers=tm_g)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            dist.barrier()
        stream = torch.cuda.current_stream()

        K = args.steps
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(K)]
        tm = [StepTimers(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(K)]
        clocks = bench.Clocks(local) if rank == 0 else None
        torch.cuda.synchronize()
        dist.barrier()
        if clocks:
            clocks.start()
        gemm_list = []
        for i in range(K):
            flush.zero_()
            ev[i][0].record(stream)
            if graph is not None:
                graph.replay()
                out = out_static
            else:
                out = ep.forward(hidden, ids, timers=tm[i])
            ev[i][1].record(stream)
            if graph is not None:
                torch.cuda.synchronize()
                gemm_list.append(tm_g.gemm_start.elapsed_time(tm_g.gemm_end))
        torch.cuda.synchronize()
        dist.barrier()
        clk = clocks.stop() if clocks else None
        step_ms = sum(a.elapsed_time(b) for a, b in ev) / K
        if graph is None:
            gemm_list = [t.gemm_start.elapsed_time(t.gemm_end) for t in tm]
        gemm_ms = sum(gemm_list) / K

        # e2e: host buffers in, host buffer out, through the same public API
        h_hidden = hidden.cpu().pin_memory()
        h_ids = ids.cpu().pin_memory()
        h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        d_hidden, d_ids = torch.empty_like(hidden), torch.empty_like(ids)
        ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(K)]
        dist.barrier()
        for i in range(K):
            flush.zero_()
            ev2[i][0].record(stream)
            if graph is not None:
                hidden.copy_(h_hidden, non_blocking=True)     # the graph's static inputs
                ids.copy_(h_ids, non_blocking=True)
                graph.replay()
                o = out_static
            else:
                d_hidden.copy_(h_hidden, non_blocking=True)
                d_ids.copy_(h_ids, non_blocking=True)
                o = ep.forward(d_hidden, d_ids)
            h_out.copy_(o, non_blocking=True)
            ev2[i][1].record(stream)
        torch.cuda.synchronize()
        e2e_ms = sum(a.elapsed_time(b) for a, b in ev2) / K

        # local GEMM algorithmic bytes (this rank's experts and received rows)
        flat = ids_g.reshape(-1)
        owner_slot = torch.empty(cfg.E, dtype=torch.int64)
        owner_slot[table.long()] = torch.arange(cfg.E)
        loc_counts = torch.bincount(owner_slot[flat.long()], minlength=cfg.E)[rank * El:(rank + 1) * El]
        byts, _, active = bench.fp8_algorithmic(cfg, loc_counts.tolist())
        R_global = int(flat.numel())
        flops = 2.0 * R_global * cfg.N * cfg.K

        if mode == "p2p":
            # quant, publish, ready, ids, permute (1, or count/scan/scatter), row gather, GEMM, done
            from ._lib import lib
            chunked = lib().ferret_moe_permute_workspace_size(G * Tl, cfg.topk, El) > 0
            launches = 7 + (3 if chunked else 1)
        else:
            launches = 4
        max_step = _max(step_ms, dev)
        max_gemm = _max(gemm_ms, dev)
        max_e2e = _max(e2e_ms, dev)
        gemm_bw = byts / (gemm_ms * 1e-3) / 1e9
        min_bw = -_max(-gemm_bw, dev)
        sum_active = _sum(float(active), dev)
        max_rows = _max(float(loc_counts.sum()), dev)
        if rank != 0:
            return None
        pk = bench.peaks()
        return {
            "metric": "grouped W13 GEMM TFLOPS & HBM GB/s vs roofline",
            "value": round(flops / (max_step * 1e-3) / 1e12, 3),
            "unit": "TFLOPS",
            "n_gpus": G,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": round(max_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "e4m3 x e4m3 -> f32 accumulate, bf16 out; "
                     + ("fp8 dispatch" if mode == "p2p" else "bf16 dispatch"),
            "data": "synthetic (seeded), random-init weights",
            "config": {"workload": cfg.name, "E": cfg.E, "topk": cfg.topk, "tokens": cfg.T,
                       "routed_rows": R_global, "K": cfg.K, "N": cfg.N, "silu": cfg.silu,
                       "routing": cfg.routing,
                       "parallelism": f"ep{G} ({El} experts and {Tl} tokens per GPU, "
                                      f"{'balanced' if placement is not None else 'contiguous'} placement)",
                       "active_experts_total": int(sum_active), "max_rows_per_gpu": int(max_rows),
                       "l2": "256 MB flush between timed steps"},
            "roofline": {"bound": "hbm", "kernel": "fp8_w13_grouped_kernel (per-GPU local GEMM, slowest rank)",
                         "achieved": round(min_bw, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(min_bw / pk["hbm_gbs"], 4), "peak_source": pk["source"],
                         "kernel_ms": round(max_gemm, 4), "traffic": None},
            "e2e": {"value": round(flops / (max_e2e * 1e-3) / 1e12, 3), "unit": "TFLOPS",
                    "ms_per_step": round(max_e2e, 4),
                    "h2d_bytes_per_step": (h_hidden.numel() * 2 + h_ids.numel() * 4) * G,
                    "d2h_bytes_per_step": h_out.numel() * 2 * G},
            "gpu_launches": launches * K,
            "ep_mode": mode,
            "cuda_graph": graph is not None,
            "clocks": clk,
        }
    finally:
        graph = None        # a graph holding NCCL work must be released before teardown
        torch.cuda.synchronize()
        if ep is not None:
            ep.close()      # collective: peer-memory context (p2p)
        dist.destroy_process_group()
