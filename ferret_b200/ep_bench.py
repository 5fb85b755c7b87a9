"""Multi-GPU leg of bench.py: the same global W13 batch run expert-parallel.

Launched by torchrun (one process per GPU).  Rank r owns E/G experts (the
balanced placement by default -- greedy LPT on the routing histogram, E/G
experts per rank -- or contiguous ids with --placement contiguous) and T/G of
the tokens; one step = ExpertParallelW13.forward.  Every rank draws the one
global weight set a single GPU would hold and keeps its own experts, so the
expert-parallel output is comparable with the single-GPU run row for row.

The default exchange (--ep-mode p2p) is the library's peer-memory path:
own-token FP8 quantization, device flag barriers, routed FP8 rows pulled from
the source ranks (inside the prefill GEMM for prefill-sized batches), grouped
GEMM storing its rows into the source ranks' outputs over NVLink.
--ep-mode gather / a2a / auto use torch.distributed NCCL collectives instead.
Strong scaling: the global batch is fixed as G grows.

Modes without a host synchronisation (p2p, gather) run each step as one CUDA
graph replay; "a2a" (one host sync per step for the splits) runs eagerly.
Timing: CUDA events per step on each rank's stream, 256 MB L2 flush between
steps, barrier + synchronize around the timed region, max over ranks.  The
per-phase device times (p2p: the library's own events around the ready
barrier, the GEMM and the done barrier) come from a second, separate pass of
the same graph, so the timed steps carry no extra event records.

Parity: after timing, rank 0 runs the single-GPU path (ferret_b200.ops) on the
whole global batch with all E experts and compares every 8th (token, slot)
output row of every rank with it, bit for bit.
"""
from __future__ import annotations

import datetime
import os
import statistics

import torch
import torch.distributed as dist

FLUSH_BYTES = 256 << 20
PARITY_STRIDE = 8


def _max(x: float, dev) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum(x: float, dev) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _capture(fn):
    """fn's launches captured as one CUDA graph (a side stream, as torch asks)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            out = fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    return g, out


def _parity(cfg, ids_g, hidden_g, out_local, rank, G, Tl, dev):
    """Every PARITY_STRIDE-th (token, slot) row of every rank's expert-parallel
    output against the single-GPU W13 path on the whole batch (rank 0)."""
    from . import data, ops
    rows_local = torch.arange(0, Tl * cfg.topk, PARITY_STRIDE, device=dev)
    mine = out_local.index_select(0, rows_local).contiguous()
    allv = torch.empty(G * mine.shape[0], mine.shape[1], dtype=mine.dtype, device=dev)
    dist.all_gather_into_tensor(allv, mine)      # bf16 (NCCL has no int16)
    res = None
    if rank == 0:
        W, Ws = data.fp8_weights(cfg.E, cfg.N, cfg.K, device=dev)
        out, rows, _ = ops.fp8_moe_w13(hidden_g.to(dev), ids_g.to(dev), W, Ws, silu=cfg.silu)
        del W, Ws
        R = cfg.T * cfg.topk
        ref = torch.zeros(R, out.shape[1], dtype=out.dtype, device=dev)
        live = rows[:R] >= 0
        ref[rows[:R][live].long()] = out[:R][live]
        sel = torch.cat([g * Tl * cfg.topk + rows_local for g in range(G)])
        want = ref.index_select(0, sel)
        exact = bool(torch.equal(allv.view(torch.int16), want.view(torch.int16)))
        a, b = allv.float(), want.float()
        floor = 1e-3 * float(b.abs().max())
        rel = ((a - b).abs() / torch.clamp(b.abs(), min=floor)).max()
        res = {"checked": True, "rows_checked": int(sel.numel()),
               "against": "single-GPU W13 path (same kernels, all experts on one GPU)",
               "bit_exact": exact, "max_rel": float(rel),
               "finite": bool(torch.isfinite(a).all())}
        del out, ref
        torch.cuda.empty_cache()
    return res


def run(args, cfg):
    import bench  # contract helpers (peaks, clocks, algorithmic bytes, roofline)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    ep = graph = graph_ev = None
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
        place_kind = getattr(args, "placement", None) or "balanced"
        placement = None
        if place_kind == "balanced":
            placement = balanced_placement(torch.bincount(ids_g.reshape(-1), minlength=cfg.E), G)
        table = placement if placement is not None else torch.arange(cfg.E, dtype=torch.int32)
        mine = table[rank * El:(rank + 1) * El]
        # one global weight set (the single-GPU run's), each rank keeping its shard
        W, Ws = data.fp8_weights(cfg.E, cfg.N, cfg.K, device=dev, select=mine.tolist())
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
        if graphed:
            # the whole step -- collectives included -- as one CUDA graph; every
            # rank captures the same sequence of collectives
            graph, out_static = _capture(lambda: ep.forward(hidden, ids))
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
        for i in range(K):
            flush.zero_()
            ev[i][0].record(stream)
            if graph is not None:
                graph.replay()
                out = out_static
            else:
                out = ep.forward(hidden, ids, timers=tm[i])
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        clk = clocks.stop() if clocks else None
        step_list = [a.elapsed_time(b) for a, b in ev]
        step_ms = sum(step_list) / K

        # per-phase device times, from a separate pass
        phases = {}
        if mode == "p2p":
            pev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(5)]
            ep.set_phase_events(pev[1:])
            graph_ev, _ = _capture(lambda: (pev[0].record(), ep.forward(hidden, ids))[1])
            ep.set_phase_events([])
            acc = {"ready_ms": [], "pull_permute_ms": [], "gemm_ms": [], "done_ms": []}
            dist.barrier()
            for i in range(K):
                flush.zero_()
                graph_ev.replay()
                torch.cuda.synchronize()
                for j, key in enumerate(acc):
                    acc[key].append(pev[j].elapsed_time(pev[j + 1]))
            phases = {k: sum(v) / K for k, v in acc.items()}
            graph_ev = None
        else:
            if graph is not None:
                tm_g = StepTimers(torch.cuda.Event(enable_timing=True, external=True),
                                  torch.cuda.Event(enable_timing=True, external=True))
                graph_ev, _ = _capture(lambda: ep.forward(hidden, ids, timers=tm_g))
                g_list = []
                dist.barrier()
                for i in range(K):
                    flush.zero_()
                    graph_ev.replay()
                    torch.cuda.synchronize()
                    g_list.append(tm_g.gemm_start.elapsed_time(tm_g.gemm_end))
                graph_ev = None
            else:
                g_list = [t.gemm_start.elapsed_time(t.gemm_end) for t in tm]
            phases = {"gemm_ms": sum(g_list) / K}
        gemm_ms = phases["gemm_ms"]
        torch.cuda.synchronize()
        dist.barrier()

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
        if graph is not None:
            out = out_static
        status = ep_status = 0
        from . import ops
        ep_status = ops.last_device_status()
        status = int(_max(float(ep_status != 0), dev))
        parity = _parity(cfg, ids_g, hidden_g, out, rank, G, Tl, dev)

        # local GEMM algorithmic bytes and FLOPs (this rank's experts and received rows)
        flat = ids_g.reshape(-1)
        owner_slot = torch.empty(cfg.E, dtype=torch.int64)
        owner_slot[table.long()] = torch.arange(cfg.E)
        loc_counts = torch.bincount(owner_slot[flat.long()], minlength=cfg.E)[rank * El:(rank + 1) * El]
        byts, loc_flops, active = bench.fp8_algorithmic(cfg, loc_counts.tolist())
        R_global = int(flat.numel())
        flops = 2.0 * R_global * cfg.N * cfg.K

        if mode == "p2p":
            # quant, publish, ready, ids, permute (1, or count/scan/scatter),
            # row pull (a kernel of its own unless the prefill GEMM does it), GEMM, done
            from ._lib import lib
            chunked = lib().ferret_moe_permute_workspace_size(G * Tl, cfg.topk, El) > 0
            own = Tl * cfg.topk
            pull_in_gemm = (own + El - 1) // El > 48 and cfg.N % 256 == 0
            launches = 6 + (3 if chunked else 1) + (0 if pull_in_gemm else 1)
        else:
            launches = 4
        max_step = _max(step_ms, dev)
        med_step = _max(statistics.median(step_list), dev)
        max_phase = {k: round(_max(v, dev), 4) for k, v in phases.items()}
        max_e2e = _max(e2e_ms, dev)
        # the slowest rank's GEMM against its own roofline
        t_gemm = _max(gemm_ms, dev)
        slow = _max(float(rank) if gemm_ms >= t_gemm else -1.0, dev)
        pk = bench.peaks()
        prefill = (Tl * cfg.topk + El - 1) // El > 48 and cfg.N % 256 == 0
        kname = "fp8_w13_prefill_ep_kernel" if prefill and mode == "p2p" else \
                "fp8_w13_prefill_kernel" if prefill else "fp8_w13_grouped_kernel"
        rl = bench.roofline(byts, loc_flops, gemm_ms, pk, kname)
        rl_t = torch.tensor([rl["frac"], rl["achieved"], float(byts), loc_flops], dtype=torch.float64,
                            device=dev)
        dist.broadcast(rl_t, src=int(slow))
        sum_active = _sum(float(active), dev)
        max_rows = _max(float(loc_counts.sum()), dev)
        if rank != 0:
            return None
        rl.update({"frac": round(float(rl_t[0]), 4), "achieved": round(float(rl_t[1]), 1),
                   "algorithmic_bytes": int(rl_t[2]), "kernel_ms": round(t_gemm, 4),
                   "kernel": f"{kname} (per-GPU local GEMM, slowest rank {int(slow)})",
                   "traffic": None,
                   "traffic_note": "no ncu capture of a multi-rank run (ncu is single-GPU only here)"})
        rl.pop("hbm_frac", None)
        rl.pop("tensor_frac_fp8", None)
        rl.pop("kernel_tflops", None)
        rl.pop("roofline_frac", None)
        return {
            "metric": "grouped W13 GEMM TFLOPS & HBM GB/s vs roofline",
            "value": round(flops / (max_step * 1e-3) / 1e12, 3),
            "unit": "TFLOPS",
            "n_gpus": G,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": round(max_step, 4),
            "ms_per_step_median": round(med_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "e4m3 x e4m3 -> f32 accumulate, bf16 out; "
                     + ("fp8 dispatch" if mode == "p2p" else "bf16 dispatch"),
            "data": "synthetic (seeded), random-init weights (one global set, sharded by expert)",
            "config": {"workload": cfg.name, "E": cfg.E, "topk": cfg.topk, "tokens": cfg.T,
                       "routed_rows": R_global, "K": cfg.K, "N": cfg.N, "silu": cfg.silu,
                       "routing": cfg.routing,
                       "parallelism": f"ep{G} ({El} experts and {Tl} tokens per GPU, "
                                      f"{place_kind} placement)",
                       "active_experts_total": int(sum_active), "max_rows_per_gpu": int(max_rows),
                       "l2": "256 MB flush between timed steps"},
            "phases_ms": max_phase,
            "roofline": rl,
            "e2e": {"value": round(flops / (max_e2e * 1e-3) / 1e12, 3), "unit": "TFLOPS",
                    "ms_per_step": round(max_e2e, 4),
                    "h2d_bytes_per_step": (h_hidden.numel() * 2 + h_ids.numel() * 4) * G,
                    "d2h_bytes_per_step": h_out.numel() * 2 * G},
            "parity": parity,
            "device_status_ok": status == 0,
            "gpu_launches": launches * K,
            "ep_mode": mode,
            "cuda_graph": graph is not None,
            "clocks": clk,
        }
    finally:
        graph = graph_ev = None   # a graph holding NCCL work must be released before teardown
        torch.cuda.synchronize()
        if ep is not None:
            ep.close()      # collective: peer-memory context (p2p)
        dist.destroy_process_group()
