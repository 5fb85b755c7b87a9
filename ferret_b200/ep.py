"""Expert parallelism for the W13 path: experts sharded over ranks, tokens
dispatched to the rank that owns their expert and the W13 outputs combined
back to the token's rank, over torch.distributed (NCCL over NVLink on B200;
gloo on CPU for the host-logic tests).

One rank per GPU.  Rank r owns E/G experts (contiguous ids by default, or a
placement table, e.g. the balanced one from ``balanced_placement``) and only
holds their weights.  Three exchange schemes:

* "p2p" (the product path on GPUs; ``PeerContext`` over the library's
  ferret_ep_* entry points): no collective library on the data path.  Each
  rank quantizes its own tokens to FP8 once; the owner of an expert pulls the
  routed FP8 rows from the source rank's memory over NVLink, and the grouped
  GEMM's epilogue stores each output row straight into the source rank's
  output buffer.  Bounded device-side flag barriers replace the collectives;
  no host synchronisation, so a step can be captured in a CUDA graph.

and two over torch.distributed collectives (NCCL on GPUs, gloo on CPU for the
host-logic tests), chosen by batch size under "auto" when "p2p" is not used:

* "a2a" (prefill-sized batches), every step:
  1. remap expert ids to placement order and permute the local (token, slot)
     pairs by expert -- expert-sorted order is also destination-rank order;
  2. all_to_all of the per-expert counts (E ints), one device->host copy of
     the counts to size the variable splits;
  3. dispatch all_to_all of the bf16 token rows;
  4. locally: permute the received rows by local expert, gathered FP8
     quantization, grouped GEMM (the CUDA kernels);
  5. un-permute, combine all_to_all back, scatter into (token, slot) order.
* "gather" (decode-sized batches, no host synchronisation, fixed sizes):
  1. all_gather of every rank's token rows and top-k ids;
  2. locally: keep the pairs routed to this rank's experts, permute, gathered
     FP8 quantization, and the scatter-output grouped GEMM writing each row
     straight into a zeroed (token, slot)-ordered buffer of the whole batch;
  3. reduce_scatter (sum) of that buffer returns each rank its own rows --
     every pair has exactly one non-zero contributor, so the sum is exact.

The reference has no multi-GPU implementation of this path; parity is the
single-GPU result for every (token, slot) pair.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist


class CudaKernels:
    """The product kernels (CUDA library via ferret_b200.ops)."""

    def __init__(self):
        from . import ops
        self.ops = ops

    def permute(self, ids: torch.Tensor, E: int):
        rows, offs, _ = self.ops.moe_permute(ids, E)
        return rows, offs

    def quant(self, x: torch.Tensor, rows: torch.Tensor, div: int):
        return self.ops.per_token_cast_to_fp8(x, rows, div)

    def gemm_scatter(self, q, s, W, Ws, offsets, out_rows, out, silu: bool):
        if q.shape[0]:
            self.ops.m_grouped_fp8_gemm_scatter((q, s), (W, Ws), out, offsets, out_rows, silu=silu)

    def gemm(self, q, s, W, Ws, offsets, silu: bool):
        E, N, _ = W.shape
        out = torch.empty(q.shape[0], N // 2 if silu else N, dtype=torch.bfloat16, device=q.device)
        if q.shape[0]:
            self.ops.m_grouped_fp8_gemm_nt_contiguous((q, s), (W, Ws), out, None,
                                                      expert_offsets=offsets, silu=silu)
        return out


def contiguous_placement(E: int, G: int) -> torch.Tensor:
    """owner-order table: slot i (rank i // (E/G)) holds expert table[i]."""
    return torch.arange(E, dtype=torch.int32)


def balanced_placement(counts: torch.Tensor, G: int) -> torch.Tensor:
    """Expert placement with exactly E/G experts per rank that minimises the
    busiest rank's routed rows.  Greedy LPT first (experts by descending load,
    each to the least-loaded rank that still has room), then pairwise swaps:
    while some swap of an expert of the busiest rank with a lighter expert of
    another rank lowers the larger of the two ranks' loads below the current
    maximum, take the best one.  Under skewed routing one expert can hold most
    of a rank's share; LPT then fills its rank with mid-sized experts, and the
    swaps trade them for the smallest ones.  Returns the owner-order table
    (the experts of rank 0, then rank 1, ...)."""
    E = counts.numel()
    per = E // G
    c = [int(x) for x in counts.tolist()]
    order = sorted(range(E), key=lambda e: -c[e])          # stable: ties by expert id
    load = [0] * G
    slots = [[] for _ in range(G)]
    for e in order:
        r = min((g for g in range(G) if len(slots[g]) < per), key=lambda g: (load[g], g))
        slots[r].append(e)
        load[r] += c[e]
    while G > 1:
        m = max(range(G), key=lambda g: (load[g], -g))
        best = None
        for i, a in enumerate(slots[m]):
            for r in range(G):
                if r == m:
                    continue
                for j, b in enumerate(slots[r]):
                    d = c[a] - c[b]
                    if d <= 0:
                        continue
                    new_max = max(load[m] - d, load[r] + d)
                    if new_max < load[m] and (best is None or new_max < best[0]):
                        best = (new_max, i, r, j, d)
        if best is None:
            break
        _, i, r, j, d = best
        slots[m][i], slots[r][j] = slots[r][j], slots[m][i]
        load[m] -= d
        load[r] += d
    return torch.tensor([e for s in slots for e in sorted(s)], dtype=torch.int32)


class PeerContext:
    """One rank's ferret_ep context: buffers exported to, and mapped from, every
    peer.  Collective: every rank of `group` constructs it with the same sizes.
    The 64-byte CUDA IPC handles are exchanged with all_gather_object."""

    def __init__(self, E: int, topk: int, max_tokens: int, K: int, N: int, flags: int,
                 placement: torch.Tensor | None, group=None):
        from ._lib import check, lib
        self.L = lib()
        self.group = group
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        hb = int(self.L.ferret_ep_handle_bytes())
        handle = (ctypes.c_uint8 * hb)()
        ctx = ctypes.c_void_p()
        pl = None
        if placement is not None:
            self._placement = (ctypes.c_int32 * E)(*[int(x) for x in placement.tolist()])
            pl = ctypes.cast(self._placement, ctypes.c_void_p)
        check(self.L.ferret_ep_init(rank, world, E, topk, max_tokens, K, N, flags, pl,
                                    ctypes.cast(handle, ctypes.c_void_p), ctypes.byref(ctx)),
              "ferret_ep_init")
        self.ctx = ctx
        self.max_tokens = max_tokens
        handles = [bytes(handle)]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
        buf = (ctypes.c_uint8 * (hb * world)).from_buffer_copy(b"".join(handles))
        check(self.L.ferret_ep_connect(ctx, ctypes.cast(buf, ctypes.c_void_p)), "ferret_ep_connect")
        if world > 1:
            dist.barrier(group)

    def output_view(self, rows: int, cols: int) -> torch.Tensor:
        """The context's exported output buffer as a bf16 [rows, cols] tensor
        (no copy; rewritten by the next step)."""
        ptr = self.L.ferret_ep_output_buffer(self.ctx)

        class _Buf:
            __cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<i2",
                                        "data": (ptr, False), "version": 3, "strides": None,
                                        "stream": None}
        return torch.as_tensor(_Buf(), device=torch.cuda.current_device()).view(torch.bfloat16)

    def forward(self, hidden, topk_ids, W, Ws, out=None):
        """One step; `out` None leaves the rows in the context's buffer."""
        from ._lib import check
        T = topk_ids.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"T={T} exceeds the context's max_tokens={self.max_tokens}")
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        check(self.L.ferret_ep_w13_forward(self.ctx, ctypes.c_void_p(hidden.data_ptr()),
                                           ctypes.c_void_p(topk_ids.data_ptr()), T,
                                           ctypes.c_void_p(W.data_ptr()),
                                           ctypes.c_void_p(Ws.data_ptr()),
                                           None if out is None else ctypes.c_void_p(out.data_ptr()),
                                           stream),
              "ferret_ep_w13_forward")
        return out

    def set_events(self, events):
        """Step-phase timing events the library records in every later step
        (ferret_ep_set_events): after the ready barrier, before and after the
        GEMM, after the done barrier.  An empty list turns them off."""
        from ._lib import check
        for e in events:
            e.record()              # torch creates the CUDA event on first record
        torch.cuda.synchronize()
        self._events = list(events)
        arr = (ctypes.c_void_p * 4)(*[ctypes.c_void_p(e.cuda_event) for e in events])
        check(self.L.ferret_ep_set_events(self.ctx, ctypes.cast(arr, ctypes.c_void_p), len(events)),
              "ferret_ep_set_events")

    def close(self):
        """Collective: waits for this rank's work, meets the peers, frees."""
        if self.ctx is None:
            return
        torch.cuda.synchronize()
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.barrier(self.group)
        self.L.ferret_ep_destroy(self.ctx)
        self.ctx = None


@dataclass
class StepTimers:
    """Optional CUDA events recorded around the local GEMM of a step."""
    gemm_start: torch.cuda.Event | None = None
    gemm_end: torch.cuda.Event | None = None


class ExpertParallelW13:
    """W13 forward with experts sharded over the ranks of `group`.

    W_local / Ws_local: this rank's experts, in placement order
    ([E/G, N, K] e4m3 and [E/G, N/128, K/128] f32); `placement` is the
    owner-order table (global expert id of every slot; default identity).
    """

    GATHER_BYTES = 64 << 20    # dense combine buffer above which "auto" uses a2a

    def __init__(self, W_local, Ws_local, E: int, group=None, silu: bool = False,
                 placement: torch.Tensor | None = None, kernels=None, mode: str = "auto",
                 max_tokens: int | None = None):
        if mode not in ("auto", "a2a", "gather", "p2p"):
            raise ValueError(mode)
        self.mode = mode
        self.group = group
        self.G = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if E % self.G:
            raise ValueError(f"E={E} must be divisible by the world size {self.G}")
        self.E, self.El = E, E // self.G
        if W_local.shape[0] != self.El:
            raise ValueError(f"W_local holds {W_local.shape[0]} experts, expected {self.El}")
        self.W, self.Ws, self.silu = W_local, Ws_local, silu
        self.kernels = kernels or CudaKernels()
        dev = W_local.device
        if placement is None:
            self.remap = None
        else:
            # global expert id -> slot in owner order
            inv = torch.empty(E, dtype=torch.int32)
            inv[placement.long()] = torch.arange(E, dtype=torch.int32)
            self.remap = inv.to(dev)
        self.loc_pattern = torch.arange(self.El, dtype=torch.int32, device=dev).repeat(self.G)
        self.placement = placement
        self.max_tokens = max_tokens
        self.peer = None
        if mode == "p2p" and not (W_local.is_cuda and isinstance(self.kernels, CudaKernels)):
            raise ValueError("mode 'p2p' runs the CUDA library on GPU-resident weights")

    def set_phase_events(self, events):
        """Mode "p2p": up to 4 timing events recorded inside every later step
        (after the ready barrier, before and after the GEMM, after the done
        barrier).  Needs a first step to have created the peer context."""
        if self.peer is None:
            raise RuntimeError("set_phase_events needs the p2p context (run a step first)")
        self.peer.set_events(events)

    def close(self):
        """Collective: releases the peer-memory context (mode "p2p")."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        if self.G == 1:
            out.copy_(inp)
            return
        if out.dtype == torch.bfloat16:
            # a pure byte copy: move bf16 rows as uint8 so every backend takes them
            out = out.view(torch.uint8)
            inp = inp.view(torch.uint8)
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, hidden: torch.Tensor, topk_ids: torch.Tensor,
                timers: StepTimers | None = None) -> torch.Tensor:
        """hidden bf16 [T, K], topk_ids int32 [T, topk] (global expert ids) ->
        bf16 [T*topk, N or N/2] in (token, slot) order; pairs with an invalid
        expert id get zero rows.  Every rank passes the same T.  In mode "p2p"
        the result is a view of the context's output buffer, valid until the
        next forward (work queued on the current stream in between reads it
        safely: peers write the next step's rows only after this rank's next
        step has started)."""
        T, topk = topk_ids.shape
        N = self.W.shape[1]
        n_out = N // 2 if self.silu else N
        mode = self.mode
        if mode == "p2p":
            return self._forward_p2p(hidden, topk_ids, timers)
        if mode == "auto":
            mode = "gather" if self.G * T * topk * n_out * 2 <= self.GATHER_BYTES else "a2a"
        if mode == "gather":
            return self._forward_gather(hidden, topk_ids, timers)
        return self._forward_a2a(hidden, topk_ids, timers)

    def _forward_p2p(self, hidden, topk_ids, timers):
        from ._lib import FERRET_SILU_MUL
        T, topk = topk_ids.shape
        K = hidden.shape[1]
        N = self.W.shape[1]
        if self.peer is None:
            self.peer = PeerContext(self.E, topk, self.max_tokens or T, K, N,
                                    FERRET_SILU_MUL if self.silu else 0, self.placement, self.group)
        if timers is not None and timers.gemm_start is not None:
            timers.gemm_start.record()
        self.peer.forward(hidden.contiguous(), topk_ids.contiguous(), self.W, self.Ws)
        if timers is not None and timers.gemm_end is not None:
            timers.gemm_end.record()
        # zero-copy: the rows stay in the exported buffer until the next step
        return self.peer.output_view(T * topk, N // 2 if self.silu else N)

    def _remap(self, ids: torch.Tensor) -> torch.Tensor:
        if self.remap is None:
            return ids
        valid = (ids >= 0) & (ids < self.E)
        return torch.where(valid, self.remap[ids.clamp(0, self.E - 1).long()], -1).to(torch.int32)

    def _forward_gather(self, hidden, topk_ids, timers):
        T, topk = topk_ids.shape
        K = hidden.shape[1]
        N = self.W.shape[1]
        n_out = N // 2 if self.silu else N
        dev = hidden.device
        ids = self._remap(topk_ids).contiguous()
        if self.G > 1:
            all_h = torch.empty(self.G * T, K, dtype=hidden.dtype, device=dev)
            dist.all_gather_into_tensor(all_h.view(torch.uint8), hidden.contiguous().view(torch.uint8),
                                        group=self.group)
            all_ids = torch.empty(self.G * T, topk, dtype=torch.int32, device=dev)
            dist.all_gather_into_tensor(all_ids, ids, group=self.group)
        else:
            all_h, all_ids = hidden, ids
        loc = all_ids - self.rank * self.El
        local = torch.where((all_ids >= 0) & (loc >= 0) & (loc < self.El), loc, -1).to(torch.int32)
        rows, offs = self.kernels.permute(local.contiguous(), self.El)
        q, s = self.kernels.quant(all_h, rows, topk)
        dense = torch.zeros(self.G * T * topk, n_out, dtype=torch.bfloat16, device=dev)
        if timers is not None and timers.gemm_start is not None:
            timers.gemm_start.record()
        self.kernels.gemm_scatter(q, s, self.W, self.Ws, offs, rows, dense, self.silu)
        if timers is not None and timers.gemm_end is not None:
            timers.gemm_end.record()
        if self.G == 1:
            return dense
        out = torch.empty(T * topk, n_out, dtype=torch.bfloat16, device=dev)
        dist.reduce_scatter_tensor(out, dense, group=self.group)
        return out

    def _forward_a2a(self, hidden, topk_ids, timers):
        T, topk = topk_ids.shape
        K = hidden.shape[1]
        N = self.W.shape[1]
        n_out = N // 2 if self.silu else N
        dev = hidden.device
        ids = self._remap(topk_ids)
        rows, offs = self.kernels.permute(ids.contiguous(), self.E)
        counts = (offs[1:] - offs[:-1]).contiguous()
        recv_counts = torch.empty_like(counts)
        self._a2a(recv_counts, counts)
        both = torch.cat([counts, recv_counts]).cpu()          # the one host sync
        send_splits = both[: self.E].view(self.G, self.El).sum(1).tolist()
        recv_splits = both[self.E:].view(self.G, self.El).sum(1).tolist()
        Rv, Rr = sum(send_splits), sum(recv_splits)

        sel = rows[:Rv].long()
        send = hidden.index_select(0, sel // topk)
        recv = torch.empty(Rr, K, dtype=hidden.dtype, device=dev)
        self._a2a(recv, send, recv_splits, send_splits)

        loc_ids = torch.repeat_interleave(self.loc_pattern, recv_counts.to(torch.int64),
                                          output_size=Rr).view(Rr, 1)
        rows2, offs2 = self.kernels.permute(loc_ids.contiguous(), self.El)
        q, s = self.kernels.quant(recv, rows2, 1)
        if timers is not None and timers.gemm_start is not None:
            timers.gemm_start.record()
        out2 = self.kernels.gemm(q, s, self.W, self.Ws, offs2, self.silu)
        if timers is not None and timers.gemm_end is not None:
            timers.gemm_end.record()
        back = torch.empty_like(out2)
        back.index_copy_(0, rows2[:Rr].long(), out2)
        ret = torch.empty(Rv, n_out, dtype=out2.dtype, device=dev)
        self._a2a(ret, back, send_splits, recv_splits)
        out = torch.zeros(T * topk, n_out, dtype=ret.dtype, device=dev)
        out.index_copy_(0, sel, ret)
        return out
