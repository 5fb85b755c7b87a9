"""Expert parallelism on 2 GPUs: every (token, slot) output equals the
single-GPU W13 path on the same inputs, bit for bit -- for the NCCL exchange
modes ("a2a", "gather") and for the peer-memory mode ("p2p", the library's
ferret_ep_* entry points), eagerly and replayed from a CUDA graph.  A second
test checks that a p2p step whose peer never arrives ends with a bounded
device timeout instead of a hang.  Skips on a 1-GPU box."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    return dev


def _all_true(ok, dev):
    import torch.distributed as dist
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


def _worker(rank, world, port, q):
    import torch.distributed as dist
    dev = _init(rank, world, port)
    try:
        from ferret_b200 import data, ops
        from ferret_b200.ep import ExpertParallelW13, balanced_placement
        E, N, K, T, topk = 16, 512, 512, 64, 4
        W, Ws = data.fp8_weights(E, N, K, device=dev)
        hidden = data.activations(T, K).to(dev)
        ids = data.routing(T, E, topk, "zipf").to(dev)
        ids[3, 1] = -1            # a dropped pair: zero row in every mode
        ids[T - 1, 0] = E + 5
        refs = {}
        for silu in (False, True):
            out, rows, _ = ops.fp8_moe_w13(hidden, ids, W, Ws, silu=silu)
            ref = torch.zeros(T * topk, out.shape[1], dtype=out.dtype, device=dev)
            live = rows >= 0
            ref[rows[live].long()] = out[live]
            refs[silu] = ref
        bal = balanced_placement(torch.bincount(ids.reshape(-1).clamp(0, E - 1).cpu(), minlength=E), world)
        cases = [(p, m, False) for p in (None, bal) for m in ("a2a", "gather", "p2p")]
        cases += [(None, "p2p", True), (bal, "p2p", True)]
        cases += [("big", "p2p", False), ("big", "p2p", True)]   # prefill kernel, peer stores
        # a batch large enough (> 48 rows per local expert) for the prefill kernel
        # (its GEMM pulls the rows from the peers itself); consecutive steps
        # alternate between two token batches, so a tile that read rows left
        # over from the previous step would show
        Tb = 1024
        ids_b = data.routing(Tb, E, topk, "zipf").to(dev)
        hidden_bs = [data.activations(Tb, K, seed=sd).to(dev) for sd in (11, 12)]
        refs_bs = []
        for hb in hidden_bs:
            refs_b = {}
            for silu in (False, True):
                out, rows, _ = ops.fp8_moe_w13(hb, ids_b, W, Ws, silu=silu)
                ref = torch.zeros(Tb * topk, out.shape[1], dtype=out.dtype, device=dev)
                ref[rows.long()] = out
                refs_b[silu] = ref
            refs_bs.append(refs_b)
        El = E // world
        results = []
        for placement, mode, silu in cases:
            big = isinstance(placement, str)
            if big:
                placement = None
            Tn, hids, ids_n, refs_l = ((Tb, hidden_bs, ids_b, refs_bs) if big
                                       else (T, [hidden], ids, [refs]))
            Tl = Tn // world
            h_locs = [h[rank * Tl:(rank + 1) * Tl].contiguous() for h in hids]
            i_loc = ids_n[rank * Tl:(rank + 1) * Tl].contiguous()
            table = placement if placement is not None else torch.arange(E)
            mine = table[rank * El:(rank + 1) * El].long().to(dev)
            ep = ExpertParallelW13(W[mine].contiguous(), Ws[mine].contiguous(), E, placement=placement,
                                   mode=mode, silu=silu, max_tokens=2 * Tl)
            wants = [r[silu][rank * Tl * topk:(rank + 1) * Tl * topk] for r in refs_l]
            steps = 3 if mode == "p2p" else 1      # several epochs through one context
            ok = True
            for i in range(steps):
                got = ep.forward(h_locs[i % len(h_locs)], i_loc)
                torch.cuda.synchronize()
                ok = ok and torch.equal(got.view(torch.int16), wants[i % len(wants)].view(torch.int16))
            h_loc, want = h_locs[0], wants[0]
            if mode == "p2p" and silu:
                # the same step replayed from a CUDA graph
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                g = torch.cuda.CUDAGraph()
                with torch.cuda.stream(side):
                    with torch.cuda.graph(g, stream=side):
                        got_g = ep.forward(h_loc, i_loc)
                torch.cuda.current_stream().wait_stream(side)
                for _ in range(2):
                    got_g.zero_()
                    g.replay()
                    torch.cuda.synchronize()
                    ok = ok and torch.equal(got_g.view(torch.int16), want.view(torch.int16))
                del g
            ok = ok and ops.last_device_status() == 0
            ep.close()
            results.append(_all_true(ok, dev))
        if rank == 0:
            q.put(results)
    except Exception as e:
        q.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


def _run(worker, world=2, timeout=300):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=timeout)
    for p in procs:
        p.join(timeout=120)
    return res, [p.exitcode for p in procs]


def test_ep_two_gpus_matches_single_gpu(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res, codes = _run(_worker)
    assert isinstance(res, list) and len(res) == 10 and all(res), res
    assert all(c == 0 for c in codes)


def _timeout_worker(rank, world, port, q):
    """Step 1 runs on both ranks; in step 2 rank 1 stays on the host (alive,
    its buffers mapped), so rank 0's ready barrier must give up after the
    wait timeout and report it through the status word."""
    import torch.distributed as dist
    dev = _init(rank, world, port)
    try:
        from ferret_b200 import data, ops
        from ferret_b200.ep import ExpertParallelW13
        E, N, K, T, topk = 8, 256, 256, 8, 2
        W, Ws = data.fp8_weights(E, N, K, device=dev)
        El, Tl = E // world, T // world
        hidden = data.activations(T, K)[rank * Tl:(rank + 1) * Tl].contiguous().to(dev)
        ids = data.routing(T, E, topk, "uniform")[rank * Tl:(rank + 1) * Tl].contiguous().to(dev)
        ep = ExpertParallelW13(W[rank * El:(rank + 1) * El].contiguous(),
                               Ws[rank * El:(rank + 1) * El].contiguous(), E, mode="p2p")
        ep.forward(hidden, ids)
        torch.cuda.synchronize()
        ok1 = ops.last_device_status() == 0
        dist.barrier()
        status = 0
        if rank == 0:
            ops.set_wait_timeout(0.2)
            ep.forward(hidden, ids)          # rank 1 never arrives
            torch.cuda.synchronize()
            status = ops.last_device_status()
            ops.set_wait_timeout(2.0)
        dist.barrier()                       # rank 1 keeps its buffers until rank 0 is done
        ep.close()
        if rank == 0:
            q.put((ok1, status))
    except Exception as e:
        q.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


def test_ep_p2p_missing_peer_times_out(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res, codes = _run(_timeout_worker)
    assert isinstance(res, tuple), res
    ok1, status = res
    assert ok1
    # DEV_TIMEOUT (1) from the ready barrier (site 20) or the done barrier (21)
    assert status & 0xFF == 1 and (status >> 8) in (20, 21), hex(status)
    assert all(c == 0 for c in codes)
