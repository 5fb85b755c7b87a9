"""Expert parallelism on 2 GPUs (NCCL): every (token, slot) output equals the
single-GPU W13 path on the same inputs, bit for bit.  Skips on a 1-GPU box."""
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


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from ferret_b200 import data, ops
        from ferret_b200.ep import ExpertParallelW13, balanced_placement
        E, N, K, T, topk = 16, 512, 512, 64, 4
        W, Ws = data.fp8_weights(E, N, K, device=dev)
        hidden = data.activations(T, K).to(dev)
        ids = data.routing(T, E, topk, "zipf").to(dev)
        # single-GPU result on every rank, (token, slot) order
        out, rows, _ = ops.fp8_moe_w13(hidden, ids, W, Ws)
        ref = torch.empty_like(out)
        ref[rows.long()] = out
        cases = [(p, m) for p in (None, balanced_placement(torch.bincount(ids.reshape(-1).cpu(), minlength=E), world))
                 for m in ("a2a", "gather")]
        for placement, mode in cases:
            table = placement if placement is not None else torch.arange(E)
            El, Tl = E // world, T // world
            mine = table[rank * El:(rank + 1) * El].long().to(dev)
            ep = ExpertParallelW13(W[mine].contiguous(), Ws[mine].contiguous(), E, placement=placement,
                                   mode=mode)
            got = ep.forward(hidden[rank * Tl:(rank + 1) * Tl].contiguous(),
                             ids[rank * Tl:(rank + 1) * Tl].contiguous())
            torch.cuda.synchronize()
            want = ref[rank * Tl * topk:(rank + 1) * Tl * topk]
            ok = torch.equal(got.view(torch.int16), want.view(torch.int16))
            flag = torch.tensor([1 if ok else 0], device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            if rank == 0:
                q.put(bool(flag.item()))
    except Exception as e:
        q.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_matches_single_gpu(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(4)]
    for p in procs:
        p.join(timeout=120)
    assert all(r is True for r in results), results
    assert all(p.exitcode == 0 for p in procs)
