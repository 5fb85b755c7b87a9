"""Block-padded routing layout (vLLM's moe_align_block_size with
ignore_invalid_experts=True, baselines/kimi-moe-w13-int4/baseline_marlin.py:123-126):
bit-exact against the CPU restatement, and -- where vLLM's own op loads on the
box -- the same block experts, padded length and pairs per expert as vLLM
(vLLM's order inside an expert differs: ours is the ascending flat index)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda_device):
    from ferret_b200 import ops as _ops
    return _ops


CASES = [
    (4, 3, 4, 4, 0, 4),          # (T, topk, E, block, lo, hi)
    (1, 8, 384, 16, 0, 384),     # fewer pairs than experts
    (64, 8, 384, 16, 0, 384),    # the Kimi decode batch
    (128, 8, 256, 64, -1, 257),  # dropped ids at both ends
    (7, 2, 5, 1, 0, 5),          # block 1: no padding
    (4096, 8, 32, 16, 0, 32),    # chunked permutation underneath
]


@pytest.mark.parametrize("T,topk,E,bs,lo,hi", CASES)
def test_align_block_size_bit_exact(ops, T, topk, E, bs, lo, hi):
    rng = np.random.default_rng(T * 31 + E)
    ids = rng.integers(lo, hi, size=(T, topk)).astype(np.int32)
    s, e, n = ops.moe_align_block_size(torch.from_numpy(ids).cuda(), bs, E)
    rs, re_, rn = O.moe_align_block_size(ids, E, bs)
    assert np.array_equal(n.cpu().numpy(), rn)
    assert np.array_equal(e.cpu().numpy(), re_)
    assert np.array_equal(s.cpu().numpy(), rs)


def test_align_block_size_matches_vllm_sets(ops):
    try:
        from vllm.model_executor.layers.fused_moe.moe_align_block_size import (
            moe_align_block_size as vllm_align)
    except Exception as exc:          # vLLM or its compiled ops unavailable here
        pytest.skip(f"vLLM moe_align_block_size not importable: {type(exc).__name__}")
    rng = np.random.default_rng(5)
    for T, topk, E, bs in ((1, 8, 384, 16), (64, 8, 384, 16), (256, 8, 64, 16)):
        ids = torch.from_numpy(rng.integers(0, E, size=(T, topk)).astype(np.int32)).cuda()
        try:
            vs, ve, vn = vllm_align(ids, bs, E, ignore_invalid_experts=True)
        except Exception as exc:
            pytest.skip(f"vLLM op failed to run: {type(exc).__name__}")
        s, e, n = ops.moe_align_block_size(ids, bs, E)
        total = int(n.item())
        assert total == int(vn.item()), (T, total, int(vn.item()))
        e, ve = e.cpu().numpy(), ve.cpu().numpy()
        assert len(e) == len(ve) and len(s) == len(vs), (len(e), len(ve), len(s), len(vs))
        assert np.array_equal(e[: total // bs], ve[: total // bs]), (T, e[:8], ve[:8])
        s, vs = s.cpu().numpy(), vs.cpu().numpy()
        blk = np.repeat(e[: total // bs], bs)
        for x in np.unique(blk):              # same pairs per expert (order inside is vLLM's own)
            mine, theirs = s[:total][blk == x], vs[:total][blk == x]
            assert np.array_equal(np.sort(mine), np.sort(theirs)), (T, int(x))
