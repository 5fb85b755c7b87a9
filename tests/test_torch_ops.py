"""The operator form of the library: torch.ops.ferret_moe.* registered with
the baselines' tensor signatures (CPU: schemas; GPU: same results as ops)."""
import numpy as np
import pytest
import torch

import ferret_b200.torch_ops  # noqa: F401  (registers torch.ops.ferret_moe)


def test_schemas_registered():
    s = str(torch.ops.ferret_moe.fp8_grouped_gemm_nt_contiguous.default._schema)
    assert "Tensor(a!) out" in s and "Tensor m_indices" in s and "bool silu=False" in s
    assert "bool disable_ue8m0_cast=True" in s
    assert "bool use_ue8m0=False" in str(torch.ops.ferret_moe.per_token_cast_to_fp8.default._schema)
    for name in ("per_token_cast_to_fp8", "moe_align_block_size", "int4_moe_w13"):
        assert hasattr(torch.ops.ferret_moe, name)


@pytest.mark.gpu
def test_ops_match_python_api(cuda_device):
    from ferret_b200 import data, ops
    dev = torch.device("cuda")
    E, N, K, T, topk = 8, 512, 512, 32, 2
    W, Ws = data.fp8_weights(E, N, K, device=dev)
    hidden = data.activations(T, K).to(dev)
    ids = data.routing(T, E, topk).to(dev)
    q, s = torch.ops.ferret_moe.per_token_cast_to_fp8(hidden)
    q2, s2 = ops.per_token_cast_to_fp8(hidden)
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s, s2)
    rows, offs, mi = ops.moe_permute(ids, E)
    a, a_s = ops.per_token_cast_to_fp8(hidden, rows, topk)
    out1 = torch.empty(T * topk, N, dtype=torch.bfloat16, device=dev)
    out2 = torch.empty_like(out1)
    torch.ops.ferret_moe.fp8_grouped_gemm_nt_contiguous(a, a_s, W, Ws, out1, mi)
    ops.m_grouped_fp8_gemm_nt_contiguous((a, a_s), (W, Ws), out2, mi)
    torch.cuda.synchronize()
    assert torch.equal(out1.view(torch.int16), out2.view(torch.int16))
    qu, su = torch.ops.ferret_moe.per_token_cast_to_fp8(hidden, True)
    qv, sv = ops.per_token_cast_to_fp8(hidden, use_ue8m0=True)
    assert torch.equal(qu.view(torch.uint8), qv.view(torch.uint8)) and torch.equal(su, sv)
    si, ei, ni = torch.ops.ferret_moe.moe_align_block_size(ids, 16, E)
    sj, ej, nj = ops.moe_align_block_size(ids, 16, E)
    assert torch.equal(si, sj) and torch.equal(ei, ej) and torch.equal(ni, nj)
    raw, sc = data.int4_weights(E, N, K, device=dev)
    r1 = torch.ops.ferret_moe.int4_moe_w13(hidden, raw, sc, ids, True)
    r2 = ops.moe_wna16_w13(hidden, ops.Int4W13Weights(raw, sc), ids, silu=True)
    torch.cuda.synchronize()
    assert torch.equal(r1.view(torch.int16), r2.view(torch.int16))
    assert np.isfinite(r1.float().cpu().numpy()).all()
