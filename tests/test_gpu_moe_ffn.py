"""The MoE layer around the W13 path: the top-k weighted combine, and the
whole FP8 expert layer (W13 + SiLU -> quant -> W2 -> combine) against the CPU
restatement.  Bar: combine within one bf16 ulp of an fp32 slot-order sum;
layer max relative error < 1e-2 (denominator max(|ref|, 1e-3 max|ref|)), no NaN."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(scope="module")
def ops(cuda_device):
    from ferret_b200 import ops as _ops
    return _ops


@pytest.mark.parametrize("T,topk,H,E", [(1, 8, 7168, 256), (33, 2, 512, 8), (128, 8, 1024, 16)])
def test_combine(ops, T, topk, H, E):
    rng = np.random.default_rng(T + H)
    y = O.f32_to_bf16(rng.standard_normal((T * topk, H)).astype(np.float32))
    w = rng.random((T, topk)).astype(np.float32)
    ids = rng.integers(-1, E + 1, (T, topk)).astype(np.int32)     # some pairs dropped
    got = ops.moe_combine(torch.from_numpy(y.view(np.int16)).view(torch.bfloat16).cuda(),
                          torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda(), E)
    torch.cuda.synchronize()
    got = O.bf16_to_f32(got.view(torch.int16).cpu().numpy().view(np.uint16))
    yf = O.bf16_to_f32(y).reshape(T, topk, H).astype(np.float64)
    valid = ((ids >= 0) & (ids < E))[:, :, None]
    ref = (np.where(valid, yf, 0.0) * w[:, :, None]).sum(1)
    ulp = np.maximum(np.abs(ref), 1e-30) * 2.0 ** -7
    assert np.all(np.abs(got - ref) <= ulp + 1e-6)


@pytest.mark.parametrize("T,topk,E,H,I", [(64, 2, 8, 512, 256), (16, 8, 32, 1024, 512)])
def test_fp8_moe_ffn_vs_oracle(ops, T, topk, E, H, I):
    from ferret_b200 import data
    g = torch.Generator().manual_seed(T + E)
    w13 = torch.randn(E, 2 * I, H, generator=g) * 0.02
    w2 = torch.randn(E, H, I, generator=g) * 0.02
    w13q, w13s = data.per_block_cast_to_fp8(w13)
    w2q, w2s = data.per_block_cast_to_fp8(w2)
    hidden = data.activations(T, H, seed=T)
    ids = data.routing(T, E, topk, "zipf")
    ids[0, 0] = -1                                     # a dropped pair
    wts = torch.rand(T, topk, generator=g)
    dev = torch.device("cuda")
    got = ops.fp8_moe_ffn(hidden.to(dev), ids.to(dev), wts.to(dev), w13q.to(dev), w13s.to(dev),
                          w2q.to(dev), w2s.to(dev))
    torch.cuda.synchronize()
    assert ops.last_device_status() == 0
    got = O.bf16_to_f32(got.view(torch.int16).cpu().numpy().view(np.uint16))
    ref = O.fp8_moe_ffn(hidden.view(torch.int16).numpy().view(np.uint16), ids.numpy(), wts.numpy(),
                        w13q.view(torch.uint8).numpy(), w13s.numpy(), w2q.view(torch.uint8).numpy(),
                        w2s.numpy())
    err = O.rel_err(got, ref)
    assert err["nan"] == 0 and err["max_rel"] < TOL, err
