"""GPU parity of the UE8M0 (power-of-two scale) form of the FP8 W13 path.

The quantizer's use_ue8m0 mode must be bit-exact against the CPU oracle.  The
GEMM with FERRET_UE8M0_SCALES (plain 128-token tiles: the block-scaled kernel,
tcgen05.mma kind::mxf8f6f4.block_scale; with SiLU: the exact-scale kernel)
must match the fp32 oracle within max relative error < 1e-2 (denominator
max(|ref|, 1e-3 max|ref|), no NaN, every row) -- power-of-two scales are exact
in both, so the kernels differ only in fp32 summation order -- and the
block-scaled kernel must agree with the exact-scale kernel on the same inputs.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from test_gpu_fp8 import BF16_NAN, TOL, check, make_case, u8, u16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda_device):
    from ferret_b200 import ops as _ops
    return _ops


@pytest.mark.parametrize("R,K", [(1, 128), (37, 512), (1024, 7168)])
def test_quant_ue8m0_bit_exact(ops, R, K):
    g = torch.Generator().manual_seed(R + 11)
    x = (torch.randn(R, K, generator=g) * torch.logspace(-5, 2, R).unsqueeze(1)).to(torch.bfloat16)
    x[0, :128] = 0
    if R > 1:
        x[1, :128] = 56.0          # amax / 448 = 1/8 exactly: no rounding up
    q, s = ops.per_token_cast_to_fp8(x.cuda(), use_ue8m0=True)
    qr, sr = O.quant_act_fp8_1x128(u16(x), ue8m0=True)
    assert np.array_equal(u8(q), qr)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))
    assert (s.view(torch.int32) & 0x7FFFFF == 0).all()


def test_quant_ue8m0_gather_bit_exact(ops):
    g = torch.Generator().manual_seed(5)
    T, topk, K = 33, 4, 1024
    x = torch.randn(T, K, generator=g).to(torch.bfloat16)
    rows = torch.randperm(T * topk, generator=g).to(torch.int32)
    rows[-5:] = -1
    q, s = ops.per_token_cast_to_fp8(x.cuda(), rows.cuda(), topk, use_ue8m0=True)
    qr, sr = O.quant_act_fp8_1x128(u16(x), rows.numpy(), topk, ue8m0=True)
    assert np.array_equal(u8(q), qr)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))


def run(ops, a, a_s, w, w_s, mi, silu, ue8m0, use_offsets, pairs=False):
    M, K = a.shape
    E, N, _ = w.shape
    out = torch.full((M, N // 2 if silu else N), BF16_NAN, dtype=torch.int16).view(torch.bfloat16).cuda()
    offs = None
    if use_offsets:
        offs = torch.from_numpy(np.concatenate([[0], np.cumsum(np.bincount(mi, minlength=E))])
                                .astype(np.int32)).cuda()
    ops.m_grouped_fp8_gemm_nt_contiguous(
        (torch.from_numpy(a).cuda(), torch.from_numpy(a_s).cuda()),
        (torch.from_numpy(w).cuda(), torch.from_numpy(w_s).cuda()),
        out, None if use_offsets else torch.from_numpy(mi).cuda(),
        disable_ue8m0_cast=not ue8m0, expert_offsets=offs, silu=silu, tile=128,
        prefill_pairs=pairs)
    torch.cuda.synchronize()
    assert ops.last_device_status() == 0
    return out


CASES = [
    # (seg_counts, N, K, pad, silu)
    ([300, 129, 2, 0, 77], 512, 384, 0, False),
    ([300, 129, 2, 0, 77], 512, 384, 0, True),
    ([40, 40, 40, 40], 256, 128, 5, False),         # one K block, padding rows
    ([1000], 256, 256, 0, True),
    ([5, 100, 127, 128, 129], 256, 384, 0, False),
    ([200, 300], 512, 7168, 0, False),              # 56 K blocks: the scale ring wraps 7 times
    ([200, 300], 512, 7168, 0, True),
    ([1500] * 4, 1024, 1024, 0, False),             # 192 tiles: CTAs reuse the accumulator
    ([130, 3], 256, 16384, 0, False),               # the K limit: 128 K blocks
]


@pytest.mark.parametrize("seg,N,K,pad,silu", CASES)
@pytest.mark.parametrize("use_offsets", [False, True])
def test_ue8m0_gemm_vs_oracle(ops, seg, N, K, pad, silu, use_offsets):
    if use_offsets and pad:
        pytest.skip("offsets describe unpadded layouts")
    a, a_s, w, w_s, mi = make_case(hash((tuple(seg), N, K, 8)) & 0xFFFF, seg, N, K, pad,
                                   scale_kind="pow2")
    out = run(ops, a, a_s, w, w_s, mi, silu, True, use_offsets)
    ref = O.fp8_grouped_gemm(a, a_s, w, w_s, mi, silu=silu)
    check(out, ref, mi)


def test_ue8m0_gemm_agrees_with_exact_scale_kernel(ops):
    """Same power-of-two inputs through both kernels: equal up to the last
    bf16 rounding (fp32 summation order differs)."""
    a, a_s, w, w_s, mi = make_case(77, [700, 0, 260, 513], 512, 2048, 0, scale_kind="pow2")
    mx = O.bf16_to_f32(u16(run(ops, a, a_s, w, w_s, mi, False, True, False)))
    ex = O.bf16_to_f32(u16(run(ops, a, a_s, w, w_s, mi, False, False, False)))
    err = O.rel_err(mx, ex)
    assert err["nan"] == 0 and err["max_rel"] <= 2 ** -7, err      # one bf16 ulp


@pytest.mark.parametrize("seg,N,K", [
    ([600, 0, 256, 255, 1000, 3], 512, 512),
    ([1024], 256, 7168),
    ([513, 770], 1024, 384),
    ([100, 37], 256, 256),                          # no whole 256-row chunk
])
@pytest.mark.parametrize("use_offsets", [False, True])
def test_ue8m0_gemm_cta_pairs(ops, seg, N, K, use_offsets):
    """Block-scaled CTA-pair kernel (tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale)
    on whole 256-row chunks plus the single-CTA block-scaled kernel on the
    rest: against the fp32 oracle, and within one bf16 ulp of the single-CTA
    block-scaled kernel alone."""
    a, a_s, w, w_s, mi = make_case(hash((tuple(seg), N, K, 9)) & 0xFFFF, seg, N, K, 0,
                                   scale_kind="pow2")
    out = run(ops, a, a_s, w, w_s, mi, False, True, use_offsets, pairs=True)
    check(out, O.fp8_grouped_gemm(a, a_s, w, w_s, mi), mi)
    single = run(ops, a, a_s, w, w_s, mi, False, True, use_offsets)
    err = O.rel_err(O.bf16_to_f32(u16(out)), O.bf16_to_f32(u16(single)))
    assert err["nan"] == 0 and err["max_rel"] <= 2 ** -7, err


def test_w13_path_ue8m0_prefill_full_size(ops):
    """Benchmark configuration 3 (E=256, top-8 Zipf(1.1), 8192 tokens) with
    UE8M0 weights and activations: the expert-sorted FP8 rows and scales
    (quantize once + row gather) bit-exact against the oracle quantizer, and
    every row of 6 sampled experts (the largest among them) against the fp32
    oracle, plain and fused SiLU."""
    from ferret_b200 import data
    cfg = data.CONFIGS["dsv3_prefill"]
    dev = torch.device("cuda")
    W, Ws = data.fp8_weights(cfg.E, cfg.N, cfg.K, device=dev, use_ue8m0=True)
    assert (Ws.view(torch.int32) & 0x7FFFFF == 0).all()
    hidden = data.activations(cfg.T, cfg.K)
    ids = data.routing(cfg.T, cfg.E, cfg.topk, "zipf")
    r_rows, r_offs, _ = O.moe_permute(ids.numpy(), cfg.E)
    counts = np.diff(r_offs)
    experts = [int(np.argmax(counts))] + list(np.random.default_rng(3).choice(
        np.nonzero(counts)[0], 5, replace=False))
    qo, so = O.quant_act_fp8_1x128(u16(hidden), r_rows, cfg.topk, ue8m0=True)
    for silu in (False, True):
        bufs = ops.W13Buffers(cfg.T, cfg.topk, cfg.K, cfg.N // 2 if silu else cfg.N, cfg.E, dev)
        out, rows, offs = ops.fp8_moe_w13(hidden.cuda(), ids.cuda(), W, Ws, silu=silu,
                                          bufs=bufs, use_ue8m0=True)
        torch.cuda.synchronize()
        assert np.array_equal(offs.cpu().numpy(), r_offs)
        assert np.array_equal(rows.cpu().numpy(), r_rows)
        assert np.array_equal(u8(bufs.a), qo)
        assert np.array_equal(bufs.a_scale.cpu().numpy().view(np.uint32), so.view(np.uint32))
        got = O.bf16_to_f32(u16(out))
        for e in experts:
            r0, r1 = r_offs[e], r_offs[e + 1]
            ref = O.fp8_grouped_gemm_fast(qo[r0:r1], so[r0:r1], u8(W[e:e + 1]),
                                          Ws[e:e + 1].cpu().numpy(),
                                          np.zeros(r1 - r0, np.int32), silu=silu)
            err = O.rel_err(got[r0:r1], ref)
            assert err["nan"] == 0 and err["max_rel"] < TOL, (silu, int(e), err)
    assert ops.last_device_status() == 0
