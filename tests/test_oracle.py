"""CPU tests of the oracle: pinned against the reference's own code.

* fp8_v007_ref.npz holds the output of the reference's FP8 host reference
  cpu_ref_bs (examples/fp8-group-gemm/v007_dsv3_decode_verified_105.cu:441-467),
  compiled unmodified; the oracle must match it bit for bit.
* int4_ref_small.npz / int4_ref_kimi.npz hold outputs of the reference's
  fp32_oracle_w13_silu (correctness/compare_marlin_vs_ref.py:44-100).
Fixtures are produced by tests/golden/make_golden.py.
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_fp8_matches_reference_cpu_ref_bs_bit_exact():
    d = np.load(os.path.join(GOLD, "fp8_v007_ref.npz"))
    out = O.fp8_grouped_gemm(d["a"], d["a_scale"], d["w"], d["w_scale"], d["m_indices"])
    assert out.shape == d["out"].shape
    assert np.array_equal(out.view(np.uint32), d["out"].view(np.uint32))


def test_fp8_fast_oracle_close_to_reference():
    d = np.load(os.path.join(GOLD, "fp8_v007_ref.npz"))
    fast = O.fp8_grouped_gemm_fast(d["a"], d["a_scale"], d["w"], d["w_scale"], d["m_indices"])
    assert O.rel_err(fast, d["out"])["max_rel"] < 1e-4


def test_int4_matches_reference_oracle_small_bit_exact():
    d = np.load(os.path.join(GOLD, "int4_ref_small.npz"))
    out = O.int4_w13(d["hidden"], d["raw_q"], d["scales"], d["topk_ids"], silu=True)
    assert np.array_equal(O.f32_to_bf16(out), d["out"])


def test_int4_matches_reference_oracle_kimi_shape():
    import sys
    sys.path.insert(0, GOLD)
    import make_golden as G
    k = np.load(os.path.join(GOLD, "int4_ref_kimi.npz"))
    T, E, K, N, topk = (int(x) for x in k["shape"])
    h, rq, sc, ids = G.int4_inputs(int(k["seed"]), T, E, K, N, topk)
    assert G.digest(h, rq, sc, ids) == str(k["sha256"]), "input regeneration drifted"
    out = O.f32_to_bf16(O.int4_w13(h, rq, sc, ids, silu=True))
    ref = k["out"]
    # fp32 summation order differs from torch's matvec: allow rare 1-ulp flips
    diff = np.abs(out.astype(np.int32) - ref.astype(np.int32))
    assert diff.max() <= 1 and np.count_nonzero(diff) <= ref.size // 200
    assert O.rel_err(O.bf16_to_f32(out), O.bf16_to_f32(ref))["max_rel"] < 1e-2
    fast = O.int4_w13_fast(h, rq, sc, ids, silu=True)
    assert O.rel_err(fast, O.bf16_to_f32(ref))["max_rel"] < 1e-2


def test_e4m3_conversion_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                        for s in (1e-4, 1e-2, 1, 100)] +
                       [np.array([0, -0.0, 448, -448, 2**-10, 2**-9 * 1.5, 2**-6, 464 - 1e-3],
                                 np.float32)])
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.f32_to_e4m3(x), ref)
    lut = O.e4m3_lut()
    tl = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    same = (lut == tl) | (np.isnan(lut) & np.isnan(tl))
    assert same.all()


def _dg_per_token_cast(x: torch.Tensor):
    """The published per_token_cast_to_fp8 algorithm (use_ue8m0=False) in torch."""
    m, n = x.shape
    v = x.view(m, -1, 128)
    amax = v.abs().float().amax(dim=2).view(m, -1).clamp(1e-4)
    q = (v * (448.0 / amax.unsqueeze(2))).to(torch.float8_e4m3fn).view(m, n)
    return q, (amax / 448.0).view(m, -1)


def test_quant_oracle_matches_published_algorithm():
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(37, 512, generator=g) * torch.logspace(-6, 2, 37).unsqueeze(1)).to(torch.bfloat16)
    x[3] = 0  # all-zero row exercises the 1e-4 clamp
    q_ref, s_ref = _dg_per_token_cast(x)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    q, s = O.quant_act_fp8_1x128(xb)
    assert np.array_equal(q, q_ref.view(torch.uint8).numpy())
    assert np.array_equal(s.view(np.uint32), s_ref.numpy().view(np.uint32))


def test_quant_ue8m0_oracle_matches_exact_restatement():
    """use_ue8m0 form: scale = 2^ceil(log2(fl(amax/448))) evaluated exactly
    (float64 log2 of a float32 is exact enough for the ceiling), q = the e4m3
    of x / scale (exact)."""
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(64, 512, generator=g) * torch.logspace(-3, 3, 64).unsqueeze(1)).to(torch.bfloat16)
    x[3] = 0                     # the 1e-4 clamp
    x[5, :128] = 56.0            # amax / 448 = 1/8 exactly: kept, not rounded up
    xb = x.view(torch.int16).numpy().view(np.uint16)
    q, s = O.quant_act_fp8_1x128(xb, ue8m0=True)
    xf = x.float().numpy().reshape(64, 4, 128).astype(np.float64)
    amax = np.maximum(np.abs(xf).max(-1), 1e-4).astype(np.float32)
    s_ref = np.exp2(np.ceil(np.log2((amax / np.float32(448)).astype(np.float64)))).astype(np.float32)
    assert np.array_equal(s, s_ref)
    assert s[5, 0] == 0.125
    q_ref = torch.from_numpy((xf / s_ref[..., None]).astype(np.float32).reshape(64, 512))
    assert np.array_equal(q, q_ref.to(torch.float8_e4m3fn).view(torch.uint8).numpy())
    # the gathered form reads the same rows
    rows = np.array([9, 0, -1, 4], np.int32)
    qg, sg = O.quant_act_fp8_1x128(xb, rows, gather_div=3, ue8m0=True)
    assert np.array_equal(qg[0], q[3]) and np.array_equal(sg[3], s[1])
    assert not qg[2].any() and not sg[2].any()


@pytest.mark.parametrize("ue8m0", [False, True])
def test_weight_block_quant_matches_oracle(ue8m0):
    """The load-time weight quantizer (torch) against the oracle's restatement
    of the published per_block_cast_to_fp8, bit for bit: zero blocks (the 1e-4
    clamp), an outlier block and magnitudes over 8 decades."""
    from ferret_b200 import data
    g = torch.Generator().manual_seed(9)
    w = torch.randn(3, 384, 512, generator=g) * torch.logspace(-4, 4, 3 * 384).view(3, 384, 1)
    w[0, :128, :128] = 0
    w[1, 200, 300] = 1e5
    q, s = data.per_block_cast_to_fp8(w, use_ue8m0=ue8m0)
    qr, sr = O.per_block_cast_to_fp8(w.numpy(), ue8m0=ue8m0)
    assert np.array_equal(q.view(torch.uint8).numpy(), qr)
    assert np.array_equal(s.numpy().view(np.uint32), sr.view(np.uint32))


def test_ue8m0_weight_scales_are_powers_of_two():
    from ferret_b200 import data
    g = torch.Generator().manual_seed(8)
    w = torch.randn(2, 256, 512, generator=g) * 0.02
    q, s = data.per_block_cast_to_fp8(w, use_ue8m0=True)
    assert (s.view(torch.int32) & 0x7FFFFF == 0).all()
    q0, s0 = data.per_block_cast_to_fp8(w)
    assert (s >= s0).all() and (s < 2 * s0).all()
    deq = q.float().view(2, 2, 128, 4, 128) * s.view(2, 2, 1, 4, 1)
    assert (deq.view(2, 256, 512) - w).abs().max() <= w.abs().max() / 8


def test_quant_oracle_gather():
    g = torch.Generator().manual_seed(6)
    x = torch.randn(5, 256, generator=g).to(torch.bfloat16)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    rows = np.array([9, 0, -1, 4, 14], np.int32)      # flat t*topk + j with topk=3
    q, s = O.quant_act_fp8_1x128(xb, rows, gather_div=3)
    qd, sd = O.quant_act_fp8_1x128(xb[[3, 0, 0, 1, 4]])
    for r, src in enumerate([3, 0, None, 1, 4]):
        if src is None:
            assert not q[r].any() and not s[r].any()
        else:
            assert np.array_equal(q[r], qd[r]) and np.array_equal(s[r], sd[r])


@pytest.mark.parametrize("T,topk,E", [(1, 1, 1), (7, 3, 5), (64, 8, 384), (300, 2, 8), (0, 8, 16)])
def test_permute_oracle_is_stable_counting_sort(T, topk, E):
    rng = np.random.default_rng(T * 31 + E)
    ids = rng.integers(-2, E + 2, size=(T, topk)).astype(np.int32)
    rows, offs, mi = O.moe_permute(ids, E)
    flat = ids.reshape(-1)
    valid = (flat >= 0) & (flat < E)
    order = np.argsort(np.where(valid, flat, E), kind="stable")[: valid.sum()]
    assert np.array_equal(rows[: valid.sum()], order)
    assert np.array_equal(mi[: valid.sum()], flat[order])
    assert (rows[valid.sum():] == -1).all() and (mi[valid.sum():] == -1).all()
    assert np.array_equal(offs, np.concatenate([[0], np.cumsum(np.bincount(flat[valid], minlength=E))]))


def test_fast_and_scalar_fp8_oracles_agree():
    rng = np.random.default_rng(3)
    M, N, K, E = 40, 256, 384, 3
    a = O.f32_to_e4m3(rng.standard_normal((M, K)).astype(np.float32) * 50)
    w = O.f32_to_e4m3(rng.standard_normal((E, N, K)).astype(np.float32) * 50)
    a_s = rng.uniform(0.001, 0.01, (M, K // 128)).astype(np.float32)
    w_s = rng.uniform(0.001, 0.01, (E, N // 128, K // 128)).astype(np.float32)
    mi = np.sort(rng.integers(-1, E, M)).astype(np.int32)
    for silu in (False, True):
        ref = O.fp8_grouped_gemm(a, a_s, w, w_s, mi, silu=silu)
        fast = O.fp8_grouped_gemm_fast(a, a_s, w, w_s, mi, silu=silu)
        ok = mi >= 0
        assert O.rel_err(fast[ok], ref[ok])["max_rel"] < 1e-4
        assert np.isnan(ref[~ok]).all() and np.isnan(fast[~ok]).all()


def test_fast_and_scalar_int4_oracles_agree():
    import sys
    sys.path.insert(0, GOLD)
    import make_golden as G
    h, rq, sc, ids = G.int4_inputs(9, T=3, E=5, K=256, N=128, topk=2)
    for silu in (False, True):
        ref = O.int4_w13(h, rq, sc, ids, silu=silu)
        fast = O.int4_w13_fast(h, rq, sc, ids, silu=silu)
        assert O.rel_err(fast, ref)["max_rel"] < 1e-4


def test_torch_cpu_fp8_path_agrees_with_scalar_oracle():
    """The torch fp32 path (the timed CPU baseline, also the per-expert checker
    of the full-size GPU tests) against the scalar oracle."""
    import torch
    rng = np.random.default_rng(4)
    M, N, K, E = 24, 256, 384, 3
    a = O.f32_to_e4m3(rng.standard_normal((M, K)).astype(np.float32) * 50)
    w = O.f32_to_e4m3(rng.standard_normal((E, N, K)).astype(np.float32) * 50)
    a_s = rng.uniform(0.001, 0.01, (M, K // 128)).astype(np.float32)
    w_s = rng.uniform(0.001, 0.01, (E, N // 128, K // 128)).astype(np.float32)
    mi = np.sort(rng.integers(0, E, M)).astype(np.int32)
    offs = np.concatenate([[0], np.cumsum(np.bincount(mi, minlength=E))])
    for silu in (False, True):
        ref = O.fp8_grouped_gemm(a, a_s, w, w_s, mi, silu=silu)
        got = O.fp8_w13_torch_cpu(torch.from_numpy(a), torch.from_numpy(a_s), torch.from_numpy(w),
                                  torch.from_numpy(w_s), offs, range(E), silu=silu)
        for e in range(E):
            if offs[e + 1] > offs[e]:
                assert O.rel_err(got[e].numpy(), ref[offs[e]:offs[e + 1]])["max_rel"] < 1e-4


def test_torch_cpu_int4_path_agrees_with_scalar_oracle():
    import sys
    import torch
    sys.path.insert(0, GOLD)
    import make_golden as G
    h, rq, sc, ids = G.int4_inputs(11, T=4, E=3, K=256, N=256, topk=2)
    flat = ids.reshape(-1)
    for silu in (False, True):
        ref = O.int4_w13(h, rq, sc, ids, silu=silu)
        for e in np.unique(flat):
            pairs = np.nonzero(flat == e)[0]
            x = torch.from_numpy(h.view(np.int16)).view(torch.bfloat16)[torch.from_numpy(pairs // 2)]
            got = O.int4_w13_torch_cpu(x, torch.from_numpy(rq[e]),
                                       torch.from_numpy(sc[e].view(np.int16)).view(torch.bfloat16),
                                       silu=silu)
            assert O.rel_err(got.numpy(), ref[pairs])["max_rel"] < 1e-4


def test_rel_err_counts_nan():
    r = O.rel_err(np.array([1.0, np.nan]), np.array([1.0, 2.0]))
    assert r["nan"] == 1 and r["max_rel"] == np.inf


def test_align_block_size_oracle_layout():
    """Padded layout: each expert's ascending flat indices, padded with
    T*topk to the block size; blocks carry their expert, -1 past the end."""
    ids = np.array([[1, 0], [1, 2], [0, 5], [1, 1]], np.int32)    # 5 is invalid with E=3
    s, e, n = O.moe_align_block_size(ids, 3, 4)
    assert n.tolist() == [12]
    assert s[:12].tolist() == [1, 4, 8, 8, 0, 2, 6, 7, 3, 8, 8, 8]
    assert e.tolist()[:3] == [0, 1, 2] and all(v == -1 for v in e.tolist()[3:])
    assert len(s) == 8 + 3 * 3 and (s[12:] == 8).all()
