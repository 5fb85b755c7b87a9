"""GPU parity tests of the FP8 W13 path against the CPU oracle.

Integer outputs (permutation, quantized activations and their scales) must be
bit-exact.  GEMM outputs are bf16 and must match the fp32 oracle within max
relative error < 1e-2 (denominator max(|ref|, 1e-3 * max|ref|)), with no NaN,
over every row (the reference's check at
examples/fp8-group-gemm/v007_dsv3_decode_verified_105.cu:547-551 and
tasks/fp8-group-gemm-dsv3-decode.yaml:101, extended from 32 rows to all).
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2
GOLD = os.path.join(os.path.dirname(__file__), "golden")
BF16_NAN = 0x7FFF


@pytest.fixture(scope="module")
def ops(cuda_device):
    from ferret_b200 import ops as _ops
    return _ops


def u16(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.uint8).cpu().numpy()


# ---------------------------------------------------------------- permutation

@pytest.mark.parametrize("T,topk,E,lo,hi", [
    (1, 1, 1, 0, 1), (128, 8, 256, 0, 256), (64, 8, 384, 0, 384), (7, 3, 5, -2, 7),
    (300, 2, 8, 0, 8), (0, 8, 16, 0, 16), (4096, 8, 1024, -1, 1024), (32768, 8, 256, 0, 256),
    (1000, 4, 3, 2, 3),     # a single expert receives everything
])
def test_permute_bit_exact(ops, T, topk, E, lo, hi):
    rng = np.random.default_rng(T + 7 * E)
    ids = rng.integers(lo, hi, size=(T, topk)).astype(np.int32)
    d_rows, d_offs, d_mi = ops.moe_permute(torch.from_numpy(ids).cuda(), E)
    rows, offs, mi = O.moe_permute(ids, E)
    assert np.array_equal(d_offs.cpu().numpy(), offs)
    assert np.array_equal(d_rows.cpu().numpy(), rows)
    assert np.array_equal(d_mi.cpu().numpy(), mi)


@pytest.mark.parametrize("T,topk,E,lo,hi", [
    (513, 8, 256, 0, 256),          # 4104 ids: two chunks
    (4099, 3, 7, -1, 8),            # ragged chunks, dropped ids at both ends of the range
    (32768, 8, 32, 0, 32),          # the all-rank sort of 8-way EP prefill (1024 ids/expert)
    (262144, 8, 256, 0, 256),       # 2M ids: the 256-chunk limit
])
def test_permute_chunked_matches_single_cta(ops, T, topk, E, lo, hi):
    """The multi-CTA (workspace) form and the one-CTA form give the same bits,
    and both match the oracle."""
    import ctypes
    from ferret_b200._lib import lib
    rng = np.random.default_rng(T * 3 + E)
    ids_np = rng.integers(lo, hi, size=(T, topk)).astype(np.int32)
    ids = torch.from_numpy(ids_np).cuda()
    L = lib()
    ws_bytes = int(L.ferret_moe_permute_workspace_size(T, topk, E))
    assert ws_bytes > 0
    outs = []
    for ws in (torch.empty(ws_bytes // 4, dtype=torch.int32, device="cuda"), None):
        r = torch.full((T * topk,), 7, dtype=torch.int32, device="cuda")
        o = torch.full((E + 1,), 7, dtype=torch.int32, device="cuda")
        m = torch.full((T * topk,), 7, dtype=torch.int32, device="cuda")
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = L.ferret_moe_permute(ctypes.c_void_p(ids.data_ptr()), T, topk, E,
                                  ctypes.c_void_p(r.data_ptr()), ctypes.c_void_p(o.data_ptr()),
                                  ctypes.c_void_p(m.data_ptr()),
                                  None if ws is None else ctypes.c_void_p(ws.data_ptr()),
                                  0 if ws is None else ws_bytes, stream)
        assert rc == 0
        outs.append((r.cpu().numpy(), o.cpu().numpy(), m.cpu().numpy()))
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    if T * topk <= 300000:
        rows, offs, mi = O.moe_permute(ids_np, E)
        assert np.array_equal(outs[0][0], rows)
        assert np.array_equal(outs[0][1], offs)
        assert np.array_equal(outs[0][2], mi)
    else:   # stable-sort properties at the largest size
        r, o, m = outs[0]
        flat = ids_np.reshape(-1)
        assert np.array_equal(o, np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))]))
        assert np.array_equal(flat[r], m)
        for e in (0, E // 2, E - 1):
            seg = r[o[e]:o[e + 1]]
            assert np.all(np.diff(seg) > 0)


# ---------------------------------------------------------------- quantization

@pytest.mark.parametrize("R,K", [(1, 128), (37, 512), (1024, 7168), (3, 16384)])
def test_quant_bit_exact(ops, R, K):
    g = torch.Generator().manual_seed(R)
    x = (torch.randn(R, K, generator=g) * torch.logspace(-5, 2, R).unsqueeze(1)).to(torch.bfloat16)
    x[0, :128] = 0
    q, s = ops.per_token_cast_to_fp8(x.cuda())
    qr, sr = O.quant_act_fp8_1x128(u16(x))
    assert np.array_equal(u8(q), qr)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))


def test_quant_gather_bit_exact(ops):
    g = torch.Generator().manual_seed(1)
    T, topk, K = 33, 4, 1024
    x = torch.randn(T, K, generator=g).to(torch.bfloat16)
    rows = torch.randperm(T * topk, generator=g).to(torch.int32)
    rows[-5:] = -1
    q, s = ops.per_token_cast_to_fp8(x.cuda(), rows.cuda(), topk)
    qr, sr = O.quant_act_fp8_1x128(u16(x), rows.numpy(), topk)
    assert np.array_equal(u8(q), qr)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))


@pytest.mark.parametrize("ue8m0", [False, True])
@pytest.mark.parametrize("T,topk,E,K", [(5, 3, 4, 256), (1024, 8, 256, 7168), (3000, 8, 64, 512)])
def test_quant_scatter_equals_gathered_quant(ops, T, topk, E, K, ue8m0):
    """Quantize-and-scatter (each token once, written to its top-k expert-sorted
    rows) gives the gathered quantizer's bytes on every valid sorted row, also
    with dropped pairs; rows past the valid ones are left alone."""
    from ferret_b200 import data
    x = data.activations(T, K, seed=T).cuda()
    ids = data.routing(T, E, topk, "zipf").cuda()
    ids[1, 0] = -1
    ids[T - 1, topk - 1] = E + 3
    rows, offs, _ = ops.moe_permute(ids, E)
    R = int(offs[-1])
    qg, sg = ops.per_token_cast_to_fp8(x, rows, topk, use_ue8m0=ue8m0)
    qs = torch.full((T * topk, K), 0x55, dtype=torch.uint8, device="cuda")
    ss = torch.full((T * topk, K // 128), -7.0, device="cuda")
    ops.per_token_cast_to_fp8_scatter(x, rows, offs, topk, out=(qs, ss), use_ue8m0=ue8m0)
    torch.cuda.synchronize()
    assert torch.equal(qs[:R], qg.view(torch.uint8)[:R])
    assert torch.equal(ss[:R], sg[:R])
    assert (qs[R:] == 0x55).all() and (ss[R:] == -7.0).all()
    assert ops.last_device_status() == 0


@pytest.mark.parametrize("T,topk,K", [(5, 3, 256), (1024, 8, 7168)])
def test_gather_rows_equals_gathered_quant(ops, T, topk, K):
    """Quantize-once + ferret_fp8_gather_rows gives the bytes of the gathered
    quantizer, including zero rows for negative indices."""
    import ctypes
    from ferret_b200._lib import lib
    g = torch.Generator().manual_seed(T + K)
    x = torch.randn(T, K, generator=g).to(torch.bfloat16).cuda()
    rows = torch.randperm(T * topk, generator=g).to(torch.int32)
    rows[::7] = -1
    rows = rows.cuda()
    qa, sa = ops.per_token_cast_to_fp8(x, rows, topk)
    qt, st = ops.per_token_cast_to_fp8(x)
    R = rows.numel()
    qb = torch.full((R, K), 0x55, dtype=torch.uint8, device="cuda")
    sb = torch.full((R, K // 128), 3.0, dtype=torch.float32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib().ferret_fp8_gather_rows(ctypes.c_void_p(qt.data_ptr()), ctypes.c_void_p(st.data_ptr()), T,
                                      ctypes.c_void_p(rows.data_ptr()), topk, R, K,
                                      ctypes.c_void_p(qb.data_ptr()), ctypes.c_void_p(sb.data_ptr()),
                                      stream)
    assert rc == 0
    assert torch.equal(qa.view(torch.uint8), qb)
    assert torch.equal(sa.view(torch.int32), sb.view(torch.int32))


def test_quant_matches_torch_cuda_published_algorithm(ops):
    """The published per_token_cast_to_fp8 evaluated by torch on this GPU."""
    g = torch.Generator().manual_seed(2)
    x = (torch.randn(64, 2048, generator=g) * 3).to(torch.bfloat16).cuda()
    v = x.view(64, -1, 128)
    amax = v.abs().float().amax(dim=2).view(64, -1).clamp(1e-4)
    q_ref = (v * (448.0 / amax.unsqueeze(2))).to(torch.float8_e4m3fn).view(64, 2048)
    q, s = ops.per_token_cast_to_fp8(x)
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))
    # torch may evaluate amax / 448 as amax * (1/448) on the GPU: allow 1 ulp
    s_ref = (amax / 448.0)
    ulp = (s.view(torch.int32) - s_ref.view(torch.int32)).abs().max().item()
    assert ulp <= 1


# ---------------------------------------------------------------- grouped GEMM

def make_case(seed, seg_counts, N, K, pad_between=0, scale_kind="random"):
    """Contiguous-layout inputs: experts in order with `pad_between` padding
    rows (m_indices = -1) after every segment."""
    rng = np.random.default_rng(seed)
    E = len(seg_counts)
    mi = []
    for e, c in enumerate(seg_counts):
        mi += [e] * c + [-1] * pad_between
    mi = np.array(mi, np.int32)
    M = len(mi)
    a = O.f32_to_e4m3(rng.standard_normal((M, K)).astype(np.float32) * 100)
    w = O.f32_to_e4m3(rng.standard_normal((E, N, K)).astype(np.float32) * 100)
    if scale_kind == "pow2":
        a_s = np.ldexp(1.0, rng.integers(-12, -6, (M, K // 128))).astype(np.float32)
        w_s = np.ldexp(1.0, rng.integers(-12, -6, (E, N // 128, K // 128))).astype(np.float32)
    else:
        a_s = rng.uniform(1e-3, 1e-2, (M, K // 128)).astype(np.float32)
        w_s = rng.uniform(1e-4, 1e-3, (E, N // 128, K // 128)).astype(np.float32)
    return a, a_s, w, w_s, mi


def run_gemm(ops, a, a_s, w, w_s, mi, silu, tile, use_offsets):
    M, K = a.shape
    E, N, _ = w.shape
    n_out = N // 2 if silu else N
    out = torch.full((M, n_out), BF16_NAN, dtype=torch.int16).view(torch.bfloat16).cuda()
    offs = None
    if use_offsets:
        assert (mi >= 0).all()
        offs = torch.from_numpy(np.concatenate([[0], np.cumsum(np.bincount(mi, minlength=E))])
                                .astype(np.int32)).cuda()
    ops.m_grouped_fp8_gemm_nt_contiguous(
        (torch.from_numpy(a).cuda(), torch.from_numpy(a_s).cuda()),
        (torch.from_numpy(w).cuda(), torch.from_numpy(w_s).cuda()),
        out, None if use_offsets else torch.from_numpy(mi).cuda(),
        expert_offsets=offs, silu=silu, tile=tile)
    torch.cuda.synchronize()
    assert ops.last_device_status() == 0
    return out


def check(out, ref, mi):
    got = O.bf16_to_f32(u16(out))
    valid = mi >= 0
    err = O.rel_err(got[valid], ref[valid])
    assert err["nan"] == 0 and err["max_rel"] < TOL, err
    # padding rows are never written
    assert (u16(out)[~valid] == BF16_NAN).all()


CASES = [
    # (seg_counts, N, K, pad, silu, tile)
    ([5, 0, 17, 1, 3], 256, 256, 0, False, 16),
    ([5, 0, 17, 1, 3], 256, 256, 0, True, 16),
    ([40, 3, 0, 70], 512, 384, 0, False, 32),
    ([40, 3, 0, 70], 512, 384, 0, True, 32),
    ([130, 64, 1], 256, 512, 0, False, 64),
    ([130, 64, 1], 512, 512, 0, True, 64),
    ([300, 129, 2], 384, 256, 0, False, 128),
    ([1] * 12, 256, 1024, 0, False, 0),
    ([8, 8, 8, 8], 256, 128, 5, False, 16),     # DeepGEMM-style padding rows
    ([8, 8, 8, 8], 256, 128, 5, True, 0),
    # the prefill kernel (128-token tiles on MMA M, 256 weight rows on MMA N)
    ([300, 129, 2, 0, 77], 512, 384, 0, False, 128),
    ([300, 129, 2, 0, 77], 512, 384, 0, True, 128),
    ([40, 40, 40, 40], 256, 128, 5, False, 128),
    ([1000], 256, 256, 0, True, 128),
    # per-tile MMA N (16-row granules) inside a 64- or 128-row token tile
    ([1, 17, 33, 49, 64, 0, 70], 256, 512, 0, False, 64),
    ([1, 17, 33, 49, 64, 0, 70], 512, 512, 0, True, 64),
    ([5, 100, 127, 128, 129], 256, 384, 0, False, 128),
    # few tiles: K split over the SMs (m_indices path, with workspace), fp32
    # partials reduced in split order by the last unit of each tile
    ([32], 1024, 2048, 0, False, 0),
    ([32], 1024, 2048, 0, True, 0),
    ([3, 0, 9], 512, 7168, 0, True, 16),
    # the K limit (K = 16384: 128 K blocks) on the swap-AB and the prefill kernel
    ([3] * 16, 256, 16384, 0, False, 0),
    ([130, 3], 256, 16384, 0, True, 128),
]


@pytest.mark.parametrize("seg,N,K,pad,silu,tile", CASES)
@pytest.mark.parametrize("use_offsets", [False, True])
def test_grouped_gemm_vs_oracle(ops, seg, N, K, pad, silu, tile, use_offsets):
    if use_offsets and pad:
        pytest.skip("offsets describe unpadded layouts")
    a, a_s, w, w_s, mi = make_case(hash((tuple(seg), N, K)) & 0xFFFF, seg, N, K, pad)
    out = run_gemm(ops, a, a_s, w, w_s, mi, silu, tile, use_offsets)
    ref = O.fp8_grouped_gemm(a, a_s, w, w_s, mi, silu=silu)
    check(out, ref, mi)


PAIR_CASES = [
    # (seg_counts, N, K, silu): whole 256-row chunks on CTA pairs, the rest on single CTAs
    ([600, 0, 256, 255, 1000, 3], 512, 512, False),
    ([600, 0, 256, 255, 1000, 3], 512, 512, True),
    ([1024], 256, 7168, False),
    ([513, 770], 1024, 384, True),
    ([100, 37], 256, 256, False),                   # one pair tile per expert, second half empty
]


@pytest.mark.parametrize("seg,N,K,silu", PAIR_CASES)
@pytest.mark.parametrize("use_offsets", [False, True])
def test_grouped_gemm_cta_pairs_vs_oracle(ops, seg, N, K, silu, use_offsets):
    """FERRET_PREFILL_PAIRS: tcgen05.mma.cta_group::2 tiles of 256 rows over
    every expert's rows (the last one of an expert partly or half empty)
    against the oracle, and equal to the single-CTA prefill kernel (same
    per-K-block promotion order)."""
    a, a_s, w, w_s, mi = make_case(hash((tuple(seg), N, K, 2)) & 0xFFFF, seg, N, K)
    M = len(mi)
    outs = []
    for pairs in (True, False):
        out = torch.full((M, N // 2 if silu else N), BF16_NAN, dtype=torch.int16).view(torch.bfloat16).cuda()
        offs = None
        if use_offsets:
            offs = torch.from_numpy(np.concatenate([[0], np.cumsum(np.bincount(mi, minlength=len(seg)))])
                                    .astype(np.int32)).cuda()
        ops.m_grouped_fp8_gemm_nt_contiguous(
            (torch.from_numpy(a).cuda(), torch.from_numpy(a_s).cuda()),
            (torch.from_numpy(w).cuda(), torch.from_numpy(w_s).cuda()),
            out, None if use_offsets else torch.from_numpy(mi).cuda(),
            expert_offsets=offs, silu=silu, tile=128, prefill_pairs=pairs)
        torch.cuda.synchronize()
        assert ops.last_device_status() == 0
        outs.append(out)
    ref = O.fp8_grouped_gemm(a, a_s, w, w_s, mi, silu=silu)
    check(outs[0], ref, mi)
    err = O.rel_err(O.bf16_to_f32(u16(outs[0])), O.bf16_to_f32(u16(outs[1])))
    assert err["nan"] == 0 and err["max_rel"] <= 2 ** -7, err


def test_grouped_gemm_reference_golden(ops):
    """The inputs/outputs of the reference's own cpu_ref_bs (tests/golden)."""
    d = np.load(os.path.join(GOLD, "fp8_v007_ref.npz"))
    out = run_gemm(ops, d["a"], d["a_scale"], d["w"], d["w_scale"], d["m_indices"], False, 0, False)
    check(out, d["out"], d["m_indices"])


def test_grouped_gemm_is_deterministic(ops):
    a, a_s, w, w_s, mi = make_case(3, [33, 2, 90], 512, 512)
    o1 = run_gemm(ops, a, a_s, w, w_s, mi, False, 0, False)
    o2 = run_gemm(ops, a, a_s, w, w_s, mi, False, 0, False)
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))


def test_grouped_gemm_reports_noncontiguous_rows(ops):
    a, a_s, w, w_s, _ = make_case(4, [4, 4], 256, 128)
    mi = np.array([0, 0, 1, 1, 0, 0, 1, 1], np.int32)
    run_gemm_status = None
    M, K = a.shape
    out = torch.empty(M, 256, dtype=torch.bfloat16, device="cuda")
    ops.m_grouped_fp8_gemm_nt_contiguous(
        (torch.from_numpy(a).cuda(), torch.from_numpy(a_s).cuda()),
        (torch.from_numpy(w).cuda(), torch.from_numpy(w_s).cuda()), out,
        torch.from_numpy(mi).cuda())
    torch.cuda.synchronize()
    run_gemm_status = ops.last_device_status()
    assert run_gemm_status == 3
    assert ops.last_device_status() == 0   # read-and-clear


# ---------------------------------------------------------------- whole W13 path

def oracle_w13(hidden, ids, w, w_s, E, silu):
    rows, offs, mi = O.moe_permute(ids, E)
    R = int(offs[-1])
    q, s = O.quant_act_fp8_1x128(hidden, rows[:R], ids.shape[1])
    return O.fp8_grouped_gemm(q, s, w, w_s, mi[:R], silu=silu), rows, offs, q, s


@pytest.mark.parametrize("silu", [False, True])
def test_w13_path_cpu_config(ops, silu):
    """Benchmark configuration 1 (E=8, top-2 uniform, 256 tokens, K=512, N=1024), all rows."""
    from ferret_b200 import data
    cfg = data.CONFIGS["cpu_fp8"]
    W, Ws = data.fp8_weights(cfg.E, cfg.N, cfg.K)
    hidden = data.activations(cfg.T, cfg.K)
    ids = data.routing(cfg.T, cfg.E, cfg.topk)
    out, rows, offs = ops.fp8_moe_w13(hidden.cuda(), ids.cuda(), W.cuda(), Ws.cuda(), silu=silu)
    torch.cuda.synchronize()
    ref, r_rows, r_offs, _, _ = oracle_w13(u16(hidden), ids.numpy(), u8(W), Ws.numpy(), cfg.E, silu)
    assert np.array_equal(rows.cpu().numpy(), r_rows)
    assert np.array_equal(offs.cpu().numpy(), r_offs)
    err = O.rel_err(O.bf16_to_f32(u16(out)), ref)
    assert err["nan"] == 0 and err["max_rel"] < TOL, err


def _torch_ref(q, s, W, Ws, e, silu=False):
    """fp32 dequantize-then-matmul of one expert's rows on the host cores
    (oracle.fp8_w13_torch_cpu, checked against the scalar oracle on the CPU)."""
    n = q.shape[0]
    res = O.fp8_w13_torch_cpu(torch.from_numpy(q), torch.from_numpy(s), W[e:e + 1].cpu(),
                              Ws[e:e + 1].cpu(), [0, n], [0], silu=silu)
    return res[0].numpy()


def test_w13_path_dsv3_decode_full_size(ops):
    """Benchmark configuration 2 at full size: every output row of every active
    expert against the fp32 oracle; permutation and quantization in full."""
    from ferret_b200 import data
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = data.CONFIGS["dsv3_decode"]
    dev = torch.device("cuda")
    W, Ws = data.fp8_weights(cfg.E, cfg.N, cfg.K, device=dev)
    hidden = data.activations(cfg.T, cfg.K)
    ids = data.routing(cfg.T, cfg.E, cfg.topk)
    out, rows, offs = ops.fp8_moe_w13(hidden.cuda(), ids.cuda(), W, Ws)
    torch.cuda.synchronize()
    r_rows, r_offs, r_mi = O.moe_permute(ids.numpy(), cfg.E)
    assert np.array_equal(rows.cpu().numpy(), r_rows)
    assert np.array_equal(offs.cpu().numpy(), r_offs)
    q, s = O.quant_act_fp8_1x128(u16(hidden), r_rows, cfg.topk)
    qd, sd = ops.per_token_cast_to_fp8(hidden.cuda(), rows, cfg.topk)
    assert np.array_equal(u8(qd), q)
    got = O.bf16_to_f32(u16(out))
    experts = np.nonzero(np.diff(r_offs))[0]
    assert len(experts) == 252
    for e in experts:
        r0, r1 = r_offs[e], r_offs[e + 1]
        err = O.rel_err(got[r0:r1], _torch_ref(q[r0:r1], s[r0:r1], W, Ws, e))
        assert err["nan"] == 0 and err["max_rel"] < TOL, (int(e), err)
    assert ops.last_device_status() == 0


def test_w13_path_ep_prefill_full_size(ops):
    """Benchmark configuration 5's global batch on one GPU (E=256, top-8
    Zipf(1.1), 32,768 tokens = 262,144 routed rows, K=7168, N=4096): the
    permutation in full, and every row of the 6 largest experts (28,497 rows
    down to 8,259) and of 10 random other active experts against the fp32
    oracle, quantized by the oracle's own quantizer."""
    from ferret_b200 import data
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = data.CONFIGS["ep_prefill"]
    dev = torch.device("cuda")
    W, Ws = data.fp8_weights(cfg.E, cfg.N, cfg.K, device=dev)
    hidden = data.activations(cfg.T, cfg.K)
    ids = data.routing(cfg.T, cfg.E, cfg.topk, cfg.routing, cfg.zipf_s)
    out, rows, offs = ops.fp8_moe_w13(hidden.cuda(), ids.cuda(), W, Ws)
    torch.cuda.synchronize()
    assert ops.last_device_status() == 0
    r_rows, r_offs, _ = O.moe_permute(ids.numpy(), cfg.E)
    assert np.array_equal(rows.cpu().numpy(), r_rows)
    assert np.array_equal(offs.cpu().numpy(), r_offs)
    counts = np.diff(r_offs)
    order = np.argsort(-counts, kind="stable")
    rest = [e for e in order[6:] if counts[e] > 0]
    experts = list(order[:6]) + list(np.random.default_rng(5).choice(rest, 10, replace=False))
    h = u16(hidden)
    for e in experts:
        r0, r1 = int(r_offs[e]), int(r_offs[e + 1])
        q, s = O.quant_act_fp8_1x128(h, r_rows[r0:r1], cfg.topk)
        got = O.bf16_to_f32(u16(out[r0:r1]))
        err = O.rel_err(got, _torch_ref(q, s, W, Ws, e))
        assert err["nan"] == 0 and err["max_rel"] < TOL, (int(e), r1 - r0, err)


# ---------------------------------------------------------------- expert parallel, one rank

def test_ep_single_rank_matches_w13_path(ops):
    """ExpertParallelW13 with one rank (no communication) against fp8_moe_w13:
    bit-identical per (token, slot) pair."""
    from ferret_b200 import data
    from ferret_b200.ep import ExpertParallelW13
    cfg = data.CONFIGS["cpu_fp8"]
    dev = torch.device("cuda")
    W, Ws = data.fp8_weights(cfg.E, cfg.N, cfg.K, device=dev)
    hidden = data.activations(cfg.T, cfg.K).to(dev)
    ids = data.routing(cfg.T, cfg.E, cfg.topk, "zipf").to(dev)
    for silu in (False, True):
        out, rows, offs = ops.fp8_moe_w13(hidden, ids, W, Ws, silu=silu)
        tk = torch.empty_like(out)
        tk[rows.long()] = out
        ep = ExpertParallelW13(W, Ws, cfg.E, silu=silu)
        got = ep.forward(hidden, ids)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), tk.view(torch.int16))


def test_w13_path_dsv3_prefill_full_size(ops):
    """Benchmark configuration 3 (E=256, top-8 Zipf(1.1), 8192 tokens) at full size, plain
    and fused SiLU: every row of 6 sampled experts (the largest among them)
    against the fp32 oracle."""
    from ferret_b200 import data
    cfg = data.CONFIGS["dsv3_prefill"]
    dev = torch.device("cuda")
    W, Ws = data.fp8_weights(cfg.E, cfg.N, cfg.K, device=dev)
    hidden = data.activations(cfg.T, cfg.K)
    ids = data.routing(cfg.T, cfg.E, cfg.topk, "zipf")
    r_rows, r_offs, _ = O.moe_permute(ids.numpy(), cfg.E)
    counts = np.diff(r_offs)
    experts = [int(np.argmax(counts))] + list(np.random.default_rng(2).choice(
        np.nonzero(counts)[0], 5, replace=False))
    for silu in (False, True):
        out, rows, offs = ops.fp8_moe_w13(hidden.cuda(), ids.cuda(), W, Ws, silu=silu)
        torch.cuda.synchronize()
        assert np.array_equal(offs.cpu().numpy(), r_offs)
        got = O.bf16_to_f32(u16(out))
        qd, sd = u8(ops.per_token_cast_to_fp8(hidden.cuda(), rows, cfg.topk)[0]), None
        q, s = ops.per_token_cast_to_fp8(hidden.cuda(), rows, cfg.topk)
        q, s = u8(q), s.cpu().numpy()
        for e in experts:
            r0, r1 = r_offs[e], r_offs[e + 1]
            ref = O.fp8_grouped_gemm_fast(q[r0:r1], s[r0:r1], u8(W[e:e + 1]), Ws[e:e + 1].cpu().numpy(),
                                          np.zeros(r1 - r0, np.int32), silu=silu)
            err = O.rel_err(got[r0:r1], ref)
            assert err["nan"] == 0 and err["max_rel"] < TOL, (silu, int(e), err)
    assert ops.last_device_status() == 0


@pytest.mark.parametrize("silu,tile", [(False, 0), (True, 16), (False, 128), (True, 128)])
def test_scatter_gemm_token_order(ops, silu, tile):
    """The scatter-output GEMM writes row i of the expert-sorted operand to
    out[sorted_rows[i]]: the (token, slot) order, bit-identical to the
    contiguous GEMM's rows moved there."""
    from ferret_b200 import data
    cfg = data.CONFIGS["cpu_fp8"]
    dev = torch.device("cuda")
    W, Ws = data.fp8_weights(cfg.E, cfg.N, cfg.K, device=dev)
    hidden = data.activations(cfg.T, cfg.K).to(dev)
    ids = data.routing(cfg.T, cfg.E, cfg.topk, "zipf").to(dev)
    ids[3, 1] = -1
    out, rows, offs = ops.fp8_moe_w13(hidden, ids, W, Ws, silu=silu, tile=tile)
    q, s = ops.per_token_cast_to_fp8(hidden, rows, cfg.topk)
    tok = torch.full((cfg.R, out.shape[1]), 7.0, dtype=torch.bfloat16, device=dev)
    ops.m_grouped_fp8_gemm_scatter((q, s), (W, Ws), tok, offs, rows, silu=silu, tile=tile)
    torch.cuda.synchronize()
    R = int(offs[-1])
    want = torch.full_like(tok, 7.0)
    want[rows[:R].long()] = out[:R]
    assert torch.equal(tok.view(torch.int16), want.view(torch.int16))
