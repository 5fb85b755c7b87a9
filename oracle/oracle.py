"""CPU oracle for the quantized MoE W13 hot path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, and only as the checker.  The
product package (ferret_b200) never imports this module.

Two layers:

* ctypes bindings to ``liboracle.so`` (ferret_oracle.c): scalar restatements
  with the reference's accumulation order, used for small parity cases and
  pinned against the reference itself (tests/golden).
* numpy "dequantize-then-matmul" versions for sizes the scalar code cannot
  finish in seconds.  They follow the same formulas with BLAS fp32 matmuls:
  the fp32 dequantize-then-matmul path the reference's correctness oracle
  uses (correctness/compare_marlin_vs_ref.py:44-100) and the per-128-K-block
  promotion of examples/fp8-group-gemm/v007_dsv3_decode_verified_105.cu:441-467
  with exact fp32 scales.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_p = ctypes.c_void_p
_i = ctypes.c_int


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def build() -> str:
    """Compile liboracle.so (gcc) if it is missing or older than its source."""
    so = os.path.join(_HERE, "liboracle.so")
    src = os.path.join(_HERE, "ferret_oracle.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "liboracle.so"])
    return so


def lib():
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(build())
        L = _LIB
        L.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_e4m3_to_f32.restype = ctypes.c_float
        L.orc_f32_to_e4m3.argtypes = [ctypes.c_float]
        L.orc_f32_to_e4m3.restype = ctypes.c_uint8
        L.orc_moe_permute.argtypes = [_p, _i, _i, _i, _p, _p, _p]
        L.orc_quant_act_fp8_1x128.argtypes = [_p, _p, _i, _i, _i, _p, _p]
        L.orc_quant_act_fp8_1x128_ue8m0.argtypes = [_p, _p, _i, _i, _i, _p, _p]
        L.orc_fp8_grouped_gemm.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p]
        L.orc_int4_w13.argtypes = [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p]
    return _LIB


# ---------------------------------------------------------------------------
# scalar formats
# ---------------------------------------------------------------------------

def e4m3_lut() -> np.ndarray:
    L = lib()
    return np.array([L.orc_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)


_E4M3 = None


def e4m3_to_f32(q: np.ndarray) -> np.ndarray:
    global _E4M3
    if _E4M3 is None:
        _E4M3 = e4m3_lut()
    return _E4M3[q.astype(np.uint8)]


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (uint16)."""
    f = np.ascontiguousarray(f, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[np.isnan(f)] = 0x7FC0
    return r


def f32_to_e4m3(f: np.ndarray) -> np.ndarray:
    """Vectorised RNE fp32 -> e4m3fn with saturation (same rule as the C)."""
    f = np.asarray(f, dtype=np.float32)
    a = np.abs(f).astype(np.float64)
    sign = np.signbit(f).astype(np.uint8) << 7
    code = np.zeros(f.shape, dtype=np.int32)
    sub = a < 2.0 ** -6
    code[sub] = np.rint(a[sub] * 512.0).astype(np.int32)
    nrm = ~sub
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(nrm, a, 1.0))).astype(np.int32)
    # log2 can be off by one ulp at exact powers of two; fix the bracket
    lo = np.ldexp(1.0, e)
    e = np.where(a < lo, e - 1, e)
    e = np.where(a >= np.ldexp(1.0, e + 1), e + 1, e)
    n = np.rint(np.ldexp(a, 3 - e)).astype(np.int32)
    code = np.where(nrm, ((e + 7) << 3) + (n - 8), code)
    code = np.minimum(code, 0x7E)
    out = (code.astype(np.uint8) | sign).astype(np.uint8)
    out[np.isnan(f)] = 0x7F | sign[np.isnan(f)]
    return out


# ---------------------------------------------------------------------------
# scalar-restatement wrappers
# ---------------------------------------------------------------------------

def moe_permute(topk_ids: np.ndarray, E: int):
    ids = np.ascontiguousarray(topk_ids, dtype=np.int32)
    T, topk = ids.shape
    R = T * topk
    sorted_rows = np.empty(R, np.int32)
    offsets = np.empty(E + 1, np.int32)
    m_indices = np.empty(R, np.int32)
    lib().orc_moe_permute(_ptr(ids), T, topk, E, _ptr(sorted_rows), _ptr(offsets), _ptr(m_indices))
    return sorted_rows, offsets, m_indices


def moe_align_block_size(topk_ids: np.ndarray, E: int, block_size: int):
    """The block-padded layout of vLLM's moe_align_block_size with
    ignore_invalid_experts=True, restated from its published description
    (vllm/model_executor/layers/fused_moe/moe_align_block_size.py, the function
    called at baselines/kimi-moe-w13-int4/baseline_marlin.py:123-126), with the
    stable order inside an expert: returns (sorted_ids, expert_ids, num_post_pad)."""
    flat = np.asarray(topk_ids, np.int64).reshape(-1)
    numel = flat.size
    max_padded = numel + E * (block_size - 1)
    if numel < E:
        max_padded = min(max_padded, numel * block_size)
    max_blocks = -(-max_padded // block_size)
    sorted_ids = np.full(max_padded, numel, np.int32)
    expert_ids = np.full(max_blocks, -1, np.int32)
    p = 0
    for e in range(E):
        idx = np.nonzero(flat == e)[0]
        n = -(-idx.size // block_size) * block_size
        sorted_ids[p:p + idx.size] = idx
        expert_ids[p // block_size:(p + n) // block_size] = e
        p += n
    return sorted_ids, expert_ids, np.array([p], np.int32)


def per_block_cast_to_fp8(w: np.ndarray, ue8m0: bool = False):
    """128x128 block weight quantization: DeepGEMM per_block_cast_to_fp8 as
    called at baselines/fp8-group-gemm/baseline_dsv3_decode.py:44-47
    (use_ue8m0=False), restated with IEEE float32 steps.

    w: float32 [..., N, K], N and K multiples of 128.  Per block: amax =
    max|w| clamped at 1e-4; f = fl(fl(1/amax) * 448) (torch's `448.0 / amax`
    is reciprocal-then-multiply); q = e4m3_rne_satfinite(fl(w * f)); scale =
    fl(amax / 448).  ue8m0: scale = the smallest power of two >= fl(amax /
    448) (from the bits) and f = its exact inverse.
    Returns (e4m3 bytes [..., N, K], float32 scales [..., N/128, K/128])."""
    w = np.ascontiguousarray(w, np.float32)
    *lead, N, K = w.shape
    v = w.reshape(*lead, N // 128, 128, K // 128, 128)
    amax = np.maximum(np.abs(v).max(axis=(-3, -1), keepdims=True), np.float32(1e-4))
    s = (amax / np.float32(448)).astype(np.float32)
    if ue8m0:
        bits = s.view(np.uint32)
        ex = (bits >> 23) + ((bits & 0x7FFFFF) != 0).astype(np.uint32)
        s = (ex << 23).astype(np.uint32).view(np.float32)
        f = ((254 - ex) << 23).astype(np.uint32).view(np.float32)
    else:
        f = ((np.float32(1) / amax).astype(np.float32) * np.float32(448)).astype(np.float32)
    q = f32_to_e4m3((v * f).astype(np.float32)).reshape(*lead, N, K)
    return q, np.ascontiguousarray(s.reshape(*lead, N // 128, K // 128))


def quant_act_fp8_1x128(x_bf16: np.ndarray, gather_rows: np.ndarray | None = None,
                        gather_div: int = 1, R: int | None = None, ue8m0: bool = False):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    K = x.shape[1]
    if gather_rows is not None:
        gather_rows = np.ascontiguousarray(gather_rows, dtype=np.int32)
        R = gather_rows.shape[0] if R is None else R
    else:
        R = x.shape[0] if R is None else R
    q = np.empty((R, K), np.uint8)
    s = np.empty((R, K // 128), np.float32)
    fn = lib().orc_quant_act_fp8_1x128_ue8m0 if ue8m0 else lib().orc_quant_act_fp8_1x128
    fn(_ptr(x), _ptr(gather_rows), gather_div, R, K, _ptr(q), _ptr(s))
    return q, s


def fp8_grouped_gemm(a, a_scale, w, w_scale, m_indices, silu=False, out=None):
    a = np.ascontiguousarray(a, np.uint8)
    a_scale = np.ascontiguousarray(a_scale, np.float32)
    w = np.ascontiguousarray(w, np.uint8)
    w_scale = np.ascontiguousarray(w_scale, np.float32)
    m_indices = np.ascontiguousarray(m_indices, np.int32)
    M, K = a.shape
    E, N, _ = w.shape
    if out is None:
        out = np.full((M, N // 2 if silu else N), np.nan, np.float32)
    lib().orc_fp8_grouped_gemm(_ptr(a), _ptr(a_scale), _ptr(w), _ptr(w_scale), _ptr(m_indices),
                               M, N, K, E, int(silu), _ptr(out))
    return out


def int4_w13(hidden_bf16, raw_q, scales_bf16, topk_ids, silu=True, out=None):
    hidden = np.ascontiguousarray(hidden_bf16, np.uint16)
    raw_q = np.ascontiguousarray(raw_q, np.int32)
    scales = np.ascontiguousarray(scales_bf16, np.uint16)
    ids = np.ascontiguousarray(topk_ids, np.int32)
    T, K = hidden.shape
    E, _, N = raw_q.shape
    topk = ids.shape[1]
    if out is None:
        out = np.full((T * topk, N // 2 if silu else N), np.nan, np.float32)
    lib().orc_int4_w13(_ptr(hidden), _ptr(raw_q), _ptr(scales), _ptr(ids), T, topk, N, K, E,
                       int(silu), _ptr(out))
    return out


# ---------------------------------------------------------------------------
# numpy dequantize-then-matmul versions (large sizes, CPU baseline)
# ---------------------------------------------------------------------------

def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """correctness/compare_marlin_vs_ref.py:94-97 in fp32."""
    g = g.astype(np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))) * u


def dequant_w_fp8(w_e: np.ndarray, ws_e: np.ndarray) -> np.ndarray:
    """One expert [N, K] e4m3 with [N/128, K/128] scales -> fp32 [N, K]."""
    N, K = w_e.shape
    d = e4m3_to_f32(w_e).reshape(N // 128, 128, K // 128, 128)
    d *= ws_e[:, None, :, None]
    return d.reshape(N, K)


def fp8_grouped_gemm_fast(a, a_scale, w, w_scale, m_indices, silu=False, rows=None):
    """fp32 dequantize-then-matmul of the rows in ``rows`` (default: all)."""
    M, K = a.shape
    E, N, _ = w.shape
    m_indices = np.asarray(m_indices)
    if rows is None:
        rows = np.arange(M)
    rows = np.asarray(rows)
    out = np.full((len(rows), N // 2 if silu else N), np.nan, np.float32)
    ad = e4m3_to_f32(a[rows]).reshape(len(rows), K // 128, 128)
    ad *= a_scale[rows][:, :, None]
    ad = ad.reshape(len(rows), K)
    ex = m_indices[rows]
    for e in np.unique(ex):
        if e < 0 or e >= E:
            continue
        sel = np.nonzero(ex == e)[0]
        acc = ad[sel] @ dequant_w_fp8(w[e], w_scale[e]).T
        out[sel] = silu_mul(acc[:, : N // 2], acc[:, N // 2:]) if silu else acc
    return out


def int4_dequant(raw_q_e: np.ndarray, scales_e: np.ndarray) -> np.ndarray:
    """raw [K/8, N] int32 + bf16 bits [K/32, N] -> bf16-rounded fp32 [N, K]."""
    K8, N = raw_q_e.shape
    u = raw_q_e.astype(np.uint32)
    nib = np.stack([(u >> (4 * s)) & 0xF for s in range(8)], axis=1)  # [K/8, 8, N]
    signed = nib.reshape(K8 * 8, N).astype(np.float32) - np.float32(8.0)
    sc = np.repeat(bf16_to_f32(scales_e), 32, axis=0)                   # [K, N]
    w = bf16_to_f32(f32_to_bf16(signed * sc))
    return np.ascontiguousarray(w.T)


def int4_w13_fast(hidden_bf16, raw_q, scales_bf16, topk_ids, silu=True, pairs=None):
    T, K = hidden_bf16.shape
    E, _, N = raw_q.shape
    topk = topk_ids.shape[1]
    flat = np.asarray(topk_ids).reshape(-1)
    if pairs is None:
        pairs = np.arange(T * topk)
    pairs = np.asarray(pairs)
    a = bf16_to_f32(hidden_bf16)
    out = np.full((len(pairs), N // 2 if silu else N), np.nan, np.float32)
    ex = flat[pairs]
    for e in np.unique(ex):
        if e < 0 or e >= E:
            continue
        sel = np.nonzero(ex == e)[0]
        acc = a[pairs[sel] // topk] @ int4_dequant(raw_q[e], scales_bf16[e]).T
        out[sel] = silu_mul(acc[:, : N // 2], acc[:, N // 2:]) if silu else acc
    return out


# ---------------------------------------------------------------------------
# comparison metric
# ---------------------------------------------------------------------------

def rel_err(got: np.ndarray, ref: np.ndarray) -> dict:
    """Max relative error with denominator max(|ref|, 1e-3*max|ref|), NaN
    counted as failure (v007:547-551, tasks/kimi-moe-w13-int4-grouped-gemm.yaml:171-184)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    finite_ref = np.isfinite(ref)
    amax = np.max(np.abs(ref[finite_ref])) if finite_ref.any() else 0.0
    floor = max(amax * 1e-3, 1e-30)
    bad = ~np.isfinite(got) | ~finite_ref
    d = np.abs(got - ref)
    re = np.where(bad, np.inf, d / np.maximum(np.abs(ref), floor))
    return {
        "max_rel": float(np.max(re)) if re.size else 0.0,
        "max_abs": float(np.max(np.where(bad, np.inf, d))) if d.size else 0.0,
        "nan": int(np.count_nonzero(bad)),
    }


# ---------------------------------------------------------------------------
# torch CPU fp32 path (the CPU baseline: multi-threaded dequantize-then-matmul)
# ---------------------------------------------------------------------------

def fp8_w13_torch_cpu(a_q, a_scale, w_q, w_scale, offsets, experts, silu=False):
    """fp32 dequantize-then-matmul on the host cores with torch, one expert at a
    time (streamed: dequantizing every expert at once would need tens of GB).

    a_q e4m3 [R, K] (torch float8 or uint8), a_scale f32 [R, K/128],
    w_q e4m3 [E, N, K], w_scale f32 [E, N/128, K/128], offsets int [E+1]
    (expert-contiguous rows); `experts` lists the experts to compute.
    Returns {expert: fp32 [rows_e, N or N/2]}.
    """
    import torch
    f8 = torch.float8_e4m3fn
    a_q = a_q.view(f8) if a_q.dtype != f8 else a_q
    w_q = w_q.view(f8) if w_q.dtype != f8 else w_q
    R, K = a_q.shape
    E, N, _ = w_q.shape
    out = {}
    for e in experts:
        r0, r1 = int(offsets[e]), int(offsets[e + 1])
        if r1 <= r0:
            continue
        a = a_q[r0:r1].float().view(r1 - r0, K // 128, 128) * a_scale[r0:r1].unsqueeze(2)
        w = w_q[e].float().view(N // 128, 128, K // 128, 128) * w_scale[e].view(N // 128, 1, K // 128, 1)
        acc = a.view(r1 - r0, K) @ w.view(N, K).t()
        if silu:
            g, u = acc[:, : N // 2], acc[:, N // 2:]
            acc = g / (1.0 + torch.exp(-g)) * u
        out[e] = acc
    return out


def int4_w13_torch_cpu(x_bf16, raw_e, scales_e, silu=True):
    """One expert of the INT4 W4A16 W13 on the host cores with torch, fp32
    dequantize-then-matmul as in correctness/compare_marlin_vs_ref.py:44-100:
    w[k, n] = bf16((nibble(k, n) - 8) * scale[k // 32, n]), out = x @ w.

    x_bf16 [rows, K] bf16; raw_e int32 [K/8, N] (nibble s of word k8 is
    k = 8*k8 + s); scales_e bf16 [K/32, N].  Returns fp32 [rows, N or N/2].
    """
    import torch
    K8, N = raw_e.shape
    shifts = torch.arange(0, 32, 4, dtype=torch.int32).view(1, 8, 1)
    nib = (raw_e.view(K8, 1, N) >> shifts) & 0xF                          # [K/8, 8, N]
    w = (nib.reshape(K8 * 8, N).float() - 8.0) * scales_e.float().repeat_interleave(32, 0)
    w = w.to(torch.bfloat16).float()
    acc = x_bf16.float() @ w
    if silu:
        g, u = acc[:, : N // 2], acc[:, N // 2:]
        acc = g / (1.0 + torch.exp(-g)) * u
    return acc


def fp8_moe_ffn(hidden_bf16, topk_ids, topk_weights, w13, w13_s, w2, w2_s):
    """The FP8 MoE expert layer restated for the CPU: per (token, slot) pair,
    1x128 quant -> W13 (fp32, exact block scales) -> SiLU(gate)*up -> bf16 ->
    1x128 quant -> W2 -> bf16; then the fp32 top-k weighted sum in slot order
    -> bf16.  Pairs with an id outside [0, E) are skipped.  Returns fp32 values
    of the bf16 result, [T, H]."""
    T, H = hidden_bf16.shape
    topk = topk_ids.shape[1]
    E = w13.shape[0]
    flat = np.asarray(topk_ids).reshape(-1)
    pairs = np.nonzero((flat >= 0) & (flat < E))[0]
    a = hidden_bf16[pairs // topk]
    q1, s1 = quant_act_fp8_1x128(a)
    y1 = fp8_grouped_gemm_fast(q1, s1, w13, w13_s, flat[pairs].astype(np.int32), silu=True)
    y1 = f32_to_bf16(y1)
    q2, s2 = quant_act_fp8_1x128(y1)
    y2 = bf16_to_f32(f32_to_bf16(fp8_grouped_gemm_fast(q2, s2, w2, w2_s, flat[pairs].astype(np.int32))))
    out = np.zeros((T, H), np.float32)
    w = np.asarray(topk_weights, np.float32).reshape(-1)
    for j in range(topk):                      # slot order, as the device sums
        sel = np.nonzero(pairs % topk == j)[0]
        t = pairs[sel] // topk
        out[t] = out[t] + w[pairs[sel]][:, None] * y2[sel]
    return bf16_to_f32(f32_to_bf16(out))
