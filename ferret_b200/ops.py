"""Torch-facing operators over the C ABI (device tensors in, device tensors out).

The names and argument tuples mirror the reference's baseline call sites so
the library drops in where they are used:

* ``m_grouped_fp8_gemm_nt_contiguous((A, A_scale), (W, W_scale), out,
  m_indices, disable_ue8m0_cast=True)`` -- DeepGEMM's grouped FP8 GEMM as
  called at baselines/fp8-group-gemm/baseline_dsv3_decode.py:55-57.
* ``per_token_cast_to_fp8(x)`` -- the activation quantizer of
  baselines/fp8-group-gemm/baseline_dsv3_decode.py:42 (use_ue8m0=False).
* ``moe_permute(topk_ids, E)`` -- the routing sort the reference takes from
  vLLM's moe_align_block_size (baselines/kimi-moe-w13-int4/baseline_marlin.py:123-126),
  unpadded: (sorted_rows, expert_offsets, m_indices).
* ``fp8_moe_w13(hidden, topk_ids, W, W_scale)`` -- the whole W13 hot path:
  permute -> gathered per-token quantization -> grouped GEMM.

All calls are asynchronous on ``torch.cuda.current_stream()``.  Every op runs
the CUDA library; there is no CPU or eager-torch fallback.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import (FERRET_PREFILL_PAIRS, FERRET_SILU_MUL, FERRET_TILE_SHIFT, FERRET_UE8M0_SCALES,
                   check, lib)


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t: torch.Tensor, dtype, name: str, ndim: int | None = None):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")


def set_wait_timeout(seconds: float) -> None:
    check(lib().ferret_set_wait_timeout_ns(int(seconds * 1e9)), "ferret_set_wait_timeout_ns")


def last_device_status() -> int:
    st = ctypes.c_int32(0)
    check(lib().ferret_last_device_status(_stream(), ctypes.byref(st)), "ferret_last_device_status")
    return int(st.value)


def moe_permute(topk_ids: torch.Tensor, num_experts: int):
    """topk_ids int32 [T, topk] -> (sorted_rows [T*topk], expert_offsets [E+1], m_indices [T*topk])."""
    _need(topk_ids, torch.int32, "topk_ids", 2)
    T, topk = topk_ids.shape
    dev = topk_ids.device
    sorted_rows = torch.empty(T * topk, dtype=torch.int32, device=dev)
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    m_indices = torch.empty(T * topk, dtype=torch.int32, device=dev)
    ws_bytes = int(lib().ferret_moe_permute_workspace_size(T, topk, num_experts))
    ws = torch.empty(max(ws_bytes, 4) // 4, dtype=torch.int32, device=dev) if ws_bytes else None
    check(lib().ferret_moe_permute(_ptr(topk_ids), T, topk, num_experts, _ptr(sorted_rows),
                                   _ptr(offsets), _ptr(m_indices), _ptr(ws), ws_bytes, _stream()),
          "ferret_moe_permute")
    return sorted_rows, offsets, m_indices


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int,
                         expert_map: torch.Tensor | None = None, pad_sorted_ids: bool = False,
                         ignore_invalid_experts: bool = True):
    """vLLM's moe_align_block_size (baselines/kimi-moe-w13-int4/baseline_marlin.py:123-126):
    returns (sorted_token_ids, expert_ids, num_tokens_post_padded).  Ids outside
    [0, E) are dropped (ignore_invalid_experts=True semantics); expert_map and
    pad_sorted_ids are not supported."""
    if expert_map is not None or pad_sorted_ids:
        raise NotImplementedError("expert_map / pad_sorted_ids are not supported")
    _need(topk_ids, torch.int32, "topk_ids", 2)
    T, topk = topk_ids.shape
    L = lib()
    mp, mb = ctypes.c_int(0), ctypes.c_int(0)
    check(L.ferret_moe_align_block_size_sizes(T, topk, num_experts, block_size, ctypes.byref(mp),
                                              ctypes.byref(mb)), "ferret_moe_align_block_size_sizes")
    dev = topk_ids.device
    sorted_ids = torch.empty(mp.value, dtype=torch.int32, device=dev)
    expert_ids = torch.empty(mb.value, dtype=torch.int32, device=dev)
    post = torch.empty(1, dtype=torch.int32, device=dev)
    ws_bytes = int(L.ferret_moe_align_block_size_workspace_size(T, topk, num_experts))
    ws = torch.empty((ws_bytes + 3) // 4, dtype=torch.int32, device=dev)
    check(L.ferret_moe_align_block_size(_ptr(topk_ids), T, topk, num_experts, block_size,
                                        _ptr(sorted_ids), _ptr(expert_ids), _ptr(post), _ptr(ws),
                                        ws_bytes, _stream()), "ferret_moe_align_block_size")
    return sorted_ids, expert_ids, post


def per_token_cast_to_fp8(x: torch.Tensor, gather_rows: torch.Tensor | None = None,
                          gather_div: int = 1, out=None, use_ue8m0: bool = False):
    """bf16 [rows, K] -> (e4m3 [R, K], f32 scales [R, K/128]).  With gather_rows,
    output row r quantizes x[gather_rows[r] // gather_div] (negative -> zeros).
    use_ue8m0 rounds each scale up to a power of two (the input of the
    block-scaled GEMM, ``disable_ue8m0_cast=False``)."""
    _need(x, torch.bfloat16, "x", 2)
    K = x.shape[1]
    R = x.shape[0] if gather_rows is None else gather_rows.shape[0]
    if gather_rows is not None:
        _need(gather_rows, torch.int32, "gather_rows", 1)
    if out is None:
        q = torch.empty(R, K, dtype=torch.float8_e4m3fn, device=x.device)
        s = torch.empty(R, K // 128, dtype=torch.float32, device=x.device)
    else:
        q, s = out
    name = "ferret_quant_act_fp8_1x128_ue8m0" if use_ue8m0 else "ferret_quant_act_fp8_1x128"
    check(getattr(lib(), name)(_ptr(x), x.shape[0], _ptr(gather_rows), gather_div, R, K, _ptr(q),
                               _ptr(s), _stream()), name)
    return q, s


def per_token_cast_to_fp8_scatter(x: torch.Tensor, sorted_rows: torch.Tensor,
                                  expert_offsets: torch.Tensor, topk: int, out=None,
                                  use_ue8m0: bool = False):
    """bf16 [T, K] -> (e4m3 [T*topk, K], f32 [T*topk, K/128]) in expert-sorted
    order: row p holds token sorted_rows[p] // topk for p < expert_offsets[-1]
    (later rows are left as allocated).  Each token is quantized once; same
    bytes as per_token_cast_to_fp8(x, sorted_rows, topk) on those rows."""
    _need(x, torch.bfloat16, "x", 2)
    _need(sorted_rows, torch.int32, "sorted_rows", 1)
    _need(expert_offsets, torch.int32, "expert_offsets", 1)
    T, K = x.shape
    R = T * topk
    if out is None:
        q = torch.empty(R, K, dtype=torch.float8_e4m3fn, device=x.device)
        s = torch.empty(R, K // 128, dtype=torch.float32, device=x.device)
    else:
        q, s = out
    inv = torch.empty(R, dtype=torch.int32, device=x.device)
    check(lib().ferret_quant_act_fp8_1x128_scatter(
        _ptr(x), T, topk, _ptr(sorted_rows), _ptr(expert_offsets), expert_offsets.numel() - 1, K,
        _ptr(q), _ptr(s), _ptr(inv), FERRET_UE8M0_SCALES if use_ue8m0 else 0, _stream()),
        "ferret_quant_act_fp8_1x128_scatter")
    return q, s


def m_grouped_fp8_gemm_nt_contiguous(a, b, out: torch.Tensor, m_indices: torch.Tensor | None,
                                     disable_ue8m0_cast: bool = True,
                                     expert_offsets: torch.Tensor | None = None,
                                     silu: bool = False, tile: int = 0,
                                     prefill_pairs: bool = False) -> None:
    """out[r] = dequant(A[r]) @ dequant(W[m_indices[r]])^T with exact fp32 block scales.

    ``disable_ue8m0_cast=False`` declares every scale a power of two (UE8M0:
    ``per_token_cast_to_fp8(..., use_ue8m0=True)`` activations and
    ``data.per_block_cast_to_fp8(..., use_ue8m0=True)`` weights); 128-row
    tiles then apply the scales inside the tensor-core MMA
    (kind::mxf8f6f4.block_scale).  Other scales are never rounded: with the
    default ``True`` they are applied in fp32 as given.  ``prefill_pairs`` runs
    each expert's whole 256-row chunks on CTA pairs (tcgen05.mma.cta_group::2).
    """
    A, A_scale = a
    W, W_scale = b
    if A.dtype == torch.float8_e4m3fn:
        A = A.view(torch.uint8)
    if W.dtype == torch.float8_e4m3fn:
        W = W.view(torch.uint8)
    _need(A, torch.uint8, "A", 2)
    _need(W, torch.uint8, "W", 3)
    _need(A_scale, torch.float32, "A_scale", 2)
    _need(W_scale, torch.float32, "W_scale", 3)
    _need(out, torch.bfloat16, "out", 2)
    M, K = A.shape
    E, N, K2 = W.shape
    if K2 != K:
        raise ValueError("A and W disagree on K")
    if out.shape != (M, N // 2 if silu else N):
        raise ValueError(f"out must be [{M}, {N // 2 if silu else N}], got {tuple(out.shape)}")
    ws = None
    ws_bytes = 0
    if expert_offsets is None:
        _need(m_indices, torch.int32, "m_indices", 1)
        ws_bytes = lib().ferret_fp8_grouped_gemm_workspace_size(M, E)
        ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=A.device)
    else:
        _need(expert_offsets, torch.int32, "expert_offsets", 1)
    flags = ((FERRET_SILU_MUL if silu else 0) | (tile << FERRET_TILE_SHIFT)
             | (0 if disable_ue8m0_cast else FERRET_UE8M0_SCALES)
             | (FERRET_PREFILL_PAIRS if prefill_pairs else 0))
    check(lib().ferret_fp8_grouped_gemm_nt_contiguous(
        _ptr(A), _ptr(A_scale), _ptr(W), _ptr(W_scale), _ptr(out), _ptr(m_indices),
        _ptr(expert_offsets), M, N, K, E, flags, _ptr(ws), ws_bytes, _stream()),
        "ferret_fp8_grouped_gemm_nt_contiguous")


def m_grouped_fp8_gemm_scatter(a, b, out: torch.Tensor, expert_offsets: torch.Tensor,
                               out_rows: torch.Tensor, silu: bool = False, tile: int = 0) -> None:
    """Grouped FP8 GEMM whose expert-sorted row i lands in out[out_rows[i]]
    (rows of out_rows outside [0, out.shape[0]) are skipped)."""
    A, A_scale = a
    W, W_scale = b
    if A.dtype == torch.float8_e4m3fn:
        A = A.view(torch.uint8)
    if W.dtype == torch.float8_e4m3fn:
        W = W.view(torch.uint8)
    _need(A, torch.uint8, "A", 2)
    _need(W, torch.uint8, "W", 3)
    _need(A_scale, torch.float32, "A_scale", 2)
    _need(W_scale, torch.float32, "W_scale", 3)
    _need(out, torch.bfloat16, "out", 2)
    _need(expert_offsets, torch.int32, "expert_offsets", 1)
    _need(out_rows, torch.int32, "out_rows", 1)
    M, K = A.shape
    E, N, _ = W.shape
    if out.shape[1] != (N // 2 if silu else N):
        raise ValueError("out has the wrong number of columns")
    flags = (FERRET_SILU_MUL if silu else 0) | (tile << FERRET_TILE_SHIFT)
    check(lib().ferret_fp8_grouped_gemm_scatter(
        _ptr(A), _ptr(A_scale), _ptr(W), _ptr(W_scale), _ptr(out), _ptr(expert_offsets),
        _ptr(out_rows), M, out.shape[0], N, K, E, flags, _stream()),
        "ferret_fp8_grouped_gemm_scatter")


# Routed rows above which the W13 path quantizes each token once and scatters
# its FP8 row to its routed copies (identical bytes; topk-fold less quantizer
# arithmetic, and no separate row-gather pass).
QUANT_ONCE_ROWS = 8192


class W13Buffers:
    """Preallocated intermediates of the fused W13 path for fixed sizes."""

    def __init__(self, T: int, topk: int, K: int, N_out: int, E: int, device):
        R = T * topk
        self.sorted_rows = torch.empty(R, dtype=torch.int32, device=device)
        self.offsets = torch.empty(E + 1, dtype=torch.int32, device=device)
        self.m_indices = torch.empty(R, dtype=torch.int32, device=device)
        self.a = torch.empty(R, K, dtype=torch.uint8, device=device)
        self.a_scale = torch.empty(R, K // 128, dtype=torch.float32, device=device)
        self.out = torch.empty(R, N_out, dtype=torch.bfloat16, device=device)
        ws = int(lib().ferret_moe_permute_workspace_size(T, topk, E))
        self.perm_ws = torch.empty(ws // 4, dtype=torch.int32, device=device) if ws else None
        self.perm_ws_bytes = ws
        self.quant_once = R > QUANT_ONCE_ROWS and topk > 1
        if self.quant_once:
            self.inv = torch.empty(R, dtype=torch.int32, device=device)


def fp8_moe_w13(hidden: torch.Tensor, topk_ids: torch.Tensor, W: torch.Tensor,
                W_scale: torch.Tensor, silu: bool = False, bufs: W13Buffers | None = None,
                tile: int = 0, use_ue8m0: bool = False, prefill_pairs: bool = False):
    """The W13 hot path on one GPU.

    hidden bf16 [T, K], topk_ids int32 [T, topk], W e4m3 [E, N, K],
    W_scale f32 [E, N/128, K/128].  Returns (out, sorted_rows, expert_offsets):
    out bf16 [T*topk, N or N/2] in expert-sorted order; row i of out belongs to
    the (token, slot) pair sorted_rows[i] (= token*topk + slot).
    use_ue8m0: W_scale holds powers of two (``per_block_cast_to_fp8(...,
    use_ue8m0=True)``); activations get power-of-two scales too and the GEMM
    applies both inside the MMA.  prefill_pairs: CTA-pair tiles for whole
    256-row expert chunks.
    """
    _need(hidden, torch.bfloat16, "hidden", 2)
    _need(topk_ids, torch.int32, "topk_ids", 2)
    if W.dtype == torch.float8_e4m3fn:
        W = W.view(torch.uint8)
    T, K = hidden.shape
    topk = topk_ids.shape[1]
    E, N, _ = W.shape
    n_out = N // 2 if silu else N
    if bufs is None:
        bufs = W13Buffers(T, topk, K, n_out, E, hidden.device)
    L = lib()
    s = _stream()
    R = T * topk
    check(L.ferret_moe_permute(_ptr(topk_ids), T, topk, E, _ptr(bufs.sorted_rows),
                               _ptr(bufs.offsets), _ptr(bufs.m_indices), _ptr(bufs.perm_ws),
                               bufs.perm_ws_bytes, s),
          "ferret_moe_permute")
    qname = "ferret_quant_act_fp8_1x128_ue8m0" if use_ue8m0 else "ferret_quant_act_fp8_1x128"
    quant = getattr(L, qname)
    if bufs.quant_once:
        # each token quantized once, written straight to its topk expert-sorted rows
        check(L.ferret_quant_act_fp8_1x128_scatter(
            _ptr(hidden), T, topk, _ptr(bufs.sorted_rows), _ptr(bufs.offsets), E, K, _ptr(bufs.a),
            _ptr(bufs.a_scale), _ptr(bufs.inv), FERRET_UE8M0_SCALES if use_ue8m0 else 0, s),
            "ferret_quant_act_fp8_1x128_scatter")
    else:
        check(quant(_ptr(hidden), T, _ptr(bufs.sorted_rows), topk, R, K, _ptr(bufs.a),
                    _ptr(bufs.a_scale), s), qname)
    flags = ((FERRET_SILU_MUL if silu else 0) | (tile << FERRET_TILE_SHIFT)
             | (FERRET_UE8M0_SCALES if use_ue8m0 else 0)
             | (FERRET_PREFILL_PAIRS if prefill_pairs else 0))
    check(L.ferret_fp8_grouped_gemm_nt_contiguous(
        _ptr(bufs.a), _ptr(bufs.a_scale), _ptr(W), _ptr(W_scale), _ptr(bufs.out), None,
        _ptr(bufs.offsets), R, N, K, E, flags, None, 0, s), "ferret_fp8_grouped_gemm_nt_contiguous")
    return bufs.out, bufs.sorted_rows, bufs.offsets


def moe_combine(y: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor | None = None,
                num_experts: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum_j topk_weights[t, j] * y[t*topk + j] (fp32, slot order, bf16 out);
    pairs whose id is outside [0, num_experts) are skipped when topk_ids is given."""
    _need(y, torch.bfloat16, "y", 2)
    _need(topk_weights, torch.float32, "topk_weights", 2)
    T, topk = topk_weights.shape
    H = y.shape[1]
    if y.shape[0] != T * topk:
        raise ValueError("y must hold T*topk rows")
    if topk_ids is not None:
        _need(topk_ids, torch.int32, "topk_ids", 2)
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=y.device)
    check(lib().ferret_moe_combine(_ptr(y), _ptr(topk_weights), _ptr(topk_ids), num_experts, T,
                                   topk, H, _ptr(out), _stream()), "ferret_moe_combine")
    return out


def fp8_moe_ffn(hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                W13: torch.Tensor, W13_scale: torch.Tensor, W2: torch.Tensor,
                W2_scale: torch.Tensor) -> torch.Tensor:
    """The FP8 MoE expert layer on one GPU: permute -> 1x128 quant -> W13 grouped
    GEMM with fused SiLU(gate)*up -> 1x128 quant of the intermediate -> W2
    grouped GEMM writing (token, slot) order -> top-k weighted combine.

    hidden bf16 [T, H]; topk_ids int32 / topk_weights f32 [T, topk];
    W13 e4m3 [E, 2I, H] + scales [E, 2I/128, H/128]; W2 e4m3 [E, H, I] + scales
    [E, H/128, I/128].  Returns bf16 [T, H]."""
    T, H = hidden.shape
    topk = topk_ids.shape[1]
    E, N13, _ = W13.shape
    if W2.shape[0] != E or W2.shape[1] != H or W2.shape[2] != N13 // 2:
        raise ValueError("W2 must be [E, H, I] with I = W13.shape[1] / 2")
    y1, rows, offs = fp8_moe_w13(hidden, topk_ids, W13, W13_scale, silu=True)
    q2, s2 = per_token_cast_to_fp8(y1)
    y2 = torch.empty(T * topk, H, dtype=torch.bfloat16, device=hidden.device)
    m_grouped_fp8_gemm_scatter((q2, s2), (W2, W2_scale), y2, offs, rows)
    return moe_combine(y2, topk_weights, topk_ids, E)


# ---------------------------------------------------------------- INT4 W4A16

class Int4W13Weights:
    """INT4 W13 weights in the kernel's blob layout (see ferret_int4_repack_w13).

    Built once at load time from the raw compressed-tensors tensors
    (int32 [E, K/8, N], bf16 scales [E, K/32, N])."""

    def __init__(self, w_raw: torch.Tensor, w_scale: torch.Tensor):
        _need(w_raw, torch.int32, "w_raw", 3)
        _need(w_scale, torch.bfloat16, "w_scale", 3)
        E, K8, N = w_raw.shape
        K = K8 * 8
        if tuple(w_scale.shape) != (E, K // 32, N):
            raise ValueError(f"w_scale must be [{E}, {K // 32}, {N}]")
        nbytes = lib().ferret_int4_blob_bytes(E, K, N)
        if nbytes == 0:
            raise ValueError("K and N must be multiples of 128")
        self.E, self.K, self.N = E, K, N
        self.blob = torch.empty(nbytes, dtype=torch.uint8, device=w_raw.device)
        check(lib().ferret_int4_repack_w13(_ptr(w_raw), _ptr(w_scale), _ptr(self.blob), E, K, N,
                                           _stream()), "ferret_int4_repack_w13")


def moe_wna16_w13(hidden: torch.Tensor, weights: Int4W13Weights, topk_ids: torch.Tensor,
                  silu: bool = True, out: torch.Tensor | None = None, tile: int = 0, perm=None,
                  workspace: torch.Tensor | None = None):
    """INT4 W4A16 W13: moe_wna16_marlin_gemm + apply_moe_activation(SILU) in one call.

    hidden bf16 [T, K]; weights from Int4W13Weights; topk_ids int32 [T, topk].
    Returns bf16 [T*topk, N/2 if silu else N] in (token, slot) order; rows of
    pairs with an invalid expert id are left as allocated (zeros when `out` is None).
    """
    _need(hidden, torch.bfloat16, "hidden", 2)
    _need(topk_ids, torch.int32, "topk_ids", 2)
    T, K = hidden.shape
    E, N = weights.E, weights.N
    topk = topk_ids.shape[1]
    if K != weights.K:
        raise ValueError("hidden and weights disagree on K")
    n_out = N // 2 if silu else N
    if out is None:
        out = torch.zeros(T * topk, n_out, dtype=torch.bfloat16, device=hidden.device)
    if perm is None:
        perm = moe_permute(topk_ids, E)
    sorted_rows, offsets, _ = perm
    ws_bytes = lib().ferret_int4_moe_w13_workspace_size(T, topk, K)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=hidden.device)
    flags = (FERRET_SILU_MUL if silu else 0) | (tile << FERRET_TILE_SHIFT)
    check(lib().ferret_int4_moe_w13(_ptr(hidden), _ptr(weights.blob), _ptr(sorted_rows),
                                    _ptr(offsets), _ptr(out), T, topk, N, K, E, flags,
                                    _ptr(workspace), ws_bytes, _stream()), "ferret_int4_moe_w13")
    return out
