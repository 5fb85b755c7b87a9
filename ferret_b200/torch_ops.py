"""Torch operator registrations: ``torch.ops.ferret_moe.*``.

The reference's kernels are reached from torch code either through ctypes
shims or as TORCH_LIBRARY operators (examples/tcgen05-gemm/matmul.cpp:73-95);
this module gives the library the operator form, with the tensor signatures
of the baselines it replaces:

* ``ferret_moe::fp8_grouped_gemm_nt_contiguous(Tensor a, Tensor a_scale,
  Tensor w, Tensor w_scale, Tensor(a!) out, Tensor m_indices, bool silu=False,
  bool disable_ue8m0_cast=True) -> ()`` -- DeepGEMM's
  m_grouped_fp8_gemm_nt_contiguous (baselines/fp8-group-gemm/baseline_dsv3_decode.py:55-57;
  ``disable_ue8m0_cast=False`` declares power-of-two scales);
* ``ferret_moe::per_token_cast_to_fp8(Tensor x, bool use_ue8m0=False) ->
  (Tensor, Tensor)`` (baseline_dsv3_decode.py:42);
* ``ferret_moe::moe_align_block_size(Tensor topk_ids, int block_size,
  int num_experts) -> (Tensor, Tensor, Tensor)``
  (baselines/kimi-moe-w13-int4/baseline_marlin.py:123-126);
* ``ferret_moe::int4_moe_w13(Tensor hidden, Tensor w_raw, Tensor w_scale,
  Tensor topk_ids, bool silu=True) -> Tensor`` -- the raw compressed-tensors
  INT4 weights ([E, K/8, N] int32, [E, K/32, N] bf16), repacked once per
  weight tensor pair (the last pair is cached, by identity and version), then
  moe_wna16_marlin_gemm + SiLU
  (baseline_marlin.py:140-168).

Every operator runs the CUDA library (CUDA tensors only); importing this
module registers them.
"""
from __future__ import annotations

import torch

from . import ops

_LIB = torch.library.Library("ferret_moe", "DEF")
_LIB.define("fp8_grouped_gemm_nt_contiguous(Tensor a, Tensor a_scale, Tensor w, Tensor w_scale, "
            "Tensor(a!) out, Tensor m_indices, bool silu=False, bool disable_ue8m0_cast=True) -> ()")
_LIB.define("per_token_cast_to_fp8(Tensor x, bool use_ue8m0=False) -> (Tensor, Tensor)")
_LIB.define("moe_align_block_size(Tensor topk_ids, int block_size, int num_experts) "
            "-> (Tensor, Tensor, Tensor)")
_LIB.define("int4_moe_w13(Tensor hidden, Tensor w_raw, Tensor w_scale, Tensor topk_ids, "
            "bool silu=True) -> Tensor")

# the last repacked INT4 weight set: (w_raw, w_scale, their versions, blob);
# holding the raw tensors keeps their memory from being reused by others
_INT4_CACHE: list = []


def _fp8_gemm(a, a_scale, w, w_scale, out, m_indices, silu=False, disable_ue8m0_cast=True):
    ops.m_grouped_fp8_gemm_nt_contiguous((a, a_scale), (w, w_scale), out, m_indices,
                                         disable_ue8m0_cast=disable_ue8m0_cast, silu=silu)


def _quant(x, use_ue8m0=False):
    return ops.per_token_cast_to_fp8(x, use_ue8m0=use_ue8m0)


def _align(topk_ids, block_size, num_experts):
    return ops.moe_align_block_size(topk_ids, block_size, num_experts)


def _int4(hidden, w_raw, w_scale, topk_ids, silu=True):
    versions = (w_raw._version, w_scale._version)
    if (_INT4_CACHE and _INT4_CACHE[0] is w_raw and _INT4_CACHE[1] is w_scale
            and _INT4_CACHE[2] == versions):
        packed = _INT4_CACHE[3]
    else:
        _INT4_CACHE.clear()          # one weight set at a time: repacks are GBs
        packed = ops.Int4W13Weights(w_raw, w_scale)
        _INT4_CACHE.extend([w_raw, w_scale, versions, packed])
    return ops.moe_wna16_w13(hidden, packed, topk_ids, silu=silu)


_LIB.impl("fp8_grouped_gemm_nt_contiguous", _fp8_gemm, "CUDA")
_LIB.impl("per_token_cast_to_fp8", _quant, "CUDA")
_LIB.impl("moe_align_block_size", _align, "CUDA")
_LIB.impl("int4_moe_w13", _int4, "CUDA")
