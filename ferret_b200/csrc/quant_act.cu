// quant_act.cu -- per-token 1x128 FP8 (e4m3) activation quantization with an
// optional row gather, so that the expert-sorted A operand is produced in one
// pass straight from the token-ordered hidden states.
//
// Algorithm (DeepGEMM per_token_cast_to_fp8 with use_ue8m0=False, as called at
// baselines/fp8-group-gemm/baseline_dsv3_decode.py:42): per 128-element block,
// amax = max(|x|) clamped at 1e-4, f = fl(fl(1/amax) * 448) (torch evaluates
// `448.0 / amax` as reciprocal-then-multiply), q = e4m3(fl(x * f)) with
// round-to-nearest-even and saturation, scale = fl(amax / 448).  Every step is
// IEEE round-to-nearest (no fast-math), so the result is bit-identical to the
// CPU restatement.  The UE8M0 form (use_ue8m0=True) rounds the scale up to a
// power of two and multiplies by its exact inverse.
//
// HBM-bound: a warp quantizes 4 blocks of a row per task, 16 bytes per lane in.
#include "capi_internal.h"

namespace ferret {
namespace {

constexpr int kQuantThreads = 256;
constexpr int kBlocksPerTask = 4;     // 128-element blocks one warp handles per task

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// A warp task is (row, 4 consecutive 128-element blocks).  Each half-warp
// covers one block with 16-byte loads; both loads of a lane are issued before
// either is used, so 1 KB per warp is in flight (the kernel is bound by the
// latency of the gathered row reads, not by HBM, at decode sizes).
// UE8M0: the scale is the smallest power of two >= fl(amax / 448), taken from
// the fp32 bits (exact; no log2), and x is multiplied by its exact inverse.
// SCATTER: row r is token r (R = x_rows), and its quantized row is written to
// every row inv[r * gather_div + j], j < gather_div, that is not negative (the
// expert-sorted positions of the token's top-k pairs): each token is
// quantized once and its bytes go straight to its routed copies.
template <bool UE8M0, bool SCATTER = false>
__global__ void __launch_bounds__(kQuantThreads)
    quant_act_kernel(const __nv_bfloat16* __restrict__ x, int x_rows,
                     const int32_t* __restrict__ gather, int gather_div, int R, int K,
                     uint8_t* __restrict__ q, float* __restrict__ scale, DevCtl ctl) {
    pdl_begin();
    const int nk = K >> 7;
    const int tasks_per_row = (nk + kBlocksPerTask - 1) / kBlocksPerTask;
    const long long tasks = (long long)R * tasks_per_row;
    const int lane = threadIdx.x & 31;
    const int half = lane >> 4, hl = lane & 15;
    const long long warps = (long long)gridDim.x * (kQuantThreads / 32);
    for (long long task = (long long)blockIdx.x * (kQuantThreads / 32) + (threadIdx.x >> 5);
         task < tasks; task += warps) {
        const int r = (int)(task / tasks_per_row);
        const int b0 = (int)(task - (long long)r * tasks_per_row) * kBlocksPerTask;
        long long src = r;
        if (!SCATTER && gather) {
            const int g = gather[r];
            src = g < 0 ? -1 : g / gather_div;
            if (src >= x_rows) {            // out-of-range gather: zero row + status
                if (lane == 0) report(ctl, DEV_BAD_ROW);
                src = -1;
            }
        }
        uint4 raw[kBlocksPerTask / 2];
#pragma unroll
        for (int i = 0; i < kBlocksPerTask / 2; ++i) {
            const int b = b0 + 2 * i + half;
            raw[i] = (src >= 0 && b < nk)
                         ? *reinterpret_cast<const uint4*>(x + src * K + b * 128 + hl * 8)
                         : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < kBlocksPerTask / 2; ++i) {
            const int b = b0 + 2 * i + half;
            const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
            float v[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[2 * j] = bf16_lo(w[j]);
                v[2 * j + 1] = bf16_hi(w[j]);
            }
            float amax = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
            for (int off = 8; off > 0; off >>= 1)      // within the 16-lane half
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            if (b >= nk) continue;
            amax = fmaxf(amax, 1e-4f);
            float f, sc;
            if (UE8M0) {
                const uint32_t bits = __float_as_uint(__fdiv_rn(amax, 448.0f));
                const uint32_t ex = (bits >> 23) + ((bits & 0x7FFFFFu) ? 1u : 0u);
                sc = __uint_as_float(ex >= 255u ? 0x7F800000u : ex << 23);
                f = ex >= 255u ? 0.0f
                               : __uint_as_float(ex == 254u ? 0x00400000u : (254u - ex) << 23);
            } else {
                // `448.0 / amax` in the published torch code is reciprocal-then-multiply
                f = __fmul_rn(__frcp_rn(amax), 448.0f);
                sc = __fdiv_rn(amax, 448.0f);
            }
            uint32_t packed[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
                    make_float2(__fmul_rn(v[4 * j], f), __fmul_rn(v[4 * j + 1], f)), __NV_SATFINITE,
                    __NV_E4M3);
                const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
                    make_float2(__fmul_rn(v[4 * j + 2], f), __fmul_rn(v[4 * j + 3], f)),
                    __NV_SATFINITE, __NV_E4M3);
                packed[j] = (uint32_t)lo | ((uint32_t)hi << 16);
            }
            if (SCATTER) {
                for (int j = 0; j < gather_div; ++j) {
                    const int p = __ldg(gather + (long long)r * gather_div + j);
                    if (p < 0) continue;
                    *reinterpret_cast<uint2*>(q + (long long)p * K + b * 128 + hl * 8) =
                        make_uint2(packed[0], packed[1]);
                    if (hl == 0) scale[(long long)p * nk + b] = sc;
                }
                continue;
            }
            uint8_t* qdst = q + (long long)r * K + b * 128 + hl * 8;
            if (src < 0) {
                packed[0] = packed[1] = 0u;
            }
            *reinterpret_cast<uint2*>(qdst) = make_uint2(packed[0], packed[1]);
            if (hl == 0) scale[(long long)r * nk + b] = src < 0 ? 0.0f : sc;
        }
    }
}

}  // namespace
}  // namespace ferret

using namespace ferret;

template <bool UE8M0>
static int quant_act(const void* x_bf16, int x_rows, const int32_t* gather_rows, int gather_div,
                     int R, int K, void* a_fp8, float* a_scale, void* stream) {
    if (R < 0 || K <= 0 || (K % 128) != 0 || x_rows < 0) return FERRET_ERR_SHAPE;
    if (!gather_rows && R > x_rows) return FERRET_ERR_SHAPE;
    if (R == 0) return FERRET_OK;
    if (!x_bf16 || !a_fp8 || !a_scale) return FERRET_ERR_NULL;
    if (gather_rows && gather_div <= 0) return FERRET_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(x_bf16) & 15u) || (reinterpret_cast<uintptr_t>(a_fp8) & 7u) ||
        (reinterpret_cast<uintptr_t>(a_scale) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    const long long tasks = (long long)R * ((K / 128 + kBlocksPerTask - 1) / kBlocksPerTask);
    const long long want = (tasks + (kQuantThreads / 32) - 1) / (kQuantThreads / 32);
    const int grid = (int)(want < (long long)info->num_sms * 16 ? want : (long long)info->num_sms * 16);
    return launch_kernel(quant_act_kernel<UE8M0>, dim3(grid), dim3(kQuantThreads), 0,
                         as_stream(stream), static_cast<const __nv_bfloat16*>(x_bf16), x_rows,
                         gather_rows, gather_div, R, K, static_cast<uint8_t*>(a_fp8), a_scale,
                         make_ctl(info));
}

extern "C" int ferret_quant_act_fp8_1x128(const void* x_bf16, int x_rows,
                                          const int32_t* gather_rows, int gather_div, int R, int K,
                                          void* a_fp8, float* a_scale, void* stream) {
    return quant_act<false>(x_bf16, x_rows, gather_rows, gather_div, R, K, a_fp8, a_scale, stream);
}

extern "C" int ferret_quant_act_fp8_1x128_ue8m0(const void* x_bf16, int x_rows,
                                                const int32_t* gather_rows, int gather_div, int R,
                                                int K, void* a_fp8, float* a_scale, void* stream) {
    return quant_act<true>(x_bf16, x_rows, gather_rows, gather_div, R, K, a_fp8, a_scale, stream);
}

// ---------------------------------------------------------------------------
// Quantize-and-scatter: each token row is quantized once and written to the
// expert-sorted positions of its top-k pairs (the inverse of the permutation's
// sorted_rows), which gives the same A operand as the gathered quantizer with
// topk-fold less arithmetic and without a separate row-gather pass.
// ---------------------------------------------------------------------------
namespace ferret {
namespace {

// inv[sorted[p]] = p for the valid sorted positions p < offsets[E]
// (inv pre-filled with -1: pairs whose expert id is invalid keep -1).
__global__ void __launch_bounds__(256)
    inverse_rows_kernel(const int32_t* __restrict__ sorted, const int32_t* __restrict__ off_end,
                        int R, int32_t* __restrict__ inv, DevCtl ctl) {
    pdl_begin();
    const int valid = *off_end;
    for (int p = blockIdx.x * 256 + threadIdx.x; p < R; p += gridDim.x * 256) {
        if (p >= valid) continue;
        const int v = sorted[p];
        if (v < 0 || v >= R) {
            report(ctl, DEV_BAD_ROW);
            continue;
        }
        inv[v] = p;
    }
}

}  // namespace
}  // namespace ferret

extern "C" int ferret_quant_act_fp8_1x128_scatter(const void* x_bf16, int T, int topk,
                                                  const int32_t* sorted_rows,
                                                  const int32_t* expert_offsets, int E, int K,
                                                  void* a_fp8, float* a_scale, int32_t* inv_ws,
                                                  int flags, void* stream) {
    if (T < 0 || topk <= 0 || E <= 0 || K <= 0 || (K % 128) != 0) return FERRET_ERR_SHAPE;
    if ((long long)T * topk >= (1ll << 31)) return FERRET_ERR_SHAPE;
    if (T == 0) return FERRET_OK;
    if (!x_bf16 || !sorted_rows || !expert_offsets || !a_fp8 || !a_scale || !inv_ws)
        return FERRET_ERR_NULL;
    if ((reinterpret_cast<uintptr_t>(x_bf16) & 15u) || (reinterpret_cast<uintptr_t>(a_fp8) & 7u) ||
        (reinterpret_cast<uintptr_t>(a_scale) & 3u) || (reinterpret_cast<uintptr_t>(inv_ws) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    cudaStream_t s = as_stream(stream);
    const int R = T * topk;
    if (cudaMemsetAsync(inv_ws, 0xFF, (size_t)R * sizeof(int32_t), s) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    {
        const int want = (R + 255) / 256;
        const int grid = want < info->num_sms * 8 ? want : info->num_sms * 8;
        if ((rc = launch_kernel(inverse_rows_kernel, dim3(grid), dim3(256), 0, s, sorted_rows,
                                expert_offsets + E, R, inv_ws, make_ctl(info))) != FERRET_OK)
            return rc;
    }
    const long long tasks = (long long)T * ((K / 128 + kBlocksPerTask - 1) / kBlocksPerTask);
    const long long want = (tasks + (kQuantThreads / 32) - 1) / (kQuantThreads / 32);
    const int grid = (int)(want < (long long)info->num_sms * 16 ? want : (long long)info->num_sms * 16);
    const bool ue8m0 = (flags & FERRET_UE8M0_SCALES) != 0;
    return launch_kernel(ue8m0 ? quant_act_kernel<true, true> : quant_act_kernel<false, true>,
                         dim3(grid), dim3(kQuantThreads), 0, s,
                         static_cast<const __nv_bfloat16*>(x_bf16), T,
                         static_cast<const int32_t*>(inv_ws), topk, T, K,
                         static_cast<uint8_t*>(a_fp8), a_scale, make_ctl(info));
}

// ---------------------------------------------------------------------------
// Row gather of already-quantized FP8 rows: out row r = source row
// rows[r] / div (negative -> zero row, scale 0).  Quantizing the T token rows
// once and gathering the T*topk routed copies gives the same bytes as the
// gathered quantizer above at a fraction of its arithmetic (prefill sizes).
// ---------------------------------------------------------------------------
namespace ferret {
namespace {

constexpr int kGatherThreads = 256;

__global__ void __launch_bounds__(kGatherThreads)
    fp8_gather_rows_kernel(const uint4* __restrict__ q, const float* __restrict__ s, int src_rows,
                           const int32_t* __restrict__ rows, int div, int R, int K,
                           uint4* __restrict__ q_out, float* __restrict__ s_out, DevCtl ctl) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int vec = K >> 4, nk = K >> 7;
    const int warps = gridDim.x * (kGatherThreads / 32);
    for (int r = blockIdx.x * (kGatherThreads / 32) + (threadIdx.x >> 5); r < R; r += warps) {
        const int g = rows[r];
        int src = g < 0 ? -1 : g / div;
        if (src >= src_rows) {
            if (lane == 0) report(ctl, DEV_BAD_ROW);
            src = -1;
        }
        uint4* dst = q_out + (size_t)r * vec;
        float* sd = s_out + (size_t)r * nk;
        if (src < 0) {
            for (int c = lane; c < vec; c += 32) dst[c] = make_uint4(0, 0, 0, 0);
            for (int c = lane; c < nk; c += 32) sd[c] = 0.0f;
            continue;
        }
        const uint4* sq = q + (size_t)src * vec;
        const float* ss = s + (size_t)src * nk;
        for (int c = lane; c < vec; c += 32) dst[c] = __ldg(sq + c);
        for (int c = lane; c < nk; c += 32) sd[c] = __ldg(ss + c);
    }
}

}  // namespace
}  // namespace ferret

extern "C" int ferret_fp8_gather_rows(const void* q_fp8, const float* q_scale, int src_rows,
                                      const int32_t* rows, int div, int R, int K, void* out_fp8,
                                      float* out_scale, void* stream) {
    if (R < 0 || K <= 0 || (K % 128) != 0 || src_rows < 0 || div <= 0) return FERRET_ERR_SHAPE;
    if (R == 0) return FERRET_OK;
    if (!q_fp8 || !q_scale || !rows || !out_fp8 || !out_scale) return FERRET_ERR_NULL;
    if (!aligned16(q_fp8) || !aligned16(out_fp8) || (reinterpret_cast<uintptr_t>(q_scale) & 3u) ||
        (reinterpret_cast<uintptr_t>(out_scale) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    const long long want = ((long long)R + kGatherThreads / 32 - 1) / (kGatherThreads / 32);
    const int grid = (int)(want < (long long)info->num_sms * 8 ? want : (long long)info->num_sms * 8);
    return launch_kernel(fp8_gather_rows_kernel, dim3(grid), dim3(kGatherThreads), 0,
                         as_stream(stream), static_cast<const uint4*>(q_fp8), q_scale, src_rows,
                         rows, div, R, K, static_cast<uint4*>(out_fp8), out_scale, make_ctl(info));
}
