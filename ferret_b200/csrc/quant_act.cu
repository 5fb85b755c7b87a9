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
// CPU restatement.
//
// HBM-bound: one warp per 128-element block, 8 bytes per lane in, 4 out.
#include "capi_internal.h"

namespace ferret {
namespace {

constexpr int kQuantThreads = 256;

__global__ void __launch_bounds__(kQuantThreads)
    quant_act_kernel(const __nv_bfloat16* __restrict__ x, int x_rows,
                     const int32_t* __restrict__ gather, int gather_div, int R, int K,
                     uint8_t* __restrict__ q, float* __restrict__ scale, DevCtl ctl) {
    const int nk = K >> 7;
    const long long tasks = (long long)R * nk;
    const int lane = threadIdx.x & 31;
    const long long warps = (long long)gridDim.x * (kQuantThreads / 32);
    for (long long task = (long long)blockIdx.x * (kQuantThreads / 32) + (threadIdx.x >> 5);
         task < tasks; task += warps) {
        const int r = (int)(task / nk), b = (int)(task % nk);
        long long src = r;
        if (gather) {
            const int g = gather[r];
            src = g < 0 ? -1 : g / gather_div;
            if (src >= x_rows) {            // out-of-range gather: zero row + status
                if (lane == 0) report(ctl, DEV_BAD_ROW);
                src = -1;
            }
        }
        uint8_t* qdst = q + (long long)r * K + b * 128 + lane * 4;
        if (src < 0) {
            *reinterpret_cast<uint32_t*>(qdst) = 0u;
            if (lane == 0) scale[(long long)r * nk + b] = 0.0f;
            continue;
        }
        const uint2 raw =
            *reinterpret_cast<const uint2*>(x + src * K + b * 128 + lane * 4);
        const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
        const __nv_bfloat162 p1 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
        const float v0 = __low2float(p0), v1 = __high2float(p0);
        const float v2 = __low2float(p1), v3 = __high2float(p1);
        float amax = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        amax = fmaxf(amax, 1e-4f);
        // `448.0 / amax` in the published torch code is reciprocal-then-multiply
        const float f = __fmul_rn(__frcp_rn(amax), 448.0f);
        const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
            make_float2(__fmul_rn(v0, f), __fmul_rn(v1, f)), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
            make_float2(__fmul_rn(v2, f), __fmul_rn(v3, f)), __NV_SATFINITE, __NV_E4M3);
        *reinterpret_cast<uint32_t*>(qdst) = (uint32_t)lo | ((uint32_t)hi << 16);
        if (lane == 0) scale[(long long)r * nk + b] = __fdiv_rn(amax, 448.0f);
    }
}

}  // namespace
}  // namespace ferret

using namespace ferret;

extern "C" int ferret_quant_act_fp8_1x128(const void* x_bf16, int x_rows,
                                          const int32_t* gather_rows, int gather_div, int R, int K,
                                          void* a_fp8, float* a_scale, void* stream) {
    if (R < 0 || K <= 0 || (K % 128) != 0 || x_rows < 0) return FERRET_ERR_SHAPE;
    if (!gather_rows && R > x_rows) return FERRET_ERR_SHAPE;
    if (R == 0) return FERRET_OK;
    if (!x_bf16 || !a_fp8 || !a_scale) return FERRET_ERR_NULL;
    if (gather_rows && gather_div <= 0) return FERRET_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(x_bf16) & 7u) || (reinterpret_cast<uintptr_t>(a_fp8) & 3u) ||
        (reinterpret_cast<uintptr_t>(a_scale) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    const long long tasks = (long long)R * (K / 128);
    const long long want = (tasks + (kQuantThreads / 32) - 1) / (kQuantThreads / 32);
    const int grid = (int)(want < (long long)info->num_sms * 8 ? want : (long long)info->num_sms * 8);
    quant_act_kernel<<<grid, kQuantThreads, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(x_bf16), x_rows, gather_rows, gather_div, R, K,
        static_cast<uint8_t*>(a_fp8), a_scale, make_ctl(info));
    return launch_status();
}
