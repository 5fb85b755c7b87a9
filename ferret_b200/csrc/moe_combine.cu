// moe_combine.cu -- top-k weighted combine of the expert outputs, the step
// after the W2 (down) projection that completes the MoE layer:
//
//   out[t, h] = bf16( sum_{j < topk, id(t, j) in [0, E)} w[t, j] * y[t*topk + j, h] )
//
// y holds the W2 rows in (token, slot) order (the scatter form of the grouped
// GEMM writes them there directly); the sum runs in fp32 in slot order, so the
// result is deterministic.  HBM-bound: T*topk*H*2 bytes read, T*H*2 written;
// a thread owns 8 consecutive columns of one token (16-byte loads and stores).
#include "capi_internal.h"

namespace ferret {
namespace {

constexpr int kCombThreads = 256;

__global__ void __launch_bounds__(kCombThreads)
    moe_combine_kernel(const uint4* __restrict__ y, const float* __restrict__ w,
                       const int32_t* __restrict__ ids, int E, int T, int topk, int H,
                       uint4* __restrict__ out) {
    pdl_begin();
    const int vec = H >> 3;                           // 16-byte chunks per row
    const long long total = (long long)T * vec;
    for (long long i = (long long)blockIdx.x * kCombThreads + threadIdx.x; i < total;
         i += (long long)gridDim.x * kCombThreads) {
        const int t = (int)(i / vec), c = (int)(i - (long long)t * vec);
        float acc[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
        for (int j = 0; j < topk; ++j) {
            const int p = t * topk + j;
            if (ids) {
                const int e = __ldg(ids + p);
                if (e < 0 || e >= E) continue;
            }
            const float wj = __ldg(w + p);
            const uint4 v = __ldg(y + (size_t)p * vec + c);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                acc[2 * k] = fmaf(wj, __uint_as_float(u[k] << 16), acc[2 * k]);
                acc[2 * k + 1] = fmaf(wj, __uint_as_float(u[k] & 0xFFFF0000u), acc[2 * k + 1]);
            }
        }
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
            ow[k] = *reinterpret_cast<const uint32_t*>(&b);
        }
        out[(size_t)t * vec + c] = o;
    }
}

}  // namespace
}  // namespace ferret

using namespace ferret;

extern "C" int ferret_moe_combine(const void* y_bf16, const float* topk_weights,
                                  const int32_t* topk_ids, int E, int T, int topk, int H,
                                  void* out_bf16, void* stream) {
    if (T < 0 || topk <= 0 || H <= 0 || H % 8 || (topk_ids && E <= 0)) return FERRET_ERR_SHAPE;
    if (T == 0) return FERRET_OK;
    if (!y_bf16 || !topk_weights || !out_bf16) return FERRET_ERR_NULL;
    if (!aligned16(y_bf16) || !aligned16(out_bf16) ||
        (reinterpret_cast<uintptr_t>(topk_weights) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    const long long total = (long long)T * (H / 8);
    const long long want = (total + kCombThreads - 1) / kCombThreads;
    const int grid = (int)(want < (long long)info->num_sms * 8 ? want : (long long)info->num_sms * 8);
    return launch_kernel(moe_combine_kernel, dim3(grid), dim3(kCombThreads), 0, as_stream(stream),
                         static_cast<const uint4*>(y_bf16), topk_weights, topk_ids, E, T, topk, H,
                         static_cast<uint4*>(out_bf16));
}
