// int4_common.cuh -- pieces shared by the two INT4 W13 kernels (the tensor-core
// kernel in int4_grouped_gemm.cu and the decode kernel in int4_decode.cu): the
// exact dequantization of a repacked word and the decode kernel's launcher.
#pragma once

#include <algorithm>

#include "capi_internal.h"

namespace ferret {
namespace {

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// One repacked word (slots hold k offsets 0,2,4,6,1,3,5,7) and the scale
// pair (s, s) -> 8 bf16 weights for k offsets 0..7, as four bf16x2 words.
__device__ __forceinline__ uint4 dequant_word(uint32_t w, uint32_t s2) {
    const uint32_t kMask = 0x000F000Fu, kMagic = 0x43004300u, kBias = 0x43084308u;  // 128, 136
    uint4 r;
    r.x = bf16x2_mul(bf16x2_sub(lop3_and_or(w, kMask, kMagic), kBias), s2);
    r.y = bf16x2_mul(bf16x2_sub(lop3_and_or(w >> 4, kMask, kMagic), kBias), s2);
    r.z = bf16x2_mul(bf16x2_sub(lop3_and_or(w >> 8, kMask, kMagic), kBias), s2);
    r.w = bf16x2_mul(bf16x2_sub(lop3_and_or(w >> 12, kMask, kMagic), kBias), s2);
    return r;
}

}  // namespace

// Register-dequant decode kernel (int4_decode.cu): few token rows per expert.
// a_sorted: [R, K] expert-sorted activation rows; split_ws (nullable): tile
// counters (zeroed before the launch, `ncnt` of them) followed by fp32
// partials, `split_bytes` in all.
int launch_int4_decode(const DeviceInfo* info, const void* a_sorted, const uint8_t* blob,
                       const int32_t* sorted_rows, const int32_t* offsets, void* out, int T,
                       int topk, int N, int K, int E, int R, bool pair, cudaStream_t stream,
                       uint8_t* split_ws, size_t split_bytes, int ncnt);

// Upper bound on the decode kernel's work items (expert, 8-token pass, 128-column
// output block) for R routed rows over E experts -- the split-K counter count.
inline long long int4_decode_items_bound(int R, int E, int N, bool pair) {
    return ((long long)std::min(R, E) + R / 8) * (pair ? N / 256 : N / 128);
}

}  // namespace ferret
