// moe_permute.cu -- top-k routing ids -> expert-contiguous row order.
//
// A stable counting sort of the flat (token*topk + slot) index by expert,
// the order the contiguous grouped-GEMM layout needs
// (tasks/fp8-group-gemm-dsv3-prefill.yaml:18-21).  One CTA of 16 warps:
//   1. each warp walks its contiguous share of the ids 32 at a time and
//      builds a private histogram with warp-ballot aggregation
//      (__match_any_sync: one leader per distinct expert adds the group size);
//   2. block scan over experts -> expert_offsets, then each warp's base per
//      expert = offset + counts of the warps before it;
//   3. the warps re-walk their shares; an item's slot is its warp base plus
//      its rank among equal ids in the 32-wide batch (popc of the match mask
//      below the lane), so the order inside an expert is the index order.
// Integer-only; bit-exact with the CPU restatement.
#include "capi_internal.h"

namespace ferret {
namespace {

constexpr int kPermWarps = 16;
constexpr int kPermThreads = kPermWarps * 32;

__global__ void __launch_bounds__(kPermThreads, 1)
    moe_permute_kernel(const int32_t* __restrict__ ids, int R, int E,
                       int32_t* __restrict__ sorted_rows, int32_t* __restrict__ offsets_out,
                       int32_t* __restrict__ m_indices) {
    extern __shared__ int smem[];
    int* hist = smem;                                   // [kPermWarps][E]
    int* offs = hist + kPermWarps * E;                  // [E+1]
    int* part = offs + E + 1;                           // [kPermThreads+1]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const unsigned lt_mask = (1u << lane) - 1u;
    // each warp's share is a multiple of 32 so batches never straddle warps
    const int share = ((R + kPermWarps - 1) / kPermWarps + 31) & ~31;
    const int lo = min(R, warp * share), hi = min(R, lo + share);
    int* my = hist + warp * E;

    for (int i = tid; i < kPermWarps * E; i += kPermThreads) hist[i] = 0;
    __syncthreads();

    // 1. per-warp histograms
    for (int base = lo; base < hi; base += 32) {
        const int i = base + lane;
        int e = (i < hi) ? ids[i] : -1;
        if (e < 0 || e >= E) e = -1;
        const unsigned grp = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(grp) - 1) my[e] += __popc(grp);
        __syncwarp();
    }
    __syncthreads();

    // 2. offsets and per-warp bases
    for (int e = tid; e < E; e += kPermThreads) {
        int t = 0;
        for (int w = 0; w < kPermWarps; ++w) t += hist[w * E + e];
        offs[e] = t;
    }
    __syncthreads();
    block_exclusive_scan(offs, E, part);
    for (int e = tid; e < E; e += kPermThreads) {
        int run = offs[e];
        for (int w = 0; w < kPermWarps; ++w) {
            const int c = hist[w * E + e];
            hist[w * E + e] = run;
            run += c;
        }
    }
    for (int e = tid; e <= E; e += kPermThreads) offsets_out[e] = offs[e];
    __syncthreads();

    // 3. stable scatter
    for (int base = lo; base < hi; base += 32) {
        const int i = base + lane;
        int e = (i < hi) ? ids[i] : -1;
        if (e < 0 || e >= E) e = -1;
        const unsigned grp = __match_any_sync(0xffffffffu, e);
        if (e >= 0) {
            const int pos = my[e] + __popc(grp & lt_mask);
            sorted_rows[pos] = i;
            m_indices[pos] = e;
        }
        __syncwarp();
        if (e >= 0 && lane == __ffs(grp) - 1) my[e] += __popc(grp);
        __syncwarp();
    }
    // tail: dropped ids leave unused slots at the end
    for (int p = offs[E] + tid; p < R; p += kPermThreads) {
        sorted_rows[p] = -1;
        m_indices[p] = -1;
    }
}

}  // namespace
}  // namespace ferret

using namespace ferret;

extern "C" int ferret_moe_permute(const int32_t* topk_ids, int T, int topk, int E,
                                  int32_t* sorted_rows, int32_t* expert_offsets,
                                  int32_t* m_indices, void* workspace, size_t ws_bytes,
                                  void* stream) {
    (void)workspace;
    (void)ws_bytes;
    if (T < 0 || topk <= 0 || E <= 0 || E > 1024) return FERRET_ERR_SHAPE;
    if (!expert_offsets) return FERRET_ERR_NULL;
    const long long R = (long long)T * topk;
    if (R > (1ll << 30)) return FERRET_ERR_SHAPE;
    if (R > 0 && (!topk_ids || !sorted_rows || !m_indices)) return FERRET_ERR_NULL;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    const size_t smem = sizeof(int) * ((size_t)kPermWarps * E + E + 1 + kPermThreads + 1);
    if (smem > (size_t)info->max_smem_optin) return FERRET_ERR_SHAPE;
    if (cudaFuncSetAttribute(moe_permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    moe_permute_kernel<<<1, kPermThreads, smem, as_stream(stream)>>>(
        topk_ids, (int)R, E, sorted_rows, expert_offsets, m_indices);
    return launch_status();
}
