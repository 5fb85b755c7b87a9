// moe_permute.cu -- top-k routing ids -> expert-contiguous row order.
//
// A stable counting sort of the flat (token*topk + slot) index by expert,
// the order the contiguous grouped-GEMM layout needs
// (tasks/fp8-group-gemm-dsv3-prefill.yaml:18-21).  A CTA of 16 warps sorts a
// contiguous chunk of the ids:
//   1. each warp walks its contiguous share of the chunk 32 ids at a time and
//      builds a private histogram with warp-ballot aggregation
//      (__match_any_sync: one leader per distinct expert adds the group size);
//   2. every (warp, expert) gets a base = the expert's offset + the counts of
//      all ids of that expert before the warp's share;
//   3. the warps re-walk their shares; an item's slot is its warp base plus
//      its rank among equal ids in the 32-wide batch (popc of the match mask
//      below the lane), so the order inside an expert is the index order.
// Small batches (decode) run as one CTA over all ids.  Large ones (prefill,
// and the all-rank sort of expert parallelism) split the ids into up to 256
// chunks, one CTA each: a histogram kernel, a one-CTA scan kernel turning the
// per-chunk counts into per-chunk bases, and a scatter kernel.
// Integer-only; bit-exact with the CPU restatement.
#include <algorithm>

#include "capi_internal.h"

namespace ferret {
namespace {

constexpr int kPermWarps = 16;
constexpr int kPermThreads = kPermWarps * 32;
constexpr int kMaxChunks = 256;
constexpr int kChunkMin = 4096;      // ids per CTA below which one CTA does it all
constexpr int kScanThreads = 1024;

__device__ __forceinline__ int expert_of(const int32_t* ids, int i, int hi, int E) {
    int e = (i < hi) ? ids[i] : -1;
    return (e < 0 || e >= E) ? -1 : e;
}

// Step 1 for the CTA's chunk [c0, c1): per-warp histograms in hist[warp][E].
// Returns the warp's share [lo, hi).
__device__ void chunk_histograms(const int32_t* __restrict__ ids, int c0, int c1, int E, int* hist,
                                 int& lo, int& hi) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // each warp's share is a multiple of 32 so batches never straddle warps
    const int share = ((c1 - c0 + kPermWarps - 1) / kPermWarps + 31) & ~31;
    lo = min(c1, c0 + warp * share);
    hi = min(c1, lo + share);
    for (int i = tid; i < kPermWarps * E; i += kPermThreads) hist[i] = 0;
    __syncthreads();
    int* my = hist + warp * E;
    for (int base = lo; base < hi; base += 32) {
        const int e = expert_of(ids, base + lane, hi, E);
        const unsigned grp = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(grp) - 1) my[e] += __popc(grp);
        __syncwarp();
    }
    __syncthreads();
}

// Step 3: hist[warp][e] holds the warp's base slot for expert e.
__device__ void chunk_scatter(const int32_t* __restrict__ ids, int lo, int hi, int E, int* hist,
                              int32_t* __restrict__ sorted_rows, int32_t* __restrict__ m_indices) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned lt_mask = (1u << lane) - 1u;
    int* my = hist + warp * E;
    for (int base = lo; base < hi; base += 32) {
        const int i = base + lane;
        const int e = expert_of(ids, i, hi, E);
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
}

// Unused slots at the end (dropped ids) get -1; grid-strided.
__device__ void fill_tail(int R, int filled, int32_t* sorted_rows, int32_t* m_indices) {
    for (int p = filled + blockIdx.x * blockDim.x + threadIdx.x; p < R; p += gridDim.x * blockDim.x) {
        sorted_rows[p] = -1;
        m_indices[p] = -1;
    }
}

__global__ void __launch_bounds__(kPermThreads, 1)
    moe_permute_kernel(const int32_t* __restrict__ ids, int R, int E,
                       int32_t* __restrict__ sorted_rows, int32_t* __restrict__ offsets_out,
                       int32_t* __restrict__ m_indices) {
    pdl_begin();
    extern __shared__ int smem[];
    int* hist = smem;                                   // [kPermWarps][E]
    int* offs = hist + kPermWarps * E;                  // [E+1]
    int* part = offs + E + 1;                           // [kPermThreads+1]
    const int tid = threadIdx.x;
    int lo, hi;
    chunk_histograms(ids, 0, R, E, hist, lo, hi);
    // offsets and per-warp bases
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
    chunk_scatter(ids, lo, hi, E, hist, sorted_rows, m_indices);
    fill_tail(R, offs[E], sorted_rows, m_indices);
}

// Multi-CTA form, kernel 1: per-chunk expert counts into counts[chunk][E].
__global__ void __launch_bounds__(kPermThreads, 1)
    permute_count_kernel(const int32_t* __restrict__ ids, int R, int E, int chunk,
                         int32_t* __restrict__ counts) {
    pdl_begin();
    extern __shared__ int hist[];                       // [kPermWarps][E]
    const int c0 = blockIdx.x * chunk, c1 = min(R, c0 + chunk);
    int lo, hi;
    chunk_histograms(ids, c0, c1, E, hist, lo, hi);
    for (int e = threadIdx.x; e < E; e += kPermThreads) {
        int t = 0;
        for (int w = 0; w < kPermWarps; ++w) t += hist[w * E + e];
        counts[(size_t)blockIdx.x * E + e] = t;
    }
}

// Kernel 2 (one CTA): counts[c][e] -> base slot of chunk c's first id of
// expert e, in place; expert offsets.
__global__ void __launch_bounds__(kScanThreads, 1)
    permute_scan_kernel(int32_t* __restrict__ counts, int C, int E, int32_t* __restrict__ offsets_out) {
    pdl_begin();
    extern __shared__ int s[];
    int* tot = s;                   // [E+1]
    int* part = tot + E + 1;        // [kScanThreads+1]
    for (int e = threadIdx.x; e < E; e += kScanThreads) {
        int t = 0;
        for (int c = 0; c < C; ++c) t += counts[(size_t)c * E + e];
        tot[e] = t;
    }
    __syncthreads();
    block_exclusive_scan(tot, E, part);
    for (int e = threadIdx.x; e < E; e += kScanThreads) {
        int run = tot[e];
        for (int c = 0; c < C; ++c) {
            const int v = counts[(size_t)c * E + e];
            counts[(size_t)c * E + e] = run;
            run += v;
        }
    }
    for (int e = threadIdx.x; e <= E; e += kScanThreads) offsets_out[e] = tot[e];
}

// Kernel 3: the stable scatter of each chunk from its bases.
__global__ void __launch_bounds__(kPermThreads, 1)
    permute_scatter_kernel(const int32_t* __restrict__ ids, int R, int E, int chunk,
                           const int32_t* __restrict__ bases, const int32_t* __restrict__ offsets,
                           int32_t* __restrict__ sorted_rows, int32_t* __restrict__ m_indices) {
    pdl_begin();
    extern __shared__ int hist[];                       // [kPermWarps][E]
    const int c0 = blockIdx.x * chunk, c1 = min(R, c0 + chunk);
    int lo, hi;
    chunk_histograms(ids, c0, c1, E, hist, lo, hi);
    for (int e = threadIdx.x; e < E; e += kPermThreads) {
        int run = bases[(size_t)blockIdx.x * E + e];
        for (int w = 0; w < kPermWarps; ++w) {
            const int c = hist[w * E + e];
            hist[w * E + e] = run;
            run += c;
        }
    }
    __syncthreads();
    chunk_scatter(ids, lo, hi, E, hist, sorted_rows, m_indices);
    fill_tail(R, offsets[E], sorted_rows, m_indices);
}

int permute_chunks(long long R) {
    long long c = (R + kChunkMin - 1) / kChunkMin;
    return (int)(c < 1 ? 1 : c > kMaxChunks ? kMaxChunks : c);
}

}  // namespace
}  // namespace ferret

using namespace ferret;

extern "C" size_t ferret_moe_permute_workspace_size(int T, int topk, int E) {
    if (T < 0 || topk <= 0 || E <= 0) return 0;
    const int C = permute_chunks((long long)T * topk);
    return C > 1 ? (size_t)C * E * sizeof(int32_t) : 0;
}

extern "C" int ferret_moe_permute(const int32_t* topk_ids, int T, int topk, int E,
                                  int32_t* sorted_rows, int32_t* expert_offsets,
                                  int32_t* m_indices, void* workspace, size_t ws_bytes,
                                  void* stream) {
    if (T < 0 || topk <= 0 || E <= 0 || E > 1024) return FERRET_ERR_SHAPE;
    if (!expert_offsets) return FERRET_ERR_NULL;
    const long long R = (long long)T * topk;
    if (R > (1ll << 30)) return FERRET_ERR_SHAPE;
    if (R > 0 && (!topk_ids || !sorted_rows || !m_indices)) return FERRET_ERR_NULL;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    cudaStream_t s = as_stream(stream);
    const int C = permute_chunks(R);
    const size_t need = (size_t)C * E * sizeof(int32_t);
    if (C > 1 && workspace && ws_bytes >= need && !(reinterpret_cast<uintptr_t>(workspace) & 3u)) {
        // chunked: count, scan, scatter
        const int chunk = (int)((R + C - 1) / C);
        int32_t* counts = static_cast<int32_t*>(workspace);
        const size_t hsm = sizeof(int) * (size_t)kPermWarps * E;
        const size_t ssm = sizeof(int) * ((size_t)E + 1 + kScanThreads + 1);
        if (hsm > (size_t)info->max_smem_optin) return FERRET_ERR_SHAPE;
        if (cudaFuncSetAttribute(permute_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)hsm) != cudaSuccess ||
            cudaFuncSetAttribute(permute_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)hsm) != cudaSuccess) {
            cudaGetLastError();
            return FERRET_ERR_CUDA;
        }
        if ((rc = launch_kernel(permute_count_kernel, dim3(C), dim3(kPermThreads), hsm, s,
                                topk_ids, (int)R, E, chunk, counts)) != FERRET_OK) return rc;
        if ((rc = launch_kernel(permute_scan_kernel, dim3(1), dim3(kScanThreads), ssm, s, counts,
                                C, E, expert_offsets)) != FERRET_OK) return rc;
        return launch_kernel(permute_scatter_kernel, dim3(C), dim3(kPermThreads), hsm, s, topk_ids,
                             (int)R, E, chunk, counts, expert_offsets, sorted_rows, m_indices);
    }
    // one CTA over all ids (decode sizes, or no workspace given)
    const size_t smem = sizeof(int) * ((size_t)kPermWarps * E + E + 1 + kPermThreads + 1);
    if (smem > (size_t)info->max_smem_optin) return FERRET_ERR_SHAPE;
    if (cudaFuncSetAttribute(moe_permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    return launch_kernel(moe_permute_kernel, dim3(1), dim3(kPermThreads), smem, s, topk_ids,
                         (int)R, E, sorted_rows, expert_offsets, m_indices);
}

// ---------------------------------------------------------------------------
// Block-padded layout of vLLM's moe_align_block_size(topk_ids, block_size, E,
// ignore_invalid_experts=True) (baselines/kimi-moe-w13-int4/baseline_marlin.py:123-126):
// every expert's rows padded to a multiple of block_size, padding entries =
// T*topk, expert_ids per block (-1 past the used blocks), and the padded total.
// Built from the stable permutation above: one CTA turns the expert offsets
// into padded offsets and block experts, then a grid fills the padded rows.
// ---------------------------------------------------------------------------
namespace ferret {
namespace {

constexpr int kPadThreads = 1024;

__global__ void __launch_bounds__(kPadThreads, 1)
    align_blocks_kernel(const int32_t* __restrict__ offs, int E, int bs, int max_blocks,
                        int32_t* __restrict__ pad_offs, int32_t* __restrict__ expert_ids,
                        int32_t* __restrict__ num_post_pad) {
    pdl_begin();
    extern __shared__ int sm[];
    int* po = sm;                    // [E+1]
    int* part = sm + E + 1;          // [kPadThreads+1]
    for (int e = threadIdx.x; e < E; e += kPadThreads) {
        const int c = offs[e + 1] - offs[e];
        po[e] = (c + bs - 1) / bs * bs;
    }
    __syncthreads();
    block_exclusive_scan(po, E, part);
    for (int e = threadIdx.x; e <= E; e += kPadThreads) pad_offs[e] = po[e];
    if (threadIdx.x == 0) *num_post_pad = po[E];
    for (int b = threadIdx.x; b < max_blocks; b += kPadThreads) {
        const int p = b * bs;
        int v = -1;
        if (p < po[E]) {
            int lo = 0, hi = E - 1;          // last expert whose padded range starts at or before p
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (po[mid] <= p) lo = mid;
                else hi = mid - 1;
            }
            v = lo;
        }
        expert_ids[b] = v;
    }
}

__global__ void __launch_bounds__(256)
    align_fill_kernel(const int32_t* __restrict__ sorted_rows, const int32_t* __restrict__ offs,
                      const int32_t* __restrict__ pad_offs, int E, int max_padded, int sentinel,
                      int32_t* __restrict__ sorted_ids) {
    pdl_begin();
    const int total = pad_offs[E];
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < max_padded; p += gridDim.x * blockDim.x) {
        int v = sentinel;
        if (p < total) {
            int lo = 0, hi = E - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (pad_offs[mid] <= p) lo = mid;
                else hi = mid - 1;
            }
            const int i = p - pad_offs[lo];
            if (i < offs[lo + 1] - offs[lo]) v = sorted_rows[offs[lo] + i];
        }
        sorted_ids[p] = v;
    }
}

}  // namespace
}  // namespace ferret

extern "C" int ferret_moe_align_block_size_sizes(int T, int topk, int E, int block_size,
                                                  int* max_padded, int* max_blocks) {
    if (T < 0 || topk <= 0 || E <= 0 || block_size <= 0 || !max_padded || !max_blocks)
        return FERRET_ERR_SHAPE;
    const long long numel = (long long)T * topk;
    long long m = numel + (long long)E * (block_size - 1);
    if (numel < E) m = std::min(m, numel * block_size);
    if (m >= (1ll << 31)) return FERRET_ERR_SHAPE;
    *max_padded = (int)m;
    *max_blocks = (int)((m + block_size - 1) / block_size);
    return FERRET_OK;
}

extern "C" size_t ferret_moe_align_block_size_workspace_size(int T, int topk, int E) {
    if (T < 0 || topk <= 0 || E <= 0) return 0;
    const size_t R = (size_t)T * topk;
    const size_t perm = ferret_moe_permute_workspace_size(T, topk, E);
    return (2 * R + 2 * ((size_t)E + 1)) * sizeof(int32_t) + 256 + perm;
}

extern "C" int ferret_moe_align_block_size(const int32_t* topk_ids, int T, int topk, int E,
                                           int block_size, int32_t* sorted_ids,
                                           int32_t* expert_ids, int32_t* num_tokens_post_pad,
                                           void* workspace, size_t ws_bytes, void* stream) {
    int max_padded = 0, max_blocks = 0;
    int rc = ferret_moe_align_block_size_sizes(T, topk, E, block_size, &max_padded, &max_blocks);
    if (rc != FERRET_OK) return rc;
    if (E > 1024) return FERRET_ERR_SHAPE;
    if (!sorted_ids || !expert_ids || !num_tokens_post_pad) return FERRET_ERR_NULL;
    if (T > 0 && !topk_ids) return FERRET_ERR_NULL;
    if (!workspace || ws_bytes < ferret_moe_align_block_size_workspace_size(T, topk, E))
        return FERRET_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 3u) return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    if ((rc = current_device(&info)) != FERRET_OK) return rc;
    cudaStream_t s = as_stream(stream);
    const size_t R = (size_t)T * topk;
    int32_t* w = static_cast<int32_t*>(workspace);
    int32_t* rows = w;
    int32_t* midx = rows + R;
    int32_t* offs = midx + R;
    int32_t* pad_offs = offs + E + 1;
    uint8_t* pws = reinterpret_cast<uint8_t*>(pad_offs + E + 1);
    pws += (256 - (reinterpret_cast<uintptr_t>(pws) & 255)) & 255;
    const size_t pws_bytes = ferret_moe_permute_workspace_size(T, topk, E);
    rc = ferret_moe_permute(topk_ids, T, topk, E, rows, offs, midx, pws_bytes ? pws : nullptr,
                            pws_bytes, stream);
    if (rc != FERRET_OK) return rc;
    const size_t smem = sizeof(int) * ((size_t)E + 1 + kPadThreads + 1);
    if ((rc = launch_kernel(align_blocks_kernel, dim3(1), dim3(kPadThreads), smem, s, offs, E,
                            block_size, max_blocks, pad_offs, expert_ids, num_tokens_post_pad)) !=
        FERRET_OK)
        return rc;
    const int grid = std::max(1, std::min((max_padded + 255) / 256, info->num_sms * 8));
    return launch_kernel(align_fill_kernel, dim3(grid), dim3(256), 0, s, rows, offs, pad_offs, E,
                         max_padded, (int)R, sorted_ids);
}
