// fp8_grouped_gemm.cu -- entry points of the FP8 block-scaled grouped GEMM
// (include/ferret_moe.h): argument checks, segment derivation from
// m_indices, split-K workspace, and the choice between the kernel families
// (fp8_decode.cu: swap-AB token tiles; fp8_prefill.cu: 128 x 256 tiles;
// fp8_prefill_mx.cu: block-scaled UE8M0 tiles).
#include "fp8_gemm_common.cuh"

namespace ferret {
namespace {

int pick_tile(int M, int E, int K, int flags, bool pair) {
    int nt = (flags >> FERRET_TILE_SHIFT) & 0xFF;
    if (nt == 0) {
        // measured on B200 (graph-timed): at K = 7168 the 32-row tile streams
        // the decode weights 4 % faster than the 16-row one (same tiles, one
        // stage fewer); at K = 2048 the 16-row tile is faster
        const int avg = (M + E - 1) / std::max(E, 1);
        nt = (avg <= 12 && K < 4096) ? 16 : avg <= 24 ? 32 : avg <= 48 ? 64 : 128;
    }
    if (pair && nt > 64) nt = 64;
    return nt;
}

}  // namespace

// 128-token tiles (requested, or experts averaging more than 48 rows) run on
// the prefill kernel when the weight tiles (256 rows) divide N.
bool fp8_gemm_uses_prefill(int rows_hint, int E, int flags, int N) {
    int nt = (flags >> FERRET_TILE_SHIFT) & 0xFF;
    if (nt == 0) nt = ((rows_hint + E - 1) / std::max(E, 1)) > 48 ? 128 : 0;
    return nt == 128 && N % 256 == 0;
}

int run_fp8_gemm(const DeviceInfo* info, const void* a, const float* a_scale, const void* w,
                 const float* w_scale, void* out, const int32_t* seg, int seg_pairs, int M, int N,
                 int K, int E, int flags, int rows_hint, cudaStream_t s, const OutMap& om,
                 const SplitWs& sw) {
    const bool pair = (flags & FERRET_SILU_MUL) != 0;
    const bool prefill = fp8_gemm_uses_prefill(rows_hint, E, flags, N);
    // rows pulled from the peers inside the GEMM: only the prefill kernel's
    // staged-store form does that
    if (om.gather && (!prefill || !om.peers)) return FERRET_ERR_SHAPE;
    // power-of-two scales: the block-scaled kernel for plain 128-token tiles
    // (with SiLU the exact-scale kernel is faster and exact for such scales)
    if (prefill && (flags & FERRET_UE8M0_SCALES) && !pair && !om.peers)
        return (flags & FERRET_PREFILL_PAIRS)
                   ? launch_fp8_prefill_mx_pairs(info, a, a_scale, w, w_scale, out, seg, seg_pairs,
                                                 M, N, K, E, s, om)
                   : launch_fp8_prefill_mx(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M, N,
                                           K, E, s, om);
    // CTA pairs for whole 256-row expert chunks, single CTAs for the rest
    if (prefill && (flags & FERRET_PREFILL_PAIRS) && !om.peers)
        return launch_fp8_prefill_pairs(pair, info, a, a_scale, w, w_scale, out, seg, seg_pairs, M,
                                        N, K, E, s, om);
    if (prefill)
        return launch_fp8_prefill(pair, info, a, a_scale, w, w_scale, out, seg, seg_pairs, M, N, K,
                                  E, s, om);
    return launch_fp8_decode(pick_tile(rows_hint, E, K, flags, pair), pair, info, a, a_scale, w,
                             w_scale, out, seg, seg_pairs, M, N, K, E, s, om, sw);
}

}  // namespace ferret

using namespace ferret;

// Batches up to kSplitMaxRows rows also get room for split-K partials (a
// launch with fewer tiles than SMs splits K across them).
constexpr int kSplitMaxRows = 4096;
constexpr size_t kSplitBytes = (size_t)16 << 20;

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

extern "C" size_t ferret_fp8_grouped_gemm_workspace_size(int M, int E) {
    if (E <= 0) return 0;
    const size_t seg = align256((size_t)E * 2 * sizeof(int32_t));
    return M >= 0 && M <= kSplitMaxRows ? seg + kSplitBytes : seg;
}

extern "C" int ferret_fp8_grouped_gemm_nt_contiguous(
    const void* a_fp8, const float* a_scale, const void* w_fp8, const float* w_scale,
    void* out_bf16, const int32_t* m_indices, const int32_t* expert_offsets, int M, int N, int K,
    int E, int flags, void* workspace, size_t ws_bytes, void* stream) {
    const bool pair = (flags & FERRET_SILU_MUL) != 0;
    if (M < 0 || N <= 0 || K <= 0 || E <= 0 || E > kMaxE) return FERRET_ERR_SHAPE;
    if (K % 128 || N % 128 || (pair && N % 256) || K / 128 > kMaxNK) return FERRET_ERR_SHAPE;
    if ((long long)E * N >= (1ll << 31) || (long long)M * K >= (1ll << 40)) return FERRET_ERR_SHAPE;
    if (M == 0) return FERRET_OK;
    if (!a_fp8 || !a_scale || !w_fp8 || !w_scale || !out_bf16) return FERRET_ERR_NULL;
    if (!expert_offsets && !m_indices) return FERRET_ERR_NULL;
    if (!aligned16(a_fp8) || !aligned16(w_fp8) || !aligned16(out_bf16) ||
        (reinterpret_cast<uintptr_t>(a_scale) & 3u) || (reinterpret_cast<uintptr_t>(w_scale) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    cudaStream_t s = as_stream(stream);

    const int32_t* seg = expert_offsets;
    int seg_pairs = 0;
    const size_t seg_bytes = expert_offsets ? 0 : align256((size_t)E * 2 * sizeof(int32_t));
    if (!expert_offsets && (!workspace || ws_bytes < seg_bytes)) return FERRET_ERR_WORKSPACE;
    if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 3u)) return FERRET_ERR_ALIGN;
    // split-K room past the segments: tile counters (bounded by the tiles any
    // token tile of >= 16 rows can give), then fp32 partials
    SplitWs sw;
    int ncnt = 0;
    if (workspace && M <= kSplitMaxRows && ws_bytes > seg_bytes) {
        const long long tiles_up = ((long long)std::min(M, E) + M / 16) * (N / 128);
        const size_t cnt_bytes = align256((size_t)tiles_up * sizeof(int));
        if (ws_bytes > seg_bytes + cnt_bytes + 4096) {
            uint8_t* base = static_cast<uint8_t*>(workspace) + seg_bytes;
            sw.cnt = reinterpret_cast<int*>(base);
            sw.part = reinterpret_cast<float*>(base + cnt_bytes);
            sw.bytes = ws_bytes - seg_bytes - cnt_bytes;
            sw.smax = K / 128;
            ncnt = (int)tiles_up;
        }
    }
    if (!expert_offsets) {
        if ((rc = launch_derive_segments(info, m_indices, M, E, static_cast<int32_t*>(workspace),
                                         sw.cnt, ncnt, s)) != FERRET_OK) return rc;
        seg = static_cast<const int32_t*>(workspace);
        seg_pairs = 1;
    } else if (sw.cnt) {
        if (cudaMemsetAsync(sw.cnt, 0, (size_t)ncnt * sizeof(int), s) != cudaSuccess) {
            cudaGetLastError();
            return FERRET_ERR_CUDA;
        }
    }

    // many tokens per expert: the prefill kernel (tokens on MMA M, 256 weight rows on N);
    // otherwise the swap-AB kernel with a token tile sized to the rows per expert
    return run_fp8_gemm(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, seg, seg_pairs, M, N, K, E,
                        flags, M, s, OutMap{}, sw);
}

#include <mutex>

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Callers such as a serving process that hands nearly all HBM to weights and
// the KV cache up front, or a plugin host that binds this library through an
// FFI and has no handle on the framework's allocator, cannot obtain a
// workspace at call time.  This entry point keeps the derived expert segments
// in a fixed device array instead, so it needs no workspace and calls no
// allocator.  The array lives in this library's module on every GPU that
// loads the library, until the process exits.
// ---------------------------------------------------------------------------
namespace ferret {
namespace {

constexpr int kNoAllocMaxExperts = kMaxE;                       // 1024 experts
static __device__ __align__(256) int32_t g_noalloc_segments[2 * kNoAllocMaxExperts];  // 8 KB

constexpr int kNoAllocMaxDevices = 64;
int32_t* g_noalloc_ptr[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Device address of the array on device `dev` (which must be current): host
// code only ever sees a host-side stand-in for the array, so the address is
// queried, once per device.  A failed query is not remembered: the next call
// tries again (for instance after a first call made, against the advice in
// the header, inside a stream capture that refused it).
int noalloc_scratch(int dev, int32_t** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_segments) != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return FERRET_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = static_cast<int32_t*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return FERRET_OK;
}

}  // namespace
}  // namespace ferret

extern "C" int ferret_fp8_grouped_gemm_nt_contiguous_noalloc(
    const void* a_fp8, const float* a_scale, const void* w_fp8, const float* w_scale,
    void* out_bf16, const int32_t* m_indices, int M, int N, int K, int E, int flags,
    void* stream) {
    const bool pair = (flags & FERRET_SILU_MUL) != 0;
    if (M < 0 || N <= 0 || K <= 0 || E <= 0) return FERRET_ERR_SHAPE;
    if (E > kNoAllocMaxExperts) return FERRET_ERR_SHAPE;   // beyond the fixed scratch
    if (K % 128 || N % 128 || (pair && N % 256) || K / 128 > kMaxNK) return FERRET_ERR_SHAPE;
    if ((long long)E * N >= (1ll << 31) || (long long)M * K >= (1ll << 40)) return FERRET_ERR_SHAPE;
    if (M == 0) return FERRET_OK;
    if (!a_fp8 || !a_scale || !w_fp8 || !w_scale || !out_bf16 || !m_indices) return FERRET_ERR_NULL;
    if (!aligned16(a_fp8) || !aligned16(w_fp8) || !aligned16(out_bf16) ||
        (reinterpret_cast<uintptr_t>(a_scale) & 3u) || (reinterpret_cast<uintptr_t>(w_scale) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    if (info->device < 0 || info->device >= kNoAllocMaxDevices) return FERRET_ERR_UNSUPPORTED;
    int32_t* seg = nullptr;
    if ((rc = noalloc_scratch(info->device, &seg)) != FERRET_OK) return rc;
    cudaStream_t s = as_stream(stream);
    // every call rewrites all 2E (start, count) entries before the GEMM reads them
    if ((rc = launch_derive_segments(info, m_indices, M, E, seg, nullptr, 0, s)) != FERRET_OK)
        return rc;
    // the same kernel choice as the workspace entry point; without a workspace
    // there is no split-K, so small launches may sum K in another order
    return run_fp8_gemm(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, seg, 1, M, N, K, E, flags,
                        M, s, OutMap{}, SplitWs{});
}


// Scatter-output form: rows of expert segment e are [off[e], off[e+1]) of A as
// usual, but expert-sorted row i is written to output row out_rows[i] (rows
// outside [0, out_total) are skipped).  With out_rows = the permutation's
// sorted_rows this writes the W13 result straight into (token, slot) order.
extern "C" int ferret_fp8_grouped_gemm_scatter(const void* a_fp8, const float* a_scale,
                                               const void* w_fp8, const float* w_scale,
                                               void* out_bf16, const int32_t* expert_offsets,
                                               const int32_t* out_rows, int M, int out_total, int N,
                                               int K, int E, int flags, void* stream) {
    const bool pair = (flags & FERRET_SILU_MUL) != 0;
    if (M < 0 || out_total < 0 || N <= 0 || K <= 0 || E <= 0 || E > kMaxE) return FERRET_ERR_SHAPE;
    if (K % 128 || N % 128 || (pair && N % 256) || K / 128 > kMaxNK) return FERRET_ERR_SHAPE;
    if ((long long)E * N >= (1ll << 31) || (long long)M * K >= (1ll << 40)) return FERRET_ERR_SHAPE;
    if (M == 0 || out_total == 0) return FERRET_OK;
    if (!a_fp8 || !a_scale || !w_fp8 || !w_scale || !out_bf16 || !expert_offsets || !out_rows)
        return FERRET_ERR_NULL;
    if (!aligned16(a_fp8) || !aligned16(w_fp8) || !aligned16(out_bf16) ||
        (reinterpret_cast<uintptr_t>(a_scale) & 3u) || (reinterpret_cast<uintptr_t>(w_scale) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    cudaStream_t s = as_stream(stream);
    OutMap om;
    om.rows = out_rows;
    om.total = out_total;
    return run_fp8_gemm(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, expert_offsets, 0, M, N, K,
                        E, flags, M, s, om);
}
