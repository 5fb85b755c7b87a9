// fp8_gemm_common.cuh -- definitions shared by the FP8 grouped GEMM kernel
// families (swap-AB decode, prefill, block-scaled prefill) and their entry
// points: kernel arguments, tile decoding, shared-memory layouts, and the
// launchers each family exports to the entry points.
#pragma once

#include <algorithm>

#include "capi_internal.h"

namespace ferret {
namespace {


constexpr int kThreads = 192;     // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kEpiThreads = 128;
constexpr int kMaxE = 1024;
constexpr int kMaxNK = 128;       // K <= 16384
constexpr int kMaxStages = 16;
constexpr int kMaxAcc = 8;
constexpr int kWTile = 128 * 128; // one 128x128 e4m3 weight box

// wait sites recorded in the status word
enum : int {
    SITE_EMPTY = 1, SITE_FULL = 2, SITE_TEMPTY = 3, SITE_TFULL = 4, SITE_DRAIN = 5, SITE_EPI = 6
};

constexpr int kABox = 16;         // token rows per activation TMA box (the MMA N granule)

struct GemmArgs {
    const float* a_scale;
    const float* w_scale;
    const int32_t* seg;    // offsets[E+1] (seg_pairs == 0) or [E][2] (start, count)
    int seg_pairs;
    __nv_bfloat16* out;
    const int32_t* out_rows;   // nullable: output row of expert-sorted row i is out_rows[i]
    int out_total;             // rows of `out` when out_rows is set (others are skipped)
    __nv_bfloat16* const* out_peers;   // nullable: row o lives on buffer o / peer_rows
    int peer_rows;
    int M, N, K, E;
    int stages;
    DevCtl ctl;
};

// Split-K for launches with fewer tiles than SMs (swap-AB kernel): the kernel
// picks S <= splits_max from the actual tile count so that the fp32 partials
// part[unit][col][128] fit part_bytes; cnt[tile] (zeroed before the launch)
// finds the last unit of a tile, which reduces in split order.  splits_max <= 1
// disables it.  (A separate kernel argument: the prefill kernel's code
// generation measured sensitive to the size of its argument struct.)
struct SplitArgs {
    int splits_max;
    float* part;
    int* cnt;
    size_t part_bytes;
};

// Address of output row `orow` (row stride ldo): the local matrix, or, with a
// peer table, row orow % peer_rows of buffer orow / peer_rows (another GPU's
// memory over NVLink when the table holds peer pointers).
__device__ __forceinline__ __nv_bfloat16* out_row_ptr(const GemmArgs& a, int orow, int ldo) {
    if (a.out_peers) {
        const int g = orow / a.peer_rows;
        return a.out_peers[g] + (size_t)(orow - g * a.peer_rows) * ldo;
    }
    return a.out + (size_t)orow * ldo;
}

// Tile t -> (expert, first row, rows, n-block).  Tiles are ordered token-tile
// major so the CTAs of one wave share an expert's token rows through L2 while
// each streams distinct weight blocks.
template <int NT>
__device__ __forceinline__ void decode_tile(int t, int nbc, int E, const int* mt_start,
                                            const int* seg_s, const int* seg_c, int& e, int& row0,
                                            int& rows, int& nb) {
    const int mt = t / nbc;
    nb = t - mt * nbc;
    int lo = 0, hi = E - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (mt_start[mid] <= mt) lo = mid;
        else hi = mid - 1;
    }
    e = lo;
    const int local = (mt - mt_start[e]) * NT;
    row0 = seg_s[e] + local;
    rows = min(NT, seg_c[e] - local);
}

// ---------------------------------------------------------------------------
// Prefill-shaped kernel: tokens on the MMA M axis.
//
// When experts carry many tokens the swap-AB orientation wastes issue slots:
// its per-column (per-token) scales cost a multiply per accumulator element.
// Here a CTA tile is 128 token rows (MMA M) x 256 weight rows (MMA N: two
// 128-row weight blocks -- consecutive ones, or gate block j and up block
// N/256 + j with SiLU), 128-wide K blocks (48 KB stages, TMA, 128-byte
// swizzle).  tcgen05.mma kind::f8f6f4 M=128 N=256 K=32 writes each K block's
// partial into one of two 256-column TMEM buffers; 8 epilogue warps promote
// it: thread (row r, column half h) owns 64 columns of each weight block and
// needs just two scale products per K block (a_scale[r] * w_scale[block]),
// then 128 FMAs.  SiLU pairs land in the same thread (gate column c and up
// column 128 + c), so the fused epilogue needs no exchange.
// ---------------------------------------------------------------------------
constexpr int kPfThreads = 320;          // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kPfEpi = 256;
constexpr int kPfStage = 128 * 128 + 256 * 128;   // A 16 KB + B 32 KB
constexpr int kPfMaxStages = 6;

// The expert-parallel form adds six warps (warps 2-3 and a fourth warpgroup,
// warps 12-15; the epilogue moves to warps 4-11): four pull the tile rows
// from the peers and two push finished rows to them while the tile pipeline
// runs.
constexpr int kPfPullWarps = 4, kPfPushWarps = 2;
constexpr int kPfPeerThreads = 16 * 32;

// waits for pulled rows to land / for a tile's rows to be stored before the push
enum : int { SITE_ROWS = 11, SITE_PUSH = 12 };

struct PfLayout {
    int stages_off, segs_off, segc_off, mts_off, part_off, bar_off, misc_off, total;
};

// ep: the expert-parallel form (more threads for the block scan's scratch)
__host__ __device__ inline PfLayout pf_layout(int stages, int E, bool ep) {
    PfLayout L;
    int o = 0;
    L.stages_off = o;
    o += kPfStage * stages;
    L.segs_off = o;
    o += 4 * E;
    L.segc_off = o;
    o += 4 * E;
    L.mts_off = o;
    o += 4 * (E + 1);
    L.part_off = o;
    o += 4 * ((ep ? kPfPeerThreads : kPfThreads) + 1);
    o = (o + 7) & ~7;
    L.bar_off = o;
    o += 8 * (2 * kPfMaxStages + 2 * 2 + 2);
    L.misc_off = o;
    o += 16;
    L.total = o;
    return L;
}

constexpr int kMxThreads = 448;
constexpr int kMxEpi = 256;
constexpr int kMxSfSlots = 8;
constexpr int kMxSfCol0 = 256;      // accumulator: columns 0-255
constexpr int kMxSfCols = 16;       // per slot: A scales cols 0-3, B scales cols 8-15

enum : int { SITE_SFULL = 7, SITE_SEMPTY = 8 };

struct MxLayout {
    int stages_off, segs_off, segc_off, mts_off, part_off, bar_off, misc_off, total;
};

__host__ __device__ inline MxLayout mx_layout(int stages, int E) {
    MxLayout L;
    int o = 0;
    L.stages_off = o;
    o += kPfStage * stages;
    L.segs_off = o;
    o += 4 * E;
    L.segc_off = o;
    o += 4 * E;
    L.mts_off = o;
    o += 4 * (E + 1);
    L.part_off = o;
    o += 4 * (kMxThreads + 1);
    o = (o + 7) & ~7;
    L.bar_off = o;
    o += 8 * (2 * kPfMaxStages + 2 + 2 * kMxSfSlots + 1);
    L.misc_off = o;
    o += 16;
    L.total = o;
    return L;
}

// UE8M0 byte of a power-of-two scale (its fp32 exponent field), in all 4 bytes.
__device__ __forceinline__ uint32_t ue8m0_word(float s) {
    return ((__float_as_uint(s) >> 23) & 0xFFu) * 0x01010101u;
}

constexpr int kPpStage = 128 * 128 + 128 * 128;    // A half 16 KB + B half 16 KB
constexpr int kPpMaxStages = 6;

enum : int { SITE_PEER_EMPTY = 9, SITE_PEER_TAIL = 10 };

struct PpLayout {
    int stages_off, segs_off, segc_off, mts_off, part_off, bar_off, misc_off, total;
};

__host__ __device__ inline PpLayout pp_layout(int stages, int E) {
    PpLayout L;
    int o = 0;
    L.stages_off = o;
    o += kPpStage * stages;
    L.segs_off = o;
    o += 4 * E;
    L.segc_off = o;
    o += 4 * E;
    L.mts_off = o;
    o += 4 * (E + 1);
    L.part_off = o;
    o += 4 * (kPfThreads + 1);
    o = (o + 7) & ~7;
    L.bar_off = o;
    o += 8 * (2 * kPpMaxStages + 2 * 2 + 1);
    L.misc_off = o;
    o += 16;
    L.total = o;
    return L;
}

struct MxpLayout {
    int stages_off, segs_off, segc_off, mts_off, part_off, bar_off, misc_off, total;
};

__host__ __device__ inline MxpLayout mxp_layout(int stages, int E) {
    MxpLayout L;
    int o = 0;
    L.stages_off = o;
    o += kPpStage * stages;
    L.segs_off = o;
    o += 4 * E;
    L.segc_off = o;
    o += 4 * E;
    L.mts_off = o;
    o += 4 * (E + 1);
    L.part_off = o;
    o += 4 * (kMxThreads + 1);
    o = (o + 7) & ~7;
    L.bar_off = o;
    o += 8 * (2 * kPpMaxStages + 2 + 2 * kMxSfSlots + 1);
    L.misc_off = o;
    o += 16;
    L.total = o;
    return L;
}

}  // namespace

// Launchers exported by the kernel-family files to the entry points.

// Swap-AB kernel with an NT-row token tile (16, 32, 64 or 128; 128 without SiLU only).
int launch_fp8_decode(int nt, bool pair, const DeviceInfo* info, const void* a, const float* a_scale,
                      const void* w, const float* w_scale, void* out, const int32_t* seg,
                      int seg_pairs, int M, int N, int K, int E, cudaStream_t stream,
                      const OutMap& om, const SplitWs& sw);

// m_indices -> per-expert (start, count) pairs in seg[2E]; zeroes cnt[0, ncnt).
int launch_derive_segments(const DeviceInfo* info, const int32_t* m_indices, int M, int E,
                           int32_t* seg, int* cnt, int ncnt, cudaStream_t stream);

// Prefill kernel (128 token rows x 256 weight rows per tile); om.gather selects
// its expert-parallel form, which pulls its A rows from and pushes its output
// rows to the peers itself.
int launch_fp8_prefill(bool pair, const DeviceInfo* info, const void* a, const float* a_scale,
                       const void* w, const float* w_scale, void* out, const int32_t* seg,
                       int seg_pairs, int M, int N, int K, int E, cudaStream_t stream,
                       const OutMap& om);

// CTA-pair prefill kernel for whole 256-row chunks + the single-CTA remainder.
int launch_fp8_prefill_pairs(bool pair, const DeviceInfo* info, const void* a,
                             const float* a_scale, const void* w, const float* w_scale, void* out,
                             const int32_t* seg, int seg_pairs, int M, int N, int K, int E,
                             cudaStream_t stream, const OutMap& om);

// Block-scaled (UE8M0) prefill kernel, single CTAs or CTA pairs + remainder.
int launch_fp8_prefill_mx(const DeviceInfo* info, const void* a, const float* a_scale,
                          const void* w, const float* w_scale, void* out, const int32_t* seg,
                          int seg_pairs, int M, int N, int K, int E, cudaStream_t stream,
                          const OutMap& om);
int launch_fp8_prefill_mx_pairs(const DeviceInfo* info, const void* a, const float* a_scale,
                                const void* w, const float* w_scale, void* out, const int32_t* seg,
                                int seg_pairs, int M, int N, int K, int E, cudaStream_t stream,
                                const OutMap& om);

}  // namespace ferret
