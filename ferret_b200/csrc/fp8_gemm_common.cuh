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

// One K block of the prefill epilogue: this thread's row of the 2*HALF-column
// TMEM partial at `tb` (CPH columns of each half, the thread's column group)
// scaled into its accumulators, acc0 for the first half's weight rows
// (s0 = a_scale * w_scale[their block]) and acc1 for the second's (s1).
// The caller waits for the partial (tfull) before and releases the buffer after.
// PACKED: one fma.rn.f32x2 per two columns, else one fmaf per column (the same
// roundings; which is faster depends on the kernel around it).
template <int CPH, int LD, int HALF = 128, bool PACKED = true>
__device__ __forceinline__ void promote_kblock(uint32_t tb, float (&acc0)[CPH], float (&acc1)[CPH],
                                               float s0, float s1) {
#pragma unroll
    for (int c = 0; c < CPH; c += LD) {
        float v[LD], u[LD];
        tmem_ld_cols<LD>(tb + c, v);
        tmem_ld_cols<LD>(tb + HALF + c, u);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < LD; j += 2) {
            if constexpr (PACKED) {
                ffma2(acc0[c + j], acc0[c + j + 1], v[j], v[j + 1], s0);
                ffma2(acc1[c + j], acc1[c + j + 1], u[j], u[j + 1], s1);
            } else {
                acc0[c + j] = fmaf(v[j], s0, acc0[c + j]);
                acc0[c + j + 1] = fmaf(v[j + 1], s0, acc0[c + j + 1]);
                acc1[c + j] = fmaf(u[j], s1, acc1[c + j]);
                acc1[c + j + 1] = fmaf(u[j + 1], s1, acc1[c + j + 1]);
            }
        }
    }
}

// Stores one row of a finished prefill tile (2*HALF weight rows) as bf16
// (16-byte stores) at output row `o`, output tile nb, column group h: the
// thread's CPH columns of each half.  PAIR (SiLU): silu(gate) * up of the two
// halves into HALF output columns per tile; otherwise both halves side by side.
template <bool PAIR, int CPH, int HALF = 128>
__device__ __forceinline__ void store_tile_row(__nv_bfloat16* o, int nb, int h,
                                               const float (&acc0)[CPH], const float (&acc1)[CPH]) {
    if (PAIR) {
        uint4* dst = reinterpret_cast<uint4*>(o + nb * HALF + h * CPH);
#pragma unroll
        for (int c = 0; c < CPH; c += 8) {
            uint4 pk;
            uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const __nv_bfloat162 b = __floats2bfloat162_rn(
                    silu_mul(acc0[c + 2 * j], acc1[c + 2 * j]),
                    silu_mul(acc0[c + 2 * j + 1], acc1[c + 2 * j + 1]));
                pw[j] = *reinterpret_cast<const uint32_t*>(&b);
            }
            dst[c >> 3] = pk;
        }
    } else {
        uint4* d0 = reinterpret_cast<uint4*>(o + nb * 2 * HALF + h * CPH);
        uint4* d1 = reinterpret_cast<uint4*>(o + nb * 2 * HALF + HALF + h * CPH);
#pragma unroll
        for (int c = 0; c < CPH; c += 8) {
            uint4 p0, p1;
            uint32_t* w0 = reinterpret_cast<uint32_t*>(&p0);
            uint32_t* w1 = reinterpret_cast<uint32_t*>(&p1);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const __nv_bfloat162 b0 = __floats2bfloat162_rn(acc0[c + 2 * j], acc0[c + 2 * j + 1]);
                const __nv_bfloat162 b1 = __floats2bfloat162_rn(acc1[c + 2 * j], acc1[c + 2 * j + 1]);
                w0[j] = *reinterpret_cast<const uint32_t*>(&b0);
                w1[j] = *reinterpret_cast<const uint32_t*>(&b1);
            }
            d0[c >> 3] = p0;
            d1[c >> 3] = p1;
        }
    }
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
// partial into one of two 256-column TMEM buffers; the epilogue warps promote
// it: thread (row r, column group h) owns 512 / (epilogue warps) columns of
// each weight block and needs just two scale products per K block
// (a_scale[r] * w_scale[block]), then one packed FMA per two columns.  SiLU
// pairs land in the same thread (gate column c and up column 128 + c), so the
// fused epilogue needs no exchange.
// ---------------------------------------------------------------------------
constexpr int kPfEpiWarps = 8;           // single-GPU form: epilogue warps (8 or 16)
constexpr bool kPfRegSplit = false;      // single-GPU form: warpgroup 0 (TMA, MMA, 2 idle
                                         // warps) hands registers to the epilogue warpgroups
constexpr int kPfLdCols = 16;            // TMEM columns per tcgen05.ld in the epilogue (16 or 32)
constexpr int kPfEpi0 = kPfRegSplit ? 4 : 2;                // first epilogue warp
constexpr int kPfThreads = 32 * (kPfEpi0 + kPfEpiWarps);
constexpr int kPfStage = 128 * 128 + 256 * 128;   // A 16 KB + B 32 KB
constexpr int kPfMaxStages = 6;

// The expert-parallel form adds six warps (warps 2-3 and a fourth warpgroup,
// warps 12-15; the epilogue is warps 4-11): four pull the tile rows from the
// peers and two push finished rows to them while the tile pipeline runs.
constexpr int kPfPullWarps = 4, kPfPushWarps = 2;
constexpr int kPfEpEpiWarps = 8;
constexpr int kPfEpLdCols = 16;         // its TMEM columns per tcgen05.ld (192-register epilogue)
constexpr int kPfPeerThreads = 16 * 32;

// Register split (setmaxnreg) of a launch with `threads` threads and one CTA
// per SM.  Each of the 4 SM sub-partitions holds 16384 registers and every
// 4th warp, so a thread gets 16384 / (32 x ceil(warps / 4)) rounded down to 8;
// `ctl_warpgroups` warpgroups drop to `ctl` and the epilogue warps take what
// is left (rounded down to 8, at most 256).  The sum never exceeds the
// launch's registers, so every setmaxnreg.inc is satisfiable.
__host__ __device__ constexpr int pf_launch_regs(int threads) {
    return (16384 / (32 * ((threads / 32 + 3) / 4))) & ~7;
}
__host__ __device__ constexpr int pf_epi_regs(int threads, int ctl_warpgroups, int ctl,
                                              int epi_warps) {
    const int r =
        ((pf_launch_regs(threads) * threads - 128 * ctl_warpgroups * ctl) / (32 * epi_warps)) & ~7;
    return r > 256 ? 256 : r;
}
constexpr int kPfCtlRegs = 56;           // single-GPU form, warpgroup 0
constexpr int kPfEpiRegs = pf_epi_regs(kPfThreads, 1, kPfCtlRegs, kPfEpiWarps);
constexpr int kPfEpCtlRegs = 64;         // expert-parallel form, warpgroups 0 and 3
constexpr int kPfEpEpiRegs = pf_epi_regs(kPfPeerThreads, 2, kPfEpCtlRegs, kPfEpEpiWarps);
static_assert(!kPfRegSplit || kPfThreads % 128 == 0, "register split needs whole warpgroups");
static_assert(kPfEpiWarps == 8 || kPfEpiWarps == 16, "8 or 16 epilogue warps");

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
constexpr int kPpEpiWarps = kPfEpiWarps;    // CTA-pair form: the single-CTA form's warp roles
constexpr int kPpThreads = kPfThreads;
constexpr int kPpBN = 256;                   // its weight rows per pair tile (256 or 128)

// CTA-pair tile of 256 tokens x BN weight rows: each CTA loads 128 token rows
// and BN/2 weight rows per 128-wide K block and holds a 128 x BN fp32 partial
// per K block in Tensor Memory (512 / BN buffers).
template <int BN>
struct PpTile {
    static constexpr int kB = (BN / 2) * 128;            // this CTA's weight rows x 128 bytes
    static constexpr int kStage = 128 * 128 + kB;        // A 16 KB + B 16 or 8 KB
    static constexpr int kBufs = 512 / BN;
    static constexpr int kMaxStages = BN == 256 ? 6 : 9;
};

struct Pp2Layout {
    int stages_off, segs_off, segc_off, mts_off, part_off, bar_off, misc_off, total;
};

template <int BN>
__host__ __device__ inline Pp2Layout pp2_layout(int stages, int E) {
    using T = PpTile<BN>;
    Pp2Layout L;
    int o = 0;
    L.stages_off = o;
    o += T::kStage * stages;
    L.segs_off = o;
    o += 4 * E;
    L.segc_off = o;
    o += 4 * E;
    L.mts_off = o;
    o += 4 * (E + 1);
    L.part_off = o;
    o += 4 * (kPpThreads + 1);
    o = (o + 7) & ~7;
    L.bar_off = o;
    o += 8 * (2 * T::kMaxStages + 2 * T::kBufs + 1);
    L.misc_off = o;
    o += 16;
    L.total = o;
    return L;
}

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
    o += 4 * (kPpThreads + 1);
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
