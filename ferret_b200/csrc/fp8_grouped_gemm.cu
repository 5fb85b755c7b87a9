// fp8_grouped_gemm.cu -- FP8 (e4m3) block-scaled grouped GEMM for the MoE
// W13 projection, contiguous layout, on sm_100a tensor cores.
//
//   out[r, n] = sum_kb a_scale[r, kb] * w_scale[e(r), n/128, kb]
//                      * sum_{k in kb} a[r, k] * w[e(r), n, k]          (bf16)
//   optional fused epilogue: out[r, j] = silu(x[r, j]) * x[r, N/2 + j]
//
// Design (one persistent CTA per SM, 6 warps):
//   * swap-AB: the 128 weight rows of an n-block sit on the MMA M axis and the
//     token rows of one expert (a tile of NT = 16..128 rows) on the MMA N
//     axis, so the weight stream is read once, K-major, by whole 128x128-byte
//     TMA boxes, however few tokens an expert has (decode).
//   * warp 0 streams W and A tiles with TMA into an NS-deep shared-memory
//     ring (128-byte swizzle); weights carry an evict-first L2 hint.
//   * warp 1 issues tcgen05.mma kind::f8f6f4 (M=128, K=32, N = the tile's
//     live token rows rounded up to 16) from one elected thread; each 128-wide
//     K block goes to its own TMEM accumulator buffer (up to 8 in flight) so
//     the scales can be applied exactly.  Activation rows arrive in 16-row
//     TMA boxes, only as many as the tile holds.
//   * warps 2-5 (128 threads, one TMEM lane = one weight row each) read each
//     K-block partial with tcgen05.ld and promote it in fp32 registers:
//     acc += partial * (a_scale * w_scale) -- the exact-fp32-scale contract
//     (no UE8M0 rounding of the scales).  With FERRET_SILU_MUL the CTA pairs
//     gate block j with up block j + N/256 so SiLU(gate)*up is formed in
//     registers and only N/2 columns are written.
//   * tiles never straddle experts: the schedule is built per CTA in the
//     prologue from the expert segments (prefix offsets, or (start, count)
//     pairs derived from m_indices), so ragged groups of any size are exact.
//   * when the tiles cannot fill half the SMs, K is split over them: fp32
//     partials in the workspace, reduced in split order by the last unit of
//     each tile (an atomic tile counter) -- deterministic.
// Every mbarrier wait is bounded (ferret_common.cuh).
// The prefill-shaped kernel (tokens on MMA M) follows further below.
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

template <int NT, bool PAIR>
struct Cfg {
    static constexpr int kW = PAIR ? 2 : 1;
    static constexpr int kATile = NT * 128;
    static constexpr int kStage = kW * kWTile + kATile;     // multiple of 1024
    static constexpr int kCols = NT * kW;                   // TMEM columns per accumulator
    static constexpr int kAcc = (512 / kCols) > kMaxAcc ? kMaxAcc : (512 / kCols);
    static constexpr int kUsedCols = kAcc * kCols;
    static constexpr int kTmemCols = kUsedCols <= 32 ? 32
                                   : kUsedCols <= 64 ? 64
                                   : kUsedCols <= 128 ? 128
                                   : kUsedCols <= 256 ? 256 : 512;
};

// Shared-memory layout, identical on host (sizing) and device (carving).
struct Layout {
    int stages_off, asc_off, wsc_off, segs_off, segc_off, mts_off, part_off, bar_off, misc_off, total;
};

__host__ __device__ inline Layout make_layout(int stage_bytes, int stages, int NT, int kW, int nk,
                                              int E) {
    Layout L;
    int o = 0;
    L.stages_off = o;
    o += stage_bytes * stages;
    L.asc_off = o;
    o += 4 * NT * nk;
    L.wsc_off = o;
    o += 4 * kW * nk;
    L.segs_off = o;
    o += 4 * E;
    L.segc_off = o;
    o += 4 * E;
    L.mts_off = o;
    o += 4 * (E + 1);
    L.part_off = o;
    o += 4 * (kThreads + 1);
    o = (o + 7) & ~7;
    L.bar_off = o;
    o += 8 * (2 * kMaxStages + 2 * kMaxAcc + 2);
    L.misc_off = o;
    o += 16;
    L.total = o;
    return L;
}

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

template <int NT, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_w13_grouped_kernel(const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_a, const GemmArgs args,
                           const SplitArgs split) {
    pdl_begin();
    using C = Cfg<NT, PAIR>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int M = args.M, N = args.N, K = args.K, E = args.E, NS = args.stages;
    const int nk = K >> 7;
    const int nbc = PAIR ? (N >> 8) : (N >> 7);
    const Layout L = make_layout(C::kStage, NS, NT, C::kW, nk, E);

    float* a_sc = reinterpret_cast<float*>(smem + L.asc_off);     // [nk][NT]
    float* w_sc = reinterpret_cast<float*>(smem + L.wsc_off);     // [kW][nk]
    int* seg_s = reinterpret_cast<int*>(smem + L.segs_off);
    int* seg_c = reinterpret_cast<int*>(smem + L.segc_off);
    int* mt_start = reinterpret_cast<int*>(smem + L.mts_off);
    int* part = reinterpret_cast<int*>(smem + L.part_off);
    const uint32_t bar0 = smem_addr(smem + L.bar_off);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kMaxStages + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kMaxStages + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kMaxStages + kMaxAcc + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kMaxStages + 2 * kMaxAcc);
    const uint32_t epi_bar = drain_bar + 8u;   // epilogue-warps rendezvous (bounded)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    const uint32_t stage_base = smem_addr(smem + L.stages_off);

    // ---- prologue: barriers, TMEM, expert schedule
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < C::kAcc; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), kEpiThreads);
        }
        mbar_init(drain_bar, 1);
        mbar_init(epi_bar, kEpiThreads);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    bool seg_bad = false;
    for (int e = tid; e < E; e += kThreads) {
        int s, c;
        if (args.seg_pairs) {
            s = args.seg[2 * e];
            c = args.seg[2 * e + 1];
        } else {
            s = args.seg[e];
            c = args.seg[e + 1] - s;
        }
        // clamp to [0, M): a malformed segment never addresses outside out / A
        if (s < 0 || s > M || c < 0 || c > M - s) {
            seg_bad = true;
            s = min(max(s, 0), M);
            c = min(max(c, 0), M - s);
        }
        seg_s[e] = s;
        seg_c[e] = c;
        mt_start[e] = (c + NT - 1) / NT;
    }
    if (seg_bad) report(args.ctl, DEV_LAYOUT);
    __syncthreads();
    block_exclusive_scan(mt_start, E, part);   // ends with __syncthreads
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int tiles = mt_start[E] * nbc;
    // split-K when the tiles cannot fill the SMs (every CTA derives the same S)
    int S = 1;
    if (split.splits_max > 1 && tiles > 0 && 2 * tiles <= (int)gridDim.x) {
        S = min((int)gridDim.x / tiles, min(split.splits_max, nk));
        const size_t unit_bytes = (size_t)C::kCols * 128 * sizeof(float);
        while (S > 1 && (size_t)tiles * S * unit_bytes > split.part_bytes) --S;
    }
    const int total = tiles * S;                  // work units: (tile, K split)

    if (warp == 0) {
        // ================= TMA producer =================
        if (elect_one()) {
            tma_prefetch_desc(&tm_w);
            tma_prefetch_desc(&tm_a);
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_a = policy_evict_last();
            int it = 0;
            RingPos rp;
            for (int u = blockIdx.x; u < total; u += gridDim.x) {
                const int t = u / S, sp = u - t * S;
                int e, row0, rows, nb;
                decode_tile<NT>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
                const int nl = (rows + kABox - 1) & ~(kABox - 1);   // live token rows, 16-row granule
                const int wrow = e * N + nb * 128;
                const int wrow_up = e * N + (N >> 1) + nb * 128;
                bool ok = true;
                for (int kb = sp * nk / S; kb < (sp + 1) * nk / S; ++kb, ++it, rp.advance(NS)) {
                    const int s = rp.slot;
                    if (!mbar_wait(empty_bar(s), rp.phase ^ 1u, abort_flag, args.ctl,
                                   SITE_EMPTY)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = stage_base + s * C::kStage;
                    mbar_expect_tx(full_bar(s), C::kW * kWTile + nl * 128);
                    tma_load_2d_hint(dst, &tm_w, kb * 128, wrow, full_bar(s), pol_w);
                    if (PAIR) tma_load_2d_hint(dst + kWTile, &tm_w, kb * 128, wrow_up, full_bar(s), pol_w);
                    for (int b = 0; b < nl; b += kABox)
                        tma_load_2d_hint(dst + C::kW * kWTile + b * 128, &tm_a, kb * 128, row0 + b,
                                         full_bar(s), pol_a);
                }
                if (!ok) break;
            }
            // drain: the last load issued into each stage may still be in flight
            for (int i = max(0, it - NS); i < it; ++i)
                mbar_wait(full_bar(i % NS), (i / NS) & 1, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else if (warp == 1) {
        // ================= MMA issuer =================
        if (elect_one()) {
            RingPos rs, ra;
            for (int u = blockIdx.x; u < total; u += gridDim.x) {
                const int t = u / S, sp = u - t * S;
                int e, row0, rows, nb;
                decode_tile<NT>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
                // MMA N = the tile's live token rows rounded up to 16
                const uint32_t idesc = make_idesc(128, (rows + kABox - 1) & ~(kABox - 1), 0, 0);
                bool ok = true;
                for (int kb = sp * nk / S; kb < (sp + 1) * nk / S; ++kb, rs.advance(NS), ra.advance(C::kAcc)) {
                    const int s = rs.slot, a = ra.slot;
                    if (!mbar_wait(tempty_bar(a), ra.phase ^ 1u, abort_flag, args.ctl,
                                   SITE_TEMPTY) ||
                        !mbar_wait(full_bar(s), rs.phase, abort_flag, args.ctl, SITE_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = stage_base + s * C::kStage;
                    const uint32_t a_tile = st + C::kW * kWTile;
                    const uint32_t d = tmem_base + a * C::kCols;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t bdesc = sdesc_k_sw128(a_tile + ks * 32);
                        mma_f8f6f4(d, sdesc_k_sw128(st + ks * 32), bdesc, idesc, ks > 0);
                        if (PAIR) mma_f8f6f4(d + NT, sdesc_k_sw128(st + kWTile + ks * 32), bdesc, idesc, ks > 0);
                    }
                    tc_commit(empty_bar(s));
                    tc_commit(tfull_bar(a));
                }
                if (!ok) break;
            }
            // every MMA this thread issued has finished before TMEM is freed
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else {
        // ================= epilogue: promotion + store =================
        const int q = warp & 3;              // TMEM lanes [32q, 32q+32)
        const int et = tid - 64;             // 0..127
        const int lane = tid & 31;
        const int ldo = PAIR ? (N >> 1) : N;
        int ai = 0;
        uint32_t epi_phase = 0;
        // rendezvous of the 128 epilogue threads; bounded and abort-aware so a
        // warp that gave up never strands the others
        auto epi_sync = [&]() -> bool {
            mbar_arrive(epi_bar);
            bool ok = mbar_wait(epi_bar, epi_phase & 1u, abort_flag, args.ctl, SITE_EPI);
            ++epi_phase;
            return __all_sync(0xffffffffu, ok);
        };
        __shared__ int s_last;
        for (int u = blockIdx.x; u < total; u += gridDim.x) {
            const int t = u / S, sp = u - t * S;
            const int kb0 = sp * nk / S, kb1 = (sp + 1) * nk / S;
            int e, row0, rows, nb;
            decode_tile<NT>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            const int nl = (rows + kABox - 1) & ~(kABox - 1);
            // stage this tile's scales: a_sc[kb][j], w_sc[g][kb]
            if (!epi_sync()) break;
            for (int i = et; i < nl * nk; i += kEpiThreads) {
                const int j = i / nk, kb = i - j * nk;
                a_sc[kb * NT + j] = (j < rows) ? __ldg(args.a_scale + (size_t)(row0 + j) * nk + kb) : 0.0f;
            }
            const size_t wsb = ((size_t)e * (N >> 7) + nb) * nk;
            for (int i = et; i < nk; i += kEpiThreads) {
                w_sc[i] = __ldg(args.w_scale + wsb + i);
                if (PAIR) w_sc[nk + i] = __ldg(args.w_scale + wsb + (size_t)(N >> 8) * nk + i);
            }
            if (!epi_sync()) break;

            float acc_g[NT];
            float acc_u[PAIR ? NT : 1];
#pragma unroll
            for (int j = 0; j < NT; ++j) acc_g[j] = 0.0f;
#pragma unroll
            for (int j = 0; j < (PAIR ? NT : 1); ++j) acc_u[j] = 0.0f;

            bool ok = true;
            for (int kb = kb0; kb < kb1; ++kb, ++ai) {
                const int a = ai % C::kAcc;
                ok = __all_sync(0xffffffffu, mbar_wait(tfull_bar(a), (ai / C::kAcc) & 1, abort_flag,
                                                       args.ctl, SITE_TFULL));
                if (!ok) break;
                tc_fence_after();
                const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + a * C::kCols;
                const float ws = w_sc[kb];
                const float wsu = PAIR ? w_sc[nk + kb] : 0.0f;
                const float* asc = a_sc + kb * NT;
#pragma unroll
                for (int c = 0; c < NT; c += 16) {
                    if (c >= nl) break;                  // columns past the tile's MMA N
                    float v[16], uu[16];
                    tmem_ld16(tb + c, v);
                    if (PAIR) tmem_ld16(tb + NT + c, uu);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float sa = asc[c + j];
                        acc_g[c + j] = fmaf(v[j], sa * ws, acc_g[c + j]);
                        if (PAIR) acc_u[c + j] = fmaf(uu[j], sa * wsu, acc_u[c + j]);
                    }
                }
                tc_fence_before();
                mbar_arrive(tempty_bar(a));
            }
            if (!ok) break;
            if (S > 1) {
                // this unit's fp32 partial, [col][128 rows]: a warp writes 128 contiguous bytes
                float* pu = split.part + (size_t)u * C::kCols * 128 + et;
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    if (j < nl) {
                        pu[(size_t)j * 128] = acc_g[j];
                        if (PAIR) pu[(size_t)(NT + j) * 128] = acc_u[PAIR ? j : 0];
                    }
                }
                __threadfence();
                if (!epi_sync()) break;
                if (et == 0) s_last = (atomicAdd(split.cnt + t, 1) == S - 1);
                if (!epi_sync()) break;
                if (!s_last) continue;
                __threadfence();
                // last unit of the tile: the S partials, summed in split order
                const float* pt = split.part + (size_t)t * S * C::kCols * 128 + et;
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    if (j < nl) {
                        float g = 0.0f, v2 = 0.0f;
                        for (int s2 = 0; s2 < S; ++s2) {
                            g += __ldcg(pt + ((size_t)s2 * C::kCols + j) * 128);
                            if (PAIR) v2 += __ldcg(pt + ((size_t)s2 * C::kCols + NT + j) * 128);
                        }
                        acc_g[j] = g;
                        if (PAIR) acc_u[PAIR ? j : 0] = v2;
                    }
                }
                if (et == 0) split.cnt[t] = 0;
            }
            // store: this thread owns output column n for the tile's rows
            const int n = nb * 128 + q * 32 + lane;
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                if (j < rows) {
                    int orow = row0 + j;
                    if (args.out_rows) {
                        orow = __ldg(args.out_rows + row0 + j);
                        if (orow < 0 || orow >= args.out_total) continue;
                    }
                    const float val = PAIR ? silu_mul(acc_g[j], acc_u[PAIR ? j : 0]) : acc_g[j];
                    out_row_ptr(args, orow, ldo)[n] = __float2bfloat16_rn(val);
                }
            }
        }
    }

    // ---- teardown
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// m_indices -> per-expert (start, count), single CTA.  A row starts a segment
// when its predecessor holds another expert, ends one when its successor does.
// Two starts for one expert mean its rows are not contiguous (DEV_LAYOUT).
constexpr int kSegThreads = 1024;

__global__ void __launch_bounds__(kSegThreads, 1)
    derive_segments_kernel(const int32_t* __restrict__ m, int M, int E, int32_t* __restrict__ seg,
                           DevCtl ctl, int* __restrict__ cnt, int ncnt) {
    pdl_begin();
    extern __shared__ int sm[];
    for (int i = threadIdx.x; i < ncnt; i += kSegThreads) cnt[i] = 0;   // split-K tile counters
    int* nst = sm;
    int* fst = sm + E;
    int* lst = sm + 2 * E;
    for (int e = threadIdx.x; e < E; e += kSegThreads) {
        nst[e] = 0;
        fst[e] = 0;
        lst[e] = -1;
    }
    __syncthreads();
    bool bad_e = false;
    for (int r = threadIdx.x; r < M; r += kSegThreads) {
        const int e = m[r];
        if (e < 0) continue;
        if (e >= E) {
            bad_e = true;
            continue;
        }
        const int prev = r > 0 ? m[r - 1] : -1;
        const int next = r + 1 < M ? m[r + 1] : -1;
        if (prev != e) {
            atomicAdd(&nst[e], 1);
            fst[e] = r;
        }
        if (next != e) lst[e] = r;
    }
    if (bad_e) report(ctl, DEV_BAD_EXPERT);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += kSegThreads) {
        int s = 0, c = 0;
        if (nst[e] > 0) {
            if (nst[e] > 1) report(ctl, DEV_LAYOUT);
            s = fst[e];
            c = max(0, lst[e] - fst[e] + 1);
        }
        seg[2 * e] = s;
        seg[2 * e + 1] = c;
    }
}

template <int NT, bool PAIR>
int launch_fp8(const DeviceInfo* info, const void* a, const float* a_scale, const void* w,
               const float* w_scale, void* out, const int32_t* seg, int seg_pairs, int M, int N,
               int K, int E, cudaStream_t stream, const OutMap& om = OutMap{},
               const SplitWs& sw = SplitWs{}) {
    using C = Cfg<NT, PAIR>;
    CUtensorMap tm_w, tm_a;
    int rc = make_tmap_2d(&tm_w, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)E * N, K, K, 128,
                          128, true);
    if (rc != FERRET_OK) return rc;
    rc = make_tmap_2d(&tm_a, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, K, 128, kABox, true);
    if (rc != FERRET_OK) return rc;
    const int nk = K / 128;
    const int budget = info->max_smem_optin - 1024;   // 1 KB for base alignment
    const Layout l0 = make_layout(C::kStage, 0, NT, C::kW, nk, E);
    int stages = std::min(kMaxStages, (budget - l0.total) / C::kStage);
    if (stages < 2) return FERRET_ERR_SHAPE;
    const Layout L = make_layout(C::kStage, stages, NT, C::kW, nk, E);
    const int smem = L.total + 1024;
    auto kern = fp8_w13_grouped_kernel<NT, PAIR>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    GemmArgs g;
    g.a_scale = a_scale;
    g.w_scale = w_scale;
    g.seg = seg;
    g.seg_pairs = seg_pairs;
    g.out = static_cast<__nv_bfloat16*>(out);
    g.out_rows = om.rows;
    g.out_total = om.total;
    g.out_peers = om.peers;
    g.peer_rows = om.peer_rows;
    g.M = M;
    g.N = N;
    g.K = K;
    g.E = E;
    g.stages = stages;
    g.ctl = make_ctl(info);
    SplitArgs sp;
    sp.splits_max = sw.part ? sw.smax : 1;
    sp.part = sw.part;
    sp.cnt = sw.cnt;
    sp.part_bytes = sw.bytes;
    return launch_kernel(kern, dim3(info->num_sms), dim3(kThreads), smem, stream, tm_w, tm_a, g, sp);
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

// Per epilogue warp: a 32-row x 32-column bf16 staging block (rows padded to
// 80 bytes: conflict-free 16-byte writes) and the 32 rows' output pointers.
constexpr int kPfStgRow = 80;
constexpr int kPfStgWarp = 32 * kPfStgRow + 32 * 8;

struct PfLayout {
    int stages_off, segs_off, segc_off, mts_off, part_off, stg_off, bar_off, misc_off, total;
};

__host__ __device__ inline PfLayout pf_layout(int stages, int E, bool staged) {
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
    o += 4 * (kPfThreads + 1);
    o = (o + 7) & ~7;
    L.stg_off = o;
    if (staged) {
        o = (o + 15) & ~15;
        L.stg_off = o;
        o += kPfStgWarp * (kPfEpi / 32);
    }
    L.bar_off = o;
    o += 8 * (2 * kPfMaxStages + 2 * 2 + 2);
    L.misc_off = o;
    o += 16;
    L.total = o;
    return L;
}

// REM: only the rows of each expert past its whole 256-row chunks (which the
// CTA-pair kernel below takes), i.e. its last count % 256 rows.
template <bool PAIR, bool REM = false>
__global__ void __launch_bounds__(kPfThreads, 1)
    fp8_w13_prefill_kernel(const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_a, const GemmArgs args) {
    pdl_begin();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = args.M, N = args.N, K = args.K, E = args.E, NS = args.stages;
    const int nk = K >> 7;
    const int nbc = N >> 8;                        // 256-row weight tiles
    const PfLayout L = pf_layout(NS, E, false);
    int* seg_s = reinterpret_cast<int*>(smem + L.segs_off);
    int* seg_c = reinterpret_cast<int*>(smem + L.segc_off);
    int* mt_start = reinterpret_cast<int*>(smem + L.mts_off);
    int* part = reinterpret_cast<int*>(smem + L.part_off);
    const uint32_t bar0 = smem_addr(smem + L.bar_off);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kPfMaxStages + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kPfMaxStages + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kPfMaxStages + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kPfMaxStages + 4);
    const uint32_t epi_bar = drain_bar + 8u;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    const uint32_t stage_base = smem_addr(smem + L.stages_off);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), kPfEpi);
        }
        mbar_init(drain_bar, 1);
        mbar_init(epi_bar, kPfEpi);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), 512);
        tmem_relinquish();
    }
    bool seg_bad = false;
    for (int e = tid; e < E; e += kPfThreads) {
        int s, c;
        if (args.seg_pairs) {
            s = args.seg[2 * e];
            c = args.seg[2 * e + 1];
        } else {
            s = args.seg[e];
            c = args.seg[e + 1] - s;
        }
        if (s < 0 || s > M || c < 0 || c > M - s) {
            seg_bad = true;
            s = min(max(s, 0), M);
            c = min(max(c, 0), M - s);
        }
        if (REM) {
            s += c & ~255;
            c &= 255;
        }
        seg_s[e] = s;
        seg_c[e] = c;
        mt_start[e] = (c + 127) >> 7;
    }
    if (seg_bad) report(args.ctl, DEV_LAYOUT);
    __syncthreads();
    block_exclusive_scan(mt_start, E, part);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = mt_start[E] * nbc;

    if (warp == 0) {
        // ================= TMA producer =================
        if (elect_one()) {
            tma_prefetch_desc(&tm_w);
            tma_prefetch_desc(&tm_a);
            const uint64_t pol_w = policy_evict_last();     // reused by the expert's token tiles
            const uint64_t pol_a = policy_evict_last();
            int it = 0;
            RingPos rp;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int e, row0, rows, nb;
                decode_tile<128>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
                const int w0 = PAIR ? e * N + nb * 128 : e * N + nb * 256;
                const int w1 = PAIR ? e * N + (N >> 1) + nb * 128 : w0 + 128;
                for (int kb = 0; kb < nk; ++kb, ++it, rp.advance(NS)) {
                    const int s = rp.slot;
                    if (!mbar_wait(empty_bar(s), rp.phase ^ 1u, abort_flag, args.ctl, SITE_EMPTY)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = stage_base + s * kPfStage;
                    mbar_expect_tx(full_bar(s), kPfStage);
                    tma_load_2d_hint(dst, &tm_a, kb * 128, row0, full_bar(s), pol_a);
                    tma_load_2d_hint(dst + 16384, &tm_w, kb * 128, w0, full_bar(s), pol_w);
                    tma_load_2d_hint(dst + 32768, &tm_w, kb * 128, w1, full_bar(s), pol_w);
                }
            }
            for (int i = max(0, it - NS); i < it; ++i)
                mbar_wait(full_bar(i % NS), (i / NS) & 1, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else if (warp == 1) {
        // ================= MMA issuer =================
        if (elect_one()) {
            constexpr uint32_t idesc = make_idesc(128, 256, 0, 0);
            RingPos rs, ra;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                for (int kb = 0; kb < nk; ++kb, rs.advance(NS), ra.advance(2)) {
                    const int s = rs.slot, a = ra.slot;
                    if (!mbar_wait(tempty_bar(a), ra.phase ^ 1u, abort_flag, args.ctl, SITE_TEMPTY) ||
                        !mbar_wait(full_bar(s), rs.phase, abort_flag, args.ctl, SITE_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = stage_base + s * kPfStage;
                    const uint32_t d = tmem_base + a * 256;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f8f6f4(d, sdesc_k_sw128(st + ks * 32), sdesc_k_sw128(st + 16384 + ks * 32),
                                   idesc, ks > 0);
                    tc_commit(empty_bar(s));
                    tc_commit(tfull_bar(a));
                }
            }
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else {
        // ================= epilogue: promotion + store =================
        const int h = (warp - 2) >> 2;           // column half: [64h, 64h+64) of each block
        const int q = warp & 3;                  // TMEM lanes [32q, 32q+32) = tile rows
        const int r = q * 32 + lane;
        const int ldo = PAIR ? (N >> 1) : N;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        RingPos ra;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int e, row0, rows, nb;
            decode_tile<128>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            const bool live = r < rows;
            const float* as_row = args.a_scale + (size_t)(row0 + (live ? r : 0)) * nk;
            const int blk0 = PAIR ? nb : 2 * nb;
            const int blk1 = PAIR ? (N >> 8) + nb : 2 * nb + 1;
            const float* ws0 = args.w_scale + ((size_t)e * (N >> 7) + blk0) * nk;
            const float* ws1 = args.w_scale + ((size_t)e * (N >> 7) + blk1) * nk;
            float acc0[64], acc1[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                acc0[j] = 0.0f;
                acc1[j] = 0.0f;
            }
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb, ra.advance(2)) {
                const float sa = live ? __ldg(as_row + kb) : 0.0f;
                const float s0 = sa * __ldg(ws0 + kb), s1 = sa * __ldg(ws1 + kb);
                ok = __all_sync(0xffffffffu, mbar_wait(tfull_bar(ra.slot), ra.phase, abort_flag,
                                                       args.ctl, SITE_TFULL));
                if (!ok) break;
                tc_fence_after();
                const uint32_t tb = tmem_base + lane_addr + ra.slot * 256 + h * 64;
#pragma unroll
                for (int c = 0; c < 64; c += 16) {
                    float v[16], u[16];
                    tmem_ld16(tb + c, v);
                    tmem_ld16(tb + 128 + c, u);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        acc0[c + j] = fmaf(v[j], s0, acc0[c + j]);
                        acc1[c + j] = fmaf(u[j], s1, acc1[c + j]);
                    }
                }
                tc_fence_before();
                mbar_arrive(tempty_bar(ra.slot));
            }
            if (!ok) break;
            int orow = row0 + r;
            if (live && args.out_rows) {
                orow = __ldg(args.out_rows + row0 + r);
                if (orow < 0 || orow >= args.out_total) orow = -1;
            }
            if (live && orow >= 0) {
                __nv_bfloat16* o = out_row_ptr(args, orow, ldo);
                if (PAIR) {
                    uint4* dst = reinterpret_cast<uint4*>(o + nb * 128 + h * 64);
#pragma unroll
                    for (int c = 0; c < 64; c += 8) {
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
                    uint4* d0 = reinterpret_cast<uint4*>(o + nb * 256 + h * 64);
                    uint4* d1 = reinterpret_cast<uint4*>(o + nb * 256 + 128 + h * 64);
#pragma unroll
                    for (int c = 0; c < 64; c += 8) {
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
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}

// The same kernel for output rows on other GPUs (expert parallelism): rows are
// written through shared memory, 64 contiguous bytes of 8 rows per store
// instruction, because 16-byte writes scattered over 32 rows make poor NVLink
// transactions.  A separate function rather than a template switch of the one
// above, so that the local kernel's code generation stays as measured.
template <bool PAIR>
__global__ void __launch_bounds__(kPfThreads, 1)
    fp8_w13_prefill_peer_kernel(const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_a, const GemmArgs args) {
    pdl_begin();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = args.M, N = args.N, K = args.K, E = args.E, NS = args.stages;
    const int nk = K >> 7;
    const int nbc = N >> 8;                        // 256-row weight tiles
    const PfLayout L = pf_layout(NS, E, true);
    int* seg_s = reinterpret_cast<int*>(smem + L.segs_off);
    int* seg_c = reinterpret_cast<int*>(smem + L.segc_off);
    int* mt_start = reinterpret_cast<int*>(smem + L.mts_off);
    int* part = reinterpret_cast<int*>(smem + L.part_off);
    const uint32_t bar0 = smem_addr(smem + L.bar_off);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kPfMaxStages + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kPfMaxStages + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kPfMaxStages + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kPfMaxStages + 4);
    const uint32_t epi_bar = drain_bar + 8u;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    const uint32_t stage_base = smem_addr(smem + L.stages_off);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), kPfEpi);
        }
        mbar_init(drain_bar, 1);
        mbar_init(epi_bar, kPfEpi);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), 512);
        tmem_relinquish();
    }
    bool seg_bad = false;
    for (int e = tid; e < E; e += kPfThreads) {
        int s, c;
        if (args.seg_pairs) {
            s = args.seg[2 * e];
            c = args.seg[2 * e + 1];
        } else {
            s = args.seg[e];
            c = args.seg[e + 1] - s;
        }
        if (s < 0 || s > M || c < 0 || c > M - s) {
            seg_bad = true;
            s = min(max(s, 0), M);
            c = min(max(c, 0), M - s);
        }
        seg_s[e] = s;
        seg_c[e] = c;
        mt_start[e] = (c + 127) >> 7;
    }
    if (seg_bad) report(args.ctl, DEV_LAYOUT);
    __syncthreads();
    block_exclusive_scan(mt_start, E, part);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = mt_start[E] * nbc;

    if (warp == 0) {
        // ================= TMA producer =================
        if (elect_one()) {
            tma_prefetch_desc(&tm_w);
            tma_prefetch_desc(&tm_a);
            const uint64_t pol_w = policy_evict_last();     // reused by the expert's token tiles
            const uint64_t pol_a = policy_evict_last();
            int it = 0;
            RingPos rp;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int e, row0, rows, nb;
                decode_tile<128>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
                const int w0 = PAIR ? e * N + nb * 128 : e * N + nb * 256;
                const int w1 = PAIR ? e * N + (N >> 1) + nb * 128 : w0 + 128;
                for (int kb = 0; kb < nk; ++kb, ++it, rp.advance(NS)) {
                    const int s = rp.slot;
                    if (!mbar_wait(empty_bar(s), rp.phase ^ 1u, abort_flag, args.ctl, SITE_EMPTY)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = stage_base + s * kPfStage;
                    mbar_expect_tx(full_bar(s), kPfStage);
                    tma_load_2d_hint(dst, &tm_a, kb * 128, row0, full_bar(s), pol_a);
                    tma_load_2d_hint(dst + 16384, &tm_w, kb * 128, w0, full_bar(s), pol_w);
                    tma_load_2d_hint(dst + 32768, &tm_w, kb * 128, w1, full_bar(s), pol_w);
                }
            }
            for (int i = max(0, it - NS); i < it; ++i)
                mbar_wait(full_bar(i % NS), (i / NS) & 1, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else if (warp == 1) {
        // ================= MMA issuer =================
        if (elect_one()) {
            constexpr uint32_t idesc = make_idesc(128, 256, 0, 0);
            RingPos rs, ra;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                for (int kb = 0; kb < nk; ++kb, rs.advance(NS), ra.advance(2)) {
                    const int s = rs.slot, a = ra.slot;
                    if (!mbar_wait(tempty_bar(a), ra.phase ^ 1u, abort_flag, args.ctl, SITE_TEMPTY) ||
                        !mbar_wait(full_bar(s), rs.phase, abort_flag, args.ctl, SITE_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = stage_base + s * kPfStage;
                    const uint32_t d = tmem_base + a * 256;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f8f6f4(d, sdesc_k_sw128(st + ks * 32), sdesc_k_sw128(st + 16384 + ks * 32),
                                   idesc, ks > 0);
                    tc_commit(empty_bar(s));
                    tc_commit(tfull_bar(a));
                }
            }
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else {
        // ================= epilogue: promotion + store =================
        const int h = (warp - 2) >> 2;           // column half: [64h, 64h+64) of each block
        const int q = warp & 3;                  // TMEM lanes [32q, 32q+32) = tile rows
        const int r = q * 32 + lane;
        const int ldo = PAIR ? (N >> 1) : N;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        uint8_t* stg = smem + L.stg_off + (warp - 2) * kPfStgWarp;
        __nv_bfloat16** rowp = reinterpret_cast<__nv_bfloat16**>(stg + 32 * kPfStgRow);
        RingPos ra;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int e, row0, rows, nb;
            decode_tile<128>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            const bool live = r < rows;
            const float* as_row = args.a_scale + (size_t)(row0 + (live ? r : 0)) * nk;
            const int blk0 = PAIR ? nb : 2 * nb;
            const int blk1 = PAIR ? (N >> 8) + nb : 2 * nb + 1;
            const float* ws0 = args.w_scale + ((size_t)e * (N >> 7) + blk0) * nk;
            const float* ws1 = args.w_scale + ((size_t)e * (N >> 7) + blk1) * nk;
            float acc0[64], acc1[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                acc0[j] = 0.0f;
                acc1[j] = 0.0f;
            }
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb, ra.advance(2)) {
                const float sa = live ? __ldg(as_row + kb) : 0.0f;
                const float s0 = sa * __ldg(ws0 + kb), s1 = sa * __ldg(ws1 + kb);
                ok = __all_sync(0xffffffffu, mbar_wait(tfull_bar(ra.slot), ra.phase, abort_flag,
                                                       args.ctl, SITE_TFULL));
                if (!ok) break;
                tc_fence_after();
                const uint32_t tb = tmem_base + lane_addr + ra.slot * 256 + h * 64;
#pragma unroll
                for (int c = 0; c < 64; c += 16) {
                    float v[16], u[16];
                    tmem_ld16(tb + c, v);
                    tmem_ld16(tb + 128 + c, u);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        acc0[c + j] = fmaf(v[j], s0, acc0[c + j]);
                        acc1[c + j] = fmaf(u[j], s1, acc1[c + j]);
                    }
                }
                tc_fence_before();
                mbar_arrive(tempty_bar(ra.slot));
            }
            if (!ok) break;
            int orow = row0 + r;
            if (live && args.out_rows) {
                orow = __ldg(args.out_rows + row0 + r);
                if (orow < 0 || orow >= args.out_total) orow = -1;
            }
            // Staged: every store instruction writes 64 contiguous bytes of 8
            // rows instead of 16 bytes of 32 rows.
            rowp[lane] = (live && orow >= 0) ? out_row_ptr(args, orow, ldo) : nullptr;
#pragma unroll
            for (int k = 0; k < (PAIR ? 2 : 4); ++k) {
                // chunk k: 32 columns of this thread's row
                uint4 pk[4];
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    uint32_t* pw = reinterpret_cast<uint32_t*>(&pk[v]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int c = (PAIR ? k * 32 : (k & 1) * 32) + v * 8 + 2 * j;
                        __nv_bfloat162 b;
                        if (PAIR)
                            b = __floats2bfloat162_rn(silu_mul(acc0[c], acc1[c]),
                                                      silu_mul(acc0[c + 1], acc1[c + 1]));
                        else if (k < 2)
                            b = __floats2bfloat162_rn(acc0[c], acc0[c + 1]);
                        else
                            b = __floats2bfloat162_rn(acc1[c], acc1[c + 1]);
                        pw[j] = *reinterpret_cast<const uint32_t*>(&b);
                    }
                }
                uint4* srow = reinterpret_cast<uint4*>(stg + lane * kPfStgRow);
#pragma unroll
                for (int v = 0; v < 4; ++v) srow[v] = pk[v];
                __syncwarp();
                const int col = PAIR ? nb * 128 + h * 64 + k * 32
                                     : nb * 256 + (k >> 1) * 128 + h * 64 + (k & 1) * 32;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int idx = i * 32 + lane, row = idx >> 2, part = idx & 3;
                    __nv_bfloat16* o = rowp[row];
                    if (o)
                        reinterpret_cast<uint4*>(o + col)[part] =
                            *reinterpret_cast<const uint4*>(stg + row * kPfStgRow + part * 16);
                }
                __syncwarp();
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}

// ---------------------------------------------------------------------------
// UE8M0 form of the prefill kernel (FERRET_UE8M0_SCALES).  When every scale is
// a power of two (UE8M0-quantized checkpoints and activations), the tensor
// core applies the scales itself: tcgen05.mma kind::mxf8f6f4.block_scale
// multiplies each K=32 slice of row m / column n by 2^(ea-127) * 2^(eb-127),
// read from Tensor Memory, so one accumulator holds the whole K sum and the
// per-K-block promotion in registers disappears.  The products are exact, so
// the result equals the exact-fp32-scale kernel's up to fp32 summation order.
//
// Scale factors sit in TMEM as the MMA reads them (scale vector 1X): the
// scale of row m of a 128-row operand (A: token rows; B: weight rows, 256 =
// two blocks) at column m / 32, lane m % 32, repeated in each of the four
// 32-lane sub-partitions.  One 16-column slot per K block holds A's 4 columns
// (cols 0-3) and B's 8 (cols 8-15); each 32-bit word repeats its exponent
// byte 4 times, so the descriptor's scale-factor id (the byte) is always 0.
//
//   warp 0      TMA producer (as above, 48 KB stages)
//   warp 1      MMA issuer: per K block, 4 block-scaled MMAs into the single
//               256-column accumulator, reading the K block's scale slot
//   warps 2-5   scale writers (one per sub-partition): exponent bytes of
//               a_scale / w_scale -> a ring of 8 TMEM slots, loads issued one
//               group of 4 K blocks ahead
//   warps 6-13  epilogue: the finished tile -> registers as bf16, accumulator
//               released, then the stores
//
// Measured on B200 at benchmark configuration 3 (GEMM alone, CUDA graphs,
// 256 MB flush): 2.664 ms against 2.708 ms for the exact-scale kernel -- both
// sit on the L2->SM operand traffic of the 128x256 tiling, so removing the
// promotion buys little.  With the fused SiLU epilogue the single accumulator
// has to wait for the SiLU arithmetic of the previous tile (2.845 ms against
// 2.721 ms), so SiLU launches keep the exact-scale kernel, which is exact for
// power-of-two scales too.
// ---------------------------------------------------------------------------
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

// REM: only the rows past each expert's whole 256-row chunks (the block-scaled
// CTA-pair kernel takes those).
template <bool REM = false>
__global__ void __launch_bounds__(kMxThreads, 1)
    fp8_w13_prefill_mx_kernel(const __grid_constant__ CUtensorMap tm_w,
                              const __grid_constant__ CUtensorMap tm_a, const GemmArgs args) {
    pdl_begin();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = args.M, N = args.N, K = args.K, E = args.E, NS = args.stages;
    const int nk = K >> 7;
    const int nbc = N >> 8;
    const MxLayout L = mx_layout(NS, E);
    int* seg_s = reinterpret_cast<int*>(smem + L.segs_off);
    int* seg_c = reinterpret_cast<int*>(smem + L.segc_off);
    int* mt_start = reinterpret_cast<int*>(smem + L.mts_off);
    int* part = reinterpret_cast<int*>(smem + L.part_off);
    const uint32_t bar0 = smem_addr(smem + L.bar_off);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kPfMaxStages + s); };
    const uint32_t tfull_bar = bar0 + 8u * (2 * kPfMaxStages);
    const uint32_t tempty_bar = tfull_bar + 8u;
    auto sfull_bar = [&](int j) { return bar0 + 8u * (2 * kPfMaxStages + 2 + j); };
    auto sempty_bar = [&](int j) { return bar0 + 8u * (2 * kPfMaxStages + 2 + kMxSfSlots + j); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kPfMaxStages + 2 + 2 * kMxSfSlots);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    const uint32_t stage_base = smem_addr(smem + L.stages_off);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(tfull_bar, 1);
        mbar_init(tempty_bar, kMxEpi);
        for (int j = 0; j < kMxSfSlots; ++j) {
            mbar_init(sfull_bar(j), 4);           // one arrive per scale-writer warp
            mbar_init(sempty_bar(j), 1);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), 512);
        tmem_relinquish();
    }
    bool seg_bad = false;
    for (int e = tid; e < E; e += kMxThreads) {
        int s, c;
        if (args.seg_pairs) {
            s = args.seg[2 * e];
            c = args.seg[2 * e + 1];
        } else {
            s = args.seg[e];
            c = args.seg[e + 1] - s;
        }
        if (s < 0 || s > M || c < 0 || c > M - s) {
            seg_bad = true;
            s = min(max(s, 0), M);
            c = min(max(c, 0), M - s);
        }
        if (REM) {
            s += c & ~255;
            c &= 255;
        }
        seg_s[e] = s;
        seg_c[e] = c;
        mt_start[e] = (c + 127) >> 7;
    }
    if (seg_bad) report(args.ctl, DEV_LAYOUT);
    __syncthreads();
    block_exclusive_scan(mt_start, E, part);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = mt_start[E] * nbc;

    if (warp == 0) {
        // ================= TMA producer =================
        if (elect_one()) {
            tma_prefetch_desc(&tm_w);
            tma_prefetch_desc(&tm_a);
            const uint64_t pol_w = policy_evict_last();
            const uint64_t pol_a = policy_evict_last();
            int it = 0;
            RingPos rp;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int e, row0, rows, nb;
                decode_tile<128>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
                const int w0 = e * N + nb * 256;
                for (int kb = 0; kb < nk; ++kb, ++it, rp.advance(NS)) {
                    const int s = rp.slot;
                    if (!mbar_wait(empty_bar(s), rp.phase ^ 1u, abort_flag, args.ctl, SITE_EMPTY)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = stage_base + s * kPfStage;
                    mbar_expect_tx(full_bar(s), kPfStage);
                    tma_load_2d_hint(dst, &tm_a, kb * 128, row0, full_bar(s), pol_a);
                    tma_load_2d_hint(dst + 16384, &tm_w, kb * 128, w0, full_bar(s), pol_w);
                    tma_load_2d_hint(dst + 32768, &tm_w, kb * 128, w0 + 128, full_bar(s), pol_w);
                }
            }
            for (int i = max(0, it - NS); i < it; ++i)
                mbar_wait(full_bar(i % NS), (i / NS) & 1, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else if (warp == 1) {
        // ================= MMA issuer =================
        if (elect_one()) {
            constexpr uint32_t idesc = make_idesc_mx(128, 256);
            RingPos rs, rf, ra;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ra.advance(1)) {
                if (!mbar_wait(tempty_bar, ra.phase ^ 1u, abort_flag, args.ctl, SITE_TEMPTY)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < nk; ++kb, rs.advance(NS), rf.advance(kMxSfSlots)) {
                    const int s = rs.slot, f = rf.slot;
                    if (!mbar_wait(sfull_bar(f), rf.phase, abort_flag, args.ctl, SITE_SFULL) ||
                        !mbar_wait(full_bar(s), rs.phase, abort_flag, args.ctl, SITE_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = stage_base + s * kPfStage;
                    const uint32_t sfa = tmem_base + kMxSfCol0 + f * kMxSfCols;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        mma_mxf8f6f4(tmem_base, sdesc_k_sw128(st + ks * 32),
                                     sdesc_k_sw128(st + 16384 + ks * 32), idesc, sfa, sfa + 8,
                                     (kb | ks) != 0);
                    tc_commit(empty_bar(s));
                    tc_commit(sempty_bar(f));
                }
                if (ok) tc_commit(tfull_bar);
            }
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else if (warp < 6) {
        // ================= scale writers =================
        const int q = warp & 3;
        const uint32_t sf_lane = tmem_base + ((uint32_t)(q * 32) << 16) + kMxSfCol0;
        const int nsb = N >> 7;
        // scales of 4 consecutive K blocks from kb0 for tile t: a[m][j] for
        // token rows 32m + lane, w[i][j] for the tile's two weight blocks
        auto load = [&](int t, int kb0, float (&a)[4][4], float (&w)[2][4]) {
            int e, row0, rows, nb;
            decode_tile<128>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            const float* ws0 = args.w_scale + ((size_t)e * nsb + 2 * nb) * nk;
            const float* ws1 = ws0 + nk;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kb = min(kb0 + j, nk - 1);
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const int r = 32 * m + lane;
                    a[m][j] = r < rows ? __ldg(args.a_scale + (size_t)(row0 + r) * nk + kb) : 1.0f;
                }
                w[0][j] = __ldg(ws0 + kb);
                w[1][j] = __ldg(ws1 + kb);
            }
        };
        RingPos rf;
        int t = blockIdx.x, kb0 = 0;
        float a[4][4], w[2][4];
        if (t < total) load(t, 0, a, w);
        bool ok = true;
        while (t < total && ok) {
            int tn = t, kn = kb0 + 4;
            if (kn >= nk) {
                tn = t + gridDim.x;
                kn = 0;
            }
            float an[4][4], wn[2][4];
            if (tn < total) load(tn, kn, an, wn);          // in flight while this group is written
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (kb0 + j >= nk) break;
                ok = __all_sync(0xffffffffu, mbar_wait(sempty_bar(rf.slot), rf.phase ^ 1u,
                                                       abort_flag, args.ctl, SITE_SEMPTY));
                if (!ok) break;
                tc_fence_after();
                const uint32_t col = sf_lane + rf.slot * kMxSfCols;
                tmem_st4(col, ue8m0_word(a[0][j]), ue8m0_word(a[1][j]), ue8m0_word(a[2][j]),
                         ue8m0_word(a[3][j]));
                const uint32_t b0 = ue8m0_word(w[0][j]), b1 = ue8m0_word(w[1][j]);
                const uint32_t bw[8] = {b0, b0, b0, b0, b1, b1, b1, b1};
                tmem_st8(col + 8, bw);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(sfull_bar(rf.slot));
                rf.advance(kMxSfSlots);
            }
            t = tn;
            kb0 = kn;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int m = 0; m < 4; ++m) a[m][j] = an[m][j];
                w[0][j] = wn[0][j];
                w[1][j] = wn[1][j];
            }
        }
    } else {
        // ================= epilogue =================
        const int h = (warp - 6) >> 2;           // column half: [64h, 64h+64) of each block
        const int q = warp & 3;                  // TMEM lanes [32q, 32q+32) = tile rows
        const int r = q * 32 + lane;
        const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + h * 64;
        RingPos ra;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ra.advance(1)) {
            int e, row0, rows, nb;
            decode_tile<128>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            if (!__all_sync(0xffffffffu,
                            mbar_wait(tfull_bar, ra.phase, abort_flag, args.ctl, SITE_TFULL)))
                break;
            tc_fence_after();
            uint32_t p0[32], p1[32];       // bf16 pairs of block 0 / block 1 columns
#pragma unroll
            for (int c = 0; c < 64; c += 16) {
                float v[16], u[16];
                tmem_ld16(tb + c, v);
                tmem_ld16(tb + 128 + c, u);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const __nv_bfloat162 b0 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                    const __nv_bfloat162 b1 = __floats2bfloat162_rn(u[2 * j], u[2 * j + 1]);
                    p0[(c >> 1) + j] = *reinterpret_cast<const uint32_t*>(&b0);
                    p1[(c >> 1) + j] = *reinterpret_cast<const uint32_t*>(&b1);
                }
            }
            tc_fence_before();
            mbar_arrive(tempty_bar);
            const bool live = r < rows;
            int orow = row0 + r;
            if (live && args.out_rows) {
                orow = __ldg(args.out_rows + row0 + r);
                if (orow < 0 || orow >= args.out_total) orow = -1;
            }
            if (live && orow >= 0) {
                __nv_bfloat16* o = out_row_ptr(args, orow, N);
                uint4* d0 = reinterpret_cast<uint4*>(o + nb * 256 + h * 64);
                uint4* d1 = reinterpret_cast<uint4*>(o + nb * 256 + 128 + h * 64);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    d0[c] = make_uint4(p0[4 * c], p0[4 * c + 1], p0[4 * c + 2], p0[4 * c + 3]);
                    d1[c] = make_uint4(p1[4 * c], p1[4 * c + 1], p1[4 * c + 2], p1[4 * c + 3]);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}

int launch_fp8_prefill_mx(const DeviceInfo* info, const void* a, const float* a_scale,
                          const void* w, const float* w_scale, void* out, const int32_t* seg,
                          int seg_pairs, int M, int N, int K, int E, cudaStream_t stream,
                          const OutMap& om) {
    CUtensorMap tm_w, tm_a;
    int rc = make_tmap_2d(&tm_w, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)E * N, K, K, 128,
                          128, true);
    if (rc != FERRET_OK) return rc;
    rc = make_tmap_2d(&tm_a, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, K, 128, 128, true);
    if (rc != FERRET_OK) return rc;
    const int budget = info->max_smem_optin - 1024;
    const int stages = std::min(kPfMaxStages, (budget - mx_layout(0, E).total) / kPfStage);
    if (stages < 2) return FERRET_ERR_SHAPE;
    const int smem = mx_layout(stages, E).total + 1024;
    auto kern = fp8_w13_prefill_mx_kernel<false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    GemmArgs g;
    g.a_scale = a_scale;
    g.w_scale = w_scale;
    g.seg = seg;
    g.seg_pairs = seg_pairs;
    g.out = static_cast<__nv_bfloat16*>(out);
    g.out_rows = om.rows;
    g.out_total = om.total;
    g.out_peers = nullptr;
    g.peer_rows = 0;
    g.M = M;
    g.N = N;
    g.K = K;
    g.E = E;
    g.stages = stages;
    g.ctl = make_ctl(info);
    return launch_kernel(kern, dim3(info->num_sms), dim3(kMxThreads), smem, stream, tm_w, tm_a, g);
}

// ---------------------------------------------------------------------------
// CTA-pair form of the prefill kernel (FERRET_PREFILL_PAIRS) for each expert's
// whole 256-row chunks; the rows past them go to fp8_w13_prefill_kernel<.., true>.
//
// A pair (thread-block cluster of 2) computes a 256-token x 256-weight-row
// tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32): CTA r holds
// token rows [128r, 128r+128) of the tile and weight rows [128r, 128r+128)
// (gate block for r = 0 and up block for r = 1 with SiLU), and receives the
// 128 x 256 partial of its own token rows in its own Tensor Memory.  Per SM
// that is 32 KB of operands per K block instead of 48 KB for the same MMA
// work, so the L2->SM stream shrinks by a third and 6 stages fit.
//
// Protocol (every load is a plain TMA load into the issuing CTA's own shared memory):
//   * both CTAs load their halves with .cta_group::2 TMA, completing on the
//     leader's (rank 0) full barrier, which the leader arms with both halves'
//     bytes;
//   * the leader's single MMA thread waits for it, issues the pair MMAs and
//     commits to each CTA's empty barrier (stage free) and tfull barrier
//     (K-block partial ready);
//   * each CTA's 8 epilogue warps promote their own partial exactly as the
//     single-CTA kernel does and release the buffer with one arrive per warp
//     on the leader's tempty barrier (16 arrivals);
//   * a cluster barrier after the roles finish keeps either CTA from leaving
//     while the other still reads its shared memory or Tensor Memory.
//
// Measured on B200 (benchmark configuration 3, GEMM alone): 4.311 ms for this
// kernel plus the single-CTA remainder launch, against 2.708 ms for the
// single-CTA kernel alone.  With exact fp32 scales every K block's partial has
// to be promoted by both CTAs before the leader can reuse one of the two TMEM
// buffers, which puts a cross-SM round trip (tfull to the peer, the peer's
// promotion, its arrive back on the leader) on every K block.  Hence opt-in;
// the pair protocol itself is the base for the block-scaled pair tile, whose
// single accumulator needs one such handshake per tile.
// ---------------------------------------------------------------------------
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

template <bool PAIR>
__global__ void __launch_bounds__(kPfThreads, 1)
    fp8_w13_prefill_pair_kernel(const __grid_constant__ CUtensorMap tm_w,
                                const __grid_constant__ CUtensorMap tm_a, const GemmArgs args) {
    pdl_begin();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = args.M, N = args.N, K = args.K, E = args.E, NS = args.stages;
    const int nk = K >> 7;
    const int nbc = N >> 8;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const PpLayout L = pp_layout(NS, E);
    int* seg_s = reinterpret_cast<int*>(smem + L.segs_off);
    int* seg_c = reinterpret_cast<int*>(smem + L.segc_off);
    int* mt_start = reinterpret_cast<int*>(smem + L.mts_off);
    int* part = reinterpret_cast<int*>(smem + L.part_off);
    const uint32_t bar0 = smem_addr(smem + L.bar_off);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kPpMaxStages + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kPpMaxStages + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kPpMaxStages + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kPpMaxStages + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    const uint32_t stage_base = smem_addr(smem + L.stages_off);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 1);            // the leader's arm; bytes from both CTAs
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 2 * (kPfEpi / 32));   // one per epilogue warp of both CTAs
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_addr(tmem_slot), 512);
        tmem_relinquish_pair();
    }
    bool seg_bad = false;
    for (int e = tid; e < E; e += kPfThreads) {
        int s, c;
        if (args.seg_pairs) {
            s = args.seg[2 * e];
            c = args.seg[2 * e + 1];
        } else {
            s = args.seg[e];
            c = args.seg[e + 1] - s;
        }
        if (s < 0 || s > M || c < 0 || c > M - s) {
            seg_bad = true;
            s = min(max(s, 0), M);
            c = min(max(c, 0), M - s);
        }
        seg_s[e] = s;
        seg_c[e] = c & ~255;                      // whole 256-row chunks only
        mt_start[e] = c >> 8;
    }
    if (seg_bad && leader) report(args.ctl, DEV_LAYOUT);
    __syncthreads();
    block_exclusive_scan(mt_start, E, part);
    tc_fence_before();
    __syncthreads();
    cluster_sync();                               // both CTAs' barriers are initialised
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = mt_start[E] * nbc;

    if (warp == 0) {
        // ================= TMA producer (both CTAs) =================
        if (elect_one()) {
            tma_prefetch_desc(&tm_w);
            tma_prefetch_desc(&tm_a);
            const uint64_t pol = policy_evict_last();
            int it = 0;
            RingPos rp;
            bool ok = true;
            for (int t = pair; t < total && ok; t += npairs) {
                int e, row0, rows, nb;
                decode_tile<256>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
                const int arow = row0 + 128 * (int)rank;
                const int wrow = PAIR ? e * N + (rank ? (N >> 1) : 0) + nb * 128
                                      : e * N + nb * 256 + 128 * (int)rank;
                for (int kb = 0; kb < nk; ++kb, ++it, rp.advance(NS)) {
                    const int s = rp.slot;
                    if (!mbar_wait_cl(empty_bar(s), rp.phase ^ 1u, abort_flag, args.ctl,
                                      SITE_PEER_EMPTY)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_expect_tx(full_bar(s), 2 * kPpStage);
                    const uint32_t dst = stage_base + s * kPpStage;
                    const uint32_t bar = mapa_shared(full_bar(s), 0);
                    tma_load_2d_pair(dst, &tm_a, kb * 128, arow, bar, pol);
                    tma_load_2d_pair(dst + 16384, &tm_w, kb * 128, wrow, bar, pol);
                }
            }
            // the last stages are free again once the leader's MMAs consumed
            // them, which also means this CTA's loads into them have landed
            for (int i = max(0, it - NS); i < it; ++i)
                if (!mbar_wait_cl(empty_bar(i % NS), (i / NS) & 1, abort_flag, args.ctl,
                                  SITE_PEER_TAIL, false))
                    break;
        }
    } else if (warp == 1) {
        // ================= MMA issuer (leader CTA) =================
        if (leader && elect_one()) {
            constexpr uint32_t idesc = make_idesc(256, 256, 0, 0);
            RingPos rs, ra;
            bool ok = true;
            for (int t = pair; t < total && ok; t += npairs) {
                for (int kb = 0; kb < nk; ++kb, rs.advance(NS), ra.advance(2)) {
                    const int s = rs.slot, a = ra.slot;
                    if (!mbar_wait_cl(tempty_bar(a), ra.phase ^ 1u, abort_flag, args.ctl,
                                      SITE_TEMPTY) ||
                        !mbar_wait_cl(full_bar(s), rs.phase, abort_flag, args.ctl, SITE_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = stage_base + s * kPpStage;
                    const uint32_t d = tmem_base + a * 256;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f8f6f4_pair(d, sdesc_k_sw128(st + ks * 32),
                                        sdesc_k_sw128(st + 16384 + ks * 32), idesc, ks > 0);
                    tc_commit_pair(empty_bar(s));
                    tc_commit_pair(mapa_shared(empty_bar(s), 1));
                    tc_commit_pair(tfull_bar(a));
                    tc_commit_pair(mapa_shared(tfull_bar(a), 1));
                }
            }
            tc_commit_pair(drain_bar);
            mbar_wait(drain_bar, 0, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else {
        // ================= epilogue: promotion + store (both CTAs) =================
        const int h = (warp - 2) >> 2;           // column half: [64h, 64h+64) of each block
        const int q = warp & 3;                  // TMEM lanes [32q, 32q+32) = this CTA's rows
        const int r = q * 32 + lane;
        const int ldo = PAIR ? (N >> 1) : N;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        RingPos ra;
        for (int t = pair; t < total; t += npairs) {
            int e, row0, rows, nb;
            decode_tile<256>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            const int my0 = row0 + 128 * (int)rank;
            const bool live = 128 * (int)rank + r < rows;
            const float* as_row = args.a_scale + (size_t)(my0 + (live ? r : 0)) * nk;
            const int blk0 = PAIR ? nb : 2 * nb;
            const int blk1 = PAIR ? (N >> 8) + nb : 2 * nb + 1;
            const float* ws0 = args.w_scale + ((size_t)e * (N >> 7) + blk0) * nk;
            const float* ws1 = args.w_scale + ((size_t)e * (N >> 7) + blk1) * nk;
            float acc0[64], acc1[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                acc0[j] = 0.0f;
                acc1[j] = 0.0f;
            }
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb, ra.advance(2)) {
                const float sa = live ? __ldg(as_row + kb) : 0.0f;
                const float s0 = sa * __ldg(ws0 + kb), s1 = sa * __ldg(ws1 + kb);
                ok = __all_sync(0xffffffffu, mbar_wait_cl(tfull_bar(ra.slot), ra.phase, abort_flag,
                                                          args.ctl, SITE_TFULL));
                if (!ok) break;
                tc_fence_after();
                const uint32_t tb = tmem_base + lane_addr + ra.slot * 256 + h * 64;
#pragma unroll
                for (int c = 0; c < 64; c += 16) {
                    float v[16], u[16];
                    tmem_ld16(tb + c, v);
                    tmem_ld16(tb + 128 + c, u);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        acc0[c + j] = fmaf(v[j], s0, acc0[c + j]);
                        acc1[c + j] = fmaf(u[j], s1, acc1[c + j]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar(ra.slot), 0));
            }
            if (!ok) break;
            int orow = my0 + r;
            if (live && args.out_rows) {
                orow = __ldg(args.out_rows + my0 + r);
                if (orow < 0 || orow >= args.out_total) orow = -1;
            }
            if (live && orow >= 0) {
                __nv_bfloat16* o = args.out + (size_t)orow * ldo;
                if (PAIR) {
                    uint4* dst = reinterpret_cast<uint4*>(o + nb * 128 + h * 64);
#pragma unroll
                    for (int c = 0; c < 64; c += 8) {
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
                    uint4* d0 = reinterpret_cast<uint4*>(o + nb * 256 + h * 64);
                    uint4* d1 = reinterpret_cast<uint4*>(o + nb * 256 + 128 + h * 64);
#pragma unroll
                    for (int c = 0; c < 64; c += 8) {
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
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();                               // the pair's MMAs and arrivals are done
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

template <bool PAIR>
int launch_fp8_prefill_pairs(const DeviceInfo* info, const void* a, const float* a_scale,
                             const void* w, const float* w_scale, void* out, const int32_t* seg,
                             int seg_pairs, int M, int N, int K, int E, cudaStream_t stream,
                             const OutMap& om) {
    CUtensorMap tm_w, tm_a;
    int rc = make_tmap_2d(&tm_w, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)E * N, K, K, 128,
                          128, true);
    if (rc != FERRET_OK) return rc;
    rc = make_tmap_2d(&tm_a, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, K, 128, 128, true);
    if (rc != FERRET_OK) return rc;
    const int budget = info->max_smem_optin - 1024;
    const int stages = std::min(kPpMaxStages, (budget - pp_layout(0, E).total) / kPpStage);
    if (stages < 2) return FERRET_ERR_SHAPE;
    const int smem = pp_layout(stages, E).total + 1024;
    auto kern = fp8_w13_prefill_pair_kernel<PAIR>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    const int pairs = std::min(max_resident_pairs(kern, dim3(kPfThreads), smem), info->num_sms / 2);
    if (pairs < 1) return FERRET_ERR_UNSUPPORTED;
    GemmArgs g;
    g.a_scale = a_scale;
    g.w_scale = w_scale;
    g.seg = seg;
    g.seg_pairs = seg_pairs;
    g.out = static_cast<__nv_bfloat16*>(out);
    g.out_rows = om.rows;
    g.out_total = om.total;
    g.out_peers = nullptr;
    g.peer_rows = 0;
    g.M = M;
    g.N = N;
    g.K = K;
    g.E = E;
    g.stages = stages;
    g.ctl = make_ctl(info);
    rc = launch_kernel_pairs(kern, dim3(2 * pairs), dim3(kPfThreads), smem, stream, tm_w, tm_a, g);
    if (rc != FERRET_OK) return rc;
    // the rows past each expert's whole 256-row chunks
    const int stages1 = std::min(kPfMaxStages, (budget - pf_layout(0, E, false).total) / kPfStage);
    if (stages1 < 2) return FERRET_ERR_SHAPE;
    const int smem1 = pf_layout(stages1, E, false).total + 1024;
    auto kern1 = fp8_w13_prefill_kernel<PAIR, true>;
    if (cudaFuncSetAttribute(kern1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1) !=
        cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    g.stages = stages1;
    return launch_kernel(kern1, dim3(info->num_sms), dim3(kPfThreads), smem1, stream, tm_w, tm_a, g);
}

// ---------------------------------------------------------------------------
// Block-scaled CTA-pair kernel (FERRET_UE8M0_SCALES | FERRET_PREFILL_PAIRS,
// plain outputs): the pair protocol above with the UE8M0 kernel's roles.
// tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale M = 256, N = 256: each
// CTA's tensor core reads the scales from its own Tensor Memory, laid out as
// in the single-CTA block-scaled kernel -- A's for its own 128 token rows (4
// columns) and B's for all 256 weight rows of the tile (8 columns), since
// each CTA's accumulator spans the whole N.  Each CTA's 4 scale writers fill
// its own slot and arrive on the leader's sfull barrier (8 arrivals); the
// leader's MMA commits each slot free to both CTAs.  One 256-column
// accumulator per CTA, handed over once per tile.  The rows past each
// expert's whole 256-row chunks run on fp8_w13_prefill_mx_kernel<true>.
//
// Measured on B200 (benchmark configuration 3, GEMM alone): 3.448 ms with the
// remainder launch against 2.664 ms for the single-CTA block-scaled kernel;
// all 148 SMs hold a CTA (74 resident pairs), so the per-FLOP cost of the
// pair tile itself is what remains to be profiled.  Hence opt-in.
// ---------------------------------------------------------------------------
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

__global__ void __launch_bounds__(kMxThreads, 1)
    fp8_w13_prefill_mx_pair_kernel(const __grid_constant__ CUtensorMap tm_w,
                                   const __grid_constant__ CUtensorMap tm_a, const GemmArgs args) {
    pdl_begin();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = args.M, N = args.N, K = args.K, E = args.E, NS = args.stages;
    const int nk = K >> 7;
    const int nbc = N >> 8;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const MxpLayout L = mxp_layout(NS, E);
    int* seg_s = reinterpret_cast<int*>(smem + L.segs_off);
    int* seg_c = reinterpret_cast<int*>(smem + L.segc_off);
    int* mt_start = reinterpret_cast<int*>(smem + L.mts_off);
    int* part = reinterpret_cast<int*>(smem + L.part_off);
    const uint32_t bar0 = smem_addr(smem + L.bar_off);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kPpMaxStages + s); };
    const uint32_t tfull_bar = bar0 + 8u * (2 * kPpMaxStages);
    const uint32_t tempty_bar = tfull_bar + 8u;
    auto sfull_bar = [&](int j) { return bar0 + 8u * (2 * kPpMaxStages + 2 + j); };
    auto sempty_bar = [&](int j) { return bar0 + 8u * (2 * kPpMaxStages + 2 + kMxSfSlots + j); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kPpMaxStages + 2 + 2 * kMxSfSlots);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    const uint32_t stage_base = smem_addr(smem + L.stages_off);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(tfull_bar, 1);
        mbar_init(tempty_bar, 2 * (kMxEpi / 32));          // epilogue warps of both CTAs
        for (int j = 0; j < kMxSfSlots; ++j) {
            mbar_init(sfull_bar(j), 2 * 4);                // scale-writer warps of both CTAs
            mbar_init(sempty_bar(j), 1);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_addr(tmem_slot), 512);
        tmem_relinquish_pair();
    }
    bool seg_bad = false;
    for (int e = tid; e < E; e += kMxThreads) {
        int s, c;
        if (args.seg_pairs) {
            s = args.seg[2 * e];
            c = args.seg[2 * e + 1];
        } else {
            s = args.seg[e];
            c = args.seg[e + 1] - s;
        }
        if (s < 0 || s > M || c < 0 || c > M - s) {
            seg_bad = true;
            s = min(max(s, 0), M);
            c = min(max(c, 0), M - s);
        }
        seg_s[e] = s;
        seg_c[e] = c & ~255;                      // whole 256-row chunks only
        mt_start[e] = c >> 8;
    }
    if (seg_bad && leader) report(args.ctl, DEV_LAYOUT);
    __syncthreads();
    block_exclusive_scan(mt_start, E, part);
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = mt_start[E] * nbc;

    if (warp == 0) {
        // ================= TMA producer (both CTAs) =================
        if (elect_one()) {
            tma_prefetch_desc(&tm_w);
            tma_prefetch_desc(&tm_a);
            const uint64_t pol = policy_evict_last();
            int it = 0;
            RingPos rp;
            bool ok = true;
            for (int t = pair; t < total && ok; t += npairs) {
                int e, row0, rows, nb;
                decode_tile<256>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
                const int arow = row0 + 128 * (int)rank;
                const int wrow = e * N + nb * 256 + 128 * (int)rank;
                for (int kb = 0; kb < nk; ++kb, ++it, rp.advance(NS)) {
                    const int s = rp.slot;
                    if (!mbar_wait_cl(empty_bar(s), rp.phase ^ 1u, abort_flag, args.ctl,
                                      SITE_PEER_EMPTY)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_expect_tx(full_bar(s), 2 * kPpStage);
                    const uint32_t dst = stage_base + s * kPpStage;
                    const uint32_t bar = mapa_shared(full_bar(s), 0);
                    tma_load_2d_pair(dst, &tm_a, kb * 128, arow, bar, pol);
                    tma_load_2d_pair(dst + 16384, &tm_w, kb * 128, wrow, bar, pol);
                }
            }
            for (int i = max(0, it - NS); i < it; ++i)
                if (!mbar_wait_cl(empty_bar(i % NS), (i / NS) & 1, abort_flag, args.ctl,
                                  SITE_PEER_TAIL, false))
                    break;
        }
    } else if (warp == 1) {
        // ================= MMA issuer (leader CTA) =================
        if (leader && elect_one()) {
            constexpr uint32_t idesc = make_idesc_mx(256, 256);
            RingPos rs, rf, ra;
            bool ok = true;
            for (int t = pair; t < total && ok; t += npairs, ra.advance(1)) {
                if (!mbar_wait_cl(tempty_bar, ra.phase ^ 1u, abort_flag, args.ctl, SITE_TEMPTY)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < nk; ++kb, rs.advance(NS), rf.advance(kMxSfSlots)) {
                    const int s = rs.slot, f = rf.slot;
                    if (!mbar_wait_cl(sfull_bar(f), rf.phase, abort_flag, args.ctl, SITE_SFULL) ||
                        !mbar_wait_cl(full_bar(s), rs.phase, abort_flag, args.ctl, SITE_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = stage_base + s * kPpStage;
                    const uint32_t sfa = tmem_base + kMxSfCol0 + f * kMxSfCols;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        mma_mxf8f6f4_pair(tmem_base, sdesc_k_sw128(st + ks * 32),
                                          sdesc_k_sw128(st + 16384 + ks * 32), idesc, sfa, sfa + 8,
                                          (kb | ks) != 0);
                    tc_commit_pair(empty_bar(s));
                    tc_commit_pair(mapa_shared(empty_bar(s), 1));
                    tc_commit_pair(sempty_bar(f));
                    tc_commit_pair(mapa_shared(sempty_bar(f), 1));
                }
                if (ok) {
                    tc_commit_pair(tfull_bar);
                    tc_commit_pair(mapa_shared(tfull_bar, 1));
                }
            }
            tc_commit_pair(drain_bar);
            mbar_wait(drain_bar, 0, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    } else if (warp < 6) {
        // ================= scale writers (both CTAs, own Tensor Memory) =================
        const int q = warp & 3;
        const uint32_t sf_lane = tmem_base + ((uint32_t)(q * 32) << 16) + kMxSfCol0;
        const int nsb = N >> 7;
        auto load = [&](int t, int kb0, float (&a)[4][4], float (&w)[2][4]) {
            int e, row0, rows, nb;
            decode_tile<256>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            const int my0 = row0 + 128 * (int)rank;
            const int my_rows = min(max(rows - 128 * (int)rank, 0), 128);
            const float* ws0 = args.w_scale + ((size_t)e * nsb + 2 * nb) * nk;
            const float* ws1 = ws0 + nk;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kb = min(kb0 + j, nk - 1);
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const int r = 32 * m + lane;
                    a[m][j] = r < my_rows ? __ldg(args.a_scale + (size_t)(my0 + r) * nk + kb) : 1.0f;
                }
                w[0][j] = __ldg(ws0 + kb);
                w[1][j] = __ldg(ws1 + kb);
            }
        };
        const uint32_t sfull_leader0 = mapa_shared(sfull_bar(0), 0);
        RingPos rf;
        int t = pair, kb0 = 0;
        float a[4][4], w[2][4];
        if (t < total) load(t, 0, a, w);
        bool ok = true;
        while (t < total && ok) {
            int tn = t, kn = kb0 + 4;
            if (kn >= nk) {
                tn = t + npairs;
                kn = 0;
            }
            float an[4][4], wn[2][4];
            if (tn < total) load(tn, kn, an, wn);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (kb0 + j >= nk) break;
                ok = __all_sync(0xffffffffu, mbar_wait_cl(sempty_bar(rf.slot), rf.phase ^ 1u,
                                                          abort_flag, args.ctl, SITE_SEMPTY));
                if (!ok) break;
                tc_fence_after();
                const uint32_t col = sf_lane + rf.slot * kMxSfCols;
                tmem_st4(col, ue8m0_word(a[0][j]), ue8m0_word(a[1][j]), ue8m0_word(a[2][j]),
                         ue8m0_word(a[3][j]));
                const uint32_t b0 = ue8m0_word(w[0][j]), b1 = ue8m0_word(w[1][j]);
                const uint32_t bw[8] = {b0, b0, b0, b0, b1, b1, b1, b1};
                tmem_st8(col + 8, bw);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(sfull_leader0 + 8u * rf.slot);
                rf.advance(kMxSfSlots);
            }
            t = tn;
            kb0 = kn;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int m = 0; m < 4; ++m) a[m][j] = an[m][j];
                w[0][j] = wn[0][j];
                w[1][j] = wn[1][j];
            }
        }
    } else {
        // ================= epilogue (both CTAs, own rows) =================
        const int h = (warp - 6) >> 2;
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + h * 64;
        const uint32_t tempty_leader = mapa_shared(tempty_bar, 0);
        RingPos ra;
        for (int t = pair; t < total; t += npairs, ra.advance(1)) {
            int e, row0, rows, nb;
            decode_tile<256>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            if (!__all_sync(0xffffffffu,
                            mbar_wait_cl(tfull_bar, ra.phase, abort_flag, args.ctl, SITE_TFULL)))
                break;
            tc_fence_after();
            uint32_t p0[32], p1[32];
#pragma unroll
            for (int c = 0; c < 64; c += 16) {
                float v[16], u[16];
                tmem_ld16(tb + c, v);
                tmem_ld16(tb + 128 + c, u);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const __nv_bfloat162 b0 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                    const __nv_bfloat162 b1 = __floats2bfloat162_rn(u[2 * j], u[2 * j + 1]);
                    p0[(c >> 1) + j] = *reinterpret_cast<const uint32_t*>(&b0);
                    p1[(c >> 1) + j] = *reinterpret_cast<const uint32_t*>(&b1);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader);
            const int my0 = row0 + 128 * (int)rank;
            const bool live = 128 * (int)rank + r < rows;
            int orow = my0 + r;
            if (live && args.out_rows) {
                orow = __ldg(args.out_rows + my0 + r);
                if (orow < 0 || orow >= args.out_total) orow = -1;
            }
            if (live && orow >= 0) {
                __nv_bfloat16* o = args.out + (size_t)orow * N;
                uint4* d0 = reinterpret_cast<uint4*>(o + nb * 256 + h * 64);
                uint4* d1 = reinterpret_cast<uint4*>(o + nb * 256 + 128 + h * 64);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    d0[c] = make_uint4(p0[4 * c], p0[4 * c + 1], p0[4 * c + 2], p0[4 * c + 3]);
                    d1[c] = make_uint4(p1[4 * c], p1[4 * c + 1], p1[4 * c + 2], p1[4 * c + 3]);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

int launch_fp8_prefill_mx_pairs(const DeviceInfo* info, const void* a, const float* a_scale,
                                const void* w, const float* w_scale, void* out, const int32_t* seg,
                                int seg_pairs, int M, int N, int K, int E, cudaStream_t stream,
                                const OutMap& om) {
    CUtensorMap tm_w, tm_a;
    int rc = make_tmap_2d(&tm_w, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)E * N, K, K, 128,
                          128, true);
    if (rc != FERRET_OK) return rc;
    rc = make_tmap_2d(&tm_a, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, K, 128, 128, true);
    if (rc != FERRET_OK) return rc;
    const int budget = info->max_smem_optin - 1024;
    const int stages = std::min(kPpMaxStages, (budget - mxp_layout(0, E).total) / kPpStage);
    if (stages < 2) return FERRET_ERR_SHAPE;
    const int smem = mxp_layout(stages, E).total + 1024;
    auto kern = fp8_w13_prefill_mx_pair_kernel;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    const int pairs = std::min(max_resident_pairs(kern, dim3(kMxThreads), smem), info->num_sms / 2);
    if (pairs < 1) return FERRET_ERR_UNSUPPORTED;
    GemmArgs g;
    g.a_scale = a_scale;
    g.w_scale = w_scale;
    g.seg = seg;
    g.seg_pairs = seg_pairs;
    g.out = static_cast<__nv_bfloat16*>(out);
    g.out_rows = om.rows;
    g.out_total = om.total;
    g.out_peers = nullptr;
    g.peer_rows = 0;
    g.M = M;
    g.N = N;
    g.K = K;
    g.E = E;
    g.stages = stages;
    g.ctl = make_ctl(info);
    rc = launch_kernel_pairs(kern, dim3(2 * pairs), dim3(kMxThreads), smem, stream, tm_w, tm_a, g);
    if (rc != FERRET_OK) return rc;
    // the rows past each expert's whole 256-row chunks
    const int stages1 = std::min(kPfMaxStages, (budget - mx_layout(0, E).total) / kPfStage);
    if (stages1 < 2) return FERRET_ERR_SHAPE;
    const int smem1 = mx_layout(stages1, E).total + 1024;
    auto kern1 = fp8_w13_prefill_mx_kernel<true>;
    if (cudaFuncSetAttribute(kern1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1) !=
        cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    g.stages = stages1;
    return launch_kernel(kern1, dim3(info->num_sms), dim3(kMxThreads), smem1, stream, tm_w, tm_a, g);
}

template <bool PAIR, bool STAGED>
int launch_fp8_prefill_t(const DeviceInfo* info, const void* a, const float* a_scale, const void* w,
                       const float* w_scale, void* out, const int32_t* seg, int seg_pairs, int M,
                       int N, int K, int E, cudaStream_t stream, const OutMap& om = OutMap{}) {
    CUtensorMap tm_w, tm_a;
    int rc = make_tmap_2d(&tm_w, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)E * N, K, K, 128,
                          128, true);
    if (rc != FERRET_OK) return rc;
    rc = make_tmap_2d(&tm_a, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, K, 128, 128, true);
    if (rc != FERRET_OK) return rc;
    const int budget = info->max_smem_optin - 1024;
    const int stages = std::min(kPfMaxStages, (budget - pf_layout(0, E, STAGED).total) / kPfStage);
    if (stages < 2) return FERRET_ERR_SHAPE;
    const int smem = pf_layout(stages, E, STAGED).total + 1024;
    auto kern = STAGED ? fp8_w13_prefill_peer_kernel<PAIR> : fp8_w13_prefill_kernel<PAIR>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    GemmArgs g;
    g.a_scale = a_scale;
    g.w_scale = w_scale;
    g.seg = seg;
    g.seg_pairs = seg_pairs;
    g.out = static_cast<__nv_bfloat16*>(out);
    g.out_rows = om.rows;
    g.out_total = om.total;
    g.out_peers = om.peers;
    g.peer_rows = om.peer_rows;
    g.M = M;
    g.N = N;
    g.K = K;
    g.E = E;
    g.stages = stages;
    g.ctl = make_ctl(info);
    return launch_kernel(kern, dim3(info->num_sms), dim3(kPfThreads), smem, stream, tm_w, tm_a, g);
}

template <bool PAIR>
int launch_fp8_prefill(const DeviceInfo* info, const void* a, const float* a_scale, const void* w,
                       const float* w_scale, void* out, const int32_t* seg, int seg_pairs, int M,
                       int N, int K, int E, cudaStream_t stream, const OutMap& om = OutMap{}) {
    return om.peers ? launch_fp8_prefill_t<PAIR, true>(info, a, a_scale, w, w_scale, out, seg,
                                                       seg_pairs, M, N, K, E, stream, om)
                    : launch_fp8_prefill_t<PAIR, false>(info, a, a_scale, w, w_scale, out, seg,
                                                        seg_pairs, M, N, K, E, stream, om);
}

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

// 128-token tiles (requested, or experts averaging more than 48 rows) run on
// the prefill kernel when the weight tiles (256 rows) divide N.
bool use_prefill(int M, int E, int flags, int N) {
    int nt = (flags >> FERRET_TILE_SHIFT) & 0xFF;
    if (nt == 0) nt = ((M + E - 1) / std::max(E, 1)) > 48 ? 128 : 0;
    return nt == 128 && N % 256 == 0;
}

}  // namespace

int run_fp8_gemm(const DeviceInfo* info, const void* a, const float* a_scale, const void* w,
                 const float* w_scale, void* out, const int32_t* seg, int seg_pairs, int M, int N,
                 int K, int E, int flags, int rows_hint, cudaStream_t s, const OutMap& om,
                 const SplitWs& sw) {
    const bool pair = (flags & FERRET_SILU_MUL) != 0;
    // power-of-two scales: the block-scaled kernel for plain 128-token tiles
    // (with SiLU the exact-scale kernel is faster and exact for such scales)
    if (use_prefill(rows_hint, E, flags, N) && (flags & FERRET_UE8M0_SCALES) && !pair && !om.peers)
        return (flags & FERRET_PREFILL_PAIRS)
                   ? launch_fp8_prefill_mx_pairs(info, a, a_scale, w, w_scale, out, seg, seg_pairs,
                                                 M, N, K, E, s, om)
                   : launch_fp8_prefill_mx(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M, N,
                                           K, E, s, om);
    // CTA pairs for whole 256-row expert chunks, single CTAs for the rest
    if (use_prefill(rows_hint, E, flags, N) && (flags & FERRET_PREFILL_PAIRS) && !om.peers)
        return pair ? launch_fp8_prefill_pairs<true>(info, a, a_scale, w, w_scale, out, seg,
                                                     seg_pairs, M, N, K, E, s, om)
                    : launch_fp8_prefill_pairs<false>(info, a, a_scale, w, w_scale, out, seg,
                                                      seg_pairs, M, N, K, E, s, om);
    if (use_prefill(rows_hint, E, flags, N))
        return pair ? launch_fp8_prefill<true>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M,
                                               N, K, E, s, om)
                    : launch_fp8_prefill<false>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M,
                                                N, K, E, s, om);
#define FERRET_FP8_CASE(NT_)                                                                    \
    case NT_:                                                                                   \
        return pair ? launch_fp8<NT_, true>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M, \
                                            N, K, E, s, om, sw)                                 \
                    : launch_fp8<NT_, false>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M,\
                                             N, K, E, s, om, sw);
    switch (pick_tile(rows_hint, E, K, flags, pair)) {
        FERRET_FP8_CASE(16)
        FERRET_FP8_CASE(32)
        FERRET_FP8_CASE(64)
        case 128:
            return launch_fp8<128, false>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M, N,
                                          K, E, s, om, sw);
        default:
            return FERRET_ERR_SHAPE;
    }
#undef FERRET_FP8_CASE
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
        const int smem = 3 * E * (int)sizeof(int);
        if ((rc = launch_kernel(derive_segments_kernel, dim3(1), dim3(kSegThreads), smem, s,
                                m_indices, M, E, static_cast<int32_t*>(workspace), make_ctl(info),
                                sw.cnt, ncnt)) != FERRET_OK) return rc;
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
int g_noalloc_err[kNoAllocMaxDevices];
std::once_flag g_noalloc_once[kNoAllocMaxDevices];

// Runs once per device, with that device current: host code only ever sees a
// host-side stand-in for the array, so its device address must be queried.
void noalloc_setup(int dev) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_segments);
    if (e != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        g_noalloc_err[dev] = FERRET_ERR_CUDA;
        return;
    }
    g_noalloc_ptr[dev] = static_cast<int32_t*>(p);
    g_noalloc_err[dev] = FERRET_OK;
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
    std::call_once(g_noalloc_once[info->device], noalloc_setup, info->device);
    if (g_noalloc_err[info->device] != FERRET_OK) return g_noalloc_err[info->device];
    int32_t* seg = g_noalloc_ptr[info->device];
    cudaStream_t s = as_stream(stream);
    // every call rewrites all 2E (start, count) entries before the GEMM reads them
    if ((rc = launch_kernel(derive_segments_kernel, dim3(1), dim3(kSegThreads),
                            3 * E * (int)sizeof(int), s, m_indices, M, E, seg, make_ctl(info),
                            (int*)nullptr, 0)) != FERRET_OK) return rc;
    const int nt = pick_tile(M, E, K, flags, pair);
    switch (nt) {
        case 16:
            return pair ? launch_fp8<16, true>(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, seg, 1, M, N, K, E, s)
                        : launch_fp8<16, false>(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, seg, 1, M, N, K, E, s);
        case 32:
            return pair ? launch_fp8<32, true>(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, seg, 1, M, N, K, E, s)
                        : launch_fp8<32, false>(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, seg, 1, M, N, K, E, s);
        case 64:
            return pair ? launch_fp8<64, true>(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, seg, 1, M, N, K, E, s)
                        : launch_fp8<64, false>(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, seg, 1, M, N, K, E, s);
        case 128:
            return launch_fp8<128, false>(info, a_fp8, a_scale, w_fp8, w_scale, out_bf16, seg, 1, M, N, K, E, s);
        default:
            return FERRET_ERR_SHAPE;
    }
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
