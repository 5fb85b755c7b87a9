// int4_grouped_gemm.cu -- W4A16 (INT4 group-32 symmetric weights, bf16
// activations) grouped GEMM for the MoE W13 projection on sm_100a, the
// operation of vLLM's moe_wna16_marlin_gemm + apply_moe_activation(SILU) as
// the reference times it (baselines/kimi-moe-w13-int4/baseline_marlin.py:140-168).
//
//   w[e, n, k]   = bf16((nibble(e, k, n) - 8) * scale[e, k/32, n])
//   out[p, n]    = sum_k hidden[p / topk, k] * w[e(p), n, k]            (bf16)
//   SiLU variant = silu(out[p, j]) * out[p, N/2 + j]  for j < N/2
// with p the flat (token, slot) index; rows are written in that (token, slot)
// order, as Marlin writes them.
//
// Data path, designed so each 128-wide K block costs three copy operations (the
// per-SM copy engine, not HBM, limits a design that issues one small copy per
// activation row and separate scale boxes):
//   * load time (ferret_int4_repack_w13): every 128 (n) x 128 (k) weight block
//     and its 128 x 4 bf16 group scales become one contiguous 9 KB blob, nibbles
//     reordered so each (k, k+1) pair sits 16 bits apart, and word row k8's
//     entry for weight row n stored at n ^ 8 (k8 % 4) (which keeps this
//     kernel's per-row reads conflict-free and makes the decode kernel's
//     16-byte fragment reads so);
//   * per call, a gather pass writes the expert-sorted activation rows
//     contiguously (workspace), so one tensor-map box brings NT token rows of
//     a 64-wide K half in the 128-byte-swizzled layout;
//   * warp 0 (one thread): per K block, one bulk copy of the weight blob (two
//     with SiLU: gate and up) and two B-tile boxes into an NS-deep ring;
//   * warps 2-17 (dequant, four warpgroups taking 128x128 weight tiles in
//     turn): the thread of weight row n turns its 16 packed words (128 K
//     values) into 64 bf16x2 words and stores them with tcgen05.st into TMEM
//     lane n -- the dequantized A operand never touches shared memory, which
//     a decode-sized MMA (N = 8 tokens) would otherwise re-read per K step;
//   * warp 1 (MMA): tcgen05.mma.kind::f16 with A read from TMEM (bf16 x bf16
//     -> f32), M = 128 weight rows, N = NT token rows (swap-AB), K = 16,
//     accumulating the whole K range in one TMEM buffer per tile
//     (double-buffered across tiles);
//   * warps 18-21 (epilogue): TMEM -> registers -> optional SiLU*up -> bf16.
// A dequant warp leaves a tile's TMEM stores in flight while it dequantizes
// its next tile, and only then hands the slot to the MMA.  With fewer tiles
// than SMs (a handful of tokens) the K blocks are split over the SMs; fp32
// partials go to the workspace and the last unit of each tile reduces them
// in split order (deterministic).
// The dequant arithmetic is exact: nibble pairs become bf16 (128 + n) with one
// lop3 against the 0x4300 exponent, minus 136 gives n - 8 exactly, and one
// bf16x2 multiply by the scale rounds once -- the oracle's bf16((n-8)*s).
#include <algorithm>

#include "int4_common.cuh"

namespace ferret {
namespace {

constexpr int kDqWarp0 = 2, kDqWarps = 16;
constexpr int kEpiWarp0 = kDqWarp0 + kDqWarps, kI4EpiThreads = 128;
constexpr int kI4Threads = (kEpiWarp0 + 4) * 32;   // 22 warps
constexpr int kI4MaxE = 1024;
constexpr int kDqGroups = kDqWarps / 4;            // dequant warpgroups
constexpr int kI4MaxStages = 16, kI4MaxQ = 8, kI4MaxAcc = 4;
constexpr int kRawW = 128 * 16 * 4;    // packed words: 16 k8 rows x 128 n
constexpr int kRawS = 128 * 4 * 2;     // scales: 4 groups x 128 n bf16
constexpr int kBlob = kRawW + kRawS;   // 9216 B per 128 x 128 weight block
constexpr int kQCols = 64;             // TMEM columns of one dequantized 128x128 tile

enum : int { I4_EMPTY = 1, I4_FULL = 2, I4_QE = 3, I4_QF = 4, I4_TE = 5, I4_TF = 6, I4_DRAIN = 7,
             I4_EPI = 8 };

struct Int4Args {
    const uint8_t* blob;          // [E][N/128][K/128] x kBlob
    const int32_t* sorted_rows;   // flat (token, slot) of each expert-sorted row
    const int32_t* offsets;       // [E+1]
    __nv_bfloat16* out;
    int T, topk, N, K, E, R;
    int stages;
    // split-K (splits > 1): unit u = tile * splits + s covers K blocks
    // [s*nk/splits, (s+1)*nk/splits); fp32 partials go to part[u][col][128],
    // cnt[tile] counts finished units and the last one reduces in s order
    int splits;
    float* part;
    int* cnt;
    DevCtl ctl;
};

template <int NT, bool PAIR>
struct I4Cfg {
    static constexpr int kW = PAIR ? 2 : 1;
    static constexpr int kBTile = NT * 256;                     // NT rows x 128 k bf16
    static constexpr int kStage = kW * kBlob + kBTile;          // multiple of 1024
    static constexpr int kCols = NT * kW;                       // accumulator columns per tile
    static constexpr int kAcc = 2;
    static constexpr int kAccCols = kAcc * kCols;
    static constexpr int kQ0 = (512 - kAccCols) / kQCols;       // dequantized-tile slots
    static constexpr int kQ = kQ0 > kI4MaxQ ? kI4MaxQ : kQ0;
    static constexpr int kTmemCols = 512;
};

struct I4Layout {
    int raw_off, mts_off, part_off, bar_off, misc_off, total;
};

__host__ __device__ inline I4Layout i4_layout(int stage_bytes, int stages, int E) {
    I4Layout L;
    int o = 0;
    L.raw_off = o;                           // B tiles inside need 1024 alignment
    o += stage_bytes * stages;
    L.mts_off = o;
    o += 4 * (E + 1);
    L.part_off = o;
    o += 4 * (kI4Threads + 1);
    o = (o + 7) & ~7;
    L.bar_off = o;
    o += 8 * (2 * kI4MaxStages + 2 * kI4MaxQ + 2 * kI4MaxAcc + 2);
    L.misc_off = o;
    o += 16;
    L.total = o;
    return L;
}

template <int NT>
__device__ __forceinline__ void i4_decode_tile(int t, int nbc, int E, const int* mt_start,
                                               const int32_t* offs, int& e, int& row0, int& rows,
                                               int& nb) {
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
    row0 = __ldg(offs + e) + local;
    rows = min(NT, __ldg(offs + e + 1) - row0);
}

template <int NT, bool PAIR>
__global__ void __launch_bounds__(kI4Threads, 1)
    int4_w13_grouped_kernel(const __grid_constant__ CUtensorMap tm_a, const Int4Args args) {
    pdl_begin();
    using C = I4Cfg<NT, PAIR>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int N = args.N, K = args.K, E = args.E, NS = args.stages;
    constexpr int NQ = C::kQ;
    const int nk = K >> 7;
    const int nbc = PAIR ? (N >> 8) : (N >> 7);
    const I4Layout L = i4_layout(C::kStage, NS, E);
    int* mt_start = reinterpret_cast<int*>(smem + L.mts_off);
    int* part = reinterpret_cast<int*>(smem + L.part_off);
    const uint32_t bar0 = smem_addr(smem + L.bar_off);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kI4MaxStages + s); };
    auto qf_bar = [&](int q) { return bar0 + 8u * (2 * kI4MaxStages + q); };
    auto qe_bar = [&](int q) { return bar0 + 8u * (2 * kI4MaxStages + kI4MaxQ + q); };
    auto tf_bar = [&](int a) { return bar0 + 8u * (2 * kI4MaxStages + 2 * kI4MaxQ + a); };
    auto te_bar = [&](int a) { return bar0 + 8u * (2 * kI4MaxStages + 2 * kI4MaxQ + kI4MaxAcc + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kI4MaxStages + 2 * kI4MaxQ + 2 * kI4MaxAcc);
    const uint32_t epi_bar = drain_bar + 8u;      // epilogue rendezvous (split-K), bounded
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    uint8_t* raw = smem + L.raw_off;
    const uint32_t raw_base = smem_addr(raw);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int q = 0; q < NQ; ++q) {
            mbar_init(qf_bar(q), 4);             // one arrival per warp of a dequant group
            mbar_init(qe_bar(q), 1);
        }
        for (int a = 0; a < C::kAcc; ++a) {
            mbar_init(tf_bar(a), 1);
            mbar_init(te_bar(a), kI4EpiThreads);
        }
        mbar_init(drain_bar, 1);
        mbar_init(epi_bar, kI4EpiThreads);
        *abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    bool seg_bad = false;
    for (int e = tid; e < E; e += kI4Threads) {
        const int s = args.offsets[e], c = args.offsets[e + 1] - s;
        const bool bad = s < 0 || c < 0 || s + c > args.R;
        seg_bad |= bad;
        mt_start[e] = bad ? 0 : (c + NT - 1) / NT;
    }
    if (seg_bad) report(args.ctl, DEV_LAYOUT);
    __syncthreads();
    block_exclusive_scan(mt_start, E, part);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t q_base = tmem_base + C::kAccCols;          // dequantized-tile slots
    const int S = args.splits;
    const int total = mt_start[E] * nbc * S;                  // work units
    const size_t blob_nb = (size_t)(K >> 7) * kBlob;          // bytes per (e, n-block)

    if (warp == 0) {
        // ================= copy producer =================
        if (elect_one()) {
            tma_prefetch_desc(&tm_a);
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_a = policy_evict_last();
            int it = 0;
            RingPos rp;
            bool ok = true;
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                const int t = u / S, sp = u - t * S;
                int e, row0, rows, nb;
                i4_decode_tile<NT>(t, nbc, E, mt_start, args.offsets, e, row0, rows, nb);
                const uint8_t* wg = args.blob + ((size_t)e * (N >> 7) + nb) * blob_nb;
                const uint8_t* wu = args.blob + ((size_t)e * (N >> 7) + (N >> 8) + nb) * blob_nb;
                for (int kb = sp * nk / S; kb < (sp + 1) * nk / S; ++kb, ++it, rp.advance(NS)) {
                    const int s = rp.slot;
                    if (!mbar_wait(empty_bar(s), rp.phase ^ 1u, abort_flag, args.ctl, I4_EMPTY)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = raw_base + s * C::kStage;
                    mbar_expect_tx(full_bar(s), C::kStage);
                    bulk_load_hint(st, wg + (size_t)kb * kBlob, kBlob, full_bar(s), pol_w);
                    if (PAIR) bulk_load_hint(st + kBlob, wu + (size_t)kb * kBlob, kBlob, full_bar(s), pol_w);
                    tma_load_2d_hint(st + C::kW * kBlob, &tm_a, kb * 128, row0, full_bar(s), pol_a);
                    tma_load_2d_hint(st + C::kW * kBlob + NT * 128, &tm_a, kb * 128 + 64, row0,
                                     full_bar(s), pol_a);
                }
            }
            // drain: the last load issued into each stage may still be in flight
            for (int i = max(0, it - NS); i < it; ++i)
                mbar_wait(full_bar(i % NS), (i / NS) & 1, abort_flag, args.ctl, I4_DRAIN, false);
        }
    } else if (warp == 1) {
        // ================= MMA issuer =================
        if (elect_one()) {
            constexpr uint32_t idesc = make_idesc(128, NT, 1, 1);
            RingPos rs, rq, ra;
            bool ok = true;
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ra.advance(C::kAcc)) {
                const int sp = u % S;
                const int kb0 = sp * nk / S, kb1 = (sp + 1) * nk / S;
                const int a = ra.slot;
                if (!mbar_wait(te_bar(a), ra.phase ^ 1u, abort_flag, args.ctl, I4_TE)) break;
                const uint32_t d_acc = tmem_base + a * C::kCols;
                for (int kb = kb0; kb < kb1; ++kb, rs.advance(NS)) {
                    const int s = rs.slot;
                    RingPos qw[C::kW];
                    qw[0] = rq;
                    rq.advance(NQ);
                    if (PAIR) {
                        qw[C::kW - 1] = rq;
                        rq.advance(NQ);
                    }
                    // the B tile comes straight from the copy engine; the
                    // dequantized A tiles from the dequant warpgroups
                    bool ready = mbar_wait(full_bar(s), rs.phase, abort_flag, args.ctl, I4_FULL);
#pragma unroll
                    for (int w = 0; w < C::kW; ++w)
                        ready = ready && mbar_wait(qf_bar(qw[w].slot), qw[w].phase, abort_flag,
                                                   args.ctl, I4_QF);
                    if (!ready) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t bt = raw_base + s * C::kStage + C::kW * kBlob;
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint32_t acc = (kb > kb0 || ks) ? 1u : 0u;
                        const uint64_t bdesc =
                            sdesc_k_sw128(bt + (ks >> 2) * NT * 128 + (ks & 3) * 32);
#pragma unroll
                        for (int w = 0; w < C::kW; ++w)
                            mma_f16_tmem_a(d_acc + w * NT, q_base + qw[w].slot * kQCols + ks * 8, bdesc,
                                           idesc, acc);
                    }
                    tc_commit(empty_bar(s));
#pragma unroll
                    for (int w = 0; w < C::kW; ++w) tc_commit(qe_bar(qw[w].slot));
                }
                if (!ok) break;
                tc_commit(tf_bar(a));
            }
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_flag, args.ctl, I4_DRAIN, false);
        }
    } else if (warp < kEpiWarp0) {
        // ================= dequant =================
        // group g takes the weight tiles g, g+4, g+8, ... in issue order; the
        // thread of TMEM lane n (its warp's lane quarter) owns weight row n
        const int g = (warp - kDqWarp0) >> 2;
        const int n = ((warp & 3) << 5) + lane;
        const uint32_t lane_addr = (uint32_t)((warp & 3) << 5) << 16;
        RingPos rs, rq;
        int job = 0;
        bool ok = true;
        // Software pipeline: a job's TMEM stores are left in flight while the
        // next job's words are fetched and dequantized; only then does the
        // warp wait for them and hand the slot to the MMA (pend).
        int pend = -1;
        auto release_pending = [&]() {
            if (pend >= 0) {
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(qf_bar(pend));
                pend = -1;
            }
        };
        for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
            const int sp = u % S;
            for (int kb = sp * nk / S; kb < (sp + 1) * nk / S && ok; ++kb, rs.advance(NS)) {
#pragma unroll
                for (int w = 0; w < C::kW; ++w, ++job, rq.advance(NQ)) {
                    if ((job & (kDqGroups - 1)) != g) continue;
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(full_bar(rs.slot), rs.phase, abort_flag, args.ctl, I4_FULL) &&
                                        mbar_wait(qe_bar(rq.slot), rq.phase ^ 1u, abort_flag, args.ctl,
                                                  I4_QE));
                    if (!ok) break;
                    const uint8_t* blob = raw + rs.slot * C::kStage + w * kBlob;
                    const uint32_t* words = reinterpret_cast<const uint32_t*>(blob);
                    const uint16_t* sc = reinterpret_cast<const uint16_t*>(blob + kRawW);
                    const uint32_t col = q_base + rq.slot * kQCols + lane_addr;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {          // K halves: 64 values, 32 columns
                        uint32_t wv[8];
                        uint32_t s0 = sc[(2 * h) * 128 + n], s1 = sc[(2 * h + 1) * 128 + n];
#pragma unroll
                        for (int i = 0; i < 8; ++i) wv[i] = words[(8 * h + i) * 128 + (n ^ ((i & 3) << 3))];
                        s0 |= s0 << 16;
                        s1 |= s1 << 16;
                        uint32_t r[32];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint4 v = dequant_word(wv[i], i < 4 ? s0 : s1);
                            r[4 * i + 0] = v.x;
                            r[4 * i + 1] = v.y;
                            r[4 * i + 2] = v.z;
                            r[4 * i + 3] = v.w;
                        }
                        if (h == 0) release_pending();     // the previous job's stores are done
                        tmem_st32(col + h * 32, r);
                    }
                    pend = rq.slot;
                }
            }
        }
        release_pending();
    } else {
        // ================= epilogue =================
        const int q = warp & 3;
        const int ldo = PAIR ? (N >> 1) : N;
        const int et = tid - kEpiWarp0 * 32;             // 0..127 = weight row of the tile
        __shared__ int s_last;
        uint32_t epi_phase = 0;
        auto epi_sync = [&]() -> bool {                  // bounded, abort-aware rendezvous
            mbar_arrive(epi_bar);
            const bool ok = mbar_wait(epi_bar, epi_phase & 1u, abort_flag, args.ctl, I4_EPI);
            ++epi_phase;
            return __all_sync(0xffffffffu, ok);
        };
        RingPos ra;
        for (int u = blockIdx.x; u < total; u += gridDim.x, ra.advance(C::kAcc)) {
            const int t = u / S;
            int e, row0, rows, nb;
            i4_decode_tile<NT>(t, nbc, E, mt_start, args.offsets, e, row0, rows, nb);
            const int a = ra.slot;
            if (!__all_sync(0xffffffffu, mbar_wait(tf_bar(a), ra.phase, abort_flag, args.ctl, I4_TF)))
                break;
            tc_fence_after();
            const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + a * C::kCols;
            const int ncol = nb * 128 + q * 32 + lane;
            if (S > 1) {
                // this unit's fp32 partial, [col][row] so a warp writes 128 contiguous bytes
                float* pu = args.part + (size_t)u * C::kCols * 128 + et;
#pragma unroll
                for (int c = 0; c < C::kCols; c += 8) {
                    uint32_t r[8];
                    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
                                   "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                                 : "r"(tb + c));
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 8; ++j) pu[(size_t)(c + j) * 128] = __uint_as_float(r[j]);
                }
                tc_fence_before();
                mbar_arrive(te_bar(a));
                __threadfence();
                if (!epi_sync()) break;
                if (et == 0) s_last = (atomicAdd(args.cnt + t, 1) == S - 1);
                if (!epi_sync()) break;
                if (!s_last) continue;
                __threadfence();
                // last unit of the tile: sum the S partials in split order
                const float* pt = args.part + (size_t)t * S * C::kCols * 128 + et;
#pragma unroll
                for (int c = 0; c < NT; c += 8) {
                    float g[8], v[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) g[j] = v[j] = 0.0f;
                    for (int s2 = 0; s2 < S; ++s2) {
                        const float* ps = pt + (size_t)s2 * C::kCols * 128;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            g[j] += __ldcg(ps + (size_t)(c + j) * 128);
                            if (PAIR) v[j] += __ldcg(ps + (size_t)(NT + c + j) * 128);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (c + j < rows) {
                            const int orow = __ldg(args.sorted_rows + row0 + c + j);
                            const float val = PAIR ? silu_mul(g[j], v[j]) : g[j];
                            args.out[(size_t)orow * ldo + ncol] = __float2bfloat16_rn(val);
                        }
                    }
                }
                if (et == 0) args.cnt[t] = 0;     // ready for the next launch
                continue;
            }
            // 8 token columns at a time: few live registers
#pragma unroll
            for (int c = 0; c < NT; c += 8) {
                uint32_t r[8], v[8];
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                             : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                               "=r"(r[6]), "=r"(r[7])
                             : "r"(tb + c));
                if (PAIR)
                    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]),
                                   "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                                 : "r"(tb + NT + c));
                tmem_ld_wait();
                if (c + 8 >= NT) {
                    tc_fence_before();
                    mbar_arrive(te_bar(a));      // the accumulator is free for the next tile
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (c + j < rows) {
                        const int orow = __ldg(args.sorted_rows + row0 + c + j);
                        const float g = __uint_as_float(r[j]);
                        const float val = PAIR ? silu_mul(g, __uint_as_float(v[j])) : g;
                        args.out[(size_t)orow * ldo + ncol] = __float2bfloat16_rn(val);
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
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// Load-time repack into 9 KB blobs: block (e, nb, kb) = 2048 words
// [k8][n ^ 8 (k8 % 4)] with the nibbles of each word reordered to K offsets
// {0,2,4,6,1,3,5,7}, then 4 x 128 bf16 scales [g][n].
__global__ void int4_repack_kernel(const uint32_t* __restrict__ raw, const uint16_t* __restrict__ sc,
                                   uint32_t* __restrict__ blob, int E, int K, int N) {
    pdl_begin();
    const int nbn = N >> 7, nbk = K >> 7;
    const size_t words_per_block = kBlob / 4;                 // 2304
    const size_t total = (size_t)E * nbn * nbk * words_per_block;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t b = i / words_per_block;
        const int w = (int)(i - b * words_per_block);
        const int kb = (int)(b % nbk);
        const int nb = (int)((b / nbk) % nbn);
        const int e = (int)(b / ((size_t)nbk * nbn));
        uint32_t r;
        if (w < 2048) {
            const int k8 = w >> 7, n = (w & 127) ^ ((k8 & 3) << 3);
            const uint32_t v = raw[((size_t)e * (K >> 3) + kb * 16 + k8) * N + nb * 128 + n];
            r = 0;
#pragma unroll
            for (int slot = 0; slot < 8; ++slot) {
                const int k = slot < 4 ? 2 * slot : 2 * (slot - 4) + 1;
                r |= ((v >> (4 * k)) & 0xFu) << (4 * slot);
            }
        } else {
            const int idx = (w - 2048) * 2, g = idx >> 7, n = idx & 127;
            const size_t src = ((size_t)e * (K >> 5) + kb * 4 + g) * N + nb * 128 + n;
            r = (uint32_t)sc[src] | ((uint32_t)sc[src + 1] << 16);
        }
        blob[i] = r;
    }
}

// Expert-sorted activation rows: out[r] = hidden[rows[r] / topk]
// (zero row for a negative entry or a token >= T, the latter reported).
// Also clears the ncnt split-K tile counters for the GEMM that follows.
__global__ void gather_rows_kernel(const uint4* __restrict__ hidden, const int32_t* __restrict__ rows,
                                   int topk, int T, int R, int K, uint4* __restrict__ out,
                                   int* __restrict__ cnt, int ncnt, DevCtl ctl) {
    pdl_begin();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ncnt; i += gridDim.x * blockDim.x)
        cnt[i] = 0;
    const int per_row = K >> 3;                                // 16-byte chunks
    const size_t total = (size_t)R * per_row;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / per_row), c = (int)(i - (size_t)r * per_row);
        const int src = rows[r];
        int tok = src < 0 ? -1 : src / topk;
        if (tok >= T) {
            if (c == 0) report(ctl, DEV_BAD_ROW);
            tok = -1;
        }
        out[i] = tok < 0 ? make_uint4(0, 0, 0, 0) : hidden[(size_t)tok * per_row + c];
    }
}

template <int NT, bool PAIR>
int launch_int4(const DeviceInfo* info, const void* a_sorted, const uint8_t* blob,
                const int32_t* sorted_rows, const int32_t* offsets, void* out, int T, int topk,
                int N, int K, int E, int R, cudaStream_t stream, uint8_t* split_ws,
                size_t split_bytes) {
    using C = I4Cfg<NT, PAIR>;
    CUtensorMap tm_a;
    // gathered activations [R, K] bf16, box = 64 K values x NT rows
    int rc = make_tmap_2d(&tm_a, a_sorted, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, R, K, (uint64_t)K * 2,
                          64, NT, true);
    if (rc != FERRET_OK) return rc;
    static_assert(C::kQ >= C::kW * 2, "too few TMEM tile slots");
    // Each dequant group may hold a finished slot while it waits for a free one
    // for its next job; the slot it waits for must belong to an MMA step that
    // needs none of the held jobs (an MMA step takes kW consecutive jobs).
    static_assert(C::kQ >= kDqGroups + C::kW, "too few TMEM tile slots for the dequant pipeline");
    const int budget = info->max_smem_optin - 1024;
    const I4Layout l0 = i4_layout(C::kStage, 0, E);
    const int stages = std::min(kI4MaxStages, (budget - l0.total) / C::kStage);
    if (stages < 2) return FERRET_ERR_SHAPE;
    const I4Layout L = i4_layout(C::kStage, stages, E);
    const int smem = L.total + 1024;
    auto kern = int4_w13_grouped_kernel<NT, PAIR>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    Int4Args a;
    a.blob = blob;
    a.sorted_rows = sorted_rows;
    a.offsets = offsets;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.T = T;
    a.topk = topk;
    a.N = N;
    a.K = K;
    a.E = E;
    a.R = R;
    a.stages = stages;
    a.ctl = make_ctl(info);
    // Split K when the tiles cannot fill the SMs (decode with a handful of
    // tokens): at most the bound on tiles, floor(SMs / tiles) splits of at
    // least 4 K blocks, if the workspace holds the partials.
    a.splits = 1;
    a.part = nullptr;
    a.cnt = nullptr;
    const int nbc = PAIR ? N / 256 : N / 128;
    const long long tiles_up = ((long long)std::min(R, E) + R / NT) * nbc;
    if (split_ws && tiles_up > 0) {
        // (the counters, tiles_up ints at split_ws, were cleared by the row gather)
        const int S = (int)std::min<long long>(info->num_sms / tiles_up, (K / 128) / 4);
        const size_t part_bytes = (size_t)tiles_up * S * C::kCols * 128 * sizeof(float);
        const size_t cnt_bytes = (size_t)tiles_up * sizeof(int);
        if (S >= 2 && part_bytes + cnt_bytes <= split_bytes) {
            a.splits = S;
            a.cnt = reinterpret_cast<int*>(split_ws);
            a.part = reinterpret_cast<float*>(split_ws + ((cnt_bytes + 255) & ~size_t(255)));
        }
    }
    return launch_kernel(kern, dim3(info->num_sms), dim3(kI4Threads), smem, stream, tm_a, a);
}

}  // namespace
}  // namespace ferret

using namespace ferret;

extern "C" size_t ferret_int4_blob_bytes(int E, int K, int N) {
    if (E <= 0 || K <= 0 || N <= 0 || K % 128 || N % 128) return 0;
    return (size_t)E * (N / 128) * (K / 128) * kBlob;
}

// Routed rows up to which the workspace also holds split-K partials (decode
// with a handful of tokens), and the space reserved for them.
constexpr int kSplitMaxRows = 64;
constexpr size_t kSplitBytes = (size_t)9 << 20;

extern "C" size_t ferret_int4_moe_w13_workspace_size(int T, int topk, int K) {
    if (T < 0 || topk <= 0 || K <= 0) return 0;
    const size_t rows = (size_t)T * topk * K * 2;
    return T * topk <= kSplitMaxRows ? ((rows + 255) & ~size_t(255)) + kSplitBytes : rows;
}

extern "C" int ferret_int4_repack_w13(const int32_t* w_raw, const void* w_scale_bf16, void* w_blob,
                                      int E, int K, int N, void* stream) {
    if (E <= 0 || K <= 0 || N <= 0 || K % 128 || N % 128) return FERRET_ERR_SHAPE;
    if (!w_raw || !w_scale_bf16 || !w_blob) return FERRET_ERR_NULL;
    if (!aligned16(w_blob) || (reinterpret_cast<uintptr_t>(w_raw) & 3u) ||
        (reinterpret_cast<uintptr_t>(w_scale_bf16) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    const size_t words = ferret_int4_blob_bytes(E, K, N) / 4;
    const int grid = (int)std::min<size_t>((words + 255) / 256, (size_t)info->num_sms * 16);
    return launch_kernel(int4_repack_kernel, dim3(grid), dim3(256), 0, as_stream(stream),
                         reinterpret_cast<const uint32_t*>(w_raw),
                         static_cast<const uint16_t*>(w_scale_bf16),
                         static_cast<uint32_t*>(w_blob), E, K, N);
}

extern "C" int ferret_int4_moe_w13(const void* hidden_bf16, const void* w_blob,
                                   const int32_t* sorted_rows, const int32_t* expert_offsets,
                                   void* out_bf16, int T, int topk, int N, int K, int E, int flags,
                                   void* workspace, size_t ws_bytes, void* stream) {
    const bool pair = (flags & FERRET_SILU_MUL) != 0;
    if (T < 0 || topk <= 0 || N <= 0 || K <= 0 || E <= 0 || E > kI4MaxE) return FERRET_ERR_SHAPE;
    if (K % 128 || N % 128 || (pair && N % 256)) return FERRET_ERR_SHAPE;
    if ((long long)T * topk >= (1ll << 31) || (long long)E * (N / 128) * (K / 128) >= (1ll << 31))
        return FERRET_ERR_SHAPE;
    if (T == 0) return FERRET_OK;
    if (!hidden_bf16 || !w_blob || !sorted_rows || !expert_offsets || !out_bf16)
        return FERRET_ERR_NULL;
    if (!workspace || ws_bytes < ferret_int4_moe_w13_workspace_size(T, topk, K))
        return FERRET_ERR_WORKSPACE;
    if (!aligned16(hidden_bf16) || !aligned16(w_blob) || !aligned16(workspace) ||
        (reinterpret_cast<uintptr_t>(out_bf16) & 1u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    cudaStream_t s = as_stream(stream);
    const int R = T * topk;
    const uint8_t* blob = static_cast<const uint8_t*>(w_blob);
    int nt = (flags >> FERRET_TILE_SHIFT) & 0xFF;
    // A few rows per active expert (at most 4 on average, counting every
    // expert that can be active): the register-dequant decode kernel, which
    // streams the weights once without materialising them; more rows, or a
    // forced token tile: the tensor-core kernel.
    const bool decode = nt == 0 && R > kSplitMaxRows && (long long)R <= 4ll * std::min(R, E) &&
                        (reinterpret_cast<uintptr_t>(out_bf16) & 7u) == 0;
    if (nt == 0) {
        const int avg = (R + E - 1) / E;
        nt = avg <= 4 ? 8 : avg <= 12 ? 16 : 32;
    }
    // the workspace tail past the gathered rows holds split-K counters + partials
    const size_t rows_bytes = ((size_t)R * K * 2 + 255) & ~size_t(255);
    uint8_t* split_ws = nullptr;
    size_t split_bytes = 0;
    int ncnt = 0;
    if (R <= kSplitMaxRows && ws_bytes > rows_bytes) {
        split_ws = static_cast<uint8_t*>(workspace) + rows_bytes;
        split_bytes = ws_bytes - rows_bytes;
        const long long tiles_up =
            decode ? int4_decode_items_bound(R, E, N, pair)
                   : ((long long)std::min(R, E) + R / std::max(nt, 1)) * (pair ? N / 256 : N / 128);
        ncnt = (int)std::min<long long>(tiles_up, (long long)(split_bytes / sizeof(int)));
    }
    {
        const size_t chunks = (size_t)R * (K / 8);
        const int grid = (int)std::min<size_t>((chunks + 255) / 256, (size_t)info->num_sms * 8);
        if ((rc = launch_kernel(gather_rows_kernel, dim3(grid), dim3(256), 0, s,
                                static_cast<const uint4*>(hidden_bf16), sorted_rows, topk, T, R, K,
                                static_cast<uint4*>(workspace), reinterpret_cast<int*>(split_ws),
                                ncnt, make_ctl(info))) != FERRET_OK) return rc;
    }
    if (decode)
        return launch_int4_decode(info, workspace, blob, sorted_rows, expert_offsets, out_bf16, T,
                                  topk, N, K, E, R, pair, s, split_ws, split_bytes, ncnt);
#define FERRET_I4_CASE(NT_)                                                                        \
    case NT_:                                                                                      \
        return pair ? launch_int4<NT_, true>(info, workspace, blob, sorted_rows, expert_offsets,   \
                                             out_bf16, T, topk, N, K, E, R, s, split_ws,           \
                                             split_bytes)                                          \
                    : launch_int4<NT_, false>(info, workspace, blob, sorted_rows, expert_offsets,  \
                                              out_bf16, T, topk, N, K, E, R, s, split_ws,          \
                                              split_bytes);
    switch (nt) {
        FERRET_I4_CASE(8)
        FERRET_I4_CASE(16)
        FERRET_I4_CASE(32)
        default:
            return FERRET_ERR_SHAPE;
    }
#undef FERRET_I4_CASE
}
