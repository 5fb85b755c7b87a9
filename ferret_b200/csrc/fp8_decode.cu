// fp8_decode.cu -- FP8 (e4m3) block-scaled grouped GEMM for the MoE
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
#include "fp8_gemm_common.cuh"

namespace ferret {
namespace {

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
    const bool few_units = total <= 4 * (int)gridDim.x;   // at most ~4 units per CTA

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
            // stage this unit's scales, K blocks kb0..kb1 only: a_sc[kb - kb0][j],
            // w_sc[g][kb - kb0].  With few units per CTA (small batches) the
            // staging latency is exposed, so up to 8 loads per thread are in
            // flight before their stores and the first batch is loaded before
            // the rendezvous that frees the previous tile's copy; with many units
            // per CTA the producer runs ahead of the epilogue and the plain loop
            // measured faster (fewer registers and instructions).
            const int nkb = kb1 - kb0;
            const int n_as = nl * nkb;
            const size_t wsb = ((size_t)e * (N >> 7) + nb) * nk;
            if (few_units) {
                auto load_batch = [&](int base, float (&v)[8]) {
#pragma unroll
                    for (int x = 0; x < 8; ++x) {
                        const int i = base + x * kEpiThreads;
                        const int j = i / nkb, kb = kb0 + (i - j * nkb);
                        v[x] = (i < n_as && j < rows)
                                   ? __ldg(args.a_scale + (size_t)(row0 + j) * nk + kb)
                                   : 0.0f;
                    }
                };
                auto store_batch = [&](int base, const float (&v)[8]) {
#pragma unroll
                    for (int x = 0; x < 8; ++x) {
                        const int i = base + x * kEpiThreads;
                        const int j = i / nkb;
                        if (i < n_as) a_sc[(i - j * nkb) * NT + j] = v[x];
                    }
                };
                float v0[8];
                load_batch(et, v0);
                const float w0 = et < nkb ? __ldg(args.w_scale + wsb + kb0 + et) : 0.0f;
                const float w1 = (PAIR && et < nkb)
                                     ? __ldg(args.w_scale + wsb + (size_t)(N >> 8) * nk + kb0 + et)
                                     : 0.0f;
                if (!epi_sync()) break;
                store_batch(et, v0);
                for (int base = et + 8 * kEpiThreads; base < n_as; base += 8 * kEpiThreads) {
                    float v[8];
                    load_batch(base, v);
                    store_batch(base, v);
                }
                if (et < nkb) {
                    w_sc[et] = w0;
                    if (PAIR) w_sc[nk + et] = w1;
                }
            } else {
                if (!epi_sync()) break;
                for (int i = et; i < n_as; i += kEpiThreads) {
                    const int j = i / nkb, kb = kb0 + (i - j * nkb);
                    a_sc[(kb - kb0) * NT + j] =
                        (j < rows) ? __ldg(args.a_scale + (size_t)(row0 + j) * nk + kb) : 0.0f;
                }
                if (et < nkb) {
                    w_sc[et] = __ldg(args.w_scale + wsb + kb0 + et);
                    if (PAIR) w_sc[nk + et] = __ldg(args.w_scale + wsb + (size_t)(N >> 8) * nk + kb0 + et);
                }
            }
            for (int i = et + kEpiThreads; i < nkb; i += kEpiThreads) {
                w_sc[i] = __ldg(args.w_scale + wsb + kb0 + i);
                if (PAIR) w_sc[nk + i] = __ldg(args.w_scale + wsb + (size_t)(N >> 8) * nk + kb0 + i);
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
                const float ws = w_sc[kb - kb0];
                const float wsu = PAIR ? w_sc[nk + kb - kb0] : 0.0f;
                const float* asc = a_sc + (kb - kb0) * NT;
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

}  // namespace

int launch_fp8_decode(int nt, bool pair, const DeviceInfo* info, const void* a, const float* a_scale,
                      const void* w, const float* w_scale, void* out, const int32_t* seg,
                      int seg_pairs, int M, int N, int K, int E, cudaStream_t s,
                      const OutMap& om, const SplitWs& sw) {
#define FERRET_FP8_CASE(NT_)                                                                    \
    case NT_:                                                                                   \
        return pair ? launch_fp8<NT_, true>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M, \
                                            N, K, E, s, om, sw)                                 \
                    : launch_fp8<NT_, false>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M,\
                                             N, K, E, s, om, sw);
    switch (nt) {
        FERRET_FP8_CASE(16)
        FERRET_FP8_CASE(32)
        FERRET_FP8_CASE(64)
        case 128:
            if (pair) return FERRET_ERR_SHAPE;
            return launch_fp8<128, false>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M, N,
                                          K, E, s, om, sw);
        default:
            return FERRET_ERR_SHAPE;
    }
#undef FERRET_FP8_CASE
}

int launch_derive_segments(const DeviceInfo* info, const int32_t* m_indices, int M, int E,
                           int32_t* seg, int* cnt, int ncnt, cudaStream_t stream) {
    return launch_kernel(derive_segments_kernel, dim3(1), dim3(kSegThreads),
                         3 * E * (int)sizeof(int), stream, m_indices, M, E, seg, make_ctl(info),
                         cnt, ncnt);
}

}  // namespace ferret
