// fp8_prefill_mx.cu -- the block-scaled (UE8M0) prefill FP8 grouped GEMM,
// single-CTA and CTA-pair forms (FERRET_UE8M0_SCALES).
#include "fp8_gemm_common.cuh"

namespace ferret {
namespace {


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


}  // namespace

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

namespace {


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

}  // namespace


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

}  // namespace ferret
