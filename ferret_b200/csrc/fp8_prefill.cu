// fp8_prefill.cu -- the prefill-shaped FP8 grouped GEMM (tokens on the MMA M
// axis, 128 x 256 tiles), its expert-parallel form (token rows pulled from
// and results pushed to the other GPUs by extra warps of the same kernel,
// while the tiles run), and the opt-in CTA-pair form.
#include "fp8_gemm_common.cuh"

namespace ferret {
namespace {

// Expert-parallel form of the prefill kernel.  Extra warps move the rows
// while the tiles run:
//   * four pull warps per CTA copy the routed token rows (e4m3 + 1x128 scales) out of
//     the source ranks' memory into the A operand, in tile order, with plain
//     16-byte peer loads (NVLink), counting each landed row on its 128-row
//     tile's `ready` counter (release).  The TMA producer waits for a tile's
//     count before its first A load (acquire, then a proxy fence so the
//     async-proxy loads see the rows); the epilogue waits the same way before
//     reading the rows' scales.
//   * the epilogue stores each tile into a local staging matrix, exactly as
//     the single-GPU kernel stores its output, and each epilogue warp counts
//     its part of the tile on the tile's `done` counter; the push warp, once
//     every epilogue warp of every 256-column block of a 128-row tile has
//     counted, two push warps per CTA copy those rows to their destination (row sorted[i] % own of
//     rank sorted[i] / own) as whole contiguous rows: 8 KB (4 KB with SiLU)
//     NVLink writes.
// Neither mover waits on anything but counters that the other roles raise
// without waiting on the movers, so every count completes while all CTAs are
// resident (one CTA per SM, grid = SMs); every wait is bounded all the same.
struct EpMoveArgs {
    const int32_t* src;                 // [rows] global pair index of each sorted row
    const uint8_t* const* q_peers;      // [world] every rank's e4m3 token rows
    const float* const* s_peers;        // [world] every rank's 1x128 scales
    __nv_bfloat16* const* out_peers;    // [world] every rank's output rows, (token, slot) order
    uint8_t* a;                         // the A operand: pulled row i is written here
    float* a_s;                         // its scales
    int* ready;                         // [128-row tiles] rows landed, zero at launch
    int* done;                          // [128-row tiles] warp-tiles stored, zero at launch
    int own;                            // pairs per rank (tokens * topk)
    int topk;
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Orders this thread's generic-proxy view (the acquire before it) before its
// later async-proxy accesses (the TMA loads of the rows that were pulled).
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until counter *cnt reaches `want` (acquire).
__device__ bool wait_count(const int* cnt, int want, volatile int* abort_flag, const DevCtl& ctl,
                           int site) {
    if (ld_acquire_gpu(cnt) >= want) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        __nanosleep(128);
        if (ld_acquire_gpu(cnt) >= want) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > ctl.timeout_ns) {
            *abort_flag = 1;
            report(ctl, DEV_TIMEOUT | (site << 8));
            return false;
        }
    }
}

// Pull warp pw of this CTA: row slots blockIdx.x * kPfPullWarps + pw, then
// every gridDim.x * kPfPullWarps-th, of the tile-ordered slot list (128 per
// tile), so the rows land roughly in the order the tiles need them.
__device__ __forceinline__ void ep_pull_rows(const EpMoveArgs& mv, int K, int E, const int* mt_start,
                                             const int* seg_s, const int* seg_c, int pw, int lane) {
    const int nk = K >> 7;
    const int vec = K >> 4;                    // 16-byte words per row
    const int slots = mt_start[E] * 128;
    for (int idx = blockIdx.x * kPfPullWarps + pw; idx < slots; idx += gridDim.x * kPfPullWarps) {
        const int mt = idx >> 7, i = idx & 127;
        int e, row0, rows, nb;
        decode_tile<128>(mt, 1, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
        if (i >= rows) continue;
        const int r = row0 + i;
        const int src = __ldg(mv.src + r);
        const int g = src / mv.own;
        const int tok = (src - g * mv.own) / mv.topk;
        const uint4* q = reinterpret_cast<const uint4*>(mv.q_peers[g] + (size_t)tok * K);
        const float* sc = mv.s_peers[g] + (size_t)tok * nk;
        uint4* dst = reinterpret_cast<uint4*>(mv.a + (size_t)r * K);
        // all of a lane's loads for a 4 KB piece of the row before its
        // stores: one NVLink latency per piece
        for (int base = 0; base < vec; base += 32 * 8) {
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = base + lane + 32 * j;
                if (c < vec) v[j] = __ldcv(q + c);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = base + lane + 32 * j;
                if (c < vec) dst[c] = v[j];
            }
        }
        for (int c = lane; c < nk; c += 32) mv.a_s[(size_t)r * nk + c] = __ldcv(sc + c);
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_gpu_add(mv.ready + mt, 1);
    }
}

// Push warp pw of this CTA: the same kind of slot walk; a row moves once
// every epilogue warp of every 256-column block of its tile has counted.
__device__ __forceinline__ void ep_push_rows(const EpMoveArgs& mv, const __nv_bfloat16* stage,
                                             int ldo, int nbc, int E, const int* mt_start,
                                             const int* seg_s, const int* seg_c, int pw, int lane,
                                             volatile int* abort_flag, const DevCtl& ctl) {
    const int vec = ldo >> 3;                  // 16-byte words per output row
    const int slots = mt_start[E] * 128;
    const int want = nbc * kPfEpEpiWarps;
    for (int idx = blockIdx.x * kPfPushWarps + pw; idx < slots; idx += gridDim.x * kPfPushWarps) {
        const int mt = idx >> 7, i = idx & 127;
        int e, row0, rows, nb;
        decode_tile<128>(mt, 1, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
        if (i >= rows) continue;
        if (!__all_sync(0xffffffffu, wait_count(mv.done + mt, want, abort_flag, ctl, SITE_PUSH)))
            return;
        const int r = row0 + i;
        const int src = __ldg(mv.src + r);
        const int g = src / mv.own;
        const uint4* sp = reinterpret_cast<const uint4*>(stage + (size_t)r * ldo);
        uint4* d = reinterpret_cast<uint4*>(mv.out_peers[g] + (size_t)(src - g * mv.own) * ldo);
        for (int base = 0; base < vec; base += 32 * 8) {
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = base + lane + 32 * j;
                if (c < vec) v[j] = __ldcg(sp + c);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = base + lane + 32 * j;
                if (c < vec) d[c] = v[j];
            }
        }
    }
}

// The tile pipeline of the prefill kernel and of its expert-parallel form.
// EP: the expert-parallel form (EpMoveArgs), kPfPeerThreads threads.
template <bool PAIR, bool EP>
__device__ __forceinline__ void prefill_body(const CUtensorMap* tm_w, const CUtensorMap* tm_a,
                                             const GemmArgs& args, const EpMoveArgs& mv) {
    constexpr int kNT = EP ? kPfPeerThreads : kPfThreads;
    constexpr int kEW = EP ? kPfEpEpiWarps : kPfEpiWarps;      // epilogue warps
    constexpr int kEpi0 = EP ? 4 : kPfEpi0;                    // first epilogue warp
    constexpr int kCPH = 512 / kEW;          // columns per thread in each 128-column half
    constexpr int kLDmax = EP ? kPfEpLdCols : kPfLdCols;
    constexpr int kLD = kCPH < kLDmax ? kCPH : kLDmax;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = args.M, N = args.N, K = args.K, E = args.E, NS = args.stages;
    const int nk = K >> 7;
    const int nbc = N >> 8;                        // 256-row weight tiles
    const PfLayout L = pf_layout(NS, E, EP);
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
            // single-GPU form: one arrive per epilogue warp; EP form: one per
            // epilogue thread (each measured faster in its own kernel)
            mbar_init(tempty_bar(a), EP ? kEW * 32 : kEW);
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
    for (int e = tid; e < E; e += kNT) {
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

    auto producer = [&]() {
        // ================= TMA producer =================
        if (elect_one()) {
            tma_prefetch_desc(tm_w);
            tma_prefetch_desc(tm_a);
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
                if constexpr (EP) {
                    // the tile's A rows are pulled by this kernel's own mover warp
                    if (!wait_count(mv.ready + t / nbc, rows, abort_flag, args.ctl, SITE_ROWS)) {
                        ok = false;
                        break;
                    }
                    fence_proxy_async_global();
                }
                for (int kb = 0; kb < nk; ++kb, ++it, rp.advance(NS)) {
                    const int s = rp.slot;
                    if (!mbar_wait(empty_bar(s), rp.phase ^ 1u, abort_flag, args.ctl, SITE_EMPTY)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = stage_base + s * kPfStage;
                    mbar_expect_tx(full_bar(s), kPfStage);
                    tma_load_2d_hint(dst, tm_a, kb * 128, row0, full_bar(s), pol_a);
                    tma_load_2d_hint(dst + 16384, tm_w, kb * 128, w0, full_bar(s), pol_w);
                    tma_load_2d_hint(dst + 32768, tm_w, kb * 128, w1, full_bar(s), pol_w);
                }
            }
            for (int i = max(0, it - NS); i < it; ++i)
                mbar_wait(full_bar(i % NS), (i / NS) & 1, abort_flag, args.ctl, SITE_DRAIN, false);
        }
    };
    auto mma_issuer = [&]() {
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
    };
    auto epilogue = [&]() {
        // ================= epilogue: promotion + store =================
        const int h = (warp - kEpi0) >> 2;       // columns [kCPH h, kCPH (h+1)) of each block
        const int q = warp & 3;                  // TMEM lanes [32q, 32q+32) = tile rows
        const int r = q * 32 + lane;
        const int ldo = PAIR ? (N >> 1) : N;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        RingPos ra;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int e, row0, rows, nb;
            decode_tile<128>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            if constexpr (EP) {
                // the rows' scales come from this kernel's own pull
                if (!__all_sync(0xffffffffu, wait_count(mv.ready + t / nbc, rows, abort_flag,
                                                        args.ctl, SITE_ROWS)))
                    break;
            }
            const bool live = r < rows;
            const float* as_row = args.a_scale + (size_t)(row0 + (live ? r : 0)) * nk;
            const int blk0 = PAIR ? nb : 2 * nb;
            const int blk1 = PAIR ? (N >> 8) + nb : 2 * nb + 1;
            const float* ws0 = args.w_scale + ((size_t)e * (N >> 7) + blk0) * nk;
            const float* ws1 = args.w_scale + ((size_t)e * (N >> 7) + blk1) * nk;
            float acc0[kCPH], acc1[kCPH];
#pragma unroll
            for (int j = 0; j < kCPH; ++j) {
                acc0[j] = 0.0f;
                acc1[j] = 0.0f;
            }
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb, ra.advance(2)) {
                // EP: a plain (L1-caching) load, ordered after the pull by the
                // acquire above (the read-only path would not be)
                const float sa = live ? (EP ? __ldca(as_row + kb) : __ldg(as_row + kb)) : 0.0f;
                const float s0 = sa * __ldg(ws0 + kb), s1 = sa * __ldg(ws1 + kb);
                ok = __all_sync(0xffffffffu, mbar_wait(tfull_bar(ra.slot), ra.phase, abort_flag,
                                                       args.ctl, SITE_TFULL));
                if (!ok) break;
                tc_fence_after();
                promote_kblock<kCPH, kLD, 128, !EP>(tmem_base + lane_addr + ra.slot * 256 + h * kCPH,
                                                    acc0, acc1, s0, s1);
                // this thread's loads of the buffer are complete (wait::ld)
                // before it releases the buffer to the MMA: each thread (EP), or
                // the warp once all its lanes have (single-GPU form)
                tc_fence_before();
                if constexpr (EP) {
                    mbar_arrive(tempty_bar(ra.slot));
                } else {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty_bar(ra.slot));
                }
            }
            if (!ok) break;
            int orow = row0 + r;
            if (live && args.out_rows) {
                orow = __ldg(args.out_rows + row0 + r);
                if (orow < 0 || orow >= args.out_total) orow = -1;
            }
            if (live && orow >= 0)
                store_tile_row<PAIR, kCPH>(out_row_ptr(args, orow, ldo), nb, h, acc0, acc1);
            if constexpr (EP) {
                // this warp's rows of the tile are stored: count it for the push
                __threadfence();
                __syncwarp();
                if (lane == 0) red_release_gpu_add(mv.done + t / nbc, 1);
            }
        }
    };

    if constexpr (EP) {
        // Warpgroups 0 (TMA, MMA, pull, push) and 3 (pull x3, push) hand
        // registers to the two epilogue warpgroups (1, 2), which then hold their
        // accumulators without spilling: launched at 128 per thread, 2 x 128 x 64
        // + 2 x 128 x 192 = 512 x 128.
        static_assert(kPfEpEpiWarps == 8 && kPfEpCtlRegs == 64 && kPfEpEpiRegs == 192,
                      "warp roles below assume this split");
        if (warp < 4 || warp >= 12) {
            setmaxnreg_dec<kPfEpCtlRegs>();
            if (warp == 0) producer();
            else if (warp == 1) mma_issuer();
            else if (warp == 2 || warp >= 13)
                ep_pull_rows(mv, K, E, mt_start, seg_s, seg_c, warp == 2 ? 0 : warp - 12, lane);
            else
                ep_push_rows(mv, args.out, PAIR ? (N >> 1) : N, nbc, E, mt_start, seg_s, seg_c,
                             warp == 3 ? 0 : 1, lane, abort_flag, args.ctl);
        } else {
            setmaxnreg_inc<kPfEpEpiRegs>();
            epilogue();
        }
    } else if constexpr (kPfRegSplit) {
        // warpgroup 0 (TMA, MMA; warps 2-3 idle) hands registers to the
        // epilogue warpgroups (the launcher checks that the kernel was built
        // with pf_launch_regs(kPfThreads) registers per thread)
        static_assert(128 * kPfCtlRegs + 32 * kPfEpiWarps * kPfEpiRegs <=
                          kPfThreads * pf_launch_regs(kPfThreads),
                      "register split above the launch's registers");
        if (warp < 4) {
            setmaxnreg_dec<kPfCtlRegs>();
            if (warp == 0) producer();
            else if (warp == 1) mma_issuer();
        } else {
            setmaxnreg_inc<kPfEpiRegs>();
            epilogue();
        }
    } else {
        if (warp == 0) producer();
        else if (warp == 1) mma_issuer();
        else epilogue();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}


template <bool PAIR>
__global__ void __launch_bounds__(kPfThreads, 1)
    fp8_w13_prefill_kernel(const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_a, const GemmArgs args) {
    pdl_begin();
    prefill_body<PAIR, false>(&tm_w, &tm_a, args, EpMoveArgs{});
}

template <bool PAIR>
__global__ void __launch_bounds__(kPfPeerThreads, 1)
    fp8_w13_prefill_ep_kernel(const __grid_constant__ CUtensorMap tm_w,
                              const __grid_constant__ CUtensorMap tm_a, const GemmArgs args,
                              const EpMoveArgs mv) {
    pdl_begin();
    prefill_body<PAIR, true>(&tm_w, &tm_a, args, mv);
}

// ---------------------------------------------------------------------------
// CTA-pair form of the prefill kernel (FERRET_PREFILL_PAIRS).
//
// A pair (thread-block cluster of 2 on two SMs) computes a 256-token x
// 256-weight-row tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32):
// CTA r loads token rows [128r, 128r+128) of the tile and weight rows
// [128r, 128r+128) of its 256-row block (gate block for r = 0 and up block for
// r = 1 with SiLU), and receives the 128 x 256 partial of its own token rows in
// its own Tensor Memory.  Per SM that is 32 KB of operands per 128-wide K block
// instead of 48 KB for the same MMA work, so the same shared-memory ring keeps
// 1.5x more MMA work in flight.  Every expert's rows are covered by 256-row
// pair tiles; in the last one the rows past the expert are computed and
// dropped (a half with none of the expert's rows loads no A tile and skips its
// promotion).
//
// Protocol (every load is a plain TMA load into the issuing CTA's own shared memory):
//   * both CTAs load their halves with .cta_group::2 TMA, completing on the
//     leader's (rank 0) full barrier, which the leader arms with the tile's
//     byte count of both CTAs;
//   * the leader's MMA thread waits for it and for the TMEM buffer's release,
//     issues the 4 pair MMAs of the K block and commits to each CTA's empty
//     barrier (stage free) and tfull barrier (partial ready);
//   * each CTA's epilogue warps promote their own partial exactly as the
//     single-CTA kernel does and release the buffer with one arrive per warp on
//     the leader's tempty barrier;
//   * a cluster barrier after the roles finish keeps either CTA from leaving
//     while the other still reads its shared memory or writes its Tensor Memory.
// ---------------------------------------------------------------------------

template <bool PAIR, int BN>
__global__ void __launch_bounds__(kPpThreads, 1)
    fp8_w13_prefill_pair_kernel(const __grid_constant__ CUtensorMap tm_w,
                                const __grid_constant__ CUtensorMap tm_a, const GemmArgs args) {
    pdl_begin();
    using T = PpTile<BN>;
    constexpr int kHalf = BN / 2;                  // weight rows per CTA = partial columns per half
    constexpr int kEW = kPpEpiWarps;
    constexpr int kEpi0 = kPfEpi0;
    constexpr int kCPH = kHalf / (kEW / 4);        // columns per thread in each half
    constexpr int kLD = kCPH < kPfLdCols ? kCPH : kPfLdCols;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = args.M, N = args.N, K = args.K, E = args.E, NS = args.stages;
    const int nk = K >> 7;
    const int nbc = N / BN;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const Pp2Layout L = pp2_layout<BN>(NS, E);
    int* seg_s = reinterpret_cast<int*>(smem + L.segs_off);
    int* seg_c = reinterpret_cast<int*>(smem + L.segc_off);
    int* mt_start = reinterpret_cast<int*>(smem + L.mts_off);
    int* part = reinterpret_cast<int*>(smem + L.part_off);
    const uint32_t bar0 = smem_addr(smem + L.bar_off);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (T::kMaxStages + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * T::kMaxStages + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * T::kMaxStages + T::kBufs + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * T::kMaxStages + 2 * T::kBufs);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
    const uint32_t stage_base = smem_addr(smem + L.stages_off);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 1);            // the leader's arm; bytes from both CTAs
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < T::kBufs; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 2 * kEW);   // one per epilogue warp of both CTAs
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
    for (int e = tid; e < E; e += kPpThreads) {
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
        mt_start[e] = (c + 255) >> 8;
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

    auto producer = [&]() {
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
                const bool a_live = 128 * (int)rank < rows;      // this CTA's A rows exist
                const uint32_t bytes = 16384 + 2 * T::kB + (rows > 128 ? 16384 : 0);
                const int arow = row0 + 128 * (int)rank;
                const int wrow = PAIR ? e * N + (rank ? (N >> 1) : 0) + nb * kHalf
                                      : e * N + nb * BN + kHalf * (int)rank;
                for (int kb = 0; kb < nk; ++kb, ++it, rp.advance(NS)) {
                    const int s = rp.slot;
                    if (!mbar_wait_cl(empty_bar(s), rp.phase ^ 1u, abort_flag, args.ctl,
                                      SITE_PEER_EMPTY)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_expect_tx(full_bar(s), bytes);
                    const uint32_t dst = stage_base + s * T::kStage;
                    const uint32_t bar = mapa_shared(full_bar(s), 0);
                    if (a_live) tma_load_2d_pair(dst, &tm_a, kb * 128, arow, bar, pol);
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
    };
    auto mma_issuer = [&]() {
        // ================= MMA issuer (leader CTA) =================
        if (leader && elect_one()) {
            constexpr uint32_t idesc = make_idesc(256, BN, 0, 0);
            RingPos rs, ra;
            bool ok = true;
            for (int t = pair; t < total && ok; t += npairs) {
                for (int kb = 0; kb < nk; ++kb, rs.advance(NS), ra.advance(T::kBufs)) {
                    const int s = rs.slot, a = ra.slot;
                    if (!mbar_wait_cl(tempty_bar(a), ra.phase ^ 1u, abort_flag, args.ctl,
                                      SITE_TEMPTY) ||
                        !mbar_wait_cl(full_bar(s), rs.phase, abort_flag, args.ctl, SITE_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = stage_base + s * T::kStage;
                    const uint32_t d = tmem_base + a * BN;
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
    };
    auto epilogue = [&]() {
        // ================= epilogue: promotion + store (both CTAs) =================
        const int h = (warp - kEpi0) >> 2;       // columns [kCPH h, kCPH (h+1)) of each block
        const int q = warp & 3;                  // TMEM lanes [32q, 32q+32) = this CTA's rows
        const int r = q * 32 + lane;
        const int ldo = PAIR ? (N >> 1) : N;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        RingPos ra;
        for (int t = pair; t < total; t += npairs) {
            int e, row0, rows, nb;
            decode_tile<256>(t, nbc, E, mt_start, seg_s, seg_c, e, row0, rows, nb);
            const int my0 = row0 + 128 * (int)rank;
            const int my_rows = min(max(rows - 128 * (int)rank, 0), 128);
            const bool live = r < my_rows;
            const float* as_row = args.a_scale + (size_t)(my0 + (live ? r : 0)) * nk;
            // 128-row weight blocks of the two halves' rows (one block for both
            // halves when BN = 128 without SiLU)
            const int blk0 = (PAIR ? nb * kHalf : nb * BN) >> 7;
            const int blk1 = (PAIR ? (N >> 1) + nb * kHalf : nb * BN + kHalf) >> 7;
            const float* ws0 = args.w_scale + ((size_t)e * (N >> 7) + blk0) * nk;
            const float* ws1 = args.w_scale + ((size_t)e * (N >> 7) + blk1) * nk;
            float acc0[kCPH], acc1[kCPH];
#pragma unroll
            for (int j = 0; j < kCPH; ++j) {
                acc0[j] = 0.0f;
                acc1[j] = 0.0f;
            }
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb, ra.advance(T::kBufs)) {
                const float sa = live ? __ldg(as_row + kb) : 0.0f;
                const float s0 = sa * __ldg(ws0 + kb), s1 = sa * __ldg(ws1 + kb);
                ok = __all_sync(0xffffffffu, mbar_wait_cl(tfull_bar(ra.slot), ra.phase, abort_flag,
                                                          args.ctl, SITE_TFULL));
                if (!ok) break;
                tc_fence_after();
                if (my_rows > 0)
                    promote_kblock<kCPH, kLD, kHalf>(tmem_base + lane_addr + ra.slot * BN + h * kCPH,
                                                     acc0, acc1, s0, s1);
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
            if (live && orow >= 0)
                store_tile_row<PAIR, kCPH, kHalf>(args.out + (size_t)orow * ldo, nb, h, acc0, acc1);
        }
    };

    if constexpr (kPfRegSplit) {
        if (warp < 4) {
            setmaxnreg_dec<kPfCtlRegs>();
            if (warp == 0) producer();
            else if (warp == 1) mma_issuer();
        } else {
            setmaxnreg_inc<kPfEpiRegs>();
            epilogue();
        }
    } else {
        if (warp == 0) producer();
        else if (warp == 1) mma_issuer();
        else epilogue();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();             // neither CTA leaves while the other may still touch it
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

template <bool PAIR, int BN = kPpBN>
int launch_fp8_prefill_pairs_p(const DeviceInfo* info, const void* a, const float* a_scale,
                               const void* w, const float* w_scale, void* out, const int32_t* seg,
                               int seg_pairs, int M, int N, int K, int E, cudaStream_t stream,
                               const OutMap& om) {
    using T = PpTile<BN>;
    if (N % BN) return FERRET_ERR_SHAPE;
    CUtensorMap tm_w, tm_a;
    int rc = make_tmap_2d(&tm_w, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)E * N, K, K, 128,
                          BN / 2, true);
    if (rc != FERRET_OK) return rc;
    rc = make_tmap_2d(&tm_a, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, K, 128, 128, true);
    if (rc != FERRET_OK) return rc;
    const int budget = info->max_smem_optin - 1024;
    const int stages = std::min(T::kMaxStages, (budget - pp2_layout<BN>(0, E).total) / T::kStage);
    if (stages < 2) return FERRET_ERR_SHAPE;
    const int smem = pp2_layout<BN>(stages, E).total + 1024;
    auto kern = fp8_w13_prefill_pair_kernel<PAIR, BN>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    static const bool regs_ok = !kPfRegSplit || kernel_has_regs(kern, pf_launch_regs(kPpThreads));
    if (!regs_ok) return FERRET_ERR_CUDA;
    const int pairs = std::min(max_resident_pairs(kern, dim3(kPpThreads), smem), info->num_sms / 2);
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
    return launch_kernel_pairs(kern, dim3(2 * pairs), dim3(kPpThreads), smem, stream, tm_w, tm_a,
                               g);
}

template <bool PAIR, bool EP>
int launch_fp8_prefill_t(const DeviceInfo* info, const void* a, const float* a_scale, const void* w,
                         const float* w_scale, void* out, const int32_t* seg, int seg_pairs, int M,
                         int N, int K, int E, cudaStream_t stream, const OutMap& om) {
    CUtensorMap tm_w, tm_a;
    int rc = make_tmap_2d(&tm_w, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)E * N, K, K, 128,
                          128, true);
    if (rc != FERRET_OK) return rc;
    rc = make_tmap_2d(&tm_a, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, K, 128, 128, true);
    if (rc != FERRET_OK) return rc;
    const int budget = info->max_smem_optin - 1024;
    const int stages = std::min(kPfMaxStages, (budget - pf_layout(0, E, EP).total) / kPfStage);
    if (stages < 2) return FERRET_ERR_SHAPE;
    const int smem = pf_layout(stages, E, EP).total + 1024;
    auto kern_local = fp8_w13_prefill_kernel<PAIR>;
    auto kern_ep = fp8_w13_prefill_ep_kernel<PAIR>;
    const cudaError_t ae =
        EP ? cudaFuncSetAttribute(kern_ep, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)
           : cudaFuncSetAttribute(kern_local, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (ae != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    GemmArgs g;
    g.a_scale = a_scale;
    g.w_scale = w_scale;
    g.seg = seg;
    g.seg_pairs = seg_pairs;
    g.out = static_cast<__nv_bfloat16*>(out);
    g.out_rows = EP ? nullptr : om.rows;     // EP: tiles go to the local staging rows
    g.out_total = om.total;
    g.out_peers = EP ? nullptr : om.peers;
    g.peer_rows = om.peer_rows;
    g.M = M;
    g.N = N;
    g.K = K;
    g.E = E;
    g.stages = stages;
    g.ctl = make_ctl(info);
    if (!EP) {
        static const bool regs_ok = !kPfRegSplit || kernel_has_regs(kern_local, pf_launch_regs(kPfThreads));
        if (!regs_ok) return FERRET_ERR_CUDA;
        return launch_kernel(kern_local, dim3(info->num_sms), dim3(kPfThreads), smem, stream, tm_w,
                             tm_a, g);
    }
    static const bool regs_ok_ep = kernel_has_regs(kern_ep, pf_launch_regs(kPfPeerThreads));
    if (!regs_ok_ep) return FERRET_ERR_CUDA;
    if (!om.rows || !om.peers || !om.q_peers || !om.s_peers || !om.ready || !om.done ||
        om.peer_rows <= 0 || om.gather_topk <= 0)
        return FERRET_ERR_NULL;
    EpMoveArgs mv;
    mv.src = om.rows;
    mv.q_peers = om.q_peers;
    mv.s_peers = om.s_peers;
    mv.out_peers = om.peers;
    mv.a = static_cast<uint8_t*>(const_cast<void*>(a));
    mv.a_s = const_cast<float*>(a_scale);
    mv.ready = om.ready;
    mv.done = om.done;
    mv.own = om.peer_rows;
    mv.topk = om.gather_topk;
    return launch_kernel(kern_ep, dim3(info->num_sms), dim3(kPfPeerThreads), smem, stream, tm_w,
                         tm_a, g, mv);
}

template <bool PAIR>
int launch_fp8_prefill_p(const DeviceInfo* info, const void* a, const float* a_scale, const void* w,
                         const float* w_scale, void* out, const int32_t* seg, int seg_pairs, int M,
                         int N, int K, int E, cudaStream_t stream, const OutMap& om) {
    return om.gather ? launch_fp8_prefill_t<PAIR, true>(info, a, a_scale, w, w_scale, out, seg,
                                                        seg_pairs, M, N, K, E, stream, om)
                     : launch_fp8_prefill_t<PAIR, false>(info, a, a_scale, w, w_scale, out, seg,
                                                         seg_pairs, M, N, K, E, stream, om);
}

}  // namespace

int launch_fp8_prefill(bool pair, const DeviceInfo* info, const void* a, const float* a_scale,
                       const void* w, const float* w_scale, void* out, const int32_t* seg,
                       int seg_pairs, int M, int N, int K, int E, cudaStream_t stream,
                       const OutMap& om) {
    return pair ? launch_fp8_prefill_p<true>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M,
                                             N, K, E, stream, om)
                : launch_fp8_prefill_p<false>(info, a, a_scale, w, w_scale, out, seg, seg_pairs, M,
                                              N, K, E, stream, om);
}

int launch_fp8_prefill_pairs(bool pair, const DeviceInfo* info, const void* a,
                             const float* a_scale, const void* w, const float* w_scale, void* out,
                             const int32_t* seg, int seg_pairs, int M, int N, int K, int E,
                             cudaStream_t stream, const OutMap& om) {
    return pair ? launch_fp8_prefill_pairs_p<true>(info, a, a_scale, w, w_scale, out, seg,
                                                   seg_pairs, M, N, K, E, stream, om)
                : launch_fp8_prefill_pairs_p<false>(info, a, a_scale, w, w_scale, out, seg,
                                                    seg_pairs, M, N, K, E, stream, om);
}

}  // namespace ferret
