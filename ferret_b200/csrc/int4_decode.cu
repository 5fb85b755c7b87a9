// int4_decode.cu -- W4A16 INT4 W13 grouped GEMM for decode-sized batches (a
// few token rows per expert: benchmark configuration 4 has 512 routed rows
// over ~285 active experts, 1.8 rows each), without materialising the
// dequantized weights anywhere.
//
// At ~2 token rows per expert a weight element is used ~twice, so the job is
// to stream the 4-bit weights from HBM once and spend as few issue slots per
// weight as possible.  The tensor-core kernel (int4_grouped_gemm.cu) writes
// every dequantized weight into Tensor Memory for tcgen05.mma, and that store
// volume, not HBM, bounds it at this shape.  Here the weights go from the
// load straight into registers, are dequantized there with the same exact
// steps (bf16((n - 8) * s): one lop3 into a bf16 with exponent 128, one
// bf16x2 subtract, one bf16x2 multiply -- the reference's formula,
// correctness/compare_marlin_vs_ref.py:44-100), and are fed to the warp-level
// mma.sync.m16n8k16 bf16 x bf16 -> fp32 from those registers: the tensor core
// serves as the multiply-accumulate unit (products exact in fp32, fp32
// accumulation), eight token rows per instruction, with no shared-memory or
// Tensor-Memory round trip for either operand.  (tcgen05.mma reads A from
// shared or Tensor Memory, so it cannot take fragments from registers.)
//
// Fragment mapping.  The MMA's reduction index order is free as long as both
// operands use the same one, so each thread takes whole repacked words:
// thread (g = lane / 4, t = lane % 4) of a warp loads, per 32-wide K group q
// of a 128-wide K block, word k8 = 4q + t of four adjacent weight rows
// (one 16-byte load: the repacked blob stores words [k8][n]) and the 8
// activation values of that word's K range for token row g (one 16-byte
// load).  Word pairs (k, k+1), (k+2, k+3) of rows 4g / 4g+1 form the A
// fragment of one m16n8k16 (logical rows g and g + 8), the activation pairs
// its B fragment; pairs (k+4 .. k+7) the next one; rows 4g+2 / 4g+3 a second
// 16-row slice.  A warp thus covers 32 weight rows, a CTA of 4 warps one
// 128-row block; with the fused SiLU epilogue each warp also carries the
// matching 32 rows of the up block.
//
// Work items: (active expert, pass of up to 8 token rows, 128-column output
// block), listed per CTA from the expert offsets (block scan), walked
// persistently.  When the items cannot fill the SMs (a handful of tokens),
// each item's K blocks are split over several units; fp32 partials go to the
// workspace and the last unit of an item (atomic counter) sums them in split
// order -- deterministic -- and stores.
//
// Feeding the warps.  A warp that loads its own weights from global memory
// can keep only one K block of loads in flight (its registers hold them), far
// fewer bytes per SM than it takes to cover the HBM latency.  So a fifth warp
// copies each K block into a shared-memory ring ahead of use: the weight blob
// of the (expert, 128-row block, K block) -- 9 KB contiguous, one bulk copy;
// two with SiLU -- and the pass's 8 activation rows of that K block (one 2 KB
// tensor-map box; rows past the expert are computed and never stored).  The
// four math warps read their fragments from shared memory and release the
// stage before the MMAs.  The blob's 16-byte chunks are XOR-swizzled by the
// repack (chunk c of word row k8 stored at c ^ 2 (k8 % 4)), which makes the
// fragment reads -- 8 lanes at 4 word rows x 2 chunks -- conflict-free.
#include <algorithm>

#include "int4_common.cuh"

namespace ferret {
namespace {

constexpr int kRdWarps = 4;                 // math warps: 4 x 32 weight rows = one 128-row block
constexpr int kRdMath = kRdWarps * 32;
constexpr int kRdThreads = kRdMath + 32;    // + the copy warp
constexpr int kRdTok = 8;                   // token rows per pass: the MMA's N
constexpr int kRdMaxE = 1024;
constexpr int kRdBlob = 9216;               // bytes: 2048 packed words [k8][n] + 512 scale words
constexpr int kRdXTile = kRdTok * 128 * 2;  // 8 token rows x 128 K values, bf16
constexpr int kRdPart = 16;                 // fp32 partials per thread (4 accumulators x 4)
constexpr int kRdCtas = 3;                  // CTAs per SM
constexpr int kRdMaxStages = 8;

enum : int { RD_EMPTY = 1, RD_FULL = 2, RD_DRAIN = 3, RD_SPLIT = 4 };

struct Int4DecArgs {
    const uint8_t* blob;                    // repacked blobs [E][N/128][K/128] x kRdBlob
    const int32_t* sorted_rows;             // (token, slot) index of each sorted row
    const int32_t* offsets;                 // [E+1]
    __nv_bfloat16* out;                     // [T*topk, N or N/2] in (token, slot) order
    int N, K, E, R;
    int splits;                             // K splits per item (1: none)
    int stages;
    float* part;                            // [unit][kRdMath][kRdPart]
    int* cnt;                               // [item] finished units, zero at launch
    DevCtl ctl;
};

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (s, s) from the low / high bf16 of a scale word
__device__ __forceinline__ uint32_t rep_lo(uint32_t w) { return __byte_perm(w, 0, 0x1010); }
__device__ __forceinline__ uint32_t rep_hi(uint32_t w) { return __byte_perm(w, 0, 0x3232); }

// One 32-wide K group: four repacked words (rows 4g..4g+3 at one k8), their
// two scale words and the token row's 8 activation values -> 4 MMAs into the
// two 16-row slices' accumulators.
__device__ __forceinline__ void group_mma(const uint4 w, const uint2 sc, const uint4 x,
                                          float (&acc0)[4], float (&acc1)[4]) {
    const uint4 d0 = dequant_word(w.x, rep_lo(sc.x));   // row 4g
    const uint4 d1 = dequant_word(w.y, rep_hi(sc.x));   // row 4g+1
    const uint4 d2 = dequant_word(w.z, rep_lo(sc.y));   // row 4g+2
    const uint4 d3 = dequant_word(w.w, rep_hi(sc.y));   // row 4g+3
    mma_16816(acc0, d0.x, d1.x, d0.y, d1.y, x.x, x.y);
    mma_16816(acc0, d0.z, d1.z, d0.w, d1.w, x.z, x.w);
    mma_16816(acc1, d2.x, d3.x, d2.y, d3.y, x.x, x.y);
    mma_16816(acc1, d2.z, d3.z, d2.w, d3.w, x.z, x.w);
}

// Unit u -> (expert, first sorted row of the pass, live rows, output block,
// K-block range); the copy warp and the math warps walk the same sequence.
struct RdUnit {
    int item, e, r0, cc, ob, kb0, kb1;
};

__device__ __forceinline__ RdUnit rd_unit(int u, int S, int E, int nob, int nk,
                                          const int* it_start, const int32_t* offsets) {
    RdUnit w;
    w.item = u / S;
    const int s = u - w.item * S;
    int lo = 0, hi = E - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (it_start[mid] <= w.item) lo = mid;
        else hi = mid - 1;
    }
    w.e = lo;
    const int local = w.item - it_start[w.e];
    const int pass = local / nob;
    w.ob = local - pass * nob;
    w.r0 = __ldg(offsets + w.e) + pass * kRdTok;
    w.cc = min(kRdTok, __ldg(offsets + w.e + 1) - w.r0);
    w.kb0 = s * nk / S;
    w.kb1 = (s + 1) * nk / S;
    return w;
}

template <bool PAIR>
__global__ void __launch_bounds__(kRdThreads, kRdCtas)
    int4_w13_decode_kernel(const __grid_constant__ CUtensorMap tm_x, const Int4DecArgs args) {
    pdl_begin();
    constexpr int kW = PAIR ? 2 : 1;
    constexpr int kStage = kW * kRdBlob + kRdXTile;    // multiple of 1024
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    __shared__ int it_start[kRdMaxE + 1];
    __shared__ int scan_part[kRdThreads + 1];
    __shared__ __align__(8) uint64_t bars[2 * kRdMaxStages + 1];
    __shared__ int s_last;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int N = args.N, K = args.K, E = args.E, NS = args.stages;
    const int nk = K >> 7, nbn = N >> 7;
    const int nob = PAIR ? N >> 8 : N >> 7;          // 128-column output blocks
    const int ldo = PAIR ? N >> 1 : N;
    const int S = args.splits;
    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kRdMaxStages + s); };
    const uint32_t split_bar = bar0 + 8u * (2 * kRdMaxStages);   // math-thread rendezvous
    volatile int* abort_flag = &s_abort;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), kRdWarps);
        }
        mbar_init(split_bar, kRdMath);
        s_abort = 0;
        mbar_init_fence();
    }
    for (int e = tid; e < E; e += kRdThreads) {
        const int c = __ldg(args.offsets + e + 1) - __ldg(args.offsets + e);
        it_start[e] = c > 0 ? ((c + kRdTok - 1) / kRdTok) * nob : 0;
    }
    __syncthreads();
    block_exclusive_scan(it_start, E, scan_part);   // ends with __syncthreads
    const int units = it_start[E] * S;

    if (warp == kRdWarps) {
        // ================= copy warp =================
        if (elect_one()) {
            tma_prefetch_desc(&tm_x);
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            RingPos rp;
            int it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const RdUnit w = rd_unit(u, S, E, nob, nk, it_start, args.offsets);
                const uint8_t* bg = args.blob + ((size_t)w.e * nbn + w.ob) * nk * kRdBlob;
                const uint8_t* bu = args.blob + ((size_t)w.e * nbn + w.ob + (N >> 8)) * nk * kRdBlob;
                for (int kb = w.kb0; kb < w.kb1; ++kb, ++it, rp.advance(NS)) {
                    if (!mbar_wait(empty_bar(rp.slot), rp.phase ^ 1u, abort_flag, args.ctl, RD_EMPTY)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = smem_addr(ring + rp.slot * kStage);
                    mbar_expect_tx(full_bar(rp.slot), kStage);
                    bulk_load_hint(st, bg + (size_t)kb * kRdBlob, kRdBlob, full_bar(rp.slot), pol_w);
                    if (PAIR)
                        bulk_load_hint(st + kRdBlob, bu + (size_t)kb * kRdBlob, kRdBlob,
                                       full_bar(rp.slot), pol_w);
                    tma_load_2d_hint(st + kW * kRdBlob, &tm_x, kb * 128, w.r0, full_bar(rp.slot),
                                     pol_x);
                }
            }
            // the copies into the last stages land before the CTA may exit
            for (int i = max(0, it - NS); i < it; ++i)
                mbar_wait(full_bar(i % NS), (i / NS) & 1, abort_flag, args.ctl, RD_DRAIN, false);
        }
        return;
    }

    // ================= math warps =================
    const int g = lane >> 2, t = lane & 3;
    const int wrow = 32 * warp + 4 * g;             // this thread's rows: wrow .. wrow + 3
    // fragment offsets inside a stage (bytes): word row k8 = 4q + t of the
    // swizzled blob, the scale pair words of group q, token row g's 8 values
    const int w_off = (t * 128 + (wrow ^ (t << 3))) * 4;
    const int s_off = 8192 + ((wrow >> 1) * 4);
    const int x_off = kW * kRdBlob + g * 256 + t * 16;
    RingPos rs;
    uint32_t split_phase = 0;
    // rendezvous of the math threads (split-K): bounded and abort-aware, so a
    // warp that gave up on a wait never strands the others
    auto math_sync = [&]() -> bool {
        mbar_arrive(split_bar);
        const bool ok = mbar_wait(split_bar, split_phase & 1u, abort_flag, args.ctl, RD_SPLIT);
        ++split_phase;
        return __all_sync(0xffffffffu, ok);
    };
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const RdUnit w = rd_unit(u, S, E, nob, nk, it_start, args.offsets);
        float ag0[4] = {0, 0, 0, 0}, ag1[4] = {0, 0, 0, 0};
        float au0[4] = {0, 0, 0, 0}, au1[4] = {0, 0, 0, 0};
        bool ok = true;
        for (int kb = w.kb0; kb < w.kb1; ++kb, rs.advance(NS)) {
            ok = __all_sync(0xffffffffu,
                            mbar_wait(full_bar(rs.slot), rs.phase, abort_flag, args.ctl, RD_FULL));
            if (!ok) break;
            const uint8_t* st = ring + rs.slot * kStage;
            uint4 vg[4], vu[4], x[4];
            uint2 sg[4], su[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                vg[q] = *reinterpret_cast<const uint4*>(st + w_off + q * 4 * 512);
                sg[q] = *reinterpret_cast<const uint2*>(st + s_off + q * 256);
                if (PAIR) {
                    vu[q] = *reinterpret_cast<const uint4*>(st + kRdBlob + w_off + q * 4 * 512);
                    su[q] = *reinterpret_cast<const uint2*>(st + kRdBlob + s_off + q * 256);
                }
                x[q] = *reinterpret_cast<const uint4*>(st + x_off + q * 64);
            }
            // the fragments are in registers: the stage can be refilled
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar(rs.slot));
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                group_mma(vg[q], sg[q], x[q], ag0, ag1);
                if (PAIR) group_mma(vu[q], su[q], x[q], au0, au1);
            }
        }
        if (!ok) break;

        // accumulator element i of slice h: weight row wrow + 2h + (i >> 1),
        // token 2t + (i & 1)
        if (S > 1) {
            float* my = args.part + ((size_t)u * kRdMath + tid) * kRdPart;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                my[i] = ag0[i];
                my[4 + i] = ag1[i];
                if (PAIR) {
                    my[8 + i] = au0[i];
                    my[12 + i] = au1[i];
                }
            }
            __threadfence();
            if (!math_sync()) break;
            if (tid == 0) s_last = atomicAdd(args.cnt + w.item, 1) == S - 1;
            if (!math_sync()) break;
            if (!s_last) continue;
            __threadfence();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                ag0[i] = ag1[i] = au0[i] = au1[i] = 0.0f;
            }
            for (int j = 0; j < S; ++j) {    // split order: deterministic
                const float* p = args.part + ((size_t)(w.item * S + j) * kRdMath + tid) * kRdPart;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    ag0[i] += __ldcg(p + i);
                    ag1[i] += __ldcg(p + 4 + i);
                    if (PAIR) {
                        au0[i] += __ldcg(p + 8 + i);
                        au1[i] += __ldcg(p + 12 + i);
                    }
                }
            }
        }
        // store: for each of this thread's two tokens, its four adjacent columns
#pragma unroll
        for (int jt = 0; jt < 2; ++jt) {
            const int j = 2 * t + jt;
            if (j >= w.cc) continue;
            const int orow = __ldg(args.sorted_rows + w.r0 + j);
            float v[4] = {ag0[jt], ag0[2 + jt], ag1[jt], ag1[2 + jt]};
            if (PAIR) {
                const float u4[4] = {au0[jt], au0[2 + jt], au1[jt], au1[2 + jt]};
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = silu_mul(v[i], u4[i]);
            }
            const __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]);
            const __nv_bfloat162 p1 = __floats2bfloat162_rn(v[2], v[3]);
            uint2 pk;
            pk.x = *reinterpret_cast<const uint32_t*>(&p0);
            pk.y = *reinterpret_cast<const uint32_t*>(&p1);
            *reinterpret_cast<uint2*>(args.out + (size_t)orow * ldo + w.ob * 128 + wrow) = pk;
        }
    }
}

template <bool PAIR>
int launch_int4_decode_t(const DeviceInfo* info, const void* a_sorted, const uint8_t* blob,
                         const int32_t* sorted_rows, const int32_t* offsets, void* out, int N,
                         int K, int E, int R, cudaStream_t stream, uint8_t* split_ws,
                         size_t split_bytes, int ncnt) {
    if (E > kRdMaxE) return FERRET_ERR_SHAPE;
    constexpr int kStage = (PAIR ? 2 : 1) * kRdBlob + kRdXTile;
    CUtensorMap tm_x;
    int rc = make_tmap_2d(&tm_x, a_sorted, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, R, K, (uint64_t)K * 2,
                          128, kRdTok, false);
    if (rc != FERRET_OK) return rc;
    // stages: what kRdCtas CTAs per SM leave each (1 KB reserved per CTA, the
    // static arrays, 1 KB of alignment slack)
    const int per_cta = 233472 / kRdCtas - 1024 - (kRdMaxE + 1) * 4 - (kRdThreads + 1) * 4 - 256;
    const int stages = std::min(kRdMaxStages, (per_cta - 1024) / kStage);
    if (stages < 2) return FERRET_ERR_SHAPE;
    const int smem = stages * kStage + 1024;
    auto kern = int4_w13_decode_kernel<PAIR>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kRdThreads, smem) != cudaSuccess ||
        occ < 1) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    Int4DecArgs a;
    a.blob = blob;
    a.sorted_rows = sorted_rows;
    a.offsets = offsets;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.N = N;
    a.K = K;
    a.E = E;
    a.R = R;
    a.stages = stages;
    a.ctl = make_ctl(info);
    a.splits = 1;
    a.part = nullptr;
    a.cnt = nullptr;
    const int grid = info->num_sms * std::min(occ, kRdCtas);
    // Split K when the items cannot fill the resident CTAs: at most the bound
    // on items, splits of at least 2 K blocks, if the workspace holds the
    // partials (the counters, ncnt ints at split_ws, were cleared by the row
    // gather).
    const long long items_up = int4_decode_items_bound(R, E, N, PAIR);
    if (split_ws && items_up > 0 && items_up <= ncnt) {
        const int S = (int)std::min<long long>(grid / items_up, (K / 128) / 2);
        const size_t cnt_bytes = ((size_t)items_up * sizeof(int) + 255) & ~size_t(255);
        const size_t part_bytes = (size_t)items_up * S * kRdMath * kRdPart * sizeof(float);
        if (S >= 2 && cnt_bytes + part_bytes <= split_bytes) {
            a.splits = S;
            a.cnt = reinterpret_cast<int*>(split_ws);
            a.part = reinterpret_cast<float*>(split_ws + cnt_bytes);
        }
    }
    return launch_kernel(kern, dim3(grid), dim3(kRdThreads), smem, stream, tm_x, a);
}

}  // namespace

int launch_int4_decode(const DeviceInfo* info, const void* a_sorted, const uint8_t* blob,
                       const int32_t* sorted_rows, const int32_t* offsets, void* out, int T,
                       int topk, int N, int K, int E, int R, bool pair, cudaStream_t stream,
                       uint8_t* split_ws, size_t split_bytes, int ncnt) {
    (void)T;
    (void)topk;
    return pair ? launch_int4_decode_t<true>(info, a_sorted, blob, sorted_rows, offsets, out, N, K,
                                             E, R, stream, split_ws, split_bytes, ncnt)
                : launch_int4_decode_t<false>(info, a_sorted, blob, sorted_rows, offsets, out, N, K,
                                              E, R, stream, split_ws, split_bytes, ncnt);
}

}  // namespace ferret
