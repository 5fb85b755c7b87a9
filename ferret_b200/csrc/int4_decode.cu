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
#include <algorithm>

#include "int4_common.cuh"

namespace ferret {
namespace {

constexpr int kRdWarps = 4;                 // 4 warps x 32 weight rows = one 128-row block
constexpr int kRdThreads = kRdWarps * 32;
constexpr int kRdTok = 8;                   // token rows per pass: the MMA's N
constexpr int kRdMaxE = 1024;
constexpr int kRdBlobWords = 2304;          // 2048 packed words [k8][n] + 256 scale words
constexpr int kRdPart = 16;                 // fp32 partials per thread (4 accumulators x 4)

struct Int4DecArgs {
    const uint32_t* blob;                   // repacked blobs [E][N/128][K/128] x 2304 words
    const __nv_bfloat16* a;                 // [R, K] expert-sorted activation rows
    const int32_t* sorted_rows;             // (token, slot) index of each sorted row
    const int32_t* offsets;                 // [E+1]
    __nv_bfloat16* out;                     // [T*topk, N or N/2] in (token, slot) order
    int N, K, E, R;
    int splits;                             // K splits per item (1: none)
    float* part;                            // [unit][kRdThreads][kRdPart]
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

template <bool PAIR>
__global__ void __launch_bounds__(kRdThreads, 4)
    int4_w13_decode_kernel(const Int4DecArgs args) {
    pdl_begin();
    __shared__ int it_start[kRdMaxE + 1];
    __shared__ int scan_part[kRdThreads + 1];
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int N = args.N, K = args.K, E = args.E;
    const int nk = K >> 7, nbn = N >> 7;
    const int nob = PAIR ? N >> 8 : N >> 7;          // 128-column output blocks
    const int ldo = PAIR ? N >> 1 : N;
    const int S = args.splits;

    for (int e = tid; e < E; e += kRdThreads) {
        const int c = __ldg(args.offsets + e + 1) - __ldg(args.offsets + e);
        it_start[e] = c > 0 ? ((c + kRdTok - 1) / kRdTok) * nob : 0;
    }
    __syncthreads();
    block_exclusive_scan(it_start, E, scan_part);
    const int items = it_start[E];

    for (int u = blockIdx.x; u < items * S; u += gridDim.x) {
        const int item = u / S, s = u - item * S;
        int lo = 0, hi = E - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (it_start[mid] <= item) lo = mid;
            else hi = mid - 1;
        }
        const int e = lo;
        const int local = item - it_start[e];
        const int pass = local / nob, ob = local - pass * nob;
        const int r0 = __ldg(args.offsets + e) + pass * kRdTok;
        const int cc = min(kRdTok, __ldg(args.offsets + e + 1) - r0);
        const int kb0 = s * nk / S, kb1 = (s + 1) * nk / S;

        // this thread's rows: 32*warp + 4g .. +3 of the gate (or plain) block
        // and of the up block
        const int nb_g = ob, nb_u = ob + (N >> 8);
        const uint32_t* bg = args.blob + ((size_t)e * nbn + nb_g) * nk * kRdBlobWords;
        const uint32_t* bu = args.blob + ((size_t)e * nbn + nb_u) * nk * kRdBlobWords;
        const int wrow = 32 * warp + 4 * g;
        const bool live = g < cc;
        const __nv_bfloat16* xrow = args.a + (size_t)(r0 + (live ? g : 0)) * K;

        float ag0[4] = {0, 0, 0, 0}, ag1[4] = {0, 0, 0, 0};
        float au0[4] = {0, 0, 0, 0}, au1[4] = {0, 0, 0, 0};
        for (int kb = kb0; kb < kb1; ++kb) {
            const uint32_t* wg = bg + (size_t)kb * kRdBlobWords;
            const uint32_t* wu = bu + (size_t)kb * kRdBlobWords;
            uint4 vg[4], vu[4], x[4];
            uint2 sg[4], su[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                vg[q] = __ldcs(reinterpret_cast<const uint4*>(wg + (4 * q + t) * 128 + wrow));
                sg[q] = __ldcs(reinterpret_cast<const uint2*>(wg + 2048 + ((q * 128 + wrow) >> 1)));
                if (PAIR) {
                    vu[q] = __ldcs(reinterpret_cast<const uint4*>(wu + (4 * q + t) * 128 + wrow));
                    su[q] = __ldcs(reinterpret_cast<const uint2*>(wu + 2048 + ((q * 128 + wrow) >> 1)));
                }
                x[q] = live ? __ldg(reinterpret_cast<const uint4*>(xrow + kb * 128 + 8 * (4 * q + t)))
                            : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                group_mma(vg[q], sg[q], x[q], ag0, ag1);
                if (PAIR) group_mma(vu[q], su[q], x[q], au0, au1);
            }
        }

        // accumulator element i of slice h: weight row wrow + 2h + (i >> 1),
        // token 2t + (i & 1)
        if (S > 1) {
            float* my = args.part + ((size_t)u * kRdThreads + tid) * kRdPart;
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
            __syncthreads();
            if (tid == 0) s_last = atomicAdd(args.cnt + item, 1) == S - 1;
            __syncthreads();
            if (!s_last) continue;
            __threadfence();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                ag0[i] = ag1[i] = au0[i] = au1[i] = 0.0f;
            }
            for (int j = 0; j < S; ++j) {    // split order: deterministic
                const float* p = args.part + ((size_t)(item * S + j) * kRdThreads + tid) * kRdPart;
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
            if (j >= cc) continue;
            const int orow = __ldg(args.sorted_rows + r0 + j);
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
            *reinterpret_cast<uint2*>(args.out + (size_t)orow * ldo + ob * 128 + wrow) = pk;
        }
    }
}

}  // namespace

int launch_int4_decode(const DeviceInfo* info, const void* a_sorted, const uint8_t* blob,
                       const int32_t* sorted_rows, const int32_t* offsets, void* out, int T,
                       int topk, int N, int K, int E, int R, bool pair, cudaStream_t stream,
                       uint8_t* split_ws, size_t split_bytes, int ncnt) {
    (void)T;
    (void)topk;
    if (E > kRdMaxE) return FERRET_ERR_SHAPE;
    Int4DecArgs a;
    a.blob = reinterpret_cast<const uint32_t*>(blob);
    a.a = static_cast<const __nv_bfloat16*>(a_sorted);
    a.sorted_rows = sorted_rows;
    a.offsets = offsets;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.N = N;
    a.K = K;
    a.E = E;
    a.R = R;
    a.ctl = make_ctl(info);
    a.splits = 1;
    a.part = nullptr;
    a.cnt = nullptr;
    constexpr int kCtasPerSm = 4;
    const int grid = info->num_sms * kCtasPerSm;
    // Split K when the items cannot fill the resident CTAs: at most the bound
    // on items, splits of at least 2 K blocks, if the workspace holds the
    // partials (the counters, ncnt ints at split_ws, were cleared by the row
    // gather).
    const long long items_up = int4_decode_items_bound(R, E, N, pair);
    if (split_ws && items_up > 0 && items_up <= ncnt) {
        const int S = (int)std::min<long long>(grid / items_up, (K / 128) / 2);
        const size_t cnt_bytes = ((size_t)items_up * sizeof(int) + 255) & ~size_t(255);
        const size_t part_bytes = (size_t)items_up * S * kRdThreads * kRdPart * sizeof(float);
        if (S >= 2 && cnt_bytes + part_bytes <= split_bytes) {
            a.splits = S;
            a.cnt = reinterpret_cast<int*>(split_ws);
            a.part = reinterpret_cast<float*>(split_ws + cnt_bytes);
        }
    }
    return pair ? launch_kernel(int4_w13_decode_kernel<true>, dim3(grid), dim3(kRdThreads), 0, stream, a)
                : launch_kernel(int4_w13_decode_kernel<false>, dim3(grid), dim3(kRdThreads), 0, stream, a);
}

}  // namespace ferret
