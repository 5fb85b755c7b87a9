/*
 * ferret_oracle.c -- CPU restatement of the quantized MoE W13 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg compare the CUDA
 * library against.  Nothing in the shipped product path (ferret_b200/) links,
 * loads or calls it.
 *
 * Every function states the reference code it restates (paths relative to
 * the xinhaoc/ferret repository):
 *
 *   orc_e4m3_to_f32 / orc_f32_to_e4m3   e4m3fn format (max 448, NaN 0x7F/0xFF),
 *       docs/quantization/fp8-fp4-guide.md:5-11; the host decode the reference
 *       kernels use is __nv_cvt_fp8_to_halfraw(..., __NV_E4M3)
 *       (examples/fp8-group-gemm/v007_dsv3_decode_verified_105.cu:458-459).
 *   orc_quant_act_fp8_1x128            DeepGEMM per_token_cast_to_fp8 as
 *       called at baselines/fp8-group-gemm/baseline_dsv3_decode.py:42
 *       (use_ue8m0=False) with the layout of
 *       tasks/fp8-group-gemm-dsv3-decode.yaml:18-24; orc_quant_act_fp8_1x128_ue8m0
 *       the use_ue8m0=True form (power-of-two scales, the input of the
 *       block-scaled UE8M0 MMA of
 *       examples/fp8-group-gemm/v007_dsv3_decode_verified_105.cu:262).
 *   orc_fp8_grouped_gemm               the host reference cpu_ref_bs of
 *       examples/fp8-group-gemm/v007_dsv3_decode_verified_105.cu:441-467
 *       (same per-128-K-block fp32 dot, then sum += dot*sfa*sfb) but with
 *       exact fp32 scales (no UE8M0 rounding, v007:454-455) and the expert
 *       taken per row from m_indices (v007:449-450 uses the first row of the
 *       128-row tile, a defect for ragged groups).
 *   orc_moe_permute                    the expert-contiguous order that
 *       m_indices describes (tasks/fp8-group-gemm-dsv3-prefill.yaml:18-21,
 *       baselines/fp8-group-gemm/baseline_dsv3_decode.py:50) produced from
 *       top-k ids as vLLM's moe_align_block_size is used at
 *       baselines/kimi-moe-w13-int4/baseline_marlin.py:123-126: a stable
 *       counting sort of the flat (token*topk + slot) index by expert.
 *   orc_int4_w13                       fp32_oracle_w13_silu of
 *       correctness/compare_marlin_vs_ref.py:44-100: low-nibble-first unpack,
 *       minus 8, times the bf16 group-32 scale, round to bf16, fp32 matvec,
 *       SiLU(gate)*up in fp32, round to bf16.
 *
 * Compiled with -ffp-contract=off so no fused multiply-add changes the
 * rounding of the restated formulas.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* scalar formats                                                      */
/* ------------------------------------------------------------------ */

ORC_API float orc_e4m3_to_f32(uint8_t v) {
    int sign = v >> 7;
    int exp = (v >> 3) & 0xF;
    int man = v & 0x7;
    float r;
    if (exp == 0xF && man == 0x7) return NAN;
    if (exp == 0)
        r = ldexpf((float)man, -9);               /* subnormal: m * 2^-9 */
    else
        r = ldexpf(1.0f + (float)man / 8.0f, exp - 7);
    return sign ? -r : r;
}

/* fp32 -> e4m3fn, round to nearest even, saturating to +-448 (the
 * __NV_SATFINITE behaviour; the quantizers below never produce a magnitude
 * above 448*(1+2^-23), which rounds to 448 under either convention). */
ORC_API uint8_t orc_f32_to_e4m3(float f) {
    uint8_t sign = signbit(f) ? 0x80 : 0x00;
    float a = fabsf(f);
    if (isnan(f)) return (uint8_t)(sign | 0x7F);
    if (a >= 448.0f) return (uint8_t)(sign | 0x7E);
    int code;
    if (a < 0.015625f) {                          /* below 2^-6: step 2^-9 */
        float n = nearbyintf(a * 512.0f);         /* exact scaling, RNE */
        code = (int)n;                            /* n == 8 is 2^-6, code 0x08 */
    } else {
        int e2;
        frexpf(a, &e2);                           /* a = m * 2^e2, m in [0.5,1) */
        int e = e2 - 1;                           /* a in [2^e, 2^(e+1)) */
        float n = nearbyintf(ldexpf(a, 3 - e));   /* in [8, 16] */
        code = ((e + 7) << 3) + ((int)n - 8);
    }
    if (code > 0x7E) code = 0x7E;
    return (uint8_t)(sign | code);
}

ORC_API float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

ORC_API uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if (isnan(f)) return 0x7FC0;
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float silu_mul(float g, float u) {
    /* correctness/compare_marlin_vs_ref.py:94-97 */
    float s = g / (1.0f + expf(-g));
    return s * u;
}

/* ------------------------------------------------------------------ */
/* routing permutation                                                 */
/* ------------------------------------------------------------------ */

/* topk_ids: [T*topk] flat.  Ids outside [0,E) are dropped (the
 * ignore_invalid_experts=True call of baseline_marlin.py:123-126).
 * sorted_rows[R]: flat source index, expert-contiguous, ascending within an
 * expert; positions past the valid count hold -1.  expert_offsets[E+1].
 * m_indices[R]: expert of each sorted row, -1 in the tail. */
ORC_API void orc_moe_permute(const int32_t* topk_ids, int T, int topk, int E,
                             int32_t* sorted_rows, int32_t* expert_offsets,
                             int32_t* m_indices) {
    long R = (long)T * topk;
    int32_t* cursor = (int32_t*)calloc((size_t)E + 1, sizeof(int32_t));
    for (long i = 0; i < R; i++) {
        int e = topk_ids[i];
        if (e >= 0 && e < E) cursor[e + 1]++;
    }
    expert_offsets[0] = 0;
    for (int e = 0; e < E; e++) expert_offsets[e + 1] = expert_offsets[e] + cursor[e + 1];
    for (int e = 0; e < E; e++) cursor[e] = expert_offsets[e];
    for (long i = 0; i < R; i++) {
        int e = topk_ids[i];
        if (e < 0 || e >= E) continue;
        int pos = cursor[e]++;
        sorted_rows[pos] = (int32_t)i;
        m_indices[pos] = e;
    }
    for (long p = expert_offsets[E]; p < R; p++) {
        sorted_rows[p] = -1;
        m_indices[p] = -1;
    }
    free(cursor);
}

/* ------------------------------------------------------------------ */
/* per-token 1x128 activation quantization                             */
/* ------------------------------------------------------------------ */

/* x: bf16 [rows_src, K].  Output row r reads source row
 * gather_rows ? gather_rows[r] / gather_div : r.  q: e4m3 [R, K];
 * scale: f32 [R, K/128] row-major.  The published per_token_cast_to_fp8
 * algorithm as torch executes it: amax clamped at 1e-4,
 * f = fl(fl(1/amax) * 448) (torch's `448.0 / t` is reciprocal-then-multiply),
 * q = e4m3_rne_satfinite(fl(x * f)), scale = fl(amax / 448). */
static void quant_act(const uint16_t* x, const int32_t* gather_rows, int gather_div, int R,
                      int K, uint8_t* q, float* scale, int ue8m0) {
    int nk = K / 128;
    for (int r = 0; r < R; r++) {
        long src = r;
        if (gather_rows) {
            int g = gather_rows[r];
            if (g < 0) {                            /* tail row: zero */
                memset(q + (long)r * K, 0, (size_t)K);
                for (int b = 0; b < nk; b++) scale[(long)r * nk + b] = 0.0f;
                continue;
            }
            src = g / (gather_div > 0 ? gather_div : 1);
        }
        const uint16_t* xr = x + src * (long)K;
        for (int b = 0; b < nk; b++) {
            float amax = 0.0f;
            for (int i = 0; i < 128; i++) {
                float v = fabsf(orc_bf16_to_f32(xr[b * 128 + i]));
                if (v > amax) amax = v;
            }
            if (amax < 1e-4f) amax = 1e-4f;
            float f, sc;
            if (ue8m0) {
                /* smallest power of two >= fl(amax/448), from the fp32 bits */
                float s0 = amax / 448.0f;
                uint32_t bits, ex, sb, fb;
                memcpy(&bits, &s0, 4);
                ex = (bits >> 23) + ((bits & 0x7FFFFFu) ? 1u : 0u);
                sb = ex >= 255u ? 0x7F800000u : ex << 23;
                fb = ex >= 255u ? 0u : ex == 254u ? 0x00400000u : (254u - ex) << 23;
                memcpy(&sc, &sb, 4);
                memcpy(&f, &fb, 4);
            } else {
                /* torch evaluates `448.0 / amax` as reciprocal(amax) * 448 */
                f = (1.0f / amax) * 448.0f;
                sc = amax / 448.0f;
            }
            for (int i = 0; i < 128; i++)
                q[(long)r * K + b * 128 + i] = orc_f32_to_e4m3(orc_bf16_to_f32(xr[b * 128 + i]) * f);
            scale[(long)r * nk + b] = sc;
        }
    }
}

ORC_API void orc_quant_act_fp8_1x128(const uint16_t* x, const int32_t* gather_rows,
                                     int gather_div, int R, int K, uint8_t* q,
                                     float* scale) {
    quant_act(x, gather_rows, gather_div, R, K, q, scale, 0);
}

/* The use_ue8m0=True form of the same quantizer (DeepGEMM
 * per_token_cast_to_fp8(x, use_ue8m0=True)): the scale is rounded up to a
 * power of two -- here exactly, from the fp32 bits, rather than through a
 * floating-point log2 -- and x is multiplied by its exact inverse. */
ORC_API void orc_quant_act_fp8_1x128_ue8m0(const uint16_t* x, const int32_t* gather_rows,
                                           int gather_div, int R, int K, uint8_t* q,
                                           float* scale) {
    quant_act(x, gather_rows, gather_div, R, K, q, scale, 1);
}

/* ------------------------------------------------------------------ */
/* FP8 grouped GEMM (contiguous layout)                                */
/* ------------------------------------------------------------------ */

/* a: e4m3 [M, K], a_scale: f32 [M, K/128], w: e4m3 [E, N, K],
 * w_scale: f32 [E, ceil(N/128), K/128], m_indices: [M] (rows < 0 skipped).
 * out: f32 [M, N] (silu=0) or [M, N/2] (silu=1: gate cols [0,N/2), up cols
 * [N/2,N)).  Skipped rows are left untouched. */
ORC_API void orc_fp8_grouped_gemm(const uint8_t* a, const float* a_scale, const uint8_t* w,
                                  const float* w_scale, const int32_t* m_indices, int M,
                                  int N, int K, int E, int silu, float* out) {
    int nk = K / 128;
    int nsn = (N + 127) / 128;
    float lut[256];
    for (int i = 0; i < 256; i++) lut[i] = orc_e4m3_to_f32((uint8_t)i);
    float* acc = (float*)malloc(sizeof(float) * (size_t)N);
    float* arow = (float*)malloc(sizeof(float) * (size_t)K);
    for (int m = 0; m < M; m++) {
        int e = m_indices[m];
        if (e < 0 || e >= E) continue;
        for (int k = 0; k < K; k++) arow[k] = lut[a[(long)m * K + k]];
        for (int n = 0; n < N; n++) {
            const uint8_t* wr = w + ((long)e * N + n) * K;
            float sum = 0.0f;
            for (int kb = 0; kb < nk; kb++) {
                float sfa = a_scale[(long)m * nk + kb];
                float sfb = w_scale[((long)e * nsn + n / 128) * nk + kb];
                float dot = 0.0f;
                for (int k = kb * 128; k < kb * 128 + 128; k++) dot += arow[k] * lut[wr[k]];
                sum += dot * sfa * sfb;
            }
            acc[n] = sum;
        }
        if (silu) {
            int h = N / 2;
            for (int j = 0; j < h; j++) out[(long)m * h + j] = silu_mul(acc[j], acc[h + j]);
        } else {
            memcpy(out + (long)m * N, acc, sizeof(float) * (size_t)N);
        }
    }
    free(acc);
    free(arow);
}

/* ------------------------------------------------------------------ */
/* INT4 W4A16 grouped GEMM                                             */
/* ------------------------------------------------------------------ */

/* Dequantized weight of expert e at (k, n): bf16((nib - 8) * scale).
 * raw_q: int32 [E, K/8, N], low nibble first along K, offset 8.
 * scales: bf16 [E, K/32, N]. */
static float int4_weight(const int32_t* raw_q, const uint16_t* scales, int N, int K, int e,
                         int k, int n) {
    uint32_t word = (uint32_t)raw_q[((long)e * (K / 8) + k / 8) * N + n];
    int nib = (int)((word >> (4 * (k % 8))) & 0xFu);
    float s = orc_bf16_to_f32(scales[((long)e * (K / 32) + k / 32) * N + n]);
    float v = (float)(nib - 8) * s;
    return orc_bf16_to_f32(orc_f32_to_bf16(v));
}

/* hidden: bf16 [T, K]; topk_ids: [T*topk]; out row p = t*topk + j (the
 * (token, slot) order of correctness/compare_marlin_vs_ref.py:89-98).
 * silu=1: out f32 [T*topk, N/2]; silu=0: out f32 [T*topk, N].  Pairs with an
 * invalid expert id are left untouched. */
ORC_API void orc_int4_w13(const uint16_t* hidden, const int32_t* raw_q, const uint16_t* scales,
                          const int32_t* topk_ids, int T, int topk, int N, int K, int E,
                          int silu, float* out) {
    float* wcol = (float*)malloc(sizeof(float) * (size_t)K);
    float* acc = (float*)malloc(sizeof(float) * (size_t)N);
    float* arow = (float*)malloc(sizeof(float) * (size_t)K);
    for (int t = 0; t < T; t++) {
        for (int k = 0; k < K; k++) arow[k] = orc_bf16_to_f32(hidden[(long)t * K + k]);
        for (int j = 0; j < topk; j++) {
            int e = topk_ids[t * topk + j];
            if (e < 0 || e >= E) continue;
            for (int n = 0; n < N; n++) {
                for (int k = 0; k < K; k++) wcol[k] = int4_weight(raw_q, scales, N, K, e, k, n);
                float s = 0.0f;
                for (int k = 0; k < K; k++) s += arow[k] * wcol[k];
                acc[n] = s;
            }
            long p = (long)t * topk + j;
            if (silu) {
                int h = N / 2;
                for (int c = 0; c < h; c++) out[p * h + c] = silu_mul(acc[c], acc[h + c]);
            } else {
                memcpy(out + p * N, acc, sizeof(float) * (size_t)N);
            }
        }
    }
    free(wcol);
    free(acc);
    free(arow);
}
