/*
 * ferret_moe.h -- C ABI of the B200 quantized MoE W13 (gate+up) library.
 *
 * Conventions (the ctypes shim convention of the reference,
 * tests/compare_decode_linear.py:103-129): plain device pointers and ints,
 * caller-owned buffers, the CUDA stream passed as `void*` (NULL = legacy
 * default stream), every call asynchronous on that stream.  Every entry
 * point returns 0 on success or a negative FERRET_ERR_* code; nothing throws
 * across this boundary.  Calls on distinct streams are thread-safe.
 *
 * Errors that only the device can see (a bounded wait that ran out, an
 * expert id >= E, non-contiguous expert rows) are recorded in a per-device
 * status word; read and clear it with ferret_last_device_status().
 *
 * Tensor layouts are the reference's (paths relative to xinhaoc/ferret):
 *   FP8 contiguous grouped layout   tasks/fp8-group-gemm-dsv3-decode.yaml:18-24
 *   INT4 compressed-tensors layout  baselines/kimi-moe-w13-int4/baseline_marlin.py:62-89
 */
#ifndef FERRET_MOE_H
#define FERRET_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FERRET_API __attribute__((visibility("default")))
#else
#define FERRET_API
#endif

#define FERRET_MOE_VERSION 1

/* return codes */
#define FERRET_OK 0
#define FERRET_ERR_SHAPE (-1)       /* unsupported or inconsistent sizes */
#define FERRET_ERR_ALIGN (-2)       /* a pointer misses its 16-byte alignment */
#define FERRET_ERR_NULL (-3)        /* a required pointer is NULL */
#define FERRET_ERR_CUDA (-4)        /* a CUDA runtime / driver call failed */
#define FERRET_ERR_TIMEOUT (-5)     /* a device wait ran out (status word) */
#define FERRET_ERR_NCCL (-6)        /* reserved for the collective layer */
#define FERRET_ERR_WORKSPACE (-7)   /* workspace missing or too small */
#define FERRET_ERR_UNSUPPORTED (-8) /* no sm_100 device / feature */
#define FERRET_ERR_DEVICE (-9)      /* device reported a data error */

/* flags for the GEMM entry points */
#define FERRET_SILU_MUL 0x1         /* fused SiLU(gate)*up epilogue, N_out = N/2 */
#define FERRET_TILE_SHIFT 8         /* bits 8-15: force token tile (16,32,64,128); 0 = auto */
#define FERRET_UE8M0_SCALES 0x2     /* every a_scale / w_scale is a power of two (UE8M0):
                                       plain (no SiLU) 128-token-tile launches apply them inside
                                       the tensor-core MMA (kind::mxf8f6f4.block_scale) from
                                       their exponent bits; other launches keep the exact-scale
                                       kernels (exact for such scales) */
#define FERRET_PREFILL_PAIRS 0x4    /* 128-token-tile launches on CTA pairs
                                       (tcgen05.mma.cta_group::2, 256-token x 256-row tiles over
                                       every expert's rows; with FERRET_UE8M0_SCALES the
                                       block-scaled pair kernel on whole 256-row chunks, the rest
                                       on single CTAs); same results, measured slower */

/* Library version (FERRET_MOE_VERSION). */
FERRET_API int ferret_version(void);

/* Human-readable text for a return code. */
FERRET_API const char* ferret_strerror(int code);

/* Upper bound, in nanoseconds, for any single device-side wait; 0 restores
 * the default (2 s).  Applies to launches issued after the call. */
FERRET_API int ferret_set_wait_timeout_ns(unsigned long long ns);

/* Reads and clears the current device's status word (stream-ordered on
 * `stream`, then synchronises that stream).  *status receives 0 or a device
 * code: 1 timeout (bits 8-15: wait site), 2 expert id >= E, 3 non-contiguous
 * expert rows, 4 gather index out of range. */
FERRET_API int ferret_last_device_status(void* stream, int32_t* status);

/* Self-test of the device-side failure detection: launches one CTA whose
 * only wait can never complete; the wait gives up after timeout_ns (at most
 * 10 s), records status 1 | (15 << 8) and the kernel returns.  No counterpart
 * in the reference (its waits spin forever, v007:31-41). */
FERRET_API int ferret_selftest_wait_timeout(unsigned long long timeout_ns, void* stream);

/*
 * Routing -> expert-contiguous permutation (stable counting sort).
 * Replaces: the routing sort the reference takes from vLLM's
 *   moe_align_block_size(topk_ids, block, E, ignore_invalid_experts=True)
 *   (baselines/kimi-moe-w13-int4/baseline_marlin.py:123-126) and the
 *   synthetic m_indices of baselines/fp8-group-gemm/baseline_dsv3_decode.py:50.
 * topk_ids:       int32 [T*topk] (ids outside [0,E) are dropped)
 * sorted_rows:    int32 [T*topk] flat source index t*topk+j, grouped by
 *                 expert, ascending inside an expert; -1 past the valid count
 * expert_offsets: int32 [E+1] exclusive prefix of the per-expert counts
 * m_indices:      int32 [T*topk] expert of each sorted row (-1 in the tail)
 * workspace: NULL (one CTA sorts all ids -- the fastest form for decode
 *   sizes) or ferret_moe_permute_workspace_size(T, topk, E) bytes, 4-byte
 *   aligned, which lets large batches (more than 4096 ids) sort in chunks
 *   over many CTAs.  The result is identical either way.  A size of 0 means
 *   no workspace is used at that size.  Limits: E <= 1024.
 */
FERRET_API size_t ferret_moe_permute_workspace_size(int T, int topk, int E);
FERRET_API int ferret_moe_permute(const int32_t* topk_ids, int T, int topk, int E, int32_t* sorted_rows,
                       int32_t* expert_offsets, int32_t* m_indices, void* workspace,
                       size_t ws_bytes, void* stream);

/*
 * Block-padded routing layout, the output of vLLM's
 *   moe_align_block_size(topk_ids, block_size, E, ignore_invalid_experts=True)
 *   (baselines/kimi-moe-w13-int4/baseline_marlin.py:123-126), built from the
 *   stable permutation above.
 * ferret_moe_align_block_size_sizes: max_padded = T*topk + E*(block_size-1)
 *   (at most T*topk*block_size when T*topk < E), max_blocks =
 *   ceil(max_padded / block_size) -- vLLM's buffer sizes.
 * sorted_ids [max_padded]: every expert's flat (token, slot) indices in
 *   ascending order, padded to a multiple of block_size with T*topk (also
 *   past the used length); expert_ids [max_blocks]: the expert of each block,
 *   -1 past the used blocks; num_tokens_post_pad [1]: the padded length.
 * Ids outside [0, E) are dropped.  Order inside an expert is the ascending
 * flat index (vLLM's own order inside an expert is not specified).
 * workspace: ferret_moe_align_block_size_workspace_size(T, topk, E) bytes,
 * 4-byte aligned.  Limits: E <= 1024.
 */
FERRET_API int ferret_moe_align_block_size_sizes(int T, int topk, int E, int block_size,
                                                  int* max_padded, int* max_blocks);
FERRET_API size_t ferret_moe_align_block_size_workspace_size(int T, int topk, int E);
FERRET_API int ferret_moe_align_block_size(const int32_t* topk_ids, int T, int topk, int E,
                                           int block_size, int32_t* sorted_ids,
                                           int32_t* expert_ids, int32_t* num_tokens_post_pad,
                                           void* workspace, size_t ws_bytes, void* stream);

/*
 * Per-token 1x128 FP8 activation quantization (with optional row gather).
 * Replaces: DeepGEMM per_token_cast_to_fp8(x, use_ue8m0=False)
 *   (baselines/fp8-group-gemm/baseline_dsv3_decode.py:42).
 * x_bf16:      bf16 [x_rows, K]
 * gather_rows: NULL (row r reads x row r; needs R <= x_rows) or int32 [R]:
 *              row r reads x row gather_rows[r] / gather_div (negative ->
 *              zero row, scale 0; a source row >= x_rows is skipped like a
 *              negative one and reported as device status 4)
 * a_fp8:       e4m3 [R, K]; a_scale: f32 [R, K/128] row-major
 * amax is clamped at 1e-4; f = fl(fl(1/amax)*448); q = e4m3_satfinite(fl(x*f));
 * scale = fl(amax/448).
 * Limits: K % 128 == 0.
 */
FERRET_API int ferret_quant_act_fp8_1x128(const void* x_bf16, int x_rows, const int32_t* gather_rows,
                                          int gather_div, int R, int K, void* a_fp8,
                                          float* a_scale, void* stream);

/*
 * The same quantizer with power-of-two (UE8M0) scales, the input of
 * FERRET_UE8M0_SCALES.
 * Replaces: DeepGEMM per_token_cast_to_fp8(x, use_ue8m0=True).
 * Arguments and layouts as ferret_quant_act_fp8_1x128.  amax is clamped at
 * 1e-4; scale = the smallest power of two >= fl(amax/448) (exact, from the
 * fp32 bits); q = e4m3_satfinite(x * (1/scale)) (an exact product).
 */
FERRET_API int ferret_quant_act_fp8_1x128_ue8m0(const void* x_bf16, int x_rows,
                                                const int32_t* gather_rows, int gather_div, int R,
                                                int K, void* a_fp8, float* a_scale, void* stream);

/*
 * Quantize-and-scatter form of the 1x128 activation quantizer (the A operand
 * of the W13 grouped GEMM in one pass from the token-ordered hidden states):
 * each token row of x_bf16 [T, K] is quantized once (the algorithm of
 * ferret_quant_act_fp8_1x128, or of its UE8M0 form with flags =
 * FERRET_UE8M0_SCALES) and written to the expert-sorted rows of its top-k
 * pairs: row p of a_fp8 [T*topk, K] / a_scale [T*topk, K/128] gets token
 * sorted_rows[p] / topk for every p < expert_offsets[E] (sorted_rows and
 * expert_offsets [E+1] from ferret_moe_permute); rows from expert_offsets[E]
 * on are not written.  Bit-identical to ferret_quant_act_fp8_1x128 with
 * gather_rows = sorted_rows, gather_div = topk on those rows.
 * inv_ws: int32 [T*topk] scratch (the inverse permutation), caller-owned.
 * No reference counterpart as one call: it replaces per_token_cast_to_fp8
 * (baselines/fp8-group-gemm/baseline_dsv3_decode.py:42) followed by the row
 * order the grouped GEMM needs.  Limits: K % 128 == 0.
 */
FERRET_API int ferret_quant_act_fp8_1x128_scatter(const void* x_bf16, int T, int topk,
                                                  const int32_t* sorted_rows,
                                                  const int32_t* expert_offsets, int E, int K,
                                                  void* a_fp8, float* a_scale, int32_t* inv_ws,
                                                  int flags, void* stream);

/*
 * Row gather of quantized rows (no reference counterpart; an alternative to
 * the gathered quantizer above with identical output): out row r = row
 * rows[r] / div of q_fp8 [src_rows, K] / q_scale [src_rows, K/128]
 * (negative -> zero row and scale; a source row >= src_rows is treated like
 * a negative one and reported as device status 4).  Quantizing T token rows
 * once and gathering their T*topk routed copies saves topk-fold quantizer
 * arithmetic at prefill sizes.  Limits: K % 128 == 0; 16-byte aligned rows.
 */
FERRET_API int ferret_fp8_gather_rows(const void* q_fp8, const float* q_scale, int src_rows,
                                      const int32_t* rows, int div, int R, int K, void* out_fp8,
                                      float* out_scale, void* stream);

/*
 * FP8 block-scaled grouped GEMM, contiguous layout, W13 (gate+up).
 * Replaces: DeepGEMM m_grouped_fp8_gemm_nt_contiguous((A, A_scale),
 *   (W, W_scale), out, m_indices, disable_ue8m0_cast=True)
 *   (baselines/fp8-group-gemm/baseline_dsv3_decode.py:55-57,68-70) and the
 *   reference kernel launcher launch_grouped_gemm_bs
 *   (examples/fp8-group-gemm/v007_dsv3_decode_verified_105.cu:373-439).
 * a_fp8 [M,K] e4m3, a_scale [M,K/128] f32, w_fp8 [E,N,K] e4m3,
 * w_scale [E,N/128,K/128] f32, out_bf16 [M,N] (or [M,N/2] with
 * FERRET_SILU_MUL: out = silu(x[:, :N/2]) * x[:, N/2:]).
 * Rows of one expert must be contiguous; rows with m_indices < 0 are padding
 * and their output rows are not written.
 * expert_offsets: NULL -> the expert segments are derived on the device from
 *   m_indices (needs ferret_fp8_grouped_gemm_workspace_size() bytes of
 *   workspace); non-NULL int32 [E+1] -> rows [off[e], off[e+1]) belong to
 *   expert e (m_indices is then not read and may be NULL).
 * workspace (4-byte aligned): with M <= 4096, ferret_fp8_grouped_gemm_workspace_size
 *   also reserves room for split-K: a launch with fewer tiles than half the
 *   SMs then splits K over them and reduces the fp32 partials in a fixed order
 *   (deterministic).  A smaller workspace (or NULL with expert_offsets) only
 *   disables the split.
 * Limits: K % 128 == 0, N % 128 == 0 (N % 256 == 0 with SILU), E <= 1024,
 *   K <= 16384; pointers 16-byte aligned.
 */
FERRET_API int ferret_fp8_grouped_gemm_nt_contiguous(const void* a_fp8, const float* a_scale, const void* w_fp8,
                                          const float* w_scale, void* out_bf16,
                                          const int32_t* m_indices, const int32_t* expert_offsets,
                                          int M, int N, int K, int E, int flags, void* workspace,
                                          size_t ws_bytes, void* stream);

/*
 * Scatter-output form of the FP8 grouped GEMM: expert segments from
 * expert_offsets [E+1] over the rows of a_fp8 [M, K], and expert-sorted row i
 * written to output row out_rows[i] of out_bf16 [out_total, N or N/2] (rows
 * whose out_rows entry lies outside [0, out_total) are skipped).  With
 * out_rows = ferret_moe_permute's sorted_rows the result lands directly in
 * (token, slot) order -- the order Marlin's MoE output uses
 * (baselines/kimi-moe-w13-int4/baseline_marlin.py:140-168) and the one the
 * expert-parallel combine needs.  Same limits as
 * ferret_fp8_grouped_gemm_nt_contiguous.
 */
FERRET_API int ferret_fp8_grouped_gemm_scatter(const void* a_fp8, const float* a_scale,
                                               const void* w_fp8, const float* w_scale,
                                               void* out_bf16, const int32_t* expert_offsets,
                                               const int32_t* out_rows, int M, int out_total, int N,
                                               int K, int E, int flags, void* stream);

/* Workspace bytes ferret_fp8_grouped_gemm_nt_contiguous needs when
 * expert_offsets is NULL. */
FERRET_API size_t ferret_fp8_grouped_gemm_workspace_size(int M, int E);

/*
 * Allocation-free variant of ferret_fp8_grouped_gemm_nt_contiguous (m_indices
 * form).  No counterpart in the reference: it exists for callers that cannot
 * allocate device memory when they call -- a serving process that has handed
 * almost all HBM to weights and the KV cache, or a plugin host that reaches
 * this library through an FFI and has no access to its framework's allocator.
 * Same arguments as the workspace entry point with expert_offsets = NULL,
 * minus the workspace, and the same kernel choice; results agree with that
 * entry point within the GEMM's tolerance, not always bit for bit (without a
 * workspace there is no split-K, which the workspace entry point uses for
 * launches with few tiles).  The per-expert segments derived
 * from m_indices live in a fixed 8 KB device array inside this library
 * (2 x 1024 int32), which every GPU that loads the library keeps until the
 * process exits.  It allocates nothing and calls no allocator.
 * Limit: E <= 1024 (the array's size); larger E returns FERRET_ERR_SHAPE.
 * The first call on a device looks up the array's device address with that
 * device current; make that first call before any stream capture (a lookup
 * that fails returns FERRET_ERR_CUDA and is retried by the next call).
 * All calls share the one array and each call rewrites the entries it uses
 * before reading them; calls that overlap on the GPU (e.g. on two streams at
 * once) race on it and must be serialised by the caller.
 */
FERRET_API int ferret_fp8_grouped_gemm_nt_contiguous_noalloc(
    const void* a_fp8, const float* a_scale, const void* w_fp8, const float* w_scale,
    void* out_bf16, const int32_t* m_indices, int M, int N, int K, int E, int flags, void* stream);

/*
 * One-time (load-time) repack of raw compressed-tensors INT4 W13 weights and
 * their scales into the blob ferret_int4_moe_w13 reads: for every expert,
 * 128-row n block and 128-wide K block, 9216 contiguous bytes = 2048 int32
 * words [k/8][n ^ 8 (k/8 mod 4)] (the 8 nibbles of each word reordered to K
 * offsets {0,2,4,6,1,3,5,7}; the XOR spreads the kernels' shared-memory reads
 * over all banks) followed by the 4 x 128 bf16 group scales [k/32][n].
 * The one-time pre-permutation the reference contract allows
 * (tasks/kimi-moe-w13-int4-grouped-gemm.yaml:69-71); it replaces the Marlin
 * repack gptq_marlin_moe_repack (baselines/kimi-moe-w13-int4/baseline_marlin.py:80-82).
 * w_raw int32 [E, K/8, N] (offset-8 nibbles, low nibble first along K),
 * w_scale_bf16 [E, K/32, N], w_blob: ferret_int4_blob_bytes(E, K, N) bytes.
 * Limits: K % 128 == 0, N % 128 == 0.
 */
FERRET_API size_t ferret_int4_blob_bytes(int E, int K, int N);
FERRET_API int ferret_int4_repack_w13(const int32_t* w_raw, const void* w_scale_bf16, void* w_blob,
                                      int E, int K, int N, void* stream);

/*
 * Top-k weighted combine after the W2 (down) projection -- the step that
 * completes the MoE layer.  No reference counterpart: the reference times the
 * grouped GEMMs alone (its W2 shapes: tasks/fp8-group-gemm-dsv3-decode.yaml:67-86).
 * out[t, h] = bf16(sum_j w[t, j] * y[t*topk + j, h]), fp32 in slot order,
 * pairs whose topk_ids entry is outside [0, E) skipped (topk_ids may be NULL:
 * every pair counts).  y_bf16 [T*topk, H] in (token, slot) order -- the
 * scatter grouped GEMM with out_rows = sorted_rows writes it so;
 * topk_weights f32 [T, topk]; out_bf16 [T, H].  Limits: H % 8 == 0.
 */
FERRET_API int ferret_moe_combine(const void* y_bf16, const float* topk_weights,
                                  const int32_t* topk_ids, int E, int T, int topk, int H,
                                  void* out_bf16, void* stream);

/*
 * INT4 W4A16 grouped GEMM for the W13 projection (group-32 symmetric bf16
 * scales, offset-8 nibbles), optional fused SiLU(gate)*up.
 * Replaces: vLLM ops.moe_wna16_marlin_gemm(...) followed by
 *   apply_moe_activation(SILU, ...) (baselines/kimi-moe-w13-int4/baseline_marlin.py:140-168).
 * hidden_bf16 [T, K]; w_blob from ferret_int4_repack_w13; sorted_rows /
 * expert_offsets from ferret_moe_permute (T*topk flat (token, slot) indices
 * grouped by expert).  out_bf16 [T*topk, N] (or [T*topk, N/2] with
 * FERRET_SILU_MUL), row p = (token p/topk, slot p%topk) -- Marlin's output
 * order; rows of dropped pairs are not written.  The workspace receives the
 * expert-sorted activation rows: ferret_int4_moe_w13_workspace_size() bytes,
 * 16-byte aligned.
 * Limits: K % 128 == 0, N % 128 == 0 (N % 256 == 0 with SILU), E <= 1024.
 */
FERRET_API size_t ferret_int4_moe_w13_workspace_size(int T, int topk, int K);
FERRET_API int ferret_int4_moe_w13(const void* hidden_bf16, const void* w_blob,
                                   const int32_t* sorted_rows, const int32_t* expert_offsets,
                                   void* out_bf16, int T, int topk, int N, int K, int E, int flags,
                                   void* workspace, size_t ws_bytes, void* stream);

/*
 * Expert-parallel FP8 W13 over NVLink peer memory, one process per GPU.
 * No reference counterpart: the reference has no multi-GPU implementation of
 * this path.  The entry points keep its shim conventions
 * (tests/compare_decode_linear.py:110-128: raw device pointers and ints,
 * caller-owned buffers, stream as void*, int status) and the per-rank result
 * equals the single-GPU ferret_fp8_grouped_gemm_nt_contiguous output for the
 * rank's own (token, slot) pairs.
 *
 * Setup, on every rank with its GPU current:
 *   ferret_ep_init(rank, world, E, topk, max_tokens, K, N, flags, placement,
 *                  handle, &ctx)  -- allocates this rank's buffers and writes
 *                  its ferret_ep_handle_bytes()-byte export handle;
 *   all-gather the handles in rank order over any bootstrap;
 *   ferret_ep_connect(ctx, handles) -- maps every peer's buffers.
 * placement: NULL (rank r owns experts [r*E/world, (r+1)*E/world)) or a host
 * array of E distinct expert ids in owner order (slot i on rank i/(E/world)).
 * flags: FERRET_SILU_MUL and the token-tile bits, as for the grouped GEMM.
 *
 * Step (every rank, same T <= max_tokens, collective over the ranks):
 *   ferret_ep_w13_forward(ctx, hidden [T, K] bf16, topk_ids [T, topk] int32
 *       (global expert ids; ids outside [0, E) give zero rows),
 *       T, w_fp8 [E/world, N, K] e4m3 and w_scale [E/world, N/128, K/128] f32
 *       of this rank's experts in placement order, out [T*topk, N or N/2]
 *       bf16 in (token, slot) order or NULL to leave the result in
 *       ferret_ep_output_buffer(ctx), stream).
 * It enqueues kernels only (no host synchronisation, no allocation), so a
 * step can be captured in a CUDA graph.  A peer that does not arrive within
 * the wait timeout makes the step record a device timeout
 * (ferret_last_device_status: 1 | site << 8, site 20 or 21); the context is
 * then out of step and must be destroyed.
 * ferret_ep_destroy: only after every rank's last step has completed.
 */
typedef struct ferret_ep ferret_ep;
FERRET_API size_t ferret_ep_handle_bytes(void);
FERRET_API int ferret_ep_init(int rank, int world, int num_experts, int topk, int max_tokens, int K,
                              int N, int flags, const int32_t* placement, void* handle_out,
                              ferret_ep** ctx);
FERRET_API int ferret_ep_connect(ferret_ep* ctx, const void* all_handles);
FERRET_API int ferret_ep_w13_forward(ferret_ep* ctx, const void* hidden_bf16, const int32_t* topk_ids,
                                     int T, const void* w_fp8, const float* w_scale, void* out_bf16,
                                     void* stream);
FERRET_API void* ferret_ep_output_buffer(ferret_ep* ctx);
/*
 * Optional step-phase timing: up to 4 cudaEvent_t handles (passed as void*,
 * created by the caller with timing enabled) that every later
 * ferret_ep_w13_forward records on its stream -- [0] after the ready barrier,
 * [1] before the grouped GEMM (after the permutation and, for decode-sized
 * batches, the separate row pull), [2] after the GEMM, [3] after the done
 * barrier.  Inside a stream capture they become external record nodes, so a
 * replayed graph stamps them.  n = 0 turns the recording off.
 */
FERRET_API int ferret_ep_set_events(ferret_ep* ctx, void* const* events, int n);
FERRET_API int ferret_ep_destroy(ferret_ep* ctx);

#ifdef __cplusplus
}
#endif

#endif /* FERRET_MOE_H */
