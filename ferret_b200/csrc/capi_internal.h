// capi_internal.h -- host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cstdint>
#include <utility>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/ferret_moe.h"
#include "ferret_common.cuh"

namespace ferret {

// Per-device facts resolved once: SM count, shared-memory limit, address of
// the status word, compute capability.
struct DeviceInfo {
    int device = -1;
    int num_sms = 0;
    int max_smem_optin = 0;
    int cc_major = 0, cc_minor = 0;
    int* status = nullptr;
};

// Fills `info` for the current device; returns FERRET_OK or an error code.
int current_device(DeviceInfo** info);

// Builds the DevCtl passed to every kernel launch.
DevCtl make_ctl(const DeviceInfo* info);

// 2-D tensor map over a row-major [rows, cols] matrix of `elem_bytes`
// elements with a (box_cols x box_rows) box.  swizzle128 selects the
// 128-byte swizzle (box_cols * elem_bytes must then be 128).
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t rows, uint64_t cols, uint64_t row_stride_bytes, uint32_t box_cols,
                 uint32_t box_rows, bool swizzle128);

// 3-D tensor map: dims[0] innermost (elements), byte strides of dims 1 and 2,
// box[0..2]; 128-byte swizzle when swizzle128.
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 const uint64_t dims[3], const uint64_t strides_bytes[2], const uint32_t box[3],
                 bool swizzle128);

// Where the grouped GEMM writes expert-sorted row i: row i of `out` (rows ==
// nullptr), or row rows[i] (skipped outside [0, total)).  With a peer table,
// output row o goes to row o % peer_rows of buffer peers[o / peer_rows] -- a
// device array of G pointers, other GPUs' memory included.
struct OutMap {
    const int32_t* rows = nullptr;
    int total = 0;
    __nv_bfloat16* const* peers = nullptr;
    int peer_rows = 0;
    // Expert parallelism, prefill kernel only (requires `rows` and `peers`):
    // the GEMM moves the rows itself.  Expert-sorted row i is row
    // (rows[i] % peer_rows) / gather_topk of rank rows[i] / peer_rows, read
    // from q_peers (e4m3, K bytes per row) and s_peers (K/128 fp32 scales per
    // row) into row i of the A operand and its scales before any tile reads
    // it; the tiles are stored to row i of `out` (a local staging matrix) and
    // then copied to row rows[i] % peer_rows of peers[rows[i] / peer_rows].
    // ready[m] / done[m] count rows landed / warp-tiles stored for 128-row
    // tile m and must be zero when the launch starts.
    bool gather = false;
    const uint8_t* const* q_peers = nullptr;
    const float* const* s_peers = nullptr;
    int gather_topk = 0;
    int* ready = nullptr;
    int* done = nullptr;
};

// Workspace for split-K of the swap-AB kernel: tile counters (zeroed before
// the launch) and fp32 partials; part == nullptr disables splitting.
struct SplitWs {
    int* cnt = nullptr;
    float* part = nullptr;
    size_t bytes = 0;
    int smax = 1;
};

// Whether run_fp8_gemm takes the prefill kernel (128-token tiles) for these
// arguments (rows_hint = expected rows holding data).
bool fp8_gemm_uses_prefill(int rows_hint, int E, int flags, int N);

// FP8 grouped GEMM launch shared by the entry points: picks the prefill kernel
// or the swap-AB token tile from rows_hint (expected rows holding data) and E.
int run_fp8_gemm(const DeviceInfo* info, const void* a, const float* a_scale, const void* w,
                 const float* w_scale, void* out, const int32_t* seg, int seg_pairs, int M, int N,
                 int K, int E, int flags, int rows_hint, cudaStream_t s, const OutMap& om,
                 const SplitWs& sw = SplitWs{});

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Launches a library kernel with programmatic stream serialization (the
// kernel starts with pdl_begin()); returns FERRET_OK or FERRET_ERR_CUDA.
template <typename... KArgs, typename... Args>
inline int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                         cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    return FERRET_OK;
}

// True when `kern` launches with at least `regs` registers per thread.  A
// kernel whose warpgroups trade registers with setmaxnreg assumes the launch
// total (threads x registers) its split adds up to; with fewer, an increase
// could never be granted.
template <typename... KArgs>
inline bool kernel_has_regs(void (*kern)(KArgs...), int regs) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return fa.numRegs >= regs;
}

// The same for a kernel of CTA pairs (thread-block clusters of 2 along x).
// grid.x must be even.
template <typename... KArgs, typename... Args>
inline int launch_kernel_pairs(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    return FERRET_OK;
}

// How many CTA pairs of `kern` (block threads, smem bytes) can be resident at
// once; 0 if the query fails.
template <typename... KArgs>
inline int max_resident_pairs(void (*kern)(KArgs...), dim3 block, size_t smem) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// Maps a launch error to FERRET_ERR_CUDA (and clears it).
inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FERRET_OK : FERRET_ERR_CUDA;
}

}  // namespace ferret
