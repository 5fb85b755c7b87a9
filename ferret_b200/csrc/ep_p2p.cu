// ep_p2p.cu -- expert-parallel W13 over NVLink peer memory (one process per
// GPU, no collective library on the data path).
//
// Every rank owns E/G experts and holds only their weights.  A step moves no
// bf16 activations: each rank quantizes its own T token rows once (1x128 FP8,
// the same bytes the single-GPU path would produce for those rows), the owner
// of an expert pulls the FP8 rows routed to it straight out of the source
// rank's memory, and the grouped GEMM's epilogue stores every output row into
// the source rank's output buffer over NVLink.  The steps on each rank:
//
//   1. quant_act  : own hidden [T, K] -> e4m3 rows + 1x128 scales in the
//                   exported buffer                               (local)
//   2. publish    : copy own top-k ids into the exported buffer, zero the
//                   output rows of invalid ids                    (local)
//      ready      : raise "ready(epoch)" on every peer, wait for every
//                   peer's (one CTA)
//      ids        : read all G*T*topk ids from the peers and map them to
//                   local experts (-1 when the expert lives elsewhere)
//                                                                 (peer loads)
//   3. permute    : stable counting sort of the G*T*topk pairs by local expert
//   4. gather     : expert-sorted FP8 rows + scales pulled from the source
//                   ranks into the local A operand                (peer loads)
//   5. grouped GEMM (swap-AB or prefill kernel) whose epilogue writes row i to
//                   row sorted[i] % (T*topk) of rank sorted[i] / (T*topk)'s
//                   output buffer                                 (peer stores)
//      With the prefill kernel (many rows per expert) steps 4 and 5 are one
//      kernel: a mover warp per CTA pulls the rows in tile order while the
//      tensor cores work on earlier tiles (each tile's loads wait for its
//      rows), the tiles are stored to a local staging matrix, and a second
//      mover warp copies each finished 128-row tile's rows to the source
//      ranks as whole rows (per-tile counters, zeroed by the ids kernel).
//   6. done       : system fence, raise "done(epoch)" on every peer, wait for
//                   every peer's -- after it every rank's output is complete
//   7. copy the exported output buffer to the caller's output (optional).
//
// The step counter (epoch) lives in device memory and is advanced by the
// ready kernel, so a captured CUDA graph of the step replays correctly.
// Every wait is bounded (the library's wait timeout); a rank that times out
// records DEV_TIMEOUT with site 20 (ready) or 21 (done) in the status word,
// turns the rest of its step into no-ops and returns -- the context is then
// out of step with its peers and must be destroyed.
//
// Buffers are exchanged as CUDA IPC handles: ferret_ep_init exports this
// rank's buffer, the caller all-gathers the handles over its own bootstrap
// (torch.distributed, MPI, a file) and hands them to ferret_ep_connect.
#include <cstring>
#include <vector>

#include "capi_internal.h"

namespace ferret {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kGatherThreads = 256;
constexpr int SITE_EP_READY = 20, SITE_EP_DONE = 21;

// Everything the EP kernels need, by value.
struct EpDev {
    int rank, world, T, topk, E, K;
    uint32_t* my_flags;                 // this rank's flag words: ready[8] at 0, done[8] at 32
    uint32_t* const* flag_peers;        // [world] every rank's flag words (self included)
    const int32_t* const* ids_peers;    // [world] every rank's exported top-k ids
    const uint8_t* const* q_peers;      // [world] every rank's e4m3 rows
    const float* const* s_peers;        // [world] every rank's 1x128 scales
    int32_t* ids_sym;                   // this rank's exported ids
    __nv_bfloat16* out_sym;             // this rank's exported output rows
    int n_out;
    const int32_t* remap;               // [E] global expert -> local expert or -1
    int32_t* all_ids;                   // [world*T*topk] local expert per pair or -1
    const int32_t* sorted;              // [world*T*topk] expert-sorted global pair index
    const int32_t* offsets;             // [El+1]
    int El;
    uint8_t* a;                         // [world*T*topk, K] gathered e4m3 rows
    float* a_s;                         // [world*T*topk, K/128]
    uint32_t* epoch;                    // device step counter
    int* failed;                        // set by a ready barrier that ran out (this step)
    int* ready;                         // [n_ready] per-tile landed-row counts of the in-GEMM pull
    int* done;                          // [n_ready] per-tile stored-warp counts for the in-GEMM push
    int n_ready;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Raise flag word `slot` (ready or done, at this rank's index) on every rank,
// then wait until every rank has raised this rank's copy to `epoch`.  Threads
// 0..world-1 each handle one rank.  Returns false when a wait ran out.
__device__ bool ep_barrier(const EpDev& d, int slot_base, uint32_t epoch, DevCtl ctl, int site) {
    const int g = threadIdx.x;
    bool ok = true;
    if (g < d.world) {
        st_release_sys(d.flag_peers[g] + slot_base + d.rank, epoch);
        const uint32_t* f = d.my_flags + slot_base + g;
        const uint64_t t0 = global_ns();
        while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
            if (global_ns() - t0 > ctl.timeout_ns) {
                ok = false;
                report(ctl, DEV_TIMEOUT | (site << 8));
                break;
            }
            __nanosleep(64);
        }
    }
    return __syncthreads_and(ok) != 0;
}

// This rank's ids into the exported buffer; output rows of invalid ids are
// zeroed here (no rank's GEMM writes them).  Grid-wide, one id per thread.
__global__ void __launch_bounds__(kGatherThreads)
    ep_publish_kernel(const EpDev d, const int32_t* __restrict__ topk_ids) {
    pdl_begin();
    const int own = d.T * d.topk;
    for (int i = blockIdx.x * kGatherThreads + threadIdx.x; i < own; i += gridDim.x * kGatherThreads) {
        const int id = topk_ids[i];
        d.ids_sym[i] = id;
        if (id < 0 || id >= d.E) {
            uint4* row = reinterpret_cast<uint4*>(d.out_sym + (size_t)i * d.n_out);
            for (int c = 0; c < d.n_out / 8; ++c) row[c] = make_uint4(0, 0, 0, 0);
        }
    }
}

// One CTA: advance the step counter, raise "ready" on every rank (after a
// system fence: the quantized rows, ids and zeroed rows written by the
// kernels before this one are visible first), wait for every rank's.
__global__ void __launch_bounds__(32, 1) ep_ready_kernel(const EpDev d, DevCtl ctl) {
    pdl_begin();
    __shared__ uint32_t s_epoch;
    if (threadIdx.x == 0) {
        s_epoch = *d.epoch + 1u;
        *d.epoch = s_epoch;
        __threadfence_system();
    }
    __syncthreads();
    const bool ok = ep_barrier(d, 0, s_epoch, ctl, SITE_EP_READY);
    if (threadIdx.x == 0) *d.failed = ok ? 0 : 1;
}

// Every rank's ids (peer loads, many CTAs) -> local expert per pair, or -1.
// After a failed ready barrier no pair is routed here: the rest of the step
// is empty and touches no peer memory.
__global__ void __launch_bounds__(kGatherThreads)
    ep_ids_kernel(const EpDev d) {
    pdl_begin();
    const int own = d.T * d.topk;
    const int total = d.world * own;
    const bool failed = *d.failed != 0;
    for (int i = blockIdx.x * kGatherThreads + threadIdx.x; i < d.n_ready; i += gridDim.x * kGatherThreads) {
        d.ready[i] = 0;     // this step's GEMM counts its pulled rows and stored tiles from zero
        d.done[i] = 0;
    }
    for (int i = blockIdx.x * kGatherThreads + threadIdx.x; i < total; i += gridDim.x * kGatherThreads) {
        int v = -1;
        if (!failed) {
            const int g = i / own;
            const int id = __ldcv(d.ids_peers[g] + (i - g * own));
            v = (id >= 0 && id < d.E) ? d.remap[id] : -1;
        }
        d.all_ids[i] = v;
    }
}

// Pull the expert-sorted rows: one warp per row, 16-byte peer loads, all of
// a lane's loads for the row (up to 16: K <= 16384) issued before any store so
// the NVLink latency is paid once per row, not once per load.
__global__ void __launch_bounds__(kGatherThreads)
    ep_gather_kernel(const EpDev d) {
    pdl_begin();
    constexpr int kMaxVec = 16;
    const int rows = d.offsets[d.El];
    const int lane = threadIdx.x & 31;
    const int nk = d.K >> 7;
    const int vec = d.K >> 4;                 // 16-byte words per row
    const int own = d.T * d.topk;
    const int warps = gridDim.x * (kGatherThreads / 32);
    for (int r = blockIdx.x * (kGatherThreads / 32) + (threadIdx.x >> 5); r < rows; r += warps) {
        const int src = d.sorted[r];
        const int g = src / own;
        const int t = (src - g * own) / d.topk;
        const uint4* q = reinterpret_cast<const uint4*>(d.q_peers[g] + (size_t)t * d.K);
        const float* s = d.s_peers[g] + (size_t)t * nk;
        uint4* dst = reinterpret_cast<uint4*>(d.a + (size_t)r * d.K);
        float sc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {         // nk <= 128
            const int c = lane + 32 * j;
            if (c < nk) sc[j] = __ldcv(s + c);
        }
        for (int base = 0; base < vec; base += 32 * kMaxVec) {   // 8 KB of the row per pass
            uint4 v[kMaxVec];
#pragma unroll
            for (int j = 0; j < kMaxVec; ++j) {
                const int c = base + lane + 32 * j;
                if (c < vec) v[j] = __ldcv(q + c);
            }
#pragma unroll
            for (int j = 0; j < kMaxVec; ++j) {
                const int c = base + lane + 32 * j;
                if (c < vec) dst[c] = v[j];
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = lane + 32 * j;
            if (c < nk) d.a_s[(size_t)r * nk + c] = sc[j];
        }
    }
}

__global__ void __launch_bounds__(32, 1) ep_done_kernel(const EpDev d, DevCtl ctl) {
    pdl_begin();
    __shared__ uint32_t s_epoch;
    if (threadIdx.x == 0) {
        __threadfence_system();     // this rank's peer stores (the GEMM) before the flag
        s_epoch = *d.epoch;
    }
    __syncthreads();
    ep_barrier(d, 32, s_epoch, ctl, SITE_EP_DONE);
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Records `ev` (if set) on stream s; inside a stream capture as an external
// record node, so a replayed graph still stamps it.
int record_event(cudaEvent_t ev, cudaStream_t s) {
    if (!ev) return FERRET_OK;
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &st) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    const cudaError_t e = st == cudaStreamCaptureStatusActive
                              ? cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal)
                              : cudaEventRecord(ev, s);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    return FERRET_OK;
}

}  // namespace
}  // namespace ferret

using namespace ferret;

// Opaque to C callers (include/ferret_moe.h declares `struct ferret_ep`).
struct ferret_ep {
    int rank = 0, world = 1, E = 0, El = 0, topk = 0, max_T = 0, K = 0, N = 0, n_out = 0;
    int flags = 0, device = -1;
    bool connected = false;
    // exported allocation: flags | q | s | ids | out
    uint8_t* sym = nullptr;
    size_t off_q = 0, off_s = 0, off_ids = 0, off_out = 0, sym_bytes = 0;
    // local allocation: tables | remap | epoch | all_ids | sorted | m_idx | offsets | a | a_s
    uint8_t* loc = nullptr;
    void** tables = nullptr;            // 5 x kMaxRanks device pointers
    int32_t* remap = nullptr;
    uint32_t* epoch = nullptr;
    int32_t *all_ids = nullptr, *sorted = nullptr, *m_idx = nullptr, *offsets = nullptr;
    int32_t* perm_ws = nullptr;         // chunked-permutation counts
    size_t perm_ws_bytes = 0;
    uint8_t* a = nullptr;
    float* a_s = nullptr;
    int* ready = nullptr;               // per-tile counters of the in-GEMM row pull
    int* done = nullptr;                // per-tile counters of the in-GEMM push
    int n_ready = 0;
    __nv_bfloat16* stage = nullptr;     // [pairs, n_out] local output rows before the push
    cudaEvent_t ev[4] = {};             // optional step-phase timing events
    uint8_t* peer_base[kMaxRanks] = {};
    bool opened[kMaxRanks] = {};
};

namespace {

void ep_free(ferret_ep* c) {
    if (!c) return;
    int prev = -1;
    cudaGetDevice(&prev);
    if (c->device >= 0) cudaSetDevice(c->device);
    for (int g = 0; g < kMaxRanks; ++g)
        if (c->opened[g]) cudaIpcCloseMemHandle(c->peer_base[g]);
    if (c->sym) cudaFree(c->sym);
    if (c->loc) cudaFree(c->loc);
    cudaGetLastError();
    if (prev >= 0) cudaSetDevice(prev);
    delete c;
}

}  // namespace

extern "C" size_t ferret_ep_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int ferret_ep_init(int rank, int world, int num_experts, int topk, int max_tokens, int K,
                              int N, int flags, const int32_t* placement, void* handle_out,
                              ferret_ep** ctx) {
    if (!ctx || !handle_out) return FERRET_ERR_NULL;
    *ctx = nullptr;
    const bool pair = (flags & FERRET_SILU_MUL) != 0;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return FERRET_ERR_SHAPE;
    if (num_experts <= 0 || num_experts % world || num_experts / world > 1024) return FERRET_ERR_SHAPE;
    if (topk <= 0 || max_tokens <= 0 || K <= 0 || K % 128 || N <= 0 || N % 128 || (pair && N % 256))
        return FERRET_ERR_SHAPE;
    if (K > 16384 || (long long)(num_experts / world) * N >= (1ll << 31)) return FERRET_ERR_SHAPE;
    const long long pairs = (long long)world * max_tokens * topk;
    if (pairs >= (1ll << 30) || pairs * K >= (1ll << 40)) return FERRET_ERR_SHAPE;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;

    ferret_ep* c = new ferret_ep;
    c->rank = rank;
    c->world = world;
    c->E = num_experts;
    c->El = num_experts / world;
    c->topk = topk;
    c->max_T = max_tokens;
    c->K = K;
    c->N = N;
    c->n_out = pair ? N / 2 : N;
    c->flags = flags;
    c->device = info->device;

    // global expert -> local expert on this rank (placement: owner-order table)
    std::vector<int32_t> remap(num_experts, -1);
    std::vector<int> seen(num_experts, 0);
    for (int slot = 0; slot < num_experts; ++slot) {
        const int e = placement ? placement[slot] : slot;
        if (e < 0 || e >= num_experts || seen[e]++) {
            delete c;
            return FERRET_ERR_SHAPE;   // not a permutation of [0, E)
        }
        if (slot / c->El == rank) remap[e] = slot % c->El;
    }

    const size_t nk = K / 128;
    size_t o = 256;   // flag words: ready[8] at 0, done[8] at 128 bytes
    c->off_q = o;
    o = align_up(o + (size_t)max_tokens * K, 256);
    c->off_s = o;
    o = align_up(o + (size_t)max_tokens * nk * 4, 256);
    c->off_ids = o;
    o = align_up(o + (size_t)max_tokens * topk * 4, 256);
    c->off_out = o;
    o = align_up(o + (size_t)max_tokens * topk * c->n_out * 2, 256);
    c->sym_bytes = o;

    size_t l = 0;
    const size_t off_tables = l;
    l += 5 * kMaxRanks * sizeof(void*);
    const size_t off_remap = l = align_up(l, 256);
    l += (size_t)num_experts * 4;
    const size_t off_epoch = l = align_up(l, 256);
    l += 256;
    const size_t off_all = l;
    l = align_up(l + (size_t)pairs * 4, 256);
    const size_t off_sorted = l;
    l = align_up(l + (size_t)pairs * 4, 256);
    const size_t off_midx = l;
    l = align_up(l + (size_t)pairs * 4, 256);
    const size_t off_offs = l;
    l = align_up(l + (size_t)(c->El + 1) * 4, 256);
    c->perm_ws_bytes = ferret_moe_permute_workspace_size(world * max_tokens, topk, c->El);
    const size_t off_pws = l;
    l = align_up(l + c->perm_ws_bytes, 256);
    const size_t off_a = l;
    l = align_up(l + (size_t)pairs * K, 256);
    const size_t off_as = l;
    l = align_up(l + (size_t)pairs * nk * 4, 256);
    c->n_ready = (int)(pairs / 128 + c->El + 1);   // >= sum over experts of ceil(rows / 128)
    const size_t off_ready = l;
    l = align_up(l + (size_t)c->n_ready * 4 * 2, 256);     // ready, then done
    const size_t off_stage = l;
    l = align_up(l + (size_t)pairs * c->n_out * 2, 256);

    if (cudaMalloc(&c->sym, c->sym_bytes) != cudaSuccess || cudaMalloc(&c->loc, l) != cudaSuccess ||
        cudaMemset(c->sym, 0, c->sym_bytes) != cudaSuccess ||
        cudaMemset(c->loc, 0, l) != cudaSuccess) {
        ep_free(c);
        return FERRET_ERR_CUDA;
    }
    c->tables = reinterpret_cast<void**>(c->loc + off_tables);
    c->remap = reinterpret_cast<int32_t*>(c->loc + off_remap);
    c->epoch = reinterpret_cast<uint32_t*>(c->loc + off_epoch);
    c->all_ids = reinterpret_cast<int32_t*>(c->loc + off_all);
    c->sorted = reinterpret_cast<int32_t*>(c->loc + off_sorted);
    c->m_idx = reinterpret_cast<int32_t*>(c->loc + off_midx);
    c->offsets = reinterpret_cast<int32_t*>(c->loc + off_offs);
    c->perm_ws = reinterpret_cast<int32_t*>(c->loc + off_pws);
    c->a = c->loc + off_a;
    c->a_s = reinterpret_cast<float*>(c->loc + off_as);
    c->ready = reinterpret_cast<int*>(c->loc + off_ready);
    c->done = c->ready + c->n_ready;
    c->stage = reinterpret_cast<__nv_bfloat16*>(c->loc + off_stage);
    cudaIpcMemHandle_t h;
    if (cudaMemcpy(c->remap, remap.data(), remap.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaIpcGetMemHandle(&h, c->sym) != cudaSuccess) {
        ep_free(c);
        return FERRET_ERR_CUDA;
    }
    std::memcpy(handle_out, &h, sizeof(h));
    *ctx = c;
    return FERRET_OK;
}

namespace {
int ep_open_peers(ferret_ep* c, const void* all_handles);
}

extern "C" int ferret_ep_connect(ferret_ep* c, const void* all_handles) {
    if (!c || !all_handles) return FERRET_ERR_NULL;
    if (c->connected) return FERRET_OK;
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(c->device) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    const int rc = ep_open_peers(c, all_handles);
    cudaSetDevice(prev);
    return rc;
}

namespace {

int ep_open_peers(ferret_ep* c, const void* all_handles) {
    const uint8_t* hs = static_cast<const uint8_t*>(all_handles);
    for (int g = 0; g < c->world; ++g) {
        if (g == c->rank) {
            c->peer_base[g] = c->sym;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + (size_t)g * sizeof(h), sizeof(h));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            return FERRET_ERR_UNSUPPORTED;   // no peer access between these GPUs
        }
        c->peer_base[g] = static_cast<uint8_t*>(p);
        c->opened[g] = true;
    }
    // device tables: flags, ids, q, s, out of every rank (identical layouts)
    void* tab[5 * kMaxRanks] = {};
    for (int g = 0; g < c->world; ++g) {
        tab[0 * kMaxRanks + g] = c->peer_base[g];
        tab[1 * kMaxRanks + g] = c->peer_base[g] + c->off_ids;
        tab[2 * kMaxRanks + g] = c->peer_base[g] + c->off_q;
        tab[3 * kMaxRanks + g] = c->peer_base[g] + c->off_s;
        tab[4 * kMaxRanks + g] = c->peer_base[g] + c->off_out;
    }
    if (cudaMemcpy(c->tables, tab, sizeof(tab), cudaMemcpyHostToDevice) != cudaSuccess)
        return FERRET_ERR_CUDA;
    c->connected = true;
    return FERRET_OK;
}

}  // namespace

extern "C" void* ferret_ep_output_buffer(ferret_ep* c) {
    return c ? static_cast<void*>(c->sym + c->off_out) : nullptr;
}

extern "C" int ferret_ep_w13_forward(ferret_ep* c, const void* hidden_bf16, const int32_t* topk_ids,
                                     int T, const void* w_fp8, const float* w_scale, void* out_bf16,
                                     void* stream) {
    if (!c) return FERRET_ERR_NULL;
    if (!c->connected) return FERRET_ERR_SHAPE;
    if (T < 0 || T > c->max_T) return FERRET_ERR_SHAPE;
    if (T == 0) return FERRET_OK;     // every rank passes the same T
    if (!hidden_bf16 || !topk_ids || !w_fp8 || !w_scale) return FERRET_ERR_NULL;
    if (!aligned16(hidden_bf16) || !aligned16(w_fp8) || (out_bf16 && !aligned16(out_bf16)) ||
        (reinterpret_cast<uintptr_t>(w_scale) & 3u) || (reinterpret_cast<uintptr_t>(topk_ids) & 3u))
        return FERRET_ERR_ALIGN;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    if (info->device != c->device) return FERRET_ERR_SHAPE;
    cudaStream_t s = as_stream(stream);
    const int own = T * c->topk;
    const int pairs = c->world * own;
    uint8_t* my = c->sym;

    // 1. own rows -> e4m3 + scales in the exported buffer
    rc = ferret_quant_act_fp8_1x128(hidden_bf16, T, nullptr, 1, T, c->K, my + c->off_q,
                                    reinterpret_cast<float*>(my + c->off_s), stream);
    if (rc != FERRET_OK) return rc;

    EpDev d;
    d.rank = c->rank;
    d.world = c->world;
    d.T = T;
    d.topk = c->topk;
    d.E = c->E;
    d.K = c->K;
    d.my_flags = reinterpret_cast<uint32_t*>(my);
    d.flag_peers = reinterpret_cast<uint32_t* const*>(c->tables + 0 * kMaxRanks);
    d.ids_peers = reinterpret_cast<const int32_t* const*>(c->tables + 1 * kMaxRanks);
    d.q_peers = reinterpret_cast<const uint8_t* const*>(c->tables + 2 * kMaxRanks);
    d.s_peers = reinterpret_cast<const float* const*>(c->tables + 3 * kMaxRanks);
    d.ids_sym = reinterpret_cast<int32_t*>(my + c->off_ids);
    d.out_sym = reinterpret_cast<__nv_bfloat16*>(my + c->off_out);
    d.n_out = c->n_out;
    d.remap = c->remap;
    d.all_ids = c->all_ids;
    d.sorted = c->sorted;
    d.offsets = c->offsets;
    d.El = c->El;
    d.a = c->a;
    d.a_s = c->a_s;
    d.epoch = c->epoch;
    d.failed = reinterpret_cast<int*>(c->epoch + 1);
    d.ready = c->ready;
    d.done = c->done;
    d.n_ready = c->n_ready;
    const DevCtl ctl = make_ctl(info);
    // the prefill kernel pulls its rows itself (own = the rows one rank receives
    // on average, the same hint the GEMM's kernel choice uses below)
    const bool pull_in_gemm = fp8_gemm_uses_prefill(own, c->El, c->flags, c->N);

    // 2. publish ids, meet the peers, read every rank's ids
    {
        const int want = (own + kGatherThreads - 1) / kGatherThreads;
        const int grid = want < info->num_sms * 4 ? want : info->num_sms * 4;
        if ((rc = launch_kernel(ep_publish_kernel, dim3(grid), dim3(kGatherThreads), 0, s, d,
                                topk_ids)) != FERRET_OK) return rc;
    }
    if ((rc = launch_kernel(ep_ready_kernel, dim3(1), dim3(32), 0, s, d, ctl)) != FERRET_OK) return rc;
    if ((rc = record_event(c->ev[0], s)) != FERRET_OK) return rc;
    {
        const int want = (pairs + kGatherThreads - 1) / kGatherThreads;
        const int grid = want < info->num_sms * 4 ? want : info->num_sms * 4;
        if ((rc = launch_kernel(ep_ids_kernel, dim3(grid), dim3(kGatherThreads), 0, s, d)) != FERRET_OK) return rc;
    }
    // 3. local expert order of all pairs
    rc = ferret_moe_permute(c->all_ids, c->world * T, c->topk, c->El, c->sorted, c->offsets,
                            c->m_idx, c->perm_ws, c->perm_ws_bytes, stream);
    if (rc != FERRET_OK) return rc;
    // 4. pull the routed FP8 rows (inside the GEMM for the prefill kernel)
    if (!pull_in_gemm) {
        const int want = (pairs + kGatherThreads / 32 - 1) / (kGatherThreads / 32);
        const int grid = want < info->num_sms * 8 ? want : info->num_sms * 8;
        if ((rc = launch_kernel(ep_gather_kernel, dim3(grid), dim3(kGatherThreads), 0, s, d)) != FERRET_OK) return rc;
    }
    // 5. grouped GEMM, epilogue stores into the source ranks' output buffers
    OutMap om;
    om.rows = c->sorted;
    om.total = pairs;
    om.peers = reinterpret_cast<__nv_bfloat16* const*>(c->tables + 4 * kMaxRanks);
    om.peer_rows = own;
    if (pull_in_gemm) {
        om.gather = true;
        om.q_peers = reinterpret_cast<const uint8_t* const*>(c->tables + 2 * kMaxRanks);
        om.s_peers = reinterpret_cast<const float* const*>(c->tables + 3 * kMaxRanks);
        om.gather_topk = c->topk;
        om.ready = c->ready;
        om.done = c->done;
    }
    if ((rc = record_event(c->ev[1], s)) != FERRET_OK) return rc;
    // (with the in-GEMM movers, `out` is the local staging matrix)
    rc = run_fp8_gemm(info, c->a, c->a_s, w_fp8, w_scale,
                      pull_in_gemm ? static_cast<void*>(c->stage) : static_cast<void*>(my + c->off_out),
                      c->offsets, 0, pairs, c->N, c->K, c->El, c->flags, own, s, om);
    if (rc != FERRET_OK) return rc;
    if ((rc = record_event(c->ev[2], s)) != FERRET_OK) return rc;
    // 6. every rank's rows have landed
    if ((rc = launch_kernel(ep_done_kernel, dim3(1), dim3(32), 0, s, d, ctl)) != FERRET_OK) return rc;
    if ((rc = record_event(c->ev[3], s)) != FERRET_OK) return rc;
    // 7. to the caller's buffer
    if (out_bf16 && out_bf16 != my + c->off_out) {
        if (cudaMemcpyAsync(out_bf16, my + c->off_out, (size_t)own * c->n_out * 2,
                            cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
            cudaGetLastError();
            return FERRET_ERR_CUDA;
        }
    }
    return FERRET_OK;
}

extern "C" int ferret_ep_set_events(ferret_ep* c, void* const* events, int n) {
    if (!c) return FERRET_ERR_NULL;
    if (n < 0 || n > 4 || (n > 0 && !events)) return FERRET_ERR_SHAPE;
    for (int i = 0; i < 4; ++i) c->ev[i] = i < n ? static_cast<cudaEvent_t>(events[i]) : nullptr;
    return FERRET_OK;
}

extern "C" int ferret_ep_destroy(ferret_ep* c) {
    if (!c) return FERRET_ERR_NULL;
    ep_free(c);
    return FERRET_OK;
}
