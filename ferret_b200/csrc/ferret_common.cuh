// ferret_common.cuh -- sm_100a device helpers shared by the W13 kernels.
//
// Inline-PTX wrappers for mbarriers, TMA tile loads and the tcgen05 tensor
// core family (TMEM alloc/ld, mma, commit), plus the bounded wait every
// kernel here uses: no wait spins forever.  A wait that sees no progress for
// `timeout_ns` (measured on %globaltimer) records FERRET_DEV_TIMEOUT in the
// device status word, raises the CTA's abort flag and returns false; the
// caller then leaves its loop and the kernel tears down (drains its own
// in-flight copies and MMAs with bounded waits, frees TMEM) and returns.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

namespace ferret {

// Device status codes (low byte); the site of a timeout goes in bits 8-15.
enum DevStatus : int {
    DEV_OK = 0,
    DEV_TIMEOUT = 1,
    DEV_BAD_EXPERT = 2,   // m_indices value >= E
    DEV_LAYOUT = 3,       // an expert's rows are not contiguous
    DEV_BAD_ROW = 4,      // gather index out of range
};

struct DevCtl {
    int* status;                 // device status word (first error wins)
    unsigned long long timeout_ns;
};

__device__ __forceinline__ void report(const DevCtl& c, int code) {
    if (c.status) atomicCAS(c.status, 0, code);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ bool elect_one() {
    uint32_t is_leader = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(is_leader));
    return is_leader != 0;
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps until it completes or `hint_ns` passes, instead of spinning and
// taking issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_test_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return done != 0;
}

// Bounded wait for the phase with the given parity to complete.
//   abort_flag: CTA-wide flag in shared memory; when `respect_abort` is true
//               the wait gives up as soon as another role raised it.
//   site:       identifies the wait in the recorded status.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          const DevCtl& ctl, int site, bool respect_abort = true) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        // sleep up to 0.5 ms per try; completion wakes the thread early
        if (mbar_test_sleep(bar, parity, 500000u)) return true;
        if (respect_abort && *abort_flag) return false;
        if (global_ns() - t0 > ctl.timeout_ns) {
            *abort_flag = 1;
            report(ctl, DEV_TIMEOUT | (site << 8));
            return false;
        }
    }
}

// Position in a ring of n slots: the slot and the parity of the current lap
// (the mbarrier phase to wait for).  Advanced incrementally, so the pipeline
// loops need no integer division by a runtime stage count.
struct RingPos {
    int slot = 0;
    uint32_t phase = 0;
    __device__ __forceinline__ void advance(int n) {
        if (++slot == n) {
            slot = 0;
            phase ^= 1u;
        }
    }
};

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}

// 2-D tiled load global -> shared, completion counted on `bar` in bytes.
// The innermost coordinate x must be a multiple of 16 bytes of elements.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, int x, int y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(m), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Same, with an L2 eviction-priority hint (createpolicy result).
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* m, int x, int y,
                                                 uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(m), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}

// 3-D tiled load (same completion rule as the 2-D form).
__device__ __forceinline__ void tma_load_3d_hint(uint32_t dst, const CUtensorMap* m, int x, int y,
                                                 int z, uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
        "l"(m), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
        : "memory");
}

// Contiguous bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completion counted on `bar` in bytes.
__device__ __forceinline__ void bulk_load_hint(uint32_t dst, const void* src, uint32_t bytes,
                                               uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// Arrive once on `bar` when every tcgen05 op this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, fp8/fp6/fp4 operands, fp32 accumulate.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "setp.ne.b32 P, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, P;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= (A[smem] * 2^sfa) * (B[smem] * 2^sfb)^T, e4m3 operands with
// UE8M0 block scales read from Tensor Memory (one per row and per K=32 slice,
// scale vector 1X), fp32 accumulate.
__device__ __forceinline__ void mma_mxf8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "setp.ne.b32 P, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], P;\n\t}" ::
            "r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// ------------------------------------------------- CTA pairs (cta_group::2)
// A pair is a thread-block cluster of 2; the even CTA (rank 0) leads: it
// issues the pair's MMAs, which read A and B from both CTAs' shared memory at
// the same offsets and write each CTA's own Tensor Memory.

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Every thread of both CTAs: release this CTA's prior writes, wait for the peer.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}

// Shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

// Arrive on an mbarrier of either CTA of the cluster, with the default
// semantics (release at CTA scope) of a local arrive.  The handoffs it signals
// are ordered by the tcgen05 fences around it (Tensor Memory reads finished
// before a buffer is released); a cluster-scope release would also make every
// call wait for a memory fence, once per warp and K block.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cl_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}

// try_wait with the suspend-time hint for a barrier that also receives
// arrivals from the peer CTA (tcgen05.commit, TMA byte counts, remote
// arrives); default acquire semantics, as for the local waits.
__device__ __forceinline__ bool mbar_test_cl(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// Pair MMA: D (each CTA: its 128 rows x N) (+)= A (128 rows per CTA) * B^T (N/2
// rows per CTA), e4m3 operands, fp32 accumulate.  Leader CTA only.
__device__ __forceinline__ void mma_f8f6f4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "setp.ne.b32 P, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, P;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Block-scaled pair MMA (kind::mxf8f6f4.block_scale, cta_group::2): each CTA's
// tensor core reads the scale factors from its own Tensor Memory at the given
// addresses.  Leader CTA only.
__device__ __forceinline__ void mma_mxf8f6f4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                  uint32_t idesc, uint32_t sfa_tmem,
                                                  uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "setp.ne.b32 P, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], P;\n\t}" ::
            "r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// Arrive once on the mbarrier at shared::cluster address `cl_bar` (either CTA)
// when the pair MMAs this thread issued so far are done.
__device__ __forceinline__ void tc_commit_pair(uint32_t cl_bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     cl_bar)
                 : "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion (bytes) is
// counted on the mbarrier at shared::cluster address `cl_bar`, which may be
// the leader CTA's.  Same x alignment rule as tma_load_2d.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, int x, int y,
                                                 uint32_t cl_bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(m), "r"(x), "r"(y), "r"(cl_bar), "l"(policy)
        : "memory");
}

// mbar_wait for barriers that receive arrivals from the peer CTA of a pair.
__device__ __forceinline__ bool mbar_wait_cl(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                             const DevCtl& ctl, int site, bool respect_abort = true) {
    if (mbar_test_cl(bar, parity, 0u)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_test_cl(bar, parity, 500000u)) return true;
        if (respect_abort && *abort_flag) return false;
        if (global_ns() - t0 > ctl.timeout_ns) {
            *abort_flag = 1;
            report(ctl, DEV_TIMEOUT | (site << 8));
            return false;
        }
    }
}

// D[tmem] (+)= A[smem] * B[smem]^T, f16/bf16 operands, fp32 accumulate.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "setp.ne.b32 P, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, P;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, f16/bf16 operands, fp32 accumulate.  A sits
// row-major in Tensor Memory: row m in lane m, two 16-bit K values per column.
__device__ __forceinline__ void mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "setp.ne.b32 P, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, P;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 32 columns of 32-bit registers -> TMEM (thread l writes lane l).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
        " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// 32 lanes x 4 / 8 columns of 32-bit registers -> TMEM.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2,
                                         uint32_t r3) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr),
                 "r"(r0), "r"(r1), "r"(r2), "r"(r3)
                 : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(
                     taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
                 "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row groups 1024 bytes apart).  The
// tile base must be 1024-byte aligned; advancing along K inside the 128-byte
// row is done by adding the byte offset to `saddr`.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4)        // start address
           | ((uint64_t)1 << 16)                       // LBO (unused for swizzled K-major)
           | ((uint64_t)(1024 >> 4) << 32)             // SBO: 8 rows * 128 B
           | ((uint64_t)1 << 46)                       // fixed 0b001
           | ((uint64_t)2 << 61);                      // 128-byte swizzle
}

// Instruction descriptor: dense, D=f32, A/B K-major.
//   kind::f8f6f4 with e4m3 inputs: a_fmt = b_fmt = 0.
//   kind::f16 with bf16 inputs:    a_fmt = b_fmt = 1.
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, uint32_t a_fmt, uint32_t b_fmt) {
    return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor of the block-scaled kind::mxf8f6f4 MMA: e4m3 A and B
// (formats 0), both K-major, UE8M0 scale factors (bit 23), scale-factor ids
// (bits 4-5 for B, 29-30 for A: the byte of the 32-bit TMEM word) 0, K = 32.
// The accumulator of this kind is always f32 (no D-format field).
__host__ __device__ constexpr uint32_t make_idesc_mx(int M, int N) {
    return ((uint32_t)(N >> 3) << 17) | (1u << 23) | ((uint32_t)(M >> 4) << 24);
}

// 32 lanes x 16 columns of 32-bit TMEM -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32"
        " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 8 columns of 32-bit TMEM -> 8 registers per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 columns of 32-bit TMEM -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32"
        " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x N (16 or 32) columns -> N registers per thread.
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&v)[N]) {
    static_assert(N == 16 || N == 32, "16 or 32 columns per load");
    if constexpr (N == 16) tmem_ld16(taddr, v);
    else tmem_ld32(taddr, v);
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// (a0, a1) = (v0, v1) * s + (a0, a1) in one packed fma.rn.f32x2: each lane is
// a fused multiply-add rounded to nearest, exactly what fmaf gives, at half
// the instruction count.
__device__ __forceinline__ void ffma2(float& a0, float& a1, float v0, float v1, float s) {
    uint64_t a, v, ss;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(v0), "f"(v1));
    asm("mov.b64 %0, {%1, %1};" : "=l"(ss) : "f"(s));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(v), "l"(ss));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(a));
}

// Programmatic dependent launch: every kernel of the library is launched
// with programmatic stream serialization, so the next kernel in the stream
// can be scheduled while this one runs.  Each kernel therefore first waits
// until the previous grid in the stream has completed and its memory is
// visible (griddepcontrol.wait; a no-op without a programmatic predecessor),
// then lets its own dependent launch early.
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Warpgroup register reallocation (all threads of the warpgroup execute it):
// lower this warpgroup's per-thread register count, or raise it from the
// registers other warpgroups released.
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    return g / (1.0f + __expf(-g)) * u;
}

// Block-wide exclusive scan of data[0..n) in place; data[n] receives the
// total.  `part` needs blockDim.x ints of shared scratch.  All threads of the
// block must call it.
__device__ inline void block_exclusive_scan(int* data, int n, int* part) {
    const int nthr = blockDim.x, tid = threadIdx.x;
    const int per = (n + nthr - 1) / nthr;
    const int lo = min(n, tid * per), hi = min(n, lo + per);
    int s = 0;
    for (int i = lo; i < hi; ++i) s += data[i];
    part[tid] = s;
    __syncthreads();
    if (tid < 32) {
        const int per2 = (nthr + 31) / 32;
        const int plo = min(nthr, tid * per2), phi = min(nthr, plo + per2);
        int x = 0;
        for (int i = plo; i < phi; ++i) x += part[i];
        int inc = x;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, inc, off);
            if (tid >= off) inc += y;
        }
        int run = inc - x;
        for (int i = plo; i < phi; ++i) {
            int t = part[i];
            part[i] = run;
            run += t;
        }
        if (tid == 31) part[nthr] = inc;   // grand total (part has nthr+1 slots)
    }
    __syncthreads();
    int run = part[tid];
    for (int i = lo; i < hi; ++i) {
        int t = data[i];
        data[i] = run;
        run += t;
    }
    __syncthreads();
    if (tid == 0) data[n] = part[nthr];
    __syncthreads();
}

}  // namespace ferret
