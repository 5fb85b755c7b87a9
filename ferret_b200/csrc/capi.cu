// capi.cu -- library-wide C-ABI entry points and host helpers: version,
// error text, device facts, the device status word, TMA descriptor encoding.
#include <atomic>
#include <cstring>
#include <mutex>

#include "capi_internal.h"

namespace ferret {

// One status word per device that loads the library (first error wins).
__device__ int g_device_status;

namespace {

constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
std::once_flag g_info_once[kMaxDevices];
int g_info_err[kMaxDevices];

std::atomic<unsigned long long> g_timeout_ns{2000000000ull};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

void resolve_encode() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
}

void init_device(int dev) {
    DeviceInfo& d = g_info[dev];
    d.device = dev;
    g_info_err[dev] = FERRET_OK;
    if (cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
        g_info_err[dev] = FERRET_ERR_CUDA;
        return;
    }
    if (d.cc_major != 10) {
        g_info_err[dev] = FERRET_ERR_UNSUPPORTED;
        return;
    }
    // The status word's device address, taken once with this device current.
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) {
        g_info_err[dev] = FERRET_ERR_CUDA;
        return;
    }
    d.status = static_cast<int*>(p);
}

}  // namespace

int current_device(DeviceInfo** info) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) return FERRET_ERR_UNSUPPORTED;
    std::call_once(g_info_once[dev], init_device, dev);
    if (g_info_err[dev] != FERRET_OK) return g_info_err[dev];
    *info = &g_info[dev];
    return FERRET_OK;
}

DevCtl make_ctl(const DeviceInfo* info) {
    DevCtl c;
    c.status = info->status;
    c.timeout_ns = g_timeout_ns.load(std::memory_order_relaxed);
    return c;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t rows, uint64_t cols, uint64_t row_stride_bytes, uint32_t box_cols,
                 uint32_t box_rows, bool swizzle128) {
    std::call_once(g_encode_once, resolve_encode);
    if (!g_encode) return FERRET_ERR_UNSUPPORTED;
    if (rows == 0 || cols == 0) return FERRET_ERR_SHAPE;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    (void)elem_bytes;
    CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FERRET_OK : FERRET_ERR_CUDA;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 const uint64_t dims[3], const uint64_t strides_bytes[2], const uint32_t box[3],
                 bool swizzle128) {
    std::call_once(g_encode_once, resolve_encode);
    if (!g_encode) return FERRET_ERR_UNSUPPORTED;
    if (dims[0] == 0 || dims[1] == 0 || dims[2] == 0) return FERRET_ERR_SHAPE;
    cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
    cuuint32_t bx[3] = {box[0], box[1], box[2]};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, dtype, 3, const_cast<void*>(base), d, st, bx, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FERRET_OK : FERRET_ERR_CUDA;
}

}  // namespace ferret

using namespace ferret;

extern "C" int ferret_version(void) { return FERRET_MOE_VERSION; }

extern "C" const char* ferret_strerror(int code) {
    switch (code) {
        case FERRET_OK: return "ok";
        case FERRET_ERR_SHAPE: return "unsupported or inconsistent sizes";
        case FERRET_ERR_ALIGN: return "pointer not 16-byte aligned";
        case FERRET_ERR_NULL: return "required pointer is NULL";
        case FERRET_ERR_CUDA: return "CUDA call failed";
        case FERRET_ERR_TIMEOUT: return "device wait timed out";
        case FERRET_ERR_NCCL: return "collective failed";
        case FERRET_ERR_WORKSPACE: return "workspace missing or too small";
        case FERRET_ERR_UNSUPPORTED: return "no sm_100 device or unsupported feature";
        case FERRET_ERR_DEVICE: return "device reported a data error";
        default: return "unknown error";
    }
}

extern "C" int ferret_set_wait_timeout_ns(unsigned long long ns) {
    g_timeout_ns.store(ns ? ns : 2000000000ull, std::memory_order_relaxed);
    return FERRET_OK;
}

extern "C" int ferret_last_device_status(void* stream, int32_t* status) {
    if (!status) return FERRET_ERR_NULL;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    cudaStream_t s = as_stream(stream);
    int host = 0;
    if (cudaMemcpyAsync(&host, info->status, sizeof(int), cudaMemcpyDeviceToHost, s) !=
            cudaSuccess ||
        cudaMemsetAsync(info->status, 0, sizeof(int), s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return FERRET_ERR_CUDA;
    }
    *status = host;
    return FERRET_OK;
}

// ---------------------------------------------------------------------------
// Self-test of the bounded-wait machinery: one CTA waits on an mbarrier that
// nothing ever arrives on.  The wait must give up after `timeout_ns`, record
// DEV_TIMEOUT (site 15) in the status word and let the kernel return -- the
// same path every pipeline wait takes when a peer role stops making progress.
// ---------------------------------------------------------------------------
namespace ferret {
namespace {

__global__ void wait_timeout_selftest_kernel(DevCtl ctl) {
    pdl_begin();
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(smem_addr(&bar), 1);
        abort_flag = 0;
        mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(smem_addr(&bar), 0, &abort_flag, ctl, 15);
    __syncthreads();
}

}  // namespace
}  // namespace ferret

extern "C" int ferret_selftest_wait_timeout(unsigned long long timeout_ns, void* stream) {
    if (timeout_ns == 0 || timeout_ns > 10000000000ull) return FERRET_ERR_SHAPE;
    DeviceInfo* info = nullptr;
    int rc = current_device(&info);
    if (rc != FERRET_OK) return rc;
    DevCtl c = make_ctl(info);
    c.timeout_ns = timeout_ns;
    return launch_kernel(wait_timeout_selftest_kernel, dim3(1), dim3(32), 0, as_stream(stream), c);
}
