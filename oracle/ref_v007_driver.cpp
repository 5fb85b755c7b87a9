// ref_v007_driver.cpp -- runs the reference's own FP8 host reference.
//
// TEST INFRASTRUCTURE ONLY.  Linked against the object file that
// oracle/Makefile compiles, unmodified, from the reference source
// examples/fp8-group-gemm/v007_dsv3_decode_verified_105.cu (its main() is
// renamed on the compiler command line so this driver can own main()).
// Only the host functions cpu_ref_bs (v007:441-467) and prepare_sf /
// float_to_ue8m0 (v007:341-371) are called; no GPU code runs.
//
// Input file (little-endian): int32 M, N, K, E; then
//   A      u8  [M*K]
//   W      u8  [E*N*K]
//   a_sc   f32 [M*nk]
//   w_sc   f32 [E*(N/128)*nk]
//   m_idx  i32 [M]
// Output file: f32 [M*N] = cpu_ref_bs(...) with the weight scales expanded to
// one row per output column exactly as v007's main() does (v007:508-511).
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <vector>
#include <cuda.h>

void cpu_ref_bs(const uint8_t* A, const uint8_t* B, const float* a_scale,
                const float* w_scale_expanded, float* C, const int* m_indices,
                int M_total, int N, int K, int E);

// v007 references these driver entry points from its (unused) launcher.  The
// driver never calls the launcher, so inert definitions let the binary link
// and run on a machine without libcuda.
extern "C" CUresult cuInit(unsigned int) { return CUDA_ERROR_NOT_SUPPORTED; }
extern "C" CUresult cuGetErrorString(CUresult, const char** s) {
    *s = "unavailable";
    return CUDA_SUCCESS;
}
extern "C" CUresult cuTensorMapEncodeTiled(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                           const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                           const cuuint32_t*, CUtensorMapInterleave,
                                           CUtensorMapSwizzle, CUtensorMapL2promotion,
                                           CUtensorMapFloatOOBfill) {
    return CUDA_ERROR_NOT_SUPPORTED;
}

template <typename T>
static void rd(FILE* f, T* p, size_t n) {
    if (fread(p, sizeof(T), n, f) != n) {
        fprintf(stderr, "short read\n");
        exit(2);
    }
}

int main(int argc, char** argv) {
    if (argc != 3) {
        fprintf(stderr, "usage: %s in.bin out.bin\n", argv[0]);
        return 2;
    }
    FILE* f = fopen(argv[1], "rb");
    if (!f) return 2;
    int32_t hdr[4];
    rd(f, hdr, 4);
    int M = hdr[0], N = hdr[1], K = hdr[2], E = hdr[3];
    int nk = K / 128, ns = N / 128;
    std::vector<uint8_t> A((size_t)M * K), W((size_t)E * N * K);
    std::vector<float> as((size_t)M * nk), ws((size_t)E * ns * nk);
    std::vector<int> mi(M);
    rd(f, A.data(), A.size());
    rd(f, W.data(), W.size());
    rd(f, as.data(), as.size());
    rd(f, ws.data(), ws.size());
    rd(f, mi.data(), mi.size());
    fclose(f);
    std::vector<float> wexp((size_t)E * N * nk);
    for (int e = 0; e < E; e++)
        for (int n = 0; n < N; n++)
            for (int k = 0; k < nk; k++)
                wexp[((size_t)e * N + n) * nk + k] = ws[((size_t)e * ns + n / 128) * nk + k];
    std::vector<float> C((size_t)M * N);
    cpu_ref_bs(A.data(), W.data(), as.data(), wexp.data(), C.data(), mi.data(), M, N, K, E);
    FILE* o = fopen(argv[2], "wb");
    if (!o) return 2;
    fwrite(C.data(), sizeof(float), C.size(), o);
    fclose(o);
    return 0;
}
