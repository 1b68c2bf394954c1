// ORACLE — test infrastructure only.
//
// C-linkage shim around the reference's own checking helpers, compiled from
// the reference's headers where they lie (oracle/Makefile passes
// -I<reference>/include) into oracle/_ref/libref.so.  Nothing here is product
// code: it lets the tests call
//   fill_random          include/random_fill.cuh:31-60
//   read_back_as_float   include/random_fill.cuh:69-89
//   reference_matmul_cublas  include/reference_matmul.cuh:33-91
//   check_close          include/reference_matmul.cuh:99-145
// exactly as the reference harness (vmm/main.cpp:259-260,316-320) does, so the
// CPU restatement in orc_rng.c / orc_gemm.c can be pinned against them.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstring>
#include <vector>

#include "random_fill.cuh"
#include "reference_matmul.cuh"

namespace {

template <typename T>
struct ShimTensor {
    using dtype = T;
    void* raw_ptr;
    size_t n;
    size_t numel() const { return n; }
};

}  // namespace

extern "C" {

// fill_random on a bf16 tensor of n elements at device pointer `dev`
// (may be null when no GPU is present: the reference then reports the failed
// cudaMemcpy on stderr and still returns its host-side values).
int ref_fill_random_bf16(unsigned seed, float lo, float hi, size_t n, void* dev, float* host_out) {
    ShimTensor<__nv_bfloat16> t{dev, n};
    std::vector<float> v = fill_random(t, seed, lo, hi);
    if (v.size() != n) return -1;
    std::memcpy(host_out, v.data(), n * sizeof(float));
    return 0;
}

int ref_fill_random_f32(unsigned seed, float lo, float hi, size_t n, void* dev, float* host_out) {
    ShimTensor<float> t{dev, n};
    std::vector<float> v = fill_random(t, seed, lo, hi);
    if (v.size() != n) return -1;
    std::memcpy(host_out, v.data(), n * sizeof(float));
    return 0;
}

int ref_read_back_bf16(const void* dev, size_t n, float* host_out) {
    std::vector<float> v = read_back_as_float(static_cast<const __nv_bfloat16*>(dev), n);
    std::memcpy(host_out, v.data(), n * sizeof(float));
    return 0;
}

// C[M, N] = A[M, K] . B[N, K]^T through the reference's cuBLAS path.
int ref_matmul_cublas(const float* A, int M, int K, const float* B, int N, float* C_out) {
    std::vector<float> a(A, A + static_cast<size_t>(M) * K);
    std::vector<float> b(B, B + static_cast<size_t>(N) * K);
    std::vector<float> c = reference_matmul_cublas(a, M, K, b, N);
    if (c.size() != static_cast<size_t>(M) * N) return -1;
    std::memcpy(C_out, c.data(), c.size() * sizeof(float));
    return 0;
}

int ref_check_close(const float* actual, const float* expected, int rows, int cols, float atol,
                    float rtol) {
    const size_t n = static_cast<size_t>(rows) * cols;
    std::vector<float> a(actual, actual + n), e(expected, expected + n);
    return check_close(a, e, rows, cols, atol, rtol, "C") ? 1 : 0;
}

int ref_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

}  // extern "C"
