#pragma once
// Correctness check of the harness API (include/reference_matmul.cuh of the
// reference):
//
//   reference_matmul_cublas(A_host, M, K, B_host, N) -> C[M*N] (row-major fp32)
//       C[m, n] = sum_k A[m, k] * B[n, k]: A row-major [M, K], B row-major
//       [N, K] (the weight layout of the fused kernel), inputs uploaded as
//       bf16, cuBLAS with fp32 compute (reference_matmul.cuh:17-32, 59-77).
//       Row-major C = A . B^T is the column-major product B^T(NxK as KxN
//       transposed) . A, i.e. cublasGemmEx(T, N, N, M, K, B, ld K, A, ld K, C, ld N).
//   check_close(actual, expected, rows, cols, atol = 0.1, rtol = 0.02, label)
//       |a - e| <= atol + rtol * |e| everywhere; prints the first 5 failures
//       and the count (reference_matmul.cuh:93-145).
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <vector>

namespace agg_check {

template <typename T>
struct DevBuf {
    T* p = nullptr;
    explicit DevBuf(size_t n) {
        if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) p = nullptr;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
};

inline std::vector<__nv_bfloat16> to_bf16(const std::vector<float>& v) {
    std::vector<__nv_bfloat16> out(v.size());
    for (size_t i = 0; i < v.size(); ++i) out[i] = __float2bfloat16(v[i]);
    return out;
}

}  // namespace agg_check

inline std::vector<float> reference_matmul_cublas(const std::vector<float>& A_host, int M, int K,
                                                   const std::vector<float>& B_host, int N) {
    std::vector<float> C(static_cast<size_t>(M) * N, 0.0f);
    const std::vector<__nv_bfloat16> a = agg_check::to_bf16(A_host);
    const std::vector<__nv_bfloat16> b = agg_check::to_bf16(B_host);
    agg_check::DevBuf<__nv_bfloat16> da(a.size()), db(b.size());
    agg_check::DevBuf<float> dc(C.size());
    if (!da.p || !db.p || !dc.p) {
        std::fprintf(stderr, "reference_matmul_cublas: cudaMalloc failed\n");
        return C;
    }
    cudaMemcpy(da.p, a.data(), a.size() * sizeof(__nv_bfloat16), cudaMemcpyHostToDevice);
    cudaMemcpy(db.p, b.data(), b.size() * sizeof(__nv_bfloat16), cudaMemcpyHostToDevice);
    cublasHandle_t h = nullptr;
    if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) {
        std::fprintf(stderr, "reference_matmul_cublas: cublasCreate failed\n");
        return C;
    }
    const float one = 1.0f, zero = 0.0f;
    const cublasStatus_t st = cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, N, M, K, &one, db.p, CUDA_R_16BF, K, da.p,
                                           CUDA_R_16BF, K, &zero, dc.p, CUDA_R_32F, N, CUBLAS_COMPUTE_32F,
                                           CUBLAS_GEMM_DEFAULT);
    if (st != CUBLAS_STATUS_SUCCESS)
        std::fprintf(stderr, "reference_matmul_cublas: cublasGemmEx failed (status %d)\n", static_cast<int>(st));
    cudaMemcpy(C.data(), dc.p, C.size() * sizeof(float), cudaMemcpyDeviceToHost);
    cublasDestroy(h);
    return C;
}

inline bool check_close(const std::vector<float>& actual, const std::vector<float>& expected, int rows, int cols,
                        float atol = 1e-1f, float rtol = 2e-2f, const char* label = "C") {
    const size_t n = static_cast<size_t>(rows) * cols;
    if (actual.size() != n || expected.size() != n) {
        std::fprintf(stderr, "%s: size mismatch (actual=%zu, expected=%zu, rows*cols=%zu)\n", label, actual.size(),
                     expected.size(), n);
        return false;
    }
    long bad = 0;
    for (size_t i = 0; i < n; ++i) {
        const float a = actual[i], e = expected[i];
        const float tol = atol + rtol * std::fabs(e);
        if (!(std::fabs(a - e) <= tol)) {
            if (bad < 5)
                std::fprintf(stderr, "%s mismatch at (row %zu, col %zu): got %.4f, expected %.4f (tol %.4f)\n", label,
                             i / cols, i % cols, a, e, tol);
            ++bad;
        }
    }
    if (bad) std::fprintf(stderr, "%s: %ld/%zu elements out of tolerance\n", label, bad, n);
    return bad == 0;
}
