#pragma once
// Error-checking macros of the harness API (include/util.cuh of the reference):
//   MKERNEL_CUCHECK(cmd)  a driver call that must succeed; prints file:line and exits;
//   DKF(x) / CKF(x)       driver / runtime calls inside a bool-returning setup
//                         function: print "... (disabled)" and return false.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

using bf16 = __nv_bfloat16;

#define MKERNEL_CUCHECK(cmd)                                                                   \
    do {                                                                                       \
        CUresult mk_err_ = (cmd);                                                              \
        if (mk_err_ != CUDA_SUCCESS) {                                                         \
            const char* mk_s_ = nullptr;                                                       \
            cuGetErrorString(mk_err_, &mk_s_);                                                 \
            std::fprintf(stderr, "CUDA driver error %s:%d '%s'\n", __FILE__, __LINE__,         \
                         mk_s_ ? mk_s_ : "");                                                  \
            std::exit(EXIT_FAILURE);                                                           \
        }                                                                                      \
    } while (0)

#define DKF(x)                                                                                 \
    do {                                                                                       \
        CUresult dkf_r_ = (x);                                                                 \
        if (dkf_r_ != CUDA_SUCCESS) {                                                          \
            const char* dkf_s_ = "?";                                                          \
            cuGetErrorString(dkf_r_, &dkf_s_);                                                 \
            std::fprintf(stderr, "mInfer SP_MM: %s -> %s (disabled)\n", #x, dkf_s_);           \
            return false;                                                                      \
        }                                                                                      \
    } while (0)

#define CKF(x)                                                                                 \
    do {                                                                                       \
        cudaError_t ckf_e_ = (x);                                                              \
        if (ckf_e_ != cudaSuccess) {                                                           \
            std::fprintf(stderr, "mInfer SP_MM: %s -> %s (disabled)\n", #x,                    \
                         cudaGetErrorString(ckf_e_));                                          \
            return false;                                                                      \
        }                                                                                      \
    } while (0)
