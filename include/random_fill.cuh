#pragma once
// Input generation of the harness API (include/random_fill.cuh of the reference):
//
//   fill_random(t, seed, lo, hi)  element i of tensor `t` is the i-th draw of
//       std::uniform_real_distribution<float>(lo, hi) over std::mt19937(seed),
//       narrowed to t's dtype (round to nearest even); the narrowed values,
//       widened back to float, are returned as the host reference, so a check
//       sees exactly the device bits (random_fill.cuh:22-30).
//   read_back_as_float(ptr, count)  copy `count` elements back and widen.
//
// `t` is any type with `raw_ptr`, `numel()` and a `dtype` member type
// (bf16, fp16, float or e4m3).  Generation is single-threaded, as in the
// reference; the same (seed, lo, hi) give the same values on every rank.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <random>
#include <type_traits>
#include <vector>

namespace agg_fill {

template <typename T>
inline T narrow(float v) {
    if constexpr (std::is_same_v<T, __nv_bfloat16>) return __float2bfloat16(v);
    else if constexpr (std::is_same_v<T, __half>) return __float2half(v);
    else if constexpr (std::is_same_v<T, __nv_fp8_e4m3>) return __nv_fp8_e4m3(v);
    else return static_cast<T>(v);
}

template <typename T>
inline float widen(T v) {
    if constexpr (std::is_same_v<T, __nv_bfloat16>) return __bfloat162float(v);
    else if constexpr (std::is_same_v<T, __half>) return __half2float(v);
    else if constexpr (std::is_same_v<T, __nv_fp8_e4m3>) return static_cast<float>(v);
    else return static_cast<float>(v);
}

inline void* device_ptr(void* p) { return p; }
inline void* device_ptr(uint64_t p) { return reinterpret_cast<void*>(static_cast<uintptr_t>(p)); }

}  // namespace agg_fill

template <typename LocalTensor>
std::vector<float> fill_random(LocalTensor& t, unsigned seed, float lo = -1.0f, float hi = 1.0f) {
    using T = typename LocalTensor::dtype;
    const size_t n = t.numel();
    std::vector<T> payload(n);
    std::vector<float> host(n);
    std::mt19937 engine(seed);
    std::uniform_real_distribution<float> draw(lo, hi);
    for (size_t i = 0; i < n; ++i) {
        payload[i] = agg_fill::narrow<T>(draw(engine));
        host[i] = agg_fill::widen<T>(payload[i]);
    }
    const cudaError_t e =
        cudaMemcpy(agg_fill::device_ptr(t.raw_ptr), payload.data(), n * sizeof(T), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) std::fprintf(stderr, "fill_random: cudaMemcpy failed -> %s\n", cudaGetErrorString(e));
    return host;
}

template <typename T>
std::vector<float> read_back_as_float(const T* device_ptr, size_t count) {
    std::vector<T> payload(count);
    const cudaError_t e = cudaMemcpy(payload.data(), device_ptr, count * sizeof(T), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) std::fprintf(stderr, "read_back_as_float: cudaMemcpy failed -> %s\n", cudaGetErrorString(e));
    std::vector<float> host(count);
    for (size_t i = 0; i < count; ++i) host[i] = agg_fill::widen<T>(payload[i]);
    return host;
}
