// Multicast primitives and their checks:
//   * agg_mc_broadcast      — 16-byte multimem.st push of a local buffer into the
//                             multicast VA (the multicast-bandwidth sweep; the
//                             copy-engine push of vmm/test_vmm_multicast_speed.cu:172-194
//                             done by SMs instead);
//   * agg_verify_*          — byte-exact checks (vmm/test_vmm_multicast_speed.cu:99-126);
//   * agg_multimem_ops_test — the reference's multimem smoke (include/test_kernel.cuh:46-74);
//   * agg_mm_barrier        — the cross-GPU CTA barrier of vmm/multimem.cu:103-119,
//                             with a bounded wait;
//   * agg_wait_flag         — a bounded device wait on a flag (failure detection).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "agg.h"
#include "agg_internal.h"
#include "agg_ptx.cuh"

namespace agg {
namespace {

constexpr int kCopyThreads = 512;
constexpr int kUnroll = 4;

__global__ void __launch_bounds__(kCopyThreads) mc_broadcast_kernel(const uint4* __restrict__ src,
                                                                    uint4* mc_dst, size_t n16,
                                                                    uint32_t* flag_mc) {
    const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = tid; i < n16; i += stride * kUnroll) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const size_t j = i + u * stride;
            if (j < n16) v[u] = __ldg(src + j);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const size_t j = i + u * stride;
            if (j < n16) mm_st_v4(mc_dst + j, v[u]);
        }
    }
    if (flag_mc) {
        fence_acq_rel_sys();
        __syncthreads();
        if (threadIdx.x == 0) mm_red_add_release_u32(flag_mc, 1u);
    }
}

__device__ __forceinline__ unsigned long long block_sum(unsigned long long v) {
    __shared__ unsigned long long part[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) part[w] = v;
    __syncthreads();
    unsigned long long s = 0;
    if (threadIdx.x == 0)
        for (int i = 0; i < (blockDim.x + 31) / 32; ++i) s += part[i];
    return s;
}

__global__ void verify_bytes_kernel(const uint64_t* __restrict__ a, const uint64_t* __restrict__ b,
                                    size_t words, unsigned long long* mismatches) {
    unsigned long long bad = 0;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < words;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        bad += (a[i] != b[i]) ? 1ull : 0ull;
    const unsigned long long s = block_sum(bad);
    if (threadIdx.x == 0 && s) atomicAdd(mismatches, s);
}

__global__ void verify_pattern_gather_kernel(const uint64_t* __restrict__ g, size_t words_per_shard,
                                             int world, unsigned long long* mismatches) {
    constexpr uint64_t kRepeated = 0x0101010101010101ull;
    const size_t total = words_per_shard * static_cast<size_t>(world);
    unsigned long long bad = 0;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint64_t expect = static_cast<uint64_t>(i / words_per_shard + 1) * kRepeated;
        bad += (g[i] != expect) ? 1ull : 0ull;
    }
    const unsigned long long s = block_sum(bad);
    if (threadIdx.x == 0 && s) atomicAdd(mismatches, s);
}

__global__ void alias_fence_kernel() {
    if (blockIdx.x == 0 && threadIdx.x == 0) fence_proxy_alias();
}

// Record layout of include/test_kernel.cuh:12-17.
struct alignas(16) McRecord {
    float reduce_input;
    float store_output;
    float red_target;
    float reduced_local;
};

__global__ void multimem_ops_kernel(McRecord* mc, float* reduced_out, float addend) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    const float sum = mm_ld_reduce_add_acquire_f32(&mc->reduce_input);
    mm_st_release_b32(&mc->store_output, __float_as_uint(sum));
    mm_red_add_release_f32(&mc->red_target, addend);
    fence_proxy_alias();
    *reduced_out = sum;
}

__global__ void ld_reduce_v4_kernel(const float* mc_src, float4* out, size_t n4) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = mm_ld_reduce_add_v4_f32(mc_src + 4 * i);
}

__global__ void red_add_v4_kernel(float* mc_dst, float addend, size_t n4) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        mm_red_add_v4_f32(mc_dst + 4 * i, addend, addend, addend, addend);
}

constexpr int kMaxBarrierCtas = 256;  // vmm/multimem.cu:103

__global__ void mm_barrier_kernel(uint32_t* mc_flags, const uint32_t* uc_flags, int row, uint32_t target,
                                  uint32_t* status, unsigned long long timeout_ns) {
    if (threadIdx.x == 0) {
        Deadline dl{globaltimer_ns() + timeout_ns, status};
        const int idx = row * kMaxBarrierCtas + static_cast<int>(blockIdx.x);
        mm_red_add_release_u32(mc_flags + idx, 1u);
        if (!wait_flag_geq(uc_flags + idx, target, dl))
            record_failure(status, AGG_ROLE_BARRIER, blockIdx.x);
        fence_proxy_alias();
    }
    __syncthreads();
}

__global__ void wait_flag_kernel(const uint32_t* flag, uint32_t target, uint32_t* status,
                                 unsigned long long timeout_ns) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        Deadline dl{globaltimer_ns() + timeout_ns, status};
        if (!wait_flag_geq(flag, target, dl)) record_failure(status, AGG_ROLE_FLAG, 0u);
    }
}

int default_blocks() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace
}  // namespace agg

using namespace agg;

extern "C" {

int agg_mc_broadcast(const void* src, uint64_t mc_dst, size_t bytes, uint32_t* flag_mc, int num_blocks,
                     void* stream) {
    if (!src || !mc_dst) return fail(AGG_EINVAL, "agg_mc_broadcast: null pointer");
    if (bytes % 16 || reinterpret_cast<uintptr_t>(src) % 16 || mc_dst % 16)
        return fail(AGG_EINVAL, "agg_mc_broadcast: pointers and size must be 16-byte multiples");
    const size_t n16 = bytes / 16;
    int blocks = num_blocks > 0 ? num_blocks : default_blocks();
    mc_broadcast_kernel<<<blocks, kCopyThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src), reinterpret_cast<uint4*>(mc_dst), n16, flag_mc);
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

int agg_verify_bytes(const void* data, const void* expect, size_t bytes, unsigned long long* mismatches,
                     void* stream) {
    if (!data || !expect || !mismatches) return fail(AGG_EINVAL, "agg_verify_bytes: null pointer");
    if (bytes % 8) return fail(AGG_EINVAL, "agg_verify_bytes: size must be a multiple of 8");
    verify_bytes_kernel<<<1024, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint64_t*>(data), static_cast<const uint64_t*>(expect), bytes / 8, mismatches);
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

int agg_verify_pattern_gather(const void* gathered, size_t shard_bytes, int world,
                              unsigned long long* mismatches, void* stream) {
    if (!gathered || !mismatches || world < 1) return fail(AGG_EINVAL, "agg_verify_pattern_gather: bad args");
    if (shard_bytes % 8) return fail(AGG_EINVAL, "agg_verify_pattern_gather: shard size must be a multiple of 8");
    verify_pattern_gather_kernel<<<1024, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint64_t*>(gathered), shard_bytes / 8, world, mismatches);
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

int agg_alias_fence(void* stream) {
    alias_fence_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>();
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

int agg_multimem_ops_test(uint64_t mc_rec, float* reduced_out, float addend, void* stream) {
    if (!mc_rec || !reduced_out || mc_rec % 16) return fail(AGG_EINVAL, "agg_multimem_ops_test: bad pointer");
    multimem_ops_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<McRecord*>(mc_rec),
                                                                       reduced_out, addend);
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

int agg_multimem_ld_reduce_v4(uint64_t mc_src, float* out, size_t n4, void* stream) {
    if (!mc_src || !out || mc_src % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return fail(AGG_EINVAL, "agg_multimem_ld_reduce_v4: bad pointer");
    const int blocks = static_cast<int>(std::min<size_t>((n4 + 255) / 256, 4096));
    if (blocks == 0) return AGG_OK;
    ld_reduce_v4_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const float*>(mc_src), reinterpret_cast<float4*>(out), n4);
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

int agg_multimem_red_add_v4(uint64_t mc_dst, float addend, size_t n4, void* stream) {
    if (!mc_dst || mc_dst % 16) return fail(AGG_EINVAL, "agg_multimem_red_add_v4: bad pointer");
    const int blocks = static_cast<int>(std::min<size_t>((n4 + 255) / 256, 4096));
    if (blocks == 0) return AGG_OK;
    red_add_v4_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<float*>(mc_dst),
                                                                            addend, n4);
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

int agg_mm_barrier(uint32_t* mc_flags, const uint32_t* uc_flags, int row, uint32_t target, int blocks,
                   uint32_t* status, uint64_t timeout_ns, void* stream) {
    if (!mc_flags || !uc_flags || blocks < 1 || blocks > kMaxBarrierCtas || row < 0)
        return fail(AGG_EINVAL, "agg_mm_barrier: bad args");
    mm_barrier_kernel<<<blocks, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        mc_flags, uc_flags, row, target, status, timeout_ns ? timeout_ns : 10000000000ull);
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

int agg_wait_flag(const uint32_t* flag, uint32_t target, uint32_t* status, uint64_t timeout_ns, void* stream) {
    if (!flag) return fail(AGG_EINVAL, "agg_wait_flag: null flag");
    wait_flag_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag, target, status,
                                                                      timeout_ns ? timeout_ns : 1000000000ull);
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

}  // extern "C"
