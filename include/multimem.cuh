#pragma once
// Multicast slab + multimem PTX of the harness API (include/multimem.cuh of the
// reference), on top of libagg.so:
//   kDmwChannels, kSlab, kFlagOff, RankState, extern g_rs[8]   (multimem.cuh:7-21)
//   minfer_spmm_init(rank, world, device, data_bytes)          (multimem.cuh:23)
//   mm_barrier(mc_flags, uc_flags, row, target)                (multimem.cuh:25-28),
//       here bounded: it gives up after a time limit instead of spinning forever
// plus named device wrappers for the multimem instructions the reference wrote
// inline (include/test_kernel.cuh:55-72).
//
// g_rs is defined by the harness executable, as in the reference
// (vmm/main.cpp:22).  Unlike the reference, the slab grows past 512 MiB when
// data_bytes asks for more, and minfer_spmm_finalize releases it.
#include <cuda.h>
#include <stdint.h>

#include <mutex>

#include "agg.h"

constexpr int kDmwChannels = 2;
constexpr size_t kSlab = (512ull << 20);
constexpr size_t kFlagOff = 320ull << 20;

struct RankState {
    CUdeviceptr uc = 0, mc = 0;
    unsigned ag_calls = 0, rs_calls = 0;
    bool ready = false;   // slab usable by the fused kernels
    bool mapped = false;  // slab mapped
    bool dmw = false;
    unsigned* dmw_cnt[kDmwChannels] = {nullptr, nullptr};
    unsigned* lat_cnt = nullptr;
    CUdeviceptr peer_addresses[8];
    // added: geometry of this rank's slab
    size_t slab_bytes = 0;
    size_t flag_off = 0;
};
extern RankState g_rs[8];

// Bring up this rank's slab (one host thread per GPU, rank == device).  0 / -1.
inline int minfer_spmm_init(int rank, int world, int device, size_t data_bytes) {
    if (rank < 0 || rank >= 8) return -1;
    agg_rank_info info;
    if (agg_spmm_init(rank, world, device, data_bytes, &info) != AGG_OK) {
        std::fprintf(stderr, "mInfer SP_MM: %s (disabled)\n", agg_last_error());
        return -1;
    }
    RankState& r = g_rs[rank];
    r.uc = static_cast<CUdeviceptr>(info.uc);
    r.mc = static_cast<CUdeviceptr>(info.mc);
    r.slab_bytes = info.slab_bytes;
    r.flag_off = info.flag_off;
    r.mapped = true;
    r.ready = true;
    std::printf("[rank %d] SP_MM ready: %zu MB multicast slab, flags at +%zu MB\n", rank, info.slab_bytes >> 20,
                info.flag_off >> 20);
    return 0;
}

inline int minfer_spmm_finalize(int rank) {
    if (rank < 0 || rank >= 8) return -1;
    g_rs[rank].ready = g_rs[rank].mapped = false;
    return agg_spmm_finalize(rank) == AGG_OK ? 0 : -1;
}

#ifdef __CUDACC__
// ---- multimem wrappers (16-byte vector forms are what the fused kernel uses) ----
__device__ __forceinline__ void mm_st_v4(void* mc_addr, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "r"(v.x),
                 "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void mm_st_release_b32(void* mc_addr, uint32_t v) {
    asm volatile("multimem.st.release.sys.global.b32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}
__device__ __forceinline__ void mm_red_add_u32(unsigned* mc_addr, unsigned v) {
    asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}
__device__ __forceinline__ void mm_red_add_f32(float* mc_addr, float v) {
    asm volatile("multimem.red.release.sys.global.add.f32 [%0], %1;" ::"l"(mc_addr), "f"(v) : "memory");
}
__device__ __forceinline__ float mm_ld_reduce_add_f32(const float* mc_addr) {
    float r;
    asm volatile("multimem.ld_reduce.acquire.sys.global.add.f32 %0, [%1];" : "=f"(r) : "l"(mc_addr) : "memory");
    return r;
}
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// Cross-GPU CTA barrier: thread 0 adds 1 to this CTA's flag on every GPU
// (multicast), then waits until its own GPU's copy reaches `target`.  Gives up
// after `timeout_ns` (default 10 s) and returns false instead of hanging.
constexpr int kMaxCtas = 256;
__device__ __forceinline__ bool mm_barrier(unsigned* mc_flags, const unsigned* uc_flags, int row, unsigned target,
                                           unsigned long long timeout_ns = 10000000000ull) {
    __shared__ int mm_ok;
    if (threadIdx.x == 0) {
        mm_red_add_u32(mc_flags + row * kMaxCtas + blockIdx.x, 1u);
        const unsigned* l = uc_flags + row * kMaxCtas + blockIdx.x;
        unsigned long long t0;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        unsigned v = 0;
        int ok = 1;
        for (unsigned spin = 0;; ++spin) {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(l) : "memory");
            if (v >= target) break;
            if ((spin & 63u) == 63u) {
                unsigned long long t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                if (t - t0 > timeout_ns) {
                    ok = 0;
                    break;
                }
            }
        }
        fence_proxy_alias();
        mm_ok = ok;
    }
    __syncthreads();
    return mm_ok != 0;
}
#endif
