// Copy-engine all-gather: the alternatives to the kernel's multimem.st producers
// that the reference measures in vmm/test_vmm_multicast_speed.cu:172-263.
//
//   * agg_ce_allgather     — a standalone all-gather of one shard per rank into
//                            every slab: one cudaMemcpyAsync into the multicast
//                            VA, a push ring over the peers' unicast mappings
//                            (r-1, r-2, ...), or a pull ring (r+1, r+2, ...);
//   * agg_stream_write_u32 — cuStreamWriteValue32, the copy-engine path's flag;
//   * ce_begin / ce_push_shard / ce_end — the producer side of the fused kernel
//                            in the AGG_ARGS_CE_* modes: the shard is copied in
//                            chunk order on an internal stream and each chunk's
//                            arrival flag is written on every GPU after its copy
//                            (the write is ordered after the copy by the stream
//                            and carries a memory barrier), while the kernel's
//                            loaders wait on those flags exactly as they wait on
//                            the multimem producers';
//   * ce_rs_exchange       — the reduce-scatter twin's exchange in the same way,
//                            the other direction: the internal stream waits
//                            (cuStreamWaitValue32) for the kernel to store each
//                            owner's partial block, copies it into the owner's
//                            inbox and writes the owner's arrival word.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "agg.h"
#include "agg_internal.h"

namespace agg {
namespace {

// Internal streams and events per device, created on first use: `stream`
// carries the copies; the reduce-scatter exchange can spread each copy over
// `extra` streams too (more copy engines), joined back through `ev_join`.
constexpr int kCeExtra = 3;
struct CeDev {
    std::once_flag once;
    std::mutex mu;
    int rc = AGG_OK;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    cudaStream_t extra[kCeExtra] = {};
    cudaEvent_t ev_join[kCeExtra] = {};
};
CeDev g_ce[64];

int ce_dev(int dev, CeDev** out) {
    if (dev < 0 || dev >= 64) return fail(AGG_EINVAL, "device ordinal %d out of range", dev);
    CeDev& c = g_ce[dev];
    std::call_once(c.once, [&c] {
        auto setup = [&]() -> int {
            AGG_RT(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
            AGG_RT(cudaEventCreateWithFlags(&c.ev_in, cudaEventDisableTiming));
            AGG_RT(cudaEventCreateWithFlags(&c.ev_out, cudaEventDisableTiming));
            for (int i = 0; i < kCeExtra; ++i) {
                AGG_RT(cudaStreamCreateWithFlags(&c.extra[i], cudaStreamNonBlocking));
                AGG_RT(cudaEventCreateWithFlags(&c.ev_join[i], cudaEventDisableTiming));
            }
            return AGG_OK;
        };
        c.rc = setup();
    });
    if (c.rc) return fail(c.rc, "copy-engine stream set-up failed on device %d", dev);
    *out = &c;
    return AGG_OK;
}

int copy(uint64_t dst, const void* src, size_t bytes, cudaStream_t s) {
    AGG_RT(cudaMemcpyAsync(reinterpret_cast<void*>(dst), src, bytes, cudaMemcpyDeviceToDevice, s));
    return AGG_OK;
}

int write_u32(uint64_t addr, uint32_t value, cudaStream_t s) {
    const DriverApi& d = driver();
    if (!d.ok) return fail(AGG_EDRIVER, "CUDA driver unavailable: %s", d.why.c_str());
    AGG_DRV(d.cuStreamWriteValue32(reinterpret_cast<CUstream>(s), static_cast<CUdeviceptr>(addr), value,
                                   CU_STREAM_WRITE_VALUE_DEFAULT));
    return AGG_OK;
}

int wait_geq_u32(const uint32_t* addr, uint32_t value, cudaStream_t s) {
    const DriverApi& d = driver();
    if (!d.ok) return fail(AGG_EDRIVER, "CUDA driver unavailable: %s", d.why.c_str());
    AGG_DRV(d.cuStreamWaitValue32(reinterpret_cast<CUstream>(s), reinterpret_cast<CUdeviceptr>(addr), value,
                                  CU_STREAM_WAIT_VALUE_GEQ));
    return AGG_OK;
}

}  // namespace

// Orders the internal stream after everything enqueued on `caller` so far
// (the shard is ready; this slab's previous launch, copies included, is done).
int ce_begin(cudaStream_t caller, cudaStream_t* ce) {
    int dev = 0;
    AGG_RT(cudaGetDevice(&dev));
    CeDev* c = nullptr;
    int rc = ce_dev(dev, &c);
    if (rc) return rc;
    c->mu.lock();
    cudaError_t e = cudaEventRecord(c->ev_in, caller);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(c->stream, c->ev_in, 0);
    for (int i = 0; i < kCeExtra && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(c->extra[i], c->ev_in, 0);
    if (e != cudaSuccess) {
        c->mu.unlock();
        return check_rt(e, "copy-engine stream ordering");
    }
    *ce = c->stream;
    return AGG_OK;
}

// `caller` waits for the internal stream's copies; releases the device's CE state.
int ce_end(cudaStream_t caller) {
    int dev = 0;
    AGG_RT(cudaGetDevice(&dev));
    CeDev& c = g_ce[dev];
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < kCeExtra && e == cudaSuccess; ++i) {
        e = cudaEventRecord(c.ev_join[i], c.extra[i]);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c.stream, c.ev_join[i], 0);
    }
    if (e == cudaSuccess) e = cudaEventRecord(c.ev_out, c.stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(caller, c.ev_out, 0);
    c.mu.unlock();
    if (e != cudaSuccess) return check_rt(e, "copy-engine completion");
    return AGG_OK;
}

// Copies this rank's shard (m_local rows of row_bytes) into slot `rank` of
// gathered region `region_off` on every GPU, in chunk order, a few 128-row
// chunks per copy; after each copy, writes `target` into the arrival flag of
// each chunk it carried on every GPU (flag word parity*8*1024 + rank*1024 + c).
int ce_push_shard(const agg_args* a, const void* src, int m_local, size_t row_bytes, uint64_t region_off,
                  uint32_t parity, uint32_t target, bool multicast, cudaStream_t ce) {
    const int P = a->world, r = a->dev_idx;
    const uint64_t base = a->A_peer[r];
    const uint64_t flag_off = reinterpret_cast<uint64_t>(a->A_copy_ready) - base;
    const size_t chunk_bytes = static_cast<size_t>(AGG_TILE_M) * row_bytes;
    const int num_chunks = m_local / AGG_TILE_M;
    const int per_copy = std::max(1, std::min(num_chunks, static_cast<int>((size_t(4) << 20) / chunk_bytes)));
    const uint64_t slot = region_off + static_cast<uint64_t>(r) * m_local * row_bytes;
    const uint8_t* s8 = static_cast<const uint8_t*>(src);
    int rc = AGG_OK;
    for (int c0 = 0; c0 < num_chunks && rc == AGG_OK; c0 += per_copy) {
        const int n = std::min(per_copy, num_chunks - c0);
        const uint64_t off = static_cast<uint64_t>(c0) * chunk_bytes;
        const size_t bytes = static_cast<size_t>(n) * chunk_bytes;
        for (int step = 1; step <= P && rc == AGG_OK; ++step) {
            const int d = (r - step + P) % P;  // r-1, r-2, ..., r itself last
            if (multicast) {
                if (step == 1) rc = copy(a->A_mc + slot + off, s8 + off, bytes, ce);
            } else {
                rc = copy(a->A_peer[d] + slot + off, s8 + off, bytes, ce);
            }
            for (int c = c0; c < c0 + n && rc == AGG_OK; ++c) {
                const uint64_t word = static_cast<uint64_t>(parity) * AGG_MAX_RANKS * AGG_MAX_CHUNKS +
                                      static_cast<uint64_t>(r) * AGG_MAX_CHUNKS + c;
                rc = write_u32(a->A_peer[d] + flag_off + 4 * word, target, ce);
            }
        }
    }
    return rc;
}

int ce_rs_exchange(int rank, int world, const uint64_t* inbox_slot, const uint8_t* stage, size_t slot_bytes,
                   size_t m_tile_bytes, int L, int gm, int n_tiles, uint32_t* cnt, const uint64_t* rx_word,
                   uint32_t epoch, int streams, cudaStream_t ce) {
    int dev = 0;
    AGG_RT(cudaGetDevice(&dev));
    CeDev& c = g_ce[dev];  // held by ce_begin: `ce` is c.stream
    const int n = std::max(1, std::min(streams, 1 + kCeExtra));
    const int chunks = (L + gm - 1) / gm;
    int rc = AGG_OK;
    for (int b = 1; b < world && rc == AGG_OK; ++b) {
        const int s = (rank + b) % world;
        const uint8_t* src = stage + static_cast<size_t>(s) * slot_bytes;
        bool used[1 + kCeExtra] = {};
        for (int k = 0; k < chunks && rc == AGG_OK; ++k) {
            const int rows = std::min(gm, L - k * gm);
            const size_t beg = static_cast<size_t>(k) * gm * m_tile_bytes;
            const uint32_t target = 8u * static_cast<uint32_t>(rows) * static_cast<uint32_t>(n_tiles) * epoch;
            const int i = k % n;
            cudaStream_t st = i == 0 ? ce : c.extra[i - 1];
            used[i] = true;
            rc = wait_geq_u32(cnt + s * chunks + k, target, st);
            if (rc == AGG_OK) rc = copy(inbox_slot[s] + beg, src + beg, static_cast<size_t>(rows) * m_tile_bytes, st);
        }
        for (int i = 1; i < n && rc == AGG_OK; ++i) {
            if (!used[i]) continue;
            AGG_RT(cudaEventRecord(c.ev_join[i - 1], c.extra[i - 1]));
            AGG_RT(cudaStreamWaitEvent(ce, c.ev_join[i - 1], 0));
        }
        if (rc == AGG_OK) rc = write_u32(rx_word[s], epoch, ce);  // after every chunk of the block
    }
    return rc;
}

}  // namespace agg

extern "C" {

int agg_ce_allgather(const agg_rank_info* info, uint64_t region_off, const void* src, size_t shard_bytes, int mode,
                     void* stream) {
    using namespace agg;
    if (!info) return fail(AGG_EINVAL, "agg_ce_allgather: null info");
    const int P = info->world, r = info->rank;
    if (P < 1 || P > AGG_MAX_RANKS || r < 0 || r >= P) return fail(AGG_EINVAL, "agg_ce_allgather: bad rank info");
    if (region_off + static_cast<uint64_t>(P) * shard_bytes > info->flag_off)
        return fail(AGG_EINVAL, "agg_ce_allgather: %d x %zu bytes at %llu overrun the slab's data area", P,
                    shard_bytes, static_cast<unsigned long long>(region_off));
    for (int s = 0; s < P; ++s)
        if (!info->peer_uc[s]) return fail(AGG_ESTATE, "agg_ce_allgather: rank %d's slab is not mapped here", s);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint64_t own = region_off + static_cast<uint64_t>(r) * shard_bytes;
    switch (mode) {
        case AGG_CE_MC_PUSH:
            if (!src) return fail(AGG_EINVAL, "agg_ce_allgather: null src");
            return copy(info->mc + own, src, shard_bytes, st);
        case AGG_CE_PEER_PUSH: {
            if (!src) return fail(AGG_EINVAL, "agg_ce_allgather: null src");
            for (int step = 1; step <= P; ++step) {
                const int d = (r - step + P) % P;
                int rc = copy(info->peer_uc[d] + own, src, shard_bytes, st);
                if (rc) return rc;
            }
            return AGG_OK;
        }
        case AGG_CE_PEER_PULL:
            for (int dist = 1; dist < P; ++dist) {
                const int s = (r + dist) % P;
                const uint64_t slot = region_off + static_cast<uint64_t>(s) * shard_bytes;
                int rc = copy(info->uc + slot, reinterpret_cast<const void*>(info->peer_uc[s] + slot), shard_bytes,
                              st);
                if (rc) return rc;
            }
            return AGG_OK;
        default:
            return fail(AGG_EINVAL, "agg_ce_allgather: unknown mode %d", mode);
    }
}

int agg_stream_write_u32(uint64_t addr, uint32_t value, void* stream) {
    if (!addr || addr % 4) return agg::fail(AGG_EINVAL, "agg_stream_write_u32: bad address");
    return agg::write_u32(addr, value, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
