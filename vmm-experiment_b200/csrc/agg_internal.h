// Host-side internals shared by the library's translation units: the CUDA
// driver entry points (fetched through the runtime, so libagg.so has no link
// dependency on libcuda and loads on machines without a GPU driver), and the
// per-thread error message behind agg_last_error().
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <string>

#include "agg.h"

namespace agg {

#define AGG_DRIVER_FUNCS(X)             \
    X(cuInit)                           \
    X(cuGetErrorString)                 \
    X(cuDeviceGet)                      \
    X(cuDeviceGetAttribute)             \
    X(cuMemCreate)                      \
    X(cuMemRelease)                     \
    X(cuMemAddressReserve)              \
    X(cuMemAddressFree)                 \
    X(cuMemMap)                         \
    X(cuMemUnmap)                       \
    X(cuMemSetAccess)                   \
    X(cuMemGetAllocationGranularity)    \
    X(cuMemExportToShareableHandle)     \
    X(cuMemImportFromShareableHandle)   \
    X(cuMulticastCreate)                \
    X(cuMulticastAddDevice)             \
    X(cuMulticastBindMem)               \
    X(cuMulticastUnbind)                \
    X(cuMulticastGetGranularity)        \
    X(cuStreamWriteValue32)             \
    X(cuStreamWaitValue32)              \
    X(cuCtxGetCurrent)                  \
    X(cuCtxGetId)                       \
    X(cuTensorMapEncodeTiled)

struct DriverApi {
#define AGG_DECLARE_PFN(name) decltype(&::name) name = nullptr;
    AGG_DRIVER_FUNCS(AGG_DECLARE_PFN)
#undef AGG_DECLARE_PFN
    bool ok = false;
    std::string why;
};

// Loads the table once (thread-safe).  ok == false when no driver is present.
const DriverApi& driver();

// Records a formatted message for agg_last_error() and returns `code`.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Helpers that turn CUDA failures into library error codes.
int check_rt(cudaError_t e, const char* what);
int check_drv(CUresult r, const char* what);

// Copy-engine producers of the fused kernel (agg_ce.cu).  ce_begin orders the
// device's internal stream after `caller` and holds the device's copy-engine
// state until ce_end, which makes `caller` wait for the copies; call ce_end
// after every successful ce_begin.
int ce_begin(cudaStream_t caller, cudaStream_t* ce);
int ce_end(cudaStream_t caller);
int ce_push_shard(const agg_args* a, const void* src, int m_local, size_t row_bytes, uint64_t region_off,
                  uint32_t parity, uint32_t target, bool multicast, cudaStream_t ce);
// The reduce-scatter twin's copy-engine exchange, on the internal stream `ce`:
// for owners rank+1, rank+2, ... (the kernel's block order) and each chunk c
// of gm m-tiles (m_tile_bytes each, L per block) of the owner's block, wait
// until cnt[owner * chunks + c] >= 8 x tiles of the chunk x epoch (the kernel
// has stored the chunk in `stage`, at the owner's rows), copy it into
// inbox_slot[owner] (slot `rank` of that owner's inbox, as mapped here); after
// the block's last chunk write `epoch` into rx_word[owner] (this source's
// arrival word in the owner's flag area).  Chunk c goes on internal stream
// c % streams (1-4); the write waits for all of them.
int ce_rs_exchange(int rank, int world, const uint64_t* inbox_slot, const uint8_t* stage, size_t slot_bytes,
                   size_t m_tile_bytes, int L, int gm, int n_tiles, uint32_t* cnt, const uint64_t* rx_word,
                   uint32_t epoch, int streams, cudaStream_t ce);

}  // namespace agg

#define AGG_RT(expr)                                        \
    do {                                                    \
        cudaError_t e__ = (expr);                           \
        if (e__ != cudaSuccess) return ::agg::check_rt(e__, #expr); \
    } while (0)

#define AGG_DRV(expr)                                       \
    do {                                                    \
        CUresult r__ = (expr);                              \
        if (r__ != CUDA_SUCCESS) return ::agg::check_drv(r__, #expr); \
    } while (0)
