// Split-K GEMM for callers that cannot allocate device memory.
//
//   C[M, N] = A[M, K] . B[N, K]^T      (bf16 in, fp32 accumulate, bf16 out)
//
// Some callers of this library may not call cudaMalloc at all: a plugin loaded
// into a host program whose caching allocator owns every byte of device memory
// (a foreign cudaMalloc fragments the pool it reserved and synchronises the
// device behind its back), or a latency-bound loop that must never take the
// allocator's device-wide synchronisation.  Such a caller can still hand us its
// inputs and output, but it cannot hand us a workspace.  This entry point
// needs no workspace argument: its scratch memory is one file-scope __device__
// array of AGG_NOALLOC_SCRATCH_BYTES that the CUDA runtime places on every GPU
// whose context loads this library's kernels, held until the process exits.
//
// The kernel splits K into `splits` ranges so that small M x N outputs with a
// long K still fill the GPU:
//
//   work unit   (tile, split): a 128 x 256 output tile over one K range.
//   warp 0      TMA loader (4-stage ring of 16 KiB A + 32 KiB B k-blocks);
//   warp 1      tcgen05.mma issuer, two 128 x 256 fp32 accumulators in TMEM;
//   warps 2-5   epilogue: each warp drains 32 accumulator rows, writes them as
//               an fp32 partial tile into the scratch, then counts its arrival
//               on that 32-row quarter's counter.  The warp that arrives last
//               (the splits-th arrival) adds the partials of all splits in
//               split order - so the result does not depend on arrival order -
//               rounds to bf16, writes C and resets the counter to zero.
//
// Scratch layout: [0, 64 KiB) u32 arrival counters, one per (tile, quarter);
// then one fp32 128 x 256 partial tile (128 KiB) per work unit.
//
// Every wait is bounded by a deadline (10 s); a timeout writes the status word
// and the roles wind down, TMEM is always released.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "agg.h"
#include "agg_internal.h"
#include "agg_ptx.cuh"

namespace agg {
namespace noalloc {

constexpr int TM = 128;                       // output tile rows
constexpr int TN = 256;                       // output tile columns
constexpr int KB_BYTES = 128;                 // one 128-byte swizzle row: 64 bf16
constexpr int KB_ELEMS = KB_BYTES / 2;
constexpr int STAGES = 4;
constexpr int A_BYTES = TM * KB_BYTES;        // 16 KiB
constexpr int B_BYTES = TN * KB_BYTES;        // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int NUM_THREADS = (2 + EPI_WARPS) * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr int BAR_OFF = STAGES * STAGE_BYTES;
constexpr int NUM_BARS = 2 * STAGES + 2 + 2 + 1;
constexpr int SLOT_OFF = BAR_OFF + NUM_BARS * 8;
constexpr int SMEM_ALLOC = SLOT_OFF + 16 + 1024;  // + slack to align the base to 1024 B
static_assert(SMEM_ALLOC <= 232448, "shared memory budget");

constexpr size_t COUNTER_BYTES = 64u << 10;
constexpr int MAX_QUARTERS = static_cast<int>(COUNTER_BYTES / sizeof(uint32_t));
constexpr int MAX_TILES = MAX_QUARTERS / 4;
constexpr size_t PART_BYTES = static_cast<size_t>(TM) * TN * sizeof(float);  // 128 KiB per unit
constexpr int MAX_UNITS = static_cast<int>((AGG_NOALLOC_SCRATCH_BYTES - COUNTER_BYTES) / PART_BYTES);
constexpr int MAX_SPLITS = 64;
static_assert(AGG_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size");

constexpr uint32_t IDESC = make_idesc(1, 1, TM, TN);

// The scratch.  In host code this name only identifies the variable; the
// device address is obtained per device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_scratch[AGG_NOALLOC_SCRATCH_BYTES];

struct Params {
    CUtensorMap tm_a;
    CUtensorMap tm_b;
    __nv_bfloat16* c;
    uint32_t* counters;  // scratch + 0
    float* parts;        // scratch + COUNTER_BYTES
    uint32_t* status;
    uint64_t timeout_ns;
    int M, N, K;
    int num_n_tiles, num_tiles, num_kb, splits, num_units;
};

__device__ __forceinline__ void unit_coords(const Params& p, int u, int& tile, int& s, int& kb0, int& kb1) {
    tile = u / p.splits;
    s = u - tile * p.splits;
    // Balanced K ranges; splits <= num_kb, so none is empty.
    kb0 = static_cast<int>((static_cast<long long>(s) * p.num_kb) / p.splits);
    kb1 = static_cast<int>((static_cast<long long>(s + 1) * p.num_kb) / p.splits);
}

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void loader(const Params& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                       const Deadline& dl) {
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
    int stage = 0;
    uint32_t phase = 0;
    uint32_t used = 0, last_par = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
        int tile, s, kb0, kb1;
        unit_coords(p, u, tile, s, kb0, kb1);
        const int mt = tile / p.num_n_tiles;
        const int nt = tile - mt * p.num_n_tiles;
        for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, dl)) {
                record_failure(p.status, AGG_ROLE_TMA, static_cast<uint32_t>(u));
                ok = false;
                break;
            }
            uint8_t* sa = smem + stage * STAGE_BYTES;
            mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
            tma_load_2d(&p.tm_a, sa, &full[stage], kb * KB_ELEMS, mt * TM);
            tma_load_2d(&p.tm_b, sa + A_BYTES, &full[stage], kb * KB_ELEMS, nt * TN);
            used |= 1u << stage;
            last_par = (last_par & ~(1u << stage)) | (phase << stage);
            if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
    // Never leave the CTA with TMA writes still landing in shared memory.
    for (int st = 0; st < STAGES; ++st)
        if (used & (1u << st))
            if (!mbar_wait_for(&full[st], (last_par >> st) & 1u, 200000000ull))
                record_failure(p.status, AGG_ROLE_DRAIN, 1u);
}

__device__ __forceinline__ void issuer(const Params& p, uint8_t* smem, uint32_t tmem_base, uint64_t* full,
                                       uint64_t* empty, uint64_t* tfull, uint64_t* tempty, uint64_t* drain,
                                       const Deadline& dl) {
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
        int tile, s, kb0, kb1;
        unit_coords(p, u, tile, s, kb0, kb1);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, dl)) {
            record_failure(p.status, AGG_ROLE_MMA, static_cast<uint32_t>(u));
            break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * TN);
        for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(&full[stage], phase, dl)) {
                record_failure(p.status, AGG_ROLE_MMA, static_cast<uint32_t>(u));
                ok = false;
                break;
            }
            const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
            const uint64_t adesc = sw128_kmajor_desc(sa);
            const uint64_t bdesc = sw128_kmajor_desc(sa + A_BYTES);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                // +32 bytes along K inside the 128-byte swizzle row (>> 4 in the descriptor)
                const uint64_t off = static_cast<uint64_t>(k * 2);
                umma_f16(d_tmem, adesc + off, bdesc + off, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
            }
            umma_commit(&empty[stage]);
            if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
        }
    }
    umma_commit(drain);
    if (!mbar_wait_for(drain, 0, 500000000ull)) record_failure(p.status, AGG_ROLE_DRAIN, 2u);
}

__device__ __forceinline__ void epilogue(const Params& p, uint32_t tmem_base, uint64_t* tfull, uint64_t* tempty,
                                         int warp, const Deadline& dl) {
    const int q = warp & 3;  // TMEM lane quarter this warp may access = its 32 rows of the tile
    const uint32_t lane = lane_id();
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
        int tile, s, kb0, kb1;
        unit_coords(p, u, tile, s, kb0, kb1);
        int got = 1;
        if (lane == 0) got = mbar_wait_sleepy(&tfull[acc], acc_phase, dl) ? 1 : 0;
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_EPI, static_cast<uint32_t>(u));
            break;
        }
        tc_fence_after();
        // This warp's 32 rows of the fp32 partial: row (q*32 + lane), 256 columns.
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * TN);
        float4* prow = reinterpret_cast<float4*>(p.parts + (static_cast<size_t>(u) * TM + q * 32 + lane) * TN);
#pragma unroll 1
        for (int j = 0; j < TN / 64; ++j) {
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(j * 64), r0);
            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(j * 64 + 32), r1);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i)
                __stcg(prow + j * 16 + i, make_float4(__uint_as_float(r0[4 * i]), __uint_as_float(r0[4 * i + 1]),
                                                      __uint_as_float(r0[4 * i + 2]), __uint_as_float(r0[4 * i + 3])));
#pragma unroll
            for (int i = 0; i < 8; ++i)
                __stcg(prow + j * 16 + 8 + i,
                       make_float4(__uint_as_float(r1[4 * i]), __uint_as_float(r1[4 * i + 1]),
                                   __uint_as_float(r1[4 * i + 2]), __uint_as_float(r1[4 * i + 3])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
        }

        // Publish this quarter's partial (every lane's stores, then one release
        // fence and arrival); the splits-th arrival reduces it.
        __syncwarp();
        __threadfence();
        uint32_t* cnt = p.counters + tile * 4 + q;
        uint32_t prev = 0;
        if (lane == 0) {
            prev = atomicAdd(cnt, 1u);
            __threadfence();  // lane 0 acquires the other splits' partials ...
        }
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != static_cast<uint32_t>(p.splits) - 1u) continue;
        __syncwarp();        // ... and the warp barrier orders lanes 1-31 after lane 0
        __threadfence();
        const int mt = tile / p.num_n_tiles;
        const int nt = tile - mt * p.num_n_tiles;
        const int col = nt * TN + static_cast<int>(lane) * 8;
        const float* base = p.parts + (static_cast<size_t>(tile) * p.splits * TM + q * 32) * TN + lane * 8;
        const size_t split_stride = static_cast<size_t>(TM) * TN;
        for (int r = 0; r < 32; ++r) {
            const int row = mt * TM + q * 32 + r;
            if (row >= p.M) break;
            if (col >= p.N) continue;  // N % 8 == 0: a lane's 8 columns are all in or all out
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
            const float* src = base + static_cast<size_t>(r) * TN;
            for (int sp = 0; sp < p.splits; ++sp) {
                const float4 x = __ldcg(reinterpret_cast<const float4*>(src + sp * split_stride));
                const float4 y = __ldcg(reinterpret_cast<const float4*>(src + sp * split_stride + 4));
                v[0] += x.x;
                v[1] += x.y;
                v[2] += x.z;
                v[3] += x.w;
                v[4] += y.x;
                v[5] += y.y;
                v[6] += y.z;
                v[7] += y.w;
            }
            const uint4 out = make_uint4(bf16x2(v[0], v[1]), bf16x2(v[2], v[3]), bf16x2(v[4], v[5]),
                                         bf16x2(v[6], v[7]));
            *reinterpret_cast<uint4*>(p.c + static_cast<size_t>(row) * p.N + col) = out;
        }
        if (lane == 0) atomicExch(cnt, 0u);  // ready for the next call
        __syncwarp();
    }
}

__global__ void __launch_bounds__(NUM_THREADS, 1) splitk_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SLOT_OFF);

    const int warp = static_cast<int>(threadIdx.x >> 5);
    const uint32_t lane = lane_id();
    Deadline dl;
    dl.end_ns = globaltimer_ns() + (p.timeout_ns ? p.timeout_ns : 10000000000ull);
    dl.status = p.status;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], EPI_WARPS);
        }
        mbar_init(drain, 1);
        fence_mbarrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

    if (warp == 0) {
        if (lane == 0) loader(p, smem, full, empty, dl);
    } else if (warp == 1) {
        if (lane == 0) issuer(p, smem, tmem_base, full, empty, tfull, tempty, drain, dl);
        __syncwarp();
    } else {
        epilogue(p, tmem_base, tfull, tempty, warp, dl);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------------------------------------------------------- host side
// Per-device set-up, redone whenever the device's current context differs
// from the one it was done in (a cudaDeviceReset or a new primary context
// reloads the module, which may move the scratch and drops the kernel's
// shared-memory attribute): the scratch's device address, looked up with that
// device current, and the kernel's attributes.  A failed set-up is not kept,
// so the next call tries again.
struct DevState {
    unsigned long long ctx_id = 0;  // context the set-up was done in (0: none yet)
    unsigned char* scratch = nullptr;
    int sms = 0;
};
DevState g_state[64];
std::mutex g_state_mu;

int device_state(int dev, DevState* out) {
    if (dev < 0 || dev >= 64) return fail(AGG_EINVAL, "device ordinal %d out of range", dev);
    const DriverApi& d = driver();
    if (!d.ok) return fail(AGG_EDRIVER, "CUDA driver unavailable: %s", d.why.c_str());
    CUcontext ctx = nullptr;
    AGG_DRV(d.cuCtxGetCurrent(&ctx));
    unsigned long long id = 0;
    if (ctx) AGG_DRV(d.cuCtxGetId(ctx, &id));
    std::lock_guard<std::mutex> lock(g_state_mu);
    DevState& st = g_state[dev];
    if (!ctx || st.ctx_id != id) {
        // (With no context current yet, the runtime binds the device's primary
        // context in the first call below.)
        DevState fresh;
        void* ptr = nullptr;
        AGG_RT(cudaGetSymbolAddress(&ptr, g_scratch));
        fresh.scratch = static_cast<unsigned char*>(ptr);
        AGG_RT(cudaDeviceGetAttribute(&fresh.sms, cudaDevAttrMultiProcessorCount, dev));
        AGG_RT(cudaFuncSetAttribute(splitk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC));
        AGG_DRV(d.cuCtxGetCurrent(&ctx));
        if (!ctx) return fail(AGG_ESTATE, "no CUDA context current on device %d", dev);
        AGG_DRV(d.cuCtxGetId(ctx, &id));
        fresh.ctx_id = id;
        st = fresh;
    }
    *out = st;
    return AGG_OK;
}

int encode(CUtensorMap* m, const void* base, int inner, int outer, uint32_t box_outer, const char* what) {
    const DriverApi& d = driver();
    if (!d.ok) return fail(AGG_EDRIVER, "CUDA driver unavailable: %s", d.why.c_str());
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(KB_ELEMS), box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = d.cuTensorMapEncodeTiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return check_drv(r, what);
    return AGG_OK;
}

int launch(const void* A, const void* B, void* C, int M, int N, int K, int splits, uint32_t* status,
           cudaStream_t stream) {
    const char* fn = "agg_gemm_bf16_noalloc";
    if (!A || !B || !C) return fail(AGG_EINVAL, "%s: null A, B or C", fn);
    if (M <= 0 || N <= 0 || K <= 0) return fail(AGG_EINVAL, "%s: empty shape %d x %d x %d", fn, M, N, K);
    if (K % 8) return fail(AGG_EINVAL, "%s: K=%d must be a multiple of 8", fn, K);
    if (N % 8) return fail(AGG_EINVAL, "%s: N=%d must be a multiple of 8", fn, N);
    if (reinterpret_cast<uintptr_t>(A) % 16 || reinterpret_cast<uintptr_t>(B) % 16 ||
        reinterpret_cast<uintptr_t>(C) % 16)
        return fail(AGG_EINVAL, "%s: A, B and C must be 16-byte aligned", fn);
    if (splits < 0 || splits > MAX_SPLITS) return fail(AGG_EINVAL, "%s: splits=%d outside [0, %d]", fn, splits, MAX_SPLITS);

    const int num_m_tiles = (M + TM - 1) / TM;
    const int num_n_tiles = (N + TN - 1) / TN;
    const long long tiles = static_cast<long long>(num_m_tiles) * num_n_tiles;
    const int num_kb = (K + KB_ELEMS - 1) / KB_ELEMS;
    const long long min_bytes = static_cast<long long>(COUNTER_BYTES) + tiles * static_cast<long long>(PART_BYTES);
    if (tiles > MAX_TILES || tiles > MAX_UNITS)
        return fail(AGG_EINVAL,
                    "%s: %d x %d output needs %lld bytes of scratch even without splitting K, more than the "
                    "%u-byte static scratch (at most %d tiles of 128 x 256)",
                    fn, M, N, min_bytes, AGG_NOALLOC_SCRATCH_BYTES, std::min(MAX_TILES, MAX_UNITS));

    int dev = 0;
    AGG_RT(cudaGetDevice(&dev));
    DevState state;
    int rc = device_state(dev, &state);
    if (rc) return rc;
    const DevState* ds = &state;

    int s = splits;
    const int fit = static_cast<int>(MAX_UNITS / tiles);
    if (s == 0) {
        // Enough splits to give every SM a unit, within the scratch and K.
        s = static_cast<int>((ds->sms + tiles - 1) / tiles);
        s = std::max(1, std::min({s, fit, num_kb, MAX_SPLITS}));
    } else {
        if (s > num_kb) return fail(AGG_EINVAL, "%s: splits=%d exceeds the %d k-blocks of 64 in K=%d", fn, s, num_kb, K);
        if (s > fit)
            return fail(AGG_EINVAL, "%s: %lld tiles x %d splits need %lld bytes of scratch, more than the %u-byte static scratch",
                        fn, tiles, s,
                        static_cast<long long>(COUNTER_BYTES) + tiles * s * static_cast<long long>(PART_BYTES),
                        AGG_NOALLOC_SCRATCH_BYTES);
    }

    Params p;
    std::memset(&p, 0, sizeof(p));
    rc = encode(&p.tm_a, A, K, M, TM, "tensor map A");
    if (rc) return rc;
    rc = encode(&p.tm_b, B, K, N, TN, "tensor map B");
    if (rc) return rc;
    p.c = static_cast<__nv_bfloat16*>(C);
    p.counters = reinterpret_cast<uint32_t*>(ds->scratch);
    p.parts = reinterpret_cast<float*>(ds->scratch + COUNTER_BYTES);
    p.status = status;
    p.M = M;
    p.N = N;
    p.K = K;
    p.num_n_tiles = num_n_tiles;
    p.num_tiles = static_cast<int>(tiles);
    p.num_kb = num_kb;
    p.splits = s;
    p.num_units = static_cast<int>(tiles) * s;

    // The counters must start at zero.  A completed call leaves them at zero,
    // but one cut short (a timeout) may not, so clear this call's share first.
    AGG_RT(cudaMemsetAsync(p.counters, 0, static_cast<size_t>(tiles) * 4 * sizeof(uint32_t), stream));
    const int grid = std::max(1, std::min(ds->sms, p.num_units));
    splitk_kernel<<<grid, NUM_THREADS, SMEM_ALLOC, stream>>>(p);
    AGG_RT(cudaGetLastError());
    return AGG_OK;
}

}  // namespace noalloc
}  // namespace agg

extern "C" int agg_gemm_bf16_noalloc(const void* A, const void* B, void* C, int M, int N, int K, int splits,
                                     uint32_t* status, void* stream) {
    return agg::noalloc::launch(A, B, C, M, N, K, splits, status, static_cast<cudaStream_t>(stream));
}
