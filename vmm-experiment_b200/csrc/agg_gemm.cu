// The fused all-gather GEMM for sm_100a.
//
//   C_r[M, N_r] = AllGather(A_r)[M, K] . B_r[N_r, K]^T
//
// One persistent, warp-specialised kernel per rank (one CTA per SM, 256 threads):
//
//   warp 0      operand loader: one lane issues TMA loads of A (128 x 128 B) and
//               B (256 x 128 B) k-blocks into a 4-stage shared-memory ring.  A tile
//               of a remote rank's rows is loaded only after that chunk's arrival
//               flag (in this GPU's own slab) has reached its target.
//   warp 1      tensor-core issuer: owns 512 TMEM columns (two 128 x 256 fp32
//               accumulators), one lane issues tcgen05.mma (M=128, N=256, K=16
//               for bf16 / K=32 for e4m3) and tcgen05.commit to free stages and
//               publish finished accumulators.
//   warps 2-5   epilogue: tcgen05.ld 32 TMEM lanes x 64 columns at a time, (e4m3:
//               apply per-row x per-column scales), round to bf16, stage through a
//               128 B-swizzled buffer and TMA-store 32 x 64 boxes of C.  Runs one
//               accumulator behind the MMAs (double buffering).
//   warps 6-7   multicast producers (world > 1): stream this rank's A shard from
//               HBM and write it with 16-byte multimem.st into the NVLink multicast
//               object, so NVSwitch delivers it into every GPU's slab; after each
//               part a release-ordered multimem.red raises that chunk's flag on
//               every GPU.
//
// Tile order: this rank's own rows first (no wait), then the remote chunks in
// the order they are produced (chunk-major, sources r+1, r+2, ...), grouped
// `group_m` m-tiles at a time so concurrently running CTAs share A and B in L2.
//
// Every wait is bounded by the launch's deadline; a timeout writes the status
// word and all roles wind down (no traps, no unbounded spins), TMEM is always
// released.
//
// Reference: the kernel replaces launch_ag_gemm_warp_specialized<128,256,2,5>
// called at vmm/main.cpp:296 with the fused_globals of vmm/main.cpp:272-294
// (its own source is in an absent submodule).  The numerics follow the
// reference's check, include/reference_matmul.cuh:17-32 / 59-77: bf16 inputs,
// fp32 accumulation.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "agg.h"
#include "agg_internal.h"
#include "agg_ptx.cuh"

namespace agg {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK_BYTES = 128;  // one 128-byte swizzle row: 64 bf16 or 128 e4m3
constexpr int STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK_BYTES;  // 16 KiB
constexpr int B_STAGE_BYTES = BN * BK_BYTES;  // 32 KiB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int EPI_ROWS = 32;
constexpr int EPI_COLS = 64;
constexpr int EPI_BUF_BYTES = EPI_ROWS * EPI_COLS * 2;  // 4 KiB of bf16
constexpr int PROD_WARPS = 2;
constexpr int NUM_WARPS = 2 + EPI_WARPS + PROD_WARPS;
constexpr int NUM_THREADS = NUM_WARPS * 32;
constexpr uint32_t TMEM_COLS = 512;

constexpr int SMEM_STAGE_OFF = 0;
constexpr int SMEM_EPI_OFF = STAGES * STAGE_BYTES;
constexpr int SMEM_BAR_OFF = SMEM_EPI_OFF + EPI_WARPS * 2 * EPI_BUF_BYTES;
constexpr int NUM_BARS = 2 * STAGES + 2 + 2 + 1;
constexpr int SMEM_TMEM_SLOT_OFF = SMEM_BAR_OFF + NUM_BARS * 8;
constexpr int SMEM_USED = SMEM_TMEM_SLOT_OFF + 16;
constexpr int SMEM_ALLOC = SMEM_USED + 1024;  // slack to align the base to 1024 B
static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
static_assert(SMEM_EPI_OFF % 1024 == 0 && STAGE_BYTES % 1024 == 0, "swizzle alignment");

constexpr uint32_t IDESC_BF16 = make_idesc(1, 1, BM, BN);
constexpr uint32_t IDESC_E4M3 = make_idesc(0, 0, BM, BN);

struct alignas(64) KParams {
    CUtensorMap tm_a_src;   // this rank's shard (the whole A when world == 1)
    CUtensorMap tm_a_gath;  // gathered A [M, K] in this GPU's slab
    CUtensorMap tm_b;       // B_r [N, K]
    CUtensorMap tm_c;       // C_r [M, N] bf16
    CUtensorMap tm_out[AGG_MAX_RANKS];  // reduce-scatter: slot `rank` of every owner's inbox [M/P, N]
    const uint4* a_src;     // shard, for the producers' loads
    uint4* a_mc;            // multicast VA of this rank's slot in gathered A
    unsigned long long shard_bytes;
    unsigned long long chunk_bytes;
    uint32_t* flags_uc;     // this launch's parity set, [AGG_MAX_RANKS][AGG_MAX_CHUNKS]
    uint32_t* flags_mc;
    uint32_t* done_uc;
    uint32_t* done_mc;
    uint32_t* cta_counter;  // this GPU's count of CTAs done with the launch
    uint32_t* chunk_cnt;    // this GPU's count of pieces pushed, per chunk
    unsigned long long* ticket;  // this GPU's next piece to push
    unsigned long long piece_bytes;
    uint32_t flag_target;   // a chunk has arrived when its counter reaches this
    uint32_t gate_done;     // producers start once the done counter reaches this
    const float* scale_a;     // e4m3: row scales of A_src ([M] at world 1, the shard's [M/world] otherwise)
    const float* scale_b;     // e4m3: row scales of B ([N])
    const float* scale_gath;  // e4m3, world > 1: gathered row scales [M] (this GPU's view)
    float* scale_mc;          // e4m3, world > 1: this rank's slot of them, multicast view
    void* c_ptr;  // C, for the epilogue that stores without TMA
    uint32_t* status;
    unsigned long long* trace;  // optional per-CTA event times (AGG_TR_*)
    unsigned long long timeout_ns;
    uint32_t epoch;
    int rank, world;
    int M, N, K;
    int m_local;
    int num_m_tiles, num_n_tiles, num_tiles, num_kb;
    int num_chunks;
    int group_m;   // tiles per raster group (m-tiles, or n-tiles when raster_n)
    int raster_n;  // 1: group n-tiles instead of m-tiles
    int dtype;
    int tile_m;  // rows per m-tile: 128 (one CTA) or 256 (a CTA pair)
    // reduce-scatter twin (flags_* are then the per-tile counters of this launch's parity)
    const uint8_t* inbox;    // this GPU's inbox of this launch: [P][M/P, N] bf16, slot s from rank s
    __nv_bfloat16* y;        // this rank's rows of the sum [M/world, N]
    uint32_t rs_target;      // a tile's partials are all stored when its counter reaches this
    int ext_producer;        // 1: copy engines move the shard (AGG_ARGS_CE_*), no producer warps
    int peer_push;           // 1: producers store into every rank's slab (AGG_ARGS_SM_PEER_PUSH)
    uint64_t peer_dst[AGG_MAX_RANKS];  // peer_push: this rank's slot in every rank's slab, this launch's region
    // reduce-scatter with the copy-engine exchange (AGG_ARGS_RS_COPY_ENGINE)
    int rs_ce;                  // 1: other owners' partials go to the local stage; copy engines move them
    uint32_t* ce_cnt;           // this GPU's slices stored per owner and chunk, u32 [AGG_MAX_RANKS][ce_chunks]
    int ce_chunks;              // chunks per owner block: groups of min(group_m, m_local/256) m-tiles
    const uint32_t* ce_rx;      // this GPU's arrival words, per source rank (written by the sources' copies)
    const uint32_t* ce_fail;    // this GPU's failure marks, per source rank
    uint64_t ce_fail_peer[AGG_MAX_RANKS];  // this rank's failure mark in every rank's flag area
    // CTA-pair kernels: tiles are handed out in raster order from this launch's
    // slot of g_sched (dynamic = 1), or round-robin by cluster (dynamic = 0).
    int sched_slot;
    int dynamic;
    // wide kernel: work items [0, split_from) are 256 x 512 tiles, the rest
    // halves of the remaining tiles (num_tiles counts items)
    int split_from;
};

// Tile counters of the CTA-pair kernels' dynamic schedule.  Each launch takes
// the next slot of a per-device ring (host side), counts its tiles out of
// `next` and its finished CTAs into `done`; the last CTA to finish zeroes both,
// so the slot is ready for its next launch.  Launches that run at the same
// time (different streams) use different slots unless AGG_SCHED_SLOTS of them
// are in flight at once.
constexpr int AGG_SCHED_SLOTS = 1024;
struct SchedSlot {
    unsigned int next;
    unsigned int done;
};
static __device__ SchedSlot g_sched[AGG_SCHED_SLOTS];

// Position `pos` of the m-tile visiting order -> global m-tile index.
__device__ __forceinline__ int m_tile_at(const KParams& p, int pos) {
    if (p.world == 1) return pos;
    const int L = p.m_local / p.tile_m;
    if (pos < L) return p.rank * L + pos;
    const int q = pos - L;
    const int c = q / (p.world - 1);
    const int k = q - c * (p.world - 1);
    int s = p.rank + 1 + k;
    if (s >= p.world) s -= p.world;
    return s * L + c;
}

// Tile t of the launch -> (m-tile, n-tile).  Tiles are visited in groups so that
// the CTAs running at the same time share operand panels in L2:
//   m-major (raster_n == 0): groups of `group` m-tiles, all n-tiles of a group
//       before the next, m fastest (consecutive tiles share a B panel);
//   n-major (raster_n == 1): groups of `group` n-tiles, all m positions of a
//       group before the next, n fastest (consecutive tiles share an A panel).
// m positions follow m_tile_at (this rank's shard first, then arrival order).
__device__ __forceinline__ void tile_coords(const KParams& p, int t, int& mt, int& nt) {
    if (p.raster_n) {
        const int per_group = p.group_m * p.num_m_tiles;
        const int g = t / per_group;
        const int j = t - g * per_group;
        const int first = g * p.group_m;
        const int gs = min(p.group_m, p.num_n_tiles - first);
        const int pos = j / gs;
        nt = first + (j - pos * gs);
        mt = m_tile_at(p, pos);
        return;
    }
    const int per_group = p.group_m * p.num_n_tiles;
    const int g = t / per_group;
    const int j = t - g * per_group;
    const int first = g * p.group_m;
    const int gs = min(p.group_m, p.num_m_tiles - first);
    nt = j / gs;
    mt = m_tile_at(p, first + (j - nt * gs));
}

// Reduce-scatter tile order, the same on every rank: m-major groups of
// `group_m` m positions as above, where position pos is local m-tile pos / P
// of owner pos % P, so that every owner's tiles complete at an even rate on all
// ranks at once and its reducers always have finished tiles to work on.
// With the copy-engine exchange the order is owner-major instead: owner
// rank+1's block, then rank+2's, ..., this rank's own block last, each in
// groups of `group_m` m-tiles; a block is copied out as soon as it is stored.
__device__ __forceinline__ void rs_block_tile(const KParams& p, int owner, int j, int& mt, int& nt) {
    const int L = p.m_local / 256;
    const int gm = min(p.group_m, L);
    const int per_group = gm * p.num_n_tiles;
    const int g = j / per_group;
    j -= g * per_group;
    const int first = g * gm;
    const int gs = min(gm, L - first);
    nt = j / gs;
    mt = owner * L + first + (j - nt * gs);
}

__device__ __forceinline__ void rs_tile_coords(const KParams& p, int t, int& mt, int& nt) {
    if (p.rs_ce) {
        const int per_owner = (p.m_local / 256) * p.num_n_tiles;
        const int b = t / per_owner;
        int owner = p.rank + 1 + b;
        if (owner >= p.world) owner -= p.world;
        rs_block_tile(p, owner, t - b * per_owner, mt, nt);
        return;
    }
    const int per_group = p.group_m * p.num_n_tiles;
    const int g = t / per_group;
    const int j = t - g * per_group;
    const int first = g * p.group_m;
    const int gs = min(p.group_m, p.num_m_tiles - first);
    nt = j / gs;
    const int pos = first + (j - nt * gs);
    mt = (pos % p.world) * (p.m_local / 256) + pos / p.world;
}

// Copy-engine exchange, a launch that gave up: the copy stream waits for
// every chunk of every owner's block.  Mark this launch failed in every peer's
// flag area, then release the waits (each chunk counter to its target: 8
// slices x its tiles x epoch), so that the owners give up instead of adding
// what the copies bring.  Run by the last CTA, after every other CTA is done.
__device__ __noinline__ void rs_ce_release(const KParams& p) {
    for (int s = 0; s < p.world; ++s)
        if (s != p.rank) st_relaxed_sys_u32(reinterpret_cast<uint32_t*>(p.ce_fail_peer[s]), p.epoch);
    fence_acq_rel_sys();
    const int L = p.m_local / 256;
    const int gm = min(p.group_m, L);
    for (int s = 0; s < p.world; ++s) {
        if (s == p.rank) continue;
        for (int c = 0; c < p.ce_chunks; ++c) {
            const uint32_t rows = static_cast<uint32_t>(min(gm, L - c * gm));
            atomicExch(p.ce_cnt + s * p.ce_chunks + c, 8u * rows * static_cast<uint32_t>(p.num_n_tiles) * p.epoch);
        }
    }
}

// ---- optional event trace (one row of AGG_TRACE_SLOTS u64 per CTA)
__device__ __forceinline__ void trace_set(const KParams& p, int slot, unsigned long long v) {
    if (p.trace) p.trace[blockIdx.x * AGG_TRACE_SLOTS + slot] = v;
}
__device__ __forceinline__ void trace_max(const KParams& p, int slot, unsigned long long v) {
    if (p.trace) atomicMax(p.trace + blockIdx.x * AGG_TRACE_SLOTS + slot, v);
}

// An mbarrier wait that, with tracing on, adds the time it blocked to `acc`
// and counts the blocking waits in `n`.
__device__ __forceinline__ bool mbar_wait_timed(uint64_t* bar, uint32_t parity, const Deadline& dl, bool on,
                                                unsigned long long& acc, unsigned long long& n) {
    if (!on) return mbar_wait(bar, parity, dl);
    if (mbar_try_wait(smem_u32(bar), parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    const bool ok = mbar_wait(bar, parity, dl);
    acc += globaltimer_ns() - t0;
    ++n;
    return ok;
}

// Bookkeeping of a loader's waits on remote chunks and on free stages.
struct FlagWaitLog {
    unsigned long long first_wait = 0, first_ready = 0, last_ready = 0, waited = 0;
    unsigned long long stage_wait = 0, stage_waits = 0;
    int tiles = 0;
    __device__ __forceinline__ bool wait(const KParams& p, const uint32_t* f, const Deadline& dl) {
        const unsigned long long t0 = p.trace ? globaltimer_ns() : 0ull;
        const bool ok = wait_flag_geq(f, p.flag_target, dl);
        if (p.trace) {
            const unsigned long long t1 = globaltimer_ns();
            if (!first_wait) {
                first_wait = t0;
                first_ready = t1;
            }
            last_ready = t1;
            waited += t1 - t0;
        }
        return ok;
    }
    __device__ __forceinline__ void flush(const KParams& p) const {
        if (!p.trace) return;
        trace_set(p, AGG_TR_FIRST_WAIT, first_wait);
        trace_set(p, AGG_TR_FIRST_READY, first_ready);
        trace_set(p, AGG_TR_LAST_READY, last_ready);
        trace_set(p, AGG_TR_FLAG_WAIT_NS, waited);
        trace_set(p, AGG_TR_LOADER_DONE, globaltimer_ns());
        trace_set(p, AGG_TR_TILES, static_cast<unsigned long long>(tiles));
        trace_set(p, AGG_TR_LOAD_WAIT_NS, stage_wait);
    }
};

// e4m3 epilogue: the scale of row (row0 + lane).  A remote shard's scales came
// with its chunk (see the producer); the warp's 32 rows lie in one chunk, whose
// arrival lane 0 re-acquires before the lanes read the gathered scales.
__device__ __forceinline__ float epilogue_row_scale(const KParams& p, int row0, uint32_t lane, const Deadline& dl) {
    const int row = row0 + static_cast<int>(lane);
    if (p.world == 1) return row < p.M ? __ldg(p.scale_a + row) : 0.0f;
    const int src = row0 / p.m_local;
    if (src == p.rank) return __ldg(p.scale_a + (row - src * p.m_local));
    int ok = 1;
    if (lane == 0) {
        const uint32_t* f = p.flags_uc + src * AGG_MAX_CHUNKS + (row0 - src * p.m_local) / BM;
        ok = wait_flag_geq(f, p.flag_target, dl) ? 1 : 0;
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) return 0.0f;
    float v;
    asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p.scale_gath + row) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint4 ld_nc_v4(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// ---------------------------------------------------------------- roles
__device__ __forceinline__ void role_loader(const KParams& p, uint8_t* smem, uint64_t* full,
                                            uint64_t* empty, const Deadline& dl) {
    tma_prefetch_desc(&p.tm_a_src);
    tma_prefetch_desc(&p.tm_b);
    if (p.world > 1) tma_prefetch_desc(&p.tm_a_gath);
    const int kb_elems = p.dtype == AGG_DTYPE_BF16 ? BK_BYTES / 2 : BK_BYTES;
    const int L = p.m_local / BM;
    int stage = 0;
    uint32_t phase = 0;
    uint32_t used = 0, last_par = 0;
    bool ok = true;
    FlagWaitLog log;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int mt, nt;
        tile_coords(p, t, mt, nt);
        ++log.tiles;
        const CUtensorMap* tma = &p.tm_a_src;
        int a_row;
        if (p.world == 1) {
            a_row = mt * BM;
        } else {
            const int src = mt / L;
            if (src == p.rank) {
                a_row = (mt - src * L) * BM;
            } else {
                const uint32_t* f = p.flags_uc + src * AGG_MAX_CHUNKS + (mt - src * L);
                if (!log.wait(p, f, dl)) {
                    record_failure(p.status, AGG_ROLE_FLAG, static_cast<uint32_t>(mt));
                    ok = false;
                    break;
                }
                // The chunk arrived through the multicast alias and is read here
                // through the unicast alias by the async (TMA) proxy.
                fence_proxy_alias();
                fence_proxy_async_global();
                tma = &p.tm_a_gath;
                a_row = mt * BM;
            }
        }
        for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!mbar_wait_timed(&empty[stage], phase ^ 1u, dl, p.trace != nullptr, log.stage_wait, log.stage_waits)) {
                record_failure(p.status, AGG_ROLE_TMA, static_cast<uint32_t>(t));
                ok = false;
                break;
            }
            uint8_t* sa = smem + SMEM_STAGE_OFF + stage * STAGE_BYTES;
            uint8_t* sb = sa + A_STAGE_BYTES;
            mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
            tma_load_2d(tma, sa, &full[stage], kb * kb_elems, a_row);
            tma_load_2d(&p.tm_b, sb, &full[stage], kb * kb_elems, nt * BN);
            used |= 1u << stage;
            last_par = (last_par & ~(1u << stage)) | (phase << stage);
            if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
    log.flush(p);
    // Never leave the CTA with TMA writes still landing in shared memory.
    for (int s = 0; s < STAGES; ++s)
        if (used & (1u << s))
            if (!mbar_wait_for(&full[s], (last_par >> s) & 1u, 200000000ull))
                record_failure(p.status, AGG_ROLE_DRAIN, 1u);
}

// The whole warp runs the loop, one elected lane issues (see pair_mma_loop).
template <bool F8>
__device__ __forceinline__ void role_mma_loop(const KParams& p, uint8_t* smem, uint32_t tmem_base, uint64_t* full,
                                              uint64_t* empty, uint64_t* tfull, uint64_t* tempty,
                                              const Deadline& dl) {
    constexpr uint32_t IDESC = F8 ? IDESC_E4M3 : IDESC_BF16;
    const uint32_t lane = lane_id();
    const bool tr = p.trace != nullptr;
    const uint64_t desc0 = sw128_kmajor_desc(smem_u32(smem + SMEM_STAGE_OFF));
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    unsigned long long full_wait = 0, full_waits = 0, acc_wait = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        const unsigned long long ta = tr ? globaltimer_ns() : 0ull;
        if (!mbar_wait_warp(&tempty[acc], acc_phase ^ 1u, dl)) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_MMA, static_cast<uint32_t>(t));
            break;
        }
        if (tr) acc_wait += globaltimer_ns() - ta;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!__all_sync(0xffffffffu, mbar_try_wait(smem_u32(&full[stage]), phase))) {
                const unsigned long long t0 = tr ? globaltimer_ns() : 0ull;
                ok = mbar_wait_warp(&full[stage], phase, dl);
                if (tr) {
                    full_wait += globaltimer_ns() - t0;
                    ++full_waits;
                }
                if (!ok) {
                    if (lane == 0) record_failure(p.status, AGG_ROLE_MMA, static_cast<uint32_t>(t));
                    break;
                }
            }
            // (No tcgen05 fence here: the stage was filled by TMA and the mbarrier
            // wait already orders those async-proxy writes before the MMA reads.)
            const uint64_t adesc = desc0 + static_cast<uint64_t>((stage * STAGE_BYTES) >> 4);
            const uint64_t bdesc = adesc + static_cast<uint64_t>(A_STAGE_BYTES >> 4);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                // +32 bytes along K inside the 128-byte swizzle row (>> 4 in the descriptor)
                const uint64_t off = static_cast<uint64_t>(k * 2);
                const uint32_t accumulate = (kb > 0 || k > 0) ? 1u : 0u;
                if constexpr (F8)
                    umma_f8_warp(d_tmem, adesc + off, bdesc + off, IDESC, accumulate);
                else
                    umma_f16_warp(d_tmem, adesc + off, bdesc + off, IDESC, accumulate);
            }
            umma_commit_warp(&empty[stage]);  // stage is free once these MMAs have read it
            if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if (!ok) break;
        umma_commit_warp(&tfull[acc]);  // accumulator complete
        if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
        }
    }
    if (tr && lane == 0) {
        trace_set(p, AGG_TR_MMA_WAIT_NS, full_wait);
        trace_set(p, AGG_TR_MMA_ACC_NS, acc_wait);
        trace_set(p, AGG_TR_MMA_STALLS, full_waits);
    }
}

__device__ __forceinline__ void role_mma(const KParams& p, uint8_t* smem, uint32_t tmem_base, uint64_t* full,
                                         uint64_t* empty, uint64_t* tfull, uint64_t* tempty, uint64_t* drain,
                                         const Deadline& dl) {
    if (p.dtype == AGG_DTYPE_E4M3)
        role_mma_loop<true>(p, smem, tmem_base, full, empty, tfull, tempty, dl);
    else
        role_mma_loop<false>(p, smem, tmem_base, full, empty, tfull, tempty, dl);
    // Every MMA this warp issued has finished once `drain` flips.
    umma_commit_warp(drain);
    if (lane_id() == 0) {
        if (!mbar_wait_for(drain, 0, 500000000ull)) record_failure(p.status, AGG_ROLE_DRAIN, 2u);
        if (p.trace) trace_set(p, AGG_TR_MMA_DONE, globaltimer_ns());
    }
    __syncwarp();
}

__device__ __forceinline__ void role_epilogue(const KParams& p, uint8_t* smem, uint32_t tmem_base,
                                              uint64_t* tfull, uint64_t* tempty, int warp,
                                              const Deadline& dl) {
    const int eg = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane = lane_id();
    uint8_t* stg = smem + SMEM_EPI_OFF + (warp - 2) * 2 * EPI_BUF_BYTES;
    const bool f8 = p.dtype == AGG_DTYPE_E4M3;
    int acc = 0;
    uint32_t acc_phase = 0;
    int buf = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        int mt, nt;
        tile_coords(p, t, mt, nt);
        int got = 1;
        if (lane == 0) got = mbar_wait_sleepy(&tfull[acc], acc_phase, dl) ? 1 : 0;
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_EPI, static_cast<uint32_t>(t));
            break;
        }
        tc_fence_after();
        const uint32_t tbase =
            tmem_base + (static_cast<uint32_t>(eg * 32) << 16) + static_cast<uint32_t>(acc * BN);
        const int row0 = mt * BM + eg * 32;
        const float row_scale = f8 ? epilogue_row_scale(p, row0, lane, dl) : 1.0f;
#pragma unroll 1
        for (int j = 0; j < BN / EPI_COLS; ++j) {
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(j * EPI_COLS), r0);
            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(j * EPI_COLS + 32), r1);
            tmem_wait_ld();
            const int col0 = nt * BN + j * EPI_COLS;
            uint32_t packed[32];
            if (f8) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = col0 + 2 * i;
                    const float s0 = c < p.N ? __ldg(p.scale_b + c) : 0.0f;
                    const float s1 = c + 1 < p.N ? __ldg(p.scale_b + c + 1) : 0.0f;
                    packed[i] = pack_bf16x2(__uint_as_float(r0[2 * i]) * row_scale * s0,
                                            __uint_as_float(r0[2 * i + 1]) * row_scale * s1);
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = col0 + 32 + 2 * i;
                    const float s0 = c < p.N ? __ldg(p.scale_b + c) : 0.0f;
                    const float s1 = c + 1 < p.N ? __ldg(p.scale_b + c + 1) : 0.0f;
                    packed[16 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]) * row_scale * s0,
                                                 __uint_as_float(r1[2 * i + 1]) * row_scale * s1);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    packed[i] = pack_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    packed[16 + i] =
                        pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
            }
            // The buffer is free once the TMA store issued two chunks ago has read it.
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
            uint8_t* b = stg + buf * EPI_BUF_BYTES;
            const uint32_t row_base = smem_u32(b) + lane * 128u;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint32_t addr = row_base + ((static_cast<uint32_t>(c) ^ (lane & 7u)) << 4);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                             "r"(packed[4 * c]), "r"(packed[4 * c + 1]), "r"(packed[4 * c + 2]),
                             "r"(packed[4 * c + 3])
                             : "memory");
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&p.tm_c, b, col0, row0);
                bulk_commit_group();
            }
            buf ^= 1;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
        }
    }
    if (lane == 0) {
        bulk_wait_group<0>();
        if (p.trace) trace_max(p, AGG_TR_EPI_DONE, globaltimer_ns());
    }
    __syncwarp();
}

__device__ __forceinline__ void role_producer(const KParams& p, int pw, const Deadline& dl) {
    if (p.ext_producer) return;  // the copy engines move the shard and raise the flags
    const uint32_t lane = lane_id();
    int ok = 1;
    if (p.gate_done > 0) {
        // Every rank must be done reading the gathered region this launch is
        // about to overwrite (the previous launch, or the one before it when the
        // region is double-buffered) before this rank writes its slot on all GPUs.
        if (lane == 0) ok = wait_flag_geq(p.done_uc, p.gate_done, dl) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_PROD, 0u);
            return;
        }
        fence_proxy_alias();
    }
    if (p.trace && pw == 0 && lane == 0) trace_set(p, AGG_TR_PROD_GATE, globaltimer_ns());
    // The shard is cut into pieces of `piece_bytes`, numbered in chunk order and
    // handed out by a ticket counter, so the pieces in flight are always the
    // earliest unfinished ones: chunks complete in the order the consumers need
    // them.  The piece size (host-chosen) keeps enough bytes in flight to cover
    // the NVLink round trip that each piece's system-scope fence waits for.
    const unsigned long long pieces_per_chunk = (p.chunk_bytes + p.piece_bytes - 1) / p.piece_bytes;
    const unsigned long long total = pieces_per_chunk * static_cast<unsigned long long>(p.num_chunks);
    for (;;) {
        unsigned long long ticket = 0;
        if (lane == 0) ticket = atomicAdd(p.ticket, 1ull);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket >= total) break;
        const int c = static_cast<int>(ticket / pieces_per_chunk);
        const unsigned long long cbeg = static_cast<unsigned long long>(c) * p.chunk_bytes;
        unsigned long long cend = cbeg + p.chunk_bytes;
        if (cend > p.shard_bytes) cend = p.shard_bytes;
        const unsigned long long beg = cbeg + (ticket - static_cast<unsigned long long>(c) * pieces_per_chunk) *
                                                  p.piece_bytes;
        unsigned long long end = beg + p.piece_bytes;
        if (end > cend) end = cend;
        if (beg < end) {
            const uint4* s = p.a_src + beg / 16;
            uint4* d = p.a_mc + beg / 16;
            const unsigned long long n = (end - beg) / 16;
            for (unsigned long long i = lane; i < n; i += 32ull * 8ull) {
                uint4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const unsigned long long j = i + 32ull * u;
                    if (j < n) v[u] = ld_nc_v4(s + j);
                }
                if (p.peer_push) {
                    // one unicast copy per rank (this GPU's own slot included), the
                    // ranks interleaved so every link carries traffic at once
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const unsigned long long j = i + 32ull * u;
                        if (j < n)
                            for (int r = 0; r < p.world; ++r)
                                reinterpret_cast<uint4*>(p.peer_dst[r] + beg)[j] = v[u];
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const unsigned long long j = i + 32ull * u;
                        if (j < n) mm_st_v4(d + j, v[u]);
                    }
                }
            }
        }
        if (p.scale_mc && ticket == static_cast<unsigned long long>(c) * pieces_per_chunk) {
            // e4m3: the first piece of a chunk also carries the chunk's 128 row
            // scales (512 bytes, one 16-byte store per lane), so the chunk's
            // arrival counter covers them too.
            const int row = c * BM + static_cast<int>(lane) * 4;
            if (row < p.m_local) {
                const float4 sv = *reinterpret_cast<const float4*>(p.scale_a + row);
                mm_st_v4(p.scale_mc + row, make_uint4(__float_as_uint(sv.x), __float_as_uint(sv.y),
                                                      __float_as_uint(sv.z), __float_as_uint(sv.w)));
            }
        }
        // This warp's piece is out: order its multicast stores (system scope)
        // before its count; the warp that completes the count raises the
        // chunk's arrival counter on every GPU, once per chunk and launch.
        fence_acq_rel_sys();
        __syncwarp();
        if (lane == 0) {
            const uint32_t prev = atomicAdd(p.chunk_cnt + c, 1u);
            if (prev == static_cast<uint32_t>(pieces_per_chunk) - 1u) {
                atomicExch(p.chunk_cnt + c, 0u);  // ready for the next launch
                fence_acq_rel_sys();
                mm_red_add_release_u32(p.flags_mc + p.rank * AGG_MAX_CHUNKS + c, 1u);
            }
        }
        if (failed(p.status)) break;
    }
    if (p.trace && lane == 0) trace_max(p, AGG_TR_PROD_DONE, globaltimer_ns());
}

// Reduce-scatter: this rank owns m-tiles [rank*L, (rank+1)*L).  Every rank's
// epilogue has TMA-stored its partial of each such tile into slot `its rank`
// of this GPU's inbox.  The epilogue warps, once their own tiles are out, take
// 32-row slices of the owned tiles by ticket, in the order the tiles complete
// (rs_tile_coords restricted to this owner), wait until all ranks' slices are
// stored (the tile's counter reaches rs_target), and add the P slots from
// local memory in source order (fp32), one 16-byte load per lane, row and
// slot.  (Pulling the sum through NVSwitch with multimem.ld_reduce instead
// moved only ~100 GB/s and stalled the SMs.)
//
// With the copy-engine exchange the other ranks' slots arrive as whole blocks:
// a reducer first waits (once) for every source's arrival word, then for each
// tile only for this rank's own partial (stored last, in rs_block_tile order).
__device__ __forceinline__ bool rs_ce_sources_arrived(const KParams& p, const Deadline& dl) {
    for (int s = 0; s < p.world; ++s) {
        if (s == p.rank) continue;
        for (uint32_t spin = 0;; ++spin) {
            if (ld_relaxed_sys(p.ce_fail + s) >= p.epoch) return false;
            if (ld_relaxed_sys(p.ce_rx + s) >= p.epoch) break;
            __nanosleep(500);
            if ((spin & 15u) == 15u && (globaltimer_ns() > dl.end_ns || failed(dl.status))) return false;
        }
    }
    fence_acq_rel_sys();
    // a source that failed marks it before it releases its copies
    for (int s = 0; s < p.world; ++s)
        if (s != p.rank && ld_relaxed_sys(p.ce_fail + s) >= p.epoch) return false;
    return true;
}

__device__ __forceinline__ void role_reducer(const KParams& p, const Deadline& dl) {
    const uint32_t lane = lane_id();
    const int L = p.m_local / 256;
    const int nN = p.num_n_tiles;
    const int P = p.world;
    const unsigned long long units = static_cast<unsigned long long>(L) * nN * 8ull;
    bool sources = !p.rs_ce;  // copy-engine exchange: the other ranks' blocks are in
    for (;;) {
        unsigned long long ticket = 0;
        if (lane == 0) ticket = atomicAdd(p.ticket, 1ull);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket >= units) break;
        const int slice = static_cast<int>(ticket & 7ull);
        int k = static_cast<int>(ticket >> 3);
        int mt = -1, nt = 0;
        if (p.rs_ce) {
            rs_block_tile(p, p.rank, k, mt, nt);
        } else {
            // k-th owned tile in completion order: walk the m-position groups.
            for (int first = 0; first < p.num_m_tiles; first += p.group_m) {
                const int gs = min(p.group_m, p.num_m_tiles - first);
                const int f_own = first + ((p.rank - first) % P + P) % P;  // first owned position >= first
                const int owned = f_own < first + gs ? (first + gs - 1 - f_own) / P + 1 : 0;
                if (k < owned * nN) {
                    nt = k / owned;
                    mt = p.rank * L + (f_own + (k - nt * owned) * P) / P;
                    break;
                }
                k -= owned * nN;
            }
        }
        if (mt < 0) break;  // not reached: units counts exactly the owned tiles
        int ok = 1;
        if (!sources) {
            if (lane == 0) {
                const unsigned long long t0 = p.trace ? globaltimer_ns() : 0ull;
                ok = rs_ce_sources_arrived(p, dl) ? 1 : 0;
                if (p.trace) {  // when this CTA's reducers had every block, and how long they waited
                    const unsigned long long t1 = globaltimer_ns();
                    trace_max(p, AGG_TR_LAST_READY, t1);
                    atomicAdd(p.trace + blockIdx.x * AGG_TRACE_SLOTS + AGG_TR_FLAG_WAIT_NS, t1 - t0);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            sources = true;
        }
        if (lane == 0 && ok) ok = wait_flag_geq_quiet(p.flags_uc + mt * nN + nt, p.rs_target, dl) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_REDUCE, static_cast<uint32_t>(mt * nN + nt));
            break;
        }
        __syncwarp();
        fence_proxy_alias();
        const int col = nt * 256 + static_cast<int>(lane) * 8;
        if (col < p.N) {
            // row lr of the owner's block, slot s: inbox + ((s * m_local + lr) * N + col) * 2
            const int lr0 = (mt - p.rank * L) * 256 + slice * 32;
            const size_t pitch = static_cast<size_t>(p.N);
            const size_t slot = static_cast<size_t>(p.m_local) * pitch;
            const uint4* src = reinterpret_cast<const uint4*>(
                reinterpret_cast<const __nv_bfloat16*>(p.inbox) + static_cast<size_t>(lr0) * pitch + col);
            __nv_bfloat16* dst = p.y + static_cast<size_t>(lr0) * pitch + col;
            constexpr int R = 8;  // rows per pass: R loads in flight per lane and slot
#pragma unroll 1
            for (int r = 0; r < 32; r += R) {
                float acc[R][8];
#pragma unroll
                for (int i = 0; i < R; ++i)
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[i][e] = 0.0f;
                for (int s = 0; s < P; ++s) {  // fixed source order: the sum does not depend on timing
                    uint4 v[R];
#pragma unroll
                    for (int i = 0; i < R; ++i) v[i] = __ldcg(src + (s * slot + (r + i) * pitch) / 8);
#pragma unroll
                    for (int i = 0; i < R; ++i) {
                        const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            acc[i][2 * e] += __uint_as_float(w[e] << 16);
                            acc[i][2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < R; ++i)
                    *reinterpret_cast<uint4*>(dst + (r + i) * pitch) =
                        make_uint4(pack_bf16x2(acc[i][0], acc[i][1]), pack_bf16x2(acc[i][2], acc[i][3]),
                                   pack_bf16x2(acc[i][4], acc[i][5]), pack_bf16x2(acc[i][6], acc[i][7]));
            }
        }
        if (failed(p.status)) break;
    }
    if (p.trace && lane == 0) trace_max(p, AGG_TR_PROD_DONE, globaltimer_ns());
}

// ---------------------------------------------------------------- kernel
__global__ void __launch_bounds__(NUM_THREADS, 1) ag_gemm_kernel(const __grid_constant__ KParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_BAR_OFF);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SMEM_TMEM_SLOT_OFF);

    const int warp = static_cast<int>(threadIdx.x >> 5);
    const uint32_t lane = lane_id();
    Deadline dl;
    dl.end_ns = globaltimer_ns() + (p.timeout_ns ? p.timeout_ns : 10000000000ull);
    dl.status = p.status;
    if (p.trace && threadIdx.x == 0) trace_set(p, AGG_TR_START, globaltimer_ns());

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
        if (lane == 0) role_loader(p, smem, full, empty, dl);
    } else if (warp == 1) {
        role_mma(p, smem, tmem_base, full, empty, tfull, tempty, drain, dl);
        __syncwarp();
    } else if (warp < 2 + EPI_WARPS) {
        role_epilogue(p, smem, tmem_base, tfull, tempty, warp, dl);
    } else if (p.world > 1) {
        role_producer(p, warp - 2 - EPI_WARPS, dl);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
    if (p.trace && threadIdx.x == 0) trace_set(p, AGG_TR_END, globaltimer_ns());
    if (p.world > 1 && threadIdx.x == 0) {
        // This CTA has finished reading gathered A for this launch.  The last CTA
        // on this GPU tells every GPU (release, system scope).
        __threadfence();
        const uint32_t prev = atomicAdd(p.cta_counter, 1u);
        if (prev == gridDim.x - 1u) {
            if (p.rs_ce && failed(p.status)) rs_ce_release(p);
            atomicExch(p.cta_counter, 0u);
            atomicExch(p.ticket, 0ull);  // every producer of this launch is done
            fence_acq_rel_sys();
            mm_red_add_release_u32(p.done_mc, 1u);
        }
    }
}

// ================================================================ CTA-pair kernel
//
// The same roles on a cluster of two CTAs that share one tcgen05.mma.cta_group::2
// per k-step: the pair computes a 256 x BN tile, each CTA holding 128 rows of A
// and BN/2 rows of B in its shared memory and 128 x BN accumulators in its TMEM.
// Per SM that halves the B traffic from L2 and the smem bytes the tensor core
// reads per FLOP.  A stage holds SUB 128-byte-wide k sub-blocks (one TMA box
// per operand and sub-block): with SUB = 2 the issuer runs 8 MMAs per barrier
// round trip, which is what keeps the tensor pipe busy; 3 (BN=256) or 4
// (BN=128) such stages fill the shared memory.
//
//   both CTAs   loader: waits on its own `empty` barrier, TMA-loads its A half
//               and B half, completion counted on the EVEN CTA's `full` barrier
//               (the even CTA arms it with both CTAs' bytes);
//   even CTA    MMA issuer: waits `full`, issues the pair MMA, commits to
//               `empty` in both CTAs, and to `tfull` in both CTAs per tile;
//   both CTAs   epilogue: drains its own TMEM, arrives on the even CTA's `tempty`.
// The pair's tile queue: the even CTA's loader takes each tile (from the
// launch's counter, or round-robin) and publishes its index into a ring of
// TQ_DEPTH slots in both CTAs' shared memory; the odd CTA's loader, the MMA
// issuer and the eight epilogue warps read it from there.  -1 ends the launch.
constexpr int TQ_DEPTH = 4;
constexpr uint32_t TQ_READERS = 2 + 2 * EPI_WARPS;

struct TileQueue {
    int* ids;         // this CTA's ring
    uint64_t* full;   // this CTA's, one arrival (from the even CTA's loader) per slot fill
    uint64_t* empty;  // the even CTA's are used: TQ_READERS arrivals per slot drain
    int pos;          // ring position of this role's next read or fill
};

// A reader's next tile: the id, -1 at the end, -2 when the wait gave up.
__device__ __forceinline__ int tq_read(TileQueue& q, const Deadline& dl) {
    const int s = q.pos % TQ_DEPTH;
    const uint32_t ph = static_cast<uint32_t>(q.pos / TQ_DEPTH) & 1u;
    ++q.pos;
    if (!mbar_wait_cluster(&q.full[s], ph, dl)) return -2;
    const int t = ld_shared_volatile_s32(&q.ids[s]);
    mbar_arrive_cluster(mapa_shared(smem_u32(&q.empty[s]), 0));
    return t;
}

// The even CTA's loader: take the next tile and publish it to both CTAs.
__device__ __forceinline__ int tq_fill(const KParams& p, TileQueue& q, int& rr, const Deadline& dl) {
    const int s = q.pos % TQ_DEPTH;
    const uint32_t ph = static_cast<uint32_t>(q.pos / TQ_DEPTH) & 1u;
    ++q.pos;
    if (!mbar_wait_cluster(&q.empty[s], ph ^ 1u, dl)) return -2;
    int t;
    if (p.dynamic) {
        const unsigned int n = atomicAdd(&g_sched[p.sched_slot].next, 1u);
        t = n < static_cast<unsigned int>(p.num_tiles) ? static_cast<int>(n) : -1;
    } else {
        t = rr < p.num_tiles ? rr : -1;
        rr += static_cast<int>(gridDim.x >> 1);
    }
    q.ids[s] = t;
    st_shared_cluster_u32(mapa_shared(smem_u32(&q.ids[s]), 1), static_cast<uint32_t>(t));
    mbar_arrive(&q.full[s]);
    mbar_arrive_cluster(mapa_shared(smem_u32(&q.full[s]), 1));
    return t;
}

template <int BN2, int ST, int SUB, int EB = 2>
struct PairCfg {
    static constexpr int TILE_M = 256;
    static constexpr int B_ROWS = BN2 / 2;
    static constexpr int A_SUB = 128 * BK_BYTES;     // one k sub-block of A (16 KiB)
    static constexpr int B_SUB = B_ROWS * BK_BYTES;  // one k sub-block of B
    static constexpr int A_BYTES = SUB * A_SUB;
    static constexpr int B_BYTES = SUB * B_SUB;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int STAGES = ST;
    static constexpr int EPI_OFF = STAGES * STAGE;
    // The epilogue stages C through EB swizzled 4 KiB buffers per warp for TMA
    // stores when there is room; with one stage more it writes 16-byte row
    // segments straight to HBM.
    static constexpr int EPI_BUFS = EB;
    static constexpr bool STAGED_EPI = EPI_OFF + EPI_WARPS * EB * EPI_BUF_BYTES + 256 + 1024 <= 232448;
    static constexpr int BAR_OFF = EPI_OFF + (STAGED_EPI ? EPI_WARPS * EB * EPI_BUF_BYTES : 0);
    static constexpr int NUM_BARS = 2 * STAGES + 2 + 2 + 1 + 2 * TQ_DEPTH;
    static constexpr int SLOT_OFF = BAR_OFF + NUM_BARS * 8;
    static constexpr int TQ_OFF = SLOT_OFF + 16;  // int tile ids [TQ_DEPTH]
    static constexpr int SMEM = TQ_OFF + 4 * TQ_DEPTH + 1024;
    static constexpr uint32_t TMEM_COLS = 2 * BN2;  // two accumulators: 512 or 256 columns
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(EPI_OFF % 1024 == 0 && STAGE % 1024 == 0 && A_BYTES % 1024 == 0, "swizzle alignment");
    static_assert(STAGES <= 32, "stage masks are 32-bit");
};

// The pair kernel's shared-memory layout.  The reduce-scatter twin stores its
// partial tiles into other GPUs' memory, where a TMA store frees its staging
// buffer only after a round trip over NVLink: it keeps four buffers per warp
// (and 1-k-block stages to make room) so that three stores can be in flight.
template <int BN2, int ST, int SUB, bool RS>
using PairG = PairCfg<BN2, ST, SUB, RS ? 4 : 2>;

template <int BN2, int ST, int SUB, bool RS = false>
__device__ __forceinline__ void pair_loader(const KParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                            TileQueue& q, uint32_t crank, const Deadline& dl) {
    using G = PairG<BN2, ST, SUB, RS>;
    tma_prefetch_desc(&p.tm_a_src);
    tma_prefetch_desc(&p.tm_b);
    if (!RS && p.world > 1) tma_prefetch_desc(&p.tm_a_gath);
    const int kb_elems = p.dtype == AGG_DTYPE_BF16 ? BK_BYTES / 2 : BK_BYTES;
    int rr = static_cast<int>(blockIdx.x >> 1);  // round-robin schedule: this pair's next tile
    int stage = 0;
    uint32_t phase = 0;
    uint32_t used = 0, last_par = 0;
    bool ok = true;
    FlagWaitLog log;
    while (ok) {
        const int t = crank == 0 ? tq_fill(p, q, rr, dl) : tq_read(q, dl);
        if (t == -2) {
            record_failure(p.status, AGG_ROLE_TMA, 0xFFFFFFu);
            break;
        }
        if (t < 0) break;
        int mt, nt;
        if constexpr (RS)
            rs_tile_coords(p, t, mt, nt);
        else
            tile_coords(p, t, mt, nt);
        ++log.tiles;
        const int row = mt * G::TILE_M + static_cast<int>(crank) * 128;  // this CTA's first row of gathered A
        const CUtensorMap* tma = &p.tm_a_src;
        int a_row = row;
        if (!RS && p.world > 1) {
            const int src = row / p.m_local;
            if (src == p.rank) {
                a_row = row - src * p.m_local;
            } else {
                const uint32_t* f = p.flags_uc + src * AGG_MAX_CHUNKS + (row - src * p.m_local) / BM;
                if (!log.wait(p, f, dl)) {
                    record_failure(p.status, AGG_ROLE_FLAG, static_cast<uint32_t>(row / BM));
                    ok = false;
                    break;
                }
                fence_proxy_alias();
                fence_proxy_async_global();
                tma = &p.tm_a_gath;
            }
        }
        const int b_row = nt * BN2 + static_cast<int>(crank) * G::B_ROWS;
        for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!mbar_wait_timed(&empty[stage], phase ^ 1u, dl, p.trace != nullptr, log.stage_wait, log.stage_waits)) {
                record_failure(p.status, AGG_ROLE_TMA, static_cast<uint32_t>(t));
                ok = false;
                break;
            }
            uint8_t* sa = smem + stage * G::STAGE;
            uint8_t* sb = sa + G::A_BYTES;
            if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * G::STAGE);
            const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
#pragma unroll
            for (int u = 0; u < SUB; ++u) {
                const int kx = (kb * SUB + u) * kb_elems;
                tma_load_2d_pair(tma, sa + u * G::A_SUB, bar, kx, a_row);
                tma_load_2d_pair(&p.tm_b, sb + u * G::B_SUB, bar, kx, b_row);
            }
            used |= 1u << stage;
            last_par = (last_par & ~(1u << stage)) | (phase << stage);
            if (++stage == G::STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
    log.flush(p);
    // The even CTA's `full` barriers count both CTAs' bytes of every phase it armed.
    if (crank == 0)
        for (int s = 0; s < G::STAGES; ++s)
            if (used & (1u << s))
                if (!mbar_wait_for(&full[s], (last_par >> s) & 1u, 200000000ull))
                    record_failure(p.status, AGG_ROLE_DRAIN, 1u);
}

// The MMA issuer: the whole warp runs the loop (so descriptors stay in
// uniform registers), one elected lane issues each tcgen05 instruction.
template <int BN2, int ST, int SUB, bool F8>
__device__ __forceinline__ void pair_mma_loop(const KParams& p, uint8_t* smem, uint32_t tmem_base, uint64_t* full,
                                              uint64_t* empty, uint64_t* tfull, uint64_t* tempty, TileQueue& q,
                                              const Deadline& dl) {
    using G = PairCfg<BN2, ST, SUB>;
    constexpr uint32_t IDESC = F8 ? make_idesc(0, 0, G::TILE_M, BN2) : make_idesc(1, 1, G::TILE_M, BN2);
    const uint32_t lane = lane_id();
    const bool tr = p.trace != nullptr;
    const uint64_t desc0 = sw128_kmajor_desc(smem_u32(smem));
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    unsigned long long full_wait = 0, full_waits = 0, acc_wait = 0;
    for (;;) {
        int t = 0;
        if (lane == 0) t = tq_read(q, dl);
        t = __shfl_sync(0xffffffffu, t, 0);
        if (t == -2) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_MMA, 0xFFFFFFu);
            break;
        }
        if (t < 0) break;
        const unsigned long long ta = tr ? globaltimer_ns() : 0ull;
        if (!mbar_wait_warp(&tempty[acc], acc_phase ^ 1u, dl)) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_MMA, static_cast<uint32_t>(t));
            break;
        }
        if (tr) acc_wait += globaltimer_ns() - ta;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN2);
        bool ok = true;
        for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!__all_sync(0xffffffffu, mbar_try_wait(smem_u32(&full[stage]), phase))) {
                const unsigned long long t0 = tr ? globaltimer_ns() : 0ull;
                ok = mbar_wait_warp(&full[stage], phase, dl);
                if (tr) {
                    full_wait += globaltimer_ns() - t0;
                    ++full_waits;
                }
            }
            if (!ok) {
                if (lane == 0) record_failure(p.status, AGG_ROLE_MMA, static_cast<uint32_t>(t));
                break;
            }
            // (No tcgen05 fence here: TMA filled the stage, the mbarrier orders it.)
            const uint64_t sdesc = desc0 + static_cast<uint64_t>((stage * G::STAGE) >> 4);
#pragma unroll
            for (int u = 0; u < SUB; ++u) {
                const uint64_t adesc = sdesc + static_cast<uint64_t>((u * G::A_SUB) >> 4);
                const uint64_t bdesc = sdesc + static_cast<uint64_t>((G::A_BYTES + u * G::B_SUB) >> 4);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    // +32 bytes along K inside the 128-byte swizzle row
                    const uint64_t off = static_cast<uint64_t>(k * 2);
                    const uint32_t accumulate = (kb > 0 || u > 0 || k > 0) ? 1u : 0u;
                    if constexpr (F8)
                        umma_f8_pair_warp(d_tmem, adesc + off, bdesc + off, IDESC, accumulate);
                    else
                        umma_f16_pair_warp(d_tmem, adesc + off, bdesc + off, IDESC, accumulate);
                }
            }
            umma_commit_pair_mc_warp(&empty[stage], 0x3);
            if (++stage == G::STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if (!ok) break;
        umma_commit_pair_mc_warp(&tfull[acc], 0x3);
        if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
        }
    }
    if (tr && lane == 0) {
        trace_set(p, AGG_TR_MMA_WAIT_NS, full_wait);
        trace_set(p, AGG_TR_MMA_ACC_NS, acc_wait);
        trace_set(p, AGG_TR_MMA_STALLS, full_waits);
    }
}

template <int BN2, int ST, int SUB>
__device__ __forceinline__ void pair_mma(const KParams& p, uint8_t* smem, uint32_t tmem_base, uint64_t* full,
                                         uint64_t* empty, uint64_t* tfull, uint64_t* tempty, uint64_t* drain,
                                         TileQueue& q, const Deadline& dl) {
    if (p.dtype == AGG_DTYPE_E4M3)
        pair_mma_loop<BN2, ST, SUB, true>(p, smem, tmem_base, full, empty, tfull, tempty, q, dl);
    else
        pair_mma_loop<BN2, ST, SUB, false>(p, smem, tmem_base, full, empty, tfull, tempty, q, dl);
    // Every MMA issued has finished once `drain` flips.
    umma_commit_pair_mc_warp(drain, 0x1);
    int drained = 1;
    if (lane_id() == 0) {
        drained = mbar_wait_for(drain, 0, 500000000ull) ? 1 : 0;
        if (!drained) record_failure(p.status, AGG_ROLE_DRAIN, 2u);
        if (p.trace) trace_set(p, AGG_TR_MMA_DONE, globaltimer_ns());
    }
    __syncwarp();
}

// Reduce-scatter: one warp's slice of tile `tile` has landed in the owner's
// inbox (its TMA stores completed): order it before the count, then raise the
// tile's counter on every GPU.
//
// With the copy-engine exchange a slice of another owner's tile has landed in
// the local stage: count it on this GPU's counter for that owner, which the
// copy stream waits on.  A slice of an own tile is counted on this GPU only.
__device__ __forceinline__ void rs_publish(const KParams& p, int tile) {
    fence_proxy_async_global();
    fence_acq_rel_sys();
    if (p.rs_ce) {
        const int L = p.m_local / 256;
        const int mt = tile / p.num_n_tiles;
        const int owner = mt / L;
        const int chunk = (mt - owner * L) / min(p.group_m, L);  // the group of m-tiles rs_block_tile runs together
        red_add_release_sys_u32(owner == p.rank ? p.flags_uc + tile : p.ce_cnt + owner * p.ce_chunks + chunk, 1u);
        return;
    }
    mm_red_add_release_u32(p.flags_mc + tile, 1u);
}

template <int BN2, int ST, int SUB, bool RS = false>
__device__ __forceinline__ void pair_epilogue(const KParams& p, uint8_t* smem, uint32_t tmem_base, uint64_t* tfull,
                                              uint64_t* tempty, TileQueue& q, int warp, uint32_t crank,
                                              const Deadline& dl) {
    using G = PairG<BN2, ST, SUB, RS>;
    const int eg = warp & 3;
    const uint32_t lane = lane_id();
    uint8_t* stg = smem + G::EPI_OFF + (warp - 2) * G::EPI_BUFS * EPI_BUF_BYTES;
    const bool f8 = p.dtype == AGG_DTYPE_E4M3;
    int acc = 0;
    uint32_t acc_phase = 0;
    int buf = 0;
    int rs_pending = -1;  // reduce-scatter: the tile whose slice awaits its count
    if constexpr (RS) {
        // The inbox slots this launch writes were last read (by every owner's
        // reducers) two launches ago with double buffering, else by the
        // previous launch: wait until every rank is done.
        if (p.gate_done > 0) {
            int ok = 1;
            if (lane == 0) ok = wait_flag_geq(p.done_uc, p.gate_done, dl) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) record_failure(p.status, AGG_ROLE_PROD, 1u);
                return;
            }
            fence_proxy_alias();
        }
    }
    for (;;) {
        int t = 0;
        if (lane == 0) t = tq_read(q, dl);
        t = __shfl_sync(0xffffffffu, t, 0);
        if (t == -2) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_EPI, 0xFFFFFFu);
            break;
        }
        if (t < 0) break;
        int mt, nt;
        if constexpr (RS)
            rs_tile_coords(p, t, mt, nt);
        else
            tile_coords(p, t, mt, nt);
        int got = 1;
        if (lane == 0) got = mbar_wait_sleepy(&tfull[acc], acc_phase, dl) ? 1 : 0;
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_EPI, static_cast<uint32_t>(t));
            break;
        }
        tc_fence_after();
        const uint32_t tbase =
            tmem_base + (static_cast<uint32_t>(eg * 32) << 16) + static_cast<uint32_t>(acc * BN2);
        const int row0 = mt * G::TILE_M + static_cast<int>(crank) * 128 + eg * 32;
        const float row_scale = f8 ? epilogue_row_scale(p, row0, lane, dl) : 1.0f;
#pragma unroll 1
        for (int j = 0; j < BN2 / EPI_COLS; ++j) {
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(j * EPI_COLS), r0);
            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(j * EPI_COLS + 32), r1);
            tmem_wait_ld();
            const int col0 = nt * BN2 + j * EPI_COLS;
            uint32_t packed[32];
            if (f8) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = col0 + 2 * i;
                    const float s0 = c < p.N ? __ldg(p.scale_b + c) : 0.0f;
                    const float s1 = c + 1 < p.N ? __ldg(p.scale_b + c + 1) : 0.0f;
                    packed[i] = pack_bf16x2(__uint_as_float(r0[2 * i]) * row_scale * s0,
                                            __uint_as_float(r0[2 * i + 1]) * row_scale * s1);
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = col0 + 32 + 2 * i;
                    const float s0 = c < p.N ? __ldg(p.scale_b + c) : 0.0f;
                    const float s1 = c + 1 < p.N ? __ldg(p.scale_b + c + 1) : 0.0f;
                    packed[16 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]) * row_scale * s0,
                                                 __uint_as_float(r1[2 * i + 1]) * row_scale * s1);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    packed[i] = pack_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    packed[16 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
            }
            if (j == BN2 / EPI_COLS - 1) {
                // Every TMEM read of this accumulator is done: hand it back to the
                // MMA issuer before the last stores go out.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
            }
            if constexpr (G::STAGED_EPI) {
                if (lane == 0) bulk_wait_group_read<G::EPI_BUFS - 1>();
                __syncwarp();
                uint8_t* b = stg + buf * EPI_BUF_BYTES;
                const uint32_t row_base = smem_u32(b) + lane * 128u;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint32_t addr = row_base + ((static_cast<uint32_t>(c) ^ (lane & 7u)) << 4);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(packed[4 * c]),
                                 "r"(packed[4 * c + 1]), "r"(packed[4 * c + 2]), "r"(packed[4 * c + 3])
                                 : "memory");
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (RS) {
                        // into slot `rank` of the owner's inbox (over NVLink for the
                        // other ranks), row within the owner's block
                        const int owner = row0 / p.m_local;
                        tma_store_2d(&p.tm_out[owner], b, col0, row0 - owner * p.m_local);
                    } else {
                        tma_store_2d(&p.tm_c, b, col0, row0);
                    }
                    bulk_commit_group();
                }
                if (++buf == G::EPI_BUFS) buf = 0;
            } else {
                // One row per thread, 16-byte segments straight to global memory.
                const int row = row0 + static_cast<int>(lane);
                if (row < p.M) {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.c_ptr) +
                                                          static_cast<size_t>(row) * p.N + col0);
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        if (col0 + 8 * c < p.N)
                            __stcs(dst + c, make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2],
                                                       packed[4 * c + 3]));
                }
            }
        }
        if constexpr (RS) {
            // This warp's 32-row slice of the partial tile is out.  It is counted
            // (on the tile's counter in every GPU, 8 slices per tile and rank) once
            // its TMA stores have landed, which the warp checks only after issuing
            // the next tile's stores: the wait then leaves that tile's
            // BN2/EPI_COLS store groups in flight.
            // With the copy-engine exchange every store is local and lands within
            // a microsecond or two, far inside the next tile's MMA time: the warp
            // waits for it and counts the slice at once, so that a block's copy
            // and an own tile's reduction do not wait a tile longer.
            static_assert(G::STAGED_EPI, "reduce-scatter publishes TMA-stored slices");
            if (lane == 0 && p.rs_ce) {
                bulk_wait_group<0>();
                rs_publish(p, mt * p.num_n_tiles + nt);
            } else if (lane == 0) {
                if (rs_pending >= 0) {
                    bulk_wait_group<BN2 / EPI_COLS>();
                    rs_publish(p, rs_pending);
                }
                rs_pending = mt * p.num_n_tiles + nt;
            }
            __syncwarp();
        }
        if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
        }
    }
    if (lane == 0) {
        bulk_wait_group<0>();
        if (RS && rs_pending >= 0) rs_publish(p, rs_pending);
        if (p.trace) trace_max(p, AGG_TR_EPI_DONE, globaltimer_ns());
    }
    __syncwarp();
}

template <int BN2, int ST, int SUB, bool RS = false>
__global__ void __launch_bounds__(NUM_THREADS, 1) ag_gemm_pair_kernel(const __grid_constant__ KParams p) {
    using G = PairG<BN2, ST, SUB, RS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::BAR_OFF);
    uint64_t* full = bars;
    uint64_t* empty = bars + G::STAGES;
    uint64_t* tfull = bars + 2 * G::STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::SLOT_OFF);
    TileQueue q{reinterpret_cast<int*>(smem + G::TQ_OFF), drain + 1, drain + 1 + TQ_DEPTH, 0};

    const int warp = static_cast<int>(threadIdx.x >> 5);
    const uint32_t lane = lane_id();
    const uint32_t crank = cluster_ctarank();
    Deadline dl;
    dl.end_ns = globaltimer_ns() + (p.timeout_ns ? p.timeout_ns : 10000000000ull);
    dl.status = p.status;
    if (p.trace && threadIdx.x == 0) trace_set(p, AGG_TR_START, globaltimer_ns());

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * EPI_WARPS);
        }
        mbar_init(drain, 1);
        for (int s = 0; s < TQ_DEPTH; ++s) {
            mbar_init(&q.full[s], 1);
            mbar_init(&q.empty[s], TQ_READERS);
        }
        fence_mbarrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, G::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or complete_tx
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

    // Reduce-scatter: every warp that has no GEMM work left sums owned tiles
    // (role_reducer takes them by ticket, in completion order): the loader,
    // MMA and epilogue warps as soon as their part of the GEMM is done, and
    // the two warps that produce nothing in this mode together with the
    // loader (named barrier 1).  Reducing from the start of the launch instead
    // slowed the GEMM by more than it saved.
    if (warp == 0) {
        if (lane == 0) pair_loader<BN2, ST, SUB, RS>(p, smem, full, empty, q, crank, dl);
        __syncwarp();
        if constexpr (RS) {
            named_barrier_sync(1, 3 * 32);
            role_reducer(p, dl);
        }
    } else if (warp == 1) {
        if (crank == 0) pair_mma<BN2, ST, SUB>(p, smem, tmem_base, full, empty, tfull, tempty, drain, q, dl);
        __syncwarp();
        if constexpr (RS) role_reducer(p, dl);
    } else if (warp < 2 + EPI_WARPS) {
        pair_epilogue<BN2, ST, SUB, RS>(p, smem, tmem_base, tfull, tempty, q, warp, crank, dl);
        if constexpr (RS) role_reducer(p, dl);
    } else if constexpr (RS) {
        static_assert(NUM_WARPS - 2 - EPI_WARPS == 2, "warps 0, 6, 7 meet at barrier 1");
        named_barrier_sync(1, 3 * 32);
        role_reducer(p, dl);
    } else if (p.world > 1) {
        role_producer(p, warp - 2 - EPI_WARPS, dl);
    }

    tc_fence_before();
    __syncthreads();
    if (failed(p.status)) {
        // A role gave up: let copies the peer CTA issued toward this CTA land
        // before the pair dissolves.
        const uint64_t until = globaltimer_ns() + 2000000ull;
        while (globaltimer_ns() < until) {
        }
    }
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, G::TMEM_COLS);
    }
    if (p.trace && threadIdx.x == 0) trace_set(p, AGG_TR_END, globaltimer_ns());
    if (p.dynamic && threadIdx.x == 0) {
        // Every tile this CTA took was taken above (program order, then the
        // fence): the last CTA to get here readies the slot for its next launch.
        __threadfence();
        SchedSlot& sl = g_sched[p.sched_slot];
        if (atomicAdd(&sl.done, 1u) == gridDim.x - 1u) {
            atomicExch(&sl.next, 0u);
            atomicExch(&sl.done, 0u);
        }
    }
    if (p.world > 1 && threadIdx.x == 0) {
        __threadfence();
        const uint32_t prev = atomicAdd(p.cta_counter, 1u);
        if (prev == gridDim.x - 1u) {
            if (p.rs_ce && failed(p.status)) rs_ce_release(p);
            atomicExch(p.cta_counter, 0u);
            atomicExch(p.ticket, 0ull);  // every producer of this launch is done
            fence_acq_rel_sys();
            mm_red_add_release_u32(p.done_mc, 1u);
        }
    }
}

// ================================================================ wide CTA-pair kernel
//
// The pair computes a 256 x 512 tile as two N=256 halves that share every A
// k-block: per k-step the even CTA issues two tcgen05.mma.cta_group::2, one per
// half.  Per SM that is 25% fewer operand bytes from L2 per FLOP than the
// 256 x 256 tile.  The accumulator (128 x 512 fp32 per CTA) fills TMEM, so
// there is one accumulator; the epilogue releases each half (tempty[0], [1])
// as soon as it has read it, and the next tile's first MMAs into a half wait
// only for that half.
//
// ST stages of 48 KiB.  The epilogue writes C in one of three ways:
//   EB >= 2  stage each 32 x 64 chunk in one of EB 4 KiB buffers per warp and
//            TMA-store it (a buffer is reused once its store has read it);
//   EB == 1  stage the chunk in the warp's one buffer, read it back transposed
//            (8 lanes per 128-byte row) and write whole rows with coalesced
//            16-byte st.global: no async-proxy fence, no wait for a store to
//            finish reading shared memory, so the accumulator drains fastest;
//   EB == 0  each lane writes its own row straight from registers.
template <int ST, int EB>
struct WideCfg {
    static constexpr int TILE_M = 256;
    static constexpr int TILE_N = 512;
    static constexpr int A_BYTES = 128 * BK_BYTES;     // 16 KiB
    static constexpr int B_HALF = 128 * BK_BYTES;      // this CTA's 128 rows of one N half
    static constexpr int STAGE = A_BYTES + 2 * B_HALF;  // 48 KiB
    static constexpr int STAGES = ST;
    static constexpr int EPI_BUFS = EB;
    static constexpr int EPI_OFF = STAGES * STAGE;
    static constexpr int BAR_OFF = EPI_OFF + EPI_WARPS * EB * EPI_BUF_BYTES;
    static constexpr int NUM_BARS = 2 * STAGES + 1 + 2 + 1 + 2 * TQ_DEPTH;
    static constexpr int SLOT_OFF = BAR_OFF + NUM_BARS * 8;
    static constexpr int TQ_OFF = SLOT_OFF + 16;  // int tile ids [TQ_DEPTH]
    static constexpr int SMEM = TQ_OFF + 4 * TQ_DEPTH + 1024;
    static constexpr uint32_t TMEM_COLS = 512;
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(EPI_OFF % 1024 == 0 && STAGE % 1024 == 0, "swizzle alignment");
};

// The wide kernel's work item i: a whole 256 x 512 tile (halves = 3), or, for
// the tiles of a short last wave, one 256 x 256 half of it (halves = 1 or 2),
// so that the last wave takes half a tile's time on twice as many pairs.
__device__ __forceinline__ void wide_item(const KParams& p, int i, int& t, uint32_t& halves) {
    if (i < p.split_from) {
        t = i;
        halves = 3u;
        return;
    }
    const int j = i - p.split_from;
    t = p.split_from + (j >> 1);
    halves = 1u << (j & 1);
}

template <int ST, int EB>
__device__ __forceinline__ void wide_loader(const KParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                            TileQueue& q, uint32_t crank, const Deadline& dl) {
    using G = WideCfg<ST, EB>;
    tma_prefetch_desc(&p.tm_a_src);
    tma_prefetch_desc(&p.tm_b);
    if (p.world > 1) tma_prefetch_desc(&p.tm_a_gath);
    const int kb_elems = p.dtype == AGG_DTYPE_BF16 ? BK_BYTES / 2 : BK_BYTES;
    int rr = static_cast<int>(blockIdx.x >> 1);  // round-robin schedule: this pair's next tile
    int stage = 0;
    uint32_t phase = 0;
    uint32_t used = 0, last_par = 0;
    bool ok = true;
    FlagWaitLog log;
    while (ok) {
        const int item = crank == 0 ? tq_fill(p, q, rr, dl) : tq_read(q, dl);
        if (item == -2) {
            record_failure(p.status, AGG_ROLE_TMA, 0xFFFFFFu);
            break;
        }
        if (item < 0) break;
        int t, mt, nt;
        uint32_t halves;
        wide_item(p, item, t, halves);
        tile_coords(p, t, mt, nt);
        ++log.tiles;
        const int row = mt * G::TILE_M + static_cast<int>(crank) * 128;
        const CUtensorMap* tma = &p.tm_a_src;
        int a_row = row;
        if (p.world > 1) {
            const int src = row / p.m_local;
            if (src == p.rank) {
                a_row = row - src * p.m_local;
            } else {
                const uint32_t* f = p.flags_uc + src * AGG_MAX_CHUNKS + (row - src * p.m_local) / BM;
                if (!log.wait(p, f, dl)) {
                    record_failure(p.status, AGG_ROLE_FLAG, static_cast<uint32_t>(row / BM));
                    ok = false;
                    break;
                }
                fence_proxy_alias();
                fence_proxy_async_global();
                tma = &p.tm_a_gath;
            }
        }
        const int b_row0 = nt * G::TILE_N + static_cast<int>(crank) * 128;  // half 0; half 1 is +256
        for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!mbar_wait_timed(&empty[stage], phase ^ 1u, dl, p.trace != nullptr, log.stage_wait, log.stage_waits)) {
                record_failure(p.status, AGG_ROLE_TMA, static_cast<uint32_t>(t));
                ok = false;
                break;
            }
            uint8_t* sa = smem + stage * G::STAGE;
            uint8_t* sb = sa + G::A_BYTES;
            if (crank == 0)
                mbar_arrive_expect_tx(&full[stage], 2u * (G::A_BYTES + (halves == 3u ? 2u : 1u) * G::B_HALF));
            const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
            const int kx = kb * kb_elems;
            tma_load_2d_pair(tma, sa, bar, kx, a_row);
            if (halves & 1u) tma_load_2d_pair(&p.tm_b, sb, bar, kx, b_row0);
            if (halves & 2u) tma_load_2d_pair(&p.tm_b, sb + G::B_HALF, bar, kx, b_row0 + 256);
            used |= 1u << stage;
            last_par = (last_par & ~(1u << stage)) | (phase << stage);
            if (++stage == G::STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
    log.flush(p);
    if (crank == 0)
        for (int s = 0; s < G::STAGES; ++s)
            if (used & (1u << s))
                if (!mbar_wait_for(&full[s], (last_par >> s) & 1u, 200000000ull))
                    record_failure(p.status, AGG_ROLE_DRAIN, 1u);
}

// The whole warp runs the loop, one elected lane issues (see pair_mma_loop).
template <int ST, int EB, bool F8>
__device__ __forceinline__ void wide_mma_loop(const KParams& p, uint8_t* smem, uint32_t tmem_base, uint64_t* full,
                                              uint64_t* empty, uint64_t* tfull, uint64_t* tempty, TileQueue& q,
                                              const Deadline& dl) {
    using G = WideCfg<ST, EB>;
    constexpr uint32_t IDESC = F8 ? make_idesc(0, 0, G::TILE_M, 256) : make_idesc(1, 1, G::TILE_M, 256);
    const uint32_t lane = lane_id();
    const bool tr = p.trace != nullptr;
    const uint64_t desc0 = sw128_kmajor_desc(smem_u32(smem));
    int stage = 0;
    uint32_t phase = 0;
    uint32_t uses[2] = {0u, 0u};  // items so far that accumulated into each half
    unsigned long long full_wait = 0, full_waits = 0, acc_wait = 0;
    for (;;) {
        int item = 0;
        if (lane == 0) item = tq_read(q, dl);
        item = __shfl_sync(0xffffffffu, item, 0);
        if (item == -2) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_MMA, 0xFFFFFFu);
            break;
        }
        if (item < 0) break;
        int t;
        uint32_t halves;
        wide_item(p, item, t, halves);
        bool ok = true;
        for (int kb = 0; kb < p.num_kb && ok; ++kb) {
            if (!__all_sync(0xffffffffu, mbar_try_wait(smem_u32(&full[stage]), phase))) {
                const unsigned long long t0 = tr ? globaltimer_ns() : 0ull;
                ok = mbar_wait_warp(&full[stage], phase, dl);
                if (tr) {
                    full_wait += globaltimer_ns() - t0;
                    ++full_waits;
                }
                if (!ok) break;
            }
            const uint64_t adesc = desc0 + static_cast<uint64_t>((stage * G::STAGE) >> 4);
            const uint64_t bdesc0 = adesc + static_cast<uint64_t>(G::A_BYTES >> 4);
            const uint64_t bdesc1 = bdesc0 + static_cast<uint64_t>(G::B_HALF >> 4);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint64_t off = static_cast<uint64_t>(k * 2);
                const uint32_t accumulate = (kb > 0 || k > 0) ? 1u : 0u;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (!((halves >> h) & 1u)) continue;
                    if (kb == 0 && k == 0) {
                        // the epilogue must have read this half of the last item that used it
                        const unsigned long long ta = tr ? globaltimer_ns() : 0ull;
                        ok = mbar_wait_warp(&tempty[h], (uses[h] & 1u) ^ 1u, dl);
                        if (tr) acc_wait += globaltimer_ns() - ta;
                        if (!ok) break;
                        tc_fence_after();
                    }
                    const uint32_t d = tmem_base + static_cast<uint32_t>(h * 256);
                    const uint64_t bd = (h ? bdesc1 : bdesc0) + off;
                    if constexpr (F8)
                        umma_f8_pair_warp(d, adesc + off, bd, IDESC, accumulate);
                    else
                        umma_f16_pair_warp(d, adesc + off, bd, IDESC, accumulate);
                }
                if (!ok) break;
            }
            if (!ok) break;
            umma_commit_pair_mc_warp(&empty[stage], 0x3);
            if (++stage == G::STAGES) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if (!ok) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_MMA, static_cast<uint32_t>(t));
            break;
        }
        umma_commit_pair_mc_warp(tfull, 0x3);
        for (int h = 0; h < 2; ++h) uses[h] += (halves >> h) & 1u;
    }
    if (tr && lane == 0) {
        trace_set(p, AGG_TR_MMA_WAIT_NS, full_wait);
        trace_set(p, AGG_TR_MMA_ACC_NS, acc_wait);
        trace_set(p, AGG_TR_MMA_STALLS, full_waits);
    }
}

template <int ST, int EB>
__device__ __forceinline__ void wide_mma(const KParams& p, uint8_t* smem, uint32_t tmem_base, uint64_t* full,
                                         uint64_t* empty, uint64_t* tfull, uint64_t* tempty, uint64_t* drain,
                                         TileQueue& q, const Deadline& dl) {
    if (p.dtype == AGG_DTYPE_E4M3)
        wide_mma_loop<ST, EB, true>(p, smem, tmem_base, full, empty, tfull, tempty, q, dl);
    else
        wide_mma_loop<ST, EB, false>(p, smem, tmem_base, full, empty, tfull, tempty, q, dl);
    umma_commit_pair_mc_warp(drain, 0x1);
    if (lane_id() == 0) {
        if (!mbar_wait_for(drain, 0, 500000000ull)) record_failure(p.status, AGG_ROLE_DRAIN, 2u);
        if (p.trace) trace_set(p, AGG_TR_MMA_DONE, globaltimer_ns());
    }
    __syncwarp();
}

template <int ST, int EB>
__device__ __forceinline__ void wide_epilogue(const KParams& p, uint8_t* smem, uint32_t tmem_base, uint64_t* tfull,
                                              uint64_t* tempty, TileQueue& q, int warp, uint32_t crank,
                                              const Deadline& dl) {
    using G = WideCfg<ST, EB>;
    const int eg = warp & 3;
    const uint32_t lane = lane_id();
    uint8_t* stg = smem + G::EPI_OFF + (warp - 2) * EB * EPI_BUF_BYTES;
    const bool f8 = p.dtype == AGG_DTYPE_E4M3;
    uint32_t acc_phase = 0;
    int buf = 0;
    for (;;) {
        int item = 0;
        if (lane == 0) item = tq_read(q, dl);
        item = __shfl_sync(0xffffffffu, item, 0);
        if (item == -2) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_EPI, 0xFFFFFFu);
            break;
        }
        if (item < 0) break;
        int t, mt, nt;
        uint32_t halves;
        wide_item(p, item, t, halves);
        tile_coords(p, t, mt, nt);
        int got = 1;
        if (lane == 0) got = mbar_wait_sleepy(tfull, acc_phase, dl) ? 1 : 0;
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
            if (lane == 0) record_failure(p.status, AGG_ROLE_EPI, static_cast<uint32_t>(t));
            break;
        }
        tc_fence_after();
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(eg * 32) << 16);
        const int row0 = mt * G::TILE_M + static_cast<int>(crank) * 128 + eg * 32;
        const float row_scale = f8 ? epilogue_row_scale(p, row0, lane, dl) : 1.0f;
        // Chunk j: columns [64j, 64j + 64) of this warp's 32 accumulator rows.
        // Its TMEM load is issued one chunk ahead, so the load's latency
        // (about 400 cycles before the registers can be used) overlaps the
        // previous chunk's conversion and stores.
        auto chunk_out = [&](const uint32_t (&r0)[32], const uint32_t (&r1)[32], int j) {
            if ((j & 3) == 3) {
                // this N half is read: the next tile may accumulate into it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[j >> 2]), 0));
            }
            const int col0 = nt * G::TILE_N + j * EPI_COLS;
            uint32_t packed[32];
            if (f8) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = col0 + 2 * i;
                    const float s0 = c < p.N ? __ldg(p.scale_b + c) : 0.0f;
                    const float s1 = c + 1 < p.N ? __ldg(p.scale_b + c + 1) : 0.0f;
                    packed[i] = pack_bf16x2(__uint_as_float(r0[2 * i]) * row_scale * s0,
                                            __uint_as_float(r0[2 * i + 1]) * row_scale * s1);
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = col0 + 32 + 2 * i;
                    const float s0 = c < p.N ? __ldg(p.scale_b + c) : 0.0f;
                    const float s1 = c + 1 < p.N ? __ldg(p.scale_b + c + 1) : 0.0f;
                    packed[16 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]) * row_scale * s0,
                                                 __uint_as_float(r1[2 * i + 1]) * row_scale * s1);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    packed[i] = pack_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    packed[16 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
            }
            if constexpr (EB == 1) {
                // Rows go into the buffer one per lane (128-byte swizzle, no bank
                // conflicts), come back 8 lanes per row, and leave as 4 whole rows
                // per store instruction.
                const uint32_t buf_base = smem_u32(stg);
                const uint32_t row_base = buf_base + lane * 128u;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint32_t addr = row_base + ((static_cast<uint32_t>(c) ^ (lane & 7u)) << 4);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(packed[4 * c]),
                                 "r"(packed[4 * c + 1]), "r"(packed[4 * c + 2]), "r"(packed[4 * c + 3])
                                 : "memory");
                }
                __syncwarp();
                const uint32_t seg = lane & 7u;
                const int col = col0 + static_cast<int>(seg) * 8;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t r = static_cast<uint32_t>(i) * 4u + (lane >> 3);
                    uint4 v;
                    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                                 : "r"(buf_base + r * 128u + ((seg ^ (r & 7u)) << 4))
                                 : "memory");
                    const int row = row0 + static_cast<int>(r);
                    if (row < p.M && col < p.N)
                        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.c_ptr) +
                                                  static_cast<size_t>(row) * p.N + col) = v;
                }
                __syncwarp();  // every lane has read the buffer before the next chunk fills it
            } else if constexpr (EB == 0) {
                // One row per lane, 16-byte segments straight to global memory.
                const int row = row0 + static_cast<int>(lane);
                if (row < p.M && col0 < p.N) {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.c_ptr) +
                                                          static_cast<size_t>(row) * p.N + col0);
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        if (col0 + 8 * c < p.N)
                            __stcs(dst + c, make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2],
                                                       packed[4 * c + 3]));
                }
            } else if (col0 < p.N) {
                // The buffer is free once the TMA store issued EB chunks ago has read it.
                if (lane == 0) bulk_wait_group_read<EB - 1>();
                __syncwarp();
                uint8_t* b = stg + buf * EPI_BUF_BYTES;
                const uint32_t row_base = smem_u32(b) + lane * 128u;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint32_t addr = row_base + ((static_cast<uint32_t>(c) ^ (lane & 7u)) << 4);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(packed[4 * c]),
                                 "r"(packed[4 * c + 1]), "r"(packed[4 * c + 2]), "r"(packed[4 * c + 3])
                                 : "memory");
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&p.tm_c, b, col0, row0);
                    bulk_commit_group();
                }
                if (++buf == EB) buf = 0;
            }
        };
        const int jbeg = (halves & 1u) ? 0 : 4;
        const int jend = (halves & 2u) ? 8 : 4;
        uint32_t a0[32], a1[32], b0[32], b1[32];
        tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(jbeg * EPI_COLS), a0);
        tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(jbeg * EPI_COLS + 32), a1);
        tmem_wait_ld();
        regs_ready(a0);
        regs_ready(a1);
#pragma unroll 1
        for (int j = jbeg; j < jend; j += 2) {  // a half has 4 chunks: they come in pairs
            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>((j + 1) * EPI_COLS), b0);
            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>((j + 1) * EPI_COLS + 32), b1);
            chunk_out(a0, a1, j);
            tmem_wait_ld();
            regs_ready(b0);
            regs_ready(b1);
            const bool more = j + 2 < jend;
            if (more) {
                tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>((j + 2) * EPI_COLS), a0);
                tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>((j + 2) * EPI_COLS + 32), a1);
            }
            chunk_out(b0, b1, j + 1);
            if (more) {
                tmem_wait_ld();
                regs_ready(a0);
                regs_ready(a1);
            }
        }
        acc_phase ^= 1u;
    }
    if (lane == 0) {
        bulk_wait_group<0>();
        if (p.trace) trace_max(p, AGG_TR_EPI_DONE, globaltimer_ns());
    }
    __syncwarp();
}

template <int ST, int EB>
__global__ void __launch_bounds__(NUM_THREADS, 1) ag_gemm_wide_kernel(const __grid_constant__ KParams p) {
    using G = WideCfg<ST, EB>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::BAR_OFF);
    uint64_t* full = bars;
    uint64_t* empty = bars + G::STAGES;
    uint64_t* tfull = bars + 2 * G::STAGES;
    uint64_t* tempty = tfull + 1;  // [2]: one per N half
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::SLOT_OFF);
    TileQueue q{reinterpret_cast<int*>(smem + G::TQ_OFF), drain + 1, drain + 1 + TQ_DEPTH, 0};

    const int warp = static_cast<int>(threadIdx.x >> 5);
    const uint32_t lane = lane_id();
    const uint32_t crank = cluster_ctarank();
    Deadline dl;
    dl.end_ns = globaltimer_ns() + (p.timeout_ns ? p.timeout_ns : 10000000000ull);
    dl.status = p.status;
    if (p.trace && threadIdx.x == 0) trace_set(p, AGG_TR_START, globaltimer_ns());

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(&tempty[0], 2 * EPI_WARPS);
        mbar_init(&tempty[1], 2 * EPI_WARPS);
        mbar_init(drain, 1);
        for (int s = 0; s < TQ_DEPTH; ++s) {
            mbar_init(&q.full[s], 1);
            mbar_init(&q.empty[s], TQ_READERS);
        }
        fence_mbarrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, G::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

    if (warp == 0) {
        if (lane == 0) wide_loader<ST, EB>(p, smem, full, empty, q, crank, dl);
    } else if (warp == 1) {
        if (crank == 0) wide_mma<ST, EB>(p, smem, tmem_base, full, empty, tfull, tempty, drain, q, dl);
        __syncwarp();
    } else if (warp < 2 + EPI_WARPS) {
        wide_epilogue<ST, EB>(p, smem, tmem_base, tfull, tempty, q, warp, crank, dl);
    } else if (p.world > 1) {
        role_producer(p, warp - 2 - EPI_WARPS, dl);
    }

    tc_fence_before();
    __syncthreads();
    if (failed(p.status)) {
        const uint64_t until = globaltimer_ns() + 2000000ull;
        while (globaltimer_ns() < until) {
        }
    }
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, G::TMEM_COLS);
    }
    if (p.trace && threadIdx.x == 0) trace_set(p, AGG_TR_END, globaltimer_ns());
    if (p.dynamic && threadIdx.x == 0) {
        __threadfence();
        SchedSlot& sl = g_sched[p.sched_slot];
        if (atomicAdd(&sl.done, 1u) == gridDim.x - 1u) {
            atomicExch(&sl.next, 0u);
            atomicExch(&sl.done, 0u);
        }
    }
    if (p.world > 1 && threadIdx.x == 0) {
        __threadfence();
        const uint32_t prev = atomicAdd(p.cta_counter, 1u);
        if (prev == gridDim.x - 1u) {
            if (p.rs_ce && failed(p.status)) rs_ce_release(p);
            atomicExch(p.cta_counter, 0u);
            atomicExch(p.ticket, 0ull);
            fence_acq_rel_sys();
            mm_red_add_release_u32(p.done_mc, 1u);
        }
    }
}

// ---------------------------------------------------------------- host side
namespace {

int encode_2d(CUtensorMap* m, CUtensorMapDataType dt, size_t elem, const void* base, uint64_t inner,
              uint64_t outer, uint32_t box_inner, uint32_t box_outer, const char* what) {
    const DriverApi& d = driver();
    if (!d.ok) return fail(AGG_EDRIVER, "CUDA driver unavailable: %s", d.why.c_str());
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
        return fail(AGG_EINVAL, "%s: base address %p is not 16-byte aligned", what, base);
    if ((inner * elem) % 16 != 0)
        return fail(AGG_EINVAL, "%s: row pitch %llu bytes is not a multiple of 16", what,
                    static_cast<unsigned long long>(inner * elem));
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * elem};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = d.cuTensorMapEncodeTiled(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return check_drv(r, what);
    return AGG_OK;
}

// First tile of the wide kernel to run as two half tiles: when the last wave
// would hold r whole tiles, and 2r half tiles still fit in one wave of
// `clusters` pairs, the last wave takes half a tile's time instead of a whole
// one.  AGG_WIDE_SPLIT=0 keeps whole tiles.
int env_int(const char* name, int dflt);
int wide_split(long tiles, int clusters) {
    if (clusters < 1 || tiles <= clusters || env_int("AGG_WIDE_SPLIT", 1) == 0) return static_cast<int>(tiles);
    const long r = tiles % clusters;
    if (r == 0 || 2 * r > clusters) return static_cast<int>(tiles);
    return static_cast<int>(tiles - r);
}

int current_sms(int* dev_out) {
    int dev = 0;
    AGG_RT(cudaGetDevice(&dev));
    int sms = 0;
    AGG_RT(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (dev_out) *dev_out = dev;
    return sms;
}

int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    if (!v || !*v) return dflt;
    return atoi(v);
}

}  // namespace

namespace {

// The CTA-pair kernel instantiations: tile width x pipeline depth x k sub-blocks
// per stage.  SUB = 2 (8 MMAs per stage) is the default; SUB = 1 with twice the
// stages is kept for comparison.
struct PairKernel {
    const void* fn;
    int smem;
    int bn;      // output columns per pair tile
    int b_box;   // B rows one CTA loads per TMA box
    int stages;
    int sub;     // 128-byte k sub-blocks per stage
    bool wide;   // 256 x 512 tile with one accumulator
    float cost;  // relative time per output element (measured on the 70B MLP shape)
    int clusters;  // resident CTA pairs on this device
};

template <int BN2, int ST, int SUB>
PairKernel pair_kernel_entry(float cost) {
    using G = PairCfg<BN2, ST, SUB>;
    return PairKernel{reinterpret_cast<const void*>(&ag_gemm_pair_kernel<BN2, ST, SUB>), G::SMEM, BN2, BN2 / 2, ST, SUB,
                      false, cost, 0};
}

template <int ST, int EB>
PairKernel wide_kernel_entry(float cost) {
    using G = WideCfg<ST, EB>;
    return PairKernel{reinterpret_cast<const void*>(&ag_gemm_wide_kernel<ST, EB>), G::SMEM, G::TILE_N, 128,
                      G::STAGES, 1, true, cost, 0};
}

// pair[0..3]: 256 x 256 / 256 x 128 forms; pair[4 + w]: the wide kernel's form w
// (AGG_WIDE, read at each launch; kDefaultWide when unset).
constexpr int kNumPairKernels = 9;
constexpr int kDefaultWide = 1;

// Per-device launch facts, filled once: SM count and how many CTA pairs of each
// pair kernel can be resident at once (clusters must fit inside a GPC).
struct DevInfo {
    int sms = 0;
    PairKernel pair[kNumPairKernels];
    PairKernel rs;  // the reduce-scatter instantiation (256 x 256, 5 stages of 1 k-block, 4 buffers)
    int rc = AGG_OK;
    std::string err;
};
DevInfo g_dev[64];
std::once_flag g_dev_once[64];

int max_pair_clusters(const void* kern, int smem, int sms, int* out) {
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1), 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    AGG_RT(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    *out = n;
    return AGG_OK;
}

int device_info(int dev, const DevInfo** out) {
    if (dev < 0 || dev >= 64) return fail(AGG_EINVAL, "device ordinal %d out of range", dev);
    std::call_once(g_dev_once[dev], [dev] {
        DevInfo& d = g_dev[dev];
        // Relative cost per output element, from sustained (power-capped) runs
        // of each variant on the 16384 x 57344 x 8192 and 16384 x 7168 x 8192
        // GEMMs.  The wide 256 x 512 tile reads a quarter fewer operand bytes
        // from L2 per FLOP, which the 1 kW cap turns into clock; its epilogue
        // is partly exposed (one accumulator fills TMEM), and it still comes
        // out ahead wherever its coarser waves do not cost more.
        d.pair[0] = pair_kernel_entry<256, 3, 2>(1.00f);
        d.pair[1] = pair_kernel_entry<256, 6, 1>(1.02f);
        d.pair[2] = pair_kernel_entry<128, 4, 2>(1.12f);
        d.pair[3] = pair_kernel_entry<128, 8, 1>(1.15f);
        // The wide kernel's stage / epilogue forms, by AGG_WIDE: 0 = 4 stages and
        // two TMA-store buffers per warp, 1 = 3 stages and four, 2 = 4 stages
        // and direct global stores, 3 = 4 stages and coalesced stores through
        // one buffer, 4 = the same with 3 stages.
        d.pair[4] = wide_kernel_entry<4, 2>(0.93f);
        d.pair[5] = wide_kernel_entry<3, 4>(0.93f);
        d.pair[6] = wide_kernel_entry<4, 0>(0.93f);
        d.pair[7] = wide_kernel_entry<4, 1>(0.93f);
        d.pair[8] = wide_kernel_entry<3, 1>(0.93f);
        d.rs = PairKernel{reinterpret_cast<const void*>(&ag_gemm_pair_kernel<256, 5, 1, true>),
                          PairG<256, 5, 1, true>::SMEM, 256, 128, 5, 1, false, 1.0f, 0};
        auto setup = [&]() -> int {
            AGG_RT(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
            AGG_RT(cudaFuncSetAttribute(ag_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC));
            for (PairKernel& k : d.pair) {
                AGG_RT(cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem));
                int rc = max_pair_clusters(k.fn, k.smem, d.sms, &k.clusters);
                if (rc) return rc;
            }
            AGG_RT(cudaFuncSetAttribute(d.rs.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, d.rs.smem));
            return max_pair_clusters(d.rs.fn, d.rs.smem, d.sms, &d.rs.clusters);
        };
        d.rc = setup();
        if (d.rc) d.err = agg_last_error();
    });
    if (g_dev[dev].rc) return fail(g_dev[dev].rc, "kernel setup failed: %s", g_dev[dev].err.c_str());
    *out = &g_dev[dev];
    return AGG_OK;
}


// One launch of a CTA-pair kernel: a persistent grid of as many pairs as fit
// at once (never more than there are tiles).
std::atomic<unsigned int> g_sched_seq[64];

int launch_pair(const PairKernel& k, KParams& p, cudaStream_t stream, int dev) {
    const int clusters = std::max(1, std::min(k.clusters, p.num_tiles));
    // Tile schedule: dynamic (tiles in raster order to whichever pair is free)
    // unless AGG_SCHED=static asks for the round-robin one.
    const char* sched = getenv("AGG_SCHED");
    p.dynamic = (sched && std::strcmp(sched, "static") == 0) ? 0 : 1;
    p.sched_slot = static_cast<int>(g_sched_seq[dev & 63].fetch_add(1u) % AGG_SCHED_SLOTS);
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters), 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(k.smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* kargs[] = {&p};
    AGG_RT(cudaLaunchKernelExC(&cfg, k.fn, kargs));
    return AGG_OK;
}

}  // namespace

int launch_ag_gemm(const agg_args* a, cudaStream_t stream) {
    if (!a) return fail(AGG_EINVAL, "agg_launch: null args");
    const int world = a->world;
    const bool f8 = a->dtype == AGG_DTYPE_E4M3;
    if (a->dtype != AGG_DTYPE_BF16 && !f8) return fail(AGG_EINVAL, "agg_launch: unknown dtype %d", a->dtype);
    if (world < 1 || world > AGG_MAX_RANKS) return fail(AGG_EINVAL, "agg_launch: world %d", world);
    if (a->dev_idx < 0 || a->dev_idx >= world) return fail(AGG_EINVAL, "agg_launch: rank %d", a->dev_idx);
    if (a->M <= 0 || a->N <= 0 || a->K <= 0) return fail(AGG_EINVAL, "agg_launch: empty shape");
    if (a->M % world) return fail(AGG_EINVAL, "agg_launch: M=%d not divisible by world=%d", a->M, world);
    const int m_local = a->M / world;
    const size_t elem = f8 ? 1 : 2;
    if ((static_cast<size_t>(a->K) * elem) % 16) return fail(AGG_EINVAL, "agg_launch: K*elem must be a multiple of 16");
    if (a->N % 8) return fail(AGG_EINVAL, "agg_launch: N must be a multiple of 8");
    if (!a->B || !a->C) return fail(AGG_EINVAL, "agg_launch: null B or C");
    if (f8 && (!a->scale_a || !a->scale_b)) return fail(AGG_EINVAL, "agg_launch: e4m3 needs scale_a and scale_b");
    if (world > 1) {
        if (m_local % BM) return fail(AGG_EINVAL, "agg_launch: M/world=%d must be a multiple of %d", m_local, BM);
        if (m_local / BM > AGG_MAX_CHUNKS) return fail(AGG_EINVAL, "agg_launch: M/world too large");
        if (!a->A_local_buf || !a->A_mc || !a->A_copy_ready || !a->A_copy_ready_mc || !a->done_uc || !a->done_mc)
            return fail(AGG_EINVAL, "agg_launch: multicast buffers missing");
        if (a->A_copy_epoch < 1) return fail(AGG_EINVAL, "agg_launch: epoch must start at 1");
    }
    const uint32_t ce_mode = a->flags & (AGG_ARGS_CE_MC_PUSH | AGG_ARGS_CE_PEER_PUSH);
    const bool peer_push = world > 1 && (a->flags & AGG_ARGS_SM_PEER_PUSH) != 0;
    if (peer_push) {
        if (ce_mode) return fail(AGG_EINVAL, "agg_launch: choose the copy engines or the SM peer push");
        if (f8) return fail(AGG_EINVAL, "agg_launch: the SM peer push moves bf16 shards only");
        for (int s = 0; s < world; ++s)
            if (!a->A_peer[s] || a->A_peer[s] % 16)
                return fail(AGG_EINVAL, "agg_launch: the SM peer push needs A_peer[%d] (16-byte aligned)", s);
        const uint64_t lb = reinterpret_cast<uint64_t>(a->A_local_buf);
        if (lb < a->A_peer[a->dev_idx] || (lb - a->A_peer[a->dev_idx]) % 16)
            return fail(AGG_EINVAL, "agg_launch: A_local_buf must lie in this rank's slab (A_peer[rank])");
    }
    if (ce_mode && world > 1) {
        if (ce_mode == (AGG_ARGS_CE_MC_PUSH | AGG_ARGS_CE_PEER_PUSH))
            return fail(AGG_EINVAL, "agg_launch: choose one copy-engine mode");
        if (!(a->flags & AGG_ARGS_DOUBLE_BUFFER) || f8)
            return fail(AGG_EINVAL, "agg_launch: copy-engine producers need bf16 and AGG_ARGS_DOUBLE_BUFFER");
        for (int s = 0; s < world; ++s)
            if (!a->A_peer[s]) return fail(AGG_EINVAL, "agg_launch: copy-engine producers need A_peer[%d]", s);
        const uint64_t ready = reinterpret_cast<uint64_t>(a->A_copy_ready);
        if (ready < a->A_peer[a->dev_idx] || ready % 4)
            return fail(AGG_EINVAL, "agg_launch: A_copy_ready must lie in this rank's slab (A_peer[rank])");
    }
    const void* a_src = a->A_src;
    if (!a_src) {
        if (!a->A_local_buf) return fail(AGG_EINVAL, "agg_launch: no A");
        a_src = static_cast<const uint8_t*>(a->A_local_buf) +
                static_cast<size_t>(a->dev_idx) * m_local * a->K * elem;
    }

    int dev = 0;
    AGG_RT(cudaGetDevice(&dev));
    const DevInfo* di = nullptr;
    int rc = device_info(dev, &di);
    if (rc) return rc;

    // ---- kernel choice.  A CTA-pair kernel unless the shard height forbids it
    // (a 256-row tile must not straddle two shards); among them the one with the
    // smallest estimated time = waves of tiles x tile area x relative cost, so
    // that wave quantisation of small problems is weighed against efficiency.
    // AGG_KERNEL=1sm|pair|wide, AGG_BN=128|256 and AGG_SUB=1|2 override it.
    const PairKernel* pk = nullptr;
    const char* kenv = getenv("AGG_KERNEL");
    const bool force_1sm = kenv && std::strcmp(kenv, "1sm") == 0;
    const bool force_wide = kenv && std::strcmp(kenv, "wide") == 0;
    const bool force_pair = kenv && std::strcmp(kenv, "pair") == 0;
    if (!force_1sm && !(world > 1 && m_local % 256)) {
        const int bn_env = env_int("AGG_BN", 0);
        const int sub_env = env_int("AGG_SUB", 2);
        const int wide_env = env_int("AGG_WIDE", kDefaultWide);
        double best = 0.0;
        for (int ki = 0; ki < kNumPairKernels; ++ki) {
            const PairKernel& k = di->pair[ki];
            if (k.clusters < 1) continue;
            if (k.wide && ki - 4 != wide_env) continue;
            if (force_wide && !k.wide) continue;
            if (force_pair && k.wide) continue;
            if (!k.wide && (k.sub != sub_env || (bn_env && k.bn != bn_env))) continue;
            if (k.wide && (bn_env || sub_env != 2)) continue;
            const long tiles = static_cast<long>((a->M + 255) / 256) * ((a->N + k.bn - 1) / k.bn);
            double waves = static_cast<double>((tiles + k.clusters - 1) / k.clusters);
            // the wide kernel runs a short last wave as half tiles (wide_split)
            if (k.wide && wide_split(tiles, k.clusters) < tiles) waves -= 0.5;
            const double est = waves * 256.0 * k.bn * k.cost;
            if (!pk || est < best) {
                pk = &k;
                best = est;
            }
        }
    }
    const int tile_m = pk ? 256 : BM;
    const int tile_n = pk ? pk->bn : BN;
    const int b_box = pk ? pk->b_box : BN;

    KParams p;
    std::memset(&p, 0, sizeof(p));
    const CUtensorMapDataType dt = f8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint32_t kb_elems = BK_BYTES / static_cast<uint32_t>(elem);
    // Double buffering: launch e uses gathered region and flag set (e & 1).
    const bool dbl = world > 1 && (a->flags & AGG_ARGS_DOUBLE_BUFFER) != 0;
    const uint32_t parity = dbl ? (a->A_copy_epoch & 1u) : 0u;
    const size_t region_off = static_cast<size_t>(parity) * a->M * a->K * elem;
    rc = encode_2d(&p.tm_a_src, dt, elem, a_src, a->K, world == 1 ? a->M : m_local, kb_elems, BM, "tensor map A shard");
    if (rc) return rc;
    if (world > 1) {
        rc = encode_2d(&p.tm_a_gath, dt, elem, static_cast<uint8_t*>(a->A_local_buf) + region_off, a->K, a->M,
                       kb_elems, BM, "tensor map gathered A");
        if (rc) return rc;
    }
    rc = encode_2d(&p.tm_b, dt, elem, a->B, a->K, a->N, kb_elems, static_cast<uint32_t>(b_box), "tensor map B");
    if (rc) return rc;
    rc = encode_2d(&p.tm_c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->C, a->N, a->M, EPI_COLS, EPI_ROWS, "tensor map C");
    if (rc) return rc;

    p.a_src = static_cast<const uint4*>(a_src);
    p.c_ptr = a->C;
    p.M = a->M;
    p.N = a->N;
    p.K = a->K;
    p.rank = a->dev_idx;
    p.world = world;
    p.m_local = m_local;
    p.tile_m = tile_m;
    p.num_m_tiles = (a->M + tile_m - 1) / tile_m;
    p.num_n_tiles = (a->N + tile_n - 1) / tile_n;
    p.num_tiles = p.num_m_tiles * p.num_n_tiles;
    p.split_from = p.num_tiles;
    if (pk && pk->wide) {
        // work items: whole tiles, then the last wave's tiles as halves
        p.split_from = wide_split(p.num_tiles, pk->clusters);
        p.num_tiles = p.split_from + 2 * (p.num_tiles - p.split_from);
    }
    const size_t kblock_bytes = static_cast<size_t>(BK_BYTES) * (pk ? pk->sub : 1);
    p.num_kb = static_cast<int>((static_cast<size_t>(a->K) * elem + kblock_bytes - 1) / kblock_bytes);
    // m-tiles of 256 rows per group.  One GPU: 12 (on the 16384 x 57344 x 8192
    // workload DRAM reads fall from 24 GB with 8 to 17 GB with 10 to 14).  Across
    // GPUs, where remote chunks are loaded from the slab as they arrive: 8
    // (1.54-1.58 ms against 1.68-1.69 ms with 12 on that workload at P = 8).
    p.group_m = std::max(1, env_int("AGG_GROUP_M", pk ? (world > 1 ? 8 : 12) : 16));
    p.raster_n = env_int("AGG_RASTER_N", 0) ? 1 : 0;
    p.dtype = a->dtype;
    p.scale_a = a->scale_a;
    p.scale_b = a->scale_b;
    p.status = a->status;
    p.timeout_ns = a->timeout_ns;
    p.trace = reinterpret_cast<unsigned long long*>(a->trace);
    p.epoch = a->A_copy_epoch;

    if (world > 1) {
        if (peer_push) {
            // the gathered region sits at the same offset in every rank's slab
            const uint64_t goff = reinterpret_cast<uint64_t>(a->A_local_buf) - a->A_peer[a->dev_idx];
            p.peer_push = 1;
            for (int s = 0; s < world; ++s)
                p.peer_dst[s] = a->A_peer[s] + goff + region_off +
                                static_cast<uint64_t>(a->dev_idx) * m_local * a->K * elem;
        }
        p.a_mc = reinterpret_cast<uint4*>(a->A_mc + region_off +
                                          static_cast<uint64_t>(a->dev_idx) * m_local * a->K * elem);
        p.shard_bytes = static_cast<unsigned long long>(m_local) * a->K * elem;
        p.chunk_bytes = static_cast<unsigned long long>(BM) * a->K * elem;
        p.num_chunks = m_local / BM;
        // Each chunk's counter grows by exactly one per launch (the last producer
        // warp done with it raises it), so the target is the launch's ordinal
        // within its flag set; the producer gate is the done count of the last
        // launch that read the region being overwritten.
        const uint32_t e = a->A_copy_epoch;
        const uint32_t sets_per_rank = static_cast<uint32_t>(AGG_MAX_RANKS * AGG_MAX_CHUNKS);
        p.flags_uc = a->A_copy_ready + parity * sets_per_rank;
        p.flags_mc = a->A_copy_ready_mc + parity * sets_per_rank;
        p.flag_target = dbl ? (e + 1u) >> 1 : e;
        const uint32_t prior = dbl ? (e > 2u ? e - 2u : 0u) : e - 1u;
        p.gate_done = prior * static_cast<uint32_t>(world);
        p.done_uc = a->done_uc;
        p.done_mc = a->done_mc;
        p.cta_counter = a->done_uc + 16;                                        // +64 B
        p.ticket = reinterpret_cast<unsigned long long*>(a->done_uc + 32);      // +128 B
        p.chunk_cnt = a->done_uc + 1024;                                        // +4 KiB
        if (f8) {
            // Gathered row scales follow the gathered region(s): float [M] per parity.
            const size_t scales_off = static_cast<size_t>(dbl ? 2 : 1) * a->M * a->K * elem +
                                      static_cast<size_t>(parity) * a->M * sizeof(float);
            p.scale_gath = reinterpret_cast<const float*>(static_cast<uint8_t*>(a->A_local_buf) + scales_off);
            p.scale_mc = reinterpret_cast<float*>(a->A_mc + scales_off) + static_cast<size_t>(a->dev_idx) * m_local;
            if (reinterpret_cast<uintptr_t>(a->scale_a) % 16)
                return fail(AGG_EINVAL, "agg_launch: scale_a must be 16-byte aligned");
        }
        // Piece size: the bytes in flight (producer warps x piece) should cover
        // one system-scope round trip (~15 us) at this rank's share of the
        // receivers' NVLink ingress (~600 GB/s, shared by world-1 senders), and
        // never less than two chunks, so that chunks still complete in order.
        const double egress = 600e9 / static_cast<double>(world - 1);
        double window = egress * 15e-6;
        window = std::max(window, 2.0 * static_cast<double>(p.chunk_bytes));
        const int grid_ctas = pk ? 2 * std::max(1, std::min(pk->clusters, p.num_tiles))
                                 : std::max(1, std::min(di->sms, p.num_tiles));
        unsigned long long piece = static_cast<unsigned long long>(window / (grid_ctas * PROD_WARPS));
        const int piece_env_kb = env_int("AGG_PIECE_KB", 0);
        if (piece_env_kb > 0) piece = static_cast<unsigned long long>(piece_env_kb) << 10;
        piece = std::min<unsigned long long>(std::max<unsigned long long>(piece, 4096ull), p.chunk_bytes);
        p.piece_bytes = (piece + 511) / 512 * 512;
        if (reinterpret_cast<uintptr_t>(a_src) % 16 || (p.a_mc && reinterpret_cast<uintptr_t>(p.a_mc) % 16))
            return fail(AGG_EINVAL, "agg_launch: shard pointers must be 16-byte aligned");
    }

    auto launch_kernel = [&]() -> int {
        if (!pk) {
            const int grid = std::max(1, std::min(di->sms, p.num_tiles));
            ag_gemm_kernel<<<grid, NUM_THREADS, SMEM_ALLOC, stream>>>(p);
            AGG_RT(cudaGetLastError());
            return AGG_OK;
        }
        return launch_pair(*pk, p, stream, dev);
    };
    if (!(ce_mode && world > 1)) return launch_kernel();

    // Copy-engine producers: the copies (internal stream) and the kernel (the
    // caller's stream) run side by side; the launch completes on `stream` when
    // both have.  The region being overwritten is free without a device-side
    // gate: this rank's previous launch has completed (stream order), so every
    // rank has delivered its previous-launch chunks, which its own copies
    // started only after its launch before that -- the last reader of this
    // parity's region -- had completed.
    p.ext_producer = 1;
    cudaStream_t ce = nullptr;
    rc = ce_begin(stream, &ce);
    if (rc) return rc;
    rc = ce_push_shard(a, a_src, m_local, static_cast<size_t>(a->K) * elem, region_off, parity, p.flag_target,
                       (ce_mode & AGG_ARGS_CE_MC_PUSH) != 0, ce);
    if (rc == AGG_OK) rc = launch_kernel();
    const int rc_end = ce_end(stream);
    return rc ? rc : rc_end;
}

int launch_gemm_rs(const agg_rs_args* a, cudaStream_t stream) {
    if (!a) return fail(AGG_EINVAL, "agg_launch_rs: null args");
    const int world = a->world;
    if (world < 2 || world > AGG_MAX_RANKS) return fail(AGG_EINVAL, "agg_launch_rs: world %d (2..8)", world);
    if (a->rank < 0 || a->rank >= world) return fail(AGG_EINVAL, "agg_launch_rs: rank %d", a->rank);
    if (a->M <= 0 || a->N <= 0 || a->K <= 0) return fail(AGG_EINVAL, "agg_launch_rs: empty shape");
    if (a->M % world) return fail(AGG_EINVAL, "agg_launch_rs: M=%d not divisible by world=%d", a->M, world);
    const int m_local = a->M / world;
    if (m_local % 256) return fail(AGG_EINVAL, "agg_launch_rs: M/world=%d must be a multiple of 256", m_local);
    if (a->K % 8 || a->N % 8) return fail(AGG_EINVAL, "agg_launch_rs: N and K must be multiples of 8");
    if (!a->X || !a->W || !a->Y) return fail(AGG_EINVAL, "agg_launch_rs: null X, W or Y");
    if (reinterpret_cast<uintptr_t>(a->Y) % 16) return fail(AGG_EINVAL, "agg_launch_rs: Y must be 16-byte aligned");
    if (!a->cnt_uc || !a->cnt_mc || !a->done_uc || !a->done_mc)
        return fail(AGG_EINVAL, "agg_launch_rs: multicast buffers missing");
    for (int s = 0; s < world; ++s)
        if (!a->part_peer[s] || a->part_peer[s] % 16)
            return fail(AGG_EINVAL, "agg_launch_rs: inbox of rank %d missing or not 16-byte aligned", s);
    if (a->epoch < 1) return fail(AGG_EINVAL, "agg_launch_rs: epoch must start at 1");
    const bool ce = (a->flags & AGG_ARGS_RS_COPY_ENGINE) != 0;
    if (ce && (!a->stage || reinterpret_cast<uintptr_t>(a->stage) % 16))
        return fail(AGG_EINVAL, "agg_launch_rs: the copy-engine exchange needs a 16-byte aligned stage [M, N]");
    if (ce && !a->status)
        return fail(AGG_EINVAL, "agg_launch_rs: the copy-engine exchange needs a status word");
    if (ce && reinterpret_cast<uint64_t>(a->done_uc) <= a->part_peer[a->rank])
        return fail(AGG_EINVAL, "agg_launch_rs: done_uc must lie in this rank's slab, after its inbox");
    const int num_m_tiles = a->M / 256;
    const int num_n_tiles = (a->N + 255) / 256;
    if (static_cast<long long>(num_m_tiles) * num_n_tiles > AGG_RS_MAX_TILES)
        return fail(AGG_EINVAL, "agg_launch_rs: %d x %d tiles exceed %d", num_m_tiles, num_n_tiles, AGG_RS_MAX_TILES);

    int dev = 0;
    AGG_RT(cudaGetDevice(&dev));
    const DevInfo* di = nullptr;
    int rc = device_info(dev, &di);
    if (rc) return rc;
    if (di->rs.clusters < 1) return fail(AGG_ECUDA, "agg_launch_rs: kernel cannot be resident");

    KParams p;
    std::memset(&p, 0, sizeof(p));
    const bool dbl = (a->flags & AGG_ARGS_DOUBLE_BUFFER) != 0;
    const uint32_t e = a->epoch;
    const uint32_t parity = dbl ? (e & 1u) : 0u;
    const size_t region = static_cast<size_t>(a->M) * a->N * 2;
    const uint32_t kb_elems = BK_BYTES / 2;
    rc = encode_2d(&p.tm_a_src, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->X, a->K, a->M, kb_elems, BM, "tensor map X");
    if (rc) return rc;
    rc = encode_2d(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->W, a->K, a->N, kb_elems, di->rs.b_box,
                   "tensor map W");
    if (rc) return rc;
    // Slot `rank` of owner s's inbox (in its slab, as mapped here): rows of s's
    // block.  With the copy-engine exchange, the other owners' blocks go to the
    // local stage instead, at their own rows.
    const size_t slot_bytes = static_cast<size_t>(m_local) * a->N * 2;
    uint64_t inbox_slot[AGG_MAX_RANKS] = {};
    for (int s = 0; s < world; ++s) {
        inbox_slot[s] = a->part_peer[s] + parity * region + a->rank * slot_bytes;
        const uint64_t dst = (ce && s != a->rank) ? reinterpret_cast<uint64_t>(a->stage) + s * slot_bytes
                                                   : inbox_slot[s];
        rc = encode_2d(&p.tm_out[s], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, reinterpret_cast<const void*>(dst), a->N,
                       m_local, EPI_COLS, EPI_ROWS, "tensor map inbox");
        if (rc) return rc;
    }
    p.M = a->M;
    p.N = a->N;
    p.K = a->K;
    p.rank = a->rank;
    p.world = world;
    p.m_local = m_local;
    p.tile_m = 256;
    p.num_m_tiles = num_m_tiles;
    p.num_n_tiles = num_n_tiles;
    p.num_tiles = num_m_tiles * num_n_tiles;
    p.num_kb = static_cast<int>((static_cast<size_t>(a->K) * 2 + BK_BYTES * di->rs.sub - 1) / (BK_BYTES * di->rs.sub));
    p.group_m = std::max(1, env_int("AGG_GROUP_M", 12));
    p.dtype = AGG_DTYPE_BF16;
    p.status = a->status;
    p.timeout_ns = a->timeout_ns;
    p.trace = reinterpret_cast<unsigned long long*>(a->trace);
    p.epoch = e;
    p.flags_uc = a->cnt_uc + parity * AGG_RS_MAX_TILES;
    p.flags_mc = a->cnt_mc + parity * AGG_RS_MAX_TILES;
    // Every tile's counter grows by 8 slices x world ranks per launch of its parity set.
    const uint32_t ordinal = dbl ? (e + 1u) >> 1 : e;
    p.rs_target = 8u * static_cast<uint32_t>(world) * ordinal;
    const uint32_t prior = dbl ? (e > 2u ? e - 2u : 0u) : e - 1u;
    p.gate_done = prior * static_cast<uint32_t>(world);
    p.done_uc = a->done_uc;
    p.done_mc = a->done_mc;
    p.cta_counter = a->done_uc + 16;                                    // +64 B
    p.ticket = reinterpret_cast<unsigned long long*>(a->done_uc + 32);  // +128 B
    p.inbox = reinterpret_cast<const uint8_t*>(a->part_peer[a->rank] + parity * region);
    p.y = static_cast<__nv_bfloat16*>(a->Y);
    if (!ce) return launch_pair(di->rs, p, stream, dev);

    // Copy-engine exchange.  Own tiles count 8 slices per launch of their
    // parity on this GPU only.  Each owner's block runs as chunks of gm m-tiles
    // (all n-tiles of a chunk before the next), counted per (owner, chunk): 8
    // slices per tile per launch, so a chunk's copy can start as soon as it is
    // stored.  Default: groups of 12 m-tiles, i.e. whole blocks at P = 8 on the
    // 70B down projection.  Smaller chunks (AGG_RS_CE_GROUP=2) start the copies
    // earlier but measured slower there: 1.03 ms with one copy stream and
    // 0.87 ms with two, against 0.83-0.87 ms with whole 32 MiB blocks; at P = 2
    // they also stream all of W (235 MB) through L2 once per chunk.
    // At most 128 chunks per owner fit the counter area (flag area + 4 KiB).
    const int L = m_local / 256;
    int gm = std::max(1, std::min(L, env_int("AGG_RS_CE_GROUP", 12)));
    gm = std::max(gm, (L + 127) / 128);
    p.group_m = gm;
    p.rs_ce = 1;
    p.rs_target = 8u * ordinal;
    p.ce_chunks = (L + gm - 1) / gm;
    p.ce_cnt = a->done_uc + 1024;  // +4 KiB: u32 [AGG_MAX_RANKS][ce_chunks]
    p.ce_rx = a->done_uc + 80;     // +320 B
    p.ce_fail = a->done_uc + 96;  // +384 B
    // the flag area sits at the same offset from the inbox in every slab
    const uint64_t flag_rel = reinterpret_cast<uint64_t>(a->done_uc) - a->part_peer[a->rank];
    uint64_t rx_word[AGG_MAX_RANKS] = {};
    for (int s = 0; s < world; ++s) {
        p.ce_fail_peer[s] = a->part_peer[s] + flag_rel + 4u * (96u + static_cast<uint32_t>(a->rank));
        rx_word[s] = a->part_peer[s] + flag_rel + 4u * (80u + static_cast<uint32_t>(a->rank));
    }
    cudaStream_t cs = nullptr;
    rc = ce_begin(stream, &cs);  // before the launch: the copy stream must not wait for the kernel to end
    if (rc) return rc;
    rc = launch_pair(di->rs, p, stream, dev);
    if (rc == AGG_OK)
        rc = ce_rs_exchange(a->rank, world, inbox_slot, static_cast<const uint8_t*>(a->stage), slot_bytes,
                            static_cast<size_t>(256) * a->N * 2, L, gm, num_n_tiles, p.ce_cnt, rx_word, e,
                            env_int("AGG_RS_CE_STREAMS", 1), cs);
    const int rc_end = ce_end(stream);
    return rc ? rc : rc_end;
}

}  // namespace agg

extern "C" {

int agg_launch(const agg_args* args, void* stream) {
    return agg::launch_ag_gemm(args, static_cast<cudaStream_t>(stream));
}

int agg_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, uint32_t* status,
                  void* stream) {
    agg_args a;
    std::memset(&a, 0, sizeof(a));
    a.A_src = A;
    a.B = B;
    a.C = C;
    a.M = M;
    a.N = N;
    a.K = K;
    a.world = 1;
    a.dev_idx = 0;
    a.A_copy_epoch = 1;
    a.dtype = AGG_DTYPE_BF16;
    a.status = status;
    return agg::launch_ag_gemm(&a, static_cast<cudaStream_t>(stream));
}

int agg_gemm_e4m3(const void* A, const void* B, void* C, const float* scale_a, const float* scale_b,
                  int M, int N, int K, uint32_t* status, void* stream) {
    agg_args a;
    std::memset(&a, 0, sizeof(a));
    a.A_src = A;
    a.B = B;
    a.C = C;
    a.M = M;
    a.N = N;
    a.K = K;
    a.world = 1;
    a.dev_idx = 0;
    a.A_copy_epoch = 1;
    a.dtype = AGG_DTYPE_E4M3;
    a.scale_a = scale_a;
    a.scale_b = scale_b;
    a.status = status;
    return agg::launch_ag_gemm(&a, static_cast<cudaStream_t>(stream));
}

int agg_launch_rs(const agg_rs_args* args, void* stream) {
    return agg::launch_gemm_rs(args, static_cast<cudaStream_t>(stream));
}

size_t agg_rs_args_size(void) { return sizeof(agg_rs_args); }

int agg_num_sms(void) {
    const int s = agg::current_sms(nullptr);
    return s > 0 ? s : 0;
}

}  // extern "C"
