/*
 * agg.h — C ABI of the B200 (sm_100a) fused all-gather GEMM library, libagg.so.
 *
 * The library computes, on each of P ranks (one GPU each),
 *     C_r[M, N_r] = AllGather_r(A_r)[M, K] . B_r[N_r, K]^T
 * bf16 (or e4m3) inputs, fp32 accumulation in tensor memory, bf16 output,
 * in ONE kernel: producer warps broadcast this rank's A shard into an NVLink
 * multicast object with multimem.st and raise per-chunk arrival flags, while
 * the tensor-core warps already consume the arrived tiles.
 *
 * Every entry point takes plain pointers and sizes; CUDA streams are passed as
 * `void*` (a cudaStream_t, NULL = legacy default stream).  Return values are
 * 0 on success and a negative AGG_E* code otherwise; agg_last_error() gives
 * the message of the calling thread's last failure.
 *
 * Interfaces of the reference (ShawnWeiChew/vmm-experiment) replaced here:
 *   agg_spmm_init / agg_rank_info   minfer_spmm_init + RankState
 *                                   (vmm/multimem.cu:74-101, include/multimem.cuh:11-23)
 *   agg_vm_alloc / agg_vm_map /     vm_alloc / vm_map (include/vmm.cuh:12-38); the
 *   agg_vm_set_access               access grant the reference leaves out is added
 *   agg_args / agg_launch           fused_globals<128,256,2> +
 *                                   launch_ag_gemm_warp_specialized<128,256,2,5>
 *                                   (call site vmm/main.cpp:226,272-296; the kernel's
 *                                   own source is an absent submodule)
 *   agg_multimem_ops_test           multicast_ops_kernel (include/test_kernel.cuh:46-74)
 *   agg_alias_fence                 multicast_alias_fence_kernel (include/test_kernel.cuh:41-44)
 *   agg_mm_barrier                  mm_barrier (vmm/multimem.cu:103-119), bounded
 *   agg_mc_broadcast / agg_verify_* multicast push + byte-exact verify
 *                                   (vmm/test_vmm_multicast_speed.cu:99-126,172-194)
 *   agg_mp_*                        no counterpart (the reference is one process with a
 *                                   thread per GPU); POSIX-fd export/import of the same
 *                                   handles so ranks can be separate processes.
 */
#ifndef AGG_H_
#define AGG_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- error codes ---------------------------------------------------------------- */
#define AGG_OK 0
#define AGG_EINVAL (-1)        /* bad argument (shape, alignment, rank/device mismatch) */
#define AGG_ECUDA (-2)         /* a CUDA runtime call failed */
#define AGG_EDRIVER (-3)       /* a CUDA driver call failed */
#define AGG_ENOMULTICAST (-4)  /* a device lacks NVLink multicast support */
#define AGG_ESTATE (-5)        /* called in the wrong order / not initialised */
#define AGG_ESYS (-6)          /* an OS call (socket, fd passing) failed */
#define AGG_ETIMEOUT (-7)      /* a device-side wait ran out (see agg_status_* below) */

/* ---- device status word (written by kernels, read by the host) ------------------- */
/* 0 = ok.  Otherwise bits 0-7 hold the failing role, bits 8-31 where it gave up.    */
#define AGG_STATUS_OK 0u
#define AGG_ROLE_TMA 1u        /* operand loader waiting for a free stage            */
#define AGG_ROLE_MMA 2u        /* tensor-core issuer waiting for operands/TMEM        */
#define AGG_ROLE_EPI 3u        /* epilogue waiting for an accumulator                 */
#define AGG_ROLE_FLAG 4u       /* loader waiting for a remote chunk's arrival flag    */
#define AGG_ROLE_PROD 5u       /* multicast producer waiting for the previous launch  */
#define AGG_ROLE_BARRIER 6u    /* mm_barrier gave up                                  */
#define AGG_ROLE_DRAIN 7u      /* teardown wait for in-flight copies / MMAs          */
#define AGG_ROLE_REDUCE 8u     /* reduce-scatter: reducer waiting for a tile's partials */

/* ---- dtypes ----------------------------------------------------------------------- */
#define AGG_DTYPE_BF16 0
#define AGG_DTYPE_E4M3 1

/* ---- slab / flag layout constants ------------------------------------------------ */
#define AGG_MAX_RANKS 8
#define AGG_TILE_M 128                 /* rows per arrival chunk (= MMA tile height)     */
#define AGG_MAX_CHUNKS 1024            /* per source rank: M/P <= 131072 rows            */
#define AGG_FLAG_BYTES (128u << 10)    /* flag area, zeroed at init:                     */
#define AGG_FLAG_CHUNK_OFF 0u          /* u32 [2][AGG_MAX_RANKS][AGG_MAX_CHUNKS] arrival */
                                       /* counters, one set per launch parity; each     */
                                       /* chunk's counter grows by one per launch       */
#define AGG_FLAG_DONE_OFF (64u << 10)  /* u32 end-of-launch counter (one per rank and    */
                                       /* launch); +64 B: this GPU's CTA counter;        */
                                       /* +4 KiB: u32 [AGG_MAX_CHUNKS] producer counters */
#define AGG_FLAG_USER_OFF (72u << 10)  /* free for mm_barrier rows / tests (56 KiB)      */
#define AGG_RS_MAX_TILES 8192          /* reduce-scatter: the chunk-counter area holds   */
                                       /* u32 [2][AGG_RS_MAX_TILES] per-tile counters    */

/* agg_args.flags bits */
#define AGG_ARGS_DOUBLE_BUFFER 1u      /* gathered A has two [M, K] regions used by     */
                                       /* launch parity (A_local_buf / A_mc point at    */
                                       /* region 0, region 1 follows), so a launch never */
                                       /* waits for the other ranks' previous launch    */
/* Who moves this rank's shard (default: the kernel's own producer warps, multimem.st).
   The copy-engine modes (vmm/test_vmm_multicast_speed.cu:172-263) leave the SMs to the
   GEMM: an internal stream, ordered after the caller's prior work on `stream`, copies
   the shard in chunk order with cudaMemcpyAsync and raises each chunk's flag on every
   GPU with cuStreamWriteValue32 through the peers' unicast mappings (A_peer[]); the
   launch completes on `stream` once the copies have.  They need
   AGG_ARGS_DOUBLE_BUFFER, bf16, A_peer[s] = every rank's slab base as mapped here
   (A_peer[rank] = this GPU's, containing A_copy_ready), and consecutive launches on
   one slab issued on the same stream. */
#define AGG_ARGS_CE_MC_PUSH 2u         /* one copy per chunk into the multicast VA       */
#define AGG_ARGS_CE_PEER_PUSH 4u       /* one copy per chunk and peer (order r-1, r-2..) */
/* The kernel's producer warps store each piece of the shard into every rank's slab
   (this GPU's included) through the unicast peer mappings A_peer[] with 16-byte
   st.global, instead of one multimem.st into the multicast VA: the NVSwitch then
   carries (P-1) unicast copies, which all-to-all can move faster than one multicast.
   Needs bf16, A_peer[s] = every rank's slab base as mapped here, and A_local_buf
   inside this rank's slab (the gathered region sits at the same offset in every slab). */
#define AGG_ARGS_SM_PEER_PUSH 8u

/* Per-rank view of the multicast slab (RankState of the reference, C layout). */
typedef struct agg_rank_info {
    uint64_t uc;                        /* this GPU's physical slab, unicast VA          */
    uint64_t mc;                        /* the multicast VA of the same slab             */
    uint64_t peer_uc[AGG_MAX_RANKS];    /* every rank's slab as mapped in this process  */
    uint64_t slab_bytes;                /* size of each slab                              */
    uint64_t flag_off;                  /* offset of the flag area inside the slab       */
    int32_t rank, world, device;
    int32_t reserved;
} agg_rank_info;

/*
 * Launch arguments: the fields of the reference's fused_globals in its order
 * (A, A_local_buf, B, C, A_copy_ready, A_copy_epoch, dev_idx, M, N;
 * vmm/main.cpp:272-294) followed by what the reference fixed at compile time.
 */
typedef struct agg_args {
    /* A: the distributed activation.  A_mc is the multicast VA where gathered A
       starts (rank s's shard at A_mc + s*M_local*K*elem); A_peer[s] are the
       unicast VAs of every rank's slab (informational; the kernel only reads
       its own GPU's memory). */
    uint64_t A_mc;
    uint64_t A_peer[AGG_MAX_RANKS];
    /* Gathered A [M, K] on this GPU (unicast VA of the same slab region). */
    void* A_local_buf;
    /* B_r [N_r, K] row-major (K-major), this rank's weight shard. */
    const void* B;
    /* C_r [M, N_r] row-major bf16 output. */
    void* C;
    /* Arrival counters, this GPU's unicast view of the flag area's chunk sets
       (u32 [2][AGG_MAX_RANKS][AGG_MAX_CHUNKS], AGG_FLAG_CHUNK_OFF). */
    uint32_t* A_copy_ready;
    /* Launch epoch, >= 1, incremented by exactly one per launch on every rank. */
    uint32_t A_copy_epoch;
    int32_t dev_idx; /* this rank */
    int32_t M;       /* total rows of gathered A = world * M_local */
    int32_t N;       /* N_r, columns of this rank's output */
    /* ---- added: what the reference template fixed at compile time ---- */
    int32_t K;
    int32_t world;
    int32_t dtype;                 /* AGG_DTYPE_BF16 / AGG_DTYPE_E4M3 */
    int32_t flags;                 /* AGG_ARGS_* bits */
    const void* A_src;             /* this rank's shard [M/world, K]; NULL = inside A_local_buf */
    uint32_t* A_copy_ready_mc;     /* multicast view of the flag array */
    uint32_t* done_uc;             /* end-of-launch counter, unicast view (AGG_FLAG_DONE_OFF) */
    uint32_t* done_mc;             /* end-of-launch counter, multicast view */
    const float* scale_a;          /* e4m3: per-row scales of A_src, 16-byte aligned: [M] at
                                      world 1, this rank's [M/world] otherwise (the kernel
                                      gathers them into the slab right after the gathered
                                      A region(s): float [M] per region) */
    const float* scale_b;          /* e4m3: per-row scale of B_r [N_r] (per output column) */
    uint32_t* status;              /* device status word (AGG_STATUS_*), may be NULL */
    uint64_t timeout_ns;           /* bound on every device-side wait; 0 = 10 s */
    uint64_t* trace;               /* optional: u64 [grid][AGG_TRACE_SLOTS] event times (ns) */
} agg_args;

/* Per-CTA trace slots written when agg_args.trace is not NULL (%globaltimer, ns;
   0 = event did not happen).  The grid never exceeds agg_num_sms() CTAs, so a
   buffer of agg_num_sms() * AGG_TRACE_SLOTS u64 (zeroed) always suffices. */
#define AGG_TRACE_SLOTS 16
#define AGG_TR_START 0          /* CTA start                                          */
#define AGG_TR_PROD_GATE 1      /* producers may overwrite the gathered buffer        */
#define AGG_TR_PROD_DONE 2      /* this CTA's producers pushed all their parts        */
#define AGG_TR_FIRST_WAIT 3     /* loader starts its first wait for a remote chunk    */
#define AGG_TR_FIRST_READY 4    /* ... and sees it                                    */
#define AGG_TR_LAST_READY 5     /* loader sees its last remote chunk (reduce-scatter  */
                                /* copy-engine exchange: reducers see every block)    */
#define AGG_TR_FLAG_WAIT_NS 6   /* total time the loader waited on remote chunks      */
                                /* (... the reducers waited for the blocks)           */
#define AGG_TR_LOADER_DONE 7    /* loader issued its last k-block                     */
#define AGG_TR_MMA_DONE 8       /* tensor-core issuer committed its last tile         */
#define AGG_TR_EPI_DONE 9       /* epilogue stored its last tile                      */
#define AGG_TR_END 10           /* CTA end                                            */
#define AGG_TR_TILES 11         /* tiles this CTA processed (a count, not a time)     */
#define AGG_TR_MMA_WAIT_NS 12   /* total time the MMA issuer waited for operand stages */
#define AGG_TR_MMA_ACC_NS 13    /* ... and for a free accumulator                     */
#define AGG_TR_LOAD_WAIT_NS 14  /* total time the loader waited for free stages       */
#define AGG_TR_MMA_STALLS 15    /* operand-stage waits of the MMA issuer that blocked  */

/* ---- library ---------------------------------------------------------------------- */
int agg_version(void);                 /* 100 * major + minor */
int agg_abi_sizes(size_t* args_bytes, size_t* rank_info_bytes); /* sizeof(agg_args/agg_rank_info) */
const char* agg_last_error(void);      /* message of this thread's last failure */
int agg_device_count(void);

/* ---- VMM helpers (include/vmm.cuh:12-38) ------------------------------------------- */
int agg_vm_alloc(uint64_t* handle, size_t* allocated_size, size_t size, int device_id);
int agg_vm_map(uint64_t* ptr, uint64_t handle, size_t size);
int agg_vm_set_access(uint64_t ptr, size_t size, const int* devices, int ndevices);
int agg_vm_unmap_free(uint64_t ptr, size_t size);
int agg_vm_release(uint64_t handle);

/* ---- one process, one thread per GPU (minfer_spmm_init, vmm/multimem.cu:74-101) --- */
/* rank must equal device; the first caller creates the multicast object for
   devices 0..world-1; every rank binds its own slab.  Idempotent per rank. */
int agg_spmm_init(int rank, int world, int device, size_t data_bytes, agg_rank_info* out);
/* Unmaps and releases this rank's slab; the multicast object goes with the last rank. */
int agg_spmm_finalize(int rank);

/* ---- one process per GPU: POSIX-fd handle exchange over abstract unix sockets ----- */
/* Call order on every rank, with a host barrier between the steps:
     agg_mp_open -> barrier -> agg_mp_exchange -> agg_mp_add_device -> barrier ->
     agg_mp_bind -> barrier -> (launches) -> agg_mp_close.
   job_id must be the same string on every rank and unique on the machine. */
typedef struct agg_mp_ctx agg_mp_ctx;
int agg_mp_open(int rank, int world, int device, size_t data_bytes, const char* job_id,
                agg_mp_ctx** out);
int agg_mp_exchange(agg_mp_ctx* ctx);
int agg_mp_add_device(agg_mp_ctx* ctx);
int agg_mp_bind(agg_mp_ctx* ctx, agg_rank_info* out);
int agg_mp_close(agg_mp_ctx* ctx);

/* ---- the fused all-gather GEMM ----------------------------------------------------- */
/* Enqueue one launch on `stream`.  Shapes: M % world == 0, (M/world) % 128 == 0
   when world > 1, K % 8 == 0, N % 8 == 0 (16-byte row pitch).  Returns AGG_EINVAL
   without launching on bad arguments.
   After a launch whose status word is nonzero (a wait gave up), the slab's
   arrival and done counters no longer match the epochs: once every rank's
   launches have ended, zero each slab's flag area (AGG_FLAG_BYTES at flag_off)
   and restart A_copy_epoch at 1 on every rank before launching again.  The
   same holds for agg_launch_rs. */
int agg_launch(const agg_args* args, void* stream);
/* Single-GPU GEMM through the same kernel: C[M,N] = A[M,K] . B[N,K]^T (bf16). */
int agg_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, uint32_t* status,
                  void* stream);
/* Same for e4m3 operands with per-row scales of A [M] and of B [N], bf16 output. */
int agg_gemm_e4m3(const void* A, const void* B, void* C, const float* scale_a,
                  const float* scale_b, int M, int N, int K, uint32_t* status, void* stream);
/* Number of SMs the persistent grid uses on the current device (0 on failure). */
int agg_num_sms(void);

/* Single-GPU bf16 GEMM, C[M,N] = A[M,K] . B[N,K]^T, that allocates nothing: for
   callers that may not call cudaMalloc (a plugin inside a program whose caching
   allocator owns all device memory, a loop that must not take the allocator's
   device-wide synchronisation).  No counterpart in the reference.
   K is split into `splits` ranges (0 = chosen from the SM count); the fp32
   partial tiles and their arrival counters live in one static device array of
   AGG_NOALLOC_SCRATCH_BYTES that every GPU whose context loads this library's
   kernels holds until exit.  Limit: (ceil(M/128) * ceil(N/256)) * splits <= 255
   and splits <= ceil(K/64); larger requests return AGG_EINVAL with the bytes
   they would need.  Same shape rules as agg_gemm_bf16, and A, B, C 16-byte aligned.
   The first call on a device looks up the array's device address (with that
   device current); make that first call before any stream capture.  The lookup
   is redone, by the next call, whenever the device's current CUDA context is
   not the one it was made in (after a cudaDeviceReset, for instance).  All calls
   on a device share the array and it keeps the last call's contents: each call
   first clears the counters it uses, so calls whose executions overlap on the
   GPU (concurrent streams) race and must be serialised by the caller. */
#define AGG_NOALLOC_SCRATCH_BYTES (32u << 20)
int agg_gemm_bf16_noalloc(const void* A, const void* B, void* C, int M, int N, int K, int splits,
                          uint32_t* status, void* stream);

/* ---- the fused GEMM + reduce-scatter (row-parallel twin) ---------------------------- */
/*
 * Y_r[M/P, N] = rows [r*M/P, (r+1)*M/P) of  sum_s X_s[M, K_s] . W_s[N, K_s]^T
 * (bf16 in, fp32 accumulate, bf16 partials, fp32 sum in source order, bf16 out),
 * in one kernel per rank: the tensor-core warps compute every [256 x 256] tile of
 * this rank's partial product and TMA-store it straight into the owning rank's
 * inbox (slot r of its slab region, over NVLink for the other ranks), then raise
 * the tile's counter on every GPU (multimem.red); reducer warps on the owner add
 * the P slots of each of its tiles from local memory as the tiles complete.  The
 * reduce-scatter channels that the reference's RankState reserves (rs_calls,
 * dmw_cnt[kDmwChannels]; include/multimem.cuh:13-17) have no kernel in the
 * reference; this is that path.
 * Shapes: M % P == 0, (M/P) % 256 == 0, N % 8 == 0, K % 8 == 0,
 * ceil(M/256) * ceil(N/256) <= AGG_RS_MAX_TILES.
 * Slab data: one inbox region of [P][M/P, N] bf16 (two with
 * AGG_ARGS_DOUBLE_BUFFER, region 1 right after region 0) at the same offset in
 * every rank's slab.  Counters and the done counter live in the slab's flag area
 * (AGG_FLAG_CHUNK_OFF, AGG_FLAG_DONE_OFF).
 *
 * With AGG_ARGS_RS_COPY_ENGINE the SMs store nothing to a peer: the kernel
 * visits the owners' row blocks in the order rank+1, rank+2, ..., rank itself
 * last, each in chunks of 12 m-tiles (a whole block when M/P <= 3072;
 * AGG_RS_CE_GROUP overrides, fixed for all launches on a slab), and
 * TMA-stores the partials of the other owners into `stage` (this GPU's memory,
 * [M, N] bf16, block s at rows [s*M/P, (s+1)*M/P)).  An internal stream waits
 * (cuStreamWaitValue32) until each chunk is stored, copies it into slot `rank`
 * of that owner's inbox with cudaMemcpyAsync and, after a block's last chunk,
 * writes the owner's arrival word for this source (cuStreamWriteValue32
 * through the peer mapping); the owner's reducers wait for all P-1 arrival
 * words, then add the
 * slots of each of its own tiles as they complete.  A launch that fails marks
 * itself failed in every peer's flag area before it releases the copies, so
 * the owners fail too instead of reducing a partial sum.  The launch completes
 * on `stream` once the copies have.  All launches on one slab use one mode.
 * Flag area words (after AGG_FLAG_DONE_OFF): +320 B arrival words per source,
 * +384 B failure marks per source, +4 KiB u32 [AGG_MAX_RANKS][chunks] slices
 * stored per owner and chunk (at most 128 chunks per owner).
 */
#define AGG_ARGS_RS_COPY_ENGINE 16u
typedef struct agg_rs_args {
    const void* X;        /* this rank's activation slice [M, K] bf16, K-major       */
    const void* W;        /* this rank's weight slice [N, K] bf16, K-major           */
    void* Y;              /* this rank's rows of the sum [M/world, N] bf16           */
    uint64_t part_peer[AGG_MAX_RANKS];  /* inbox region 0 in every rank's slab as     */
                                        /* mapped here (part_peer[rank]: this GPU's)  */
    uint32_t* cnt_uc;     /* per-tile counters (flag area + AGG_FLAG_CHUNK_OFF), UC   */
    uint32_t* cnt_mc;     /* the same, multicast VA                                   */
    uint32_t* done_uc;    /* end-of-launch counter (flag area + AGG_FLAG_DONE_OFF), UC */
    uint32_t* done_mc;    /* the same, multicast VA                                   */
    uint32_t epoch;       /* launch ordinal on this slab: 1, 2, ... on every rank     */
    int32_t rank, world;
    int32_t M, N, K;      /* K: this rank's slice of the contraction                  */
    uint32_t flags;       /* AGG_ARGS_DOUBLE_BUFFER | AGG_ARGS_RS_COPY_ENGINE         */
    uint32_t* status;     /* device status word, may be NULL                          */
    uint64_t timeout_ns;  /* bound on every device-side wait; 0 = 10 s                */
    uint64_t* trace;      /* optional: u64 [grid][AGG_TRACE_SLOTS] event times (ns)   */
    void* stage;          /* AGG_ARGS_RS_COPY_ENGINE: [M, N] bf16 on this GPU, 16-byte */
                          /* aligned; the other owners' partial blocks before the copy */
} agg_rs_args;

/* Enqueue one launch on `stream`; AGG_EINVAL without launching on bad arguments. */
int agg_launch_rs(const agg_rs_args* args, void* stream);
/* sizeof(agg_rs_args), for bindings to check their layout. */
size_t agg_rs_args_size(void);

/* ---- copy-engine all-gather (vmm/test_vmm_multicast_speed.cu:172-263) ---------------- */
#define AGG_CE_MC_PUSH 0     /* one cudaMemcpyAsync of the shard into the multicast VA
                                (enqueue_multicast_push, :183-194)                       */
#define AGG_CE_PEER_PUSH 1   /* one copy into every peer's slot, destinations r-1, r-2, ...
                                (enqueue_quack_ag_push, :207-231)                          */
#define AGG_CE_PEER_PULL 2   /* one copy from every peer's slot into this GPU's, sources
                                r+1, r+2, ... (enqueue_mkernel_ag_pull, :233-254); the
                                peers' shards must already be in their own slots           */
/* Copy-engine all-gather of `shard_bytes` per rank into slot `rank` (offset
   region_off + rank * shard_bytes) of every rank's slab, on `stream`.  `src` is
   this rank's shard (PUSH modes; the local slot is filled too).  Uses the slab
   addresses of `info` (agg_spmm_init / agg_mp_bind). */
int agg_ce_allgather(const agg_rank_info* info, uint64_t region_off, const void* src, size_t shard_bytes,
                     int mode, void* stream);
/* cuStreamWriteValue32 of `value` to a local or peer (unicast) address on `stream`
   (enqueue_stream_write_value, :256-263): the copy-engine path's flag write. */
int agg_stream_write_u32(uint64_t addr, uint32_t value, void* stream);

/* ---- multicast primitives ---------------------------------------------------------- */
/* Broadcast `bytes` (multiple of 16) from local `src` to `mc_dst` with 16-byte
   multimem.st, then raise the u32 at `flag_mc` by one (release, system scope)
   when flag_mc is not NULL. */
int agg_mc_broadcast(const void* src, uint64_t mc_dst, size_t bytes, uint32_t* flag_mc,
                     int num_blocks, void* stream);
/* Count 64-bit words of `data` (bytes/8 of them) that differ from `expect`
   into *mismatches (device u64, accumulated). */
int agg_verify_bytes(const void* data, const void* expect, size_t bytes,
                     unsigned long long* mismatches, void* stream);
/* Count words of a gathered buffer [world][shard_bytes] whose bytes are not
   (source rank + 1) repeated (vmm/test_vmm_multicast_speed.cu:99-114). */
int agg_verify_pattern_gather(const void* gathered, size_t shard_bytes, int world,
                              unsigned long long* mismatches, void* stream);
/* fence.proxy.alias on the stream (include/test_kernel.cuh:41-44). */
int agg_alias_fence(void* stream);
/* The reference's multimem smoke (include/test_kernel.cuh:46-74) on a 16-byte
   record {reduce_input, store_output, red_target, reduced_local} at mc_rec:
   ld_reduce.add.f32 of reduce_input over all GPUs, st of the sum to
   store_output, red.add.f32 of `addend` to red_target, sum also to *reduced_out. */
int agg_multimem_ops_test(uint64_t mc_rec, float* reduced_out, float addend, void* stream);
/* Vectorised variants: v4 ld_reduce.add.f32 over n4 float4s (sum of all GPUs' copies
   written to local out), and v4 red.add.f32 of `addend` into every GPU's copy. */
int agg_multimem_ld_reduce_v4(uint64_t mc_src, float* out, size_t n4, void* stream);
int agg_multimem_red_add_v4(uint64_t mc_dst, float addend, size_t n4, void* stream);
/* mm_barrier (vmm/multimem.cu:103-119) as a kernel of `blocks` CTAs: each CTA adds 1
   to mc_flags[row*256 + cta] and waits (bounded by timeout_ns) until its unicast
   copy reaches `target`; a timeout is recorded in *status (AGG_ROLE_BARRIER). */
int agg_mm_barrier(uint32_t* mc_flags, const uint32_t* uc_flags, int row, uint32_t target,
                   int blocks, uint32_t* status, uint64_t timeout_ns, void* stream);
/* Device-side bounded wait on a u32 flag reaching `target` (no writer needed):
   the failure-detection path; records AGG_ROLE_FLAG on timeout. */
int agg_wait_flag(const uint32_t* flag, uint32_t target, uint32_t* status, uint64_t timeout_ns,
                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AGG_H_ */
