"""Host side of the fused all-gather GEMM: ctypes bindings of libagg.so and the
torch.distributed plumbing around them.

Mirrors the reference harness's API for this path (ShawnWeiChew/vmm-experiment):

  * ``spmm_init(rank, world, device, data_bytes)`` — minfer_spmm_init
    (vmm/multimem.cu:74-101) for one process driving several GPUs from threads;
  * ``RankState`` — include/multimem.cuh:11-20 (uc / mc / peer_addresses);
  * ``AllGatherGemm`` — the launch of ag_gemm_warp_specialized at
    vmm/main.cpp:272-296 for one process per GPU, the multicast slab set up
    with POSIX-fd handle exchange under torch.distributed;
  * ``gemm`` — the same kernel on one GPU (world == 1).

Everything runs on libagg.so: there is no fallback.  A missing library or a
CUDA-less host raises ``AggError`` instead of computing anything elsewhere.
"""
from __future__ import annotations

import ctypes
import os
import uuid

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libagg.so")

# ---- constants of include/agg.h -------------------------------------------------
AGG_OK = 0
AGG_DTYPE_BF16 = 0
AGG_DTYPE_E4M3 = 1
AGG_MAX_RANKS = 8
AGG_TILE_M = 128
AGG_MAX_CHUNKS = 1024
AGG_FLAG_BYTES = 128 << 10
AGG_FLAG_CHUNK_OFF = 0
AGG_FLAG_DONE_OFF = 64 << 10
AGG_FLAG_USER_OFF = 72 << 10
AGG_ARGS_DOUBLE_BUFFER = 1
AGG_ARGS_CE_MC_PUSH = 2
AGG_ARGS_CE_PEER_PUSH = 4
AGG_ARGS_SM_PEER_PUSH = 8
AGG_ARGS_RS_COPY_ENGINE = 16
AGG_CE_MC_PUSH, AGG_CE_PEER_PUSH, AGG_CE_PEER_PULL = 0, 1, 2
PRODUCERS = {"sm": 0, "ce_mc": AGG_ARGS_CE_MC_PUSH, "ce_push": AGG_ARGS_CE_PEER_PUSH,
             "sm_peer": AGG_ARGS_SM_PEER_PUSH}
ROLE_NAMES = {1: "tma", 2: "mma", 3: "epilogue", 4: "flag", 5: "producer", 6: "barrier", 7: "drain",
              8: "reducer"}
AGG_TRACE_SLOTS = 16
TRACE_EVENTS = ["start", "prod_gate", "prod_done", "first_wait", "first_ready", "last_ready", "flag_wait_ns",
                "loader_done", "mma_done", "epi_done", "end", "tiles", "mma_wait_ns", "mma_acc_ns", "load_wait_ns",
                "mma_stalls"]


def trace_summary(rows):
    """Summarise a [grid, AGG_TRACE_SLOTS] u64 trace (numpy) of one launch: for
    each event, microseconds after the earliest CTA start (min / median / max
    over the CTAs that recorded it); durations and counts as they are."""
    import numpy as np

    rows = np.asarray(rows, dtype=np.uint64)
    t0 = rows[:, 0][rows[:, 0] > 0].min()
    out = {}
    for i, name in enumerate(TRACE_EVENTS):
        col = rows[:, i]
        col = col[col > 0]
        if col.size == 0:
            continue
        if name.endswith("_ns") or name in ("tiles", "mma_stalls"):
            v = col.astype(np.float64) / (1e3 if name.endswith("_ns") else 1.0)
        else:
            v = (col - t0).astype(np.float64) / 1e3
        out[name] = {"n": int(col.size), "min": float(v.min()), "med": float(np.median(v)), "max": float(v.max())}
    return out

# Every function the C ABI exports (include/agg.h).
EXPORTS = [
    "agg_version", "agg_abi_sizes", "agg_last_error", "agg_device_count",
    "agg_vm_alloc", "agg_vm_map", "agg_vm_set_access", "agg_vm_unmap_free", "agg_vm_release",
    "agg_spmm_init", "agg_spmm_finalize",
    "agg_mp_open", "agg_mp_exchange", "agg_mp_add_device", "agg_mp_bind", "agg_mp_close",
    "agg_launch", "agg_gemm_bf16", "agg_gemm_e4m3", "agg_num_sms",
    "agg_mc_broadcast", "agg_verify_bytes", "agg_verify_pattern_gather", "agg_alias_fence",
    "agg_multimem_ops_test", "agg_multimem_ld_reduce_v4", "agg_multimem_red_add_v4",
    "agg_mm_barrier", "agg_wait_flag", "agg_gemm_bf16_noalloc",
    "agg_launch_rs", "agg_rs_args_size", "agg_ce_allgather", "agg_stream_write_u32",
]


class AggError(RuntimeError):
    pass


class agg_rank_info(ctypes.Structure):
    _fields_ = [
        ("uc", ctypes.c_uint64),
        ("mc", ctypes.c_uint64),
        ("peer_uc", ctypes.c_uint64 * AGG_MAX_RANKS),
        ("slab_bytes", ctypes.c_uint64),
        ("flag_off", ctypes.c_uint64),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class agg_args(ctypes.Structure):
    _fields_ = [
        ("A_mc", ctypes.c_uint64),
        ("A_peer", ctypes.c_uint64 * AGG_MAX_RANKS),
        ("A_local_buf", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("C", ctypes.c_void_p),
        ("A_copy_ready", ctypes.c_void_p),
        ("A_copy_epoch", ctypes.c_uint32),
        ("dev_idx", ctypes.c_int32),
        ("M", ctypes.c_int32),
        ("N", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("A_src", ctypes.c_void_p),
        ("A_copy_ready_mc", ctypes.c_void_p),
        ("done_uc", ctypes.c_void_p),
        ("done_mc", ctypes.c_void_p),
        ("scale_a", ctypes.c_void_p),
        ("scale_b", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_uint64),
        ("trace", ctypes.c_void_p),
    ]


class agg_rs_args(ctypes.Structure):
    _fields_ = [
        ("X", ctypes.c_void_p),
        ("W", ctypes.c_void_p),
        ("Y", ctypes.c_void_p),
        ("part_peer", ctypes.c_uint64 * AGG_MAX_RANKS),
        ("cnt_uc", ctypes.c_void_p),
        ("cnt_mc", ctypes.c_void_p),
        ("done_uc", ctypes.c_void_p),
        ("done_mc", ctypes.c_void_p),
        ("epoch", ctypes.c_uint32),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("M", ctypes.c_int32),
        ("N", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("status", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_uint64),
        ("trace", ctypes.c_void_p),
        ("stage", ctypes.c_void_p),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    """Load libagg.so (built in-tree by ``make -C vmm-experiment_b200/csrc``)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise AggError(f"{LIB_PATH} is not built; run __graft_entry__.build() or make -C csrc")
    L = ctypes.CDLL(LIB_PATH)
    vp, u64, sz, i32, u32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32
    sig = {
        "agg_version": ([], i32),
        "agg_abi_sizes": ([ctypes.POINTER(sz), ctypes.POINTER(sz)], i32),
        "agg_last_error": ([], ctypes.c_char_p),
        "agg_device_count": ([], i32),
        "agg_vm_alloc": ([ctypes.POINTER(u64), ctypes.POINTER(sz), sz, i32], i32),
        "agg_vm_map": ([ctypes.POINTER(u64), u64, sz], i32),
        "agg_vm_set_access": ([u64, sz, ctypes.POINTER(i32), i32], i32),
        "agg_vm_unmap_free": ([u64, sz], i32),
        "agg_vm_release": ([u64], i32),
        "agg_spmm_init": ([i32, i32, i32, sz, ctypes.POINTER(agg_rank_info)], i32),
        "agg_spmm_finalize": ([i32], i32),
        "agg_mp_open": ([i32, i32, i32, sz, ctypes.c_char_p, ctypes.POINTER(vp)], i32),
        "agg_mp_exchange": ([vp], i32),
        "agg_mp_add_device": ([vp], i32),
        "agg_mp_bind": ([vp, ctypes.POINTER(agg_rank_info)], i32),
        "agg_mp_close": ([vp], i32),
        "agg_launch": ([ctypes.POINTER(agg_args), vp], i32),
        "agg_gemm_bf16": ([vp, vp, vp, i32, i32, i32, vp, vp], i32),
        "agg_gemm_e4m3": ([vp, vp, vp, vp, vp, i32, i32, i32, vp, vp], i32),
        "agg_num_sms": ([], i32),
        "agg_mc_broadcast": ([vp, u64, sz, vp, i32, vp], i32),
        "agg_verify_bytes": ([vp, vp, sz, vp, vp], i32),
        "agg_verify_pattern_gather": ([vp, sz, i32, vp, vp], i32),
        "agg_alias_fence": ([vp], i32),
        "agg_multimem_ops_test": ([u64, vp, ctypes.c_float, vp], i32),
        "agg_multimem_ld_reduce_v4": ([u64, vp, sz, vp], i32),
        "agg_multimem_red_add_v4": ([u64, ctypes.c_float, sz, vp], i32),
        "agg_mm_barrier": ([vp, vp, i32, u32, i32, vp, u64, vp], i32),
        "agg_wait_flag": ([vp, u32, vp, u64, vp], i32),
        "agg_gemm_bf16_noalloc": ([vp, vp, vp, i32, i32, i32, i32, vp, vp], i32),
        "agg_launch_rs": ([ctypes.POINTER(agg_rs_args), vp], i32),
        "agg_rs_args_size": ([], sz),
        "agg_ce_allgather": ([ctypes.POINTER(agg_rank_info), u64, vp, sz, i32, vp], i32),
        "agg_stream_write_u32": ([u64, u32, vp], i32),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def check(rc: int, what: str = "") -> None:
    if rc != AGG_OK:
        msg = lib().agg_last_error().decode(errors="replace")
        raise AggError(f"{what or 'libagg'} failed ({rc}): {msg}")


def describe_status(word: int) -> str:
    if word == 0:
        return "ok"
    return f"{ROLE_NAMES.get(word & 0xFF, '?')} wait timed out at {word >> 8}"


# ---- torch plumbing -------------------------------------------------------------
def _torch():
    import torch

    return torch


def _stream_ptr(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class _DevView:
    """__cuda_array_interface__ over raw device memory (a slab region)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape),
            "typestr": typestr,
            "data": (int(ptr), False),
            "version": 3,
            "strides": None,
        }


def device_view(ptr: int, shape, dtype, device=None):
    """A torch tensor aliasing device memory at `ptr` (no copy)."""
    torch = _torch()
    typestr = {torch.bfloat16: "<f2", torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1",
               torch.int64: "<i8", torch.uint32: "<u4"}[dtype]
    if dtype == torch.bfloat16:
        # bf16 has no array-interface code: view the bytes as int16 and reinterpret
        t = torch.as_tensor(_DevView(ptr, shape, "<i2"), device=device or "cuda")
        return t.view(torch.bfloat16)
    return torch.as_tensor(_DevView(ptr, shape, typestr), device=device or "cuda")


def _check_operand(t, name, dtype=None):
    torch = _torch()
    if not t.is_cuda:
        raise AggError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise AggError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise AggError(f"{name} must be {dtype}, got {t.dtype}")
    return t


def gemm(A, B, out=None, status=None, stream=None):
    """C[M, N] = A[M, K] . B[N, K]^T on one GPU (bf16 in, fp32 accumulate, bf16 out)."""
    torch = _torch()
    _check_operand(A, "A", torch.bfloat16)
    _check_operand(B, "B", torch.bfloat16)
    M, K = A.shape
    N, K2 = B.shape
    if K != K2:
        raise AggError(f"K mismatch {K} vs {K2}")
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=A.device)
    st = ctypes.c_void_p(status.data_ptr()) if status is not None else None
    check(lib().agg_gemm_bf16(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                              ctypes.c_void_p(out.data_ptr()), M, N, K, st, _stream_ptr(stream)),
          "agg_gemm_bf16")
    return out


def quantize_rows_e4m3(x):
    """Per-row amax scaling to e4m3 on the device: s = amax/448 (1 for an all-zero
    row), q = e4m3(x / s) rounded to nearest even.  Returns (uint8 payload, float32 s)."""
    torch = _torch()
    xf = x.float()
    amax = xf.abs().amax(dim=1)
    # tensor / tensor is an IEEE division (a Python scalar divisor becomes a
    # multiplication by its rounded reciprocal)
    s = torch.where(amax > 0, amax / torch.full_like(amax, 448.0), torch.ones_like(amax)).contiguous()
    q = (xf / s[:, None]).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8).contiguous()
    return q, s


def gemm_e4m3(A_q, B_q, scale_a, scale_b, out=None, status=None, stream=None):
    """C = (s_a[:,None] * A_q) . (s_b[:,None] * B_q)^T with e4m3 operands (uint8 payloads)."""
    torch = _torch()
    M, K = A_q.shape
    N, _ = B_q.shape
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=A_q.device)
    st = ctypes.c_void_p(status.data_ptr()) if status is not None else None
    check(lib().agg_gemm_e4m3(ctypes.c_void_p(A_q.data_ptr()), ctypes.c_void_p(B_q.data_ptr()),
                              ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(scale_a.data_ptr()),
                              ctypes.c_void_p(scale_b.data_ptr()), M, N, K, st, _stream_ptr(stream)),
          "agg_gemm_e4m3")
    return out


# ---- one process driving several GPUs (the reference's model) -------------------
class RankState:
    """include/multimem.cuh:11-20 as seen from Python."""

    def __init__(self, info: agg_rank_info):
        self.info = info
        self.uc = info.uc
        self.mc = info.mc
        self.peer_addresses = [info.peer_uc[i] for i in range(AGG_MAX_RANKS)]
        self.slab_bytes = info.slab_bytes
        self.flag_off = info.flag_off


def spmm_init(rank: int, world: int, device: int, data_bytes: int) -> RankState:
    info = agg_rank_info()
    check(lib().agg_spmm_init(rank, world, device, data_bytes, ctypes.byref(info)), "agg_spmm_init")
    return RankState(info)


# ---- one process per GPU ----------------------------------------------------------
class MulticastSlab:
    """This rank's slab of an NVLink multicast object shared by `world` processes.

    Collective: every rank constructs it in the same order.  `barrier` is a
    callable that blocks until all ranks reach it (torch.distributed.barrier on
    a gloo group by default); `job_id` must match across ranks.
    """

    def __init__(self, rank: int, world: int, device: int, data_bytes: int, job_id: str, barrier):
        self.rank, self.world, self.device = rank, world, device
        ctx = ctypes.c_void_p()
        check(lib().agg_mp_open(rank, world, device, data_bytes, job_id.encode(), ctypes.byref(ctx)),
              "agg_mp_open")
        self._ctx = ctx
        try:
            barrier()
            check(lib().agg_mp_exchange(ctx), "agg_mp_exchange")
            check(lib().agg_mp_add_device(ctx), "agg_mp_add_device")
            barrier()
            info = agg_rank_info()
            check(lib().agg_mp_bind(ctx, ctypes.byref(info)), "agg_mp_bind")
            barrier()
        except Exception:
            lib().agg_mp_close(ctx)
            self._ctx = None
            raise
        self.info = info
        self.uc, self.mc = info.uc, info.mc
        self.peer_uc = [info.peer_uc[i] for i in range(world)]
        self.slab_bytes, self.flag_off = info.slab_bytes, info.flag_off

    # addresses inside the slab
    def flags(self, mc: bool = False) -> int:
        return (self.mc if mc else self.uc) + self.flag_off + AGG_FLAG_CHUNK_OFF

    def done(self, mc: bool = False) -> int:
        return (self.mc if mc else self.uc) + self.flag_off + AGG_FLAG_DONE_OFF

    def user(self, mc: bool = False) -> int:
        return (self.mc if mc else self.uc) + self.flag_off + AGG_FLAG_USER_OFF

    def close(self):
        if self._ctx is not None:
            lib().agg_mp_close(self._ctx)
            self._ctx = None


def _default_group_barrier(group):
    import torch.distributed as dist

    return lambda: dist.barrier(group=group)


def make_job_id(group=None) -> str:
    """A token equal on every rank of `group` and unique on the machine."""
    import torch.distributed as dist

    obj = [uuid.uuid4().hex[:16] if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


class _SlabEpochs:
    """Launch bookkeeping shared by the fused operators.  Every launch on a slab
    raises its counters by a fixed amount, and the kernels compute their wait
    targets from the launch epoch.  A launch that gave up (nonzero status)
    leaves the counters short, so later launches would wait for counts that
    never come, or start early: after a failure the operator refuses to launch
    until `reset()` (collective: every rank calls it) has zeroed the slab's
    counters and restarted the epochs."""

    def _init_epochs(self):
        self.epoch = 0
        self._failed = None

    def _before_launch(self):
        if self._failed:
            raise AggError(f"a previous launch failed ({self._failed}); call reset() on every rank first")
        self.epoch += 1

    def _status_word(self):
        word = int(self.status.item())
        if word:
            self._failed = describe_status(word)
            raise AggError(f"device status: {self._failed}")

    def reset(self):
        """Collective: wait for this GPU, meet the other ranks, zero this GPU's
        slab counters (flag area), meet again, and start the epochs over."""
        torch = _torch()
        torch.cuda.synchronize(self.device)
        if self.slab is not None:
            import torch.distributed as dist

            dist.barrier(group=self._host_group)
            device_view(self.slab.uc + self.slab.flag_off, (AGG_FLAG_BYTES,), torch.uint8, self.device).zero_()
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self._host_group)
        self.status.zero_()
        self._init_epochs()


class AllGatherGemm(_SlabEpochs):
    """C_r = AllGather(A_r) . B_r^T across the ranks of torch.distributed, fused in one kernel.

    world == 1 (or no process group) runs the same kernel as a plain GEMM.
    The gathered activation lives in this GPU's multicast slab; the rank's own
    shard is read from the caller's tensor.  With `double_buffer` (default) the
    slab holds two gathered regions used by launch parity, so consecutive
    launches never wait for each other across ranks.
    """

    def __init__(self, m_local: int, k: int, *, dtype: str = "bf16", group=None, device=None,
                 timeout_s: float = 10.0, host_group=None, double_buffer: bool = True, producer: str = "auto"):
        """`producer` chooses who moves this rank's shard: "sm" (the kernel's own
        warps, multimem.st; default), "sm_peer" (the same warps, one 16-byte
        store per rank through the unicast peer mappings; bf16), "ce_mc" (copy
        engines, one copy per chunk into the multicast VA) or "ce_push" (copy
        engines, one copy per chunk and peer); the copy-engine modes need bf16
        and double buffering.  "auto" (default) picks "sm_peer" for bf16 on 2-4
        ranks and "sm" otherwise: measured on the fused kernel, the unicast
        stores win up to P = 4 (the multicast path delivers 345-540 GB/s of
        ingress per GPU there) and lose at P = 8, where their 7x egress from
        the SMs competes with the GEMM."""
        torch = _torch()
        import torch.distributed as dist

        if producer == "auto":
            w = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
            producer = "sm_peer" if dtype == "bf16" and 2 <= w <= 4 else "sm"
        if producer not in PRODUCERS:
            raise AggError(f"producer must be one of {sorted(PRODUCERS) + ['auto']}")
        if producer.startswith("ce") and (dtype != "bf16" or not double_buffer):
            raise AggError("copy-engine producers need bf16 and double buffering")
        if producer == "sm_peer" and dtype != "bf16":
            raise AggError("the SM peer push moves bf16 shards only")
        self.producer = producer
        self.dtype = dtype
        self.elem = 1 if dtype == "e4m3" else 2
        self.m_local, self.k = m_local, k
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.timeout_ns = int(timeout_s * 1e9)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._init_epochs()
        self.slab = None
        self._host_group = None
        self.double_buffer = double_buffer
        if self.world > 1:
            if m_local % AGG_TILE_M:
                raise AggError(f"rows per rank ({m_local}) must be a multiple of {AGG_TILE_M}")
            hg = host_group if host_group is not None else dist.new_group(backend="gloo")
            self._host_group = hg
            job = make_job_id(hg)
            regions = 2 if double_buffer else 1
            M = self.world * m_local
            data = regions * M * k * self.elem + (regions * M * 4 if self.elem == 1 else 0)  # + gathered scales
            self.slab = MulticastSlab(self.rank, self.world, self.device.index, data, job,
                                      _default_group_barrier(hg))

    @property
    def M(self) -> int:
        return self.world * self.m_local

    def gathered(self):
        """The gathered activation [M, K] of the latest launch in this GPU's slab
        (valid once that launch has completed)."""
        torch = _torch()
        if self.slab is None:
            raise AggError("no slab at world == 1")
        dt = torch.bfloat16 if self.elem == 2 else torch.uint8
        region = (self.epoch & 1) if self.double_buffer else 0
        return device_view(self.slab.uc + region * self.M * self.k * self.elem, (self.M, self.k), dt, self.device)

    def new_trace(self):
        """A zeroed trace buffer for one launch (pass as `trace=`)."""
        torch = _torch()
        return torch.zeros((lib().agg_num_sms(), AGG_TRACE_SLOTS), dtype=torch.int64, device=self.device)

    def __call__(self, A_r, B_r, out=None, scale_a=None, scale_b=None, stream=None, trace=None):
        torch = _torch()
        if A_r.shape != (self.m_local, self.k):
            raise AggError(f"A_r must be [{self.m_local}, {self.k}], got {tuple(A_r.shape)}")
        N, K = B_r.shape
        if K != self.k:
            raise AggError("B_r must be [N_r, K]")
        _check_operand(A_r, "A_r")
        _check_operand(B_r, "B_r")
        if out is None:
            out = torch.empty((self.M, N), dtype=torch.bfloat16, device=self.device)
        self._before_launch()
        a = agg_args()
        a.B = B_r.data_ptr()
        a.C = out.data_ptr()
        a.A_src = A_r.data_ptr()
        a.A_copy_epoch = self.epoch
        a.dev_idx = self.rank
        a.M, a.N, a.K = self.M, N, self.k
        a.world = self.world
        a.dtype = AGG_DTYPE_E4M3 if self.elem == 1 else AGG_DTYPE_BF16
        a.status = self.status.data_ptr()
        a.timeout_ns = self.timeout_ns
        if trace is not None:
            a.trace = trace.data_ptr()
        if self.elem == 1:
            a.scale_a = scale_a.data_ptr()
            a.scale_b = scale_b.data_ptr()
        if self.slab is not None:
            s = self.slab
            a.A_mc = s.mc
            for i in range(self.world):
                a.A_peer[i] = s.peer_uc[i]
            a.A_local_buf = s.uc
            a.A_copy_ready = s.flags()
            a.A_copy_ready_mc = s.flags(mc=True)
            a.done_uc = s.done()
            a.done_mc = s.done(mc=True)
            if self.double_buffer:
                a.flags |= AGG_ARGS_DOUBLE_BUFFER
            a.flags |= PRODUCERS[self.producer]
        check(lib().agg_launch(ctypes.byref(a), _stream_ptr(stream)), "agg_launch")
        return out

    def check_status(self):
        self._status_word()

    def close(self):
        if self.slab is not None:
            self.slab.close()
            self.slab = None


class GemmReduceScatter(_SlabEpochs):
    """Y_r = rows [r*M/P, (r+1)*M/P) of sum_s X_s . W_s^T, fused in one kernel per rank.

    The row-parallel twin of AllGatherGemm (a tensor-parallel down projection):
    rank s holds X_s [M, K_s] and W_s [N, K_s], slices of the contraction.  Each
    rank's kernel stores its bf16 partial product tile by tile straight into
    the owning rank's inbox (a slot per source rank in every slab); the owner
    adds the slots of each of its tiles (fp32, source order) as they complete.
    world == 1 runs the plain GEMM.  With `double_buffer` (default) the slab
    holds two [M, N] partial regions used by launch parity.

    `exchange` chooses who moves the partials to their owners: "sm" (the
    epilogue warps TMA-store them into the owners' inboxes over NVLink) or
    "ce" (the epilogue stores them into a local stage in owner order and the
    copy engines copy each owner's block as soon as it is complete, so the SMs
    only do the GEMM and the reduction; needs an extra [M, N] bf16 buffer).
    "auto" (default) picks "ce".
    """

    EXCHANGES = ("sm", "ce")

    def __init__(self, m: int, n: int, k_local: int, *, group=None, device=None, timeout_s: float = 10.0,
                 host_group=None, double_buffer: bool = True, exchange: str = "auto"):
        torch = _torch()
        import torch.distributed as dist

        if exchange == "auto":
            exchange = "ce"
        if exchange not in self.EXCHANGES:
            raise AggError(f"unknown exchange {exchange!r} (one of {', '.join(self.EXCHANGES)} or auto)")
        self.exchange = exchange
        self.stage = None
        self.M, self.N, self.k = m, n, k_local
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.timeout_ns = int(timeout_s * 1e9)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._init_epochs()
        self.slab = None
        self._host_group = None
        self.double_buffer = double_buffer
        if m % self.world or (self.world > 1 and (m // self.world) % 256):
            raise AggError(f"M ({m}) must split into row blocks of a multiple of 256 over {self.world} ranks")
        if self.world > 1:
            hg = host_group if host_group is not None else dist.new_group(backend="gloo")
            self._host_group = hg
            job = make_job_id(hg)
            regions = 2 if double_buffer else 1
            self.slab = MulticastSlab(self.rank, self.world, self.device.index, regions * m * n * 2, job,
                                      _default_group_barrier(hg))
            if exchange == "ce":
                self.stage = torch.empty((m, n), dtype=torch.bfloat16, device=self.device)

    @property
    def m_local(self) -> int:
        return self.M // self.world

    def new_trace(self):
        torch = _torch()
        return torch.zeros((lib().agg_num_sms(), AGG_TRACE_SLOTS), dtype=torch.int64, device=self.device)

    def __call__(self, X_r, W_r, out=None, stream=None, trace=None):
        torch = _torch()
        if tuple(X_r.shape) != (self.M, self.k) or tuple(W_r.shape) != (self.N, self.k):
            raise AggError(f"X_r must be [{self.M}, {self.k}] and W_r [{self.N}, {self.k}]")
        _check_operand(X_r, "X_r", torch.bfloat16)
        _check_operand(W_r, "W_r", torch.bfloat16)
        if out is None:
            out = torch.empty((self.m_local, self.N), dtype=torch.bfloat16, device=self.device)
        if self.world == 1:
            return gemm(X_r, W_r, out=out, status=self.status, stream=stream)
        self._before_launch()
        s = self.slab
        a = agg_rs_args()
        a.X, a.W, a.Y = X_r.data_ptr(), W_r.data_ptr(), out.data_ptr()
        for i in range(self.world):
            a.part_peer[i] = s.peer_uc[i]
        a.cnt_uc, a.cnt_mc = s.flags(), s.flags(mc=True)
        a.done_uc, a.done_mc = s.done(), s.done(mc=True)
        a.epoch = self.epoch
        a.rank, a.world = self.rank, self.world
        a.M, a.N, a.K = self.M, self.N, self.k
        a.flags = AGG_ARGS_DOUBLE_BUFFER if self.double_buffer else 0
        if self.stage is not None:
            a.flags |= AGG_ARGS_RS_COPY_ENGINE
            a.stage = self.stage.data_ptr()
        a.status = self.status.data_ptr()
        a.timeout_ns = self.timeout_ns
        if trace is not None:
            a.trace = trace.data_ptr()
        check(lib().agg_launch_rs(ctypes.byref(a), _stream_ptr(stream)), "agg_launch_rs")
        return out

    def check_status(self):
        self._status_word()

    def close(self):
        if self.slab is not None:
            self.slab.close()
            self.slab = None
        self.stage = None
