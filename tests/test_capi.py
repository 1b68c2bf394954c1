"""The C-ABI library loads on a host without a GPU and exports what include/agg.h declares."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "agg.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(agg_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol(pkg):
    L = pkg.lib()
    declared = header_functions()
    assert len(declared) >= 25
    nm = subprocess.run(["nm", "-D", "--defined-only", pkg.agg.LIB_PATH], capture_output=True, text=True,
                        check=True).stdout
    exported = set(re.findall(r" T (agg_[a-z0-9_]+)", nm))
    missing = [f for f in declared if f not in exported]
    assert not missing, f"declared in agg.h but not exported: {missing}"
    assert set(pkg.agg.EXPORTS) == set(declared)
    for f in declared:
        getattr(L, f)


def test_library_has_no_driver_link_dependency(pkg):
    ldd = subprocess.run(["ldd", pkg.agg.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in ldd and "libtorch" not in ldd


def test_abi_struct_sizes_match_python(pkg):
    a = ctypes.c_size_t()
    r = ctypes.c_size_t()
    assert pkg.lib().agg_abi_sizes(ctypes.byref(a), ctypes.byref(r)) == 0
    assert a.value == ctypes.sizeof(pkg.agg.agg_args) == 208
    assert r.value == ctypes.sizeof(pkg.agg.agg_rank_info)
    assert pkg.lib().agg_version() == 100


def test_launch_rejects_bad_arguments_before_touching_the_gpu(pkg):
    agg = pkg.agg
    L = pkg.lib()
    base = dict(M=256, N=256, K=256, world=1, dev_idx=0, A_copy_epoch=1)

    def launch(**kw):
        a = agg.agg_args()
        a.A_src, a.B, a.C = 0x1000, 0x2000, 0x3000
        for k, v in {**base, **kw}.items():
            setattr(a, k, v)
        return L.agg_launch(ctypes.byref(a), None)

    assert launch(N=12) == -1                 # N*2 bytes not a 16-byte pitch
    assert launch(K=12) == -1                 # K*2 bytes not a 16-byte pitch
    assert launch(world=9) == -1
    assert launch(world=2, M=256 + 2) == -1   # M not divisible by world
    assert launch(world=2, M=2 * 100) == -1   # shard not a multiple of 128 rows
    assert launch(world=2, M=512) == -1       # multicast buffers missing
    assert launch(dtype=7) == -1
    assert launch(dtype=1) == -1              # e4m3 without scales
    assert b"scale" in L.agg_last_error()
    # copy-engine producers: one mode, double buffering, bf16, every rank's slab
    mc = dict(world=2, M=512, A_mc=0x100000, A_local_buf=0x200000, A_copy_ready=0x300000, A_copy_ready_mc=0x400000,
              done_uc=0x500000, done_mc=0x600000)
    both = agg.AGG_ARGS_CE_MC_PUSH | agg.AGG_ARGS_CE_PEER_PUSH
    assert launch(flags=both | agg.AGG_ARGS_DOUBLE_BUFFER, **mc) == -1
    assert launch(flags=agg.AGG_ARGS_CE_MC_PUSH, **mc) == -1               # single buffer
    assert b"DOUBLE_BUFFER" in L.agg_last_error()
    assert launch(flags=agg.AGG_ARGS_CE_MC_PUSH | agg.AGG_ARGS_DOUBLE_BUFFER, **mc) == -1   # no A_peer
    assert b"A_peer" in L.agg_last_error()


def test_reduce_scatter_layout_and_argument_checks(pkg):
    agg = pkg.agg
    L = pkg.lib()
    assert L.agg_rs_args_size() == ctypes.sizeof(agg.agg_rs_args)
    base = dict(X=0x1000, W=0x2000, Y=0x3000, cnt_uc=0x4000, cnt_mc=0x5000,
                done_uc=0x6000, done_mc=0x7000, epoch=1, rank=0, world=2, M=512, N=256, K=256)

    def launch(peers=(0x10000, 0x20000), **kw):
        a = agg.agg_rs_args()
        for k, v in {**base, **kw}.items():
            setattr(a, k, v)
        for i, v in enumerate(peers):
            a.part_peer[i] = v
        return L.agg_launch_rs(ctypes.byref(a), None)

    assert launch(world=1) == -1              # the twin needs 2..8 ranks
    assert launch(world=9) == -1
    assert launch(rank=2) == -1
    assert launch(M=2 * 384) == -1            # row block not a multiple of 256
    assert b"256" in L.agg_last_error()
    assert launch(N=12) == -1
    assert launch(K=12) == -1
    assert launch(epoch=0) == -1
    assert launch(Y=0x3008) == -1             # Y not 16-byte aligned
    assert launch(cnt_mc=0) == -1
    assert launch(peers=(0x10000, 0)) == -1   # a rank's inbox missing
    assert launch(peers=(0x10000, 0x20008)) == -1
    assert launch(M=2 * 256 * 64, N=256 * 129) == -1   # more tiles than counters
    assert b"tiles" in L.agg_last_error()
    ce = agg.AGG_ARGS_RS_COPY_ENGINE
    assert launch(flags=ce, status=0x8000) == -1                  # copy-engine exchange without a stage
    assert b"stage" in L.agg_last_error()
    assert launch(flags=ce, status=0x8000, stage=0x9008) == -1    # stage not 16-byte aligned
    assert launch(flags=ce, stage=0x9000) == -1                   # ... or without a status word
    assert b"status" in L.agg_last_error()
    assert launch(flags=ce, status=0x8000, stage=0x9000, done_uc=0x10000) == -1  # flags before the inbox
    assert b"done_uc" in L.agg_last_error()


def test_errors_without_gpu_are_reported_not_raised(pkg):
    import torch

    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    L = pkg.lib()
    assert L.agg_device_count() == 0
    info = pkg.agg.agg_rank_info()
    rc = L.agg_spmm_init(0, 2, 0, 1 << 20, ctypes.byref(info))
    assert rc < 0 and L.agg_last_error()
    assert L.agg_spmm_init(0, 2, 1, 1 << 20, ctypes.byref(info)) == -1  # rank != device


def test_nvlink_counter_reader_degrades_without_nvml(pkg):
    """The benchmark's NVLink byte counters come from NVML; where NVML or the
    fields are missing, the reader says why and reads nothing (no exception)."""
    import importlib

    nv = importlib.import_module(pkg.__name__ + ".nvlink_counters")
    c = nv.NvlinkCounters(0)
    if c.available:  # a GPU host with NVLink: the counters only grow
        a = c.read()
        b = c.read()
        assert b[0] >= a[0] and b[1] >= a[1]
    else:
        assert c.read() is None
        assert "unavailable" in c.describe() and c.why
    assert nv.delta(None, (1, 2)) is None
    assert nv.delta((1, 2), (4, 7)) == (3, 5)


def test_fused_ops_refuse_launches_after_a_failed_one(pkg):
    """A launch that gave up leaves the slab's counters short of their epoch
    targets; the operators then refuse to launch until a collective reset."""
    for cls in (pkg.agg.AllGatherGemm, pkg.agg.GemmReduceScatter):
        op = object.__new__(cls)
        op._init_epochs()
        op._before_launch()
        op._before_launch()
        assert op.epoch == 2
        op._failed = "flag wait timed out at 3"
        with pytest.raises(pkg.AggError, match="reset"):
            op._before_launch()
        assert op.epoch == 2
