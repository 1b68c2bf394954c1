"""Multicast write bandwidth sweep: a rank-local buffer pushed with 16-byte
multimem.st into the multicast slab, every GPU's copy checked byte for byte.

This is the SM-driven counterpart of the reference's copy-engine multicast
cases (vmm/test_vmm_multicast_speed.cu:172-194 single and concurrent pushes,
verified at :301-429): message sizes from 1 MiB to 1 GiB, P = 2/4/8.

Patterns per size:
  single      rank 0 broadcasts `size` bytes into slot 0 (one writer, P copies);
  concurrent  every rank broadcasts its own `size` bytes into its slot at the
              same time — an all-gather through NVSwitch; each GPU receives
              (P-1) * size bytes;
  allgather_ce_mc / _ce_push / _ce_pull  (with copy_engines=True) the same
              all-gather by the copy engines, as the reference measures it:
              one cudaMemcpyAsync into the multicast VA, a push ring to the
              peers' unicast mappings, a pull ring from them (agg_ce_allgather).
Times are device time (CUDA events) per all-gather or push, the max over ranks.
Beside them, each rank's NVLink hardware counters (NVML, bytes sent and
received over all links during the timed pushes) give the traffic on the wire.
"""
from __future__ import annotations

import ctypes

from . import agg
from .nvlink_counters import NvlinkCounters, delta


def _src(torch, size, rank, device):
    g = torch.Generator(device=device).manual_seed(7919 * rank + size)
    return (torch.rand(size // 2, device=device, generator=g) * 2 - 1).bfloat16()


CE_MODES = {"allgather_ce_mc": agg.AGG_CE_MC_PUSH, "allgather_ce_push": agg.AGG_CE_PEER_PUSH,
            "allgather_ce_pull": agg.AGG_CE_PEER_PULL}


def run(slab, sizes, reps=10, warmup=3, group=None, copy_engines=False):
    """Runs the sweep on an initialised MulticastSlab (collective over `group`)."""
    import torch
    import torch.distributed as dist

    L = agg.lib()
    rank, world = slab.rank, slab.world
    device = torch.device("cuda", torch.cuda.current_device())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    bad = torch.zeros(1, dtype=torch.int64, device=device)
    rows = []
    counters = NvlinkCounters(device.index)

    def per_rank(x):
        out = [None] * world
        dist.all_gather_object(out, x, group=group)
        return out

    def barrier():
        dist.barrier(group=group)

    def max_ranks(x):
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item())

    for size in sizes:
        if world * size > slab.flag_off:
            raise agg.AggError(f"slab too small for {size} bytes x {world}")
        src = _src(torch, size, rank, device)
        row = {"bytes": size}
        patterns = ["single", "concurrent"] + (list(CE_MODES) if copy_engines else [])
        for pattern in patterns:
            writer = pattern != "single" or rank == 0
            dst = slab.mc + (rank if pattern == "concurrent" else 0) * size

            def push():
                if pattern in CE_MODES:
                    agg.check(L.agg_ce_allgather(ctypes.byref(slab.info), 0, ctypes.c_void_p(src.data_ptr()), size,
                                                 CE_MODES[pattern], stream))
                else:
                    agg.check(L.agg_mc_broadcast(ctypes.c_void_p(src.data_ptr()), dst, size, None, 0, stream))

            # clear every GPU's copy so stale data cannot pass the check
            agg.device_view(slab.uc, (world * size,), torch.uint8, device).zero_()
            if pattern == "allgather_ce_pull":  # the pull ring reads the peers' own slots
                agg.device_view(slab.uc + rank * size, (size // 2,), torch.bfloat16, device).copy_(src)
            torch.cuda.synchronize()
            barrier()
            if writer:
                for _ in range(warmup):
                    push()
            torch.cuda.synchronize()
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0 = counters.read()
            e0.record()
            if writer:
                for _ in range(reps):
                    push()
            e1.record()
            torch.cuda.synchronize()
            c1 = counters.read()
            barrier()
            ms = max_ranks(e0.elapsed_time(e1) / reps if writer else 0.0)
            d = delta(c0, c1)
            wire = per_rank(None if d is None else (d[0] / reps, d[1] / reps))
            agg.check(L.agg_alias_fence(stream))
            bad.zero_()
            slots = [0] if pattern == "single" else range(world)
            for s in slots:
                exp = _src(torch, size, s, device)
                agg.check(L.agg_verify_bytes(ctypes.c_void_p(slab.uc + s * size), ctypes.c_void_p(exp.data_ptr()),
                                             size, ctypes.c_void_p(bad.data_ptr()), stream))
            torch.cuda.synchronize()
            mism = int(max_ranks(float(bad.item())))
            recv = size if pattern == "single" else (world - 1) * size
            row[pattern] = {"ms": ms, "sender_gbs": size / (ms * 1e-3) / 1e9,
                            "ingress_gbs_per_gpu": recv / (ms * 1e-3) / 1e9,
                            "delivered_gbs": (world * size if pattern == "single" else world * (world - 1) * size)
                            / (ms * 1e-3) / 1e9,
                            "mismatched_words": mism}
            if all(w is not None for w in wire):
                # bytes on this GPU's links per push, and that over the max-over-ranks push time
                row[pattern]["nvlink_counters"] = {
                    "tx_bytes_per_push": [w[0] for w in wire], "rx_bytes_per_push": [w[1] for w in wire],
                    "tx_gbs": [w[0] / (ms * 1e-3) / 1e9 for w in wire],
                    "rx_gbs": [w[1] / (ms * 1e-3) / 1e9 for w in wire]}
        rows.append(row)
        del src
    return rows, counters.describe()
