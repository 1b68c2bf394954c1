"""Child-process bodies of the multi-GPU tests (one process per GPU, gloo for
the host-side rendezvous).  Each function returns a dict of results; the
parent collects them through a queue.  Kept free of pytest so spawn-started
children import it cheaply.

Every worker ends in _teardown(), also after an exception, so that no rank
leaves while its slab is still bound to the multicast object and the others
are still using it."""
from __future__ import annotations

import datetime
import os
import sys
import traceback

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def _init(rank, world, port):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    import __graft_entry__ as ge

    return ge.load_package()


def _teardown(*objs):
    """Wait for this GPU's work (every device wait is bounded), meet the other
    ranks, release the multicast slabs, meet again, leave the group."""
    import torch
    import torch.distributed as dist

    try:
        torch.cuda.synchronize()
    finally:
        try:
            dist.barrier()
        finally:
            for o in objs:
                if o is not None:
                    o.close()
            try:
                dist.barrier()
            finally:
                dist.destroy_process_group()


def _bits_to_dev(bits, shape):
    import numpy as np
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).reshape(shape)).view(torch.bfloat16).cuda()


def ag_gemm_parity(rank, world, port, m_local, k, n_r, launches, scheme, double_buffer=True, producer="sm"):
    """Fused all-gather GEMM vs the oracle on the reference harness's inputs
    (`producer`: who moves the shards, the kernel's warps or the copy engines)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import oracle

    pkg = _init(rank, world, port)
    op = None
    try:
        A_bits, A_ref, B_bits, B_ref = oracle.harness_inputs(world, m_local, k, n_r, scheme)
        A_r = _bits_to_dev(A_bits[rank], (m_local, k))
        B_r = _bits_to_dev(B_bits[rank], (n_r, k))
        op = pkg.AllGatherGemm(m_local, k, host_group=dist.group.WORLD, double_buffer=double_buffer,
                               producer=producer)
        outs = []
        for _ in range(launches):
            C = op(A_r, B_r)
            torch.cuda.synchronize()
            op.check_status()
            outs.append(C.clone())
        gathered = op.gathered().clone()
        torch.cuda.synchronize()
        want_gather = np.concatenate([b.reshape(m_local, k) for b in A_bits]).view(np.int16)
        gather_ok = bool(np.array_equal(gathered.view(torch.int16).cpu().numpy(), want_gather))
        full_A = np.concatenate([a.reshape(m_local, k) for a in A_ref])
        want = oracle.gemm_f64(full_A, B_ref[rank].reshape(n_r, k)).astype(np.float32)
        got = outs[-1].float().cpu().numpy()
        stats = oracle.error_stats(got, want)
        bad, where = oracle.check_close(got, want)
        same = all(torch.equal(o, outs[0]) for o in outs)
        return {"rank": rank, "gather_ok": gather_ok, "bad": bad, "where": where, "stats": stats,
                "launches_identical": same, "epoch": op.epoch}
    finally:
        _teardown(op)


def ag_gemm_e4m3_parity(rank, world, port, m_local, k, n_r, launches):
    """e4m3 fused all-gather GEMM (scales gathered with the chunks) vs the oracle."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import oracle

    pkg = _init(rank, world, port)
    op = None
    try:
        shards = []
        for s in range(world):
            x = np.random.default_rng(11 + s).standard_normal((m_local, k)).astype(np.float32)
            shards.append(oracle.quantize_e4m3_rows(x))
        wb = (np.random.default_rng(99 + rank).standard_normal((n_r, k)) * 0.02).astype(np.float32)
        qb, sb = oracle.quantize_e4m3_rows(wb)
        dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
        qa, sa = shards[rank]
        op = pkg.AllGatherGemm(m_local, k, dtype="e4m3", host_group=dist.group.WORLD)
        A_r, S_a, B_r, S_b = dev(qa), dev(sa), dev(qb), dev(sb)
        outs = []
        for _ in range(launches):
            outs.append(op(A_r, B_r, scale_a=S_a, scale_b=S_b))
        torch.cuda.synchronize()
        op.check_status()
        full = np.concatenate([oracle.dequantize_e4m3_rows(q, s) for q, s in shards])
        want = oracle.gemm_f64(full, oracle.dequantize_e4m3_rows(qb, sb)).astype(np.float32)
        got = outs[-1].float().cpu().numpy()
        stats = oracle.error_stats(got, want)
        bad, where = oracle.check_close(got, want)
        gathered = op.gathered().cpu().numpy()
        gather_ok = bool(np.array_equal(gathered, np.concatenate([q for q, _ in shards])))
        same = all(torch.equal(o, outs[0]) for o in outs)
        return {"rank": rank, "stats": stats, "bad": bad, "where": where, "gather_ok": gather_ok,
                "launches_identical": same}
    finally:
        _teardown(op)


def ag_gemm_changing_inputs(rank, world, port, m_local, k, n_r, launches, producer="sm"):
    """Back-to-back launches with different activations: each output must match
    its own inputs (checks the end-of-launch barrier that guards the gathered
    buffer against being overwritten while a slower rank still reads it, or,
    with copy-engine producers, the stream ordering that stands in for it)."""
    import torch
    import torch.distributed as dist

    pkg = _init(rank, world, port)
    op = None
    try:
        op = pkg.AllGatherGemm(m_local, k, host_group=dist.group.WORLD, producer=producer)
        g = torch.Generator(device="cuda").manual_seed(rank)
        B_r = (torch.randn(n_r, k, device="cuda", generator=g) * 0.05).bfloat16()
        outs = []
        shards = []
        for e in range(launches):
            ge_ = torch.Generator(device="cuda").manual_seed(100 * e + rank)
            A_r = torch.randn(m_local, k, device="cuda", generator=ge_).bfloat16()
            shards.append(A_r)
            outs.append(op(A_r, B_r))
        torch.cuda.synchronize()
        op.check_status()
        worst = 0.0
        for e in range(launches):
            parts = []
            for s in range(world):
                ge_ = torch.Generator(device="cuda").manual_seed(100 * e + s)
                parts.append(torch.randn(m_local, k, device="cuda", generator=ge_).bfloat16())
            ref = torch.cat(parts).float() @ B_r.float().t()
            err = ((outs[e].float() - ref).abs().max() / ref.abs().max()).item()
            worst = max(worst, err)
        return {"rank": rank, "worst_rel_err": worst}
    finally:
        _teardown(op)


def gemm_rs_parity(rank, world, port, m_per_rank, n, k, launches, double_buffer=True, exchange="auto",
                   compare_exchange=None):
    """Fused GEMM + reduce-scatter vs the oracle: launch e uses X_s, W_s drawn by
    fill_random from seeds 5000 + 100e + s and 6000 + s (U[-1, 1], bf16); rank r's
    output must be rows [r*M/P, (r+1)*M/P) of sum_s X_s . W_s^T.  With
    `compare_exchange`, a second operator using that exchange runs the same
    launches and its outputs must be bit-identical (same partials, same order)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import oracle

    pkg = _init(rank, world, port)
    op = other = None
    try:
        M = world * m_per_rank
        Ws = [oracle.fill_random_bf16(6000 + s, n * k) for s in range(world)]
        op = pkg.GemmReduceScatter(M, n, k, host_group=dist.group.WORLD, double_buffer=double_buffer,
                                   exchange=exchange)
        if compare_exchange:
            other = pkg.GemmReduceScatter(M, n, k, host_group=dist.group.WORLD, double_buffer=double_buffer,
                                          exchange=compare_exchange)
        W_r = _bits_to_dev(Ws[rank][0], (n, k))
        outs, inputs, identical = [], [], True
        for e in range(launches):
            Xs = [oracle.fill_random_bf16(5000 + 100 * e + s, M * k) for s in range(world)]
            inputs.append(Xs)
            X_r = _bits_to_dev(Xs[rank][0], (M, k))
            outs.append(op(X_r, W_r))
            if other is not None:
                identical = identical and torch.equal(other(X_r, W_r), outs[-1])
        torch.cuda.synchronize()
        op.check_status()
        if other is not None:
            other.check_status()
        worst, bad_total, bound_total, nan_total = 0.0, 0, 0, 0
        rows = slice(rank * m_per_rank, (rank + 1) * m_per_rank)
        for e in range(launches):
            parts = [oracle.gemm_f64(inputs[e][s][1].reshape(M, k)[rows], Ws[s][1].reshape(n, k))
                     for s in range(world)]
            want64 = sum(parts)
            want = want64.astype(np.float32)
            got = outs[e].float().cpu().numpy()
            stats = oracle.error_stats(got, want)
            bad, _ = oracle.check_close(got, want)
            # Each rank's partial is rounded to bf16 before the sum (as in a bf16
            # reduce-scatter): up to 2^-9 of every |partial| on top of the
            # reference's element check (atol 0.1, rtol 0.02).
            tol = 0.1 + 0.02 * np.abs(want64) + 2.0 ** -8 * sum(np.abs(p) for p in parts)
            bound_total += int(np.count_nonzero(~(np.abs(got - want64) <= tol)))
            worst = max(worst, stats["max_rel_err"])
            bad_total += bad
            nan_total += stats["nan"]
        return {"rank": rank, "worst_rel_err": worst, "bad_check_close": bad_total, "bad": bound_total,
                "nan": nan_total, "epoch": op.epoch, "exchange": op.exchange, "identical": identical}
    finally:
        _teardown(op, other)


def torch_ops_mlp(rank, world, port, m, k, n):
    """A tensor-parallel MLP (up: ColumnParallelLinear, down: RowParallelLinear)
    through the torch.library operators, against direct calls of the same kernels
    (bit-identical) and the up projection against torch on gathered inputs."""
    import importlib

    import torch
    import torch.distributed as dist

    pkg = _init(rank, world, port)
    ops = importlib.import_module(pkg.__name__ + ".torch_ops")
    up = down = ref_ag = ref_rs = None
    try:
        m_local, n_r = m // world, n // world
        g = torch.Generator(device="cuda").manual_seed(77 + rank)
        x_r = torch.randn(m_local, k, device="cuda", generator=g).bfloat16()
        w_up = (torch.randn(n_r, k, device="cuda", generator=g) * 0.05).bfloat16()
        w_down = (torch.randn(k, n_r, device="cuda", generator=g) * 0.05).bfloat16()
        up = ops.ColumnParallelLinear(w_up, m_local, host_group=dist.group.WORLD)
        down = ops.RowParallelLinear(w_down, m, host_group=dist.group.WORLD)
        h = up(x_r)       # [M, N/P]
        y_r = down(h)     # [M/P, K]
        ref_ag = pkg.AllGatherGemm(m_local, k, host_group=dist.group.WORLD)
        ref_rs = pkg.GemmReduceScatter(m, k, n_r, host_group=dist.group.WORLD)
        h2 = ref_ag(x_r, w_up)
        y2 = ref_rs(h2, w_down)
        torch.cuda.synchronize()
        up.op.check_status()
        down.op.check_status()
        parts = [torch.empty_like(x_r).cpu() for _ in range(world)]
        dist.all_gather(parts, x_r.cpu())
        ref = torch.cat(parts).cuda().float() @ w_up.float().t()
        up_err = float(((h.float() - ref).abs().max() / ref.abs().max()).item())
        return {"rank": rank, "up_identical": bool(torch.equal(h, h2)), "down_identical": bool(torch.equal(y_r, y2)),
                "up_rel_err": up_err, "shape_ok": tuple(y_r.shape) == (m_local, k)}
    finally:
        _teardown(up, down, ref_ag, ref_rs)


def multicast_sweep(rank, world, port, sizes, reps=1, mode="sm"):
    """Each rank moves `size` bytes into its slot on every GPU -- mode "sm":
    multimem.st (agg_mc_broadcast); "ce_mc" / "ce_push" / "ce_pull": the copy
    engines (agg_ce_allgather) -- and every rank's copy of every slot must be
    byte-identical to the sender's source."""
    import ctypes

    import torch
    import torch.distributed as dist

    pkg = _init(rank, world, port)
    agg = pkg.agg
    L = pkg.lib()
    slab = None
    try:
        maxb = max(sizes)
        slab = agg.MulticastSlab(rank, world, rank, world * maxb, agg.make_job_id(), lambda: dist.barrier())
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        bad = torch.zeros(1, dtype=torch.int64, device="cuda")
        res = []
        for size in sizes:
            def src_of(s):
                g = torch.Generator(device="cuda").manual_seed(7919 * s + size)
                return (torch.rand(size // 2, device="cuda", generator=g) * 2 - 1).bfloat16()

            src = src_of(rank)
            ce = {"ce_mc": agg.AGG_CE_MC_PUSH, "ce_push": agg.AGG_CE_PEER_PUSH, "ce_pull": agg.AGG_CE_PEER_PULL}

            def move():
                if mode == "sm":
                    agg.check(L.agg_mc_broadcast(ctypes.c_void_p(src.data_ptr()), slab.mc + rank * size, size, None,
                                                 0, stream))
                else:
                    agg.check(L.agg_ce_allgather(ctypes.byref(slab.info), 0, ctypes.c_void_p(src.data_ptr()), size,
                                                 ce[mode], stream))

            if mode == "ce_pull":  # the pull ring reads the peers' own slots: stage them first
                agg.device_view(slab.uc + rank * size, (size // 2,), torch.bfloat16).copy_(src)
                torch.cuda.synchronize()
                dist.barrier()
            for _ in range(2):  # warm-up
                move()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                move()
            e1.record()
            torch.cuda.synchronize()
            dist.barrier()
            agg.check(L.agg_alias_fence(stream))
            bad.zero_()
            for s in range(world):
                exp = src_of(s)
                agg.check(L.agg_verify_bytes(ctypes.c_void_p(slab.uc + s * size), ctypes.c_void_p(exp.data_ptr()),
                                             size, ctypes.c_void_p(bad.data_ptr()), stream))
            torch.cuda.synchronize()
            res.append({"size": size, "mismatched_words": int(bad.item()), "ms": e0.elapsed_time(e1) / reps})
        return {"rank": rank, "sweep": res}
    finally:
        _teardown(slab)


def multimem_known_answers(rank, world, port):
    """include/test_kernel.cuh:46-74 and vmm/main.cpp:121-204 generalised to P ranks,
    plus mm_barrier (vmm/multimem.cu:103-119) with a bounded wait."""
    import ctypes

    import numpy as np
    import torch
    import torch.distributed as dist

    pkg = _init(rank, world, port)
    agg = pkg.agg
    L = pkg.lib()
    slab = None
    try:
        slab = agg.MulticastSlab(rank, world, rank, 1 << 20, agg.make_job_id(), lambda: dist.barrier())
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rec_off = 4096  # kMulticastTestOffset, include/test_kernel.cuh:9
        rec = agg.device_view(slab.uc + rec_off, (4,), torch.float32)
        rec.copy_(torch.tensor([rank + 1.0, 0.0, rank + 1.0, 0.0]))
        torch.cuda.synchronize()
        agg.check(L.agg_alias_fence(stream))
        torch.cuda.synchronize()
        dist.barrier()
        reduced = torch.zeros(1, device="cuda")
        if rank == 0:
            agg.check(L.agg_multimem_ops_test(slab.mc + rec_off, ctypes.c_void_p(reduced.data_ptr()), 10.0, stream))
            torch.cuda.synchronize()
        dist.barrier()
        agg.check(L.agg_alias_fence(stream))
        torch.cuda.synchronize()
        observed = rec.cpu().tolist()
        expect_sum = float(sum(r + 1 for r in range(world)))
        out = {"rank": rank, "store_ok": observed[1] == expect_sum, "red_ok": observed[2] == rank + 1.0 + 10.0,
               "reduce_ok": (rank != 0) or float(reduced.item()) == expect_sum, "observed": observed}

        # vector ld_reduce / red over 1024 float4s
        n4 = 1024
        voff = 64 << 10
        vec = agg.device_view(slab.uc + voff, (4 * n4,), torch.float32)
        vec.copy_(torch.arange(4 * n4, device="cuda", dtype=torch.float32) * (rank + 1))
        torch.cuda.synchronize()
        dist.barrier()
        summed = torch.zeros(4 * n4, device="cuda")
        agg.check(L.agg_multimem_ld_reduce_v4(slab.mc + voff, ctypes.c_void_p(summed.data_ptr()), n4, stream))
        torch.cuda.synchronize()
        dist.barrier()
        agg.check(L.agg_multimem_red_add_v4(slab.mc + voff, 1.0, n4, stream))
        torch.cuda.synchronize()
        dist.barrier()
        agg.check(L.agg_alias_fence(stream))
        torch.cuda.synchronize()
        w = float(sum(r + 1 for r in range(world)))
        ar = np.arange(4 * n4, dtype=np.float32)
        out["ld_reduce_ok"] = bool(np.array_equal(summed.cpu().numpy(), ar * w))
        out["red_v4_ok"] = bool(np.array_equal(vec.cpu().numpy(), ar * (rank + 1) + world))

        # mm_barrier: every CTA of every rank adds 1 on all GPUs; wait for it * world
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        for it in (1, 2):
            agg.check(L.agg_mm_barrier(ctypes.c_void_p(slab.user(mc=True)), ctypes.c_void_p(slab.user()), 0,
                                       it * world, 8, ctypes.c_void_p(status.data_ptr()), 5_000_000_000, stream))
            torch.cuda.synchronize()
        out["barrier_status"] = int(status.item())
        flags = agg.device_view(slab.user(), (8,), torch.int32).cpu().tolist()
        out["barrier_flags_ok"] = flags == [2 * world] * 8
        return out
    finally:
        _teardown(slab)


def run_child(fn_name, rank, world, port, q, kwargs):
    try:
        fn = globals()[fn_name]
        q.put(("ok", rank, fn(rank, world, port, **kwargs)))
    except BaseException:
        q.put(("err", rank, traceback.format_exc()))
