"""Host-side logic of the multi-rank path, run as two gloo ranks on the CPU.

What the GPU tests cannot isolate: that every rank agrees on the job token that
names the multicast rendezvous, that a set-up failure (here: no GPU driver)
surfaces as the same AggError on every rank instead of leaving one rank waiting
in a barrier, and that under torchrun only rank 0 of the reference arm prints
its result line.
"""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    import __graft_entry__ as ge

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    pkg = ge.load_package()
    agg = pkg.agg
    res = {"job": [agg.make_job_id(), agg.make_job_id()]}
    try:
        agg.MulticastSlab(rank, world, 0, 1 << 20, res["job"][0], lambda: dist.barrier())
        res["slab"] = "opened"
    except agg.AggError as e:
        res["slab"] = "AggError"
        res["slab_msg"] = str(e)
    # every rank reaches this barrier: nobody was left behind in set-up
    dist.barrier()
    dist.destroy_process_group()
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


def test_two_ranks_agree_on_job_and_fail_setup_alike(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.is_available():
        pytest.skip("checks the set-up failure path of a host without a GPU")
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    r0 = json.load(open(tmp_path / "rank0.json"))
    r1 = json.load(open(tmp_path / "rank1.json"))
    assert r0["job"] == r1["job"]
    assert r0["job"][0] != r0["job"][1] and len(r0["job"][0]) == 16
    assert r0["slab"] == r1["slab"] == "AggError"
    assert "agg_mp_open" in r0["slab_msg"]


def test_reference_arm_under_torchrun_prints_one_line_from_rank_zero():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3",
           "--workload", "qkv8b"]
    p = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, p.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2
    assert d["config"]["P"] == 2 and d["config"]["N_per_rank"] == 6144 // 2
    assert d["cpu_baseline"]["kind"] == "port" and d["e2e"]["h2d_bytes_per_step"] == 0
