"""Host logic of the multi-GPU paths with two gloo ranks on the CPU (no GPU):
the max-over-ranks device time and the barrier the bench uses under
torchrun, the peer exchange of the column-sharded variant's IPC handles, and
the reference arm, which only rank 0 runs while the other ranks exit quietly."""
import contextlib
import io
import json
import multiprocessing as mp
import os
import socket
from datetime import timedelta
from types import SimpleNamespace

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, what, q):
    try:
        import torch.distributed as dist
        os.environ.update(RANK=str(rank), WORLD_SIZE="2", LOCAL_RANK=str(rank))
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                                timeout=timedelta(seconds=60))
        import bench
        if what == "max":
            bench.barrier(2)
            got = bench.max_over_ranks([1.5, 3.25][rank], 2, "cpu")
            q.put((rank, got))
        elif what == "exchange":
            from swarmlora_b200.engine import exchange_with_peer
            mine = bytes([rank]) * 64 * 3  # three 64-byte handles
            q.put((rank, exchange_with_peer(mine, rank)))
        elif what == "reference":
            args = SimpleNamespace(gpus=2, steps=1, warmup=0, slots=4, ctx_lo=256, ctx_hi=1024)
            out = io.StringIO()
            with contextlib.redirect_stdout(out):
                rc = bench.reference_arm(args)
            q.put((rank, (rc, out.getvalue())))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, f"error: {type(e).__name__}: {e}"))


def _run(what, timeout=300):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, what, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, v = q.get(timeout=timeout)
            res[r] = v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


def test_max_over_ranks_takes_the_slowest_rank():
    res = _run("max")
    assert res == {0: 3.25, 1: 3.25}


def test_peer_exchange_returns_the_other_ranks_handles():
    res = _run("exchange")
    assert res[0] == bytes([1]) * 192
    assert res[1] == bytes([0]) * 192


def test_reference_arm_runs_on_rank_zero_only():
    res = _run("reference")
    assert not isinstance(res[0], str), res[0]
    rc0, out0 = res[0]
    rc1, out1 = res[1]
    assert rc0 == 0 and rc1 == 0
    assert out1 == ""
    line = json.loads(out0.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
    assert line["metric"] == "decode tok/s/GPU (Llama-3.1-8B shape, N=4 slots)"


def test_metric_names_the_headline_configuration_and_other_slot_counts():
    import bench
    assert bench.metric_for(28) == "decode tok/s/GPU (Llama-3.1-8B shape, N=28 slots)"
    assert bench.metric_for(32) == "decode tok/s/GPU (Llama-3.1-8B shape, N=32 slots)"
