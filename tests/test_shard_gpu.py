"""Column-sharded base weights over two GPUs (the multi-GPU configuration's
variant with an NVLink all-gather of the round outputs): two processes, one
GPU each, build the same slot group from the same seeds; every round then
computes one GPU's half of the output columns and stores it into both GPUs'
slot outputs by peer stores, ordered by epoch flags in each GPU's memory.

Checks, on the engine test's model (Llama-3.1-8B layer shapes, 2 layers,
4096-entry vocabulary, ragged contexts, one slot without adapter): both GPUs
end every step with bit-identical tokens and hidden states, these match the
CPU oracle like the one-GPU engine, a replayed CUDA graph reproduces the
eager tokens, and no bounded wait of the exchange ran out; and, with a peer
that never runs the round, that the round gives up after the 2 s limit,
reports it through swl_round_device_error and leaves the context usable.
Needs two GPUs; host-side failures surface as exceptions in the children.
"""
import copy
import io
import multiprocessing as mp
import socket
from datetime import timedelta

import pytest
import torch

from tests.tolerances import ATOL_RMS_MULTILAYER, assert_close

pytestmark = pytest.mark.gpu
BF_ULP = 2.0 ** -7
CTX = [20, 0, 31, 100, 7]
TOKENS0 = [5, 4095, 17, 0, 1234]
STEPS = 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _child(rank, port, q):
    try:
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                                timeout=timedelta(seconds=120))
        from swarmlora_b200 import rounds
        from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
        cfg = ModelConfig(layers=2, vocab=4096)
        base = random_base(cfg, seed=1, device=dev, norm_noise=0.1)
        adapters = [random_adapter(cfg, seed=10 + i, device=dev) if i != 2 else None for i in range(len(CTX))]
        grp = SlotGroup(cfg, base, adapters, CTX, max_new=8, device=rank, seed=3)
        try:
            kc0 = [k.clone() for k in grp.k_cache]
            vc0 = [v.clone() for v in grp.v_cache]
            grp.shard(rank)
            grp.tokens.copy_(torch.tensor(TOKENS0))
            stream = torch.cuda.current_stream(dev)
            steps = []
            for _ in range(STEPS):
                grp.enqueue_step(stream)
                torch.cuda.synchronize(dev)
                steps.append((grp.tokens.cpu(), grp.h.cpu(), grp.read_slot_rows("in", cfg.hidden).cpu()))
            err_eager = rounds.device_error()
            for l in range(cfg.layers):
                grp.k_cache[l].copy_(kc0[l])
                grp.v_cache[l].copy_(vc0[l])
            grp.reset_positions()
            grp.tokens.copy_(torch.tensor(TOKENS0))
            grp.capture()
            replay = []
            for _ in range(STEPS):
                grp.replay()
                torch.cuda.synchronize(dev)
                replay.append(grp.tokens.cpu())
            err_replay = rounds.device_error()
        finally:
            grp.close()
            dist.destroy_process_group()
        buf = io.BytesIO()  # plain bytes: nothing of the child's must outlive it
        torch.save((steps, replay), buf)
        q.put((rank, None, buf.getvalue(), (err_eager, err_replay)))
    except Exception as e:  # reported by the parent
        q.put((rank, f"{type(e).__name__}: {e}", None, None))


def _child_missing_peer(rank, port, q):
    """Rank 1 connects but never runs the round: rank 0's round gives up its
    wait for the peer's start flag after the time limit, records the error
    and returns (no peer stores), and the context stays usable."""
    try:
        import time
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                                timeout=timedelta(seconds=120))
        from swarmlora_b200 import ext_aggregator as agg
        from swarmlora_b200 import rounds
        from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
        cfg = ModelConfig(layers=1, vocab=4096)
        base = random_base(cfg, seed=1, device=dev)
        grp = SlotGroup(cfg, base, [random_adapter(cfg, seed=10 + i, device=dev) for i in range(2)], [4, 9],
                        max_new=4, device=rank, seed=3)
        result = None
        try:
            rounds.device_error()  # start clean
            grp.shard(rank)
            if rank == 0:
                s = torch.cuda.current_stream(dev)
                t0 = time.perf_counter()
                grp._round(agg.OP_QKV_FUSED, 0, s.cuda_stream)
                torch.cuda.synchronize(dev)
                elapsed = time.perf_counter() - t0
                code = rounds.device_error()
                ok = bool(torch.ones(4, device=dev).sum().item() == 4.0)  # the context still works
                result = (code, elapsed, ok)
            dist.barrier()  # rank 1 waits here, on the host, with nothing in flight
        finally:
            grp.close()
            dist.destroy_process_group()
        q.put((rank, None, result))
    except Exception as e:  # reported by the parent
        q.put((rank, f"{type(e).__name__}: {e}", None))


def _cpu(x):
    if isinstance(x, torch.Tensor):
        return x.cpu()
    if isinstance(x, list):
        return [_cpu(v) for v in x]
    if isinstance(x, dict):
        return {k: _cpu(v) for k, v in x.items()}
    if isinstance(x, tuple):
        return tuple(_cpu(v) for v in x)
    if x is None:
        return None
    out = copy.copy(x)
    for k, v in vars(x).items():
        setattr(out, k, _cpu(v))
    return out


def test_column_sharded_rounds_on_two_gpus(native, cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_child, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, err, blob, errs = q.get(timeout=600)
            steps, replay = torch.load(io.BytesIO(blob)) if blob is not None else (None, None)
            res[rank] = (err, steps, replay, errs)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert res[r][0] is None, f"rank {r}: {res[r][0]}"
        assert res[r][3] == (0, 0), f"rank {r}: a bounded wait of the exchange ran out {res[r][3]}"
    # both GPUs hold the same full outputs
    for step in range(STEPS):
        for a, b in zip(res[0][1][step], res[1][1][step]):
            assert torch.equal(a, b), f"step {step}: the GPUs disagree"
        assert torch.equal(res[0][2][step], res[0][1][step][0]), f"graph replay step {step} differs"
        assert torch.equal(res[1][2][step], res[1][1][step][0])
    # and they match the CPU oracle
    from oracle.decode import decode_step
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    base = random_base(cfg, seed=1, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=10 + i, device=cuda) if i != 2 else None for i in range(len(CTX))]
    grp = SlotGroup(cfg, base, adapters, CTX, max_new=8, seed=3)
    try:
        kc = [k.cpu() for k in grp.k_cache]
        vc = [v.cpu() for v in grp.v_cache]
        bts = [t.tolist() for t in grp.block_tables]
    finally:
        grp.close()
    base_c, ad_c = _cpu(base), _cpu(adapters)
    tokens, seq = list(TOKENS0), list(CTX)
    for step in range(STEPS):
        want, final, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, seq, tokens)
        got_tok, got_h, got_final = res[0][1][step]
        assert_close(got_h, h_last, f"sharded step {step} last-layer hidden", atol_rms=ATOL_RMS_MULTILAYER)
        assert_close(got_final, final, f"sharded step {step} LM-head input", atol_rms=ATOL_RMS_MULTILAYER)
        for i, (g, w) in enumerate(zip(got_tok.tolist(), want.tolist())):
            if g != w:
                lg = logits[i].float()
                assert lg[g] >= lg.max() - BF_ULP * lg.max().abs(), f"step {step}: slot {i} token {g} != {w}"
        tokens = got_tok.tolist()
        seq = [s + 1 for s in seq]


def test_missing_peer_round_gives_up_and_reports(native, cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_child_missing_peer, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, err, result = q.get(timeout=600)
            res[rank] = (err, result)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert res[r][0] is None, f"rank {r}: {res[r][0]}"
    code, elapsed, ok = res[0][1]
    assert code == 5, f"expected the peer-start wait to give up (5), got {code}"
    # one 2 s limit for the whole round: the other CTAs give up at once
    assert 1.5 < elapsed < 15.0, elapsed
    assert ok
