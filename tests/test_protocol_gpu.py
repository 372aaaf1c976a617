"""The reference's deployment shape with this library's worker kernels: the
aggregator's main loop (aggregator_main_loop_slots) serving native worker
clients that request every round through the shared-memory ring and epoch
barrier (worker_sync.py:230-389, 1274-1425), one host thread per client.

* one client owning every slot (device-published completion with a flag
  input wait, event completion, event completion with per-segment graphs):
  the same launches as the in-process engine's step, so tokens and hidden
  rows are bit-identical to it;
* one client per two slots (the reference's host completion with a
  stream-sync input wait, and event completion): tokens and last-layer
  hidden rows against the CPU oracle (attention splits its work by the
  launch's rows, so this launch shape rounds differently from the engine's)."""
import copy

import pytest
import torch

from oracle.decode import decode_step
from tests.tolerances import ATOL_RMS_MULTILAYER, assert_close

pytestmark = pytest.mark.gpu
BF_ULP = 2.0 ** -8


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


def _group(cuda):
    from swarmlora_b200.engine import ModelConfig, SlotGroup, random_adapter, random_base
    cfg = ModelConfig(layers=2, vocab=4096)
    ctx = [20, 0, 31, 100, 7, 64]
    base = random_base(cfg, seed=1, device=cuda, norm_noise=0.1)
    adapters = [random_adapter(cfg, seed=10 + i, device=cuda) if i != 2 else None for i in range(len(ctx))]
    grp = SlotGroup(cfg, base, adapters, ctx, max_new=8, seed=3)
    return cfg, base, adapters, ctx, grp


@pytest.mark.parametrize("completion,input_ready,graphs", [("device", "flag", False), ("event", "event", False),
                                                            ("event", "event", True)])
def test_one_client_matches_the_engine_bit_for_bit(native, cuda, completion, input_ready, graphs):
    from swarmlora_b200.protocol import ProtocolRun
    cfg, base, adapters, ctx, grp = _group(cuda)
    try:
        k0 = [k.clone() for k in grp.k_cache]
        v0 = [v.clone() for v in grp.v_cache]
        first = torch.tensor([5, 4095, 17, 0, 1234, 77])
        grp.tokens.copy_(first)
        stream = torch.cuda.current_stream()
        want, want_h = [], []
        for _ in range(3):
            grp.enqueue_step(stream)
            torch.cuda.synchronize()
            want.append(grp.tokens.cpu().clone())
            want_h.append(grp.h.cpu().clone())
        for l in range(cfg.layers):
            grp.k_cache[l].copy_(k0[l])
            grp.v_cache[l].copy_(v0[l])
        grp.reset_positions()
        grp.tokens.copy_(first)
        run = ProtocolRun(grp, workers=1, completion=completion, input_ready=input_ready, graphs=graphs)
        try:
            got = run.run(3, record=True)
        finally:
            run.close()
        hist = got["history"].cpu()
        assert got["rounds"] == 3 * (1 + 4 * cfg.layers + 1)
        assert torch.equal(hist[-1], want[-1])
        for t in range(3):
            assert torch.equal(hist[t], want[t]), f"token {t}: {hist[t].tolist()} vs engine {want[t].tolist()}"
        assert torch.equal(grp.h.cpu(), want_h[-1])
        assert grp.seqlens.cpu().tolist() == [c + 3 for c in ctx]
    finally:
        grp.close()


@pytest.mark.parametrize("completion,input_ready,graphs", [("host", "sync", False), ("event", "event", False),
                                                            ("event", "event", True)])
def test_clients_of_two_slots_match_the_oracle(native, cuda, completion, input_ready, graphs):
    from swarmlora_b200.protocol import ProtocolRun
    cfg, base, adapters, ctx, grp = _group(cuda)
    try:
        base_c, ad_c = _cpu(base), _cpu(adapters)
        kc = [k.cpu() for k in grp.k_cache]
        vc = [v.cpu() for v in grp.v_cache]
        bts = [t.tolist() for t in grp.block_tables]
        tokens = [5, 4095, 17, 0, 1234, 77]
        grp.tokens.copy_(torch.tensor(tokens))
        run = ProtocolRun(grp, workers=3, completion=completion, input_ready=input_ready, graphs=graphs)
        try:  # all tokens in one go: the aggregator evicts a slot not ready within 500 ms
            got = run.run(3, record=True)
        finally:
            run.close()
        hist = got["history"].cpu()
        seq = list(ctx)
        for step in range(3):
            want, _, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, seq, tokens)
            picks = hist[step]
            for i, (g, w) in enumerate(zip(picks.tolist(), want.tolist())):
                if g != w:  # a tie within one bf16 ulp of the maximum logit
                    lg = logits[i].float()
                    assert lg[g] >= lg.max() - BF_ULP * lg.max().abs(), f"step {step} slot {i}: {g} != {w}"
            tokens = picks.tolist()  # the oracle follows the clients' picks
            seq = [s + 1 for s in seq]
        assert_close(grp.h, h_last, "last-layer hidden after three tokens", atol_rms=ATOL_RMS_MULTILAYER)
        assert grp.seqlens.cpu().tolist() == seq
    finally:
        grp.close()


def test_stalled_client_is_evicted_and_the_other_finishes(native, cuda):
    """Event completion with graphs: one of two clients runs one token and
    stops (its worker process died between tokens, as far as the aggregator
    can tell); the aggregator evicts its slots after the barrier timeout and
    the other client's remaining tokens still match the oracle."""
    import ctypes as C
    import threading
    from swarmlora_b200._native import lib
    from swarmlora_b200 import ext_ipc_queue as extq
    from swarmlora_b200.protocol import ProtocolRun
    cfg, base, adapters, ctx, grp = _group(cuda)
    try:
        base_c, ad_c = _cpu(base), _cpu(adapters)
        kc = [k.cpu() for k in grp.k_cache]
        vc = [v.cpu() for v in grp.v_cache]
        bts = [t.tolist() for t in grp.block_tables]
        tokens = [5, 4095, 17, 0, 1234, 77]
        grp.tokens.copy_(torch.tensor(tokens))
        run = ProtocolRun(grp, workers=2, completion="event", input_ready="event", graphs=True)
        try:
            run._start_loop()
            L = lib()
            hist = torch.zeros(3, 3, dtype=torch.int64, device=cuda)
            L.swl_wc_configure(run.handles[1], 2, 30000, C.c_void_p(hist.data_ptr()))
            L.swl_wc_configure(run.handles[0], 2, 30000, None)
            status = {}

            def client(i, n):
                status[i] = L.swl_wc_run(run.handles[i], n, None)
            t0 = threading.Thread(target=client, args=(0, 1))
            t1 = threading.Thread(target=client, args=(1, 3))
            t0.start()
            t1.start()
            t0.join(timeout=60)
            t1.join(timeout=60)
            assert status == {0: 0, 1: 0}, status
            gone = [extq.is_slot_evicted(grp.slot_ids[i]) for i in range(6)]
            assert gone == [True] * 3 + [False] * 3, gone
        finally:
            run.close()
        # the surviving slots (3..5) against the oracle over their three tokens
        seq = list(ctx)
        picks = hist.cpu()
        for step in range(3):
            want, _, logits, h_last = decode_step(cfg, base_c, ad_c, kc, vc, bts, seq, tokens)
            for j, i in enumerate(range(3, 6)):
                g = int(picks[step, j])
                if g != int(want[i]):
                    lg = logits[i].float()
                    assert lg[g] >= lg.max() - BF_ULP * lg.max().abs(), f"step {step} slot {i}: {g} != {int(want[i])}"
            # slots 0..2 stopped after the first token: the oracle keeps them
            # decoding, their rows do not touch the others'
            tokens = [int(x) for x in want.tolist()[:3]] + [int(picks[step, j]) for j in range(3)]
            seq = [s + 1 for s in seq]
        assert_close(grp.h[3:], h_last[3:], "surviving slots' last-layer hidden", atol_rms=ATOL_RMS_MULTILAYER)
    finally:
        grp.close()
