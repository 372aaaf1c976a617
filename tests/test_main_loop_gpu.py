"""The drop-in protocol end to end on one GPU: aggregator_main_loop_slots
(ext_aggregator.cpp:1024-1210) serving two workers through the shared-memory
ring and epoch barrier (ext_ipc_queue) and the slot buffers
(ext_unified_barrier), each worker issuing one token's ops in the reference
worker's order (worker_sync.py:1274-1425: embed, QKV, O, Gate+Up, Down, LM
head; epoch captured before slot_signal_ready). Every round's output is
checked against the CPU oracle; in the sampling variant one worker's LM
head samples (top_k = 1, posted before its join), the other's is greedy."""
import threading

import pytest
import torch

from oracle import reference_math as ref
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


@pytest.mark.parametrize("sampling", [False, True], ids=["greedy", "sampling"])
def test_main_loop_serves_two_workers(native, cuda, sampling):
    from swarmlora_b200 import ext_aggregator as agg
    from swarmlora_b200 import ext_ipc_queue as extq
    from swarmlora_b200 import ext_unified_barrier as ub
    H, I, hq, hkv, D, V = 256, 512, 2, 1, 128, 64
    g = torch.Generator().manual_seed(5)

    def w(o, i):
        return (torch.randn(o, i, generator=g) * 0.05).to(BF)

    q, k, v, o = w(hq * D, H), w(hkv * D, H), w(hkv * D, H), w(H, hq * D)
    gate, up, down = w(I, H), w(I, H), w(H, I)
    embed, lm = w(V, H), w(V, H)
    dev = {name: t.to(cuda) for name, t in dict(q=q, k=k, v=v, o=o, gate=gate, up=up, down=down,
                                                 embed=embed, lm=lm).items()}
    agg.init_slot_pool(2, 0, H, I, hkv, D, 16, 2)
    agg.init_aggregator_begin(1, 0)
    agg.init_aggregator_layer(0, dev["q"], dev["k"], dev["v"], dev["o"], torch.empty(0), dev["gate"],
                              dev["up"], dev["down"], torch.empty(0))
    agg.init_aggregator_finalize()
    agg.init_embed_lm_head_weights(dev["embed"], dev["lm"])
    info = extq.create_queue(64, 64)
    agg.init_aggregator_queue(info["shm_name"], 64)
    extq.init_batch_control(2)
    ub.init_worker_slot_manager(1001, 0, 0, H, I, (hq + 2 * hkv) * D)
    slots = []
    for wid in (1001, 1002):
        c = agg.claim_slot(wid)
        a_in, a_out = agg.slot_buffers(c["slot_id"])
        ub.attach_slot(c["slot_id"], a_in, a_out, c["input_buffer_size"], c["output_buffer_size"])
        slots.append((c["slot_id"], wid))
    if sampling:
        # the second worker posts sampling with top_k = 1 before it joins: its
        # LM-head round goes through the sampling kernel and keeps only the
        # maximum (worker_sync.py posts its request's parameters this way)
        extq.slot_set_pending_sampling(slots[1][0], True, 1.0, 1, 1.0)
    for s, _ in slots:  # both join before the loop starts: they activate together
        extq.slot_signal_join(s)

    loop_err = []

    def run_loop():
        try:
            agg.aggregator_main_loop_slots(2, 15)
        except Exception as e:  # surfaced by the assertion below
            loop_err.append(e)

    loop = threading.Thread(target=run_loop, daemon=True)
    loop.start()
    results, errors = {}, []

    def worker(slot, wid, token, seed):
        try:
            torch.cuda.set_device(0)
            gw = torch.Generator().manual_seed(seed)
            for _ in range(2000):
                if extq.slot_is_active(slot):
                    break
                threading.Event().wait(0.005)
            assert extq.slot_is_active(slot), "slot never became active"

            def step(op, dx, prepare):
                prepare()
                e = extq.get_barrier_done_epoch()
                extq.submit_slot_command(op, 0, slot, wid, 1, 1, dx, 0, 0, 0, 0, 0)
                extq.slot_signal_ready(slot)
                extq.wait_for_epoch(e, timeout_ms=30000)

            r = {}
            step(ub.OP_EMBED, 1, lambda: ub.prepare_token_ids_slot(slot, torch.tensor([[token]], device=cuda)))
            r["embed"] = ub.get_embeddings_slot(slot, BF)[0].cpu()
            for name, op, K, dims in (("qkv", ub.OP_QKV_FUSED, H, [hq * D, hkv * D, hkv * D]),
                                      ("o", ub.OP_O_PROJ, hq * D, [H]),
                                      ("gate_up", ub.OP_GATE_UP_FUSED, H, [I, I]),
                                      ("down", ub.OP_DOWN_PROJ, I, [H])):
                x = torch.randn(1, 1, K, generator=gw).to(BF)
                step(op, K, lambda: ub.prepare_input_slot(slot, op, x.to(cuda)))
                outs = ub.get_outputs_slot(slot, dims, x.to(cuda))
                r[name] = (x[0], torch.cat([t.cpu() for t in outs], -1)[0])
            hid = torch.randn(1, 1, H, generator=gw).to(BF)
            step(ub.OP_LM_HEAD, H, lambda: ub.prepare_hidden_for_lm_head_slot(slot, hid.to(cuda)))
            r["lm_head"] = (hid[0], ub.get_next_token_slot(slot))
            results[slot] = (token, r)
        except Exception as e:
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(s, wid, 7 + i * 20, 100 + i))
               for i, (s, wid) in enumerate(slots)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    extq.set_quit(1)
    loop.join(timeout=60)
    try:
        assert not errors, errors
        assert not loop_err, loop_err
        assert not loop.is_alive(), "main loop did not stop on quit"
        fused = {"qkv": ref.fuse_qkv(q, k, v), "o": o, "gate_up": ref.fuse_gate_up(gate, up), "down": down}
        for slot, (token, r) in results.items():
            assert torch.equal(r["embed"], embed[token:token + 1])
            for name, W in fused.items():
                x, got = r[name]
                assert_close(got, ref.slot_round([x], W)[0], f"slot {slot} {name} round")
            hid, tok = r["lm_head"]
            logits = ref.lm_head_logits(hid, lm)[0].float()
            assert logits[tok] >= logits.max() - 2.0 ** -7 * logits.max().abs()
        assert len(results) == 2
    finally:
        agg.set_worker_sampling(slots[1][1], False)  # later tests see a greedy worker
        for s, wid in slots:
            ub.close_slot(s)
            agg.release_slot(s, wid)
        ub.cleanup_worker_slots()
        extq.close_queue()
        agg.cleanup_slot_pool()
