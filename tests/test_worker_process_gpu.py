"""The reference's deployment shape on one GPU: the aggregator's main loop in
this process, a worker in another process that opens the queue by name
(open_queue), maps its slot from the 64-byte CUDA IPC handles claim_slot
returned (open_slot, ext_unified_barrier.cpp:97-160, called with the
reference's keyword arguments), and issues one token's rounds in the
reference worker's order (worker_sync.py:1274-1425). The worker sends its
outputs back as bytes; they are checked here against the CPU oracle. No
kernel waits on another process: the processes meet only on the host
(shared-memory ring and epoch)."""
import io
import multiprocessing as mp
import threading
import traceback

import pytest
import torch

from oracle import reference_math as ref
from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
H, I, HQ, HKV, D, V = 256, 512, 2, 1, 128, 64
WID = 2001


def _worker(shm_name, slot, claim, q):
    try:
        import torch
        from swarmlora_b200 import ext_ipc_queue as extq
        from swarmlora_b200 import ext_unified_barrier as ub
        torch.cuda.set_device(0)
        cuda = torch.device("cuda", 0)
        extq.open_queue(shm_name, 64, 64)
        ub.init_worker_slot_manager(worker_id=WID, worker_device=0, aggregator_device=0, hidden_dim=H,
                                    intermediate_dim=I, qkv_dim=(HQ + 2 * HKV) * D)
        ub.open_slot(slot_id=slot, input_handle=claim["input_handle"], output_handle=claim["output_handle"],
                     input_buffer_size=claim["input_buffer_size"], output_buffer_size=claim["output_buffer_size"])
        # everything slow happens before the join: once active, the aggregator
        # evicts a slot that is not ready within 500 ms of a round
        g = torch.Generator().manual_seed(31)
        ops = (("qkv", ub.OP_QKV_FUSED, H, [HQ * D, HKV * D, HKV * D]), ("o", ub.OP_O_PROJ, HQ * D, [H]),
               ("gate_up", ub.OP_GATE_UP_FUSED, H, [I, I]), ("down", ub.OP_DOWN_PROJ, I, [H]))
        xs = {name: torch.randn(1, 1, K, generator=g).to(BF) for name, _, K, _ in ops}
        xs_dev = {name: x.to(cuda) for name, x in xs.items()}
        hid = torch.randn(1, 1, H, generator=g).to(BF)
        hid_dev = hid.to(cuda)
        token = 17
        ids_dev = torch.tensor([[token]], device=cuda)
        torch.cuda.synchronize()
        extq.slot_signal_join(slot)
        for _ in range(4000):
            if extq.slot_is_active(slot):
                break
            threading.Event().wait(0.005)
        assert extq.slot_is_active(slot), "slot never became active"

        def step(op, dx, prepare):
            prepare()
            e = extq.get_barrier_done_epoch()
            extq.submit_slot_command(op, 0, slot, WID, 1, 1, dx, 0, 0, 0, 0, 0)
            extq.slot_signal_ready(slot)
            extq.wait_for_epoch(e, timeout_ms=30000)  # bounded here; the reference waits without one

        r, got = {}, {}
        step(ub.OP_EMBED, 1, lambda: ub.prepare_token_ids_slot(slot, ids_dev))
        r["embed"] = ub.get_embeddings_slot(slot, BF)[0]
        for name, op, K, dims in ops:
            step(op, K, lambda: ub.prepare_input_slot(slot, op, xs_dev[name]))
            got[name] = torch.cat(ub.get_outputs_slot(slot, dims, xs_dev[name]), -1)[0]
        step(ub.OP_LM_HEAD, H, lambda: ub.prepare_hidden_for_lm_head_slot(slot, hid_dev))
        tok = int(ub.get_next_token_slot(slot))
        # host copies after the last round
        r = {"embed": r["embed"].cpu(), "lm_head": (hid[0], tok),
             **{name: (xs[name][0], got[name].cpu()) for name in got}}
        extq.slot_signal_leave(slot)
        for _ in range(4000):
            if not extq.slot_is_active(slot):
                break
            threading.Event().wait(0.005)
        ub.close_slot(slot)
        ub.cleanup_worker_slots()
        buf = io.BytesIO()
        torch.save((token, r), buf)
        q.put(("ok", buf.getvalue()))
    except Exception:
        q.put(("error", traceback.format_exc()))


def test_worker_process_maps_its_slot_by_ipc_handles(native, cuda):
    from swarmlora_b200 import ext_aggregator as agg
    from swarmlora_b200 import ext_ipc_queue as extq
    g = torch.Generator().manual_seed(30)

    def w(o, i):
        return (torch.randn(o, i, generator=g) * 0.05).to(BF)
    q_, k_, v_, o_ = w(HQ * D, H), w(HKV * D, H), w(HKV * D, H), w(H, HQ * D)
    gate, up, down = w(I, H), w(I, H), w(H, I)
    embed, lm = w(V, H), w(V, H)
    dev = [t.to(cuda) for t in (q_, k_, v_, o_, gate, up, down, embed, lm)]
    agg.init_slot_pool(1, 0, H, I, HKV, D, 16, 2)
    agg.init_aggregator_begin(1, 0)
    agg.init_aggregator_layer(0, dev[0], dev[1], dev[2], dev[3], torch.empty(0), dev[4], dev[5], dev[6],
                              torch.empty(0))
    agg.init_aggregator_finalize()
    agg.init_embed_lm_head_weights(dev[7], dev[8])
    info = extq.create_queue(64, 64)
    agg.init_aggregator_queue(info["shm_name"], 64)
    extq.init_batch_control(1)
    claim = agg.claim_slot(WID)
    assert len(claim["input_handle"]) == 64 and len(claim["output_handle"]) == 64
    loop_err = []

    def run_loop():
        try:
            agg.aggregator_main_loop_slots(1, 15)
        except Exception as e:
            loop_err.append(e)
    loop = threading.Thread(target=run_loop, daemon=True)
    loop.start()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_worker, args=(info["shm_name"], claim["slot_id"], claim, q))
    p.start()
    try:
        status, payload = q.get(timeout=600)
        assert status == "ok", payload
        token, r = torch.load(io.BytesIO(payload))
        assert torch.equal(r["embed"], embed[token:token + 1])
        fused = {"qkv": ref.fuse_qkv(q_, k_, v_), "o": o_, "gate_up": ref.fuse_gate_up(gate, up), "down": down}
        for name, W in fused.items():
            x, got = r[name]
            assert_close(got, ref.slot_round([x], W)[0], f"{name} round through the worker process")
        hid, tok = r["lm_head"]
        logits = ref.lm_head_logits(hid, lm)[0].float()
        assert logits[tok] >= logits.max() - 2.0 ** -7 * logits.max().abs()
    finally:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
        extq.set_quit(1)
        loop.join(timeout=60)
        agg.release_slot(claim["slot_id"], WID)
        extq.close_queue()
        agg.cleanup_slot_pool()
    assert not loop_err, loop_err
    assert p.exitcode == 0
