"""Donor weight transfer (export_weight_ipc_handles / import_weights_from_ipc,
ext_aggregator.cpp:1216-1406) between two processes on one GPU: the donor
initialises an aggregator whose borrowed weights (o, down, embed, lm_head)
are views at non-zero offsets inside one allocation, exports, and keeps its
weights alive until the receiver is done; the receiver imports and checks

* every weight's bytes against the donor's (sha256 per weight),
* a QKV round, a Down round, an embed round and a greedy LM-head round on
  the imported weights against torch on the same weights.

Only bytes, ints and dicts cross the process queues.
"""
import hashlib
import multiprocessing as mp
import traceback

import pytest
import torch

from tests.tolerances import assert_close

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
H, I, HQ, HKV, D, VOCAB, LAYERS = 512, 1024, 4, 2, 128, 2048, 2
OPS = (9, 3, 10, 6)  # OP_QKV_FUSED, OP_O_PROJ, OP_GATE_UP_FUSED, OP_DOWN_PROJ
OP_EMBED, OP_LM_HEAD = 11, 12


def _digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).cpu().numpy().tobytes()).hexdigest()


def _weight_bytes(lib, C, layer, op):
    """The aggregator's weight of (layer, op) copied into a torch tensor."""
    from swarmlora_b200._native import check, i64_array, ptr_array
    W, N, K = C.c_void_p(), C.c_int64(), C.c_int64()
    check(lib.swl_agg_weight(layer, op, C.byref(W), C.byref(N), C.byref(K)))
    out = torch.empty(N.value, K.value, dtype=BF, device="cuda:0")
    check(lib.swl_copy_rows(1, ptr_array([W.value]), ptr_array([out.data_ptr()]),
                            i64_array([N.value * K.value * 2]), None))
    torch.cuda.synchronize()
    return out


def _donor(q_out, q_done):
    try:
        import ctypes as C
        from swarmlora_b200 import ext_aggregator as agg
        from swarmlora_b200._native import lib
        torch.cuda.set_device(0)
        dev = torch.device("cuda:0")
        g = torch.Generator(device=dev).manual_seed(5)

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=dev) * 0.02).to(BF)
        # o / down / embed / lm_head as views inside one allocation, each at a
        # 1 KiB-aligned non-zero offset
        sizes = [H * HQ * D, H * I] * LAYERS + [VOCAB * H] * 2
        offs, at = [], 512
        for n in sizes:
            offs.append(at)
            at += (n + 511) // 512 * 512
        arena = torch.empty(at, dtype=BF, device=dev)
        views = []
        for n, o, shape in zip(sizes, offs, [(H, HQ * D), (H, I)] * LAYERS + [(VOCAB, H)] * 2):
            v = arena[o:o + n].view(shape)
            v.copy_(w(*shape))
            views.append(v)
        agg.init_aggregator_begin(LAYERS, 0)
        for l in range(LAYERS):
            agg.init_aggregator_layer(l, w(HQ * D, H), w(HKV * D, H), w(HKV * D, H), views[2 * l], torch.empty(0),
                                      w(I, H), w(I, H), views[2 * l + 1], torch.empty(0))
        agg.init_aggregator_finalize()
        agg.init_embed_lm_head_weights(views[-2], views[-1])
        digests = {(l, op): _digest(_weight_bytes(lib(), C, l, op)) for l in range(LAYERS) for op in OPS}
        digests[("embed",)] = _digest(views[-2])
        digests[("lm_head",)] = _digest(views[-1])
        handles = agg.export_weight_ipc_handles()
        q_out.put(("ok", handles, digests))
        q_done.get(timeout=300)  # weights stay alive until the receiver has finished
    except Exception:
        q_out.put(("error", traceback.format_exc(), None))


def _receiver(handles, digests, q_res):
    try:
        import ctypes as C
        from swarmlora_b200 import ext_aggregator as agg
        from swarmlora_b200._native import check, i64_array, lib, ptr_array
        torch.cuda.set_device(0)
        agg.import_weights_from_ipc(handles, 0)
        L = lib()
        for l in range(LAYERS):
            for op in OPS:
                assert _digest(_weight_bytes(L, C, l, op)) == digests[(l, op)], f"layer {l} op {op} bytes differ"
        emb, lm = _weight_bytes(L, C, 0, OP_EMBED), _weight_bytes(L, C, 0, OP_LM_HEAD)
        assert _digest(emb) == digests[("embed",)] and _digest(lm) == digests[("lm_head",)]
        # rounds on the imported weights through one pool slot
        agg.init_slot_pool(1, 0, H, I, HKV, D, 16, 2)
        sid = agg.claim_slot(7)["slot_id"]
        s_in, s_out = agg.slot_buffers(sid)

        def copy(dst, src, nbytes):
            check(L.swl_copy_rows(1, ptr_array([src]), ptr_array([dst]), i64_array([nbytes]), None))
            torch.cuda.synchronize()
        gx = torch.Generator().manual_seed(9)
        for layer, op, K in ((1, 9, H), (0, 6, I)):
            W = _weight_bytes(L, C, layer, op)
            x = torch.randn(3, K, generator=gx).to(BF).cuda()
            copy(s_in, x.data_ptr(), x.numel() * 2)
            agg.execute_round(op, layer, [sid], [7], [1], [3])
            torch.cuda.synchronize()
            y = torch.empty(3, W.shape[0], dtype=BF, device="cuda:0")
            copy(y.data_ptr(), s_out, y.numel() * 2)
            want = (x.float() @ W.float().t()).to(BF)
            assert_close(y.cpu(), want.cpu(), f"imported layer {layer} op {op} round")
        ids = torch.tensor([3, VOCAB - 1, 0], dtype=torch.int64, device="cuda:0")
        copy(s_in, ids.data_ptr(), 24)
        agg.execute_round(OP_EMBED, 0, [sid], [7], [1], [3])
        torch.cuda.synchronize()
        e = torch.empty(3, H, dtype=BF, device="cuda:0")
        copy(e.data_ptr(), s_out, e.numel() * 2)
        assert torch.equal(e, emb[ids]), "embed round on imported table"
        x = (lm[1234].float() * 50).to(BF).reshape(1, H)  # logit 1234 dominates by a wide margin
        copy(s_in, x.data_ptr(), H * 2)
        agg.execute_round(OP_LM_HEAD, 0, [sid], [7], [1], [1])
        torch.cuda.synchronize()
        tok = torch.empty(1, dtype=torch.int64, device="cuda:0")
        copy(tok.data_ptr(), s_out, 8)
        assert int(tok.item()) == int((x.float() @ lm.float().t()).argmax()) == 1234
        agg.release_slot(sid, 7)
        agg.cleanup_slot_pool()
        q_res.put(("ok", None))
    except Exception:
        q_res.put(("error", traceback.format_exc()))


def test_import_weights_from_a_donor_process(native, cuda):
    ctx = mp.get_context("spawn")
    q_out, q_done, q_res = ctx.Queue(), ctx.Queue(), ctx.Queue()
    donor = ctx.Process(target=_donor, args=(q_out, q_done))
    donor.start()
    receiver = None
    try:
        status, handles, digests = q_out.get(timeout=300)
        assert status == "ok", handles
        assert handles["num_layers"] == LAYERS and handles["dtype_code"] == 15
        assert handles["layers"][0]["o_weight_offset"] > 0  # borrowed views inside one allocation
        assert handles["layers"][0]["o_weight_handle"] == handles["embed_weight_handle"]
        receiver = ctx.Process(target=_receiver, args=(handles, digests, q_res))
        receiver.start()
        status, err = q_res.get(timeout=300)
        assert status == "ok", err
    finally:
        q_done.put(1)
        for p in (receiver, donor):
            if p is not None:
                p.join(timeout=120)
                if p.is_alive():
                    p.kill()
    assert donor.exitcode == 0 and receiver.exitcode == 0
