"""Drop-in for the reference's `ext_aggregator` module
(src/cpp_extensions/ext_aggregator.cpp:1436-1517): slot pool, frozen base
weights and the blocking main loop of the per-GPU aggregator.

Same function names, argument names and return values; failures raise
RuntimeError. Weight tensors are bf16 CUDA tensors with HF nn.Linear layout
[out, in]; q|k|v and gate|up are fused into library-owned copies (so the
caller may free its originals, as src/aggregator.py:351-356 does), while
o / down / embed / lm_head are borrowed — this module keeps a reference so
they stay alive, as the reference's detach() does.

Additions (not in the reference): `execute_round` runs one round over pool
slots on a given stream, `slot_buffers` returns a slot's device addresses
for in-process drivers, `set_round_algo` selects the round kernel. The
donor weight transfer (`export_weight_ipc_handles` /
`import_weights_from_ipc`) carries each weight's offset inside its
allocation next to the reference's keys.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._native import WeightIpc, check, i32_array, i64_array, lib

OP_O_PROJ = 3
OP_DOWN_PROJ = 6
OP_QKV_FUSED = 9
OP_GATE_UP_FUSED = 10
OP_EMBED = 11
OP_LM_HEAD = 12
OP_SET_SAMPLING = 13
MAX_SLOTS = 128

_borrowed: dict = {}


def _bf16_cuda(t: torch.Tensor, what: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.bfloat16:
        raise RuntimeError(f"{what} must be a bf16 CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{what} must be contiguous")
    return t


def init_slot_pool(num_slots: int, device_index: int, hidden_dim: int, intermediate_dim: int,
                   num_kv_heads: int, head_dim: int, max_seq_per_step: int, dtype_size: int) -> dict:
    """ext_aggregator.cpp:138-187."""
    ib, ob = C.c_size_t(0), C.c_size_t(0)
    check(lib().swl_agg_init_slot_pool(int(num_slots), int(device_index), int(hidden_dim),
                                       int(intermediate_dim), int(num_kv_heads), int(head_dim),
                                       int(max_seq_per_step), int(dtype_size), C.byref(ib), C.byref(ob)))
    return {"num_slots": int(num_slots), "input_buffer_size": ib.value, "output_buffer_size": ob.value}


def claim_slot(worker_id: int) -> dict:
    """ext_aggregator.cpp:190-245."""
    sid = C.c_int(-1)
    hin, hout = C.create_string_buffer(64), C.create_string_buffer(64)
    ib, ob = C.c_size_t(0), C.c_size_t(0)
    check(lib().swl_agg_claim_slot(int(worker_id), C.byref(sid), hin, hout, C.byref(ib), C.byref(ob)))
    return {"slot_id": sid.value, "worker_id": int(worker_id), "input_handle": hin.raw,
            "output_handle": hout.raw, "input_buffer_size": ib.value, "output_buffer_size": ob.value}


def release_slot(slot_id: int, worker_id: int) -> None:
    """ext_aggregator.cpp:248-296."""
    check(lib().swl_agg_release_slot(int(slot_id), int(worker_id)))


def get_slot_owner(slot_id: int) -> int:
    return int(lib().swl_agg_get_slot_owner(int(slot_id)))


def get_slot_pool_status() -> dict:
    """ext_aggregator.cpp:307-328."""
    init, n, active = C.c_int(0), C.c_int(0), C.c_int(0)
    masks = (C.c_uint64 * 4)()
    owners = (C.c_int * MAX_SLOTS)()
    check(lib().swl_agg_get_slot_pool_status(C.byref(init), C.byref(n), masks, C.byref(active), owners))
    free_lo, free_hi, act_lo, act_hi = (int(m) for m in masks)
    return {
        "initialized": bool(init.value), "num_slots": n.value,
        "free_mask_lo": free_lo, "free_mask_hi": free_hi,
        "active_mask_lo": act_lo, "active_mask_hi": act_hi,
        "free_count": bin(free_lo).count("1") + bin(free_hi).count("1"),
        "active_count": bin(act_lo).count("1") + bin(act_hi).count("1"),
        "active_slot_count": active.value,
        "slot_owners": [int(owners[i]) for i in range(n.value)],
    }


def cleanup_slot_pool() -> None:
    check(lib().swl_agg_cleanup_slot_pool())


def init_aggregator_begin(num_layers: int, device_index: int) -> None:
    check(lib().swl_agg_init_begin(int(num_layers), int(device_index)))
    _borrowed.clear()


def init_aggregator_layer(layer_idx: int, q_weight, k_weight, v_weight, o_weight, o_bias,
                          gate_weight, up_weight, down_weight, down_bias) -> None:
    """ext_aggregator.cpp:347-376 (an empty bias tensor means no bias)."""
    q = _bf16_cuda(q_weight, "q_weight")
    k = _bf16_cuda(k_weight, "k_weight")
    v = _bf16_cuda(v_weight, "v_weight")
    o = _bf16_cuda(o_weight, "o_weight")
    g = _bf16_cuda(gate_weight, "gate_weight")
    u = _bf16_cuda(up_weight, "up_weight")
    d = _bf16_cuda(down_weight, "down_weight")
    ob = _bf16_cuda(o_bias, "o_bias") if o_bias is not None and o_bias.numel() > 0 else None
    db = _bf16_cuda(down_bias, "down_bias") if down_bias is not None and down_bias.numel() > 0 else None
    hidden, inter = int(q.shape[1]), int(d.shape[1])
    check(lib().swl_agg_init_layer(
        int(layer_idx), q.data_ptr(), q.shape[0], k.data_ptr(), k.shape[0], v.data_ptr(), v.shape[0],
        o.data_ptr(), o.shape[0], ob.data_ptr() if ob is not None else None,
        g.data_ptr(), g.shape[0], u.data_ptr(), u.shape[0], d.data_ptr(), d.shape[0],
        db.data_ptr() if db is not None else None, hidden, inter))
    _borrowed[("layer", int(layer_idx))] = (o, d, ob, db)


def init_aggregator_finalize() -> None:
    check(lib().swl_agg_init_finalize())


def init_embed_lm_head_weights(embed_weight, lm_head_weight) -> None:
    """ext_aggregator.cpp:413-424."""
    e = _bf16_cuda(embed_weight, "embed_weight")
    h = _bf16_cuda(lm_head_weight, "lm_head_weight")
    check(lib().swl_agg_init_embed_lm_head(e.data_ptr(), h.data_ptr(), int(e.shape[0]), int(e.shape[1])))
    _borrowed["embed_lm_head"] = (e, h)


def init_aggregator_queue(shm_name: str, capacity: int) -> None:
    check(lib().swl_agg_init_queue(shm_name.encode(), int(capacity)))


def aggregator_main_loop_slots(num_slots: int, dtype_code: int) -> None:
    """ext_aggregator.cpp:1024-1210. Blocks until the quit flag is set; the
    GIL is released for the duration (ctypes foreign call)."""
    check(lib().swl_agg_main_loop_slots(int(num_slots), int(dtype_code)))


# ---------------------------------------------------------------------------
# additions
# ---------------------------------------------------------------------------

_LAYER_WEIGHTS = ("qkv_weight", "o_weight", "gate_up_weight", "down_weight")
_LAYER_DIMS = ("q_dim", "k_dim", "v_dim", "gate_dim", "up_dim")
_DTYPE_BF16 = 15  # c10::ScalarType::BFloat16, the code the reference's export carries


def export_weight_ipc_handles() -> dict:
    """ext_aggregator.cpp:1216-1291: the reference's dict (handles as 64-byte
    bytes, shapes as tuples, bias flags, per-layer dims, dtype_code) plus a
    `*_offset` entry per handle: the weight's byte offset inside the
    exported allocation. Keep this process's weights alive until every
    importer has returned."""
    L, dev = C.c_int(0), C.c_int(0)
    check(lib().swl_agg_export_weights(None, 0, None, C.byref(L), C.byref(dev)))
    n = 6 * L.value + 2
    recs = (WeightIpc * n)()
    dims = (C.c_int64 * (5 * L.value))()
    check(lib().swl_agg_export_weights(recs, n, dims, C.byref(L), C.byref(dev)))

    def put(d, name, r, one_d=False):
        d[f"{name}_handle"] = bytes(r.handle)
        d[f"{name}_offset"] = int(r.offset)
        if one_d:
            d[f"{name}_size"] = int(r.rows)
        else:
            d[f"{name}_shape"] = (int(r.rows), int(r.cols))
    layers = []
    for l in range(L.value):
        r = recs[6 * l:6 * l + 6]
        lh = {}
        for name, rec in zip(_LAYER_WEIGHTS, r[:4]):
            put(lh, name, rec)
        for name, rec in (("o_bias", r[4]), ("down_bias", r[5])):
            lh[f"has_{name}"] = rec.rows > 0
            if rec.rows > 0:
                put(lh, name, rec, one_d=True)
        for j, k in enumerate(_LAYER_DIMS):
            lh[k] = int(dims[5 * l + j])
        layers.append(lh)
    out = {"num_layers": L.value, "device_index": dev.value, "layers": layers, "dtype_code": _DTYPE_BF16}
    put(out, "embed_weight", recs[6 * L.value])
    put(out, "lm_head_weight", recs[6 * L.value + 1])
    return out


def import_weights_from_ipc(handles_dict: dict, target_device_index: int) -> None:
    """ext_aggregator.cpp:1294-1406: copies a donor aggregator's weights
    (export_weight_ipc_handles of another process) onto this process's
    device; the aggregator is then as after init_aggregator_finalize and
    init_embed_lm_head_weights. A dict without `*_offset` entries (the
    reference's own export) reads each weight from its allocation's start."""
    if int(handles_dict.get("dtype_code", _DTYPE_BF16)) != _DTYPE_BF16:
        raise RuntimeError("import_weights_from_ipc: only bf16 weights are supported")
    L = int(handles_dict["num_layers"])
    layers = handles_dict["layers"]
    if len(layers) != L:
        raise RuntimeError(f"import_weights_from_ipc: {len(layers)} layer entries for num_layers={L}")
    n = 6 * L + 2
    recs = (WeightIpc * n)()
    dims = (C.c_int64 * (5 * L))()

    def get(r, d, name, one_d=False):
        h = bytes(d[f"{name}_handle"])
        if len(h) != 64:
            raise RuntimeError(f"import_weights_from_ipc: {name}_handle must be 64 bytes")
        C.memmove(r.handle, h, 64)
        r.offset = int(d.get(f"{name}_offset", 0))
        if one_d:
            r.rows, r.cols = int(d[f"{name}_size"]), 1
        else:
            r.rows, r.cols = (int(x) for x in d[f"{name}_shape"])
    for l, lh in enumerate(layers):
        for j, name in enumerate(_LAYER_WEIGHTS):
            get(recs[6 * l + j], lh, name)
        for j, name in ((4, "o_bias"), (5, "down_bias")):
            if lh.get(f"has_{name}"):
                get(recs[6 * l + j], lh, name, one_d=True)
        for j, k in enumerate(_LAYER_DIMS):
            dims[5 * l + j] = int(lh[k])
    get(recs[6 * L], handles_dict, "embed_weight")
    get(recs[6 * L + 1], handles_dict, "lm_head_weight")
    check(lib().swl_agg_import_weights(recs, n, dims, L, int(target_device_index)))
    _borrowed.clear()  # the imported weights are library-owned


def execute_round(op: int, layer: int, slot_ids, worker_ids, bx, tx, stream=None) -> None:
    """One round over pool slots (what the main loop runs per op), queued on
    `stream` (a torch.cuda.Stream; None = the default stream, waited for)."""
    n = len(slot_ids)
    st = stream.cuda_stream if stream is not None else None
    check(lib().swl_agg_execute_round(int(op), int(layer), n, i32_array(slot_ids), i32_array(worker_ids),
                                      i64_array(bx), i64_array(tx), st))


def shard_begin(rank: int, world: int = 2) -> None:
    """Column-sharded base weights over a pair of GPUs (one process each):
    builds this GPU's half of every fused weight (a row view). Call after the
    pool, the layers and the LM head are initialised."""
    check(lib().swl_agg_shard_begin(int(rank), int(world)))


def shard_handles() -> bytes:
    """IPC handles (64 bytes each) of this GPU's sync words, logits and slot
    outputs, for the peer's shard_connect."""
    n = C.c_int(0)
    lib().swl_agg_shard_handles(None, 0, C.byref(n))
    buf = (C.c_ubyte * (64 * n.value))()
    check(lib().swl_agg_shard_handles(buf, n.value, C.byref(n)))
    return bytes(buf)


def shard_connect(peer_handles: bytes) -> None:
    """Maps the peer's buffers; from here on every round is column-sharded
    and both GPUs must run the same rounds in the same order."""
    n = len(peer_handles) // 64
    buf = (C.c_ubyte * len(peer_handles)).from_buffer_copy(peer_handles)
    check(lib().swl_agg_shard_connect(buf, n))


def shard_end() -> None:
    """Unmaps the peer's buffers (on both GPUs before either frees its pool)."""
    check(lib().swl_agg_shard_end())


def slot_buffers(slot_id: int) -> tuple[int, int]:
    """Aggregator-local device addresses (input, output) of a pool slot."""
    a, b = C.c_void_p(), C.c_void_p()
    check(lib().swl_agg_slot_buffers(int(slot_id), C.byref(a), C.byref(b)))
    return int(a.value), int(b.value)


def set_worker_sampling(worker_id: int, do_sample: bool, temperature: float = 1.0, top_k: int = 0,
                        top_p: float = 1.0) -> None:
    """Sampling state of a worker for in-process drivers (the protocol sets it
    through OP_SET_SAMPLING or slot_set_pending_sampling): the LM-head round
    samples that worker's slot with it."""
    check(lib().swl_agg_set_worker_sampling(int(worker_id), int(bool(do_sample)), float(temperature),
                                            int(top_k), float(top_p)))


def set_sampling_seed(seed: int) -> None:
    """Seed of the LM-head sampling draws (their offset restarts at 0)."""
    check(lib().swl_agg_set_sampling_seed(int(seed)))


def set_round_algo(algo: int, splits: int = 0) -> None:
    """0/1: tensor-core round kernel (default); 2: CUDA-core cross-check kernel."""
    check(lib().swl_agg_set_round_algo(int(algo), int(splits)))
