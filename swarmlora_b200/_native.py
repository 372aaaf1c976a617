"""ctypes binding to libswarmlora_b200.so, the C-ABI library.

Every entry point returns an int status (0 = ok); `check` turns a failure into
RuntimeError carrying the library's message, the same exception type the
reference's pybind modules raise. There is no Python fallback: if the library
is missing, importing any module of this package that needs it fails loudly.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libswarmlora_b200.so"

_i32, _i64, _u64, _f32 = C.c_int, C.c_int64, C.c_uint64, C.c_float
_p, _sz, _cp = C.c_void_p, C.c_size_t, C.c_char_p
_pi32 = C.POINTER(C.c_int)
_pi64 = C.POINTER(C.c_int64)
_pu64 = C.POINTER(C.c_uint64)
_psz = C.POINTER(C.c_size_t)
_pp = C.POINTER(C.c_void_p)
_pu32 = C.POINTER(C.c_uint)


class WeightIpc(C.Structure):
    """swl_weight_ipc: one weight of a donor export (allocation handle, byte
    offset in it, bf16 [rows, cols]; rows 0 = absent)."""
    _fields_ = [("handle", C.c_ubyte * 64), ("offset", C.c_uint64), ("rows", C.c_int64), ("cols", C.c_int64)]


_pwipc = C.POINTER(WeightIpc)


class Sampling(C.Structure):
    """swl_sampling: one row's sampling parameters."""
    _fields_ = [("do_sample", C.c_int), ("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float)]

# name -> (restype, argtypes). Kept in the same order as include/swarmlora_b200.h.
SIGNATURES: dict[str, tuple] = {
    "swl_last_error": (_cp, []),
    "swl_abi_version": (_i32, []),
    "swl_set_pdl": (_i32, [_i32]),
    # ---- ext_ipc_queue
    "swl_q_create": (_i32, [_i32, _i32, C.c_char_p, _i32]),
    "swl_q_open": (_i32, [_cp, _i32, _i32]),
    "swl_q_close": (_i32, []),
    "swl_q_init_batch_control": (_i32, [_i32]),
    "swl_q_set_quit": (_i32, [_i32]),
    "swl_q_slot_set_pending_sampling": (_i32, [_i32, _i32, _f32, _i32, _f32]),
    "swl_q_slot_signal_join": (_i32, [_i32]),
    "swl_q_slot_signal_leave": (_i32, [_i32]),
    "swl_q_slot_signal_ready": (_i32, [_i32]),
    "swl_q_wait_for_epoch": (_i32, [_i64, _i64, _pi64]),
    "swl_q_slot_is_active": (_i32, [_i32]),
    "swl_q_get_barrier_done_epoch": (_i64, []),
    "swl_q_is_slot_evicted": (_i32, [_i32]),
    "swl_q_clear_evicted_slot": (None, [_i32]),
    "swl_q_submit_slot_command": (_i32, [_i32, _i32, _i32, _i32, _i64, _i64, _i64,
                                         _u64, _u64, _u64, _u64, _i32]),
    "swl_q_control_block": (_p, []),
    "swl_q_capacity": (_i32, []),
    "swl_q_control_block_size": (_sz, []),
    "swl_q_command_size": (_sz, []),
    # ---- ext_aggregator
    "swl_agg_init_slot_pool": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _psz, _psz]),
    "swl_agg_claim_slot": (_i32, [_i32, _pi32, C.c_char_p, C.c_char_p, _psz, _psz]),
    "swl_agg_release_slot": (_i32, [_i32, _i32]),
    "swl_agg_get_slot_owner": (_i32, [_i32]),
    "swl_agg_get_slot_pool_status": (_i32, [_pi32, _pi32, _pu64, _pi32, _pi32]),
    "swl_agg_slot_buffers": (_i32, [_i32, _pp, _pp]),
    "swl_agg_cleanup_slot_pool": (_i32, []),
    "swl_agg_init_begin": (_i32, [_i32, _i32]),
    "swl_agg_init_layer": (_i32, [_i32, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _p,
                                  _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i64]),
    "swl_agg_init_finalize": (_i32, []),
    "swl_agg_init_embed_lm_head": (_i32, [_p, _p, _i64, _i64]),
    "swl_agg_init_queue": (_i32, [_cp, _i32]),
    "swl_agg_set_round_algo": (_i32, [_i32, _i32]),
    "swl_agg_set_worker_sampling": (_i32, [_i32, _i32, _f32, _i32, _f32]),
    "swl_agg_set_sampling_seed": (_i32, [_u64]),
    "swl_agg_weight": (_i32, [_i32, _i32, _pp, _pi64, _pi64]),
    "swl_agg_execute_round": (_i32, [_i32, _i32, _i32, _pi32, _pi32, _pi64, _pi64, _p]),
    "swl_agg_execute_qkv_rope_round": (_i32, [_i32, _i32, _pi32, _pi32, _pi64, _pi64, _pp, _i32, _p, _i32, _pp, _pp, _pp,
                                               _pp, _i32, _i32, _i32, _i32, _p, _p, _p]),
    "swl_agg_export_weights": (_i32, [_pwipc, _i32, _pi64, _pi32, _pi32]),
    "swl_agg_import_weights": (_i32, [_pwipc, _i32, _pi64, _i32, _i32]),
    "swl_agg_shard_begin": (_i32, [_i32, _i32]),
    "swl_agg_shard_handles": (_i32, [_p, _i32, _pi32]),
    "swl_agg_shard_connect": (_i32, [_p, _i32]),
    "swl_agg_shard_end": (_i32, []),
    "swl_agg_main_loop_slots": (_i32, [_i32, _i32]),
    "swl_agg_set_completion_mode": (_i32, [_i32]),
    "swl_agg_completion_mode": (_i32, []),
    "swl_agg_set_round_graphs": (_i32, [_i32]),
    "swl_agg_round_event_handle": (_i32, [C.c_char_p, _sz]),
    "swl_agg_round_event": (_i32, [C.POINTER(C.c_void_p)]),
    "swl_agg_set_slot_input_event": (_i32, [_i32, C.c_char_p, _sz]),
    "swl_agg_set_slot_input_event_local": (_i32, [_i32, _p]),
    # ---- ext_unified_barrier
    "swl_ub_init_worker_slot_manager": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "swl_ub_open_slot": (_i32, [_i32, C.c_char_p, _sz, C.c_char_p, _sz, _sz, _sz]),
    "swl_ub_attach_slot": (_i32, [_i32, _p, _p, _sz, _sz]),
    "swl_ub_close_slot": (_i32, [_i32]),
    "swl_ub_slot_buffers": (_i32, [_i32, _pp, _pp, _psz, _psz]),
    "swl_ub_prepare_input_slot": (_i32, [_i32, _i32, _p, _sz, _i64, _i64, _i64, _p]),
    "swl_ub_slot_shape": (_i32, [_i32, _pi64, _pi64, _pi64]),
    "swl_ub_get_outputs_slot": (_i32, [_i32, _p, _sz, _p]),
    "swl_ub_prepare_token_ids_slot": (_i32, [_i32, _p, _i64, _i64, _p]),
    "swl_ub_get_embeddings_slot": (_i32, [_i32, _p, _sz, _p]),
    "swl_ub_prepare_hidden_for_lm_head_slot": (_i32, [_i32, _p, _sz, _i64, _i64, _i64, _p]),
    "swl_ub_get_next_token_slot": (_i32, [_i32, _pi64, _p]),
    "swl_ub_cleanup_worker_slots": (_i32, []),
    # ---- kernels callable directly
    "swl_slot_gemm": (_i32, [_p, _i64, _i64, _p, _i32, _pp, _pp, _pi32, _i64, _i64, _i32, _i32, _p]),
    "swl_argmax_rows": (_i32, [_p, _i32, _i64, _i64, _p, _p]),
    "swl_sample_rows": (_i32, [_p, _i32, _i64, _i64, C.POINTER(Sampling), _p, _u64, _u64, _p, _p]),
    "swl_round_device_error": (_i32, [_pu32]),
    "swl_round_set_streamk_ctas_per_sm": (_i32, [_i32]),
    "swl_round_set_streamk_ctas": (_i32, [_i32]),
    "swl_round_tune": (_i32, [_i32, _i32, _i32, _i32]),
    # ---- worker kernels
    "swl_lora_shrink": (_i32, [_i32, _pi32, _pp, _i64, _pp, _i64, _i32, _i32, _p, _p]),
    "swl_lora_expand": (_i32, [_i32, _pi32, _pp, _i64, _pp, _pp, _i64, _pp, _i64, _i64, _i32,
                               _i32, _pi64, _f32, _i32, _i32, _p, _p]),
    "swl_rope_append": (_i32, [_i32, _pi32, _pp, _i64, _pp, _pp, _pp, _pp, _i32, _i32, _i32, _i32,
                               _p, _i32, _p, _p]),
    "swl_attention_part_floats": (_i64, [_i32, _i32, _i32, _i32]),
    "swl_attention_tune": (_i32, [_i32, _i32, _i32]),
    "swl_attention_pairing": (_i32, [_i32]),
    "swl_attention_tma": (_i32, [_i32]),
    "swl_paged_attention": (_i32, [_i32, _pi32, _pp, _pp, _pp, _pp, _pp, _i64, _i32, _i32, _i32,
                                   _i32, _f32, _i32, _p, _p, _p]),
    "swl_paged_attention_noalloc": (_i32, [_i32, _pi32, _pp, _pp, _pp, _pp, _pp, _i64, _i32, _i32,
                                           _i32, _i32, _f32, _i32, _p, _p]),
    "swl_noalloc_forget_device": (_i32, []),
    "swl_rms_norm": (_i32, [_i32, _pi32, _pp, _i64, _pp, _i64, _p, _i64, _f32, _p]),
    "swl_copy_rows": (_i32, [_i32, _pp, _pp, _pi64, _p]),
    "swl_paged_attention_shrink": (_i32, [_i32, _pi32, _pp, _pp, _pp, _pp, _pp, _i64, _i32, _i32, _i32,
                                          _i32, _f32, _i32, _p, _p, _pp, _i32, _p, _p, _i64, _p]),
    "swl_fused_qkv_rope": (_i32, [_i32, _pi32, _pp, _i64, _pp, _i32, _p, _i32, _pp, _pp, _pp, _pp,
                                  _i32, _i32, _i32, _i32, _p, _p, _p, _i64, _p]),
    "swl_fused_resid_norm_shrink": (_i32, [_i32, _pi32, _pp, _i64, _pp, _i32, _f32, _p, _i32, _i32,
                                           _pp, _i64, _p, _i64, _f32, _pp, _i64, _pp, _i32, _p, _p, _i64,
                                           _p]),
    "swl_fused_gu_silu_shrink": (_i32, [_i32, _pi32, _pp, _i64, _pp, _i32, _p, _i32, _i64, _pp, _i64,
                                        _pp, _i32, _p, _p, _i64, _p]),
    "swl_fused_norm_splits": (_i32, [_i32]),
    "swl_fused_silu_splits": (_i32, [_i64]),
    "swl_advance_i32": (_i32, [_p, _i32, _i32, _p]),
    "swl_wc_create": (_i32, [_i32, _pi32, _pi32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _f32,
                             _i32, C.POINTER(C.c_void_p)]),
    "swl_wc_set_buffers": (_i32, [_p, _pp, _pp, _pp, _pp, _pp, _pp, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "swl_wc_set_layer": (_i32, [_p, _i32, _p, _p, _pp, _pp, _pp, _pp, _pp, _pp, _pp, _pp, _pp, _pp]),
    "swl_wc_configure": (_i32, [_p, _i32, _i64, _p]),
    "swl_wc_run": (_i32, [_p, _i32, _pi64]),
    "swl_wc_rounds": (_i64, [_p]),
    "swl_wc_use_graphs": (_i32, [_p, _i32]),
    "swl_wc_destroy": (_i32, [_p]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads the library once (ctypes.CDLL releases the GIL around calls)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m swarmlora_b200.build` "
                "(there is no fallback implementation)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().swl_last_error()
    return msg.decode() if msg else "unknown error"


def check(status: int) -> None:
    if status != 0:
        raise RuntimeError(last_error())


def ptr_array(values) -> C.Array:
    arr = (C.c_void_p * max(1, len(values)))()
    for i, v in enumerate(values):
        arr[i] = v
    return arr


def i32_array(values) -> C.Array:
    arr = (C.c_int * max(1, len(values)))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr


def i64_array(values) -> C.Array:
    arr = (C.c_int64 * max(1, len(values)))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr
