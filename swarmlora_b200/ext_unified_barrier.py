"""Drop-in for the reference's `ext_unified_barrier` module
(src/cpp_extensions/ext_unified_barrier.cpp:562-630): the worker's view of its
aggregator slot buffers, mapped through CUDA IPC.

Same function names, argument names and return values; failures raise
RuntimeError. Copies go on the caller's current torch stream; the prepare_*
calls wait for their copy (the aggregator reads the slot from another process
once the ready bit is set), the get_* calls do not (same-stream ordering).

Additions: `attach_slot` (in-process workers, where CUDA IPC cannot map the
process's own allocations) and `slot_buffers` (device addresses for fused
kernels that read the slot output in place).
"""
from __future__ import annotations

import ctypes as C

import torch

from ._native import check, lib

OP_O_PROJ = 3
OP_DOWN_PROJ = 6
OP_QKV_FUSED = 9
OP_GATE_UP_FUSED = 10
OP_EMBED = 11
OP_LM_HEAD = 12
OP_SET_SAMPLING = 13

_state = {"device": 0, "hidden": 0}


def _stream():
    return torch.cuda.current_stream(_state["device"]).cuda_stream


def init_worker_slot_manager(worker_id: int, worker_device: int, aggregator_device: int,
                             hidden_dim: int, intermediate_dim: int, qkv_dim: int) -> None:
    check(lib().swl_ub_init_worker_slot_manager(int(worker_id), int(worker_device),
                                                int(aggregator_device), int(hidden_dim),
                                                int(intermediate_dim), int(qkv_dim)))
    _state["device"] = int(worker_device)
    _state["hidden"] = int(hidden_dim)


def open_slot(slot_id: int, input_handle: bytes, output_handle: bytes, input_buffer_size: int,
              output_buffer_size: int) -> None:
    """ext_unified_barrier.cpp:97-160 (handles must be 64-byte cudaIpcMemHandle_t)."""
    check(lib().swl_ub_open_slot(int(slot_id), bytes(input_handle), len(input_handle),
                                 bytes(output_handle), len(output_handle),
                                 int(input_buffer_size), int(output_buffer_size)))


def attach_slot(slot_id: int, input_ptr: int, output_ptr: int, input_buffer_size: int,
                output_buffer_size: int) -> None:
    check(lib().swl_ub_attach_slot(int(slot_id), int(input_ptr), int(output_ptr),
                                   int(input_buffer_size), int(output_buffer_size)))


def close_slot(slot_id: int) -> None:
    check(lib().swl_ub_close_slot(int(slot_id)))


def slot_buffers(slot_id: int) -> tuple[int, int, int, int]:
    a, b = C.c_void_p(), C.c_void_p()
    ia, ib = C.c_size_t(0), C.c_size_t(0)
    check(lib().swl_ub_slot_buffers(int(slot_id), C.byref(a), C.byref(b), C.byref(ia), C.byref(ib)))
    return int(a.value), int(b.value), ia.value, ib.value


def prepare_input_slot(slot_id: int, op_type: int, input: torch.Tensor) -> None:
    """ext_unified_barrier.cpp:225-273: input must be 3-D [B, T, D]."""
    if input.dim() != 3:
        raise RuntimeError("Input must be 3D [B, T, D]")
    x = input.contiguous()
    b, t, d = x.shape
    check(lib().swl_ub_prepare_input_slot(int(slot_id), int(op_type), x.data_ptr(),
                                          x.numel() * x.element_size(), b, t, d, _stream()))


def _shape(slot_id: int):
    b, t, d = C.c_int64(), C.c_int64(), C.c_int64()
    check(lib().swl_ub_slot_shape(int(slot_id), C.byref(b), C.byref(t), C.byref(d)))
    return b.value, t.value, d.value


def get_outputs_slot(slot_id: int, out_dims, input_template: torch.Tensor) -> list:
    """ext_unified_barrier.cpp:276-347: [B, T, sum(out_dims)] split on the last dim."""
    b, t, _ = _shape(slot_id)
    total = int(sum(out_dims))
    out = torch.empty((b, t, total), dtype=input_template.dtype, device=input_template.device)
    check(lib().swl_ub_get_outputs_slot(int(slot_id), out.data_ptr(),
                                        out.numel() * out.element_size(), _stream()))
    if len(out_dims) > 1:
        return list(out.split([int(d) for d in out_dims], -1))
    return [out]


def prepare_token_ids_slot(slot_id: int, token_ids: torch.Tensor) -> None:
    """ext_unified_barrier.cpp:350-393: token_ids [B, T] int64."""
    if token_ids.dim() != 2:
        raise RuntimeError("token_ids must be 2D [B, T]")
    ids = token_ids.to(torch.int64).contiguous()
    check(lib().swl_ub_prepare_token_ids_slot(int(slot_id), ids.data_ptr(), ids.shape[0],
                                              ids.shape[1], _stream()))


def get_embeddings_slot(slot_id: int, dtype: torch.dtype) -> torch.Tensor:
    """ext_unified_barrier.cpp:396-440."""
    b, t, _ = _shape(slot_id)
    emb = torch.empty((b, t, _state["hidden"]), dtype=dtype, device=f"cuda:{_state['device']}")
    check(lib().swl_ub_get_embeddings_slot(int(slot_id), emb.data_ptr(), emb.element_size(), _stream()))
    return emb


def prepare_hidden_for_lm_head_slot(slot_id: int, hidden_states: torch.Tensor) -> None:
    """ext_unified_barrier.cpp:443-486."""
    if hidden_states.dim() != 3:
        raise RuntimeError("hidden_states must be 3D [B, T, D]")
    h = hidden_states.contiguous()
    b, t, d = h.shape
    check(lib().swl_ub_prepare_hidden_for_lm_head_slot(int(slot_id), h.data_ptr(),
                                                       h.numel() * h.element_size(), b, t, d,
                                                       _stream()))


def get_next_token_slot(slot_id: int) -> int:
    """ext_unified_barrier.cpp:489-518."""
    tok = C.c_int64(0)
    check(lib().swl_ub_get_next_token_slot(int(slot_id), C.byref(tok), _stream()))
    return int(tok.value)


def cleanup_worker_slots() -> None:
    check(lib().swl_ub_cleanup_worker_slots())
