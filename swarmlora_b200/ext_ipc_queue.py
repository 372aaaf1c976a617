"""Drop-in for the reference's `ext_ipc_queue` module
(src/cpp_extensions/ext_ipc_queue.cpp:413-483): the shared-memory command ring
and slot barrier used by both the aggregator and every worker process.

Same function names, argument names and return values; failures raise
RuntimeError with the library's message. One queue is mapped per process.
"""
from __future__ import annotations

import ctypes as C

from ._native import check, lib


def create_queue(capacity: int, max_tickets: int) -> dict:
    """ext_ipc_queue.cpp:111-145: create and map a new segment."""
    buf = C.create_string_buffer(128)
    check(lib().swl_q_create(int(capacity), int(max_tickets), buf, 128))
    return {"shm_name": buf.value.decode(), "capacity": int(capacity), "max_tickets": int(max_tickets)}


def open_queue(shm_name: str, capacity: int, max_tickets: int) -> dict:
    """ext_ipc_queue.cpp:147-176: map an existing segment."""
    check(lib().swl_q_open(shm_name.encode(), int(capacity), int(max_tickets)))
    return {"capacity": int(capacity), "max_tickets": int(max_tickets)}


def close_queue() -> None:
    """Unmaps this process's view (unlinks the segment if this process created it)."""
    check(lib().swl_q_close())


def init_batch_control(num_slots: int) -> None:
    check(lib().swl_q_init_batch_control(int(num_slots)))


def set_quit(value: int) -> None:
    check(lib().swl_q_set_quit(int(value)))


def slot_set_pending_sampling(slot_id: int, do_sample: bool, temperature: float, top_k: int,
                              top_p: float) -> None:
    check(lib().swl_q_slot_set_pending_sampling(int(slot_id), int(bool(do_sample)), float(temperature),
                                                int(top_k), float(top_p)))


def slot_signal_join(slot_id: int) -> None:
    check(lib().swl_q_slot_signal_join(int(slot_id)))


def slot_signal_leave(slot_id: int) -> None:
    check(lib().swl_q_slot_signal_leave(int(slot_id)))


def slot_signal_ready(slot_id: int) -> None:
    check(lib().swl_q_slot_signal_ready(int(slot_id)))


def wait_for_epoch(expected_epoch: int, timeout_ms: int = 0) -> int:
    """ext_ipc_queue.cpp:272-300. Capture expected_epoch BEFORE slot_signal_ready().

    timeout_ms (not in the reference) bounds the wait; 0 waits until the epoch
    moves or the quit flag is set, as the reference does.
    """
    out = C.c_int64(0)
    check(lib().swl_q_wait_for_epoch(int(expected_epoch), int(timeout_ms), C.byref(out)))
    return int(out.value)


def slot_is_active(slot_id: int) -> bool:
    return bool(lib().swl_q_slot_is_active(int(slot_id)))


def get_barrier_done_epoch() -> int:
    return int(lib().swl_q_get_barrier_done_epoch())


def is_slot_evicted(slot_id: int) -> bool:
    return bool(lib().swl_q_is_slot_evicted(int(slot_id)))


def clear_evicted_slot(slot_id: int) -> None:
    lib().swl_q_clear_evicted_slot(int(slot_id))


def submit_slot_command(op_type: int, layer_idx: int, slot_id: int, worker_id: int, bx: int,
                        tx: int, dx: int, x_key: int, y0_key: int, y1_key: int, y2_key: int,
                        ticket_id: int) -> None:
    check(lib().swl_q_submit_slot_command(int(op_type), int(layer_idx), int(slot_id), int(worker_id),
                                          int(bx), int(tx), int(dx), int(x_key), int(y0_key),
                                          int(y1_key), int(y2_key), int(ticket_id)))
