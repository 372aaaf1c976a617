"""The shared-memory command ring and slot barrier (ext_ipc_queue drop-in,
src/cpp_extensions/ext_ipc_queue.cpp:111-410) on CPU: segment layout, command
encoding, validation, ring-full behaviour, the join/leave/ready/sampling
signals, bounded and quit-aborted epoch waits, and a second process (spawned)
writing into the same segment."""
import ctypes as C
import multiprocessing as mp

import pytest

from swarmlora_b200 import ext_ipc_queue as extq
from swarmlora_b200._native import lib


class Mask(C.Structure):
    _fields_ = [("w", C.c_uint64 * 2)]

    def bits(self):
        return [i for i in range(128) if (self.w[i >> 6] >> (i & 63)) & 1]


class Sampling(C.Structure):
    _fields_ = [("do_sample", C.c_bool), ("temperature", C.c_float), ("top_k", C.c_int),
                ("top_p", C.c_float)]


class ControlBlockHead(C.Structure):
    """Leading fields of ControlBlock (ipc_types.h:160-217 layout)."""
    _fields_ = [("head", C.c_int), ("tail", C.c_int), ("capacity", C.c_int), ("quit_flag", C.c_int),
                ("num_workers", C.c_int), ("num_slots", C.c_int), ("unused_free_mask", Mask),
                ("active_slot_mask", Mask), ("pending_slot_joins", Mask), ("pending_slot_leaves", Mask),
                ("per_slot_ready_mask", Mask), ("evicted_slot_mask", Mask), ("active_slot_count", C.c_int),
                ("slot_ready_count", C.c_int), ("barrier_done_epoch", C.c_int64),
                ("pending_sampling_mask", Mask), ("pending_sampling", Sampling * 128)]


class Command(C.Structure):
    _fields_ = [("ready", C.c_int), ("op_type", C.c_int), ("layer_idx", C.c_int), ("slot_id", C.c_int),
                ("worker_id", C.c_int), ("bx", C.c_int64), ("tx", C.c_int64), ("dx", C.c_int64),
                ("x_key", C.c_uint64), ("y0_key", C.c_uint64), ("y1_key", C.c_uint64), ("y2_key", C.c_uint64),
                ("ticket_id", C.c_int)]


def _views():
    base = lib().swl_q_control_block()
    cb = ControlBlockHead.from_address(base)
    cb_size = lib().swl_q_control_block_size()
    ring = (Command * cb.capacity).from_address(base + cb_size)
    return cb, ring


@pytest.fixture
def queue():
    info = extq.create_queue(8, 16)
    extq.init_batch_control(4)
    yield info
    extq.close_queue()


def test_layout_sizes(native):
    assert lib().swl_q_command_size() == 128  # alignas(64) around 88 bytes of fields
    assert lib().swl_q_control_block_size() % 64 == 0
    assert C.sizeof(Command) <= 128


def test_submit_encodes_command_and_advances_head(native, queue):
    assert queue["shm_name"].startswith("/")
    cb, ring = _views()
    assert cb.capacity == 8 and cb.num_slots == 4 and cb.head == 0 and cb.tail == 0
    extq.submit_slot_command(9, 3, 2, 1001, 1, 5, 4096, 11, 12, 13, 14, 7)
    c = ring[0]
    assert (c.ready, c.op_type, c.layer_idx, c.slot_id, c.worker_id) == (1, 9, 3, 2, 1001)
    assert (c.bx, c.tx, c.dx, c.x_key, c.y0_key, c.y1_key, c.y2_key, c.ticket_id) == (1, 5, 4096, 11, 12, 13, 14, 7)
    assert cb.head == 1


def test_submit_validates_before_reserving(native, queue):
    cb, _ = _views()
    for bad in [dict(slot_id=200), dict(slot_id=-1), dict(worker_id=-5), dict(bx=0), dict(tx=70000)]:
        args = dict(op_type=9, layer_idx=0, slot_id=0, worker_id=1, bx=1, tx=1, dx=8, x_key=0, y0_key=0,
                    y1_key=0, y2_key=0, ticket_id=0)
        args.update(bad)
        with pytest.raises(RuntimeError):
            extq.submit_slot_command(**args)
    assert cb.head == 0  # nothing reserved


def test_ring_full(native, queue):
    for i in range(7):  # capacity 8 keeps one entry free
        extq.submit_slot_command(3, 0, i % 4, 1, 1, 1, 8, 0, 0, 0, 0, i)
    with pytest.raises(RuntimeError, match="FULL"):
        extq.submit_slot_command(3, 0, 0, 1, 1, 1, 8, 0, 0, 0, 0, 99)


def test_slot_signals_and_sampling(native, queue):
    cb, _ = _views()
    extq.slot_set_pending_sampling(1, True, 0.7, 50, 0.9)
    extq.slot_signal_join(1)
    extq.slot_signal_join(3)
    extq.slot_signal_leave(2)
    extq.slot_signal_ready(3)
    assert cb.pending_slot_joins.bits() == [1, 3]
    assert cb.pending_slot_leaves.bits() == [2]
    assert cb.per_slot_ready_mask.bits() == [3]
    assert cb.pending_sampling_mask.bits() == [1]
    s = cb.pending_sampling[1]
    assert s.do_sample and abs(s.temperature - 0.7) < 1e-6 and s.top_k == 50 and abs(s.top_p - 0.9) < 1e-6
    assert not extq.slot_is_active(1)  # only the aggregator applies joins
    cb.active_slot_mask.w[0] = 0b1010
    assert extq.slot_is_active(1) and extq.slot_is_active(3) and not extq.slot_is_active(0)
    for bad in (-1, 128, 500):  # the range is MAX_SLOTS, as in the reference
        with pytest.raises(RuntimeError):
            extq.slot_signal_ready(bad)


def test_eviction_flags(native, queue):
    cb, _ = _views()
    assert not extq.is_slot_evicted(2)
    cb.evicted_slot_mask.w[0] = 1 << 2
    assert extq.is_slot_evicted(2)
    extq.clear_evicted_slot(2)
    assert not extq.is_slot_evicted(2)


def test_wait_for_epoch_bounded_moved_and_quit(native, queue):
    cb, _ = _views()
    e0 = extq.get_barrier_done_epoch()
    with pytest.raises(RuntimeError, match="stayed at"):
        extq.wait_for_epoch(e0, timeout_ms=50)
    cb.barrier_done_epoch = e0 + 1  # what the aggregator's signal_done does
    assert extq.wait_for_epoch(e0, timeout_ms=50) == e0 + 1
    extq.set_quit(1)
    with pytest.raises(RuntimeError, match="quit"):
        extq.wait_for_epoch(e0 + 1, timeout_ms=5000)


def _worker(shm_name, capacity, slot, wid, q):
    from swarmlora_b200 import ext_ipc_queue as wq
    try:
        wq.open_queue(shm_name, capacity, 16)
        wq.slot_signal_join(slot)
        wq.submit_slot_command(10, 5, slot, wid, 1, 2, 4096, 0, 0, 0, 0, 42)
        wq.slot_signal_ready(slot)
        wq.close_queue()
        q.put("ok")
    except Exception as e:  # report into the parent's assertion
        q.put(repr(e))


def test_second_process_writes_same_segment(native, queue):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_worker, args=(queue["shm_name"], 8, 2, 1002, q))
    p.start()
    assert q.get(timeout=120) == "ok"
    p.join(timeout=60)
    assert p.exitcode == 0
    cb, ring = _views()
    assert cb.head == 1
    c = ring[0]
    assert (c.ready, c.op_type, c.layer_idx, c.slot_id, c.worker_id, c.tx, c.ticket_id) == (1, 10, 5, 2, 1002, 2, 42)
    assert cb.pending_slot_joins.bits() == [2]
    assert cb.per_slot_ready_mask.bits() == [2]
