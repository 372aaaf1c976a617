"""swarmlora_b200: a B200-native (sm_100a) implementation of SwarmLoRA's
aggregator hot path behind the reference's slot-pool API.

Modules mirroring the reference's native extensions (same function names,
argument names and error behaviour):
  * swarmlora_b200.ext_ipc_queue       <- src/cpp_extensions/ext_ipc_queue.cpp
  * swarmlora_b200.ext_aggregator      <- src/cpp_extensions/ext_aggregator.cpp
  * swarmlora_b200.ext_unified_barrier <- src/cpp_extensions/ext_unified_barrier.cpp
Worker-side kernels (LoRA delta, paged decode attention, norms) live in
swarmlora_b200.worker_ops. All compute goes through libswarmlora_b200.so.
"""
from ._native import LIB_PATH, lib  # noqa: F401

OP_O_PROJ = 3
OP_DOWN_PROJ = 6
OP_QKV_FUSED = 9
OP_GATE_UP_FUSED = 10
OP_EMBED = 11
OP_LM_HEAD = 12
OP_SET_SAMPLING = 13
MAX_SLOTS = 128


def set_pdl(on: bool) -> bool:
    """Programmatic dependent launch for the library's later kernel launches
    (on by default); returns the previous setting."""
    return bool(lib().swl_set_pdl(1 if on else 0))
