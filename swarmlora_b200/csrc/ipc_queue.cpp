// Worker <-> aggregator lock-step protocol over POSIX shared memory: the
// command ring, the join / leave / ready slot masks and the epoch barrier.
// Host-only code (no CUDA). Behaviour follows the reference's ext_ipc_queue
// module (src/cpp_extensions/ext_ipc_queue.cpp); each entry point cites the
// function it replaces.
//
// One queue is mapped per process (module-level state), exactly as in the
// reference, so the aggregator calls create, every worker calls open.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <chrono>
#include <cstring>
#include <thread>

#include "common.h"
#include "shm_abi.h"

using namespace swl;

namespace {

struct QueueState {
  void* base = nullptr;
  size_t bytes = 0;
  char name[128] = {0};
  bool owner = false;  // created (and will unlink) the segment
  ControlBlock* ctrl = nullptr;
  Command* ring = nullptr;
  int capacity = 0;
};
QueueState g_q;

int map_segment(const char* name, int capacity, bool create) {
  size_t bytes = shm_bytes(capacity);
  int fd = create ? shm_open(name, O_CREAT | O_EXCL | O_RDWR, 0600)
                  : shm_open(name, O_RDWR, 0600);
  if (fd < 0) {
    return set_error(SWL_ERR_SYS, "shm_open (%s) failed for %s", create ? "create" : "open", name);
  }
  if (create && ftruncate(fd, static_cast<off_t>(bytes)) != 0) {
    close(fd);
    shm_unlink(name);
    return set_error(SWL_ERR_SYS, "ftruncate failed for shm %s", name);
  }
  if (!create) {
    struct stat st;
    if (fstat(fd, &st) != 0 || static_cast<size_t>(st.st_size) < bytes) {
      close(fd);
      return set_error(SWL_ERR_ARG, "shm %s is smaller than capacity %d needs", name, capacity);
    }
  }
  void* base = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (base == MAP_FAILED) {
    if (create) shm_unlink(name);
    return set_error(SWL_ERR_SYS, "mmap failed for shm %s", name);
  }
  if (g_q.base) munmap(g_q.base, g_q.bytes);
  g_q.base = base;
  g_q.bytes = bytes;
  snprintf(g_q.name, sizeof(g_q.name), "%s", name);
  g_q.owner = create;
  g_q.ctrl = static_cast<ControlBlock*>(base);
  g_q.ring = reinterpret_cast<Command*>(static_cast<char*>(base) + sizeof(ControlBlock));
  g_q.capacity = capacity;
  return SWL_OK;
}

inline bool valid_slot(int s) { return s >= 0 && s < kMaxSlots; }

}  // namespace

// ext_ipc_queue.cpp:111-145 create_queue. Writes the generated segment name
// ("/gpuqueue_<pid>_<ns>") into name_out.
SWL_EXPORT int swl_q_create(int capacity, int max_tickets, char* name_out, int name_cap) {
  if (capacity <= 0) return set_error(SWL_ERR_ARG, "capacity must be > 0");
  if (max_tickets <= 0) return set_error(SWL_ERR_ARG, "max_tickets must be > 0");
  char name[128];
  long long ns = std::chrono::duration_cast<std::chrono::nanoseconds>(
                     std::chrono::steady_clock::now().time_since_epoch())
                     .count();
  snprintf(name, sizeof(name), "/gpuqueue_%d_%lld", static_cast<int>(getpid()), ns);
  SWL_TRY(map_segment(name, capacity, true));
  std::memset(g_q.base, 0, g_q.bytes);
  ControlBlock* c = g_q.ctrl;
  c->head.store(0, std::memory_order_relaxed);
  c->tail.store(0, std::memory_order_relaxed);
  c->capacity = capacity;
  c->quit_flag.store(0, std::memory_order_relaxed);
  c->num_workers = 0;
  std::atomic_thread_fence(std::memory_order_release);
  if (name_out && name_cap > 0) snprintf(name_out, name_cap, "%s", name);
  return SWL_OK;
}

// ext_ipc_queue.cpp:147-176 open_queue.
SWL_EXPORT int swl_q_open(const char* name, int capacity, int max_tickets) {
  if (capacity <= 0) return set_error(SWL_ERR_ARG, "capacity must be > 0");
  if (max_tickets <= 0) return set_error(SWL_ERR_ARG, "max_tickets must be > 0");
  if (!name || !name[0]) return set_error(SWL_ERR_ARG, "shm_name cannot be empty");
  return map_segment(name, capacity, false);
}

// Unmaps this process's view (and unlinks the segment when this process
// created it). Not in the reference, which leaks the mapping until exit.
SWL_EXPORT int swl_q_close(void) {
  if (!g_q.base) return SWL_OK;
  munmap(g_q.base, g_q.bytes);
  if (g_q.owner) shm_unlink(g_q.name);
  g_q = QueueState();
  return SWL_OK;
}

// ext_ipc_queue.cpp:180-209 init_batch_control.
SWL_EXPORT int swl_q_init_batch_control(int num_slots) {
  if (!g_q.ctrl) return set_error(SWL_ERR_STATE, "init_batch_control: queue not initialized");
  if (num_slots <= 0 || num_slots > kMaxSlots)
    return set_error(SWL_ERR_ARG, "init_batch_control: num_slots must be between 1 and %d", kMaxSlots);
  ControlBlock* c = g_q.ctrl;
  c->num_workers = num_slots;
  c->num_slots = num_slots;
  Mask128 zero;
  c->unused_free_mask.store(zero, std::memory_order_relaxed);
  c->active_slot_mask.store(zero, std::memory_order_relaxed);
  c->pending_slot_joins.store(zero, std::memory_order_relaxed);
  c->pending_slot_leaves.store(zero, std::memory_order_relaxed);
  c->per_slot_ready_mask.store(zero, std::memory_order_relaxed);
  c->evicted_slot_mask.store(zero, std::memory_order_relaxed);
  c->active_slot_count.store(0, std::memory_order_relaxed);
  c->slot_ready_count.store(0, std::memory_order_relaxed);
  c->barrier_done_epoch.store(0, std::memory_order_relaxed);
  c->pending_sampling_mask.store(zero, std::memory_order_release);
  return SWL_OK;
}

// ext_ipc_queue.cpp:404-410 set_quit.
SWL_EXPORT int swl_q_set_quit(int value) {
  if (!g_q.ctrl) return set_error(SWL_ERR_STATE, "set_quit: queue not initialized");
  g_q.ctrl->quit_flag.store(value, std::memory_order_release);
  return SWL_OK;
}

// ext_ipc_queue.cpp:217-233 slot_set_pending_sampling.
SWL_EXPORT int swl_q_slot_set_pending_sampling(int slot_id, int do_sample, float temperature,
                                               int top_k, float top_p) {
  if (!g_q.ctrl) return set_error(SWL_ERR_STATE, "slot_set_pending_sampling: queue not initialized");
  if (!valid_slot(slot_id))
    return set_error(SWL_ERR_ARG, "slot_set_pending_sampling: slot_id out of range (0-%d)", kMaxSlots - 1);
  PendingSampling& p = g_q.ctrl->pending_sampling[slot_id];
  p.do_sample = do_sample != 0;
  p.temperature = temperature;
  p.top_k = top_k;
  p.top_p = top_p;
  g_q.ctrl->pending_sampling_mask.set_bit(slot_id);
  return SWL_OK;
}

// ext_ipc_queue.cpp:235-243 slot_signal_join.
SWL_EXPORT int swl_q_slot_signal_join(int slot_id) {
  if (!g_q.ctrl) return set_error(SWL_ERR_STATE, "slot_signal_join: queue not initialized");
  if (!valid_slot(slot_id))
    return set_error(SWL_ERR_ARG, "slot_signal_join: slot_id out of range (0-%d)", kMaxSlots - 1);
  g_q.ctrl->pending_slot_joins.set_bit(slot_id);
  return SWL_OK;
}

// ext_ipc_queue.cpp:246-254 slot_signal_leave.
SWL_EXPORT int swl_q_slot_signal_leave(int slot_id) {
  if (!g_q.ctrl) return set_error(SWL_ERR_STATE, "slot_signal_leave: queue not initialized");
  if (!valid_slot(slot_id))
    return set_error(SWL_ERR_ARG, "slot_signal_leave: slot_id out of range (0-%d)", kMaxSlots - 1);
  g_q.ctrl->pending_slot_leaves.set_bit(slot_id);
  return SWL_OK;
}

// ext_ipc_queue.cpp:257-268 slot_signal_ready.
SWL_EXPORT int swl_q_slot_signal_ready(int slot_id) {
  if (!g_q.ctrl) return set_error(SWL_ERR_STATE, "slot_signal_ready: queue not initialized");
  if (!valid_slot(slot_id))
    return set_error(SWL_ERR_ARG, "slot_signal_ready: slot_id out of range (0-%d)", kMaxSlots - 1);
  g_q.ctrl->per_slot_ready_mask.set_bit(slot_id);
  g_q.ctrl->slot_ready_count.fetch_add(1, std::memory_order_release);
  return SWL_OK;
}

// ext_ipc_queue.cpp:272-300 wait_for_epoch: returns once barrier_done_epoch
// exceeds `expected` (capture `expected` BEFORE signalling ready). Spins,
// then pauses, then yields, then sleeps 10 us per poll. timeout_ms <= 0 waits
// until the epoch moves or the quit flag is raised, like the reference.
SWL_EXPORT int swl_q_wait_for_epoch(int64_t expected, int64_t timeout_ms, int64_t* epoch_out) {
  if (!g_q.ctrl) return set_error(SWL_ERR_STATE, "wait_for_epoch: queue not initialized");
  ControlBlock* c = g_q.ctrl;
  auto t0 = std::chrono::steady_clock::now();
  long spins = 0;
  int64_t e;
  while ((e = c->barrier_done_epoch.load(std::memory_order_acquire)) <= expected) {
    if (c->quit_flag.load(std::memory_order_acquire) != 0)
      return set_error(SWL_ERR_QUIT, "wait_for_epoch: quit flag set");
    ++spins;
    if (spins < kSpinTight) {
    } else if (spins < kSpinPause) {
      cpu_relax();
    } else if (spins < kSpinYield) {
      std::this_thread::yield();
    } else {
      std::this_thread::sleep_for(std::chrono::microseconds(10));
      if (timeout_ms > 0 && (spins & 63) == 0 &&
          std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
        return set_error(SWL_ERR_TIMEOUT, "wait_for_epoch: epoch stayed at %lld for %lld ms",
                         static_cast<long long>(e), static_cast<long long>(timeout_ms));
    }
  }
  if (epoch_out) *epoch_out = e;
  return SWL_OK;
}

// ext_ipc_queue.cpp:303-311 slot_is_active (0/1; invalid ids read as 0).
SWL_EXPORT int swl_q_slot_is_active(int slot_id) {
  if (!g_q.ctrl || !valid_slot(slot_id)) return 0;
  return g_q.ctrl->active_slot_mask.test(slot_id) ? 1 : 0;
}

// ext_ipc_queue.cpp:314-319 get_barrier_done_epoch.
SWL_EXPORT int64_t swl_q_get_barrier_done_epoch(void) {
  if (!g_q.ctrl) return 0;
  return g_q.ctrl->barrier_done_epoch.load(std::memory_order_acquire);
}

// ext_ipc_queue.cpp:322-327 is_slot_evicted.
SWL_EXPORT int swl_q_is_slot_evicted(int slot_id) {
  if (!g_q.ctrl || !valid_slot(slot_id)) return 0;
  return g_q.ctrl->evicted_slot_mask.test(slot_id) ? 1 : 0;
}

// ext_ipc_queue.cpp:330-336 clear_evicted_slot.
SWL_EXPORT void swl_q_clear_evicted_slot(int slot_id) {
  if (!g_q.ctrl || !valid_slot(slot_id)) return;
  g_q.ctrl->evicted_slot_mask.clear_bit(slot_id);
}

// ext_ipc_queue.cpp:339-402 submit_slot_command. Every field is validated
// before a ring entry is reserved, so a rejected command never leaves a
// reserved-but-unwritten entry for the aggregator to stall on.
SWL_EXPORT int swl_q_submit_slot_command(int op_type, int layer_idx, int slot_id, int worker_id,
                                         int64_t bx, int64_t tx, int64_t dx, uint64_t x_key,
                                         uint64_t y0_key, uint64_t y1_key, uint64_t y2_key,
                                         int ticket_id) {
  if (!g_q.ctrl || !g_q.ring) return set_error(SWL_ERR_STATE, "submit_slot_command: queue not initialized");
  if (!valid_slot(slot_id))
    return set_error(SWL_ERR_ARG, "submit_slot_command: slot_id out of range: %d", slot_id);
  if (worker_id < 0 || worker_id > 100000)
    return set_error(SWL_ERR_ARG, "submit_slot_command: invalid worker_id: %d", worker_id);
  if (bx <= 0 || tx <= 0 || bx > 65536 || tx > 65536)
    return set_error(SWL_ERR_ARG, "submit_slot_command: invalid bx/tx: bx=%lld tx=%lld",
                     static_cast<long long>(bx), static_cast<long long>(tx));
  ControlBlock* c = g_q.ctrl;
  int head, next;
  do {
    head = c->head.load(std::memory_order_acquire);
    next = (head + 1) % g_q.capacity;
    if (next == c->tail.load(std::memory_order_acquire))
      return set_error(SWL_ERR_FULL, "command ring buffer FULL");
  } while (!c->head.compare_exchange_weak(head, next, std::memory_order_acq_rel,
                                          std::memory_order_acquire));
  Command& cmd = g_q.ring[head];
  cmd.op_type = op_type;
  cmd.layer_idx = layer_idx;
  cmd.slot_id = slot_id;
  cmd.worker_id = worker_id;
  cmd.bx = bx;
  cmd.tx = tx;
  cmd.dx = dx;
  cmd.x_key = x_key;
  cmd.y0_key = y0_key;
  cmd.y1_key = y1_key;
  cmd.y2_key = y2_key;
  cmd.ticket_id = ticket_id;
  cmd.ready.store(1, std::memory_order_release);
  return SWL_OK;
}

// Read-only view used by the aggregator library and by tests: pointer to the
// mapped control block (nullptr when none is mapped).
SWL_EXPORT void* swl_q_control_block(void) { return g_q.ctrl; }
SWL_EXPORT int swl_q_capacity(void) { return g_q.capacity; }
SWL_EXPORT size_t swl_q_control_block_size(void) { return sizeof(ControlBlock); }
SWL_EXPORT size_t swl_q_command_size(void) { return sizeof(Command); }
