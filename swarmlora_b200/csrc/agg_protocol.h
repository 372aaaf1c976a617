// Host side of the aggregator's lock-step protocol over the shared-memory
// control block and command ring (ext_aggregator.cpp:879-1210): the slot
// barrier with mid-op leaves and eviction of stuck slots, the epoch signal,
// the ring drain and the per-token main loop. Free of CUDA: the aggregator
// library runs it with its GPU rounds as hooks, and
// tests/native/protocol_stress.cpp runs the same code with a host round
// under ThreadSanitizer and AddressSanitizer.
#pragma once

#include <chrono>
#include <cstdio>
#include <thread>
#include <vector>

#include "shm_abi.h"

namespace swl {

// One command taken off the ring.
struct DrainedCmd {
  int slot_id;
  int worker_id;
  int op_type;
  int layer_idx;
  int64_t rows;  // bx * tx
  uint64_t x_key, y0_key, y1_key;
};

struct ProtocolTimes {
  std::chrono::milliseconds evict_after{500};  // a slot not ready this long is evicted (ext_aggregator.cpp:883)
  std::chrono::milliseconds leave_every{10};   // mid-op leave poll
  long drain_spin_limit = 10000000;            // polls of one ring entry before the loop gives up
};

// aggregator_wait_for_slots (ext_aggregator.cpp:879-978): waits until every
// active slot has set its ready bit; drops slots that signal leave mid-op
// and evicts slots not ready within t.evict_after. Returns the remaining
// slot count, or -1 when the quit flag is raised.
inline int wait_for_slots(ControlBlock* ctrl, Mask128& active, const ProtocolTimes& t) {
  using clk = std::chrono::steady_clock;
  auto start = clk::now(), last_leave = start;
  long spins = 0;
  for (;;) {
    Mask128 ready = ctrl->per_slot_ready_mask.load();
    Mask128 missing = active & ~ready;
    if (missing.empty()) return active.count();
    if (ctrl->quit_flag.load(std::memory_order_acquire)) return -1;
    ++spins;
    if (spins < kSpinTight) continue;
    if (spins < kSpinYield) {
      cpu_relax();
      continue;
    }
    auto now = clk::now();
    if (now - last_leave > t.leave_every) {
      last_leave = now;
      Mask128 leaving = ctrl->pending_slot_leaves.load() & active;
      if (!leaving.empty()) {
        active = active & ~leaving;
        ctrl->pending_slot_leaves.and_with(~leaving);
        ctrl->active_slot_mask.store(active);
        ctrl->active_slot_count.store(active.count());
        if (active.empty()) return 0;
      }
    }
    if (now - start > t.evict_after) {
      Mask128 stuck = active & ~ctrl->per_slot_ready_mask.load();
      if (!stuck.empty()) {
        active = active & ~stuck;
        ctrl->active_slot_mask.store(active);
        ctrl->active_slot_count.store(active.count());
        for (Mask128 r = stuck; !r.empty();) {
          int sid = r.lowest();
          r.clear(sid);
          ctrl->evicted_slot_mask.set_bit(sid);
        }
        fprintf(stderr, "[swl aggregator] evicting stuck slot(s) mask=0x%llx:%llx; %d continue\n",
                (unsigned long long)stuck.w[1], (unsigned long long)stuck.w[0], active.count());
        if (active.empty()) return 0;
        start = clk::now();
        spins = 0;
      }
    }
    cpu_relax();
    cpu_relax();
  }
}

// First half of aggregator_signal_done_slots (ext_aggregator.cpp:981-987):
// the round's ready state (count and the active slots' ready bits) is reset.
// A worker sets its next ready bit only after it has seen the epoch move, so
// resetting before the epoch is published (by the host below, or by the
// device once the round's kernels have finished) never loses a ready bit.
inline void clear_ready(ControlBlock* ctrl) {
  ctrl->slot_ready_count.store(0, std::memory_order_release);
  Mask128 active = ctrl->active_slot_mask.load();
  ctrl->per_slot_ready_mask.and_with(~active);
}

// aggregator_signal_done_slots (ext_aggregator.cpp:981-987).
inline void signal_done(ControlBlock* ctrl) {
  clear_ready(ctrl);
  ctrl->barrier_done_epoch.fetch_add(1, std::memory_order_release);
}

inline void evict_slots(ControlBlock* ctrl, const std::vector<int>& slots, Mask128& active) {
  for (int sid : slots) {
    active.clear(sid);
    ctrl->evicted_slot_mask.set_bit(sid);
  }
  ctrl->active_slot_mask.store(active);
  ctrl->active_slot_count.store(active.count());
}

// apply_pending_sampling_states (ext_aggregator.cpp:991-1020): hands the
// sampling parameters that joining slots posted (slot_set_pending_sampling)
// to fn(slot, params) and clears their pending bits.
template <class Fn>
inline void take_pending_sampling(ControlBlock* ctrl, const Mask128& joins, Fn&& fn) {
  Mask128 todo = ctrl->pending_sampling_mask.load() & joins;
  for (Mask128 r = todo; !r.empty();) {
    int sid = r.lowest();
    r.clear(sid);
    fn(sid, ctrl->pending_sampling[sid]);
  }
  ctrl->pending_sampling_mask.and_with(~todo);
}

// Takes ring entries until n commands of active slots are collected,
// discarding entries of slots evicted or gone meanwhile. Returns false when
// the quit flag is raised (or raised here after an entry stayed unwritten
// for t.drain_spin_limit polls).
inline bool drain_commands(ControlBlock* ctrl, Command* ring, int capacity, const Mask128& active, int n,
                           std::vector<DrainedCmd>* out, const ProtocolTimes& t) {
  int tail = ctrl->tail.load(std::memory_order_acquire);
  int drained = 0;
  bool quit = false;
  while (static_cast<int>(out->size()) < n && drained < kMaxSlots + 8) {
    Command* c = &ring[tail];
    long spin = 0;
    while (c->ready.load(std::memory_order_acquire) != 1) {
      if (ctrl->quit_flag.load(std::memory_order_acquire)) {
        quit = true;
        break;
      }
      if (++spin > t.drain_spin_limit) {
        fprintf(stderr, "[swl aggregator] command not ready after drain wait; quitting\n");
        ctrl->quit_flag.store(1, std::memory_order_release);
        quit = true;
        break;
      }
      if (spin > kSpinYield) cpu_relax();
    }
    if (quit) break;
    const DrainedCmd d{c->slot_id, c->worker_id, c->op_type, c->layer_idx, c->bx * c->tx,
                       c->x_key, c->y0_key, c->y1_key};
    c->ready.store(0, std::memory_order_release);
    tail = (tail + 1) % capacity;
    ++drained;
    if (d.slot_id >= 0 && d.slot_id < kMaxSlots && active.test(d.slot_id)) out->push_back(d);
  }
  ctrl->tail.store(tail, std::memory_order_release);
  return !quit && ctrl->quit_flag.load(std::memory_order_acquire) == 0;
}

// aggregator_main_loop_slots (ext_aggregator.cpp:1024-1210). Joins and
// leaves are applied at token boundaries; each token is ops_per_token
// rounds: wait for every active slot's ready bit, drain one command per
// slot, run the round, signal the epoch.
//
// Completion. With h.deferred_epoch() false the host signals each round
// after h.round returns (the reference: the round has finished, the host
// bumps the epoch). With it true the loop clears the ready state first and
// passes h.round the epoch value that completes the round; the hook
// arranges for that value to be stored into barrier_done_epoch once the
// round's results are in place (a device write after the round's kernels)
// and returns at once, so the host goes on to wait for the next round's
// ready bits while the round runs. The loop keeps the last value it handed
// out; before the host itself signals (quit, a failed drain, a sampling-only
// round) it calls h.flush(), which must return only once every handed-out
// value has been stored. Hooks:
//   void on_membership(const Mask128& active, const Mask128& joins)
//       after a token boundary's joins / leaves are applied;
//   void on_sampling(const DrainedCmd& c)   for each set-sampling command;
//   void validate(int op, int layer, const std::vector<DrainedCmd>& cmds,
//                 std::vector<int>* bad)     slots whose commands are refused
//                                            (evicted; the round runs without them);
//   int round(int op, int layer, const std::vector<DrainedCmd>& cmds,
//             const std::vector<int>& bad, int64_t epoch)
//                                            0 or a failure status, which ends the loop;
//                                            `epoch` is the value to publish (deferred
//                                            completion) or 0;
//   bool deferred_epoch()                    see Completion above;
//   void flush()                             every handed-out epoch stored.
// Returns 0 when the quit flag ends the loop.
template <class Hooks>
int run_main_loop(ControlBlock* ctrl, Command* ring, int capacity, int ops_per_token, Hooks& h,
                  const ProtocolTimes& t = ProtocolTimes()) {
  Mask128 active;
  std::vector<DrainedCmd> cmds;
  std::vector<int> bad;
  cmds.reserve(kMaxSlots);
  // last epoch value handed to the hooks (deferred completion)
  int64_t handed = ctrl->barrier_done_epoch.load(std::memory_order_acquire);
  auto host_signal = [&] {
    h.flush();
    signal_done(ctrl);
    handed = ctrl->barrier_done_epoch.load(std::memory_order_acquire);
  };
  while (ctrl->quit_flag.load(std::memory_order_acquire) == 0) {
    Mask128 leaves, joins;
    if (!ctrl->pending_slot_leaves.load().empty()) leaves = ctrl->pending_slot_leaves.take_all();
    if (!leaves.empty()) active = active & ~leaves;
    if (!ctrl->pending_slot_joins.load().empty()) joins = ctrl->pending_slot_joins.take_all();
    if (!joins.empty()) active = active | joins;
    // A joining worker reads the epoch once it sees itself active and waits
    // for it to move: every round's epoch must be stored before then, or a
    // late store would release its first wait before its round ran.
    if (!joins.empty() && h.deferred_epoch()) h.flush();
    int N = active.count();
    ctrl->active_slot_mask.store(active);
    ctrl->active_slot_count.store(N);
    h.on_membership(active, joins);
    if (N == 0) {
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
      continue;
    }
    for (int op_idx = 0; op_idx < ops_per_token; ++op_idx) {
      int got = wait_for_slots(ctrl, active, t);
      if (got < 0) {
        host_signal();
        break;
      }
      if (got == 0) break;
      N = got;
      cmds.clear();
      if (!drain_commands(ctrl, ring, capacity, active, N, &cmds, t)) {
        host_signal();
        break;
      }
      if (cmds.empty()) continue;
      const int op = cmds[0].op_type, layer = cmds[0].layer_idx;
      for (const DrainedCmd& c : cmds)
        if (c.op_type == kOpSetSampling) h.on_sampling(c);
      if (op == kOpSetSampling) {
        host_signal();
        continue;
      }
      bad.clear();
      h.validate(op, layer, cmds, &bad);
      if (!bad.empty()) evict_slots(ctrl, bad, active);
      int st;
      if (h.deferred_epoch()) {
        clear_ready(ctrl);
        st = h.round(op, layer, cmds, bad, ++handed);
        if (st != 0) {
          host_signal();  // publish what the failed round would have, so no worker waits on it
          return st;
        }
      } else {
        st = h.round(op, layer, cmds, bad, 0);
        signal_done(ctrl);
        if (st != 0) return st;  // device state is unknown; stop like the reference does
      }
    }
  }
  h.flush();
  return 0;
}

}  // namespace swl
