// Shared-memory ABI between the aggregator process and its worker processes.
//
// The byte layout of `ControlBlock` and `Command` is kept identical to the
// reference's (src/cpp_extensions/common/ipc_types.h:153-217) so a mixed
// deployment could read either side's segment; the mask type and helpers are
// this library's own. Op codes and MAX_SLOTS follow ipc_types.h:16-25.
#pragma once

#include <atomic>
#include <cstdint>
#include <pthread.h>

namespace swl {

constexpr int kMaxSlots = 128;             // ipc_types.h:16
constexpr int kMaskWords = kMaxSlots / 64;  // two 64-bit words

// Op codes carried in Command::op_type (ipc_types.h:19-25).
constexpr int kOpOProj = 3;
constexpr int kOpDownProj = 6;
constexpr int kOpQkvFused = 9;
constexpr int kOpGateUpFused = 10;
constexpr int kOpEmbed = 11;
constexpr int kOpLmHead = 12;
constexpr int kOpSetSampling = 13;

// Progressive back-off thresholds for host spin loops (ipc_types.h:29-31).
constexpr int kSpinTight = 64;
constexpr int kSpinPause = 1024;
constexpr int kSpinYield = 10000;

// Plain 128-bit slot set (one bit per slot) for local use.
struct Mask128 {
  uint64_t w[kMaskWords] = {0, 0};
  Mask128() = default;
  Mask128(uint64_t lo, uint64_t hi) { w[0] = lo; w[1] = hi; }
  static Mask128 bit(int i) { Mask128 m; m.set(i); return m; }
  static Mask128 first_n(int n) {
    Mask128 m;
    for (int k = 0; k < kMaskWords; ++k) {
      int lo = k * 64, take = n - lo;
      if (take >= 64) m.w[k] = ~0ull;
      else if (take > 0) m.w[k] = (1ull << take) - 1;
    }
    return m;
  }
  void set(int i) { w[i >> 6] |= 1ull << (i & 63); }
  void clear(int i) { w[i >> 6] &= ~(1ull << (i & 63)); }
  bool test(int i) const { return (w[i >> 6] >> (i & 63)) & 1ull; }
  bool empty() const { return (w[0] | w[1]) == 0; }
  int count() const { return __builtin_popcountll(w[0]) + __builtin_popcountll(w[1]); }
  int lowest() const {
    if (w[0]) return __builtin_ctzll(w[0]);
    if (w[1]) return 64 + __builtin_ctzll(w[1]);
    return -1;
  }
  Mask128 operator&(const Mask128& o) const { return {w[0] & o.w[0], w[1] & o.w[1]}; }
  Mask128 operator|(const Mask128& o) const { return {w[0] | o.w[0], w[1] | o.w[1]}; }
  Mask128 operator~() const { return {~w[0], ~w[1]}; }
  bool operator==(const Mask128& o) const { return w[0] == o.w[0] && w[1] == o.w[1]; }
};

// 128-bit slot set living in shared memory. Every mutation touches one bit
// (or applies an AND mask word by word), so per-word atomics suffice.
struct SharedMask128 {
  std::atomic<uint64_t> w[kMaskWords];
  Mask128 load(std::memory_order o = std::memory_order_acquire) const {
    return {w[0].load(o), w[1].load(o)};
  }
  void store(const Mask128& m, std::memory_order o = std::memory_order_release) {
    w[0].store(m.w[0], o);
    w[1].store(m.w[1], o);
  }
  Mask128 take_all(std::memory_order o = std::memory_order_acq_rel) {
    return {w[0].exchange(0, o), w[1].exchange(0, o)};
  }
  void set_bit(int i, std::memory_order o = std::memory_order_release) {
    w[i >> 6].fetch_or(1ull << (i & 63), o);
  }
  void and_with(const Mask128& m, std::memory_order o = std::memory_order_release) {
    w[0].fetch_and(m.w[0], o);
    w[1].fetch_and(m.w[1], o);
  }
  void clear_bit(int i, std::memory_order o = std::memory_order_release) {
    w[i >> 6].fetch_and(~(1ull << (i & 63)), o);
  }
  bool test(int i, std::memory_order o = std::memory_order_acquire) const {
    return (w[i >> 6].load(o) >> (i & 63)) & 1ull;
  }
  bool cas_word(int k, uint64_t& expect, uint64_t desired) {
    return w[k].compare_exchange_weak(expect, desired, std::memory_order_acq_rel,
                                      std::memory_order_acquire);
  }
};

// Sampling parameters a worker posts out of band before it joins.
struct PendingSampling {
  bool do_sample;
  float temperature;
  int top_k;
  float top_p;
};

// One ring entry. Field order is the shared-memory contract; with alignas(64)
// the 88 bytes of fields round up to 128 bytes, as in the reference.
struct alignas(64) Command {
  std::atomic<int> ready;  // 0 = empty, 1 = written
  int op_type;
  int layer_idx;
  int slot_id;
  int worker_id;
  int64_t bx, tx, dx;
  uint64_t x_key;
  uint64_t y0_key;
  uint64_t y1_key;
  uint64_t y2_key;
  int ticket_id;
  char pad_[4];
};

// Header of the shm segment; the Command ring follows it.
struct alignas(64) ControlBlock {
  std::atomic<int> head;
  std::atomic<int> tail;
  int capacity;
  std::atomic<int> quit_flag;
  int num_workers;
  int num_slots;
  SharedMask128 unused_free_mask;  // kept for layout compatibility
  SharedMask128 active_slot_mask;
  SharedMask128 pending_slot_joins;
  SharedMask128 pending_slot_leaves;
  SharedMask128 per_slot_ready_mask;
  SharedMask128 evicted_slot_mask;
  std::atomic<int> active_slot_count;
  std::atomic<int> slot_ready_count;
  std::atomic<int64_t> barrier_done_epoch;
  SharedMask128 pending_sampling_mask;
  PendingSampling pending_sampling[kMaxSlots];
  char pad1[64];
  pthread_mutex_t unused_mutex;  // layout compatibility only
  pthread_cond_t unused_cond0;
  pthread_cond_t unused_cond1;
};

static_assert(sizeof(Command) == 128, "Command layout changed");
static_assert(sizeof(ControlBlock) % 64 == 0, "ring must stay 64-byte aligned");

inline size_t shm_bytes(int capacity) {
  return sizeof(ControlBlock) + static_cast<size_t>(capacity) * sizeof(Command);
}

inline void cpu_relax() {
#if defined(__x86_64__)
  __builtin_ia32_pause();
#endif
}

}  // namespace swl
