// Stress run of the aggregator's host protocol in one process, for the
// thread and address sanitizers: worker threads drive the worker-side queue
// API (swarmlora_b200/csrc/ipc_queue.cpp: join, submit, ready, wait for the
// epoch, leave) against an aggregator thread running run_main_loop
// (swarmlora_b200/csrc/agg_protocol.h) with a host "round" in place of the
// GPU round. Per-slot inputs and outputs are plain (non-atomic) arrays, so
// the sanitizer sees whether the ring and the epoch publish them.
//
// Scenarios: workers joining at different times (half of them posting
// sampling parameters first) and leaving after different token counts, one worker that stops mid-token (evicted by the barrier
// timeout), one that submits a command under another worker's id (evicted
// by validation). With --deferred the rounds complete the way the library's
// device-published completion does: the loop clears the ready state, hands
// the round's epoch to a publisher thread (standing in for the device) and
// goes on; the publisher stores it after a short random delay. Exit status
// 0 and "protocol stress ok" on success.
#include <signal.h>
#include <sys/mman.h>
#include <sys/wait.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <mutex>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "agg_protocol.h"
#include "common.h"
#include "swarmlora_b200.h"

namespace swl {
static thread_local std::string g_err;
int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}
const char* last_error() { return g_err.c_str(); }
}  // namespace swl

using namespace swl;

namespace {

constexpr int kWorkers = 10;
constexpr int kLayers = 2;
constexpr int kOpsPerToken = 1 + 4 * kLayers + 1;
constexpr int kStall = 3;  // stops submitting mid-token
constexpr int kRogue = 6;  // submits one command under another worker's id

// A worker's input of the current op and the round's output for its slot
// (plain data); in the process mode they live in a shared mapping.
uint64_t g_in_local[kMaxSlots], g_out_local[kMaxSlots];
uint64_t* g_in = g_in_local;
uint64_t* g_out = g_out_local;
constexpr int kVictim = 5;  // process mode: dies by SIGKILL mid-token
bool g_processes = false;
std::atomic<int> g_failures{0};
std::atomic<int> g_rounds{0};
std::atomic<int> g_evicted_seen{0};

void fail(const char* what, int slot) {
  fprintf(stderr, "FAIL slot %d: %s\n", slot, what);
  g_failures.fetch_add(1);
}

void op_of(int k, int* op, int* layer) {
  static const int per_layer[4] = {kOpQkvFused, kOpOProj, kOpGateUpFused, kOpDownProj};
  if (k == 0) { *op = kOpEmbed; *layer = 0; return; }
  if (k == kOpsPerToken - 1) { *op = kOpLmHead; *layer = 0; return; }
  *op = per_layer[(k - 1) % 4];
  *layer = (k - 1) / 4;
}

bool wait_until(bool (*pred)(int), int slot, int ms) {
  auto t0 = std::chrono::steady_clock::now();
  while (!pred(slot)) {
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(ms)) return false;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  return true;
}
bool is_active(int s) { return swl_q_slot_is_active(s) == 1; }
bool is_inactive(int s) { return swl_q_slot_is_active(s) == 0; }
bool is_evicted(int s) { return swl_q_is_slot_evicted(s) == 1; }

std::atomic<int> g_sampling_taken{0};

// Stores handed-out epochs into the control block after a short delay, in
// order, as the device does after a round's kernels.
struct Publisher {
  ControlBlock* ctrl = nullptr;
  std::mutex mu;
  std::condition_variable cv;
  std::deque<int64_t> todo;
  int64_t stored = 0;
  bool stop = false;
  std::thread th;
  void start(ControlBlock* c) {
    ctrl = c;
    stored = c->barrier_done_epoch.load();
    th = std::thread([this] { run(); });
  }
  void run() {
    unsigned seed = 12345;
    std::unique_lock<std::mutex> lk(mu);
    for (;;) {
      cv.wait(lk, [this] { return stop || !todo.empty(); });
      if (todo.empty()) return;
      const int64_t v = todo.front();
      lk.unlock();
      seed = seed * 1103515245u + 12345u;
      std::this_thread::sleep_for(std::chrono::microseconds((seed >> 16) % 50));
      ctrl->barrier_done_epoch.store(v, std::memory_order_release);
      lk.lock();
      todo.pop_front();
      stored = v;
      cv.notify_all();
    }
  }
  void publish(int64_t v) {
    std::lock_guard<std::mutex> lk(mu);
    if (v <= stored || (!todo.empty() && v <= todo.back())) fail("epochs handed out of order", -1);
    todo.push_back(v);
    cv.notify_all();
  }
  void flush() {
    std::unique_lock<std::mutex> lk(mu);
    cv.wait(lk, [this] { return todo.empty(); });
  }
  void finish() {
    {
      std::lock_guard<std::mutex> lk(mu);
      stop = true;
      cv.notify_all();
    }
    th.join();
  }
};

struct HostHooks {
  std::vector<int> owner;  // slot -> worker id
  ControlBlock* ctrl = nullptr;
  Publisher* pub = nullptr;  // deferred completion
  bool deferred_epoch() const { return pub != nullptr; }
  void flush() {
    if (pub) pub->flush();
  }
  void on_membership(const Mask128&, const Mask128& joins) {
    take_pending_sampling(ctrl, joins, [](int sid, const PendingSampling& p) {
      // the joining worker posted temperature 0.5 + slot and top_k = slot
      if (!p.do_sample || p.top_k != sid || p.temperature != 0.5f + static_cast<float>(sid) || p.top_p != 0.9f)
        fail("pending sampling parameters not visible at the join", sid);
      g_sampling_taken.fetch_add(1);
    });
  }
  void on_sampling(const DrainedCmd&) {}
  void validate(int, int, const std::vector<DrainedCmd>& cmds, std::vector<int>* bad) {
    for (const DrainedCmd& c : cmds)
      if (c.worker_id != owner[c.slot_id] || c.rows != 1) bad->push_back(c.slot_id);
  }
  int round(int op, int layer, const std::vector<DrainedCmd>& cmds, const std::vector<int>& bad, int64_t epoch) {
    if (pub && !ctrl->per_slot_ready_mask.load().empty() &&
        !(ctrl->per_slot_ready_mask.load() & ctrl->active_slot_mask.load()).empty())
      fail("ready bits of the round still set when it runs", -1);
    for (const DrainedCmd& c : cmds) {
      if (c.op_type != op || c.layer_idx != layer) fail("round mixes ops", c.slot_id);
      bool refused = false;
      for (int b : bad) refused |= b == c.slot_id;
      if (refused) continue;
      if (g_in[c.slot_id] != c.x_key) fail("slot input not visible to the round", c.slot_id);
      g_out[c.slot_id] = c.x_key + 1;
    }
    g_rounds.fetch_add(1);
    if (pub) pub->publish(epoch);
    return 0;
  }
};

void worker(int slot, int tokens, int join_delay_ms) {
  const int wid = 1000 + slot;
  std::this_thread::sleep_for(std::chrono::milliseconds(join_delay_ms));
  if (slot % 2 == 0)  // posted before the join, applied at the token boundary that admits the slot
    swl_q_slot_set_pending_sampling(slot, 1, 0.5f + static_cast<float>(slot), slot, 0.9f);
  swl_q_slot_signal_join(slot);
  if (!wait_until(is_active, slot, 5000)) return fail("never activated", slot);
  uint64_t counter = 0;
  for (int t = 0; t < tokens; ++t) {
    for (int k = 0; k < kOpsPerToken; ++k) {
      if (slot == kStall && t == 2 && k == 3) {  // hang mid-token: the barrier evicts the slot
        if (!wait_until(is_evicted, slot, 5000)) return fail("stalled slot was not evicted", slot);
        g_evicted_seen.fetch_add(1);
        return;
      }
      int op, layer;
      op_of(k, &op, &layer);
      const int64_t e0 = swl_q_get_barrier_done_epoch();
      const uint64_t key = (static_cast<uint64_t>(slot) << 40) | ++counter;
      g_in[slot] = key;
      const int as = (slot == kRogue && t == 3 && k == 5) ? wid + 1 : wid;
      int rc;
      while ((rc = swl_q_submit_slot_command(op, layer, slot, as, 1, 1, 4096, key, 0, 0, 0, 0)) == SWL_ERR_FULL)
        std::this_thread::yield();
      if (rc != SWL_OK) return fail("submit failed", slot);
      swl_q_slot_signal_ready(slot);
      if (g_processes && slot == kVictim && t == 2 && k == 4) raise(SIGKILL);  // the fault driver's kill
      int64_t e = 0;
      if (swl_q_wait_for_epoch(e0, 5000, &e) != SWL_OK) return fail("epoch did not move", slot);
      if (is_evicted(slot)) {
        if (as == wid) return fail("evicted without cause", slot);
        g_evicted_seen.fetch_add(1);
        return;
      }
      if (as != wid) return fail("foreign command was not refused", slot);
      if (g_out[slot] != key + 1) return fail("round output missing", slot);
    }
  }
  swl_q_slot_signal_leave(slot);
  if (!wait_until(is_inactive, slot, 5000)) fail("leave not acknowledged", slot);
}

}  // namespace

// Process mode: the workers are forked processes sharing the queue segment
// (inherited mapping) and a shared page for the slot data; kVictim kills
// itself after signalling ready mid-token, as the reference's fault driver
// (security_eval/common/fault_driver.py) kills a worker; the aggregator must
// evict it after the barrier timeout and every other worker must finish.
int run_processes(ControlBlock* ctrl, Command* ring, HostHooks& hooks, const ProtocolTimes& times) {
  void* shared = mmap(nullptr, 2 * sizeof(uint64_t) * kMaxSlots, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_ANONYMOUS,
                      -1, 0);
  if (shared == MAP_FAILED) return 2;
  g_in = static_cast<uint64_t*>(shared);
  g_out = g_in + kMaxSlots;
  std::vector<pid_t> pids;
  for (int s = 0; s < kWorkers; ++s) {
    if (s == kStall || s == kRogue) continue;  // this mode tests the kill alone
    pid_t pid = fork();
    if (pid == 0) {
      worker(s, 12 + 2 * (s % 3), (s % 3) * 10);
      _exit(g_failures.load() ? 1 : 0);
    }
    pids.push_back(pid);
  }
  int loop_status = -99;
  const auto t0 = std::chrono::steady_clock::now();
  std::thread agg([&] { loop_status = run_main_loop(ctrl, ring, swl_q_capacity(), kOpsPerToken, hooks, times); });
  int killed = 0, ok = 0;
  for (pid_t pid : pids) {
    int st = 0;
    waitpid(pid, &st, 0);
    if (WIFSIGNALED(st) && WTERMSIG(st) == SIGKILL) ++killed;
    else if (WIFEXITED(st) && WEXITSTATUS(st) == 0) ++ok;
    else fail("a surviving worker failed", -1);
  }
  const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  swl_q_set_quit(1);
  agg.join();
  if (loop_status != 0) fail("main loop returned an error", -1);
  if (killed != 1) fail("expected exactly one killed worker", -1);
  if (ctrl->evicted_slot_mask.test(kVictim) == false) fail("the killed worker's slot was not evicted", kVictim);
  if (g_failures.load()) return 1;
  printf("protocol stress ok: processes, %d survived, 1 killed and evicted, %.2f s\n", ok, secs);
  return 0;
}

int main(int argc, char** argv) {
  g_processes = argc > 1 && std::string(argv[1]) == "--processes";
  const bool deferred = argc > 1 && std::string(argv[1]) == "--deferred";
  char name[128];
  if (swl_q_create(256, 256, name, sizeof(name)) != SWL_OK || swl_q_init_batch_control(kWorkers) != SWL_OK) {
    fprintf(stderr, "queue setup failed: %s\n", last_error());
    return 2;
  }
  auto* ctrl = static_cast<ControlBlock*>(swl_q_control_block());
  auto* ring = reinterpret_cast<Command*>(reinterpret_cast<char*>(ctrl) + sizeof(ControlBlock));
  HostHooks hooks;
  hooks.ctrl = ctrl;
  hooks.owner.assign(kMaxSlots, -1);
  for (int s = 0; s < kWorkers; ++s) hooks.owner[s] = 1000 + s;
  ProtocolTimes times;
  times.evict_after = std::chrono::milliseconds(100);
  times.leave_every = std::chrono::milliseconds(2);
  if (g_processes) {
    const int rc = run_processes(ctrl, ring, hooks, times);
    swl_q_close();
    return rc;
  }
  Publisher pub;
  if (deferred) {
    pub.start(ctrl);
    hooks.pub = &pub;
  }
  int loop_status = -99;
  std::thread agg([&] { loop_status = run_main_loop(ctrl, ring, swl_q_capacity(), kOpsPerToken, hooks, times); });
  std::vector<std::thread> ws;
  for (int s = 0; s < kWorkers; ++s) ws.emplace_back(worker, s, 40 + 10 * (s % 4), (s % 3) * 15);
  for (auto& w : ws) w.join();
  swl_q_set_quit(1);
  agg.join();
  if (deferred) {
    if (!pub.todo.empty()) fail("the loop returned with epochs still to store", -1);
    pub.finish();
  }
  swl_q_close();
  if (loop_status != 0) fail("main loop returned an error", -1);
  if (g_evicted_seen.load() != 2) fail("expected exactly the stalled and the rogue slot evicted", -1);
  if (g_sampling_taken.load() != (kWorkers + 1) / 2) fail("every posted sampling state taken once", -1);
  if (g_failures.load()) return 1;
  printf("protocol stress ok: %d rounds, %d workers, 2 evicted%s\n", g_rounds.load(), kWorkers,
         deferred ? ", epochs published by a deferred publisher" : "");
  return 0;
}
