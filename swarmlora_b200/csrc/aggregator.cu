// Aggregator side of the slot protocol: the slot pool (per-slot cudaMalloc +
// CUDA IPC handles), the fused frozen base weights, one round over pool slots,
// and the barrier-driven main loop. Mirrors the reference module
// ext_aggregator (src/cpp_extensions/ext_aggregator.cpp); each entry point
// cites the function whose behaviour it keeps.
//
// Differences by design:
//  * a round is one kernel (slot_round.cu) reading the slot buffers through a
//    slot table; no concatenated input or staging output exists;
//  * commands naming a bad slot, a non-owner or an oversized shape are
//    dropped and that slot is evicted, instead of ending the main loop;
//  * o_proj / down_proj / embed / lm_head weights are borrowed (the caller
//    keeps them alive), q|k|v and gate|up are fused into library-owned copies,
//    the same memory behaviour as the reference's detach()/cat().
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

#include "common.h"
#include "agg_protocol.h"
#include "shm_abi.h"
#include "swarmlora_b200.h"
#include "slot_round.h"
#include "vocab_ops.h"
#include "worker_ops.h"

using namespace swl;

namespace {

struct Slot {
  std::atomic<int> owner{-1};
  void* in = nullptr;
  void* out = nullptr;
  cudaIpcMemHandle_t in_handle;
  cudaIpcMemHandle_t out_handle;
  // event completion: the worker's event recorded after the work that
  // writes the slot's round input (opened from an IPC handle: owned here)
  cudaEvent_t input_event = nullptr;
  bool input_event_owned = false;
};

struct Pool {
  Slot slots[kMaxSlots];
  std::atomic<uint64_t> free_w[kMaskWords];
  std::atomic<uint64_t> active_w[kMaskWords];
  std::atomic<int> active_slot_count{0};
  int num_slots = 0;
  int device = 0;
  int hidden = 0, inter = 0, qkv = 0;
  size_t in_bytes = 0, out_bytes = 0;
  int max_seq_per_step = 0;
  bool initialized = false;
};

struct Layer {
  void* qkv = nullptr;  // owned [q+k+v, hidden]
  void* gu = nullptr;   // owned [gate+up, hidden]
  const void* o = nullptr;     // borrowed [hidden_out, hidden]
  const void* down = nullptr;  // borrowed [hidden, inter]
  const void* o_bias = nullptr;
  const void* down_bias = nullptr;
  int64_t q_dim = 0, k_dim = 0, v_dim = 0, gate_dim = 0, up_dim = 0;
  int64_t hidden = 0, inter = 0, o_out = 0, down_out = 0;
  bool owns_fused = true;  // qkv / gu are separate allocations (not in g_arena)
  CUtensorMap tm_qkv, tm_o, tm_gu, tm_down;
};

struct SamplingState {
  bool do_sample = false;
  float temperature = 1.0f;
  int top_k = 0;
  float top_p = 1.0f;
};

Pool g_pool;
std::vector<Layer> g_layers;
int g_num_layers = 0;
bool g_weights_ready = false;
int g_device = 0;

const void* g_embed = nullptr;    // borrowed [vocab, hidden] (or in g_arena)
const void* g_lm_head = nullptr;  // borrowed [vocab, hidden] (or in g_arena)
void* g_arena = nullptr;          // every weight, after swl_agg_import_weights
CUtensorMap g_tm_lm;
int64_t g_vocab = 0, g_embed_hidden = 0;
bool g_vocab_ready = false;
void* g_logits = nullptr;  // [kMaxSlots, vocab] bf16 LM-head scratch

ControlBlock* g_ctrl = nullptr;
Command* g_ring = nullptr;
int g_capacity = 0;
size_t g_map_bytes = 0;

cudaStream_t g_stream = nullptr;
int g_round_algo = kAlgoAuto;
int g_round_splits = 0;
std::map<int, SamplingState> g_sampling;  // worker_id -> params
std::mutex g_sampling_mu;                 // the loop thread and in-process setters both touch it
std::atomic<uint64_t> g_sample_seed{0};    // LM-head sampling: uniforms from (seed, offset, row)
std::atomic<uint64_t> g_sample_offset{0};  // advanced by every sampling LM-head round

// Column-sharded base weights over two GPUs (one process per GPU; the
// variant of the multi-GPU configuration with an NVLink all-gather of the
// outputs): every round reads a row view of the fused weight holding this
// GPU's half of the output columns and writes those columns into both GPUs'
// slot outputs (the LM head into both GPUs' logits). The peer's buffers are
// mapped from the IPC handles it exported; the worker-side kernels run on
// both GPUs over the same inputs.
struct ShardView {
  int64_t col0 = 0, n = 0;
  CUtensorMap tm;
};
struct Shard {
  bool on = false;
  int rank = 0;
  unsigned int* sync = nullptr;       // this GPU's sync words (kSyncWords, zeroed)
  unsigned int* peer_sync = nullptr;  // the peer's, mapped
  void* peer_logits = nullptr;        // the peer's LM-head logits, mapped
  std::vector<void*> peer_out;        // the peer's slot outputs by slot id, mapped
  std::vector<std::array<ShardView, 4>> layer;  // QKV, O, Gate+Up, Down
  ShardView lm;
};
Shard g_shard;

// This GPU's half of an [N, K] weight: columns [col0, col0 + n), split at a
// multiple of 8.
int shard_view(ShardView* v, const void* W, int64_t N, int64_t K, int rank) {
  const int64_t half = N / 2 / 8 * 8;
  v->col0 = rank == 0 ? 0 : half;
  v->n = rank == 0 ? half : N - half;
  return encode_weight_tmap(&v->tm, static_cast<const char*>(W) + v->col0 * K * 2, v->n, K);
}

Mask128 load_mask(const std::atomic<uint64_t>* w) {
  return {w[0].load(std::memory_order_acquire), w[1].load(std::memory_order_acquire)};
}
void store_mask(std::atomic<uint64_t>* w, const Mask128& m) {
  w[0].store(m.w[0], std::memory_order_release);
  w[1].store(m.w[1], std::memory_order_release);
}

int ensure_stream() {
  if (!g_stream) SWL_CUDA_TRY(cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking));
  return SWL_OK;
}

// One validated command of a round.
struct RoundCmd {
  int slot_id;
  int worker_id;
  int64_t rows;
};

// Checks slot id, ownership and shape of each command against the pool; bad
// ones are reported in *bad (slot ids) and left out of *good.
void validate(const RoundCmd* cmds, int n, int64_t in_row_bytes, int64_t out_row_bytes,
              std::vector<RoundCmd>* good, std::vector<int>* bad, std::string* why) {
  good->clear();
  bad->clear();
  for (int i = 0; i < n; ++i) {
    const RoundCmd& c = cmds[i];
    char buf[256];
    if (c.slot_id < 0 || c.slot_id >= g_pool.num_slots) {
      snprintf(buf, sizeof(buf), "invalid slot_id %d; ", c.slot_id);
      *why += buf;
      continue;  // cannot evict an out-of-range id
    }
    int owner = g_pool.slots[c.slot_id].owner.load(std::memory_order_acquire);
    if (owner != c.worker_id) {
      snprintf(buf, sizeof(buf), "worker %d does not own slot %d (owner=%d); ", c.worker_id,
               c.slot_id, owner);
      *why += buf;
      bad->push_back(c.slot_id);
      continue;
    }
    if (c.rows <= 0 || c.rows * in_row_bytes > static_cast<int64_t>(g_pool.in_bytes) ||
        c.rows * out_row_bytes > static_cast<int64_t>(g_pool.out_bytes)) {
      snprintf(buf, sizeof(buf), "slot %d: %lld rows exceed the slot buffers; ", c.slot_id,
               static_cast<long long>(c.rows));
      *why += buf;
      bad->push_back(c.slot_id);
      continue;
    }
    good->push_back(c);
  }
}

// Unmaps the peer's buffers and frees the sync words (back to unsharded rounds).
int shard_end() {
  if (!g_shard.sync && !g_shard.on) return SWL_OK;
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  SWL_CUDA_TRY(cudaDeviceSynchronize());
  if (g_shard.peer_sync) cudaIpcCloseMemHandle(g_shard.peer_sync);
  if (g_shard.peer_logits) cudaIpcCloseMemHandle(g_shard.peer_logits);
  for (void* q : g_shard.peer_out)
    if (q) cudaIpcCloseMemHandle(q);
  if (g_shard.sync) cudaFree(g_shard.sync);
  g_shard = Shard();
  return SWL_OK;
}

// Shard arguments of a round: slot i's peer rows are the peer's output
// buffer of the same slot id, or row i of the peer's logits (LM head).
ShardArgs shard_args(const std::vector<RoundCmd>& cmds, int64_t col0, bool logits, int64_t vocab) {
  ShardArgs a;
  for (int i = 0; i < kMaxSlots; ++i) a.peer_out[i] = nullptr;
  for (size_t i = 0; i < cmds.size(); ++i)
    a.peer_out[i] = logits ? static_cast<__nv_bfloat16*>(g_shard.peer_logits) + static_cast<int64_t>(i) * vocab
                           : static_cast<__nv_bfloat16*>(g_shard.peer_out[cmds[i].slot_id]);
  a.col0 = col0;
  a.sync = g_shard.sync;
  a.peer_sync = g_shard.peer_sync;
  return a;
}

// Runs one round over validated commands on `stream` (no synchronisation).
int run_round(int op, int layer, const std::vector<RoundCmd>& cmds, cudaStream_t stream) {
  if (cmds.empty()) return SWL_OK;
  const int n = static_cast<int>(cmds.size());
  if (op == kOpEmbed) {
    if (!g_vocab_ready) return set_error(SWL_ERR_STATE, "embed: weights not initialized");
    TokenTable tab;
    tab.nslots = n;
    int acc = 0;
    for (int i = 0; i < n; ++i) {
      const Slot& s = g_pool.slots[cmds[i].slot_id];
      tab.row_start[i] = acc;
      tab.tokens[i] = static_cast<const int64_t*>(s.in);
      tab.out[i] = static_cast<__nv_bfloat16*>(s.out);
      acc += static_cast<int>(cmds[i].rows);
    }
    tab.row_start[n] = acc;
    tab.total_rows = acc;
    return launch_embed_gather(tab, g_embed, g_vocab, g_embed_hidden, stream);
  }
  if (op == kOpLmHead) {
    if (!g_vocab_ready) return set_error(SWL_ERR_STATE, "lm_head: weights not initialized");
    SlotTable tab;
    TokenOuts outs;
    tab.nslots = n;
    for (int i = 0; i < n; ++i) {
      const Slot& s = g_pool.slots[cmds[i].slot_id];
      tab.row_start[i] = i;
      tab.in[i] = static_cast<const __nv_bfloat16*>(s.in) + (cmds[i].rows - 1) * g_embed_hidden;
      tab.out[i] = static_cast<__nv_bfloat16*>(g_logits) + static_cast<int64_t>(i) * g_vocab;
      outs.p[i] = static_cast<int64_t*>(s.out);
    }
    tab.row_start[n] = n;
    tab.total_rows = n;
    RoundShape shape{g_vocab, g_embed_hidden, g_embed_hidden, g_vocab, nullptr};
    if (g_shard.on) {
      const ShardView& v = g_shard.lm;
      shape.N = v.n;
      const ShardArgs sh = shard_args(cmds, v.col0, true, g_vocab);
      SWL_TRY(launch_slot_round_shard(tab, shape, static_cast<const char*>(g_lm_head) + v.col0 * g_embed_hidden * 2,
                                      &v.tm, sh, g_round_splits, stream));
    } else {
      SWL_TRY(launch_slot_round(tab, shape, g_lm_head, &g_tm_lm, g_round_algo, g_round_splits, stream));
    }
    // each row with its own worker's sampling state (the reference applies
    // the first command's worker's state to the whole batch,
    // ext_aggregator.cpp:717-734); greedy when no row samples
    SampleTable params;
    bool any = false;
    for (int i = 0; i < n; ++i) {
      SampleParams q{0, 1.0f, 0, 1.0f};
      std::lock_guard<std::mutex> lock(g_sampling_mu);
      auto it = g_sampling.find(cmds[i].worker_id);
      if (it != g_sampling.end())
        q = {it->second.do_sample ? 1 : 0, it->second.temperature, it->second.top_k, it->second.top_p};
      params.p[i] = q;
      any = any || q.do_sample != 0;
    }
    if (!any) return launch_argmax_rows(g_logits, n, g_vocab, g_vocab, outs, stream);
    return launch_sample_rows(g_logits, n, g_vocab, g_vocab, params, nullptr, g_sample_seed.load(),
                              g_sample_offset.fetch_add(1), outs, stream);
  }
  if (layer < 0 || layer >= g_num_layers)
    return set_error(SWL_ERR_ARG, "round: layer_idx %d out of range [0, %d)", layer, g_num_layers);
  const Layer& L = g_layers[layer];
  const void* W;
  const CUtensorMap* tm;
  RoundShape shape;
  int view = 0;
  switch (op) {
    case kOpQkvFused:
      W = L.qkv; tm = &L.tm_qkv; view = 0;
      shape = {L.q_dim + L.k_dim + L.v_dim, L.hidden, 0, 0, nullptr};
      break;
    case kOpOProj:
      W = L.o; tm = &L.tm_o; view = 1;
      shape = {L.o_out, L.hidden, 0, 0, static_cast<const __nv_bfloat16*>(L.o_bias)};
      break;
    case kOpGateUpFused:
      W = L.gu; tm = &L.tm_gu; view = 2;
      shape = {L.gate_dim + L.up_dim, L.hidden, 0, 0, nullptr};
      break;
    case kOpDownProj:
      W = L.down; tm = &L.tm_down; view = 3;
      shape = {L.down_out, L.inter, 0, 0, static_cast<const __nv_bfloat16*>(L.down_bias)};
      break;
    default:
      return set_error(SWL_ERR_ARG, "round: unknown op %d", op);
  }
  shape.in_stride = shape.K;
  shape.out_stride = shape.N;
  SlotTable tab;
  tab.nslots = n;
  int acc = 0;
  for (int i = 0; i < n; ++i) {
    const Slot& s = g_pool.slots[cmds[i].slot_id];
    tab.row_start[i] = acc;
    tab.in[i] = static_cast<const __nv_bfloat16*>(s.in);
    tab.out[i] = static_cast<__nv_bfloat16*>(s.out);
    acc += static_cast<int>(cmds[i].rows);
  }
  tab.row_start[n] = acc;
  tab.total_rows = acc;
  if (g_shard.on) {
    const ShardView& v = g_shard.layer[layer][view];
    shape.N = v.n;  // the row stride of the outputs stays the full width
    if (shape.bias) shape.bias += v.col0;
    const ShardArgs sh = shard_args(cmds, v.col0, false, 0);
    return launch_slot_round_shard(tab, shape, static_cast<const char*>(W) + v.col0 * shape.K * 2, &v.tm, sh,
                                   g_round_splits, stream);
  }
  return launch_slot_round(tab, shape, W, tm, g_round_algo, g_round_splits, stream);
}

void row_bytes_for(int op, int layer, int64_t* in_row, int64_t* out_row) {
  int64_t H = g_pool.hidden, I = g_pool.inter;
  *in_row = 2 * H;
  *out_row = 2 * H;
  if (op == kOpEmbed) { *in_row = 8; *out_row = 2 * H; return; }
  if (op == kOpLmHead) { *in_row = 2 * H; *out_row = 0; return; }
  if (layer >= 0 && layer < g_num_layers) {
    const Layer& L = g_layers[layer];
    if (op == kOpQkvFused) *out_row = 2 * (L.q_dim + L.k_dim + L.v_dim);
    if (op == kOpGateUpFused) *out_row = 2 * (L.gate_dim + L.up_dim);
    if (op == kOpDownProj) *in_row = 2 * I;
  }
}

}  // namespace

// ===== slot pool ============================================================

// ext_aggregator.cpp:138-187 init_slot_pool. Per-slot buffers: input
// max_seq_per_step * max(inter, hidden) * dtype_size bytes, output
// max_seq_per_step * max(2 * inter, qkv) * dtype_size bytes, each its own
// cudaMalloc with its own IPC handle (a worker can map only its own slot).
SWL_EXPORT int swl_agg_init_slot_pool(int num_slots, int device_index, int hidden_dim,
                                      int intermediate_dim, int num_kv_heads, int head_dim,
                                      int max_seq_per_step, int dtype_size, size_t* in_bytes,
                                      size_t* out_bytes) {
  if (num_slots <= 0 || num_slots > kMaxSlots)
    return set_error(SWL_ERR_ARG, "num_slots must be between 1 and %d", kMaxSlots);
  if (hidden_dim <= 0 || intermediate_dim <= 0 || max_seq_per_step <= 0 || dtype_size <= 0)
    return set_error(SWL_ERR_ARG, "init_slot_pool: dimensions must be positive");
  if (g_pool.initialized) return set_error(SWL_ERR_STATE, "init_slot_pool: already initialized");
  SWL_CUDA_TRY(cudaSetDevice(device_index));
  Pool& p = g_pool;
  p.num_slots = num_slots;
  p.device = device_index;
  p.hidden = hidden_dim;
  p.inter = intermediate_dim;
  p.qkv = hidden_dim + num_kv_heads * head_dim * 2;
  p.max_seq_per_step = max_seq_per_step;
  p.in_bytes = static_cast<size_t>(max_seq_per_step) * std::max(intermediate_dim, hidden_dim) * dtype_size;
  p.out_bytes = static_cast<size_t>(max_seq_per_step) * std::max(intermediate_dim * 2, p.qkv) * dtype_size;
  store_mask(p.free_w, Mask128::first_n(num_slots));
  store_mask(p.active_w, Mask128());
  p.active_slot_count.store(0);
  for (int i = 0; i < num_slots; ++i) {
    Slot& s = p.slots[i];
    s.owner.store(-1);
    SWL_CUDA_TRY(cudaMalloc(&s.in, p.in_bytes));
    SWL_CUDA_TRY(cudaMemset(s.in, 0, p.in_bytes));
    SWL_CUDA_TRY(cudaIpcGetMemHandle(&s.in_handle, s.in));
    SWL_CUDA_TRY(cudaMalloc(&s.out, p.out_bytes));
    SWL_CUDA_TRY(cudaMemset(s.out, 0, p.out_bytes));
    SWL_CUDA_TRY(cudaIpcGetMemHandle(&s.out_handle, s.out));
  }
  SWL_TRY(ensure_streamk_workspace());
  p.initialized = true;
  if (in_bytes) *in_bytes = p.in_bytes;
  if (out_bytes) *out_bytes = p.out_bytes;
  return SWL_OK;
}

// ext_aggregator.cpp:190-245 claim_slot: lowest free slot by CAS on its mask
// word; scrubs stale ready / evicted bits of the previous tenant.
SWL_EXPORT int swl_agg_claim_slot(int worker_id, int* slot_id, unsigned char* in_handle,
                                  unsigned char* out_handle, size_t* in_bytes, size_t* out_bytes) {
  if (!g_pool.initialized) return set_error(SWL_ERR_STATE, "claim_slot: slot pool not initialized");
  for (;;) {
    Mask128 freem = load_mask(g_pool.free_w);
    if (freem.empty()) return set_error(SWL_ERR_FULL, "No free slots available");
    int sid = freem.lowest();
    int k = sid >> 6;
    uint64_t expect = freem.w[k];
    if (g_pool.free_w[k].compare_exchange_weak(expect, expect & ~(1ull << (sid & 63)),
                                               std::memory_order_acq_rel,
                                               std::memory_order_acquire)) {
      Slot& s = g_pool.slots[sid];
      s.owner.store(worker_id, std::memory_order_release);
      if (g_ctrl) {
        g_ctrl->per_slot_ready_mask.clear_bit(sid);
        g_ctrl->evicted_slot_mask.clear_bit(sid);
      }
      if (slot_id) *slot_id = sid;
      if (in_handle) std::memcpy(in_handle, &s.in_handle, sizeof(cudaIpcMemHandle_t));
      if (out_handle) std::memcpy(out_handle, &s.out_handle, sizeof(cudaIpcMemHandle_t));
      if (in_bytes) *in_bytes = g_pool.in_bytes;
      if (out_bytes) *out_bytes = g_pool.out_bytes;
      return SWL_OK;
    }
  }
}

// ext_aggregator.cpp:248-296 release_slot: owner CAS, zero both buffers and
// wait for the zeroing before the slot becomes claimable again.
SWL_EXPORT int swl_agg_release_slot(int slot_id, int worker_id) {
  if (!g_pool.initialized) return set_error(SWL_ERR_STATE, "release_slot: slot pool not initialized");
  if (slot_id < 0 || slot_id >= g_pool.num_slots)
    return set_error(SWL_ERR_ARG, "release_slot: invalid slot_id");
  Slot& s = g_pool.slots[slot_id];
  int expect = worker_id;
  if (!s.owner.compare_exchange_strong(expect, -1, std::memory_order_acq_rel,
                                       std::memory_order_acquire))
    return set_error(SWL_ERR_OWNER, "release_slot: worker does not own slot %d", slot_id);
  SWL_CUDA_TRY(cudaSetDevice(g_pool.device));
  cudaStream_t st;
  SWL_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  cudaMemsetAsync(s.in, 0, g_pool.in_bytes, st);
  cudaMemsetAsync(s.out, 0, g_pool.out_bytes, st);
  cudaError_t e = cudaStreamSynchronize(st);
  cudaStreamDestroy(st);
  if (e != cudaSuccess) return set_error(SWL_ERR_CUDA, "release_slot: %s", cudaGetErrorString(e));
  if (s.input_event && s.input_event_owned) cudaEventDestroy(s.input_event);
  s.input_event = nullptr;
  s.input_event_owned = false;
  g_pool.free_w[slot_id >> 6].fetch_or(1ull << (slot_id & 63), std::memory_order_release);
  g_pool.active_w[slot_id >> 6].fetch_and(~(1ull << (slot_id & 63)), std::memory_order_release);
  return SWL_OK;
}

// ext_aggregator.cpp:299-304 get_slot_owner (-1 if free or invalid).
SWL_EXPORT int swl_agg_get_slot_owner(int slot_id) {
  if (!g_pool.initialized || slot_id < 0 || slot_id >= g_pool.num_slots) return -1;
  return g_pool.slots[slot_id].owner.load(std::memory_order_acquire);
}

// ext_aggregator.cpp:307-328 get_slot_pool_status. masks = {free_lo, free_hi,
// active_lo, active_hi}; owners receives num_slots entries (cap kMaxSlots).
SWL_EXPORT int swl_agg_get_slot_pool_status(int* initialized, int* num_slots, uint64_t* masks,
                                            int* active_slot_count, int* owners) {
  if (initialized) *initialized = g_pool.initialized ? 1 : 0;
  if (num_slots) *num_slots = g_pool.num_slots;
  Mask128 f = load_mask(g_pool.free_w), a = load_mask(g_pool.active_w);
  if (masks) {
    masks[0] = f.w[0];
    masks[1] = f.w[1];
    masks[2] = a.w[0];
    masks[3] = a.w[1];
  }
  if (active_slot_count) *active_slot_count = g_pool.active_slot_count.load();
  if (owners)
    for (int i = 0; i < g_pool.num_slots; ++i) owners[i] = g_pool.slots[i].owner.load();
  return SWL_OK;
}

// Aggregator-local device addresses of a slot's buffers (for in-process
// drivers such as tests and the benchmark; workers use the IPC handles).
SWL_EXPORT int swl_agg_slot_buffers(int slot_id, void** in, void** out) {
  if (!g_pool.initialized || slot_id < 0 || slot_id >= g_pool.num_slots)
    return set_error(SWL_ERR_ARG, "slot_buffers: invalid slot %d", slot_id);
  if (in) *in = g_pool.slots[slot_id].in;
  if (out) *out = g_pool.slots[slot_id].out;
  return SWL_OK;
}

// ext_aggregator.cpp:1410-1431 cleanup_slot_pool.
SWL_EXPORT int swl_agg_cleanup_slot_pool(void) {
  if (!g_pool.initialized) return SWL_OK;
  SWL_CUDA_TRY(cudaSetDevice(g_pool.device));
  SWL_CUDA_TRY(cudaDeviceSynchronize());
  SWL_TRY(shard_end());  // a column-shard setup maps the peer's buffers by slot
  for (int i = 0; i < g_pool.num_slots; ++i) {
    Slot& s = g_pool.slots[i];
    if (s.in) cudaFree(s.in);
    if (s.out) cudaFree(s.out);
    s.in = s.out = nullptr;
    if (s.input_event && s.input_event_owned) cudaEventDestroy(s.input_event);
    s.input_event = nullptr;
    s.input_event_owned = false;
    s.owner.store(-1);
  }
  g_pool.initialized = false;
  g_pool.num_slots = 0;
  return SWL_OK;
}

// ===== weights ===============================================================

// Frees the library-owned weights: the fused copies, or the arena of an
// import (which also held embed / lm_head, so those are forgotten with it).
int free_weights() {
  SWL_TRY(shard_end());  // its row views point into these weights
  for (Layer& L : g_layers) {
    if (L.owns_fused) {
      if (L.qkv) cudaFree(L.qkv);
      if (L.gu) cudaFree(L.gu);
    }
    L.qkv = L.gu = nullptr;
  }
  if (g_arena) {
    SWL_CUDA_TRY(cudaDeviceSynchronize());
    cudaFree(g_arena);
    g_arena = nullptr;
    g_embed = g_lm_head = nullptr;
    g_vocab_ready = false;
  }
  g_weights_ready = false;
  return SWL_OK;
}

// ext_aggregator.cpp:338-345 init_aggregator_begin.
SWL_EXPORT int swl_agg_init_begin(int num_layers, int device_index) {
  if (num_layers <= 0) return set_error(SWL_ERR_ARG, "init_aggregator_begin: num_layers must be > 0");
  SWL_CUDA_TRY(cudaSetDevice(device_index));
  SWL_TRY(free_weights());
  g_layers.assign(num_layers, Layer());
  g_num_layers = num_layers;
  g_device = device_index;
  g_weights_ready = false;
  return ensure_stream();
}

// ext_aggregator.cpp:347-376 init_aggregator_layer: W_qkv = cat(q, k, v) and
// W_gu = cat(gate, up) along the output dimension into library-owned
// buffers; o / down (and optional biases, NULL = none) are borrowed. All
// weights are row-major [out, in] bf16 on the aggregator device.
SWL_EXPORT int swl_agg_init_layer(int layer_idx, const void* q, int64_t q_rows, const void* k,
                                  int64_t k_rows, const void* v, int64_t v_rows, const void* o,
                                  int64_t o_rows, const void* o_bias, const void* gate,
                                  int64_t gate_rows, const void* up, int64_t up_rows,
                                  const void* down, int64_t down_rows, const void* down_bias,
                                  int64_t hidden, int64_t inter) {
  if (layer_idx < 0 || layer_idx >= g_num_layers)
    return set_error(SWL_ERR_ARG, "init_aggregator_layer: layer_idx %d out of range [0, %d)",
                     layer_idx, g_num_layers);
  if (!q || !k || !v || !o || !gate || !up || !down)
    return set_error(SWL_ERR_ARG, "init_aggregator_layer: null weight");
  Layer& L = g_layers[layer_idx];
  if (L.owns_fused) {
    if (L.qkv) cudaFree(L.qkv);
    if (L.gu) cudaFree(L.gu);
  }
  L = Layer();
  L.q_dim = q_rows; L.k_dim = k_rows; L.v_dim = v_rows;
  L.gate_dim = gate_rows; L.up_dim = up_rows;
  L.hidden = hidden; L.inter = inter; L.o_out = o_rows; L.down_out = down_rows;
  const size_t row_h = static_cast<size_t>(hidden) * 2;
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  SWL_CUDA_TRY(cudaMalloc(&L.qkv, (q_rows + k_rows + v_rows) * row_h));
  SWL_CUDA_TRY(cudaMalloc(&L.gu, (gate_rows + up_rows) * row_h));
  // The caller's weights may still be in flight on any of its streams (the
  // copy stream below does not wait for them).
  SWL_CUDA_TRY(cudaDeviceSynchronize());
  char* dq = static_cast<char*>(L.qkv);
  SWL_CUDA_TRY(cudaMemcpyAsync(dq, q, q_rows * row_h, cudaMemcpyDeviceToDevice, g_stream));
  SWL_CUDA_TRY(cudaMemcpyAsync(dq + q_rows * row_h, k, k_rows * row_h, cudaMemcpyDeviceToDevice, g_stream));
  SWL_CUDA_TRY(cudaMemcpyAsync(dq + (q_rows + k_rows) * row_h, v, v_rows * row_h,
                               cudaMemcpyDeviceToDevice, g_stream));
  char* dg = static_cast<char*>(L.gu);
  SWL_CUDA_TRY(cudaMemcpyAsync(dg, gate, gate_rows * row_h, cudaMemcpyDeviceToDevice, g_stream));
  SWL_CUDA_TRY(cudaMemcpyAsync(dg + gate_rows * row_h, up, up_rows * row_h, cudaMemcpyDeviceToDevice,
                               g_stream));
  SWL_CUDA_TRY(cudaStreamSynchronize(g_stream));
  L.o = o;
  L.down = down;
  L.o_bias = o_bias;
  L.down_bias = down_bias;
  SWL_TRY(encode_weight_tmap(&L.tm_qkv, L.qkv, q_rows + k_rows + v_rows, hidden));
  SWL_TRY(encode_weight_tmap(&L.tm_o, L.o, o_rows, hidden));
  SWL_TRY(encode_weight_tmap(&L.tm_gu, L.gu, gate_rows + up_rows, hidden));
  SWL_TRY(encode_weight_tmap(&L.tm_down, L.down, down_rows, inter));
  return SWL_OK;
}

// ext_aggregator.cpp:378-410 init_aggregator_finalize. No staging buffers are
// needed: the round kernel writes straight into the slot outputs.
SWL_EXPORT int swl_agg_init_finalize(void) {
  for (int i = 0; i < g_num_layers; ++i)
    if (!g_layers[i].qkv) return set_error(SWL_ERR_STATE, "init_aggregator_finalize: layer %d missing", i);
  g_weights_ready = true;
  return SWL_OK;
}

// ext_aggregator.cpp:413-424 init_embed_lm_head_weights (both borrowed).
SWL_EXPORT int swl_agg_init_embed_lm_head(const void* embed, const void* lm_head, int64_t vocab,
                                          int64_t hidden) {
  if (!embed || !lm_head || vocab <= 0 || hidden <= 0)
    return set_error(SWL_ERR_ARG, "init_embed_lm_head_weights: invalid arguments");
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  SWL_TRY(ensure_stream());
  g_embed = embed;
  g_lm_head = lm_head;
  g_vocab = vocab;
  g_embed_hidden = hidden;
  SWL_TRY(encode_weight_tmap(&g_tm_lm, lm_head, vocab, hidden));
  if (g_logits) cudaFree(g_logits);
  SWL_CUDA_TRY(cudaMalloc(&g_logits, static_cast<size_t>(kMaxSlots) * vocab * 2));
  g_vocab_ready = true;
  return SWL_OK;
}

// ===== donor weight transfer ==================================================

constexpr int kRecsPerLayer = 6;  // qkv, o, gate_up, down, o_bias, down_bias
constexpr size_t kArenaAlign = 512;

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

// The allocation holding `p`: its base and size.
int swl::allocation_of(const void* p, char** base, size_t* size) {
  auto fn = address_range_fn();
  if (!fn) return set_error(SWL_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  CUdeviceptr b = 0;
  size_t n = 0;
  CUresult r = fn(&b, &n, reinterpret_cast<CUdeviceptr>(p));
  if (r != CUDA_SUCCESS) return set_error(SWL_ERR_CUDA, "cuMemGetAddressRange failed (%d)", static_cast<int>(r));
  *base = reinterpret_cast<char*>(b);
  *size = n;
  return SWL_OK;
}

// One handle per allocation, so a receiver maps each allocation once.
using HandleCache = std::vector<std::pair<char*, cudaIpcMemHandle_t>>;

int export_one(HandleCache& cache, swl_weight_ipc* rec, const void* p, int64_t rows, int64_t cols) {
  memset(rec, 0, sizeof(*rec));
  if (!p || rows <= 0) return SWL_OK;  // absent (bias)
  char* base = nullptr;
  size_t size = 0;
  SWL_TRY(allocation_of(p, &base, &size));
  const cudaIpcMemHandle_t* hp = nullptr;
  for (const auto& c : cache)
    if (c.first == base) hp = &c.second;
  if (!hp) {
    cudaIpcMemHandle_t h;
    SWL_CUDA_TRY(cudaIpcGetMemHandle(&h, base));
    cache.emplace_back(base, h);
    hp = &cache.back().second;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(rec->handle), "IPC handle size");
  memcpy(rec->handle, hp, sizeof(rec->handle));
  rec->offset = static_cast<uint64_t>(static_cast<const char*>(p) - base);
  rec->rows = rows;
  rec->cols = cols;
  return SWL_OK;
}

// export_weight_ipc_handles (ext_aggregator.cpp:1216-1291), as records with
// offsets (layout in the public header).
SWL_EXPORT int swl_agg_export_weights(swl_weight_ipc* recs, int cap, int64_t* dims, int* num_layers,
                                      int* device_index) {
  if (!g_weights_ready) return set_error(SWL_ERR_STATE, "export_weight_ipc_handles: weights not initialized");
  if (!g_vocab_ready)
    return set_error(SWL_ERR_STATE, "export_weight_ipc_handles: embed/lm_head not initialized");
  if (num_layers) *num_layers = g_num_layers;
  if (device_index) *device_index = g_device;
  if (!recs) return SWL_OK;
  const int need = kRecsPerLayer * g_num_layers + 2;
  if (cap < need || !dims) return set_error(SWL_ERR_ARG, "export_weight_ipc_handles: room for %d records needed", need);
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  HandleCache cache;
  for (int l = 0; l < g_num_layers; ++l) {
    const Layer& L = g_layers[l];
    swl_weight_ipc* r = recs + kRecsPerLayer * l;
    SWL_TRY(export_one(cache, r + 0, L.qkv, L.q_dim + L.k_dim + L.v_dim, L.hidden));
    SWL_TRY(export_one(cache, r + 1, L.o, L.o_out, L.hidden));
    SWL_TRY(export_one(cache, r + 2, L.gu, L.gate_dim + L.up_dim, L.hidden));
    SWL_TRY(export_one(cache, r + 3, L.down, L.down_out, L.inter));
    SWL_TRY(export_one(cache, r + 4, L.o_bias, L.o_bias ? L.o_out : 0, 1));
    SWL_TRY(export_one(cache, r + 5, L.down_bias, L.down_bias ? L.down_out : 0, 1));
    int64_t* d = dims + 5 * l;
    d[0] = L.q_dim; d[1] = L.k_dim; d[2] = L.v_dim; d[3] = L.gate_dim; d[4] = L.up_dim;
  }
  SWL_TRY(export_one(cache, recs + kRecsPerLayer * g_num_layers, g_embed, g_vocab, g_embed_hidden));
  SWL_TRY(export_one(cache, recs + kRecsPerLayer * g_num_layers + 1, g_lm_head, g_vocab, g_embed_hidden));
  return SWL_OK;
}

// Checks the records' shapes against each other before anything is mapped.
int check_import_records(const swl_weight_ipc* recs, const int64_t* dims, int L) {
  const swl_weight_ipc& emb = recs[kRecsPerLayer * L];
  const swl_weight_ipc& lm = recs[kRecsPerLayer * L + 1];
  const int64_t hidden = emb.cols;
  if (emb.rows <= 0 || hidden <= 0 || lm.rows != emb.rows || lm.cols != hidden)
    return set_error(SWL_ERR_ARG, "import_weights_from_ipc: embed / lm_head shapes disagree");
  for (int l = 0; l < L; ++l) {
    const swl_weight_ipc* r = recs + kRecsPerLayer * l;
    const int64_t* d = dims + 5 * l;
    for (int j = 0; j < 5; ++j)
      if (d[j] <= 0) return set_error(SWL_ERR_ARG, "import_weights_from_ipc: layer %d has a dimension <= 0", l);
    const int64_t inter = r[3].cols;
    const bool ok = r[0].rows == d[0] + d[1] + d[2] && r[0].cols == hidden && r[1].rows > 0 &&
                    r[1].cols == hidden && r[2].rows == d[3] + d[4] && r[2].cols == hidden &&
                    r[3].rows > 0 && inter > 0 && (r[4].rows == 0 || (r[4].rows == r[1].rows && r[4].cols == 1)) &&
                    (r[5].rows == 0 || (r[5].rows == r[3].rows && r[5].cols == 1));
    if (!ok) return set_error(SWL_ERR_ARG, "import_weights_from_ipc: layer %d shapes disagree", l);
  }
  return SWL_OK;
}

// import_weights_from_ipc (ext_aggregator.cpp:1294-1406).
SWL_EXPORT int swl_agg_import_weights(const swl_weight_ipc* recs, int count, const int64_t* dims,
                                      int num_layers, int device_index) {
  if (!recs || !dims || num_layers <= 0 || count != kRecsPerLayer * num_layers + 2)
    return set_error(SWL_ERR_ARG, "import_weights_from_ipc: expected %d records for %d layers",
                     kRecsPerLayer * num_layers + 2, num_layers);
  SWL_TRY(check_import_records(recs, dims, num_layers));
  SWL_CUDA_TRY(cudaSetDevice(device_index));
  SWL_TRY(free_weights());
  g_device = device_index;
  SWL_TRY(ensure_stream());
  std::vector<size_t> at(count, 0);
  size_t total = 0;
  for (int i = 0; i < count; ++i) {
    if (recs[i].rows <= 0) continue;
    at[i] = total;
    total += (static_cast<size_t>(recs[i].rows) * recs[i].cols * 2 + kArenaAlign - 1) / kArenaAlign * kArenaAlign;
  }
  SWL_CUDA_TRY(cudaMalloc(&g_arena, total));
  struct Mapped { cudaIpcMemHandle_t h; char* base; size_t size; };
  std::vector<Mapped> maps;
  int st = SWL_OK;
  for (int i = 0; st == SWL_OK && i < count; ++i) {
    const swl_weight_ipc& rec = recs[i];
    if (rec.rows <= 0) continue;
    const Mapped* m = nullptr;
    for (const Mapped& x : maps)
      if (!memcmp(&x.h, rec.handle, sizeof(x.h))) m = &x;
    if (!m) {
      Mapped x;
      memcpy(&x.h, rec.handle, sizeof(x.h));
      void* p = nullptr;
      cudaError_t e = cudaIpcOpenMemHandle(&p, x.h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        st = set_error(SWL_ERR_CUDA, "import_weights_from_ipc: mapping record %d failed: %s", i, cudaGetErrorString(e));
        break;
      }
      x.base = static_cast<char*>(p);
      char* b2 = nullptr;
      size_t n2 = 0;
      st = allocation_of(p, &b2, &n2);
      x.size = st == SWL_OK ? static_cast<size_t>(b2 + n2 - x.base) : 0;  // bytes mapped from x.base on
      maps.push_back(x);
      if (st != SWL_OK) break;
      m = &maps.back();
    }
    const size_t bytes = static_cast<size_t>(rec.rows) * rec.cols * 2;
    if (rec.offset > m->size || bytes > m->size - rec.offset) {
      st = set_error(SWL_ERR_ARG, "import_weights_from_ipc: record %d (%zu bytes at %llu) lies outside its %zu-byte allocation",
                     i, bytes, static_cast<unsigned long long>(rec.offset), m->size);
      break;
    }
    cudaError_t e = cudaMemcpyAsync(static_cast<char*>(g_arena) + at[i], m->base + rec.offset, bytes,
                                    cudaMemcpyDefault, g_stream);
    if (e != cudaSuccess) st = set_error(SWL_ERR_CUDA, "import_weights_from_ipc: copy of record %d failed: %s", i, cudaGetErrorString(e));
  }
  cudaError_t se = cudaStreamSynchronize(g_stream);
  if (st == SWL_OK && se != cudaSuccess)
    st = set_error(SWL_ERR_CUDA, "import_weights_from_ipc: copies failed: %s", cudaGetErrorString(se));
  for (const Mapped& x : maps) cudaIpcCloseMemHandle(x.base);
  if (st != SWL_OK) {
    const std::string why = last_error();
    cudaFree(g_arena);
    g_arena = nullptr;
    g_layers.clear();
    g_num_layers = 0;
    return set_error(st, "%s", why.c_str());
  }
  char* arena = static_cast<char*>(g_arena);
  g_layers.assign(num_layers, Layer());
  g_num_layers = num_layers;
  const int64_t hidden = recs[kRecsPerLayer * num_layers].cols;
  for (int l = 0; l < num_layers && st == SWL_OK; ++l) {
    Layer& L = g_layers[l];
    const swl_weight_ipc* r = recs + kRecsPerLayer * l;
    const size_t* a = at.data() + kRecsPerLayer * l;
    const int64_t* d = dims + 5 * l;
    L.owns_fused = false;
    L.q_dim = d[0]; L.k_dim = d[1]; L.v_dim = d[2]; L.gate_dim = d[3]; L.up_dim = d[4];
    L.hidden = hidden; L.inter = r[3].cols; L.o_out = r[1].rows; L.down_out = r[3].rows;
    L.qkv = arena + a[0];
    L.o = arena + a[1];
    L.gu = arena + a[2];
    L.down = arena + a[3];
    L.o_bias = r[4].rows ? arena + a[4] : nullptr;
    L.down_bias = r[5].rows ? arena + a[5] : nullptr;
    st = encode_weight_tmap(&L.tm_qkv, L.qkv, r[0].rows, hidden);
    if (st == SWL_OK) st = encode_weight_tmap(&L.tm_o, L.o, L.o_out, hidden);
    if (st == SWL_OK) st = encode_weight_tmap(&L.tm_gu, L.gu, r[2].rows, hidden);
    if (st == SWL_OK) st = encode_weight_tmap(&L.tm_down, L.down, L.down_out, L.inter);
  }
  if (st != SWL_OK) return st;
  g_weights_ready = true;
  const int64_t vocab = recs[kRecsPerLayer * num_layers].rows;
  g_embed = arena + at[kRecsPerLayer * num_layers];
  g_lm_head = arena + at[kRecsPerLayer * num_layers + 1];
  g_vocab = vocab;
  g_embed_hidden = hidden;
  SWL_TRY(encode_weight_tmap(&g_tm_lm, g_lm_head, vocab, hidden));
  if (g_logits) cudaFree(g_logits);
  g_logits = nullptr;
  SWL_CUDA_TRY(cudaMalloc(&g_logits, static_cast<size_t>(kMaxSlots) * vocab * 2));
  g_vocab_ready = true;
  return SWL_OK;
}

// ===== device-published round completion =======================================
//
// Completion mode 0 (the reference, ext_aggregator.cpp:1196-1202): after a
// round's launches the main loop synchronizes the stream, then bumps the
// epoch on the host. Mode 1: the control block is registered with CUDA as
// mapped host memory, and after the round's kernels the loop enqueues a
// one-thread kernel that stores the round's epoch into barrier_done_epoch;
// the loop does not wait, so the workers see the epoch as soon as the round
// has finished on the GPU while the host already waits for the next round's
// ready bits (agg_protocol.h, deferred completion).
namespace {
int g_completion_mode = 0;
bool g_round_graphs = false;
void* g_ctrl_registered = nullptr;  // the mapping registered with cudaHostRegister
size_t g_ctrl_registered_bytes = 0;
int64_t* g_epoch_dev = nullptr;     // device address of barrier_done_epoch

// Launched in stream order without programmatic serialization: it starts
// after every earlier kernel on the stream has completed.
__global__ void publish_epoch_kernel(int64_t* epoch, int64_t value) {
  __threadfence_system();
  asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(epoch), "l"(value) : "memory");
}

void unregister_ctrl() {
  if (g_ctrl_registered) {
    cudaHostUnregister(g_ctrl_registered);
    cudaGetLastError();
  }
  g_ctrl_registered = nullptr;
  g_ctrl_registered_bytes = 0;
  g_epoch_dev = nullptr;
}

int register_ctrl() {
  if (!g_ctrl) return set_error(SWL_ERR_STATE, "completion mode: aggregator queue not initialized");
  if (g_ctrl_registered == g_ctrl && g_epoch_dev) return SWL_OK;
  unregister_ctrl();
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  const size_t page = static_cast<size_t>(sysconf(_SC_PAGESIZE));
  const size_t len = (g_map_bytes + page - 1) / page * page;  // the mapping starts on a page
  cudaError_t e = cudaHostRegister(g_ctrl, len, cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(SWL_ERR_CUDA, "completion mode: registering the control block failed: %s",
                     cudaGetErrorString(e));
  }
  void* d = nullptr;
  e = cudaHostGetDevicePointer(&d, &g_ctrl->barrier_done_epoch, 0);
  if (e != cudaSuccess || !d) {
    cudaHostUnregister(g_ctrl);
    cudaGetLastError();
    return set_error(SWL_ERR_CUDA, "completion mode: no device address for the control block: %s",
                     cudaGetErrorString(e));
  }
  g_ctrl_registered = g_ctrl;
  g_ctrl_registered_bytes = len;
  g_epoch_dev = static_cast<int64_t*>(d);
  return SWL_OK;
}
}  // namespace

// Event completion (mode 2). Every slot's worker records a CUDA event after
// the work that writes the slot's round input and only then sets its ready
// bit; the round's stream waits for those events, the round's kernels are
// enqueued, the round event is recorded after them, and the host bumps the
// epoch at once. A worker that sees the epoch makes its stream wait for the
// round event before it reads the outputs. Neither side's host waits for the
// GPU; the GPU orders the work by stream-level event dependencies. Only for
// workers that follow this (swl_wc_* clients, or a worker that registers
// its input event and waits for the round event).
namespace {
cudaEvent_t g_round_event = nullptr;

int ensure_round_event() {
  if (g_round_event) return SWL_OK;
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  SWL_CUDA_TRY(cudaEventCreateWithFlags(&g_round_event, cudaEventDisableTiming | cudaEventInterprocess));
  return SWL_OK;
}

int slot_for_event(int slot_id, Slot** out) {
  if (!g_pool.initialized || slot_id < 0 || slot_id >= g_pool.num_slots)
    return set_error(SWL_ERR_ARG, "input event: invalid slot %d", slot_id);
  *out = &g_pool.slots[slot_id];
  if ((*out)->input_event && (*out)->input_event_owned) cudaEventDestroy((*out)->input_event);
  (*out)->input_event = nullptr;
  (*out)->input_event_owned = false;
  return SWL_OK;
}
}  // namespace

// The round event's IPC handle (64 bytes), for workers in other processes
// (cudaIpcOpenEventHandle).
SWL_EXPORT int swl_agg_round_event_handle(unsigned char* out, size_t len) {
  if (!out || len < sizeof(cudaIpcEventHandle_t)) return set_error(SWL_ERR_ARG, "round event: 64-byte buffer needed");
  SWL_TRY(ensure_round_event());
  cudaIpcEventHandle_t h;
  SWL_CUDA_TRY(cudaIpcGetEventHandle(&h, g_round_event));
  memcpy(out, &h, sizeof(h));
  return SWL_OK;
}

// The round event itself (cudaEvent_t), for workers in this process.
SWL_EXPORT int swl_agg_round_event(void** event) {
  if (!event) return set_error(SWL_ERR_ARG, "round event: null pointer");
  SWL_TRY(ensure_round_event());
  *event = g_round_event;
  return SWL_OK;
}

// A slot's input event from its worker's IPC handle (a worker in another
// process), or (len 0, handle NULL) none.
SWL_EXPORT int swl_agg_set_slot_input_event(int slot_id, const unsigned char* handle, size_t len) {
  Slot* s = nullptr;
  SWL_TRY(slot_for_event(slot_id, &s));
  if (!handle || len == 0) return SWL_OK;
  if (len != sizeof(cudaIpcEventHandle_t)) return set_error(SWL_ERR_ARG, "input event: handle of 64 bytes expected");
  cudaIpcEventHandle_t h;
  memcpy(&h, handle, sizeof(h));
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  SWL_CUDA_TRY(cudaIpcOpenEventHandle(&s->input_event, h));
  s->input_event_owned = true;
  return SWL_OK;
}

// A slot's input event created in this process (not owned; NULL = none).
SWL_EXPORT int swl_agg_set_slot_input_event_local(int slot_id, void* event) {
  Slot* s = nullptr;
  SWL_TRY(slot_for_event(slot_id, &s));
  s->input_event = static_cast<cudaEvent_t>(event);
  return SWL_OK;
}

// 0: the host signals each round after a stream sync (the reference);
// 1: the device publishes each round's epoch (needs the queue mapped by
// swl_agg_init_queue; registers it); 2: event completion (above). Takes
// effect at the next main loop.
SWL_EXPORT int swl_agg_set_completion_mode(int mode) {
  if (mode < 0 || mode > 2) return set_error(SWL_ERR_ARG, "completion mode must be 0, 1 or 2");
  if (mode == 1) SWL_TRY(register_ctrl());
  if (mode == 2) SWL_TRY(ensure_round_event());
  g_completion_mode = mode;
  return SWL_OK;
}

SWL_EXPORT int swl_agg_completion_mode(void) { return g_completion_mode; }

// Under event completion: 1 replays each (op, layer) round from a CUDA graph
// (the input-event waits, the round's kernels and the round event's record),
// captured when the same slots send the same rows a second time; the LM-head
// round always runs eagerly. Takes effect at the next main loop.
SWL_EXPORT int swl_agg_set_round_graphs(int on) {
  g_round_graphs = on != 0;
  return SWL_OK;
}

// ext_aggregator.cpp:427-459 init_aggregator_queue: map the queue segment
// created by ext_ipc_queue.create_queue (this module's own view).
SWL_EXPORT int swl_agg_init_queue(const char* shm_name, int capacity) {
  if (capacity <= 0) return set_error(SWL_ERR_ARG, "init_aggregator_queue: capacity must be positive");
  if (!shm_name || !shm_name[0]) return set_error(SWL_ERR_ARG, "init_aggregator_queue: shm_name cannot be empty");
  int fd = shm_open(shm_name, O_RDWR, 0600);
  if (fd < 0) return set_error(SWL_ERR_SYS, "Failed to open shared memory: %s", shm_name);
  size_t bytes = shm_bytes(capacity);
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return set_error(SWL_ERR_SYS, "Failed to mmap shared memory");
  unregister_ctrl();
  g_completion_mode = 0;  // a new segment starts with host completion
  if (g_ctrl) munmap(g_ctrl, g_map_bytes);
  g_ctrl = static_cast<ControlBlock*>(p);
  g_ring = reinterpret_cast<Command*>(static_cast<char*>(p) + sizeof(ControlBlock));
  g_capacity = capacity;
  g_map_bytes = bytes;
  return SWL_OK;
}

// Sampling state of a worker for in-process drivers (the protocol sets it
// with OP_SET_SAMPLING or slot_set_pending_sampling).
SWL_EXPORT int swl_agg_set_worker_sampling(int worker_id, int do_sample, float temperature, int top_k,
                                           float top_p) {
  if (worker_id < 0 || worker_id > 100000) return set_error(SWL_ERR_ARG, "set_worker_sampling: invalid worker_id");
  std::lock_guard<std::mutex> lock(g_sampling_mu);
  g_sampling[worker_id] = {do_sample != 0, temperature, top_k, top_p};
  return SWL_OK;
}

// Seed of the LM-head sampling; the draw offset restarts at 0.
SWL_EXPORT int swl_agg_set_sampling_seed(uint64_t seed) {
  g_sample_seed.store(seed);
  g_sample_offset.store(0);
  return SWL_OK;
}

// Round kernel selection: 0 auto (cluster split-K), 1 cluster split-K,
// 2 CUDA cores, 3 stream-K (<= 64 rows); splits <= 0 = automatic K split for
// the cluster kernel.
SWL_EXPORT int swl_agg_set_round_algo(int algo, int splits) {
  if (algo < 0 || algo > 3) return set_error(SWL_ERR_ARG, "unknown round algo %d", algo);
  g_round_algo = algo;
  g_round_splits = splits;
  return SWL_OK;
}

// The fused weight of (layer, op) and its [N, K] shape, for callers that
// check a round against their own reference; OP_EMBED / OP_LM_HEAD give the
// [vocab, hidden] tables (layer ignored).
SWL_EXPORT int swl_agg_weight(int layer, int op, const void** W, int64_t* N, int64_t* K) {
  if (op == kOpEmbed || op == kOpLmHead) {
    if (!g_vocab_ready) return set_error(SWL_ERR_STATE, "weight: embed/lm_head not initialized");
    *W = op == kOpEmbed ? g_embed : g_lm_head;
    *N = g_vocab;
    *K = g_embed_hidden;
    return SWL_OK;
  }
  if (layer < 0 || layer >= g_num_layers) return set_error(SWL_ERR_ARG, "weight: bad layer");
  const Layer& L = g_layers[layer];
  switch (op) {
    case kOpQkvFused: *W = L.qkv; *N = L.q_dim + L.k_dim + L.v_dim; *K = L.hidden; break;
    case kOpOProj: *W = L.o; *N = L.o_out; *K = L.hidden; break;
    case kOpGateUpFused: *W = L.gu; *N = L.gate_dim + L.up_dim; *K = L.hidden; break;
    case kOpDownProj: *W = L.down; *N = L.down_out; *K = L.inter; break;
    default: return set_error(SWL_ERR_ARG, "weight: bad op");
  }
  return SWL_OK;
}

// One round over pool slots, asynchronously on `stream` (NULL = the
// library's own stream, then synchronised). Slot i of the round has
// bx[i] * tx[i] token rows in its input buffer. Ownership and buffer bounds
// are checked first; any failure rejects the whole call with an error. This
// is the unit the main loop runs per op (ext_aggregator.cpp:1187-1193).
SWL_EXPORT int swl_agg_execute_round(int op, int layer, int n, const int* slot_ids,
                                     const int* worker_ids, const int64_t* bx, const int64_t* tx,
                                     void* stream) {
  if (!g_pool.initialized) return set_error(SWL_ERR_STATE, "execute_round: slot pool not initialized");
  if (op != kOpEmbed && op != kOpLmHead && !g_weights_ready)
    return set_error(SWL_ERR_STATE, "execute_round: weights not initialized");
  if (n < 0 || n > g_pool.num_slots) return set_error(SWL_ERR_ARG, "execute_round: bad slot count %d", n);
  std::vector<RoundCmd> cmds(n);
  for (int i = 0; i < n; ++i) {
    if (bx[i] <= 0 || tx[i] <= 0 || bx[i] > 65536 || tx[i] > 65536)
      return set_error(SWL_ERR_ARG, "execute_round: invalid bx/tx dimensions");
    cmds[i] = {slot_ids[i], worker_ids[i], bx[i] * tx[i]};
  }
  int64_t in_row, out_row;
  row_bytes_for(op, layer, &in_row, &out_row);
  std::vector<RoundCmd> good;
  std::vector<int> bad;
  std::string why;
  validate(cmds.data(), n, in_row, out_row, &good, &bad, &why);
  if (static_cast<int>(good.size()) != n) return set_error(SWL_ERR_OWNER, "execute_round: %s", why.c_str());
  // A null stream is the legacy default stream (torch's default): the round
  // runs there, ordered after whatever the caller queued on it, and the call
  // returns once it is done.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SWL_TRY(run_round(op, layer, good, st));
  if (st == nullptr) SWL_CUDA_TRY(cudaStreamSynchronize(st));
  return SWL_OK;
}

// The QKV round of `layer` over the given slots fused with the RoPE epilogue
// (swl_fused_qkv_rope's arguments, table entry i = command i): each round
// tile adds its head's LoRA delta, applies RoPE and writes rotated q to
// q_rot and the new token's k / v into the caches; the QKV slot outputs are
// not written. Above kQkvRopeMaxRows rows, or with column-sharded weights,
// it runs as the round followed by the separate RoPE epilogue (which then
// also leaves the round output in the slot outputs), with the same results.
SWL_EXPORT int swl_agg_execute_qkv_rope_round(int layer, int n, const int* slot_ids, const int* worker_ids,
                                              const int64_t* bx, const int64_t* tx, const void* const* B,
                                              int r, const float* ws_in, int splits_in,
                                              const void* const* block_tables, void* const* k_cache,
                                              void* const* v_cache, const void* const* seqlens, int hq,
                                              int hkv, int head_dim, int page, const void* cos_sin,
                                              void* q_rot, void* stream) {
  if (!g_pool.initialized || !g_weights_ready)
    return set_error(SWL_ERR_STATE, "qkv/rope round: pool or weights not initialized");
  if (n <= 0 || n > g_pool.num_slots || !slot_ids || !worker_ids || !bx || !tx || !block_tables || !k_cache ||
      !v_cache || !seqlens)
    return set_error(SWL_ERR_ARG, "qkv/rope round: invalid arguments");
  if (layer < 0 || layer >= g_num_layers)
    return set_error(SWL_ERR_ARG, "qkv/rope round: layer_idx %d out of range [0, %d)", layer, g_num_layers);
  if (head_dim != 128) return set_error(SWL_ERR_ARG, "qkv/rope round: head_dim must be 128");
  std::vector<RoundCmd> cmds(n);
  for (int i = 0; i < n; ++i) {
    if (bx[i] <= 0 || tx[i] <= 0 || bx[i] > 65536 || tx[i] > 65536)
      return set_error(SWL_ERR_ARG, "qkv/rope round: invalid bx/tx dimensions");
    cmds[i] = {slot_ids[i], worker_ids[i], bx[i] * tx[i]};
  }
  int64_t in_row, out_row;
  row_bytes_for(kOpQkvFused, layer, &in_row, &out_row);
  std::vector<RoundCmd> good;
  std::vector<int> bad;
  std::string why;
  validate(cmds.data(), n, in_row, out_row, &good, &bad, &why);
  if (static_cast<int>(good.size()) != n) return set_error(SWL_ERR_OWNER, "qkv/rope round: %s", why.c_str());
  const Layer& L = g_layers[layer];
  if (L.q_dim != static_cast<int64_t>(hq) * 128 || L.k_dim != static_cast<int64_t>(hkv) * 128 || L.v_dim != L.k_dim)
    return set_error(SWL_ERR_ARG, "qkv/rope round: head counts do not match the layer's q/k/v rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t rows = 0;
  for (const RoundCmd& c : good) rows += c.rows;
  if (rows > kQkvRopeMaxRows || g_shard.on || g_round_algo == kAlgoSimt || g_round_algo == kAlgoStreamK) {
    SWL_TRY(run_round(kOpQkvFused, layer, good, st));
    QkvRopeTable t;
    t.seg.nseg = n;
    int acc = 0;
    for (int i = 0; i < n; ++i) {
      const Slot& sl = g_pool.slots[good[i].slot_id];
      t.seg.row_start[i] = acc;
      acc += static_cast<int>(good[i].rows);
      t.base[i] = static_cast<const __nv_bfloat16*>(sl.out);
      t.B[i] = B ? static_cast<const __nv_bfloat16*>(B[i]) : nullptr;
      t.block_table[i] = static_cast<const int*>(block_tables[i]);
      t.k_cache[i] = static_cast<__nv_bfloat16*>(k_cache[i]);
      t.v_cache[i] = static_cast<__nv_bfloat16*>(v_cache[i]);
      t.seqlen[i] = static_cast<const int*>(seqlens[i]);
    }
    t.seg.row_start[n] = acc;
    t.seg.total_rows = acc;
    QkvRopeParams p{};
    p.hq = hq; p.hkv = hkv; p.head_dim = head_dim; p.page = page;
    p.base_stride = L.q_dim + L.k_dim + L.v_dim;
    p.ws_in = ws_in;
    p.splits_in = splits_in;
    p.cos_sin = static_cast<const __nv_bfloat16*>(cos_sin);
    p.q_rot = static_cast<__nv_bfloat16*>(q_rot);
    SWL_TRY(launch_qkv_rope(t, p, r, st));
  } else {
    SlotTable tab;
    QkvRopeEpi epi;
    tab.nslots = n;
    int acc = 0;
    for (int i = 0; i < n; ++i) {
      const Slot& sl = g_pool.slots[good[i].slot_id];
      tab.row_start[i] = acc;
      tab.in[i] = static_cast<const __nv_bfloat16*>(sl.in);
      tab.out[i] = static_cast<__nv_bfloat16*>(sl.out);
      acc += static_cast<int>(good[i].rows);
      epi.B[i] = B ? static_cast<const __nv_bfloat16*>(B[i]) : nullptr;
      epi.block_table[i] = static_cast<const int*>(block_tables[i]);
      epi.k_cache[i] = static_cast<__nv_bfloat16*>(k_cache[i]);
      epi.v_cache[i] = static_cast<__nv_bfloat16*>(v_cache[i]);
      epi.seqlen[i] = static_cast<const int*>(seqlens[i]);
    }
    for (int i = n; i < kMaxSlots; ++i) {
      epi.B[i] = nullptr;
      epi.block_table[i] = nullptr;
      epi.k_cache[i] = epi.v_cache[i] = nullptr;
      epi.seqlen[i] = nullptr;
    }
    tab.row_start[n] = acc;
    tab.total_rows = acc;
    epi.ws_in = ws_in;
    epi.splits_in = splits_in;
    epi.rank = r;
    epi.hq = hq;
    epi.hkv = hkv;
    epi.page = page;
    epi.cos_sin = static_cast<const __nv_bfloat16*>(cos_sin);
    epi.q_rot = static_cast<__nv_bfloat16*>(q_rot);
    const int64_t N = L.q_dim + L.k_dim + L.v_dim;
    RoundShape shape{N, L.hidden, L.hidden, N, nullptr};
    SWL_TRY(launch_slot_round_qkv_rope(tab, shape, L.qkv, &L.tm_qkv, epi, g_round_splits, st));
  }
  if (st == nullptr) SWL_CUDA_TRY(cudaStreamSynchronize(st));
  return SWL_OK;
}

// ===== column-sharded base weights (two GPUs) ==================================

// After the slot pool, the layers and the LM head are initialised: builds this
// GPU's row views of every fused weight and of the LM head (no copies) and
// allocates its sync words. rank is 0 or 1 of a pair of GPUs (world 2). The
// rounds stay unsharded until swl_agg_shard_connect has mapped the peer.
SWL_EXPORT int swl_agg_shard_begin(int rank, int world) {
  if (world != 2 || rank < 0 || rank > 1)
    return set_error(SWL_ERR_ARG, "shard: a pair of GPUs (world 2, rank 0 or 1) is supported");
  if (!g_pool.initialized || !g_weights_ready || !g_vocab_ready)
    return set_error(SWL_ERR_STATE, "shard: initialise the slot pool, the layers and the LM head first");
  SWL_TRY(shard_end());
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  g_shard.rank = rank;
  g_shard.layer.assign(g_num_layers, {});
  for (int l = 0; l < g_num_layers; ++l) {
    const Layer& L = g_layers[l];
    SWL_TRY(shard_view(&g_shard.layer[l][0], L.qkv, L.q_dim + L.k_dim + L.v_dim, L.hidden, rank));
    SWL_TRY(shard_view(&g_shard.layer[l][1], L.o, L.o_out, L.hidden, rank));
    SWL_TRY(shard_view(&g_shard.layer[l][2], L.gu, L.gate_dim + L.up_dim, L.hidden, rank));
    SWL_TRY(shard_view(&g_shard.layer[l][3], L.down, L.down_out, L.inter, rank));
  }
  SWL_TRY(shard_view(&g_shard.lm, g_lm_head, g_vocab, g_embed_hidden, rank));
  void* p = nullptr;
  SWL_CUDA_TRY(cudaMalloc(&p, kSyncWords * sizeof(unsigned int)));
  SWL_CUDA_TRY(cudaMemset(p, 0, kSyncWords * sizeof(unsigned int)));
  SWL_CUDA_TRY(cudaDeviceSynchronize());
  g_shard.sync = static_cast<unsigned int*>(p);
  return SWL_OK;
}

// IPC handles (64 bytes each) of this GPU's sync words, LM-head logits and
// slot output buffers (slot ids 0 .. num_slots-1), in that order, for the
// peer's swl_agg_shard_connect; *count = 2 + num_slots.
SWL_EXPORT int swl_agg_shard_handles(unsigned char* out, int max_handles, int* count) {
  if (!g_shard.sync) return set_error(SWL_ERR_STATE, "shard: call swl_agg_shard_begin first");
  const int need = 2 + g_pool.num_slots;
  if (count) *count = need;
  if (!out || max_handles < need) return set_error(SWL_ERR_ARG, "shard: room for %d handles needed", need);
  cudaIpcMemHandle_t h;
  SWL_CUDA_TRY(cudaIpcGetMemHandle(&h, g_shard.sync));
  memcpy(out, &h, sizeof(h));
  SWL_CUDA_TRY(cudaIpcGetMemHandle(&h, g_logits));
  memcpy(out + 64, &h, sizeof(h));
  for (int i = 0; i < g_pool.num_slots; ++i) memcpy(out + 64 * (2 + i), &g_pool.slots[i].out_handle, 64);
  return SWL_OK;
}

// Maps the peer's buffers from its handles (the layout of
// swl_agg_shard_handles) and switches every round to the sharded kernel.
// From then on both GPUs must run the same rounds in the same order: a
// round waits for the peer's (with a time limit, after which the kernel
// records an error that swl_round_device_error reports).
SWL_EXPORT int swl_agg_shard_connect(const unsigned char* peer, int count) {
  if (!g_shard.sync) return set_error(SWL_ERR_STATE, "shard: call swl_agg_shard_begin first");
  if (!peer || count != 2 + g_pool.num_slots)
    return set_error(SWL_ERR_ARG, "shard: expected %d peer handles", 2 + g_pool.num_slots);
  if (g_shard.on) return set_error(SWL_ERR_STATE, "shard: already connected");
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  auto open = [&](int i, void** ptr) -> int {
    cudaIpcMemHandle_t h;
    memcpy(&h, peer + 64 * i, sizeof(h));
    SWL_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return SWL_OK;
  };
  void* p = nullptr;
  int st = open(0, &p);
  g_shard.peer_sync = static_cast<unsigned int*>(p);
  if (st == SWL_OK) st = open(1, &g_shard.peer_logits);
  g_shard.peer_out.assign(g_pool.num_slots, nullptr);
  for (int i = 0; st == SWL_OK && i < g_pool.num_slots; ++i) st = open(2 + i, &g_shard.peer_out[i]);
  if (st != SWL_OK) {
    const std::string why = last_error();
    shard_end();
    return set_error(SWL_ERR_CUDA, "shard: mapping the peer's buffers failed: %s", why.c_str());
  }
  g_shard.on = true;
  return SWL_OK;
}

// Unmaps the peer's buffers and returns to unsharded rounds. Call it on both
// GPUs (and wait for both) before either frees its slot pool.
SWL_EXPORT int swl_agg_shard_end(void) { return shard_end(); }

// ===== main loop ===============================================================

namespace {

// ext_aggregator.cpp:991-1020 apply_pending_sampling_states.
void apply_pending_sampling(const Mask128& joins) {
  take_pending_sampling(g_ctrl, joins, [](int sid, const PendingSampling& p) {
    int wid = g_pool.slots[sid].owner.load(std::memory_order_acquire);
    if (wid >= 0) {
      std::lock_guard<std::mutex> lock(g_sampling_mu);
      g_sampling[wid] = {p.do_sample, p.temperature, p.top_k, p.top_p};
    }
  });
}

// The aggregator's side of run_main_loop: GPU rounds over validated
// commands, sampling state, the pool's copy of the active set.
struct AggHooks {
  std::vector<RoundCmd> all, good;
  void on_membership(const Mask128& active, const Mask128& joins) {
    if (!joins.empty()) apply_pending_sampling(joins);
    store_mask(g_pool.active_w, active);
    g_pool.active_slot_count.store(active.count());
  }
  void on_sampling(const DrainedCmd& c) {
    SamplingState s;
    s.do_sample = (c.x_key & 1) != 0;
    s.temperature = static_cast<float>(c.x_key >> 1) / 10000.0f;
    s.top_k = static_cast<int>(c.y0_key);
    s.top_p = static_cast<float>(c.y1_key) / 10000.0f;
    std::lock_guard<std::mutex> lock(g_sampling_mu);
    g_sampling[c.worker_id] = s;
  }
  void validate(int op, int layer, const std::vector<DrainedCmd>& cmds, std::vector<int>* bad) {
    all.clear();
    for (const DrainedCmd& c : cmds) all.push_back({c.slot_id, c.worker_id, c.rows});
    int64_t in_row, out_row;
    row_bytes_for(op, layer, &in_row, &out_row);
    std::string why;
    ::validate(all.data(), static_cast<int>(all.size()), in_row, out_row, &good, bad, &why);
    if (!why.empty()) fprintf(stderr, "[swl aggregator] dropping commands: %s\n", why.c_str());
    if (g_completion_mode == 2) {
      // event completion reads a slot's input only after its worker's event;
      // a slot without one cannot be ordered, so its command is refused
      size_t k = 0;
      for (const RoundCmd& c : good) {
        if (g_pool.slots[c.slot_id].input_event) {
          good[k++] = c;
        } else {
          bad->push_back(c.slot_id);
          fprintf(stderr, "[swl aggregator] slot %d has no input event under event completion; evicted\n",
                  c.slot_id);
        }
      }
      good.resize(k);
    }
  }
  bool deferred = false;  // device-published completion (mode 1)
  bool events = false;    // event completion (mode 2)
  bool graphs = false;    // event completion: replay each (op, layer) round from a CUDA graph
  std::vector<cudaEvent_t> waits;
  // A round's graph: the waits for its slots' input events, its kernels, the
  // round event's record; valid while the same slots send the same rows
  // with the same events (the steady state of decode).
  struct RoundGraph {
    std::vector<int> slots;
    std::vector<int64_t> rows;
    std::vector<cudaEvent_t> events;
    int seen = 0;  // eager runs of this command set (capture after the first)
    cudaGraphExec_t exec = nullptr;
  };
  std::map<std::pair<int, int>, RoundGraph> graph_cache;
  ~AggHooks() {
    for (auto& kv : graph_cache)
      if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  }
  bool deferred_epoch() const { return deferred; }
  void flush() {
    if (deferred || events) cudaStreamSynchronize(g_stream);
  }
  // The cached graph of this round if it matches the commands, capturing it
  // when the same command set comes a second time; nullptr = run eagerly.
  // The LM-head round is not cached: its sampling draws move every token.
  cudaGraphExec_t round_graph(int op, int layer) {
    if (!graphs || op == kOpLmHead) return nullptr;
    RoundGraph& g = graph_cache[{op, layer}];
    bool same = g.slots.size() == good.size() && g.events == waits;
    for (size_t i = 0; same && i < good.size(); ++i)
      same = g.slots[i] == good[i].slot_id && g.rows[i] == good[i].rows;
    if (!same) {
      if (g.exec) cudaGraphExecDestroy(g.exec);
      g = RoundGraph();
      for (const RoundCmd& c : good) {
        g.slots.push_back(c.slot_id);
        g.rows.push_back(c.rows);
      }
      g.events = waits;
    }
    if (g.exec) return g.exec;
    if (g.seen++ == 0) return nullptr;  // the first run sets the kernels' attributes outside any capture
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(g_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    bool ok = true;
    for (cudaEvent_t e : waits) ok = ok && cudaStreamWaitEvent(g_stream, e, cudaEventWaitExternal) == cudaSuccess;
    ok = ok && run_round(op, layer, good, g_stream) == SWL_OK;
    ok = ok && cudaEventRecordWithFlags(g_round_event, g_stream, cudaEventRecordExternal) == cudaSuccess;
    const bool ended = cudaStreamEndCapture(g_stream, &graph) == cudaSuccess;
    if (ok && ended && graph && cudaGraphInstantiate(&g.exec, graph, 0) != cudaSuccess) g.exec = nullptr;
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return g.exec;
  }
  int round(int op, int layer, const std::vector<DrainedCmd>&, const std::vector<int>&, int64_t epoch) {
    if (events) {
      waits.clear();
      for (const RoundCmd& c : good) {
        cudaEvent_t e = g_pool.slots[c.slot_id].input_event;
        if (std::find(waits.begin(), waits.end(), e) == waits.end()) waits.push_back(e);
      }
      if (cudaGraphExec_t exec = round_graph(op, layer)) {
        const cudaError_t e = cudaGraphLaunch(exec, g_stream);
        if (e == cudaSuccess) return SWL_OK;
        set_error(SWL_ERR_CUDA, "round: replaying the round graph: %s", cudaGetErrorString(e));
        fprintf(stderr, "[swl aggregator] %s\n", last_error());
        return SWL_ERR_CUDA;
      }
      for (cudaEvent_t e : waits) {
        const cudaError_t err = cudaStreamWaitEvent(g_stream, e, 0);
        if (err != cudaSuccess) {
          set_error(SWL_ERR_CUDA, "round: waiting for a worker's input event: %s", cudaGetErrorString(err));
          fprintf(stderr, "[swl aggregator] %s\n", last_error());
          return SWL_ERR_CUDA;
        }
      }
    }
    int st = run_round(op, layer, good, g_stream);
    if (st == SWL_OK && events) {
      const cudaError_t e = cudaEventRecord(g_round_event, g_stream);
      if (e != cudaSuccess) st = set_error(SWL_ERR_CUDA, "round: recording the round event: %s", cudaGetErrorString(e));
    } else if (st == SWL_OK && deferred) {
      publish_epoch_kernel<<<1, 1, 0, g_stream>>>(g_epoch_dev, epoch);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) st = set_error(SWL_ERR_CUDA, "round: publishing the epoch: %s", cudaGetErrorString(e));
    } else if (st == SWL_OK) {
      cudaError_t e = cudaStreamSynchronize(g_stream);
      if (e != cudaSuccess) st = set_error(SWL_ERR_CUDA, "round: %s", cudaGetErrorString(e));
    }
    if (st != SWL_OK) fprintf(stderr, "[swl aggregator] round op=%d layer=%d failed: %s\n", op, layer, last_error());
    return st;
  }
};

}  // namespace

// ext_aggregator.cpp:1024-1210 aggregator_main_loop_slots. Blocking; the
// Python binding calls it without the GIL. Joins/leaves are applied at token
// boundaries; each token is 1 + 4 * num_layers + 1 rounds.
SWL_EXPORT int swl_agg_main_loop_slots(int num_slots, int dtype_code) {
  (void)num_slots;
  if (!g_ctrl || !g_ring) return set_error(SWL_ERR_STATE, "Aggregator queue not initialized");
  if (!g_weights_ready) return set_error(SWL_ERR_STATE, "Aggregator weights not initialized");
  if (!g_pool.initialized) return set_error(SWL_ERR_STATE, "Slot pool not initialized");
  if (dtype_code != 15) return set_error(SWL_ERR_ARG, "only bf16 (dtype_code 15) is supported");
  SWL_CUDA_TRY(cudaSetDevice(g_device));
  SWL_TRY(ensure_stream());
  AggHooks hooks;
  if (g_completion_mode == 1) {
    SWL_TRY(register_ctrl());
    hooks.deferred = true;
  } else if (g_completion_mode == 2) {
    SWL_TRY(ensure_round_event());
    hooks.events = true;
    hooks.graphs = g_round_graphs;
  }
  const int st = run_main_loop(g_ctrl, g_ring, g_capacity, 1 + g_num_layers * 4 + 1, hooks);
  if (st == SWL_OK && (hooks.deferred || hooks.events)) {
    cudaError_t e = cudaStreamSynchronize(g_stream);
    if (e != cudaSuccess) return set_error(SWL_ERR_CUDA, "main loop: %s", cudaGetErrorString(e));
  }
  return st;
}
