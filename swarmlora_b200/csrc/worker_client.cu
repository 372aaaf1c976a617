// A native worker client of the aggregator's slot protocol.
//
// The reference runs every adapter worker as its own process whose engine
// thread makes, per generated token, the worker's 1 + 4L + 1 requests to the
// aggregator (worker_sync.py:1274-1425, _generate_one_token_all) through
// BatchedAggregatorOps (worker_sync.py:230-389): per round it copies its
// activation into its slot (prepare_input_slot: memcpy + stream sync),
// captures the epoch, submits one command per slot, sets the slots' ready
// bits, computes the LoRA delta while the aggregator runs, waits for the
// epoch to move, then reads the slot output and adds the delta, the residual
// and so on.
//
// This client does the same protocol for the slots it owns, from one host
// thread, with this library's worker kernels between the rounds: the fused
// epilogue kernels read each round's output in place from the slot output
// buffer and write the next round's input straight into the slot input
// buffer (no copies), carrying the LoRA shrink of that input so the expand
// is one pass over the round's output. The rounds themselves are requested
// exactly as the reference's worker requests them: epoch captured before the
// ready bits, one command per slot, ready bits, wait for the epoch.
//
// Before the ready bits the host must know that the round's input has been
// written. Input mode 0 waits the way the reference's prepare_input_slot
// does (cudaStreamSynchronize). Input mode 1 ends the epilogue with a
// one-thread kernel that stores a sequence number into pinned host memory
// and polls it (no driver call while polling, so many client threads do not
// contend inside the driver). Input mode 2 goes with the aggregator's event
// completion (swl_agg_set_completion_mode(2)): the client records its input
// event after the epilogue and sets the ready bits without waiting; once the
// epoch moves its stream waits for the aggregator's round event before the
// next kernels read the round's outputs. The host never waits for the GPU
// inside a token.
#include <chrono>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "common.h"
#include "shm_abi.h"
#include "swarmlora_b200.h"

using namespace swl;

namespace {

struct WcLayer {
  const void* in_norm = nullptr;
  const void* post_norm = nullptr;
  std::vector<void*> k_cache, v_cache;
  std::vector<const void*> A_qkv, B_qkv, A_o, B_o, A_gu, B_gu, A_dn, B_dn;
};

struct WorkerClient {
  int n = 0;
  std::vector<int> slot_ids, worker_ids;
  int layers = 0, hidden = 0, inter = 0, hq = 0, hkv = 0, head_dim = 0, page = 0, rank = 0, max_len = 0;
  float eps = 0.f, scaling = 0.f;
  int norm_splits = 0, dn_splits = 0;
  std::vector<int> rows;
  std::vector<int64_t> tok_bytes;
  std::vector<void*> slot_in, slot_out, h_rows, tokens;
  std::vector<const void*> block_tables, seqlens;
  int* seqlen_base = nullptr;  // the slots' positions, contiguous int32
  void* q_rot = nullptr;
  float *part = nullptr, *ws_qkv = nullptr, *ws_o = nullptr, *ws_gu = nullptr, *ws_dn = nullptr;
  const void* cos_sin = nullptr;
  const void* final_norm = nullptr;
  void* history = nullptr;  // optional int64 [tokens][n]: each token's picks
  std::vector<WcLayer> L;
  bool buffers_set = false;
  cudaStream_t stream = nullptr;
  int input_mode = 0;
  cudaEvent_t input_event = nullptr;  // mode 2: recorded after each round's input
  cudaEvent_t round_event = nullptr;  // mode 2: the aggregator's, recorded after each round
  bool use_graphs = false;            // mode 2: one CUDA graph per segment between rounds
  std::vector<cudaGraphExec_t> graphs;
  uint32_t* flag_host = nullptr;
  uint32_t* flag_dev = nullptr;
  uint32_t flag_seq = 0;
  int64_t timeout_ms = 30000;
  int64_t rounds_done = 0;
};

__global__ void input_ready_kernel(uint32_t* flag, uint32_t seq) {
  __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(seq) : "memory");
}

int check_client(const WorkerClient* c) {
  if (!c) return set_error(SWL_ERR_ARG, "worker client: null handle");
  if (!c->buffers_set) return set_error(SWL_ERR_STATE, "worker client: buffers not set");
  for (int l = 0; l < c->layers; ++l)
    if (c->L[l].k_cache.empty() || !c->L[l].in_norm)
      return set_error(SWL_ERR_STATE, "worker client: layer %d not set", l);
  if (!c->final_norm) return set_error(SWL_ERR_STATE, "worker client: final norm not set");
  return SWL_OK;
}

// The round's input is in the slot input buffers once the work enqueued so
// far has run.
int wait_input_written(WorkerClient* c) {
  if (c->input_mode == 0) {
    SWL_CUDA_TRY(cudaStreamSynchronize(c->stream));
    return SWL_OK;
  }
  if (c->input_mode == 2) {
    SWL_CUDA_TRY(cudaEventRecord(c->input_event, c->stream));
    return SWL_OK;
  }
  const uint32_t seq = ++c->flag_seq;
  input_ready_kernel<<<1, 1, 0, c->stream>>>(c->flag_dev, seq);
  SWL_CUDA_TRY(cudaGetLastError());
  const volatile uint32_t* f = c->flag_host;
  auto t0 = std::chrono::steady_clock::now();
  long spins = 0;
  while (static_cast<int32_t>(*f - seq) < 0) {
    if (++spins < kSpinPause) continue;
    cpu_relax();
    if ((spins & 4095) == 0) {
      const cudaError_t e = cudaStreamQuery(c->stream);
      if (e != cudaSuccess && e != cudaErrorNotReady)
        return set_error(SWL_ERR_CUDA, "worker client: %s", cudaGetErrorString(e));
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(c->timeout_ms))
        return set_error(SWL_ERR_TIMEOUT, "worker client: input of a round not written within %lld ms",
                         static_cast<long long>(c->timeout_ms));
    }
  }
  return SWL_OK;
}

// Rounds of one token: EMBED, per layer QKV / O / Gate+Up / Down, LM_HEAD.
int rounds_per_token(const WorkerClient* c) { return 4 * c->layers + 2; }

void round_of(const WorkerClient* c, int i, int* op, int* layer, int64_t* dx) {
  if (i == 0) {
    *op = kOpEmbed, *layer = 0, *dx = c->hidden;
    return;
  }
  if (i == rounds_per_token(c) - 1) {
    *op = kOpLmHead, *layer = 0, *dx = c->hidden;
    return;
  }
  const int l = (i - 1) / 4;
  *layer = l;
  switch ((i - 1) % 4) {
    case 0: *op = kOpQkvFused, *dx = c->hidden; break;
    case 1: *op = kOpOProj, *dx = static_cast<int64_t>(c->hq) * c->head_dim; break;
    case 2: *op = kOpGateUpFused, *dx = c->hidden; break;
    default: *op = kOpDownProj, *dx = c->inter; break;
  }
}

// One round through the protocol (BatchedAggregatorOps.*_submit_all +
// barrier_sync, worker_sync.py:250-389), for every slot of the client. With
// `launched` the segment just enqueued already ends with the input event
// and the next one starts by waiting for the round event (per-segment graphs).
int protocol_round(WorkerClient* c, int op, int layer, int64_t dx, bool launched = false) {
  if (!launched) SWL_TRY(wait_input_written(c));
  const int64_t e0 = swl_q_get_barrier_done_epoch();
  for (int i = 0; i < c->n; ++i) {
    int st;
    const auto t0 = std::chrono::steady_clock::now();
    while ((st = swl_q_submit_slot_command(op, layer, c->slot_ids[i], c->worker_ids[i], 1, c->rows[i], dx, 0, 0,
                                           0, 0, 0)) == SWL_ERR_FULL) {
      // the ring drains as the aggregator takes commands; give up with the client's time limit
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(c->timeout_ms))
        return set_error(SWL_ERR_TIMEOUT, "worker client: command ring stayed full for %lld ms",
                         static_cast<long long>(c->timeout_ms));
      std::this_thread::yield();
    }
    SWL_TRY(st);
  }
  for (int i = 0; i < c->n; ++i) SWL_TRY(swl_q_slot_signal_ready(c->slot_ids[i]));
  int64_t e = 0;
  SWL_TRY(swl_q_wait_for_epoch(e0, c->timeout_ms, &e));
  for (int i = 0; i < c->n; ++i)
    if (swl_q_is_slot_evicted(c->slot_ids[i]))
      return set_error(SWL_ERR_STATE, "worker client: slot %d evicted by the aggregator", c->slot_ids[i]);
  // the round is enqueued, not finished: order the reads of its outputs after it
  if (c->input_mode == 2 && !launched) SWL_CUDA_TRY(cudaStreamWaitEvent(c->stream, c->round_event, 0));
  ++c->rounds_done;
  return SWL_OK;
}

// The launches between round i - 1 and round i of a token (segment 0: before
// the EMBED round; segment rounds_per_token: after the LM head), with this
// library's fused epilogues: the same sequence as the in-process engine's
// step. The epilogues read each round's output in place and write the next
// round's input straight into the slot input buffers.
int enqueue_segment(WorkerClient* c, int i, int t) {
  const int n = c->n;
  const int H = c->hidden, I = c->inter, D = c->head_dim, r = c->rank;
  const int64_t qkv_n = static_cast<int64_t>(c->hq + 2 * c->hkv) * D;
  void* st = c->stream;
  const int* rows = c->rows.data();
  void* const* out = c->slot_out.data();
  void* const* in = c->slot_in.data();
  void* const* h = c->h_rows.data();
  const int R = rounds_per_token(c);
  if (i == 0) return swl_copy_rows(n, c->tokens.data(), in, c->tok_bytes.data(), st);
  if (i == 1)
    return swl_fused_resid_norm_shrink(n, rows, out, H, nullptr, 0, 0.f, nullptr, 0, 0, h, H, c->L[0].in_norm, H,
                                       c->eps, in, H, c->L[0].A_qkv.data(), 3 * r, c->ws_qkv, nullptr, 0, st);
  if (i == R) {
    SWL_TRY(swl_copy_rows(n, out, c->tokens.data(), c->tok_bytes.data(), st));
    if (c->history) {
      std::vector<void*> dst(n);
      for (int k = 0; k < n; ++k) dst[k] = static_cast<int64_t*>(c->history) + static_cast<int64_t>(t) * n + k;
      SWL_TRY(swl_copy_rows(n, out, dst.data(), c->tok_bytes.data(), st));
    }
    return swl_advance_i32(c->seqlen_base, n, 1, st);
  }
  const int l = (i - 2) / 4;  // the layer of the round just finished
  const WcLayer& w = c->L[l];
  switch ((i - 2) % 4) {
    case 0:  // after QKV: LoRA expand + RoPE + K/V append, attention -> O input
      SWL_TRY(swl_fused_qkv_rope(n, rows, out, qkv_n, w.B_qkv.data(), r, c->ws_qkv, c->norm_splits,
                                 c->block_tables.data(), w.k_cache.data(), w.v_cache.data(), c->seqlens.data(), c->hq,
                                 c->hkv, D, c->page, c->cos_sin, c->q_rot, nullptr, 0, st));
      return swl_paged_attention_shrink(n, rows, c->block_tables.data(), w.k_cache.data(), w.v_cache.data(),
                                        c->seqlens.data(), in, static_cast<int64_t>(c->hq) * D, c->hq, c->hkv, D,
                                        c->page, 1.0f / sqrtf(static_cast<float>(D)), c->max_len, c->q_rot, c->part,
                                        w.A_o.data(), r, c->ws_o, nullptr, 0, st);
    case 1:  // after O: LoRA expand, + residual, RMSNorm -> Gate+Up input
      return swl_fused_resid_norm_shrink(n, rows, out, H, w.B_o.data(), r, c->scaling, c->ws_o, c->hq, 1, h, H,
                                         w.post_norm, H, c->eps, in, H, w.A_gu.data(), 2 * r, c->ws_gu, nullptr, 0,
                                         st);
    case 2:  // after Gate+Up: LoRA expand, SiLU * up -> Down input
      return swl_fused_gu_silu_shrink(n, rows, out, 2 * static_cast<int64_t>(I), w.B_gu.data(), r, c->ws_gu,
                                      c->norm_splits, I, in, I, w.A_dn.data(), r, c->ws_dn, nullptr, 0, st);
    default: {  // after Down: LoRA expand, + residual, next RMSNorm -> next QKV (or LM-head) input
      const bool last = l == c->layers - 1;
      return swl_fused_resid_norm_shrink(n, rows, out, H, w.B_dn.data(), r, c->scaling, c->ws_dn, c->dn_splits, 1,
                                         h, H, last ? c->final_norm : c->L[l + 1].in_norm, H, c->eps, in, H,
                                         last ? nullptr : c->L[l + 1].A_qkv.data(), 3 * r, c->ws_qkv, nullptr, 0,
                                         st);
    }
  }
}

void drop_graphs(WorkerClient* c) {
  for (cudaGraphExec_t g : c->graphs)
    if (g) cudaGraphExecDestroy(g);
  c->graphs.clear();
}

// Event mode with graphs: segment i (0 .. rounds_per_token - 1) captured
// once, as [wait for the round event] + launches + [record the input event]
// (segment 0 has no wait: it follows the token-end launches on the stream).
// Each segment is captured just before its first graphed launch, so a round
// waits for one capture, not the aggregator for a whole token's worth (which
// could outlast its barrier's eviction time).
int build_graph(WorkerClient* c, int i) {
  const int R = rounds_per_token(c);
  if (static_cast<int>(c->graphs.size()) != R) c->graphs.assign(R, nullptr);
  cudaGraph_t g = nullptr;
  SWL_CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  int st = SWL_OK;
  if (i > 0 && cudaStreamWaitEvent(c->stream, c->round_event, cudaEventWaitExternal) != cudaSuccess)
    st = set_error(SWL_ERR_CUDA, "worker client: capturing the round-event wait");
  if (st == SWL_OK) st = enqueue_segment(c, i, 0);
  if (st == SWL_OK && cudaEventRecordWithFlags(c->input_event, c->stream, cudaEventRecordExternal) != cudaSuccess)
    st = set_error(SWL_ERR_CUDA, "worker client: capturing the input-event record");
  const cudaError_t e = cudaStreamEndCapture(c->stream, &g);
  if (st != SWL_OK || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return st != SWL_OK ? st : set_error(SWL_ERR_CUDA, "worker client: capture: %s", cudaGetErrorString(e));
  }
  const cudaError_t ie = cudaGraphInstantiate(&c->graphs[i], g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) {
    c->graphs[i] = nullptr;
    return set_error(SWL_ERR_CUDA, "worker client: instantiating a segment graph: %s", cudaGetErrorString(ie));
  }
  return SWL_OK;
}

// One decode token for every slot of the client: the reference worker's
// per-token sequence, segment by segment, each round through the protocol.
// With graphs, every token after the first (eager) one launches each
// segment as its graph (the first eager token sets the kernels' attributes
// outside any capture).
int run_token(WorkerClient* c, int t) {
  const int R = rounds_per_token(c);
  const bool graphed = c->use_graphs && c->input_mode == 2 && c->rounds_done > 0;
  for (int i = 0; i < R; ++i) {
    int op, layer;
    int64_t dx;
    round_of(c, i, &op, &layer, &dx);
    if (graphed) {
      if (static_cast<int>(c->graphs.size()) != R || !c->graphs[i]) SWL_TRY(build_graph(c, i));
      SWL_CUDA_TRY(cudaGraphLaunch(c->graphs[i], c->stream));
    } else {
      SWL_TRY(enqueue_segment(c, i, t));
    }
    SWL_TRY(protocol_round(c, op, layer, dx, graphed));
  }
  // token end: the stream waits for the LM-head round before reading its picks
  if (graphed) SWL_CUDA_TRY(cudaStreamWaitEvent(c->stream, c->round_event, 0));
  return enqueue_segment(c, R, t);
}

}  // namespace

// Creates a client over `nslots` claimed slots (slot_ids / worker_ids as
// claimed from the aggregator). Shapes as the aggregator's model; `rank` the
// LoRA rank the adapters are packed at, `scaling` the O / Down scale applied
// after the expand, `max_len` the longest context any slot reaches.
SWL_EXPORT int swl_wc_create(int nslots, const int* slot_ids, const int* worker_ids, int layers, int hidden,
                             int inter, int hq, int hkv, int head_dim, int page, int rank, float eps,
                             float scaling, int max_len, void** out) {
  if (!out || nslots <= 0 || nslots > kMaxSlots || !slot_ids || !worker_ids || layers <= 0 || hidden <= 0 ||
      inter <= 0 || hq <= 0 || hkv <= 0 || head_dim <= 0 || page <= 0 || rank <= 0 || max_len <= 0)
    return set_error(SWL_ERR_ARG, "worker client: invalid arguments");
  auto* c = new WorkerClient();
  c->n = nslots;
  c->slot_ids.assign(slot_ids, slot_ids + nslots);
  c->worker_ids.assign(worker_ids, worker_ids + nslots);
  c->layers = layers;
  c->hidden = hidden;
  c->inter = inter;
  c->hq = hq;
  c->hkv = hkv;
  c->head_dim = head_dim;
  c->page = page;
  c->rank = rank;
  c->eps = eps;
  c->scaling = scaling;
  c->max_len = max_len;
  c->norm_splits = swl_fused_norm_splits(rank);
  c->dn_splits = swl_fused_silu_splits(inter);
  c->rows.assign(nslots, 1);
  c->tok_bytes.assign(nslots, 8);
  c->L.resize(layers);
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaHostAlloc(&c->flag_host, 64, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e == cudaSuccess) {
    *c->flag_host = 0;
    void* d = nullptr;
    e = cudaHostGetDevicePointer(&d, c->flag_host, 0);
    c->flag_dev = static_cast<uint32_t*>(d);
  }
  if (e != cudaSuccess) {
    if (c->stream) cudaStreamDestroy(c->stream);
    if (c->flag_host) cudaFreeHost(c->flag_host);
    delete c;
    return set_error(SWL_ERR_CUDA, "worker client: %s", cudaGetErrorString(e));
  }
  *out = c;
  return SWL_OK;
}

// Per-slot device buffers (arrays of nslots): the slot pool's input and
// output buffers, the hidden rows [max rows, hidden], the int64 token of each
// slot, block tables and int32 positions; `seqlen_base` is the slots'
// positions as one contiguous int32 array (the same memory as seqlens[i]).
// Scratch owned by the caller, sized for nslots rows: q_rot [n, hq*D] bf16,
// attention partials (swl_attention_part_floats), the shrink partials of the
// four rounds; the cos/sin cache and the final norm weight.
SWL_EXPORT int swl_wc_set_buffers(void* handle, void* const* slot_in, void* const* slot_out, void* const* h_rows,
                                  void* const* tokens, const void* const* block_tables,
                                  const void* const* seqlens, int* seqlen_base, void* q_rot, float* part,
                                  float* ws_qkv, float* ws_o, float* ws_gu, float* ws_dn, const void* cos_sin,
                                  const void* final_norm) {
  auto* c = static_cast<WorkerClient*>(handle);
  if (!c || !slot_in || !slot_out || !h_rows || !tokens || !block_tables || !seqlens || !seqlen_base || !q_rot ||
      !part || !ws_qkv || !ws_o || !ws_gu || !ws_dn || !cos_sin || !final_norm)
    return set_error(SWL_ERR_ARG, "worker client: null buffer");
  const int n = c->n;
  c->slot_in.assign(slot_in, slot_in + n);
  c->slot_out.assign(slot_out, slot_out + n);
  c->h_rows.assign(h_rows, h_rows + n);
  c->tokens.assign(tokens, tokens + n);
  c->block_tables.assign(block_tables, block_tables + n);
  c->seqlens.assign(seqlens, seqlens + n);
  c->seqlen_base = seqlen_base;
  c->q_rot = q_rot;
  c->part = part;
  c->ws_qkv = ws_qkv;
  c->ws_o = ws_o;
  c->ws_gu = ws_gu;
  c->ws_dn = ws_dn;
  c->cos_sin = cos_sin;
  c->final_norm = final_norm;
  c->buffers_set = true;
  return SWL_OK;
}

// One layer: the two RMSNorm weights, each slot's K / V cache and its packed
// adapter (arrays of nslots; an entry of A_qkv NULL = the slot has no
// adapter, as in the fused kernels).
SWL_EXPORT int swl_wc_set_layer(void* handle, int layer, const void* in_norm, const void* post_norm,
                                void* const* k_cache, void* const* v_cache, const void* const* A_qkv,
                                const void* const* B_qkv, const void* const* A_o, const void* const* B_o,
                                const void* const* A_gu, const void* const* B_gu, const void* const* A_dn,
                                const void* const* B_dn) {
  auto* c = static_cast<WorkerClient*>(handle);
  if (!c || layer < 0 || layer >= c->layers) return set_error(SWL_ERR_ARG, "worker client: bad layer");
  if (!in_norm || !post_norm || !k_cache || !v_cache || !A_qkv || !B_qkv || !A_o || !B_o || !A_gu || !B_gu || !A_dn ||
      !B_dn)
    return set_error(SWL_ERR_ARG, "worker client: null layer argument");
  const int n = c->n;
  WcLayer& w = c->L[layer];
  w.in_norm = in_norm;
  w.post_norm = post_norm;
  w.k_cache.assign(k_cache, k_cache + n);
  w.v_cache.assign(v_cache, v_cache + n);
  w.A_qkv.assign(A_qkv, A_qkv + n);
  w.B_qkv.assign(B_qkv, B_qkv + n);
  w.A_o.assign(A_o, A_o + n);
  w.B_o.assign(B_o, B_o + n);
  w.A_gu.assign(A_gu, A_gu + n);
  w.B_gu.assign(B_gu, B_gu + n);
  w.A_dn.assign(A_dn, A_dn + n);
  w.B_dn.assign(B_dn, B_dn + n);
  return SWL_OK;
}

// input_mode 0: wait for a round's input with cudaStreamSynchronize (as the
// reference's prepare_input_slot); 1: with a device-written host flag; 2:
// events (the aggregator in this process must use completion mode 2; the
// client registers its input event for each of its slots).
// timeout_ms bounds every wait (epoch, input flag). history: optional int64
// device buffer [tokens][nslots] receiving each token's picks, or NULL.
SWL_EXPORT int swl_wc_configure(void* handle, int input_mode, int64_t timeout_ms, void* history) {
  auto* c = static_cast<WorkerClient*>(handle);
  if (!c || input_mode < 0 || input_mode > 2 || timeout_ms <= 0)
    return set_error(SWL_ERR_ARG, "worker client: input_mode 0, 1 or 2, positive timeout");
  if (input_mode == 2) {
    if (!c->input_event) SWL_CUDA_TRY(cudaEventCreateWithFlags(&c->input_event, cudaEventDisableTiming));
    void* ev = nullptr;
    SWL_TRY(swl_agg_round_event(&ev));
    c->round_event = static_cast<cudaEvent_t>(ev);
    for (int i = 0; i < c->n; ++i) SWL_TRY(swl_agg_set_slot_input_event_local(c->slot_ids[i], c->input_event));
  } else if (c->input_mode == 2) {
    for (int i = 0; i < c->n; ++i) swl_agg_set_slot_input_event_local(c->slot_ids[i], nullptr);
  }
  if (input_mode != 2) drop_graphs(c);
  c->input_mode = input_mode;
  c->timeout_ms = timeout_ms;
  c->history = history;
  return SWL_OK;
}

// Runs `tokens` decode tokens for the client's slots through the protocol
// (blocking; the slots must be active in the aggregator's main loop). On
// return token_ns[t] (if given) holds token t's host wall time in
// nanoseconds, measured from the first launch of the token to the return of
// its last round's wait. The work of the last token is synchronized.
SWL_EXPORT int swl_wc_run(void* handle, int tokens, int64_t* token_ns) {
  auto* c = static_cast<WorkerClient*>(handle);
  SWL_TRY(check_client(c));
  if (tokens < 0) return set_error(SWL_ERR_ARG, "worker client: negative token count");
  for (int t = 0; t < tokens; ++t) {
    const auto t0 = std::chrono::steady_clock::now();
    SWL_TRY(run_token(c, t));
    if (token_ns)
      token_ns[t] = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
  }
  SWL_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return SWL_OK;
}

// Rounds this client has completed through the protocol.
SWL_EXPORT int64_t swl_wc_rounds(void* handle) {
  auto* c = static_cast<WorkerClient*>(handle);
  return c ? c->rounds_done : 0;
}

// Event mode (input mode 2) only: 1 captures the launches between each pair
// of rounds into one CUDA graph (one launch per round instead of several),
// after the client's first eager token; 0 launches them one by one.
SWL_EXPORT int swl_wc_use_graphs(void* handle, int on) {
  auto* c = static_cast<WorkerClient*>(handle);
  if (!c) return set_error(SWL_ERR_ARG, "worker client: null handle");
  c->use_graphs = on != 0;
  if (!c->use_graphs) drop_graphs(c);
  return SWL_OK;
}

SWL_EXPORT int swl_wc_destroy(void* handle) {
  auto* c = static_cast<WorkerClient*>(handle);
  if (!c) return SWL_OK;
  drop_graphs(c);
  if (c->stream) {
    cudaStreamSynchronize(c->stream);
    cudaStreamDestroy(c->stream);
  }
  if (c->flag_host) cudaFreeHost(c->flag_host);
  if (c->input_event) {
    if (c->input_mode == 2)
      for (int i = 0; i < c->n; ++i) swl_agg_set_slot_input_event_local(c->slot_ids[i], nullptr);
    cudaEventDestroy(c->input_event);
  }
  delete c;
  return SWL_OK;
}
