// Worker side of the slot protocol: map the aggregator's per-slot buffers
// through CUDA IPC and move activations in and out of them. Mirrors the
// reference module ext_unified_barrier
// (src/cpp_extensions/ext_unified_barrier.cpp); each entry point cites the
// function whose behaviour it keeps. Copies are issued on the caller's
// stream; tensors never cross this boundary, only device pointers and sizes.
#include <cstring>

#include "common.h"
#include "shm_abi.h"

using namespace swl;

namespace {

constexpr int kMaxSlotsPerWorker = 8;  // ext_unified_barrier.cpp:22

struct SlotCtx {
  int slot_id = -1;
  bool open = false;
  bool mapped = false;  // true: pointers came from cudaIpcOpenMemHandle
  void* in = nullptr;
  void* out = nullptr;
  size_t in_bytes = 0, out_bytes = 0;
  int64_t bx = 0, tx = 0, dx = 0;
};

struct Manager {
  int worker_id = -1;
  int worker_device = 0;
  int aggregator_device = 0;
  int hidden = 0, inter = 0, qkv = 0;
  SlotCtx slots[kMaxSlotsPerWorker];
  int num_open = 0;
  bool initialized = false;
};

Manager g_w;

SlotCtx* find(int slot_id) {
  for (auto& c : g_w.slots)
    if (c.open && c.slot_id == slot_id) return &c;
  return nullptr;
}

int require(const char* fn, int slot_id, SlotCtx** ctx) {
  if (!g_w.initialized) return set_error(SWL_ERR_STATE, "%s: worker slot manager not initialized", fn);
  *ctx = find(slot_id);
  if (!*ctx) return set_error(SWL_ERR_ARG, "%s: slot %d not found", fn, slot_id);
  return SWL_OK;
}

}  // namespace

// ext_unified_barrier.cpp:60-94 init_worker_slot_manager.
SWL_EXPORT int swl_ub_init_worker_slot_manager(int worker_id, int worker_device,
                                               int aggregator_device, int hidden_dim,
                                               int intermediate_dim, int qkv_dim) {
  g_w = Manager();
  g_w.worker_id = worker_id;
  g_w.worker_device = worker_device;
  g_w.aggregator_device = aggregator_device;
  g_w.hidden = hidden_dim;
  g_w.inter = intermediate_dim;
  g_w.qkv = qkv_dim;
  SWL_CUDA_TRY(cudaSetDevice(worker_device));
  g_w.initialized = true;
  return SWL_OK;
}

// ext_unified_barrier.cpp:97-160 open_slot: map both IPC handles (lazy peer
// access), after checking the handle sizes.
SWL_EXPORT int swl_ub_open_slot(int slot_id, const unsigned char* in_handle, size_t in_handle_len,
                                const unsigned char* out_handle, size_t out_handle_len,
                                size_t in_bytes, size_t out_bytes) {
  if (!g_w.initialized) return set_error(SWL_ERR_STATE, "open_slot: worker slot manager not initialized");
  if (g_w.num_open >= kMaxSlotsPerWorker) return set_error(SWL_ERR_FULL, "open_slot: max slots per worker exceeded");
  if (in_handle_len != sizeof(cudaIpcMemHandle_t) || out_handle_len != sizeof(cudaIpcMemHandle_t))
    return set_error(SWL_ERR_ARG, "open_slot: invalid IPC handle size (got %zu/%zu, expected %zu)",
                     in_handle_len, out_handle_len, sizeof(cudaIpcMemHandle_t));
  SlotCtx* ctx = nullptr;
  for (auto& c : g_w.slots)
    if (!c.open) { ctx = &c; break; }
  if (!ctx) return set_error(SWL_ERR_FULL, "open_slot: no free slot context");
  SWL_CUDA_TRY(cudaSetDevice(g_w.worker_device));
  cudaIpcMemHandle_t hi, ho;
  std::memcpy(&hi, in_handle, sizeof(hi));
  std::memcpy(&ho, out_handle, sizeof(ho));
  void *pi = nullptr, *po = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&pi, hi, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return set_error(SWL_ERR_CUDA, "open_slot: input IPC open failed: %s", cudaGetErrorString(e));
  e = cudaIpcOpenMemHandle(&po, ho, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaIpcCloseMemHandle(pi);
    return set_error(SWL_ERR_CUDA, "open_slot: output IPC open failed: %s", cudaGetErrorString(e));
  }
  *ctx = SlotCtx();
  ctx->slot_id = slot_id;
  ctx->open = true;
  ctx->mapped = true;
  ctx->in = pi;
  ctx->out = po;
  ctx->in_bytes = in_bytes;
  ctx->out_bytes = out_bytes;
  ++g_w.num_open;
  return SWL_OK;
}

// In-process variant of open_slot for a worker living in the aggregator's own
// process (CUDA IPC cannot map a process's own allocations): attach the
// slot's buffers by device address. Not in the reference.
SWL_EXPORT int swl_ub_attach_slot(int slot_id, void* in, void* out, size_t in_bytes,
                                  size_t out_bytes) {
  if (!g_w.initialized) return set_error(SWL_ERR_STATE, "attach_slot: worker slot manager not initialized");
  if (g_w.num_open >= kMaxSlotsPerWorker) return set_error(SWL_ERR_FULL, "attach_slot: max slots per worker exceeded");
  if (!in || !out) return set_error(SWL_ERR_ARG, "attach_slot: null buffer");
  SlotCtx* ctx = nullptr;
  for (auto& c : g_w.slots)
    if (!c.open) { ctx = &c; break; }
  *ctx = SlotCtx();
  ctx->slot_id = slot_id;
  ctx->open = true;
  ctx->in = in;
  ctx->out = out;
  ctx->in_bytes = in_bytes;
  ctx->out_bytes = out_bytes;
  ++g_w.num_open;
  return SWL_OK;
}

// ext_unified_barrier.cpp:163-211 close_slot: device sync, then unmap.
SWL_EXPORT int swl_ub_close_slot(int slot_id) {
  SlotCtx* ctx;
  SWL_TRY(require("close_slot", slot_id, &ctx));
  SWL_CUDA_TRY(cudaDeviceSynchronize());
  if (ctx->mapped) {
    if (ctx->in) cudaIpcCloseMemHandle(ctx->in);
    if (ctx->out) cudaIpcCloseMemHandle(ctx->out);
  }
  *ctx = SlotCtx();
  --g_w.num_open;
  return SWL_OK;
}

// Device addresses of an open slot's mapped buffers (for fused kernels that
// read the slot output in place). Not in the reference.
SWL_EXPORT int swl_ub_slot_buffers(int slot_id, void** in, void** out, size_t* in_bytes,
                                   size_t* out_bytes) {
  SlotCtx* ctx;
  SWL_TRY(require("slot_buffers", slot_id, &ctx));
  if (in) *in = ctx->in;
  if (out) *out = ctx->out;
  if (in_bytes) *in_bytes = ctx->in_bytes;
  if (out_bytes) *out_bytes = ctx->out_bytes;
  return SWL_OK;
}

// ext_unified_barrier.cpp:225-273 prepare_input_slot: copy `bytes` of the
// worker's [bx, tx, dx] activation into the slot input, then wait for the
// copy (the aggregator reads it from another process once ready is set).
SWL_EXPORT int swl_ub_prepare_input_slot(int slot_id, int op_type, const void* src, size_t bytes,
                                         int64_t bx, int64_t tx, int64_t dx, void* stream) {
  (void)op_type;
  SlotCtx* ctx;
  SWL_TRY(require("prepare_input_slot", slot_id, &ctx));
  if (bytes > ctx->in_bytes)
    return set_error(SWL_ERR_ARG, "prepare_input_slot: input tensor (%zu bytes) exceeds slot buffer size (%zu bytes)",
                     bytes, ctx->in_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SWL_CUDA_TRY(cudaMemcpyAsync(ctx->in, src, bytes, cudaMemcpyDefault, st));
  SWL_CUDA_TRY(cudaStreamSynchronize(st));
  ctx->bx = bx;
  ctx->tx = tx;
  ctx->dx = dx;
  return SWL_OK;
}

// Shape recorded by the last prepare_* call of a slot.
SWL_EXPORT int swl_ub_slot_shape(int slot_id, int64_t* bx, int64_t* tx, int64_t* dx) {
  SlotCtx* ctx;
  SWL_TRY(require("slot_shape", slot_id, &ctx));
  *bx = ctx->bx;
  *tx = ctx->tx;
  *dx = ctx->dx;
  return SWL_OK;
}

// ext_unified_barrier.cpp:276-347 get_outputs_slot: copy bx*tx*sum(out_dims)
// elements of the slot output into the caller's buffer `dst` (the Python
// binding allocates it and splits the last dimension).
SWL_EXPORT int swl_ub_get_outputs_slot(int slot_id, void* dst, size_t bytes, void* stream) {
  SlotCtx* ctx;
  SWL_TRY(require("get_outputs_slot", slot_id, &ctx));
  if (bytes > ctx->out_bytes)
    return set_error(SWL_ERR_ARG, "get_outputs_slot: output (%zu bytes) exceeds slot output buffer (%zu bytes)",
                     bytes, ctx->out_bytes);
  SWL_CUDA_TRY(cudaMemcpyAsync(dst, ctx->out, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
  return SWL_OK;
}

// ext_unified_barrier.cpp:350-393 prepare_token_ids_slot (int64 ids [B, T]).
SWL_EXPORT int swl_ub_prepare_token_ids_slot(int slot_id, const void* ids, int64_t bx, int64_t tx,
                                             void* stream) {
  SlotCtx* ctx;
  SWL_TRY(require("prepare_token_ids_slot", slot_id, &ctx));
  size_t bytes = static_cast<size_t>(bx * tx) * sizeof(int64_t);
  if (bytes > ctx->in_bytes)
    return set_error(SWL_ERR_ARG, "prepare_token_ids_slot: token_ids (%zu bytes) exceeds slot buffer size (%zu bytes)",
                     bytes, ctx->in_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SWL_CUDA_TRY(cudaMemcpyAsync(ctx->in, ids, bytes, cudaMemcpyDefault, st));
  SWL_CUDA_TRY(cudaStreamSynchronize(st));
  ctx->bx = bx;
  ctx->tx = tx;
  ctx->dx = g_w.hidden;
  return SWL_OK;
}

// ext_unified_barrier.cpp:396-440 get_embeddings_slot: bx*tx*hidden elements.
SWL_EXPORT int swl_ub_get_embeddings_slot(int slot_id, void* dst, size_t elem_size, void* stream) {
  SlotCtx* ctx;
  SWL_TRY(require("get_embeddings_slot", slot_id, &ctx));
  size_t bytes = static_cast<size_t>(ctx->bx * ctx->tx) * g_w.hidden * elem_size;
  if (bytes > ctx->out_bytes)
    return set_error(SWL_ERR_ARG, "get_embeddings_slot: output (%zu bytes) exceeds slot output buffer (%zu bytes)",
                     bytes, ctx->out_bytes);
  SWL_CUDA_TRY(cudaMemcpyAsync(dst, ctx->out, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
  return SWL_OK;
}

// ext_unified_barrier.cpp:443-486 prepare_hidden_for_lm_head_slot.
SWL_EXPORT int swl_ub_prepare_hidden_for_lm_head_slot(int slot_id, const void* src, size_t bytes,
                                                      int64_t bx, int64_t tx, int64_t dx,
                                                      void* stream) {
  SlotCtx* ctx;
  SWL_TRY(require("prepare_hidden_for_lm_head_slot", slot_id, &ctx));
  if (bytes > ctx->in_bytes)
    return set_error(SWL_ERR_ARG, "prepare_hidden_for_lm_head_slot: hidden_states (%zu bytes) exceeds slot buffer size (%zu bytes)",
                     bytes, ctx->in_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SWL_CUDA_TRY(cudaMemcpyAsync(ctx->in, src, bytes, cudaMemcpyDefault, st));
  SWL_CUDA_TRY(cudaStreamSynchronize(st));
  ctx->bx = bx;
  ctx->tx = tx;
  ctx->dx = dx;
  return SWL_OK;
}

// ext_unified_barrier.cpp:489-518 get_next_token_slot: drain the caller's
// stream, then read the int64 token at the start of the slot output.
SWL_EXPORT int swl_ub_get_next_token_slot(int slot_id, int64_t* token, void* stream) {
  SlotCtx* ctx;
  SWL_TRY(require("get_next_token_slot", slot_id, &ctx));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SWL_CUDA_TRY(cudaStreamSynchronize(st));
  int64_t v = 0;
  SWL_CUDA_TRY(cudaMemcpyAsync(&v, ctx->out, sizeof(v), cudaMemcpyDefault, st));
  SWL_CUDA_TRY(cudaStreamSynchronize(st));
  *token = v;
  return SWL_OK;
}

// ext_unified_barrier.cpp:521-557 cleanup_worker_slots.
SWL_EXPORT int swl_ub_cleanup_worker_slots(void) {
  if (!g_w.initialized) return SWL_OK;
  cudaSetDevice(g_w.worker_device);
  cudaDeviceSynchronize();
  for (auto& c : g_w.slots) {
    if (c.open && c.mapped) {
      if (c.in) cudaIpcCloseMemHandle(c.in);
      if (c.out) cudaIpcCloseMemHandle(c.out);
    }
    c = SlotCtx();
  }
  g_w.num_open = 0;
  g_w.initialized = false;
  return SWL_OK;
}
