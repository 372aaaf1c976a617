/*
 * swarmlora_b200 — C ABI of the B200 (sm_100a) implementation of SwarmLoRA's
 * aggregator hot path: the gather -> frozen-base GEMM -> scatter round over
 * the CUDA-IPC slot pool, the shared-memory lock-step protocol around it, the
 * worker-side slot I/O, and the worker kernels (LoRA delta, RoPE + paged KV,
 * paged decode attention, RMSNorm) that surround each round.
 *
 * Library: swarmlora_b200/_lib/libswarmlora_b200.so (built by
 * `python -m swarmlora_b200.build`; CUDA runtime linked statically).
 *
 * Conventions
 *   - Every function returning int returns 0 on success and a negative status
 *     on failure; swl_last_error() then holds a message (thread-local). The
 *     reference's pybind modules raise RuntimeError in the same situations.
 *   - Pointers named *dev* or documented as device pointers are CUDA device
 *     addresses on the current device; `stream` is a cudaStream_t (NULL = the
 *     legacy default stream unless stated otherwise).
 *   - bf16 data is IEEE bfloat16 stored as 2-byte values; weights are
 *     row-major [out_features, in_features] (HF nn.Linear layout).
 *   - Reference citations are path:line in the SwarmLoRA source tree.
 */
#ifndef SWARMLORA_B200_H
#define SWARMLORA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define SWL_OK 0
#define SWL_ERR_ARG -1
#define SWL_ERR_STATE -2
#define SWL_ERR_CUDA -3
#define SWL_ERR_SYS -4
#define SWL_ERR_FULL -5
#define SWL_ERR_QUIT -6
#define SWL_ERR_TIMEOUT -7
#define SWL_ERR_OWNER -8

/* Op codes carried in ring commands (src/cpp_extensions/common/ipc_types.h:19-25). */
#define SWL_OP_O_PROJ 3
#define SWL_OP_DOWN_PROJ 6
#define SWL_OP_QKV_FUSED 9
#define SWL_OP_GATE_UP_FUSED 10
#define SWL_OP_EMBED 11
#define SWL_OP_LM_HEAD 12
#define SWL_OP_SET_SAMPLING 13
#define SWL_MAX_SLOTS 128 /* ipc_types.h:16 */

const char* swl_last_error(void);
int swl_abi_version(void);
/* Programmatic dependent launch for every later kernel launch of the library
 * (on by default): each kernel may start while the previous kernel of its
 * stream finishes, and waits for it before touching its outputs. Returns the
 * previous setting. No counterpart in the reference (a launch option). */
int swl_set_pdl(int on);

/* ======================================================================
 * Shared-memory command ring and slot barrier — replaces the pybind module
 * ext_ipc_queue (src/cpp_extensions/ext_ipc_queue.cpp:413-483). One queue
 * is mapped per process. Segment layout (ControlBlock followed by the
 * Command ring) is byte-identical to ipc_types.h:153-217.
 * ==================================================================== */

/* create_queue (ext_ipc_queue.cpp:111-145); writes "/gpuqueue_<pid>_<ns>". */
int swl_q_create(int capacity, int max_tickets, char* name_out, int name_cap);
/* open_queue (ext_ipc_queue.cpp:147-176). */
int swl_q_open(const char* shm_name, int capacity, int max_tickets);
/* Unmap (and unlink when created by this process); not in the reference. */
int swl_q_close(void);
/* init_batch_control (ext_ipc_queue.cpp:180-209). */
int swl_q_init_batch_control(int num_slots);
/* set_quit (ext_ipc_queue.cpp:404-410). */
int swl_q_set_quit(int value);
/* slot_set_pending_sampling (ext_ipc_queue.cpp:217-233). */
int swl_q_slot_set_pending_sampling(int slot_id, int do_sample, float temperature, int top_k,
                                    float top_p);
/* slot_signal_join / leave / ready (ext_ipc_queue.cpp:235-268). */
int swl_q_slot_signal_join(int slot_id);
int swl_q_slot_signal_leave(int slot_id);
int swl_q_slot_signal_ready(int slot_id);
/* wait_for_epoch (ext_ipc_queue.cpp:272-300): returns once the epoch exceeds
 * `expected` (capture it before signalling ready). timeout_ms <= 0 waits until
 * the epoch moves or quit is raised (as the reference); > 0 bounds the wait. */
int swl_q_wait_for_epoch(int64_t expected, int64_t timeout_ms, int64_t* epoch_out);
/* slot_is_active, get_barrier_done_epoch, is_slot_evicted, clear_evicted_slot
 * (ext_ipc_queue.cpp:303-336). */
int swl_q_slot_is_active(int slot_id);
int64_t swl_q_get_barrier_done_epoch(void);
int swl_q_is_slot_evicted(int slot_id);
void swl_q_clear_evicted_slot(int slot_id);
/* submit_slot_command (ext_ipc_queue.cpp:339-402): validates before reserving. */
int swl_q_submit_slot_command(int op_type, int layer_idx, int slot_id, int worker_id, int64_t bx,
                              int64_t tx, int64_t dx, uint64_t x_key, uint64_t y0_key,
                              uint64_t y1_key, uint64_t y2_key, int ticket_id);
/* Introspection of this process's mapping (tests). */
void* swl_q_control_block(void);
int swl_q_capacity(void);
size_t swl_q_control_block_size(void);
size_t swl_q_command_size(void);

/* ======================================================================
 * Aggregator: slot pool, frozen base weights, rounds, main loop — replaces
 * the pybind module ext_aggregator (src/cpp_extensions/ext_aggregator.cpp:1436-1517).
 * ==================================================================== */

/* init_slot_pool (ext_aggregator.cpp:138-187): per-slot cudaMalloc input and
 * output buffers with CUDA IPC handles; returns their byte sizes. */
int swl_agg_init_slot_pool(int num_slots, int device_index, int hidden_dim, int intermediate_dim,
                           int num_kv_heads, int head_dim, int max_seq_per_step, int dtype_size,
                           size_t* in_bytes, size_t* out_bytes);
/* claim_slot (ext_aggregator.cpp:190-245): 64-byte cudaIpcMemHandle_t each. */
int swl_agg_claim_slot(int worker_id, int* slot_id, unsigned char* in_handle,
                       unsigned char* out_handle, size_t* in_bytes, size_t* out_bytes);
/* release_slot (ext_aggregator.cpp:248-296): zeroes both buffers first. */
int swl_agg_release_slot(int slot_id, int worker_id);
/* get_slot_owner (ext_aggregator.cpp:299-304): -1 if free or invalid. */
int swl_agg_get_slot_owner(int slot_id);
/* get_slot_pool_status (ext_aggregator.cpp:307-328): masks = {free_lo,
 * free_hi, active_lo, active_hi}; owners receives num_slots entries. */
int swl_agg_get_slot_pool_status(int* initialized, int* num_slots, uint64_t* masks,
                                 int* active_slot_count, int* owners);
/* Aggregator-local device addresses of a slot (in-process drivers). */
int swl_agg_slot_buffers(int slot_id, void** in_dev, void** out_dev);
/* cleanup_slot_pool (ext_aggregator.cpp:1410-1431). */
int swl_agg_cleanup_slot_pool(void);
/* init_aggregator_begin / _layer / _finalize (ext_aggregator.cpp:338-410):
 * q|k|v and gate|up are fused into library-owned copies; o, down and the
 * optional biases (NULL = none) are borrowed device pointers. */
int swl_agg_init_begin(int num_layers, int device_index);
int swl_agg_init_layer(int layer_idx, const void* q, int64_t q_rows, const void* k, int64_t k_rows,
                       const void* v, int64_t v_rows, const void* o, int64_t o_rows,
                       const void* o_bias, const void* gate, int64_t gate_rows, const void* up,
                       int64_t up_rows, const void* down, int64_t down_rows, const void* down_bias,
                       int64_t hidden, int64_t inter);
int swl_agg_init_finalize(void);
/* init_embed_lm_head_weights (ext_aggregator.cpp:413-424); both borrowed. */
int swl_agg_init_embed_lm_head(const void* embed, const void* lm_head, int64_t vocab,
                               int64_t hidden);
/* init_aggregator_queue (ext_aggregator.cpp:427-459). */
int swl_agg_init_queue(const char* shm_name, int capacity);
/* Round kernel: 0 auto (= 1), 1 tcgen05 cluster split-K, 2 CUDA cores,
 * 3 tcgen05 stream-K (<= 64 rows); splits <= 0 = automatic K split. */
int swl_agg_set_round_algo(int algo, int splits);
/* Sampling state of a worker for in-process drivers (the protocol sets it
 * with OP_SET_SAMPLING / slot_set_pending_sampling, ext_aggregator.cpp:991-1020).
 * The LM-head round samples each row with its own worker's state (the
 * reference applies the first command's worker's state to the batch). */
int swl_agg_set_worker_sampling(int worker_id, int do_sample, float temperature, int top_k, float top_p);
/* Seed of the LM-head sampling; each sampling round draws with the next
 * offset (restarted at 0 here). */
int swl_agg_set_sampling_seed(uint64_t seed);
/* Fused weight of (layer, op) and its [N, K] shape; OP_EMBED / OP_LM_HEAD
 * give the [vocab, hidden] tables (layer ignored). */
int swl_agg_weight(int layer, int op, const void** W, int64_t* N, int64_t* K);
/* One round over pool slots — execute_batched_gemm_slots (ext_aggregator.cpp:
 * 470-626), execute_batched_embed_slots (:630-706) or the greedy LM head
 * (:710-875) — on `stream` (NULL = the library's stream, synchronised).
 * Slot i has bx[i] * tx[i] rows. Ownership and buffer bounds are checked. */
int swl_agg_execute_round(int op, int layer, int n, const int* slot_ids, const int* worker_ids,
                          const int64_t* bx, const int64_t* tx, void* stream);
/* aggregator_main_loop_slots (ext_aggregator.cpp:1024-1210); blocking. */
int swl_agg_main_loop_slots(int num_slots, int dtype_code);
/* How the main loop completes a round (not in the reference). 0: it
 * synchronizes the round's stream, then bumps barrier_done_epoch on the host
 * (ext_aggregator.cpp:1196-1202). 1: the control block is registered as
 * mapped host memory and a device store after the round's kernels bumps the
 * epoch; the loop goes on without waiting (workers see the epoch as soon as
 * the round has finished on the GPU). Needs swl_agg_init_queue first;
 * mapping a new queue resets the mode to 0. */
int swl_agg_set_completion_mode(int mode);
int swl_agg_completion_mode(void);
/* Event completion (mode 2 of swl_agg_set_completion_mode; not in the
 * reference): each slot's worker records an event after the work that
 * writes the slot's round input and then sets its ready bit; the round's
 * stream waits for those events, the round event is recorded after the
 * round's kernels and the host bumps the epoch at once; a worker that sees
 * the epoch makes its stream wait for the round event before reading the
 * outputs. A slot without an input event is refused under mode 2. The round
 * event: its IPC handle (64 bytes) for workers in other processes, or the
 * cudaEvent_t for workers in this process. A slot's input event: from the
 * worker's IPC handle (NULL / 0 = none), or a cudaEvent_t of this process. */
/* Under event completion, 1 = replay each (op, layer) round from a CUDA
 * graph holding the input-event waits, the round's kernels and the round
 * event's record, captured when the same slots send the same rows a second
 * time (the LM-head round always runs eagerly); 0 = launch each round. */
int swl_agg_set_round_graphs(int on);
int swl_agg_round_event_handle(unsigned char* out, size_t len);
int swl_agg_round_event(void** event);
int swl_agg_set_slot_input_event(int slot_id, const unsigned char* handle, size_t len);
int swl_agg_set_slot_input_event_local(int slot_id, void* event);
/* The QKV round of `layer` fused with the RoPE epilogue (swl_fused_qkv_rope's
 * arguments; table entry i belongs to command i): each round tile is one head
 * and adds its LoRA delta, applies NeoX RoPE and writes rotated q to q_rot
 * and the new token's k / v into the paged caches; the QKV slot outputs are
 * not written. Same results as swl_agg_execute_round(OP_QKV_FUSED) followed
 * by swl_fused_qkv_rope, which it runs instead above 64 rows or with
 * column-sharded weights. No reference counterpart (a fusion). */
int swl_agg_execute_qkv_rope_round(int layer, int n, const int* slot_ids, const int* worker_ids,
                                   const int64_t* bx, const int64_t* tx, const void* const* B, int r,
                                   const float* ws_in, int splits_in, const void* const* block_tables,
                                   void* const* k_cache, void* const* v_cache, const void* const* seqlens,
                                   int hq, int hkv, int head_dim, int page, const void* cos_sin, void* q_rot,
                                   void* stream);
/* Donor weight transfer for multi-GPU bring-up — export_weight_ipc_handles /
 * import_weights_from_ipc (ext_aggregator.cpp:1216-1406). One record per
 * weight, in this order: per layer l, records 6l..6l+5 = fused qkv
 * [q+k+v, hidden], o [o_out, hidden], fused gate_up [gate+up, hidden], down
 * [down_out, inter], o_bias [o_out, 1], down_bias [down_out, 1] (rows 0 =
 * absent); then embed and lm_head [vocab, hidden]. All bf16 row-major.
 * dims holds 5 int64 per layer: q, k, v, gate, up output sizes. Unlike the
 * reference's handles, a record names the allocation holding the weight
 * and the weight's byte offset in it, so weights inside a larger allocation
 * (a caching allocator's block) are exported correctly. */
typedef struct swl_weight_ipc {
  unsigned char handle[64]; /* cudaIpcMemHandle_t of the allocation */
  uint64_t offset;          /* bytes from the allocation's base */
  int64_t rows, cols;
} swl_weight_ipc;
/* Fills `recs` (room for cap = 6 * num_layers + 2 records) and `dims`
 * (5 * num_layers) from this aggregator's weights; with recs == NULL only
 * *num_layers and *device_index are returned. Needs the layers and the LM
 * head initialised. The donor process must keep its weights alive until
 * every receiver's import has returned. */
int swl_agg_export_weights(swl_weight_ipc* recs, int cap, int64_t* dims, int* num_layers,
                           int* device_index);
/* Replaces this aggregator's weights with copies of a donor's (another
 * process, any GPU of the node): maps each distinct allocation once, checks
 * every record against the mapped range, copies all weights into one
 * library-owned arena on device_index (peer copies over NVLink when the
 * donor is another GPU), unmaps, and leaves the aggregator as after
 * init_aggregator_finalize + init_embed_lm_head_weights. */
int swl_agg_import_weights(const swl_weight_ipc* recs, int count, const int64_t* dims, int num_layers,
                           int device_index);
/* Column-sharded base weights over a pair of GPUs, one process each (the
 * multi-GPU configuration's variant with an NVLink all-gather of outputs; no
 * reference counterpart). After the pool, layers and LM head are set up:
 * swl_agg_shard_begin builds this GPU's row views (output columns
 * [rank*N/2, ...)) of every fused weight; swl_agg_shard_handles exports the
 * IPC handles (64 bytes each: sync words, logits, slot outputs 0..n-1) that
 * the peer passes to swl_agg_shard_connect, which maps them and switches
 * every round to the sharded kernel: each GPU computes its half of the
 * columns and writes it into both GPUs' slot outputs by peer stores. Both
 * GPUs must then run the same rounds in the same order; a round whose peer
 * does not follow within 2 s records an error (swl_round_device_error).
 * swl_agg_shard_end unmaps (call it on both GPUs before freeing a pool). */
int swl_agg_shard_begin(int rank, int world);
int swl_agg_shard_handles(unsigned char* out, int max_handles, int* count);
int swl_agg_shard_connect(const unsigned char* peer, int count);
int swl_agg_shard_end(void);

/* ======================================================================
 * Worker slot I/O — replaces the pybind module ext_unified_barrier
 * (src/cpp_extensions/ext_unified_barrier.cpp:562-630).
 * ==================================================================== */

/* init_worker_slot_manager (ext_unified_barrier.cpp:60-94). */
int swl_ub_init_worker_slot_manager(int worker_id, int worker_device, int aggregator_device,
                                    int hidden_dim, int intermediate_dim, int qkv_dim);
/* open_slot (ext_unified_barrier.cpp:97-160): maps both IPC handles. */
int swl_ub_open_slot(int slot_id, const unsigned char* in_handle, size_t in_handle_len,
                     const unsigned char* out_handle, size_t out_handle_len, size_t in_bytes,
                     size_t out_bytes);
/* In-process variant of open_slot (device addresses instead of handles). */
int swl_ub_attach_slot(int slot_id, void* in_dev, void* out_dev, size_t in_bytes, size_t out_bytes);
/* close_slot (ext_unified_barrier.cpp:163-211). */
int swl_ub_close_slot(int slot_id);
/* Mapped device addresses of an open slot. */
int swl_ub_slot_buffers(int slot_id, void** in_dev, void** out_dev, size_t* in_bytes,
                        size_t* out_bytes);
/* prepare_input_slot (ext_unified_barrier.cpp:225-273): copy + wait. */
int swl_ub_prepare_input_slot(int slot_id, int op_type, const void* src_dev, size_t bytes,
                              int64_t bx, int64_t tx, int64_t dx, void* stream);
/* Shape recorded by the last prepare_* call. */
int swl_ub_slot_shape(int slot_id, int64_t* bx, int64_t* tx, int64_t* dx);
/* get_outputs_slot (ext_unified_barrier.cpp:276-347): async copy of the slot
 * output into dst (the Python binding splits the last dimension). */
int swl_ub_get_outputs_slot(int slot_id, void* dst_dev, size_t bytes, void* stream);
/* prepare_token_ids_slot / get_embeddings_slot /
 * prepare_hidden_for_lm_head_slot / get_next_token_slot / cleanup_worker_slots
 * (ext_unified_barrier.cpp:350-557). */
int swl_ub_prepare_token_ids_slot(int slot_id, const void* ids_dev, int64_t bx, int64_t tx,
                                  void* stream);
int swl_ub_get_embeddings_slot(int slot_id, void* dst_dev, size_t elem_size, void* stream);
int swl_ub_prepare_hidden_for_lm_head_slot(int slot_id, const void* src_dev, size_t bytes,
                                           int64_t bx, int64_t tx, int64_t dx, void* stream);
int swl_ub_get_next_token_slot(int slot_id, int64_t* token, void* stream);
int swl_ub_cleanup_worker_slots(void);

/* ======================================================================
 * Kernels callable directly (no pool): the round over caller buffers and the
 * worker-side kernels, batched over slots. Segment i covers rows[i] rows.
 * ==================================================================== */

/* The round of execute_batched_gemm_slots (ext_aggregator.cpp:526-625) over
 * caller slot buffers: out_ptrs[i][r] = in_ptrs[i][r] @ W^T (+ bias). */
int swl_slot_gemm(const void* W, int64_t N, int64_t K, const void* bias, int nslots,
                  const void* const* in_ptrs, void* const* out_ptrs, const int* rows,
                  int64_t in_stride, int64_t out_stride, int algo, int splits, void* stream);
/* Greedy pick of the LM-head op (ext_aggregator.cpp:821-874, torch.argmax per
 * row): out[r] (int64, device) = lowest index of the largest bf16 logit of
 * row r (row stride ld elements); NaN never wins, no finite maximum gives 0. */
int swl_argmax_rows(const void* logits, int rows, int64_t vocab, int64_t ld, int64_t* out, void* stream);
/* Sampling parameters of one row (OP_SET_SAMPLING state). */
typedef struct swl_sampling {
  int do_sample;
  float temperature;
  int top_k;
  float top_p;
} swl_sampling;
/* Next token of each row (ext_aggregator.cpp:757-787, :821-874): rows with
 * do_sample draw from softmax(bf16(logit / max(temperature, 0.01))) limited
 * to the top_k largest (ties kept, 0 = no limit) and then to the top_p
 * nucleus (kept while the running probability in descending order stays
 * <= top_p; the first always), by the inverse CDF in index order at u[r]
 * (device floats in [0, 1); NULL: derived from seed, offset and r); other
 * rows take the argmax as swl_argmax_rows. params is a host array of rows
 * entries; out is int64 device memory. */
int swl_sample_rows(const void* logits, int rows, int64_t vocab, int64_t ld, const swl_sampling* params,
                    const float* u, uint64_t seed, uint64_t offset, int64_t* out, void* stream);
/* Bounded-wait status of the round kernels (0 = none ran out); synchronous. */
int swl_round_device_error(unsigned int* code);
/* Tuning of the stream-K round (algo 3). */
int swl_round_set_streamk_ctas_per_sm(int n);
int swl_round_set_streamk_ctas(int n);
/* Tuning of the tensor-core round: rounds of up to max_rows token rows (32,
 * 64, 96, 128; 0 = above 128) use a tile of bn rows with a ring of `stages`
 * K-blocks (bn 0 = the default); flags bit 0: the gather warps poll without
 * sleeping; bit 1: split-K sums reduced through a per-device global-memory
 * workspace instead of across a thread-block cluster (then rounds with
 * split-K on one device share that workspace and must run in stream order,
 * never concurrently); bit 2: before its dependency wait each CTA prefetches
 * into L2 the W tiles its ring cannot hold (up to 12 K-blocks); bits 0-2
 * apply to every class. Bit 3 (with bn != 0): the class's token rows are
 * packed into a per-device staging copy by a launch ahead of the round,
 * which then loads its token tiles by TMA (default above 128 rows, and for
 * the large weights from 65 rows); such rounds on one device share the
 * staging copy and run in stream order. */
int swl_round_tune(int max_rows, int bn, int stages, int flags);

/* LoRA shrink (model_builder.py:258-262 x @ fused_A; worker_sync.py:305/375
 * lora_A): ws[split][row][R] fp32 partials of x @ A, A[i] = [K, R] or NULL. */
int swl_lora_shrink(int nseg, const int* rows, const void* const* x, int64_t x_stride,
                    const void* const* A, int64_t K, int R, int splits, float* ws, void* stream);
/* LoRA expand + round epilogue (worker_sync.py:270-389): mode 0 base + d,
 * 1 resid + (base + d) with d scaled after the expand, 2 silu(gate+dg)*(up+du). */
int swl_lora_expand(int nseg, const int* rows, const void* const* base, int64_t base_stride,
                    const void* const* B, const void* const* resid, int64_t resid_stride,
                    void* const* out, int64_t out_stride, int64_t n_total, int r, int nblocks,
                    const int64_t* block_end, float post_scale, int mode, int splits,
                    const float* ws, void* stream);
/* NeoX RoPE + paged KV append (vLLM rotary_embedding + the append inside
 * flash_attn_with_kvcache, worker_sync.py:192-203). */
int swl_rope_append(int nseg, const int* rows, const void* const* qkv, int64_t qkv_stride,
                    const void* const* block_tables, void* const* k_cache, void* const* v_cache,
                    const void* const* seqlens, int hq, int hkv, int head_dim, int page,
                    const void* cos_sin, int max_pos, void* q_rot, void* stream);
/* Tuning of the attention launch: pages per context chunk, page-ring depth
 * (2..4) and kv head groups (1, 2, 4, 8: CTAs that share one page's heads,
 * each holding its group's slices); 0 = automatic. A launch option, no
 * counterpart in the reference. */
int swl_attention_tune(int chunk_pages, int stages, int groups);
/* 1 (default): two consecutive rows of one slot (a prefill chunk) share each
 * page read, their query heads filling the MMA's columns together; 0: every
 * row reads its pages alone. A launch option, no counterpart in the reference. */
int swl_attention_pairing(int on);
/* 1 (default): the attention kernel loads its K/V pages with TMA (one lane
 * per warp issues its kv head's 128B-swizzled halves) when every row's pages
 * lie in one cache allocation; 0: per-lane cp.async copies always. A launch
 * option, no counterpart in the reference. */
int swl_attention_tma(int on);
/* fp32 scratch floats swl_paged_attention needs in `part`. */
int64_t swl_attention_part_floats(int total_rows, int hq, int hkv, int max_len);
/* Causal GQA attention over paged KV (flash_attn_with_kvcache semantics,
 * worker_sync.py:196-203); `part` is caller scratch. The context lengths and
 * block tables are read before the launch waits for the kernel launched just
 * ahead of it on the stream (programmatic dependent launch): that launch,
 * when it is one of this library's kernels, must not write them (the
 * RoPE/append launches that normally precede attention do not). */
int swl_paged_attention(int nseg, const int* rows, const void* const* block_tables,
                        const void* const* k_cache, const void* const* v_cache,
                        const void* const* seqlens, void* const* out, int64_t out_stride, int hq,
                        int hkv, int head_dim, int page, float scale, int max_len,
                        const void* q_rot, float* part, void* stream);
/* swl_paged_attention without the `part` argument, for callers that cannot
 * allocate: a host whose memory is not managed by torch, or code on a path
 * where allocating is not allowed. No counterpart in the reference (its
 * attention, flash_attn_with_kvcache at worker_sync.py:196-203, allocates
 * its own temporaries). The partial results live in an array compiled into
 * the library, SWL_NOALLOC_ATTN_SCRATCH_FLOATS fp32 values per device
 * (4 MiB); a launch needing more (swl_attention_part_floats) fails with
 * SWL_ERR_ARG. Nothing is allocated. All calls on a device share that array
 * and it keeps the last call's contents; calls on one stream are safe, calls
 * that overlap on the GPU corrupt each other. Nothing in it needs to start at
 * zero. The first call on a device looks up the array's address (this may
 * load the library's code onto the device): make it before any stream
 * capture begins. The address is cached per device for the life of the
 * device's primary context; after cudaDeviceReset call
 * swl_noalloc_forget_device with that device current. */
#define SWL_NOALLOC_ATTN_SCRATCH_FLOATS 1048576
int swl_paged_attention_noalloc(int nseg, const int* rows, const void* const* block_tables,
                                const void* const* k_cache, const void* const* v_cache,
                                const void* const* seqlens, void* const* out, int64_t out_stride,
                                int hq, int hkv, int head_dim, int page, float scale, int max_len,
                                const void* q_rot, void* stream);
/* Forgets the current device's cached address of the no-allocation scratch
 * array, so the next swl_paged_attention_noalloc looks it up again (needed
 * only after the device's primary context was destroyed, e.g. by
 * cudaDeviceReset). No counterpart in the reference. */
int swl_noalloc_forget_device(void);
/* swl_paged_attention + the O projection's LoRA shrink on its output. */
int swl_paged_attention_shrink(int nseg, const int* rows, const void* const* block_tables,
                               const void* const* k_cache, const void* const* v_cache,
                               const void* const* seqlens, void* const* out, int64_t out_stride,
                               int hq, int hkv, int head_dim, int page, float scale, int max_len,
                               const void* q_rot, float* part, const void* const* A_o, int r,
                               float* ws_o, const void* pf, int64_t pf_bytes, void* stream);
/* LlamaRMSNorm (HF modeling_llama; worker_sync.py:1346, 1380, 1416). */
int swl_rms_norm(int nseg, const int* rows, const void* const* x, int64_t x_stride,
                 void* const* out, int64_t out_stride, const void* w, int64_t hidden, float eps,
                 void* stream);
/* Fused round epilogues (one launch between two rounds; worker_sync.py:1337-1409).
 * Each reads its adapters and the shrink partials of its round's input
 * (swl_fused_resid_norm_shrink also the residual and norm weight,
 * swl_fused_qkv_rope the context lengths, block tables and cos/sin cache)
 * before waiting for the round launched just ahead of it, which must not
 * write them. */
int swl_fused_qkv_rope(int nseg, const int* rows, const void* const* base, int64_t base_stride,
                       const void* const* B, int r, const float* ws_in, int splits_in,
                       const void* const* block_tables, void* const* k_cache,
                       void* const* v_cache, const void* const* seqlens, int hq, int hkv,
                       int head_dim, int page, const void* cos_sin, void* q_rot, const void* pf,
                       int64_t pf_bytes, void* stream);
int swl_fused_resid_norm_shrink(int nseg, const int* rows, const void* const* base,
                                int64_t base_stride, const void* const* B, int r_in,
                                float post_scale, const float* ws_in, int splits_in, int has_resid,
                                void* const* h, int64_t h_stride, const void* w, int64_t hidden,
                                float eps, void* const* x_out, int64_t x_stride,
                                const void* const* A_next, int r_next, float* ws_next,
                                const void* pf, int64_t pf_bytes, void* stream);
int swl_fused_gu_silu_shrink(int nseg, const int* rows, const void* const* base,
                             int64_t base_stride, const void* const* B, int r, const float* ws_in,
                             int splits_in, int64_t inter, void* const* act, int64_t act_stride,
                             const void* const* A_next, int r_next, float* ws_next, const void* pf,
                             int64_t pf_bytes, void* stream);
/* Shrink partials per row that swl_fused_resid_norm_shrink writes for a
 * group packed at LoRA rank `rank` (its cluster size: 4 up to rank 16, else 8). */
int swl_fused_norm_splits(int rank);
int swl_fused_silu_splits(int64_t inter);
/* Batched device copies and an in-place counter advance. */
int swl_copy_rows(int n, const void* const* src, void* const* dst, const int64_t* bytes,
                  void* stream);
int swl_advance_i32(int* p, int n, int delta, void* stream);

/* ======================================================================
 * Worker client of the slot protocol — the reference worker's per-token
 * loop (worker_sync.py:1274-1425) and its round requests
 * (BatchedAggregatorOps.*_submit_all / barrier_sync, worker_sync.py:230-389)
 * for the slots one client owns, from one host thread, with this library's
 * fused worker kernels between the rounds (slot outputs read in place, the
 * next round's input written straight into the slot input). Each round:
 * the input is known written (input mode 0: cudaStreamSynchronize, as
 * prepare_input_slot; 1: a device-written host flag; 2: an event recorded
 * for the aggregator's event completion), the epoch is captured, one command
 * per slot is submitted, the ready bits are set, the client waits for the
 * epoch (mode 2: then its stream waits for the round event). Uses this process's queue mapping (swl_q_create or
 * swl_q_open); the slots must have joined and be active.
 * ==================================================================== */
int swl_wc_create(int nslots, const int* slot_ids, const int* worker_ids, int layers, int hidden,
                  int inter, int hq, int hkv, int head_dim, int page, int rank, float eps,
                  float scaling, int max_len, void** out);
int swl_wc_set_buffers(void* handle, void* const* slot_in, void* const* slot_out,
                       void* const* h_rows, void* const* tokens, const void* const* block_tables,
                       const void* const* seqlens, int* seqlen_base, void* q_rot, float* part,
                       float* ws_qkv, float* ws_o, float* ws_gu, float* ws_dn,
                       const void* cos_sin, const void* final_norm);
int swl_wc_set_layer(void* handle, int layer, const void* in_norm, const void* post_norm,
                     void* const* k_cache, void* const* v_cache, const void* const* A_qkv,
                     const void* const* B_qkv, const void* const* A_o, const void* const* B_o,
                     const void* const* A_gu, const void* const* B_gu, const void* const* A_dn,
                     const void* const* B_dn);
int swl_wc_configure(void* handle, int input_mode, int64_t timeout_ms, void* history);
/* Runs `tokens` decode tokens (blocking); token_ns[t] = token t's host wall
 * time in ns, or NULL. */
int swl_wc_run(void* handle, int tokens, int64_t* token_ns);
/* Input mode 2 only: 1 = capture the launches between each pair of rounds
 * into one CUDA graph (external event wait / record nodes at its ends), after
 * the client's first eager token; 0 = launch them one by one. */
int swl_wc_use_graphs(void* handle, int on);
int64_t swl_wc_rounds(void* handle);
int swl_wc_destroy(void* handle);

#ifdef __cplusplus
}
#endif

#endif /* SWARMLORA_B200_H */
