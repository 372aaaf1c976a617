// Gather -> frozen-base GEMM -> scatter over the slot pool, as one kernel.
//
// A round computes, for every active slot s with rows_s tokens,
//   out_s[r, :] = in_s[r, :] @ W^T (+ bias)   for r in [0, rows_s)
// where in_s is the slot's [rows_s, K] bf16 input buffer and out_s its
// [rows_s, N] bf16 output buffer, W is the fused [N, K] weight. This is
// the reference's execute_batched_gemm_slots (ext_aggregator.cpp:470-626:
// torch::cat of the slot inputs, matmul_out against W.t(), copy_ back per
// slot) without the concatenated or staged intermediate.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "shm_abi.h"

namespace swl {

// Slot table handed to the kernel by value (kernel parameter space): the
// rows of slot i are global rows [row_start[i], row_start[i+1]).
struct SlotTable {
  int nslots;
  int total_rows;
  int row_start[kMaxSlots + 1];
  const __nv_bfloat16* in[kMaxSlots];
  __nv_bfloat16* out[kMaxSlots];
};

struct RoundShape {
  int64_t N;            // output features (rows of W)
  int64_t K;            // input features
  int64_t in_stride;    // elements between consecutive rows of a slot input
  int64_t out_stride;   // elements between consecutive rows of a slot output
  const __nv_bfloat16* bias;  // [N] or nullptr
};

// Column shard of a round over two GPUs (the column-sharded base-weight
// variant): this GPU holds rows [col0, col0 + N) of the fused weight, i.e.
// output columns [col0, col0 + N), and its epilogue writes them both into its
// own slot outputs and, by peer stores over NVLink, into the peer GPU's slot
// outputs (the all-gather of the outputs, fused into the round). Two epoch
// flags in each GPU's sync words order the exchange: a round stores into the
// peer only after the peer has started the same round (so the peer's readers
// of the previous round's outputs are done), and it completes only after the
// peer's half has landed here.
struct ShardArgs {
  __nv_bfloat16* peer_out[kMaxSlots];  // the peer's slot output rows (slot i as tab.out[i])
  int64_t col0;                        // first output column of this shard
  unsigned int* sync;                  // this GPU's sync words (kSyncWords, zeroed once)
  unsigned int* peer_sync;             // the peer's sync words, mapped into this process
};
// Sync word offsets (unsigned ints, each on its own 64-byte line).
constexpr int kSyncArrive = 0;   // CTAs of this round that finished their stores
constexpr int kSyncEpoch = 16;   // rounds completed on this GPU
constexpr int kSyncDone = 32;    // written by the peer: rounds whose stores into us landed
constexpr int kSyncStart = 48;   // written by the peer: rounds the peer has started
constexpr int kSyncWords = 64;

// The QKV round fused with its RoPE epilogue (decode launches, <= 64 rows):
// a round tile is one head (128 output columns), so instead of the round's
// bf16 output each tile adds the head's LoRA delta (bf16(t @ B^T) with t from
// the shrink partials), applies NeoX RoPE to q and k heads at position
// *seqlen + local row, and writes rotated q to q_rot and the new token's k / v
// into its cache page; the same arithmetic, in the same order, as the round
// followed by the separate RoPE epilogue.
struct QkvRopeEpi {
  const __nv_bfloat16* B[kMaxSlots];  // [(hq + 2 hkv) * 128, rank] lora_B rows per slot, or nullptr
  const int* block_table[kMaxSlots];
  __nv_bfloat16* k_cache[kMaxSlots];  // [pages, page, hkv, 128]
  __nv_bfloat16* v_cache[kMaxSlots];
  const int* seqlen[kMaxSlots];
  const float* ws_in;                 // shrink partials [rows][splits_in][3 rank]
  int splits_in, rank, hq, hkv, page;
  const __nv_bfloat16* cos_sin;       // [positions, 128]: cos (64) | sin (64)
  __nv_bfloat16* q_rot;               // [rows, hq * 128]
};
// Rows a fused QKV/RoPE launch takes at most (the tile's per-row tables live
// in shared memory next to the pipeline).
constexpr int kQkvRopeMaxRows = 64;

// Split-K through global memory (no thread-block cluster): split s of tile t
// writes its fp32 partial tile to part[(t * splits + s) * tile_floats] and
// counts itself in count[t]; the last of a tile's splits to arrive sums the
// partials in split order (the same order as the cluster reduction, so the
// results are bit-identical to it), writes the outputs and resets count[t].
// part == nullptr selects the cluster reduction.
struct SplitWs {
  float* part;
  int* count;
};

// The per-device split-K workspace (inside the stream-K workspace, allocated
// with the slot pool or on first use outside a stream capture): room for
// `floats` partial values and `tiles` counters, or SWL_ERR_STATE.
int splitk_workspace(SplitWs* out, size_t floats, int tiles);

enum RoundAlgo : int {
  kAlgoAuto = 0,        // cluster split-K (measured faster than stream-K on B200)
  kAlgoTensorCore = 1,  // tcgen05 + TMA, K split across a thread-block cluster (DSMEM reduce)
  kAlgoSimt = 2,        // plain CUDA-core kernel, used as an on-device cross-check
  kAlgoStreamK = 3,     // tcgen05 + TMA, persistent stream-K (<= 64 rows)
};

// Encodes the TMA descriptor for a row-major [N, K] bf16 weight (box 64 x 128,
// 128-byte swizzle). Returns SWL_OK or an error status.
int encode_weight_tmap(CUtensorMap* map, const void* W, int64_t N, int64_t K);

// Encodes the TMA descriptor of a paged KV cache, viewed as [tokens][hkv][128]
// bf16 with `tokens` rows (pages x page tokens): box 64 dims x 1 head x 16
// tokens, 128-byte swizzle (one kv head's half of a page per load).
int encode_kv_page_tmap(CUtensorMap* map, const void* cache, int64_t tokens, int hkv);

// Launches one round on `stream`. `tmap` may be nullptr (encoded on the fly).
// `splits` <= 0 picks the split-K factor automatically.
int launch_slot_round(const SlotTable& tab, const RoundShape& shape, const void* W,
                      const CUtensorMap* tmap, int algo, int splits, cudaStream_t stream);

// Launches one column-sharded round (tensor-core path only): W is this GPU's
// [shape.N, K] row block of the fused weight, outputs go to columns
// sh.col0 + [0, shape.N) of both GPUs' slot outputs.
int launch_slot_round_shard(const SlotTable& tab, const RoundShape& shape, const void* W,
                            const CUtensorMap* tmap, const ShardArgs& sh, int splits, cudaStream_t stream);

// Launches the fused QKV/RoPE round (tab.total_rows <= kQkvRopeMaxRows, head
// dim 128, no bias); tab's row-to-slot map is the one of the epilogue tables.
int launch_slot_round_qkv_rope(const SlotTable& tab, const RoundShape& shape, const void* W,
                               const CUtensorMap* tmap, const QkvRopeEpi& epi, int splits,
                               cudaStream_t stream);

// Device error word written by bounded waits inside round kernels (0 = ok).
int read_and_clear_device_error(unsigned int* code);

// Stream-K rounds (slot_round_sk.cu). The workspace (fp32 partial tiles and
// per-tile arrival counters) is allocated once per device; allocate it
// before capturing a launch into a CUDA graph.
int ensure_streamk_workspace();
int reset_streamk_counters();
int launch_slot_round_streamk(const SlotTable& tab, const RoundShape& shape, const CUtensorMap& map,
                              cudaStream_t stream);
int read_and_clear_sk_error(unsigned int* code);
int set_streamk_ctas_per_sm(int n);
int set_streamk_ctas(int n);

}  // namespace swl
