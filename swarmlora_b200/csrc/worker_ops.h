// Worker-side kernels around each aggregator round, batched over slots: each
// slot (worker) brings its own adapter, residual and KV-cache pointers
// through a by-value table, so one launch serves one worker or many.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "shm_abi.h"

namespace swl {

// Rows of slot i are global rows [row_start[i], row_start[i+1]).
struct RowSegments {
  int nseg;
  int total_rows;
  int row_start[kMaxSlots + 1];
};

// LoRA shrink: t[rows, R] = x[rows, K] @ A[K, R] (A row-major, R contiguous).
struct LoraShrinkTable {
  RowSegments seg;
  const __nv_bfloat16* x[kMaxSlots];  // slot activations, row stride x_stride
  const __nv_bfloat16* A[kMaxSlots];  // [K, R] or nullptr (no adapter)
};

// LoRA expand + epilogue over the fused output of a round.
struct LoraExpandTable {
  RowSegments seg;
  const __nv_bfloat16* base[kMaxSlots];   // round output rows [rows, n_total] (row stride base_stride)
  const __nv_bfloat16* B[kMaxSlots];      // [n_total, r] lora_B rows, or nullptr
  const __nv_bfloat16* resid[kMaxSlots];  // [rows, n_out] residual (mode kResidual) or nullptr
  __nv_bfloat16* out[kMaxSlots];          // destination rows (row stride out_stride)
};

enum ExpandMode : int {
  kExpandAdd = 0,       // out = base + delta                              (QKV)
  kExpandResidual = 1,  // out = resid + (base + delta)                    (O, Down)
  kExpandSiluMul = 2,   // out = silu(gate + dg) * (up + du), n_out = n/2 (Gate+Up)
};

struct ExpandParams {
  int64_t n_total;      // columns of the round output
  int r;                // rank
  int nblocks;          // fused projections (1, 2 or 3)
  int64_t block_end[3]; // exclusive column end of each projection
  float post_scale;     // delta scale applied after the expand (O/Down), 0 = none
  int mode;
  int64_t base_stride, out_stride, resid_stride;
  int splits;           // shrink partial count
};

// RoPE + paged KV append + attention tables.
struct AttnTable {
  RowSegments seg;
  const __nv_bfloat16* qkv[kMaxSlots];  // [rows, (Hq + 2 Hkv) * D] (LoRA already added)
  const int* block_table[kMaxSlots];    // device int32 page ids of the slot
  __nv_bfloat16* k_cache[kMaxSlots];    // [pages, page, Hkv, D] of this layer
  __nv_bfloat16* v_cache[kMaxSlots];
  __nv_bfloat16* out[kMaxSlots];        // [rows, Hq * D] attention output
  const int* seqlen[kMaxSlots];         // device int: cached tokens before this step
};

struct AttnParams {
  int hq, hkv, head_dim, page;
  int64_t qkv_stride, out_stride;
  float scale;
  const __nv_bfloat16* cos_sin;  // [max_pos, D]: cos (D/2) | sin (D/2)
  int max_pos;
  int max_len;                   // upper bound of any slot's context after this step
  __nv_bfloat16* q_rot;          // [total_rows, Hq * D] scratch for rotated q
  float* part;                   // per-chunk records, attention_part_floats() floats
  const void* pf;                // next round's weight to prefetch into L2 (or nullptr)
  int64_t pf_bytes;
};

// Context chunks the attention launch will use (each at most chunk_pages
// pages of a row's context), and the fp32 partial-record scratch it needs.
struct AttnSplit {
  int chunk_pages;
  int chunks;
};
AttnSplit attention_split(int total_rows, int hkv, int max_len);
int attention_splits(int total_rows, int hkv, int max_len);
// Overrides of the chunk size (pages) and page-ring depth; 0 = automatic.
int set_attention_tuning(int chunk_pages, int stages, int groups);
int set_attention_pairing(int on);
int set_attention_tma(int on);
int64_t attention_part_floats(int total_rows, int hq, int splits);

// RMSNorm over rows.
struct NormTable {
  RowSegments seg;
  const __nv_bfloat16* x[kMaxSlots];
  __nv_bfloat16* out[kMaxSlots];
};

// Batched device copies (one per entry; at most kMaxSlots per launch).
struct CopyTable {
  const void* src[kMaxSlots];
  void* dst[kMaxSlots];
  int64_t bytes[kMaxSlots];
};
int launch_copy_rows(const CopyTable& tab, int n, cudaStream_t stream);
int launch_advance_i32(int* p, int n, int delta, cudaStream_t stream);

int launch_lora_shrink(const LoraShrinkTable& tab, int64_t K, int R, int64_t x_stride, int splits,
                       float* ws, cudaStream_t stream);
int launch_lora_expand(const LoraExpandTable& tab, const ExpandParams& p, const float* ws,
                       cudaStream_t stream);
int launch_rope_append(const AttnTable& tab, const AttnParams& p, cudaStream_t stream);
// Optional LoRA shrink fused into the attention combine (O projection):
// ws[row][head][j] = sum_d out[row, head*D + d] * A[head*D + d, j].
struct ShrinkSide {
  const __nv_bfloat16* A[kMaxSlots];  // [hq*D, r] per slot, or nullptr
  int r;
  float* ws;
};
int launch_paged_attention(const AttnTable& tab, const AttnParams& p, cudaStream_t stream,
                           const ShrinkSide* shrink = nullptr);
int launch_rms_norm(const NormTable& tab, const __nv_bfloat16* w, int64_t hidden, float eps,
                    int64_t x_stride, int64_t out_stride, cudaStream_t stream);

// ---- fused round epilogues (fused_ops.cu) ------------------------------------------------
struct QkvRopeTable {
  RowSegments seg;
  const __nv_bfloat16* base[kMaxSlots];  // QKV round output rows [rows, (hq + 2 hkv) * D]
  const __nv_bfloat16* B[kMaxSlots];     // [(hq + 2 hkv) * D, r] lora_B rows, or nullptr
  const int* block_table[kMaxSlots];
  __nv_bfloat16* k_cache[kMaxSlots];
  __nv_bfloat16* v_cache[kMaxSlots];
  const int* seqlen[kMaxSlots];
};
struct QkvRopeParams {
  int hq, hkv, head_dim, page;
  int64_t base_stride;
  const float* ws_in;  // QKV shrink partials [total_rows][splits_in][3 r]
  int splits_in;
  const __nv_bfloat16* cos_sin;
  __nv_bfloat16* q_rot;  // [total_rows, hq * D]
  const void* pf;        // next round's weight to prefetch into L2 (or nullptr)
  int64_t pf_bytes;
};

struct ResidNormTable {
  RowSegments seg;
  const __nv_bfloat16* base[kMaxSlots];    // round output (or embedding) rows [rows, hidden]
  const __nv_bfloat16* B[kMaxSlots];       // [hidden, r_in] lora_B of the finished round, or nullptr
  __nv_bfloat16* h[kMaxSlots];             // hidden rows: residual in, new hidden out
  __nv_bfloat16* x_out[kMaxSlots];         // normed rows (next round's slot input)
  const __nv_bfloat16* A_next[kMaxSlots];  // [hidden, r_next] next round's shrink matrix, or nullptr
};
struct ResidNormParams {
  int64_t hidden;
  float post_scale;       // delta scale after the expand (0 = none)
  const float* ws_in;     // finished round's shrink partials [total_rows][splits_in][r_in]
  int splits_in;
  int has_resid;          // 0: h = base (+ delta); 1: h = h + (base + delta)
  const __nv_bfloat16* w; // RMSNorm weight [hidden]
  float eps;
  int64_t base_stride, h_stride, x_stride;
  int r_next;
  float* ws_next;         // [total_rows][8][r_next]
  const void* pf;         // next round's weight to prefetch into L2 (or nullptr)
  int64_t pf_bytes;
};

struct GuSiluTable {
  RowSegments seg;
  const __nv_bfloat16* base[kMaxSlots];    // Gate+Up round output rows [rows, 2 inter]
  const __nv_bfloat16* B[kMaxSlots];       // [2 inter, r] lora_B rows, or nullptr
  __nv_bfloat16* act[kMaxSlots];           // SiLU(gate) * up rows (Down round slot input)
  const __nv_bfloat16* A_next[kMaxSlots];  // [inter, r_next] Down shrink matrix, or nullptr
};
struct GuSiluParams {
  int64_t inter;
  int64_t base_stride, act_stride;
  const float* ws_in;  // Gate+Up shrink partials [total_rows][splits_in][2 r]
  int splits_in;
  int r_next;
  float* ws_next;      // [total_rows][gu_silu_splits(inter)][r_next]
  const void* pf;      // next round's weight to prefetch into L2 (or nullptr)
  int64_t pf_bytes;
};

int launch_qkv_rope(const QkvRopeTable& tab, const QkvRopeParams& p, int r, cudaStream_t stream);
int launch_resid_norm_shrink(const ResidNormTable& tab, const ResidNormParams& p, int r_in,
                             cudaStream_t stream);
int launch_gu_silu_shrink(const GuSiluTable& tab, const GuSiluParams& p, int r, cudaStream_t stream);
int resid_norm_splits(int rank);  // shrink partials per row for a group of this LoRA rank
int gu_silu_splits(int64_t inter);

}  // namespace swl
