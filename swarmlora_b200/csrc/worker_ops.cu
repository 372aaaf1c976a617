// Worker-side kernels around each round, batched over slots.
//
//  * lora_shrink   t = x @ A (A = [K, R], R = rank * fused projections),
//                  split over K into fp32 partials.
//  * lora_expand   d = bf16(t) @ B^T per fused projection, then the
//                  epilogue of the round read in place from the slot output:
//                  QKV: base + d; O/Down: resid + (base + bf16(d * s));
//                  Gate+Up: silu(gate + dg) * (up + du).
//  * rope_append   NeoX RoPE on q and k, k/v appended to the paged cache.
//  * paged_attention  causal GQA attention of each new token over its slot's
//                  pages (split over the context, partials combined).
//  * rms_norm      LlamaRMSNorm.
//
// Rounding follows the reference's bf16 tensors: the LoRA intermediate t and
// delta d are bf16 (model_builder.py:258-262, worker_sync.py:305/:375), the
// adds are bf16 adds (worker_sync.py:270-389), RoPE arithmetic is per-op bf16
// (vLLM rotary_embedding), RMSNorm rounds the normalised row before the weight
// multiply (HF LlamaRMSNorm), silu(g) is rounded before the multiply by up.
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

#include "common.h"
#include "launch.h"
#include "ptx.cuh"
#include "slot_round.h"
#include "worker_ops.h"

namespace swl {

namespace {

__device__ __forceinline__ float bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ int seg_of_row(const RowSegments& s, int gr) {
  int lo = 0, hi = s.nseg - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (s.row_start[mid] <= gr) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// ---- LoRA shrink ---------------------------------------------------------------
// CTA = (segment, K split). Threads are (column group cg of 8 columns, k lane
// kg); each accumulates ROWS rows x 8 columns over its k values, then the k
// lanes are summed through shared memory. Output: ws[split][row][R] fp32.
template <int ROWS>
__global__ void __launch_bounds__(256) lora_shrink_kernel(const __grid_constant__ LoraShrinkTable tab,
                                                          int64_t K, int R, int64_t x_stride,
                                                          int splits, float* __restrict__ ws) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  extern __shared__ float red[];  // [256][ROWS * 8]
  const int seg = blockIdx.x / splits, split = blockIdx.x % splits;
  const __nv_bfloat16* A = tab.A[seg];
  if (!A) return;
  const int G = R / 8;
  const int kgroups = 256 / G;
  const int t = threadIdx.x;
  const bool active = t < kgroups * G;
  const int cg = t % G, kg = t / G;
  const int64_t kb = (K * split / splits) & ~int64_t(7);
  const int64_t ke = split == splits - 1 ? K : ((K * (split + 1) / splits) & ~int64_t(7));
  const int row0 = tab.seg.row_start[seg], rows = tab.seg.row_start[seg + 1] - row0;
  const int total = tab.seg.total_rows;
  for (int r0 = 0; r0 < rows; r0 += ROWS) {
    float acc[ROWS][8];
#pragma unroll
    for (int rr = 0; rr < ROWS; ++rr)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[rr][j] = 0.f;
    if (active) {
      const __nv_bfloat16* xr[ROWS];
#pragma unroll
      for (int rr = 0; rr < ROWS; ++rr)
        xr[rr] = tab.x[seg] + static_cast<int64_t>(min(r0 + rr, rows - 1)) * x_stride;
      for (int64_t k = kb + kg; k < ke; k += kgroups) {
        float a[8];
        load8(A + k * R + cg * 8, a);
#pragma unroll
        for (int rr = 0; rr < ROWS; ++rr) {
          const float xv = __bfloat162float(xr[rr][k]);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[rr][j] = fmaf(xv, a[j], acc[rr][j]);
        }
      }
    }
#pragma unroll
    for (int rr = 0; rr < ROWS; ++rr)
#pragma unroll
      for (int j = 0; j < 8; ++j) red[t * (ROWS * 8) + rr * 8 + j] = acc[rr][j];
    __syncthreads();
    for (int o = t; o < ROWS * R; o += 256) {
      const int rr = o / R, c = o % R;
      if (r0 + rr < rows) {
        float s = 0.f;
        for (int g = 0; g < kgroups; ++g) s += red[(g * G + c / 8) * (ROWS * 8) + rr * 8 + (c & 7)];
        ws[(static_cast<int64_t>(split) * total + row0 + r0 + rr) * R + c] = s;
      }
    }
    __syncthreads();
  }
}

// ---- LoRA expand + round epilogue ---------------------------------------------------
// CTA = (segment, column tile of 256 outputs), one thread per output column;
// the bf16 shrink result t of the segment's rows is rebuilt in shared memory
// from the fp32 partials.
template <int RANK>
__global__ void __launch_bounds__(256) lora_expand_kernel(const __grid_constant__ LoraExpandTable tab,
                                                          const ExpandParams p,
                                                          const float* __restrict__ ws) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  extern __shared__ float tsm[];  // [rows_chunk][R]
  constexpr int kRowsChunk = 16;
  const int seg = blockIdx.x;
  const int R = RANK * p.nblocks;
  const int64_t n_out = p.mode == kExpandSiluMul ? p.n_total / 2 : p.n_total;
  const int64_t n = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x;
  const __nv_bfloat16* B = tab.B[seg];
  const int row0 = tab.seg.row_start[seg], rows = tab.seg.row_start[seg + 1] - row0;
  const int total = tab.seg.total_rows;
  // This thread's B rows (one, or gate+up for the SwiGLU epilogue), kept in registers.
  float b0[RANK], b1[RANK];
  int blk0 = 0, blk1 = 1;
  const bool live = n < n_out;
  if (B && live) {
    const int64_t c0 = n;
    blk0 = c0 < p.block_end[0] ? 0 : (c0 < p.block_end[1] ? 1 : 2);
#pragma unroll
    for (int j = 0; j < RANK; j += 8) {
      float v[8];
      load8(B + c0 * RANK + j, v);
#pragma unroll
      for (int q = 0; q < 8; ++q) b0[j + q] = v[q];
    }
    if (p.mode == kExpandSiluMul) {
      const int64_t c1 = n + n_out;
      blk1 = c1 < p.block_end[0] ? 0 : (c1 < p.block_end[1] ? 1 : 2);
#pragma unroll
      for (int j = 0; j < RANK; j += 8) {
        float v[8];
        load8(B + c1 * RANK + j, v);
#pragma unroll
        for (int q = 0; q < 8; ++q) b1[j + q] = v[q];
      }
    }
  }
  for (int r0 = 0; r0 < rows; r0 += kRowsChunk) {
    const int nr = min(kRowsChunk, rows - r0);
    if (B) {
      __syncthreads();
      for (int o = threadIdx.x; o < nr * R; o += blockDim.x) {
        const int rr = o / R, c = o % R;
        float s = 0.f;
        for (int sp = 0; sp < p.splits; ++sp)
          s += ws[(static_cast<int64_t>(sp) * total + row0 + r0 + rr) * R + c];
        tsm[rr * R + c] = bf(s);  // t is a bf16 tensor in the reference
      }
      __syncthreads();
    }
    if (!live) continue;
    for (int rr = 0; rr < nr; ++rr) {
      const int64_t lr = r0 + rr;
      const __nv_bfloat16* base = tab.base[seg] + lr * p.base_stride;
      __nv_bfloat16* out = tab.out[seg] + lr * p.out_stride;
      float d0 = 0.f, d1 = 0.f;
      if (B) {
        const float* t = tsm + rr * R;
#pragma unroll
        for (int j = 0; j < RANK; ++j) d0 = fmaf(t[blk0 * RANK + j], b0[j], d0);
        d0 = bf(d0);
        if (p.post_scale != 0.f) d0 = bf(d0 * p.post_scale);
        if (p.mode == kExpandSiluMul) {
#pragma unroll
          for (int j = 0; j < RANK; ++j) d1 = fmaf(t[blk1 * RANK + j], b1[j], d1);
          d1 = bf(d1);
        }
      }
      if (p.mode == kExpandSiluMul) {
        const float g = B ? bf(__bfloat162float(base[n]) + d0) : __bfloat162float(base[n]);
        const float u = B ? bf(__bfloat162float(base[n + n_out]) + d1) : __bfloat162float(base[n + n_out]);
        const float sg = bf(g / (1.f + __expf(-g)));
        out[n] = __float2bfloat16_rn(sg * u);
      } else {
        float v = B ? bf(__bfloat162float(base[n]) + d0) : __bfloat162float(base[n]);
        if (p.mode == kExpandResidual) v = __bfloat162float(tab.resid[seg][lr * p.resid_stride + n]) + v;
        out[n] = __float2bfloat16_rn(v);
      }
    }
  }
}

// ---- RoPE + KV append ----------------------------------------------------------------
__global__ void __launch_bounds__(256) rope_append_kernel(const __grid_constant__ AttnTable tab,
                                                          const AttnParams p) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int gr = blockIdx.x;
  const int s = seg_of_row(tab.seg, gr);
  const int local = gr - tab.seg.row_start[s];
  const int pos = *tab.seqlen[s] + local;
  const int D = p.head_dim, half = D / 2;
  const __nv_bfloat16* row = tab.qkv[s] + static_cast<int64_t>(local) * p.qkv_stride;
  const __nv_bfloat16* cs = p.cos_sin + static_cast<int64_t>(pos) * D;
  const int page = tab.block_table[s][pos / p.page];
  const int off = pos % p.page;
  const int64_t kv_row = (static_cast<int64_t>(page) * p.page + off) * p.hkv;
  const int q_pairs = p.hq * half, k_pairs = p.hkv * half;
  for (int i = threadIdx.x; i < q_pairs + k_pairs; i += blockDim.x) {
    const bool is_q = i < q_pairs;
    const int ii = is_q ? i : i - q_pairs;
    const int h = ii / half, d = ii % half;
    const __nv_bfloat16* src = row + (is_q ? 0 : p.hq * D) + h * D;
    const float x = __bfloat162float(src[d]), y = __bfloat162float(src[d + half]);
    const float c = __bfloat162float(cs[d]), sn = __bfloat162float(cs[half + d]);
    const float o1 = bf(bf(x * c) - bf(y * sn));
    const float o2 = bf(bf(y * c) + bf(x * sn));
    __nv_bfloat16* dst = is_q ? p.q_rot + static_cast<int64_t>(gr) * p.hq * D + h * D
                              : tab.k_cache[s] + (kv_row + h) * D;
    dst[d] = __float2bfloat16_rn(o1);
    dst[d + half] = __float2bfloat16_rn(o2);
  }
  const __nv_bfloat16* vsrc = row + (p.hq + p.hkv) * D;
  for (int i = threadIdx.x; i < p.hkv * D; i += blockDim.x)
    tab.v_cache[s][kv_row * D + i] = vsrc[i];
}

// ---- paged attention -------------------------------------------------------------------
// The work of one call is a stream of units, one unit = one 16-token page of
// one token row (all kv heads): rows in order, then pages. Each CTA takes an
// equal contiguous range of at least `min_units` units, so every CTA does the
// same amount of work whatever the rows' context lengths; where its range
// crosses a row boundary it finishes one partial result ("piece") and starts
// the next.
// A CTA has one warp per kv head. Warp w streams its head's slice of each page
// (K and V token rows, 256 B each, plus the G query rows of its head group at
// the first page of a piece) into its own slots of a ring of page stages with
// cp.async, zero-filling tokens past the causal end; the warps never wait for
// one another. Token rows sit hkv * 256 + 16 bytes apart, so the 8 rows one
// ldmatrix reads fall in 8 different bank groups. Per page the warp computes,
// on tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate), with the
// 16 tokens as the M dimension and the G query heads (padded to 8) as N:
//   S^T[tok, head]  = K[tok, :] . Q[head, :]      (A = K via ldmatrix, B = Q^T)
//   P = exp2(S*scale*log2e - m)                   (online softmax per head)
//   O^T[dim, head] += V^T[dim, tok] . P^T[tok, head]  (A = V^T via ldmatrix.trans,
//                                                      B = P^T from registers)
// Each piece writes one record [m, l, o[128]] per query head at
// [row][head][piece][...], the piece index counted from the first CTA whose
// range touches the row; attention_combine_kernel merges them.
constexpr int kD = 128;
constexpr int kPageTok = 16;
constexpr int kAttnStagesMax = 4;
constexpr int kAttnMaxHkv = 8;
constexpr int kAttnMaxRows = 256;
constexpr int kMinUnits = 8;                             // pages per CTA at least
constexpr int kAttnSmemMax = 227 * 1024 - 8192;          // dynamic ring budget (static tables take ~5 KB)
constexpr uint64_t kAttnWaitNs = 2000000000ull;

// Tuning overrides (0 = automatic): minimum pages per CTA, ring depth, kv
// head groups per page (CTAs sharing one page's heads).
std::atomic<int> g_attn_min_units{0};
std::atomic<int> g_attn_stages{0};
std::atomic<int> g_attn_groups{0};
std::atomic<int> g_attn_no_pair{0};  // tuning: never pair a slot's rows
std::atomic<int> g_attn_tma{1};      // K/V pages by TMA where every row's pages share one cache

__host__ __device__ __forceinline__ int attn_row_bytes(int hkv) { return hkv * kD * 2 + 16; }
// One page stage: K and V token rows of the CTA's kv heads, and the query
// rows of `qrows` token rows (a group) for its query heads.
__host__ __device__ __forceinline__ int attn_stage_bytes(int hq, int hkv, int qrows = 1) {
  return 2 * kPageTok * attn_row_bytes(hkv) + qrows * hq * kD * 2;
}

// TMA layout of one warp's share of a page stage: its kv head's K then V
// slice of the page, each as two 128B-swizzled [16 tokens][64 dims] halves
// (2 KB each), then the query rows (dense), padded to 1024 bytes so every
// warp's halves start on the 1024-byte boundary the swizzle pattern needs.
__host__ __device__ __forceinline__ int attn_tma_warp_bytes(int G, int qrows = 1) {
  return 4 * kPageTok * 128 + (qrows * G * kD * 2 + 1023) / 1024 * 1024;
}

// The partial scratch starts with a header the combine step reads: [0] units
// per CTA, [1 + 2r] and [2 + 2r] the page prefix at the start and the end of
// row r's group (r = 0..rows-1), padded to 32 floats.
__host__ __device__ __forceinline__ int64_t attn_hdr_floats(int rows) { return (2 * rows + 1 + 31) / 32 * 32; }

// Units per CTA: at least min_units, and enough that `grid` CTAs cover all.
__device__ __forceinline__ int64_t attn_units_per_cta(int64_t total, int grid, int min_units) {
  const int64_t w = (total + grid - 1) / grid;
  return w > min_units ? w : min_units;
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int kStages, bool kTma>
__global__ void __launch_bounds__(kAttnMaxHkv * 32, 1)
    paged_attention_kernel(const __grid_constant__ AttnTable tab, const AttnParams p, int max_pieces,
                           int min_units, int pair, float* __restrict__ part,
                           const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(128) uint8_t att_dyn_raw[];
  // the TMA path's swizzled halves sit on 1024-byte boundaries
  uint8_t* const att_dyn =
      kTma ? reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(att_dyn_raw) + 1023) & ~uintptr_t(1023))
           : att_dyn_raw;
  __shared__ __align__(8) uint64_t tbar[kAttnMaxHkv][kAttnStagesMax];  // TMA: one per (warp, stage)
  __shared__ int pre[kAttnMaxRows + 1];  // page prefix over groups
  __shared__ int keys[kAttnMaxRows];     // keys (causal length) of each row
  __shared__ int gfirst[kAttnMaxRows];   // first row of each group
  __shared__ int gcount[kAttnMaxRows];   // rows of each group (1 or 2)
  __shared__ int rgroup[kAttnMaxRows];   // group of each row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the kv heads are split into gridDim.y groups; this CTA's group is
  // blockIdx.y and it holds only that group's slices of each page
  const int hkv = p.hkv, G = p.hq / p.hkv;
  const int hkv_c = hkv / static_cast<int>(gridDim.y);
  const int row_bytes = attn_row_bytes(hkv_c);
  const int kv_bytes = kPageTok * row_bytes;
  // pair: two consecutive rows of a slot share each page read (their query
  // heads fill the MMA's 8 columns: column = 4 * row-in-group + head)
  const int qrows = pair ? 2 : 1;
  const int wblk = attn_tma_warp_bytes(G, qrows);
  const int stage_bytes = kTma ? hkv_c * wblk : attn_stage_bytes(hkv_c * G, hkv_c, qrows);
  if (kTma && lane == 0) {
    for (int st = 0; st < kStages; ++st) ptx::mbar_init(&tbar[warp][st], 1);
    ptx::fence_mbar_init();
  }

  // Page prefix over the rows (every CTA derives the same unit stream). The
  // context lengths and block tables are not written by the launch just
  // ahead of this one (that launch writes the new tokens' K/V and q): the
  // prefix, this CTA's range and its first page id are set up before
  // waiting for it.
  const int rows = tab.seg.total_rows;
  __shared__ int ngroups_sh;
  if (warp == 0) {
    // rows -> keys and groups (a group starts at every row, or with pairing
    // at every other row of a slot)
    int gcarry = 0;
    for (int r0 = 0; r0 < rows; r0 += 32) {
      const int r = r0 + lane;
      bool start = false;
      int n_in = 1;
      if (r < rows) {
        const int sg = seg_of_row(tab.seg, r);
        const int local = r - tab.seg.row_start[sg];
        keys[r] = *tab.seqlen[sg] + local + 1;
        start = !pair || (local & 1) == 0;
        if (pair && start && r + 1 < tab.seg.row_start[sg + 1]) n_in = 2;
      }
      const unsigned m = __ballot_sync(0xffffffffu, start);
      const int gi = gcarry + __popc(m & ((1u << lane) - 1u));
      if (start) {
        gfirst[gi] = r;
        gcount[gi] = n_in;
        rgroup[r] = gi;
        if (n_in == 2) rgroup[r + 1] = gi;
      }
      gcarry += __popc(m);
    }
    if (lane == 0) ngroups_sh = gcarry;
    __syncwarp();
    // page prefix over groups: a group has the pages of its last row
    int carry = 0;
    for (int j0 = 0; j0 < gcarry; j0 += 32) {
      const int j = j0 + lane;
      int v = 0;
      if (j < gcarry) v = (keys[gfirst[j] + gcount[j] - 1] + kPageTok - 1) / kPageTok;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      if (j < gcarry) pre[j + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) pre[0] = 0;
  }
  __syncthreads();
  const int ngroups = ngroups_sh;
  const int64_t total = pre[ngroups];
  const int64_t W = attn_units_per_cta(total, gridDim.x, min_units);
  float* const recs = part + attn_hdr_floats(rows);
  const int64_t u0 = static_cast<int64_t>(blockIdx.x) * W;
  const int64_t u1 = min(total, u0 + W);
  const bool idle = u0 >= u1;
  const int nunits = idle ? 0 : static_cast<int>(u1 - u0);
  int r_start;  // the first group of this CTA's range
  {
    int lo = 0, hi = ngroups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pre[mid] <= u0) lo = mid;
      else hi = mid - 1;
    }
    r_start = lo;
  }
  const int t_start = static_cast<int>(u0 - pre[r_start]);

  const int kvh = static_cast<int>(blockIdx.y) * hkv_c + warp;  // this warp's kv head
  const uint32_t sm0 = ptx::smem_addr(att_dyn);
  const uint32_t head_off = warp * kD * 2;
  const uint32_t q_off = 2 * kv_bytes + warp * qrows * G * kD * 2;  // this head's query rows in a stage

  // ---- loads: this warp's slice of unit (lr, lt) into stage `st` ----
  const int ld_tok = lane >> 4, ld_ch = lane & 15;  // token parity and 16-byte chunk of this lane
  // load position (row lr, page lt), its slot, and its page id fetched one
  // unit ahead so the copies of a page never wait on the block-table read
  int lr = r_start, lt = t_start;  // load position: group lr, page lt
  int lsg = idle ? 0 : seg_of_row(tab.seg, gfirst[lr]);
  int next_page = idle ? 0 : tab.block_table[lsg][lt];
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  if (blockIdx.x == 0 && blockIdx.y == 0 && warp == 0) {
    int* hdr = reinterpret_cast<int*>(part);
    if (lane == 0) hdr[0] = static_cast<int>(W);
    for (int r = lane; r < rows; r += 32) {
      hdr[1 + 2 * r] = pre[rgroup[r]];
      hdr[2 + 2 * r] = pre[rgroup[r] + 1];
    }
  }
  if (idle) return;
  auto issue = [&](int j) {
    const int st = j % kStages;
    const uint32_t ss = sm0 + st * stage_bytes;
    const int glast = gfirst[lr] + gcount[lr] - 1;  // the group's longest row
    const int live = min(kPageTok, keys[glast] - lt * kPageTok);
    const int64_t page = next_page;
    if constexpr (kTma) {
      // one lane issues the warp's K and V halves (4 boxes) and, at a new
      // piece, the group's query rows; a missing second row reads as zeros
      uint8_t* wb = att_dyn + st * stage_bytes + warp * wblk;
      const bool newq = j == 0 || lt == 0;
      uint32_t qbytes = 0;
      if (newq)
        for (int ri = 0; ri < qrows; ++ri) {
          if (ri < gcount[lr]) {
            qbytes += G * kD * 2;
          } else {
            uint4* z = reinterpret_cast<uint4*>(wb + 4 * kPageTok * 128 + ri * G * kD * 2);
            for (int e = lane; e < G * kD * 2 / 16; e += 32) z[e] = make_uint4(0u, 0u, 0u, 0u);
            ptx::fence_proxy_async_smem();  // before a later copy into the same bytes
          }
        }
      __syncwarp();
      if (lane == 0) {
        ptx::fence_proxy_async_smem();
        uint64_t* bar = &tbar[warp][st];
        ptx::mbar_arrive_expect_tx(bar, 4 * kPageTok * 128 + qbytes);
        const int tok0 = static_cast<int>(page * p.page);
        const uint32_t ws = ptx::smem_addr(wb);
        ptx::tma_load_3d(ws, &kmap, bar, 0, kvh, tok0);
        ptx::tma_load_3d(ws + kPageTok * 128, &kmap, bar, 64, kvh, tok0);
        ptx::tma_load_3d(ws + 2 * kPageTok * 128, &vmap, bar, 0, kvh, tok0);
        ptx::tma_load_3d(ws + 3 * kPageTok * 128, &vmap, bar, 64, kvh, tok0);
        if (newq)
          for (int ri = 0; ri < qrows && ri < gcount[lr]; ++ri)
            ptx::bulk_load(wb + 4 * kPageTok * 128 + ri * G * kD * 2,
                           p.q_rot + (static_cast<int64_t>(gfirst[lr] + ri) * p.hq + kvh * G) * kD,
                           static_cast<uint32_t>(G * kD * 2), bar);
      }
      (void)live;
    } else {
      const int64_t e0 = ((page * p.page + ld_tok) * hkv + kvh) * kD + ld_ch * 8;  // element offset, token ld_tok
      const __nv_bfloat16* kp = tab.k_cache[lsg] + e0;
      const __nv_bfloat16* vp = tab.v_cache[lsg] + e0;
      const int64_t tstep = 2 * hkv * kD;  // two tokens
#pragma unroll
      for (int i = 0; i < kPageTok / 2; ++i) {
        const int tok = ld_tok + 2 * i;
        const bool ok = tok < live;
        const uint32_t d = ss + tok * row_bytes + head_off + ld_ch * 16;
        ptx::cp_async_16(d, ok ? static_cast<const void*>(kp + i * tstep) : static_cast<const void*>(kp), ok ? 16u : 0u);
        ptx::cp_async_16(d + kv_bytes, ok ? static_cast<const void*>(vp + i * tstep) : static_cast<const void*>(vp),
                         ok ? 16u : 0u);
      }
      if (j == 0 || lt == 0) {
        // the group's query rows (a missing second row reads as zeros)
        for (int ri = 0; ri < qrows; ++ri) {
          const bool have = ri < gcount[lr];
          const char* qp = reinterpret_cast<const char*>(
              p.q_rot + (static_cast<int64_t>(gfirst[lr] + (have ? ri : 0)) * p.hq + kvh * G) * kD);
          for (int e = lane; e < G * kD * 2 / 16; e += 32)
            ptx::cp_async_16(ss + q_off + (ri * G * kD * 2) + e * 16, qp + e * 16, have ? 16u : 0u);
        }
      }
    }
    if (++lt == pre[lr + 1] - pre[lr]) {
      lt = 0;
      ++lr;
      if (lr < ngroups) lsg = seg_of_row(tab.seg, gfirst[lr]);
    }
    if (j + 1 < nunits) next_page = tab.block_table[lsg][lt];
  };
#pragma unroll
  for (int i = 0; i < kStages - 1; ++i) {
    if (i < nunits) issue(i);
    ptx::cp_async_commit();
  }

  const int g = lane >> 2, c = lane & 3;  // mma fragment coordinates
  const int mi = lane >> 3, r8 = lane & 7;  // ldmatrix matrix / row of this lane
  const float sl2 = p.scale * 1.4426950408889634f;
  uint32_t qb[8][2];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads 2c, 2c+1
  float o[8][4];                                            // O^T tiles: dims 16mt + (g, g+8) x heads (2c, 2c+1)
  int r = r_start, t = t_start;
  for (int j = 0; j < nunits; ++j) {
    const int st = j % kStages;
    const uint32_t ss = sm0 + st * stage_bytes;
    const int tiles = pre[r + 1] - pre[r];
    if constexpr (kTma) {
      ptx::mbar_wait(&tbar[warp][st], (j / kStages) & 1, nullptr, 0, kAttnWaitNs);
      // V token rows past the group's causal end: zeros (the page may hold
      // stale values there; their weights are 0, but 0 * NaN is not)
      const int live = min(kPageTok, keys[gfirst[r] + gcount[r] - 1] - t * kPageTok);
      if (live < kPageTok) {
        uint4* v0 = reinterpret_cast<uint4*>(att_dyn + st * stage_bytes + warp * wblk + 2 * kPageTok * 128);
        for (int e = lane; e < 2 * (kPageTok - live) * 8; e += 32) {
          const int half = e / ((kPageTok - live) * 8), rem = e % ((kPageTok - live) * 8);
          v0[half * kPageTok * 8 + (live + rem / 8) * 8 + rem % 8] = make_uint4(0u, 0u, 0u, 0u);
        }
        ptx::fence_proxy_async_smem();  // before a later copy into the same bytes
      }
      __syncwarp();
      if (j + kStages - 1 < nunits) issue(j + kStages - 1);
    } else {
      ptx::cp_async_wait_group<kStages - 2>();
      __syncwarp();
      if (j + kStages - 1 < nunits) issue(j + kStages - 1);
      ptx::cp_async_commit();
    }
    // causal length of this thread's columns (2c, 2c+1: row c >> 1 of the group)
    const int my_ri = pair ? (c >> 1) : 0;
    const int L = (pair && my_ri >= gcount[r]) ? 0 : keys[gfirst[r] + my_ri];
    if (j == 0 || t == 0) {
      // new piece: Q^T as the B operand (k = dims, n = column g: query head
      // g & 3 of the group's row g >> 2 with pairing, head g without),
      // fresh softmax state
      const uint8_t* qs = att_dyn + st * stage_bytes + (kTma ? warp * wblk + 4 * kPageTok * 128 : q_off);
      const int q_ri = pair ? (g >> 2) : 0, q_h = pair ? (g & 3) : g;
      const bool real = q_h < G && q_ri < qrows;
      const int q_col = q_ri * G + q_h;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qb[ks][0] = real ? *reinterpret_cast<const uint32_t*>(qs + (q_col * kD + ks * 16 + 2 * c) * 2) : 0u;
        qb[ks][1] = real ? *reinterpret_cast<const uint32_t*>(qs + (q_col * kD + ks * 16 + 8 + 2 * c) * 2) : 0u;
      }
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    }
    // S^T = K Q^T: A = K rows (tokens) x 16 dims per k-step, two chains
    float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int tok = (mi & 1) * 8 + r8;
      const uint32_t a_row = ss + tok * row_bytes + head_off + (mi >> 1) * 16;
      // TMA layout: 16-byte chunk c of token row `tok` of a 64-dim half sits
      // at chunk c ^ (tok & 7) (128-byte swizzle)
      const uint32_t kb = ss + warp * wblk + tok * 128;
      auto kaddr = [&](int ch) { return kb + (ch >> 3) * (kPageTok * 128) + (((ch & 7) ^ (tok & 7)) << 4); };
#pragma unroll
      for (int ks = 0; ks < 8; ks += 2) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        ldsm_x4(kTma ? kaddr(ks * 2 + (mi >> 1)) : a_row + ks * 32, a0, a1, a2, a3);
        ldsm_x4(kTma ? kaddr(ks * 2 + 2 + (mi >> 1)) : a_row + ks * 32 + 32, b0, b1, b2, b3);
        mma_bf16_16816(sa, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
        mma_bf16_16816(sb, b0, b1, b2, b3, qb[ks + 1][0], qb[ks + 1][1]);
      }
    }
    // online softmax; this thread holds tokens g, g+8 of heads 2c, 2c+1
    const int tok0 = t * kPageTok;
    const bool live_lo = tok0 + g < L, live_hi = tok0 + g + 8 < L;
    float v0 = live_lo ? (sa[0] + sb[0]) * sl2 : -INFINITY;  // tok g,   head 2c
    float v1 = live_lo ? (sa[1] + sb[1]) * sl2 : -INFINITY;  // tok g,   head 2c+1
    float v2 = live_hi ? (sa[2] + sb[2]) * sl2 : -INFINITY;  // tok g+8, head 2c
    float v3 = live_hi ? (sa[3] + sb[3]) * sl2 : -INFINITY;  // tok g+8, head 2c+1
    float mx0 = fmaxf(v0, v2), mx1 = fmaxf(v1, v3);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float corr0 = mn0 == -INFINITY ? 1.f : exp2f(m0 - mn0);
    const float corr1 = mn1 == -INFINITY ? 1.f : exp2f(m1 - mn1);
    const float p0 = mn0 == -INFINITY ? 0.f : exp2f(v0 - mn0);
    const float p2 = mn0 == -INFINITY ? 0.f : exp2f(v2 - mn0);
    const float p1 = mn1 == -INFINITY ? 0.f : exp2f(v1 - mn1);
    const float p3 = mn1 == -INFINITY ? 0.f : exp2f(v3 - mn1);
    l0 = l0 * corr0 + p0 + p2;
    l1 = l1 * corr1 + p1 + p3;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      o[mt][0] *= corr0;
      o[mt][2] *= corr0;
      o[mt][1] *= corr1;
      o[mt][3] *= corr1;
    }
    // P^T as the B operand: thread (g, c) needs P[head g][tok 2c, 2c+1, 2c+8, 2c+9],
    // held by lanes (2c, g/2) and (2c+1, g/2) as (tok, tok+8) pairs of heads
    // 2c', 2c'+1
    uint32_t pb0, pb1;
    {
      const uint32_t xe = pack_bf16(p0, p2), xo = pack_bf16(p1, p3);
      const int srcA = (2 * c) * 4 + (g >> 1), srcB = srcA + 4;
      const uint32_t ae = __shfl_sync(0xffffffffu, xe, srcA), ao = __shfl_sync(0xffffffffu, xo, srcA);
      const uint32_t be = __shfl_sync(0xffffffffu, xe, srcB), bo = __shfl_sync(0xffffffffu, xo, srcB);
      const uint32_t A = (g & 1) ? ao : ae, B = (g & 1) ? bo : be;
      pb0 = __byte_perm(A, B, 0x5410);
      pb1 = __byte_perm(A, B, 0x7632);
    }
    // O^T += V^T P^T: A = V^T (16 dims x 16 tokens) via ldmatrix.trans
    {
      const int tok = (mi >> 1) * 8 + r8;
      const uint32_t a_row = ss + kv_bytes + tok * row_bytes + head_off + (mi & 1) * 16;
      const uint32_t vb = ss + warp * wblk + 2 * kPageTok * 128 + tok * 128;
      auto vaddr = [&](int ch) { return vb + (ch >> 3) * (kPageTok * 128) + (((ch & 7) ^ (tok & 7)) << 4); };
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_trans(kTma ? vaddr(mt * 2 + (mi & 1)) : a_row + mt * 32, a0, a1, a2, a3);
        mma_bf16_16816(o[mt], a0, a1, a2, a3, pb0, pb1);
      }
    }
    if (j == nunits - 1 || t == tiles - 1) {
      // end of a piece: its record per query head
      float lt0 = l0, lt1 = l1;
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        lt0 += __shfl_xor_sync(0xffffffffu, lt0, off);
        lt1 += __shfl_xor_sync(0xffffffffu, lt1, off);
      }
      const int piece = static_cast<int>(blockIdx.x - pre[r] / W);
      if (piece < max_pieces) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int col = 2 * c + hh;
          const int ri = pair ? (col >> 2) : 0, hg = pair ? (col & 3) : col;
          if (hg >= G || ri >= gcount[r]) continue;
          const int64_t row = gfirst[r] + ri;
          float* rec = recs + ((row * p.hq + kvh * G + hg) * max_pieces + piece) * (kD + 2);
          if (g == 0) {
            rec[0] = hh ? m1 : m0;
            rec[1] = hh ? lt1 : lt0;
          }
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            rec[2 + mt * 16 + g] = o[mt][hh];
            rec[2 + mt * 16 + g + 8] = o[mt][2 + hh];
          }
        }
      }
    }
    __syncwarp();
    if (++t == tiles) {
      t = 0;
      ++r;
    }
  }
  if constexpr (!kTma) ptx::cp_async_wait_all();
}

// Merges the pieces of one (row, head): O = sum_j 2^(m_j - M) o_j /
// sum_j 2^(m_j - M) l_j, written as bf16 to the slot's attention output. The
// pieces of a row are found from the header the attention kernel wrote (page
// prefix over rows, units per CTA). With a shrink side (A != nullptr) it also
// emits this head's share of the O projection's LoRA shrink:
// ws[row][h][j] = sum_d out[d] * A[h*128 + d, j]; the adapter rows are read
// before waiting for the attention kernel.
__global__ void __launch_bounds__(128) attention_combine_kernel(const __grid_constant__ AttnTable tab,
                                                                const AttnParams p, int max_pieces,
                                                                const float* __restrict__ part,
                                                                const __grid_constant__ ShrinkSide sh) {
  const int gr = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int s = seg_of_row(tab.seg, gr);
  const int local = gr - tab.seg.row_start[s];
  const __nv_bfloat16* A = sh.A[s];
  const int nvec = sh.r / 8;
  uint4 av[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    av[j] = (A && j < nvec) ? reinterpret_cast<const uint4*>(A + (static_cast<int64_t>(h) * kD + d) * sh.r)[j]
                            : make_uint4(0u, 0u, 0u, 0u);
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  // The header and the first kBatch records are loaded together (a record
  // slot past the row's piece count holds stale data and is not used), so
  // the common case costs one round trip to L2.
  constexpr int kBatch = 12;
  const int* hdr = reinterpret_cast<const int*>(part);
  const float* rec = part + attn_hdr_floats(tab.seg.total_rows) +
                     (static_cast<int64_t>(gr) * p.hq + h) * max_pieces * (kD + 2);
  float mv[kBatch], lv[kBatch], ov[kBatch];
#pragma unroll
  for (int i = 0; i < kBatch; ++i) {
    const bool in = i < max_pieces;
    mv[i] = in ? rec[i * (kD + 2)] : 0.f;
    lv[i] = in ? rec[i * (kD + 2) + 1] : 0.f;
    ov[i] = in ? rec[i * (kD + 2) + 2 + d] : 0.f;
  }
  const int W = hdr[0], p0 = hdr[1 + 2 * gr], p1 = hdr[2 + 2 * gr];
  const int nch = min((p1 - 1) / W - p0 / W + 1, max_pieces);
  float M = -INFINITY, lsum = 0.f, acc = 0.f;
  if (nch <= kBatch) {
#pragma unroll
    for (int i = 0; i < kBatch; ++i)
      if (i < nch) M = fmaxf(M, mv[i]);
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (i < nch) {
        const float wgt = mv[i] == -INFINITY ? 0.f : exp2f(mv[i] - M);
        lsum += wgt * lv[i];
        acc += wgt * ov[i];
      }
    }
  } else {
    for (int i = 0; i < nch; ++i) M = fmaxf(M, rec[i * (kD + 2)]);
    for (int i = 0; i < nch; ++i) {
      const float mi = rec[i * (kD + 2)];
      const float wgt = mi == -INFINITY ? 0.f : exp2f(mi - M);
      lsum += wgt * rec[i * (kD + 2) + 1];
      acc += wgt * rec[i * (kD + 2) + 2 + d];
    }
  }
  const __nv_bfloat16 ob = __float2bfloat16_rn(lsum > 0.f ? acc / lsum : 0.f);
  tab.out[s][static_cast<int64_t>(local) * p.out_stride + h * kD + d] = ob;
  if (!A) return;
  // shrink share of this head (r <= 32 columns)
  __shared__ float red[4][32];
  const float x = __bfloat162float(ob);
  const int w = d >> 5, lane = d & 31;
#pragma unroll
  for (int jv = 0; jv < 4; ++jv) {
    if (jv >= nvec) break;
    const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&av[jv]);
#pragma unroll
    for (int e2 = 0; e2 < 4; ++e2) {
      const float2 f = __bfloat1622float2(hv[e2]);
      float t0 = x * f.x, t1 = x * f.y;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        t0 += __shfl_xor_sync(0xffffffffu, t0, off);
        t1 += __shfl_xor_sync(0xffffffffu, t1, off);
      }
      if (lane == 0) {
        red[w][jv * 8 + 2 * e2] = t0;
        red[w][jv * 8 + 2 * e2 + 1] = t1;
      }
    }
  }
  __syncthreads();
  if (d < sh.r) {
    const float v = red[0][d] + red[1][d] + red[2][d] + red[3][d];
    sh.ws[(static_cast<int64_t>(gr) * p.hq + h) * sh.r + d] = v;
  }
}

// ---- RMSNorm ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rms_norm_kernel(const __grid_constant__ NormTable tab,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       int64_t hidden, float eps, int64_t x_stride,
                                                       int64_t out_stride) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int gr = blockIdx.x;
  const int s = seg_of_row(tab.seg, gr);
  const int64_t local = gr - tab.seg.row_start[s];
  const __nv_bfloat16* x = tab.x[s] + local * x_stride;
  __nv_bfloat16* y = tab.out[s] + local * out_stride;
  float ss = 0.f;
  for (int64_t i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    float v[8];
    load8(x + i, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / static_cast<float>(hidden) + eps);
  for (int64_t i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    float v[8], g[8];
    load8(x + i, v);
    load8(w + i, g);
    __align__(16) __nv_bfloat162 o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = __floats2bfloat162_rn(g[2 * j] * bf(v[2 * j] * inv), g[2 * j + 1] * bf(v[2 * j + 1] * inv));
    *reinterpret_cast<uint4*>(y + i) = *reinterpret_cast<uint4*>(o);
  }
}

// ---- batched copies / counters -------------------------------------------------------
// One CTA per copy; 16-byte vectors when both ends and the size allow it.
__global__ void copy_rows_kernel(const __grid_constant__ CopyTable tab) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int i = blockIdx.x;
  const char* src = static_cast<const char*>(tab.src[i]);
  char* dst = static_cast<char*>(tab.dst[i]);
  const int64_t n = tab.bytes[i];
  const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | n) & 15) == 0;
  if (vec) {
    for (int64_t k = threadIdx.x; k < n / 16; k += blockDim.x)
      reinterpret_cast<uint4*>(dst)[k] = reinterpret_cast<const uint4*>(src)[k];
  } else {
    for (int64_t k = threadIdx.x; k < n; k += blockDim.x) dst[k] = src[k];
  }
}

__global__ void advance_i32_kernel(int* p, int n, int delta) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] += delta;
}

}  // namespace

int launch_copy_rows(const CopyTable& tab, int n, cudaStream_t stream) {
  if (n <= 0) return SWL_OK;
  if (n > kMaxSlots) return set_error(SWL_ERR_ARG, "copy_rows: at most %d copies per call", kMaxSlots);
  SWL_CUDA_TRY(launch_kernel(copy_rows_kernel, dim3(n), dim3(256), 0, stream, 1, tab));
  return SWL_OK;
}

int launch_advance_i32(int* p, int n, int delta, cudaStream_t stream) {
  if (n <= 0) return SWL_OK;
  SWL_CUDA_TRY(launch_kernel(advance_i32_kernel, dim3((n + 255) / 256), dim3(256), 0, stream, 1, p, n, delta));
  return SWL_OK;
}

int launch_lora_shrink(const LoraShrinkTable& tab, int64_t K, int R, int64_t x_stride, int splits,
                       float* ws, cudaStream_t stream) {
  if (tab.seg.nseg <= 0 || tab.seg.total_rows <= 0) return SWL_OK;
  if (R % 8 || R <= 0 || R > 256 || K % 8) return set_error(SWL_ERR_ARG, "lora_shrink: R must be a multiple of 8 (<= 256), K of 8");
  if (splits <= 0) return set_error(SWL_ERR_ARG, "lora_shrink: splits must be positive");
  const int rows_max = [&] {
    int m = 0;
    for (int i = 0; i < tab.seg.nseg; ++i) m = std::max(m, tab.seg.row_start[i + 1] - tab.seg.row_start[i]);
    return m;
  }();
  dim3 grid(tab.seg.nseg * splits);
  if (rows_max <= 1) {
    SWL_CUDA_TRY(launch_kernel(lora_shrink_kernel<1>, grid, dim3(256), 256 * 8 * sizeof(float), stream, 1,
                               tab, K, R, x_stride, splits, ws));
  } else {
    SWL_CUDA_TRY(launch_kernel(lora_shrink_kernel<4>, grid, dim3(256), 256 * 32 * sizeof(float), stream, 1,
                               tab, K, R, x_stride, splits, ws));
  }
  return SWL_OK;
}

int launch_lora_expand(const LoraExpandTable& tab, const ExpandParams& p, const float* ws,
                       cudaStream_t stream) {
  if (tab.seg.nseg <= 0 || tab.seg.total_rows <= 0) return SWL_OK;
  if (p.r % 8 || p.r <= 0 || p.r > 32) return set_error(SWL_ERR_ARG, "lora_expand: rank must be 8, 16, 24 or 32");
  if (p.nblocks < 1 || p.nblocks > 3) return set_error(SWL_ERR_ARG, "lora_expand: 1..3 fused projections");
  const int64_t n_out = p.mode == kExpandSiluMul ? p.n_total / 2 : p.n_total;
  dim3 grid(tab.seg.nseg, static_cast<unsigned>((n_out + 255) / 256));
  const size_t smem = 16 * p.r * p.nblocks * sizeof(float);
  switch (p.r) {
    case 8: SWL_CUDA_TRY(launch_kernel(lora_expand_kernel<8>, grid, dim3(256), smem, stream, 1, tab, p, ws)); break;
    case 16: SWL_CUDA_TRY(launch_kernel(lora_expand_kernel<16>, grid, dim3(256), smem, stream, 1, tab, p, ws)); break;
    case 24: SWL_CUDA_TRY(launch_kernel(lora_expand_kernel<24>, grid, dim3(256), smem, stream, 1, tab, p, ws)); break;
    default: SWL_CUDA_TRY(launch_kernel(lora_expand_kernel<32>, grid, dim3(256), smem, stream, 1, tab, p, ws)); break;
  }
  return SWL_OK;
}

int launch_rope_append(const AttnTable& tab, const AttnParams& p, cudaStream_t stream) {
  if (tab.seg.total_rows <= 0) return SWL_OK;
  if (p.head_dim != kD) return set_error(SWL_ERR_ARG, "rope: head_dim must be 128");
  SWL_CUDA_TRY(launch_kernel(rope_append_kernel, dim3(tab.seg.total_rows), dim3(256), 0, stream, 1, tab, p));
  return SWL_OK;
}

AttnSplit attention_split(int total_rows, int hkv, int max_len) {
  // Each CTA takes at least chunk_pages pages of the unit stream, so a row of
  // P pages is cut into at most ceil(P / chunk_pages) + 1 pieces; `chunks`
  // bounds the pieces of any row (the record stride).
  (void)total_rows;
  (void)hkv;
  AttnSplit a;
  const int o = g_attn_min_units.load(std::memory_order_relaxed);
  a.chunk_pages = o > 0 ? o : kMinUnits;
  const int pages = std::max(1, (max_len + kPageTok - 1) / kPageTok);
  a.chunks = (pages + a.chunk_pages - 1) / a.chunk_pages + 1;
  return a;
}

int attention_splits(int total_rows, int hkv, int max_len) {
  return attention_split(total_rows, hkv, max_len).chunks;
}

int64_t attention_part_floats(int total_rows, int hq, int splits) {
  return attn_hdr_floats(total_rows) + static_cast<int64_t>(total_rows) * hq * splits * (kD + 2);
}

namespace {

int sm_count_attn() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <int S, bool Tma>
int launch_attention_stages(const AttnTable& tab, const AttnParams& p, int grid, int groups, int pair, size_t smem,
                            const AttnSplit& sp, const CUtensorMap& kmap, const CUtensorMap& vmap,
                            cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(paged_attention_kernel<S, Tma>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kAttnSmemMax);
  });
  if (attr_err != cudaSuccess)
    return set_error(SWL_ERR_CUDA, "attention: smem attribute: %s", cudaGetErrorString(attr_err));
  SWL_CUDA_TRY(launch_kernel(paged_attention_kernel<S, Tma>, dim3(grid, groups), dim3(p.hkv / groups * 32), smem,
                             stream, 1, tab, p, sp.chunks, sp.chunk_pages, pair, p.part, kmap, vmap));
  return SWL_OK;
}

// The TMA path: every row's K (and V) pages lie in one cache allocation,
// whose extent bounds the tensor map. Returns false when the slots use
// different caches (the per-lane copies then load each slot's own pages).
bool attention_tmaps(const AttnTable& tab, const AttnParams& p, CUtensorMap* kmap, CUtensorMap* vmap) {
  for (int i = 1; i < tab.seg.nseg; ++i)
    if (tab.k_cache[i] != tab.k_cache[0] || tab.v_cache[i] != tab.v_cache[0]) return false;
  const int64_t row = static_cast<int64_t>(p.hkv) * kD * 2;  // bytes per token row
  char *kb = nullptr, *vb = nullptr;
  size_t kn = 0, vn = 0;
  if (allocation_of(tab.k_cache[0], &kb, &kn) != SWL_OK || allocation_of(tab.v_cache[0], &vb, &vn) != SWL_OK)
    return false;
  const int64_t kt = (kb + kn - reinterpret_cast<const char*>(tab.k_cache[0])) / row;
  const int64_t vt = (vb + vn - reinterpret_cast<const char*>(tab.v_cache[0])) / row;
  return encode_kv_page_tmap(kmap, tab.k_cache[0], kt, p.hkv) == SWL_OK &&
         encode_kv_page_tmap(vmap, tab.v_cache[0], vt, p.hkv) == SWL_OK;
}

}  // namespace

int launch_paged_attention(const AttnTable& tab, const AttnParams& p, cudaStream_t stream,
                           const ShrinkSide* shrink) {
  if (tab.seg.total_rows <= 0) return SWL_OK;
  if (p.head_dim != kD || p.page != kPageTok || p.hq <= 0 || p.hkv <= 0 || p.hkv > kAttnMaxHkv ||
      p.hq % p.hkv || p.hq / p.hkv > 8)
    return set_error(SWL_ERR_ARG, "attention: head_dim 128, page 16, 1..%d kv heads, at most 8 query heads per kv head",
                     kAttnMaxHkv);
  if (tab.seg.total_rows > kAttnMaxRows)
    return set_error(SWL_ERR_ARG, "attention: at most %d token rows per call", kAttnMaxRows);
  if (p.max_len <= 0 || p.max_len > (1 << 20)) return set_error(SWL_ERR_ARG, "attention: max_len out of range");
  if (reinterpret_cast<uintptr_t>(p.q_rot) & 15) return set_error(SWL_ERR_ARG, "attention: q must be 16-byte aligned");
  for (int i = 0; i < tab.seg.nseg; ++i)
    if ((reinterpret_cast<uintptr_t>(tab.k_cache[i]) | reinterpret_cast<uintptr_t>(tab.v_cache[i])) & 15)
      return set_error(SWL_ERR_ARG, "attention: KV caches must be 16-byte aligned");
  if (!p.part) return set_error(SWL_ERR_ARG, "attention: missing partial scratch");
  const AttnSplit sp = attention_split(tab.seg.total_rows, p.hkv, p.max_len);
  // kv head groups: CTAs that share a page's heads (each holds only its
  // group's slices, so a smaller ring per CTA and more CTAs per SM)
  const int og = g_attn_groups.load(std::memory_order_relaxed);
  int groups = og > 0 ? og : 1;
  while (groups > 1 && p.hkv % groups) --groups;
  // rows of one slot are paired (one page read for both) when a slot has
  // several rows and two rows' query heads fit the MMA's 8 columns
  int max_seg_rows = 0;
  for (int i = 0; i < tab.seg.nseg; ++i)
    max_seg_rows = std::max(max_seg_rows, tab.seg.row_start[i + 1] - tab.seg.row_start[i]);
  const int pair = (max_seg_rows >= 2 && p.hq / p.hkv <= 4 && !g_attn_no_pair.load(std::memory_order_relaxed)) ? 1 : 0;
  // K/V pages by TMA (one lane per warp issues its kv head's 128B-swizzled
  // halves) when every row's pages lie in one cache; else per-lane copies
  CUtensorMap kmap, vmap;
  memset(&kmap, 0, sizeof(kmap));
  memset(&vmap, 0, sizeof(vmap));
  const bool tma = g_attn_tma.load(std::memory_order_relaxed) != 0 && attention_tmaps(tab, p, &kmap, &vmap);
  const int G = p.hq / p.hkv;
  const int stage_bytes = tma ? p.hkv / groups * attn_tma_warp_bytes(G, pair ? 2 : 1)
                              : attn_stage_bytes(p.hq / groups, p.hkv / groups, pair ? 2 : 1);
  // Page stages per warp by default: with per-lane copies two (one in flight
  // while one is consumed; the 148 KB ring lets a CTA sit beside the RoPE
  // epilogue's CTAs; deeper rings measured no faster); with TMA three
  // (216 KB: 18.0 vs 18.5 us with two at the decode shape, and 1% faster
  // whole steps at contexts U[1024, 4096])
  const int o = g_attn_stages.load(std::memory_order_relaxed);
  const int budget = kAttnSmemMax - (tma ? 1024 : 0);  // TMA: 1024-byte alignment slack
  const int stages = std::min(std::min(kAttnStagesMax, budget / stage_bytes), o > 0 ? o : (tma ? 3 : 2));
  if (stages < 2) return set_error(SWL_ERR_ARG, "attention: page stage of %d bytes too large", stage_bytes);
  const size_t smem = static_cast<size_t>(stages) * stage_bytes + (tma ? 1024 : 0);
  // one CTA per SM, but no more CTAs than the units can keep busy
  const int64_t units_max =
      static_cast<int64_t>(tab.seg.total_rows) * ((p.max_len + kPageTok - 1) / kPageTok);
  const int grid = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>((units_max + sp.chunk_pages - 1) / sp.chunk_pages, sm_count_attn())));
#define SWL_ATTN_LAUNCH(S)                                                                                 \
  (tma ? launch_attention_stages<S, true>(tab, p, grid, groups, pair, smem, sp, kmap, vmap, stream)          \
       : launch_attention_stages<S, false>(tab, p, grid, groups, pair, smem, sp, kmap, vmap, stream))
  switch (stages) {
    case 2: SWL_TRY(SWL_ATTN_LAUNCH(2)); break;
    case 3: SWL_TRY(SWL_ATTN_LAUNCH(3)); break;
    default: SWL_TRY(SWL_ATTN_LAUNCH(4)); break;
  }
#undef SWL_ATTN_LAUNCH
  ShrinkSide none;
  if (!shrink) {
    for (int i = 0; i < kMaxSlots; ++i) none.A[i] = nullptr;
    none.r = 0;
    none.ws = nullptr;
  } else if (shrink->r % 8 || shrink->r > 32) {
    return set_error(SWL_ERR_ARG, "attention: shrink rank must be 8..32 in steps of 8");
  }
  SWL_CUDA_TRY(launch_kernel(attention_combine_kernel, dim3(tab.seg.total_rows, p.hq), dim3(kD), 0, stream, 1,
                             tab, p, sp.chunks, static_cast<const float*>(p.part), shrink ? *shrink : none));
  return SWL_OK;
}

int launch_rms_norm(const NormTable& tab, const __nv_bfloat16* w, int64_t hidden, float eps,
                    int64_t x_stride, int64_t out_stride, cudaStream_t stream) {
  if (tab.seg.total_rows <= 0) return SWL_OK;
  if (hidden % 8) return set_error(SWL_ERR_ARG, "rms_norm: hidden must be a multiple of 8");
  SWL_CUDA_TRY(launch_kernel(rms_norm_kernel, dim3(tab.seg.total_rows), dim3(256), 0, stream, 1, tab, w, hidden, eps,
                             x_stride, out_stride));
  return SWL_OK;
}

int set_attention_pairing(int on) {
  g_attn_no_pair.store(on ? 0 : 1);
  return SWL_OK;
}

int set_attention_tma(int on) {
  g_attn_tma.store(on ? 1 : 0);
  return SWL_OK;
}

int set_attention_tuning(int chunk_pages, int stages, int groups) {
  if (chunk_pages < 0 || chunk_pages > 4096 || (stages != 0 && (stages < 2 || stages > kAttnStagesMax)) ||
      (groups != 0 && groups != 1 && groups != 2 && groups != 4 && groups != 8))
    return set_error(SWL_ERR_ARG, "attention tuning: chunk_pages 0..4096, stages 0 or 2..%d, groups 0/1/2/4/8",
                     kAttnStagesMax);
  g_attn_min_units.store(chunk_pages);
  g_attn_stages.store(stages);
  g_attn_groups.store(groups);
  return SWL_OK;
}

}  // namespace swl
