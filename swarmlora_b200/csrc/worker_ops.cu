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

#include "common.h"
#include "launch.h"
#include "ptx.cuh"
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
// CTA = one warp = (token row, kv head, context split). The warp computes all
// G query heads of the kv head at once on tensor cores (mma.sync m16n8k16,
// bf16 in, fp32 accumulate): per 16-token page,
//   S[head, tok]  = Q[head, :] . K[tok, :]      (A = Q, heads padded to 16 rows;
//                                                B = K^T via ldmatrix)
//   P = exp2(S*scale*log2e - m)                 (online softmax in registers)
//   O[head, dim] += P[head, tok] . V[tok, dim]  (A = P reused from the S
//                                                accumulator, B = V via ldmatrix.trans)
// Pages stream through a 3-stage cp.async ring in shared memory; each 16-byte
// piece of a token row is stored XOR-swizzled by (token & 7) so the 8-row
// ldmatrix reads hit 8 different bank groups. Tokens past the causal end are
// zero-filled and masked. Each CTA writes one record [m, l, o[128]] per
// query head; attention_combine_kernel merges the splits.
constexpr int kD = 128;
constexpr int kPageTok = 16;
constexpr int kAttnStages = 3;
constexpr int kTileBytes = kPageTok * kD * 2;  // one page of K (or V) of one head: 4 KB
constexpr int kMaxSplitPages = 256;

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

__global__ void __launch_bounds__(32) paged_attention_kernel(const __grid_constant__ AttnTable tab,
                                                             const AttnParams p, int splits,
                                                             float* __restrict__ part) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  __shared__ __align__(128) uint8_t kv_sm[kAttnStages][2][kTileBytes];
  __shared__ int pages[kMaxSplitPages];
  const int gr = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  ptx::prefetch_l2_share(p.pf, p.pf_bytes,
                         (split * gridDim.y + kvh) * gridDim.x + gr, gridDim.x * gridDim.y * gridDim.z);
  const int lane = threadIdx.x;
  const int G = p.hq / p.hkv;
  const int g = lane >> 2, c = lane & 3;  // mma fragment coordinates
  const int s = seg_of_row(tab.seg, gr);
  const int local = gr - tab.seg.row_start[s];
  const int L = *tab.seqlen[s] + local + 1;  // causal: keys 0 .. pos
  const int ntiles = (L + kPageTok - 1) / kPageTok;
  const int tb = static_cast<int>(static_cast<int64_t>(ntiles) * split / splits);
  const int te = static_cast<int>(static_cast<int64_t>(ntiles) * (split + 1) / splits);
  const int nt = min(te - tb, kMaxSplitPages);
  const int* bt = tab.block_table[s];
  for (int i = lane; i < nt; i += 32) pages[i] = bt[tb + i];
  __syncwarp();
  const __nv_bfloat16* kc = tab.k_cache[s];
  const __nv_bfloat16* vc = tab.v_cache[s];
  const uint32_t sm0 = static_cast<uint32_t>(__cvta_generic_to_shared(&kv_sm[0][0][0]));

  auto load_tile = [&](int i, int st) {
    const int64_t page = pages[i];
    const int tok0 = (tb + i) * kPageTok;
#pragma unroll 4
    for (int cidx = lane; cidx < 2 * kPageTok * 16; cidx += 32) {
      const int kv = cidx >> 8, cc = cidx & 255;
      const int tok = cc >> 4, ch = cc & 15;
      const bool live = tok0 + tok < L;
      const __nv_bfloat16* src = (kv ? vc : kc) + ((page * p.page + tok) * p.hkv + kvh) * kD + ch * 8;
      const uint32_t dst = sm0 + (st * 2 + kv) * kTileBytes + tok * 256 + ((ch ^ (tok & 7)) << 4);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(live ? src : kc),
                   "r"(live ? 16 : 0)
                   : "memory");
    }
  };
#pragma unroll
  for (int i = 0; i < kAttnStages - 1; ++i) {
    if (i < nt) load_tile(i, i);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  // Q as the A operand: rows = query heads of this kv head (g < G), k = dims.
  uint32_t qa[8][2];
  {
    const bool real = g < G;
    const __nv_bfloat16* qp = p.q_rot + (static_cast<int64_t>(gr) * p.hq + kvh * G + (real ? g : 0)) * kD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = real ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 2 * c) : 0u;
      qa[ks][1] = real ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 8 + 2 * c) : 0u;
    }
  }
  const float sl2 = p.scale * 1.4426950408889634f;
  float m = -INFINITY, l = 0.f;
  float o[16][4];
#pragma unroll
  for (int nt8 = 0; nt8 < 16; ++nt8) o[nt8][0] = o[nt8][1] = o[nt8][2] = o[nt8][3] = 0.f;
  // ldmatrix row address pieces of this lane
  const int mi = lane >> 3, r8 = lane & 7;

  for (int i = 0; i < nt; ++i) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kAttnStages - 2) : "memory");
    __syncwarp();
    const int nx = i + kAttnStages - 1;
    if (nx < nt) load_tile(nx, nx % kAttnStages);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const int st = i % kAttnStages;
    const uint32_t ks_base = sm0 + (st * 2 + 0) * kTileBytes;
    const uint32_t vs_base = sm0 + (st * 2 + 1) * kTileBytes;
    // S = Q K^T for tokens 0-7 (sa) and 8-15 (sb)
    float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      // matrices: (tok 0-7, dims 16ks..+7), (tok 0-7, +8..15), (tok 8-15, ..), (tok 8-15, +8..)
      const int tok = (mi >> 1) * 8 + r8;
      const int ch = ks * 2 + (mi & 1);
      uint32_t b0a, b1a, b0b, b1b;
      ldsm_x4(ks_base + tok * 256 + ((ch ^ (tok & 7)) << 4), b0a, b1a, b0b, b1b);
      mma_bf16_16816(sa, qa[ks][0], 0u, qa[ks][1], 0u, b0a, b1a);
      mma_bf16_16816(sb, qa[ks][0], 0u, qa[ks][1], 0u, b0b, b1b);
    }
    const int tok0 = (tb + i) * kPageTok;
    float sv[4] = {sa[0] * sl2, sa[1] * sl2, sb[0] * sl2, sb[1] * sl2};
    const int tk[4] = {2 * c, 2 * c + 1, 8 + 2 * c, 9 + 2 * c};
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (tok0 + tk[e] >= L) sv[e] = -INFINITY;
    float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m, mx);
    const float corr = (mn == -INFINITY) ? 1.f : exp2f(m - mn);
    float pv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pv[e] = (mn == -INFINITY) ? 0.f : exp2f(sv[e] - mn);
    l = l * corr + (pv[0] + pv[1] + pv[2] + pv[3]);
    m = mn;
    const uint32_t pa0 = pack_bf16(pv[0], pv[1]), pa2 = pack_bf16(pv[2], pv[3]);
#pragma unroll
    for (int nt8 = 0; nt8 < 16; ++nt8) {
      o[nt8][0] *= corr;
      o[nt8][1] *= corr;
    }
    // O += P V: per 16 dims one ldmatrix.trans x4 ->
    // (tok 0-7, dims n0..n0+7), (tok 8-15, n0..), (tok 0-7, n0+8..), (tok 8-15, n0+8..)
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      const int tok = (mi & 1) * 8 + r8;
      const int ch = nd * 2 + (mi >> 1);
      uint32_t b0a, b1a, b0b, b1b;
      ldsm_x4_trans(vs_base + tok * 256 + ((ch ^ (tok & 7)) << 4), b0a, b1a, b0b, b1b);
      mma_bf16_16816(o[2 * nd], pa0, 0u, pa2, 0u, b0a, b1a);
      mma_bf16_16816(o[2 * nd + 1], pa0, 0u, pa2, 0u, b0b, b1b);
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  if (g >= G) return;
  const int h = kvh * G + g;
  float* rec = part + ((static_cast<int64_t>(gr) * p.hq + h) * splits + split) * (kD + 2);
  if (c == 0) {
    rec[0] = m;
    rec[1] = l;
  }
#pragma unroll
  for (int nt8 = 0; nt8 < 16; ++nt8) {
    rec[2 + nt8 * 8 + 2 * c] = o[nt8][0];
    rec[2 + nt8 * 8 + 2 * c + 1] = o[nt8][1];
  }
}

// Merges the context splits of one (row, head): O = sum_s 2^(m_s - M) o_s /
// sum_s 2^(m_s - M) l_s, written as bf16 to the slot's attention output. With
// a shrink side (A != nullptr) it also emits this head's share of the O
// projection's LoRA shrink: ws[row][h][j] = sum_d out[d] * A[h*128 + d, j].
__global__ void __launch_bounds__(128) attention_combine_kernel(const __grid_constant__ AttnTable tab,
                                                                const AttnParams p, int splits,
                                                                const float* __restrict__ part,
                                                                const __grid_constant__ ShrinkSide sh) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int gr = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int s = seg_of_row(tab.seg, gr);
  const int local = gr - tab.seg.row_start[s];
  const float* rec = part + (static_cast<int64_t>(gr) * p.hq + h) * splits * (kD + 2);
  float M = -INFINITY;
  for (int i = 0; i < splits; ++i) M = fmaxf(M, rec[i * (kD + 2)]);
  float lsum = 0.f, acc = 0.f;
  for (int i = 0; i < splits; ++i) {
    const float mi = rec[i * (kD + 2)];
    const float wgt = mi == -INFINITY ? 0.f : exp2f(mi - M);
    lsum += wgt * rec[i * (kD + 2) + 1];
    acc += wgt * rec[i * (kD + 2) + 2 + d];
  }
  const __nv_bfloat16 ob = __float2bfloat16_rn(lsum > 0.f ? acc / lsum : 0.f);
  tab.out[s][static_cast<int64_t>(local) * p.out_stride + h * kD + d] = ob;
  const __nv_bfloat16* A = sh.A[s];
  if (!A) return;
  // shrink share of this head (r <= 32 columns)
  __shared__ float red[4][32];
  const float x = __bfloat162float(ob);
  float t[32];
  const __nv_bfloat16* ar = A + (static_cast<int64_t>(h) * kD + d) * sh.r;
  for (int j = 0; j < sh.r; j += 8) {
    float v[8];
    load8(ar + j, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) t[j + e] = x * v[e];
  }
  const int w = d >> 5, lane = d & 31;
  for (int j = 0; j < sh.r; ++j) {
    float v = t[j];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) red[w][j] = v;
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

int attention_splits(int total_rows, int hkv, int max_len) {
  // One-warp CTAs: enough context splits for ~8 CTAs per SM with at least 2
  // pages per split, and few enough pages per split for the page-id buffer.
  const int base = std::max(1, total_rows * hkv);
  const int pages = (max_len + kPageTok - 1) / kPageTok;
  int splits = std::max(1, std::min(8 * 148 / base, pages / 2));
  splits = std::max(splits, (pages + kMaxSplitPages - 1) / kMaxSplitPages);
  return std::min(splits, 64);
}

int64_t attention_part_floats(int total_rows, int hq, int splits) {
  return static_cast<int64_t>(total_rows) * hq * splits * (kD + 2);
}

int launch_paged_attention(const AttnTable& tab, const AttnParams& p, cudaStream_t stream,
                           const ShrinkSide* shrink) {
  if (tab.seg.total_rows <= 0) return SWL_OK;
  if (p.head_dim != kD || p.page != kPageTok || p.hq % p.hkv || p.hq / p.hkv > 8)
    return set_error(SWL_ERR_ARG, "attention: head_dim 128, page 16, at most 8 query heads per kv head");
  if (p.max_len > 64 * kMaxSplitPages * kPageTok) return set_error(SWL_ERR_ARG, "attention: context too long");
  const int splits = attention_splits(tab.seg.total_rows, p.hkv, p.max_len);
  if (!p.part) return set_error(SWL_ERR_ARG, "attention: missing partial scratch");
  dim3 grid(tab.seg.total_rows, p.hkv, splits);
  SWL_CUDA_TRY(launch_kernel(paged_attention_kernel, grid, dim3(32), 0, stream, 1, tab, p, splits, p.part));
  ShrinkSide none;
  if (!shrink) {
    for (int i = 0; i < kMaxSlots; ++i) none.A[i] = nullptr;
    none.r = 0;
    none.ws = nullptr;
  } else if (shrink->r % 8 || shrink->r > 32) {
    return set_error(SWL_ERR_ARG, "attention: shrink rank must be 8..32 in steps of 8");
  }
  SWL_CUDA_TRY(launch_kernel(attention_combine_kernel, dim3(tab.seg.total_rows, p.hq), dim3(kD), 0, stream, 1,
                             tab, p, splits, static_cast<const float*>(p.part), shrink ? *shrink : none));
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

}  // namespace swl
