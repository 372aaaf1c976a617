// Fused worker-side epilogues of the rounds (one launch between two rounds):
//
//  qkv_rope          after the QKV round: LoRA expand + add (q, k, v),
//                    NeoX RoPE on q and k, k/v appended to the paged cache,
//                    rotated q to the attention scratch.
//  resid_norm_shrink after the O / Down round (and after the embedding):
//                    LoRA expand (scaled after), + residual, RMSNorm of the
//                    row (sum of squares reduced across a cluster of 4 CTAs
//                    through distributed shared memory), normed row written
//                    into the next round's slot input, and the next round's
//                    LoRA shrink partials computed from it.
//  gu_silu_shrink    after the Gate+Up round: LoRA expand + add on gate and
//                    up, SiLU(gate) * up written into the Down round's slot
//                    input, and the Down projection's LoRA shrink partials.
//
// The arithmetic (bf16 rounding points) is the same as the separate kernels
// in worker_ops.cu and the reference's tensor ops (worker_sync.py:250-389,
// model_builder.py:258-262, HF LlamaRMSNorm, vLLM rotary_embedding).
#include <mutex>
#include <cuda_bf16.h>

#include "common.h"
#include "launch.h"
#include "ptx.cuh"
#include "worker_ops.h"

namespace swl {

namespace {

// resid_norm_shrink: a cluster of CL CTAs per row (hidden 4096), CTA q owns
// 4096 / CL columns, 2048 / CL threads with 2 columns each. CL = 4 when the
// staged adapter tiles fit (input rank <= 16, next shrink width <= 48),
// else 8; the next round's shrink gets one partial per CTA.
constexpr int kNormHidden = 4096;
__host__ __device__ constexpr int norm_threads(int cl) { return 2048 / cl; }
int norm_cluster(int r_in, int r_next) { return (r_in <= 16 && r_next <= 48) ? 4 : 8; }

__device__ __forceinline__ float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ int seg_row(const RowSegments& s, int gr) {
  int lo = 0, hi = s.nseg - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (s.row_start[mid] <= gr) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

constexpr int kPartialsMax = 2048;  // floats of one row's shrink partials (splits * n)

// Rebuilds the bf16-rounded LoRA intermediate t[0..n) of row gr from `splits`
// fp32 partials laid out ws[row][split][n]: the CTA stages the row's
// splits * n contiguous floats in shared memory, then n threads add them in
// split order. Ends with a barrier.
__device__ __forceinline__ void rebuild_t(float* t, float* buf, const float* ws, int splits,
                                          int gr, int n) {
  const float* src = ws + static_cast<int64_t>(gr) * splits * n;
  for (int e = threadIdx.x; e < splits * n; e += blockDim.x) buf[e] = src[e];
  __syncthreads();
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += buf[sp * n + j];
    t[j] = bfr(s);
  }
  __syncthreads();
}

template <int RANK>
__device__ __forceinline__ float lora_dot(const float* t, const __nv_bfloat16* brow) {
  float d = 0.f;
#pragma unroll
  for (int j = 0; j < RANK; j += 8) {
    float v[8];
    ld8(brow + j, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) d = fmaf(t[j + e], v[e], d);
  }
  return d;
}

// Dot product of the rebuilt t (RANK floats) with a lora_B row held in
// registers as RANK/8 16-byte vectors.
template <int RANK>
__device__ __forceinline__ float dot_regs(const float* t, const uint4 (&b)[RANK / 8]) {
  float d = 0.f;
#pragma unroll
  for (int j = 0; j < RANK / 8; ++j) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&b[j]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      d = fmaf(t[8 * j + 2 * e], f.x, d);
      d = fmaf(t[8 * j + 2 * e + 1], f.y, d);
    }
  }
  return d;
}

template <int RANK>
__device__ __forceinline__ void load_row(uint4 (&b)[RANK / 8], const __nv_bfloat16* row) {
#pragma unroll
  for (int j = 0; j < RANK / 8; ++j) b[j] = reinterpret_cast<const uint4*>(row)[j];
}

// Issues one bulk copy per non-null (dst, src, bytes) triple on a fresh
// mbarrier (thread 0), so the CTA's big contiguous operand reads run on the
// TMA engine instead of the load/store unit. Returns whether anything was issued.
__device__ __forceinline__ bool stage_bulk(uint64_t* bar, void* d0, const void* s0, uint32_t b0,
                                           void* d1, const void* s1, uint32_t b1, void* d2,
                                           const void* s2, uint32_t b2) {
  const uint32_t total = (s0 ? b0 : 0u) + (s1 ? b1 : 0u) + (s2 ? b2 : 0u);
  if (total == 0) return false;
  if (threadIdx.x == 0) {
    ptx::mbar_init(bar, 1);
    ptx::fence_mbar_init();
    ptx::mbar_arrive_expect_tx(bar, total);
    if (s0) ptx::bulk_load(d0, s0, b0, bar);
    if (s1) ptx::bulk_load(d1, s1, b1, bar);
    if (s2) ptx::bulk_load(d2, s2, b2, bar);
  }
  return true;
}

__device__ __forceinline__ float smem_dot(const float* t, const __nv_bfloat16* row, int rank) {
  float d = 0.f;
  for (int j = 0; j < rank; j += 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + j);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      d = fmaf(t[j + 2 * e], f.x, d);
      d = fmaf(t[j + 2 * e + 1], f.y, d);
    }
  }
  return d;
}

// ---- after the QKV round -------------------------------------------------------------
// CTA = (row, 4 heads = 512 columns); thread = (head, d < 64) pair of columns.
template <int RANK>
__global__ void __launch_bounds__(256) qkv_rope_kernel(const __grid_constant__ QkvRopeTable tab,
                                                       const QkvRopeParams p) {
  __shared__ __align__(128) __nv_bfloat16 bs[512 * RANK];
  __shared__ float t[3 * 32];
  __shared__ float buf[kPartialsMax];
  __shared__ __align__(8) uint64_t bar;
  const int gr = blockIdx.x;
  ptx::prefetch_l2_share(p.pf, p.pf_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
  const int s = seg_row(tab.seg, gr);
  const int64_t local = gr - tab.seg.row_start[s];
  const __nv_bfloat16* B = tab.B[s];
  const int half = p.head_dim / 2;
  const int heads = p.hq + 2 * p.hkv;
  const int64_t col0 = static_cast<int64_t>(blockIdx.y) * 4 * p.head_dim;
  const int64_t ncols = min(static_cast<int64_t>(4 * p.head_dim), static_cast<int64_t>(heads) * p.head_dim - col0);
  const bool staged = B && stage_bulk(&bar, bs, B + col0 * RANK, static_cast<uint32_t>(ncols * RANK * 2),
                                      nullptr, nullptr, 0, nullptr, nullptr, 0);
  const int pi = blockIdx.y * blockDim.x + threadIdx.x;
  const bool live = pi < heads * half;
  const int head = live ? pi / half : 0, d = pi % half;
  const int blk = head < p.hq ? 0 : (head < p.hq + p.hkv ? 1 : 2);
  const int64_t n1 = static_cast<int64_t>(head) * p.head_dim + d, n2 = n1 + half;
  // The token's position, its cos/sin and its cache page come from tables the
  // QKV round ahead of this launch does not write: read before waiting for it.
  const int pos = *tab.seqlen[s] + static_cast<int>(local);
  float c = 0.f, sn = 0.f;
  int page = 0;
  if (live) {
    if (blk != 2) {
      const __nv_bfloat16* cs = p.cos_sin + static_cast<int64_t>(pos) * p.head_dim;
      c = __bfloat162float(cs[d]);
      sn = __bfloat162float(cs[half + d]);
    }
    if (blk != 0) page = tab.block_table[s][pos / p.page];
  }
  // the LoRA intermediate of the QKV input: shrink partials written two
  // launches back, by the epilogue ahead of the QKV round
  if (B) rebuild_t(t, buf, p.ws_in, p.splits_in, gr, 3 * RANK);
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const __nv_bfloat16* base = tab.base[s] + local * p.base_stride;
  float x1 = 0.f, x2 = 0.f;
  if (live) {
    x1 = __bfloat162float(base[n1]);
    x2 = __bfloat162float(base[n2]);
  }
  if (staged) ptx::mbar_wait(&bar, 0, nullptr, 0, 2000000000ull);
  if (!live) return;
  if (B) {
    x1 = bfr(x1 + bfr(smem_dot(t + blk * RANK, bs + (n1 - col0) * RANK, RANK)));
    x2 = bfr(x2 + bfr(smem_dot(t + blk * RANK, bs + (n2 - col0) * RANK, RANK)));
  }
  if (blk == 2) {
    const int64_t row = ((static_cast<int64_t>(page) * p.page + pos % p.page) * p.hkv + (head - p.hq - p.hkv)) * p.head_dim;
    tab.v_cache[s][row + d] = __float2bfloat16_rn(x1);
    tab.v_cache[s][row + d + half] = __float2bfloat16_rn(x2);
    return;
  }
  const float o1 = bfr(bfr(x1 * c) - bfr(x2 * sn));
  const float o2 = bfr(bfr(x2 * c) + bfr(x1 * sn));
  __nv_bfloat16* dst;
  if (blk == 0) {
    dst = p.q_rot + (static_cast<int64_t>(gr) * p.hq + head) * p.head_dim;
  } else {
    dst = tab.k_cache[s] + ((static_cast<int64_t>(page) * p.page + pos % p.page) * p.hkv + (head - p.hq)) * p.head_dim;
  }
  dst[d] = __float2bfloat16_rn(o1);
  dst[d + half] = __float2bfloat16_rn(o2);
}

// ---- after the O / Down round (and the embedding) ------------------------------------
// Cluster of kCluster CTAs per token row; CTA q owns columns [q*C, (q+1)*C),
// thread t the columns c0 + t + k*blockDim (k < C / blockDim). The finished
// round's lora_B rows and the next shrink's A rows of those columns are
// staged in shared memory by two bulk copies.
template <int RANK, int CL>
__global__ void __launch_bounds__(norm_threads(CL)) resid_norm_shrink_kernel(const __grid_constant__ ResidNormTable tab,
                                                                const ResidNormParams p) {
  extern __shared__ __align__(128) uint8_t dsm[];  // a_tile [C][R] | b_tile [C][RANK] | red [warps][R]
  __shared__ float t[32];
  __shared__ float buf[kPartialsMax];
  __shared__ float ss_part;
  constexpr int kNormThreads = norm_threads(CL);
  constexpr int kCluster = CL;
  __shared__ float warp_ss[kNormThreads / 32];
  __shared__ __align__(8) uint64_t bar;
  constexpr int RB = RANK > 0 ? RANK : 8;
  constexpr int kCols = kNormHidden / CL / kNormThreads;  // columns per thread (C = kCols * blockDim)
  const int q = static_cast<int>(ptx::cluster_rank());
  const int gr = blockIdx.x / kCluster;
  ptx::prefetch_l2_share(p.pf, p.pf_bytes, blockIdx.x, gridDim.x);
  const int s = seg_row(tab.seg, gr);
  const int64_t local = gr - tab.seg.row_start[s];
  const int64_t C = p.hidden / kCluster;
  const int64_t c0 = q * C;
  const int R = p.r_next;
  const __nv_bfloat16* A = tab.A_next[s];
  const __nv_bfloat16* B = RANK > 0 ? tab.B[s] : nullptr;
  __nv_bfloat16* a_tile = reinterpret_cast<__nv_bfloat16*>(dsm);
  __nv_bfloat16* b_tile = a_tile + C * R;
  float* red = reinterpret_cast<float*>(b_tile + C * RB);  // [warp][R] shrink sums
  const bool staged = stage_bulk(&bar, a_tile, A ? A + c0 * R : nullptr, static_cast<uint32_t>(C * R * 2),
                                 b_tile, B ? B + c0 * RANK : nullptr, static_cast<uint32_t>(C * RB * 2),
                                 nullptr, nullptr, 0);
  // The residual, the norm weight and the finished round's shrink partials
  // are written two or more launches back: read them before waiting for the
  // round just ahead, whose output (base) is read after.
  __nv_bfloat16* h = tab.h[s] + local * p.h_stride;
  float v[kCols], rv[kCols], wv[kCols];
#pragma unroll
  for (int k = 0; k < kCols; ++k) {
    const int64_t n = c0 + threadIdx.x + k * blockDim.x;
    rv[k] = p.has_resid ? __bfloat162float(h[n]) : 0.f;
    wv[k] = __bfloat162float(p.w[n]);
  }
  if (B) rebuild_t(t, buf, p.ws_in, p.splits_in, gr, RANK);
  else __syncthreads();  // barrier init visible before anyone waits on it
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const __nv_bfloat16* base = tab.base[s] + local * p.base_stride;
#pragma unroll
  for (int k = 0; k < kCols; ++k) v[k] = __bfloat162float(base[c0 + threadIdx.x + k * blockDim.x]);
  if (staged) ptx::mbar_wait(&bar, 0, nullptr, 0, 2000000000ull);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kCols; ++k) {
    const int64_t c = threadIdx.x + k * blockDim.x;
    if (B) {
      float d = bfr(smem_dot(t, b_tile + c * RANK, RANK));
      if (p.post_scale != 0.f) d = bfr(d * p.post_scale);
      v[k] = bfr(v[k] + d);
    }
    if (p.has_resid) v[k] = bfr(rv[k] + v[k]);
    h[c0 + c] = __float2bfloat16_rn(v[k]);
    ss = fmaf(v[k], v[k], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) warp_ss[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) a += warp_ss[w];
    ss_part = a;
  }
  ptx::cluster_sync();
  // every CTA's part is loaded first (one round trip), then summed in order
  const uint32_t my = static_cast<uint32_t>(__cvta_generic_to_shared(&ss_part));
  float pv[kCluster];
#pragma unroll
  for (int r = 0; r < kCluster; ++r)
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv[r]) : "r"(ptx::map_peer(my, r)) : "memory");
  float total = 0.f;
#pragma unroll
  for (int r = 0; r < kCluster; ++r) total += pv[r];
  ptx::cluster_arrive();  // done with the peers' ss_part; waited for before exit
  const float inv = rsqrtf(total / static_cast<float>(p.hidden) + p.eps);
  __nv_bfloat16* xo = tab.x_out[s] + local * p.x_stride;
  float xv[kCols];
#pragma unroll
  for (int k = 0; k < kCols; ++k) {
    const int64_t c = threadIdx.x + k * blockDim.x;
    xv[k] = bfr(wv[k] * bfr(v[k] * inv));
    xo[c0 + c] = __float2bfloat16_rn(xv[k]);
  }
  if (A) {
    // next round's LoRA shrink over this CTA's columns, ws_next[gr][q][j]:
    // each thread multiplies its columns into their A rows, eight partial
    // columns at a time; a halving exchange over the warp leaves column
    // 4*b4 + 2*b3 + b2 (bits of the lane) summed over 8 lanes, two more
    // steps sum the rest; the warps' sums meet in red
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int jv = 0; jv < R / 8; ++jv) {
      float a8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < kCols; ++k) {
        const int64_t c = threadIdx.x + k * blockDim.x;
        const uint4 w4 = *reinterpret_cast<const uint4*>(a_tile + c * R + jv * 8);
        const uint32_t wq[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          a8[2 * e] = fmaf(xv[k], __uint_as_float(wq[e] << 16), a8[2 * e]);
          a8[2 * e + 1] = fmaf(xv[k], __uint_as_float(wq[e] & 0xffff0000u), a8[2 * e + 1]);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool up = lane & 16;
        const float send = up ? a8[e] : a8[e + 4], kept = up ? a8[e + 4] : a8[e];
        a8[e] = kept + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool up = lane & 8;
        const float send = up ? a8[e] : a8[e + 2], kept = up ? a8[e + 2] : a8[e];
        a8[e] = kept + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      {
        const bool up = lane & 4;
        const float send = up ? a8[0] : a8[1], kept = up ? a8[1] : a8[0];
        a8[0] = kept + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      a8[0] += __shfl_xor_sync(0xffffffffu, a8[0], 2);
      a8[0] += __shfl_xor_sync(0xffffffffu, a8[0], 1);
      if ((lane & 3) == 0)
        red[warp * R + jv * 8 + ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1)] = a8[0];
    }
    __syncthreads();
    if (threadIdx.x < R) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kNormThreads / 32; ++w) sum += red[w * R + threadIdx.x];
      p.ws_next[(static_cast<int64_t>(gr) * kCluster + q) * R + threadIdx.x] = sum;
    }
  }
  ptx::cluster_wait();  // peers may still read ss_part
}

// ---- after the Gate+Up round ----------------------------------------------------------
// Work units = (token row, block of kGuCols SiLU columns), rows in order. A
// CTA of kGuCols threads (thread = column) walks an equal contiguous range of
// units; each unit's operands (gate and up lora_B rows, the Down shrink's A
// rows, the round's gate and up outputs) stream through a ring of kGuStages
// shared-memory stages, five bulk copies per unit issued by one thread, so
// loads of later units overlap the math of the current one. The adapter
// copies of the first stages are issued before the wait for the Gate+Up
// round. Per unit: LoRA expand + add on gate and up, SiLU(gate) * up written
// into the Down round's slot input, and the unit's Down shrink partial to
// ws_next[row][block][j] (each thread multiplies its column into its A row,
// a warp sums its 32 columns by halving exchanges, the 8 warps through
// shared memory).
constexpr int kGuCols = 256;
constexpr int kGuStages = 2;  // with 4 CTAs per SM (the register limit at 64 per thread)
constexpr int kGuPartialsMax = 512;  // floats of one row's Gate/Up shrink partials

template <int RANK>
__global__ void __launch_bounds__(kGuCols) gu_silu_shrink_kernel(const __grid_constant__ GuSiluTable tab,
                                                                 const GuSiluParams p) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ float t[2 * 32], t_next[2 * 32];
  __shared__ float red_sm[kGuCols / 32][32];
  __shared__ float part_sm[kGuPartialsMax];
  const int R = p.r_next;
  // stage: bg [kGuCols][RANK] | bu [kGuCols][RANK] | an [kGuCols][R] | g [kGuCols] | u [kGuCols]
  const int b_bytes = kGuCols * RANK * 2, a_bytes = kGuCols * R * 2, v_bytes = kGuCols * 2;
  const int stage_bytes = 2 * b_bytes + a_bytes + 2 * v_bytes;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nblk = static_cast<int>((p.inter + kGuCols - 1) / kGuCols);
  const int total = tab.seg.total_rows * nblk;
  const int W = (total + gridDim.x - 1) / gridDim.x;
  const int u0 = blockIdx.x * W;
  const int u1 = min(total, u0 + W);
  if (u0 >= u1) {
    ptx::grid_dep_wait();
    ptx::grid_dep_launch();
    return;
  }
  const int nunits = u1 - u0;
  __shared__ __align__(8) uint64_t full[kGuStages];
  if (tid == 0) {
    for (int i = 0; i < kGuStages; ++i) ptx::mbar_init(&full[i], 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();

  // Thread 0 stages unit j on the stage's mbarrier: the adapter rows (gate
  // and up lora_B, the Down shrink's A) with issue_w, the Gate+Up round's
  // outputs with issue_v; the mbarrier expects both.
  auto unit_at = [&](int j, int& gr_, int64_t& n0_, int& nc_, int& s_) {
    const int u = u0 + j;
    gr_ = u / nblk;
    n0_ = static_cast<int64_t>(u - gr_ * nblk) * kGuCols;
    nc_ = static_cast<int>(min(static_cast<int64_t>(kGuCols), p.inter - n0_));
    s_ = seg_row(tab.seg, gr_);
  };
  auto issue_w = [&](int j) {
    int gr_, nc_, s_;
    int64_t n0_;
    unit_at(j, gr_, n0_, nc_, s_);
    uint8_t* ss = dsm + (j % kGuStages) * stage_bytes;
    uint64_t* bar = &full[j % kGuStages];
    const __nv_bfloat16* B = tab.B[s_];
    const __nv_bfloat16* A = tab.A_next[s_];
    const uint32_t bb = static_cast<uint32_t>(nc_) * RANK * 2, ab = static_cast<uint32_t>(nc_) * R * 2,
                   vb = static_cast<uint32_t>(nc_) * 2;
    ptx::mbar_arrive_expect_tx(bar, (B ? 2 * bb : 0u) + (A ? ab : 0u) + 2 * vb);
    if (B) {
      ptx::bulk_load(ss, B + n0_ * RANK, bb, bar);
      ptx::bulk_load(ss + b_bytes, B + (n0_ + p.inter) * RANK, bb, bar);
    }
    if (A) ptx::bulk_load(ss + 2 * b_bytes, A + n0_ * R, ab, bar);
  };
  auto issue_v = [&](int j) {
    int gr_, nc_, s_;
    int64_t n0_;
    unit_at(j, gr_, n0_, nc_, s_);
    uint8_t* ss = dsm + (j % kGuStages) * stage_bytes;
    uint64_t* bar = &full[j % kGuStages];
    const uint32_t vb = static_cast<uint32_t>(nc_) * 2;
    const __nv_bfloat16* base = tab.base[s_] + (gr_ - tab.seg.row_start[s_]) * p.base_stride + n0_;
    ptx::bulk_load(ss + 2 * b_bytes + a_bytes, base, vb, bar);
    ptx::bulk_load(ss + 2 * b_bytes + a_bytes + v_bytes, base + p.inter, vb, bar);
  };
  // A row's gate and up LoRA intermediates, bf16-rounded, from the shrink
  // partials ws_in[row][split][2 RANK] (written two launches back, by the
  // epilogue ahead of the Gate+Up round): all threads fetch the partials at
  // once, then 2 RANK threads add them in split order into dst. Ends with a
  // barrier. The range's first two rows are done before the wait.
  float tg[RANK], tu[RANK];
  auto sum_t = [&](int row, float* dst) {
    const float* src = p.ws_in + static_cast<int64_t>(row) * p.splits_in * 2 * RANK;
    for (int e = tid; e < p.splits_in * 2 * RANK; e += kGuCols) part_sm[e] = src[e];
    __syncthreads();
    if (tid < 2 * RANK) {
      float a = 0.f;
      for (int sp = 0; sp < p.splits_in; ++sp) a += part_sm[sp * 2 * RANK + tid];
      dst[tid] = bfr(a);
    }
    __syncthreads();
  };
  auto use_t = [&](const float* src) {
#pragma unroll
    for (int e = 0; e < RANK; ++e) {
      tg[e] = src[e];
      tu[e] = src[RANK + e];
    }
  };
  const int npre = min(kGuStages - 1, nunits);
  if (tid == 0)
    for (int i = 0; i < npre; ++i) issue_w(i);
  int gr = u0 / nblk, blk = u0 - gr * nblk;
  int s = seg_row(tab.seg, gr);
  const int r0 = gr;
  const bool next_pre = (u1 - 1) / nblk > r0 && tab.B[seg_row(tab.seg, r0 + 1)] != nullptr;
  if (tab.B[s]) {
    sum_t(r0, t);
    use_t(t);
  }
  if (next_pre) sum_t(r0 + 1, t_next);
  int cur_row = gr;
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  if (tid == 0)
    for (int i = 0; i < npre; ++i) issue_v(i);

  for (int j = 0; j < nunits; ++j) {
    __syncthreads();  // every thread is done with unit j-1: its stage may be refilled
    if (tid == 0 && j + kGuStages - 1 < nunits) {
      issue_w(j + kGuStages - 1);
      issue_v(j + kGuStages - 1);
    }
    ptx::mbar_wait(&full[j % kGuStages], (j / kGuStages) & 1, nullptr, 0, 2000000000ull);
    const int64_t local = gr - tab.seg.row_start[s];
    const int64_t n0 = static_cast<int64_t>(blk) * kGuCols;
    const int nc = static_cast<int>(min(static_cast<int64_t>(kGuCols), p.inter - n0));
    const __nv_bfloat16* B = tab.B[s];
    const __nv_bfloat16* A = tab.A_next[s];
    if (B && gr != cur_row) {
      if (gr == r0 + 1 && next_pre) {
        use_t(t_next);
      } else {
        sum_t(gr, t);
        use_t(t);
      }
    }
    cur_row = gr;
    const uint8_t* st = dsm + (j % kGuStages) * stage_bytes;
    const __nv_bfloat16* sg = reinterpret_cast<const __nv_bfloat16*>(st + 2 * b_bytes + a_bytes);
    const __nv_bfloat16* su = reinterpret_cast<const __nv_bfloat16*>(st + 2 * b_bytes + a_bytes + v_bytes);
    float a = 0.f;
    if (tid < nc) {
      float g = __bfloat162float(sg[tid]), uu = __bfloat162float(su[tid]);
      if (B) {
        const uint4* bgr = reinterpret_cast<const uint4*>(st + tid * RANK * 2);
        const uint4* bur = reinterpret_cast<const uint4*>(st + b_bytes + tid * RANK * 2);
        float dg = 0.f, du = 0.f;
#pragma unroll
        for (int q = 0; q < RANK / 8; ++q) {
          const uint4 x = bgr[q], y = bur[q];
          const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&x);
          const __nv_bfloat162* hy = reinterpret_cast<const __nv_bfloat162*>(&y);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 fx = __bfloat1622float2(hx[e]), fy = __bfloat1622float2(hy[e]);
            dg = fmaf(tg[8 * q + 2 * e], fx.x, dg);
            dg = fmaf(tg[8 * q + 2 * e + 1], fx.y, dg);
            du = fmaf(tu[8 * q + 2 * e], fy.x, du);
            du = fmaf(tu[8 * q + 2 * e + 1], fy.y, du);
          }
        }
        g = bfr(g + bfr(dg));
        uu = bfr(uu + bfr(du));
      }
      const float sgm = bfr(g / (1.f + expf(-g)));
      a = bfr(sgm * uu);
      tab.act[s][local * p.act_stride + n0 + tid] = __float2bfloat16_rn(a);
    }
    if (A) {
      // Down shrink partial of this block: column tid times its A row, eight
      // partial columns at a time; a halving exchange over the warp leaves
      // column 4*b4 + 2*b3 + b2 (bits of the lane) summed over 8 lanes, two
      // more steps sum the rest; then the warps' sums meet in red_sm
      const __nv_bfloat16* an = reinterpret_cast<const __nv_bfloat16*>(st + 2 * b_bytes);
      for (int jv = 0; jv < R / 8; ++jv) {
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (tid < nc) {
          const uint4 a4 = *reinterpret_cast<const uint4*>(an + tid * R + jv * 8);
          const uint32_t w4[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            v[2 * q] = a * __uint_as_float(w4[q] << 16);
            v[2 * q + 1] = a * __uint_as_float(w4[q] & 0xffff0000u);
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const bool up = lane & 16;
          const float send = up ? v[e] : v[e + 4], kept = up ? v[e + 4] : v[e];
          v[e] = kept + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool up = lane & 8;
          const float send = up ? v[e] : v[e + 2], kept = up ? v[e + 2] : v[e];
          v[e] = kept + __shfl_xor_sync(0xffffffffu, send, 8);
        }
        {
          const bool up = lane & 4;
          const float send = up ? v[0] : v[1], kept = up ? v[1] : v[0];
          v[0] = kept + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
        if ((lane & 3) == 0)
          red_sm[warp][jv * 8 + ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1)] = v[0];
      }
      __syncthreads();
      if (tid < R) {
        float x = 0.f;
#pragma unroll
        for (int w = 0; w < kGuCols / 32; ++w) x += red_sm[w][tid];
        p.ws_next[(static_cast<int64_t>(gr) * nblk + blk) * R + tid] = x;
      }
    }
    if (++blk == nblk) {
      blk = 0;
      if (++gr < tab.seg.total_rows) s = seg_row(tab.seg, gr);
    }
  }
}

}  // namespace

int launch_qkv_rope(const QkvRopeTable& tab, const QkvRopeParams& p, int r, cudaStream_t stream) {
  if (tab.seg.total_rows <= 0) return SWL_OK;
  if (p.head_dim % 2 || p.head_dim > 256) return set_error(SWL_ERR_ARG, "qkv_rope: bad head_dim");
  if (p.splits_in * 3 * r > kPartialsMax) return set_error(SWL_ERR_ARG, "qkv_rope: too many shrink partials");
  const int pairs = (p.hq + 2 * p.hkv) * (p.head_dim / 2);
  dim3 grid(tab.seg.total_rows, (pairs + 255) / 256);
  switch (r) {
    case 8: SWL_CUDA_TRY(launch_kernel(qkv_rope_kernel<8>, grid, dim3(256), 0, stream, 1, tab, p)); break;
    case 16: SWL_CUDA_TRY(launch_kernel(qkv_rope_kernel<16>, grid, dim3(256), 0, stream, 1, tab, p)); break;
    case 32: SWL_CUDA_TRY(launch_kernel(qkv_rope_kernel<32>, grid, dim3(256), 0, stream, 1, tab, p)); break;
    default: return set_error(SWL_ERR_ARG, "qkv_rope: rank must be 8, 16 or 32");
  }
  return SWL_OK;
}

namespace {
template <int RANK, int CL>
int launch_resid_norm_cl(const ResidNormTable& tab, const ResidNormParams& p, size_t smem, cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t ae = cudaSuccess;
  std::call_once(once, [] {
    ae = cudaFuncSetAttribute(resid_norm_shrink_kernel<RANK, CL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              200 * 1024);
  });
  if (ae != cudaSuccess) return set_error(SWL_ERR_CUDA, "resid_norm: %s", cudaGetErrorString(ae));
  const dim3 grid(static_cast<unsigned>(tab.seg.total_rows * CL), 1, 1);
  SWL_CUDA_TRY(launch_kernel(resid_norm_shrink_kernel<RANK, CL>, grid, dim3(norm_threads(CL)), smem, stream, CL, tab,
                             p));
  return SWL_OK;
}
template <int CL>
int launch_resid_norm_rank(const ResidNormTable& tab, const ResidNormParams& p, int r_in, size_t smem,
                           cudaStream_t stream) {
  switch (r_in) {
    case 0: return launch_resid_norm_cl<0, CL>(tab, p, smem, stream);
    case 8: return launch_resid_norm_cl<8, CL>(tab, p, smem, stream);
    case 16: return launch_resid_norm_cl<16, CL>(tab, p, smem, stream);
    case 32: return launch_resid_norm_cl<32, CL>(tab, p, smem, stream);
    default: return set_error(SWL_ERR_ARG, "resid_norm: input rank must be 0, 8, 16 or 32");
  }
}
}  // namespace

int launch_resid_norm_shrink(const ResidNormTable& tab, const ResidNormParams& p, int r_in,
                             cudaStream_t stream) {
  if (tab.seg.total_rows <= 0) return SWL_OK;
  if (p.hidden != kNormHidden) return set_error(SWL_ERR_ARG, "resid_norm: hidden must be %d", kNormHidden);
  if (p.r_next % 8 || p.r_next > 96) return set_error(SWL_ERR_ARG, "resid_norm: next rank layout must be 8..96 in steps of 8");
  if (p.splits_in * r_in > kPartialsMax) return set_error(SWL_ERR_ARG, "resid_norm: too many shrink partials");
  const int cl = norm_cluster(r_in, p.r_next);
  const int64_t C = p.hidden / cl;
  const int rb = r_in > 0 ? r_in : 8;
  const size_t smem = C * p.r_next * 2 + C * rb * 2 + static_cast<size_t>(norm_threads(cl) / 32) * p.r_next * sizeof(float);
  if (smem > 200 * 1024) return set_error(SWL_ERR_ARG, "resid_norm: shared memory too large");
  return cl == 4 ? launch_resid_norm_rank<4>(tab, p, r_in, smem, stream)
                 : launch_resid_norm_rank<8>(tab, p, r_in, smem, stream);
}

int launch_gu_silu_shrink(const GuSiluTable& tab, const GuSiluParams& p, int r, cudaStream_t stream) {
  if (tab.seg.total_rows <= 0) return SWL_OK;
  if (p.r_next % 8 || p.r_next > 32) return set_error(SWL_ERR_ARG, "gu_silu: next rank must be 8..32 in steps of 8");
  if (p.inter % 8) return set_error(SWL_ERR_ARG, "gu_silu: inter must be a multiple of 8");
  if (p.splits_in * 2 * r > kGuPartialsMax) return set_error(SWL_ERR_ARG, "gu_silu: too many shrink partials");
  if (r != 8 && r != 16 && r != 32) return set_error(SWL_ERR_ARG, "gu_silu: rank must be 8, 16 or 32");
  const size_t stage = static_cast<size_t>(kGuCols) * (2 * r + p.r_next) * 2 + 2 * kGuCols * 2;
  const size_t smem = kGuStages * stage;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int64_t units = static_cast<int64_t>(tab.seg.total_rows) * ((p.inter + kGuCols - 1) / kGuCols);
  // CTAs one SM holds (227 KB of shared memory, ~4 KB static and reserved per CTA)
  const int per_sm = static_cast<int>(std::max<size_t>(1, std::min<size_t>(4, (227 * 1024) / (smem + 4096))));
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(units, sms * per_sm)));
  cudaError_t ae = cudaSuccess;
  switch (r) {
    case 8:
      ae = cudaFuncSetAttribute(gu_silu_shrink_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (ae == cudaSuccess) ae = launch_kernel(gu_silu_shrink_kernel<8>, dim3(grid), dim3(kGuCols), smem, stream, 1, tab, p);
      break;
    case 16:
      ae = cudaFuncSetAttribute(gu_silu_shrink_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (ae == cudaSuccess) ae = launch_kernel(gu_silu_shrink_kernel<16>, dim3(grid), dim3(kGuCols), smem, stream, 1, tab, p);
      break;
    default:
      ae = cudaFuncSetAttribute(gu_silu_shrink_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (ae == cudaSuccess) ae = launch_kernel(gu_silu_shrink_kernel<32>, dim3(grid), dim3(kGuCols), smem, stream, 1, tab, p);
      break;
  }
  if (ae != cudaSuccess) return set_error(SWL_ERR_CUDA, "gu_silu: %s", cudaGetErrorString(ae));
  return SWL_OK;
}

int resid_norm_splits(int rank) { return norm_cluster(rank, 3 * rank); }
int gu_silu_splits(int64_t inter) { return static_cast<int>((inter + kGuCols - 1) / kGuCols); }

}  // namespace swl
