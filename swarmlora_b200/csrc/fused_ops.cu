// Fused worker-side epilogues of the rounds (one launch between two rounds):
//
//  qkv_rope          after the QKV round: LoRA expand + add (q, k, v),
//                    NeoX RoPE on q and k, k/v appended to the paged cache,
//                    rotated q to the attention scratch.
//  resid_norm_shrink after the O / Down round (and after the embedding):
//                    LoRA expand (scaled after), + residual, RMSNorm of the
//                    row (sum of squares reduced across a cluster of 8 CTAs
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
#include <cuda_bf16.h>

#include "common.h"
#include "ptx.cuh"
#include "worker_ops.h"

namespace swl {

namespace {

constexpr int kCluster = 8;  // CTAs per row in resid_norm_shrink

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

constexpr int kPartialsMax = 1024;  // floats of one row's shrink partials (splits * n)

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

// ---- after the QKV round -------------------------------------------------------------
template <int RANK>
__global__ void __launch_bounds__(256) qkv_rope_kernel(const __grid_constant__ QkvRopeTable tab,
                                                       const QkvRopeParams p) {
  __shared__ float t[3 * 32];
  __shared__ float buf[kPartialsMax];
  const int gr = blockIdx.x;
  ptx::prefetch_l2_share(p.pf, p.pf_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
  const int s = seg_row(tab.seg, gr);
  const int64_t local = gr - tab.seg.row_start[s];
  const __nv_bfloat16* B = tab.B[s];
  const int pi = blockIdx.y * blockDim.x + threadIdx.x;
  const int heads = p.hq + 2 * p.hkv;
  const int half = p.head_dim / 2;
  const bool live = pi < heads * half;
  const int head = live ? pi / half : 0, d = pi % half;
  const int blk = head < p.hq ? 0 : (head < p.hq + p.hkv ? 1 : 2);
  const int64_t n1 = static_cast<int64_t>(head) * p.head_dim + d, n2 = n1 + half;
  // loads that do not depend on the LoRA intermediate go first
  const __nv_bfloat16* base = tab.base[s] + local * p.base_stride;
  float x1 = 0.f, x2 = 0.f;
  uint4 b1[RANK / 8], b2[RANK / 8];
  if (live) {
    x1 = __bfloat162float(base[n1]);
    x2 = __bfloat162float(base[n2]);
    if (B) {
      load_row<RANK>(b1, B + n1 * RANK);
      load_row<RANK>(b2, B + n2 * RANK);
    }
  }
  const int pos = *tab.seqlen[s] + static_cast<int>(local);
  if (B) rebuild_t(t, buf, p.ws_in, p.splits_in, gr, 3 * RANK);
  if (!live) return;
  if (B) {
    x1 = bfr(x1 + bfr(dot_regs<RANK>(t + blk * RANK, b1)));
    x2 = bfr(x2 + bfr(dot_regs<RANK>(t + blk * RANK, b2)));
  }
  if (blk == 2) {
    const int page = tab.block_table[s][pos / p.page];
    const int64_t row = ((static_cast<int64_t>(page) * p.page + pos % p.page) * p.hkv + (head - p.hq - p.hkv)) * p.head_dim;
    tab.v_cache[s][row + d] = __float2bfloat16_rn(x1);
    tab.v_cache[s][row + d + half] = __float2bfloat16_rn(x2);
    return;
  }
  const __nv_bfloat16* cs = p.cos_sin + static_cast<int64_t>(pos) * p.head_dim;
  const float c = __bfloat162float(cs[d]), sn = __bfloat162float(cs[half + d]);
  const float o1 = bfr(bfr(x1 * c) - bfr(x2 * sn));
  const float o2 = bfr(bfr(x2 * c) + bfr(x1 * sn));
  __nv_bfloat16* dst;
  if (blk == 0) {
    dst = p.q_rot + (static_cast<int64_t>(gr) * p.hq + head) * p.head_dim;
  } else {
    const int page = tab.block_table[s][pos / p.page];
    dst = tab.k_cache[s] + ((static_cast<int64_t>(page) * p.page + pos % p.page) * p.hkv + (head - p.hq)) * p.head_dim;
  }
  dst[d] = __float2bfloat16_rn(o1);
  dst[d + half] = __float2bfloat16_rn(o2);
}

// ---- after the O / Down round (and the embedding) ------------------------------------
// Cluster of kCluster CTAs per token row; CTA q owns columns [q*C, (q+1)*C),
// one thread per 4 columns (blockDim = C / 4). The next shrink's A rows of the
// CTA's columns (contiguous, C * R * 2 bytes) stream into shared memory with
// cp.async from the start, overlapping the expand and the norm.
template <int RANK>
__global__ void __launch_bounds__(1024) resid_norm_shrink_kernel(const __grid_constant__ ResidNormTable tab,
                                                                 const ResidNormParams p) {
  extern __shared__ __align__(16) float sm[];  // a_tile | xs[C] | t[32] | red[blockDim * 8]
  __shared__ float buf[kPartialsMax];
  __shared__ float ss_part;
  __shared__ float warp_ss[32];
  constexpr int RB = RANK > 0 ? RANK : 8;
  const int q = static_cast<int>(ptx::cluster_rank());
  const int gr = blockIdx.x / kCluster;
  ptx::prefetch_l2_share(p.pf, p.pf_bytes, blockIdx.x, gridDim.x);
  const int s = seg_row(tab.seg, gr);
  const int64_t local = gr - tab.seg.row_start[s];
  const int64_t C = p.hidden / kCluster;
  const int64_t c0 = q * C;
  const int R = p.r_next;
  const __nv_bfloat16* A = tab.A_next[s];
  __nv_bfloat16* a_tile = reinterpret_cast<__nv_bfloat16*>(sm);
  float* xs = sm + (C * R) / 2;
  float* t = xs + C;
  float* red = t + 32;
  if (A) {
    const uint32_t dst0 = static_cast<uint32_t>(__cvta_generic_to_shared(a_tile));
    const char* src0 = reinterpret_cast<const char*>(A + c0 * R);
    for (int64_t k = threadIdx.x; k < C * R / 8; k += blockDim.x)
      ptx::cp_async_16(dst0 + static_cast<uint32_t>(k * 16), src0 + k * 16, 16);
    ptx::cp_async_commit();
  }
  const __nv_bfloat16* B = tab.B[s];
  const int64_t n = c0 + threadIdx.x * 4;
  const __nv_bfloat16* base = tab.base[s] + local * p.base_stride;
  __nv_bfloat16* h = tab.h[s] + local * p.h_stride;
  const uint2 bu = *reinterpret_cast<const uint2*>(base + n);
  uint2 ru = make_uint2(0u, 0u);
  if (p.has_resid) ru = *reinterpret_cast<const uint2*>(h + n);
  const uint2 wu = *reinterpret_cast<const uint2*>(p.w + n);
  uint4 bq[4][RB / 8];
  if (RANK > 0 && B) {
#pragma unroll
    for (int e = 0; e < 4; ++e) load_row<RB>(bq[e], B + (n + e) * RANK);
  }
  if (RANK > 0 && B) rebuild_t(t, buf, p.ws_in, p.splits_in, gr, RANK);
  float v[4];
  {
    const __nv_bfloat162* bv = reinterpret_cast<const __nv_bfloat162*>(&bu);
    const float2 b01 = __bfloat1622float2(bv[0]), b23 = __bfloat1622float2(bv[1]);
    v[0] = b01.x; v[1] = b01.y; v[2] = b23.x; v[3] = b23.y;
  }
  if (RANK > 0 && B) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float d = bfr(dot_regs<RB>(t, bq[e]));
      if (p.post_scale != 0.f) d = bfr(d * p.post_scale);
      v[e] = bfr(v[e] + d);
    }
  }
  if (p.has_resid) {
    const __nv_bfloat162* rv = reinterpret_cast<const __nv_bfloat162*>(&ru);
    const float2 r01 = __bfloat1622float2(rv[0]), r23 = __bfloat1622float2(rv[1]);
    v[0] = bfr(r01.x + v[0]); v[1] = bfr(r01.y + v[1]);
    v[2] = bfr(r23.x + v[2]); v[3] = bfr(r23.y + v[3]);
  }
  {
    __align__(8) __nv_bfloat162 hv[2] = {__floats2bfloat162_rn(v[0], v[1]), __floats2bfloat162_rn(v[2], v[3])};
    *reinterpret_cast<uint2*>(h + n) = *reinterpret_cast<uint2*>(hv);
  }
  float ss = v[0] * v[0];
  ss = fmaf(v[1], v[1], ss);
  ss = fmaf(v[2], v[2], ss);
  ss = fmaf(v[3], v[3], ss);
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
  float total = 0.f;
  const uint32_t my = static_cast<uint32_t>(__cvta_generic_to_shared(&ss_part));
  for (int r = 0; r < kCluster; ++r) {
    float pv;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv) : "r"(ptx::map_peer(my, r)) : "memory");
    total += pv;
  }
  const float inv = rsqrtf(total / static_cast<float>(p.hidden) + p.eps);
  {
    const __nv_bfloat162* wv = reinterpret_cast<const __nv_bfloat162*>(&wu);
    const float2 w01 = __bfloat1622float2(wv[0]), w23 = __bfloat1622float2(wv[1]);
    const float wf[4] = {w01.x, w01.y, w23.x, w23.y};
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      x[e] = bfr(wf[e] * bfr(v[e] * inv));
      xs[threadIdx.x * 4 + e] = x[e];
    }
    __align__(8) __nv_bfloat162 xv[2] = {__floats2bfloat162_rn(x[0], x[1]), __floats2bfloat162_rn(x[2], x[3])};
    *reinterpret_cast<uint2*>(tab.x_out[s] + local * p.x_stride + n) = *reinterpret_cast<uint2*>(xv);
  }
  if (A) {
    ptx::cp_async_wait_all();
    __syncthreads();
    // next round's LoRA shrink over this CTA's columns: ws_next[gr][q][j]
    const int G = R / 8;
    const int kgroups = blockDim.x / G;
    const int tid = threadIdx.x;
    const bool active = tid < kgroups * G;
    const int cg = tid % G, kg = tid / G;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (active) {
#pragma unroll 4
      for (int64_t k = kg; k < C; k += kgroups) {
        float a[8];
        ld8(a_tile + k * R + cg * 8, a);
        const float xv = xs[k];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(xv, a[e], acc[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) red[tid * 8 + e] = acc[e];
    __syncthreads();
    for (int j = tid; j < R; j += blockDim.x) {
      float sum = 0.f;
      for (int g = 0; g < kgroups; ++g) sum += red[(g * G + j / 8) * 8 + (j & 7)];
      p.ws_next[(static_cast<int64_t>(gr) * kCluster + q) * R + j] = sum;
    }
  }
  ptx::cluster_sync();  // peers may still read ss_part
}

// ---- after the Gate+Up round ----------------------------------------------------------
// One thread per 4 consecutive columns of the SiLU product; CTA = (row, 512
// columns). The Down shrink partial of the CTA's columns goes to
// ws_next[row][blockIdx.y][j].
template <int RANK>
__global__ void __launch_bounds__(128) gu_silu_shrink_kernel(const __grid_constant__ GuSiluTable tab,
                                                             const GuSiluParams p) {
  __shared__ float t[2 * 32];
  __shared__ float buf[kPartialsMax];
  __shared__ float red[4][32];
  const int gr = blockIdx.x;
  ptx::prefetch_l2_share(p.pf, p.pf_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
  const int s = seg_row(tab.seg, gr);
  const int64_t local = gr - tab.seg.row_start[s];
  const __nv_bfloat16* B = tab.B[s];
  const __nv_bfloat16* A = tab.A_next[s];
  const int R = p.r_next;
  const int64_t n0 = (static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x) * 4;
  const bool live = n0 < p.inter;
  // loads that do not depend on the LoRA intermediate go first
  uint2 gu = make_uint2(0u, 0u), uu = make_uint2(0u, 0u);
  uint4 bg[4][RANK / 8], bu[4][RANK / 8], an[4][4];
  if (live) {
    const __nv_bfloat16* base = tab.base[s] + local * p.base_stride;
    gu = *reinterpret_cast<const uint2*>(base + n0);
    uu = *reinterpret_cast<const uint2*>(base + n0 + p.inter);
    if (B) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        load_row<RANK>(bg[e], B + (n0 + e) * RANK);
        load_row<RANK>(bu[e], B + (n0 + e + p.inter) * RANK);
      }
    }
    if (A) {
#pragma unroll
      for (int e = 0; e < 4; ++e)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (j * 8 < R) an[e][j] = reinterpret_cast<const uint4*>(A + (n0 + e) * R)[j];
    }
  }
  if (B) rebuild_t(t, buf, p.ws_in, p.splits_in, gr, 2 * RANK);
  float a[4] = {0.f, 0.f, 0.f, 0.f};
  if (live) {
    const __nv_bfloat162* gv = reinterpret_cast<const __nv_bfloat162*>(&gu);
    const __nv_bfloat162* uv = reinterpret_cast<const __nv_bfloat162*>(&uu);
    float g[4], u[4];
    const float2 g01 = __bfloat1622float2(gv[0]), g23 = __bfloat1622float2(gv[1]);
    const float2 u01 = __bfloat1622float2(uv[0]), u23 = __bfloat1622float2(uv[1]);
    g[0] = g01.x; g[1] = g01.y; g[2] = g23.x; g[3] = g23.y;
    u[0] = u01.x; u[1] = u01.y; u[2] = u23.x; u[3] = u23.y;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (B) {
        g[e] = bfr(g[e] + bfr(dot_regs<RANK>(t, bg[e])));
        u[e] = bfr(u[e] + bfr(dot_regs<RANK>(t + RANK, bu[e])));
      }
      const float sg = bfr(g[e] / (1.f + expf(-g[e])));
      a[e] = bfr(sg * u[e]);
    }
    __align__(8) __nv_bfloat162 av[2] = {__floats2bfloat162_rn(a[0], a[1]), __floats2bfloat162_rn(a[2], a[3])};
    *reinterpret_cast<uint2*>(tab.act[s] + local * p.act_stride + n0) = *reinterpret_cast<uint2*>(av);
  }
  if (!A) return;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j0 = 0; j0 < 32; j0 += 8) {
    if (j0 >= R) break;
    float part[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&an[e][j0 / 8]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(hv[q]);
          part[2 * q] = fmaf(a[e], f.x, part[2 * q]);
          part[2 * q + 1] = fmaf(a[e], f.y, part[2 * q + 1]);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float v = part[q];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[w][j0 + q] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < R) {
    float v = 0.f;
    for (int ww = 0; ww < static_cast<int>(blockDim.x >> 5); ++ww) v += red[ww][threadIdx.x];
    p.ws_next[(static_cast<int64_t>(gr) * gridDim.y + blockIdx.y) * R + threadIdx.x] = v;
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
    case 8: qkv_rope_kernel<8><<<grid, 256, 0, stream>>>(tab, p); break;
    case 16: qkv_rope_kernel<16><<<grid, 256, 0, stream>>>(tab, p); break;
    case 32: qkv_rope_kernel<32><<<grid, 256, 0, stream>>>(tab, p); break;
    default: return set_error(SWL_ERR_ARG, "qkv_rope: rank must be 8, 16 or 32");
  }
  SWL_CUDA_TRY(cudaGetLastError());
  return SWL_OK;
}

int launch_resid_norm_shrink(const ResidNormTable& tab, const ResidNormParams& p, int r_in,
                             cudaStream_t stream) {
  if (tab.seg.total_rows <= 0) return SWL_OK;
  if (p.hidden % (kCluster * 4)) return set_error(SWL_ERR_ARG, "resid_norm: hidden must be a multiple of 32");
  if (p.r_next % 8 || p.r_next > 96) return set_error(SWL_ERR_ARG, "resid_norm: next rank layout must be 8..96 in steps of 8");
  if (p.splits_in * r_in > kPartialsMax) return set_error(SWL_ERR_ARG, "resid_norm: too many shrink partials");
  const int64_t C = p.hidden / kCluster;
  const int threads = static_cast<int>(C / 4);
  if (threads > 1024 || threads % 32) return set_error(SWL_ERR_ARG, "resid_norm: hidden must be a multiple of 1024 and <= 32768");
  const size_t smem = C * p.r_next * 2 + (C + 32 + static_cast<size_t>(threads) * 8) * sizeof(float);
  if (smem > 200 * 1024) return set_error(SWL_ERR_ARG, "resid_norm: shared memory too large");
  cudaError_t ae = cudaSuccess;
  switch (r_in) {
    case 0: ae = cudaFuncSetAttribute(resid_norm_shrink_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); break;
    case 8: ae = cudaFuncSetAttribute(resid_norm_shrink_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); break;
    case 16: ae = cudaFuncSetAttribute(resid_norm_shrink_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); break;
    case 32: ae = cudaFuncSetAttribute(resid_norm_shrink_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); break;
    default: break;
  }
  if (ae != cudaSuccess) return set_error(SWL_ERR_CUDA, "resid_norm: %s", cudaGetErrorString(ae));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(tab.seg.total_rows * kCluster), 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  switch (r_in) {
    case 0: SWL_CUDA_TRY(cudaLaunchKernelEx(&cfg, resid_norm_shrink_kernel<0>, tab, p)); break;
    case 8: SWL_CUDA_TRY(cudaLaunchKernelEx(&cfg, resid_norm_shrink_kernel<8>, tab, p)); break;
    case 16: SWL_CUDA_TRY(cudaLaunchKernelEx(&cfg, resid_norm_shrink_kernel<16>, tab, p)); break;
    case 32: SWL_CUDA_TRY(cudaLaunchKernelEx(&cfg, resid_norm_shrink_kernel<32>, tab, p)); break;
    default: return set_error(SWL_ERR_ARG, "resid_norm: input rank must be 0, 8, 16 or 32");
  }
  return SWL_OK;
}

int launch_gu_silu_shrink(const GuSiluTable& tab, const GuSiluParams& p, int r, cudaStream_t stream) {
  if (tab.seg.total_rows <= 0) return SWL_OK;
  if (p.r_next % 8 || p.r_next > 32) return set_error(SWL_ERR_ARG, "gu_silu: next rank must be 8..32 in steps of 8");
  if (p.inter % 4) return set_error(SWL_ERR_ARG, "gu_silu: inter must be a multiple of 4");
  if (p.splits_in * 2 * r > kPartialsMax) return set_error(SWL_ERR_ARG, "gu_silu: too many shrink partials");
  dim3 grid(tab.seg.total_rows, static_cast<unsigned>((p.inter + 511) / 512));
  switch (r) {
    case 8: gu_silu_shrink_kernel<8><<<grid, 128, 0, stream>>>(tab, p); break;
    case 16: gu_silu_shrink_kernel<16><<<grid, 128, 0, stream>>>(tab, p); break;
    case 32: gu_silu_shrink_kernel<32><<<grid, 128, 0, stream>>>(tab, p); break;
    default: return set_error(SWL_ERR_ARG, "gu_silu: rank must be 8, 16 or 32");
  }
  SWL_CUDA_TRY(cudaGetLastError());
  return SWL_OK;
}

int resid_norm_splits() { return kCluster; }
int gu_silu_splits(int64_t inter) { return static_cast<int>((inter + 511) / 512); }

}  // namespace swl
