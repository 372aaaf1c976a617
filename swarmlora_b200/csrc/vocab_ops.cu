// Vocabulary-side round kernels: the embedding gather of OP_EMBED and the
// greedy next-token pick of OP_LM_HEAD (the LM-head GEMM itself is a slot
// round, see slot_round.cu).
//
// Reference behaviour replaced: ext_aggregator.cpp:630-706
// (execute_batched_embed_slots: clamp + torch::embedding + copy per slot) and
// ext_aggregator.cpp:757-787, :821-874 (LM head logits, greedy argmax).
#include <cuda_bf16.h>

#include "common.h"
#include "launch.h"
#include "ptx.cuh"
#include "shm_abi.h"
#include "swarmlora_b200.h"
#include "vocab_ops.h"

namespace swl {

namespace {

// One CTA per gathered token; 16-byte vectors along the hidden dimension.
__global__ void embed_gather_kernel(const __grid_constant__ TokenTable tab,
                                    const __nv_bfloat16* __restrict__ table, int64_t vocab,
                                    int64_t hidden) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int gr = blockIdx.x;
  int lo = 0, hi = tab.nslots - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (tab.row_start[mid] <= gr) lo = mid;
    else hi = mid - 1;
  }
  const int64_t local = gr - tab.row_start[lo];
  int64_t tok = tab.tokens[lo][local];
  tok = tok < 0 ? 0 : (tok >= vocab ? vocab - 1 : tok);  // clamp(0, vocab-1) as the reference
  const uint4* src = reinterpret_cast<const uint4*>(table + tok * hidden);
  uint4* dst = reinterpret_cast<uint4*>(tab.out[lo] + local * hidden);
  for (int64_t i = threadIdx.x; i < hidden / 8; i += blockDim.x) dst[i] = src[i];
}

// A cluster of kArgmaxSplit CTAs per row: CTA q takes the q-th slice of the
// row (16-byte vectors when the rows are 16-byte aligned), keeps the largest
// bf16 logit with the lowest index among equals (torch.argmax returns the
// first maximal index), and CTA 0 merges the slices' winners through
// distributed shared memory.
constexpr int kArgmaxSplit = 8;
constexpr int kArgmaxThreads = 256;

__device__ __forceinline__ void argmax_take(float& best, int64_t& besti, float v, int64_t i) {
  if (v > best || (v == best && i < besti)) {
    best = v;
    besti = i;
  }
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const __nv_bfloat16* __restrict__ logits,
                                                                     int64_t vocab, int64_t ld,
                                                                     const __grid_constant__ TokenOuts outs) {
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int64_t si[kArgmaxThreads / 32];
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int row = blockIdx.x / kArgmaxSplit;
  const int q = static_cast<int>(ptx::cluster_rank());
  const __nv_bfloat16* x = logits + row * ld;
  const int64_t slice = (vocab + kArgmaxSplit * 8 - 1) / (kArgmaxSplit * 8) * 8;  // multiple of 8
  const int64_t c0 = min(vocab, q * slice), c1 = min(vocab, c0 + slice);
  float best = -INFINITY;
  int64_t besti = vocab;  // sentinel larger than any index
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const int64_t v1 = c1 / 8;  // full vectors of the slice (c0 is a multiple of 8)
#pragma unroll 4
    for (int64_t vi = c0 / 8 + threadIdx.x; vi < v1; vi += kArgmaxThreads) {
      const uint4 u = reinterpret_cast<const uint4*>(x)[vi];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        argmax_take(best, besti, __uint_as_float(w[e] << 16), vi * 8 + 2 * e);
        argmax_take(best, besti, __uint_as_float(w[e] & 0xffff0000u), vi * 8 + 2 * e + 1);
      }
    }
    for (int64_t i = v1 * 8 + threadIdx.x; i < c1; i += kArgmaxThreads)
      argmax_take(best, besti, __bfloat162float(x[i]), i);
  } else {
    for (int64_t i = c0 + threadIdx.x; i < c1; i += kArgmaxThreads)
      argmax_take(best, besti, __bfloat162float(x[i]), i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_take(best, besti, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, besti, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = best;
    si[w] = besti;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < kArgmaxThreads / 32; ++k) argmax_take(best, besti, sv[k], si[k]);
    sv[0] = best;
    si[0] = besti;
  }
  ptx::cluster_sync();
  if (q == 0 && threadIdx.x == 0) {
    const uint32_t mv = static_cast<uint32_t>(__cvta_generic_to_shared(&sv[0]));
    const uint32_t mi = static_cast<uint32_t>(__cvta_generic_to_shared(&si[0]));
    for (int r = 1; r < kArgmaxSplit; ++r) {
      float pv;
      int64_t pi;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv) : "r"(ptx::map_peer(mv, r)) : "memory");
      asm volatile("ld.shared::cluster.s64 %0, [%1];" : "=l"(pi) : "r"(ptx::map_peer(mi, r)) : "memory");
      argmax_take(best, besti, pv, pi);
    }
    *outs.p[row] = besti < vocab ? besti : 0;
  }
  ptx::cluster_sync();  // CTA 0 has read every slice's winner
}

// ---- sampling ---------------------------------------------------------------
// One CTA per row. Values are x_i = bf16(logit_i / T) (the reference divides
// the bf16 logits by the temperature, ext_aggregator.cpp:758); every pass
// re-reads the row from L2 and maps x_i to an order-preserving 32-bit key.
constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;

// Larger float -> larger key; NaN -> 0 (below -inf, never kept); -0 and +0
// share a key (they compare equal, so they tie as in torch's top-k / sort).
__device__ __forceinline__ uint32_t order_key(float f) {
  if (f != f) return 0u;
  const uint32_t b = __float_as_uint(f == 0.0f ? 0.0f : f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SampleShared {
  uint32_t cnt[256];
  float mass[256];
  float wf[kSampleWarps];
  uint32_t wu[kSampleWarps];
  int sel;
  uint32_t selu;
  float self;
};

__device__ __forceinline__ float block_sum(float v, SampleShared& sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.wf[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < kSampleWarps; ++k) t += sh.wf[k];
    sh.self = t;
  }
  __syncthreads();
  return sh.self;
}

__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, SampleShared& sh) {
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.wu[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int k = 0; k < kSampleWarps; ++k) t = max(t, sh.wu[k]);
    sh.selu = t;
  }
  __syncthreads();
  return sh.selu;
}

// Exclusive prefix over threads (in thread order) and the total.
template <class T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* total, T* warp_buf, T* tot_buf) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  T inc = v;
  for (int o = 1; o < 32; o <<= 1) {
    const T n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  __syncthreads();
  if (lane == 31) warp_buf[w] = inc;
  __syncthreads();
  if (threadIdx.x == 0) {
    T run = T(0);
    for (int k = 0; k < kSampleWarps; ++k) {
      const T t = warp_buf[k];
      warp_buf[k] = run;
      run += t;
    }
    *tot_buf = run;
  }
  __syncthreads();
  *total = *tot_buf;
  return warp_buf[w] + inc - v;
}

__device__ __forceinline__ float scaled(const __nv_bfloat16* x, int64_t i, float inv_t) {
  return __bfloat162float(__float2bfloat16_rn(__bfloat162float(x[i]) * inv_t));
}

// A uniform in [0, 1) from (seed, offset, row): SplitMix64 (Steele, Lea and
// Flood, 2014) of their combination, top 24 bits.
__device__ __forceinline__ float hashed_uniform(uint64_t seed, uint64_t offset, uint64_t row) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ull * (offset * 0x100000001ull + row + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}

__global__ void __launch_bounds__(kSampleThreads) sample_rows_kernel(
    const __nv_bfloat16* __restrict__ logits, int64_t vocab, int64_t ld, const __grid_constant__ SampleTable tab,
    const float* __restrict__ u_in, uint64_t seed, uint64_t offset, const __grid_constant__ TokenOuts outs) {
  __shared__ SampleShared sh;
  __shared__ float fscan[kSampleWarps];
  __shared__ float ftot;
  __shared__ int iscan[kSampleWarps];
  __shared__ int itot;
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int row = blockIdx.x, tid = threadIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  const SampleParams p = tab.p[row];

  if (!p.do_sample) {  // greedy: the lowest index of the largest logit (torch.argmax)
    uint32_t best = 0;
    for (int64_t i = tid; i < vocab; i += kSampleThreads) best = max(best, order_key(__bfloat162float(x[i])));
    const uint32_t m = block_max_u32(best, sh);
    int64_t first = vocab;
    if (m != 0u)
      for (int64_t i = tid; i < vocab; i += kSampleThreads)
        if (order_key(__bfloat162float(x[i])) == m) { first = i; break; }
    uint32_t lo = static_cast<uint32_t>(min(first, vocab));
    lo = ~block_max_u32(~lo, sh);  // minimum index holding the maximum
    if (tid == 0) *outs.p[row] = (m == 0u || lo >= vocab) ? 0 : static_cast<int64_t>(lo);
    return;
  }

  const float inv_t = 1.0f / fmaxf(p.temperature, 0.01f);  // temperature clamped as the reference
  // top-k threshold: the k-th largest key (ties at it are kept, as
  // `logits < threshold -> -inf` keeps them); radix select, 8 bits per pass
  uint32_t klo = 1u;  // NaN keys (0) are never kept
  if (p.top_k > 0 && p.top_k < vocab) {
    uint32_t prefix = 0, mask = 0;
    int remaining = p.top_k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += kSampleThreads) sh.cnt[b] = 0;
      __syncthreads();
      for (int64_t i = tid; i < vocab; i += kSampleThreads) {
        const uint32_t k = order_key(scaled(x, i, inv_t));
        if ((k & mask) == prefix) atomicAdd(&sh.cnt[(k >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        int cum = 0, b = 255;
        for (; b > 0; --b) {
          if (cum + static_cast<int>(sh.cnt[b]) >= remaining) break;
          cum += static_cast<int>(sh.cnt[b]);
        }
        sh.sel = b;
        sh.selu = static_cast<uint32_t>(remaining - cum);
      }
      __syncthreads();
      prefix |= static_cast<uint32_t>(sh.sel) << shift;
      mask |= 255u << shift;
      remaining = static_cast<int>(sh.selu);
      __syncthreads();
    }
    klo = max(prefix, 1u);
  }
  // the largest key and the softmax weights exp(x - x_max) of the kept tokens
  uint32_t kmax = 0;
  for (int64_t i = tid; i < vocab; i += kSampleThreads) kmax = max(kmax, order_key(scaled(x, i, inv_t)));
  kmax = block_max_u32(kmax, sh);
  if (kmax == 0u) {  // nothing but NaN
    if (tid == 0) *outs.p[row] = 0;
    return;
  }
  const float xmax = key_value(kmax);
  auto weight = [&](uint32_t k, float v) -> float { return k >= klo ? expf(v - xmax) : 0.f; };

  // top-p: keep tokens in descending (value, then index) order while the
  // running probability stays <= top_p, and always the first one
  // (ext_aggregator.cpp:769-783). Radix descent on the mass per key bucket
  // finds the boundary key kp; of the tokens holding kp, the first `tie_keep`
  // in index order are kept.
  bool cut = false;
  uint32_t kp = 0;
  int tie_keep = 0;
  if (p.top_p < 1.0f) {
    float zl = 0.f;
    for (int64_t i = tid; i < vocab; i += kSampleThreads) {
      const float v = scaled(x, i, inv_t);
      zl += weight(order_key(v), v);
    }
    const float target = p.top_p * block_sum(zl, sh);
    uint32_t prefix = 0, mask = 0;
    float above = 0.f;  // mass of kept tokens with keys above the current bucket
    bool all_fit = false;
    for (int shift = 24; shift >= 0 && !all_fit; shift -= 8) {
      for (int b = tid; b < 256; b += kSampleThreads) {
        sh.cnt[b] = 0;
        sh.mass[b] = 0.f;
      }
      __syncthreads();
      for (int64_t i = tid; i < vocab; i += kSampleThreads) {
        const float v = scaled(x, i, inv_t);
        const uint32_t k = order_key(v);
        if (k >= klo && (k & mask) == prefix) {
          const uint32_t b = (k >> shift) & 255u;
          atomicAdd(&sh.cnt[b], 1u);
          atomicAdd(&sh.mass[b], weight(k, v));
        }
      }
      __syncthreads();
      if (tid == 0) {
        int found = -1, lowest = -1;
        float a = above;
        for (int b = 255; b >= 0; --b) {
          if (sh.cnt[b] == 0u) continue;
          if (a + sh.mass[b] > target) {
            found = b;
            break;
          }
          a += sh.mass[b];
          lowest = b;
        }
        // below the top level the range came from a bucket that did not fit;
        // if rounding of the sums says otherwise, cut below its lowest bucket
        if (found < 0 && shift != 24 && lowest >= 0) {
          found = lowest;
          a -= sh.mass[lowest];
        }
        sh.sel = found;
        sh.self = a;
      }
      __syncthreads();
      if (sh.sel < 0) {
        all_fit = true;  // every kept token of this range fits under top_p
      } else {
        prefix |= static_cast<uint32_t>(sh.sel) << shift;
        mask |= 255u << shift;
        above = sh.self;
      }
      __syncthreads();
    }
    if (!all_fit) {
      cut = true;
      kp = prefix;
      const float e = expf(key_value(kp) - xmax);
      const float room = target - above;
      const float q = room > 0.f ? room / e : 0.f;  // e may underflow to 0: q = inf
      tie_keep = q >= 2.0e9f ? 2000000000 : static_cast<int>(floorf(q));
      if (kp == kmax && tie_keep == 0) tie_keep = 1;  // the most probable token is always kept
    }
  }

  // draw: inverse CDF in index order over the kept tokens; each thread owns
  // a contiguous chunk of indices
  const int64_t chunk = (vocab + kSampleThreads - 1) / kSampleThreads;
  const int64_t c0 = min(vocab, tid * chunk), c1 = min(vocab, c0 + chunk);
  int ties = 0;
  if (cut)
    for (int64_t i = c0; i < c1; ++i) ties += order_key(scaled(x, i, inv_t)) == kp;
  int tie_total = 0;
  const int tie_base = cut ? block_exclusive_scan<int>(ties, &tie_total, iscan, &itot) : 0;
  auto kept = [&](uint32_t k, int& tie_rank) -> bool {
    if (k < klo) return false;
    if (!cut || k > kp) return true;
    if (k < kp) return false;
    return tie_rank++ < tie_keep;
  };
  float mine = 0.f;
  {
    int tr = tie_base;
    for (int64_t i = c0; i < c1; ++i) {
      const float v = scaled(x, i, inv_t);
      const uint32_t k = order_key(v);
      if (kept(k, tr)) mine += expf(v - xmax);
    }
  }
  float z = 0.f;
  const float before = block_exclusive_scan<float>(mine, &z, fscan, &ftot);
  const float u = u_in ? u_in[row] : hashed_uniform(seed, offset, static_cast<uint64_t>(row));
  const float target = u * z;
  const int claim = (mine > 0.f && before <= target) ? tid : -1;
  const uint32_t finder = block_max_u32(static_cast<uint32_t>(claim + 1), sh);  // 0: none
  if (finder != 0u && tid == static_cast<int>(finder) - 1) {
    int tr = tie_base;
    float run = before;
    int64_t pick = -1, last = -1;
    for (int64_t i = c0; i < c1; ++i) {
      const float v = scaled(x, i, inv_t);
      const uint32_t k = order_key(v);
      if (!kept(k, tr)) continue;
      last = i;
      run += expf(v - xmax);
      if (run > target) {
        pick = i;
        break;
      }
    }
    *outs.p[row] = pick >= 0 ? pick : last;
  } else if (finder == 0u && tid == 0) {
    *outs.p[row] = 0;
  }
}

}  // namespace

int launch_embed_gather(const TokenTable& tab, const void* table, int64_t vocab, int64_t hidden,
                        cudaStream_t stream) {
  if (tab.total_rows <= 0) return SWL_OK;
  if (hidden % 8) return set_error(SWL_ERR_ARG, "embed: hidden must be a multiple of 8");
  SWL_CUDA_TRY(launch_kernel(embed_gather_kernel, dim3(tab.total_rows), dim3(256), 0, stream, 1, tab,
                             static_cast<const __nv_bfloat16*>(table), vocab, hidden));
  return SWL_OK;
}

int launch_sample_rows(const void* logits, int rows, int64_t vocab, int64_t ld, const SampleTable& params,
                       const float* u, uint64_t seed, uint64_t offset, const TokenOuts& outs,
                       cudaStream_t stream) {
  if (rows <= 0) return SWL_OK;
  if (rows > kMaxSlots) return set_error(SWL_ERR_ARG, "sample: too many rows");
  if (vocab <= 0 || vocab > (int64_t{1} << 31) - kSampleThreads)
    return set_error(SWL_ERR_ARG, "sample: vocab %lld out of range", static_cast<long long>(vocab));
  SWL_CUDA_TRY(launch_kernel(sample_rows_kernel, dim3(rows), dim3(kSampleThreads), 0, stream, 1,
                             static_cast<const __nv_bfloat16*>(logits), vocab, ld, params, u, seed, offset, outs));
  return SWL_OK;
}

int launch_argmax_rows(const void* logits, int rows, int64_t vocab, int64_t ld,
                       const TokenOuts& outs, cudaStream_t stream) {
  if (rows <= 0) return SWL_OK;
  if (rows > kMaxSlots) return set_error(SWL_ERR_ARG, "argmax: too many rows");
  SWL_CUDA_TRY(launch_kernel(argmax_rows_kernel, dim3(rows * kArgmaxSplit), dim3(kArgmaxThreads), 0, stream,
                             kArgmaxSplit, static_cast<const __nv_bfloat16*>(logits), vocab, ld, outs));
  return SWL_OK;
}

}  // namespace swl

using namespace swl;

// Greedy next-token pick of the LM-head op (ext_aggregator.cpp:821-874,
// torch.argmax over each row's logits): out[r] = the lowest index of the
// largest value among logits[r * ld + 0 .. vocab). NaN entries never win; a
// row with no finite maximum yields 0. out is int64 device memory.
SWL_EXPORT int swl_argmax_rows(const void* logits, int rows, int64_t vocab, int64_t ld, int64_t* out,
                               void* stream) {
  if (rows < 0 || rows > kMaxSlots || vocab <= 0 || ld < vocab || (rows > 0 && (!logits || !out)))
    return set_error(SWL_ERR_ARG, "argmax: invalid arguments");
  TokenOuts outs;
  for (int i = 0; i < kMaxSlots; ++i) outs.p[i] = i < rows ? out + i : nullptr;
  return launch_argmax_rows(logits, rows, vocab, ld, outs, static_cast<cudaStream_t>(stream));
}

// Next token of each row of bf16 logits (row r at logits + r * ld, vocab
// entries): rows whose params say do_sample draw from the softmax of
// bf16(logit / max(temperature, 0.01)) restricted to the top_k largest (ties
// kept; 0 = all) and then to the top_p nucleus (keep while the running
// probability in descending order stays <= top_p, always the first), as the
// reference's LM head does (ext_aggregator.cpp:757-787, :821-874); the draw
// is the inverse CDF in index order at u[r] (device floats in [0, 1), or
// derived from (seed, offset, r) when u is NULL). Other rows take the argmax.
SWL_EXPORT int swl_sample_rows(const void* logits, int rows, int64_t vocab, int64_t ld,
                               const swl_sampling* params, const float* u, uint64_t seed, uint64_t offset,
                               int64_t* out, void* stream) {
  if (rows < 0 || rows > kMaxSlots || vocab <= 0 || ld < vocab || (rows > 0 && (!logits || !out || !params)))
    return set_error(SWL_ERR_ARG, "sample: invalid arguments");
  static_assert(sizeof(swl_sampling) == sizeof(SampleParams), "swl_sampling layout");
  SampleTable tab;
  TokenOuts outs;
  for (int i = 0; i < kMaxSlots; ++i) {
    tab.p[i] = i < rows ? SampleParams{params[i].do_sample, params[i].temperature, params[i].top_k, params[i].top_p}
                        : SampleParams{0, 1.0f, 0, 1.0f};
    outs.p[i] = i < rows ? out + i : nullptr;
  }
  return launch_sample_rows(logits, rows, vocab, ld, tab, u, seed, offset, outs, static_cast<cudaStream_t>(stream));
}
