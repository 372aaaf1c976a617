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

}  // namespace

int launch_embed_gather(const TokenTable& tab, const void* table, int64_t vocab, int64_t hidden,
                        cudaStream_t stream) {
  if (tab.total_rows <= 0) return SWL_OK;
  if (hidden % 8) return set_error(SWL_ERR_ARG, "embed: hidden must be a multiple of 8");
  SWL_CUDA_TRY(launch_kernel(embed_gather_kernel, dim3(tab.total_rows), dim3(256), 0, stream, 1, tab,
                             static_cast<const __nv_bfloat16*>(table), vocab, hidden));
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

