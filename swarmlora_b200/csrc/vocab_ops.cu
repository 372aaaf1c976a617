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

// One CTA per row: max over bf16 logits, ties broken towards the lowest index
// (torch.argmax returns the first maximal index).
__global__ void argmax_rows_kernel(const __nv_bfloat16* __restrict__ logits, int64_t vocab,
                                   int64_t ld, const __grid_constant__ TokenOuts outs) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  float best = -INFINITY;
  int64_t besti = vocab;  // sentinel larger than any index
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    float v = __bfloat162float(x[i]);
    if (v > best || (v == best && i < besti)) {
      best = v;
      besti = i;
    }
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int64_t oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (ov > best || (ov == best && oi < besti)) {
      best = ov;
      besti = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = best;
    si[w] = besti;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = l < nw ? sv[l] : -INFINITY;
    besti = l < nw ? si[l] : vocab;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int64_t oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ov > best || (ov == best && oi < besti)) {
        best = ov;
        besti = oi;
      }
    }
    if (l == 0) *outs.p[row] = besti < vocab ? besti : 0;
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

int launch_argmax_rows(const void* logits, int rows, int64_t vocab, int64_t ld,
                       const TokenOuts& outs, cudaStream_t stream) {
  if (rows <= 0) return SWL_OK;
  if (rows > kMaxSlots) return set_error(SWL_ERR_ARG, "argmax: too many rows");
  SWL_CUDA_TRY(launch_kernel(argmax_rows_kernel, dim3(rows), dim3(1024), 0, stream, 1,
                             static_cast<const __nv_bfloat16*>(logits), vocab, ld, outs));
  return SWL_OK;
}

}  // namespace swl
