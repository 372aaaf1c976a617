// Embedding gather and greedy token pick over slot buffers.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "shm_abi.h"

namespace swl {

// Token ids of slot i are tokens[i][0 .. row_start[i+1]-row_start[i]) (int64),
// the gathered bf16 rows go to out[i] (row stride = hidden).
struct TokenTable {
  int nslots;
  int total_rows;
  int row_start[kMaxSlots + 1];
  const int64_t* tokens[kMaxSlots];
  __nv_bfloat16* out[kMaxSlots];
};

int launch_embed_gather(const TokenTable& tab, const void* table, int64_t vocab, int64_t hidden,
                        cudaStream_t stream);

// Destination of each row's token id (passed to the kernel by value).
struct TokenOuts {
  int64_t* p[kMaxSlots];
};

// Row r's argmax (int64) goes to *outs.p[r]; rows <= kMaxSlots.
int launch_argmax_rows(const void* logits, int rows, int64_t vocab, int64_t ld,
                       const TokenOuts& outs, cudaStream_t stream);

// Sampling parameters of one row (its worker's OP_SET_SAMPLING state);
// the layout of the public swl_sampling.
struct SampleParams {
  int do_sample;
  float temperature;
  int top_k;
  float top_p;
};
struct SampleTable {
  SampleParams p[kMaxSlots];
};

// Row r's next token (int64) goes to *outs.p[r]: greedy rows take the
// argmax, sampling rows draw from the temperature / top-k / top-p filtered
// softmax with uniform u[r] (device floats in [0, 1)) or, when u is null,
// one derived from (seed, offset, r).
int launch_sample_rows(const void* logits, int rows, int64_t vocab, int64_t ld, const SampleTable& params,
                       const float* u, uint64_t seed, uint64_t offset, const TokenOuts& outs,
                       cudaStream_t stream);

}  // namespace swl
