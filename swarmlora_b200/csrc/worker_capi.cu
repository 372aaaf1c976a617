// C-ABI entry points for the worker-side kernels (worker_ops.cu). Every
// argument is a plain pointer, size or array of per-slot device pointers;
// segment i of a call covers rows[i] token rows of slot i.
#include "common.h"
#include "worker_ops.h"

#include <atomic>
#include <mutex>

using namespace swl;

namespace {

int fill_segments(RowSegments* s, int nseg, const int* rows) {
  if (nseg < 0 || nseg > kMaxSlots) return set_error(SWL_ERR_ARG, "segment count %d out of range", nseg);
  if (nseg > 0 && !rows) return set_error(SWL_ERR_ARG, "null rows array");
  s->nseg = nseg;
  int acc = 0;
  for (int i = 0; i < nseg; ++i) {
    if (rows[i] < 0) return set_error(SWL_ERR_ARG, "negative row count");
    s->row_start[i] = acc;
    acc += rows[i];
  }
  s->row_start[nseg] = acc;
  s->total_rows = acc;
  return SWL_OK;
}

template <class T>
T* cast(const void* p) {
  return static_cast<T*>(const_cast<void*>(p));
}

}  // namespace

// LoRA shrink (model_builder.py:258-262 first GEMM, worker_sync.py:305/:375
// lora_A): ws[split][row][R] = partial sums of x[row] @ A over a K split.
// A[i] is [K, R] row-major (NULL: slot has no adapter, nothing written).
SWL_EXPORT int swl_lora_shrink(int nseg, const int* rows, const void* const* x, int64_t x_stride,
                               const void* const* A, int64_t K, int R, int splits, float* ws,
                               void* stream) {
  LoraShrinkTable t;
  SWL_TRY(fill_segments(&t.seg, nseg, rows));
  for (int i = 0; i < nseg; ++i) {
    t.x[i] = cast<const __nv_bfloat16>(x[i]);
    t.A[i] = cast<const __nv_bfloat16>(A[i]);
  }
  return launch_lora_shrink(t, K, R, x_stride, splits, ws, static_cast<cudaStream_t>(stream));
}

// LoRA expand fused with the round epilogue. mode 0: out = base + d (QKV);
// mode 1: out = resid + (base + d) (O / Down, d scaled by post_scale after
// the expand); mode 2: out = silu(gate + dg) * (up + du) over the Gate+Up
// output (out has n_total / 2 columns). block_end[nblocks] gives the fused
// projections' column ends; B[i] is [n_total, r] (lora_B rows), NULL = none.
SWL_EXPORT int swl_lora_expand(int nseg, const int* rows, const void* const* base,
                               int64_t base_stride, const void* const* B, const void* const* resid,
                               int64_t resid_stride, void* const* out, int64_t out_stride,
                               int64_t n_total, int r, int nblocks, const int64_t* block_end,
                               float post_scale, int mode, int splits, const float* ws,
                               void* stream) {
  if (nblocks < 1 || nblocks > 3 || !block_end) return set_error(SWL_ERR_ARG, "lora_expand: bad block layout");
  if (mode < 0 || mode > 2) return set_error(SWL_ERR_ARG, "lora_expand: bad mode");
  if (mode == kExpandResidual && !resid) return set_error(SWL_ERR_ARG, "lora_expand: residual mode needs resid");
  LoraExpandTable t;
  SWL_TRY(fill_segments(&t.seg, nseg, rows));
  for (int i = 0; i < nseg; ++i) {
    t.base[i] = cast<const __nv_bfloat16>(base[i]);
    t.B[i] = B ? cast<const __nv_bfloat16>(B[i]) : nullptr;
    t.resid[i] = resid ? cast<const __nv_bfloat16>(resid[i]) : nullptr;
    t.out[i] = cast<__nv_bfloat16>(out[i]);
  }
  ExpandParams p;
  p.n_total = n_total;
  p.r = r;
  p.nblocks = nblocks;
  for (int b = 0; b < 3; ++b) p.block_end[b] = b < nblocks ? block_end[b] : n_total;
  p.post_scale = post_scale;
  p.mode = mode;
  p.base_stride = base_stride;
  p.out_stride = out_stride;
  p.resid_stride = resid_stride;
  p.splits = splits;
  return launch_lora_expand(t, p, ws, static_cast<cudaStream_t>(stream));
}

namespace {
int fill_attn(AttnTable* t, int nseg, const int* rows, const void* const* qkv,
              const void* const* block_tables, void* const* k_cache, void* const* v_cache,
              const void* const* seqlens, void* const* out) {
  SWL_TRY(fill_segments(&t->seg, nseg, rows));
  for (int i = 0; i < nseg; ++i) {
    t->qkv[i] = qkv ? cast<const __nv_bfloat16>(qkv[i]) : nullptr;
    t->block_table[i] = cast<const int>(block_tables[i]);
    t->k_cache[i] = cast<__nv_bfloat16>(k_cache[i]);
    t->v_cache[i] = cast<__nv_bfloat16>(v_cache[i]);
    t->seqlen[i] = cast<const int>(seqlens[i]);
    t->out[i] = out ? cast<__nv_bfloat16>(out[i]) : nullptr;
    if (!t->block_table[i] || !t->k_cache[i] || !t->v_cache[i] || !t->seqlen[i])
      return set_error(SWL_ERR_ARG, "attention: null per-slot pointer");
  }
  return SWL_OK;
}
}  // namespace

// NeoX rotary embedding of q and k (vLLM rotary_embedding, is_neox=True, as
// called at worker_sync.py:192-193) and the paged KV append done inside
// flash_attn_with_kvcache (worker_sync.py:196-203): token t of slot i sits at
// position *seqlens[i] + t; rotated q goes to q_rot [total_rows, hq*D].
SWL_EXPORT int swl_rope_append(int nseg, const int* rows, const void* const* qkv,
                               int64_t qkv_stride, const void* const* block_tables,
                               void* const* k_cache, void* const* v_cache,
                               const void* const* seqlens, int hq, int hkv, int head_dim, int page,
                               const void* cos_sin, int max_pos, void* q_rot, void* stream) {
  AttnTable t;
  SWL_TRY(fill_attn(&t, nseg, rows, qkv, block_tables, k_cache, v_cache, seqlens, nullptr));
  AttnParams p = {};
  p.hq = hq; p.hkv = hkv; p.head_dim = head_dim; p.page = page;
  p.qkv_stride = qkv_stride;
  p.cos_sin = cast<const __nv_bfloat16>(cos_sin);
  p.max_pos = max_pos;
  p.q_rot = cast<__nv_bfloat16>(q_rot);
  return launch_rope_append(t, p, static_cast<cudaStream_t>(stream));
}

// Number of fp32 scratch floats swl_paged_attention needs in `part` for this
// launch shape (0 when the context is not split).
SWL_EXPORT int64_t swl_attention_part_floats(int total_rows, int hq, int hkv, int max_len) {
  return attention_part_floats(total_rows, hq, attention_splits(total_rows, hkv, max_len));
}

// Tuning knob of the attention launch: pages per context chunk, depth of
// the page ring (2..4) and kv head groups (1, 2, 4, 8: CTAs sharing one
// page's heads); 0 restores the automatic choice.
SWL_EXPORT int swl_attention_tune(int chunk_pages, int stages, int groups) {
  return set_attention_tuning(chunk_pages, stages, groups);
}

// 1 (default): two consecutive rows of a slot share each page read when a
// launch has slots with several rows; 0: every row reads its pages alone.
SWL_EXPORT int swl_attention_pairing(int on) { return set_attention_pairing(on); }

// 1 (default): K/V pages loaded by TMA when every row's pages lie in one
// cache allocation; 0: per-lane copies always.
SWL_EXPORT int swl_attention_tma(int on) { return set_attention_tma(on); }

// Causal GQA attention of each new token over its slot's paged cache
// (flash_attn_with_kvcache semantics, worker_sync.py:196-203): token t of
// slot i attends to cache positions 0 .. *seqlens[i] + t. max_len bounds
// every slot's *seqlens + rows (it sizes the context split). out[i] rows get
// [hq * D] bf16 (row stride out_stride).
SWL_EXPORT int swl_paged_attention(int nseg, const int* rows, const void* const* block_tables,
                                   const void* const* k_cache, const void* const* v_cache,
                                   const void* const* seqlens, void* const* out, int64_t out_stride,
                                   int hq, int hkv, int head_dim, int page, float scale, int max_len,
                                   const void* q_rot, float* part, void* stream) {
  AttnTable t;
  SWL_TRY(fill_attn(&t, nseg, rows, nullptr, block_tables, const_cast<void* const*>(k_cache),
                    const_cast<void* const*>(v_cache), seqlens, out));
  AttnParams p = {};
  p.hq = hq; p.hkv = hkv; p.head_dim = head_dim; p.page = page;
  p.out_stride = out_stride;
  p.scale = scale;
  p.max_len = max_len;
  p.q_rot = cast<__nv_bfloat16>(q_rot);
  p.part = part;
  return launch_paged_attention(t, p, static_cast<cudaStream_t>(stream));
}

// swl_paged_attention plus the O projection's LoRA shrink on its output:
// ws_o[row][head][j] = sum_d out[row, head*D + d] * A_o[i][head*D + d, j]
// (A_o[i] = lora_A(o_proj)^T, [hq*D, r]; NULL for a slot without adapter).
SWL_EXPORT int swl_paged_attention_shrink(int nseg, const int* rows, const void* const* block_tables,
                                          const void* const* k_cache, const void* const* v_cache,
                                          const void* const* seqlens, void* const* out,
                                          int64_t out_stride, int hq, int hkv, int head_dim, int page,
                                          float scale, int max_len, const void* q_rot, float* part,
                                          const void* const* A_o, int r, float* ws_o,
                                          const void* pf, int64_t pf_bytes, void* stream) {
  AttnTable t;
  SWL_TRY(fill_attn(&t, nseg, rows, nullptr, block_tables, const_cast<void* const*>(k_cache),
                    const_cast<void* const*>(v_cache), seqlens, out));
  AttnParams p = {};
  p.hq = hq; p.hkv = hkv; p.head_dim = head_dim; p.page = page;
  p.out_stride = out_stride;
  p.scale = scale;
  p.max_len = max_len;
  p.q_rot = cast<__nv_bfloat16>(q_rot);
  p.part = part;
  p.pf = pf;
  p.pf_bytes = pf_bytes;
  ShrinkSide sh;
  for (int i = 0; i < kMaxSlots; ++i) sh.A[i] = (A_o && i < nseg) ? cast<const __nv_bfloat16>(A_o[i]) : nullptr;
  sh.r = r;
  sh.ws = ws_o;
  if (!ws_o) return set_error(SWL_ERR_ARG, "attention shrink: null ws");
  return launch_paged_attention(t, p, static_cast<cudaStream_t>(stream), &sh);
}

// Fused epilogue of the QKV round: q|k|v = round output + LoRA delta (shrink
// partials ws_in [rows][splits_in][3r], lora_B rows B[i] [(hq+2hkv)*D, r]),
// NeoX RoPE of q and k at position *seqlens[i] + t, k and v appended to the
// paged cache, rotated q written to q_rot [total_rows, hq*D].
SWL_EXPORT int swl_fused_qkv_rope(int nseg, const int* rows, const void* const* base,
                                  int64_t base_stride, const void* const* B, int r,
                                  const float* ws_in, int splits_in,
                                  const void* const* block_tables, void* const* k_cache,
                                  void* const* v_cache, const void* const* seqlens, int hq,
                                  int hkv, int head_dim, int page, const void* cos_sin,
                                  void* q_rot, const void* pf, int64_t pf_bytes, void* stream) {
  QkvRopeTable t;
  SWL_TRY(fill_segments(&t.seg, nseg, rows));
  for (int i = 0; i < nseg; ++i) {
    t.base[i] = cast<const __nv_bfloat16>(base[i]);
    t.B[i] = B ? cast<const __nv_bfloat16>(B[i]) : nullptr;
    t.block_table[i] = cast<const int>(block_tables[i]);
    t.k_cache[i] = cast<__nv_bfloat16>(k_cache[i]);
    t.v_cache[i] = cast<__nv_bfloat16>(v_cache[i]);
    t.seqlen[i] = cast<const int>(seqlens[i]);
  }
  QkvRopeParams p;
  p.hq = hq; p.hkv = hkv; p.head_dim = head_dim; p.page = page;
  p.base_stride = base_stride;
  p.ws_in = ws_in;
  p.splits_in = splits_in;
  p.cos_sin = cast<const __nv_bfloat16>(cos_sin);
  p.q_rot = cast<__nv_bfloat16>(q_rot);
  p.pf = pf;
  p.pf_bytes = pf_bytes;
  return launch_qkv_rope(t, p, r, static_cast<cudaStream_t>(stream));
}

// Fused epilogue of the O / Down round (and of the embedding): h = [h +]
// (base + bf16(bf16(t @ B^T) * post_scale)), then x = RMSNorm(h) * w written to
// x_out (the next round's slot input) and the next round's LoRA shrink
// partials ws_next[rows][8][r_next] = x @ A_next (A_next[i] NULL: none).
SWL_EXPORT int swl_fused_resid_norm_shrink(int nseg, const int* rows, const void* const* base,
                                           int64_t base_stride, const void* const* B, int r_in,
                                           float post_scale, const float* ws_in, int splits_in,
                                           int has_resid, void* const* h, int64_t h_stride,
                                           const void* w, int64_t hidden, float eps,
                                           void* const* x_out, int64_t x_stride,
                                           const void* const* A_next, int r_next, float* ws_next,
                                           const void* pf, int64_t pf_bytes, void* stream) {
  ResidNormTable t;
  SWL_TRY(fill_segments(&t.seg, nseg, rows));
  for (int i = 0; i < nseg; ++i) {
    t.base[i] = cast<const __nv_bfloat16>(base[i]);
    t.B[i] = B ? cast<const __nv_bfloat16>(B[i]) : nullptr;
    t.h[i] = cast<__nv_bfloat16>(h[i]);
    t.x_out[i] = cast<__nv_bfloat16>(x_out[i]);
    t.A_next[i] = A_next ? cast<const __nv_bfloat16>(A_next[i]) : nullptr;
  }
  ResidNormParams p;
  p.hidden = hidden;
  p.post_scale = post_scale;
  p.ws_in = ws_in;
  p.splits_in = splits_in;
  p.has_resid = has_resid;
  p.w = cast<const __nv_bfloat16>(w);
  p.eps = eps;
  p.base_stride = base_stride;
  p.h_stride = h_stride;
  p.x_stride = x_stride;
  p.r_next = A_next ? r_next : 0;
  p.ws_next = ws_next;
  p.pf = pf;
  p.pf_bytes = pf_bytes;
  return launch_resid_norm_shrink(t, p, B ? r_in : 0, static_cast<cudaStream_t>(stream));
}

// Fused epilogue of the Gate+Up round: gate/up = round output + LoRA delta
// (partials ws_in [rows][splits_in][2r], lora_B rows B[i] [2*inter, r]),
// act = SiLU(gate) * up written to act[i] (the Down round's slot input), and
// the Down LoRA shrink partials ws_next[rows][ceil(inter/512)][r_next].
SWL_EXPORT int swl_fused_gu_silu_shrink(int nseg, const int* rows, const void* const* base,
                                        int64_t base_stride, const void* const* B, int r,
                                        const float* ws_in, int splits_in, int64_t inter,
                                        void* const* act, int64_t act_stride,
                                        const void* const* A_next, int r_next, float* ws_next,
                                        const void* pf, int64_t pf_bytes, void* stream) {
  GuSiluTable t;
  SWL_TRY(fill_segments(&t.seg, nseg, rows));
  for (int i = 0; i < nseg; ++i) {
    t.base[i] = cast<const __nv_bfloat16>(base[i]);
    t.B[i] = B ? cast<const __nv_bfloat16>(B[i]) : nullptr;
    t.act[i] = cast<__nv_bfloat16>(act[i]);
    t.A_next[i] = A_next ? cast<const __nv_bfloat16>(A_next[i]) : nullptr;
  }
  GuSiluParams p;
  p.inter = inter;
  p.base_stride = base_stride;
  p.act_stride = act_stride;
  p.ws_in = ws_in;
  p.splits_in = splits_in;
  p.r_next = r_next;
  p.ws_next = ws_next;
  p.pf = pf;
  p.pf_bytes = pf_bytes;
  return launch_gu_silu_shrink(t, p, r, static_cast<cudaStream_t>(stream));
}

// Number of shrink partials swl_fused_resid_norm_shrink writes per row (its
// cluster size) for a group whose adapters are packed at LoRA rank `rank`.
SWL_EXPORT int swl_fused_norm_splits(int rank) { return resid_norm_splits(rank); }

// Number of Down-shrink partials swl_fused_gu_silu_shrink writes per row.
SWL_EXPORT int swl_fused_silu_splits(int64_t inter) { return gu_silu_splits(inter); }

// LlamaRMSNorm over rows: out = w * bf16(x * rsqrt(mean(x^2) + eps)).
SWL_EXPORT int swl_rms_norm(int nseg, const int* rows, const void* const* x, int64_t x_stride,
                            void* const* out, int64_t out_stride, const void* w, int64_t hidden,
                            float eps, void* stream) {
  NormTable t;
  SWL_TRY(fill_segments(&t.seg, nseg, rows));
  for (int i = 0; i < nseg; ++i) {
    t.x[i] = cast<const __nv_bfloat16>(x[i]);
    t.out[i] = cast<__nv_bfloat16>(out[i]);
  }
  return launch_rms_norm(t, cast<const __nv_bfloat16>(w), hidden, eps, x_stride, out_stride,
                         static_cast<cudaStream_t>(stream));
}

// n device-to-device copies in one launch: bytes[i] from src[i] to dst[i]
// (used to move tokens, embeddings and next-token ids between slot buffers
// and worker buffers without one memcpy call per slot).
SWL_EXPORT int swl_copy_rows(int n, const void* const* src, void* const* dst, const int64_t* bytes,
                             void* stream) {
  if (n < 0 || n > kMaxSlots || (n > 0 && (!src || !dst || !bytes)))
    return set_error(SWL_ERR_ARG, "copy_rows: invalid arguments");
  CopyTable t;
  for (int i = 0; i < n; ++i) {
    if (bytes[i] < 0 || (bytes[i] > 0 && (!src[i] || !dst[i])))
      return set_error(SWL_ERR_ARG, "copy_rows: bad entry %d", i);
    t.src[i] = src[i];
    t.dst[i] = dst[i];
    t.bytes[i] = bytes[i];
  }
  return launch_copy_rows(t, n, static_cast<cudaStream_t>(stream));
}

// p[0..n) += delta on the device (KV positions after a step).
SWL_EXPORT int swl_advance_i32(int* p, int n, int delta, void* stream) {
  if (n > 0 && !p) return set_error(SWL_ERR_ARG, "advance_i32: null pointer");
  return launch_advance_i32(p, n, delta, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Attention without caller scratch and without allocation.
//
// swl_paged_attention needs `part`, an fp32 buffer for the per-split partial
// results that the combine step merges. Some callers cannot provide one: a
// host whose allocator is not torch's (a foreign runtime bound over the C
// ABI), or code running where any allocation is forbidden (inside a region
// that must not touch the allocator, or on a path that must not fail on
// memory). For them this entry point keeps the partials in a fixed array
// compiled into the library, one copy per device, and allocates nothing.
//
// The array holds kNoAllocPartFloats fp32 values (4 MiB per device). A launch
// shape that needs more (swl_attention_part_floats) is rejected with
// SWL_ERR_ARG before anything is launched.
//
// The array is shared by every call on a device and keeps whatever the last
// call wrote. Calls issued on one stream run one after another and are safe;
// calls that can overlap on the GPU (two streams, two host threads) write the
// same records and produce wrong results. Nothing in the array needs to start
// at zero: each call writes every partial record before its combine step reads
// it.
//
// The first call on a device looks up the array's device address
// (cudaGetSymbolAddress, which may load this part of the library onto the
// device) and caches it; later calls only launch. Make that first call before
// any stream capture begins. The cached address belongs to the device's
// primary context: after cudaDeviceReset (or anything else that destroys and
// recreates that context) call swl_noalloc_forget_device so that the next
// call looks the address up again.
namespace {
constexpr int64_t kNoAllocPartFloats = int64_t{1} << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_attn_part[kNoAllocPartFloats];

std::mutex g_noalloc_mu;
std::atomic<float*> g_noalloc_part[kNoAllocMaxDevices];

int noalloc_scratch(float** out) {
  int dev = 0;
  SWL_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(SWL_ERR_ARG, "paged_attention_noalloc: device %d beyond %d", dev, kNoAllocMaxDevices);
  float* p = g_noalloc_part[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    p = g_noalloc_part[dev].load(std::memory_order_relaxed);
    if (!p) {
      void* addr = nullptr;
      SWL_CUDA_TRY(cudaGetSymbolAddress(&addr, g_noalloc_attn_part));
      if (!addr) return set_error(SWL_ERR_CUDA, "paged_attention_noalloc: null scratch address");
      p = static_cast<float*>(addr);
      g_noalloc_part[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return SWL_OK;
}
}  // namespace

// Drops the cached scratch address of the current device (after a device
// reset); the array itself stays as compiled.
SWL_EXPORT int swl_noalloc_forget_device(void) {
  int dev = 0;
  SWL_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return SWL_OK;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  g_noalloc_part[dev].store(nullptr, std::memory_order_release);
  return SWL_OK;
}

// swl_paged_attention with the same arguments minus `part`; the partials live
// in the library's static per-device array described above.
SWL_EXPORT int swl_paged_attention_noalloc(int nseg, const int* rows, const void* const* block_tables,
                                           const void* const* k_cache, const void* const* v_cache,
                                           const void* const* seqlens, void* const* out,
                                           int64_t out_stride, int hq, int hkv, int head_dim, int page,
                                           float scale, int max_len, const void* q_rot, void* stream) {
  AttnTable t;
  SWL_TRY(fill_attn(&t, nseg, rows, nullptr, block_tables, const_cast<void* const*>(k_cache),
                    const_cast<void* const*>(v_cache), seqlens, out));
  if (hq <= 0 || hkv <= 0)
    return set_error(SWL_ERR_ARG, "paged_attention_noalloc: hq and hkv must be positive");
  const int64_t need = attention_part_floats(t.seg.total_rows, hq,
                                             attention_splits(t.seg.total_rows, hkv, max_len));
  if (need > kNoAllocPartFloats)
    return set_error(SWL_ERR_ARG,
                     "paged_attention_noalloc: this launch needs %lld scratch floats, the static "
                     "scratch holds %lld (use swl_paged_attention with caller scratch)",
                     static_cast<long long>(need), static_cast<long long>(kNoAllocPartFloats));
  float* part = nullptr;
  SWL_TRY(noalloc_scratch(&part));
  AttnParams p = {};
  p.hq = hq; p.hkv = hkv; p.head_dim = head_dim; p.page = page;
  p.out_stride = out_stride;
  p.scale = scale;
  p.max_len = max_len;
  p.q_rot = cast<__nv_bfloat16>(q_rot);
  p.part = part;
  return launch_paged_attention(t, p, static_cast<cudaStream_t>(stream));
}
