// Persistent stream-K variant of the slot round (decode: M <= 256 tokens).
//
// One CTA per SM walks an equal, contiguous share of the round's work units
// (128 weight rows x 64 k) in tile-major order, so every SM streams the same
// number of weight bytes whatever the tile count (the split-K cluster kernel
// quantises work to whole tiles per CTA). A tile whose k range is shared by
// several CTAs is reduced through an fp32 workspace: each contributor stores
// its partial, then bumps the tile's arrival counter; the CTA that arrives
// last adds the partials in contributor order (deterministic), writes the bf16
// rows into the slot outputs and resets the counter. No CTA ever waits for
// another.
//
// Warp roles (256 threads): warp 0 TMA producer for W, warp 1 TMEM allocator
// and tcgen05.mma issuer, warps 2-3 gather producers (cp.async of the slot
// rows into the 128B-swizzled B operand), warps 4-7 epilogue. The TMEM
// accumulator is double-buffered so the epilogue of one tile segment overlaps
// the MMAs of the next.
//
// Reference behaviour replaced: ext_aggregator.cpp:470-626.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.h"
#include "ptx.cuh"
#include "slot_round.h"

namespace swl {

__device__ unsigned int g_sk_error_word = 0;

namespace {

constexpr int kBlockW = 128;
constexpr int kBlockK = 64;
constexpr int kWStageBytes = kBlockW * kBlockK * 2;
constexpr int kThreads = 256;
constexpr int kGather = 64;
constexpr int kEpi = 128;
constexpr uint64_t kTimeoutNs = 2000000000ull;

enum SkErr : unsigned int {
  kSkEmptyW = 11,
  kSkFull = 12,
  kSkEmptyX = 13,
  kSkAccFull = 14,
  kSkAccEmpty = 15,
};

template <int BN, int STAGES>
struct SkCfg {
  static_assert(BN == 32 || BN == 64, "stream-K rounds cover decode (<= 64 rows)");
  static constexpr int kStages = STAGES;
  static constexpr int kXStage = BN * 128;
  static constexpr int kPipe = kStages * (kWStageBytes + kXStage);
  static constexpr int kSmem = 1024 + kPipe + 512 + BN * 16;
  static constexpr int kTmemCols = 2 * BN;
};

struct SkParams {
  int nkb;         // k-blocks per tile
  int64_t units;   // n_tiles * nkb
  int ctas;        // persistent CTAs (grid size)
  int max_parts;   // workspace parts per tile
  float* ws;       // [n_tiles][max_parts][BN][128]
  int* counters;   // [n_tiles], zero between launches
};

__device__ __forceinline__ int sk_slot_of_row(const SlotTable& tab, int gr) {
  int lo = 0, hi = tab.nslots - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (tab.row_start[mid] <= gr) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// CTA whose unit range contains unit u: largest c with floor(c*U/P) <= u.
__device__ __forceinline__ int cta_of_unit(int64_t u, int64_t U, int P) {
  return static_cast<int>(((u + 1) * P + U - 1) / U) - 1;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    slot_round_sk_kernel(const __grid_constant__ CUtensorMap wmap,
                         const __grid_constant__ SlotTable tab, const RoundShape shape,
                         const SkParams sk) {
  using Cfg = SkCfg<BN, STAGES>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* w_st = smem;
  uint8_t* x_st = smem + S * kWStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(x_st + S * Cfg::kXStage);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;   // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* flag = reinterpret_cast<int*>(tmem_holder + 1);
  const __nv_bfloat16** row_in = reinterpret_cast<const __nv_bfloat16**>(tmem_holder + 4);
  __nv_bfloat16** row_out = reinterpret_cast<__nv_bfloat16**>(tmem_holder + 4 + 2 * BN);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  const int64_t U = sk.units;
  const int P = sk.ctas;
  const int64_t u0 = static_cast<int64_t>(c) * U / P;
  const int64_t u1 = static_cast<int64_t>(c + 1) * U / P;
  const int nkb = sk.nkb;
  const int rows = min(BN, tab.total_rows);
  unsigned int* err = &g_sk_error_word;

  for (int r = tid; r < BN; r += kThreads) {
    const __nv_bfloat16* pin = nullptr;
    __nv_bfloat16* pout = nullptr;
    if (r < rows) {
      const int s = sk_slot_of_row(tab, r);
      const int64_t local = r - tab.row_start[s];
      pin = tab.in[s] + local * shape.in_stride;
      pout = tab.out[s] + local * shape.out_stride;
    }
    row_in[r] = pin;
    row_out[r] = pout;
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1 + kGather);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&acc_full[a], 1);
      ptx::mbar_init(&acc_empty[a], kEpi);
    }
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&wmap);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_holder, Cfg::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = ptx::policy_evict_first();
      int i = 0;
      for (int64_t u = u0; u < u1; ++u, ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!ptx::mbar_wait(&empty[s], ph ^ 1, err, kSkEmptyW, kTimeoutNs)) break;
        ptx::mbar_arrive_expect_tx(&full[s], kWStageBytes);
        ptx::tma_load_2d(w_st + s * kWStageBytes, &wmap, &full[s], static_cast<int>(u % nkb) * kBlockK,
                         static_cast<int>(u / nkb) * kBlockW, pol);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_bf16_f32(kBlockW, BN);
      int i = 0, j = 0;
      bool ok = true;
      for (int64_t u = u0; u < u1 && ok; ++j) {
        const int64_t t = u / nkb;
        const int64_t seg_end = min(u1, (t + 1) * nkb);
        const int a = j & 1;
        if (!ptx::mbar_wait(&acc_empty[a], ((j >> 1) & 1) ^ 1, err, kSkAccEmpty, kTimeoutNs)) break;
        ptx::tc_fence_after();
        const uint32_t d = tmem + a * BN;
        bool first = true;
        for (; u < seg_end; ++u, ++i) {
          const int s = i % S;
          const uint32_t ph = (i / S) & 1;
          if (!ptx::mbar_wait(&full[s], ph, err, kSkFull, kTimeoutNs)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          // (no proxy fence: see slot_round.cu)
          const uint32_t wa = ptx::smem_addr(w_st + s * kWStageBytes);
          const uint32_t xa = ptx::smem_addr(x_st + s * Cfg::kXStage);
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            ptx::mma_bf16_ss(d, ptx::sw128_kmajor_desc(wa + kk * 32), ptx::sw128_kmajor_desc(xa + kk * 32),
                             idesc, (first && kk == 0) ? 0u : 1u);
          }
          first = false;
          ptx::tc_commit(&empty[s]);
        }
        ptx::tc_commit(&acc_full[a]);
      }
    }
  } else if (warp < 4) {
    const int tg = tid - 64;
    int i = 0;
    for (int64_t u = u0; u < u1; ++u, ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      if (!ptx::mbar_wait_sleep(&empty[s], ph ^ 1, err, kSkEmptyX, kTimeoutNs, 64)) break;
      const int64_t k0 = (u % nkb) * kBlockK;
      const uint32_t xs = ptx::smem_addr(x_st + s * Cfg::kXStage);
      for (int ci = tg; ci < BN * 8; ci += kGather) {
        const int r = ci >> 3, q = ci & 7;
        const __nv_bfloat16* src = row_in[r];
        const int64_t kcol = k0 + q * 8;
        const bool live = src != nullptr && kcol < shape.K;
        ptx::cp_async_16(xs + r * 128 + ((q ^ (r & 7)) << 4),
                         live ? static_cast<const void*>(src + kcol) : static_cast<const void*>(tab.in[0]),
                         live ? 16u : 0u);
      }
      ptx::cp_async_arrive_noinc(&full[s]);
    }
    ptx::cp_async_wait_all();
  } else {
    // ---- epilogue warps 4..7: TMEM lane quarter q -------------------------------------
    const int q = warp & 3;
    const int et = tid - 128;
    int j = 0;
    for (int64_t u = u0; u < u1; ++j) {
      const int64_t t = u / nkb;
      const int64_t seg_end = min(u1, (t + 1) * nkb);
      u = seg_end;
      const int a = j & 1;
      const bool ok = ptx::mbar_wait_sleep(&acc_full[a], (j >> 1) & 1, err, kSkAccFull, kTimeoutNs, 256);
      __syncwarp();
      ptx::tc_fence_after();
      float v[BN];
      if (ok) {
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r32[32];
          ptx::tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(q * 32) << 16) + a * BN + c0, r32);
          ptx::tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[c0 + e] = __uint_as_float(r32[e]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < BN; ++e) v[e] = 0.f;
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&acc_empty[a]);
      const int64_t n = t * kBlockW + q * 32 + lane;
      const int c_first = cta_of_unit(t * nkb, U, P);
      const int c_last = cta_of_unit(t * nkb + nkb - 1, U, P);
      const int nparts = c_last - c_first + 1;
      bool write = true;
      if (nparts > 1) {
        const int pi = c - c_first;
        float* wsp = sk.ws + ((t * sk.max_parts + pi) * BN) * kBlockW;
#pragma unroll
        for (int r = 0; r < BN; ++r)
          if (r < rows) __stcg(wsp + r * kBlockW + q * 32 + lane, v[r]);
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"n"(kEpi) : "memory");
        if (et == 0) *flag = atomicAdd(&sk.counters[t], 1);
        asm volatile("bar.sync 1, %0;" ::"n"(kEpi) : "memory");
        const int old = *flag;
        asm volatile("bar.sync 1, %0;" ::"n"(kEpi) : "memory");
        write = old == nparts - 1;
        if (write) {
          __threadfence();
          float acc[BN];
#pragma unroll
          for (int r = 0; r < BN; ++r) acc[r] = 0.f;
          for (int pp = 0; pp < nparts; ++pp) {
            if (pp == pi) {
#pragma unroll
              for (int r = 0; r < BN; ++r) acc[r] += v[r];
            } else {
              const float* src = sk.ws + ((t * sk.max_parts + pp) * BN) * kBlockW + q * 32 + lane;
#pragma unroll
              for (int r = 0; r < BN; ++r)
                if (r < rows) acc[r] += __ldcg(src + r * kBlockW);
            }
          }
#pragma unroll
          for (int r = 0; r < BN; ++r) v[r] = acc[r];
          if (et == 0) sk.counters[t] = 0;
        }
      }
      if (write && n < shape.N) {
        const float b = shape.bias ? __bfloat162float(shape.bias[n]) : 0.f;
#pragma unroll
        for (int r = 0; r < BN; ++r)
          if (r < rows) row_out[r][n] = __float2bfloat16_rn(v[r] + b);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

struct Workspace {
  float* ws = nullptr;
  int* counters = nullptr;
  size_t ws_floats = 0;
  int counters_n = 0;
};
Workspace g_ws[16];  // per device ordinal
std::mutex g_ws_mu;

int sm_count_sk() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int g_sk_ctas_per_sm = 1;
int g_sk_ctas_override = 0;

template <int BN, int STAGES>
int launch_sk(const SlotTable& tab, const RoundShape& shape, const CUtensorMap& map,
              cudaStream_t stream, Workspace& w, int per_sm) {
  using Cfg = SkCfg<BN, STAGES>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(slot_round_sk_kernel<BN, STAGES>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  });
  if (attr_err != cudaSuccess)
    return set_error(SWL_ERR_CUDA, "stream-K round: smem attribute: %s", cudaGetErrorString(attr_err));
  const int n_tiles = static_cast<int>((shape.N + kBlockW - 1) / kBlockW);
  const int nkb = static_cast<int>((shape.K + kBlockK - 1) / kBlockK);
  SkParams sk;
  sk.nkb = nkb;
  sk.units = static_cast<int64_t>(n_tiles) * nkb;
  sk.ctas = static_cast<int>(std::min<int64_t>(static_cast<int64_t>(sm_count_sk()) * per_sm, sk.units));
  if (g_sk_ctas_override > 0) sk.ctas = static_cast<int>(std::min<int64_t>(g_sk_ctas_override, sk.units));
  const int64_t per = sk.units / sk.ctas;  // >= 1
  sk.max_parts = static_cast<int>((nkb + per - 1) / per) + 2;
  const size_t need = static_cast<size_t>(n_tiles) * sk.max_parts * BN * kBlockW;
  if (need > w.ws_floats || n_tiles > w.counters_n)
    return set_error(SWL_ERR_ARG, "stream-K round: workspace too small (%zu floats, %d tiles)", need, n_tiles);
  sk.ws = w.ws;
  sk.counters = w.counters;
  slot_round_sk_kernel<BN, STAGES><<<sk.ctas, kThreads, Cfg::kSmem, stream>>>(map, tab, shape, sk);
  SWL_CUDA_TRY(cudaGetLastError());
  return SWL_OK;
}

}  // namespace

// Allocates (once per device) the stream-K workspace: fp32 partial tiles and
// zeroed per-tile arrival counters. Call outside stream capture.
int ensure_streamk_workspace() {
  int dev = 0;
  SWL_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 16) return set_error(SWL_ERR_ARG, "stream-K: device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_ws_mu);
  Workspace& w = g_ws[dev];
  if (w.ws) return SWL_OK;
  const size_t floats = static_cast<size_t>(32) << 20;  // 128 MB
  const int counters = 1 << 16;
  SWL_CUDA_TRY(cudaMalloc(&w.ws, floats * sizeof(float)));
  SWL_CUDA_TRY(cudaMalloc(&w.counters, counters * sizeof(int)));
  SWL_CUDA_TRY(cudaMemset(w.counters, 0, counters * sizeof(int)));
  SWL_CUDA_TRY(cudaDeviceSynchronize());
  w.ws_floats = floats;
  w.counters_n = counters;
  return SWL_OK;
}

// The split-K workspace of the tensor-core round shares the stream-K buffer
// (the two never run at once: both are launched in stream order) and uses
// the upper half of its counters.
int splitk_workspace(SplitWs* out, size_t floats, int tiles) {
  int dev = 0;
  SWL_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 16) return set_error(SWL_ERR_ARG, "split-K: device ordinal out of range");
  Workspace& w = g_ws[dev];
  if (!w.ws) return set_error(SWL_ERR_STATE, "split-K: workspace not allocated");
  const int half = w.counters_n / 2;
  if (floats > w.ws_floats || tiles > half) return set_error(SWL_ERR_STATE, "split-K: workspace too small");
  out->part = w.ws;
  out->count = w.counters + half;
  return SWL_OK;
}

// Resets the arrival counters (after a round reported a bounded-wait timeout,
// a tile may have been left half-counted). Synchronous.
int reset_streamk_counters() {
  int dev = 0;
  SWL_CUDA_TRY(cudaGetDevice(&dev));
  Workspace& w = g_ws[dev];
  if (w.counters) SWL_CUDA_TRY(cudaMemset(w.counters, 0, w.counters_n * sizeof(int)));
  return SWL_OK;
}

int launch_slot_round_streamk(const SlotTable& tab, const RoundShape& shape, const CUtensorMap& map,
                              cudaStream_t stream) {
  int dev = 0;
  SWL_CUDA_TRY(cudaGetDevice(&dev));
  Workspace& w = g_ws[dev];
  if (!w.ws) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(stream, &cs);
    if (cs != cudaStreamCaptureStatusNone)
      return set_error(SWL_ERR_STATE, "stream-K round: workspace not allocated before capture");
    SWL_TRY(ensure_streamk_workspace());
  }
  const int m = tab.total_rows;
  const int per_sm = g_sk_ctas_per_sm;
  if (m <= 32) {
    if (per_sm >= 2) return launch_sk<32, 5>(tab, shape, map, stream, w, 2);
    return launch_sk<32, 9>(tab, shape, map, stream, w, 1);
  }
  if (m <= 64) {
    if (per_sm >= 2) return launch_sk<64, 4>(tab, shape, map, stream, w, 2);
    return launch_sk<64, 8>(tab, shape, map, stream, w, 1);
  }
  return set_error(SWL_ERR_ARG, "stream-K round: at most 64 token rows");
}

int set_streamk_ctas_per_sm(int n) {
  if (n < 1 || n > 2) return set_error(SWL_ERR_ARG, "stream-K: 1 or 2 CTAs per SM");
  g_sk_ctas_per_sm = n;
  return SWL_OK;
}

int set_streamk_ctas(int n) {
  g_sk_ctas_override = n > 0 ? n : 0;
  return SWL_OK;
}

int read_and_clear_sk_error(unsigned int* code) {
  unsigned int v = 0, zero = 0;
  SWL_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_sk_error_word, sizeof(v)));
  if (v) {
    SWL_CUDA_TRY(cudaMemcpyToSymbol(g_sk_error_word, &zero, sizeof(zero)));
    SWL_TRY(reset_streamk_counters());
  }
  *code = v;
  return SWL_OK;
}

}  // namespace swl
