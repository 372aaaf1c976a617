// Slot-round kernels: gather -> frozen-base GEMM -> scatter in one launch.
//
// Product path (kAlgoTensorCore), one CTA of 4 warps per (128 weight rows,
// token chunk, K split):
//   warp 0      TMA producer: streams 128x64 bf16 tiles of W (HBM, evict-first)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2-3   gather producers: cp.async the chunk's token rows straight from
//               each slot's input buffer into the 128B-swizzled B operand
//   all warps   epilogue: TMEM -> shared memory (f32), reduce the K splits of
//               the cluster through distributed shared memory, add bias, write
//               bf16 rows directly into each slot's output buffer.
// The MMA is "swap-AB": the 128 weight rows are the MMA M dimension and the
// (few) decode tokens the N dimension, so a decode round of 28 tokens is a
// 128 x 32 x 64 MMA stream whose speed is set by the W stream from HBM.
//
// Reference behaviour replaced: ext_aggregator.cpp:470-626
// (execute_batched_gemm_slots: torch::cat gather, matmul_out, per-slot copy_).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.h"
#include "launch.h"
#include "ptx.cuh"
#include "slot_round.h"

namespace swl {

__device__ unsigned int g_round_error_word = 0;

namespace {

constexpr int kBlockW = 128;                          // weight rows per CTA (MMA M)
constexpr int kBlockK = 64;                           // K elements per stage (128 bytes)
constexpr int kWStageBytes = kBlockW * kBlockK * 2;   // 16 KB
constexpr int kThreads = 128;
constexpr int kGatherThreads = 64;                    // warps 2-3
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;    // 2 s of device time

enum ErrCode : unsigned int {
  kErrWaitEmptyW = 1,
  kErrWaitFull = 2,
  kErrWaitEmptyX = 3,
  kErrWaitAcc = 4,
  kErrWaitPeerStart = 5,  // the peer GPU did not start the same sharded round
  kErrWaitPeerDone = 6,   // the peer GPU's half of a sharded round did not arrive
};

// Extra argument of a plain round (nothing).
struct NoEpi {
  int unused;
};

// Tile of BN token rows and a ring of STAGES K-blocks (each a 128 x 64 W
// tile and a BN x 64 token tile).
template <int BN, int STAGES>
struct TcCfg {
  static constexpr int kStages = STAGES;
  static constexpr int kXStageBytes = BN * 128;
  static constexpr int kPipeBytes = kStages * (kWStageBytes + kXStageBytes);
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kPipeBytes + 256 + BN * 24;
  // per-row tables of the fused QKV/RoPE epilogue: slot, position, page, t[32]
  static constexpr int kRopeBytes = BN * (3 * 4 + 32 * 4);
  // TMEM columns are allocated in powers of two, at least 32
  static constexpr int kTmemCols = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "MMA N of a 128-row tile: 16..256 in steps of 16");
  static_assert(BN * kBlockW * 4 <= kPipeBytes, "epilogue tile must fit in pipeline smem");
};

// Launch-time flags of the tensor-core round.
constexpr int kFlagGatherSpin = 1;    // gather warps poll the free-stage barrier without sleeping
constexpr int kFlagGlobalSplit = 2;   // split-K reduced through global memory instead of across a cluster
constexpr int kFlagPrefetchRest = 4;  // before the dependency wait, prefetch the rest of the CTA's W tiles into L2
constexpr int kFlagStagedX = 8;       // token tiles by TMA from a packed staging copy (set per launch)
constexpr int kPrefetchRestMax = 12;  // at most this many K-blocks per CTA (the small rounds)

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// t . B_row over `rank` (a multiple of 8), in the order of the RoPE
// epilogue's dot product (8 values per 16-byte load, pairs in order).
__device__ __forceinline__ float lora_row_dot(const float* t, const __nv_bfloat16* row, int rank) {
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

__device__ __forceinline__ void store_bf16x4(__nv_bfloat16* dst, const float (&v)[4]) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
  uint2 packed;
  packed.x = *reinterpret_cast<const uint32_t*>(&lo);
  packed.y = *reinterpret_cast<const uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(dst) = packed;
}

// Slot of global row `gr`: the largest s with row_start[s] <= gr.
__device__ __forceinline__ int slot_of_row(const SlotTable& tab, int gr) {
  int lo = 0, hi = tab.nslots - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (tab.row_start[mid] <= gr) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int BN, int STAGES, class Ex>
__global__ void __launch_bounds__(kThreads, 1)
    slot_round_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                         const __grid_constant__ SlotTable tab, const RoundShape shape,
                         int splits, int flags, const SplitWs sws, const __grid_constant__ Ex ex) {
  constexpr bool kShard = std::is_same<Ex, ShardArgs>::value;
  constexpr bool kRope = std::is_same<Ex, QkvRopeEpi>::value;
  using Cfg = TcCfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* w_st = smem;
  uint8_t* x_st = smem + STAGES * kWStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(x_st + STAGES * Cfg::kXStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accf + 1);
  const __nv_bfloat16** row_in = reinterpret_cast<const __nv_bfloat16**>(tmem_holder + 2);
  __nv_bfloat16** row_out = reinterpret_cast<__nv_bfloat16**>(tmem_holder + 2 + 2 * BN);
  __nv_bfloat16** row_peer = reinterpret_cast<__nv_bfloat16**>(tmem_holder + 2 + 4 * BN);
  int* rope_slot = reinterpret_cast<int*>(tmem_holder + 2 + 6 * BN);  // fused QKV/RoPE tables
  int* rope_pos = rope_slot + BN;
  int* rope_page = rope_pos + BN;
  float* rope_t = reinterpret_cast<float*>(rope_page + BN);  // [BN][32]
  __shared__ int shard_ok;
  __shared__ int split_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // split-K across a cluster (DSMEM reduction) or through global memory
  const bool gsplit = splits > 1 && sws.part != nullptr;
  const bool csplit = splits > 1 && !gsplit;
  const int rank = gsplit ? static_cast<int>(blockIdx.x) % splits
                          : (splits > 1 ? static_cast<int>(ptx::cluster_rank()) : 0);
  const int n0 = (blockIdx.x / splits) * kBlockW;
  const int chunk_row0 = blockIdx.y * BN;
  const int chunk_rows = min(BN, tab.total_rows - chunk_row0);
  const int nkb = static_cast<int>((shape.K + kBlockK - 1) / kBlockK);
  const int kb_begin = static_cast<int>(static_cast<int64_t>(rank) * nkb / splits);
  const int kb_end = static_cast<int>(static_cast<int64_t>(rank + 1) * nkb / splits);
  const int nk = kb_end - kb_begin;
  unsigned int* err = &g_round_error_word;

  // Row table for this token chunk: where each gathered row comes from and goes to.
  for (int r = tid; r < BN; r += kThreads) {
    const __nv_bfloat16* pin = nullptr;
    __nv_bfloat16* pout = nullptr;
    __nv_bfloat16* ppeer = nullptr;
    if (r < chunk_rows) {
      int gr = chunk_row0 + r;
      int s = slot_of_row(tab, gr);
      int64_t local = gr - tab.row_start[s];
      pin = tab.in[s] + local * shape.in_stride;
      pout = tab.out[s] + local * shape.out_stride;
      if constexpr (kShard) {
        pout += ex.col0;
        ppeer = ex.peer_out[s] + local * shape.out_stride + ex.col0;
      }
      if constexpr (kRope) {
        // this row's position and cache page, which the launch ahead does
        // not write (read before the dependency wait)
        const int pos = *ex.seqlen[s] + static_cast<int>(local);
        rope_slot[r] = s;
        rope_pos[r] = pos;
        rope_page[r] = (n0 >= ex.hq * 128) ? ex.block_table[s][pos / ex.page] : 0;
        if (ex.B[s]) ptx::prefetch_l2_bulk(ex.B[s] + static_cast<int64_t>(n0) * ex.rank, 128u * ex.rank * 2u);
      }
    }
    row_in[r] = pin;
    row_out[r] = pout;
    if constexpr (kShard) row_peer[r] = ppeer;
  }

  // Staged tokens: the chunk's token rows were packed into one [M, K] copy
  // by the launch just ahead, and the TMA warp loads each token tile with the
  // weight tile (the gather warps idle); otherwise the gather warps copy each
  // row from its slot buffer.
  const bool staged = (flags & kFlagStagedX) != 0;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], staged ? 1 : 1 + kGatherThreads);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(accf, 1);
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&wmap);
    if (staged) ptx::prefetch_tmap(&xmap);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_holder, Cfg::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // The weight does not depend on earlier kernels: fill the whole ring before
  // waiting for the kernel ahead in the stream (whose outputs are our inputs).
  const int npre = min(nk, STAGES);
  if (warp == 0 && lane == 0) {
    const uint64_t pol = ptx::policy_evict_first();
    for (int i = 0; i < npre; ++i) {
      // staged: the stage completes only with the token tile's arrival below
      if (staged) ptx::mbar_expect_tx(&full[i], kWStageBytes);
      else ptx::mbar_arrive_expect_tx(&full[i], kWStageBytes);
      ptx::tma_load_2d(w_st + i * kWStageBytes, &wmap, &full[i], (kb_begin + i) * kBlockK, n0, pol);
    }
    // the tiles that do not fit in the ring move into L2 now, while the
    // kernel ahead still runs (small rounds only: the bytes stay in L2)
    if ((flags & kFlagPrefetchRest) && nk - npre <= kPrefetchRestMax)
      for (int i = npre; i < nk; ++i) ptx::tma_prefetch_2d(&wmap, (kb_begin + i) * kBlockK, n0);
  }
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  // Sharded round: this is round `epoch` on this GPU (the count of completed
  // ones is only advanced by this launch's last CTA, after every CTA has read
  // it). Having passed the dependency wait, this GPU has finished reading the
  // previous round's outputs, which CTA 0 tells the peer.
  unsigned int epoch = 0;
  if constexpr (kShard) {
    epoch = *reinterpret_cast<volatile unsigned int*>(ex.sync + kSyncEpoch) + 1;
    if (blockIdx.x == 0 && blockIdx.y == 0 && tid == 0) ptx::st_release_sys(ex.peer_sync + kSyncStart, epoch);
  }

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = ptx::policy_evict_first();
      const uint64_t pol_x = ptx::policy_evict_last();  // every CTA of the chunk reads the token tiles
      if (staged)
        for (int i = 0; i < npre; ++i) {
          ptx::mbar_arrive_expect_tx(&full[i], Cfg::kXStageBytes);
          ptx::tma_load_2d(x_st + i * Cfg::kXStageBytes, &xmap, &full[i], (kb_begin + i) * kBlockK, chunk_row0,
                           pol_x);
        }
      for (int i = npre; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!ptx::mbar_wait(&empty[s], ph ^ 1, err, kErrWaitEmptyW, kWaitTimeoutNs)) break;
        ptx::mbar_arrive_expect_tx(&full[s], kWStageBytes + (staged ? Cfg::kXStageBytes : 0));
        ptx::tma_load_2d(w_st + s * kWStageBytes, &wmap, &full[s], (kb_begin + i) * kBlockK, n0,
                         pol);
        if (staged)
          ptx::tma_load_2d(x_st + s * Cfg::kXStageBytes, &xmap, &full[s], (kb_begin + i) * kBlockK, chunk_row0,
                           pol_x);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_bf16_f32(kBlockW, BN);
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!ptx::mbar_wait(&full[s], ph, err, kErrWaitFull, kWaitTimeoutNs)) break;
        ptx::tc_fence_after();
        // (no proxy fence: cp.async completion is tracked by the mbarrier, as in
        // CUTLASS's cp.async-fed UMMA mainloop)
        const uint32_t wa = ptx::smem_addr(w_st + s * kWStageBytes);
        const uint32_t xa = ptx::smem_addr(x_st + s * Cfg::kXStageBytes);
#pragma unroll
        for (int kk = 0; kk < kBlockK / 16; ++kk) {
          ptx::mma_bf16_ss(tmem, ptx::sw128_kmajor_desc(wa + kk * 32),
                           ptx::sw128_kmajor_desc(xa + kk * 32), idesc,
                           (i > 0 || kk > 0) ? 1u : 0u);
        }
        ptx::tc_commit(&empty[s]);
      }
      ptx::tc_commit(accf);
    }
  } else {
    // Gather producers. Row r of the B tile holds token row r of the chunk;
    // its eight 16-byte pieces are stored XOR-swizzled by (r & 7) as the
    // 128B-swizzle canonical layout requires. Rows past the chunk are zeros.
    const int t = tid - 2 * 32;
    for (int i = 0; i < (staged ? 0 : nk); ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (i / STAGES) & 1;
      const bool freed = (flags & kFlagGatherSpin)
                             ? ptx::mbar_wait(&empty[s], ph ^ 1, err, kErrWaitEmptyX, kWaitTimeoutNs)
                             : ptx::mbar_wait_sleep(&empty[s], ph ^ 1, err, kErrWaitEmptyX, kWaitTimeoutNs, 64);
      if (!freed) break;
      const int64_t k0 = static_cast<int64_t>(kb_begin + i) * kBlockK;
      const uint32_t xs = ptx::smem_addr(x_st + s * Cfg::kXStageBytes);
      for (int c = t; c < BN * 8; c += kGatherThreads) {
        const int r = c >> 3, j = c & 7;
        const __nv_bfloat16* src = row_in[r];
        const int64_t kcol = k0 + j * 8;
        const bool live = src != nullptr && kcol < shape.K;
        ptx::cp_async_16(xs + r * 128 + ((j ^ (r & 7)) << 4),
                         live ? static_cast<const void*>(src + kcol) : static_cast<const void*>(tab.in[0]),
                         live ? 16u : 0u);
      }
      // The arrival lands when this thread's copies have; no blocking here.
      ptx::cp_async_arrive_noinc(&full[s]);
    }
    if constexpr (kRope) {
      // While the MMA finishes: the LoRA intermediate of this tile's block
      // (q, k or v) per row, t = bf16(sum of the shrink partials), which
      // the epilogue ahead of this round writes (so read after the wait).
      const int blk = n0 < ex.hq * 128 ? 0 : (n0 < (ex.hq + ex.hkv) * 128 ? 1 : 2);
      const int count = chunk_rows * ex.rank;
      if (ex.splits_in <= 8) {
        // up to 8 splits: every load of 4 values is in flight at once
#pragma unroll 4
        for (int e = t; e < count; e += kGatherThreads) {
          const int r = e / ex.rank, j = e - r * ex.rank;
          const float* src = ex.ws_in + static_cast<int64_t>(chunk_row0 + r) * ex.splits_in * 3 * ex.rank +
                             blk * ex.rank + j;
          float v[8];
#pragma unroll
          for (int sp = 0; sp < 8; ++sp) v[sp] = sp < ex.splits_in ? src[sp * 3 * ex.rank] : 0.f;
          float a = 0.f;
#pragma unroll
          for (int sp = 0; sp < 8; ++sp)
            if (sp < ex.splits_in) a += v[sp];
          rope_t[r * 32 + j] = __bfloat162float(__float2bfloat16_rn(a));
        }
      } else {
        for (int e = t; e < count; e += kGatherThreads) {
          const int r = e / ex.rank, j = e - r * ex.rank;
          const float* src = ex.ws_in + static_cast<int64_t>(chunk_row0 + r) * ex.splits_in * 3 * ex.rank +
                             blk * ex.rank + j;
          float a = 0.f;
          for (int sp = 0; sp < ex.splits_in; ++sp) a += src[static_cast<int64_t>(sp) * 3 * ex.rank];
          rope_t[r * 32 + j] = __bfloat162float(__float2bfloat16_rn(a));
        }
      }
    }
    ptx::cp_async_wait_all();  // never leave copies in flight into freed smem
  }
  __syncwarp();

  // ---- epilogue ------------------------------------------------------------
  const bool acc_ok = ptx::mbar_wait_sleep(accf, 0, err, kErrWaitAcc, kWaitTimeoutNs, 128);
  __syncwarp();
  ptx::tc_fence_after();
  float* P = reinterpret_cast<float*>(smem);  // [BN tokens][128 weight rows] f32
  if (acc_ok && nk > 0) {
    const int q = warp & 3;  // TMEM lane quarter this warp may read
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t v[32];
      ptx::tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, v);
      ptx::tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) P[(c0 + j) * kBlockW + q * 32 + lane] = __uint_as_float(v[j]);
    }
  } else {
    for (int e = tid; e < BN * kBlockW; e += kThreads) P[e] = 0.f;
  }
  ptx::tc_fence_before();
  if (csplit) ptx::cluster_sync();
  else __syncthreads();

  // Sharded round: the peer may still read its previous round's outputs
  // until it has started this round; only then do our stores go there.
  bool to_peer = false;
  if constexpr (kShard) {
    if (tid == 0) shard_ok = ptx::wait_epoch_sys(ex.sync + kSyncStart, epoch, err, kErrWaitPeerStart, kWaitTimeoutNs);
    __syncthreads();
    to_peer = shard_ok != 0;
  }

  const uint32_t pbase = ptx::smem_addr(P);
  // Split-K through global memory: this split's partial tile goes to the
  // workspace; only the last split of the tile to arrive goes on, and it
  // reads every split's partial (including its own) back from L2.
  const int tile_id = static_cast<int>(blockIdx.y) * static_cast<int>(gridDim.x / splits) +
                      static_cast<int>(blockIdx.x) / splits;
  const float* gpart = gsplit ? sws.part + static_cast<int64_t>(tile_id) * splits * (BN * kBlockW) : nullptr;
  bool emit = true;
  if (gsplit) {
    float4* mine = reinterpret_cast<float4*>(sws.part + (static_cast<int64_t>(tile_id) * splits + rank) *
                                                            (BN * kBlockW));
    const float4* src = reinterpret_cast<const float4*>(P);
    for (int e = tid; e < chunk_rows * (kBlockW / 4); e += kThreads) mine[e] = src[e];
    __threadfence();
    __syncthreads();
    if (tid == 0) split_last = atomicAdd(sws.count + tile_id, 1) == splits - 1;
    __syncthreads();
    emit = split_last != 0;
    __threadfence();
  }
  // the K-split sum of the 4 outputs at (row r, column c) of the tile: every
  // split's partial is loaded first (up to 8 loads in flight, one round trip
  // to the peers or L2), then summed in split order
  auto reduce4 = [&](int r, int c) -> float4 {
    const uint32_t off = static_cast<uint32_t>((r * kBlockW + c) * 4);
    if (!gsplit && splits == 1) return *reinterpret_cast<const float4*>(P + r * kBlockW + c);
    float4 v[8];
#pragma unroll
    for (int p = 0; p < 8; ++p)
      if (p < splits)
        v[p] = gsplit ? __ldcg(reinterpret_cast<const float4*>(gpart + static_cast<int64_t>(p) * (BN * kBlockW) +
                                                                r * kBlockW + c))
                      : ptx::ld_cluster_f4(ptx::map_peer(pbase + off, p));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < 8; ++p)
      if (p < splits) {
        acc.x += v[p].x;
        acc.y += v[p].y;
        acc.z += v[p].z;
        acc.w += v[p].w;
      }
    return acc;
  };
  if constexpr (kRope) {
    // Fused RoPE epilogue. Work item = (row, 4 columns c..c+3 and their NeoX
    // partners c+64..c+67); the cluster's CTAs take equal shares.
    const int items = chunk_rows * 16;
    const int i_begin = static_cast<int>(static_cast<int64_t>(rank) * items / splits);
    const int i_end = static_cast<int>(static_cast<int64_t>(rank + 1) * items / splits);
    const int head = n0 / 128;
    const int blk = head < ex.hq ? 0 : (head < ex.hq + ex.hkv ? 1 : 2);
    for (int it = i_begin + tid; it < i_end; it += kThreads) {
      const int r = it >> 4, c = (it & 15) * 4;
      const float4 a = reduce4(r, c), b = reduce4(r, c + 64);
      float x1[4] = {bf16_round(a.x), bf16_round(a.y), bf16_round(a.z), bf16_round(a.w)};
      float x2[4] = {bf16_round(b.x), bf16_round(b.y), bf16_round(b.z), bf16_round(b.w)};
      const int s = rope_slot[r];
      const __nv_bfloat16* B = ex.B[s];
      if (B) {
        const float* t = rope_t + r * 32;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          x1[j] = bf16_round(x1[j] + bf16_round(lora_row_dot(t, B + static_cast<int64_t>(n0 + c + j) * ex.rank, ex.rank)));
          x2[j] = bf16_round(x2[j] + bf16_round(lora_row_dot(t, B + static_cast<int64_t>(n0 + c + 64 + j) * ex.rank, ex.rank)));
        }
      }
      const int gr = chunk_row0 + r;
      const int pos = rope_pos[r];
      const int64_t cache_row = (static_cast<int64_t>(rope_page[r]) * ex.page + pos % ex.page) * ex.hkv;
      if (blk == 2) {
        __nv_bfloat16* dst = ex.v_cache[s] + (cache_row + (head - ex.hq - ex.hkv)) * 128;
        store_bf16x4(dst + c, x1);
        store_bf16x4(dst + c + 64, x2);
      } else {
        const __nv_bfloat16* cs = ex.cos_sin + static_cast<int64_t>(pos) * 128;
        float o1[4], o2[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float cv = __bfloat162float(cs[c + j]), sv = __bfloat162float(cs[64 + c + j]);
          o1[j] = bf16_round(bf16_round(x1[j] * cv) - bf16_round(x2[j] * sv));
          o2[j] = bf16_round(bf16_round(x2[j] * cv) + bf16_round(x1[j] * sv));
        }
        __nv_bfloat16* dst = blk == 0 ? ex.q_rot + (static_cast<int64_t>(gr) * ex.hq + head) * 128
                                      : ex.k_cache[s] + (cache_row + (head - ex.hq)) * 128;
        store_bf16x4(dst + c, o1);
        store_bf16x4(dst + c + 64, o2);
      }
    }
  }
  // Each CTA of the cluster reduces an equal share of the tile's 4-float
  // groups; through global memory the last split to arrive reduces them all.
  const int groups = (kRope || !emit) ? 0 : chunk_rows * (kBlockW / 4);
  const int g_begin = csplit ? static_cast<int>(static_cast<int64_t>(rank) * groups / splits) : 0;
  const int g_end = csplit ? static_cast<int>(static_cast<int64_t>(rank + 1) * groups / splits) : groups;
  for (int g = g_begin + tid; g < g_end; g += kThreads) {
    const int r = g >> 5;
    const int c = (g & 31) * 4;
    const int64_t n = n0 + c;
    if (n >= shape.N) continue;
    float4 acc = reduce4(r, c);
    if (shape.bias) {
      acc.x += __bfloat162float(shape.bias[n]);
      acc.y += __bfloat162float(shape.bias[n + 1]);
      acc.z += __bfloat162float(shape.bias[n + 2]);
      acc.w += __bfloat162float(shape.bias[n + 3]);
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(row_out[r] + n) = packed;
    if (kShard && to_peer) *reinterpret_cast<uint2*>(row_peer[r] + n) = packed;
  }

  // The tile's arrival counter starts at zero for the next launch (which, in
  // stream order, reaches it only after this launch has completed).
  if (gsplit && emit && tid == 0) sws.count[tile_id] = 0;
  // Done reading the peers' P; they may still read ours, so the CTA waits
  // for the whole cluster before it exits (TMEM was last read before the
  // barrier above, so it is released in between). Every value read from a
  // peer went into a store above, so those reads are complete: the arrive
  // needs no release ordering (which would wait for the output stores).
  if (csplit) ptx::cluster_arrive_relaxed();
  else __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (csplit) ptx::cluster_wait();

  if constexpr (kShard) {
    // Every thread's peer stores are visible system-wide before its CTA
    // arrives; the last CTA to arrive publishes the round to the peer and
    // waits for the peer's half to have landed here.
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
      const unsigned int total = gridDim.x * gridDim.y;
      if (atomicAdd(ex.sync + kSyncArrive, 1u) == total - 1) {
        ex.sync[kSyncArrive] = 0;
        ex.sync[kSyncEpoch] = epoch;
        __threadfence_system();
        ptx::st_release_sys(ex.peer_sync + kSyncDone, epoch);
        ptx::wait_epoch_sys(ex.sync + kSyncDone, epoch, err, kErrWaitPeerDone, kWaitTimeoutNs);
      }
    }
  }
}

// Plain CUDA-core round: one warp per (output feature, token row). Slow but
// independent of the tensor-core machinery; used to cross-check on device.
__global__ void slot_round_simt_kernel(const __nv_bfloat16* __restrict__ W,
                                       const __grid_constant__ SlotTable tab,
                                       const RoundShape shape) {
  const int64_t n = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int gr = blockIdx.y;
  if (n >= shape.N || gr >= tab.total_rows) return;
  const int s = slot_of_row(tab, gr);
  const int64_t local = gr - tab.row_start[s];
  const __nv_bfloat16* x = tab.in[s] + local * shape.in_stride;
  const __nv_bfloat16* w = W + n * shape.K;
  float acc = 0.f;
  for (int64_t k = lane; k < shape.K; k += 32)
    acc += __bfloat162float(x[k]) * __bfloat162float(w[k]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    if (shape.bias) acc += __bfloat162float(shape.bias[n]);
    tab.out[s][local * shape.out_stride + n] = __float2bfloat16_rn(acc);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Tuning of the tensor-core round (swl_round_tune): the (tile rows, stages)
// used for each class of round row counts, and the launch flags.
constexpr int kRowClasses = 5;                  // <= 32, <= 64, <= 96, <= 128, more
constexpr int kClassRows[kRowClasses] = {32, 64, 96, 128, 1 << 30};
// Defaults from sweeps on B200 (CUDA graphs of launches over weights beyond
// L2): more CTA pipelines per SM beat deeper rings at the same bytes in flight.
// Per class (32-row decode: 4 stages at 2 CTAs/SM; 96 and 128 rows: 3
// stages at 2 CTAs/SM instead of 6 stages at one, M = 88 Gate+Up 103.7 ->
// 53.0 us; above 128 rows 256-row chunks of 3 stages).
constexpr int kDefaultTile[kRowClasses][2] = {{32, 4}, {64, 4}, {96, 3}, {128, 3}, {256, 3}};
std::atomic<int> g_tile_bn[kRowClasses] = {{0}, {0}, {0}, {0}, {0}};
std::atomic<int> g_tile_stages[kRowClasses] = {{0}, {0}, {0}, {0}, {0}};
// Token tiles staged (packed copy, loaded by TMA) per class by default when
// the weight has at least this many elements (-1: never): measured on B200,
// staging pays above 128 rows for every round (Gate+Up at M = 200: 188 -> 90
// us; Down at M = 512: 156 -> 73 us), and at 65..128 rows for the large
// weights only (Gate+Up at M = 88: 56 -> 51 us; O at M = 88: 15.3 -> 17.3
// us, the packing launch costing more than it saves).
constexpr int64_t kDefaultStagedMinElems[kRowClasses] = {-1, -1, int64_t{1} << 26, int64_t{1} << 25, 0};
std::atomic<int> g_tile_staged[kRowClasses] = {{-1}, {-1}, {-1}, {-1}, {-1}};
std::atomic<int> g_round_flags{0};

// ---- staged token rows ------------------------------------------------------------------
// A launch ahead of the round packs the round's token rows into one [M, K]
// bf16 buffer per device, so the round loads its token tiles by TMA (the same
// 128B-swizzled layout the gather warps write) instead of by per-row copies.
struct Staging {
  void* p = nullptr;
  size_t bytes = 0;
};
Staging g_stage[16];
std::mutex g_stage_mu;
constexpr size_t kStageMaxBytes = size_t{256} << 20;

// The device's staging buffer with room for `bytes`, grown outside stream
// captures (growing waits for the device); nullptr when it cannot be had.
void* staging_buffer(size_t bytes, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16 || bytes > kStageMaxBytes) return nullptr;
  std::lock_guard<std::mutex> lk(g_stage_mu);
  Staging& st = g_stage[dev];
  if (st.bytes >= bytes) return st.p;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusActive;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return nullptr;
  const size_t want = std::max(bytes, size_t{16} << 20);
  if (st.p) {
    if (cudaDeviceSynchronize() != cudaSuccess) return nullptr;
    cudaFree(st.p);
    st.p = nullptr;
    st.bytes = 0;
  }
  if (cudaMalloc(&st.p, want) != cudaSuccess) {
    cudaGetLastError();
    st.p = nullptr;
    return nullptr;
  }
  st.bytes = want;
  return st.p;
}

// Row gr of the round -> row gr of the staging copy (16-byte vectors).
__global__ void stage_rows_kernel(const __grid_constant__ SlotTable tab, int64_t in_stride, int64_t K,
                                  __nv_bfloat16* __restrict__ out) {
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int gr = blockIdx.x;
  const int s = slot_of_row(tab, gr);
  const int64_t local = gr - tab.row_start[s];
  const uint4* src = reinterpret_cast<const uint4*>(tab.in[s] + local * in_stride);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(gr) * K);
  for (int64_t k = threadIdx.x; k < K / 8; k += blockDim.x) dst[k] = src[k];
}

int row_class(int m) {
  int c = 0;
  while (c < kRowClasses - 1 && m > kClassRows[c]) ++c;
  return c;
}

// The packed token rows [rows, K] bf16, box 64 x box_rows, 128B swizzle:
// rows past `rows` read as zeros.
int encode_token_tmap(CUtensorMap* map, const void* X, int64_t rows, int64_t K, int box_rows) {
  auto enc = tmap_encoder();
  if (!enc) return set_error(SWL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlockK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(X), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(SWL_ERR_CUDA, "token tensor map: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SWL_OK;
}

template <int BN, int STAGES, class Ex>
int launch_tc(const SlotTable& tab, const RoundShape& shape, const CUtensorMap& map, int splits,
              const Ex& ex, cudaStream_t stream, const void* staged = nullptr) {
  using Cfg = TcCfg<BN, STAGES>;
  constexpr bool kShard = std::is_same<Ex, ShardArgs>::value;
  constexpr int smem_bytes = Cfg::kSmemBytes + (std::is_same<Ex, QkvRopeEpi>::value ? Cfg::kRopeBytes : 0);
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(slot_round_tc_kernel<BN, STAGES, Ex>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  });
  if (attr_err != cudaSuccess)
    return set_error(SWL_ERR_CUDA, "slot round: smem attribute: %s", cudaGetErrorString(attr_err));

  const int n_tiles = static_cast<int>((shape.N + kBlockW - 1) / kBlockW);
  // (a sharded round runs even with no rows: the peer waits for its flags)
  const int m_chunks = std::max(kShard ? 1 : 0, (tab.total_rows + BN - 1) / BN);
  const int nkb = static_cast<int>((shape.K + kBlockK - 1) / kBlockK);
  if (splits <= 0) {
    // The split that minimises the K-blocks of the busiest SM (its CTAs x
    // K-blocks per CTA), among cluster sizes that schedule well (1, 2, 4, 5,
    // 8; 3, 6 and 7 measured slow), with the grid within the resident CTA
    // capacity and at least 8 K-blocks per split; ties go to more splits.
    // Decode at M = 28: O and Down take 8, QKV 5 (13.1 vs 13.8 us with 4).
    // resident CTAs per SM by shared memory (228 KB per SM, 1 KB reserved per CTA), at most 4
    const int per_sm = std::max(1, std::min(4, (228 * 1024) / (smem_bytes + 1024)));
    const int sms = sm_count();
    const int cap = sms * per_sm;
    const int base = std::max(1, n_tiles * m_chunks);
    splits = 1;
    int64_t best = INT64_MAX;
    for (int s : {1, 2, 4, 5, 8}) {
      if (s > 1 && (base * s > cap || nkb / s < 8)) continue;
      const int64_t ctas = static_cast<int64_t>(base) * s;
      const int64_t cost = ((ctas + sms - 1) / sms) * ((nkb + s - 1) / s);
      if (cost <= best) {
        best = cost;
        splits = s;
      }
    }
  }
  splits = std::max(1, std::min(splits, std::min(8, nkb)));

  // Split-K through global memory when tuned on (not for the fused RoPE
  // epilogue): no cluster, every CTA of the grid resident at once, but the
  // last split of a tile reads all partials back alone; measured slower than
  // the cluster reduction on the decode shapes (O at M = 28: 14.1 vs 10.3 us,
  // Down 26.9 vs 23.5 us), so the cluster reduction is the default.
  int flags = g_round_flags.load(std::memory_order_relaxed);
  CUtensorMap xmap;
  memset(&xmap, 0, sizeof(xmap));
  if (staged) {
    SWL_TRY(encode_token_tmap(&xmap, staged, tab.total_rows, shape.K, BN));
    flags |= kFlagStagedX;
  }
  SplitWs sws{nullptr, nullptr};
  if (splits > 1 && !std::is_same<Ex, QkvRopeEpi>::value && (flags & kFlagGlobalSplit)) {
    const size_t need = static_cast<size_t>(n_tiles) * m_chunks * splits * BN * kBlockW;
    const int tiles = n_tiles * m_chunks;
    if (splitk_workspace(&sws, need, tiles) != SWL_OK) {
      sws = SplitWs{nullptr, nullptr};
      cudaStreamCaptureStatus cap = cudaStreamCaptureStatusActive;
      if (cudaStreamIsCapturing(stream, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusNone &&
          ensure_streamk_workspace() == SWL_OK && splitk_workspace(&sws, need, tiles) != SWL_OK)
        sws = SplitWs{nullptr, nullptr};
    }
  }
  SWL_CUDA_TRY(launch_kernel(slot_round_tc_kernel<BN, STAGES, Ex>,
                             dim3(static_cast<unsigned>(n_tiles * splits), static_cast<unsigned>(m_chunks), 1),
                             dim3(kThreads, 1, 1), smem_bytes, stream,
                             sws.part ? 1u : static_cast<unsigned>(splits), map, xmap, tab, shape, splits, flags,
                             sws, ex));
  return SWL_OK;
}

// Supported (tile rows, stages) pairs; the tile must cover the round's rows
// (rows above a tile of 256 are split into 256-row chunks).
#define SWL_ROUND_TILES(X) \
  X(32, 2) X(32, 3) X(32, 4) X(64, 2) X(64, 3) X(64, 4) X(96, 2) X(96, 3) X(96, 4) X(128, 2) X(128, 3) \
  X(128, 4) X(128, 6) X(256, 3) X(256, 4)

bool tile_supported(int bn, int stages) {
#define SWL_TILE_CASE(B, S) if (bn == B && stages == S) return true;
  SWL_ROUND_TILES(SWL_TILE_CASE)
#undef SWL_TILE_CASE
  return false;
}

// The tile for a round of m token rows: the tuned (or default) pair of its
// row class.
template <class Ex>
int launch_tc_any(const SlotTable& tab, const RoundShape& shape, const CUtensorMap& map, int splits,
                  const Ex& ex, cudaStream_t stream) {
  const int m = std::max(1, tab.total_rows);
  const int c = row_class(m);
  int bn = g_tile_bn[c].load(std::memory_order_relaxed), stages = g_tile_stages[c].load(std::memory_order_relaxed);
  if (bn == 0 || (bn < m && bn < 256)) {
    bn = kDefaultTile[c][0];
    stages = kDefaultTile[c][1];
  }
  // staged token rows (plain rounds only): pack them, then the round
  const int st_set = g_tile_staged[c].load(std::memory_order_relaxed);
  const int64_t min_elems = kDefaultStagedMinElems[c];
  const bool want_staged = std::is_same<Ex, NoEpi>::value && tab.total_rows > 0 &&
                           (st_set >= 0 ? st_set != 0 : (min_elems >= 0 && shape.N * shape.K >= min_elems));
  void* staged = nullptr;
  if (want_staged) {
    staged = staging_buffer(static_cast<size_t>(tab.total_rows) * shape.K * 2, stream);
    if (staged)
      SWL_CUDA_TRY(launch_kernel(stage_rows_kernel, dim3(static_cast<unsigned>(tab.total_rows)), dim3(256), 0, stream,
                                 1, tab, shape.in_stride, shape.K, static_cast<__nv_bfloat16*>(staged)));
  }
#define SWL_TILE_CASE(B, S) \
  if (bn == B && stages == S) return launch_tc<B, S>(tab, shape, map, splits, ex, stream, staged);
  SWL_ROUND_TILES(SWL_TILE_CASE)
#undef SWL_TILE_CASE
  return set_error(SWL_ERR_ARG, "slot round: no tile %d x %d stages", bn, stages);
}

}  // namespace

int encode_weight_tmap(CUtensorMap* map, const void* W, int64_t N, int64_t K) {
  auto enc = tmap_encoder();
  if (!enc) return set_error(SWL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(W) & 15) != 0 || (K * 2) % 16 != 0)
    return set_error(SWL_ERR_ARG, "weight must be 16-byte aligned with K*2 a multiple of 16");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlockK), static_cast<cuuint32_t>(kBlockW)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(W), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(SWL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SWL_OK;
}

int encode_kv_page_tmap(CUtensorMap* map, const void* cache, int64_t tokens, int hkv) {
  auto enc = tmap_encoder();
  if (!enc) return set_error(SWL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(cache) & 15) != 0 || hkv <= 0 || tokens < 16 || tokens > (int64_t{1} << 31))
    return set_error(SWL_ERR_ARG, "KV tensor map: bad cache base, head count or extent");
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(hkv), static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {128 * 2, static_cast<cuuint64_t>(hkv) * 128 * 2};
  cuuint32_t box[3] = {64, 1, 16};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(cache), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(SWL_ERR_CUDA, "KV tensor map: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SWL_OK;
}

int launch_slot_round(const SlotTable& tab, const RoundShape& shape, const void* W,
                      const CUtensorMap* tmap, int algo, int splits, cudaStream_t stream) {
  if (tab.nslots <= 0 || tab.total_rows <= 0) return SWL_OK;  // nothing to do
  if (tab.nslots > kMaxSlots) return set_error(SWL_ERR_ARG, "too many slots (%d)", tab.nslots);
  if (shape.N <= 0 || shape.K <= 0 || (shape.N % 8) != 0 || (shape.K % 8) != 0)
    return set_error(SWL_ERR_ARG, "round shape N=%lld K=%lld must be positive multiples of 8",
                     (long long)shape.N, (long long)shape.K);
  if (algo == kAlgoSimt) {
    if (tab.total_rows > 65535) return set_error(SWL_ERR_ARG, "simt round: too many rows");
    dim3 grid(static_cast<unsigned>((shape.N + 7) / 8), static_cast<unsigned>(tab.total_rows));
    slot_round_simt_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(W), tab,
                                                     shape);
    SWL_CUDA_TRY(cudaGetLastError());
    return SWL_OK;
  }
  CUtensorMap local;
  if (!tmap) {
    SWL_TRY(encode_weight_tmap(&local, W, shape.N, shape.K));
    tmap = &local;
  }
  const int m = tab.total_rows;
  if (algo == kAlgoStreamK) {
    if (m > 64) return set_error(SWL_ERR_ARG, "stream-K round: at most 64 token rows");
    return launch_slot_round_streamk(tab, shape, *tmap, stream);
  }
  const NoEpi none{0};
  return launch_tc_any(tab, shape, *tmap, splits, none, stream);
}

int launch_slot_round_qkv_rope(const SlotTable& tab, const RoundShape& shape, const void* W,
                               const CUtensorMap* tmap, const QkvRopeEpi& epi, int splits,
                               cudaStream_t stream) {
  if (tab.nslots <= 0 || tab.total_rows <= 0) return SWL_OK;
  if (tab.nslots > kMaxSlots) return set_error(SWL_ERR_ARG, "too many slots (%d)", tab.nslots);
  if (tab.total_rows > kQkvRopeMaxRows)
    return set_error(SWL_ERR_ARG, "fused QKV/RoPE round: at most %d rows", kQkvRopeMaxRows);
  if (epi.hq <= 0 || epi.hkv <= 0 || shape.N != static_cast<int64_t>(epi.hq + 2 * epi.hkv) * 128 ||
      shape.K <= 0 || (shape.K % 8) != 0 || shape.bias)
    return set_error(SWL_ERR_ARG, "fused QKV/RoPE round: N must be (hq + 2 hkv) * 128, K a multiple of 8, no bias");
  if (epi.rank < 0 || epi.rank > 32 || (epi.rank % 8) != 0 || epi.splits_in < 0 || epi.page <= 0 || !epi.cos_sin ||
      !epi.q_rot || (reinterpret_cast<uintptr_t>(epi.q_rot) & 7))
    return set_error(SWL_ERR_ARG, "fused QKV/RoPE round: invalid epilogue arguments");
  for (int i = 0; i < tab.nslots; ++i) {
    if (!epi.seqlen[i] || !epi.block_table[i] || !epi.k_cache[i] || !epi.v_cache[i] ||
        (reinterpret_cast<uintptr_t>(epi.k_cache[i]) & 7) || (reinterpret_cast<uintptr_t>(epi.v_cache[i]) & 7))
      return set_error(SWL_ERR_ARG, "fused QKV/RoPE round: slot %d tables missing or caches misaligned", i);
    if (epi.B[i] && ((reinterpret_cast<uintptr_t>(epi.B[i]) & 15) || epi.rank == 0 || !epi.ws_in))
      return set_error(SWL_ERR_ARG, "fused QKV/RoPE round: slot %d lora_B misaligned or without rank/partials", i);
  }
  CUtensorMap local;
  if (!tmap) {
    SWL_TRY(encode_weight_tmap(&local, W, shape.N, shape.K));
    tmap = &local;
  }
  if (tab.total_rows <= 32) return launch_tc<32, 4>(tab, shape, *tmap, splits, epi, stream);
  return launch_tc<64, 4>(tab, shape, *tmap, splits, epi, stream);
}

int launch_slot_round_shard(const SlotTable& tab, const RoundShape& shape, const void* W,
                            const CUtensorMap* tmap, const ShardArgs& sh, int splits, cudaStream_t stream) {
  if (tab.nslots > kMaxSlots) return set_error(SWL_ERR_ARG, "too many slots (%d)", tab.nslots);
  if (shape.N <= 0 || shape.K <= 0 || (shape.N % 8) != 0 || (shape.K % 8) != 0 || sh.col0 < 0 || (sh.col0 % 4) != 0)
    return set_error(SWL_ERR_ARG, "sharded round: N=%lld K=%lld col0=%lld must be multiples of 8 (col0 of 4)",
                     (long long)shape.N, (long long)shape.K, (long long)sh.col0);
  if (!sh.sync || !sh.peer_sync || (reinterpret_cast<uintptr_t>(sh.sync) & 63) ||
      (reinterpret_cast<uintptr_t>(sh.peer_sync) & 63))
    return set_error(SWL_ERR_ARG, "sharded round: sync words missing or not 64-byte aligned");
  for (int i = 0; i < tab.nslots; ++i) {
    const bool rows = tab.row_start[i + 1] > tab.row_start[i];
    if (rows && (!sh.peer_out[i] || (reinterpret_cast<uintptr_t>(sh.peer_out[i]) & 7)))
      return set_error(SWL_ERR_ARG, "sharded round: peer output of slot %d missing or not 8-byte aligned", i);
  }
  // An empty round still takes part in the exchange: the peer waits for it.
  const int m = std::max(1, tab.total_rows);
  CUtensorMap local;
  if (!tmap) {
    SWL_TRY(encode_weight_tmap(&local, W, shape.N, shape.K));
    tmap = &local;
  }
  (void)m;
  return launch_tc_any(tab, shape, *tmap, splits, sh, stream);
}

int read_and_clear_device_error(unsigned int* code) {
  unsigned int v = 0, zero = 0, v2 = 0;
  SWL_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_round_error_word, sizeof(v)));
  if (v) SWL_CUDA_TRY(cudaMemcpyToSymbol(g_round_error_word, &zero, sizeof(zero)));
  SWL_TRY(read_and_clear_sk_error(&v2));
  *code = v ? v : v2;
  return SWL_OK;
}

}  // namespace swl

using namespace swl;

// Raw C-ABI round over caller-provided slot buffers (no pool): slot i reads
// rows[i] rows of K bf16 from in_ptrs[i] (row stride in_stride elements) and
// writes rows[i] rows of N bf16 to out_ptrs[i] (row stride out_stride).
// W is [N, K] row-major bf16 on the current device; bias is [N] or NULL.
// algo: 0 auto (= 1), 1 cluster split-K, 2 CUDA cores, 3 stream-K (<= 64 rows).
// splits: K-split factor (cluster size) for the tensor-core path; <= 0 = auto.
SWL_EXPORT int swl_slot_gemm(const void* W, int64_t N, int64_t K, const void* bias, int nslots,
                             const void* const* in_ptrs, void* const* out_ptrs, const int* rows,
                             int64_t in_stride, int64_t out_stride, int algo, int splits,
                             void* stream) {
  if (!W || nslots < 0 || nslots > kMaxSlots || (nslots > 0 && (!in_ptrs || !out_ptrs || !rows)))
    return set_error(SWL_ERR_ARG, "swl_slot_gemm: invalid arguments");
  SlotTable tab;
  tab.nslots = nslots;
  int acc = 0;
  for (int i = 0; i < nslots; ++i) {
    if (rows[i] < 0) return set_error(SWL_ERR_ARG, "swl_slot_gemm: negative row count");
    if (rows[i] > 0 && (!in_ptrs[i] || !out_ptrs[i]))
      return set_error(SWL_ERR_ARG, "swl_slot_gemm: null slot buffer");
    tab.row_start[i] = acc;
    tab.in[i] = static_cast<const __nv_bfloat16*>(in_ptrs[i]);
    tab.out[i] = static_cast<__nv_bfloat16*>(out_ptrs[i]);
    acc += rows[i];
  }
  tab.row_start[nslots] = acc;
  tab.total_rows = acc;
  RoundShape shape{N, K, in_stride > 0 ? in_stride : K, out_stride > 0 ? out_stride : N,
                   static_cast<const __nv_bfloat16*>(bias)};
  for (int i = 0; i < nslots; ++i) {
    if ((reinterpret_cast<uintptr_t>(tab.in[i]) & 15) || (reinterpret_cast<uintptr_t>(tab.out[i]) & 7))
      return set_error(SWL_ERR_ARG, "swl_slot_gemm: slot buffers must be 16-byte (in) / 8-byte (out) aligned");
  }
  if ((shape.in_stride % 8) || (shape.out_stride % 4))
    return set_error(SWL_ERR_ARG, "swl_slot_gemm: row strides must keep rows aligned");
  if (algo < 0 || algo > 3) return set_error(SWL_ERR_ARG, "swl_slot_gemm: unknown algo %d", algo);
  return launch_slot_round(tab, shape, W, nullptr, algo, splits, static_cast<cudaStream_t>(stream));
}

// Reads (and clears) the device error word set by bounded waits in the round
// kernels; synchronous. *code = 0 means no wait ran out.
SWL_EXPORT int swl_round_device_error(unsigned int* code) {
  if (!code) return set_error(SWL_ERR_ARG, "null code pointer");
  return read_and_clear_device_error(code);
}

// Tuning of the tensor-core round: for rounds of up to `max_rows` token rows
// (32, 64, 96, 128, or 0 = above 128), tile `bn` rows with a ring of
// `stages` K-blocks (bn = 0 restores the default of that class; the tile
// must hold the class's rows, except 256-row chunks above 128). flags bit 0
// makes the gather warps poll the free-stage barrier without sleeping; bit 1
// reduces split-K partial sums through the global-memory workspace instead
// of across a thread-block cluster (DSMEM); bit 2 prefetches into L2, before
// the dependency wait, the W tiles of a CTA that do not fit in its ring (up
// to 12 K-blocks). Bits 0-2 apply to every class. Bit 3 (with bn != 0) packs
// the class's token rows into a staging copy that the round loads by TMA;
// bn = 0 restores the class's default tile and staging.
SWL_EXPORT int swl_round_tune(int max_rows, int bn, int stages, int flags) {
  int c = -1;
  for (int i = 0; i < kRowClasses - 1; ++i)
    if (max_rows == kClassRows[i]) c = i;
  if (max_rows == 0) c = kRowClasses - 1;
  if (c < 0) return set_error(SWL_ERR_ARG, "round tuning: max_rows 32, 64, 96, 128 or 0");
  if (flags & ~(kFlagGatherSpin | kFlagGlobalSplit | kFlagPrefetchRest | kFlagStagedX))
    return set_error(SWL_ERR_ARG, "round tuning: flags bits 0-3 only");
  if (bn != 0 && (!tile_supported(bn, stages) || (c < kRowClasses - 1 && bn < kClassRows[c]) ||
                  (c == kRowClasses - 1 && bn != 256)))
    return set_error(SWL_ERR_ARG, "round tuning: tile %d x %d stages not built or too small for %d rows", bn,
                     stages, max_rows);
  g_tile_bn[c].store(bn);
  g_tile_stages[c].store(bn ? stages : 0);
  g_tile_staged[c].store(bn ? ((flags & kFlagStagedX) ? 1 : 0) : -1);
  g_round_flags.store(flags & ~kFlagStagedX);
  return SWL_OK;
}

// Tuning: persistent CTAs per SM of the stream-K round (1: 9-stage pipeline,
// 2: two 5-stage pipelines per SM).
SWL_EXPORT int swl_round_set_streamk_ctas_per_sm(int n) { return set_streamk_ctas_per_sm(n); }

// Tuning: fixed number of stream-K CTAs (0 = SM count x CTAs per SM).
SWL_EXPORT int swl_round_set_streamk_ctas(int n) { return set_streamk_ctas(n); }
