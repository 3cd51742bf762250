// Single-pass fused checkpoint (sm_100a): router -> exit decision -> stable
// compaction -> final-norm exit scatter, every hidden row read from HBM once
// and written once.
//
// A thread-block cluster of C CTAs works on 64-row tiles; CTA c owns the
// hidden columns [c*H/C, (c+1)*H/C) (its K slice).  Each CTA keeps its slice of
// the folded router weights W' = down * norm_weight ([128 x H/C], model dtype)
// resident in shared memory for the whole launch, streams its slice of every
// tile through a TMA ring and computes the transposed partial GEMM
//     D_c[b, r] = sum_{k in slice c} W'[b, k] * x[r, k]
// on the tensor cores (tcgen05.mma, M = 128 router units, N = 64 rows, fp32 in
// TMEM).  Partial sums of x^2 (and x) come from the same shared-memory tiles.
// The C partials are reduced in a fixed order by the CTA that owns each group
// of 64/C rows.  They travel through an L2-resident exchange area of the
// workspace (coalesced 128-byte stores and L2-only loads, double-buffered per
// cluster); distributed shared memory carries only the mbarrier signals
// between the CTAs.  The owner sums, computes rstd, the router logit, the
// score and the exit flag, and publishes {score, rstd, mean, flag} of its rows
// for every CTA of the cluster.  Each CTA then writes its K slice
// of every row of the tile -- survivors copied to the dense buffer at their
// stable rank, exits final-normed to their original position -- reading the
// row slice back from L2 (the cluster's tiles in flight are a few MiB).  Tile
// offsets come from a decoupled look-back across tiles (Merrill & Garland
// 2016) published by CTA rank 0 of each cluster.
//
// Reference semantics: python/TIDE/runtime.py:128-130 and :174-178 (score,
// strict threshold, normed exit scatter), python/TIDE/scheduler.py:89-100
// (stable compaction of rows and positions).
//
// Warp roles (768 threads):
//   warp 0        TMA producer (resident W' slice once, then the x ring)
//   warp 1        TMEM owner, MMA issuer
//   warps 4-7     row statistics from the ring (two threads per row)
//   warps 8-11    epilogue (tcgen05.ld of D_c), partial exchange, owner
//                 reduction, decision and broadcast (even local tiles)
//   warps 12-15   write-out: look-back and the row moves (even local tiles)
//   warps 16-19   epilogue of the odd local tiles
//   warps 20-23   write-out of the odd local tiles
// Every wait is bounded; on expiry the CTA raises TIDE_DEVERR_TIMEOUT,
// stops, drains its in-flight copies and MMAs and meets its cluster at the
// final barrier.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>

#include <type_traits>

#include "common.cuh"
#include "tc_checkpoint.cuh"
#include "tc_ptx.cuh"

namespace tide {

namespace fused {

constexpr int kRows = 64;        // rows per tile (MMA N)
constexpr int kUnits = 128;      // router units (MMA M)
constexpr int kChunk = 64;       // columns per chunk (128 bytes of 16-bit data)
// G groups (1 or 2) of epilogue and write-out warps take alternate tiles of
// a cluster: each stage is a chain of exchanges with the other CTAs (a few us
// of latency, little work), so a second chain in flight raises the rate.
constexpr int kMaxGroups = 2;
__host__ __device__ constexpr int threads_for(int G) { return 256 + 256 * G; }
constexpr int kStages = 10;
constexpr int kMaxSliceChunks = 8;  // W' slice <= 8 chunks = 128 KB
constexpr uint32_t kTmemCols = 128;  // two 64-column fp32 accumulators
constexpr int kSmemBudget = 227 * 1024;

struct Params {
  int64_t n_cap;
  const int32_t *n_dev;
  int H, C, slice, slice_chunks;
  int norm_type;
  float eps, up_bias, threshold;
  const float *up, *colsum, *bias_proj, *w_norm, *b_norm;
  const void *x;
  const int64_t *pos_in;
  const int32_t *slot_in;
  void *out_buf;
  int64_t n_total;
  void *compact_out;
  int64_t *pos_out;
  int32_t *slot_out;
  int64_t *exit_pos_out;
  float *scores_out;
  int32_t *counts;
  uint64_t *status;
  float *xchg;          // exchange area, xchg_stride floats per cluster
  int64_t xchg_stride;
  int32_t *err;
};

// exchange area of one cluster (floats): partials [2][C][64][128], row
// statistics [2][C][64][2], decisions [2][64] x float4
__host__ __device__ inline int64_t xchg_floats(int C) {
  return 2LL * C * kRows * kUnits + 2LL * C * kRows * 2 + 2LL * kRows * 4;
}

// shared-memory layout (offsets from the 1024-aligned base)
struct Layout {
  uint32_t w, ring, slots, slot_ss, info, stat, wn, bn, up, cs, bp, red, own, wg2, pos, bars, end;
};

__host__ __device__ inline Layout layout(int slice_chunks, int C, int G) {
  Layout L;
  uint32_t o = 0;
  L.w = o;       o += (uint32_t)slice_chunks * kUnits * kChunk * 2;  // resident W' slice
  L.ring = o;    o += (uint32_t)kStages * kRows * kChunk * 2;        // x chunks
  L.slots = o;   o += 0;                                             // (exchange is in L2)
  L.slot_ss = o; o += 0;
  L.info = o;    o += G * kRows * 16;                                 // [group] the tile's decisions
  L.stat = o;    o += 2u * 2 * kRows * 2 * 4;                         // [2 bufs][2 halves][64][ss, sx]
  const uint32_t slice = (uint32_t)slice_chunks * kChunk;
  L.wn = o;      o += slice * 4;
  L.bn = o;      o += slice * 4;
  L.up = o;      o += kUnits * 4;
  L.cs = o;      o += kUnits * 4;
  L.bp = o;      o += kUnits * 4;
  L.red = o;     o += G * 4u * kRows * 4;                             // [group][4 warps][64/C]
  L.own = o;     o += G * 2u * kRows * 4;                             // [group] rstd, mean of owned rows
  L.wg2 = o;     o += G * (256 + kRows * 4);                          // [group] ranks, prefix, flags
  L.pos = o;     o += G * kRows * 8;                                  // [group] positions of the tile's rows
  o = (o + 15u) & ~15u;
  L.bars = o;    o += 64 * 8;
  L.end = o;
  (void)C;
  return L;
}

// barrier indices inside the bars array
enum Bar {
  kFull = 0,                 // [kStages]
  kEmpty = kFull + kStages,  // [kStages]
  kWFull = kEmpty + kStages,
  kAccFull,                  // [2]
  kAccEmpty = kAccFull + 2,  // [2]
  kStatFull = kAccEmpty + 2, // [2]
  kStatEmpty = kStatFull + 2,// [2]
  kSlotsFull = kStatEmpty + 2, // [2]
  kSlotFree = kSlotsFull + 2,  // [2]
  kInfoFull = kSlotFree + 2,   // [2]
  kInfoFree = kInfoFull + 2, // [2]
  kDrain = kInfoFree + 2,
  kNumBars
};
static_assert(kNumBars <= 64, "barrier area");

__device__ __forceinline__ void unpack8(const uint4 &v, float *f, bool bf16) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (bf16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      const float2 t = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
}

// Read-only look-back: exclusive prefix of `tile` from its predecessors.
__device__ __forceinline__ bool lookback_read(const uint64_t *status, uint32_t tile,
                                              uint32_t *keep_before, uint32_t *exits_before) {
  uint32_t kb = 0, eb = 0;
  int64_t j = (int64_t)tile - 1;
  while (j >= 0) {
    uint64_t s = 0;
    int spins = 0;
    while (((s = ld_status(&status[j])) >> 62) == 0) {
      if (++spins > kSpinLimit) {
        *keep_before = kb;
        *exits_before = eb;
        return false;
      }
      __nanosleep(32);
    }
    kb += (uint32_t)(s & kCountMask);
    eb += (uint32_t)((s >> 31) & kCountMask);
    if ((s >> 62) == 2) break;
    --j;
  }
  *keep_before = kb;
  *exits_before = eb;
  return true;
}

template <bool BF16, int C, int G>
__global__ void __launch_bounds__(threads_for(G), 1)
    fused_checkpoint_kernel(const __grid_constant__ CUtensorMap tmap_x,
                            const __grid_constant__ CUtensorMap tmap_w, Params p) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int R = kRows / C;  // rows owned by each CTA of the cluster
  static_assert(R % 4 == 0, "owner rows come in float4 groups");
  const bool LAYER = p.norm_type == TIDE_NORM_LAYER;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kThreads = threads_for(G);
  const Layout L = layout(p.slice_chunks, C, G);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
  const int grp = (int)(threadIdx.x >> 5) >= 8 ? ((int)(threadIdx.x >> 5) - 8) >> 3 : 0;  // group
  float4 *info = reinterpret_cast<float4 *>(smem + L.info) + grp * kRows;  // [64] decisions of the tile
  float *stat = reinterpret_cast<float *>(smem + L.stat);
  float *s_wn = reinterpret_cast<float *>(smem + L.wn);
  float *s_bn = reinterpret_cast<float *>(smem + L.bn);
  float *s_up = reinterpret_cast<float *>(smem + L.up);
  float *s_cs = reinterpret_cast<float *>(smem + L.cs);
  float *s_bp = reinterpret_cast<float *>(smem + L.bp);
  float *s_red = reinterpret_cast<float *>(smem + L.red) + grp * 4 * kRows;
  uint32_t *wg2 = reinterpret_cast<uint32_t *>(smem + L.wg2);  // [0..2]: CTA-wide words
  uint32_t *wgg = wg2 + grp * (64 + kRows);                     // this group's words
  uint32_t *tmem_slot = wg2;              // [0]
  volatile int *abort_flag = reinterpret_cast<volatile int *>(wg2 + 1);
  uint32_t *issued = wg2 + 2;
  uint32_t *s_prefix = wgg + 4;           // [4]: keep_before, exits_before, keep_t, exit_t
  uint32_t *s_rank = wgg + 64;            // [64] rank of each row among its kind
  volatile int *s_stop1 = reinterpret_cast<volatile int *>(wgg + 16);  // epilogue group
  volatile int *s_stop2 = reinterpret_cast<volatile int *>(wgg + 17);  // write-out group
  int64_t *s_pos = reinterpret_cast<int64_t *>(smem + L.pos) + grp * kRows;  // [64] tile positions
  float *s_rstd = reinterpret_cast<float *>(smem + L.own) + grp * 2 * kRows;  // [R] owned rows
  float *s_mean = s_rstd + kRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_rank();
  const int cluster_id = blockIdx.x / C;
  const int n_clusters = gridDim.x / C;
  const int slice = p.slice, nk = p.slice_chunks;
  const uint32_t chunk_bytes = kRows * kChunk * 2;      // 8 KB
  const uint32_t wchunk_bytes = kUnits * kChunk * 2;    // 16 KB

  int64_t n = p.n_cap;
  if (p.n_dev) {
    int64_t nd = (int64_t)__ldg(p.n_dev);
    if (nd < 0 || nd > p.n_cap) {
      if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(p.err, TIDE_DEVERR_COUNT);
      nd = nd < 0 ? 0 : p.n_cap;
    }
    n = nd;
  }
  const int n_tiles = (int)((n + kRows - 1) / kRows);

  // ---------------------------------------------------------------- setup
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&bars[kFull + s], 1);
      ptx::mbar_init(&bars[kEmpty + s], 1 + 4);  // MMA commit + 4 statistics warps
    }
    ptx::mbar_init(&bars[kWFull], 1);
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&bars[kAccFull + a], 1);
      ptx::mbar_init(&bars[kAccEmpty + a], 4);
      ptx::mbar_init(&bars[kStatFull + a], 4);
      ptx::mbar_init(&bars[kStatEmpty + a], 4);
      ptx::mbar_init(&bars[kInfoFull + a], kRows);  // one arrival per row
      ptx::mbar_init(&bars[kInfoFree + a], C);      // one arrival per CTA
      ptx::mbar_init(&bars[kSlotsFull + a], 4 * C); // 4 warps of every source
      ptx::mbar_init(&bars[kSlotFree + a], C);      // every owner
    }
    ptx::mbar_init(&bars[kDrain], 1);
    *abort_flag = 0;
    *issued = 0;
    for (int g = 0; g < G; ++g) {
      wg2[g * (64 + kRows) + 16] = 0;  // s_stop1, s_stop2 of every group
      wg2[g * (64 + kRows) + 17] = 0;
    }
    ptx::fence_mbar_init();
    ptx::fence_proxy_async();
  }
  const int col0 = (int)rank * slice;
  for (int i = threadIdx.x; i < slice; i += kThreads) {
    s_wn[i] = p.w_norm[col0 + i];
    s_bn[i] = (LAYER && p.b_norm) ? p.b_norm[col0 + i] : 0.f;
  }
  for (int i = threadIdx.x; i < kUnits; i += kThreads) {
    s_up[i] = p.up[i];
    s_cs[i] = LAYER ? p.colsum[i] : 0.f;
    s_bp[i] = (LAYER && p.bias_proj) ? p.bias_proj[i] : 0.f;
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, kTmemCols);
    ptx::tmem_relinquish();
  }
  if (n_tiles == 0 && blockIdx.x == 0 && threadIdx.x == 0 && p.counts) {
    p.counts[0] = 0;
    p.counts[1] = 0;
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  ptx::cluster_sync();  // every CTA's barriers exist before any remote arrive
  const uint32_t tmem_base = *tmem_slot;

  const uint32_t bars_u32 = ptx::smem_u32(bars);
  auto remote_bar = [&](int which, uint32_t cta) {
    return ptx::map_to_rank(bars_u32 + (uint32_t)which * 8u, cta);
  };

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      ptx::prefetch_tmap(&tmap_x);
      ptx::prefetch_tmap(&tmap_w);
      ptx::mbar_expect_tx(&bars[kWFull], (uint32_t)nk * wchunk_bytes);
      for (int kc = 0; kc < nk; ++kc)
        ptx::tma_load_2d(smem + L.w + (size_t)kc * wchunk_bytes, &tmap_w, &bars[kWFull],
                         col0 + kc * kChunk, 0);
      uint32_t it = 0;
      for (int tile = cluster_id; tile < n_tiles && !*abort_flag; tile += n_clusters) {
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
          if (it >= (uint32_t)kStages && !ptx::mbar_wait(&bars[kEmpty + s], ph ^ 1u, abort_flag)) {
            raise_error(p.err, TIDE_DEVERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          ptx::mbar_expect_tx(&bars[kFull + s], chunk_bytes);
          ptx::tma_load_2d(smem + L.ring + (size_t)s * chunk_bytes, &tmap_x, &bars[kFull + s],
                           col0 + kc * kChunk, tile * kRows);
          *issued = it + 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::f16_idesc(BF16, kUnits, kRows);
      bool ok = ptx::mbar_wait(&bars[kWFull], 0, abort_flag);
      uint32_t it = 0;
      int t_local = 0;
      const uint32_t w_base = ptx::smem_u32(smem + L.w);
      for (int tile = cluster_id; ok && tile < n_tiles && !*abort_flag;
           tile += n_clusters, ++t_local) {
        const int acc = t_local & 1;
        if (t_local >= 2 &&
            !ptx::mbar_wait(&bars[kAccEmpty + acc], ((uint32_t)(t_local >> 1) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kRows);
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
          if (!ptx::mbar_wait(&bars[kFull + s], ph, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t a0 = w_base + (uint32_t)kc * wchunk_bytes;
          const uint32_t b0 = ptx::smem_u32(smem + L.ring + (size_t)s * chunk_bytes);
#pragma unroll
          for (int k = 0; k < kChunk / 16; ++k)
            ptx::mma_f16_ss(d_tmem, ptx::sw128_kmajor_desc(a0 + 32u * k),
                            ptx::sw128_kmajor_desc(b0 + 32u * k), idesc,
                            (kc > 0 || k > 0) ? 1u : 0u);
          ptx::mma_commit(&bars[kEmpty + s]);
        }
        if (!ok) break;
        ptx::mma_commit(&bars[kAccFull + acc]);
      }
      if (!ok) {
        raise_error(p.err, TIDE_DEVERR_TIMEOUT);
        *abort_flag = 1;
      }
      ptx::mma_commit(&bars[kDrain]);
      volatile int never = 0;
      if (!ptx::mbar_wait(&bars[kDrain], 0, &never)) raise_error(p.err, TIDE_DEVERR_TIMEOUT);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------- row statistics
    const int t = threadIdx.x - 128;  // 0..127
    const int r = t & (kRows - 1), h = t >> 6;
    uint32_t it = 0;
    int t_local = 0;
    bool ok = true;
    for (int tile = cluster_id; ok && tile < n_tiles; tile += n_clusters, ++t_local) {
      float ss0 = 0.f, ss1 = 0.f, sx0 = 0.f, sx1 = 0.f;
      for (int kc = 0; kc < nk; ++kc, ++it) {
        const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
        if (!ptx::mbar_wait(&bars[kFull + s], ph, abort_flag)) { ok = false; break; }
        const uint8_t *row = smem + L.ring + (size_t)s * chunk_bytes + (size_t)r * 128;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int unit = (h * 4 + j + lane) & 7;
          float f[8];
          unpack8(*reinterpret_cast<const uint4 *>(row + (unit << 4)), f, BF16);
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            ss0 = fmaf(f[e], f[e], ss0);
            ss1 = fmaf(f[e + 1], f[e + 1], ss1);
            if (LAYER) { sx0 += f[e]; sx1 += f[e + 1]; }
          }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars[kEmpty + s]);
      }
      if (!ok) break;
      const int buf = t_local & 1;
      if (t_local >= 2 &&
          !ptx::mbar_wait(&bars[kStatEmpty + buf], ((uint32_t)(t_local >> 1) & 1u) ^ 1u, abort_flag)) {
        ok = false;
        break;
      }
      float *st = stat + ((size_t)(buf * 2 + h) * kRows + r) * 2;
      st[0] = ss0 + ss1;
      st[1] = sx0 + sx1;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[kStatFull + buf]);
    }
    if (!ok) {
      raise_error(p.err, TIDE_DEVERR_TIMEOUT);
      *abort_flag = 1;
    }
  } else if (warp >= 8 && (warp & 7) < 4) {
    // ---------------------- epilogue, partial exchange, owner reduction
    // (group grp: warps 8-11 or 16-19, the tiles with t_local % 2 == grp)
    // All 128 threads pass every named barrier of an iteration; a failed
    // wait only turns the rest of the iteration's work off (ok = false) and
    // the group stops together at the iteration's end (s_stop1).
    const int t = threadIdx.x - 256 - 256 * grp;  // 0..127 = router unit b = TMEM lane
    const int bar_id = 1 + 2 * grp;
    const int q = warp & 3;            // TMEM lane quarter of this warp
    float *xP = p.xchg + (size_t)cluster_id * (size_t)p.xchg_stride;
    float *xS = xP + 2 * C * kRows * kUnits;
    float4 *xI = reinterpret_cast<float4 *>(xS + 2 * C * kRows * 2);
    for (int tile = cluster_id + grp * n_clusters, t_local = grp; tile < n_tiles;
         tile += G * n_clusters, t_local += G) {
      bool ok = true;
      const int buf = t_local & 1;
      const uint32_t ph2 = (uint32_t)(t_local >> 1) & 1u;
      // (1) this CTA's partial row statistics
      float ss_part = 0.f, sx_part = 0.f;
      ok = ptx::mbar_wait(&bars[kStatFull + buf], ph2, abort_flag);
      if (ok && t < kRows) {
        const float *st0 = stat + ((size_t)(buf * 2 + 0) * kRows + t) * 2;
        const float *st1 = stat + ((size_t)(buf * 2 + 1) * kRows + t) * 2;
        ss_part = st0[0] + st1[0];
        sx_part = st0[1] + st1[1];
      }
      __syncwarp();
      if (ok && lane == 0) ptx::mbar_arrive(&bars[kStatEmpty + buf]);
      // (2) this CTA's partial D_c[b, 0..63] from TMEM
      // (3) publish the partials: xP[buf][rank][r][b], coalesced over b,
      // read from TMEM in two halves of 32 rows (registers)
      if (ok) ok = ptx::mbar_wait(&bars[kAccFull + buf], ph2, abort_flag);
      if (ok && t_local >= 2)
        ok = ptx::mbar_wait_cluster(&bars[kSlotFree + buf], ph2 ^ 1u, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        ptx::tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kRows);
        float *dst = xP + ((size_t)(buf * C + (int)rank) * kRows) * kUnits + t;
#pragma unroll
        for (int half = 0; half < kRows / 32; ++half) {
          float d[32];
          ptx::tmem_ld32(taddr + 32u * half, d);
#pragma unroll
          for (int r = 0; r < 32; ++r) __stcg(dst + (size_t)(half * 32 + r) * kUnits, d[r]);
        }
        ptx::tc_fence_before();
      }
      __syncwarp();
      if (ok && lane == 0) ptx::mbar_arrive(&bars[kAccEmpty + buf]);
      if (ok) {
        if (t < kRows) {
          float *sd = xS + ((size_t)(buf * C + (int)rank) * kRows + t) * 2;
          __stcg(sd, ss_part);
          __stcg(sd + 1, sx_part);
        }
      }
      // the warp barrier orders every lane's stores before lane 0's fence;
      // one cluster-scope fence then covers all the arrivals
      ok = __all_sync(0xffffffffu, ok);
      if (ok && lane == 0) {
        ptx::fence_cluster();
        for (int o = 0; o < C; ++o)
          ptx::mbar_arrive_cluster_relaxed(remote_bar(kSlotsFull + buf, (uint32_t)o));
      }
      // (4) owner: the statistics of the R owned rows, then their logits
      if (ok) ok = ptx::mbar_wait_cluster(&bars[kSlotsFull + buf], ph2, abort_flag);
      const int row0 = (int)rank * R;  // first owned row of the tile
      if (ok && t < R) {
        float ss = 0.f, sx = 0.f;
#pragma unroll
        for (int src = 0; src < C; ++src) {
          const float *sd = xS + ((size_t)(buf * C + src) * kRows + row0 + t) * 2;
          ss += __ldcg(sd);
          sx += __ldcg(sd + 1);
        }
        float mean = 0.f, rstd;
        if (!LAYER) {
          rstd = rsqrt_rn(ss / (float)p.H + p.eps);
        } else {
          mean = sx / (float)p.H;
          rstd = rsqrt_rn(fmaxf(ss / (float)p.H - mean * mean, 0.f) + p.eps);
        }
        s_rstd[t] = rstd;
        s_mean[t] = mean;
      }
      if (!ok) *s_stop1 = 1;
      ptx::named_sync(bar_id, 128);
      ok = !*s_stop1;
      if (ok) {
        float acc[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) acc[rr] = 0.f;
#pragma unroll
        for (int src = 0; src < C; ++src) {
          const float *sp = xP + ((size_t)(buf * C + src) * kRows + row0) * kUnits + t;
#pragma unroll
          for (int rr = 0; rr < R; ++rr) acc[rr] += __ldcg(sp + (size_t)rr * kUnits);
        }
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          const float rstd = s_rstd[rr];
          const float z = LAYER ? fmaf(rstd, acc[rr] - s_mean[rr] * s_cs[t], s_bp[t]) : rstd * acc[rr];
          const float v = warp_sum(s_up[t] * silu_tanh(z));
          if (lane == 0) s_red[q * R + rr] = v;
        }
      }
      ptx::named_sync(bar_id, 128);
      // every partial of this buffer has been read: sources may refill it
      // (the loads have returned: a relaxed signal orders nothing else)
      if (ok && t == 0)
        for (int src = 0; src < C; ++src)
          ptx::mbar_arrive_cluster_relaxed(remote_bar(kSlotFree + buf, (uint32_t)src));
      // (5) decide the owned rows and publish {score, rstd, mean, flag}
      if (ok && t < R) {
        const float logit = p.up_bias + s_red[0 * R + t] + s_red[1 * R + t] + s_red[2 * R + t] +
                            s_red[3 * R + t];
        const float score = sigmoid_f(logit);
        const int64_t grow = (int64_t)tile * kRows + row0 + t;
        float flag = 0.f;  // 0 beyond the active rows, 1 survive, 2 exit
        if (grow < n) {
          flag = score > p.threshold ? 2.f : 1.f;
          if (p.scores_out) p.scores_out[grow] = score;
        }
        if (t_local >= 2) ok = ptx::mbar_wait_cluster(&bars[kInfoFree + buf], ph2 ^ 1u, abort_flag);
        if (ok) {
          __stcg(&xI[buf * kRows + row0 + t], make_float4(score, s_rstd[t], s_mean[t], flag));
          ptx::fence_cluster();
#pragma unroll
          for (int dcta = 0; dcta < C; ++dcta)
            ptx::mbar_arrive_cluster_relaxed(remote_bar(kInfoFull + buf, (uint32_t)dcta));
        }
      }
      if (!ok || *abort_flag) *s_stop1 = 1;
      ptx::named_sync(bar_id, 128);
      if (*s_stop1) break;
    }
    if (*s_stop1) {
      raise_error(p.err, TIDE_DEVERR_TIMEOUT);
      *abort_flag = 1;
    }
  } else if (warp >= 8) {
    // -------------------------------------------- look-back, row moves
    // (group grp: warps 12-15 or 20-23, the tiles with t_local % 2 == grp)
    const int t = threadIdx.x - 384 - 256 * grp;  // 0..127
    const int bar_id = 2 + 2 * grp;
    const int w4 = t >> 5;            // 0..3
    const T *x = static_cast<const T *>(p.x);
    const int vec_per_row = slice / 8;  // 16-byte vectors of this CTA's slice (<= 64)
    const float4 *xI2 = reinterpret_cast<const float4 *>(
        p.xchg + (size_t)cluster_id * (size_t)p.xchg_stride + 2 * C * kRows * kUnits + 2 * C * kRows * 2);
    for (int tile = cluster_id + grp * n_clusters, t_local = grp; tile < n_tiles;
         tile += G * n_clusters, t_local += G) {
      const int buf = t_local & 1;
      const uint32_t ph2 = (uint32_t)(t_local >> 1) & 1u;
      bool ok = ptx::mbar_wait_cluster(&bars[kInfoFull + buf], ph2, abort_flag);
      if (ok && t < kRows) info[t] = __ldcg(&xI2[buf * kRows + t]);
      if (!ok) *s_stop2 = 1;
      ptx::named_sync(bar_id, 128);
      if (*s_stop2) break;
      // the decisions are copied: every owner may reuse this buffer
      if (t == 0)
        for (int o = 0; o < C; ++o)
          ptx::mbar_arrive_cluster_relaxed(remote_bar(kInfoFree + buf, (uint32_t)o));
      // ranks inside the tile (rows 0..63 by threads 0..63); the tile's
      // positions are fetched once here, in parallel
      if (t < kRows) {
        const int st = (int)info[t].w;
        const int64_t row = (int64_t)tile * kRows + t;
        s_pos[t] = st == 0 ? -1 : (p.pos_in ? p.pos_in[row] : row);
        const unsigned kb = __ballot_sync(0xffffffffu, st == 1);
        const unsigned eb = __ballot_sync(0xffffffffu, st == 2);
        const unsigned lt = (1u << lane) - 1u;
        s_rank[t] = st == 1 ? __popc(kb & lt) : __popc(eb & lt);
        if (lane == 0) {
          s_prefix[8 + w4 * 2] = __popc(kb);
          s_prefix[8 + w4 * 2 + 1] = __popc(eb);
        }
      }
      ptx::named_sync(bar_id, 128);
      if (t < kRows && t >= 32) {
        const int st = (int)info[t].w;
        s_rank[t] += st == 1 ? s_prefix[8] : s_prefix[9];
      }
      if (w4 == 0) {
        // The tile's prefix (rank 0 publishes the tile's counts, the other
        // CTAs only read).  Small clusters are many: up to 148 / C tiles are
        // in flight at once, and warp 12 reads their predecessors 32 per
        // round trip.  With 8 or 16 CTAs per cluster a tile has few live
        // predecessors and one thread walking them measured faster.
        const uint32_t keep_t = s_prefix[8] + s_prefix[10];
        const uint32_t exit_t = s_prefix[9] + s_prefix[11];
        uint32_t kb = 0, eb = 0;
        bool lb_ok = true;
        if constexpr (C <= 4) {
          lb_ok = warp_lookback(p.status, (uint32_t)tile, keep_t, exit_t, rank == 0, &kb, &eb);
        } else if (lane == 0) {
          lb_ok = rank == 0 ? lookback(p.status, (uint32_t)tile, keep_t, exit_t, &kb, &eb)
                            : lookback_read(p.status, (uint32_t)tile, &kb, &eb);
        }
        if (lane == 0) {
          if (!lb_ok) raise_error(p.err, TIDE_DEVERR_TIMEOUT);
          s_prefix[0] = kb;
          s_prefix[1] = eb;
          if (rank == 0 && tile == n_tiles - 1 && p.counts) {
            p.counts[0] = (int32_t)(kb + keep_t);
            p.counts[1] = (int32_t)(eb + exit_t);
          }
        }
      }
      ptx::named_sync(bar_id, 128);
      const uint32_t keep_before = s_prefix[0], exits_before = s_prefix[1];
      // token bookkeeping (rank 0 only)
      if (rank == 0 && t < kRows) {
        const int st = (int)info[t].w;
        const int64_t row = (int64_t)tile * kRows + t;
        if (st == 1) {
          const int64_t dst = (int64_t)keep_before + s_rank[t];
          if (p.pos_out) p.pos_out[dst] = s_pos[t];
          if (p.slot_out) p.slot_out[dst] = p.slot_in ? p.slot_in[row] : (int32_t)row;
        } else if (st == 2 && p.exit_pos_out) {
          p.exit_pos_out[(int64_t)exits_before + s_rank[t]] = s_pos[t];
        }
      }
      // row moves: warp w4 handles rows w4*16 .. w4*16+15 in batches of kMoveBatch
      constexpr int kMoveBatch = G == 1 ? 8 : 4;  // registers: 128 per thread with one group, 80 with two
      for (int batch = 0; batch < 16 / kMoveBatch; ++batch) {
        const int r0 = w4 * 16 + batch * kMoveBatch;
        uint4 v[kMoveBatch][2];
#pragma unroll
        for (int i = 0; i < kMoveBatch; ++i) {
          const int r = r0 + i;
          const int st = (int)info[r].w;
          const int64_t row = (int64_t)tile * kRows + r;
          const uint4 *src = reinterpret_cast<const uint4 *>(x + row * p.H + col0);
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int vi = lane + 32 * u;
            if (st != 0 && vi < vec_per_row) v[i][u] = ld_stream(src + vi);
          }
        }
#pragma unroll
        for (int i = 0; i < kMoveBatch; ++i) {
          const int r = r0 + i;
          const float4 in = info[r];
          const int st = (int)in.w;
          if (st == 0) continue;
          if (st == 1) {
            if (!p.compact_out) continue;
            const int64_t dst = (int64_t)keep_before + s_rank[r];
            uint4 *d = reinterpret_cast<uint4 *>(static_cast<T *>(p.compact_out) + dst * p.H + col0);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int vi = lane + 32 * u;
              if (vi < vec_per_row) st_stream(d + vi, v[i][u]);
            }
          } else {
            if (!p.out_buf) continue;
            const int64_t pos = s_pos[r];
            if (pos < 0 || pos >= p.n_total) {
              if (lane == 0) raise_error(p.err, TIDE_DEVERR_POSITION);
              continue;
            }
            const float rstd = in.y, mean = in.z, shift = -rstd * mean;
            uint4 *d = reinterpret_cast<uint4 *>(static_cast<T *>(p.out_buf) + pos * p.H + col0);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int vi = lane + 32 * u;
              if (vi >= vec_per_row) continue;
              float xv[8], y[8];
              unpack8(v[i][u], xv, BF16);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int c = vi * 8 + j;
                if (!LAYER) {
                  y[j] = __fmul_rn(s_wn[c], __fmul_rn(xv[j], rstd));
                } else {
                  const float tt = __fadd_rn(__fmul_rn(xv[j], rstd), shift);
                  y[j] = __fadd_rn(__fmul_rn(tt, s_wn[c]), s_bn[c]);
                }
              }
              st_stream(d + vi, pack16<T>(y));
            }
          }
        }
      }
      ptx::named_sync(bar_id, 128);
      if (*abort_flag) *s_stop2 = 1;
      ptx::named_sync(bar_id, 128);
      if (*s_stop2) break;
    }
    if (*s_stop2) {
      raise_error(p.err, TIDE_DEVERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // drain the TMA loads still in flight before the CTA can leave
    const uint32_t n_issued = *issued;
    volatile int never = 0;
    ptx::mbar_wait(&bars[kWFull], 0, &never);
    for (int s = 0; s < kStages; ++s) {
      if ((uint32_t)s >= n_issued) break;
      const uint32_t count = (n_issued - (uint32_t)s + (uint32_t)kStages - 1) / (uint32_t)kStages;
      ptx::mbar_wait(&bars[kFull + s], (count - 1) & 1u, &never);
    }
  }
  __syncthreads();
  ptx::cluster_sync();  // no CTA leaves while a peer may still write into it
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace fused

// ------------------------------------------------------------------ host
namespace {

PFN_cuTensorMapEncodeTiled_v12000 fused_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

bool fused_tmap(CUtensorMap *m, const void *base, bool bf16, uint64_t rows, uint64_t cols,
                uint32_t box_rows) {
  auto enc = fused_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)fused::kChunk, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
             const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Cluster size: the smallest C in {1, 2, 4, 8, 16} whose K slice is a
// multiple of 64 columns and whose W' slice fits the resident budget.  16 is
// a non-portable cluster size (opted into per kernel); it lets H = 5120 and
// 8192 keep a resident slice.
constexpr int kMaxCluster = 16;
int fused_cluster_size(int64_t H) {
  for (int c = 1; c <= kMaxCluster; c <<= 1) {
    if (H % c) continue;
    const int64_t slice = H / c;
    if (slice % fused::kChunk) continue;
    if (slice / fused::kChunk <= fused::kMaxSliceChunks) return c;
  }
  return 0;
}

size_t fused_smem_bytes(int64_t H, int G) {
  const int c = fused_cluster_size(H);
  if (!c) return 0;
  return 1024 + fused::layout((int)(H / c / fused::kChunk), c, G).end;
}

// Epilogue / write-out groups: TIDE_FUSED_GROUPS=1 or 2 forces a count.
// Otherwise one up to 1024 rows (a launch of a few tiles per cluster is one
// chain long, and the second group only adds its setup) and two above, where
// a second group's shared memory fits.  Measured at H = 4096, 10 % exits:
// 1024 rows 26.7 us either way, 2048 rows 32.3 (one) against 30.9 us (two),
// 4096 rows 43.5 against 39.6 us.
int fused_groups(int64_t H, int64_t n_rows) {
  static int forced = -1;
  if (forced < 0) {
    const char *e = getenv("TIDE_FUSED_GROUPS");
    forced = (e && (e[0] == '1' || e[0] == '2') && e[1] == 0) ? e[0] - '0' : 0;
  }
  if (forced) return forced;
  if (n_rows <= 1024) return 1;
  return fused_smem_bytes(H, 2) <= (size_t)fused::kSmemBudget ? 2 : 1;
}

template <bool BF16, int G>
const void *fused_fn_g(int C) {
  switch (C) {
    case 1: return (const void *)fused::fused_checkpoint_kernel<BF16, 1, G>;
    case 2: return (const void *)fused::fused_checkpoint_kernel<BF16, 2, G>;
    case 4: return (const void *)fused::fused_checkpoint_kernel<BF16, 4, G>;
    case 8: return (const void *)fused::fused_checkpoint_kernel<BF16, 8, G>;
    default: return (const void *)fused::fused_checkpoint_kernel<BF16, 16, G>;
  }
}
const void *fused_fn(bool bf16, int C, int G) {
  if (bf16) return G == 2 ? fused_fn_g<true, 2>(C) : fused_fn_g<true, 1>(C);
  return G == 2 ? fused_fn_g<false, 2>(C) : fused_fn_g<false, 1>(C);
}

}  // namespace

const char *fused_unsupported_reason(const tide_checkpoint_args *a) {
  if (a->dtype != TIDE_DTYPE_BF16 && a->dtype != TIDE_DTYPE_F16) return "dtype is not bf16/fp16";
  if (!a->folded) return "no folded router weights";
  if (a->bottleneck_dim != fused::kUnits) return "bottleneck_dim is not 128";
  if (!fused_cluster_size(a->hidden_dim)) return "hidden_dim has no cluster split with a resident weight slice";
  if (fused_smem_bytes(a->hidden_dim, fused_groups(a->hidden_dim, a->n_rows)) >
      (size_t)fused::kSmemBudget)
    return "shared memory budget";
  if (a->norm_type == TIDE_NORM_LAYER && !a->colsum) return "LayerNorm needs colsum";
  if (((uintptr_t)a->x | (uintptr_t)a->folded | (uintptr_t)a->out_buffer |
       (uintptr_t)a->compact_out) & 15u)
    return "x/folded/outputs not 16-byte aligned";
  if (a->n_rows < 1) return "no rows";
  if (a->n_rows > ((int64_t)1 << 30)) return "too many rows";
  return nullptr;
}

bool fused_supported(const tide_checkpoint_args *a) { return fused_unsupported_reason(a) == nullptr; }

// Measured crossovers against the split path (bf16, 10 % exits, one
// epilogue / write-out group up to 1024 rows and two above), by cluster size:
//   1 CTA  (H <= 512):  the split path wins at every size from 128 rows
//          (25.3 against 20.9 us at H = 512, 128 rows).
//   2 CTAs (H 768-1024): rows under 2 KB (H = 768) leave the split path the
//          SIMT mover, and the fused pass wins up to 8192 rows (30.0 against
//          30.1 us); with 2 KB rows (H = 1024) the split path wins from 128.
//   4 CTAs (H = 2048):  fused up to 4096 rows (29.1 against 30.7 us), split
//          from 4608.
//   8 CTAs (H = 4096):  fused up to 5120 rows (45.2 against 46.9 us), split
//          from 6144 (52.2 against 48.6 us).
//   16 CTAs: H = 5120 fused up to 3584 rows, split from 4096; H = 8192, whose
//          split router streams 2 MiB of W' through each CTA, fused up to
//          5120 (77.3 against 86.2 us); the two are level at 6144.
int64_t fused_auto_max_rows(int64_t H) {
  const int C = fused_cluster_size(H);
  switch (C) {
    case 0: return 0;
    case 1: return 0;
    case 2: return H * 2 < 2048 ? 8192 : 0;
    case 4: return 4096;
    case 8: return 5120;
    default: return H >= 8192 ? 5632 : 3584;
  }
}

// Workspace: 256 reserved bytes, the tile status words (zeroed per call),
// then one exchange area per cluster that can be resident on any B200
// (at most 160 SMs / C clusters).
size_t fused_status_bytes(int64_t n_rows) {
  const int64_t tiles = n_rows > 0 ? (n_rows + fused::kRows - 1) / fused::kRows : 1;
  return (((size_t)tiles * 8 + 255) / 256) * 256;
}

size_t fused_workspace_bytes(const tide_checkpoint_args *a) {
  const int C = fused_cluster_size(a->hidden_dim);
  if (!C) return 0;
  const size_t xchg = (size_t)(160 / C) * (size_t)fused::xchg_floats(C) * 4;
  return 256 + fused_status_bytes(a->n_rows) + xchg;
}

int fused_checkpoint_launch(const tide_checkpoint_args *a, cudaStream_t stream, char *err,
                            size_t err_len) {
  const bool bf16 = a->dtype == TIDE_DTYPE_BF16;
  const int C = fused_cluster_size(a->hidden_dim);
  const int slice = (int)(a->hidden_dim / C);
  CUtensorMap tx, tw;
  if (!fused_tmap(&tx, a->x, bf16, (uint64_t)a->n_rows, (uint64_t)a->hidden_dim, fused::kRows) ||
      !fused_tmap(&tw, a->folded, bf16, (uint64_t)fused::kUnits, (uint64_t)a->hidden_dim,
                  fused::kUnits)) {
    snprintf(err, err_len, "fused checkpoint: cuTensorMapEncodeTiled failed");
    return TIDE_ERR_CUDA;
  }
  char *ws = static_cast<char *>(a->workspace);
  uint64_t *status = reinterpret_cast<uint64_t *>(ws + 256);
  float *xchg = reinterpret_cast<float *>(ws + 256 + fused_status_bytes(a->n_rows));
  cudaError_t e = cudaMemsetAsync(a->workspace, 0, 256 + fused_status_bytes(a->n_rows), stream);
  if (e != cudaSuccess) {
    snprintf(err, err_len, "fused checkpoint: memset: %s", cudaGetErrorString(e));
    return TIDE_ERR_CUDA;
  }
  fused::Params p{};
  p.n_cap = a->n_rows;
  p.n_dev = a->n_rows_dev;
  p.H = (int)a->hidden_dim;
  p.C = C;
  p.slice = slice;
  p.slice_chunks = slice / fused::kChunk;
  p.norm_type = a->norm_type;
  p.eps = a->eps;
  p.up_bias = a->up_bias;
  p.threshold = a->threshold;
  p.up = a->up;
  p.colsum = a->colsum;
  p.bias_proj = a->bias_proj;
  p.w_norm = a->norm_weight;
  p.b_norm = a->norm_bias;
  p.x = a->x;
  p.pos_in = a->positions_in;
  p.slot_in = a->slots_in;
  p.out_buf = a->out_buffer;
  p.n_total = a->n_total;
  p.compact_out = a->compact_out;
  p.pos_out = a->positions_out;
  p.slot_out = a->slots_out;
  p.exit_pos_out = a->exit_positions_out;
  p.scores_out = a->scores_out;
  p.counts = a->counts_out;
  p.status = status;
  p.xchg = xchg;
  p.xchg_stride = fused::xchg_floats(C);
  p.err = a->error_word;

  const int G = fused_groups(a->hidden_dim, a->n_rows);
  const void *fn = fused_fn(bf16, C, G);
  // per device: the attributes and the occupancy belong to a device's context
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  static bool attr_set[64][2][kMaxCluster + 1][fused::kMaxGroups + 1] = {};
  if (!attr_set[dev][bf16][C][G]) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, fused::kSmemBudget);
    if (e == cudaSuccess && C > 8) e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) {
      snprintf(err, err_len, "fused checkpoint: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return TIDE_ERR_CUDA;
    }
    attr_set[dev][bf16][C][G] = true;
  }
  const size_t smem = fused_smem_bytes(a->hidden_dim, G);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3((unsigned)fused::threads_for(G), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // one resident cluster per C SMs: every cluster runs for the whole launch
  // so a look-back never waits on a tile whose cluster is not running.  A
  // device that cannot hold one cluster of this size reports
  // TIDE_ERR_UNSUPPORTED before anything is launched.
  static int max_clusters[64][2][kMaxCluster + 1][fused::kMaxGroups + 1] = {};
  if (!max_clusters[dev][bf16][C][G]) {
    cfg.gridDim = dim3((unsigned)C, 1, 1);
    int mc = 0;
    e = cudaOccupancyMaxActiveClusters(&mc, fn, &cfg);
    if (e != cudaSuccess || mc <= 0) {
      (void)cudaGetLastError();
      snprintf(err, err_len, "fused checkpoint: no resident cluster of %d CTAs (%s)", C,
               cudaGetErrorString(e));
      return TIDE_ERR_UNSUPPORTED;
    }
    max_clusters[dev][bf16][C][G] = mc;
  }
  const int64_t tiles = (a->n_rows + fused::kRows - 1) / fused::kRows;
  const int mcl = max_clusters[dev][bf16][C][G];
  int64_t g = tiles < mcl ? tiles : mcl;
  if (g > 160 / C) g = 160 / C;  // the workspace holds 160 / C exchange areas
  cfg.gridDim = dim3((unsigned)(g * C), 1, 1);
  void *args[] = {&tx, &tw, &p};
  e = cudaLaunchKernelExC(&cfg, fn, args);
  if (e != cudaSuccess) {
    snprintf(err, err_len, "fused checkpoint launch: %s", cudaGetErrorString(e));
    return TIDE_ERR_CUDA;
  }
  return TIDE_OK;
}

}  // namespace tide
