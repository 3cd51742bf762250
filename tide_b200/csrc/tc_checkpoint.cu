// Tensor-core router for the early-exit path (sm_100a: TMA + tcgen05).
//
// scores[i] = sigmoid(up_bias + sum_b up[b] * SiLU(z_ib)) with
//   RMSNorm:   z_ib = rstd_i * (x_i . W'_b)
//   LayerNorm: z_ib = rstd_i * (x_i . W'_b - mean_i * colsum_b) + bias_proj_b
// where W'[b, :] = down[b, :] * norm_weight (folded once, model dtype) so the
// norm never has to be materialised: the raw rows feed the tensor cores and
// a companion warpgroup computes each row's statistics from the same shared-
// memory tiles.  Reference semantics: python/TIDE/runtime.py:128-130 and
// python/TIDE/router.py:18-19.
//
// The product is taken transposed, D[unit][row] = W'[unit] . x[row], so one
// tcgen05.mma covers M = 128 units x N = 256 rows: half the instructions of
// row-major M = 128 tiles and fewer shared-memory operand bytes per FLOP.
//
// Persistent CTAs, one per SM.  The rows are cut into 32-row units and each
// CTA takes a contiguous, balanced range of units (so no SM does a whole
// extra tile), walked in tiles of up to 256 rows.  Per CTA:
//   warps 0, 2  TMA producers: per pipeline stage KC K-chunks of the tile,
//               x [rows x 64 cols] (boxes of 128, 64 and 32 rows; warp 2)
//               and W' [128 units x 64] (warp 0, which also arms the
//               stage), all with the 128-byte swizzle;
//   warp 1      TMEM owner and MMA issuer: 4 x tcgen05.mma (K = 16) per
//               stage and 128-unit block into an fp32 accumulator of 256
//               columns (double-buffered across tiles when TMEM holds two);
//   warps 4-11  row statistics from the x chunks (one row per thread),
//               handed to the epilogue per tile through a double-buffered
//               shared-memory slot;
//   warps 8-15  the epilogue (warps 8-11 after their statistics of the
//               tile), two groups of four warps, one per half of the
//               tile's rows: warp 8+4g+q reads units 32q..32q+31 of its rows
//               (tcgen05.ld), applies the norm scale and SiLU, weights by
//               up[unit], sums the 32 units of each row with a butterfly of
//               shuffles, then the four quarter warps' partial sums per row
//               meet in shared memory; writes the score and (mean, rstd).
// Launched as a programmatic dependent: barriers, TMEM and the tensor-map
// prefetch are set up before griddepcontrol.wait, so they overlap the end of
// the previous kernel; nothing global is read or written before it.  The
// producer starts loading right after it; the other warps fetch the per-unit
// vectors and clear the mover's workspace meanwhile (no separate memset).
// The survivors/exits are then moved by the stable-partition kernel.
//
// fp32 rows take the same pipeline with kind::tf32 MMAs and error-compensated
// products ("3xTF32"): each operand v is split as hi = v rounded to tf32 and
// lo = v - hi (exact), and D accumulates W'hi.xhi + W'lo.xhi + W'hi.xlo,
// which leaves out only W'lo.xlo and the tf32 rounding of the lo parts
// (about 2^-21 of each product) -- the fp32 score bar of 1e-5 holds, where a
// single tf32 product (2^-11) would not.  A K chunk is still 128 bytes of a
// row (32 fp32 columns), so the shared-memory layout and descriptors are the
// ones of the 16-bit case.  Warps 4-15 split each landed stage in place (hi
// over the loaded values, lo into the stage's second half, x and W' alike)
// while they take the row statistics; the MMA waits for that instead of the
// TMA.  Above H = 1024 the K range is accumulated in several TMEM
// accumulators (K groups) that the epilogue sums in fp32, since one
// accumulator over all of K loses about an ulp of its running sum per MMA.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "tc_checkpoint.cuh"
#include "tc_ptx.cuh"

namespace tide {

constexpr int kTcM = 128;         // router units per MMA (TMEM lanes)
constexpr int kTcUnit = 32;       // rows per scheduling unit / small TMA box
constexpr int kTcBigBox = 128;    // rows per large TMA box
constexpr int kTcMidBox = 64;     // rows per middle TMA box
constexpr int kTcTileUnits = 8;   // units per tile
constexpr int kTcTileRows = kTcUnit * kTcTileUnits;  // MMA N
constexpr int kTcK = 64;          // columns per chunk: 128 bytes of 16-bit data
constexpr int kTcThreads = 512;  // warps 0-1 TMA/MMA, 4-11 statistics, 8-15 epilogue
constexpr int kTcMaxStages = 12;
// K chunks per pipeline stage: the largest of 4, 2, 1 dividing the chunk
// count that still leaves kTcMinStages stages in the ring.  Every stage (one
// mbarrier phase) costs a fixed ~0.28 us on top of its bytes, so thin tiles
// move several K chunks per stage.
#ifndef TIDE_ROUTER_MAX_KC
#define TIDE_ROUTER_MAX_KC 4
#endif
#ifndef TIDE_ROUTER_MIN_STAGES
#define TIDE_ROUTER_MIN_STAGES 3
#endif
constexpr int kTcMaxKc = TIDE_ROUTER_MAX_KC;
constexpr int kTcMinStages = TIDE_ROUTER_MIN_STAGES;
constexpr int kTcSmemBudget = 227 * 1024;
// fp32 tile width in 32-row units: narrower tiles at larger H leave TMEM
// room for more K-group accumulators (2 at 256 rows, 4 at 128, 8 at 64), so
// the fp32 score error stays under 1e-5 to H = 8192 (the error of one
// accumulator grows with the K depth).
__host__ __device__ inline int f32_tile_units(int H) { return H <= 2048 ? 8 : (H <= 4096 ? 4 : 2); }
constexpr int kF32OneGroupMaxH = 1024;  // fp32 rows up to this H keep one K accumulator
constexpr int kTcAux = 12288;     // barriers, flags, per-unit vectors, row statistics, partials
static_assert((3 * kTcMaxStages + 9) * 8 + 16 + 3 * 256 * 4 + 2 * 256 * 2 * 4 + 4 * 256 * 4 +
                      8 * 4 <= kTcAux,
              "auxiliary shared-memory area");

struct TcRouteParams {
  int64_t n_cap;
  const int32_t *n_dev;
  int H, B, norm_type;
  float eps, up_bias;
  const float *up, *colsum, *bias_proj;
  float *scores;
  float2 *row_stats;
  int32_t *err;
  uint32_t ring_bytes;  // shared memory for the pipeline stages
  int a_tiles;   // 128-unit blocks of W' (1 for B <= 128, else 2)
  int w_rows;    // rows of one W' box: min(B, 128)
  int n_acc;     // accumulator sets in TMEM (2: double-buffered across tiles)
  uint32_t tmem_cols;
  uint4 *zero;        // stable-partition workspace the mover expects zeroed
  int64_t zero_vec;   // its size in 16-byte words
};

__device__ __forceinline__ void unpack8_16(const uint4 &v, float *f, bool bf16) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (bf16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
      float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
}

// Sum of v[0..31] over the 32 lanes of the warp, transposed: lane j returns
// sum over lanes of v[j] (a butterfly that halves the vector at each step,
// 31 shuffles in all).
__device__ __forceinline__ float transpose_sum32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

// v = hi + lo with hi = v rounded to tf32 (to nearest, ties away from zero:
// add half of the 13 dropped bits, then clear them) and lo = v - hi, exact
// because hi is within a factor of two of v.  Magnitudes that would round
// past the largest finite float (and Inf/NaN) are truncated instead.
__device__ __forceinline__ void split_tf32(float v, float &hi, float &lo) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t r = (b & 0x7fffffffu) < 0x7f7ff000u ? b + 0x1000u : b;
  hi = __uint_as_float(r & 0xffffe000u);
  lo = v - hi;
}
__device__ __forceinline__ void split_tf32_16(uint8_t *hi_at, uint8_t *lo_at) {
  float4 v = *reinterpret_cast<const float4 *>(hi_at), h, l;
  split_tf32(v.x, h.x, l.x);
  split_tf32(v.y, h.y, l.y);
  split_tf32(v.z, h.z, l.z);
  split_tf32(v.w, h.w, l.w);
  *reinterpret_cast<float4 *>(hi_at) = h;
  *reinterpret_cast<float4 *>(lo_at) = l;
}

template <bool BF16, bool LAYER, bool F32>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_route_kernel(const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_x_big,
                    const __grid_constant__ CUtensorMap tmap_x_mid,
                    const __grid_constant__ CUtensorMap tmap_w, TcRouteParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NA = p.n_acc, AT = p.a_tiles;
  // a K chunk is 128 bytes of a row: 64 16-bit or 32 fp32 columns
  constexpr int kCols = F32 ? 32 : kTcK;
  // units per tile; fp32 tiles are narrower at larger H, so that TMEM holds
  // several K-group accumulators (below)
  const int kTileMax = F32 ? f32_tile_units(p.H) : kTcTileUnits;
  // fp32 stages are twice as large: two of them (two K chunks each on thin
  // tiles; 256-row tiles) measured faster than more, smaller stages
  constexpr int kMinStages = F32 ? 2 : kTcMinStages;
  const uint32_t unit_bytes = kTcUnit * 128;
  const uint32_t w_tile_bytes = kTcM * 128;    // A operand: 128 units
  const uint32_t w_load_bytes = (uint32_t)AT * (uint32_t)p.w_rows * 128;
  // barriers and the small vectors first, the pipeline stages after them
  // (their size depends on the live row count, known only after the wait)
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kTcMaxStages;
  uint64_t *acc_full = empty + kTcMaxStages;  // [2] accumulator set written
  uint64_t *acc_empty = acc_full + 2;  // [2] accumulator set read
  uint64_t *stat_full = acc_empty + 2; // [2] statistics slot written
  uint64_t *stat_empty = stat_full + 2;// [2] statistics slot read
  uint64_t *drain = stat_empty + 2;
  uint64_t *conv = drain + 1;  // [kTcMaxStages] fp32: stage split into hi/lo
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(conv + kTcMaxStages);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  uint32_t *issued = reinterpret_cast<uint32_t *>(tmem_slot + 2);    // stages armed (warp 0)
  uint32_t *issued_x = reinterpret_cast<uint32_t *>(tmem_slot + 3);  // stages with x issued (warp 2)
  float *s_up = reinterpret_cast<float *>(tmem_slot + 4);  // [256], 0 beyond B
  float *s_cs = s_up + 256;
  float *s_bp = s_cs + 256;
  float *s_stat = s_bp + 256;  // [2 slots][256 rows][ss, sx]
  float *s_part = s_stat + 2 * kTcTileRows * 2;  // [4 warps][256 rows]
  volatile int *s_vote = reinterpret_cast<volatile int *>(s_part + 4 * kTcTileRows);  // [8]

  const int k_chunks = p.H / kCols;
  uint8_t *ring = smem + kTcAux;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcMaxStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      // MMA commit + 8 statistics warps; fp32: the MMA commit alone (the
      // MMAs wait for the split, the statistics warps' last use of a stage)
      ptx::mbar_init(&empty[s], F32 ? 1 : 1 + 8);
      ptx::mbar_init(&conv[s], 4 + 8);  // fp32: warps 4-15 split the stage
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&acc_full[a], 1);
      ptx::mbar_init(&acc_empty[a], 8);   // 8 epilogue warps
      ptx::mbar_init(&stat_full[a], 8);   // 8 statistics warps
      ptx::mbar_init(&stat_empty[a], 8);  // 8 epilogue warps
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    *issued = 0;
    *issued_x = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_x);
    ptx::prefetch_tmap(&tmap_x_big);
    ptx::prefetch_tmap(&tmap_x_mid);
    ptx::prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, p.tmem_cols);
    ptx::tmem_relinquish();
  }
  __syncthreads();
  ptx::grid_dependency_wait();
  if (threadIdx.x == 0) ptx::grid_dependents_launch();

  int64_t n = p.n_cap;
  if (p.n_dev) {
    int64_t nd = (int64_t)__ldg(p.n_dev);
    n = nd < 0 ? 0 : (nd > p.n_cap ? p.n_cap : nd);
  }
  // this CTA's balanced range of 32-row units
  const int64_t units = (n + kTcUnit - 1) / kTcUnit;
  const int64_t u_begin = (int64_t)blockIdx.x * units / gridDim.x;
  const int64_t u_end = ((int64_t)blockIdx.x + 1) * units / gridDim.x;
  // Stage geometry from the largest range of any CTA: one K chunk of the
  // tile is tile_units units of 32 rows (the MMA's N) plus the W' chunk; a
  // stage holds KC chunks [x_0 .. x_KC-1][W'_0 .. W'_KC-1], so a CTA with few
  // rows moves more bytes per stage and keeps the ring full.
  const int64_t max_units = (units + gridDim.x - 1) / gridDim.x;
  const int tile_units = max_units >= kTileMax ? kTileMax : (max_units < 1 ? 1 : (int)max_units);
  const uint32_t x_bytes = (uint32_t)tile_units * unit_bytes;  // one chunk of the B operand
  const uint32_t wc_bytes = (uint32_t)AT * w_tile_bytes;       // one chunk of the A operand
  // fp32 stages hold the lo parts in a second half of the same layout
  const uint32_t chunk_bytes = (F32 ? 2u : 1u) * (x_bytes + wc_bytes);
  int KC = 1;
  for (int c = kTcMaxKc; c > 1; c >>= 1)
    if (k_chunks % c == 0 && p.ring_bytes / ((uint32_t)c * chunk_bytes) >= (uint32_t)kMinStages) {
      KC = c;
      break;
    }
  const uint32_t w_off = (uint32_t)KC * x_bytes;  // W' chunks follow the x chunks
  const uint32_t lo_off = (uint32_t)KC * (x_bytes + wc_bytes);  // fp32: the lo half
  const uint32_t stage_bytes = (uint32_t)KC * chunk_bytes;
  const int S_fit = (int)(p.ring_bytes / stage_bytes);
  const int S = S_fit > kTcMaxStages ? kTcMaxStages : S_fit;
  const int k_stages = k_chunks / KC;
  // fp32: the K range is cut into KG groups, each accumulated from zero in
  // its own TMEM accumulator and summed in fp32 by the epilogue.  The
  // tensor core's fp32 accumulation loses about an ulp of the running sum per
  // MMA (measured: the score error of one accumulator over K grows linearly
  // with H, 5e-6 at H = 4096 and 1.4e-5 at 8192 for default-scale weights);
  // KG independent partial sums divide that by KG.  16-bit rows keep one,
  // and so do fp32 rows up to H = 1024 (4e-7 with one accumulator), which
  // keep two accumulator sets to overlap consecutive tiles instead.
  const bool k_groups = F32 && p.H > kF32OneGroupMaxH;
  const int acc_stride = k_groups ? tile_units * kTcUnit : kTcTileRows;  // TMEM columns per accumulator
  int KG = 1;
  if (k_groups) {
    KG = 512 / (NA * AT * acc_stride);
    KG = KG > 8 ? 8 : KG;
    KG = KG > k_stages ? k_stages : KG;
    KG = KG < 1 ? 1 : KG;
  }

  uint32_t tmem_base = 0;
  // the setup group: warps 1 and 3-15 (warps 0 and 2 are the producers)
  constexpr int kSetupThreads = kTcThreads - 64;
  if (warp != 0 && warp != 2) {
    // while the producers already stream: per-unit vectors, this CTA's
    // slice of the mover's workspace, zero padding of W' past B
    const int t1 = warp == 1 ? lane : threadIdx.x - 64;
    if (p.zero) {
      const int64_t per = (p.zero_vec + gridDim.x - 1) / gridDim.x;
      const int64_t z0 = (int64_t)blockIdx.x * per;
      const int64_t z1 = z0 + per < p.zero_vec ? z0 + per : p.zero_vec;
      for (int64_t i = z0 + t1; i < z1; i += kSetupThreads) p.zero[i] = make_uint4(0, 0, 0, 0);
    }
    for (int i = t1; i < 256; i += kSetupThreads) {
      const bool in = i < p.B;
      s_up[i] = in ? p.up[i] : 0.f;
      s_cs[i] = in && p.colsum ? p.colsum[i] : 0.f;
      s_bp[i] = in && p.bias_proj ? p.bias_proj[i] : 0.f;
    }
    if (p.w_rows < kTcM) {
      // W' rows past B are never loaded: zero them once in every stage so
      // the padded units contribute exactly 0 (the loads write other rows)
      for (int s = 0; s < S; ++s)
        for (int c = 0; c < KC; ++c) {
          uint4 *w = reinterpret_cast<uint4 *>(ring + (size_t)s * stage_bytes + w_off +
                                               (size_t)c * wc_bytes + (size_t)p.w_rows * 128);
          const int n16 = (kTcM - p.w_rows) * 128 / 16;
          for (int i = t1; i < n16; i += kSetupThreads) w[i] = make_uint4(0, 0, 0, 0);
        }
      ptx::fence_proxy_async();
    }
    ptx::tc_fence_before();
    ptx::named_sync(2, kSetupThreads);
    ptx::tc_fence_after();
    tmem_base = *tmem_slot;
  }

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------ TMA producers
    // Issuing a copy holds the issuing thread for a fixed time, so two
    // threads share each stage: warp 0 arms the stage for all its bytes and
    // loads the W' chunks, warp 2 loads the x chunks (boxes of 128, 64 and
    // 32 rows, at most three per chunk).  A copy may land before the stage
    // is armed; the barrier's transaction count absorbs that.
    if (lane == 0) {
      const bool arm = warp == 0;
      uint32_t it = 0;
      for (int64_t u0 = u_begin; u0 < u_end && !*abort_flag; u0 += kTileMax) {
        const int nu = (int)(u_end - u0 < kTileMax ? u_end - u0 : kTileMax);
        const int n_big = nu / (kTcBigBox / kTcUnit);
        const bool mid = (nu % (kTcBigBox / kTcUnit)) >= kTcMidBox / kTcUnit;
        const int u_mid = n_big * (kTcBigBox / kTcUnit);                  // first unit of the 64-row box
        const int u_small = u_mid + (mid ? kTcMidBox / kTcUnit : 0);      // first unit of the 32-row box
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (it >= (uint32_t)S && !ptx::mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
            raise_error(p.err, TIDE_DEVERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          uint8_t *st = ring + (size_t)s * stage_bytes;
          if (arm) {
            ptx::mbar_expect_tx(&full[s], (uint32_t)KC * ((uint32_t)nu * unit_bytes + w_load_bytes));
            for (int c = 0; c < KC; ++c)
              for (int a = 0; a < AT; ++a)
                ptx::tma_load_2d(st + w_off + (size_t)c * wc_bytes + (size_t)a * w_tile_bytes, &tmap_w,
                                 &full[s], (ks * KC + c) * kCols, a * kTcM);
            *issued = it + 1;
          } else {
            for (int c = 0; c < KC; ++c) {
              const int col = (ks * KC + c) * kCols;
              uint8_t *xc = st + (size_t)c * x_bytes;
              for (int j = 0; j < n_big; ++j)
                ptx::tma_load_2d(xc + (size_t)j * (kTcBigBox / kTcUnit) * unit_bytes, &tmap_x_big,
                                 &full[s], col, (int)((u0 + j * (kTcBigBox / kTcUnit)) * kTcUnit));
              if (mid)
                ptx::tma_load_2d(xc + (size_t)u_mid * unit_bytes, &tmap_x_mid, &full[s], col,
                                 (int)((u0 + u_mid) * kTcUnit));
              if (u_small < nu)
                ptx::tma_load_2d(xc + (size_t)u_small * unit_bytes, &tmap_x, &full[s], col,
                                 (int)((u0 + u_small) * kTcUnit));
            }
            *issued_x = it + 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = F32 ? ptx::tf32_idesc(kTcM, tile_units * kTcUnit)
                                 : ptx::f16_idesc(BF16, kTcM, tile_units * kTcUnit);
      uint32_t it = 0;
      int t_local = 0;
      bool ok = true;
      for (int64_t u0 = u_begin; u0 < u_end && ok && !*abort_flag;
           u0 += kTileMax, ++t_local) {
        const int acc = t_local % NA;
        const uint32_t acc_ph = (uint32_t)(t_local / NA) & 1u;
        if (t_local >= NA && !ptx::mbar_wait(&acc_empty[acc], acc_ph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * AT * KG * acc_stride);
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const int kg = ks * KG / k_stages;  // K group of this stage
          const bool group_start = ks == 0 || (ks - 1) * KG / k_stages != kg;
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (!ptx::mbar_wait(F32 ? &conv[s] : &full[s], ph, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t st = ptx::smem_u32(ring + (size_t)s * stage_bytes);
          for (int c = 0; c < KC; ++c) {
            const uint32_t xs = st + (uint32_t)c * x_bytes;
            const uint32_t ws = st + w_off + (uint32_t)c * wc_bytes;
            for (int a = 0; a < AT; ++a) {
              // four K steps of 32 bytes: 16 columns of kind::f16, 8 of tf32
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t wa = ws + (uint32_t)a * w_tile_bytes + 32u * k, xb = xs + 32u * k;
                const uint32_t d = d_tmem + (uint32_t)((a * KG + kg) * acc_stride);
                const uint32_t acc_in = (!group_start || c > 0 || k > 0) ? 1u : 0u;
                if constexpr (F32) {
                  ptx::mma_tf32_ss(d, ptx::sw128_kmajor_desc(wa), ptx::sw128_kmajor_desc(xb), idesc, acc_in);
                  ptx::mma_tf32_ss(d, ptx::sw128_kmajor_desc(wa + lo_off), ptx::sw128_kmajor_desc(xb),
                                   idesc, 1u);
                  ptx::mma_tf32_ss(d, ptx::sw128_kmajor_desc(wa), ptx::sw128_kmajor_desc(xb + lo_off),
                                   idesc, 1u);
                } else {
                  ptx::mma_f16_ss(d, ptx::sw128_kmajor_desc(wa), ptx::sw128_kmajor_desc(xb), idesc, acc_in);
                }
              }
            }
          }
          ptx::mma_commit(&empty[s]);
        }
        if (!ok) break;
        ptx::mma_commit(&acc_full[acc]);
      }
      if (!ok) {
        raise_error(p.err, TIDE_DEVERR_TIMEOUT);
        *abort_flag = 1;
      }
      // every MMA issued by this thread has finished once `drain` completes
      ptx::mma_commit(drain);
      volatile int never = 0;
      if (!ptx::mbar_wait(drain, 0, &never)) raise_error(p.err, TIDE_DEVERR_TIMEOUT);
    }
  } else if (warp >= 4) {
    // ------------------------------------- row statistics and epilogue
    // Statistics: thread t of warps 4-11 owns row t of the tile and reads
    // all eight 16-byte units of its chunk row, lane-rotated so a warp's
    // reads of the swizzled tile hit distinct banks (the sum is order-free
    // within a row).  Epilogue: warp 8 + 4g + q reads TMEM lanes 32q..32q+31
    // (units a*128 + 32q + lane) of the rows in chunks 4g..4g+3.  Warps 8-11
    // do both, in that order per tile: while the rows stream they have no
    // epilogue to run (a CTA's range is one tile up to 37888 rows), and eight
    // statistics warps keep each stage's release short.
    // fp32: warps 4-11 take the statistics and split the x chunks, warps
    // 4-15 the W' chunks, warps 8-15 before their epilogue of each tile.
    const bool do_stats = warp < 12;
    const bool do_epi = warp >= 8;
    const int t = threadIdx.x - 128;   // statistics row 0..255
    const int q = warp & 3;
    const int g = (warp - 8) >> 2;
    const int et = threadIdx.x - 256;  // 0..255 in the epilogue
    uint32_t it = 0;
    int t_local = 0;
    bool ok = true;
    for (int64_t u0 = u_begin; u0 < u_end; u0 += kTileMax, ++t_local) {
      const int nu = (int)(u_end - u0 < kTileMax ? u_end - u0 : kTileMax);
      const int buf = t_local & 1;
      if constexpr (F32) {
        if (ok) {
          // warps 4-11: the x rows.  A tile of 32/64/(96, 128)/(160-256) rows
          // gets 8/4/2/1 threads per row, each on 1/2/4/8 of the row's eight
          // 16-byte units (lane-rotated by row: distinct banks in each
          // quarter warp).  Statistics: per-chunk sums in fp32, across chunks
          // in fp64, over the row's threads with shuffles at the end of the
          // tile.  LayerNorm sums x - x[0], so a large mean does not cancel
          // the variance away.  Then warps 4-15 split the W' chunks together.
          const bool xg = warp < 12;
          const int k = threadIdx.x - 128;  // 0..383
          const int tpr = tile_units == 1 ? 8 : (tile_units == 2 ? 4 : (tile_units <= 4 ? 2 : 1));
          const int upt = 8 / tpr;
          const int r = k / tpr, part = k % tpr;
          const bool live = xg && r < nu * kTcUnit;
          double ssd = 0.0, sxd = 0.0;
          float shift = 0.f;
          for (int ks = 0; ks < k_stages; ++ks, ++it) {
            const uint32_t s = it % S, ph = (it / S) & 1u;
            if (!ptx::mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
            uint8_t *stg = ring + (size_t)s * stage_bytes;
            for (int c = 0; c < KC; ++c) {
              if (LAYER && ks == 0 && c == 0) {
                // the row's first column: 16-byte unit 0, at (0 ^ row) of the
                // swizzle; read by every thread of the row before any of them
                // writes its hi parts in place (a row's threads share a warp)
                if (live) shift = *reinterpret_cast<const float *>(stg + (size_t)r * 128 + ((r & 7) << 4));
                __syncwarp();
              }
              if (live) {
                uint8_t *row = stg + (size_t)c * x_bytes + (size_t)r * 128;
                float ss0 = 0.f, ss1 = 0.f, sx0 = 0.f, sx1 = 0.f;
                for (int j = 0; j < upt; ++j) {
                  uint8_t *at = row + (((part * upt + j + r) & 7) << 4);
                  const float4 v = *reinterpret_cast<const float4 *>(at);
                  if (LAYER) {
                    const float d0 = v.x - shift, d1 = v.y - shift, d2 = v.z - shift, d3 = v.w - shift;
                    ss0 = fmaf(d0, d0, fmaf(d2, d2, ss0));
                    ss1 = fmaf(d1, d1, fmaf(d3, d3, ss1));
                    sx0 += d0 + d2;
                    sx1 += d1 + d3;
                  } else {
                    ss0 = fmaf(v.x, v.x, fmaf(v.z, v.z, ss0));
                    ss1 = fmaf(v.y, v.y, fmaf(v.w, v.w, ss1));
                  }
                  split_tf32_16(at, at + lo_off);
                }
                ssd += (double)(ss0 + ss1);
                sxd += (double)(sx0 + sx1);
              }
              uint8_t *w = stg + w_off + (size_t)c * wc_bytes;
              for (int i = k; i < AT * (kTcM * 128 / 16); i += 384)
                split_tf32_16(w + (size_t)i * 16, w + lo_off + (size_t)i * 16);
            }
            // the MMAs read the split through the async proxy
            ptx::fence_proxy_async();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&conv[s]);
          }
          if (xg) {
            // a row's threads are adjacent lanes (tpr divides 32)
            for (int off = 1; off < tpr; off <<= 1) {
              ssd += __shfl_xor_sync(0xffffffffu, ssd, off);
              sxd += __shfl_xor_sync(0xffffffffu, sxd, off);
            }
            if (ok && t_local >= 2 &&
                !ptx::mbar_wait(&stat_empty[buf], ((uint32_t)(t_local >> 1) & 1u) ^ 1u, abort_flag))
              ok = false;
            if (ok) {
              if (part == 0) {
                float *st = s_stat + ((size_t)buf * kTcTileRows + r) * 2;
                const double inv_h = 1.0 / (double)p.H;
                if (!LAYER) {
                  st[0] = rsqrt_rn((float)(ssd * inv_h) + p.eps);
                  st[1] = 0.f;
                } else {
                  const double md = sxd * inv_h;
                  const double var = ssd * inv_h - md * md;
                  st[0] = rsqrt_rn((float)(var > 0.0 ? var : 0.0) + p.eps);
                  st[1] = (float)((double)shift + md);
                }
              }
              __syncwarp();
              if (lane == 0) ptx::mbar_arrive(&stat_full[buf]);
            }
          }
        }
      } else if (do_stats && ok) {
        const bool live = (t >> 5) < nu;  // warp-uniform: a unit is one warp
        float ss0 = 0.f, ss1 = 0.f, sx0 = 0.f, sx1 = 0.f;
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (!ptx::mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          if (live) {
            for (int c = 0; c < KC; ++c) {
              const uint8_t *row =
                  ring + (size_t)s * stage_bytes + (size_t)c * x_bytes + (size_t)t * 128;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int unit = (j + lane) & 7;
                const uint4 v = *reinterpret_cast<const uint4 *>(row + (unit << 4));
                float f[8];
                unpack8_16(v, f, BF16);
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                  ss0 = fmaf(f[e], f[e], ss0);
                  ss1 = fmaf(f[e + 1], f[e + 1], ss1);
                  if (LAYER) { sx0 += f[e]; sx1 += f[e + 1]; }
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&empty[s]);
        }
        if (ok && t_local >= 2 &&
            !ptx::mbar_wait(&stat_empty[buf], ((uint32_t)(t_local >> 1) & 1u) ^ 1u, abort_flag))
          ok = false;
        if (ok) {
          float *st = s_stat + ((size_t)buf * kTcTileRows + t) * 2;
          const float ssum = ss0 + ss1, xsum = sx0 + sx1;
          if (!LAYER) {
            st[0] = rsqrt_rn(ssum / (float)p.H + p.eps);
            st[1] = 0.f;
          } else {
            const float mean = xsum / (float)p.H;
            const float var = fmaxf(ssum / (float)p.H - mean * mean, 0.f);
            st[0] = rsqrt_rn(var + p.eps);
            st[1] = mean;
          }
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&stat_full[buf]);
        }
      }
      if (!do_epi) {
        if (!ok) break;
        continue;
      }
      // ---- epilogue of this tile (warps 8-15)
      const int acc = t_local % NA;
      bool got = ok &&
                 ptx::mbar_wait(&stat_full[buf], (uint32_t)(t_local >> 1) & 1u, abort_flag) &&
                 ptx::mbar_wait(&acc_full[acc], (uint32_t)(t_local / NA) & 1u, abort_flag);
      // the eight epilogue warps vote and leave together, so each named
      // barrier below is reached by all of them or by none
      got = __all_sync(0xffffffffu, got);
      if (lane == 0) s_vote[warp - 8] = got ? 1 : 0;
      ptx::named_sync(1, 256);
      bool all = true;
#pragma unroll
      for (int w = 0; w < 8; ++w) all = all && s_vote[w] != 0;
      if (!all) { ok = false; break; }
      ptx::tc_fence_after();
      const float *st = s_stat + (size_t)buf * kTcTileRows * 2;
      float part[4] = {0.f, 0.f, 0.f, 0.f};
      for (int a = 0; a < AT; ++a) {
        const int u = a * kTcM + q * 32 + lane;
        const float up = s_up[u], cs = s_cs[u], bp = s_bp[u];
        const uint32_t base = tmem_base + ((uint32_t)(q * 32) << 16) +
                              (uint32_t)((acc * AT + a) * KG * acc_stride);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = g * 4 + cc;
          if (c >= nu) break;  // warp-uniform
          float v[32];
          ptx::tmem_ld32(base + (uint32_t)(c * 32), v);
          if constexpr (F32) {
            for (int kg = 1; kg < KG; ++kg) {  // the K groups' partial sums, in order
              float w[32];
              ptx::tmem_ld32(base + (uint32_t)(kg * acc_stride + c * 32), w);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += w[j];
            }
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float rstd = st[(c * 32 + j) * 2];
            float z;
            if (!LAYER)
              z = rstd * v[j];
            else
              z = fmaf(rstd, v[j] - st[(c * 32 + j) * 2 + 1] * cs, bp);
            // fp32 rows: SiLU to ~1e-6 relative (the fp32 score bar is
            // 1e-5); the one-tanh form (~5e-4) serves the 1e-2 bar of 16-bit rows
            if constexpr (F32)
              v[j] = up * silu_fast(z);
            else
              v[j] = up * silu_tanh(z);
          }
          part[cc] += transpose_sum32(v, lane);
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&acc_empty[acc]);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        if (g * 4 + cc < nu) s_part[q * kTcTileRows + (g * 4 + cc) * 32 + lane] = part[cc];
      ptx::named_sync(1, 256);
      const int64_t row_lim_tile = (u0 + nu) * kTcUnit;
      const int64_t row_lim = row_lim_tile < n ? row_lim_tile : n;
      for (int r = et; r < nu * kTcUnit; r += 256) {
        const float logit = p.up_bias + ((s_part[r] + s_part[kTcTileRows + r]) +
                                         (s_part[2 * kTcTileRows + r] + s_part[3 * kTcTileRows + r]));
        const int64_t grow = u0 * kTcUnit + r;
        if (grow < row_lim) {
          p.scores[grow] = sigmoid_f(logit);
          if (p.row_stats) p.row_stats[grow] = make_float2(st[r * 2 + 1], st[r * 2]);
        }
      }
      ptx::named_sync(1, 256);  // s_part and the statistics slot are free again
      if (lane == 0) ptx::mbar_arrive(&stat_empty[buf]);
    }
    if (!ok) {
      raise_error(p.err, TIDE_DEVERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // drain the TMA loads still in flight before the CTA exits
    // a stage either producer touched (the other may have stopped first:
    // then its phase never completes and the bounded wait gives up)
    const uint32_t n_issued = *issued > *issued_x ? *issued : *issued_x;
    volatile int never = 0;
    for (int s = 0; s < S; ++s) {
      if ((uint32_t)s >= n_issued) break;
      const uint32_t count = (n_issued - (uint32_t)s + (uint32_t)S - 1) / (uint32_t)S;
      ptx::mbar_wait(&full[s], (count - 1) & 1u, &never);
    }
  }
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

// ------------------------------------------------------------------ host
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

}  // namespace

// A [rows, cols] row-major matrix of `dtype` (TIDE_DTYPE_*), read in boxes
// of 128 bytes of a row (64 16-bit or 32 fp32 columns) by box_rows rows.
bool tc_make_tmap(CUtensorMap *m, const void *base, int dtype, uint64_t rows, uint64_t cols,
                  uint32_t box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const uint64_t esize = dtype == TIDE_DTYPE_F32 ? 4 : 2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * esize};
  cuuint32_t box[2] = {(cuuint32_t)(128 / esize), box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType t = dtype == TIDE_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                : dtype == TIDE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(m, t, 2, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace {

bool make_tmap(CUtensorMap *m, const void *base, int dtype, uint64_t rows, uint64_t cols,
               uint32_t box_rows) {
  return tc_make_tmap(m, base, dtype, rows, cols, box_rows);
}

// Which router the split path runs for 16-bit rows of router width 128: the
// single-CTA kernel (default) or the paired-CTA one (TIDE_ROUTER=pair).  The
// pair takes in 27 % fewer bytes per SM (half of W' each) but measured no
// faster: 38.5 against 37.3 us at 16384 x 4096 (DRAM 44 % busy in both),
// 149 against 146 us at 32768 rows, equal at 1M rows; the router is bound by
// its stage round trip, not by its intake.
bool pair_router_enabled() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("TIDE_ROUTER");
    v = (e && strcmp(e, "pair") == 0) ? 1 : 0;
  }
  return v == 1;
}

// 128-unit blocks of W' (the MMA's M), each with a 256-column accumulator;
// two accumulator sets in TMEM's 512 columns when one block covers B.
int a_tiles_for(int B) { return B <= kTcM ? 1 : 2; }
int n_acc_for(int B) { return a_tiles_for(B) == 1 ? 2 : 1; }


int sm_count() {
  static int n[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

}  // namespace

const char *tc_unsupported_reason(const tide_checkpoint_args *a) {
  if (a->dtype != TIDE_DTYPE_BF16 && a->dtype != TIDE_DTYPE_F16 && a->dtype != TIDE_DTYPE_F32)
    return "bad dtype";
  if (!a->folded) return "no folded router weights";
  // a K chunk is 128 bytes of a row
  if (a->dtype == TIDE_DTYPE_F32 && a->hidden_dim % 32 != 0) return "hidden_dim is not a multiple of 32";
  if (a->dtype != TIDE_DTYPE_F32 && a->hidden_dim % kTcK != 0) return "hidden_dim is not a multiple of 64";
  if (a->bottleneck_dim < 1 || a->bottleneck_dim > 256) return "bottleneck_dim not in [1, 256]";
  if (a->norm_type == TIDE_NORM_LAYER && !a->colsum) return "LayerNorm needs colsum";
  if (a->n_rows < 1) return "no rows";
  if (((uintptr_t)a->x & 15u) || ((uintptr_t)a->folded & 15u)) return "x/folded not 16-byte aligned";
  if (a->n_rows > (int64_t)1 << 31) return "too many rows";
  return nullptr;
}

bool tc_supported(const tide_checkpoint_args *a) { return tc_unsupported_reason(a) == nullptr; }

size_t tc_workspace_bytes(int64_t) { return 0; }

int tc_route_launch(const tide_checkpoint_args *a, float *scores, float2 *row_stats,
                    void *zero, size_t zero_bytes, cudaStream_t stream, char *err,
                    size_t err_len) {
  if (pair_router_enabled() && tc_pair_supported(a)) {
    const int rc = tc_route_pair_launch(a, scores, row_stats, zero, zero_bytes, stream, err, err_len);
    if (rc != TIDE_ERR_UNSUPPORTED) return rc;
    err[0] = '\0';  // no CTA pair fits on this device: the single-CTA router runs
  }
  const int dt = a->dtype;
  const int B = (int)a->bottleneck_dim;
  const int w_rows = B < kTcM ? B : kTcM;
  CUtensorMap tx, txb, txm, tw;
  if (!make_tmap(&tx, a->x, dt, (uint64_t)a->n_rows, (uint64_t)a->hidden_dim, kTcUnit) ||
      !make_tmap(&txb, a->x, dt, (uint64_t)a->n_rows, (uint64_t)a->hidden_dim, kTcBigBox) ||
      !make_tmap(&txm, a->x, dt, (uint64_t)a->n_rows, (uint64_t)a->hidden_dim, kTcMidBox) ||
      !make_tmap(&tw, a->folded, dt, (uint64_t)B, (uint64_t)a->hidden_dim, (uint32_t)w_rows)) {
    snprintf(err, err_len, "tensor-core route: cuTensorMapEncodeTiled failed");
    return TIDE_ERR_CUDA;
  }
  TcRouteParams p{};
  p.n_cap = a->n_rows;
  p.n_dev = a->n_rows_dev;
  p.H = (int)a->hidden_dim;
  p.B = B;
  p.norm_type = a->norm_type;
  p.eps = a->eps;
  p.up_bias = a->up_bias;
  p.up = a->up;
  p.colsum = a->norm_type == TIDE_NORM_LAYER ? a->colsum : nullptr;
  p.bias_proj = a->norm_type == TIDE_NORM_LAYER ? a->bias_proj : nullptr;
  p.scores = scores;
  p.row_stats = row_stats;
  p.err = a->error_word;
  p.ring_bytes = (uint32_t)(kTcSmemBudget - 1024 - kTcAux);
  p.a_tiles = a_tiles_for(B);
  p.w_rows = w_rows;
  // fp32 above H = 1024: TMEM holds K-group accumulators instead of two sets
  p.n_acc = (dt == TIDE_DTYPE_F32 && a->hidden_dim > kF32OneGroupMaxH) ? 1 : n_acc_for(B);
  p.tmem_cols = 512;
  p.zero = static_cast<uint4 *>(zero);
  p.zero_vec = (int64_t)(zero_bytes / 16);
  const size_t smem = kTcSmemBudget;
  const int64_t units = (a->n_rows + kTcUnit - 1) / kTcUnit;
  const int grid = (int)(units < sm_count() ? units : sm_count());
  cudaError_t e;
  // the opt-in shared memory size is raised once per kernel to the budget
  const bool layer = a->norm_type == TIDE_NORM_LAYER;
  using Kern = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, TcRouteParams);
  // [dtype][layer]: fp32, fp16, bf16 (TIDE_DTYPE_* order)
  static const Kern kernels[3][2] = {
      {tc_route_kernel<false, false, true>, tc_route_kernel<false, true, true>},
      {tc_route_kernel<false, false, false>, tc_route_kernel<false, true, false>},
      {tc_route_kernel<true, false, false>, tc_route_kernel<true, true, false>}};
  const Kern fn = kernels[dt][layer ? 1 : 0];
  static bool attr_set[64][6] = {};
  const int which = dt * 2 + (layer ? 1 : 0);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev][which]) {
    e = cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBudget);
    if (e != cudaSuccess) {
      snprintf(err, err_len, "tensor-core route: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return TIDE_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) attr_set[dev][which] = true;
  }
  // programmatic dependent launch: the prologue overlaps the previous kernel
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, fn, tx, txb, txm, tw, p);
  if (e != cudaSuccess) {
    snprintf(err, err_len, "tensor-core route launch: %s", cudaGetErrorString(e));
    return TIDE_ERR_CUDA;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, err_len, "tensor-core route launch: %s", cudaGetErrorString(e));
    return TIDE_ERR_CUDA;
  }
  return TIDE_OK;
}

}  // namespace tide
