// Paired-CTA tensor-core router (sm_100a: TMA + tcgen05.mma.cta_group::2).
//
// Same scores as tc_route_kernel (tc_checkpoint.cu) for 16-bit rows and a
// router width of 128, with the product taken the other way round and split
// over the two CTAs of a cluster:
//     D[row][unit] = x[row] . W'[unit]      M = 256 rows (128 per CTA),
//                                           N = 128 units (64 per CTA), K = 16
// A tcgen05.mma of cta_group::2 reads its A operand (the rows) from both
// CTAs' shared memory and its B operand (the folded weights W') half from
// each, and writes each CTA's 128 rows x 128 units into that CTA's TMEM.  So
// a pair streams W' once for both CTAs' rows: every CTA takes in half of W'
// per K chunk instead of all of it.  With the rows of one checkpoint spread
// over all SMs that halves the weight bytes, which the single-CTA router
// pays in full on every SM whatever its share of rows (its intake at 32768 x
// 4096 is 1.77 MB of rows plus 1 MiB of W' per SM).
//
// Scores: sigmoid(up_bias + sum_u up[u] * SiLU(z_u)), RMSNorm
// z_u = rstd * D[row][u], LayerNorm z_u = rstd * (D[row][u] - mean * colsum[u])
// + bias_proj[u] (python/TIDE/runtime.py:128-130, python/TIDE/router.py:18-19),
// each thread of the epilogue owning one row and all 128 units.
//
// Work split: the rows are cut into 32-row units; cluster (pair) p takes a
// contiguous, balanced range of units, walked in pair tiles of up to 16
// units (512 rows): the first ceil(n/2) units of a pair tile are CTA 0's,
// the rest CTA 1's.  Per CTA (512 threads):
//   warps 0, 2  TMA producers: per stage KC K chunks, warp 0 arms the stage
//               and loads this CTA's half of W' [64 units x 64 cols], warp 2
//               the x rows [rows x 64 cols] (boxes of 128, 64, 32 rows);
//   warp 1      TMEM (cta_group::2, both CTAs); in CTA 0 the pair's MMAs;
//   warps 4-11  row statistics from the x chunks (one row per thread);
//   warps 8-15  epilogue: warp 8 + 4m + q reads TMEM lanes 32q..32q+31 of
//               M block m (rows 128m + 32q + lane), all 128 units.
// Barriers: both CTAs' copies of a stage complete on CTA 0's `full` barrier
// (CTA 1 issues its copies with the cta_group::2 form, naming CTA 0's
// barrier), which CTA 0 arms for the pair's bytes; the MMA issuer waits on
// it alone.  One commit per stage, multicast to both CTAs' `mdone`, says
// the MMAs have read the stage.  The statistics warps read a stage after
// `full` (CTA 0) or after `mdone` (CTA 1, which cannot see CTA 0's barrier)
// and arrive on their CTA's `empty`; a producer refills a stage once its
// CTA's `mdone` and `empty` have completed.  The accumulator's `acc_full` is
// a multicast commit as well, and CTA 0's `acc_empty` counts the epilogue
// warps of both CTAs.  Every wait is bounded; on expiry the CTA raises
// TIDE_DEVERR_TIMEOUT and stops, and the two meet at the final cluster
// barrier before TMEM is released (a CTA whose peer stopped reaches it only
// after one of its own waits has run out, long after any copy it issued has
// landed).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>

#include "common.cuh"
#include "tc_checkpoint.cuh"
#include "tc_ptx.cuh"

namespace tide {

namespace pair {

constexpr int kUnit = 32;          // rows per scheduling unit
constexpr int kCtaUnits = 8;       // units per CTA per pair tile (2 M blocks)
constexpr int kPairUnits = 2 * kCtaUnits;
constexpr int kMRows = 128;        // rows per CTA per M block
constexpr int kN = 128;            // router units (MMA N)
constexpr int kHalfN = kN / 2;     // W' rows held by each CTA
constexpr int kK = 64;             // columns per chunk: 128 bytes of 16-bit data
constexpr int kThreads = 512;
constexpr int kMaxStages = 12;
constexpr int kMaxKc = 4;
constexpr int kMinStages = 3;
constexpr int kSmemBudget = 227 * 1024;
constexpr int kAux = 8192;
constexpr uint32_t kTmemCols = 512;  // two accumulator sets of two M blocks

struct Params {
  int64_t n_cap;
  const int32_t *n_dev;
  int H, norm_type;
  float eps, up_bias;
  const float *up, *colsum, *bias_proj;
  float *scores;
  float2 *row_stats;
  int32_t *err;
  uint32_t ring_bytes;
  uint4 *zero;
  int64_t zero_vec;
};

__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at this shared-memory offset in both CTAs of
// the pair when every MMA this thread issued so far has completed.
__device__ __forceinline__ void commit_both(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], m;\n\t}" ::"r"(ptx::smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   ptx::smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// 2-D tiled load into this CTA's shared memory whose completion is counted
// on a barrier of the leading CTA of the pair (a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_to_lead(void *dst, const void *tmap, uint32_t lead_bar,
                                                    int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(ptx::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(lead_bar), "r"(c0), "r"(c1)
      : "memory");
}
// Release-arrive on a barrier of the peer CTA (a shared::cluster address):
// this thread's earlier accesses happen before the peer's wait returns.
__device__ __forceinline__ void arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

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

// The pair's tile geometry, computed identically by both CTAs.
struct PairTile {
  int64_t u0;   // first unit of this CTA's rows in the tile
  int nu;       // this CTA's units (may be 0)
  int mblocks;  // M blocks the pair's MMAs cover (1 or 2)
};
__device__ __forceinline__ PairTile pair_tile(int64_t pu0, int64_t pu_end, uint32_t rank) {
  const int nup = (int)(pu_end - pu0 < kPairUnits ? pu_end - pu0 : kPairUnits);
  const int n0 = (nup + 1) / 2, n1 = nup / 2;
  PairTile t;
  t.u0 = pu0 + (rank ? n0 : 0);
  t.nu = rank ? n1 : n0;
  t.mblocks = (n0 * kUnit + kMRows - 1) / kMRows;
  return t;
}

}  // namespace pair

template <bool BF16, bool LAYER>
__global__ void __launch_bounds__(pair::kThreads, 1)
    tc_route_pair_kernel(const __grid_constant__ CUtensorMap tmap_x,
                         const __grid_constant__ CUtensorMap tmap_x_big,
                         const __grid_constant__ CUtensorMap tmap_x_mid,
                         const __grid_constant__ CUtensorMap tmap_w, pair::Params p) {
  using namespace pair;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_rank();  // 0: issues the pair's MMAs
  const bool lead = rank == 0;

  uint64_t *full = reinterpret_cast<uint64_t *>(smem);  // CTA 0: both CTAs' copies
  uint64_t *empty = full + kMaxStages;                  // this CTA's statistics warps
  uint64_t *mdone = empty + kMaxStages;                 // the pair's MMAs read the stage
  uint64_t *acc_full = mdone + kMaxStages;  // [2]
  uint64_t *acc_empty = acc_full + 2;       // [2] (CTA 0: both CTAs' epilogues)
  uint64_t *stat_full = acc_empty + 2;      // [2]
  uint64_t *stat_empty = stat_full + 2;     // [2]
  uint64_t *drain = stat_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  uint32_t *issued = reinterpret_cast<uint32_t *>(tmem_slot + 2);
  uint32_t *issued_x = reinterpret_cast<uint32_t *>(tmem_slot + 3);
  float *s_up = reinterpret_cast<float *>(tmem_slot + 4);  // [128]
  float *s_cs = s_up + kN;
  float *s_bp = s_cs + kN;
  float *s_stat = s_bp + kN;  // [2 slots][256 rows][rstd, mean]
  static_assert((3 * kMaxStages + 9) * 8 + 16 + 3 * kN * 4 + 2 * 256 * 2 * 4 <= kAux,
                "auxiliary shared-memory area");
  uint8_t *ring = smem + kAux;
  const int k_chunks = p.H / kK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxStages; ++s) {
      ptx::mbar_init(&full[s], 1);   // CTA 0's arming (for the pair's bytes)
      ptx::mbar_init(&empty[s], 8);  // 8 statistics warps
      ptx::mbar_init(&mdone[s], 1);  // one commit of the pair's MMAs
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&acc_full[a], 1);
      ptx::mbar_init(&acc_empty[a], 16);  // 8 epilogue warps of each CTA (used in CTA 0)
      ptx::mbar_init(&stat_full[a], 8);
      ptx::mbar_init(&stat_empty[a], 8);
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
    pair::tmem_alloc_pair(tmem_slot, kTmemCols);
    pair::tmem_relinquish_pair();
  }
  // both CTAs' barriers exist before either arrives on the other's
  ptx::tc_fence_before();
  ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  ptx::grid_dependency_wait();
  if (threadIdx.x == 0) ptx::grid_dependents_launch();

  int64_t n = p.n_cap;
  if (p.n_dev) {
    const int64_t nd = (int64_t)__ldg(p.n_dev);
    n = nd < 0 ? 0 : (nd > p.n_cap ? p.n_cap : nd);
  }
  const int64_t n_pairs = gridDim.x / 2, pair_id = blockIdx.x / 2;
  const int64_t units = (n + kUnit - 1) / kUnit;
  const int64_t pu_begin = pair_id * units / n_pairs;
  const int64_t pu_end = (pair_id + 1) * units / n_pairs;
  // stage geometry from the largest pair range: one K chunk is the A rows
  // of a CTA (whole M blocks, which the MMA reads in full) and its half of W'
  const int64_t max_pair_units = (units + n_pairs - 1) / n_pairs;
  const int max_tile = (int)(max_pair_units < kPairUnits ? max_pair_units : kPairUnits);
  const int max_mblocks = ((max_tile + 1) / 2 * kUnit + kMRows - 1) / kMRows;
  const uint32_t x_bytes = (uint32_t)(max_mblocks < 1 ? 1 : max_mblocks) * kMRows * 128;
  const uint32_t w_bytes = kHalfN * 128;
  const uint32_t chunk_bytes = x_bytes + w_bytes;
  int KC = 1;
  for (int c = kMaxKc; c > 1; c >>= 1)
    if (k_chunks % c == 0 && p.ring_bytes / ((uint32_t)c * chunk_bytes) >= (uint32_t)kMinStages) {
      KC = c;
      break;
    }
  const uint32_t w_off = (uint32_t)KC * x_bytes;
  const uint32_t stage_bytes = (uint32_t)KC * chunk_bytes;
  const int S_fit = (int)(p.ring_bytes / stage_bytes);
  const int S = S_fit > kMaxStages ? kMaxStages : S_fit;
  const int k_stages = k_chunks / KC;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------ TMA producers
    if (lane == 0) {
      const bool arm = warp == 0;
      const uint32_t lead_full0 = ptx::map_to_rank(ptx::smem_u32(&full[0]), 0);
      uint32_t it = 0;
      for (int64_t pu0 = pu_begin; pu0 < pu_end && !*abort_flag; pu0 += kPairUnits) {
        const PairTile tl = pair_tile(pu0, pu_end, rank);
        const PairTile t0 = pair_tile(pu0, pu_end, 0), t1 = pair_tile(pu0, pu_end, 1);
        const uint32_t pair_bytes = (uint32_t)KC * ((uint32_t)(t0.nu + t1.nu) * kUnit * 128 + 2 * w_bytes);
        const int nu = tl.nu;
        const int n_big = nu / (128 / kUnit);
        const bool mid = (nu % (128 / kUnit)) >= 64 / kUnit;
        const int u_mid = n_big * (128 / kUnit);
        const int u_small = u_mid + (mid ? 64 / kUnit : 0);
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (it >= (uint32_t)S && !(ptx::mbar_wait_cluster(&mdone[s], ph ^ 1u, abort_flag) &&
                                     ptx::mbar_wait(&empty[s], ph ^ 1u, abort_flag))) {
            raise_error(p.err, TIDE_DEVERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          uint8_t *st = ring + (size_t)s * stage_bytes;
          const uint32_t bar = lead_full0 + (uint32_t)s * 8u;  // CTA 0's full[s]
          if (arm) {
            if (lead) ptx::mbar_expect_tx(&full[s], pair_bytes);
            for (int c = 0; c < KC; ++c)
              pair::tma_load_2d_to_lead(st + w_off + (size_t)c * w_bytes, &tmap_w, bar,
                                        (ks * KC + c) * kK, (int)rank * kHalfN);
            *issued = it + 1;
          } else {
            for (int c = 0; c < KC; ++c) {
              const int col = (ks * KC + c) * kK;
              uint8_t *xc = st + (size_t)c * x_bytes;
              for (int j = 0; j < n_big; ++j)
                pair::tma_load_2d_to_lead(xc + (size_t)j * 128 * 128, &tmap_x_big, bar, col,
                                          (int)((tl.u0 + j * (128 / kUnit)) * kUnit));
              if (mid)
                pair::tma_load_2d_to_lead(xc + (size_t)u_mid * kUnit * 128, &tmap_x_mid, bar, col,
                                          (int)((tl.u0 + u_mid) * kUnit));
              if (u_small < nu)
                pair::tma_load_2d_to_lead(xc + (size_t)u_small * kUnit * 128, &tmap_x, bar, col,
                                          (int)((tl.u0 + u_small) * kUnit));
            }
            *issued_x = it + 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && lead) {
      // ------------------------------------------- the pair's MMA issuer
      uint32_t it = 0;
      int t_local = 0;
      bool ok = true;
      for (int64_t pu0 = pu_begin; pu0 < pu_end && ok && !*abort_flag;
           pu0 += kPairUnits, ++t_local) {
        const PairTile tl = pair_tile(pu0, pu_end, rank);
        const uint32_t idesc = ptx::f16_idesc(BF16, 2 * kMRows, kN);
        const int acc = t_local & 1;
        const uint32_t acc_ph = (uint32_t)(t_local >> 1) & 1u;
        if (t_local >= 2 && !ptx::mbar_wait_cluster(&acc_empty[acc], acc_ph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_acc = tmem_base + (uint32_t)(acc * 2 * kN);
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (!ptx::mbar_wait_cluster(&full[s], ph, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t st = ptx::smem_u32(ring + (size_t)s * stage_bytes);
          for (int c = 0; c < KC; ++c) {
            const uint32_t xs = st + (uint32_t)c * x_bytes;
            const uint32_t ws = st + w_off + (uint32_t)c * w_bytes;
            for (int m = 0; m < tl.mblocks; ++m) {
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t acc_in = (ks > 0 || c > 0 || k > 0) ? 1u : 0u;
                pair::mma_pair(d_acc + (uint32_t)(m * kN),
                               ptx::sw128_kmajor_desc(xs + (uint32_t)m * kMRows * 128 + 32u * k),
                               ptx::sw128_kmajor_desc(ws + 32u * k), idesc, acc_in);
              }
            }
          }
          pair::commit_both(&mdone[s]);
        }
        if (!ok) break;
        pair::commit_both(&acc_full[acc]);
      }
      if (!ok) {
        raise_error(p.err, TIDE_DEVERR_TIMEOUT);
        *abort_flag = 1;
      }
      pair::commit_both(drain);  // every MMA of the pair has finished once it completes
    }
  } else if (warp >= 4) {
    // ------------------------------------- row statistics and epilogue
    const bool do_stats = warp < 12;
    const bool do_epi = warp >= 8;
    {
      // per-unit vectors (every warp from 4 up), and this CTA's share of the
      // mover's workspace, cleared while the producers stream
      const int t1 = threadIdx.x - 128;  // 0..383
      for (int i = t1; i < kN; i += 384) {
        s_up[i] = p.up[i];
        s_cs[i] = p.colsum ? p.colsum[i] : 0.f;
        s_bp[i] = p.bias_proj ? p.bias_proj[i] : 0.f;
      }
      if (p.zero) {
        const int64_t per = (p.zero_vec + gridDim.x - 1) / gridDim.x;
        const int64_t z0 = (int64_t)blockIdx.x * per;
        const int64_t z1 = z0 + per < p.zero_vec ? z0 + per : p.zero_vec;
        for (int64_t i = z0 + t1; i < z1; i += 384) p.zero[i] = make_uint4(0, 0, 0, 0);
      }
      ptx::named_sync(2, 384);
    }
    const int t = threadIdx.x - 128;   // statistics row 0..255
    const int mb = (warp - 8) >> 2;    // epilogue M block
    const int q = warp & 3;            // TMEM lane quarter
    const int er = mb * kMRows + q * 32 + lane;  // epilogue row 0..255
    const uint32_t peer_acc_empty = ptx::map_to_rank(ptx::smem_u32(&acc_empty[0]), 0);
    uint32_t it = 0;
    int t_local = 0;
    bool ok = true;
    for (int64_t pu0 = pu_begin; pu0 < pu_end; pu0 += kPairUnits, ++t_local) {
      const PairTile tl = pair_tile(pu0, pu_end, rank);
      const int nu = tl.nu;
      const int buf = t_local & 1;
      if (do_stats && ok) {
        const bool live = (t >> 5) < nu;  // warp-uniform: a unit is one warp
        float ss0 = 0.f, ss1 = 0.f, sx0 = 0.f, sx1 = 0.f;
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          // CTA 0 reads a stage once it has landed; CTA 1 once the MMAs
          // have read it (its copies complete on CTA 0's barrier)
          if (!(lead ? ptx::mbar_wait_cluster(&full[s], ph, abort_flag)
                     : ptx::mbar_wait_cluster(&mdone[s], ph, abort_flag))) {
            ok = false;
            break;
          }
          if (live) {
            for (int c = 0; c < KC; ++c) {
              const uint8_t *row = ring + (size_t)s * stage_bytes + (size_t)c * x_bytes + (size_t)t * 128;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int unit = (j + lane) & 7;
                const uint4 v = *reinterpret_cast<const uint4 *>(row + (unit << 4));
                float f[8];
                pair::unpack8(v, f, BF16);
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
          float *st = s_stat + ((size_t)buf * 256 + t) * 2;
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
      // ---- epilogue of this tile (warps 8-15): one row per thread
      const int acc = t_local & 1;
      bool got = ok &&
                 ptx::mbar_wait(&stat_full[buf], (uint32_t)(t_local >> 1) & 1u, abort_flag) &&
                 ptx::mbar_wait_cluster(&acc_full[acc], (uint32_t)(t_local >> 1) & 1u, abort_flag);
      got = __all_sync(0xffffffffu, got);
      if (!got) { ok = false; break; }
      ptx::tc_fence_after();
      const float *stt = s_stat + (size_t)buf * 256 * 2;
      const float rstd = stt[er * 2], mean = stt[er * 2 + 1];
      float logit = 0.f;
      if (mb < tl.mblocks) {  // warp-uniform
        const uint32_t base = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 2 * kN + mb * kN);
#pragma unroll 1
        for (int c = 0; c < kN / 32; ++c) {
          float v[32];
          ptx::tmem_ld32(base + (uint32_t)(c * 32), v);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int u = c * 32 + j;
            const float z = LAYER ? fmaf(rstd, v[j] - mean * s_cs[u], s_bp[u]) : rstd * v[j];
            logit = fmaf(s_up[u], silu_tanh(z), logit);
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (lead) ptx::mbar_arrive(&acc_empty[acc]);
        else pair::arrive_remote(peer_acc_empty + (uint32_t)acc * 8u);
      }
      const int64_t row_lim_tile = (tl.u0 + nu) * kUnit;
      const int64_t row_lim = row_lim_tile < n ? row_lim_tile : n;
      const int64_t grow = tl.u0 * kUnit + er;
      if (er < nu * kUnit && grow < row_lim) {
        p.scores[grow] = sigmoid_f(p.up_bias + logit);
        if (p.row_stats) p.row_stats[grow] = make_float2(mean, rstd);
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&stat_empty[buf]);
    }
    if (!ok) {
      raise_error(p.err, TIDE_DEVERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag && lead) {
    // drain the pair's TMA loads still in flight (they complete on CTA 0's
    // barriers; phases CTA 0 never armed give up after the bound)
    const uint32_t n_issued = *issued > *issued_x ? *issued : *issued_x;
    volatile int never = 0;
    for (int s = 0; s < S; ++s) {
      if ((uint32_t)s >= n_issued) break;
      const uint32_t count = (n_issued - (uint32_t)s + (uint32_t)S - 1) / (uint32_t)S;
      ptx::mbar_wait_cluster(&full[s], (count - 1) & 1u, &never);
    }
  }
  if (threadIdx.x == 32) {
    // the pair's MMAs read both CTAs' stages and write both TMEMs: neither
    // CTA leaves before the last of them has completed
    volatile int never = 0;
    if (!ptx::mbar_wait_cluster(drain, 0, &never)) raise_error(p.err, TIDE_DEVERR_TIMEOUT);
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();
  ptx::tc_fence_after();
  if (warp == 1) pair::tmem_dealloc_pair(tmem_base, kTmemCols);
}

// ------------------------------------------------------------------ host
namespace {

int pair_sm_count() {
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

using PairKern = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, pair::Params);

PairKern pair_kernel(int dtype, bool layer) {
  if (dtype == TIDE_DTYPE_BF16)
    return layer ? tc_route_pair_kernel<true, true> : tc_route_pair_kernel<true, false>;
  return layer ? tc_route_pair_kernel<false, true> : tc_route_pair_kernel<false, false>;
}

}  // namespace

bool tc_pair_supported(const tide_checkpoint_args *a) {
  if (a->dtype != TIDE_DTYPE_BF16 && a->dtype != TIDE_DTYPE_F16) return false;
  if (a->bottleneck_dim != pair::kN) return false;
  return tc_supported(a);
}

int tc_route_pair_launch(const tide_checkpoint_args *a, float *scores, float2 *row_stats,
                         void *zero, size_t zero_bytes, cudaStream_t stream, char *err,
                         size_t err_len) {
  const int dt = a->dtype;
  CUtensorMap tx, txb, txm, tw;
  if (!tc_make_tmap(&tx, a->x, dt, (uint64_t)a->n_rows, (uint64_t)a->hidden_dim, pair::kUnit) ||
      !tc_make_tmap(&txb, a->x, dt, (uint64_t)a->n_rows, (uint64_t)a->hidden_dim, 128) ||
      !tc_make_tmap(&txm, a->x, dt, (uint64_t)a->n_rows, (uint64_t)a->hidden_dim, 64) ||
      !tc_make_tmap(&tw, a->folded, dt, (uint64_t)pair::kN, (uint64_t)a->hidden_dim, pair::kHalfN)) {
    snprintf(err, err_len, "paired tensor-core route: cuTensorMapEncodeTiled failed");
    return TIDE_ERR_CUDA;
  }
  pair::Params p{};
  p.n_cap = a->n_rows;
  p.n_dev = a->n_rows_dev;
  p.H = (int)a->hidden_dim;
  p.norm_type = a->norm_type;
  p.eps = a->eps;
  p.up_bias = a->up_bias;
  p.up = a->up;
  p.colsum = a->norm_type == TIDE_NORM_LAYER ? a->colsum : nullptr;
  p.bias_proj = a->norm_type == TIDE_NORM_LAYER ? a->bias_proj : nullptr;
  p.scores = scores;
  p.row_stats = row_stats;
  p.err = a->error_word;
  p.ring_bytes = (uint32_t)(pair::kSmemBudget - 1024 - pair::kAux);
  p.zero = static_cast<uint4 *>(zero);
  p.zero_vec = (int64_t)(zero_bytes / 16);
  const bool layer = a->norm_type == TIDE_NORM_LAYER;
  const PairKern fn = pair_kernel(dt, layer);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64][4] = {};
  static int max_pairs[64][4] = {};
  const int which = (dt == TIDE_DTYPE_BF16 ? 2 : 0) + (layer ? 1 : 0);
  cudaError_t e;
  if (dev < 0 || dev >= 64 || !attr_set[dev][which]) {
    e = cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             pair::kSmemBudget);
    if (e != cudaSuccess) {
      snprintf(err, err_len, "paired tensor-core route: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return TIDE_ERR_CUDA;
    }
    // how many pairs the device holds at once: the grid is one wave of them
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3((unsigned)(pair_sm_count() & ~1));
    q.blockDim = dim3(pair::kThreads);
    q.dynamicSmemBytes = pair::kSmemBudget;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    q.attrs = qa;
    q.numAttrs = 1;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, (const void *)fn, &q);
    if (e != cudaSuccess || clusters < 1) {
      snprintf(err, err_len, "paired tensor-core route: no CTA pair fits (%s)",
               e != cudaSuccess ? cudaGetErrorString(e) : "0 clusters");
      cudaGetLastError();
      return TIDE_ERR_UNSUPPORTED;
    }
    if (dev >= 0 && dev < 64) {
      attr_set[dev][which] = true;
      max_pairs[dev][which] = clusters;
    }
  }
  const int pairs_cap = (dev >= 0 && dev < 64) ? max_pairs[dev][which] : pair_sm_count() / 2;
  const int64_t units = (a->n_rows + pair::kUnit - 1) / pair::kUnit;
  const int64_t pairs_need = (units + 1) / 2;
  const int pairs = (int)(pairs_need < pairs_cap ? (pairs_need < 1 ? 1 : pairs_need) : pairs_cap);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(pair::kThreads);
  cfg.dynamicSmemBytes = pair::kSmemBudget;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, fn, tx, txb, txm, tw, p);
  if (e != cudaSuccess) {
    snprintf(err, err_len, "paired tensor-core route launch: %s", cudaGetErrorString(e));
    return TIDE_ERR_CUDA;
  }
  return TIDE_OK;
}

}  // namespace tide
