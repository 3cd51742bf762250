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
// Persistent CTAs, one per SM.  The rows are cut into 32-row units and each
// CTA takes a contiguous, balanced range of units (so no SM does a whole
// extra tile), walked in tiles of up to 256 rows.  Per CTA:
//   warp 0      TMA producer: per pipeline stage, one [32 rows x 64 cols]
//               box per unit of the tile plus the W' chunk [B x 64]
//               (128-byte swizzle); the W' chunk is shared by both halves;
//   warp 1      TMEM owner and MMA issuer: per stage and 128-row half,
//               4 x tcgen05.mma (K = 16) into that half's fp32 accumulator
//               of B columns (double-buffered across tiles when TMEM holds
//               four);
//   warps 4-11  row statistics from the x chunks (one thread per row),
//               handed to the epilogue per tile through a double-buffered
//               shared-memory slot;
//   warps 12-15 the epilogue: tcgen05.ld of the accumulator rows, SiLU, up
//               projection, sigmoid; writes the score and (mean, rstd).  It
//               runs beside the statistics so the ring never waits for it.
// The survivors/exits are then moved by the stable-partition kernel.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>

#include "common.cuh"
#include "tc_checkpoint.cuh"
#include "tc_ptx.cuh"

namespace tide {

constexpr int kTcM = 128;         // rows per MMA half (TMEM lanes)
constexpr int kTcUnit = 32;       // rows per TMA box / scheduling unit
constexpr int kTcTileUnits = 8;   // units per tile: two 128-row halves
constexpr int kTcTileRows = kTcUnit * kTcTileUnits;
constexpr int kTcK = 64;          // columns per chunk: 128 bytes of 16-bit data
constexpr int kTcThreads = 512;  // warps 0-1 TMA/MMA, 4-11 statistics, 12-15 epilogue
constexpr int kTcMaxStages = 8;
constexpr int kTcSmemBudget = 227 * 1024;
constexpr int kTcAux = 8192;      // barriers, flags, per-unit vectors, row statistics

struct TcRouteParams {
  int64_t n_cap;
  const int32_t *n_dev;
  int H, B, norm_type;
  float eps, up_bias;
  const float *up, *colsum, *bias_proj;
  float *scores;
  float2 *row_stats;
  int32_t *err;
  int stages;
  int n_acc;  // accumulator sets in TMEM (2: double-buffered across tiles)
  uint32_t tmem_cols;
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

template <bool BF16, bool LAYER>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_route_kernel(const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_w, TcRouteParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages, B = p.B, NA = p.n_acc;
  const uint32_t unit_bytes = kTcUnit * kTcK * 2;
  const uint32_t a_bytes = kTcTileRows * kTcK * 2;
  const uint32_t b_bytes = (uint32_t)B * kTcK * 2;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * stage_bytes);
  uint64_t *empty = full + S;
  uint64_t *acc_full = empty + S;      // [2] accumulator set written
  uint64_t *acc_empty = acc_full + 2;  // [2] accumulator set read
  uint64_t *stat_full = acc_empty + 2; // [2] statistics slot written
  uint64_t *stat_empty = stat_full + 2;// [2] statistics slot read
  uint64_t *drain = stat_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  uint32_t *issued = reinterpret_cast<uint32_t *>(tmem_slot + 2);
  float *s_up = reinterpret_cast<float *>(tmem_slot + 4);
  float *s_cs = s_up + 256;
  float *s_bp = s_cs + 256;
  float *s_stat = s_bp + 256;  // [2 slots][256 rows][ss, sx]

  int64_t n = p.n_cap;
  if (p.n_dev) {
    int64_t nd = (int64_t)__ldg(p.n_dev);
    n = nd < 0 ? 0 : (nd > p.n_cap ? p.n_cap : nd);
  }
  // this CTA's balanced range of 32-row units
  const int64_t units = (n + kTcUnit - 1) / kTcUnit;
  const int64_t u_begin = (int64_t)blockIdx.x * units / gridDim.x;
  const int64_t u_end = ((int64_t)blockIdx.x + 1) * units / gridDim.x;
  const int k_chunks = p.H / kTcK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1 + 8);  // MMA commit + 8 statistics warps
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&acc_full[a], 1);
      ptx::mbar_init(&acc_empty[a], 4);   // 4 epilogue warps
      ptx::mbar_init(&stat_full[a], 8);   // 8 statistics warps
      ptx::mbar_init(&stat_empty[a], 4);  // 4 epilogue warps
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    *issued = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async();
  }
  for (int i = threadIdx.x; i < B; i += kTcThreads) {
    s_up[i] = p.up[i];
    s_cs[i] = p.colsum ? p.colsum[i] : 0.f;
    s_bp[i] = p.bias_proj ? p.bias_proj[i] : 0.f;
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, p.tmem_cols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      ptx::prefetch_tmap(&tmap_x);
      ptx::prefetch_tmap(&tmap_w);
      uint32_t it = 0;
      for (int64_t u0 = u_begin; u0 < u_end && !*abort_flag; u0 += kTcTileUnits) {
        const int nu = (int)(u_end - u0 < kTcTileUnits ? u_end - u0 : kTcTileUnits);
        for (int kc = 0; kc < k_chunks; ++kc, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (it >= (uint32_t)S && !ptx::mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
            raise_error(p.err, TIDE_DEVERR_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          uint8_t *st = smem + (size_t)s * stage_bytes;
          ptx::mbar_expect_tx(&full[s], (uint32_t)nu * unit_bytes + b_bytes);
          ptx::tma_load_2d(st + a_bytes, &tmap_w, &full[s], kc * kTcK, 0);
          for (int j = 0; j < nu; ++j)
            ptx::tma_load_2d(st + (size_t)j * unit_bytes, &tmap_x, &full[s], kc * kTcK,
                             (int)((u0 + j) * kTcUnit));
          *issued = it + 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::f16_idesc(BF16, kTcM, B);
      uint32_t it = 0;
      int t_local = 0;
      bool ok = true;
      for (int64_t u0 = u_begin; u0 < u_end && ok && !*abort_flag;
           u0 += kTcTileUnits, ++t_local) {
        const int nu = (int)(u_end - u0 < kTcTileUnits ? u_end - u0 : kTcTileUnits);
        const int halves = nu > kTcTileUnits / 2 ? 2 : 1;
        const int acc = t_local % NA;
        const uint32_t acc_ph = (uint32_t)(t_local / NA) & 1u;
        if (t_local >= NA && !ptx::mbar_wait(&acc_empty[acc], acc_ph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 2 * B);
        for (int kc = 0; kc < k_chunks; ++kc, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1u;
          if (!ptx::mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t a0 = ptx::smem_u32(smem + (size_t)s * stage_bytes);
          const uint32_t b0 = a0 + a_bytes;
          for (int h = 0; h < halves; ++h) {
#pragma unroll
            for (int k = 0; k < kTcK / 16; ++k) {
              ptx::mma_f16_ss(d_tmem + (uint32_t)(h * B),
                              ptx::sw128_kmajor_desc(a0 + (uint32_t)h * (kTcM * 128) + 32u * k),
                              ptx::sw128_kmajor_desc(b0 + 32u * k), idesc,
                              (kc > 0 || k > 0) ? 1u : 0u);
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
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------- row statistics
    // thread t of warps 4-11 owns row t of the tile and reads all eight
    // 16-byte units of its chunk row, lane-rotated so a warp's reads of the
    // swizzled tile hit distinct banks (the sum is order-free within a row).
    const int t = threadIdx.x - 128;
    uint32_t it = 0;
    int t_local = 0;
    bool ok = true;
    for (int64_t u0 = u_begin; u0 < u_end && ok; u0 += kTcTileUnits, ++t_local) {
      const int nu = (int)(u_end - u0 < kTcTileUnits ? u_end - u0 : kTcTileUnits);
      const bool live = (t >> 5) < nu;  // warp-uniform: a unit is one warp
      float ss0 = 0.f, ss1 = 0.f, sx0 = 0.f, sx1 = 0.f;
      for (int kc = 0; kc < k_chunks; ++kc, ++it) {
        const uint32_t s = it % S, ph = (it / S) & 1u;
        if (!ptx::mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
        if (live) {
          const uint8_t *row = smem + (size_t)s * stage_bytes + (size_t)t * 128;
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
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[s]);
      }
      if (!ok) break;
      const int buf = t_local & 1;
      if (t_local >= 2 &&
          !ptx::mbar_wait(&stat_empty[buf], ((uint32_t)(t_local >> 1) & 1u) ^ 1u, abort_flag)) {
        ok = false;
        break;
      }
      float *st = s_stat + ((size_t)buf * kTcTileRows + t) * 2;
      st[0] = ss0 + ss1;
      st[1] = sx0 + sx1;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&stat_full[buf]);
    }
    if (!ok) {
      raise_error(p.err, TIDE_DEVERR_TIMEOUT);
      *abort_flag = 1;
    }
  } else if (warp >= 12) {
    // ----------------------------------------------------------- epilogue
    // warp 12 + q reads TMEM lanes 32q..32q+31: rows 32q + lane of each half
    const int q = warp & 3;
    const int r = q * 32 + lane;
    int t_local = 0;
    bool ok = true;
    for (int64_t u0 = u_begin; u0 < u_end && ok; u0 += kTcTileUnits, ++t_local) {
      const int nu = (int)(u_end - u0 < kTcTileUnits ? u_end - u0 : kTcTileUnits);
      const int halves = nu > kTcTileUnits / 2 ? 2 : 1;
      const int buf = t_local & 1;
      if (!ptx::mbar_wait(&stat_full[buf], (uint32_t)(t_local >> 1) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      float mean[2], rstd[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float *st = s_stat + ((size_t)buf * kTcTileRows + h * kTcM + r) * 2;
        const float ss = st[0], sx = st[1];
        if (!LAYER) {
          mean[h] = 0.f;
          rstd[h] = rsqrt_rn(ss / (float)p.H + p.eps);
        } else {
          mean[h] = sx / (float)p.H;
          const float var = fmaxf(ss / (float)p.H - mean[h] * mean[h], 0.f);
          rstd[h] = rsqrt_rn(var + p.eps);
        }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&stat_empty[buf]);
      const int acc = t_local % NA;
      if (!ptx::mbar_wait(&acc_full[acc], (uint32_t)(t_local / NA) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const int64_t row_lim_tile = (u0 + nu) * kTcUnit;
      const int64_t row_lim = row_lim_tile < n ? row_lim_tile : n;
      for (int h = 0; h < halves; ++h) {
        float logit = p.up_bias;
        const uint32_t row_addr =
            tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 2 * B + h * B);
        for (int c = 0; c < B; c += 32) {
          float v[32];
          ptx::tmem_ld32(row_addr + (uint32_t)c, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float z;
            if (!LAYER)
              z = rstd[h] * v[j];
            else
              z = fmaf(rstd[h], v[j] - mean[h] * s_cs[c + j], s_bp[c + j]);
            logit = fmaf(s_up[c + j], silu_fast(z), logit);
          }
        }
        const int64_t grow = u0 * kTcUnit + h * kTcM + r;
        if (grow < row_lim) {
          p.scores[grow] = sigmoid_f(logit);
          if (p.row_stats) p.row_stats[grow] = make_float2(mean[h], rstd[h]);
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&acc_empty[acc]);
    }
    if (!ok) {
      raise_error(p.err, TIDE_DEVERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // drain the TMA loads still in flight before the CTA exits
    const uint32_t n_issued = *issued;
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

bool make_tmap(CUtensorMap *m, const void *base, bool bf16, uint64_t rows, uint64_t cols,
               uint32_t box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)kTcK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Two 128-row halves of B columns per accumulator set; two sets when TMEM's
// 512 columns hold them (B <= 128).
int n_acc_for(int B) { return 4 * B <= 512 ? 2 : 1; }

uint32_t tmem_cols_for(int B) {
  uint32_t need = (uint32_t)(n_acc_for(B) * 2 * B), c = 32;
  while (c < need) c <<= 1;
  return c;
}

int stages_for(int B) {
  const int stage = kTcTileRows * kTcK * 2 + B * kTcK * 2;
  int s = (kTcSmemBudget - 1024 - kTcAux) / stage;
  return s > kTcMaxStages ? kTcMaxStages : s;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace

const char *tc_unsupported_reason(const tide_checkpoint_args *a) {
  if (a->dtype != TIDE_DTYPE_BF16 && a->dtype != TIDE_DTYPE_F16) return "dtype is not bf16/fp16";
  if (!a->folded) return "no folded router weights";
  if (a->hidden_dim % kTcK != 0) return "hidden_dim is not a multiple of 64";
  if (a->bottleneck_dim % 32 != 0 || a->bottleneck_dim > 256) return "bottleneck_dim not in {32,...,256}";
  if (a->norm_type == TIDE_NORM_LAYER && !a->colsum) return "LayerNorm needs colsum";
  if (a->n_rows < 1) return "no rows";
  if (((uintptr_t)a->x & 15u) || ((uintptr_t)a->folded & 15u)) return "x/folded not 16-byte aligned";
  if (a->n_rows > (int64_t)1 << 31) return "too many rows";
  return nullptr;
}

bool tc_supported(const tide_checkpoint_args *a) { return tc_unsupported_reason(a) == nullptr; }

size_t tc_workspace_bytes(int64_t) { return 0; }

int tc_route_launch(const tide_checkpoint_args *a, float *scores, float2 *row_stats,
                    cudaStream_t stream, char *err, size_t err_len) {
  const bool bf16 = a->dtype == TIDE_DTYPE_BF16;
  const int B = (int)a->bottleneck_dim;
  CUtensorMap tx, tw;
  if (!make_tmap(&tx, a->x, bf16, (uint64_t)a->n_rows, (uint64_t)a->hidden_dim, kTcUnit) ||
      !make_tmap(&tw, a->folded, bf16, (uint64_t)B, (uint64_t)a->hidden_dim, (uint32_t)B)) {
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
  p.stages = stages_for(B);
  p.n_acc = n_acc_for(B);
  p.tmem_cols = tmem_cols_for(B);
  const size_t smem = 1024 + (size_t)p.stages * (kTcTileRows * kTcK * 2 + B * kTcK * 2) + kTcAux;
  const int64_t units = (a->n_rows + kTcUnit - 1) / kTcUnit;
  const int grid = (int)(units < sm_count() ? units : sm_count());
  cudaError_t e;
  // the opt-in shared memory size is raised once per kernel to the budget
  const bool layer = a->norm_type == TIDE_NORM_LAYER;
  const void *fn = bf16 ? (layer ? (const void *)tc_route_kernel<true, true> : (const void *)tc_route_kernel<true, false>)
                        : (layer ? (const void *)tc_route_kernel<false, true> : (const void *)tc_route_kernel<false, false>);
  static bool attr_set[4] = {false, false, false, false};
  const int which = (bf16 ? 2 : 0) + (layer ? 1 : 0);
  if (!attr_set[which]) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBudget);
    if (e != cudaSuccess) {
      snprintf(err, err_len, "tensor-core route: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return TIDE_ERR_CUDA;
    }
    attr_set[which] = true;
  }
  if (bf16) {
    if (layer) tc_route_kernel<true, true><<<grid, kTcThreads, smem, stream>>>(tx, tw, p);
    else tc_route_kernel<true, false><<<grid, kTcThreads, smem, stream>>>(tx, tw, p);
  } else {
    if (layer) tc_route_kernel<false, true><<<grid, kTcThreads, smem, stream>>>(tx, tw, p);
    else tc_route_kernel<false, false><<<grid, kTcThreads, smem, stream>>>(tx, tw, p);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(err, err_len, "tensor-core route launch: %s", cudaGetErrorString(e));
    return TIDE_ERR_CUDA;
  }
  return TIDE_OK;
}

}  // namespace tide
