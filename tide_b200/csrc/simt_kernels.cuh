// SIMT kernels of the early-exit path: the general router (any dtype, any
// H, B <= 256), the single-pass stable partition that moves rows (survivors
// to a dense buffer, exits final-normed to their original positions), the
// row scatter / norm-scatter operators and the router weight fold.
#pragma once

#include "common.cuh"

namespace tide {

// ------------------------------------------------------------------ router
// One CTA scores kRouteRows rows.  Pass 1 computes each row's norm
// statistics (warp per row); pass 2 stages kRouteChunk normalised columns of
// all rows in shared memory and each thread accumulates the down projection
// of its router unit(s) b for every row; the epilogue applies SiLU, the up
// projection, the bias and the sigmoid.  Reference semantics:
// python/TIDE/runtime.py:129-130 (router(final_norm(x.float()))) and
// python/TIDE/router.py:18-19; fp32 throughout.
constexpr int kRouteRows = 32;
constexpr int kRouteThreads = 128;
constexpr int kRouteChunk = 128;

struct RouteParams {
  const void *x;
  int64_t n_cap;
  const int32_t *n_dev;
  int H, B;
  int norm_type;
  const float *w_norm, *b_norm;
  float eps;
  const float *down_t;  // [H, B]
  const float *up;      // [B]
  float up_bias;
  float *scores;        // [n]
  float2 *row_stats;    // [n] (mean, rstd) or NULL
  int32_t *err;
};

__device__ __forceinline__ int64_t active_rows(int64_t n_cap, const int32_t *n_dev) {
  if (!n_dev) return n_cap;
  int64_t n = (int64_t)__ldg(n_dev);
  if (n < 0) n = 0;
  return n < n_cap ? n : n_cap;
}

template <typename T, int NB>
__global__ void __launch_bounds__(kRouteThreads) route_simt_kernel(RouteParams p) {
  __shared__ __align__(16) float s_x[kRouteRows][kRouteChunk + 4];
  __shared__ float s_mean[kRouteRows], s_rstd[kRouteRows];
  __shared__ float s_red[kRouteThreads / 32][kRouteRows];

  const int64_t n = active_rows(p.n_cap, p.n_dev);
  const int64_t row0 = (int64_t)blockIdx.x * kRouteRows;
  if (row0 >= n) return;
  const int rows = (int)min((int64_t)kRouteRows, n - row0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const T *x = static_cast<const T *>(p.x);
  const int H = p.H, B = p.B;

  // pass 1: per-row statistics
  for (int r = warp; r < kRouteRows; r += kRouteThreads / 32) {
    float mean = 0.f, rstd = 0.f;
    if (r < rows) {
      const T *xr = x + (row0 + r) * (int64_t)H;
      if (p.norm_type == TIDE_NORM_RMS) {
        float ss = 0.f;
        for (int i = lane; i < H; i += 32) {
          float v = Elem<T>::to_f(xr[i]);
          ss = fmaf(v, v, ss);
        }
        ss = warp_sum(ss);
        rstd = rsqrt_rn(ss / (float)H + p.eps);
      } else {
        float s = 0.f;
        for (int i = lane; i < H; i += 32) s += Elem<T>::to_f(xr[i]);
        mean = warp_sum(s) / (float)H;
        float ss = 0.f;
        for (int i = lane; i < H; i += 32) {
          float d = Elem<T>::to_f(xr[i]) - mean;
          ss = fmaf(d, d, ss);
        }
        ss = warp_sum(ss);
        rstd = rsqrt_rn(ss / (float)H + p.eps);
      }
    }
    if (lane == 0) { s_mean[r] = mean; s_rstd[r] = rstd; }
  }
  __syncthreads();

  float acc[NB][kRouteRows];
#pragma unroll
  for (int bb = 0; bb < NB; ++bb)
#pragma unroll
    for (int r = 0; r < kRouteRows; ++r) acc[bb][r] = 0.f;

  for (int c0 = 0; c0 < H; c0 += kRouteChunk) {
    const int cw = min(kRouteChunk, H - c0);
    // stage normalised values of the chunk (zero beyond the row/chunk end)
    {
      const int c = tid;  // kRouteThreads == kRouteChunk
      float wv = 0.f, bv = 0.f;
      if (c < cw) {
        wv = p.w_norm[c0 + c];
        bv = (p.norm_type == TIDE_NORM_LAYER && p.b_norm) ? p.b_norm[c0 + c] : 0.f;
      }
      for (int r = 0; r < kRouteRows; ++r) {
        float v = 0.f;
        if (r < rows && c < cw) {
          float xv = Elem<T>::to_f(x[(row0 + r) * (int64_t)H + c0 + c]);
          if (p.norm_type == TIDE_NORM_RMS) {
            v = __fmul_rn(wv, __fmul_rn(xv, s_rstd[r]));
          } else {
            float t = __fadd_rn(__fmul_rn(xv, s_rstd[r]), -s_rstd[r] * s_mean[r]);
            v = __fadd_rn(__fmul_rn(t, wv), bv);
          }
        }
        s_x[r][c] = v;
      }
    }
    __syncthreads();
#pragma unroll
    for (int bb = 0; bb < NB; ++bb) {
      const int b = tid + bb * kRouteThreads;
      if (b < B) {
        const float *wcol = p.down_t + (int64_t)c0 * B + b;
        for (int k = 0; k < cw; k += 4) {
          float w0 = wcol[(int64_t)k * B];
          float w1 = (k + 1 < cw) ? wcol[(int64_t)(k + 1) * B] : 0.f;
          float w2 = (k + 2 < cw) ? wcol[(int64_t)(k + 2) * B] : 0.f;
          float w3 = (k + 3 < cw) ? wcol[(int64_t)(k + 3) * B] : 0.f;
#pragma unroll
          for (int r = 0; r < kRouteRows; ++r) {
            float4 v = *reinterpret_cast<const float4 *>(&s_x[r][k]);
            float a = acc[bb][r];
            a = fmaf(v.x, w0, a);
            a = fmaf(v.y, w1, a);
            a = fmaf(v.z, w2, a);
            a = fmaf(v.w, w3, a);
            acc[bb][r] = a;
          }
        }
      }
    }
    __syncthreads();
  }

  // epilogue: sum_b up[b] * SiLU(down_b) per row
  float part[kRouteRows];
#pragma unroll
  for (int r = 0; r < kRouteRows; ++r) part[r] = 0.f;
#pragma unroll
  for (int bb = 0; bb < NB; ++bb) {
    const int b = tid + bb * kRouteThreads;
    if (b < B) {
      const float u = p.up[b];
#pragma unroll
      for (int r = 0; r < kRouteRows; ++r) part[r] = fmaf(silu_f(acc[bb][r]), u, part[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < kRouteRows; ++r) {
    float v = warp_sum(part[r]);
    if (lane == 0) s_red[warp][r] = v;
  }
  __syncthreads();
  if (tid < rows) {
    float z = p.up_bias;
#pragma unroll
    for (int w = 0; w < kRouteThreads / 32; ++w) z += s_red[w][tid];
    p.scores[row0 + tid] = sigmoid_f(z);
    if (p.row_stats) p.row_stats[row0 + tid] = make_float2(s_mean[tid], s_rstd[tid]);
  }
}

// -------------------------------------------------------- stable partition
// One CTA takes the next tile of kMoveTile rows by ticket, classifies every
// row (exit / survive / beyond the active count), ranks rows inside the tile
// with warp ballots, finds the tile's global offsets by decoupled look-back
// and moves rows: survivors are copied bit-exactly to compact_out[dst] with
// their position / slot; exits are written to out_buf at their original
// position, final-normed from the per-row statistics (runtime.py:177-178,
// scheduler.py:89-100), or copied raw (batch_compact.cu semantics).
constexpr int kMoveTile = 128;
constexpr int kMoveThreads = 256;

struct MoveParams {
  const void *x;
  int64_t n_cap;
  const int32_t *n_dev;
  int64_t H;
  int64_t n_total;
  // decision: scores > threshold, or mask != 0
  const float *scores;
  float threshold;
  const int32_t *mask;
  // exit rows: final norm from row statistics (NULL = raw copy)
  const float2 *row_stats;
  int norm_type;
  const float *w_norm, *b_norm;
  bool exits_dense;  // exits written to out_buf[exit rank] (batch_compact)
  const int64_t *pos_in;
  const int32_t *slot_in;
  void *out_buf;
  void *compact_out;
  int64_t *pos_out64;
  int32_t *pos_out32;
  int32_t *slot_out;
  int64_t *exit_pos_out64;
  int32_t *exit_pos_out32;
  int32_t *counts;       // {survivors, exits}
  int32_t *num_remaining;
  uint64_t *status;
  uint32_t *ticket;
  int32_t *err;
};

// Row moves: one warp per row, kRowUnroll 16-byte vectors per lane loaded
// before any is stored, so a warp keeps up to 4 KB of the row in flight.
constexpr int kRowUnroll = 8;

template <typename T, bool VEC>
__device__ __forceinline__ void copy_row(const T *__restrict__ src, T *__restrict__ dst, int64_t H,
                                         int lane) {
  if (VEC) {
    const int64_t nv = H / kVec<T>;
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    for (int64_t base = lane; base < nv; base += 32 * kRowUnroll) {
      uint4 v[kRowUnroll];
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u) {
        const int64_t i = base + 32 * u;
        if (i < nv) v[u] = ld_stream(s + i);
      }
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u) {
        const int64_t i = base + 32 * u;
        if (i < nv) st_stream(d + i, v[u]);
      }
    }
  } else {
    for (int64_t i = lane; i < H; i += 32) dst[i] = src[i];
  }
}

// y = final_norm(x) rounded to T.  RMSNorm: w * (x * rstd)
// (LlamaRMSNorm / Qwen3RMSNorm).  LayerNorm: (x * rstd - mean * rstd) * w + b.
template <typename T>
__device__ __forceinline__ float norm_elem(float xv, float wv, float bv, float rstd, float shift,
                                           int norm_type) {
  if (norm_type == TIDE_NORM_RMS) return __fmul_rn(wv, __fmul_rn(xv, rstd));
  const float t = __fadd_rn(__fmul_rn(xv, rstd), shift);
  return __fadd_rn(__fmul_rn(t, wv), bv);
}

template <typename T, bool VEC>
__device__ __forceinline__ void norm_row(const T *__restrict__ src, T *__restrict__ dst, int64_t H,
                                         int lane, float mean, float rstd, int norm_type,
                                         const float *__restrict__ w,
                                         const float *__restrict__ bias) {
  const float shift = -rstd * mean;
  if (VEC) {
    constexpr int V = kVec<T>;
    const int64_t nv = H / V;
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    const bool wvec = ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(bias)) & 15u) == 0;
    for (int64_t base = lane; base < nv; base += 32 * kRowUnroll) {
      uint4 v[kRowUnroll];
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u) {
        const int64_t i = base + 32 * u;
        if (i < nv) v[u] = ld_stream(s + i);
      }
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u) {
        const int64_t i = base + 32 * u;
        if (i >= nv) continue;
        float xv[V], y[V], wv[V], bv[V];
        unpack16<T>(v[u], xv);
        const int64_t col = i * V;
        if (wvec) {
#pragma unroll
          for (int j = 0; j < V; j += 4) {
            const float4 w4 = __ldg(reinterpret_cast<const float4 *>(w + col + j));
            wv[j] = w4.x; wv[j + 1] = w4.y; wv[j + 2] = w4.z; wv[j + 3] = w4.w;
            if (bias) {
              const float4 b4 = __ldg(reinterpret_cast<const float4 *>(bias + col + j));
              bv[j] = b4.x; bv[j + 1] = b4.y; bv[j + 2] = b4.z; bv[j + 3] = b4.w;
            } else {
              bv[j] = bv[j + 1] = bv[j + 2] = bv[j + 3] = 0.f;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < V; ++j) {
            wv[j] = __ldg(w + col + j);
            bv[j] = bias ? __ldg(bias + col + j) : 0.f;
          }
        }
#pragma unroll
        for (int j = 0; j < V; ++j) y[j] = norm_elem<T>(xv[j], wv[j], bv[j], rstd, shift, norm_type);
        st_stream(d + i, pack16<T>(y));
      }
    }
  } else {
    for (int64_t i = lane; i < H; i += 32)
      dst[i] = Elem<T>::from_f(norm_elem<T>(Elem<T>::to_f(src[i]), w[i], bias ? bias[i] : 0.f,
                                            rstd, shift, norm_type));
  }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kMoveThreads, 2) move_rows_kernel(MoveParams p) {
  __shared__ uint32_t s_tile;
  __shared__ uint32_t s_wkeep[kMoveTile / 32], s_wexit[kMoveTile / 32];
  __shared__ uint32_t s_keep_before, s_exits_before;
  __shared__ int8_t s_state[kMoveTile];
  __shared__ uint32_t s_rank[kMoveTile];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int64_t n = p.n_cap;
  if (p.n_dev) {
    int64_t nd = (int64_t)__ldg(p.n_dev);
    if (nd < 0 || nd > p.n_cap) {
      if (tid == 0 && blockIdx.x == 0) raise_error(p.err, TIDE_DEVERR_COUNT);
      nd = nd < 0 ? 0 : p.n_cap;
    }
    n = nd;
  }
  const int64_t n_tiles = n > 0 ? (n + kMoveTile - 1) / kMoveTile : 1;
  if (tid == 0) s_tile = atomicAdd(p.ticket, 1u);
  __syncthreads();
  const int64_t tile = s_tile;
  if (tile >= n_tiles) return;
  const int64_t row0 = tile * kMoveTile;

  if (tid < kMoveTile) {
    const int64_t row = row0 + tid;
    int state = 0;
    if (row < n) {
      bool ex = p.scores ? (p.scores[row] > p.threshold) : (p.mask[row] != 0);
      state = ex ? 2 : 1;
    }
    const unsigned kb = __ballot_sync(0xffffffffu, state == 1);
    const unsigned eb = __ballot_sync(0xffffffffu, state == 2);
    const unsigned lt = (1u << lane) - 1u;
    s_state[tid] = (int8_t)state;
    s_rank[tid] = state == 1 ? __popc(kb & lt) : __popc(eb & lt);
    if (lane == 0) {
      s_wkeep[warp] = __popc(kb);
      s_wexit[warp] = __popc(eb);
    }
  }
  __syncthreads();
  if (tid < kMoveTile) {
    const int st = s_state[tid];
    uint32_t add = 0;
    for (int w = 0; w < warp; ++w) add += st == 1 ? s_wkeep[w] : s_wexit[w];
    s_rank[tid] += add;
  }
  if (tid == 0) {
    uint32_t keep_t = 0, exit_t = 0;
    for (int w = 0; w < kMoveTile / 32; ++w) { keep_t += s_wkeep[w]; exit_t += s_wexit[w]; }
    uint32_t kb = 0, eb = 0;
    if (!lookback(p.status, (uint32_t)tile, keep_t, exit_t, &kb, &eb))
      raise_error(p.err, TIDE_DEVERR_TIMEOUT);
    s_keep_before = kb;
    s_exits_before = eb;
    if (tile == n_tiles - 1) {
      if (p.counts) { p.counts[0] = (int32_t)(kb + keep_t); p.counts[1] = (int32_t)(eb + exit_t); }
      if (p.num_remaining) p.num_remaining[0] = (int32_t)(kb + keep_t);
    }
  }
  __syncthreads();

  const T *x = static_cast<const T *>(p.x);
  for (int r = warp; r < kMoveTile; r += kMoveThreads / 32) {
    const int st = s_state[r];
    if (st == 0) continue;
    const int64_t row = row0 + r;
    const T *src = x + row * p.H;
    if (st == 1) {
      const int64_t dst = (int64_t)s_keep_before + s_rank[r];
      if (lane == 0) {
        if (p.pos_out64) p.pos_out64[dst] = p.pos_in ? p.pos_in[row] : row;
        if (p.pos_out32) p.pos_out32[dst] = (int32_t)(p.pos_in ? p.pos_in[row] : row);
        if (p.slot_out) p.slot_out[dst] = p.slot_in ? p.slot_in[row] : (int32_t)row;
      }
      if (p.compact_out) copy_row<T, VEC>(src, static_cast<T *>(p.compact_out) + dst * p.H, p.H, lane);
    } else {
      const int64_t e = (int64_t)s_exits_before + s_rank[r];
      const int64_t pos = p.pos_in ? p.pos_in[row] : row;
      if (lane == 0) {
        if (p.exit_pos_out64) p.exit_pos_out64[e] = pos;
        if (p.exit_pos_out32) p.exit_pos_out32[e] = (int32_t)pos;
      }
      if (!p.out_buf) continue;
      const int64_t dst_row = p.exits_dense ? e : pos;
      if (dst_row < 0 || dst_row >= p.n_total) {
        if (lane == 0) raise_error(p.err, TIDE_DEVERR_POSITION);
        continue;
      }
      T *dst = static_cast<T *>(p.out_buf) + dst_row * p.H;
      if (p.row_stats) {
        const float2 ms = p.row_stats[row];
        norm_row<T, VEC>(src, dst, p.H, lane, ms.x, ms.y, p.norm_type, p.w_norm, p.b_norm);
      } else {
        copy_row<T, VEC>(src, dst, p.H, lane);
      }
    }
  }
}

// ------------------------------------------------- scatter / norm-scatter
// output[pos[i]] = src[i]                 (exit_scatter.cu:16-37)
// output[pos[i]] = final_norm(src[i])     (exit_projection.cu:20-57 for
//                  RMSNorm; runtime.py:183-187 for the rows that never exit)
// One warp per row; positions are int32 (reference operators) or int64.
template <typename T, bool VEC, bool NORM>
__global__ void scatter_rows_kernel(const T *__restrict__ src, const int32_t *__restrict__ pos32,
                                    const int64_t *__restrict__ pos64, T *__restrict__ out,
                                    int64_t n_rows, int64_t H, int64_t n_total, int norm_type,
                                    const float *__restrict__ w, const float *__restrict__ bias,
                                    float eps, int32_t *err) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const int64_t p = pos64 ? pos64[row] : (int64_t)pos32[row];
  if (p < 0 || p >= n_total) {
    if (lane == 0) raise_error(err, TIDE_DEVERR_POSITION);
    return;
  }
  const T *s = src + row * H;
  T *d = out + p * H;
  if (!NORM) {
    copy_row<T, VEC>(s, d, H, lane);
    return;
  }
  // row statistics (two passes for LayerNorm: mean, then centred squares)
  float mean = 0.f;
  if (norm_type == TIDE_NORM_LAYER) {
    float sum = 0.f;
    for (int64_t i = lane; i < H; i += 32) sum += Elem<T>::to_f(s[i]);
    mean = warp_sum(sum) / (float)H;
  }
  float ss = 0.f;
  if (VEC) {
    constexpr int V = kVec<T>;
    const uint4 *sv = reinterpret_cast<const uint4 *>(s);
    for (int64_t i = lane; i < H / V; i += 32) {
      float xv[V];
      unpack16<T>(sv[i], xv);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float dv = xv[j] - mean;
        ss = fmaf(dv, dv, ss);
      }
    }
  } else {
    for (int64_t i = lane; i < H; i += 32) {
      const float dv = Elem<T>::to_f(s[i]) - mean;
      ss = fmaf(dv, dv, ss);
    }
  }
  ss = warp_sum(ss);
  const float rstd = rsqrt_rn(ss / (float)H + eps);
  norm_row<T, VEC>(s, d, H, lane, mean, rstd, norm_type, w, bias);
}

// ------------------------------------------------------- indexed rows
// Rows addressed through an index with a live count kept on the device, so
// that checkpoints chain without reading the count back:
//   gather (NORM = false):                 dst[i] = src[idx[i]]
//   norm in place (NORM, SRC_I = false):   dst[idx[i]] = final_norm(src[idx[i]])
//   norm scatter (NORM, SRC_I = true):     dst[idx[i]] = final_norm(src[i])
// for i < live, live = *n_dev clamped to [0, n_cap] (n_cap without n_dev);
// idx[i] is checked against n_src.  One warp per row, grid-stride over the
// capacity.
template <typename T, bool VEC, bool NORM, bool SRC_I = false>
__global__ void indexed_rows_kernel(const T *__restrict__ src, const int64_t *__restrict__ idx,
                                    const int32_t *__restrict__ n_dev, int64_t n_cap, int64_t H,
                                    int64_t n_src, T *__restrict__ dst, int norm_type,
                                    const float *__restrict__ w, const float *__restrict__ bias,
                                    float eps, int32_t *err) {
  const int lane = threadIdx.x & 31;
  int64_t live = n_cap;
  if (n_dev) {
    const int64_t nd = (int64_t)__ldg(n_dev);
    if (nd < 0 || nd > n_cap) {
      if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(err, TIDE_DEVERR_COUNT);
    }
    live = nd < 0 ? 0 : (nd > n_cap ? n_cap : nd);
  }
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); i < live; i += warps) {
    const int64_t p = idx[i];
    if (p < 0 || p >= n_src) {
      if (lane == 0) raise_error(err, TIDE_DEVERR_POSITION);
      continue;
    }
    const T *s = src + (SRC_I ? i : p) * H;
    if (!NORM) {
      copy_row<T, VEC>(s, dst + i * H, H, lane);
      continue;
    }
    float mean = 0.f;
    if (norm_type == TIDE_NORM_LAYER) {
      float sum = 0.f;
      for (int64_t k = lane; k < H; k += 32) sum += Elem<T>::to_f(s[k]);
      mean = warp_sum(sum) / (float)H;
    }
    float ss = 0.f;
    for (int64_t k = lane; k < H; k += 32) {
      const float dv = Elem<T>::to_f(s[k]) - mean;
      ss = fmaf(dv, dv, ss);
    }
    ss = warp_sum(ss);
    const float rstd = rsqrt_rn(ss / (float)H + eps);
    norm_row<T, VEC>(s, dst + p * H, H, lane, mean, rstd, norm_type, w, bias);
  }
}

// ---------------------------------------------------------- weight fold
// One CTA per router unit b.
template <typename TF>
__global__ void router_fold_kernel(const float *__restrict__ down, const float *__restrict__ w,
                                   const float *__restrict__ bn, int64_t H, int64_t B,
                                   float *__restrict__ down_t, TF *__restrict__ folded,
                                   float *__restrict__ colsum, float *__restrict__ bias_proj) {
  __shared__ float s_a[32], s_b[32];
  const int64_t b = blockIdx.x;
  float cs = 0.f, bp = 0.f;
  for (int64_t i = threadIdx.x; i < H; i += blockDim.x) {
    const float d = down[b * H + i];
    if (down_t) down_t[i * B + b] = d;
    if (folded) {
      const TF f = Elem<TF>::from_f(__fmul_rn(d, w[i]));
      folded[b * H + i] = f;
      cs += Elem<TF>::to_f(f);
    }
    if (bn) bp = fmaf(bn[i], d, bp);
  }
  cs = warp_sum(cs);
  bp = warp_sum(bp);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { s_a[warp] = cs; s_b[warp] = bp; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, c = 0.f;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i) { a += s_a[i]; c += s_b[i]; }
    if (colsum) colsum[b] = a;
    if (bias_proj) bias_proj[b] = c;
  }
}

}  // namespace tide
