// Decode attention over a KV cache addressed by slot, for the rows still
// active after the early-exit checkpoints of a decode step.
//
// The checkpoint kernels compact the surviving rows of a step together with
// their KV slot ids; the layers after a checkpoint then run on those rows
// only.  Their attention must read the cache rows of exactly those
// sequences, wherever they sit in the cache, and nothing of the exited ones.
// The reference has no such kernel: its decode runs every layer for the
// whole batch (python/TIDE/runtime.py:223-313) and pads the cache of skipped
// layers with zeros (runtime.py:194-221, "zero_pad").  This kernel keeps that
// padding convention: positions a sequence skipped hold zero keys and values
// and take part in the softmax like any other position.
//
//   o[i, h, :] = sum_j softmax_j(scale * q[i, h, :] . K[s_i, h / G, j, :]) V[s_i, h / G, j, :]
//   for j in [0, L), s_i = slots[i], G = query heads per KV head.
//
// One CTA per (active row, KV head), 128 threads, head_dim 128.  Pass 1:
// every thread scores whole key rows (256 bytes each, positions t, t+128, ...)
// against the G query heads held in shared memory, keeping the scores in
// shared memory.  Pass 2: max and sum per query head.  Pass 3: warp g owns
// query head g (G <= 4) or two of them (G = 8), each lane four output
// dimensions, and walks the value rows once (a warp reads a 256-byte value
// row per position).  fp32 throughout; output in the cache's 16-bit type.
#include <math.h>
#include <stdio.h>

#include "common.cuh"

namespace tide {

namespace dattn {
constexpr int kD = 128;
constexpr int kThreads = 128;
constexpr int kMaxG = 8;
}  // namespace dattn

template <typename T>
__global__ void __launch_bounds__(dattn::kThreads)
    decode_attention_kernel(const T *__restrict__ q, const T *__restrict__ kc,
                            const T *__restrict__ vc, const int32_t *__restrict__ slots,
                            T *__restrict__ o, int n_rows, int hq, int hkv, int64_t n_slots,
                            int64_t max_len, int L, float scale, int32_t *err) {
  using namespace dattn;
  extern __shared__ float sm[];
  const int G = hq / hkv;
  float *s_q = sm;                 // [G][128]
  float *s_p = sm + G * kD;        // [G][L] scores, then probabilities
  __shared__ float s_red[kMaxG][4];
  __shared__ float s_max[kMaxG], s_sum[kMaxG];
  const int row = blockIdx.x / hkv, kvh = blockIdx.x % hkv;
  if (row >= n_rows) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t slot = slots ? (int64_t)slots[row] : row;
  if (slot < 0 || slot >= n_slots) {  // a slot outside the cache: the row is skipped
    if (threadIdx.x == 0) raise_error(err, TIDE_DEVERR_POSITION);
    return;
  }
  const T *kb = kc + ((slot * hkv + kvh) * max_len) * kD;
  const T *vb = vc + ((slot * hkv + kvh) * max_len) * kD;
  for (int i = tid; i < G * kD; i += kThreads)
    s_q[i] = Elem<T>::to_f(q[((int64_t)row * hq + kvh * G) * kD + i]) * scale;
  __syncthreads();

  // pass 1: scores
  float mx[kMaxG];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) mx[g] = -INFINITY;
  for (int j = tid; j < L; j += kThreads) {
    const uint4 *kr = reinterpret_cast<const uint4 *>(kb + (int64_t)j * kD);
    float acc[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) acc[g] = 0.f;
#pragma unroll 4
    for (int c = 0; c < kD / 8; ++c) {
      const uint4 v = kr[c];
      float f[8];
      unpack16<T>(v, f);
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) {
        if (g >= G) break;
        const float *qg = s_q + g * kD + c * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g] = fmaf(qg[e], f[e], acc[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g >= G) break;
      s_p[g * L + j] = acc[g];
      mx[g] = fmaxf(mx[g], acc[g]);
    }
  }
  // pass 2: max and sum per query head
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g >= G) break;
    float m = mx[g];
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) s_red[g][warp] = m;
  }
  __syncthreads();
  if (tid < G) s_max[tid] = fmaxf(fmaxf(s_red[tid][0], s_red[tid][1]), fmaxf(s_red[tid][2], s_red[tid][3]));
  __syncthreads();
  float sum[kMaxG];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) sum[g] = 0.f;
  for (int j = tid; j < L; j += kThreads) {
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g >= G) break;
      const float e = __expf(s_p[g * L + j] - s_max[g]);
      s_p[g * L + j] = e;
      sum[g] += e;
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g >= G) break;
    float sg = sum[g];
    for (int off = 16; off; off >>= 1) sg += __shfl_xor_sync(0xffffffffu, sg, off);
    if (lane == 0) s_red[g][warp] = sg;
  }
  __syncthreads();
  if (tid < G) s_sum[tid] = (s_red[tid][0] + s_red[tid][1]) + (s_red[tid][2] + s_red[tid][3]);
  __syncthreads();

  // pass 3: o = P V; warp w serves query heads w, w + 4 (G = 8), lane four dims
  for (int g = warp; g < G; g += kThreads / 32) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    const float *pg = s_p + g * L;
#pragma unroll 4
    for (int j = 0; j < L; ++j) {
      const uint2 v = *reinterpret_cast<const uint2 *>(vb + (int64_t)j * kD + lane * 4);
      const T *e4 = reinterpret_cast<const T *>(&v);
      float f[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) f[e] = Elem<T>::to_f(e4[e]);
      const float pj = pg[j];
      a0 = fmaf(pj, f[0], a0);
      a1 = fmaf(pj, f[1], a1);
      a2 = fmaf(pj, f[2], a2);
      a3 = fmaf(pj, f[3], a3);
    }
    const float inv = 1.0f / s_sum[g];
    T *og = o + ((int64_t)row * hq + kvh * G + g) * kD + lane * 4;
    og[0] = Elem<T>::from_f(a0 * inv);
    og[1] = Elem<T>::from_f(a1 * inv);
    og[2] = Elem<T>::from_f(a2 * inv);
    og[3] = Elem<T>::from_f(a3 * inv);
  }
}

}  // namespace tide

namespace tide {
void set_last_error(const char *msg);
}

extern "C" int tide_decode_attention(int dtype, const void *q, const void *k_cache,
                                     const void *v_cache, const int32_t *slots, void *out,
                                     int64_t n_rows, int64_t n_q_heads, int64_t n_kv_heads,
                                     int64_t head_dim, int64_t n_slots, int64_t max_len,
                                     int64_t length, float scale, int32_t *error_word,
                                     tide_stream_t stream) {
  using namespace tide;
  if (dtype != TIDE_DTYPE_BF16 && dtype != TIDE_DTYPE_F16) {
    tide::set_last_error("decode_attention: dtype must be bf16 or fp16");
    return TIDE_ERR_UNSUPPORTED;
  }
  if (head_dim != dattn::kD) {
    tide::set_last_error("decode_attention: head_dim must be 128");
    return TIDE_ERR_UNSUPPORTED;
  }
  if (n_rows < 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0 ||
      n_q_heads / n_kv_heads > dattn::kMaxG || length < 1 || length > max_len || n_slots < 1 ||
      (!slots && n_rows > n_slots)) {
    tide::set_last_error("decode_attention: bad sizes (heads, length)");
    return TIDE_ERR_INVALID;
  }
  if (n_rows == 0) return TIDE_OK;
  if (!q || !k_cache || !v_cache || !out) {
    tide::set_last_error("decode_attention: NULL pointer");
    return TIDE_ERR_INVALID;
  }
  const int G = (int)(n_q_heads / n_kv_heads);
  const size_t smem = (size_t)G * (dattn::kD + (size_t)length) * sizeof(float);
  if (smem > 200 * 1024) {
    tide::set_last_error("decode_attention: length too long for the scores in shared memory");
    return TIDE_ERR_UNSUPPORTED;
  }
  const int64_t grid = n_rows * n_kv_heads;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  if (dtype == TIDE_DTYPE_BF16) {
    e = cudaFuncSetAttribute(decode_attention_kernel<__nv_bfloat16>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess)
      decode_attention_kernel<__nv_bfloat16><<<(unsigned)grid, dattn::kThreads, smem, s>>>(
          static_cast<const __nv_bfloat16 *>(q), static_cast<const __nv_bfloat16 *>(k_cache),
          static_cast<const __nv_bfloat16 *>(v_cache), slots, static_cast<__nv_bfloat16 *>(out),
          (int)n_rows, (int)n_q_heads, (int)n_kv_heads, n_slots, max_len, (int)length, scale,
          error_word);
  } else {
    e = cudaFuncSetAttribute(decode_attention_kernel<__half>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess)
      decode_attention_kernel<__half><<<(unsigned)grid, dattn::kThreads, smem, s>>>(
          static_cast<const __half *>(q), static_cast<const __half *>(k_cache),
          static_cast<const __half *>(v_cache), slots, static_cast<__half *>(out), (int)n_rows,
          (int)n_q_heads, (int)n_kv_heads, n_slots, max_len, (int)length, scale, error_word);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "decode_attention: %s", cudaGetErrorString(e));
    tide::set_last_error(buf);
    return TIDE_ERR_CUDA;
  }
  return TIDE_OK;
}
