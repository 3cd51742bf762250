// The elementwise work of a Llama-family decode layer, fused for the live
// decoder: each kernel replaces a chain of eager PyTorch ops of the model's
// own modules and rounds at exactly the points those ops round, so the
// results are those of the HF modules (up to the order of fp32 sums).
//
//   tide_rms_norm        y = w * to_T(s * rsqrt(mean(s^2) + eps)),  s = x or
//                        to_T(x + delta) (a residual add, also written out):
//                        HF LlamaRMSNorm / Qwen3RMSNorm (the layer's input and
//                        post-attention norms, the model's final norm).
//   tide_qk_norm_rope    per head: optional RMSNorm of q and k (Qwen3's
//                        q_norm / k_norm), the rotary embedding
//                        q*cos + rotate_half(q)*sin with cos/sin of
//                        position * inv_freq rounded to T (the decode
//                        position, or each row's own for a prefill), then q
//                        to its output and k, v into the slot-addressed cache
//                        at the decode position (what tide_kv_append does; a
//                        prefill passes [n, heads, 1, 128] outputs as the
//                        "cache", its rows' token indices as the slots, and
//                        gets q at those indices too).
//   tide_silu_mul        to_T(to_T(silu(gate)) * up): the gated MLP's
//                        act_fn(gate_proj(x)) * up_proj(x).
//
// Every kernel takes the live row count from the device (rows past it are
// not touched), so a decode step stays free of host values.  These are the
// live decoder's layer (python/TIDE/runtime.py:223-313 runs the HF model
// call instead); the norms, rotary and activation follow the HF modules the
// reference's runtime calls.
#include <math.h>
#include <stdio.h>

#include <initializer_list>

#include "common.cuh"

namespace tide {

void set_last_error(const char *msg);

namespace dlayer {
constexpr int kNormThreads = 128;
constexpr int kMaxVecPerThread = 8;  // H <= 128 threads x 8 vectors x 8 = 8192
}  // namespace dlayer

template <typename T>
__device__ __forceinline__ float round_t(float v) {
  return Elem<T>::to_f(Elem<T>::from_f(v));
}

__device__ __forceinline__ int64_t live_rows(const int32_t *n_dev, int64_t n_cap) {
  if (!n_dev) return n_cap;
  const int64_t v = (int64_t)__ldg(n_dev);
  return v < 0 ? 0 : (v > n_cap ? n_cap : v);
}

// One CTA per row (grid-stride), 128 threads, 16-byte vectors, VPT vectors
// per thread (the row's H / 1024 rounded up to a power of two: the fewer the
// registers, the more rows in flight per SM).
template <typename T, int VPT>
__global__ void __launch_bounds__(dlayer::kNormThreads)
    rms_norm_kernel(const T *__restrict__ x, const T *__restrict__ delta, T *__restrict__ sum_out,
                    const T *__restrict__ w, T *__restrict__ y, int64_t n_cap,
                    const int32_t *__restrict__ n_dev, int H, float eps) {
  using namespace dlayer;
  __shared__ float s_red[kNormThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nv = H / 8;  // 16-byte vectors per row
  const int64_t live = live_rows(n_dev, n_cap);
  for (int64_t row = blockIdx.x; row < live; row += gridDim.x) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * H);
    const uint4 *dr = delta ? reinterpret_cast<const uint4 *>(delta + row * H) : nullptr;
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < VPT; ++c) {
      const int i = tid + c * kNormThreads;
      if (i < nv) {
        unpack16<T>(xr[i], v[c]);
        if (dr) {
          float d[8];
          unpack16<T>(dr[i], d);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[c][e] = round_t<T>(v[c][e] + d[e]);
          if (sum_out) reinterpret_cast<uint4 *>(sum_out + row * H)[i] = pack16<T>(v[c]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[c][e], v[c][e], ss);
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    const float tot = (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]);
    const float rstd = rsqrtf(tot / (float)H + eps);  // torch.rsqrt on the GPU
    __syncthreads();  // s_red is rewritten by the next row
    const uint4 *wr = reinterpret_cast<const uint4 *>(w);
#pragma unroll
    for (int c = 0; c < VPT; ++c) {
      const int i = tid + c * kNormThreads;
      if (i < nv) {
        float wf[8], o[8];
        unpack16<T>(wr[i], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = wf[e] * round_t<T>(v[c][e] * rstd);
        reinterpret_cast<uint4 *>(y + row * H)[i] = pack16<T>(o);
      }
    }
  }
}

// One warp per (row, group of `group` <= 8 heads) of the row's q, k and v
// heads (in that order), head_dim 128: lane l holds dims 4l..4l+3; the
// rotary partner of a dim (d +- 64) sits 16 lanes away.  The rotary cos/sin
// of a lane's dims depend on the row's position only, so a warp computes
// them once for its group, and issues the group's loads before using any.
// A prefill (many rows) takes groups of eight heads, so the cos/sin are
// computed once per row and eight heads instead of once per head; a decode
// step (few rows) takes one head per warp, for more warps in flight.
template <typename T>
__global__ void __launch_bounds__(256)
    qk_norm_rope_kernel(const T *__restrict__ q, const T *__restrict__ k, const T *__restrict__ v,
                        int64_t q_stride, int64_t kv_stride,
                        const T *__restrict__ q_w, const T *__restrict__ k_w, float eps,
                        const float *__restrict__ inv_freq, float att_scale, int64_t pos_host,
                        const int32_t *__restrict__ pos_dev, const int64_t *__restrict__ rope_pos,
                        const int32_t *__restrict__ slots,
                        const int32_t *__restrict__ n_dev, int64_t n_cap, int hq, int hkv,
                        T *__restrict__ q_out, T *__restrict__ kc, T *__restrict__ vc,
                        int64_t n_slots, int64_t max_len, int group, int32_t *err) {
  constexpr int kD = 128;
  constexpr int kGroup = 8;  // most heads per warp
  const int lane = threadIdx.x & 31;
  const int heads = hq + 2 * hkv;
  const int groups = (heads + group - 1) / group;
  const int64_t live = live_rows(n_dev, n_cap);
  const int64_t pos = pos_dev ? (int64_t)__ldg(pos_dev) : pos_host;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int d0 = lane * 4;
  for (int64_t wid = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
       wid < live * groups; wid += warps) {
    const int64_t row = wid / groups;
    const int h0 = (int)(wid % groups) * group;
    const int h1 = min(h0 + group, heads);
    // the row's cache entry, when the group holds k or v heads; a prefill
    // (rope_pos given) also writes q at the row's slot
    const int64_t slot = slots ? (int64_t)slots[row] : row;
    const bool slot_ok = slot >= 0 && slot < n_slots;
    int64_t cache_row = 0;
    bool cache_ok = true;
    if (h1 > hq) {
      cache_ok = slot_ok && pos >= 0 && pos < max_len;
      if (!cache_ok && lane == 0) raise_error(err, TIDE_DEVERR_POSITION);
      cache_row = (slot * hkv) * max_len + pos;  // + h * max_len per head
    }
    const bool q_at_slot = rope_pos != nullptr;
    const bool q_ok = !q_at_slot || slot_ok;
    if (h0 < hq && !q_ok && lane == 0) raise_error(err, TIDE_DEVERR_POSITION);
    const int64_t q_row = q_at_slot ? slot : row;
    // loads of the group's heads, all issued before the first is used
    uint2 raw[kGroup];
#pragma unroll
    for (int i = 0; i < kGroup; ++i) {
      const int hh = h0 + i;
      raw[i] = make_uint2(0u, 0u);
      if (hh >= h1) continue;
      const T *src = hh < hq ? q + row * q_stride + (int64_t)hh * kD
                   : (hh < hq + hkv ? k + row * kv_stride + (int64_t)(hh - hq) * kD
                                    : v + row * kv_stride + (int64_t)(hh - hq - hkv) * kD);
      raw[i] = *reinterpret_cast<const uint2 *>(src + d0);
    }
    // cos / sin of the lane's dims at the row's position (q and k heads only)
    float cs[4] = {0.f, 0.f, 0.f, 0.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
    if (h0 < hq + hkv) {
      const int64_t rot_pos = rope_pos ? rope_pos[row] : pos;  // a prefill row's own position
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float freq = (float)rot_pos * inv_freq[(d0 + e) & (kD / 2 - 1)];
        cs[e] = round_t<T>(cosf(freq) * att_scale);
        sn[e] = round_t<T>(sinf(freq) * att_scale);
      }
    }
#pragma unroll
    for (int i = 0; i < kGroup; ++i) {
      const int hh = h0 + i;
      if (hh >= h1) break;
      const int kind = hh < hq ? 0 : (hh < hq + hkv ? 1 : 2);  // q, k, v
      const int h = kind == 0 ? hh : (kind == 1 ? hh - hq : hh - hq - hkv);
      if (kind == 2) {  // values go to the cache as they are
        if (cache_ok)
          *reinterpret_cast<uint2 *>(vc + (cache_row + (int64_t)h * max_len) * kD + d0) = raw[i];
        continue;
      }
      if ((kind == 1 && !cache_ok) || (kind == 0 && !q_ok)) continue;
      const T *e4 = reinterpret_cast<const T *>(&raw[i]);
      float f[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) f[e] = Elem<T>::to_f(e4[e]);
      const T *nw = kind == 0 ? q_w : k_w;
      if (nw) {  // the head's RMSNorm (HF: fp32 statistics, normalised rounded to T, times w)
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) ss = fmaf(f[e], f[e], ss);
        ss = warp_sum(ss);
        const float rstd = rsqrtf(ss / (float)kD + eps);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          f[e] = round_t<T>(Elem<T>::to_f(nw[d0 + e]) * round_t<T>(f[e] * rstd));
      }
      // rotate_half: dims < 64 take -x[d + 64], dims >= 64 take x[d - 64]
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, f[e], 16);
        const float rot = lane < 16 ? -partner : partner;
        o[e] = round_t<T>(round_t<T>(f[e] * cs[e]) + round_t<T>(rot * sn[e]));
      }
      uint2 packed;
      T *p4 = reinterpret_cast<T *>(&packed);
#pragma unroll
      for (int e = 0; e < 4; ++e) p4[e] = Elem<T>::from_f(o[e]);
      if (kind == 0)
        *reinterpret_cast<uint2 *>(q_out + (q_row * hq + h) * kD + d0) = packed;
      else
        *reinterpret_cast<uint2 *>(kc + (cache_row + (int64_t)h * max_len) * kD + d0) = packed;
    }
  }
}

// y = to_T(to_T(silu(g)) * u) over [live rows, I], 16-byte vectors.
template <typename T>
__global__ void silu_mul_kernel(const T *__restrict__ g, const T *__restrict__ u, T *__restrict__ y,
                                int64_t n_cap, const int32_t *__restrict__ n_dev, int64_t I) {
  const int64_t live = live_rows(n_dev, n_cap);
  const int64_t nv = live * I / 8;
  const uint4 *g4 = reinterpret_cast<const uint4 *>(g);
  const uint4 *u4 = reinterpret_cast<const uint4 *>(u);
  uint4 *y4 = reinterpret_cast<uint4 *>(y);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv;
       i += (int64_t)gridDim.x * blockDim.x) {
    float a[8], b[8], o[8];
    unpack16<T>(g4[i], a);
    unpack16<T>(u4[i], b);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = round_t<T>(a[e] / (1.0f + expf(-a[e]))) * b[e];
    y4[i] = pack16<T>(o);
  }
}

}  // namespace tide

namespace {

bool aligned16(std::initializer_list<const void *> ps) {
  for (const void *p : ps)
    if (reinterpret_cast<uintptr_t>(p) & 15u) return false;
  return true;
}

int fail_msg(int code, const char *msg) {
  tide::set_last_error(msg);
  return code;
}

int launched(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    tide::set_last_error(buf);
    return TIDE_ERR_CUDA;
  }
  return TIDE_OK;
}

unsigned grid_for(int64_t work, int64_t per_block, int64_t cap) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace

template <typename T>
void launch_rms_norm(int vpt, unsigned grid, cudaStream_t s, const void *x, const void *delta,
                     void *sum_out, const void *weight, void *out, int64_t n_rows,
                     const int32_t *n_rows_dev, int H, float eps) {
  const T *xx = static_cast<const T *>(x), *dd = static_cast<const T *>(delta);
  const T *ww = static_cast<const T *>(weight);
  T *ss = static_cast<T *>(sum_out), *yy = static_cast<T *>(out);
  constexpr int kT = tide::dlayer::kNormThreads;
  switch (vpt) {
    case 1: tide::rms_norm_kernel<T, 1><<<grid, kT, 0, s>>>(xx, dd, ss, ww, yy, n_rows, n_rows_dev, H, eps); break;
    case 2: tide::rms_norm_kernel<T, 2><<<grid, kT, 0, s>>>(xx, dd, ss, ww, yy, n_rows, n_rows_dev, H, eps); break;
    case 4: tide::rms_norm_kernel<T, 4><<<grid, kT, 0, s>>>(xx, dd, ss, ww, yy, n_rows, n_rows_dev, H, eps); break;
    default: tide::rms_norm_kernel<T, 8><<<grid, kT, 0, s>>>(xx, dd, ss, ww, yy, n_rows, n_rows_dev, H, eps); break;
  }
}

extern "C" int tide_rms_norm(int dtype, const void *x, const void *delta, void *sum_out,
                             const void *weight, void *out, int64_t n_rows,
                             const int32_t *n_rows_dev, int64_t hidden_dim, float eps,
                             tide_stream_t stream) {
  using namespace tide;
  if (dtype != TIDE_DTYPE_BF16 && dtype != TIDE_DTYPE_F16)
    return fail_msg(TIDE_ERR_UNSUPPORTED, "rms_norm: dtype must be bf16 or fp16");
  if (n_rows < 0 || hidden_dim < 8 || hidden_dim % 8 ||
      hidden_dim > dlayer::kNormThreads * dlayer::kMaxVecPerThread * 8)
    return fail_msg(TIDE_ERR_INVALID, "rms_norm: hidden_dim must be a multiple of 8, at most 8192");
  if (n_rows == 0) return TIDE_OK;
  if (!x || !weight || !out) return fail_msg(TIDE_ERR_INVALID, "rms_norm: NULL pointer");
  if (!aligned16({x, delta, sum_out, weight, out}))
    return fail_msg(TIDE_ERR_INVALID, "rms_norm: pointers must be 16-byte aligned");
  const unsigned grid = grid_for(n_rows, 1, 148 * 16);
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t nv = hidden_dim / 8;
  const int vpt = nv <= dlayer::kNormThreads ? 1 : nv <= 2 * dlayer::kNormThreads ? 2
                : nv <= 4 * dlayer::kNormThreads ? 4 : 8;
  if (dtype == TIDE_DTYPE_BF16)
    launch_rms_norm<__nv_bfloat16>(vpt, grid, s, x, delta, sum_out, weight, out, n_rows,
                                   n_rows_dev, (int)hidden_dim, eps);
  else
    launch_rms_norm<__half>(vpt, grid, s, x, delta, sum_out, weight, out, n_rows, n_rows_dev,
                            (int)hidden_dim, eps);
  return launched("rms_norm");
}

extern "C" int tide_qk_norm_rope(int dtype, const void *q, const void *k, const void *v,
                                 int64_t q_row_stride, int64_t kv_row_stride,
                                 const void *q_norm_weight, const void *k_norm_weight, float eps,
                                 const float *inv_freq, float attention_scaling, int64_t position,
                                 const int32_t *position_dev, const int64_t *rope_positions,
                                 const int32_t *slots, const int32_t *n_rows_dev, int64_t n_rows,
                                 int64_t n_q_heads,
                                 int64_t n_kv_heads, int64_t head_dim, void *q_out, void *k_cache,
                                 void *v_cache, int64_t n_slots, int64_t max_len,
                                 int32_t *error_word, tide_stream_t stream) {
  using namespace tide;
  if (dtype != TIDE_DTYPE_BF16 && dtype != TIDE_DTYPE_F16)
    return fail_msg(TIDE_ERR_UNSUPPORTED, "qk_norm_rope: dtype must be bf16 or fp16");
  if (head_dim != 128) return fail_msg(TIDE_ERR_UNSUPPORTED, "qk_norm_rope: head_dim must be 128");
  if (n_rows < 0 || n_q_heads < 1 || n_kv_heads < 1 || n_slots < 1 || max_len < 1 ||
      (!position_dev && (position < 0 || position >= max_len)) || (!slots && n_rows > n_slots))
    return fail_msg(TIDE_ERR_INVALID, "qk_norm_rope: bad sizes or position");
  const int64_t q_stride = q_row_stride ? q_row_stride : n_q_heads * head_dim;
  const int64_t kv_stride = kv_row_stride ? kv_row_stride : n_kv_heads * head_dim;
  if (q_stride < n_q_heads * head_dim || kv_stride < n_kv_heads * head_dim || q_stride % 8 ||
      kv_stride % 8)
    return fail_msg(TIDE_ERR_INVALID,
                    "qk_norm_rope: row strides must cover the heads and be multiples of 8");
  if (n_rows == 0) return TIDE_OK;
  if (!q || !k || !v || !inv_freq || !q_out || !k_cache || !v_cache)
    return fail_msg(TIDE_ERR_INVALID, "qk_norm_rope: NULL pointer");
  if (!aligned16({q, k, v, q_out, k_cache, v_cache}))
    return fail_msg(TIDE_ERR_INVALID, "qk_norm_rope: pointers must be 16-byte aligned");
  // heads per warp: eight once there are rows enough to fill the GPU with
  // such groups (a prefill), else one (a decode step)
  const int64_t heads = n_q_heads + 2 * n_kv_heads;
  const int group = n_rows * heads >= 148 * 8 * 64 ? 8 : 1;
  const int64_t warps = n_rows * ((heads + group - 1) / group);
  const unsigned grid = grid_for(warps, 8, 148 * 16);
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == TIDE_DTYPE_BF16)
    qk_norm_rope_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16 *>(q), static_cast<const __nv_bfloat16 *>(k),
        static_cast<const __nv_bfloat16 *>(v), q_stride, kv_stride,
        static_cast<const __nv_bfloat16 *>(q_norm_weight),
        static_cast<const __nv_bfloat16 *>(k_norm_weight), eps, inv_freq, attention_scaling,
        position, position_dev, rope_positions, slots, n_rows_dev, n_rows, (int)n_q_heads,
        (int)n_kv_heads, static_cast<__nv_bfloat16 *>(q_out), static_cast<__nv_bfloat16 *>(k_cache),
        static_cast<__nv_bfloat16 *>(v_cache), n_slots, max_len, group, error_word);
  else
    qk_norm_rope_kernel<__half><<<grid, 256, 0, s>>>(
        static_cast<const __half *>(q), static_cast<const __half *>(k),
        static_cast<const __half *>(v), q_stride, kv_stride, static_cast<const __half *>(q_norm_weight),
        static_cast<const __half *>(k_norm_weight), eps, inv_freq, attention_scaling, position,
        position_dev, rope_positions, slots, n_rows_dev, n_rows, (int)n_q_heads, (int)n_kv_heads,
        static_cast<__half *>(q_out), static_cast<__half *>(k_cache),
        static_cast<__half *>(v_cache), n_slots, max_len, group, error_word);
  return launched("qk_norm_rope");
}

extern "C" int tide_silu_mul(int dtype, const void *gate, const void *up, void *out, int64_t n_rows,
                             const int32_t *n_rows_dev, int64_t width, tide_stream_t stream) {
  using namespace tide;
  if (dtype != TIDE_DTYPE_BF16 && dtype != TIDE_DTYPE_F16)
    return fail_msg(TIDE_ERR_UNSUPPORTED, "silu_mul: dtype must be bf16 or fp16");
  if (n_rows < 0 || width < 8 || width % 8)
    return fail_msg(TIDE_ERR_INVALID, "silu_mul: width must be a multiple of 8");
  if (n_rows == 0) return TIDE_OK;
  if (!gate || !up || !out) return fail_msg(TIDE_ERR_INVALID, "silu_mul: NULL pointer");
  if (!aligned16({gate, up, out}))
    return fail_msg(TIDE_ERR_INVALID, "silu_mul: pointers must be 16-byte aligned");
  const unsigned grid = grid_for(n_rows * width / 8, 256, 148 * 8);
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == TIDE_DTYPE_BF16)
    silu_mul_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16 *>(gate), static_cast<const __nv_bfloat16 *>(up),
        static_cast<__nv_bfloat16 *>(out), n_rows, n_rows_dev, width);
  else
    silu_mul_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half *>(gate),
                                                  static_cast<const __half *>(up),
                                                  static_cast<__half *>(out), n_rows, n_rows_dev,
                                                  width);
  return launched("silu_mul");
}
