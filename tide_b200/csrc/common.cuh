// Shared device helpers for the sm_100a early-exit kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tide_b200.h"

namespace tide {

// ---------------------------------------------------------------- elements
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// A 16-byte vector holds kVec<T> elements.
template <typename T> constexpr int kVec = 16 / (int)sizeof(T);

template <typename T>
__device__ __forceinline__ void unpack16(const uint4 &v, float *f) {
  const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
  for (int i = 0; i < kVec<T>; ++i) f[i] = Elem<T>::to_f(e[i]);
}
template <typename T>
__device__ __forceinline__ uint4 pack16(const float *f) {
  uint4 v;
  T *e = reinterpret_cast<T *>(&v);
#pragma unroll
  for (int i = 0; i < kVec<T>; ++i) e[i] = Elem<T>::from_f(f[i]);
  return v;
}

// Streaming 16-byte global accesses.  Rows are read once by the movers, so
// their loads carry an L2 evict-first policy: lines they bring in from DRAM
// are the first to go, and what the router left in L2 (the late column
// chunks of every row) survives until the movers reach it.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(l2_evict_first_policy()));
  return v;
}
__device__ __forceinline__ void st_stream(uint4 *p, const uint4 &v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// ------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Correctly rounded 1/sqrt(v): one IEEE sqrt and one IEEE division, the same
// two roundings as torch.rsqrt's CPU path.
__device__ __forceinline__ float rsqrt_rn(float v) { return __fdiv_rn(1.0f, __fsqrt_rn(v)); }

// SiLU and sigmoid in fp32 (x * sigmoid(x), 1 / (1 + e^-x)).
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
// Fast SiLU for the fp32 tensor-core router (scores held to 1e-5): the
// hardware exponential and the approximate division, a few 1e-6 relative at
// most over the logits' range, and no branches, so an unrolled loop of them
// keeps the MUFU pipe busy.  The
// exponent is clamped at 80 (e^80 < 2^126, inside __fdividef's range); below
// -80 SiLU is 0 to fp32 precision anyway.
__device__ __forceinline__ float silu_fast(float x) {
  return __fdividef(x, 1.0f + __expf(fminf(-x, 80.0f)));
}
// SiLU through one hardware tanh: x * sigmoid(x) = 0.5 x (1 + tanh(x / 2)).
// tanh.approx.f32 is within ~5e-4 relative (absolute near 0), so a router
// logit summed over 128 units moves by ~1e-4, inside the 1e-2 score bar.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float silu_tanh(float x) {
  const float h = 0.5f * x;
  return fmaf(h, tanh_approx(h), h);
}

__device__ __forceinline__ void raise_error(int32_t *err, int bits) {
  if (err) atomicOr(err, bits);
}

// -------------------------------------------------------------- look-back
// Tile status word for the single-pass stable partition (decoupled
// look-back, Merrill & Garland 2016): bits 62-63 flag, 31-61 exit count,
// 0-30 survivor count.
constexpr uint64_t kFlagAggregate = 1ull << 62;
constexpr uint64_t kFlagPrefix = 2ull << 62;
constexpr uint64_t kCountMask = (1ull << 31) - 1;
// Spin bound for a look-back wait.  A predecessor tile is always held by a
// running CTA (tiles are handed out in ticket order), so this only expires
// if the device is wedged; the kernel then flags TIDE_DEVERR_TIMEOUT.
//
// The test build of the library (libtide_b200_testhooks.so, compiled with
// TIDE_TEST_UNPUBLISHED_TILE=t) makes that happen on purpose without any
// fault: tile t computes its own prefix but never publishes its status, so
// the look-back of the tiles after it waits on a word nothing sets, gives up
// after a short bound and reports TIDE_DEVERR_TIMEOUT.  The product build
// has no such tile.
#ifdef TIDE_TEST_UNPUBLISHED_TILE
constexpr int kSpinLimit = 1 << 12;
#else
constexpr int kSpinLimit = 1 << 24;
#endif

__device__ __forceinline__ bool unpublished_test_tile(uint32_t tile) {
#ifdef TIDE_TEST_UNPUBLISHED_TILE
  return tile == (uint32_t)(TIDE_TEST_UNPUBLISHED_TILE);
#else
  (void)tile;
  return false;
#endif
}

__device__ __forceinline__ uint64_t pack_status(uint64_t flag, uint32_t keep, uint32_t exits) {
  return flag | ((uint64_t)exits << 31) | (uint64_t)keep;
}
// The status words carry their own counts, so publishing and polling them
// needs no ordering with other memory: relaxed gpu-scope accesses suffice and
// avoid waiting for this thread's earlier stores at every publication.
__device__ __forceinline__ uint64_t ld_status(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_status(uint64_t *p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Decoupled look-back for tile `tile`: publishes this tile's aggregate,
// accumulates predecessors until an inclusive prefix is found, publishes the
// inclusive prefix and returns the exclusive one.  Called by one thread.
// Returns false if a wait expired (prefix then undefined).
__device__ __forceinline__ bool lookback(uint64_t *status, uint32_t tile, uint32_t keep,
                                         uint32_t exits, uint32_t *keep_before,
                                         uint32_t *exits_before) {
  uint32_t kb = 0, eb = 0;
  const bool publish = !unpublished_test_tile(tile);
  if (tile == 0) {
    if (publish) st_status(&status[0], pack_status(kFlagPrefix, keep, exits));
    *keep_before = 0;
    *exits_before = 0;
    return true;
  }
  if (publish) st_status(&status[tile], pack_status(kFlagAggregate, keep, exits));
  int64_t j = (int64_t)tile - 1;
  bool ok = true;
  while (j >= 0) {
    uint64_t s = 0;
    int spins = 0;
    while (((s = ld_status(&status[j])) >> 62) == 0) {
      if (++spins > kSpinLimit) { ok = false; break; }
      __nanosleep(32);
    }
    if (!ok) break;
    kb += (uint32_t)(s & kCountMask);
    eb += (uint32_t)((s >> 31) & kCountMask);
    if ((s >> 62) == 2) break;
    --j;
  }
  if (publish) st_status(&status[tile], pack_status(kFlagPrefix, kb + keep, eb + exits));
  *keep_before = kb;
  *exits_before = eb;
  return ok;
}

// Warp-wide decoupled look-back: the 32 lanes read 32 predecessors per
// round trip (lane l reads tile base - l) and stop at the nearest inclusive
// prefix, waiting only for the predecessors in front of it.  Where many
// tiles are in flight at once (small clusters, many of them), one thread
// reading one predecessor per round trip would walk the whole wave.  With
// `publish`, lane 0 publishes the tile's aggregate first and its inclusive
// prefix at the end.  Every lane gets the exclusive prefix.  Called by a
// whole warp; returns false (warp-uniformly) if a wait expired, the prefix
// then being a lower bound.
__device__ __forceinline__ bool warp_lookback(uint64_t *status, uint32_t tile, uint32_t keep,
                                              uint32_t exits, bool publish, uint32_t *keep_before,
                                              uint32_t *exits_before) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  publish = publish && !unpublished_test_tile(tile);
  if (publish && lane == 0)
    st_status(&status[tile], pack_status(tile == 0 ? kFlagPrefix : kFlagAggregate, keep, exits));
  uint32_t kb = 0, eb = 0;
  bool ok = true;
  for (int64_t base = (int64_t)tile - 1; base >= 0; base -= 32) {
    const int64_t j = base - lane;
    // before tile 0: an empty inclusive prefix
    uint64_t s = j >= 0 ? ld_status(&status[j]) : kFlagPrefix;
    uint32_t incl = 0;
    int stop = 31;
    for (int spins = 0;; ++spins) {
      incl = __ballot_sync(full, (s >> 62) == 2);
      stop = incl ? __ffs(incl) - 1 : 31;
      const bool wait_me = (s >> 62) == 0 && lane <= stop;
      if (!__any_sync(full, wait_me)) break;
      if (spins > kSpinLimit) { ok = false; break; }
      __nanosleep(32);
      if (wait_me) s = ld_status(&status[j]);
    }
    if (!ok) break;
    uint32_t k = lane <= stop ? (uint32_t)(s & kCountMask) : 0u;
    uint32_t e = lane <= stop ? (uint32_t)((s >> 31) & kCountMask) : 0u;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      k += __shfl_xor_sync(full, k, o);
      e += __shfl_xor_sync(full, e, o);
    }
    kb += k;
    eb += e;
    if (incl) break;
  }
  if (publish && lane == 0 && tile != 0)
    if (publish) st_status(&status[tile], pack_status(kFlagPrefix, kb + keep, eb + exits));
  *keep_before = kb;
  *exits_before = eb;
  return ok;
}

}  // namespace tide
