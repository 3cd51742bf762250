// Decode attention over a KV cache addressed by slot, for the rows still
// active after the early-exit checkpoints of a decode step, and the append of
// a step's keys and values to that cache.
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
// Split over the positions (flash decoding): a thread-block cluster of S CTAs
// per (active row, KV head), CTA s taking the blocks of 128 positions s,
// s + S, s + 2S, ...  A CTA (eight warps, four at G = 8; warp w owns the
// positions 16w .. 16w + 15 of a block, 32w .. 32w + 31 with four warps)
// walks its blocks with a running maximum and sum per query head:
//   scores   on the tensor cores (mma.sync m16n8k16, 16-bit operands, fp32
//            accumulators): the G query heads as the rows of A, 8 key rows
//            as B, two (four) tiles per warp; the four lanes that hold a key row
//            in B read it from shared memory as four 16-byte chunks each;
//   softmax  one warp per query head: block maximum, rescale factor, the
//            block's probabilities and their sum;
//   P V      each lane of warp w: four output dimensions of all G heads over
//            the warp's positions; a warp reads one 256-byte value row per
//            position from shared memory.
// (Eight warps instead of four: the same bytes in flight, the compute
// between a block's arrival and the next request spread over twice the
// warps; 3-6 % faster.)
// The S partial results (running max m_s, sum l_s, unnormalised output a_s)
// are combined through distributed shared memory: after a cluster barrier
// CTA r computes its share of the G*128 outputs as
//   o = sum_s e^(m_s - M) a_s / sum_s e^(m_s - M) l_s,   M = max_s m_s,
// and a second barrier keeps every CTA's shared memory alive until all have
// read it.  Exponentials are base 2 on log2(e)-scaled scores.  fp32
// throughout; output in the cache's 16-bit type.
//
// Loads: a block's keys and its values go to shared memory by one bulk copy
// each (32 KB, two mbarriers, so the scores start when the keys have
// landed), so that a block is fetched in one round trip; a CTA's next block
// is requested after its P V.  (Keys loaded to registers by 16-byte loads per
// lane, and a second value buffer filled while the current block is used,
// both measured slower.)  After the last block the partial outputs reuse the
// same shared memory.  The waits are bounded: on expiry the kernel raises
// TIDE_DEVERR_TIMEOUT, requests nothing more, waits once more for the copies
// it has outstanding and still meets its cluster's barriers.
//
// The active row count and the length may live on the device (a
// checkpoint's counts, the decode position), so that a decode step needs no
// host value and can be captured in a CUDA graph.  Rows at or past the live
// count return at once, so the attention of a step costs what its active
// rows read.
#include <cooperative_groups.h>
#include <math.h>
#include <stdio.h>

#include <type_traits>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace cg = cooperative_groups;

namespace tide {

namespace dattn {
constexpr int kD = 128;        // head dimension
#ifndef TIDE_DATTN_WARPS
#define TIDE_DATTN_WARPS 8
#endif
// Warps per CTA: eight, except at G = 8, whose larger per-lane accumulators
// would spill at the register budget of three eight-warp CTAs per SM.
__host__ __device__ constexpr int warps_for(int G) { return G >= 8 ? 4 : TIDE_DATTN_WARPS; }
constexpr int kBlock = 128;    // positions per block

constexpr int kMaxSplit = 8;   // CTAs per cluster (portable cluster size)
#ifndef TIDE_DATTN_MIN_BLOCKS
#define TIDE_DATTN_MIN_BLOCKS 3
#endif
constexpr int kMinBlocks = TIDE_DATTN_MIN_BLOCKS;  // resident CTAs per SM (64 KB of shared memory each)
// Grid size the split aims at.  At 256 rows x 8 KV heads x 1024 positions
// (G = 4, eight warps): 2048 (no split) 198 us with every row active, 114 and
// 71 us with 128 and 64 of them; 2368 (pairs) 212, 112 and 65 us; the decode
// step 11.4 against 11.9 ms.
#ifndef TIDE_DATTN_TARGET_CTAS
#define TIDE_DATTN_TARGET_CTAS 2048
#endif
constexpr int64_t kTargetCtas = TIDE_DATTN_TARGET_CTAS;
constexpr float kLog2e = 1.4426950408889634f;
}  // namespace dattn

// Tensor-core tile of the scores: D[16 x 8] += A[16 x 16] * B[16 x 8],
// A = query heads (rows; G <= 8 real, the rest zero), B = 8 key rows,
// 16-bit operands, fp32 accumulators (mma.sync m16n8k16).
template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                          uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

template <typename T, int G>
__global__ void __launch_bounds__(32 * dattn::warps_for(G), dattn::kMinBlocks)
    decode_attention_kernel(const T *__restrict__ q, const T *__restrict__ kc,
                            const T *__restrict__ vc, const int32_t *__restrict__ slots,
                            T *__restrict__ o, int n_rows, const int32_t *__restrict__ n_dev,
                            int hq, int hkv, int64_t n_slots, int64_t max_len, int Lmax,
                            const int32_t *__restrict__ len_dev, float scale, int32_t *err) {
  using namespace dattn;
  constexpr int kWarps = warps_for(G);
  constexpr int kThreads = 32 * kWarps;
  constexpr int kPos = kBlock / kWarps;  // positions of a block per warp (scores and P V)
  static_assert(kPos % 8 == 0, "whole 8-position score tiles per warp");
  extern __shared__ __align__(128) unsigned char dyn_smem[];
  // [128 positions][128] each: the block's keys, then its values; after the
  // last block the per-warp partial outputs s_a[kWarps][G][128] (fp32, [0] =
  // the CTA's) take the same bytes
  T *s_k = reinterpret_cast<T *>(dyn_smem);
  T *s_v = s_k + kBlock * kD;
  float(*s_a)[G][kD] = reinterpret_cast<float(*)[G][kD]>(dyn_smem);
  static_assert(kWarps * G * kD * sizeof(float) <= 2 * kBlock * kD * sizeof(T),
                "s_a fits the block");
  __shared__ __align__(16) float s_p[G][kBlock];   // block scores, then probabilities
  __shared__ float s_m[G], s_l[G], s_alpha[G];
  __shared__ __align__(8) uint64_t bar_k, bar_v;
  __shared__ int s_abort;

  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();
  const int split = (int)cluster.block_rank();
  const int64_t unit = (int64_t)blockIdx.x / S;  // row * hkv + kv head
  const int row = (int)(unit / hkv), kvh = (int)(unit % hkv);
  // Every early return below depends on (row, kv head) only, so a whole
  // cluster leaves together and no CTA waits at a barrier for one that left.
  if (row >= n_rows) return;
  if (n_dev && row >= __ldg(n_dev)) return;  // past the live row count
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t slot = slots ? (int64_t)__ldg(slots + row) : row;
  if (slot < 0 || slot >= n_slots) {  // a slot outside the cache: the row is skipped
    if (tid == 0 && split == 0) raise_error(err, TIDE_DEVERR_POSITION);
    return;
  }
  const int L = len_dev ? min(max(__ldg(len_dev), 1), Lmax) : Lmax;
  const T *kb = kc + ((slot * hkv + kvh) * max_len) * kD;
  const T *vb = vc + ((slot * hkv + kvh) * max_len) * kD;

  if (tid == 0) {
    ptx::mbar_init(&bar_k, 1);
    ptx::mbar_init(&bar_v, 1);
    ptx::fence_mbar_init();
    s_abort = 0;
  }
  if (tid < G) {
    s_m[tid] = -INFINITY;
    s_l[tid] = 0.f;
  }
  __syncthreads();
  const uint64_t pol = l2_evict_first_policy();  // the cache is read once per step
  // a block's keys and values: one bulk copy each (thread 0)
  auto load_block = [&](int b) {
    const uint32_t bytes = (uint32_t)min(kBlock, L - b) * kD * (uint32_t)sizeof(T);
    ptx::mbar_expect_tx(&bar_k, bytes);
    ptx::bulk_load(s_k, kb + (int64_t)b * kD, bytes, &bar_k, pol);
    ptx::mbar_expect_tx(&bar_v, bytes);
    ptx::bulk_load(s_v, vb + (int64_t)b * kD, bytes, &bar_v, pol);
  };
  // Keys: lane (n = lane / 4, t = lane % 4) of warp w holds, for n-tile it,
  // 32 dims of block position w*32 + it*8 + n as four 16-byte chunks, chunk c
  // = dims (c*4 + t)*8 .. +8.  They are the B fragments of the score tiles:
  // k-step 2c + h takes the chunk's words 2h and 2h+1.  The query's A
  // fragments use the same dims for row n (query head n < G), so each tile's
  // k order is a permutation shared by both operands.
  const int t4 = lane & 3, n8 = lane >> 2;
  if (tid == 0 && split * kBlock < L) load_block(split * kBlock);
  uint4 qf[4];
  if (n8 < G) {
    const T *qr = q + ((int64_t)row * hq + kvh * G + n8) * kD;
#pragma unroll
    for (int c = 0; c < 4; ++c) qf[c] = *reinterpret_cast<const uint4 *>(qr + (c * 4 + t4) * 8);
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c) qf[c] = make_uint4(0, 0, 0, 0);
  }
  const float qs = scale * kLog2e;
  uint32_t phase = 0;
  int late_k = -1, late_v = -1;  // the phases of waits that expired, if any

  float acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;

  // blocks split, split + S, ... of 128 positions (none when S exceeds the
  // block count: that CTA's partial result is empty)
  for (int b0 = split * kBlock; b0 < L; b0 += S * kBlock) {
    const int nb = min(kBlock, L - b0);
    // the block's keys in shared memory (bounded wait, as for the values)
    if (!ptx::mbar_wait(&bar_k, phase, &s_abort)) {
      if (lane == 0) raise_error(err, TIDE_DEVERR_TIMEOUT);
      s_abort = 1;
      late_k = (int)phase;
    }
    // scores: four 16 x 8 tiles per warp, eight k-steps each; rows at or
    // past nb hold an earlier block's keys (or nothing) and are masked below
#pragma unroll
    for (int it = 0; it < kPos / 8; ++it) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      const T *kr = s_k + (warp * kPos + it * 8 + n8) * kD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 kc4 = *reinterpret_cast<const uint4 *>(kr + (c * 4 + t4) * 8);
        mma_16816<T>(d, qf[c].x, qf[c].y, kc4.x, kc4.y);
        mma_16816<T>(d, qf[c].z, qf[c].w, kc4.z, kc4.w);
      }
      // d[0], d[1]: head n8 at block positions w*32 + it*8 + 2*t4 + {0, 1}
      if (n8 < G) {
        const int t = warp * kPos + it * 8 + 2 * t4;
        *reinterpret_cast<float2 *>(&s_p[n8][t]) =
            make_float2(t < nb ? d[0] * qs : -INFINITY, t + 1 < nb ? d[1] * qs : -INFINITY);
      }
    }
    __syncthreads();
    // softmax of the block, one warp per query head
    for (int g = warp; g < G; g += kWarps) {
      float v[4], mx = -INFINITY;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[k] = s_p[g][lane + 32 * k];
        mx = fmaxf(mx, v[k]);
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = s_m[g];
      const float m_new = fmaxf(m_old, mx);  // finite: the block holds a position
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float p = exp2f(v[k] - m_new);  // -inf (past the range) -> 0
        s_p[g][lane + 32 * k] = p;
        sum += p;
      }
      sum = warp_sum(sum);
      __syncwarp();
      if (lane == 0) {
        const float alpha = exp2f(m_old - m_new);  // 0 on the first block
        s_alpha[g] = alpha;
        s_l[g] = s_l[g] * alpha + sum;
        s_m[g] = m_new;
      }
    }
    __syncthreads();
    // P V: warp w takes block positions w*32 .. w*32+31, each lane four
    // output dimensions of all G heads
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float a = s_alpha[g];
      acc[g][0] *= a;
      acc[g][1] *= a;
      acc[g][2] *= a;
      acc[g][3] *= a;
    }
    // the block's values in shared memory (bounded wait; on expiry the
    // error is raised and the block's output is not to be used)
    if (!ptx::mbar_wait(&bar_v, phase, &s_abort)) {
      if (lane == 0) raise_error(err, TIDE_DEVERR_TIMEOUT);
      s_abort = 1;
      late_v = (int)phase;
    }
    phase ^= 1u;
    const int p0 = warp * kPos, p1 = min(nb, p0 + kPos);
    for (int t0 = p0; t0 < p1; t0 += 4) {
      float4 pg[G];
#pragma unroll
      for (int g = 0; g < G; ++g) pg[g] = *reinterpret_cast<const float4 *>(&s_p[g][t0]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (t0 + u < p1) {
          const uint2 vv = *reinterpret_cast<const uint2 *>(s_v + (t0 + u) * kD + lane * 4);
          const T *e4 = reinterpret_cast<const T *>(&vv);
          const float f0 = Elem<T>::to_f(e4[0]), f1 = Elem<T>::to_f(e4[1]);
          const float f2 = Elem<T>::to_f(e4[2]), f3 = Elem<T>::to_f(e4[3]);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float p = u == 0 ? pg[g].x : u == 1 ? pg[g].y : u == 2 ? pg[g].z : pg[g].w;
            acc[g][0] = fmaf(p, f0, acc[g][0]);
            acc[g][1] = fmaf(p, f1, acc[g][1]);
            acc[g][2] = fmaf(p, f2, acc[g][2]);
            acc[g][3] = fmaf(p, f3, acc[g][3]);
          }
        }
      }
    }
    __syncthreads();  // s_p, s_alpha, the keys and values are rewritten by the next block
    // (nothing more is requested once a wait has expired: at most one copy
    // per barrier is ever outstanding)
    if (tid == 0 && b0 + S * kBlock < L && !s_abort) load_block(b0 + S * kBlock);
  }

  if (tid == 0) {  // after an expired wait a copy may still be landing: wait for it once more
    volatile int none = 0;
    if (late_k >= 0) ptx::mbar_wait(&bar_k, (uint32_t)late_k, &none);
    if (late_v >= 0) ptx::mbar_wait(&bar_v, (uint32_t)late_v, &none);
  }
  __syncthreads();  // the key and value buffers become s_a
  // this CTA's unnormalised output: sum of the warps' partials
#pragma unroll
  for (int g = 0; g < G; ++g)
    *reinterpret_cast<float4 *>(&s_a[warp][g][lane * 4]) =
        make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
  __syncthreads();
  for (int e = tid; e < G * kD; e += kThreads) {
    const int g = e / kD, d = e % kD;
    float sum = s_a[0][g][d];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) sum += s_a[w][g][d];
    s_a[0][g][d] = sum;
  }

  cluster.sync();  // every CTA's m, l and output are in its shared memory
  constexpr int kOut = G * kD;
  const int share = (kOut + S - 1) / S;
  const int e_end = min(kOut, (split + 1) * share);
  for (int e = split * share + tid; e < e_end; e += kThreads) {
    const int g = e / kD, d = e % kD;
    float m[kMaxSplit], l[kMaxSplit], a[kMaxSplit];
#pragma unroll
    for (int r = 0; r < kMaxSplit; ++r) {  // independent remote reads, issued together
      if (r < S) {
        m[r] = cluster.map_shared_rank(&s_m[0], r)[g];
        l[r] = cluster.map_shared_rank(&s_l[0], r)[g];
        a[r] = cluster.map_shared_rank(&s_a[0][0][0], r)[g * kD + d];
      } else {
        m[r] = -INFINITY;
        l[r] = a[r] = 0.f;
      }
    }
    float M = m[0];  // CTA 0 always holds block 0: finite
#pragma unroll
    for (int r = 1; r < kMaxSplit; ++r) M = fmaxf(M, m[r]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxSplit; ++r) {
      const float w = exp2f(m[r] - M);  // a CTA without positions: 0
      den = fmaf(w, l[r], den);
      num = fmaf(w, a[r], num);
    }
    o[((int64_t)row * hq + kvh * G + g) * kD + d] = Elem<T>::from_f(num / den);
  }
  cluster.sync();  // no CTA leaves while another still reads its shared memory
}

// Append one decode position: k/v_new [n_rows, hkv, 128] go to
// cache[slots[i], :, pos, :] for i below the live row count.  One warp per
// (row, KV head), 8 bytes per lane.
template <typename T>
__global__ void kv_append_kernel(const T *__restrict__ k_new, const T *__restrict__ v_new,
                                 const int32_t *__restrict__ slots, const int32_t *__restrict__ n_dev,
                                 int64_t n_rows, int hkv, T *__restrict__ kc, T *__restrict__ vc,
                                 int64_t n_slots, int64_t max_len, int64_t pos,
                                 const int32_t *__restrict__ pos_dev, int32_t *err) {
  const int lane = threadIdx.x & 31;
  int64_t live = n_rows;
  if (n_dev) live = min((int64_t)max(__ldg(n_dev), 0), n_rows);
  const int64_t p = pos_dev ? (int64_t)__ldg(pos_dev) : pos;
  if (p < 0 || p >= max_len) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && live > 0) raise_error(err, TIDE_DEVERR_POSITION);
    return;
  }
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); w < live * hkv;
       w += warps) {
    const int64_t i = w / hkv;
    const int h = (int)(w % hkv);
    const int64_t slot = slots ? (int64_t)slots[i] : i;
    if (slot < 0 || slot >= n_slots) {
      if (lane == 0) raise_error(err, TIDE_DEVERR_POSITION);
      continue;
    }
    const int64_t src = (i * hkv + h) * dattn::kD + lane * 4;
    const int64_t dst = ((slot * hkv + h) * max_len + p) * dattn::kD + lane * 4;
    *reinterpret_cast<uint2 *>(kc + dst) = *reinterpret_cast<const uint2 *>(k_new + src);
    *reinterpret_cast<uint2 *>(vc + dst) = *reinterpret_cast<const uint2 *>(v_new + src);
  }
}

void set_last_error(const char *msg);

}  // namespace tide

namespace {

template <typename T, int G>
cudaError_t launch_attention(const void *q, const void *k_cache, const void *v_cache,
                             const int32_t *slots, void *out, int64_t n_rows,
                             const int32_t *n_rows_dev, int hq, int hkv, int64_t n_slots,
                             int64_t max_len, int length, const int32_t *length_dev, float scale,
                             int32_t *error_word, int splits, cudaStream_t s) {
  const size_t dyn = 2 * tide::dattn::kBlock * tide::dattn::kD * sizeof(T);
  static bool attr_set = false;  // per instantiation: static + dynamic exceed 48 KB at G = 8
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(tide::decode_attention_kernel<T, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
    if (e != cudaSuccess) return e;
    // the whole unified L1 / shared array as shared memory: three CTAs of
    // 64 KB of keys and values each per SM
    e = cudaFuncSetAttribute(tide::decode_attention_kernel<T, G>,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n_rows * hkv * splits), 1, 1);
  cfg.blockDim = dim3(32 * tide::dattn::warps_for(G), 1, 1);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tide::decode_attention_kernel<T, G>, static_cast<const T *>(q),
                            static_cast<const T *>(k_cache), static_cast<const T *>(v_cache),
                            slots, static_cast<T *>(out), (int)n_rows, n_rows_dev, hq, hkv,
                            n_slots, max_len, length, length_dev, scale, error_word);
}

template <typename T>
cudaError_t launch_attention_g(int G, const void *q, const void *k_cache, const void *v_cache,
                               const int32_t *slots, void *out, int64_t n_rows,
                               const int32_t *n_rows_dev, int hq, int hkv, int64_t n_slots,
                               int64_t max_len, int length, const int32_t *length_dev,
                               float scale, int32_t *error_word, int splits, cudaStream_t s) {
  switch (G) {
    case 1:
      return launch_attention<T, 1>(q, k_cache, v_cache, slots, out, n_rows, n_rows_dev, hq, hkv,
                                    n_slots, max_len, length, length_dev, scale, error_word,
                                    splits, s);
    case 2:
      return launch_attention<T, 2>(q, k_cache, v_cache, slots, out, n_rows, n_rows_dev, hq, hkv,
                                    n_slots, max_len, length, length_dev, scale, error_word,
                                    splits, s);
    case 4:
      return launch_attention<T, 4>(q, k_cache, v_cache, slots, out, n_rows, n_rows_dev, hq, hkv,
                                    n_slots, max_len, length, length_dev, scale, error_word,
                                    splits, s);
    default:
      return launch_attention<T, 8>(q, k_cache, v_cache, slots, out, n_rows, n_rows_dev, hq, hkv,
                                    n_slots, max_len, length, length_dev, scale, error_word,
                                    splits, s);
  }
}

int report(cudaError_t e, const char *what) {
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    tide::set_last_error(buf);
    return TIDE_ERR_CUDA;
  }
  return TIDE_OK;
}

}  // namespace

extern "C" int tide_decode_attention(int dtype, const void *q, const void *k_cache,
                                     const void *v_cache, const int32_t *slots, void *out,
                                     int64_t n_rows, const int32_t *n_rows_dev,
                                     int64_t n_q_heads, int64_t n_kv_heads, int64_t head_dim,
                                     int64_t n_slots, int64_t max_len, int64_t length,
                                     const int32_t *length_dev, float scale,
                                     int32_t *error_word, tide_stream_t stream) {
  using namespace tide;
  if (dtype != TIDE_DTYPE_BF16 && dtype != TIDE_DTYPE_F16) {
    tide::set_last_error("decode_attention: dtype must be bf16 or fp16");
    return TIDE_ERR_UNSUPPORTED;
  }
  if (head_dim != dattn::kD) {
    tide::set_last_error("decode_attention: head_dim must be 128");
    return TIDE_ERR_UNSUPPORTED;
  }
  const int64_t G = n_kv_heads > 0 ? n_q_heads / n_kv_heads : 0;
  if (n_rows < 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0 ||
      (G != 1 && G != 2 && G != 4 && G != 8) || length < 1 || length > max_len ||
      length > INT32_MAX || n_slots < 1 || (!slots && n_rows > n_slots) ||
      n_rows * n_kv_heads * dattn::kMaxSplit > INT32_MAX) {
    tide::set_last_error("decode_attention: bad sizes (heads: G of 1, 2, 4 or 8; length)");
    return TIDE_ERR_INVALID;
  }
  if (n_rows == 0) return TIDE_OK;
  if (!q || !k_cache || !v_cache || !out) {
    tide::set_last_error("decode_attention: NULL pointer");
    return TIDE_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
       reinterpret_cast<uintptr_t>(q)) & 15) {
    tide::set_last_error("decode_attention: q and the caches must be 16-byte aligned");
    return TIDE_ERR_INVALID;
  }
  // Positions split over a cluster of up to 8 CTAs (at most one per block of
  // 128): as few as keep about kTargetCtas CTAs in the grid, since every
  // CTA pays a fixed cost (its first round trip, the cluster combine).  The
  // split follows the row capacity (n_rows), not the live count on the
  // device.
  const int64_t blocks = (length + dattn::kBlock - 1) / dattn::kBlock;
  const int64_t units = n_rows * n_kv_heads;
  int64_t splits = dattn::kTargetCtas > 0 ? (dattn::kTargetCtas + units - 1) / units : blocks;
  if (splits > blocks) splits = blocks;
  if (splits > dattn::kMaxSplit) splits = dattn::kMaxSplit;
  if (splits < 1) splits = 1;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  if (dtype == TIDE_DTYPE_BF16)
    e = launch_attention_g<__nv_bfloat16>((int)G, q, k_cache, v_cache, slots, out, n_rows,
                                          n_rows_dev, (int)n_q_heads, (int)n_kv_heads, n_slots,
                                          max_len, (int)length, length_dev, scale, error_word,
                                          (int)splits, s);
  else
    e = launch_attention_g<__half>((int)G, q, k_cache, v_cache, slots, out, n_rows, n_rows_dev,
                                   (int)n_q_heads, (int)n_kv_heads, n_slots, max_len, (int)length,
                                   length_dev, scale, error_word, (int)splits, s);
  return report(e, "decode_attention");
}

extern "C" int tide_kv_append(int dtype, const void *k_new, const void *v_new,
                              const int32_t *slots, const int32_t *n_rows_dev, int64_t n_rows,
                              int64_t n_kv_heads, int64_t head_dim, void *k_cache, void *v_cache,
                              int64_t n_slots, int64_t max_len, int64_t position,
                              const int32_t *position_dev, int32_t *error_word,
                              tide_stream_t stream) {
  using namespace tide;
  if (dtype != TIDE_DTYPE_BF16 && dtype != TIDE_DTYPE_F16) {
    tide::set_last_error("kv_append: dtype must be bf16 or fp16");
    return TIDE_ERR_UNSUPPORTED;
  }
  if (head_dim != dattn::kD) {
    tide::set_last_error("kv_append: head_dim must be 128");
    return TIDE_ERR_UNSUPPORTED;
  }
  if (n_rows < 0 || n_kv_heads <= 0 || n_slots < 1 || max_len < 1 ||
      (!position_dev && (position < 0 || position >= max_len)) || (!slots && n_rows > n_slots)) {
    tide::set_last_error("kv_append: bad sizes or position");
    return TIDE_ERR_INVALID;
  }
  if (n_rows == 0) return TIDE_OK;
  if (!k_new || !v_new || !k_cache || !v_cache) {
    tide::set_last_error("kv_append: NULL pointer");
    return TIDE_ERR_INVALID;
  }
  const int64_t warps = n_rows * n_kv_heads;
  int64_t blocks = (warps + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == TIDE_DTYPE_BF16)
    kv_append_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16 *>(k_new), static_cast<const __nv_bfloat16 *>(v_new),
        slots, n_rows_dev, n_rows, (int)n_kv_heads, static_cast<__nv_bfloat16 *>(k_cache),
        static_cast<__nv_bfloat16 *>(v_cache), n_slots, max_len, position, position_dev,
        error_word);
  else
    kv_append_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(
        static_cast<const __half *>(k_new), static_cast<const __half *>(v_new), slots, n_rows_dev,
        n_rows, (int)n_kv_heads, static_cast<__half *>(k_cache), static_cast<__half *>(v_cache),
        n_slots, max_len, position, position_dev, error_word);
  return report(cudaSuccess, "kv_append");
}
