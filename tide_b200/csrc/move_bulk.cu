// Stable partition + row moves with bulk copies (sm_100a).
//
// Same contract as move_rows_kernel (simt_kernels.cuh): rows whose decision
// is "keep" go to compact_out in order with their position / slot, rows that
// exit go to out_buf at their position (final-normed from the row
// statistics, or copied raw), and counts = {survivors, exits}.  Reference
// semantics: python/TIDE/runtime.py:164-178 (compaction of the active rows and
// the exit scatter) and csrc/kernels/batch_compact.cu (stable order).
//
// The data path never goes through registers for survivors: each row is one
// cp.async.bulk load into a shared-memory slot and one cp.async.bulk store
// from it, so a CTA keeps ~190 KB of rows in flight with a handful of
// threads.  One persistent CTA per SM:
//   warp 0      scheduler: takes 32-row tiles in ticket order, decides each
//               row (score > threshold), publishes the tile's aggregate and
//               runs the decoupled look-back (Merrill & Garland 2016) for the
//               tile's exclusive prefix, then writes the positions / slots /
//               exit positions of the tile's rows itself;
//   warps 1, 10 loaders: one bulk load per row that has data to move, into
//               the ring of row slots, as soon as the tile's rows are known
//               (before its prefix is); warp 1 issues the even slot
//               sequence numbers, warp 10 the odd ones (issuing a copy holds
//               the issuing thread for ~0.3 us, which at 4 KB rows would cap
//               one loader near 2 TB/s);
//   warps 2-9   movers: slot q belongs to mover q % 8; a survivor is stored
//               with one bulk store to compact_out[prefix + rank]; an exit is
//               normed from shared memory by the warp and written with
//               16-byte stores, or bulk-stored raw.  A mover leaves its
//               stores reading their slots while it goes on and frees them
//               oldest first, at the latest before it waits for sequence q:
//               then every slot of sequence <= q - slots is free, which is
//               the one a loader needs for q, so a loader never waits on a
//               slot whose mover is waiting on it (each mover's sequence
//               numbers share one parity: it is fed by one loader).
// Every wait is bounded; on expiry the kernel sets TIDE_DEVERR_TIMEOUT, stops
// all roles, waits for its own loads in flight and returns.  Launched as a
// programmatic dependent of the router: the barriers are set up before
// griddepcontrol.wait, nothing global is touched before it.
#include "move_bulk.cuh"
#include "tc_ptx.cuh"

namespace tide {

namespace {

constexpr int kTileRows = 32;
constexpr int kMovers = 8;   // even: the slot sequence q of mover q % 8 has one parity
constexpr int kLoaders = 2;  // loader of slot sequence q: q % 2
constexpr int kThreads = 32 * (2 + kMovers + 1);
constexpr int kTiles = 4;       // tile descriptors in flight
constexpr int kMaxSlots = 64;
constexpr int kSmemBudget = 227 * 1024;
constexpr int kAux = 4096;      // barriers, descriptors, flags
constexpr uint32_t kMinRowBytes = 2048;
// 16-byte vectors per lane in flight when norming an exit row: eight for
// RMSNorm (weights only), four for LayerNorm (weights and bias), which keeps
// both within the registers of one CTA per SM without spills
template <bool LN> constexpr int kExitUnroll = LN ? 4 : 8;
constexpr int kMaxPending = 0;  // bulk stores a mover leaves reading their slots (more measured slower)

struct TileDesc {
  int64_t row0;
  uint32_t keep_mask, exit_mask, move_mask;
  uint32_t keep_before, exits_before;
  uint32_t n_move;
  uint32_t done;  // rows of the tile finished by movers (shared atomic)
  int32_t end;    // no more tiles
};

struct SlotDesc {
  uint8_t tile;    // tile descriptor index
  uint8_t row;     // row within the tile
  uint8_t parity;  // phase parity of the tile descriptor's barriers
  uint8_t end;     // no more rows for this mover
};

struct BulkSmem {
  uint64_t *full, *empty;                   // [slots]
  uint64_t *td_rows, *td_prefix, *td_free;  // [kTiles]
  SlotDesc *sdesc;                          // [slots]
  TileDesc *td;                             // [kTiles]
  volatile int *abort_flag;
  uint32_t *issued;                         // [2] next slot sequence of each loader
};

__device__ __forceinline__ BulkSmem carve(uint8_t *aux, int NS) {
  BulkSmem m;
  uint64_t *b = reinterpret_cast<uint64_t *>(aux);
  m.full = b;
  m.empty = b + NS;
  m.td_rows = b + 2 * NS;
  m.td_prefix = m.td_rows + kTiles;
  m.td_free = m.td_prefix + kTiles;
  m.sdesc = reinterpret_cast<SlotDesc *>(m.td_free + kTiles);
  m.td = reinterpret_cast<TileDesc *>(m.sdesc + kMaxSlots);
  m.abort_flag = reinterpret_cast<volatile int *>(m.td + kTiles);
  m.issued = reinterpret_cast<uint32_t *>(m.td + kTiles) + 1;  // two words
  return m;
}

__device__ __forceinline__ void fail(const MoveParams &p, const BulkSmem &m) {
  raise_error(p.err, TIDE_DEVERR_TIMEOUT);
  *m.abort_flag = 1;
}

template <typename T, bool LN>
__global__ void __launch_bounds__(kThreads, 1) move_rows_bulk_kernel(MoveParams p, int NS, int staged) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const uint32_t row_bytes = (uint32_t)(p.H * (int64_t)sizeof(T));
  uint8_t *slots = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  BulkSmem m = carve(slots + (size_t)NS * row_bytes, NS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the final norm's weight (bit 0) and bias (bit 1) vectors, staged in
  // shared memory when they fit beside the slots: an exit row reads the
  // whole weight vector, which otherwise partly misses L1 under the slots
  float *s_w = reinterpret_cast<float *>(slots + (size_t)NS * row_bytes + kAux);
  float *s_b = s_w + ((staged & 1) ? p.H : 0);
  // model weights, never written by the kernel this one overlaps with
  for (int64_t i = threadIdx.x; i < p.H; i += kThreads) {
    if (staged & 1) s_w[i] = p.w_norm[i];
    if (staged & 2) s_b[i] = p.b_norm[i];
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(&m.full[s], 1);
      ptx::mbar_init(&m.empty[s], 1);
    }
    for (int e = 0; e < kTiles; ++e) {
      ptx::mbar_init(&m.td_rows[e], 1);
      ptx::mbar_init(&m.td_prefix[e], 1);
      ptx::mbar_init(&m.td_free[e], kLoaders + 1);  // both loaders done with it + last row moved
    }
    *m.abort_flag = 0;
    m.issued[0] = 0;
    m.issued[1] = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async();
  }
  __syncthreads();
  ptx::grid_dependency_wait();
  if (threadIdx.x == 0) ptx::grid_dependents_launch();

  int64_t n = p.n_cap;
  if (p.n_dev) {
    int64_t nd = (int64_t)__ldg(p.n_dev);
    if (nd < 0 || nd > p.n_cap) {
      if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(p.err, TIDE_DEVERR_COUNT);
      nd = nd < 0 ? 0 : p.n_cap;
    }
    n = nd;
  }
  const int64_t n_tiles = n > 0 ? (n + kTileRows - 1) / kTileRows : 1;

  const uint64_t pol = l2_evict_first_policy();
  const T *x = static_cast<const T *>(p.x);

  if (warp == 0) {
    // ------------------------------------------------------------ scheduler
    const uint32_t lt = (1u << lane) - 1u;
    for (uint32_t k = 0;; ++k) {
      const int e = (int)(k % kTiles);
      const uint32_t use = k / kTiles;
      if (k >= (uint32_t)kTiles && !ptx::mbar_wait(&m.td_free[e], (use & 1u) ^ 1u, m.abort_flag)) {
        if (lane == 0) fail(p, m);
        break;
      }
      if (*m.abort_flag) break;
      uint32_t tile = 0;
      if (lane == 0) tile = atomicAdd(p.ticket, 1u);
      tile = __shfl_sync(0xffffffffu, tile, 0);
      TileDesc &d = m.td[e];
      if ((int64_t)tile >= n_tiles) {
        if (lane == 0) {
          d.end = 1;
          ptx::mbar_arrive(&m.td_rows[e]);
        }
        break;
      }
      const int64_t row0 = (int64_t)tile * kTileRows;
      const int64_t row = row0 + lane;
      int state = 0;
      int64_t pos = row;
      if (row < n) {
        const bool ex = p.scores ? (p.scores[row] > p.threshold) : (p.mask[row] != 0);
        state = ex ? 2 : 1;
        if (p.pos_in) pos = p.pos_in[row];
      }
      bool moves = false;
      if (state == 1) moves = p.compact_out != nullptr;
      if (state == 2 && p.out_buf) {
        if (p.exits_dense || (pos >= 0 && pos < p.n_total)) {
          moves = true;
        } else {
          raise_error(p.err, TIDE_DEVERR_POSITION);
        }
      }
      const uint32_t keep = __ballot_sync(0xffffffffu, state == 1);
      const uint32_t exits = __ballot_sync(0xffffffffu, state == 2);
      const uint32_t move = __ballot_sync(0xffffffffu, moves);
      if (lane == 0) {
        d.row0 = row0;
        d.keep_mask = keep;
        d.exit_mask = exits;
        d.move_mask = move;
        d.n_move = (uint32_t)__popc(move);
        d.done = 0;
        d.end = 0;
        ptx::mbar_arrive(&m.td_rows[e]);  // release: the loader may start
      }
      uint32_t kb = 0, eb = 0;
      if (lane == 0) {
        if (!lookback(p.status, tile, (uint32_t)__popc(keep), (uint32_t)__popc(exits), &kb, &eb))
          fail(p, m);
        d.keep_before = kb;
        d.exits_before = eb;
        ptx::mbar_arrive(&m.td_prefix[e]);  // release: movers may store
      }
      kb = __shfl_sync(0xffffffffu, kb, 0);
      eb = __shfl_sync(0xffffffffu, eb, 0);
      if (state == 1) {
        const int64_t dst = (int64_t)kb + __popc(keep & lt);
        if (p.pos_out64) p.pos_out64[dst] = pos;
        if (p.pos_out32) p.pos_out32[dst] = (int32_t)pos;
        if (p.slot_out) p.slot_out[dst] = p.slot_in ? p.slot_in[row] : (int32_t)row;
      } else if (state == 2) {
        const int64_t ei = (int64_t)eb + __popc(exits & lt);
        if (p.exit_pos_out64) p.exit_pos_out64[ei] = pos;
        if (p.exit_pos_out32) p.exit_pos_out32[ei] = (int32_t)pos;
      }
      if (lane == 0 && (int64_t)tile == n_tiles - 1) {
        const uint32_t kt = kb + (uint32_t)__popc(keep), et = eb + (uint32_t)__popc(exits);
        if (p.counts) { p.counts[0] = (int32_t)kt; p.counts[1] = (int32_t)et; }
        if (p.num_remaining) p.num_remaining[0] = (int32_t)kt;
      }
    }
  } else if (warp == 1 || warp == 2 + kMovers) {
    // -------------------------------------------------------------- loaders
    // Both walk every tile's rows in order, numbering them q; loader `par`
    // issues the rows with q % 2 == par.
    if (lane == 0) {
      const uint32_t par = warp == 1 ? 0u : 1u;
      uint32_t q = 0;
      bool ok = true;
      for (uint32_t k = 0; ok; ++k) {
        const int e = (int)(k % kTiles);
        const uint32_t use = k / kTiles;
        if (!ptx::mbar_wait(&m.td_rows[e], use & 1u, m.abort_flag)) { ok = false; break; }
        const TileDesc &d = m.td[e];
        if (d.end) break;
        uint32_t mm = d.move_mask;
        const int64_t row0 = d.row0;
        const uint32_t n_move = d.n_move;
        for (; mm; ++q) {
          const int r = __ffs(mm) - 1;
          mm &= mm - 1u;
          if ((q & 1u) != par) continue;
          const int s = (int)(q % (uint32_t)NS);
          if (q >= (uint32_t)NS && !ptx::mbar_wait(&m.empty[s], ((q / NS) & 1u) ^ 1u, m.abort_flag)) {
            ok = false;
            break;
          }
          m.sdesc[s] = SlotDesc{(uint8_t)e, (uint8_t)r, (uint8_t)(use & 1u), 0};
          ptx::mbar_expect_tx(&m.full[s], row_bytes);
          ptx::bulk_load(slots + (size_t)s * row_bytes, x + (row0 + r) * p.H, row_bytes, &m.full[s],
                         pol);
          m.issued[par] = q + 1;
        }
        if (!ok) break;
        ptx::mbar_arrive(&m.td_free[e]);
        if (n_move == 0 && par == 0) ptx::mbar_arrive(&m.td_free[e]);  // no row to move: stands in for the last one
      }
      // one end marker per mover
      for (int i = 0; ok && i < kMovers; ++i, ++q) {
        if ((q & 1u) != par) continue;
        const int s = (int)(q % (uint32_t)NS);
        if (q >= (uint32_t)NS && !ptx::mbar_wait(&m.empty[s], ((q / NS) & 1u) ^ 1u, m.abort_flag)) {
          ok = false;
          break;
        }
        m.sdesc[s] = SlotDesc{0, 0, 0, 1};
        ptx::mbar_arrive(&m.full[s]);
        m.issued[par] = q + 1;
      }
      if (!ok) fail(p, m);
    }
  } else {
    // --------------------------------------------------------------- movers
    const int mv = warp - 2;
    constexpr int V = kVec<T>;
    const int64_t nv = p.H / V;
    // stores still reading their slots, oldest first (lane 0): at most
    // slots / 8 - 1 <= 7 of them are younger than the age limit below
    int pend_s[8];
    uint32_t pend_q[8];
    int n_pend = 0;
    for (uint32_t q = (uint32_t)mv;; q += kMovers) {
      const int s = (int)(q % (uint32_t)NS);
      if (lane == 0) {
        while (n_pend > 0 && (pend_q[0] + (uint32_t)NS <= q || n_pend > kMaxPending)) {
          ptx::bulk_wait_read(n_pend - 1);  // the oldest store has read its slot
          ptx::mbar_arrive(&m.empty[pend_s[0]]);
          for (int i = 1; i < n_pend; ++i) { pend_s[i - 1] = pend_s[i]; pend_q[i - 1] = pend_q[i]; }
          --n_pend;
        }
      }
      __syncwarp();
      if (!ptx::mbar_wait(&m.full[s], (q / NS) & 1u, m.abort_flag)) {
        if (lane == 0) fail(p, m);
        break;
      }
      const SlotDesc sd = m.sdesc[s];
      if (sd.end) break;
      if (!ptx::mbar_wait(&m.td_prefix[sd.tile], sd.parity, m.abort_flag)) {
        if (lane == 0) fail(p, m);
        break;
      }
      TileDesc &d = m.td[sd.tile];
      const uint32_t bit = 1u << sd.row, lt = bit - 1u;
      const int64_t row = d.row0 + sd.row;
      uint8_t *src = slots + (size_t)s * row_bytes;
      bool stored = false;
      if (d.keep_mask & bit) {
        const int64_t dst = (int64_t)d.keep_before + __popc(d.keep_mask & lt);
        if (lane == 0) {
          ptx::bulk_store(static_cast<T *>(p.compact_out) + dst * p.H, src, row_bytes, pol);
          ptx::bulk_commit();
        }
        stored = true;
      } else {
        const int64_t ei = (int64_t)d.exits_before + __popc(d.exit_mask & lt);
        const int64_t dst_row = p.exits_dense ? ei : (p.pos_in ? p.pos_in[row] : row);
        T *dst = static_cast<T *>(p.out_buf) + dst_row * p.H;
        if (p.row_stats) {
          const float2 ms = p.row_stats[row];
          const float rstd = ms.y, shift = -ms.y * ms.x;
          const uint4 *sv = reinterpret_cast<const uint4 *>(src);
          uint4 *dv = reinterpret_cast<uint4 *>(dst);
          // UN independent 16-byte vectors per lane per trip: their
          // shared-memory and weight loads are all in flight before the math
          constexpr int UN = kExitUnroll<LN>;
          constexpr int NT = LN ? TIDE_NORM_LAYER : TIDE_NORM_RMS;
          for (int64_t i0 = lane; i0 < nv; i0 += 32 * UN) {
            uint4 xr[UN];
            float4 w4[UN][V / 4], b4[LN ? UN : 1][V / 4];
#pragma unroll
            for (int u = 0; u < UN; ++u) {
              const int64_t i = i0 + 32 * u;
              if (i >= nv) continue;
              xr[u] = sv[i];
#pragma unroll
              for (int j = 0; j < V / 4; ++j) {
                w4[u][j] = (staged & 1) ? reinterpret_cast<const float4 *>(s_w + i * V)[j]
                                        : __ldg(reinterpret_cast<const float4 *>(p.w_norm + i * V) + j);
                if (LN)
                  b4[LN ? u : 0][j] =
                      (staged & 2) ? reinterpret_cast<const float4 *>(s_b + i * V)[j]
                      : p.b_norm   ? __ldg(reinterpret_cast<const float4 *>(p.b_norm + i * V) + j)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
            if (!LN) {
#pragma unroll
              for (int j = 0; j < V / 4; ++j) b4[0][j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < UN; ++u) {
              const int64_t i = i0 + 32 * u;
              if (i >= nv) continue;
              float xv[V], y[V];
              unpack16<T>(xr[u], xv);
#pragma unroll
              for (int j = 0; j < V / 4; ++j) {
                const float4 bb = b4[LN ? u : 0][j];
                y[4 * j] = norm_elem<T>(xv[4 * j], w4[u][j].x, bb.x, rstd, shift, NT);
                y[4 * j + 1] = norm_elem<T>(xv[4 * j + 1], w4[u][j].y, bb.y, rstd, shift, NT);
                y[4 * j + 2] = norm_elem<T>(xv[4 * j + 2], w4[u][j].z, bb.z, rstd, shift, NT);
                y[4 * j + 3] = norm_elem<T>(xv[4 * j + 3], w4[u][j].w, bb.w, rstd, shift, NT);
              }
              st_stream(dv + i, pack16<T>(y));
            }
          }
          __syncwarp();
        } else {
          if (lane == 0) {
            ptx::bulk_store(dst, src, row_bytes, pol);
            ptx::bulk_commit();
          }
          stored = true;
        }
      }
      if (lane == 0) {
        if (stored) {
          pend_s[n_pend] = s;
          pend_q[n_pend] = q;
          ++n_pend;
        } else {
          ptx::mbar_arrive(&m.empty[s]);
        }
        if (atomicAdd(&d.done, 1u) + 1u == d.n_move) ptx::mbar_arrive(&m.td_free[sd.tile]);
      }
      __syncwarp();
    }
    if (lane == 0) {
      ptx::bulk_wait_all();
      for (int i = 0; i < n_pend; ++i) ptx::mbar_arrive(&m.empty[pend_s[i]]);
    }
  }

  __syncthreads();
  if (threadIdx.x == 32 && *m.abort_flag) {
    // wait for every bulk load this CTA issued before its shared memory goes:
    // per slot, the latest use q that its loader issued (loader q % 2 has
    // issued every q of its parity below issued[q % 2]; the loaders are
    // never more than a ring apart)
    const uint32_t next[2] = {m.issued[0], m.issued[1]};
    const uint32_t total = next[0] > next[1] ? next[0] : next[1];
    volatile int never = 0;
    for (int s = 0; s < NS && (uint32_t)s < total; ++s) {
      int64_t q = (int64_t)s + (int64_t)((total - 1u - (uint32_t)s) / (uint32_t)NS) * NS;
      for (; q >= 0; q -= NS) {
        if ((uint64_t)q < next[q & 1]) {
          ptx::mbar_wait(&m.full[s], (uint32_t)(q / NS) & 1u, &never);
          break;
        }
      }
    }
  }
}

// The slot count is a multiple of kMovers, so every use of a slot belongs to
// the same mover (q % kMovers is fixed by q % slots) and comes after its
// previous use.  The waits on a slot are by phase parity, which cannot tell
// the phase before the last from the next one: a second mover could wait on
// a slot's next use while its current load is in flight and read it early.
int slots_for(uint32_t row_bytes) {
  int s = (int)((kSmemBudget - 128 - kAux) / row_bytes);
  if (s > kMaxSlots) s = kMaxSlots;
  return s / kMovers * kMovers;
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <typename T, bool LN>
int launch_t(const MoveParams &p, cudaStream_t s) {
  const uint32_t row_bytes = (uint32_t)(p.H * (int64_t)sizeof(T));
  const int NS = slots_for(row_bytes);
  size_t smem = 128 + (size_t)NS * row_bytes + kAux;
  // stage the norm vectors in what the slots leave of the budget
  int staged = 0;
  const size_t vec_bytes = (size_t)p.H * sizeof(float);
  if (p.row_stats && p.w_norm && smem + vec_bytes <= (size_t)kSmemBudget) {
    staged |= 1;
    smem += vec_bytes;
    if (LN && p.b_norm && smem + vec_bytes <= (size_t)kSmemBudget) {
      staged |= 2;
      smem += vec_bytes;
    }
  }
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cudaFuncSetAttribute(move_rows_bulk_kernel<T, LN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBudget) != cudaSuccess)
      return TIDE_ERR_CUDA;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int64_t tiles = p.n_cap > 0 ? (p.n_cap + kTileRows - 1) / kTileRows : 1;
  const int sms = sm_count();
  const int grid = (int)(tiles < sms ? tiles : sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, move_rows_bulk_kernel<T, LN>, p, NS, staged) != cudaSuccess)
    return TIDE_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? TIDE_OK : TIDE_ERR_CUDA;
}

}  // namespace

static_assert(sizeof(TileDesc) * kTiles + sizeof(SlotDesc) * kMaxSlots +
                      8 * (2 * kMaxSlots + 3 * kTiles) + 16 <= kAux,
              "bulk mover aux area");

int bulk_tile_rows() { return kTileRows; }

bool bulk_move_supported(int dtype, int64_t H, bool vec, const MoveParams &p) {
  if (!vec) return false;
  if (p.row_stats && ((reinterpret_cast<uintptr_t>(p.w_norm) | reinterpret_cast<uintptr_t>(p.b_norm)) & 15u))
    return false;
  const int64_t row_bytes = H * (dtype == TIDE_DTYPE_F32 ? 4 : 2);
  if (row_bytes % 16 != 0 || row_bytes < kMinRowBytes) return false;
  return slots_for((uint32_t)row_bytes) >= kMovers;
}

int bulk_move_launch(int dtype, const MoveParams &p, cudaStream_t s) {
  const bool ln = p.norm_type == TIDE_NORM_LAYER;
  switch (dtype) {
    case TIDE_DTYPE_F32:
      return ln ? launch_t<float, true>(p, s) : launch_t<float, false>(p, s);
    case TIDE_DTYPE_F16:
      return ln ? launch_t<__half, true>(p, s) : launch_t<__half, false>(p, s);
    default:
      return ln ? launch_t<__nv_bfloat16, true>(p, s) : launch_t<__nv_bfloat16, false>(p, s);
  }
}

}  // namespace tide
