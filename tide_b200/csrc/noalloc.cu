// tide_batch_compact_noalloc: the stable row split of tide_batch_compact for
// callers that cannot allocate device memory.
//
// Some hosts cannot hand this library a scratch buffer.  Examples:
// - an FFI host whose GPU memory is owned by another runtime and is reserved
//   once at start-up;
// - code that runs where allocation is not allowed, such as inside a memory
//   pool's callback, or in a serving loop held to a fixed memory budget.
// Such callers still pass their inputs and outputs.  The look-back state the
// split needs (a tile ticket and one status word per 128-row tile) lives in
// the file-scope device array below.  This file allocates nothing: no
// cudaMalloc, no cudaFree, no allocating library call.
//
// The array is global to the process.  Every GPU that loads the library holds
// one copy of it until the process exits.  Every call on a device shares that
// copy, and the copy keeps whatever the last call left in it.  So each call
// first clears the ticket and the status words it will use (cudaMemsetAsync on
// the caller's stream).  Two calls whose kernels overlap on the GPU race on the
// array and corrupt each other's result: serialise them, for example by using
// one stream per device.
//
// Host code only ever sees a stand-in for the array's name, not a device
// address.  The first call on a device therefore looks the address up with
// cudaGetSymbolAddress, with that device current, and caches it for later
// calls.  That first call should happen before any stream capture.  The
// cached address belongs to the device's primary context: a cudaDeviceReset
// (or a release and re-creation of that context) makes it stale, and the
// entry point must not be called on that device again in this process.
#include <stdarg.h>
#include <stdio.h>

#include <initializer_list>
#include <mutex>

#include "common.cuh"
#include "simt_kernels.cuh"

namespace tide {
void set_last_error(const char *msg);
}

namespace {

constexpr int64_t kMaxRows = TIDE_NOALLOC_MAX_ROWS;
constexpr int64_t kMaxTiles = kMaxRows / tide::kMoveTile;
constexpr size_t kTicketBytes = 256;
constexpr size_t kScratchBytes = kTicketBytes + (size_t)kMaxTiles * 8;
constexpr int kMaxDevices = 64;

}  // namespace

// ticket (padded to 256 bytes) followed by one 64-bit status word per tile
static __device__ __align__(256) unsigned char g_partition_scratch[kScratchBytes];

namespace {

std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {};

int noalloc_fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  tide::set_last_error(buf);
  return code;
}

// Device address of g_partition_scratch on the current device, looked up
// once per device.
int scratch_address(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return noalloc_fail(TIDE_ERR_CUDA, "batch_compact_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return noalloc_fail(TIDE_ERR_UNSUPPORTED, "batch_compact_noalloc: device %d above %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_partition_scratch);
    if (e != cudaSuccess || !p)
      return noalloc_fail(TIDE_ERR_CUDA, "batch_compact_noalloc: cudaGetSymbolAddress: %s",
                          cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return TIDE_OK;
}

template <typename T, bool VEC>
void launch_split(const tide::MoveParams &p, int64_t grid, cudaStream_t s) {
  tide::move_rows_kernel<T, VEC><<<(unsigned)grid, tide::kMoveThreads, 0, s>>>(p);
}

}  // namespace

extern "C" int tide_batch_compact_noalloc(int dtype, const void *input, const int32_t *exit_mask,
                                          void *compacted, void *exited,
                                          int32_t *continue_indices, int32_t *exit_indices,
                                          int32_t *num_remaining, int64_t n_tokens,
                                          int64_t hidden_dim, int32_t *error_word,
                                          tide_stream_t stream) {
  if (dtype != TIDE_DTYPE_F32 && dtype != TIDE_DTYPE_F16 && dtype != TIDE_DTYPE_BF16)
    return noalloc_fail(TIDE_ERR_INVALID, "batch_compact_noalloc: bad dtype %d", dtype);
  if (n_tokens < 0 || hidden_dim <= 0)
    return noalloc_fail(TIDE_ERR_INVALID, "batch_compact_noalloc: bad sizes");
  if (n_tokens > kMaxRows)
    return noalloc_fail(TIDE_ERR_INVALID,
                        "batch_compact_noalloc: %lld rows exceed the limit of %lld rows of its "
                        "built-in scratch; use tide_batch_compact with a workspace",
                        (long long)n_tokens, (long long)kMaxRows);
  if (!num_remaining) return noalloc_fail(TIDE_ERR_INVALID, "batch_compact_noalloc: num_remaining is NULL");
  if (n_tokens > 0 && (!input || !exit_mask))
    return noalloc_fail(TIDE_ERR_INVALID, "batch_compact_noalloc: NULL input/mask");
  void *scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != TIDE_OK) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t tiles = n_tokens > 0 ? (n_tokens + tide::kMoveTile - 1) / tide::kMoveTile : 1;
  // the ticket and this call's tile words must start at zero
  cudaError_t e = cudaMemsetAsync(scratch, 0, kTicketBytes + (size_t)tiles * 8, s);
  if (e != cudaSuccess)
    return noalloc_fail(TIDE_ERR_CUDA, "batch_compact_noalloc: clear: %s", cudaGetErrorString(e));
  tide::MoveParams p{};
  p.x = input;
  p.n_cap = n_tokens;
  p.H = hidden_dim;
  p.n_total = n_tokens;
  p.mask = exit_mask;
  p.exits_dense = true;
  p.out_buf = exited;
  p.compact_out = compacted;
  p.pos_out32 = continue_indices;
  p.exit_pos_out32 = exit_indices;
  p.num_remaining = num_remaining;
  p.ticket = static_cast<uint32_t *>(scratch);
  p.status = reinterpret_cast<uint64_t *>(static_cast<char *>(scratch) + kTicketBytes);
  p.err = error_word;
  const size_t es = dtype == TIDE_DTYPE_F32 ? 4 : 2;
  bool vec = (hidden_dim * (int64_t)es) % 16 == 0;
  for (const void *q : {input, (const void *)compacted, (const void *)exited})
    if (q && ((uintptr_t)q & 15u)) vec = false;
  switch (dtype) {
    case TIDE_DTYPE_F32: vec ? launch_split<float, true>(p, tiles, s) : launch_split<float, false>(p, tiles, s); break;
    case TIDE_DTYPE_F16: vec ? launch_split<__half, true>(p, tiles, s) : launch_split<__half, false>(p, tiles, s); break;
    default: vec ? launch_split<__nv_bfloat16, true>(p, tiles, s) : launch_split<__nv_bfloat16, false>(p, tiles, s); break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return noalloc_fail(TIDE_ERR_CUDA, "batch_compact_noalloc: launch: %s", cudaGetErrorString(e));
  return TIDE_OK;
}
