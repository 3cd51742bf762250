// C ABI of libtide_b200.so: argument checks, workspace layout and dispatch
// to the SIMT and tensor-core kernels.  Declarations: include/tide_b200.h.
#include <stdarg.h>
#include <stdio.h>

#include <initializer_list>
#include <string.h>

#include "common.cuh"
#include "move_bulk.cuh"
#include "simt_kernels.cuh"
#include "tc_checkpoint.cuh"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TIDE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TIDE_OK;
}

size_t esize(int dtype) { return dtype == TIDE_DTYPE_F32 ? 4 : 2; }
bool valid_dtype(int d) { return d == TIDE_DTYPE_F32 || d == TIDE_DTYPE_F16 || d == TIDE_DTYPE_BF16; }
bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Row moves use 16-byte vectors when every row start is 16-byte aligned.
bool rows_vectorizable(int dtype, int64_t H, std::initializer_list<const void *> ptrs) {
  if ((H * (int64_t)esize(dtype)) % 16 != 0) return false;
  for (const void *p : ptrs)
    if (p && !aligned16(p)) return false;
  return true;
}

template <template <typename, bool> class F, typename... A>
void dispatch_rows(int dtype, bool vec, A &&...a) {
  switch (dtype) {
    case TIDE_DTYPE_F32: vec ? F<float, true>::run(a...) : F<float, false>::run(a...); break;
    case TIDE_DTYPE_F16: vec ? F<__half, true>::run(a...) : F<__half, false>::run(a...); break;
    default: vec ? F<__nv_bfloat16, true>::run(a...) : F<__nv_bfloat16, false>::run(a...); break;
  }
}

template <typename T, bool VEC> struct MoveLaunch {
  static void run(const tide::MoveParams &p, int64_t grid, cudaStream_t s) {
    tide::move_rows_kernel<T, VEC><<<(unsigned)grid, tide::kMoveThreads, 0, s>>>(p);
  }
};

template <typename T>
void launch_route_t(const tide::RouteParams &p, int64_t grid, cudaStream_t s) {
  if (p.B <= tide::kRouteThreads)
    tide::route_simt_kernel<T, 1><<<(unsigned)grid, tide::kRouteThreads, 0, s>>>(p);
  else
    tide::route_simt_kernel<T, 2><<<(unsigned)grid, tide::kRouteThreads, 0, s>>>(p);
}
void launch_route(int dtype, const tide::RouteParams &p, int64_t grid, cudaStream_t s) {
  if (dtype == TIDE_DTYPE_F32) launch_route_t<float>(p, grid, s);
  else if (dtype == TIDE_DTYPE_F16) launch_route_t<__half>(p, grid, s);
  else launch_route_t<__nv_bfloat16>(p, grid, s);
}

template <typename T, bool VEC> struct ScatterLaunch {
  static void run(const void *src, const int32_t *pos32, const int64_t *pos64, void *out, int64_t n,
                  int64_t H, int64_t n_total, int norm_type, const float *w, const float *b,
                  float eps, int32_t *err, bool norm, cudaStream_t s) {
    const int rows_per_block = 8;
    const unsigned grid = (unsigned)((n + rows_per_block - 1) / rows_per_block);
    if (norm)
      tide::scatter_rows_kernel<T, VEC, true><<<grid, 32 * rows_per_block, 0, s>>>(
          static_cast<const T *>(src), pos32, pos64, static_cast<T *>(out), n, H, n_total,
          norm_type, w, b, eps, err);
    else
      tide::scatter_rows_kernel<T, VEC, false><<<grid, 32 * rows_per_block, 0, s>>>(
          static_cast<const T *>(src), pos32, pos64, static_cast<T *>(out), n, H, n_total,
          norm_type, w, b, eps, err);
  }
};

template <typename T, bool VEC> struct IndexedLaunch {
  // norm: 0 gather, 1 norm in place at idx, 2 norm scatter (src row i to idx[i])
  static void run(const void *src, const int64_t *idx, const int32_t *n_dev, int64_t n_cap,
                  int64_t H, int64_t n_src, void *dst, int norm, int norm_type, const float *w,
                  const float *b, float eps, int32_t *err, cudaStream_t s) {
    const int warps_per_block = 8;
    int64_t blocks = (n_cap + warps_per_block - 1) / warps_per_block;
    if (blocks > 148 * 16) blocks = 148 * 16;  // grid-stride beyond 16 blocks per SM
    if (blocks < 1) blocks = 1;
    if (norm == 2)
      tide::indexed_rows_kernel<T, VEC, true, true><<<(unsigned)blocks, 32 * warps_per_block, 0, s>>>(
          static_cast<const T *>(src), idx, n_dev, n_cap, H, n_src, static_cast<T *>(dst),
          norm_type, w, b, eps, err);
    else if (norm)
      tide::indexed_rows_kernel<T, VEC, true><<<(unsigned)blocks, 32 * warps_per_block, 0, s>>>(
          static_cast<const T *>(src), idx, n_dev, n_cap, H, n_src, static_cast<T *>(dst),
          norm_type, w, b, eps, err);
    else
      tide::indexed_rows_kernel<T, VEC, false><<<(unsigned)blocks, 32 * warps_per_block, 0, s>>>(
          static_cast<const T *>(src), idx, n_dev, n_cap, H, n_src, static_cast<T *>(dst),
          norm_type, w, b, eps, err);
  }
};

// Workspace of the stable partition: ticket (u32, padded) then one status
// word per tile of `tile_rows` rows.
size_t partition_ws_bytes(int64_t n, int64_t tile_rows = tide::kMoveTile) {
  const int64_t tiles = n > 0 ? (n + tile_rows - 1) / tile_rows : 1;
  return 256 + align_up((size_t)tiles * 8, 256);
}

// SIMT checkpoint workspace: partition state, then scores, then row stats.
struct SimtWs {
  uint32_t *ticket;
  uint64_t *status;
  size_t partition_bytes;
  float *scores;
  float2 *stats;
};
// The checkpoint's partition area is sized for the bulk mover's smaller
// tiles, which covers the SIMT mover's too.
size_t simt_ws_bytes(int64_t n) {
  return partition_ws_bytes(n, tide::bulk_tile_rows()) + align_up((size_t)n * 4, 256) +
         align_up((size_t)n * 8, 256);
}
SimtWs simt_ws(void *ws, int64_t n) {
  SimtWs w;
  char *b = static_cast<char *>(ws);
  w.ticket = reinterpret_cast<uint32_t *>(b);
  w.status = reinterpret_cast<uint64_t *>(b + 256);
  w.partition_bytes = partition_ws_bytes(n, tide::bulk_tile_rows());
  w.scores = reinterpret_cast<float *>(b + w.partition_bytes);
  w.stats = reinterpret_cast<float2 *>(b + w.partition_bytes + align_up((size_t)n * 4, 256));
  return w;
}

int validate_checkpoint(const tide_checkpoint_args *a) {
  if (!a) return fail(TIDE_ERR_INVALID, "tide_checkpoint: args is NULL");
  if (!valid_dtype(a->dtype)) return fail(TIDE_ERR_INVALID, "tide_checkpoint: bad dtype %d", a->dtype);
  if (a->norm_type != TIDE_NORM_RMS && a->norm_type != TIDE_NORM_LAYER)
    return fail(TIDE_ERR_INVALID, "tide_checkpoint: bad norm_type %d", a->norm_type);
  if (a->n_rows < 0 || a->n_rows > INT32_MAX / 2)
    return fail(TIDE_ERR_INVALID, "tide_checkpoint: n_rows %lld out of range", (long long)a->n_rows);
  if (a->hidden_dim <= 0 || a->hidden_dim > (1 << 20))
    return fail(TIDE_ERR_INVALID, "tide_checkpoint: hidden_dim %lld out of range", (long long)a->hidden_dim);
  if (a->bottleneck_dim <= 0 || a->bottleneck_dim > 256)
    return fail(TIDE_ERR_INVALID, "tide_checkpoint: bottleneck_dim must be in [1, 256]");
  if (a->n_total < 0) return fail(TIDE_ERR_INVALID, "tide_checkpoint: n_total < 0");
  if (a->n_rows > 0 && !a->x) return fail(TIDE_ERR_INVALID, "tide_checkpoint: x is NULL");
  if (!a->norm_weight || !a->up) return fail(TIDE_ERR_INVALID, "tide_checkpoint: norm_weight/up NULL");
  if (!a->counts_out) return fail(TIDE_ERR_INVALID, "tide_checkpoint: counts_out is NULL");
  if (!a->workspace) return fail(TIDE_ERR_WORKSPACE, "tide_checkpoint: workspace is NULL");
  if (!aligned16(a->workspace)) return fail(TIDE_ERR_WORKSPACE, "tide_checkpoint: workspace not 16-byte aligned");
  return TIDE_OK;
}

}  // namespace

extern "C" {

int tide_abi_version(void) { return 1; }
const char *tide_last_error(void) { return g_err; }

int tide_fused_layernorm_route(int dtype, const void *input, const float *norm_weight,
                               const float *down_weight_t, const float *up_weight_t, float eps,
                               float *scores, int64_t n_tokens, int64_t hidden_dim,
                               int64_t bottleneck_dim, tide_stream_t stream) {
  if (!valid_dtype(dtype)) return fail(TIDE_ERR_INVALID, "fused_layernorm_route: bad dtype %d", dtype);
  if (n_tokens < 0 || hidden_dim <= 0 || bottleneck_dim <= 0 || bottleneck_dim > 256)
    return fail(TIDE_ERR_INVALID, "fused_layernorm_route: bad sizes n=%lld H=%lld B=%lld",
                (long long)n_tokens, (long long)hidden_dim, (long long)bottleneck_dim);
  if (n_tokens == 0) return TIDE_OK;
  if (!input || !norm_weight || !down_weight_t || !up_weight_t || !scores)
    return fail(TIDE_ERR_INVALID, "fused_layernorm_route: NULL pointer");
  tide::RouteParams p{};
  p.x = input; p.n_cap = n_tokens; p.n_dev = nullptr;
  p.H = (int)hidden_dim; p.B = (int)bottleneck_dim; p.norm_type = TIDE_NORM_RMS;
  p.w_norm = norm_weight; p.b_norm = nullptr; p.eps = eps;
  p.down_t = down_weight_t; p.up = up_weight_t; p.up_bias = 0.f;
  p.scores = scores; p.row_stats = nullptr; p.err = nullptr;
  const int64_t grid = (n_tokens + tide::kRouteRows - 1) / tide::kRouteRows;
  launch_route(dtype, p, grid, (cudaStream_t)stream);
  return check_launch("fused_layernorm_route");
}

size_t tide_batch_compact_workspace_size(int64_t n_tokens) { return partition_ws_bytes(n_tokens); }

int tide_batch_compact(int dtype, const void *input, const int32_t *exit_mask, void *compacted,
                       void *exited, int32_t *continue_indices, int32_t *exit_indices,
                       int32_t *num_remaining, int64_t n_tokens, int64_t hidden_dim,
                       void *workspace, size_t workspace_bytes, int32_t *error_word,
                       tide_stream_t stream) {
  if (!valid_dtype(dtype)) return fail(TIDE_ERR_INVALID, "batch_compact: bad dtype %d", dtype);
  if (n_tokens < 0 || n_tokens > INT32_MAX / 2 || hidden_dim <= 0)
    return fail(TIDE_ERR_INVALID, "batch_compact: bad sizes");
  if (!num_remaining) return fail(TIDE_ERR_INVALID, "batch_compact: num_remaining is NULL");
  if (n_tokens > 0 && (!input || !exit_mask))
    return fail(TIDE_ERR_INVALID, "batch_compact: NULL input/mask");
  if (!workspace || workspace_bytes < partition_ws_bytes(n_tokens) || !aligned16(workspace))
    return fail(TIDE_ERR_WORKSPACE, "batch_compact: workspace needs %zu bytes (16-aligned)",
                partition_ws_bytes(n_tokens));
  cudaStream_t s = (cudaStream_t)stream;
  const size_t zero_bytes = partition_ws_bytes(n_tokens);
  if (cudaMemsetAsync(workspace, 0, zero_bytes, s) != cudaSuccess)
    return fail(TIDE_ERR_CUDA, "batch_compact: memset failed");
  tide::MoveParams p{};
  p.x = input; p.n_cap = n_tokens; p.H = hidden_dim; p.n_total = n_tokens;
  p.mask = exit_mask; p.exits_dense = true;
  p.out_buf = exited; p.compact_out = compacted;
  p.pos_out32 = continue_indices; p.exit_pos_out32 = exit_indices;
  p.num_remaining = num_remaining;
  p.ticket = static_cast<uint32_t *>(workspace);
  p.status = reinterpret_cast<uint64_t *>(static_cast<char *>(workspace) + 256);
  p.err = error_word;
  const bool vec = rows_vectorizable(dtype, hidden_dim, {input, compacted, exited});
  const int64_t grid = n_tokens > 0 ? (n_tokens + tide::kMoveTile - 1) / tide::kMoveTile : 1;
  dispatch_rows<MoveLaunch>(dtype, vec, p, grid, s);
  return check_launch("batch_compact");
}


int tide_exit_scatter(int dtype, const void *exited_states, const int32_t *exit_positions,
                      void *output_buffer, int64_t n_exited, int64_t hidden_dim, int64_t n_total,
                      int32_t *error_word, tide_stream_t stream) {
  if (!valid_dtype(dtype)) return fail(TIDE_ERR_INVALID, "exit_scatter: bad dtype %d", dtype);
  if (n_exited < 0 || hidden_dim <= 0 || n_total < 0)
    return fail(TIDE_ERR_INVALID, "exit_scatter: bad sizes");
  if (n_exited == 0) return TIDE_OK;
  if (!exited_states || !exit_positions || !output_buffer)
    return fail(TIDE_ERR_INVALID, "exit_scatter: NULL pointer");
  const bool vec = rows_vectorizable(dtype, hidden_dim, {exited_states, output_buffer});
  dispatch_rows<ScatterLaunch>(dtype, vec, exited_states, exit_positions, (const int64_t *)nullptr,
                               output_buffer, n_exited, hidden_dim, n_total, (int)TIDE_NORM_RMS,
                               (const float *)nullptr, (const float *)nullptr, 0.f, error_word,
                               false, (cudaStream_t)stream);
  return check_launch("exit_scatter");
}

int tide_exit_projection(int dtype, const void *exited_states, const float *norm_weight,
                         const int32_t *exit_positions, void *output_buffer, float eps,
                         int64_t n_exited, int64_t hidden_dim, int64_t n_total,
                         int32_t *error_word, tide_stream_t stream) {
  if (!valid_dtype(dtype)) return fail(TIDE_ERR_INVALID, "exit_projection: bad dtype %d", dtype);
  if (n_exited < 0 || hidden_dim <= 0 || n_total < 0)
    return fail(TIDE_ERR_INVALID, "exit_projection: bad sizes");
  if (n_exited == 0) return TIDE_OK;
  if (!exited_states || !exit_positions || !output_buffer || !norm_weight)
    return fail(TIDE_ERR_INVALID, "exit_projection: NULL pointer");
  const bool vec = rows_vectorizable(dtype, hidden_dim, {exited_states, output_buffer});
  dispatch_rows<ScatterLaunch>(dtype, vec, exited_states, exit_positions, (const int64_t *)nullptr,
                               output_buffer, n_exited, hidden_dim, n_total, (int)TIDE_NORM_RMS,
                               norm_weight, (const float *)nullptr, eps, error_word, true,
                               (cudaStream_t)stream);
  return check_launch("exit_projection");
}

int tide_norm_scatter(int dtype, int norm_type, const void *rows, const int64_t *positions,
                      void *output_buffer, const float *norm_weight, const float *norm_bias,
                      float eps, int64_t n_rows, int64_t hidden_dim, int64_t n_total,
                      int32_t *error_word, tide_stream_t stream) {
  if (!valid_dtype(dtype)) return fail(TIDE_ERR_INVALID, "norm_scatter: bad dtype %d", dtype);
  if (norm_type != TIDE_NORM_RMS && norm_type != TIDE_NORM_LAYER)
    return fail(TIDE_ERR_INVALID, "norm_scatter: bad norm_type %d", norm_type);
  if (n_rows < 0 || hidden_dim <= 0 || n_total < 0) return fail(TIDE_ERR_INVALID, "norm_scatter: bad sizes");
  if (n_rows == 0) return TIDE_OK;
  if (!rows || !positions || !output_buffer || !norm_weight)
    return fail(TIDE_ERR_INVALID, "norm_scatter: NULL pointer");
  const bool vec = rows_vectorizable(dtype, hidden_dim, {rows, output_buffer});
  dispatch_rows<ScatterLaunch>(dtype, vec, rows, (const int32_t *)nullptr, positions, output_buffer,
                               n_rows, hidden_dim, n_total, norm_type, norm_weight,
                               norm_type == TIDE_NORM_LAYER ? norm_bias : (const float *)nullptr,
                               eps, error_word, true, (cudaStream_t)stream);
  return check_launch("norm_scatter");
}

int tide_gather_rows(int dtype, const void *src, int64_t n_src, const int64_t *index,
                     const int32_t *n_rows_dev, int64_t n_rows, int64_t hidden_dim, void *dst,
                     int32_t *error_word, tide_stream_t stream) {
  if (!valid_dtype(dtype)) return fail(TIDE_ERR_INVALID, "gather_rows: bad dtype %d", dtype);
  if (n_rows < 0 || n_src < 0 || hidden_dim <= 0) return fail(TIDE_ERR_INVALID, "gather_rows: bad sizes");
  if (n_rows == 0) return TIDE_OK;
  if (!src || !index || !dst) return fail(TIDE_ERR_INVALID, "gather_rows: NULL pointer");
  const bool vec = rows_vectorizable(dtype, hidden_dim, {src, dst});
  dispatch_rows<IndexedLaunch>(dtype, vec, src, index, n_rows_dev, n_rows, hidden_dim, n_src, dst,
                               0, (int)TIDE_NORM_RMS, (const float *)nullptr,
                               (const float *)nullptr, 0.f, error_word, (cudaStream_t)stream);
  return check_launch("gather_rows");
}

int tide_norm_at_positions(int dtype, int norm_type, const void *src, const int64_t *positions,
                           const int32_t *n_rows_dev, int64_t n_rows, int64_t hidden_dim,
                           int64_t n_total, void *output_buffer, const float *norm_weight,
                           const float *norm_bias, float eps, int32_t *error_word,
                           tide_stream_t stream) {
  if (!valid_dtype(dtype)) return fail(TIDE_ERR_INVALID, "norm_at_positions: bad dtype %d", dtype);
  if (norm_type != TIDE_NORM_RMS && norm_type != TIDE_NORM_LAYER)
    return fail(TIDE_ERR_INVALID, "norm_at_positions: bad norm_type %d", norm_type);
  if (n_rows < 0 || n_total < 0 || hidden_dim <= 0)
    return fail(TIDE_ERR_INVALID, "norm_at_positions: bad sizes");
  if (n_rows == 0) return TIDE_OK;
  if (!src || !positions || !output_buffer || !norm_weight)
    return fail(TIDE_ERR_INVALID, "norm_at_positions: NULL pointer");
  const bool vec = rows_vectorizable(dtype, hidden_dim, {src, output_buffer});
  dispatch_rows<IndexedLaunch>(dtype, vec, src, positions, n_rows_dev, n_rows, hidden_dim, n_total,
                               output_buffer, 1, norm_type, norm_weight,
                               norm_type == TIDE_NORM_LAYER ? norm_bias : (const float *)nullptr,
                               eps, error_word, (cudaStream_t)stream);
  return check_launch("norm_at_positions");
}

int tide_norm_scatter_rows(int dtype, int norm_type, const void *rows, const int64_t *positions,
                           const int32_t *n_rows_dev, int64_t n_rows, int64_t hidden_dim,
                           int64_t n_total, void *output_buffer, const float *norm_weight,
                           const float *norm_bias, float eps, int32_t *error_word,
                           tide_stream_t stream) {
  if (!valid_dtype(dtype)) return fail(TIDE_ERR_INVALID, "norm_scatter_rows: bad dtype %d", dtype);
  if (norm_type != TIDE_NORM_RMS && norm_type != TIDE_NORM_LAYER)
    return fail(TIDE_ERR_INVALID, "norm_scatter_rows: bad norm_type %d", norm_type);
  if (n_rows < 0 || n_total < 0 || hidden_dim <= 0)
    return fail(TIDE_ERR_INVALID, "norm_scatter_rows: bad sizes");
  if (n_rows == 0) return TIDE_OK;
  if (!rows || !positions || !output_buffer || !norm_weight)
    return fail(TIDE_ERR_INVALID, "norm_scatter_rows: NULL pointer");
  const bool vec = rows_vectorizable(dtype, hidden_dim, {rows, output_buffer});
  dispatch_rows<IndexedLaunch>(dtype, vec, rows, positions, n_rows_dev, n_rows, hidden_dim, n_total,
                               output_buffer, 2, norm_type, norm_weight,
                               norm_type == TIDE_NORM_LAYER ? norm_bias : (const float *)nullptr,
                               eps, error_word, (cudaStream_t)stream);
  return check_launch("norm_scatter_rows");
}

int tide_router_fold(int fold_dtype, const float *down, const float *norm_weight,
                     const float *norm_bias, int64_t hidden_dim, int64_t bottleneck_dim,
                     float *down_t, void *folded, float *colsum, float *bias_proj,
                     tide_stream_t stream) {
  if (!valid_dtype(fold_dtype)) return fail(TIDE_ERR_INVALID, "router_fold: bad dtype %d", fold_dtype);
  if (hidden_dim <= 0 || bottleneck_dim <= 0 || bottleneck_dim > 256)
    return fail(TIDE_ERR_INVALID, "router_fold: bad sizes");
  if (!down || !norm_weight) return fail(TIDE_ERR_INVALID, "router_fold: NULL down/norm_weight");
  if (bias_proj && !norm_bias) return fail(TIDE_ERR_INVALID, "router_fold: bias_proj needs norm_bias");
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned grid = (unsigned)bottleneck_dim;
  switch (fold_dtype) {
    case TIDE_DTYPE_F32:
      tide::router_fold_kernel<float><<<grid, 256, 0, s>>>(down, norm_weight, norm_bias, hidden_dim,
          bottleneck_dim, down_t, static_cast<float *>(folded), colsum, bias_proj);
      break;
    case TIDE_DTYPE_F16:
      tide::router_fold_kernel<__half><<<grid, 256, 0, s>>>(down, norm_weight, norm_bias, hidden_dim,
          bottleneck_dim, down_t, static_cast<__half *>(folded), colsum, bias_proj);
      break;
    default:
      tide::router_fold_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(down, norm_weight, norm_bias,
          hidden_dim, bottleneck_dim, down_t, static_cast<__nv_bfloat16 *>(folded), colsum, bias_proj);
      break;
  }
  return check_launch("router_fold");
}

int tide_checkpoint_select_path(const tide_checkpoint_args *a) {
  int rc = validate_checkpoint(a);
  if (rc != TIDE_OK) return -rc;
  if (a->path == TIDE_PATH_SIMT) return TIDE_PATH_SIMT;
  if (a->path == TIDE_PATH_TC_SPLIT) {
    if (!tide::tc_supported(a)) {
      fail(TIDE_ERR_UNSUPPORTED, "tide_checkpoint: tensor-core split path does not take these arguments (%s)",
           tide::tc_unsupported_reason(a));
      return -TIDE_ERR_UNSUPPORTED;
    }
    return TIDE_PATH_TC_SPLIT;
  }
  if (a->path == TIDE_PATH_TC) {
    if (tide::fused_supported(a)) return TIDE_PATH_TC;
    if (tide::tc_supported(a)) return TIDE_PATH_TC_SPLIT;
    fail(TIDE_ERR_UNSUPPORTED, "tide_checkpoint: tensor-core path does not take these arguments (%s)",
         tide::tc_unsupported_reason(a));
    return -TIDE_ERR_UNSUPPORTED;
  }
  // automatic choice, from measured latencies: the fused single pass (one
  // launch, ~20 us at 256 rows) up to a row count that depends on the hidden
  // size (5120 rows at H = 4096; none at H = 512 and 1024, where the split
  // path wins from 128 rows), the split path above it (its router streams
  // all of W' through each CTA, a floor of ~35 us at H = 4096).
  // SIMT otherwise.
  if (a->n_rows <= tide::fused_auto_max_rows(a->hidden_dim) && tide::fused_supported(a))
    return TIDE_PATH_TC;
  if (tide::tc_supported(a)) return TIDE_PATH_TC_SPLIT;
  if (tide::fused_supported(a)) return TIDE_PATH_TC;
  return TIDE_PATH_SIMT;
}

size_t tide_checkpoint_workspace_size(const tide_checkpoint_args *a) {
  if (!a) return 0;
  const int64_t n = a->n_rows > 0 ? a->n_rows : 0;
  size_t simt = simt_ws_bytes(n);
  size_t fused = tide::fused_workspace_bytes(a);
  return simt > fused ? simt : fused;
}

int tide_checkpoint(const tide_checkpoint_args *a, tide_stream_t stream) {
  int path = tide_checkpoint_select_path(a);
  if (path < 0) return -path;
  const int64_t n = a->n_rows;
  if (a->workspace_bytes < tide_checkpoint_workspace_size(a))
    return fail(TIDE_ERR_WORKSPACE, "tide_checkpoint: workspace needs %zu bytes, got %zu",
                tide_checkpoint_workspace_size(a), a->workspace_bytes);
  cudaStream_t s = (cudaStream_t)stream;
  if (path == TIDE_PATH_TC) {
    const int rc = tide::fused_checkpoint_launch(a, s, g_err, sizeof(g_err));
    // a device that cannot hold one cluster of the size this hidden_dim
    // needs: the automatic choice falls back to the split path
    if (!(rc == TIDE_ERR_UNSUPPORTED && a->path == TIDE_PATH_AUTO && tide::tc_supported(a))) return rc;
    g_err[0] = '\0';  // not an error of this call: it goes on with the split path
    path = TIDE_PATH_TC_SPLIT;
  }

  SimtWs w = simt_ws(a->workspace, n);
  float *scores = a->scores_out ? a->scores_out : w.scores;
  if (path == TIDE_PATH_TC_SPLIT) {
    // the router clears the partition workspace itself
    int rc = tide::tc_route_launch(a, scores, w.stats, a->workspace, w.partition_bytes, s, g_err,
                                   sizeof(g_err));
    if (rc != TIDE_OK) return rc;
  } else {
    if (cudaMemsetAsync(a->workspace, 0, w.partition_bytes, s) != cudaSuccess)
      return fail(TIDE_ERR_CUDA, "tide_checkpoint: memset failed");
  }
  if (path != TIDE_PATH_TC_SPLIT && n > 0) {
    if (!a->down_t) return fail(TIDE_ERR_INVALID, "tide_checkpoint: SIMT path needs down_t");
    tide::RouteParams rp{};
    rp.x = a->x; rp.n_cap = n; rp.n_dev = a->n_rows_dev;
    rp.H = (int)a->hidden_dim; rp.B = (int)a->bottleneck_dim; rp.norm_type = a->norm_type;
    rp.w_norm = a->norm_weight; rp.b_norm = a->norm_bias; rp.eps = a->eps;
    rp.down_t = a->down_t; rp.up = a->up; rp.up_bias = a->up_bias;
    rp.scores = scores; rp.row_stats = w.stats; rp.err = a->error_word;
    launch_route(a->dtype, rp, (n + tide::kRouteRows - 1) / tide::kRouteRows, s);
    int rc = check_launch("tide_checkpoint(route)");
    if (rc != TIDE_OK) return rc;
  }
  tide::MoveParams mp{};
  mp.x = a->x; mp.n_cap = n; mp.n_dev = a->n_rows_dev; mp.H = a->hidden_dim; mp.n_total = a->n_total;
  mp.scores = scores; mp.threshold = a->threshold;
  mp.row_stats = w.stats; mp.norm_type = a->norm_type; mp.w_norm = a->norm_weight; mp.b_norm = a->norm_bias;
  mp.exits_dense = false;
  mp.pos_in = a->positions_in; mp.slot_in = a->slots_in;
  mp.out_buf = a->out_buffer; mp.compact_out = a->compact_out;
  mp.pos_out64 = a->positions_out; mp.slot_out = a->slots_out;
  mp.exit_pos_out64 = a->exit_positions_out;
  mp.counts = a->counts_out;
  mp.ticket = w.ticket; mp.status = w.status; mp.err = a->error_word;
  const bool vec = rows_vectorizable(a->dtype, a->hidden_dim, {a->x, a->out_buffer, a->compact_out});
  if (tide::bulk_move_supported(a->dtype, a->hidden_dim, vec, mp)) {
    if (tide::bulk_move_launch(a->dtype, mp, s) != TIDE_OK) return check_launch("tide_checkpoint(bulk move)");
    return check_launch("tide_checkpoint(bulk move)");
  }
  const int64_t grid = n > 0 ? (n + tide::kMoveTile - 1) / tide::kMoveTile : 1;
  dispatch_rows<MoveLaunch>(a->dtype, vec, mp, grid, s);
  return check_launch("tide_checkpoint(move)");
}

}  // extern "C"

namespace tide {
// Lets other translation units of the library report through tide_last_error().
void set_last_error(const char *msg) { snprintf(g_err, sizeof(g_err), "%s", msg); }
}  // namespace tide
