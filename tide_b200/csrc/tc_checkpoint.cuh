// Tensor-core (tcgen05) checkpoint kernel: declarations used by the C ABI.
#pragma once

#include <stddef.h>

#include <cuda.h>

#include "common.cuh"

namespace tide {

// Tensor map of a [rows, cols] row-major matrix of a TIDE_DTYPE_*, read in
// boxes of 128 bytes of a row by box_rows rows, with the 128-byte swizzle.
bool tc_make_tmap(CUtensorMap *m, const void *base, int dtype, uint64_t rows, uint64_t cols,
                  uint32_t box_rows);

bool tc_supported(const tide_checkpoint_args *a);
const char *tc_unsupported_reason(const tide_checkpoint_args *a);
size_t tc_workspace_bytes(int64_t n_rows);
// Scores and per-row (mean, rstd) of the active rows on the tensor cores;
// also clears `zero` (zero_bytes, a multiple of 16), the stable-partition
// workspace of the mover launched after it.
int tc_route_launch(const tide_checkpoint_args *a, float *scores, float2 *row_stats, void *zero,
                    size_t zero_bytes, cudaStream_t s, char *err, size_t err_len);

// Paired-CTA router (tc_route_pair.cu): 16-bit rows, router width 128.
// tc_route_launch takes it where it applies when TIDE_ROUTER=pair.
bool tc_pair_supported(const tide_checkpoint_args *a);
int tc_route_pair_launch(const tide_checkpoint_args *a, float *scores, float2 *row_stats,
                         void *zero, size_t zero_bytes, cudaStream_t s, char *err, size_t err_len);

// Single-pass fused cluster kernel (tc_fused.cu).
bool fused_supported(const tide_checkpoint_args *a);
// Largest row count for which the automatic path choice takes the fused
// single pass at this hidden size (0: the fused kernel does not apply).
int64_t fused_auto_max_rows(int64_t H);
const char *fused_unsupported_reason(const tide_checkpoint_args *a);
size_t fused_workspace_bytes(const tide_checkpoint_args *a);
int fused_checkpoint_launch(const tide_checkpoint_args *a, cudaStream_t s, char *err, size_t err_len);

}  // namespace tide
