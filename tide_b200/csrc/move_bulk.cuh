// Bulk-copy stable partition + row moves (move_bulk.cu): declarations used
// by the C ABI.
#pragma once

#include "common.cuh"
#include "simt_kernels.cuh"

namespace tide {

// Rows per look-back tile of the bulk mover (the status array needs one word
// per tile).
int bulk_tile_rows();
// True when the bulk mover takes rows of this type and width: 16-byte rows
// (vec), 2 KB to ~24 KB per row, 16-byte aligned norm weight and bias.
bool bulk_move_supported(int dtype, int64_t H, bool vec, const MoveParams &p);
int bulk_move_launch(int dtype, const MoveParams &p, cudaStream_t s);

}  // namespace tide
