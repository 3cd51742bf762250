// Placeholder: the tensor-core path is not built yet.
#include "tc_checkpoint.cuh"

namespace tide {
bool tc_supported(const tide_checkpoint_args *) { return false; }
const char *tc_unsupported_reason(const tide_checkpoint_args *) { return "not built"; }
size_t tc_workspace_bytes(int64_t) { return 0; }
int tc_checkpoint_launch(const tide_checkpoint_args *, cudaStream_t, char *, size_t) { return TIDE_ERR_UNSUPPORTED; }
}  // namespace tide
