// smo_fused.cu -- fused single-pass step for exact-window pooled tensors.
#include "smo_internal.cuh"

namespace smo {

bool fused_takes(const smo_tensor &) { return false; }

size_t fused_workspace_size(const smo_tensor *, int32_t) { return 0; }

int fused_step(const smo_tensor *, int32_t, char *, size_t, cudaStream_t) { return SMO_OK; }

}  // namespace smo
