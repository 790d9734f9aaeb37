// smo_fused_bf16.cu -- the fused kernel's instances for __nv_bfloat16 tensors (a
// translation unit per storage type, so that the library builds them in
// parallel).
#include "smo_fused.cuh"

namespace smo {

int launch_fused_bf16(int key, FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
                      cudaStream_t stream) {
    return launch_fused_window<__nv_bfloat16>(key, b, max_w, halo_floats, ws, flag_bytes, stream);
}

}  // namespace smo
