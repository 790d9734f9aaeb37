// smo_fused_f16.cu -- the fused kernel's instances for __half tensors (a
// translation unit per storage type, so that the library builds them in
// parallel).
#include "smo_fused.cuh"

namespace smo {

int launch_fused_f16(int key, FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
                     cudaStream_t stream) {
    return launch_fused_window<__half>(key, b, max_w, halo_floats, ws, flag_bytes, stream);
}

}  // namespace smo
