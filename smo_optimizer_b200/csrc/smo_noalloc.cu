// smo_noalloc.cu -- the optimizer step for callers that cannot allocate
// device memory.
//
// smo_step() needs a caller-owned workspace.  Some callers have no way to get
// one: code that runs as a plug-in inside a host runtime which owns all device
// memory and hands it only the device pointers of its inputs and outputs (a C
// or FFI host with no CUDA allocator of its own, an embedding framework whose
// memory budget forbids side allocations).  smo_step_no_alloc() serves them:
// its scratch is a fixed array in the library's own device memory, so the call
// allocates nothing.
//
// The array is a file-scope __device__ variable, so every GPU on which the
// library's device code is loaded holds its kNoAllocScratchBytes until the
// process exits.  In host code its name is only a stand-in for the symbol; the
// device address is obtained per device with cudaGetSymbolAddress (on the first
// call made with that device current) and that address is what the kernels get.
// The address is kept for the life of the process: a cudaDeviceReset() unloads
// the module, so the entry point must not be used on a device after a reset.
#include <cstdint>
#include <cstring>
#include <mutex>

#include <cuda_runtime.h>

#include "smo_b200.h"
#include "smo_internal.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = SMO_NO_ALLOC_SCRATCH_BYTES;

__device__ __align__(256) unsigned char g_no_alloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;

std::mutex g_setup_mutex;
void *g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's copy of the scratch array (the first call
// per device resolves it; the device must be current).
int scratch_for_current_device(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (smo::g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    if (dev < 0 || dev >= kMaxDevices) return SMO_ERR_INVALID;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_no_alloc_scratch);
        if (e != cudaSuccess || !p) return (smo::g_last_cuda_error = (int)e, SMO_ERR_CUDA);
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return SMO_OK;
}

}  // namespace

extern "C" int smo_step_no_alloc(const smo_tensor *tensors, int32_t n, int32_t *device_status, void *stream_ptr) {
    if (n < 0 || (n > 0 && !tensors)) return SMO_ERR_INVALID;
    if (n == 0) return SMO_OK;
    // Every check comes before the shared array is touched: a bad descriptor
    // or an oversize step changes nothing on the device.
    int st = smo::validate_tensors(tensors, n);
    if (st != SMO_OK) return st;
    const size_t need = smo_workspace_size(tensors, n);
    if (need > kNoAllocScratchBytes) return SMO_ERR_WORKSPACE;  // step larger than the fixed scratch
    void *scratch = nullptr;
    st = scratch_for_current_device(&scratch);
    if (st != SMO_OK) return st;
    cudaStream_t stream = (cudaStream_t)stream_ptr;
    // The array keeps the previous call's contents.  The work counters and the
    // error word must start at zero; the launch epoch is kept, so flag words
    // left by earlier calls never match this call's epoch.
    smo::WsHeader *hdr = (smo::WsHeader *)scratch;
    cudaError_t e = cudaMemsetAsync(&hdr->next_item, 0, 2 * sizeof(unsigned int), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(&hdr->error, 0, 2 * sizeof(unsigned int), stream);
    if (e != cudaSuccess) return (smo::g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    st = smo_step(tensors, n, scratch, kNoAllocScratchBytes, stream_ptr);
    if (st != SMO_OK) return st;
    if (device_status) {
        e = cudaMemcpyAsync(device_status, &hdr->error, sizeof(int32_t), cudaMemcpyDeviceToDevice, stream);
        if (e != cudaSuccess) return (smo::g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    }
    return SMO_OK;
}
