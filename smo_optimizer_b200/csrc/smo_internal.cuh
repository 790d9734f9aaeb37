// smo_internal.cuh -- device descriptors, workspace layout and waits shared by
// the general path (smo_b200.cu) and the fused path (smo_fused.cu).
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "smo_b200.h"

namespace smo {

constexpr int kMaxBatch = 96;           // descriptors per launch (kernel-parameter batch)
constexpr int64_t kDenseChunk = 1024;   // elements per DENSE work item
constexpr int64_t kPooled32Chunk = 64;  // compact cells per POOLED32 work item
constexpr size_t kScratchAlign = 256;

// Validated per-tensor descriptor as the kernels see it.  The float pointers
// of p, g, scales and POOLED32 / DENSE moments point at elements of type dtype
// (the kernels cast them); codes are int8 and POOLED8 scratch is fp32.
struct DevDesc {
    float *p;
    const float *g;
    const int8_t *mq_in;
    const float *ms_in;
    const int8_t *vq_in;
    const float *vs_in;
    int8_t *mq_out;
    float *ms_out;
    int8_t *vq_out;
    float *vs_out;
    const float *m_in;
    const float *v_in;
    float *m_out;  // POOLED32 / DENSE: new state; POOLED8: post-EMA scratch
    float *v_out;
    int64_t H, W, h, w, B, band;
    int32_t kind;
    int32_t exact;  // whole windows tile the view
    int32_t same;   // identity interpolation (h == H, w == W, monolithic)
    int32_t dtype;  // smo_dtype of p, g, scales and POOLED32 / DENSE moments
    smo_hyper hp;
    // permute_basis: pooling basis (rp, cp) and its inverse (rpi, cpi); null = identity
    const int64_t *rp, *cp, *rpi, *cpi;
};

// Kernel-parameter batch (__grid_constant__, < 32 KB).
struct Batch {
    int32_t n;
    int64_t start_a[kMaxBatch + 1];
    int64_t start_b[kMaxBatch + 1];
    DevDesc d[kMaxBatch];
};

// First kWsHeader bytes of every workspace: scheduler counters, launch epoch
// and the device-side error word.
struct WsHeader {
    unsigned int next_item;   // dynamic work counter of the fused kernel
    unsigned int done_ctas;   // CTAs that finished (the last one resets the counters)
    unsigned int epoch;       // launch sequence number (flags carry it)
    unsigned int error;       // smo_status of a device-side failure, 0 = none
    unsigned int error_where; // work unit that failed
    unsigned int pad[59];
};
constexpr size_t kWsHeader = 256;
static_assert(sizeof(WsHeader) == kWsHeader, "workspace header layout");

// Spin until *flag >= target with acquire semantics, at most max_iters polls
// (with a short sleep between polls).  Returns false when the limit ran out.
__device__ __forceinline__ bool bounded_wait_geq(const unsigned int *flag, unsigned int target, int64_t max_iters) {
    for (int64_t it = 0; it <= max_iters; it++) {
        unsigned int v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v >= target) return true;
        if (it >= 32) __nanosleep(it < 1024 ? 64 : 256);
    }
    return false;
}

// fused single-pass path (smo_fused.cu).  Workspace: header, then
// flag_bytes of strip flags (nothing else writes there), then the body.
struct FusedLayout {
    size_t flag_bytes;  // strip-ready flags, right after the header
    size_t body_bytes;  // published rows and head rows, shared with the general path's scratch
};
bool fused_takes(const smo_tensor &t);
FusedLayout fused_workspace_layout(const smo_tensor *t, int32_t n);
int fused_step(const smo_tensor *t, int32_t n, char *ws, size_t flag_bytes, cudaStream_t stream);
int64_t wait_limit();
int64_t set_wait_limit(int64_t polls);
int inject_wait_timeout(int on);

// Checks every descriptor of a step (smo_b200.cu); SMO_OK or the first error.
int validate_tensors(const smo_tensor *t, int32_t n);

extern thread_local int g_last_cuda_error;
extern std::atomic<uint64_t> g_launches;

}  // namespace smo
