/*
 * smo_b200.h -- C ABI of the B200 SMO / SMO8bit optimizer-step library.
 *
 * The reference (mcarbonell/smo-optimizer) is pure Python: its "interface" for
 * this path is the torch.optim.Optimizer step of two classes.  Each entry point
 * below replaces one piece of that Python path; the Python drop-in classes in
 * smo_optimizer_b200/optimizers.py are the binding (ctypes) and build one
 * descriptor per parameter tensor.
 *
 * Conventions: plain pointers to device memory, sizes in elements, a CUDA
 * stream passed as void* (0 = legacy default stream).  No entry point
 * allocates device memory; scratch comes from the caller's workspace.  Every
 * call returns an smo_status (0 = success).  Work is enqueued asynchronously
 * on the stream; device-side failures are reported through smo_workspace_status().
 */
#ifndef SMO_B200_H
#define SMO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SMO_ABI_VERSION 3

#if defined(__GNUC__)
#define SMO_API __attribute__((visibility("default")))
#else
#define SMO_API
#endif

typedef enum smo_status {
    SMO_OK = 0,
    SMO_ERR_INVALID = 1,     /* bad descriptor: shape, kind, block or null pointer */
    SMO_ERR_ALIGNMENT = 2,   /* a pointer is not aligned to its element size */
    SMO_ERR_WORKSPACE = 3,   /* workspace missing or smaller than smo_workspace_size() */
    SMO_ERR_CUDA = 4,        /* a CUDA call failed; see smo_last_cuda_error() */
    SMO_ERR_TIMEOUT = 5,     /* a bounded inter-CTA wait gave up (device status) */
    SMO_ERR_NONFINITE = 6    /* reserved */
} smo_status;

/* How one tensor's moments are kept (the reference's per-tensor state kinds). */
typedef enum smo_kind {
    SMO_KIND_POOLED8 = 1,    /* SMO8bit pooled int8 moments  (spatial_8bit.py:171-204) */
    SMO_KIND_POOLED32 = 2,   /* SMO fp32 pooled moments      (spatial.py:108-129) */
    SMO_KIND_DENSE = 3,      /* dense fp32 Adam moments      (spatial_8bit.py:205-208, spatial.py:130-133) */
    SMO_KIND_QUANT_ONLY = 4  /* full-resolution int8 moments (spatial_8bit.py:157-169) */
} smo_kind;

/* Element type of a tensor's param, grad, block scales and POOLED32 / DENSE
 * moments (smo_tensor.dtype).  The reference computes in the parameter's
 * dtype (spatial_8bit.py:118, :167, :195, :207): for BF16 / F16 every op is
 * evaluated in fp32 and its result rounded to the dtype once, as torch's CPU
 * kernels do; the alpha of add/add_ (weight decay, 1 - beta) is itself
 * rounded to the dtype.  The int8 codes are int8 for every dtype.  Pointers of
 * the float-typed fields below then point at 2-byte elements (cast them). */
typedef enum smo_dtype {
    SMO_DTYPE_F32 = 0,
    SMO_DTYPE_BF16 = 1,
    SMO_DTYPE_F16 = 2
} smo_dtype;

/* smo_tensor.flags */
#define SMO_FLAG_GENERAL_PATH 1  /* step this tensor with the general two-launch kernels
                                    even when the fused single-pass kernel could take it */

/* fp32 scalars of one tensor's step.  The host forms each in double exactly as
 * the reference's Python does (spatial_8bit.py:210-297) and rounds once. */
typedef struct smo_hyper {
    float beta1, omb1;        /* beta1, 1 - beta1 */
    float beta2, omb2;        /* beta2, 1 - beta2 */
    float weight_decay;       /* L2-in-gradient: g + wd * p */
    int32_t wd_on;            /* weight_decay != 0 */
    float neg_step;           /* -(lr / (1 - beta1^step)) */
    float sqrt_bc2;           /* sqrt(1 - beta2^step) */
    float eps;
    int32_t reserved;
} smo_hyper;

/* One parameter tensor of a step.  Moments are read from *_in and written to
 * *_out.  in == out is allowed, but pooled tensors then take the general
 * two-launch kernels (the fused single-pass kernel needs separate buffers).
 * Fields a kind does not use must be NULL / 0.
 *
 *   POOLED8    param/grad [rows*cols]; codes [ceil(C/q_block)*q_block] int8,
 *              scales [ceil(C/q_block)], C = comp_rows*comp_cols
 *   POOLED32   param/grad [rows*cols]; m/v [comp_rows*comp_cols]
 *   DENSE      param/grad/m/v [rows] (cols = 1)
 *   QUANT_ONLY param/grad [rows] (cols = 1); codes/scales as POOLED8 over rows
 * Every non-code array holds elements of type `dtype` (fp32 for SMO_DTYPE_F32).
 */
typedef struct smo_tensor {
    float *param;
    const float *grad;
    const int8_t *m_q_in;
    const float *m_s_in;
    const int8_t *v_q_in;
    const float *v_s_in;
    int8_t *m_q_out;
    float *m_s_out;
    int8_t *v_q_out;
    float *v_s_out;
    const float *m_in;
    const float *v_in;
    float *m_out;
    float *v_out;
    int64_t rows, cols;             /* pooled row view (2-D math view of the param) */
    int64_t comp_rows, comp_cols;   /* compact moment grid (pooled kinds) */
    int64_t q_block;                /* int8 block size (POOLED8, QUANT_ONLY) */
    int64_t interp_band;            /* low_peak: compact rows per interpolation band
                                       (spatial_8bit.py:359); 0 = monolithic */
    int32_t kind;                   /* smo_kind */
    int32_t flags;                  /* SMO_FLAG_* (0 = let the library choose the kernel) */
    smo_hyper hp;
    /* permute_basis (spatial_8bit.py:202-204, 231-253; pooled kinds, monolithic
       interpolation): the gradient is pooled in the basis whose row i is view
       row row_perm[i] and column j is view column col_perm[j], and the
       reconstructed moments are mapped back with the inverse permutations
       (row_perm_inv[row_perm[i]] = i).  All four null = no permutation. */
    const int64_t *row_perm, *col_perm, *row_perm_inv, *col_perm_inv;
    int32_t dtype;                  /* smo_dtype (ABI 3) */
    int32_t reserved;               /* 0 */
} smo_tensor;

/* ---- the optimizer step ------------------------------------------------ */

/* Bytes of device workspace smo_step() needs for these tensors (0 if none). */
SMO_API size_t smo_workspace_size(const smo_tensor *tensors, int32_t n);

/* One optimizer step over n tensors, enqueued on `stream`.
 * Replaces SMO8bit.step (smo/optimizers/spatial_8bit.py:124-299), its low_peak
 * path SMO8bit._step_banded (spatial_8bit.py:307-374) and SMO.step
 * (smo/optimizers/spatial.py:82-208) for every tensor that has a gradient.
 * The workspace must stay untouched by others until the work completes, and
 * two steps that share a workspace must not overlap on the device. */
SMO_API int smo_step(const smo_tensor *tensors, int32_t n, void *workspace, size_t workspace_bytes, void *stream);

/* Device-side status of the steps that used `workspace` since the last call
 * (waits for the stream): SMO_OK or SMO_ERR_TIMEOUT.  The status is sticky
 * until read: a non-zero status is cleared by this call, so the next step
 * starts clean.  No counterpart in the reference (its step is synchronous
 * Python and raises directly). */
SMO_API int smo_workspace_status(void *workspace, void *stream);

/* Poll limit of the fused kernel's bounded inter-CTA waits for launches made
 * after this call, process-wide; a negative value restores the default
 * (2^22 polls).  Returns the previous setting (-1 = default).  A limit that
 * runs out makes the step report SMO_ERR_TIMEOUT through
 * smo_workspace_status() instead of waiting longer; the step's parameters are
 * then not valid.  Diagnostic hook for exercising the failure path without a
 * GPU fault.  No counterpart in the reference. */
SMO_API int64_t smo_set_wait_limit(int64_t max_polls);

/* Diagnostic for the failure path, process-wide: with on != 0, every
 * inter-CTA wait of later fused launches waits for a flag value that no strip
 * publishes, so each runs out its poll limit (smo_set_wait_limit) and the step
 * reports SMO_ERR_TIMEOUT; its parameters are then not valid.  Every wait
 * stays bounded, nothing faults.  on = 0 restores normal operation.  Returns
 * the previous setting.  No counterpart in the reference. */
SMO_API int smo_inject_wait_timeout(int on);

/* Bytes of the fixed scratch array behind smo_step_no_alloc(). */
#define SMO_NO_ALLOC_SCRATCH_BYTES ((size_t)32 << 20)

/* The same step as smo_step() for callers that cannot allocate device memory
 * (for instance a plug-in that only receives the device pointers of its inputs
 * and outputs from a host runtime that owns all device memory).  No
 * counterpart in the reference.
 * Scratch comes from a 32 MiB array in the library's own device memory, held
 * on every GPU where the library's device code is loaded until the process
 * exits; the call allocates nothing.  Descriptors are validated first (a bad
 * one returns its error and touches nothing); then a step whose
 * smo_workspace_size() exceeds SMO_NO_ALLOC_SCRATCH_BYTES is rejected with
 * SMO_ERR_WORKSPACE before any work is enqueued.  The first call on a device
 * resolves that device's copy of the array (cudaGetSymbolAddress, with the
 * device current) and keeps the address for the life of the process; make
 * that first call before any stream capture, and do not call this entry point
 * on a device after cudaDeviceReset().  All calls share the one array and it keeps the
 * previous call's contents: calls that overlap on the GPU (other streams,
 * other threads) race and must be serialised by the caller.  If
 * device_status is not NULL (a device int32), the step's device-side status
 * (SMO_OK or SMO_ERR_TIMEOUT) is copied there, in stream order. */
SMO_API int smo_step_no_alloc(const smo_tensor *tensors, int32_t n, int32_t *device_status, void *stream);

/* ---- stage entry points (same arithmetic as the fused step) ------------ */

/* SMO8bit._quantize_blockwise (spatial_8bit.py:85-107): x[n] -> codes
 * [ceil(n/block)*block] (tail coded from zero padding), scales [ceil(n/block)]. */
SMO_API int smo_quantize_blockwise(const float *x, int64_t n, int64_t block, int8_t *codes, float *scales, void *stream);

/* SMO8bit._dequantize_blockwise (spatial_8bit.py:109-122): codes, scales -> out[n]. */
SMO_API int smo_dequantize_blockwise(const int8_t *codes, const float *scales, int64_t n, int64_t block, float *out,
                             void *stream);

/* compress_2d_pair (smo/optimizers/_spatial_utils.py:72-91) of x = grad + wd*param
 * (wd_on = 0: x = grad): window means of x and x*x onto the (h, w) grid,
 * exact windows when they tile the (H, W) view, adaptive bins otherwise. */
SMO_API int smo_pool2d_pair(const float *grad, const float *param, int64_t H, int64_t W, int64_t h, int64_t w,
                    float weight_decay, int32_t wd_on, float *out_mean, float *out_sq_mean, void *stream);

/* upsample_2d_pair (_spatial_utils.py:128-176, bilinear, align_corners=False) of
 * one (h, w) channel onto (H, W); interp_band > 0 reproduces the low_peak band
 * interpolation of spatial_8bit.py:359-370. */
SMO_API int smo_upsample2d(const float *src, int64_t h, int64_t w, int64_t H, int64_t W, int64_t interp_band,
                   float *out, void *stream);

/* ---- utilities ---------------------------------------------------------- */

/* Seeded synthetic N(0, std) fill: out[i] = value(base, offset + i) of the
 * counter-hash generator in smo_optimizer_b200/synthetic.py (bit-identical to
 * the host generator).  No counterpart in the reference (test/bench input). */
SMO_API int smo_synth_normal(float *out, int64_t n, uint64_t base, float scale, int64_t offset, void *stream);

/* Runs the library's bounded inter-CTA wait on a flag that nothing sets (a
 * word in the workspace header), with an iteration limit, and returns its
 * status in *status_out (host memory):
 * SMO_ERR_TIMEOUT when the wait gave up as designed.  No counterpart in the
 * reference (exercise of the failure path without a GPU fault). */
SMO_API int smo_selftest_wait_timeout(void *workspace, size_t workspace_bytes, int64_t max_iters, int32_t *status_out,
                              void *stream);

/* Self-test of the fused step's FMA-only square root, reciprocal and division
 * (approximation + Markstein corrections) against the IEEE operations on this
 * device, over the input ranges where the step relies on them being exact:
 * counts_out[0] = finite v >= 2^-102 (all of them) whose square root differs,
 * counts_out[1] = normal d in [2^-126, 2^126] (all of them) whose reciprocal
 * differs, counts_out[2] = differing quotients among n_pairs pseudo-random
 * in-range pairs, counts_out[3] = quotients checked.  Uses only the workspace
 * header (>= 256 bytes, 256-byte aligned) and waits for the stream.  No
 * counterpart in the reference. */
SMO_API int smo_selftest_fastmath(void *workspace, size_t workspace_bytes, uint64_t n_pairs, uint64_t *counts_out,
                                  void *stream);

/* Number of kernels this library has launched in this process (all devices,
 * all entry points), for launch accounting in benchmarks. */
SMO_API uint64_t smo_launch_count(void);

SMO_API const char *smo_status_string(int status);
SMO_API int smo_last_cuda_error(void);
SMO_API int smo_abi_version(void);
/* sizeof(smo_tensor) as compiled into the library (ABI check for bindings). */
SMO_API size_t smo_tensor_struct_size(void);

#ifdef __cplusplus
}
#endif

#endif /* SMO_B200_H */
