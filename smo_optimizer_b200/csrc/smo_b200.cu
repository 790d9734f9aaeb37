// smo_b200.cu -- C ABI, launchers and the general (any-shape) step kernels.
//
// The step over a batch of tensors runs as two launches:
//   step_a_kernel  one warp per work item:
//                    pooled kinds: one int8 block (or 64 cells) of the compact
//                      grid: window sums of x = g + wd*p and x*x, dequant, EMA,
//                      block absmax, requant; post-EMA fp32 moments go to the
//                      compact buffers that step_b reads;
//                    QUANT_ONLY: one int8 block of elements, EMA, requant, write;
//                    DENSE: 1024 elements, EMA, write.
//   step_b_kernel  one warp per full-resolution row of a pooled tensor:
//                    bilinear reconstruction of m, v, clamp, Adam write.
// The fused single-pass kernel for exact-window pooled tensors lives in
// smo_fused.cu and is chosen by the launcher when a tensor qualifies.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "smo_common.cuh"
#include "smo_internal.cuh"

using namespace smo;

namespace smo {

thread_local int g_last_cuda_error = 0;
std::atomic<uint64_t> g_launches{0};

static int cuda_fail(cudaError_t e) {
    g_last_cuda_error = (int)e;
    return SMO_ERR_CUDA;
}

// ---------------------------------------------------------------- kernels

__device__ __forceinline__ int find_tensor(const int64_t *start, int n, int64_t item) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (start[mid] <= item) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Storage type T of param, grad, block scales and fp32-kind moments (float,
// __nv_bfloat16, __half); the post-EMA scratch of POOLED8 is fp32 (its values
// are already rounded to T).  rd<T> rounds each op to T (identity for float).
template <class T>
__device__ void pooled_block_item(const DevDesc &d, int64_t item, int lane) {
    const int64_t C = d.h * d.w;
    const bool q8 = (d.kind == SMO_KIND_POOLED8);
    const int64_t BI = q8 ? d.B : kPooled32Chunk;
    const int64_t base = item * BI;
    const smo_hyper &hp = d.hp;
    const T *g = (const T *)d.g, *p = (const T *)d.p;
    float tm = 0.0f, tv = 0.0f;
    if (q8) {
        tm = dequant_step<T>(ld<T>((const T *)d.ms_in + item));
        tv = dequant_step<T>(ld<T>((const T *)d.vs_in + item));
    }
    float am = 0.0f, av = 0.0f;
    for (int64_t k = lane; k < BI; k += 32) {
        int64_t c = base + k;
        if (c >= C) break;
        int64_t i = c / d.w, j = c - i * d.w;
        float gm, g2;
        pool_cell<T>(g, p, d.H, d.W, d.h, d.w, d.exact, i, j, hp, gm, g2, d.rp, d.cp);
        float m, v;
        if (q8) {
            m = dequant1<T>(d.mq_in[c], tm);
            v = dequant1<T>(d.vq_in[c], tv);
        } else {
            m = ld<T>((const T *)d.m_in + c);
            v = ld<T>((const T *)d.v_in + c);
        }
        m = ema<T>(m, gm, hp.beta1, hp.omb1);
        v = ema<T>(v, g2, hp.beta2, hp.omb2);
        if (q8) {
            d.m_out[c] = m;
            d.v_out[c] = v;
        } else {
            st<T>((T *)d.m_out + c, m);
            st<T>((T *)d.v_out + c, v);
        }
        am = absmax_acc(am, m);
        av = absmax_acc(av, v);
    }
    if (!q8) return;
    const float sm = block_scale<T>(warp_absmax(am));
    const float sv = block_scale<T>(warp_absmax(av));
    for (int64_t k = lane; k < BI; k += 32) {
        int64_t c = base + k;
        float m = 0.0f, v = 0.0f;
        if (c < C) {
            m = d.m_out[c];
            v = d.v_out[c];
        }
        d.mq_out[c] = quantize1<T>(m, sm);
        d.vq_out[c] = quantize1<T>(v, sv);
    }
    if (lane == 0) {
        st<T>((T *)d.ms_out + item, sm);
        st<T>((T *)d.vs_out + item, sv);
    }
}

// quant_only: one int8 block of B elements per warp, in two passes (the
// absmax, then the write).  Blocks of up to 64 elements (the default) keep
// their two elements per lane in registers between the passes; larger blocks
// re-read g, p and the codes in the second pass (from L1 or L2).  Holding
// more elements per lane was measured slower: the registers cost occupancy,
// and the kernel serves every kind.
template <class T>
__device__ void quant_only_item(const DevDesc &d, int64_t item, int lane) {
    const int64_t N = d.H;
    const int64_t B = d.B;
    const int64_t base = item * B;
    const smo_hyper &hp = d.hp;
    const T *g = (const T *)d.g;
    T *p = (T *)d.p;
    const float tm = dequant_step<T>(ld<T>((const T *)d.ms_in + item));
    const float tv = dequant_step<T>(ld<T>((const T *)d.vs_in + item));
    float am = 0.0f, av = 0.0f;
    if (B <= 64) {
        float pr[2], mr[2], vr[2];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int64_t k = lane + 32 * u, i = base + k;
            pr[u] = mr[u] = vr[u] = 0.0f;
            if (k < B && i < N) {
                pr[u] = ld<T>(p + i);
                const float x = decayed<T>(ld<T>(g + i), pr[u], hp);
                mr[u] = ema<T>(dequant1<T>(d.mq_in[i], tm), x, hp.beta1, hp.omb1);
                vr[u] = ema_sq<T>(dequant1<T>(d.vq_in[i], tv), x, hp.beta2, hp.omb2);
                am = absmax_acc(am, mr[u]);
                av = absmax_acc(av, vr[u]);
            }
        }
        const float sm = block_scale<T>(warp_absmax(am));
        const float sv = block_scale<T>(warp_absmax(av));
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int64_t k = lane + 32 * u, i = base + k;
            if (k >= B) break;
            if (i < N) {
                d.mq_out[i] = quantize1<T>(mr[u], sm);
                d.vq_out[i] = quantize1<T>(vr[u], sv);
                st<T>(p + i, adam_write<T>(pr[u], mr[u], vr[u], hp));
            } else {
                d.mq_out[i] = 0;
                d.vq_out[i] = 0;
            }
        }
        if (lane == 0) {
            st<T>((T *)d.ms_out + item, sm);
            st<T>((T *)d.vs_out + item, sv);
        }
        return;
    }
    for (int64_t k = lane; k < B; k += 32) {
        int64_t i = base + k;
        if (i >= N) break;
        float x = decayed<T>(ld<T>(g + i), ld<T>(p + i), hp);
        float m = ema<T>(dequant1<T>(d.mq_in[i], tm), x, hp.beta1, hp.omb1);
        float v = ema_sq<T>(dequant1<T>(d.vq_in[i], tv), x, hp.beta2, hp.omb2);
        am = absmax_acc(am, m);
        av = absmax_acc(av, v);
    }
    const float sm = block_scale<T>(warp_absmax(am));
    const float sv = block_scale<T>(warp_absmax(av));
    for (int64_t k = lane; k < B; k += 32) {
        int64_t i = base + k;
        if (i < N) {
            float pi = ld<T>(p + i);
            float x = decayed<T>(ld<T>(g + i), pi, hp);
            float m = ema<T>(dequant1<T>(d.mq_in[i], tm), x, hp.beta1, hp.omb1);
            float v = ema_sq<T>(dequant1<T>(d.vq_in[i], tv), x, hp.beta2, hp.omb2);
            d.mq_out[i] = quantize1<T>(m, sm);
            d.vq_out[i] = quantize1<T>(v, sv);
            st<T>(p + i, adam_write<T>(pi, m, v, hp));
        } else {
            d.mq_out[i] = 0;
            d.vq_out[i] = 0;
        }
    }
    if (lane == 0) {
        st<T>((T *)d.ms_out + item, sm);
        st<T>((T *)d.vs_out + item, sv);
    }
}

// dense Adam moments: 1024 elements per warp.  Each lane takes groups of
// four consecutive elements (16-byte fp32 / 8-byte half vector accesses when
// all six arrays are aligned for them: four independent loads in flight per
// lane); a group's loads come before its stores, so in-place moments
// (in == out) are fine.  One group per iteration keeps the kernel, which
// serves every kind, at its register budget.
template <class T>
__device__ void dense_item(const DevDesc &d, int64_t item, int lane) {
    const int64_t N = d.H;
    const int64_t base = item * kDenseChunk;
    const int64_t end = base + kDenseChunk < N ? base + kDenseChunk : N;
    const smo_hyper &hp = d.hp;
    const T *g = (const T *)d.g, *m_in = (const T *)d.m_in, *v_in = (const T *)d.v_in;
    T *p = (T *)d.p, *m_out = (T *)d.m_out, *v_out = (T *)d.v_out;
    constexpr uintptr_t kVec = 4 * sizeof(T);
    const bool vec = (((uintptr_t)(g + base) | (uintptr_t)(p + base) | (uintptr_t)(m_in + base) |
                       (uintptr_t)(v_in + base) | (uintptr_t)(m_out + base) | (uintptr_t)(v_out + base)) % kVec) == 0;
    int64_t i0 = base;
    if (vec) {
        const int64_t vend = base + (end - base) / 4 * 4;  // end of the whole groups of four
        for (int64_t i = base + 4 * lane; i < vend; i += 4 * 32) {
            float pv[4], gv[4], mv[4], vv[4];
            ld4<T>(p + i, pv);
            ld4<T>(g + i, gv);
            ld4<T>(m_in + i, mv);
            ld4<T>(v_in + i, vv);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float x = decayed<T>(gv[k], pv[k], hp);
                mv[k] = ema<T>(mv[k], x, hp.beta1, hp.omb1);
                vv[k] = ema_sq<T>(vv[k], x, hp.beta2, hp.omb2);
                pv[k] = adam_write<T>(pv[k], mv[k], vv[k], hp);
            }
            st4<T>(m_out + i, mv);
            st4<T>(v_out + i, vv);
            st4<T>(p + i, pv);
        }
        i0 = vend;
    }
    for (int64_t i = i0 + lane; i < end; i += 32) {
        float pi = ld<T>(p + i);
        float x = decayed<T>(ld<T>(g + i), pi, hp);
        float m = ema<T>(ld<T>(m_in + i), x, hp.beta1, hp.omb1);
        float v = ema_sq<T>(ld<T>(v_in + i), x, hp.beta2, hp.omb2);
        st<T>(m_out + i, m);
        st<T>(v_out + i, v);
        st<T>(p + i, adam_write<T>(pi, m, v, hp));
    }
}

template <class T>
__global__ void __launch_bounds__(256) step_a_kernel(const __grid_constant__ Batch b) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t total = b.start_a[b.n];
    for (int64_t it = warp; it < total; it += nwarps) {
        const int t = find_tensor(b.start_a, b.n, it);
        const DevDesc &d = b.d[t];
        const int64_t item = it - b.start_a[t];
        switch (d.kind) {
            case SMO_KIND_POOLED8:
            case SMO_KIND_POOLED32: pooled_block_item<T>(d, item, lane); break;
            case SMO_KIND_QUANT_ONLY: quant_only_item<T>(d, item, lane); break;
            case SMO_KIND_DENSE: dense_item<T>(d, item, lane); break;
            default: break;
        }
    }
}

// One full-resolution row r of a pooled tensor: moments of type S (fp32
// scratch for POOLED8, the state's type T for POOLED32), parameter of type T.
template <class T, class S>
__device__ __forceinline__ void adam_row(const DevDesc &d, int64_t r, int lane) {
    // the moments (scratch or the new state) and the parameter never overlap
    const S *__restrict__ mo = (const S *)d.m_out;
    const S *__restrict__ vo = (const S *)d.v_out;
    // permute_basis: parameter row r / column q sit at row rpi[r] / column
    // cpi[q] of the basis the moments were reconstructed in
    const int64_t br = d.rpi ? d.rpi[r] : r;
    int small;
    const Coef rc = row_coef(br, d.H, d.h, d.W, d.band, small);
    T *__restrict__ prow = (T *)d.p + r * d.W;
    const float cscale = d.w == d.W ? 1.0f : coef_scale(d.w, d.W);  // the same for every column
#pragma unroll 2
    for (int64_t q = lane; q < d.W; q += 32) {
        const int64_t bq = d.cpi ? d.cpi[q] : q;
        float mh, vh;
        if (d.same) {
            mh = ld<S>(mo + br * d.w + bq);
            vh = ld<S>(vo + br * d.w + bq);
        } else {
            const Coef cc = coef_for_scaled(bq, d.w, d.W, cscale);
            if (small) {
                mh = interp_small<S>(mo, d.w, rc, cc);
                vh = interp_small<S>(vo, d.w, rc, cc);
            } else {
                mh = interp_generic<S>(mo, d.w, rc, cc, br, bq);
                vh = interp_generic<S>(vo, d.w, rc, cc, br, bq);
            }
            mh = rd<T>(mh);
            vh = rd<T>(vh);
        }
        st<T>(prow + q, adam_write<T>(ld<T>(prow + q), mh, clamp_min0(vh), d.hp));
    }
}

template <class T>
__global__ void __launch_bounds__(256) step_b_kernel(const __grid_constant__ Batch b) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t total = b.start_b[b.n];
    for (int64_t it = warp; it < total; it += nwarps) {
        const int t = find_tensor(b.start_b, b.n, it);
        const DevDesc &d = b.d[t];
        const int64_t r = it - b.start_b[t];
        if (d.kind == SMO_KIND_POOLED32) adam_row<T, T>(d, r, lane);
        else adam_row<T, float>(d, r, lane);
    }
}

// ---------------------------------------------------------------- stage kernels

__global__ void quantize_kernel(const float *__restrict__ x, int64_t n, int64_t B, int8_t *codes, float *scales,
                                int64_t nb) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t b = warp; b < nb; b += nwarps) {
        float am = 0.0f;
        for (int64_t k = lane; k < B; k += 32) {
            int64_t i = b * B + k;
            if (i >= n) break;
            am = absmax_acc(am, x[i]);
        }
        const float s = block_scale(warp_absmax(am));
        for (int64_t k = lane; k < B; k += 32) {
            int64_t i = b * B + k;
            codes[i] = quantize1(i < n ? x[i] : 0.0f, s);
        }
        if (lane == 0) scales[b] = s;
    }
}

__global__ void dequantize_kernel(const int8_t *__restrict__ codes, const float *__restrict__ scales, int64_t n,
                                  int64_t B, float *out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = dequant1(codes[i], dequant_step(scales[i / B]));
}

__global__ void pool_kernel(const float *__restrict__ g, const float *__restrict__ p, int64_t H, int64_t W,
                            int64_t h, int64_t w, int exact, smo_hyper hp, float *om, float *o2) {
    const int64_t C = h * w;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < C; c += (int64_t)gridDim.x * blockDim.x) {
        int64_t i = c / w, j = c - i * w;
        pool_cell(g, p, H, W, h, w, exact, i, j, hp, om[c], o2[c]);
    }
}

__global__ void upsample_kernel(const float *__restrict__ src, int64_t h, int64_t w, int64_t H, int64_t W,
                                int64_t band, float *out) {
    const int64_t N = H * W;
    const int same = (h == H && w == W && band <= 0);
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < N; e += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = e / W, q = e - r * W;
        if (same) { out[e] = src[r * w + q]; continue; }
        int small;
        const Coef rc = row_coef(r, H, h, W, band, small);
        const Coef cc = coef_for(q, w, W);
        out[e] = small ? interp_small(src, w, rc, cc) : interp_generic(src, w, rc, cc, r, q);
    }
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void synth_normal_kernel(float *out, int64_t n, uint64_t base, float scale, int64_t offset) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        uint64_t idx = (uint64_t)(offset + i);
        uint64_t ha = splitmix64(base + 2ull * idx);
        uint64_t hb = splitmix64(base + 2ull * idx + 1ull);
        int64_t s = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) s += (int64_t)((ha >> (16 * k)) & 0xFFFFull) + (int64_t)((hb >> (16 * k)) & 0xFFFFull);
        out[i] = __fmul_rn((float)(2 * s - 8 * 65535), scale);
    }
}

__global__ void selftest_wait_kernel(const unsigned int *flag, int64_t max_iters, int32_t *status) {
    // Nothing sets *flag: the bounded wait must give up and report a timeout.
    int st = bounded_wait_geq(flag, 1u, max_iters) ? SMO_OK : SMO_ERR_TIMEOUT;
    if (threadIdx.x == 0 && blockIdx.x == 0) *status = st;
}

// Check of the FMA-only arithmetic of the fused step (smo_common.cuh) against
// the IEEE operations, on this device:
//   counts[0]: finite v >= 2^-102 (every one) where sqrt2_markstein differs
//              from __fsqrt_rn;
//   counts[1]: normal d in [2^-126, 2^126] (every one) where rcp2_newton
//              differs from __frcp_rn;
//   counts[2]: pseudo-random pairs (a of either sign, exponent -60..20; d in
//              [2^-27, 2^21)) with |q0| in [2^-76, 2^100] where div2_markstein
//              differs from __fdiv_rn;  counts[3]: pairs checked.
__device__ __forceinline__ uint64_t selftest_mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void selftest_fastmath_kernel(uint64_t n_pairs, unsigned long long *counts) {
    unsigned long long bad_sqrt = 0, bad_rcp = 0, bad_div = 0, checked = 0;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t first = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    // square roots: bit patterns 2^-102 .. max finite, two per iteration
    const uint64_t s_lo = 0x0c800000ull, s_n = (0x7f7fffffull - s_lo + 2) / 2;
    for (uint64_t i = first; i < s_n; i += stride) {
        const uint32_t b0 = (uint32_t)(s_lo + 2 * i), b1 = b0 + 1 <= 0x7f7fffffu ? b0 + 1 : b0;
        const float2 v = make_float2(__uint_as_float(b0), __uint_as_float(b1));
        const float2 r = sqrt2_markstein(v);
        bad_sqrt += (__float_as_uint(r.x) != __float_as_uint(__fsqrt_rn(v.x)));
        bad_sqrt += (__float_as_uint(r.y) != __float_as_uint(__fsqrt_rn(v.y)));
    }
    // reciprocals: 2^-126 .. 2^126
    const uint64_t r_lo = 0x00800000ull, r_n = (0x7e800000ull - r_lo + 2) / 2;
    for (uint64_t i = first; i < r_n; i += stride) {
        const uint32_t b0 = (uint32_t)(r_lo + 2 * i), b1 = b0 + 1 <= 0x7e800000u ? b0 + 1 : b0;
        const float2 d = make_float2(__uint_as_float(b0), __uint_as_float(b1));
        const float2 r = rcp2_newton(d);
        bad_rcp += (__float_as_uint(r.x) != __float_as_uint(__frcp_rn(d.x)));
        bad_rcp += (__float_as_uint(r.y) != __float_as_uint(__frcp_rn(d.y)));
    }
    for (uint64_t i = first; i < n_pairs; i += stride) {
        const uint64_t h = selftest_mix(i);
        const uint32_t ea = 127 - 60 + (uint32_t)((h >> 32) % 81), ed = 127 - 27 + (uint32_t)((h >> 48) % 48);
        const float a = __uint_as_float(((uint32_t)(h >> 31) & 0x80000000u) | (ea << 23) | ((uint32_t)h & 0x7fffffu));
        const float d = __uint_as_float((ed << 23) | ((uint32_t)(h >> 8) & 0x7fffffu));
        const float2 a2 = make_float2(a, -a), d2 = make_float2(d, d);
        float2 q0;
        const float2 q = div2_markstein(a2, d2, rcp2_newton(d2), q0);
        if (fabsf(q0.x) >= 0x1p-76f && fabsf(q0.x) <= 0x1p100f) {
            checked += 2;
            bad_div += (__float_as_uint(q.x) != __float_as_uint(__fdiv_rn(a, d)));
            bad_div += (__float_as_uint(q.y) != __float_as_uint(__fdiv_rn(-a, d)));
        }
    }
    if (bad_sqrt) atomicAdd(&counts[0], bad_sqrt);
    if (bad_rcp) atomicAdd(&counts[1], bad_rcp);
    if (bad_div) atomicAdd(&counts[2], bad_div);
    if (checked) atomicAdd(&counts[3], checked);
}

// ---------------------------------------------------------------- host side

static int device_sms() {
    static thread_local int sms = 0;
    if (!sms) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return 148;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    }
    return sms;
}

static inline bool aligned(const void *ptr, size_t a) { return ((uintptr_t)ptr % a) == 0; }

// Validates one ABI descriptor and fills the device descriptor; scratch
// offsets for POOLED8 post-EMA moments are assigned by the caller.
static int make_desc(const smo_tensor &t, DevDesc &d) {
    memset(&d, 0, sizeof(d));
    if (!t.param || !t.grad) return SMO_ERR_INVALID;
    if (t.dtype != SMO_DTYPE_F32 && t.dtype != SMO_DTYPE_BF16 && t.dtype != SMO_DTYPE_F16) return SMO_ERR_INVALID;
    // element size of param, grad, scales and fp32-kind moments
    const size_t es = t.dtype == SMO_DTYPE_F32 ? 4 : 2;
    if (!aligned(t.param, es) || !aligned(t.grad, es)) return SMO_ERR_ALIGNMENT;
    const int nperm = (t.row_perm != nullptr) + (t.col_perm != nullptr) + (t.row_perm_inv != nullptr) +
                      (t.col_perm_inv != nullptr);
    if (nperm && t.kind != SMO_KIND_POOLED8 && t.kind != SMO_KIND_POOLED32) return SMO_ERR_INVALID;
    d.p = t.param;
    d.g = t.grad;
    d.kind = t.kind;
    d.dtype = t.dtype;
    d.hp = t.hp;
    d.H = t.rows;
    d.W = t.cols;
    switch (t.kind) {
        case SMO_KIND_POOLED8:
        case SMO_KIND_POOLED32: {
            if (t.rows <= 0 || t.cols <= 0 || t.comp_rows <= 0 || t.comp_cols <= 0) return SMO_ERR_INVALID;
            if (t.comp_rows > t.rows || t.comp_cols > t.cols) return SMO_ERR_INVALID;
            d.h = t.comp_rows;
            d.w = t.comp_cols;
            d.exact = (t.rows % t.comp_rows == 0 && t.cols % t.comp_cols == 0);
            d.band = t.interp_band;
            if (d.band < 0 || (d.band > 0 && !d.exact)) return SMO_ERR_INVALID;
            d.same = (d.h == d.H && d.w == d.W && d.band == 0);
            if (nperm) {
                // permute_basis: all four index arrays, monolithic interpolation only
                // (the reference rejects low_peak with permute_basis, spatial_8bit.py:75-76)
                if (nperm != 4 || d.band != 0) return SMO_ERR_INVALID;
                if (!aligned(t.row_perm, 8) || !aligned(t.col_perm, 8) || !aligned(t.row_perm_inv, 8) ||
                    !aligned(t.col_perm_inv, 8))
                    return SMO_ERR_ALIGNMENT;
                d.rp = t.row_perm;
                d.cp = t.col_perm;
                d.rpi = t.row_perm_inv;
                d.cpi = t.col_perm_inv;
            }
            if (t.kind == SMO_KIND_POOLED8) {
                if (t.q_block <= 0) return SMO_ERR_INVALID;
                if (!t.m_q_in || !t.m_s_in || !t.v_q_in || !t.v_s_in || !t.m_q_out || !t.m_s_out || !t.v_q_out ||
                    !t.v_s_out)
                    return SMO_ERR_INVALID;
                if (!aligned(t.m_s_in, es) || !aligned(t.v_s_in, es) || !aligned(t.m_s_out, es) ||
                    !aligned(t.v_s_out, es))
                    return SMO_ERR_ALIGNMENT;
                d.B = t.q_block;
                d.mq_in = t.m_q_in; d.ms_in = t.m_s_in; d.vq_in = t.v_q_in; d.vs_in = t.v_s_in;
                d.mq_out = t.m_q_out; d.ms_out = t.m_s_out; d.vq_out = t.v_q_out; d.vs_out = t.v_s_out;
            } else {
                if (!t.m_in || !t.v_in || !t.m_out || !t.v_out) return SMO_ERR_INVALID;
                if (!aligned(t.m_in, es) || !aligned(t.v_in, es) || !aligned(t.m_out, es) || !aligned(t.v_out, es))
                    return SMO_ERR_ALIGNMENT;
                d.m_in = t.m_in; d.v_in = t.v_in; d.m_out = t.m_out; d.v_out = t.v_out;
            }
            return SMO_OK;
        }
        case SMO_KIND_DENSE:
            if (t.rows < 0 || t.cols != 1) return SMO_ERR_INVALID;
            if (!t.m_in || !t.v_in || !t.m_out || !t.v_out) return SMO_ERR_INVALID;
            if (!aligned(t.m_in, es) || !aligned(t.v_in, es) || !aligned(t.m_out, es) || !aligned(t.v_out, es))
                return SMO_ERR_ALIGNMENT;
            d.m_in = t.m_in; d.v_in = t.v_in; d.m_out = t.m_out; d.v_out = t.v_out;
            return SMO_OK;
        case SMO_KIND_QUANT_ONLY:
            if (t.rows < 0 || t.cols != 1 || t.q_block <= 0) return SMO_ERR_INVALID;
            if (!t.m_q_in || !t.m_s_in || !t.v_q_in || !t.v_s_in || !t.m_q_out || !t.m_s_out || !t.v_q_out ||
                !t.v_s_out)
                return SMO_ERR_INVALID;
            if (!aligned(t.m_s_in, es) || !aligned(t.v_s_in, es) || !aligned(t.m_s_out, es) || !aligned(t.v_s_out, es))
                return SMO_ERR_ALIGNMENT;
            d.B = t.q_block;
            d.mq_in = t.m_q_in; d.ms_in = t.m_s_in; d.vq_in = t.v_q_in; d.vs_in = t.v_s_in;
            d.mq_out = t.m_q_out; d.ms_out = t.m_s_out; d.vq_out = t.v_q_out; d.vs_out = t.v_s_out;
            return SMO_OK;
        default:
            return SMO_ERR_INVALID;
    }
}

int validate_tensors(const smo_tensor *t, int32_t n) {
    if (n < 0 || (n > 0 && !t)) return SMO_ERR_INVALID;
    for (int32_t i = 0; i < n; i++) {
        DevDesc d;
        const int st = make_desc(t[i], d);
        if (st != SMO_OK) return st;
    }
    return SMO_OK;
}

static inline int64_t items_a(const DevDesc &d) {
    switch (d.kind) {
        case SMO_KIND_POOLED8: return (d.h * d.w + d.B - 1) / d.B;
        case SMO_KIND_POOLED32: return (d.h * d.w + kPooled32Chunk - 1) / kPooled32Chunk;
        case SMO_KIND_QUANT_ONLY: return (d.H + d.B - 1) / d.B;
        case SMO_KIND_DENSE: return (d.H + kDenseChunk - 1) / kDenseChunk;
        default: return 0;
    }
}

static inline int64_t items_b(const DevDesc &d) {
    return (d.kind == SMO_KIND_POOLED8 || d.kind == SMO_KIND_POOLED32) ? d.H : 0;
}

static inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// scratch bytes of the general path for one tensor (POOLED8 post-EMA moments)
static inline size_t general_scratch(const smo_tensor &t) {
    if (t.kind != SMO_KIND_POOLED8 || fused_takes(t)) return 0;
    return 2 * round_up((size_t)t.comp_rows * (size_t)t.comp_cols * sizeof(float), kScratchAlign);
}

template <class T>
static int launch_general_t(Batch &b, cudaStream_t stream) {
    b.start_a[0] = 0;
    b.start_b[0] = 0;
    for (int i = 0; i < b.n; i++) {
        b.start_a[i + 1] = b.start_a[i] + items_a(b.d[i]);
        b.start_b[i + 1] = b.start_b[i] + items_b(b.d[i]);
    }
    const int threads = 256, warps = threads / 32;
    const int64_t cap = (int64_t)device_sms() * 16;
    if (b.start_a[b.n] > 0) {
        int64_t blocks = (b.start_a[b.n] + warps - 1) / warps;
        blocks = blocks < cap ? blocks : cap;
        step_a_kernel<T><<<(unsigned)blocks, threads, 0, stream>>>(b);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e);
        g_launches++;
    }
    if (b.start_b[b.n] > 0) {
        int64_t blocks = (b.start_b[b.n] + warps - 1) / warps;
        blocks = blocks < cap ? blocks : cap;
        step_b_kernel<T><<<(unsigned)blocks, threads, 0, stream>>>(b);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e);
        g_launches++;
    }
    return SMO_OK;
}

static int launch_general(Batch &b, int32_t dtype, cudaStream_t stream) {
    switch (dtype) {
        case SMO_DTYPE_BF16: return launch_general_t<__nv_bfloat16>(b, stream);
        case SMO_DTYPE_F16: return launch_general_t<__half>(b, stream);
        default: return launch_general_t<float>(b, stream);
    }
}

}  // namespace smo

// ===================================================================== C ABI

extern "C" {

size_t smo_workspace_size(const smo_tensor *tensors, int32_t n) {
    if (!tensors || n <= 0) return 0;
    size_t general = 0;
    for (int32_t i = 0; i < n; i++) general += general_scratch(tensors[i]);
    const FusedLayout fl = fused_workspace_layout(tensors, n);
    const size_t body = general > fl.body_bytes ? general : fl.body_bytes;
    return kWsHeader + fl.flag_bytes + body;
}

int smo_step(const smo_tensor *tensors, int32_t n, void *workspace, size_t workspace_bytes, void *stream_ptr) {
    if (n < 0 || (n > 0 && !tensors)) return SMO_ERR_INVALID;
    if (n == 0) return SMO_OK;
    cudaStream_t stream = (cudaStream_t)stream_ptr;

    // Validate everything before any launch: a bad descriptor launches nothing.
    int st = validate_tensors(tensors, n);
    if (st != SMO_OK) return st;
    const size_t need = smo_workspace_size(tensors, n);
    if (!workspace || workspace_bytes < need || !aligned(workspace, kScratchAlign)) return SMO_ERR_WORKSPACE;
    char *ws = (char *)workspace;
    const size_t flag_bytes = fused_workspace_layout(tensors, n).flag_bytes;

    // Tensors the fused single-pass kernel takes (exact-window pooled shapes).
    st = fused_step(tensors, n, ws, flag_bytes, stream);
    if (st != SMO_OK) return st;

    // Everything else goes through the general two-launch path, batched by
    // storage type; its scratch starts after the fused kernel's flag words.
    static thread_local Batch batch;
    const size_t base = kWsHeader + flag_bytes;
    for (int32_t dt = SMO_DTYPE_F32; dt <= SMO_DTYPE_F16; dt++) {
        size_t off = base;
        batch.n = 0;
        for (int32_t i = 0; i < n; i++) {
            if (tensors[i].dtype != dt || fused_takes(tensors[i])) continue;
            DevDesc &d = batch.d[batch.n];
            make_desc(tensors[i], d);
            if (d.kind == SMO_KIND_POOLED8) {
                const size_t bytes = round_up((size_t)(d.h * d.w) * sizeof(float), kScratchAlign);
                d.m_out = (float *)(ws + off);
                d.v_out = (float *)(ws + off + bytes);
                off += 2 * bytes;
            }
            batch.n++;
            if (batch.n == kMaxBatch) {
                st = launch_general(batch, dt, stream);
                if (st != SMO_OK) return st;
                batch.n = 0;
                off = base;  // stream order: the next launch pair starts after this one ends
            }
        }
        if (batch.n > 0) {
            st = launch_general(batch, dt, stream);
            if (st != SMO_OK) return st;
        }
    }
    return SMO_OK;
}

int64_t smo_set_wait_limit(int64_t max_polls) { return set_wait_limit(max_polls); }

int smo_inject_wait_timeout(int on) { return inject_wait_timeout(on); }

int smo_workspace_status(void *workspace, void *stream_ptr) {
    if (!workspace) return SMO_ERR_WORKSPACE;
    cudaStream_t stream = (cudaStream_t)stream_ptr;
    WsHeader h;
    cudaError_t e = cudaMemcpyAsync(&h, workspace, sizeof(h), cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return cuda_fail(e);
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e);
    if (h.error) {
        // read and cleared: the next step starts with a clean error word
        WsHeader *d = (WsHeader *)workspace;
        e = cudaMemsetAsync(&d->error, 0, 2 * sizeof(unsigned int), stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return cuda_fail(e);
    }
    return h.error ? (int)h.error : SMO_OK;
}

int smo_quantize_blockwise(const float *x, int64_t n, int64_t block, int8_t *codes, float *scales, void *stream) {
    if (n < 0 || block <= 0 || (n > 0 && (!x || !codes || !scales))) return SMO_ERR_INVALID;
    if (n == 0) return SMO_OK;
    const int64_t nb = (n + block - 1) / block;
    int64_t blocks = (nb + 7) / 8;
    const int64_t cap = (int64_t)device_sms() * 16;
    blocks = blocks < cap ? blocks : cap;
    quantize_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(x, n, block, codes, scales, nb);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    g_launches++;
    return SMO_OK;
}

int smo_dequantize_blockwise(const int8_t *codes, const float *scales, int64_t n, int64_t block, float *out,
                             void *stream) {
    if (n < 0 || block <= 0 || (n > 0 && (!codes || !scales || !out))) return SMO_ERR_INVALID;
    if (n == 0) return SMO_OK;
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = (int64_t)device_sms() * 16;
    blocks = blocks < cap ? blocks : cap;
    dequantize_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(codes, scales, n, block, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    g_launches++;
    return SMO_OK;
}

int smo_pool2d_pair(const float *grad, const float *param, int64_t H, int64_t W, int64_t h, int64_t w,
                    float weight_decay, int32_t wd_on, float *out_mean, float *out_sq_mean, void *stream) {
    if (H <= 0 || W <= 0 || h <= 0 || w <= 0 || h > H || w > W) return SMO_ERR_INVALID;
    if (!grad || !out_mean || !out_sq_mean || (wd_on && !param)) return SMO_ERR_INVALID;
    smo_hyper hp;
    memset(&hp, 0, sizeof(hp));
    hp.weight_decay = weight_decay;
    hp.wd_on = wd_on ? 1 : 0;
    const int exact = (H % h == 0 && W % w == 0);
    int64_t blocks = (h * w + 255) / 256;
    const int64_t cap = (int64_t)device_sms() * 16;
    blocks = blocks < cap ? blocks : cap;
    pool_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(grad, wd_on ? param : grad, H, W, h, w, exact,
                                                                     hp, out_mean, out_sq_mean);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    g_launches++;
    return SMO_OK;
}

int smo_upsample2d(const float *src, int64_t h, int64_t w, int64_t H, int64_t W, int64_t interp_band, float *out,
                   void *stream) {
    if (H <= 0 || W <= 0 || h <= 0 || w <= 0 || h > H || w > W || !src || !out) return SMO_ERR_INVALID;
    if (interp_band < 0 || (interp_band > 0 && (H % h != 0))) return SMO_ERR_INVALID;
    int64_t blocks = (H * W + 255) / 256;
    const int64_t cap = (int64_t)device_sms() * 16;
    blocks = blocks < cap ? blocks : cap;
    upsample_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(src, h, w, H, W, interp_band, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    g_launches++;
    return SMO_OK;
}

int smo_synth_normal(float *out, int64_t n, uint64_t base, float scale, int64_t offset, void *stream) {
    if (n < 0 || (n > 0 && !out)) return SMO_ERR_INVALID;
    if (n == 0) return SMO_OK;
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = (int64_t)device_sms() * 32;
    blocks = blocks < cap ? blocks : cap;
    synth_normal_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(out, n, base, scale, offset);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    g_launches++;
    return SMO_OK;
}

int smo_selftest_wait_timeout(void *workspace, size_t workspace_bytes, int64_t max_iters, int32_t *status_out,
                              void *stream_ptr) {
    if (!status_out || max_iters < 0) return SMO_ERR_INVALID;
    if (!workspace || workspace_bytes < kWsHeader || !aligned(workspace, kScratchAlign)) return SMO_ERR_WORKSPACE;
    cudaStream_t stream = (cudaStream_t)stream_ptr;
    // header words 32 (a flag nothing sets) and 33 (the status); the scheduler
    // words of a later step are untouched
    unsigned int *flag = (unsigned int *)workspace + 32;
    cudaError_t e = cudaMemsetAsync(flag, 0, 2 * sizeof(unsigned int), stream);
    if (e == cudaSuccess) {
        selftest_wait_kernel<<<1, 32, 0, stream>>>(flag, max_iters, (int32_t *)(flag + 1));
        e = cudaGetLastError();
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(status_out, flag + 1, sizeof(int32_t), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? SMO_OK : cuda_fail(e);
}

int smo_selftest_fastmath(void *workspace, size_t workspace_bytes, uint64_t n_pairs, uint64_t *counts_out,
                          void *stream_ptr) {
    if (!counts_out) return SMO_ERR_INVALID;
    if (!workspace || workspace_bytes < kWsHeader || !aligned(workspace, kScratchAlign)) return SMO_ERR_WORKSPACE;
    cudaStream_t stream = (cudaStream_t)stream_ptr;
    // header bytes 160..191 hold the four counters; a later step's words are untouched
    unsigned long long *counts = (unsigned long long *)((char *)workspace + 160);
    cudaError_t e = cudaMemsetAsync(counts, 0, 4 * sizeof(unsigned long long), stream);
    if (e == cudaSuccess) {
        selftest_fastmath_kernel<<<device_sms() * 8, 256, 0, stream>>>(n_pairs, counts);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(counts_out, counts, 4 * sizeof(unsigned long long), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? SMO_OK : cuda_fail(e);
}

const char *smo_status_string(int status) {
    switch (status) {
        case SMO_OK: return "ok";
        case SMO_ERR_INVALID: return "invalid tensor descriptor";
        case SMO_ERR_ALIGNMENT: return "misaligned pointer";
        case SMO_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
        case SMO_ERR_CUDA: return "CUDA error";
        case SMO_ERR_TIMEOUT: return "bounded device wait timed out";
        case SMO_ERR_NONFINITE: return "non-finite value";
        default: return "unknown status";
    }
}

int smo_last_cuda_error(void) { return g_last_cuda_error; }

uint64_t smo_launch_count(void) { return g_launches.load(); }

int smo_abi_version(void) { return SMO_ABI_VERSION; }

size_t smo_tensor_struct_size(void) { return sizeof(smo_tensor); }

}  // extern "C"
