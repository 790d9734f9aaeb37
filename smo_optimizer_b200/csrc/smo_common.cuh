// smo_common.cuh -- shared device arithmetic of the SMO step.
//
// Every function here reproduces one fp32 operation sequence of the reference
// step (as executed by torch's CPU kernels) with each rounding explicit:
// __fmaf_rn where torch fuses a multiply-add, __fmul_rn / __fadd_rn /
// __fdiv_rn / __fsqrt_rn where it rounds each operation.  The library is also
// compiled with -fmad=false so that nothing else is contracted.
//
// The storage type T of a tensor (float, __nv_bfloat16, __half) is a template
// parameter: for half-precision parameters the reference computes in the
// parameter's dtype, and torch's CPU kernels evaluate each op in fp32 and
// round its result to the dtype once, which rd<T>() does at each op boundary
// (the identity for float).  The alpha of add/add_ (weight decay, the EMA's
// 1 - beta) is itself rounded to the dtype; other scalars stay fp32.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "smo_b200.h"

namespace smo {

// ---------------------------------------------------------------- storage types

template <class T>
__device__ __forceinline__ float rd(float x) { return x; }
template <>
__device__ __forceinline__ float rd<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <>
__device__ __forceinline__ float rd<__half>(float x) { return __half2float(__float2half_rn(x)); }

template <class T>
__device__ __forceinline__ float ld(const T *p) { return *p; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16 *p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float ld<__half>(const __half *p) { return __half2float(*p); }

template <class T>
__device__ __forceinline__ void st(T *p, float x) { *p = x; }
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16 *p, float x) { *p = __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ void st<__half>(__half *p, float x) { *p = __float2half_rn(x); }

// Four consecutive elements (one 16-byte fp32 or 8-byte half access; the
// address must be aligned to that size) as fp32, and back.
template <class T>
__device__ __forceinline__ void ld4(const T *p, float (&v)[4]) {
    if constexpr (sizeof(T) == 4) {
        const float4 t = *reinterpret_cast<const float4 *>(p);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
        const uint2 t = *reinterpret_cast<const uint2 *>(p);
        const T *e = reinterpret_cast<const T *>(&t);
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = ld<T>(e + k);
    }
}

template <class T>
__device__ __forceinline__ void st4(T *p, const float (&v)[4]) {
    if constexpr (sizeof(T) == 4) {
        *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        uint2 t;
        T *e = reinterpret_cast<T *>(&t);
#pragma unroll
        for (int k = 0; k < 4; k++) st<T>(e + k, v[k]);
        *reinterpret_cast<uint2 *>(p) = t;
    }
}

// ---------------------------------------------------------------- scalars

// x = g + wd * p  (grad.add(p, alpha=wd), spatial_8bit.py:217-218)
template <class T = float>
__device__ __forceinline__ float decayed(float g, float p, const smo_hyper &hp) {
    return hp.wd_on ? rd<T>(__fmaf_rn(rd<T>(hp.weight_decay), p, g)) : g;
}

// m.mul_(b1).add_(u, alpha=1-b1)  (spatial_8bit.py:240-242)
template <class T = float>
__device__ __forceinline__ float ema(float m, float u, float beta, float omb) {
    return rd<T>(__fmaf_rn(rd<T>(omb), u, rd<T>(__fmul_rn(m, beta))));
}

// v.mul_(b2).addcmul_(x, x, value=1-b2)  (spatial_8bit.py:281)
template <class T = float>
__device__ __forceinline__ float ema_sq(float v, float x, float beta, float omb) {
    return rd<T>(__fmaf_rn(__fmul_rn(omb, x), x, rd<T>(__fmul_rn(v, beta))));
}

// denom = sqrt(v)/sqrt(bc2) + eps;  p.addcdiv_(m, denom, value=-step_size)
// (spatial_8bit.py:293-297)
template <class T = float>
__device__ __forceinline__ float adam_write(float p, float m, float v, const smo_hyper &hp) {
    float d = rd<T>(__fadd_rn(rd<T>(__fdiv_rn(rd<T>(__fsqrt_rn(v)), hp.sqrt_bc2)), hp.eps));
    return rd<T>(__fadd_rn(p, __fdiv_rn(__fmul_rn(hp.neg_step, m), d)));
}

// ---------------------------------------------------------------- FMA-only sqrt and division
//
// Hardware approximations refined by FMA corrections (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Dev. 34(1), 1990; Muller et al., Handbook of
// Floating-Point Arithmetic, chapters on Newton-Raphson based division and
// square root).  Each sequence is exact (bit-identical to the IEEE operation)
// only on a stated input range; smo_selftest_fastmath() checks those ranges
// on the device: every input for the square root and the reciprocal,
// pseudo-random pairs for the quotient.

__device__ __forceinline__ float rsqrt_approx(float x) {
    float y;
    asm("rsqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// NaN-propagating min / max (PTX min.NaN / max.NaN)
__device__ __forceinline__ float nan_min(float a, float b) {
    float y;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(y) : "f"(a), "f"(b));
    return y;
}

__device__ __forceinline__ float nan_max(float a, float b) {
    float y;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(y) : "f"(a), "f"(b));
    return y;
}

// sqrt of each lane: s = v y, h = y / 2 (y ~ 1/sqrt(v)), then s + (v - s s) h.
// Equals the correctly rounded square root for every finite v >= 2^-102;
// +0 and +inf give NaN.
__device__ __forceinline__ float2 sqrt2_markstein(float2 v) {
    const float2 y = make_float2(rsqrt_approx(v.x), rsqrt_approx(v.y));
    const float2 s = __fmul2_rn(v, y), h = __fmul2_rn(make_float2(0.5f, 0.5f), y);
    const float2 r = __ffma2_rn(make_float2(-s.x, -s.y), s, v);
    return __ffma2_rn(r, h, s);
}

// reciprocal of each lane by one Newton step from the approximation; equals
// RN(1/d) for every normal d in [2^-126, 2^126]
__device__ __forceinline__ float2 rcp2_newton(float2 d) {
    const float2 r0 = make_float2(rcp_approx(d.x), rcp_approx(d.y));
    const float2 e = __ffma2_rn(make_float2(-d.x, -d.y), r0, make_float2(1.0f, 1.0f));
    return __ffma2_rn(r0, e, r0);
}

// a / d per lane with r = RN(1/d): q0 = RN(a r), rem = a - d q0 (exact by
// FMA), q = RN(q0 + rem r).  By Markstein's theorem q is the correctly rounded
// quotient when d is normal, q0 is within an ulp of a/d and nothing under- or
// overflows; for d >= 2^-27 that holds whenever |q0| is in [2^-76, 2^100]
// (then exponent(d) + exponent(q0) >= -103 keeps rem representable).
__device__ __forceinline__ float2 div2_markstein(float2 a, float2 d, float2 r, float2 &q0) {
    q0 = __fmul2_rn(a, r);
    const float2 rem = __ffma2_rn(make_float2(-q0.x, -q0.y), d, a);
    return __ffma2_rn(rem, r, q0);
}

// torch.clamp(v, min=0): NaN passes through (fmaxf would drop it)
__device__ __forceinline__ float clamp_min0(float v) { return v < 0.0f ? 0.0f : v; }

// NaN-propagating running max of |x| (torch's max reduction propagates NaN)
__device__ __forceinline__ float absmax_acc(float acc, float x) {
    float a = fabsf(x);
    return (a > acc || a != a) ? a : acc;
}

__device__ __forceinline__ float warp_absmax(float acc) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float other = __shfl_xor_sync(0xffffffffu, acc, o);
        acc = (other > acc || other != other) ? other : acc;
    }
    return acc;
}

// scales.clamp(min=1e-12) (spatial_8bit.py:96), NaN passes through; in the
// moments' dtype (fp16 has no 1e-12: an all-zero block gets scale 0)
template <class T = float>
__device__ __forceinline__ float block_scale(float absmax) { return rd<T>(absmax < 1e-12f ? 1e-12f : absmax); }

// q = round(x / s * 127) half-to-even, dead-zone lift, clamp +-127
// (spatial_8bit.py:97-106).  NaN is stored as 0.
template <class T = float>
__device__ __forceinline__ int8_t quantize1(float x, float s) {
    float r = rintf(rd<T>(__fmul_rn(rd<T>(__fdiv_rn(x, s)), 127.0f)));
    if (r == 0.0f && x != 0.0f && x == x) r = x > 0.0f ? 1.0f : -1.0f;
    r = r > 127.0f ? 127.0f : r;
    r = r < -127.0f ? -127.0f : r;
    return (r == r) ? (int8_t)(int)r : (int8_t)0;
}

// q * (s / 127)  (spatial_8bit.py:118)
template <class T = float>
__device__ __forceinline__ float dequant_step(float s) { return rd<T>(__fdiv_rn(s, 127.0f)); }
template <class T = float>
__device__ __forceinline__ float dequant1(int8_t q, float t) { return rd<T>(__fmul_rn((float)q, t)); }

// ---------------------------------------------------------------- bilinear

// torch's compute_source_index_and_lambda for align_corners=False
struct Coef {
    int64_t i0, i1;
    float l0, l1;
    int ident;  // equal extents: pass-through
};

// torch's source-index scale in / out of one interpolated dimension
__device__ __forceinline__ float coef_scale(int64_t in, int64_t out) { return __fdiv_rn((float)in, (float)out); }

// coefficients of output index o, with scale = coef_scale(in, out) (callers
// that walk a whole row form it once)
__device__ __forceinline__ Coef coef_for_scaled(int64_t o, int64_t in, int64_t out, float scale) {
    Coef c;
    if (in == out) {
        c.i0 = c.i1 = o;
        c.l0 = 1.0f;
        c.l1 = 0.0f;
        c.ident = 1;
        return c;
    }
    float real = __fmaf_rn(scale, __fadd_rn((float)o, 0.5f), -0.5f);
    real = real < 0.0f ? 0.0f : real;
    int64_t i0 = (int64_t)floorf(real);
    i0 = i0 > in - 1 ? in - 1 : i0;
    float l1 = __fsub_rn(real, (float)i0);
    l1 = l1 < 0.0f ? 0.0f : (l1 > 1.0f ? 1.0f : l1);
    c.i0 = i0;
    c.i1 = i0 + (i0 < in - 1 ? 1 : 0);
    c.l1 = l1;
    c.l0 = __fsub_rn(1.0f, l1);
    c.ident = 0;
    return c;
}

__device__ __forceinline__ Coef coef_for(int64_t o, int64_t in, int64_t out) {
    return coef_for_scaled(o, in, out, in == out ? 1.0f : coef_scale(in, out));
}

// Row coefficients; interp_band > 0 reproduces the low_peak bands of
// spatial_8bit.py:359-370 (rows [a, b) interpolated onto (b-a)*kh rows).
__device__ __forceinline__ Coef row_coef(int64_t r, int64_t H, int64_t h, int64_t W, int64_t band, int &small) {
    if (band <= 0) {
        small = (H + W <= 128);
        return coef_for(r, h, H);
    }
    int64_t kh = H / h;
    int64_t s0 = ((r / kh) / band) * band;
    int64_t s1 = s0 + band < h ? s0 + band : h;
    int64_t a = s0 > 0 ? s0 - 1 : 0;
    int64_t b = s1 + 1 < h ? s1 + 1 : h;
    int64_t n = b - a;
    small = (n * kh + W <= 128);
    Coef c = coef_for(r - a * kh, n, n * kh);
    c.i0 += a;
    c.i1 += a;
    return c;
}

// torch's separable bilinear (output H+W > 128): width pass, then height pass
// (src elements of type S; the result in fp32, before any rounding to a dtype)
template <class S = float>
__device__ __forceinline__ float interp_generic(const S *src, int64_t w, const Coef &rc, const Coef &cc,
                                                int64_t r, int64_t q) {
    if (rc.ident && cc.ident) return ld<S>(src + r * w + q);
    if (rc.ident) {
        const S *s = src + r * w;
        return __fmaf_rn(ld<S>(s + cc.i0), cc.l0, __fmul_rn(ld<S>(s + cc.i1), cc.l1));
    }
    if (cc.ident)
        return __fmaf_rn(ld<S>(src + rc.i0 * w + q), rc.l0, __fmul_rn(ld<S>(src + rc.i1 * w + q), rc.l1));
    const S *s0 = src + rc.i0 * w, *s1 = src + rc.i1 * w;
    float t0 = __fmaf_rn(ld<S>(s0 + cc.i0), cc.l0, __fmul_rn(ld<S>(s0 + cc.i1), cc.l1));
    float t1 = __fmaf_rn(ld<S>(s1 + cc.i0), cc.l0, __fmul_rn(ld<S>(s1 + cc.i1), cc.l1));
    return __fmaf_rn(t0, rc.l0, __fmul_rn(t1, rc.l1));
}

// torch's channels-last bilinear kernel (used when output H+W <= 128)
template <class S = float>
__device__ __forceinline__ float interp_small(const S *src, int64_t w, const Coef &rc, const Coef &cc) {
    float w00 = __fmul_rn(rc.l0, cc.l0), w01 = __fmul_rn(rc.l0, cc.l1);
    float w10 = __fmul_rn(rc.l1, cc.l0), w11 = __fmul_rn(rc.l1, cc.l1);
    float a = ld<S>(src + rc.i0 * w + cc.i0), b = ld<S>(src + rc.i0 * w + cc.i1);
    float c = ld<S>(src + rc.i1 * w + cc.i0), d = ld<S>(src + rc.i1 * w + cc.i1);
    return __fmaf_rn(d, w11, __fmaf_rn(c, w10, __fmaf_rn(a, w00, __fmul_rn(b, w01))));
}

// ---------------------------------------------------------------- pooling

// Window sums of x and x*x for compact cell (i, j): sequential row-major from
// +0 (torch's cpu avg_pool2d / adaptive_avg_pool2d loops), then the divisions.
// With rp / cp set the window is taken in the permuted basis: its row r and
// column c are view row rp[r] and column cp[c] (g[rp][:, cp] of
// spatial_8bit.py:235-237).
template <class T = float>
__device__ __forceinline__ void pool_cell(const T *__restrict__ g, const T *__restrict__ p, int64_t H,
                                          int64_t W, int64_t h, int64_t w, int exact, int64_t i, int64_t j,
                                          const smo_hyper &hp, float &mean, float &sq_mean,
                                          const int64_t *rp = nullptr, const int64_t *cp = nullptr) {
    int64_t r0, r1, c0, c1;
    if (exact) {
        int64_t kh = H / h, kw = W / w;
        r0 = i * kh; r1 = r0 + kh;
        c0 = j * kw; c1 = c0 + kw;
    } else {
        r0 = (i * H) / h; r1 = ((i + 1) * H + h - 1) / h;
        c0 = (j * W) / w; c1 = ((j + 1) * W + w - 1) / w;
    }
    float s1 = 0.0f, s2 = 0.0f;
    for (int64_t r = r0; r < r1; r++) {
        const int64_t vr = rp ? rp[r] : r;
        const T *gr = g + vr * W, *pr = p + vr * W;
        for (int64_t c = c0; c < c1; c++) {
            const int64_t vc = cp ? cp[c] : c;
            float x = decayed<T>(ld<T>(gr + vc), ld<T>(pr + vc), hp);
            s1 = __fadd_rn(s1, x);
            s2 = __fadd_rn(s2, rd<T>(__fmul_rn(x, x)));  // torch.square, then the pool
        }
    }
    if (exact) {
        float div = (float)((r1 - r0) * (c1 - c0));
        mean = rd<T>(__fdiv_rn(s1, div));
        sq_mean = rd<T>(__fdiv_rn(s2, div));
    } else {
        float dh = (float)(r1 - r0), dw = (float)(c1 - c0);
        mean = rd<T>(__fdiv_rn(__fdiv_rn(s1, dh), dw));
        sq_mean = rd<T>(__fdiv_rn(__fdiv_rn(s2, dh), dw));
    }
}

}  // namespace smo
