// smo_fused.cuh -- fused single-pass step for exact-window pooled tensors:
// the device code and its launch, instantiated per storage type by
// smo_fused_f32.cu, smo_fused_bf16.cu and smo_fused_f16.cu; the host-side
// planning (which tensors, strips, workspace) is in smo_fused.cu.
//
// One persistent launch steps every qualifying tensor of the batch.  HBM sees
// each parameter and gradient element read once and each parameter written
// once (plus the compact moment state), instead of the general path's
// read-pool-write-scratch / read-scratch-interpolate-write round trip.
//
// Work unit: a STRIP of L compact rows (KH*L full-resolution rows), full
// width, of one tensor.  CTAs take strips in increasing order from an atomic
// counter in the workspace header.  Inside a strip the CTA runs a row pipeline
// over compact rows c:
//
//   phase 1 (row c)   window sums of x = g + wd*p and x*x (KH x KW windows,
//                     vector loads), dequant of the old codes, EMA; post-EMA
//                     fp32 m, v of the row go to a 3-row ring in shared memory;
//                     int8 blocks completed by this row are requantised and
//                     written (POOLED32: the new fp32 state is written).
//   phase 2 (row c-1) bilinear reconstruction of m, v from ring rows c-2..c
//                     (width pass, then height pass, torch's order), clamp,
//                     Adam write of the KH parameter rows.
//
// Neighbouring strips: the write of a strip's last row needs the first row of
// the next strip.  The CTA recomputes that row itself (look-ahead) from the
// next strip's g, p and OLD moment state; the old state is intact because
// the moments are double-buffered (read *_in, write *_out).  The write of a
// strip's FIRST row needs the previous strip's last row, which the previous
// strip publishes to the workspace (with a release flag) after its look-ahead
// read; so the first row is written last, after an acquire wait.  Waits only
// ever point at an earlier strip, which some running CTA took before this one,
// so they cannot deadlock whatever the residency; every wait is bounded and
// reports SMO_ERR_TIMEOUT in the workspace header instead of hanging.
//
// The parameter rows read in phase 1 are read again in phase 2 one pipeline
// step later; that second read is meant to hit L2.
#pragma once

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "smo_common.cuh"
#include "smo_internal.cuh"

namespace smo {

constexpr int kMaxFusedCtasPerSm = 6;
constexpr int kMaxFused = 104;
constexpr int64_t kStripRows = 16;          // longest strip (compact rows); shorter when a launch has few
constexpr int64_t kMaxFusedCols = 8192;     // compact columns (shared memory: 24 B per column)
constexpr int64_t kDefaultWaitIters = 1 << 22;

constexpr int kMaxDevices = 64;

// n / d for 32-bit unsigned n by a divisor fixed per tensor: multiply by a
// precomputed magic number (Granlund-Montgomery / Hacker's Delight 10-1,
// the round-up variant with a 33-bit add), set up on the host.
struct FastDiv {
    uint32_t d, m, l;
};

__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv &f) {
    const uint32_t t = __umulhi(n, f.m);
    return (uint32_t)(((uint64_t)t + n) >> f.l);
}

struct FusedDesc {
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
    float *m_out;
    float *v_out;
    int64_t H, W, band;
    int64_t halo_off;  // float offset of this tensor's published rows in the halo area
    int32_t h, w, B, L;
    FastDiv div_B;     // cell -> quant block
    FastDiv div_w;     // cell -> compact row
    int32_t kind;
    smo_hyper hp;
};

struct FusedBatch {
    int32_t n;
    int64_t strip_start[kMaxFused + 1];
    FusedDesc d[kMaxFused];
};
static_assert(sizeof(FusedBatch) < 30000, "kernel parameter batch must stay below 32 KB");

// ---------------------------------------------------------------- memory helpers

// One window row: KW consecutive elements of type T (float, __nv_bfloat16,
// __half) as fp32 values, with one or two vector accesses of KW * sizeof(T)
// bytes (fused_takes checks the alignment).  Cache hints: streaming for the
// gradient (kGrad), cached for phase 1's parameter read (the next cell was
// prefetched into L1, and the row is re-read from L2 one pipeline step later),
// last use for phase 2's.
enum { kGrad = 0, kParam = 1, kParamLast = 2 };

template <int HINT, class V>
__device__ __forceinline__ V ld_hint(const V *q) {
    if constexpr (HINT == kGrad) return __ldcs(q);
    else if constexpr (HINT == kParam) return __ldca(q);
    else return __ldlu(q);
}

// the two 16-bit elements of a 32-bit word (low one first) as fp32
template <class T>
__device__ __forceinline__ float2 widen16x2(uint32_t w) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    else
        return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}

// two fp32 values that are values of T (rounded already) as one word of T
template <class T>
__device__ __forceinline__ uint32_t narrow16x2(float lo, float hi) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t *>(&v);
    } else {
        const __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<const uint32_t *>(&v);
    }
}

template <class T, int KW, int HINT>
__device__ __forceinline__ void load_row(const T *ptr, float (&v)[KW]) {
    if constexpr (std::is_same<T, float>::value) {
        if constexpr (KW % 4 == 0) {
#pragma unroll
            for (int k = 0; k < KW / 4; k++) {
                const float4 t = ld_hint<HINT>(reinterpret_cast<const float4 *>(ptr) + k);
                v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
            }
        } else {
            static_assert(KW == 2, "window width");
            const float2 t = ld_hint<HINT>(reinterpret_cast<const float2 *>(ptr));
            v[0] = t.x; v[1] = t.y;
        }
    } else {
        uint32_t w[KW / 2];
        if constexpr (KW == 8) {
            const uint4 t = ld_hint<HINT>(reinterpret_cast<const uint4 *>(ptr));
            w[0] = t.x; w[1] = t.y; w[2] = t.z; w[3] = t.w;
        } else if constexpr (KW == 4) {
            const uint2 t = ld_hint<HINT>(reinterpret_cast<const uint2 *>(ptr));
            w[0] = t.x; w[1] = t.y;
        } else {
            static_assert(KW == 2, "window width");
            w[0] = ld_hint<HINT>(reinterpret_cast<const unsigned int *>(ptr));
        }
#pragma unroll
        for (int k = 0; k < KW / 2; k++) {
            const float2 x = widen16x2<T>(w[k]);
            v[2 * k] = x.x;
            v[2 * k + 1] = x.y;
        }
    }
}

template <class T, int KW>
__device__ __forceinline__ void store_param_row(T *ptr, const float (&v)[KW]) {
    if constexpr (std::is_same<T, float>::value) {
        if constexpr (KW % 4 == 0) {
#pragma unroll
            for (int k = 0; k < KW / 4; k++)
                __stcs(reinterpret_cast<float4 *>(ptr) + k,
                       make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]));
        } else {
            __stcs(reinterpret_cast<float2 *>(ptr), make_float2(v[0], v[1]));
        }
    } else {
        uint32_t w[KW / 2];
#pragma unroll
        for (int k = 0; k < KW / 2; k++) w[k] = narrow16x2<T>(v[2 * k], v[2 * k + 1]);
        if constexpr (KW == 8) __stcs(reinterpret_cast<uint4 *>(ptr), make_uint4(w[0], w[1], w[2], w[3]));
        else if constexpr (KW == 4) __stcs(reinterpret_cast<uint2 *>(ptr), make_uint2(w[0], w[1]));
        else __stcs(reinterpret_cast<unsigned int *>(ptr), w[0]);
    }
}

__device__ __forceinline__ void store_release(unsigned int *flag, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

__device__ __forceinline__ bool bounded_wait_eq(const unsigned int *flag, unsigned int target, int64_t max_iters,
                                                const unsigned int *error_word) {
    for (int64_t it = 0; it <= max_iters; it++) {
        unsigned int v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v == target) return true;
        if ((it & 255) == 255 && *(volatile const unsigned int *)error_word) return false;  // someone failed
        if (it >= 32) __nanosleep(it < 4096 ? 64 : 256);
    }
    return false;
}

__device__ __forceinline__ void report_error(WsHeader *hdr, unsigned int code, unsigned int where) {
    if (atomicCAS(&hdr->error, 0u, code) == 0u) hdr->error_where = where;
}

// ---------------------------------------------------------------- packed arithmetic
//
// The m and v channels see the same weights everywhere (EMA, width pass,
// height pass), so each (m, v) pair travels as one float2 and is computed with
// Blackwell's packed fp32x2 instructions; every lane is an ordinary correctly
// rounded fp32 operation, so results are bit-identical to the scalar sequence.

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 splat(float a) { return make_float2(a, a); }

// both lanes rounded to the storage type T (the identity for float): for
// half-precision tensors every op of the reference rounds its fp32 result once
// (one paired conversion, round to nearest even, and back)
template <class T>
__device__ __forceinline__ float2 rd2(float2 x) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat1622float2(__float22bfloat162_rn(x));
    else if constexpr (std::is_same<T, __half>::value) return __half22float2(__float22half2_rn(x));
    else return x;
}

// x / c with r = RN(1/c) for a finite c > 0: Markstein's correction
// (q0 = RN(x r), rem = x - q0 c exactly by fma, q = RN(q0 + rem r)) returns the
// correctly rounded quotient whenever x and the quotient are normal numbers
// (Markstein 1990; Muller et al., Handbook of Floating-Point Arithmetic, the
// correction step of reciprocal-based division).  Callers keep to that range
// or only use results for which a last-bit difference cannot matter.  x = +-inf
// gives +-inf (x / c for finite c > 0) and NaN stays NaN; no IEEE division is
// evaluated on any path.
__device__ __forceinline__ float div_rcp(float x, float c, float r) {
    const float q0 = __fmul_rn(x, r);
    const float rem = __fmaf_rn(q0, -c, x);
    const float q = __fmaf_rn(rem, r, q0);
    return fabsf(x) == __int_as_float(0x7f800000) ? x : q;
}

// the same for a pair, with per-lane constants (c.x, c.y) and reciprocals
__device__ __forceinline__ float2 div_rcp2(float2 x, float2 c, float2 r) {
    const float2 q0 = __fmul2_rn(x, r);
    const float2 rem = __ffma2_rn(q0, f2(-c.x, -c.y), x);
    const float2 q = __ffma2_rn(rem, r, q0);
    const float inf = __int_as_float(0x7f800000);
    return f2(fabsf(x.x) == inf ? x.x : q.x, fabsf(x.y) == inf ? x.y : q.y);
}

// The Adam write of two neighbouring elements (spatial_8bit.py:293-297):
// p + ((-lr/bc1) * m) / (sqrt(v)/sqrt(bc2) + eps).  sqrt(v) is 0, normal, +inf
// or NaN and sqrt(bc2) is in (0, 1], so the divide-by-constant stays normal.
struct AdamK {
    float2 sbc2, neg_sbc2, rcp_sbc2, eps, ns;
    bool fast;  // eps >= 2^-27: the denominator is >= 2^-27 (or not finite)
};

template <class T>
__device__ __forceinline__ float2 adam_write2(float2 p, float2 m, float2 v, const AdamK &k) {
    const float2 sv = rd2<T>(f2(__fsqrt_rn(v.x), __fsqrt_rn(v.y)));
    const float2 d = rd2<T>(__fadd2_rn(rd2<T>(div_rcp2(sv, k.sbc2, k.rcp_sbc2)), k.eps));
    const float2 a = __fmul2_rn(k.ns, m);
    return rd2<T>(__fadd2_rn(p, f2(__fdiv_rn(a.x, d.x), __fdiv_rn(a.y, d.y))));
}

// The same write with FMA-only arithmetic (sqrt2_markstein, Markstein's
// division by sqrt(bc2) and div2_markstein).  Returns false unless v >= 2^-100
// and |q0| is in [2^-76, 2^100] in both lanes, the ranges where every step is
// exact (zero, tiny, non-finite and NaN inputs all fail; so does a
// denominator that rounded to zero in T); the caller then redoes the pair
// with adam_write2.
template <class T>
__device__ __forceinline__ bool adam_write2_fast(float2 p, float2 m, float2 v, const AdamK &k, float2 &out) {
    const float2 sv = rd2<T>(sqrt2_markstein(v));
    const float2 t0 = __fmul2_rn(sv, k.rcp_sbc2);
    const float2 d = rd2<T>(__fadd2_rn(rd2<T>(__ffma2_rn(__ffma2_rn(t0, k.neg_sbc2, sv), k.rcp_sbc2, t0)), k.eps));
    const float2 a = __fmul2_rn(k.ns, m);
    float2 q0;
    const float2 q = div2_markstein(a, d, rcp2_newton(d), q0);
    out = rd2<T>(__fadd2_rn(p, q));
    const float lo = nan_min(__fmul_rn(nan_min(v.x, v.y), 0x1p24f), nan_min(fabsf(q0.x), fabsf(q0.y)));
    const float hi = nan_max(fabsf(q0.x), fabsf(q0.y));
    return lo >= 0x1p-76f && hi <= 0x1p100f;
}

// codes * (scales / 127) for an (m, v) pair; the block scales are clamped to
// >= 1e-12 in fp32 and bf16, so scale / 127 is normal (fp16 rounds 1e-12 to
// 0: 0 / 127 is 0 either way)
constexpr float kRcp127 = 0x1.020408p-7f;  // RN(1/127)
template <class T>
__device__ __forceinline__ float2 dequant2(int8_t qm, int8_t qv, float sm, float sv) {
    const float2 t = rd2<T>(div_rcp2(f2(sm, sv), splat(127.0f), splat(kRcp127)));
    return rd2<T>(__fmul2_rn(f2((float)qm, (float)qv), t));
}

// round(x / s * 127) with the dead-zone lift and clamp (spatial_8bit.py:97-106),
// given rs = RN(1/s).  A quotient too small for Markstein's bound is far below
// the first rounding threshold 0.5/127, so the code is the same either way.  A
// non-finite block scale comes from non-finite moments: x / inf is a signed
// zero for finite x and NaN for x = +-inf; x / NaN is NaN (stored as code 0).
template <class T>
__device__ __forceinline__ int8_t quantize_rc(float x, float s, float rs) {
    const float inf = __int_as_float(0x7f800000);
    float q = div_rcp(x, s, rs);
    if (s == inf) q = fabsf(x) == inf ? __int_as_float(0x7fffffff) : copysignf(0.0f, x);
    if (s != s) q = s;
    float r = rintf(rd<T>(__fmul_rn(rd<T>(q), 127.0f)));
    if (r == 0.0f && x != 0.0f && x == x) r = x > 0.0f ? 1.0f : -1.0f;
    r = r > 127.0f ? 127.0f : r;
    r = r < -127.0f ? -127.0f : r;
    return (r == r) ? (int8_t)(int)r : (int8_t)0;
}

// ---------------------------------------------------------------- phases

// (sum x, sum x*x) of one KH x KW window in row-major order from +0, times
// 1/(KH*KW) (a power of two: the same value as avg_pool2d's division)
// (for T = bf16 / fp16: x and x*x rounded to T, the means too; wd arrives
// rounded to T)
template <class T, int KH, int KW, bool WD>
__device__ __forceinline__ float2 pool_cell(const float (&gv)[KH][KW], const float (&pv)[KH][KW], float wd) {
    float2 acc = f2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < KH; i++) {
#pragma unroll
        for (int k = 0; k < KW; k += 2) {
            // two neighbouring elements at a time (paired conversions); the
            // sums still take the elements one by one, in row-major order
            const float2 x = WD ? rd2<T>(__ffma2_rn(splat(wd), f2(pv[i][k], pv[i][k + 1]), f2(gv[i][k], gv[i][k + 1])))
                                : f2(gv[i][k], gv[i][k + 1]);
            const float2 xx = rd2<T>(__fmul2_rn(x, x));
            acc = __fadd2_rn(acc, f2(x.x, xx.x));
            acc = __fadd2_rn(acc, f2(x.y, xx.y));
        }
    }
    constexpr float inv = 1.0f / (KH * KW);
    return rd2<T>(__fmul2_rn(acc, splat(inv)));
}

// The old moments of a cell as loaded (codes and scales, or the fp32-kind
// moments).  Phase 1 issues these loads together with the cell's g and p
// loads, so that all of a cell's DRAM reads are in flight at once (4 % faster
// on rows of 384 cells than loading them after the pooling).
struct OldCell {
    int qm, qv;
    float a, b;
};

template <class T>
__device__ __forceinline__ OldCell load_old(const FusedDesc &d, uint32_t cell) {
    OldCell o;
    if (d.kind == SMO_KIND_POOLED8) {
        const uint32_t bl = fast_div(cell, d.div_B);
        o.qm = d.mq_in[cell];
        o.qv = d.vq_in[cell];
        o.a = ld<T>((const T *)d.ms_in + bl);
        o.b = ld<T>((const T *)d.vs_in + bl);
    } else {
        o.qm = o.qv = 0;
        o.a = ld<T>((const T *)d.m_in + cell);
        o.b = ld<T>((const T *)d.v_in + cell);
    }
    return o;
}

// dequant of the old moments, EMA, post-EMA pair into the ring row (the
// ring holds fp32 values; for T = bf16 / fp16 they are values of T)
template <class T>
__device__ __forceinline__ void ema_cell(const FusedDesc &d, uint32_t cell, const OldCell &o, float2 pooled,
                                         float2 *row, int j, bool own) {
    const smo_hyper &hp = d.hp;
    float2 mv = d.kind == SMO_KIND_POOLED8 ? dequant2<T>((int8_t)o.qm, (int8_t)o.qv, o.a, o.b) : f2(o.a, o.b);
    // m.mul_(beta).add_(u, alpha=1-beta): alpha rounded to T, each op rounded
    mv = rd2<T>(__ffma2_rn(rd2<T>(f2(hp.omb1, hp.omb2)), pooled, rd2<T>(__fmul2_rn(mv, f2(hp.beta1, hp.beta2)))));
    row[j] = mv;
    if (own && d.kind == SMO_KIND_POOLED32) {
        st<T>((T *)d.m_out + cell, mv.x);
        st<T>((T *)d.v_out + cell, mv.y);
    }
}

// Phase 1 of compact row c: post-EMA (m, v) into `row` (shared memory).
// `own` rows also write the fp32 state (POOLED32); look-ahead rows only read.
// CELLS cells per thread per iteration keep CELLS*KH*KW*2 loads in flight.
template <class T, int KH, int KW, int CELLS, int NT, bool WD>
__device__ __forceinline__ void phase1_wd(const FusedDesc &d, int c, float2 *row, bool own) {
    const int w = d.w;
    const int64_t W = d.W;
    const T *gb = (const T *)d.g + (int64_t)c * KH * W;
    const T *pb = (const T *)d.p + (int64_t)c * KH * W;
    const uint32_t cell0 = (uint32_t)c * (uint32_t)w;
    const float wd = rd<T>(d.hp.weight_decay);  // add(p, alpha=wd): alpha in the tensor's dtype
    for (int j0 = threadIdx.x; j0 < w; j0 += CELLS * NT) {
        float gv[CELLS][KH][KW], pv[CELLS][KH][KW];
        OldCell old[CELLS];
#pragma unroll
        for (int u = 0; u < CELLS; u++) {
            const int j = j0 + u * NT;
            if (u == 0 || j < w) {
#pragma unroll
                for (int i = 0; i < KH; i++) load_row<T, KW, kGrad>(gb + i * W + (int64_t)j * KW, gv[u][i]);
                if (WD) {
#pragma unroll
                    for (int i = 0; i < KH; i++) load_row<T, KW, kParam>(pb + i * W + (int64_t)j * KW, pv[u][i]);
                }
                old[u] = load_old<T>(d, cell0 + j);
            }
        }
        {
            // while this cell is summed, pull the thread's next cell of the row
            // into L1 (one lane of eight covers a 128-byte line)
            const int jn = j0 + CELLS * NT;
            if (jn < w && (threadIdx.x & 7) == 0) {
#pragma unroll
                for (int i = 0; i < KH; i++) {
                    asm volatile("prefetch.global.L1 [%0];" ::"l"(gb + i * W + (int64_t)jn * KW));
                    if (WD) asm volatile("prefetch.global.L1 [%0];" ::"l"(pb + i * W + (int64_t)jn * KW));
                }
            }
        }
#pragma unroll
        for (int u = 0; u < CELLS; u++) {
            const int j = j0 + u * NT;
            if (u == 0 || j < w)
                ema_cell<T>(d, cell0 + j, old[u], pool_cell<T, KH, KW, WD>(gv[u], pv[u], wd), row, j, own);
        }
    }
}

template <class T, int KH, int KW, int CELLS, int NT>
__device__ __forceinline__ void phase1(const FusedDesc &d, int c, float2 *row, bool own) {
    if (d.hp.wd_on) phase1_wd<T, KH, KW, CELLS, NT, true>(d, c, row, own);
    else phase1_wd<T, KH, KW, CELLS, NT, false>(d, c, row, own);
}

// round(x / s * 127) with the dead-zone lift for a finite block scale
// 0 < s <= 2^126 (then |x| <= s, the quotient is at most 1 and no clamp or
// special case is needed); rs = RN(1/s)
template <class T>
__device__ __forceinline__ int8_t quantize_finite(float x, float s, float rs) {
    const float q0 = __fmul_rn(x, rs);
    const float q = __fmaf_rn(__fmaf_rn(q0, -s, x), rs, q0);
    float r = rintf(rd<T>(__fmul_rn(rd<T>(q), 127.0f)));
    const float lift = x != 0.0f ? copysignf(1.0f, x) : 0.0f;
    r = r == 0.0f ? lift : r;
    return (int8_t)__float2int_rn(r);
}

// Requantise the int8 blocks that START in compact row c, for the bottom-up
// row order: a block that runs on into row c+1 (q_block <= w, so at most one
// more row) finds that row already in the ring (Rn).  Strips start at rows
// where blocks realign, so no block runs past a strip's last row.
template <class T, int NT>
__device__ __forceinline__ void requant_row_up(const FusedDesc &d, int c, const float2 *Rc, const float2 *Rn) {
    const uint32_t w = (uint32_t)d.w, B = (uint32_t)d.B, C = (uint32_t)d.h * w;
    const uint32_t rowbase = (uint32_t)c * w, rowend = rowbase + w;
    const uint32_t b_lo = fast_div(rowbase + B - 1u, d.div_B);
    const uint32_t b_hi = fast_div(rowend + B - 1u, d.div_B);  // the last row also takes the zero-padded block
    const bool aligned = (w % B) == 0;                          // blocks never leave the row
    const int lane = threadIdx.x & 31;
    for (uint32_t b = b_lo + (threadIdx.x >> 5); b < b_hi; b += NT / 32) {
        float am = 0.0f, av = 0.0f;
        for (uint32_t k = lane; k < B; k += 32) {
            const uint32_t cell = b * B + k;
            if (cell >= C) break;
            const float2 mv = (aligned || cell < rowend) ? Rc[cell - rowbase] : Rn[cell - rowend];
            am = absmax_acc(am, mv.x);
            av = absmax_acc(av, mv.y);
        }
        const float sm = block_scale<T>(warp_absmax(am)), sv = block_scale<T>(warp_absmax(av));
        const float rm = __frcp_rn(sm), rv = __frcp_rn(sv);
        // uniform across the warp; false for NaN, and for the zero scale of an
        // all-zero fp16 block (fp32 and bf16 scales are >= 1e-12)
        const bool finite = sm <= 0x1p126f && sv <= 0x1p126f && sm > 0.0f && sv > 0.0f;
        for (uint32_t k = lane; k < B; k += 32) {
            const uint32_t cell = b * B + k;
            float2 mv = f2(0.0f, 0.0f);
            if (cell < C) mv = (aligned || cell < rowend) ? Rc[cell - rowbase] : Rn[cell - rowend];
            if (finite) {
                d.mq_out[cell] = quantize_finite<T>(mv.x, sm, rm);
                d.vq_out[cell] = quantize_finite<T>(mv.y, sv, rv);
            } else {
                d.mq_out[cell] = quantize_rc<T>(mv.x, sm, rm);
                d.vq_out[cell] = quantize_rc<T>(mv.y, sv, rv);
            }
        }
        if (lane == 0) {
            st<T>((T *)d.ms_out + b, sm);
            st<T>((T *)d.vs_out + b, sv);
        }
    }
}

struct RowCo {
    int s0, s1;  // ring-relative rows (0: c-1, 1: c, 2: c+1)
    float l0, l1;
};

// Row weights of the KH output rows of compact row c (threads 0..KH-1).
// This is row_coef (smo_common.cuh) specialised to exact KH-row windows:
// output row c*KH + i lies in compact row c, so the band of a low_peak tensor
// is (c / band) * band without 64-bit divisions, and the interpolation scale
// n / (n*KH) of a band (or h / H of the whole tensor) is exactly 1/KH because
// fused_takes keeps H below 2^24, where both operands are exact floats.  The
// remaining float operations are row_coef's, in its order.
template <int KH>
__device__ __forceinline__ void compute_rowco(const FusedDesc &d, int c, RowCo *dst) {
    if (threadIdx.x < KH) {
        const int i = threadIdx.x;
        int a = 0, n = d.h;  // rows [a, a + n) are interpolated together
        if (d.band > 0) {
            const int band = (int)d.band;
            const int s0 = (c / band) * band;
            const int s1 = s0 + band < d.h ? s0 + band : d.h;
            a = s0 > 0 ? s0 - 1 : 0;
            n = (s1 + 1 < d.h ? s1 + 1 : d.h) - a;
        }
        const int o = (c - a) * KH + i;  // output row in the band's coordinates
        float real = __fmaf_rn(1.0f / KH, __fadd_rn((float)o, 0.5f), -0.5f);
        real = real < 0.0f ? 0.0f : real;
        int i0 = (int)floorf(real);
        i0 = i0 > n - 1 ? n - 1 : i0;
        float l1 = __fsub_rn(real, (float)i0);
        l1 = l1 < 0.0f ? 0.0f : (l1 > 1.0f ? 1.0f : l1);
        const int i1 = i0 + (i0 < n - 1 ? 1 : 0);
        RowCo r;
        r.s0 = i0 + a - (c - 1);
        r.s1 = i1 + a - (c - 1);
        r.l0 = __fsub_rn(1.0f, l1);
        r.l1 = l1;
        dst[i] = r;
    }
}

// Width-pass weights of output column t of a KW-wide window (power-of-two KW):
// exactly torch's src = (q + 0.5)/KW - 0.5 split into floor and fraction.
template <int KW>
__device__ __forceinline__ float col_l1(int t) {
    return (t + 0.5f) / KW + (t < KW / 2 ? 0.5f : -0.5f);
}

// Width pass of the three compact rows at column j: the left half of the
// window interpolates columns (j-1, j), the right half (j, j+1), clamped at
// the edges exactly as torch's index/lambda computation does
template <int KW>
__device__ __forceinline__ void width_pass3(const float2 *const R[3], int j, int w, float2 (&h)[3][KW]) {
    const int jr = j + 1 < w ? j + 1 : w - 1;
    const int la = j > 0 ? j - 1 : 0;
#pragma unroll
    for (int s = 0; s < 3; s++) {
        const float2 left = R[s][la], mid = R[s][j], right = R[s][jr];
        const float2 x = j > 0 ? mid : right;
#pragma unroll
        for (int t = 0; t < KW; t++) {
            if (t < KW / 2) {
                const float l1 = j > 0 ? col_l1<KW>(t) : 0.0f;
                const float l0 = j > 0 ? 1.0f - col_l1<KW>(t) : 1.0f;
                h[s][t] = __ffma2_rn(left, splat(l0), __fmul2_rn(x, splat(l1)));
            } else {
                h[s][t] = __ffma2_rn(mid, splat(1.0f - col_l1<KW>(t)), __fmul2_rn(right, splat(col_l1<KW>(t))));
            }
        }
    }
}

// The same width pass for a cell with j > 0 (every cell but a row's first):
// no edge selects.
template <int KW>
__device__ __forceinline__ void width_pass3_inner(const float2 *const R[3], int j, int w, float2 (&h)[3][KW]) {
    const int jr = j + 1 < w ? j + 1 : w - 1;
#pragma unroll
    for (int s = 0; s < 3; s++) {
        const float2 left = R[s][j - 1], mid = R[s][j], right = R[s][jr];
#pragma unroll
        for (int t = 0; t < KW; t++) {
            if (t < KW / 2)
                h[s][t] = __ffma2_rn(left, splat(1.0f - col_l1<KW>(t)), __fmul2_rn(mid, splat(col_l1<KW>(t))));
            else
                h[s][t] = __ffma2_rn(mid, splat(1.0f - col_l1<KW>(t)), __fmul2_rn(right, splat(col_l1<KW>(t))));
        }
    }
}

// Rows of cell j (bits of `rows`) whose fast Adam write failed its range
// check: recomputed with the IEEE operations from the untouched parameters.
template <class T, int KH, int KW>
__device__ __noinline__ void phase2_fixup(const FusedDesc &d, int c, int j, const float2 *const R[3],
                                          const RowCo *rowco, const AdamK &ak, unsigned rows) {
    const int64_t W = d.W;
    float2 h[3][KW];
    width_pass3<KW>(R, j, d.w, h);
    for (int i = 0; i < KH; i++) {
        if (!((rows >> i) & 1u)) continue;
        T *prow = (T *)d.p + ((int64_t)c * KH + i) * W + (int64_t)j * KW;
        float pv[KW];
        load_row<T, KW, kParamLast>(prow, pv);
        const RowCo rc = rowco[i];
#pragma unroll
        for (int t = 0; t < KW; t += 2) {
            float2 m2[2];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const float2 a = rc.s0 == 0 ? h[0][t + e] : h[1][t + e];
                const float2 b = rc.s1 == 1 ? h[1][t + e] : h[2][t + e];
                m2[e] = rd2<T>(__ffma2_rn(a, splat(rc.l0), __fmul2_rn(b, splat(rc.l1))));
            }
            const float2 pn = adam_write2<T>(f2(pv[t], pv[t + 1]), f2(m2[0].x, m2[1].x),
                                             f2(clamp_min0(m2[0].y), clamp_min0(m2[1].y)), ak);
            pv[t] = pn.x;
            pv[t + 1] = pn.y;
        }
        store_param_row<T, KW>(prow, pv);
    }
}

// Phase 2 of compact row c: the KH parameter rows, from the post-EMA rows
// c-1 (R[0]), c (R[1]), c+1 (R[2]) in shared memory (an absent neighbour row
// is passed as row c and never weighted).  Row weights come from `rowco`; for
// an INTERIOR row (0 < c < h-1) they are compile-time constants instead:
// output row i interpolates rows (c-1, c) with weight row_l1(i) on row c for
// i < KH/2 and rows (c, c+1) for i >= KH/2, which is what compute_rowco
// yields there, exactly (also inside low_peak bands, whose one-row halo keeps
// interior rows interior).  Every element takes the FMA-only Adam write; a row
// whose range check fails is not stored and goes to phase2_fixup.
template <class T, int KH, int KW, int NT, bool INTERIOR>
__device__ __forceinline__ void phase2(const FusedDesc &d, int c, const float2 *const R[3], const RowCo *rowco,
                                       const AdamK &ak) {
    const int w = d.w;
    const int64_t W = d.W;
    for (int j = threadIdx.x; j < w; j += NT) {
        T *pbase = (T *)d.p + (int64_t)c * KH * W + (int64_t)j * KW;
        float pv[KH][KW];
#pragma unroll
        for (int i = 0; i < KH; i++) load_row<T, KW, kParamLast>(pbase + i * W, pv[i]);
        float2 h[3][KW];
        if (j > 0) width_pass3_inner<KW>(R, j, w, h);
        else width_pass3<KW>(R, j, w, h);
        unsigned fail = 0;
#pragma unroll
        for (int i = 0; i < KH; i++) {
            float2 mh[KW];
            if constexpr (INTERIOR) {
                const bool upper = i < KH / 2;  // resolved at compile time once the loop is unrolled
#pragma unroll
                for (int t = 0; t < KW; t++)
                    mh[t] = rd2<T>(__ffma2_rn(upper ? h[0][t] : h[1][t], splat(1.0f - col_l1<KH>(i)),
                                              __fmul2_rn(upper ? h[1][t] : h[2][t], splat(col_l1<KH>(i)))));
            } else {
                const RowCo rc = rowco[i];
                const bool lo0 = rc.s0 == 0, lo1 = rc.s1 == 1;  // uniform across the CTA
#pragma unroll
                for (int t = 0; t < KW; t++) {
                    const float2 a = lo0 ? h[0][t] : h[1][t];
                    const float2 b = lo1 ? h[1][t] : h[2][t];
                    mh[t] = rd2<T>(__ffma2_rn(a, splat(rc.l0), __fmul2_rn(b, splat(rc.l1))));
                }
            }
            bool ok = ak.fast;
            float pn[KW];
#pragma unroll
            for (int t = 0; t < KW; t += 2) {
                // clamp(v, min=0) as a NaN-propagating max: it differs from
                // clamp_min0 only by giving +0 for -0, and a zero v always
                // fails the fast path's range check, whose IEEE fix-up then
                // clamps with clamp_min0 itself
                float2 o;
                ok &= adam_write2_fast<T>(f2(pv[i][t], pv[i][t + 1]), f2(mh[t].x, mh[t + 1].x),
                                          f2(nan_max(mh[t].y, 0.0f), nan_max(mh[t + 1].y, 0.0f)), ak, o);
                pn[t] = o.x;
                pn[t + 1] = o.y;
            }
            if (ok) store_param_row<T, KW>(pbase + i * W, pn);
            else fail |= 1u << i;
        }
        if (fail) phase2_fixup<T, KH, KW>(d, c, j, R, rowco, ak, fail);
    }
}

template <class T, int KH, int KW, int NT>
__device__ __forceinline__ void phase2_row(const FusedDesc &d, int c, const float2 *const R[3], const RowCo *rowco,
                                           const AdamK &ak) {
    if (c > 0 && c < d.h - 1) phase2<T, KH, KW, NT, true>(d, c, R, rowco, ak);
    else phase2<T, KH, KW, NT, false>(d, c, R, rowco, ak);
}

// Barrier of the NT threads that run the row pipeline (named barrier 1).
template <int NT>
__device__ __forceinline__ void cta_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}

// One strip of compact rows [c0, c1), processed bottom-up: phase 1 of row r
// (from the look-ahead row c1, the next strip's first row, when it exists,
// down to c0), each followed by phase 2 of row r+1, which then has all three
// of its rows in the ring.  The look-ahead row is read first and the strip's
// bottom row c1-1 is published for the next strip right after it, so the
// flag the next strip waits on is set at the start of this strip's work;
// the strip's top row c0 needs the previous strip's published bottom row and
// is written last, after a bounded acquire wait that has normally long been
// satisfied.  Row c0 is also the look-ahead row of the previous strip, whose
// read of its OLD parameters is covered by the same flag: it is written only
// after the wait.
template <class T, int KH, int KW, int CELLS, int NT>
__device__ void process_strip(const FusedDesc &d, int sidx, int64_t gstrip, unsigned int epoch, float2 *ring,
                              RowCo (*rowco)[KH], WsHeader *hdr, unsigned int *flags, float *halo,
                              int64_t wait_iters, unsigned int wait_skew) {
    const int w = d.w, h = d.h;
    const int c0 = sidx * d.L;
    const int c1 = c0 + d.L < h ? c0 + d.L : h;
    const int top = c1 < h ? c1 : c1 - 1;  // first phase-1 row
    const bool q8 = (d.kind == SMO_KIND_POOLED8);
    AdamK ak;
    ak.sbc2 = splat(d.hp.sqrt_bc2);
    ak.neg_sbc2 = splat(-d.hp.sqrt_bc2);
    ak.rcp_sbc2 = splat(__frcp_rn(d.hp.sqrt_bc2));
    ak.eps = splat(d.hp.eps);
    ak.ns = splat(d.hp.neg_step);
    ak.fast = d.hp.eps >= 0x1p-27f;
    auto RR = [&](int c) { return ring + (c % 3) * w; };
    float2 *pub = reinterpret_cast<float2 *>(halo + d.halo_off) + (int64_t)sidx * w;

    for (int r = top; r >= c0; r--) {
        const bool do2 = r + 1 < c1;  // phase 2 of row r+1 (an own row) in this iteration
        if (do2) compute_rowco<KH>(d, r + 1, rowco[(r + 1) & 1]);
        phase1<T, KH, KW, CELLS, NT>(d, r, RR(r), r < c1);
        cta_sync<NT>();
        if (r < c1) {
            if (q8) requant_row_up<T, NT>(d, r, RR(r), r + 1 < c1 ? RR(r + 1) : nullptr);
            if (r == c1 - 1 && c1 < h) {
                // publish the bottom row for the next strip, after the
                // look-ahead read of that strip's first row (previous iteration)
                const float2 *src = RR(r);
                for (int j = threadIdx.x; j < w; j += NT) __stcg(pub + j, src[j]);
                cta_sync<NT>();
                if (threadIdx.x == 0) {
                    __threadfence();
                    store_release(flags + gstrip, epoch);
                }
            }
        }
        if (do2) {
            const float2 *R[3] = {RR(r), RR(r + 1), r + 2 <= top ? RR(r + 2) : RR(r + 1)};
            phase2_row<T, KH, KW, NT>(d, r + 1, R, rowco[(r + 1) & 1], ak);
        }
        cta_sync<NT>();
    }

    // row c0: its upper neighbour is the previous strip's published bottom row
    __shared__ int s_ok;
    compute_rowco<KH>(d, c0, rowco[c0 & 1]);
    if (c0 > 0 && threadIdx.x == 0) {
        const bool ok = bounded_wait_eq(flags + gstrip - 1, epoch + wait_skew, wait_iters, &hdr->error);
        if (!ok) report_error(hdr, SMO_ERR_TIMEOUT, (unsigned int)gstrip);
        s_ok = ok;
    }
    cta_sync<NT>();
    if (c0 > 0) {
        // the ring slot of row c0-1 holds row c0+2, which is no longer needed
        const float2 *prev = pub - w;
        float2 *dst = RR(c0 - 1);
        const bool ok = s_ok;
        for (int j = threadIdx.x; j < w; j += NT) dst[j] = ok ? __ldcg(prev + j) : f2(0.0f, 0.0f);
        cta_sync<NT>();
    }
    const float2 *R[3] = {c0 > 0 ? RR(c0 - 1) : RR(c0), RR(c0), c0 + 1 <= top ? RR(c0 + 1) : RR(c0)};
    phase2_row<T, KH, KW, NT>(d, c0, R, rowco[c0 & 1], ak);
    cta_sync<NT>();
}

__device__ __forceinline__ int find_strip_tensor(const FusedBatch &b, int64_t s) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (b.strip_start[mid] <= s) lo = mid; else hi = mid - 1;
    }
    return lo;
}

template <class T, int KH, int KW, int CELLS, int NT, int MINB>
__global__ void __launch_bounds__(NT, MINB)
    fused_step_kernel(const __grid_constant__ FusedBatch b, WsHeader *hdr, unsigned int *flags, float *halo,
                      int64_t wait_iters, unsigned int wait_skew) {
    extern __shared__ float2 ring[];
    __shared__ RowCo rowco[2][KH];
    __shared__ int64_t s_strip;
    __shared__ unsigned int s_epoch;
    if (threadIdx.x == 0) s_epoch = *(volatile unsigned int *)&hdr->epoch + 1u;
    const int64_t total = b.strip_start[b.n];
    for (;;) {
        if (threadIdx.x == 0) s_strip = (int64_t)atomicAdd(&hdr->next_item, 1u);
        __syncthreads();
        const int64_t s = s_strip;
        const unsigned int epoch = s_epoch;
        __syncthreads();
        if (s >= total) break;
        const int t = find_strip_tensor(b, s);
        process_strip<T, KH, KW, CELLS, NT>(b.d[t], (int)(s - b.strip_start[t]), s, epoch, ring, rowco, hdr, flags,
                                            halo, wait_iters, wait_skew);
    }
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int prev = atomicAdd(&hdr->done_ctas, 1u);
        if (prev == gridDim.x - 1) {
            // last CTA out: reset the scheduler for the next launch, advance the epoch
            hdr->next_item = 0;
            hdr->done_ctas = 0;
            hdr->epoch = s_epoch;
            __threadfence();
        }
    }
}

// host helpers defined in smo_fused.cu
int pick_threads(const FusedBatch &b);
int current_device();
int device_sm_count();
unsigned int wait_skew();

// The kernel instance of a storage type, window shape and CTA width:
// 16-element windows take one cell per thread-iteration, smaller windows two;
// 128-, 192- and 384-thread CTAs run six, four and two per SM at 80
// registers, 256-thread CTAs four (one cell, 64 registers) or three (two
// cells, 80 registers).  Half-precision tensors have the 192- and 256-thread
// instances only (cta_width maps any other width to 192).
template <class T>
int cta_width(int nt) {
    if (std::is_same<T, float>::value) return nt == 128 || nt == 192 || nt == 384 ? nt : 256;
    return nt == 256 ? 256 : 192;
}

template <class T, int KH, int KW>
auto fused_kernel_for(int nt) {
    constexpr int kCells = KH * KW >= 16 ? 1 : 2;
    constexpr int kMinBlocks256 = kCells == 1 ? 4 : 3;
    if constexpr (std::is_same<T, float>::value) {
        switch (nt) {
            case 128: return fused_step_kernel<T, KH, KW, kCells, 128, 6>;
            case 192: return fused_step_kernel<T, KH, KW, kCells, 192, 4>;
            case 384: return fused_step_kernel<T, KH, KW, kCells, 384, 2>;
            default: return fused_step_kernel<T, KH, KW, kCells, 256, kMinBlocks256>;
        }
    } else {
        return nt == 256 ? fused_step_kernel<T, KH, KW, kCells, 256, kMinBlocks256>
                         : fused_step_kernel<T, KH, KW, kCells, 192, 4>;
    }
}

inline int kernel_cache_slot(int nt) { return nt == 384 ? 1 : nt == 192 ? 4 : nt == 128 ? 5 : 0; }

// The shared-memory attribute and the occupancy of a kernel instance are set
// and queried once per device and size (the attribute is a maximum, so a
// larger earlier setting covers smaller launches).
struct KernelCache {
    size_t smem_attr = 0, smem_occ = 0;
    int per_sm = 0;
};

template <class Kern>
int occupancy(Kern kern, KernelCache &c, int nt, size_t smem, int &per_sm) {
    cudaError_t e = cudaSuccess;
    if (smem > c.smem_attr) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (g_last_cuda_error = (int)e, SMO_ERR_CUDA);
        c.smem_attr = smem;
    }
    if (c.per_sm == 0 || c.smem_occ != smem) {
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c.per_sm, kern, nt, smem);
        if (e != cudaSuccess) return (c.per_sm = 0, g_last_cuda_error = (int)e, SMO_ERR_CUDA);
        c.smem_occ = smem;
    }
    per_sm = c.per_sm;
    return SMO_OK;
}

template <class T, int KH, int KW>
int launch_fused_group(FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
                              cudaStream_t stream) {
    static KernelCache cache[kMaxDevices][6];
    static std::mutex mu;
    const int dev = current_device();
    WsHeader *hdr = (WsHeader *)ws;
    unsigned int *flags = (unsigned int *)(ws + kWsHeader);
    float *halo = (float *)(ws + kWsHeader + flag_bytes);
    const int64_t strips = b.strip_start[b.n];
    size_t smem = 0;
    int nt = 0, per_sm = 0, st = SMO_OK;
    {
        std::lock_guard<std::mutex> lock(mu);
        KernelCache scratch;
        smem = (size_t)6 * max_w * sizeof(float);  // ring: 3 rows x (m, v)
        nt = cta_width<T>(pick_threads(b));
        st = occupancy(fused_kernel_for<T, KH, KW>(nt), dev >= 0 ? cache[dev][kernel_cache_slot(nt)] : scratch, nt,
                       smem, per_sm);
    }
    if (st != SMO_OK) return st;
    per_sm = per_sm < 1 ? 1 : (per_sm > kMaxFusedCtasPerSm ? kMaxFusedCtasPerSm : per_sm);
    int64_t grid = (int64_t)device_sm_count() * per_sm;
    grid = grid < strips ? grid : strips;
    fused_kernel_for<T, KH, KW>(nt)<<<(unsigned)grid, nt, smem, stream>>>(b, hdr, flags, halo, wait_limit(),
                                                                        wait_skew());
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    g_launches++;
    return SMO_OK;
}

// One launch of a window-shape group of storage type T (key: KH * 16 + KW).
template <class T>
int launch_fused_window(int key, FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
                        cudaStream_t stream) {
    switch (key) {
#define SMO_FUSED_CASE(KH, KW) \
    case KH * 16 + KW: return launch_fused_group<T, KH, KW>(b, max_w, halo_floats, ws, flag_bytes, stream);
        SMO_FUSED_CASE(2, 2) SMO_FUSED_CASE(2, 4) SMO_FUSED_CASE(2, 8)
        SMO_FUSED_CASE(4, 2) SMO_FUSED_CASE(4, 4) SMO_FUSED_CASE(4, 8)
        SMO_FUSED_CASE(8, 2) SMO_FUSED_CASE(8, 4) SMO_FUSED_CASE(8, 8)
#undef SMO_FUSED_CASE
        default: return SMO_ERR_INVALID;
    }
}

// the instances, one translation unit per storage type
int launch_fused_f32(int key, FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
                     cudaStream_t stream);
int launch_fused_bf16(int key, FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
                      cudaStream_t stream);
int launch_fused_f16(int key, FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
                     cudaStream_t stream);

}  // namespace smo
