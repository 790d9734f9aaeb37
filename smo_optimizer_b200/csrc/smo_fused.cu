// smo_fused.cu -- fused single-pass step for exact-window pooled tensors.
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
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "smo_common.cuh"
#include "smo_internal.cuh"

namespace smo {

constexpr int kMaxFusedCtasPerSm = 6;
constexpr int kMaxFused = 104;
constexpr int64_t kStripRows = 16;          // longest strip (compact rows); shorter when a launch has few
constexpr int64_t kMaxFusedCols = 8192;     // compact columns (shared memory: 24 B per column)
constexpr int64_t kDefaultWaitIters = 1 << 22;

// Poll limit of the inter-CTA waits (smo_set_wait_limit; negative = default)
static std::atomic<int64_t> g_wait_limit{-1};
// Diagnostic: waits look for a flag value that no strip publishes
// (smo_inject_wait_timeout), so each runs out its poll limit
static std::atomic<unsigned int> g_wait_skew{0};

int64_t wait_limit() {
    const int64_t v = g_wait_limit.load(std::memory_order_relaxed);
    return v < 0 ? kDefaultWaitIters : v;
}

int64_t set_wait_limit(int64_t polls) { return g_wait_limit.exchange(polls < 0 ? -1 : polls); }

int inject_wait_timeout(int on) { return (int)g_wait_skew.exchange(on ? 1u : 0u); }

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

template <int KW>
__device__ __forceinline__ void load_grad_row(const float *ptr, float (&v)[KW]) {
    if constexpr (KW % 4 == 0) {
#pragma unroll
        for (int k = 0; k < KW / 4; k++) {
            float4 t = __ldcs(reinterpret_cast<const float4 *>(ptr) + k);
            v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
        }
    } else {
        static_assert(KW == 2, "window width");
        float2 t = __ldcs(reinterpret_cast<const float2 *>(ptr));
        v[0] = t.x; v[1] = t.y;
    }
}

// parameter loads: cached (phase 1: the next cell was prefetched into L1, and
// the row is re-read from L2 one pipeline step later) or last use (phase 2)
template <int KW, bool kLastUse>
__device__ __forceinline__ void load_param_row(const float *ptr, float (&v)[KW]) {
    if constexpr (KW % 4 == 0) {
#pragma unroll
        for (int k = 0; k < KW / 4; k++) {
            const float4 *q = reinterpret_cast<const float4 *>(ptr) + k;
            float4 t = kLastUse ? __ldlu(q) : __ldca(q);
            v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
        }
    } else {
        const float2 *q = reinterpret_cast<const float2 *>(ptr);
        float2 t = kLastUse ? __ldlu(q) : __ldca(q);
        v[0] = t.x; v[1] = t.y;
    }
}

template <int KW>
__device__ __forceinline__ void store_param_row(float *ptr, const float (&v)[KW]) {
    if constexpr (KW % 4 == 0) {
#pragma unroll
        for (int k = 0; k < KW / 4; k++)
            __stcs(reinterpret_cast<float4 *>(ptr) + k, make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]));
    } else {
        __stcs(reinterpret_cast<float2 *>(ptr), make_float2(v[0], v[1]));
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

__device__ __forceinline__ float2 adam_write2(float2 p, float2 m, float2 v, const AdamK &k) {
    const float2 sv = f2(__fsqrt_rn(v.x), __fsqrt_rn(v.y));
    const float2 d = __fadd2_rn(div_rcp2(sv, k.sbc2, k.rcp_sbc2), k.eps);
    const float2 a = __fmul2_rn(k.ns, m);
    return __fadd2_rn(p, f2(__fdiv_rn(a.x, d.x), __fdiv_rn(a.y, d.y)));
}

// The same write with FMA-only arithmetic (sqrt2_markstein, Markstein's
// division by sqrt(bc2) and div2_markstein).  Returns false unless v >= 2^-100
// and |q0| is in [2^-76, 2^100] in both lanes, the ranges where every step is
// exact (zero, tiny, non-finite and NaN inputs all fail); the caller then
// redoes the pair with adam_write2.
__device__ __forceinline__ bool adam_write2_fast(float2 p, float2 m, float2 v, const AdamK &k, float2 &out) {
    const float2 sv = sqrt2_markstein(v);
    const float2 t0 = __fmul2_rn(sv, k.rcp_sbc2);
    const float2 d = __fadd2_rn(__ffma2_rn(__ffma2_rn(t0, k.neg_sbc2, sv), k.rcp_sbc2, t0), k.eps);
    const float2 a = __fmul2_rn(k.ns, m);
    float2 q0;
    const float2 q = div2_markstein(a, d, rcp2_newton(d), q0);
    out = __fadd2_rn(p, q);
    const float lo = nan_min(__fmul_rn(nan_min(v.x, v.y), 0x1p24f), nan_min(fabsf(q0.x), fabsf(q0.y)));
    const float hi = nan_max(fabsf(q0.x), fabsf(q0.y));
    return lo >= 0x1p-76f && hi <= 0x1p100f;
}

// codes * (scales / 127) for an (m, v) pair; scales >= 1e-12 (clamped block
// scales), so scale / 127 is normal
constexpr float kRcp127 = 0x1.020408p-7f;  // RN(1/127)
__device__ __forceinline__ float2 dequant2(int8_t qm, int8_t qv, float sm, float sv) {
    const float2 t = div_rcp2(f2(sm, sv), splat(127.0f), splat(kRcp127));
    return __fmul2_rn(f2((float)qm, (float)qv), t);
}

// round(x / s * 127) with the dead-zone lift and clamp (spatial_8bit.py:97-106),
// given rs = RN(1/s).  A quotient too small for Markstein's bound is far below
// the first rounding threshold 0.5/127, so the code is the same either way.  A
// non-finite block scale comes from non-finite moments: x / inf is a signed
// zero for finite x and NaN for x = +-inf; x / NaN is NaN (stored as code 0).
__device__ __forceinline__ int8_t quantize_rc(float x, float s, float rs) {
    const float inf = __int_as_float(0x7f800000);
    float q = div_rcp(x, s, rs);
    if (s == inf) q = fabsf(x) == inf ? __int_as_float(0x7fffffff) : copysignf(0.0f, x);
    if (s != s) q = s;
    float r = rintf(__fmul_rn(q, 127.0f));
    if (r == 0.0f && x != 0.0f && x == x) r = x > 0.0f ? 1.0f : -1.0f;
    r = r > 127.0f ? 127.0f : r;
    r = r < -127.0f ? -127.0f : r;
    return (r == r) ? (int8_t)(int)r : (int8_t)0;
}

// ---------------------------------------------------------------- phases

// (sum x, sum x*x) of one KH x KW window in row-major order from +0, times
// 1/(KH*KW) (a power of two: the same value as avg_pool2d's division)
template <int KH, int KW, bool WD>
__device__ __forceinline__ float2 pool_cell(const float (&gv)[KH][KW], const float (&pv)[KH][KW], float wd) {
    float2 acc = f2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < KH; i++) {
#pragma unroll
        for (int k = 0; k < KW; k++) {
            const float x = WD ? __fmaf_rn(wd, pv[i][k], gv[i][k]) : gv[i][k];
            acc = __fadd2_rn(acc, f2(x, __fmul_rn(x, x)));
        }
    }
    constexpr float inv = 1.0f / (KH * KW);
    return __fmul2_rn(acc, splat(inv));
}

// dequant of the old moments, EMA, post-EMA pair into the ring row
__device__ __forceinline__ void ema_cell(const FusedDesc &d, uint32_t cell, float2 pooled, float2 *row, int j,
                                         bool own) {
    const smo_hyper &hp = d.hp;
    float2 mv;
    if (d.kind == SMO_KIND_POOLED8) {
        const uint32_t b = fast_div(cell, d.div_B);
        mv = dequant2(d.mq_in[cell], d.vq_in[cell], d.ms_in[b], d.vs_in[b]);
    } else {
        mv = f2(d.m_in[cell], d.v_in[cell]);
    }
    mv = __ffma2_rn(f2(hp.omb1, hp.omb2), pooled, __fmul2_rn(mv, f2(hp.beta1, hp.beta2)));
    row[j] = mv;
    if (own && d.kind == SMO_KIND_POOLED32) {
        d.m_out[cell] = mv.x;
        d.v_out[cell] = mv.y;
    }
}

// Phase 1 of compact row c: post-EMA (m, v) into `row` (shared memory).
// `own` rows also write the fp32 state (POOLED32); look-ahead rows only read.
// CELLS cells per thread per iteration keep CELLS*KH*KW*2 loads in flight.
template <int KH, int KW, int CELLS, int NT, bool WD>
__device__ __forceinline__ void phase1_wd(const FusedDesc &d, int c, float2 *row, bool own) {
    const int w = d.w;
    const int64_t W = d.W;
    const float *gb = d.g + (int64_t)c * KH * W;
    const float *pb = d.p + (int64_t)c * KH * W;
    const uint32_t cell0 = (uint32_t)c * (uint32_t)w;
    const float wd = d.hp.weight_decay;
    for (int j0 = threadIdx.x; j0 < w; j0 += CELLS * NT) {
        float gv[CELLS][KH][KW], pv[CELLS][KH][KW];
#pragma unroll
        for (int u = 0; u < CELLS; u++) {
            const int j = j0 + u * NT;
            if (u == 0 || j < w) {
#pragma unroll
                for (int i = 0; i < KH; i++) load_grad_row<KW>(gb + i * W + (int64_t)j * KW, gv[u][i]);
                if (WD) {
#pragma unroll
                    for (int i = 0; i < KH; i++) load_param_row<KW, false>(pb + i * W + (int64_t)j * KW, pv[u][i]);
                }
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
            if (u == 0 || j < w) ema_cell(d, cell0 + j, pool_cell<KH, KW, WD>(gv[u], pv[u], wd), row, j, own);
        }
    }
}

template <int KH, int KW, int CELLS, int NT>
__device__ __forceinline__ void phase1(const FusedDesc &d, int c, float2 *row, bool own) {
    if (d.hp.wd_on) phase1_wd<KH, KW, CELLS, NT, true>(d, c, row, own);
    else phase1_wd<KH, KW, CELLS, NT, false>(d, c, row, own);
}

// round(x / s * 127) with the dead-zone lift for a finite block scale
// s <= 2^126 (then |x| <= s, the quotient is at most 1 and no clamp or
// special case is needed); rs = RN(1/s)
__device__ __forceinline__ int8_t quantize_finite(float x, float s, float rs) {
    const float q0 = __fmul_rn(x, rs);
    const float q = __fmaf_rn(__fmaf_rn(q0, -s, x), rs, q0);
    float r = rintf(__fmul_rn(q, 127.0f));
    const float lift = x != 0.0f ? copysignf(1.0f, x) : 0.0f;
    r = r == 0.0f ? lift : r;
    return (int8_t)__float2int_rn(r);
}

// Requantise the int8 blocks that compact row c completes.  A block spans at
// most two compact rows (q_block <= w), both still in the ring.
__device__ __forceinline__ void requant_block(const FusedDesc &d, uint32_t b, int c, const float2 *Rc,
                                              const float2 *Rp, bool aligned) {
    const uint32_t w = (uint32_t)d.w, B = (uint32_t)d.B, C = (uint32_t)d.h * w;
    const int lane = threadIdx.x & 31;
    const uint32_t rowbase = (uint32_t)c * w;
    float am = 0.0f, av = 0.0f;
    for (uint32_t k = lane; k < B; k += 32) {
        const uint32_t cell = b * B + k;
        if (cell >= C) break;
        const float2 mv = (aligned || cell >= rowbase) ? Rc[cell - rowbase] : Rp[cell + w - rowbase];
        am = absmax_acc(am, mv.x);
        av = absmax_acc(av, mv.y);
    }
    const float sm = block_scale(warp_absmax(am)), sv = block_scale(warp_absmax(av));
    const float rm = __frcp_rn(sm), rv = __frcp_rn(sv);
    const bool finite = sm <= 0x1p126f && sv <= 0x1p126f;  // uniform across the warp; false for NaN
    for (uint32_t k = lane; k < B; k += 32) {
        const uint32_t cell = b * B + k;
        float2 mv = f2(0.0f, 0.0f);
        if (cell < C) mv = (aligned || cell >= rowbase) ? Rc[cell - rowbase] : Rp[cell + w - rowbase];
        if (finite) {
            d.mq_out[cell] = quantize_finite(mv.x, sm, rm);
            d.vq_out[cell] = quantize_finite(mv.y, sv, rv);
        } else {
            d.mq_out[cell] = quantize_rc(mv.x, sm, rm);
            d.vq_out[cell] = quantize_rc(mv.y, sv, rv);
        }
    }
    if (lane == 0) {
        d.ms_out[b] = sm;
        d.vs_out[b] = sv;
    }
}

template <int NT>
__device__ __forceinline__ void requant_row(const FusedDesc &d, int c, const float2 *Rc, const float2 *Rp) {
    const uint32_t w = (uint32_t)d.w, B = (uint32_t)d.B, C = (uint32_t)d.h * w;
    const uint32_t b_lo = fast_div((uint32_t)c * w, d.div_B);
    uint32_t b_hi = fast_div(((uint32_t)c + 1u) * w, d.div_B);
    if (c == d.h - 1 && C % B != 0) b_hi = C / B + 1;  // the zero-padded last block
    const bool aligned = (w % B) == 0;                  // blocks never leave the row
    for (uint32_t b = b_lo + (threadIdx.x >> 5); b < b_hi; b += NT / 32)
        requant_block(d, b, c, Rc, Rp, aligned);
}

// Requantise the int8 blocks that START in compact row c, for the bottom-up
// row order: a block that runs on into row c+1 (q_block <= w, so at most one
// more row) finds that row already in the ring (Rn).  Strips start at rows
// where blocks realign, so no block runs past a strip's last row.
template <int NT>
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
        const float sm = block_scale(warp_absmax(am)), sv = block_scale(warp_absmax(av));
        const float rm = __frcp_rn(sm), rv = __frcp_rn(sv);
        const bool finite = sm <= 0x1p126f && sv <= 0x1p126f;  // uniform across the warp; false for NaN
        for (uint32_t k = lane; k < B; k += 32) {
            const uint32_t cell = b * B + k;
            float2 mv = f2(0.0f, 0.0f);
            if (cell < C) mv = (aligned || cell < rowend) ? Rc[cell - rowbase] : Rn[cell - rowend];
            if (finite) {
                d.mq_out[cell] = quantize_finite(mv.x, sm, rm);
                d.vq_out[cell] = quantize_finite(mv.y, sv, rv);
            } else {
                d.mq_out[cell] = quantize_rc(mv.x, sm, rm);
                d.vq_out[cell] = quantize_rc(mv.y, sv, rv);
            }
        }
        if (lane == 0) {
            d.ms_out[b] = sm;
            d.vs_out[b] = sv;
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
template <int KH, int KW>
__device__ __noinline__ void phase2_fixup(const FusedDesc &d, int c, int j, const float2 *const R[3],
                                          const RowCo *rowco, const AdamK &ak, unsigned rows) {
    const int64_t W = d.W;
    float2 h[3][KW];
    width_pass3<KW>(R, j, d.w, h);
    for (int i = 0; i < KH; i++) {
        if (!((rows >> i) & 1u)) continue;
        float *prow = d.p + ((int64_t)c * KH + i) * W + (int64_t)j * KW;
        float pv[KW];
        load_param_row<KW, true>(prow, pv);
        const RowCo rc = rowco[i];
#pragma unroll
        for (int t = 0; t < KW; t += 2) {
            float2 m2[2];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const float2 a = rc.s0 == 0 ? h[0][t + e] : h[1][t + e];
                const float2 b = rc.s1 == 1 ? h[1][t + e] : h[2][t + e];
                m2[e] = __ffma2_rn(a, splat(rc.l0), __fmul2_rn(b, splat(rc.l1)));
            }
            const float2 pn = adam_write2(f2(pv[t], pv[t + 1]), f2(m2[0].x, m2[1].x),
                                          f2(clamp_min0(m2[0].y), clamp_min0(m2[1].y)), ak);
            pv[t] = pn.x;
            pv[t + 1] = pn.y;
        }
        store_param_row<KW>(prow, pv);
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
template <int KH, int KW, int NT, bool INTERIOR>
__device__ __forceinline__ void phase2(const FusedDesc &d, int c, const float2 *const R[3], const RowCo *rowco,
                                       const AdamK &ak) {
    const int w = d.w;
    const int64_t W = d.W;
    for (int j = threadIdx.x; j < w; j += NT) {
        float *pbase = d.p + (int64_t)c * KH * W + (int64_t)j * KW;
        float pv[KH][KW];
#pragma unroll
        for (int i = 0; i < KH; i++) load_param_row<KW, true>(pbase + i * W, pv[i]);
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
                    mh[t] = __ffma2_rn(upper ? h[0][t] : h[1][t], splat(1.0f - col_l1<KH>(i)),
                                       __fmul2_rn(upper ? h[1][t] : h[2][t], splat(col_l1<KH>(i))));
            } else {
                const RowCo rc = rowco[i];
                const bool lo0 = rc.s0 == 0, lo1 = rc.s1 == 1;  // uniform across the CTA
#pragma unroll
                for (int t = 0; t < KW; t++) {
                    const float2 a = lo0 ? h[0][t] : h[1][t];
                    const float2 b = lo1 ? h[1][t] : h[2][t];
                    mh[t] = __ffma2_rn(a, splat(rc.l0), __fmul2_rn(b, splat(rc.l1)));
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
                ok &= adam_write2_fast(f2(pv[i][t], pv[i][t + 1]), f2(mh[t].x, mh[t + 1].x),
                                       f2(nan_max(mh[t].y, 0.0f), nan_max(mh[t + 1].y, 0.0f)), ak, o);
                pn[t] = o.x;
                pn[t + 1] = o.y;
            }
            if (ok) store_param_row<KW>(pbase + i * W, pn);
            else fail |= 1u << i;
        }
        if (fail) phase2_fixup<KH, KW>(d, c, j, R, rowco, ak, fail);
    }
}

template <int KH, int KW, int NT>
__device__ __forceinline__ void phase2_row(const FusedDesc &d, int c, const float2 *const R[3], const RowCo *rowco,
                                           const AdamK &ak) {
    if (c > 0 && c < d.h - 1) phase2<KH, KW, NT, true>(d, c, R, rowco, ak);
    else phase2<KH, KW, NT, false>(d, c, R, rowco, ak);
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
template <int KH, int KW, int CELLS, int NT>
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
        phase1<KH, KW, CELLS, NT>(d, r, RR(r), r < c1);
        cta_sync<NT>();
        if (r < c1) {
            if (q8) requant_row_up<NT>(d, r, RR(r), r + 1 < c1 ? RR(r + 1) : nullptr);
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
            phase2_row<KH, KW, NT>(d, r + 1, R, rowco[(r + 1) & 1], ak);
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
    phase2_row<KH, KW, NT>(d, c0, R, rowco[c0 & 1], ak);
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

template <int KH, int KW, int CELLS, int NT, int MINB>
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
        process_strip<KH, KW, CELLS, NT>(b.d[t], (int)(s - b.strip_start[t]), s, epoch, ring, rowco, hdr, flags,
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

// ---------------------------------------------------------------- host side

static bool supported_window(int64_t k) { return k == 2 || k == 4 || k == 8; }

static int64_t gcd64(int64_t a, int64_t b) {
    while (b) {
        int64_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

static FastDiv make_fast_div(uint32_t d) {
    FastDiv f;
    f.d = d;
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < d) l++;
    f.l = l;
    f.m = (uint32_t)(((((uint64_t)1 << l) - d) << 32) / d + 1);
    return f;
}

// Compact rows per strip for a target length: a multiple of the rows after
// which int8 blocks realign with row starts, at most the tensor's rows.
static int64_t strip_rows(const smo_tensor &t, int64_t target) {
    int64_t align = 1;
    if (t.kind == SMO_KIND_POOLED8) align = t.q_block / gcd64(t.comp_cols, t.q_block);
    int64_t L = (target + align - 1) / align * align;
    return L < t.comp_rows ? L : t.comp_rows;
}

bool fused_takes(const smo_tensor &t) {
    if (t.kind != SMO_KIND_POOLED8 && t.kind != SMO_KIND_POOLED32) return false;
    if (t.flags & SMO_FLAG_GENERAL_PATH) return false;
    if (t.dtype != SMO_DTYPE_F32) return false;  // half-precision tensors take the general kernels
    if (t.row_perm || t.col_perm || t.row_perm_inv || t.col_perm_inv) return false;  // permute_basis
    if (t.rows <= 0 || t.cols <= 0 || t.comp_rows <= 0 || t.comp_cols <= 0) return false;
    if (t.rows % t.comp_rows != 0 || t.cols % t.comp_cols != 0) return false;
    const int64_t kh = t.rows / t.comp_rows, kw = t.cols / t.comp_cols;
    if (!supported_window(kh) || !supported_window(kw)) return false;
    if (t.cols <= 128) return false;  // torch's small-output interpolation order
    if (t.comp_cols > kMaxFusedCols) return false;
    if (t.comp_rows * t.comp_cols >= ((int64_t)1 << 31)) return false;  // 32-bit cell indices
    if (t.rows >= ((int64_t)1 << 24)) return false;  // exact float row coordinates (compute_rowco)
    if (t.kind == SMO_KIND_POOLED8 && t.q_block > t.comp_cols) return false;
    const size_t a = kw % 4 == 0 ? 16 : 8;
    if ((uintptr_t)t.param % a || (uintptr_t)t.grad % a) return false;
    if (t.interp_band < 0) return false;
    // the look-ahead reads the next strip's OLD state while that strip writes
    // the new one: in-place state would race, so it needs separate buffers
    if (t.kind == SMO_KIND_POOLED8 &&
        ((const void *)t.m_q_in == (const void *)t.m_q_out || (const void *)t.m_s_in == (const void *)t.m_s_out ||
         (const void *)t.v_q_in == (const void *)t.v_q_out || (const void *)t.v_s_in == (const void *)t.v_s_out))
        return false;
    if (t.kind == SMO_KIND_POOLED32 &&
        ((const void *)t.m_in == (const void *)t.m_out || (const void *)t.v_in == (const void *)t.v_out))
        return false;
    return true;
}

static int64_t num_strips(const smo_tensor &t, int64_t target) {
    const int64_t L = strip_rows(t, target);
    return (t.comp_rows + L - 1) / L;
}

static int window_key(const smo_tensor &t) {
    return (int)((t.rows / t.comp_rows) * 16 + (t.cols / t.comp_cols));
}

// CTA width of a launch: 192 threads (four CTAs of 80 registers per SM, so
// four independent row pipelines hide each other's load latency), or 256 when
// that leaves fewer idle thread-columns over the batch's compact rows (a
// compact row of w cells takes ceil(w / NT) passes of NT threads).
// SMO_B200_FUSED_THREADS (128, 192, 256 or 384) forces one width, for
// measurements.
static int pick_threads(const FusedBatch &b) {
    static int forced = -1;
    if (forced < 0) {
        const char *e = getenv("SMO_B200_FUSED_THREADS");
        forced = e ? atoi(e) : 0;
    }
    if (forced == 128 || forced == 192 || forced == 256 || forced == 384) return forced;
    int64_t idle192 = 0, idle256 = 0;
    for (int i = 0; i < b.n; i++) {
        const int64_t w = b.d[i].w, rows = b.d[i].h;
        idle192 += rows * ((w + 191) / 192 * 192 - w);
        idle256 += rows * ((w + 255) / 256 * 256 - w);
    }
    return idle256 < idle192 ? 256 : 192;
}

constexpr int kMaxDevices = 64;

static int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    return dev;
}

// SM count of the current device, queried once per device
static int device_sm_count() {
    static int cached[kMaxDevices];
    const int dev = current_device();
    if (dev < 0) return 148;
    if (cached[dev] > 0) return cached[dev];
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return 148;
    cached[dev] = sms;
    return sms;
}

static inline size_t align_up(size_t x) { return (x + kScratchAlign - 1) / kScratchAlign * kScratchAlign; }

// Launch plan: tensors the fused kernel takes, grouped by window shape in scan
// order (at most kMaxFused per launch), ordered by row width within a group,
// each with its strip length.
// Short launches get shorter strips so that every CTA slot sees several
// strips (the last strips of a launch otherwise leave SMs idle): the longest
// of 16, 8, 4 rows that gives at least 5 strips per CTA slot of a 4-CTA/SM
// grid.
struct LaunchGroup {
    int key;
    std::vector<int32_t> members;
    std::vector<int64_t> target;  // strip length target of each member
};

static int device_sm_count();

static void plan_launches(const smo_tensor *t, int32_t n, std::vector<LaunchGroup> &out) {
    out.clear();
    std::vector<char> done((size_t)n);
    for (int32_t i = 0; i < n; i++) done[i] = !fused_takes(t[i]);
    const int64_t want = 5 * 4 * (int64_t)device_sm_count();
    for (int32_t i = 0; i < n; i++) {
        if (done[i]) continue;
        LaunchGroup g;
        g.key = window_key(t[i]);
        for (int32_t k = i; k < n && (int)g.members.size() < kMaxFused; k++) {
            if (done[k] || window_key(t[k]) != g.key) continue;
            g.members.push_back(k);
            done[k] = 1;
        }
        // widest rows first: the largest strips are taken early and the
        // launch ends on the smallest ones, which shortens its tail
        std::stable_sort(g.members.begin(), g.members.end(),
                         [&](int32_t a, int32_t b) { return t[a].cols > t[b].cols; });
        int64_t rows = kStripRows;
        while (rows > 4) {
            int64_t strips = 0;
            for (int32_t k : g.members) strips += num_strips(t[k], rows);
            if (strips >= want) break;
            rows /= 2;
        }
        g.target.assign(g.members.size(), rows);
        out.push_back(std::move(g));
    }
}

// Workspace after the header: [flags: one word per strip][published rows:
// 2*w floats per strip].  Sized for the largest window-group launch of the
// set; each launch reuses the space.  The flag words sit
// in a region of their own that nothing else writes (the general path's
// scratch starts after it): a flag word may only ever hold a launch epoch,
// or a stale float could read as "strip published".
FusedLayout fused_workspace_layout(const smo_tensor *t, int32_t n) {
    std::vector<LaunchGroup> groups;
    plan_launches(t, n, groups);
    FusedLayout out{0, 0};
    for (const LaunchGroup &g : groups) {
        size_t strips = 0, halo_floats = 0;
        for (size_t m = 0; m < g.members.size(); m++) {
            const int32_t k = g.members[m];
            const int64_t s = num_strips(t[k], g.target[m]);
            strips += (size_t)s;
            halo_floats += (size_t)s * 2 * (size_t)t[k].comp_cols;
        }
        const size_t flags = align_up(strips * sizeof(unsigned int));
        const size_t body = align_up(halo_floats * sizeof(float));
        out.flag_bytes = out.flag_bytes > flags ? out.flag_bytes : flags;
        out.body_bytes = out.body_bytes > body ? out.body_bytes : body;
    }
    return out;
}

// The kernel instance of a window shape and CTA width: 16-element windows take
// one cell per thread-iteration, smaller windows two; 128-, 192- and
// 384-thread CTAs run six, four and two per SM at 80 registers, 256-thread
// CTAs four (one cell, 64 registers) or three (two cells, 80 registers).
template <int KH, int KW>
static auto fused_kernel_for(int nt) {
    constexpr int kCells = KH * KW >= 16 ? 1 : 2;
    constexpr int kMinBlocks256 = kCells == 1 ? 4 : 3;
    switch (nt) {
        case 128: return fused_step_kernel<KH, KW, kCells, 128, 6>;
        case 192: return fused_step_kernel<KH, KW, kCells, 192, 4>;
        case 384: return fused_step_kernel<KH, KW, kCells, 384, 2>;
        default: return fused_step_kernel<KH, KW, kCells, 256, kMinBlocks256>;
    }
}

static int kernel_cache_slot(int nt) { return nt == 384 ? 1 : nt == 192 ? 4 : nt == 128 ? 5 : 0; }

// The shared-memory attribute and the occupancy of a kernel instance are set
// and queried once per device and size (the attribute is a maximum, so a
// larger earlier setting covers smaller launches).
struct KernelCache {
    size_t smem_attr = 0, smem_occ = 0;
    int per_sm = 0;
};

template <class Kern>
static int occupancy(Kern kern, KernelCache &c, int nt, size_t smem, int &per_sm) {
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

template <int KH, int KW>
static int launch_fused_group(FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
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
        nt = pick_threads(b);
        st = occupancy(fused_kernel_for<KH, KW>(nt), dev >= 0 ? cache[dev][kernel_cache_slot(nt)] : scratch, nt, smem,
                       per_sm);
    }
    if (st != SMO_OK) return st;
    per_sm = per_sm < 1 ? 1 : (per_sm > kMaxFusedCtasPerSm ? kMaxFusedCtasPerSm : per_sm);
    int64_t grid = (int64_t)device_sm_count() * per_sm;
    grid = grid < strips ? grid : strips;
    fused_kernel_for<KH, KW>(nt)<<<(unsigned)grid, nt, smem, stream>>>(b, hdr, flags, halo, wait_limit(),
                                                                     g_wait_skew.load(std::memory_order_relaxed));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    g_launches++;
    return SMO_OK;
}

static int dispatch(int key, FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
                    cudaStream_t stream) {
    switch (key) {
#define SMO_FUSED_CASE(KH, KW) \
    case KH * 16 + KW: return launch_fused_group<KH, KW>(b, max_w, halo_floats, ws, flag_bytes, stream);
        SMO_FUSED_CASE(2, 2) SMO_FUSED_CASE(2, 4) SMO_FUSED_CASE(2, 8)
        SMO_FUSED_CASE(4, 2) SMO_FUSED_CASE(4, 4) SMO_FUSED_CASE(4, 8)
        SMO_FUSED_CASE(8, 2) SMO_FUSED_CASE(8, 4) SMO_FUSED_CASE(8, 8)
#undef SMO_FUSED_CASE
        default: return SMO_ERR_INVALID;
    }
}

static void fill(FusedDesc &f, const smo_tensor &t, int64_t halo_off, int64_t target_rows) {
    memset(&f, 0, sizeof(f));
    f.p = t.param;
    f.g = t.grad;
    f.mq_in = t.m_q_in; f.ms_in = t.m_s_in; f.vq_in = t.v_q_in; f.vs_in = t.v_s_in;
    f.mq_out = t.m_q_out; f.ms_out = t.m_s_out; f.vq_out = t.v_q_out; f.vs_out = t.v_s_out;
    f.m_in = t.m_in; f.v_in = t.v_in; f.m_out = t.m_out; f.v_out = t.v_out;
    f.H = t.rows; f.W = t.cols; f.band = t.interp_band;
    f.h = (int32_t)t.comp_rows; f.w = (int32_t)t.comp_cols;
    f.B = t.kind == SMO_KIND_POOLED8 ? (int32_t)t.q_block : 1;
    f.L = (int32_t)strip_rows(t, target_rows);
    f.div_B = make_fast_div((uint32_t)f.B);
    f.div_w = make_fast_div((uint32_t)f.w);
    f.halo_off = halo_off;
    f.kind = t.kind;
    f.hp = t.hp;
}

int fused_step(const smo_tensor *t, int32_t n, char *ws, size_t flag_bytes, cudaStream_t stream) {
    static thread_local FusedBatch batch;
    static thread_local std::vector<LaunchGroup> groups;
    plan_launches(t, n, groups);
    // one launch per group (window shape, at most kMaxFused tensors); the
    // groups run one after another and reuse the workspace
    for (const LaunchGroup &g : groups) {
        batch.n = 0;
        batch.strip_start[0] = 0;
        int64_t halo_off = 0, max_w = 0;
        for (size_t m = 0; m < g.members.size(); m++) {
            const int32_t k = g.members[m];
            FusedDesc &f = batch.d[batch.n];
            fill(f, t[k], halo_off, g.target[m]);
            const int64_t s = num_strips(t[k], g.target[m]);
            halo_off += s * 2 * t[k].comp_cols;
            max_w = max_w > t[k].comp_cols ? max_w : t[k].comp_cols;
            batch.strip_start[batch.n + 1] = batch.strip_start[batch.n] + s;
            batch.n++;
        }
        const int st = dispatch(g.key, batch, max_w, (size_t)halo_off, ws, flag_bytes, stream);
        if (st != SMO_OK) return st;
    }
    return SMO_OK;
}

}  // namespace smo
