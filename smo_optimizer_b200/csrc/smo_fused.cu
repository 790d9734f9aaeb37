// smo_fused.cu -- fused single-pass step for exact-window pooled tensors.
//
// One persistent launch steps every qualifying tensor of a batch.  HBM sees
// each parameter and gradient element read once and each parameter written
// once (plus the compact moment state); the parameter values are read a second
// time from L2.
//
// Work unit: a STRIP of L compact rows (KH*L full-resolution rows), full
// width, of one tensor.  CTAs take strips in increasing order from an atomic
// counter in the workspace header.  A strip is walked as a sequence of STEPS:
// compact row r is split into column chunks of CW compact cells, and step
// (r, k) does
//
//   phase 1 (row r, chunk k)     window sums of x = g + wd*p and x*x, dequant of
//                                the old codes, EMA; post-EMA (m, v) pairs go to
//                                a 3-row ring in shared memory;
//   phase 2 (row r-1, chunk k-1) bilinear reconstruction (width pass, then
//                                height pass, torch's order) and the Adam write
//                                of the KH parameter rows of that chunk.
//
// The gradient and parameter rows that phase 1 of a step reads are brought
// into a shared-memory stage by TMA bulk copies (cp.async.bulk, completion on
// an mbarrier) kStages-1 steps ahead, issued by one thread; the codes, scales
// or fp32 state of a row arrive by cp.async one row ahead; the parameter values
// phase 2 rewrites are loaded into registers at the start of the step.  When a
// row's last chunk is done its int8 blocks are requantised.
//
// Neighbouring strips: the write of a strip's last row needs the first row of
// the next strip.  The CTA recomputes that row itself (look-ahead) from the
// next strip's g, p and OLD moment state; the old state is intact because the
// moments are double-buffered (read *_in, write *_out).  The write of a
// strip's FIRST row needs the previous strip's last row, which the previous
// strip publishes to the workspace (with a release flag) after its look-ahead
// read; so the first row is written last, after an acquire wait.  Waits only
// ever point at an earlier strip, which some running CTA took before this one,
// so they cannot deadlock whatever the residency; every wait is bounded and
// reports SMO_ERR_TIMEOUT in the workspace header instead of hanging.
#include <cstdlib>
#include <cstring>
#include <vector>

#include "smo_common.cuh"
#include "smo_internal.cuh"

namespace smo {

constexpr int kThreads = 256;
constexpr int kStages = 4;                  // shared-memory stages (kStages-1 steps of look-ahead)
constexpr int kMaxFusedCtasPerSm = 2;
constexpr int kMaxFused = 104;
constexpr int64_t kStripRows = 16;          // target compact rows per strip
constexpr int64_t kMaxFusedCols = 4096;     // compact columns per tensor
constexpr int64_t kDefaultWaitIters = 1 << 22;

// Chunk geometry of a KH x KW window: CW compact cells per step (one per
// phase-1 thread); in phase 2 TPC threads share a cell, RPT rows each.
template <int KH, int KW>
struct Geo {
    static constexpr int CW = (2048 / (KH * KW)) > kThreads ? kThreads : 2048 / (KH * KW);
    static constexpr int TPC = kThreads / CW;
    static constexpr int RPT = KH / TPC;
    static constexpr int ROWF = CW * KW;               // floats of one staged full-resolution row
    static constexpr int STAGE_FLOATS = 2 * KH * ROWF; // gradient rows, then parameter rows
    // ring rows one thread's output rows draw on: two when its rows lie in one
    // half of the window, all three when they cover both halves
    static constexpr int NR = (RPT > KH / 2) ? 3 : 2;
    static_assert(RPT >= 1 && TPC * RPT == KH, "phase-2 mapping");
};

// n / d for 32-bit unsigned n by a divisor fixed per tensor: multiply by a
// precomputed magic number (Granlund-Montgomery / Hacker's Delight 10-1, the
// round-up variant with a 33-bit add), set up on the host.
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
    int32_t kind;
    smo_hyper hp;
};

struct FusedBatch {
    int32_t n;
    int64_t strip_start[kMaxFused + 1];
    FusedDesc d[kMaxFused];
};
static_assert(sizeof(FusedBatch) < 30000, "kernel parameter batch must stay below 32 KB");

// ---------------------------------------------------------------- async copies

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// 1-D TMA bulk copy global -> shared, completion counted on `bar` (both
// addresses 16-byte aligned, bytes a multiple of 16)
__device__ __forceinline__ void tma_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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
    float2 sbc2, rcp_sbc2, eps, ns;
};

__device__ __forceinline__ float2 adam_write2(float2 p, float2 m, float2 v, const AdamK &k) {
    const float2 sv = f2(__fsqrt_rn(v.x), __fsqrt_rn(v.y));
    const float2 d = __fadd2_rn(div_rcp2(sv, k.sbc2, k.rcp_sbc2), k.eps);
    const float2 a = __fmul2_rn(k.ns, m);
    return __fadd2_rn(p, f2(__fdiv_rn(a.x, d.x), __fdiv_rn(a.y, d.y)));
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

// ---------------------------------------------------------------- row state
//
// The moment state phase 1 reads for one compact row, staged by cp.async one
// row ahead: POOLED8: m codes [w] int8, v codes [w] int8, m scales and v
// scales of the blocks the row touches; POOLED32: m [w], v [w] fp32.

struct RowState {
    const int8_t *mq, *vq;
    const float *ms, *vs;
    const float *m, *v;
    uint32_t b0;  // first block of the row (POOLED8)
};

__device__ __forceinline__ RowState row_state_view(char *base, const FusedDesc &d, int r) {
    RowState s;
    const int w = d.w;
    if (d.kind == SMO_KIND_POOLED8) {
        const uint32_t first = fast_div((uint32_t)r * (uint32_t)w, d.div_B);
        const uint32_t last = fast_div(((uint32_t)r + 1u) * (uint32_t)w - 1u, d.div_B);
        s.mq = (const int8_t *)base;
        s.vq = (const int8_t *)base + w;
        s.ms = (const float *)(base + 2 * w);
        s.vs = s.ms + (last - first + 1);
        s.b0 = first;
        s.m = s.v = nullptr;
    } else {
        s.m = (const float *)base;
        s.v = (const float *)base + w;
        s.mq = s.vq = nullptr;
        s.ms = s.vs = nullptr;
        s.b0 = 0;
    }
    return s;
}

// all threads: issue the cp.async copies of row r's old state (w % 16 == 0)
__device__ __forceinline__ void fetch_row_state(char *base, const FusedDesc &d, int r) {
    const int w = d.w;
    const int64_t off = (int64_t)r * w;
    if (d.kind == SMO_KIND_POOLED8) {
        const uint32_t first = fast_div((uint32_t)r * (uint32_t)w, d.div_B);
        const uint32_t last = fast_div(((uint32_t)r + 1u) * (uint32_t)w - 1u, d.div_B);
        const int nb = (int)(last - first + 1);
        int8_t *mq = (int8_t *)base, *vq = (int8_t *)base + w;
        float *ms = (float *)(base + 2 * w), *vs = ms + nb;
        for (int i = threadIdx.x; i < w / 16; i += kThreads) {
            cp_async16(mq + 16 * i, d.mq_in + off + 16 * i);
            cp_async16(vq + 16 * i, d.vq_in + off + 16 * i);
        }
        for (int i = threadIdx.x; i < nb; i += kThreads) {
            cp_async4(ms + i, d.ms_in + first + i);
            cp_async4(vs + i, d.vs_in + first + i);
        }
    } else {
        float *m = (float *)base, *v = (float *)base + w;
        for (int i = threadIdx.x; i < w / 4; i += kThreads) {
            cp_async16(m + 4 * i, d.m_in + off + 4 * i);
            cp_async16(v + 4 * i, d.v_in + off + 4 * i);
        }
    }
}

// ---------------------------------------------------------------- phases

// (sum x, sum x*x) of one KH x KW window in row-major order from +0, times
// 1/(KH*KW) (a power of two: the same value as avg_pool2d's division)
template <int KH, int KW, bool WD>
__device__ __forceinline__ float2 pool_cell(const float *sg, const float *sp, float wd) {
    float2 acc = f2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < KH; i++) {
        float gv[KW], pv[KW];
#pragma unroll
        for (int k = 0; k < KW; k += (KW >= 4 ? 4 : 2)) {
            if constexpr (KW >= 4) {
                const float4 t = *reinterpret_cast<const float4 *>(sg + i * Geo<KH, KW>::ROWF + k);
                gv[k] = t.x; gv[k + 1] = t.y; gv[k + 2] = t.z; gv[k + 3] = t.w;
                if (WD) {
                    const float4 u = *reinterpret_cast<const float4 *>(sp + i * Geo<KH, KW>::ROWF + k);
                    pv[k] = u.x; pv[k + 1] = u.y; pv[k + 2] = u.z; pv[k + 3] = u.w;
                }
            } else {
                const float2 t = *reinterpret_cast<const float2 *>(sg + i * Geo<KH, KW>::ROWF + k);
                gv[k] = t.x; gv[k + 1] = t.y;
                if (WD) {
                    const float2 u = *reinterpret_cast<const float2 *>(sp + i * Geo<KH, KW>::ROWF + k);
                    pv[k] = u.x; pv[k + 1] = u.y;
                }
            }
        }
#pragma unroll
        for (int k = 0; k < KW; k++) {
            const float x = WD ? __fmaf_rn(wd, pv[k], gv[k]) : gv[k];
            acc = __fadd2_rn(acc, f2(x, __fmul_rn(x, x)));
        }
    }
    constexpr float inv = 1.0f / (KH * KW);
    return __fmul2_rn(acc, splat(inv));
}

// Phase 1 of (row r, chunk k): thread j < n1 owns compact cell k*CW + j.
template <int KH, int KW, bool WD>
__device__ __forceinline__ void phase1(const FusedDesc &d, int r, int k, const float *stage, const RowState &rs,
                                       float2 *ringrow, bool own) {
    using G = Geo<KH, KW>;
    const int j = threadIdx.x;
    const int n1 = min(G::CW, d.w - k * G::CW);
    if (j >= n1) return;
    const int col = k * G::CW + j;
    const float2 pooled = pool_cell<KH, KW, WD>(stage + j * KW, stage + KH * G::ROWF + j * KW, d.hp.weight_decay);
    const smo_hyper &hp = d.hp;
    float2 mv;
    if (d.kind == SMO_KIND_POOLED8) {
        const uint32_t cell = (uint32_t)r * (uint32_t)d.w + (uint32_t)col;
        const uint32_t bi = fast_div(cell, d.div_B) - rs.b0;
        mv = dequant2(rs.mq[col], rs.vq[col], rs.ms[bi], rs.vs[bi]);
    } else {
        mv = f2(rs.m[col], rs.v[col]);
    }
    mv = __ffma2_rn(f2(hp.omb1, hp.omb2), pooled, __fmul2_rn(mv, f2(hp.beta1, hp.beta2)));
    ringrow[col] = mv;
    if (own && d.kind == SMO_KIND_POOLED32) {
        const int64_t cell = (int64_t)r * d.w + col;
        d.m_out[cell] = mv.x;
        d.v_out[cell] = mv.y;
    }
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
    for (uint32_t k = lane; k < B; k += 32) {
        const uint32_t cell = b * B + k;
        float2 mv = f2(0.0f, 0.0f);
        if (cell < C) mv = (aligned || cell >= rowbase) ? Rc[cell - rowbase] : Rp[cell + w - rowbase];
        d.mq_out[cell] = quantize_rc(mv.x, sm, rm);
        d.vq_out[cell] = quantize_rc(mv.y, sv, rv);
    }
    if (lane == 0) {
        d.ms_out[b] = sm;
        d.vs_out[b] = sv;
    }
}

__device__ __forceinline__ void requant_row(const FusedDesc &d, int c, const float2 *Rc, const float2 *Rp) {
    const uint32_t w = (uint32_t)d.w, B = (uint32_t)d.B, C = (uint32_t)d.h * w;
    const uint32_t b_lo = fast_div((uint32_t)c * w, d.div_B);
    uint32_t b_hi = fast_div(((uint32_t)c + 1u) * w, d.div_B);
    if (c == d.h - 1 && C % B != 0) b_hi = C / B + 1;  // the zero-padded last block
    const bool aligned = (w % B) == 0;                  // blocks never leave the row
    for (uint32_t b = b_lo + (threadIdx.x >> 5); b < b_hi; b += kThreads / 32)
        requant_block(d, b, c, Rc, Rp, aligned);
}

struct RowCo {
    int s0, s1;  // ring-relative rows (0: c-1, 1: c, 2: c+1)
    float l0, l1;
};

// Row weights of the KH output rows of compact row c (threads 0..KH-1).
template <int KH>
__device__ __forceinline__ void compute_rowco(const FusedDesc &d, int c, RowCo *dst) {
    if (threadIdx.x < KH) {
        int small;
        const Coef rc = row_coef((int64_t)c * KH + threadIdx.x, d.H, d.h, d.W, d.band, small);
        RowCo r;
        r.s0 = (int)(rc.i0 - (c - 1));
        r.s1 = (int)(rc.i1 - (c - 1));
        r.l0 = rc.l0;
        r.l1 = rc.l1;
        dst[threadIdx.x] = r;
    }
}

// Width-pass weights of output column t of a KW-wide window (power-of-two KW):
// exactly torch's src = (q + 0.5)/KW - 0.5 split into floor and fraction.
template <int KW>
__device__ __forceinline__ float col_l1(int t) {
    return (t + 0.5f) / KW + (t < KW / 2 ? 0.5f : -0.5f);
}

// Parameter values phase 2 of a step rewrites, loaded into registers at the
// start of the step (L2 hits: phase 1 of the same row read them).
template <int KH, int KW>
struct P2Regs {
    float v[Geo<KH, KW>::RPT][KW];
};

template <int KH, int KW>
__device__ __forceinline__ void load_p2(const FusedDesc &d, int c, int k, P2Regs<KH, KW> &pr) {
    using G = Geo<KH, KW>;
    const int j = threadIdx.x % G::CW;
    const int i0 = (threadIdx.x / G::CW) * G::RPT;
    const int n = min(G::CW, d.w - k * G::CW);
    if (j >= n) return;
    const float *base = d.p + ((int64_t)c * KH + i0) * d.W + (int64_t)(k * G::CW + j) * KW;
#pragma unroll
    for (int i = 0; i < G::RPT; i++) {
#pragma unroll
        for (int t = 0; t < KW; t += 2) {
            const float2 x = __ldcg(reinterpret_cast<const float2 *>(base + i * d.W + t));
            pr.v[i][t] = x.x;
            pr.v[i][t + 1] = x.y;
        }
    }
}

// Phase 2 of (row c, chunk k): the thread's RPT output rows of cell k*CW + j,
// from the post-EMA rows c-1 (R0), c (R1), c+1 (R2) (an absent neighbour row is
// passed as row c and never weighted); row weights from `rowco`.
template <int KH, int KW>
__device__ __forceinline__ void phase2(const FusedDesc &d, int c, int k, const float2 *R0, const float2 *R1,
                                       const float2 *R2, const RowCo *rowco, const AdamK &ak,
                                       const P2Regs<KH, KW> &pr) {
    using G = Geo<KH, KW>;
    constexpr int NR = G::NR;
    const int j = threadIdx.x % G::CW;
    const int i0 = (threadIdx.x / G::CW) * G::RPT;
    const int w = d.w;
    const int n = min(G::CW, w - k * G::CW);
    if (j >= n) return;
    const int col = k * G::CW + j;
    // the ring rows the thread's output rows draw on: sa .. sa+NR-1
    int sa = 0;
    if (NR == 2) {
        sa = 2;
#pragma unroll
        for (int i = 0; i < G::RPT; i++) sa = min(sa, rowco[i0 + i].s0);
        sa = min(sa, 1);
    }
    // width pass: the left half of the window interpolates columns (col-1, col),
    // the right half (col, col+1), clamped at the edges exactly as torch does
    const int jr = col + 1 < w ? col + 1 : w - 1;
    const int la = col > 0 ? col - 1 : 0;
    float2 hw[NR][KW];
#pragma unroll
    for (int q = 0; q < NR; q++) {
        const int sr = sa + q;
        const float2 *row = sr == 0 ? R0 : (sr == 1 ? R1 : R2);
        const float2 L = row[la], M = row[col], Rr = row[jr];
        const float2 X = col > 0 ? M : Rr;
#pragma unroll
        for (int t = 0; t < KW; t++) {
            if (t < KW / 2) {
                const float l1 = col > 0 ? col_l1<KW>(t) : 0.0f;
                const float l0 = col > 0 ? 1.0f - col_l1<KW>(t) : 1.0f;
                hw[q][t] = __ffma2_rn(L, splat(l0), __fmul2_rn(X, splat(l1)));
            } else {
                hw[q][t] = __ffma2_rn(M, splat(1.0f - col_l1<KW>(t)), __fmul2_rn(Rr, splat(col_l1<KW>(t))));
            }
        }
    }
    float *base = d.p + ((int64_t)c * KH + i0) * d.W + (int64_t)col * KW;
#pragma unroll
    for (int i = 0; i < G::RPT; i++) {
        const RowCo rc = rowco[i0 + i];
        const int qa = rc.s0 - sa, qb = rc.s1 - sa;
#pragma unroll
        for (int t = 0; t < KW; t += 2) {
            float2 mh[2];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                float2 x, y;
                if (NR == 2) {
                    x = qa == 0 ? hw[0][t + u] : hw[NR - 1][t + u];
                    y = qb == 0 ? hw[0][t + u] : hw[NR - 1][t + u];
                } else {
                    x = qa == 0 ? hw[0][t + u] : (qa == 1 ? hw[1][t + u] : hw[NR - 1][t + u]);
                    y = qb == 0 ? hw[0][t + u] : (qb == 1 ? hw[1][t + u] : hw[NR - 1][t + u]);
                }
                mh[u] = __ffma2_rn(x, splat(rc.l0), __fmul2_rn(y, splat(rc.l1)));
            }
            const float2 pn = adam_write2(f2(pr.v[i][t], pr.v[i][t + 1]), f2(mh[0].x, mh[1].x),
                                          f2(clamp_min0(mh[0].y), clamp_min0(mh[1].y)), ak);
            __stcs(reinterpret_cast<float2 *>(base + i * d.W + t), pn);
        }
    }
}

// ---------------------------------------------------------------- strip driver

struct SharedCtl {
    uint64_t bar[kStages];
    RowCo rowco[2][8];
    int64_t strip;
    unsigned int epoch;
    int ok;
};

// Step cursor of a strip: main steps walk rows c0..c1 (c1 = the look-ahead
// row, or one past the tensor's last row), chunks 0..nk each; then nk deferred
// steps rewrite the strip's first row.  Step (r, k) runs phase 1 on (r, k) and
// phase 2 on (r-1, k-1).
struct Cursor {
    int r, k;
    bool deferred;
};

__device__ __forceinline__ void advance(Cursor &c, int c1, int nk) {
    if (c.deferred) {
        c.k++;
    } else if (++c.k > nk) {
        c.k = 0;
        if (++c.r > c1) {
            c.deferred = true;
            c.k = 0;
        }
    }
}

// thread 0: stage the phase-1 rows of the step at cursor `c` into slot
// (gs % kStages); a step without phase 1 still arrives once so that every slot
// phase completes
template <int KH, int KW>
__device__ __forceinline__ void issue_step(const FusedDesc &d, const Cursor &c, int c1, int nk, uint64_t gs,
                                           float *stages, uint64_t *bars) {
    using G = Geo<KH, KW>;
    const int slot = (int)(gs % kStages);
    const bool has1 = !c.deferred && c.k < nk && (c.r < c1 || c1 < d.h);
    if (!has1) {
        mbar_arrive_expect_tx(&bars[slot], 0);
        return;
    }
    const int n1 = min(G::CW, d.w - c.k * G::CW);
    const uint32_t seg = (uint32_t)(n1 * KW * 4);
    const bool wd = d.hp.wd_on != 0;
    // order this CTA's earlier reads of the slot before the async-proxy writes
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(&bars[slot], seg * KH * (wd ? 2u : 1u));
    float *st = stages + (size_t)slot * G::STAGE_FLOATS;
    const int64_t off = (int64_t)c.r * KH * d.W + (int64_t)c.k * G::CW * KW;
#pragma unroll
    for (int i = 0; i < KH; i++) tma_load(st + i * G::ROWF, d.g + off + i * d.W, seg, &bars[slot]);
    if (wd) {
#pragma unroll
        for (int i = 0; i < KH; i++) tma_load(st + (KH + i) * G::ROWF, d.p + off + i * d.W, seg, &bars[slot]);
    }
}

__device__ __forceinline__ void wait_slot(uint64_t *bar, uint64_t gs, int64_t wait_iters, WsHeader *hdr,
                                          int64_t gstrip) {
    const uint32_t parity = (uint32_t)((gs / kStages) & 1);
    int64_t it = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (++it > wait_iters) {
            if (threadIdx.x == 0) report_error(hdr, SMO_ERR_TIMEOUT, (unsigned int)gstrip);
            break;
        }
    }
}

template <int KH, int KW>
__device__ void process_strip(const FusedDesc &d, int sidx, int64_t gstrip, unsigned int epoch, float *stages,
                              float2 *ring, char *rstate, int rstate_stride, float2 *head, SharedCtl &ctl,
                              uint64_t &gstep, WsHeader *hdr, unsigned int *flags, float *halo, int64_t wait_iters) {
    using G = Geo<KH, KW>;
    const int w = d.w, h = d.h;
    const int c0 = sidx * d.L;
    const int c1 = c0 + d.L < h ? c0 + d.L : h;
    const int nk = (w + G::CW - 1) / G::CW;
    const int nsteps = (c1 - c0 + 1) * (nk + 1) + nk;
    const bool q8 = (d.kind == SMO_KIND_POOLED8);
    const bool wd = d.hp.wd_on != 0;
    AdamK ak;
    ak.sbc2 = splat(d.hp.sqrt_bc2);
    ak.rcp_sbc2 = splat(__frcp_rn(d.hp.sqrt_bc2));
    ak.eps = splat(d.hp.eps);
    ak.ns = splat(d.hp.neg_step);
    float2 *pub = reinterpret_cast<float2 *>(halo + d.halo_off) + (int64_t)sidx * w;
    // rows c0 and c0+1 are kept in this CTA's global head buffer (L2) until the
    // strip's first row is written at the end
    auto save_head = [&](const float2 *src, int slot) {
        float2 *dst = head + slot * w;
        for (int j = threadIdx.x; j < w; j += kThreads) __stcg(dst + j, src[j]);
    };

    // prologue: the first row's state, the first kStages-1 steps' rows
    fetch_row_state(rstate + (c0 & 1) * rstate_stride, d, c0);
    Cursor ic{c0, 0, false};  // thread 0's issue cursor, kStages-1 steps ahead
    if (threadIdx.x == 0) {
        for (int u = 0; u < kStages - 1 && u < nsteps; u++) {
            issue_step<KH, KW>(d, ic, c1, nk, gstep + u, stages, ctl.bar);
            advance(ic, c1, nk);
        }
    }
    cp_async_wait_all();
    __syncthreads();

    Cursor cur{c0, 0, false};
    // ring rows of the row in phase 1 (r) and its two predecessors
    float2 *Rm2 = ring + ((c0 + 1) % 3) * w, *Rm1 = ring + ((c0 + 2) % 3) * w, *R0 = ring + (c0 % 3) * w;
    RowState rs = row_state_view(rstate + (c0 & 1) * rstate_stride, d, c0);
    for (int u = 0; u < nsteps; u++, advance(cur, c1, nk)) {
        const uint64_t gs = gstep + u;
        const int r = cur.r, k = cur.k;
        if (cur.deferred && k == 0) {
            // deferred first row: rows c0-1 (the previous strip's published row),
            // c0 and c0+1 go back into ring slots 0, 1, 2
            compute_rowco<KH>(d, c0, ctl.rowco[c0 & 1]);
            if (c0 > 0 && threadIdx.x == 0) {
                const bool ok = bounded_wait_eq(flags + gstrip - 1, epoch, wait_iters, &hdr->error);
                if (!ok) report_error(hdr, SMO_ERR_TIMEOUT, (unsigned int)gstrip);
                ctl.ok = ok;
            }
            __syncthreads();
            const float2 *prev = pub - (sidx > 0 ? w : 0);
            const bool ok = c0 > 0 && ctl.ok;
            for (int j = threadIdx.x; j < w; j += kThreads) {
                if (c0 > 0) ring[j] = ok ? __ldcg(prev + j) : f2(0.0f, 0.0f);
                ring[w + j] = __ldcg(head + j);
                if (c0 + 1 < h) ring[2 * w + j] = __ldcg(head + w + j);
            }
            __syncthreads();
        }
        // the step kStages-1 ahead goes into the slot the previous step freed
        if (threadIdx.x == 0 && u + kStages - 1 < nsteps) {
            issue_step<KH, KW>(d, ic, c1, nk, gs + kStages - 1, stages, ctl.bar);
            advance(ic, c1, nk);
        }
        const bool has1 = !cur.deferred && k < nk && (r < c1 || c1 < h);
        const bool has2 = cur.deferred || (k >= 1 && r - 1 > c0);
        if (!cur.deferred && k == 0) {
            if (r > c0) {
                // rotate the ring: row r takes the slot of row r-3
                float2 *t = Rm2;
                Rm2 = Rm1;
                Rm1 = R0;
                R0 = t;
                rs = row_state_view(rstate + (r & 1) * rstate_stride, d, r);
            }
            if (r - 1 > c0) compute_rowco<KH>(d, r - 1, ctl.rowco[(r - 1) & 1]);
            // the next row's old state, one row ahead (the buffer of row r-1, done)
            if (r + 1 <= c1 && r + 1 < h) fetch_row_state(rstate + ((r + 1) & 1) * rstate_stride, d, r + 1);
        }
        const int pr_row = cur.deferred ? c0 : r - 1;
        const int pr_k = cur.deferred ? k : k - 1;
        P2Regs<KH, KW> pr;
        if (has2) load_p2<KH, KW>(d, pr_row, pr_k, pr);
        if (has1) {
            wait_slot(&ctl.bar[gs % kStages], gs, wait_iters, hdr, gstrip);
            const float *stage = stages + (size_t)(gs % kStages) * G::STAGE_FLOATS;
            if (wd) phase1<KH, KW, true>(d, r, k, stage, rs, R0, r < c1);
            else phase1<KH, KW, false>(d, r, k, stage, rs, R0, r < c1);
        }
        __syncthreads();
        if (!cur.deferred && k == nk) {
            if (r < c1) {
                if (q8) requant_row(d, r, R0, r > c0 ? Rm1 : nullptr);
                if (r == c0) save_head(R0, 0);
                if (r == c0 + 1) save_head(R0, 1);
                // the next row's state must have landed before its first chunk
                cp_async_wait_all();
            } else if (c1 < h) {
                // look-ahead row done: keep it as the strip's second row if the
                // strip has one row, then publish this strip's last row for the
                // next strip (after the look-ahead read of that strip's data)
                if (r == c0 + 1) save_head(R0, 1);
                for (int j = threadIdx.x; j < w; j += kThreads) __stcg(pub + j, Rm1[j]);
                __syncthreads();
                if (threadIdx.x == 0) {
                    __threadfence();
                    store_release(flags + gstrip, epoch);
                }
            }
        }
        if (has2) {
            const RowCo *rc = ctl.rowco[pr_row & 1];
            if (!cur.deferred) {
                // phase 2 of row r-1: rows r-2, r-1, r (row r absent past the tensor's end)
                phase2<KH, KW>(d, r - 1, k - 1, Rm2, Rm1, r < h ? R0 : Rm1, rc, ak, pr);
            } else {
                phase2<KH, KW>(d, c0, k, c0 > 0 ? ring : ring + w, ring + w, c0 + 1 < h ? ring + 2 * w : ring + w,
                               rc, ak, pr);
            }
        }
        __syncthreads();
    }
    gstep += (uint64_t)nsteps;
}

__device__ __forceinline__ int find_strip_tensor(const FusedBatch &b, int64_t s) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (b.strip_start[mid] <= s) lo = mid; else hi = mid - 1;
    }
    return lo;
}

template <int KH, int KW>
__global__ void __launch_bounds__(kThreads, 2)
    fused_step_kernel(const __grid_constant__ FusedBatch b, WsHeader *hdr, unsigned int *flags, float *halo,
                      float *heads, int64_t head_stride, int32_t max_w, int32_t rstate_stride, int64_t wait_iters) {
    using G = Geo<KH, KW>;
    extern __shared__ __align__(128) unsigned char dyn[];
    __shared__ SharedCtl ctl;
    float *stages = reinterpret_cast<float *>(dyn);
    float2 *ring = reinterpret_cast<float2 *>(stages + (size_t)kStages * G::STAGE_FLOATS);
    char *rstate = reinterpret_cast<char *>(ring + 3 * (size_t)max_w);
    float2 *head = reinterpret_cast<float2 *>(heads + (int64_t)blockIdx.x * head_stride);
    if (threadIdx.x == 0) {
        ctl.epoch = *(volatile unsigned int *)&hdr->epoch + 1u;
        for (int i = 0; i < kStages; i++) mbar_init(&ctl.bar[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    uint64_t gstep = 0;
    const int64_t total = b.strip_start[b.n];
    for (;;) {
        if (threadIdx.x == 0) ctl.strip = (int64_t)atomicAdd(&hdr->next_item, 1u);
        __syncthreads();
        const int64_t s = ctl.strip;
        const unsigned int epoch = ctl.epoch;
        __syncthreads();
        if (s >= total) break;
        const int t = find_strip_tensor(b, s);
        process_strip<KH, KW>(b.d[t], (int)(s - b.strip_start[t]), s, epoch, stages, ring, rstate, rstate_stride, head,
                              ctl, gstep, hdr, flags, halo, wait_iters);
    }
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int prev = atomicAdd(&hdr->done_ctas, 1u);
        if (prev == gridDim.x - 1) {
            // last CTA out: reset the scheduler for the next launch, advance the epoch
            hdr->next_item = 0;
            hdr->done_ctas = 0;
            hdr->epoch = ctl.epoch;
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

static int64_t strip_rows(const smo_tensor &t) {
    int64_t align = 1;
    if (t.kind == SMO_KIND_POOLED8) align = t.q_block / gcd64(t.comp_cols, t.q_block);
    int64_t L = (kStripRows + align - 1) / align * align;
    return L < t.comp_rows ? L : t.comp_rows;
}

bool fused_takes(const smo_tensor &t) {
    if (t.kind != SMO_KIND_POOLED8 && t.kind != SMO_KIND_POOLED32) return false;
    if (t.flags & SMO_FLAG_GENERAL_PATH) return false;
    if (t.rows <= 0 || t.cols <= 0 || t.comp_rows <= 0 || t.comp_cols <= 0) return false;
    if (t.rows % t.comp_rows != 0 || t.cols % t.comp_cols != 0) return false;
    const int64_t kh = t.rows / t.comp_rows, kw = t.cols / t.comp_cols;
    if (!supported_window(kh) || !supported_window(kw)) return false;
    if (t.cols <= 128) return false;                  // torch's small-output interpolation order
    if (t.comp_cols % 16 != 0) return false;          // 16-byte TMA / cp.async granules of every row
    if (t.comp_cols > kMaxFusedCols) return false;
    if (t.comp_rows * t.comp_cols >= ((int64_t)1 << 31)) return false;  // 32-bit cell indices
    if (t.kind == SMO_KIND_POOLED8 && t.q_block > t.comp_cols) return false;
    if ((uintptr_t)t.param % 16 || (uintptr_t)t.grad % 16) return false;
    if (t.kind == SMO_KIND_POOLED8) {
        if ((uintptr_t)t.m_q_in % 16 || (uintptr_t)t.v_q_in % 16) return false;
        if ((uintptr_t)t.m_s_in % 4 || (uintptr_t)t.v_s_in % 4) return false;
    } else {
        if ((uintptr_t)t.m_in % 16 || (uintptr_t)t.v_in % 16) return false;
    }
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

static int64_t num_strips(const smo_tensor &t) {
    const int64_t L = strip_rows(t);
    return (t.comp_rows + L - 1) / L;
}

static int window_key(const smo_tensor &t) {
    return (int)((t.rows / t.comp_rows) * 16 + (t.cols / t.comp_cols));
}

// bytes of one row-state buffer (see RowState)
static int64_t row_state_bytes(const smo_tensor &t) {
    const int64_t w = t.comp_cols;
    if (t.kind == SMO_KIND_POOLED8) return 2 * w + 8 * (w / t.q_block + 2);
    return 8 * w;
}

static int device_sm_count() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return 148;
    return sms;
}

static inline size_t align_up(size_t x) { return (x + kScratchAlign - 1) / kScratchAlign * kScratchAlign; }

// Workspace after the header: [flags: one word per strip][published rows:
// 2*w floats per strip][head rows: 4*max_w floats per CTA].  Sized for the
// whole set; each window-group launch reuses the space.
size_t fused_workspace_size(const smo_tensor *t, int32_t n) {
    size_t strips = 0, halo_floats = 0;
    int64_t max_w = 0;
    for (int32_t i = 0; i < n; i++) {
        if (!fused_takes(t[i])) continue;
        const int64_t s = num_strips(t[i]);
        strips += (size_t)s;
        halo_floats += (size_t)s * 2 * (size_t)t[i].comp_cols;
        max_w = max_w > t[i].comp_cols ? max_w : t[i].comp_cols;
    }
    if (!strips) return 0;
    const size_t ctas = (size_t)device_sm_count() * kMaxFusedCtasPerSm;
    return align_up(strips * sizeof(unsigned int)) + align_up(halo_floats * sizeof(float)) +
           ctas * 4 * (size_t)max_w * sizeof(float);
}

template <int KH, int KW>
static int launch_fused_group(FusedBatch &b, int64_t max_w, int64_t max_rs, size_t halo_floats, char *ws,
                              cudaStream_t stream) {
    using G = Geo<KH, KW>;
    const int rstride = (int)((max_rs + 15) / 16 * 16);
    const size_t smem = (size_t)kStages * G::STAGE_FLOATS * sizeof(float) + 3 * (size_t)max_w * sizeof(float2) +
                        2 * (size_t)rstride;
    auto kern = fused_step_kernel<KH, KW>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return (g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    per_sm = per_sm < 1 ? 1 : (per_sm > kMaxFusedCtasPerSm ? kMaxFusedCtasPerSm : per_sm);
    const int64_t strips = b.strip_start[b.n];
    int64_t grid = (int64_t)device_sm_count() * per_sm;
    grid = grid < strips ? grid : strips;
    WsHeader *hdr = (WsHeader *)ws;
    char *body = ws + kWsHeader;
    unsigned int *flags = (unsigned int *)body;
    body += align_up((size_t)strips * sizeof(unsigned int));
    float *halo = (float *)body;
    body += align_up(halo_floats * sizeof(float));
    float *heads = (float *)body;
    kern<<<(unsigned)grid, kThreads, smem, stream>>>(b, hdr, flags, halo, heads, 4 * max_w, (int32_t)max_w, rstride,
                                                     kDefaultWaitIters);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    g_launches++;
    return SMO_OK;
}

static int dispatch(int key, FusedBatch &b, int64_t max_w, int64_t max_rs, size_t halo_floats, char *ws,
                    cudaStream_t stream) {
    switch (key) {
#define SMO_FUSED_CASE(KH, KW) \
    case KH * 16 + KW: return launch_fused_group<KH, KW>(b, max_w, max_rs, halo_floats, ws, stream);
        SMO_FUSED_CASE(2, 2) SMO_FUSED_CASE(2, 4) SMO_FUSED_CASE(2, 8)
        SMO_FUSED_CASE(4, 2) SMO_FUSED_CASE(4, 4) SMO_FUSED_CASE(4, 8)
        SMO_FUSED_CASE(8, 2) SMO_FUSED_CASE(8, 4) SMO_FUSED_CASE(8, 8)
#undef SMO_FUSED_CASE
        default: return SMO_ERR_INVALID;
    }
}

static void fill(FusedDesc &f, const smo_tensor &t, int64_t halo_off) {
    memset(&f, 0, sizeof(f));
    f.p = t.param;
    f.g = t.grad;
    f.mq_in = t.m_q_in; f.ms_in = t.m_s_in; f.vq_in = t.v_q_in; f.vs_in = t.v_s_in;
    f.mq_out = t.m_q_out; f.ms_out = t.m_s_out; f.vq_out = t.v_q_out; f.vs_out = t.v_s_out;
    f.m_in = t.m_in; f.v_in = t.v_in; f.m_out = t.m_out; f.v_out = t.v_out;
    f.H = t.rows; f.W = t.cols; f.band = t.interp_band;
    f.h = (int32_t)t.comp_rows; f.w = (int32_t)t.comp_cols;
    f.B = t.kind == SMO_KIND_POOLED8 ? (int32_t)t.q_block : 1;
    f.L = (int32_t)strip_rows(t);
    f.div_B = make_fast_div((uint32_t)f.B);
    f.halo_off = halo_off;
    f.kind = t.kind;
    f.hp = t.hp;
}

int fused_step(const smo_tensor *t, int32_t n, char *ws, size_t ws_bytes, cudaStream_t stream) {
    (void)ws_bytes;
    static thread_local FusedBatch batch;
    // one launch per window shape (template instance), at most kMaxFused tensors each
    std::vector<char> done((size_t)n);
    for (int32_t i = 0; i < n; i++) done[i] = !fused_takes(t[i]);
    for (int32_t i = 0; i < n; i++) {
        if (done[i]) continue;
        const int key = window_key(t[i]);
        batch.n = 0;
        batch.strip_start[0] = 0;
        int64_t halo_off = 0, max_w = 0, max_rs = 0;
        for (int32_t k = i; k < n && batch.n < kMaxFused; k++) {
            if (done[k] || window_key(t[k]) != key) continue;
            FusedDesc &f = batch.d[batch.n];
            fill(f, t[k], halo_off);
            const int64_t s = num_strips(t[k]);
            halo_off += s * 2 * t[k].comp_cols;
            max_w = max_w > t[k].comp_cols ? max_w : t[k].comp_cols;
            const int64_t rs = row_state_bytes(t[k]);
            max_rs = max_rs > rs ? max_rs : rs;
            batch.strip_start[batch.n + 1] = batch.strip_start[batch.n] + s;
            batch.n++;
            done[k] = 1;
        }
        // tensors of the same window left over (batch full) start a new batch when
        // the scan reaches them
        const int st = dispatch(key, batch, max_w, max_rs, (size_t)halo_off, ws, stream);
        if (st != SMO_OK) return st;
    }
    return SMO_OK;
}

}  // namespace smo
