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
#include <cstring>
#include <vector>

#include "smo_common.cuh"
#include "smo_internal.cuh"

namespace smo {

constexpr int kFusedThreads = 256;
constexpr int kMaxFused = 112;
constexpr int64_t kStripRows = 16;          // target compact rows per strip
constexpr int64_t kMaxFusedCols = 4096;     // compact columns (shared memory: 48 B per column, 192 KB max)
constexpr int64_t kDefaultWaitIters = 1 << 22;

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
    int64_t H, W, h, w, B, band;
    int64_t L;         // compact rows per strip
    int64_t halo_off;  // float offset of this tensor's published rows in the halo area
    float col_scale;   // (float)w / (float)W, correctly rounded
    int32_t kind;
    smo_hyper hp;
};

struct FusedBatch {
    int32_t n;
    int64_t strip_start[kMaxFused + 1];
    FusedDesc d[kMaxFused];
};
static_assert(sizeof(FusedBatch) < 32000, "kernel parameter batch must stay below 32 KB");

// ---------------------------------------------------------------- memory helpers

template <int KW>
__device__ __forceinline__ void load_row(const float *ptr, float (&v)[KW]) {
    if constexpr (KW % 4 == 0) {
#pragma unroll
        for (int k = 0; k < KW / 4; k++) {
            float4 t = __ldcs(reinterpret_cast<const float4 *>(ptr) + k);
            v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
        }
    } else if constexpr (KW == 2) {
        float2 t = __ldcs(reinterpret_cast<const float2 *>(ptr));
        v[0] = t.x; v[1] = t.y;
    } else {
#pragma unroll
        for (int k = 0; k < KW; k++) v[k] = __ldcs(ptr + k);
    }
}

// parameter loads: default caching (phase 1, to be re-read) / last use (phase 2)
template <int KW>
__device__ __forceinline__ void load_param(const float *ptr, float (&v)[KW], bool last_use) {
    if constexpr (KW % 4 == 0) {
#pragma unroll
        for (int k = 0; k < KW / 4; k++) {
            const float4 *q = reinterpret_cast<const float4 *>(ptr) + k;
            float4 t = last_use ? __ldlu(q) : __ldcg(q);
            v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
        }
    } else if constexpr (KW == 2) {
        const float2 *q = reinterpret_cast<const float2 *>(ptr);
        float2 t = last_use ? __ldlu(q) : __ldcg(q);
        v[0] = t.x; v[1] = t.y;
    } else {
#pragma unroll
        for (int k = 0; k < KW; k++) v[k] = last_use ? __ldlu(ptr + k) : __ldcg(ptr + k);
    }
}

template <int KW>
__device__ __forceinline__ void store_param(float *ptr, const float (&v)[KW]) {
    if constexpr (KW % 4 == 0) {
#pragma unroll
        for (int k = 0; k < KW / 4; k++)
            __stcs(reinterpret_cast<float4 *>(ptr) + k, make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]));
    } else if constexpr (KW == 2) {
        __stcs(reinterpret_cast<float2 *>(ptr), make_float2(v[0], v[1]));
    } else {
#pragma unroll
        for (int k = 0; k < KW; k++) __stcs(ptr + k, v[k]);
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

// ---------------------------------------------------------------- phases

// Phase 1 of compact row c: post-EMA m, v into Mrow/Vrow (shared memory).
// `own` rows also write the fp32 state (POOLED32); look-ahead rows only read.
template <int KH, int KW>
__device__ __forceinline__ void phase1(const FusedDesc &d, int64_t c, float *Mrow, float *Vrow, bool own) {
    const int64_t w = d.w, W = d.W;
    const float *gb = d.g + c * KH * W;
    const float *pb = d.p + c * KH * W;
    const int64_t cell0 = c * w;
    const smo_hyper &hp = d.hp;
    const bool q8 = (d.kind == SMO_KIND_POOLED8);
    const float div = (float)(KH * KW);
    for (int64_t j = threadIdx.x; j < w; j += kFusedThreads) {
        float s1 = 0.0f, s2 = 0.0f;
        float gv[KH][KW], pv[KH][KW];
#pragma unroll
        for (int i = 0; i < KH; i++) load_row<KW>(gb + i * W + j * KW, gv[i]);
        if (hp.wd_on) {
#pragma unroll
            for (int i = 0; i < KH; i++) load_param<KW>(pb + i * W + j * KW, pv[i], false);
        }
#pragma unroll
        for (int i = 0; i < KH; i++) {
#pragma unroll
            for (int k = 0; k < KW; k++) {
                const float x = hp.wd_on ? __fmaf_rn(hp.weight_decay, pv[i][k], gv[i][k]) : gv[i][k];
                s1 = __fadd_rn(s1, x);
                s2 = __fadd_rn(s2, __fmul_rn(x, x));
            }
        }
        const float mean = __fdiv_rn(s1, div), sq = __fdiv_rn(s2, div);
        const int64_t cell = cell0 + j;
        float m, v;
        if (q8) {
            const int64_t b = cell / d.B;
            m = dequant1(d.mq_in[cell], dequant_step(d.ms_in[b]));
            v = dequant1(d.vq_in[cell], dequant_step(d.vs_in[b]));
        } else {
            m = d.m_in[cell];
            v = d.v_in[cell];
        }
        m = ema(m, mean, hp.beta1, hp.omb1);
        v = ema(v, sq, hp.beta2, hp.omb2);
        Mrow[j] = m;
        Vrow[j] = v;
        if (own && !q8) {
            d.m_out[cell] = m;
            d.v_out[cell] = v;
        }
    }
}

// Requantise the int8 blocks that compact row c completes.  A block spans at
// most two compact rows (q_block <= w), both still in the ring.
__device__ __forceinline__ void requant_row(const FusedDesc &d, int64_t c, const float *Mc, const float *Vc,
                                            const float *Mp, const float *Vp) {
    const int64_t w = d.w, B = d.B, C = d.h * d.w;
    int64_t b_lo = (c * w) / B;
    int64_t b_hi = ((c + 1) * w) / B;
    if (c == d.h - 1 && C % B != 0) b_hi = C / B + 1;  // the zero-padded last block
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t b = b_lo + warp; b < b_hi; b += kFusedThreads / 32) {
        float am = 0.0f, av = 0.0f;
        for (int64_t k = lane; k < B; k += 32) {
            const int64_t cell = b * B + k;
            if (cell >= C) break;
            const int64_t row = cell / w, col = cell - row * w;
            const float m = row == c ? Mc[col] : Mp[col];
            const float v = row == c ? Vc[col] : Vp[col];
            am = absmax_acc(am, m);
            av = absmax_acc(av, v);
        }
        const float sm = block_scale(warp_absmax(am)), sv = block_scale(warp_absmax(av));
        for (int64_t k = lane; k < B; k += 32) {
            const int64_t cell = b * B + k;
            float m = 0.0f, v = 0.0f;
            if (cell < C) {
                const int64_t row = cell / w, col = cell - row * w;
                m = row == c ? Mc[col] : Mp[col];
                v = row == c ? Vc[col] : Vp[col];
            }
            d.mq_out[cell] = quantize1(m, sm);
            d.vq_out[cell] = quantize1(v, sv);
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

// Phase 2 of compact row c: the KH parameter rows, from the post-EMA rows
// c-1 (M[0]), c (M[1]), c+1 (M[2]); absent rows are never addressed.
template <int KH, int KW>
__device__ __forceinline__ void phase2(const FusedDesc &d, int64_t c, const float *const M[3], const float *const V[3],
                                       RowCo *rowco) {
    const int64_t w = d.w, W = d.W;
    if (threadIdx.x < KH) {
        int small;
        const Coef rc = row_coef(c * KH + threadIdx.x, d.H, d.h, d.W, d.band, small);
        RowCo r;
        r.s0 = (int)(rc.i0 - (c - 1));
        r.s1 = (int)(rc.i1 - (c - 1));
        r.l0 = rc.l0;
        r.l1 = rc.l1;
        rowco[threadIdx.x] = r;
    }
    __syncthreads();
    const smo_hyper &hp = d.hp;
    for (int64_t j = threadIdx.x; j < w; j += kFusedThreads) {
        // width pass for the three compact rows
        float hm[3][KW], hv[3][KW];
#pragma unroll
        for (int t = 0; t < KW; t++) {
            const int64_t q = j * KW + t;
            float real = __fmaf_rn(d.col_scale, __fadd_rn((float)q, 0.5f), -0.5f);
            real = real < 0.0f ? 0.0f : real;
            int64_t i0 = (int64_t)floorf(real);
            i0 = i0 > w - 1 ? w - 1 : i0;
            float l1 = __fsub_rn(real, (float)i0);
            l1 = l1 < 0.0f ? 0.0f : (l1 > 1.0f ? 1.0f : l1);
            const float l0 = __fsub_rn(1.0f, l1);
            const int64_t i1 = i0 + (i0 < w - 1 ? 1 : 0);
#pragma unroll
            for (int s = 0; s < 3; s++) {
                if (M[s]) {
                    hm[s][t] = __fmaf_rn(M[s][i0], l0, __fmul_rn(M[s][i1], l1));
                    hv[s][t] = __fmaf_rn(V[s][i0], l0, __fmul_rn(V[s][i1], l1));
                } else {
                    hm[s][t] = 0.0f;
                    hv[s][t] = 0.0f;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < KH; i++) {
            const RowCo rc = rowco[i];
            float *prow = d.p + (c * KH + i) * W + j * KW;
            float pv[KW];
            load_param<KW>(prow, pv, true);
#pragma unroll
            for (int t = 0; t < KW; t++) {
                const float a_m = rc.s0 == 0 ? hm[0][t] : hm[1][t];
                const float b_m = rc.s1 == 1 ? hm[1][t] : hm[2][t];
                const float a_v = rc.s0 == 0 ? hv[0][t] : hv[1][t];
                const float b_v = rc.s1 == 1 ? hv[1][t] : hv[2][t];
                const float mh = __fmaf_rn(a_m, rc.l0, __fmul_rn(b_m, rc.l1));
                const float vh = __fmaf_rn(a_v, rc.l0, __fmul_rn(b_v, rc.l1));
                pv[t] = adam_write(pv[t], mh, clamp_min0(vh), hp);
            }
            store_param<KW>(prow, pv);
        }
    }
    __syncthreads();
}

template <int KH, int KW>
__device__ void process_strip(const FusedDesc &d, int64_t sidx, int64_t gstrip, unsigned int epoch, float *smem,
                              RowCo *rowco, WsHeader *hdr, unsigned int *flags, float *halo, int64_t wait_iters) {
    const int64_t w = d.w, h = d.h;
    const int64_t c0 = sidx * d.L;
    const int64_t c1 = c0 + d.L < h ? c0 + d.L : h;
    const bool q8 = (d.kind == SMO_KIND_POOLED8);
    float *ring = smem;          // 3 slots x (m row, v row)
    float *head = smem + 6 * w;  // rows c0-1, c0, c0+1
    auto RM = [&](int64_t c) { return ring + 2 * (c % 3) * w; };
    auto RV = [&](int64_t c) { return ring + (2 * (c % 3) + 1) * w; };
    float *HM[3] = {head, head + 2 * w, head + 4 * w};
    float *HV[3] = {head + w, head + 3 * w, head + 5 * w};

    auto copy_row = [&](int64_t c, int slot) {
        const float *sm = RM(c), *sv = RV(c);
        for (int64_t j = threadIdx.x; j < w; j += kFusedThreads) {
            HM[slot][j] = sm[j];
            HV[slot][j] = sv[j];
        }
    };

    // first row of the strip
    phase1<KH, KW>(d, c0, RM(c0), RV(c0), true);
    __syncthreads();
    if (q8) requant_row(d, c0, RM(c0), RV(c0), nullptr, nullptr);
    copy_row(c0, 1);
    __syncthreads();

    for (int64_t c = c0 + 1; c < c1; c++) {
        phase1<KH, KW>(d, c, RM(c), RV(c), true);
        __syncthreads();
        if (q8) requant_row(d, c, RM(c), RV(c), RM(c - 1), RV(c - 1));
        if (c == c0 + 1) copy_row(c, 2);
        if (c - 1 > c0) {
            const float *M[3] = {RM(c - 2), RM(c - 1), RM(c)};
            const float *V[3] = {RV(c - 2), RV(c - 1), RV(c)};
            phase2<KH, KW>(d, c - 1, M, V, rowco);  // ends with __syncthreads
        } else {
            __syncthreads();
        }
    }

    if (c1 < h) {
        // look-ahead: the next strip's first row, from its g, p and old state
        phase1<KH, KW>(d, c1, RM(c1), RV(c1), false);
        __syncthreads();
        if (c1 == c0 + 1) copy_row(c1, 2);
        // publish this strip's last row for the next strip (after the look-ahead read)
        float *out = halo + d.halo_off + sidx * 2 * w;
        const float *sm = RM(c1 - 1), *sv = RV(c1 - 1);
        for (int64_t j = threadIdx.x; j < w; j += kFusedThreads) {
            out[j] = sm[j];
            out[w + j] = sv[j];
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            store_release(flags + gstrip, epoch);
        }
    }

    if (c1 - 1 > c0) {
        const float *M[3] = {c1 - 2 >= 0 ? RM(c1 - 2) : nullptr, RM(c1 - 1), c1 < h ? RM(c1) : nullptr};
        const float *V[3] = {c1 - 2 >= 0 ? RV(c1 - 2) : nullptr, RV(c1 - 1), c1 < h ? RV(c1) : nullptr};
        phase2<KH, KW>(d, c1 - 1, M, V, rowco);
    }

    // deferred first row: needs the previous strip's last row
    if (c0 > 0) {
        __shared__ int s_ok;
        if (threadIdx.x == 0) {
            const bool ok = bounded_wait_eq(flags + gstrip - 1, epoch, wait_iters, &hdr->error);
            if (!ok) report_error(hdr, SMO_ERR_TIMEOUT, (unsigned int)gstrip);
            s_ok = ok;
        }
        __syncthreads();
        const float *in = halo + d.halo_off + (sidx - 1) * 2 * w;
        for (int64_t j = threadIdx.x; j < w; j += kFusedThreads) {
            HM[0][j] = s_ok ? __ldcg(in + j) : 0.0f;
            HV[0][j] = s_ok ? __ldcg(in + w + j) : 0.0f;
        }
        __syncthreads();
    }
    {
        const float *M[3] = {c0 > 0 ? HM[0] : nullptr, HM[1], c0 + 1 < h ? HM[2] : nullptr};
        const float *V[3] = {c0 > 0 ? HV[0] : nullptr, HV[1], c0 + 1 < h ? HV[2] : nullptr};
        phase2<KH, KW>(d, c0, M, V, rowco);
    }
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
__global__ void __launch_bounds__(kFusedThreads) fused_step_kernel(const __grid_constant__ FusedBatch b,
                                                                    WsHeader *hdr, unsigned int *flags, float *halo,
                                                                    int64_t wait_iters) {
    extern __shared__ float smem[];
    __shared__ RowCo rowco[KH];
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
        process_strip<KH, KW>(b.d[t], s - b.strip_start[t], s, epoch, smem, rowco, hdr, flags, halo, wait_iters);
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
    if (t.cols <= 128) return false;  // torch's small-output interpolation order
    if (t.comp_cols > kMaxFusedCols) return false;
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

static int64_t num_strips(const smo_tensor &t) {
    const int64_t L = strip_rows(t);
    return (t.comp_rows + L - 1) / L;
}

static int window_key(const smo_tensor &t) {
    return (int)((t.rows / t.comp_rows) * 16 + (t.cols / t.comp_cols));
}

size_t fused_workspace_size(const smo_tensor *t, int32_t n) {
    // flags (one word per strip) and published rows (2*w floats per strip),
    // sized for the whole set (each window-group launch reuses the space).
    size_t strips = 0, halo_floats = 0;
    for (int32_t i = 0; i < n; i++) {
        if (!fused_takes(t[i])) continue;
        const int64_t s = num_strips(t[i]);
        strips += (size_t)s;
        halo_floats += (size_t)s * 2 * (size_t)t[i].comp_cols;
    }
    if (!strips) return 0;
    const size_t flags_bytes = (strips * sizeof(unsigned int) + kScratchAlign - 1) / kScratchAlign * kScratchAlign;
    return flags_bytes + halo_floats * sizeof(float);
}

template <int KH, int KW>
static int launch_fused_group(FusedBatch &b, int64_t max_w, char *ws, cudaStream_t stream) {
    // ring (3 rows) + head (3 rows), each row an m and a v vector of w floats
    const size_t smem = (size_t)12 * max_w * sizeof(float);
    auto kern = fused_step_kernel<KH, KW>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFusedThreads, smem);
    if (e != cudaSuccess) return (g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (per_sm < 1) per_sm = 1;
    const int64_t strips = b.strip_start[b.n];
    int64_t grid = (int64_t)sms * per_sm;
    grid = grid < strips ? grid : strips;
    WsHeader *hdr = (WsHeader *)ws;
    size_t flags_bytes = 0;
    {
        // flags sit right after the header; published rows after the flags
        flags_bytes = ((size_t)strips * sizeof(unsigned int) + kScratchAlign - 1) / kScratchAlign * kScratchAlign;
    }
    unsigned int *flags = (unsigned int *)(ws + kWsHeader);
    float *halo = (float *)(ws + kWsHeader + flags_bytes);
    kern<<<(unsigned)grid, kFusedThreads, smem, stream>>>(b, hdr, flags, halo, kDefaultWaitIters);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (g_last_cuda_error = (int)e, SMO_ERR_CUDA);
    g_launches++;
    return SMO_OK;
}

static int dispatch(int key, FusedBatch &b, int64_t max_w, char *ws, cudaStream_t stream) {
    switch (key) {
#define SMO_FUSED_CASE(KH, KW) \
    case KH * 16 + KW: return launch_fused_group<KH, KW>(b, max_w, ws, stream);
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
    f.H = t.rows; f.W = t.cols; f.h = t.comp_rows; f.w = t.comp_cols;
    f.B = t.q_block;
    f.band = t.interp_band;
    f.L = strip_rows(t);
    f.halo_off = halo_off;
    f.col_scale = (float)t.comp_cols / (float)t.cols;
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
        int64_t halo_off = 0, max_w = 0;
        for (int32_t k = i; k < n && batch.n < kMaxFused; k++) {
            if (done[k] || window_key(t[k]) != key) continue;
            FusedDesc &f = batch.d[batch.n];
            fill(f, t[k], halo_off);
            const int64_t s = num_strips(t[k]);
            halo_off += s * 2 * t[k].comp_cols;
            max_w = max_w > t[k].comp_cols ? max_w : t[k].comp_cols;
            batch.strip_start[batch.n + 1] = batch.strip_start[batch.n] + s;
            batch.n++;
            done[k] = 1;
        }
        // tensors of the same window left over (batch full) start a new batch when
        // the scan reaches them
        const int st = dispatch(key, batch, max_w, ws, stream);
        if (st != SMO_OK) return st;
    }
    return SMO_OK;
}

}  // namespace smo
