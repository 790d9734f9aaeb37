/*
 * smo_oracle.c -- CPU restatement of the SMO / SMO8bit optimizer step.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
 * reference legs may load it.  The product path never calls it.
 *
 * It restates, in plain C with every rounding step explicit, the fp32
 * arithmetic that the reference's PyTorch code performs on the CPU:
 *
 *   smo/optimizers/spatial_8bit.py:124-299   SMO8bit.step (monolithic)
 *   smo/optimizers/spatial_8bit.py:307-374   SMO8bit._step_banded (low_peak)
 *   smo/optimizers/spatial_8bit.py:85-122    _quantize_blockwise / _dequantize_blockwise
 *   smo/optimizers/spatial.py:82-208         SMO.step (fp32 pooled moments)
 *   smo/optimizers/_spatial_utils.py:45-176  exact / adaptive pooling, bilinear upsample
 *
 * The reference delegates its arithmetic to torch (no version pinned beyond
 * torch>=2.0.0, setup.py:11-13); the op order below was established against
 * torch 2.11.0 CPU kernels and is pinned by tests/golden/:
 *
 *   grad.add(p, alpha=wd)            x = fma(wd, p, g)
 *   m.mul_(b).add_(u, alpha=1-b)     m = fma(1-b, u, m*b)
 *   v.mul_(b).addcmul_(g, g, 1-b)    v = fma((1-b)*g, g, v*b)
 *   avg_pool2d (exact window)        sequential row-major sum from +0, / (kh*kw)
 *   adaptive_avg_pool2d              sequential row-major sum from +0, / bin_h / bin_w
 *   interpolate(bilinear, ac=False)  src = fma(in/out, o+0.5, -0.5) clamped at 0;
 *                                    H+W > 128: width pass then height pass,
 *                                      t = fma(a, w0, b*w1), out = fma(t0, h0, t1*h1)
 *                                    H+W <= 128 (channels-last kernel):
 *                                      out = fma(d, h1w1, fma(c, h1w0, fma(a, h0w0, b*h0w1)))
 *   quantize                          s = max(absmax, 1e-12); q = rint((x/s)*127),
 *                                    dead-zone lift, clamp +-127
 *   dequantize                        q * (s/127)
 *   addcdiv_(m, d, value=-ss)         p + ((-ss)*m)/d,  d = sqrt(v)/sqrt(bc2) + eps
 *
 * One deliberate difference: sqrtf here is IEEE correctly rounded, while
 * torch's vectorised CPU sqrt differs from it by 1 ulp on about 0.6% of
 * elements.  That touches only the parameter write (never the int8 codes) and
 * stays far inside the rtol 1e-5 parameter tolerance.
 *
 * Half-precision parameters (bf16 / fp16, oracle_hyper.dtype): the reference
 * then computes in the parameter's dtype (its state too: moments and block
 * scales), and torch's CPU kernels for those dtypes evaluate every op in fp32
 * exactly as above and round the op's result to the dtype once (rd()).  Two
 * scalar rules were established against torch 2.11 CPU: the alpha of
 * add/add_ (the weight decay and the EMA's 1-beta) is rounded to the dtype
 * first; every other scalar (mul_, addcmul_'s value, addcdiv_'s value, the
 * divisor and eps) stays fp32.  With dtype 0 (fp32) rd() is the identity and
 * everything reduces to the sequence above.
 *
 * Build with -ffp-contract=off: every fused multiply-add is written as fmaf.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
    float beta1, omb1;      /* (float)beta1, (float)(1 - beta1) */
    float beta2, omb2;      /* (float)beta2, (float)(1 - beta2) */
    float wd;               /* (float)weight_decay */
    int32_t wd_on;          /* weight_decay != 0 (the reference skips the add otherwise) */
    float neg_step;         /* (float)(-(lr / (1 - beta1**step))) */
    float sqrt_bc2;         /* (float)sqrt(1 - beta2**step) */
    float eps;              /* (float)eps */
    int32_t dtype;          /* parameter dtype: 0 fp32, 1 bf16, 2 fp16 */
} oracle_hyper;

/* fp32 -> bf16 / fp16 -> fp32, round to nearest even (the dtype's value as a float) */
static inline float rd_bf16(float x)
{
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return x;           /* NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    memcpy(&x, &u, 4);
    return x;
}

static inline float rd(float x, int dtype)
{
    if (dtype == 1) return rd_bf16(x);
    if (dtype == 2) return (float)(_Float16)x;
    return x;
}

typedef struct {
    int64_t i0, i1;
    float l0, l1;
    int ident;              /* input and output extents are equal: pass-through */
} coef_t;

/* _spatial_utils.py:128-176 via torch: compute_source_index_and_lambda */
static coef_t coef_for(int64_t o, int64_t in, int64_t out)
{
    coef_t c;
    if (in == out) {
        c.i0 = c.i1 = o; c.l0 = 1.0f; c.l1 = 0.0f; c.ident = 1;
        return c;
    }
    float scale = (float)in / (float)out;
    float real = fmaf(scale, (float)o + 0.5f, -0.5f);
    if (real < 0.0f) real = 0.0f;
    int64_t i0 = (int64_t)floorf(real);
    if (i0 > in - 1) i0 = in - 1;
    float l1 = real - (float)i0;
    if (l1 < 0.0f) l1 = 0.0f;
    if (l1 > 1.0f) l1 = 1.0f;
    c.i0 = i0;
    c.i1 = i0 + (i0 < in - 1 ? 1 : 0);
    c.l1 = l1;
    c.l0 = 1.0f - l1;
    c.ident = 0;
    return c;
}

/* Row coefficients, including the reference's low_peak interpolation bands
 * (spatial_8bit.py:359-370): band b covers compact rows [s0, s1) and is
 * interpolated from rows [a, b) = [max(0,s0-1), min(h,s1+1)) onto
 * (b-a)*kh output rows.  interp_band == 0 means one monolithic interpolation. */
static coef_t row_coef(int64_t r, int64_t H, int64_t h, int64_t W, int64_t interp_band, int *small)
{
    if (interp_band <= 0) {
        *small = (H + W <= 128);
        return coef_for(r, h, H);
    }
    int64_t kh = H / h;
    int64_t s0 = ((r / kh) / interp_band) * interp_band;
    int64_t s1 = s0 + interp_band < h ? s0 + interp_band : h;
    int64_t a = s0 > 0 ? s0 - 1 : 0;
    int64_t b = s1 + 1 < h ? s1 + 1 : h;
    int64_t n = b - a;
    *small = (n * kh + W <= 128);
    coef_t c = coef_for(r - a * kh, n, n * kh);
    c.i0 += a;
    c.i1 += a;
    return c;
}

static inline float interp_generic(const float *src, int64_t w, coef_t rc, coef_t cc, int64_t r, int64_t q)
{
    if (rc.ident && cc.ident) return src[r * w + q];
    if (rc.ident) {
        const float *s = src + r * w;
        return fmaf(s[cc.i0], cc.l0, s[cc.i1] * cc.l1);
    }
    if (cc.ident)
        return fmaf(src[rc.i0 * w + q], rc.l0, src[rc.i1 * w + q] * rc.l1);
    const float *s0 = src + rc.i0 * w, *s1 = src + rc.i1 * w;
    float t0 = fmaf(s0[cc.i0], cc.l0, s0[cc.i1] * cc.l1);
    float t1 = fmaf(s1[cc.i0], cc.l0, s1[cc.i1] * cc.l1);
    return fmaf(t0, rc.l0, t1 * rc.l1);
}

static inline float interp_small(const float *src, int64_t w, coef_t rc, coef_t cc)
{
    float w00 = rc.l0 * cc.l0, w01 = rc.l0 * cc.l1, w10 = rc.l1 * cc.l0, w11 = rc.l1 * cc.l1;
    float a = src[rc.i0 * w + cc.i0], b = src[rc.i0 * w + cc.i1];
    float c = src[rc.i1 * w + cc.i0], d = src[rc.i1 * w + cc.i1];
    return fmaf(d, w11, fmaf(c, w10, fmaf(a, w00, b * w01)));
}

/* ------------------------------------------------------------------ */
/* primitives                                                          */
/* ------------------------------------------------------------------ */

static inline float decayed(float g, float p, const oracle_hyper *hp)
{
    return hp->wd_on ? rd(fmaf(rd(hp->wd, hp->dtype), p, g), hp->dtype) : g;
}

/* _spatial_utils.py:72-91: stack(g, g*g) then avg_pool2d (exact) or
 * adaptive_avg_pool2d, on x = g + wd*p. */
void oracle_pool_pair(const float *g, const float *p, int64_t H, int64_t W, int64_t h, int64_t w,
                      const oracle_hyper *hp, float *out_g, float *out_g2)
{
    int exact = (h > 0 && w > 0 && H % h == 0 && W % w == 0);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < h; i++) {
        int64_t r0, r1;
        if (exact) { r0 = i * (H / h); r1 = r0 + H / h; }
        else { r0 = (i * H) / h; r1 = ((i + 1) * H + h - 1) / h; }
        for (int64_t j = 0; j < w; j++) {
            int64_t c0, c1;
            if (exact) { c0 = j * (W / w); c1 = c0 + W / w; }
            else { c0 = (j * W) / w; c1 = ((j + 1) * W + w - 1) / w; }
            float s1 = 0.0f, s2 = 0.0f;
            for (int64_t r = r0; r < r1; r++)
                for (int64_t c = c0; c < c1; c++) {
                    float x = decayed(g[r * W + c], p[r * W + c], hp);
                    s1 = s1 + x;
                    s2 = s2 + rd(x * x, hp->dtype);     /* torch.square, then the pool */
                }
            if (exact) {
                float div = (float)((r1 - r0) * (c1 - c0));
                out_g[i * w + j] = rd(s1 / div, hp->dtype);
                out_g2[i * w + j] = rd(s2 / div, hp->dtype);
            } else {
                float dh = (float)(r1 - r0), dw = (float)(c1 - c0);
                out_g[i * w + j] = rd(s1 / dh / dw, hp->dtype);
                out_g2[i * w + j] = rd(s2 / dh / dw, hp->dtype);
            }
        }
    }
}

/* spatial_8bit.py:85-107.  q holds nb*B codes (the padded tail is coded too);
 * the scales are in the moments' dtype. */
void oracle_quantize_dt(const float *x, int64_t n, int64_t B, int8_t *q, float *s, int dtype)
{
    int64_t nb = (n + B - 1) / B;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; b++) {
        float m = 0.0f;
        for (int64_t k = 0; k < B; k++) {
            int64_t i = b * B + k;
            float a = i < n ? fabsf(x[i]) : 0.0f;
            if (a > m || a != a) m = a;
            if (m != m) break;
        }
        float sc = rd((m < 1e-12f) ? 1e-12f : m, dtype);
        s[b] = sc;
        for (int64_t k = 0; k < B; k++) {
            int64_t i = b * B + k;
            float v = i < n ? x[i] : 0.0f;
            float r = rintf(rd(rd(v / sc, dtype) * 127.0f, dtype));
            if (r == 0.0f && v != 0.0f && v == v) r = v > 0.0f ? 1.0f : -1.0f;
            if (r > 127.0f) r = 127.0f;
            if (r < -127.0f) r = -127.0f;
            q[i] = (r == r) ? (int8_t)r : (int8_t)0;
        }
    }
}

void oracle_quantize(const float *x, int64_t n, int64_t B, int8_t *q, float *s)
{
    oracle_quantize_dt(x, n, B, q, s, 0);
}

/* spatial_8bit.py:109-122 (dequantised to the moments' dtype) */
void oracle_dequantize_dt(const int8_t *q, const float *s, int64_t n, int64_t B, float *out, int dtype)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        float t = rd(s[i / B] / 127.0f, dtype);
        out[i] = rd((float)q[i] * t, dtype);
    }
}

void oracle_dequantize(const int8_t *q, const float *s, int64_t n, int64_t B, float *out)
{
    oracle_dequantize_dt(q, s, n, B, out, 0);
}

/* _spatial_utils.py:128-176 (one channel), with the low_peak band emulation. */
void oracle_upsample(const float *src, int64_t h, int64_t w, int64_t H, int64_t W,
                     int64_t interp_band, float *out)
{
    int same = (h == H && w == W && interp_band <= 0);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < H; r++) {
        int small;
        coef_t rc = row_coef(r, H, h, W, interp_band, &small);
        for (int64_t q = 0; q < W; q++) {
            if (same) { out[r * W + q] = src[r * w + q]; continue; }
            coef_t cc = coef_for(q, w, W);
            out[r * W + q] = small ? interp_small(src, w, rc, cc)
                                   : interp_generic(src, w, rc, cc, r, q);
        }
    }
}

/* the shared Adam write (spatial_8bit.py:289-297, :369-370; spatial.py:192-206) */
static inline float adam_write(float p, float mh, float vh, const oracle_hyper *hp)
{
    const int dt = hp->dtype;
    float d = rd(rd(rd(sqrtf(vh), dt) / hp->sqrt_bc2, dt) + hp->eps, dt);
    float u = (hp->neg_step * mh) / d;
    return rd(p + u, dt);
}

/* EMA of the compact moments and the parameter write for a pooled tensor whose
 * post-EMA compact moments are m, v (fp32, h*w each). */
static void pooled_write(float *p, const float *m, const float *v, int64_t H, int64_t W,
                         int64_t h, int64_t w, int64_t interp_band, const oracle_hyper *hp)
{
    int same = (h == H && w == W && interp_band <= 0);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < H; r++) {
        int small;
        coef_t rc = row_coef(r, H, h, W, interp_band, &small);
        for (int64_t q = 0; q < W; q++) {
            float mh, vh;
            if (same) {
                mh = m[r * w + q];
                vh = v[r * w + q];
            } else {
                coef_t cc = coef_for(q, w, W);
                if (small) {
                    mh = interp_small(m, w, rc, cc);
                    vh = interp_small(v, w, rc, cc);
                } else {
                    mh = interp_generic(m, w, rc, cc, r, q);
                    vh = interp_generic(v, w, rc, cc, r, q);
                }
                mh = rd(mh, hp->dtype);
                vh = rd(vh, hp->dtype);
            }
            if (vh < 0.0f) vh = 0.0f;           /* clamp(min=0), NaN passes through */
            p[r * W + q] = adam_write(p[r * W + q], mh, vh, hp);
        }
    }
}

/* ------------------------------------------------------------------ */
/* composite steps                                                     */
/* ------------------------------------------------------------------ */

/* SMO8bit pooled tensor, monolithic (interp_band = 0) or low_peak banded
 * (interp_band = band_comp of spatial_8bit.py:359).  Codes and scales are
 * updated in place; q holds nb*B codes. */
int oracle_smo8bit_pooled_step(float *p, const float *g, int8_t *mq, float *ms, int8_t *vq, float *vs,
                               int64_t H, int64_t W, int64_t h, int64_t w, int64_t B,
                               int64_t interp_band, const oracle_hyper *hp)
{
    int64_t C = h * w;
    float *gm = malloc(sizeof(float) * C), *g2 = malloc(sizeof(float) * C);
    float *m = malloc(sizeof(float) * C), *v = malloc(sizeof(float) * C);
    if (!gm || !g2 || !m || !v) { free(gm); free(g2); free(m); free(v); return 1; }
    const int dt = hp->dtype;
    oracle_pool_pair(g, p, H, W, h, w, hp, gm, g2);
    oracle_dequantize_dt(mq, ms, C, B, m, dt);
    oracle_dequantize_dt(vq, vs, C, B, v, dt);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < C; i++) {
        m[i] = rd(fmaf(rd(hp->omb1, dt), gm[i], rd(m[i] * hp->beta1, dt)), dt);
        v[i] = rd(fmaf(rd(hp->omb2, dt), g2[i], rd(v[i] * hp->beta2, dt)), dt);
    }
    oracle_quantize_dt(m, C, B, mq, ms, dt);
    oracle_quantize_dt(v, C, B, vq, vs, dt);
    pooled_write(p, m, v, H, W, h, w, interp_band, hp);
    free(gm); free(g2); free(m); free(v);
    return 0;
}

/* SMO (fp32 pooled moments, spatial.py:82-208); m, v are h*w, updated in place. */
int oracle_smo_pooled_step(float *p, const float *g, float *m, float *v,
                           int64_t H, int64_t W, int64_t h, int64_t w, const oracle_hyper *hp)
{
    int64_t C = h * w;
    float *gm = malloc(sizeof(float) * C), *g2 = malloc(sizeof(float) * C);
    if (!gm || !g2) { free(gm); free(g2); return 1; }
    const int dt = hp->dtype;
    oracle_pool_pair(g, p, H, W, h, w, hp, gm, g2);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < C; i++) {
        m[i] = rd(fmaf(rd(hp->omb1, dt), gm[i], rd(m[i] * hp->beta1, dt)), dt);
        v[i] = rd(fmaf(rd(hp->omb2, dt), g2[i], rd(v[i] * hp->beta2, dt)), dt);
    }
    pooled_write(p, m, v, H, W, h, w, 0, hp);
    free(gm); free(g2);
    return 0;
}

/* dense Adam moments (spatial_8bit.py:278-283, spatial.py:184-189) */
void oracle_dense_step(float *p, const float *g, float *m, float *v, int64_t n, const oracle_hyper *hp)
{
    const int dt = hp->dtype;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        float x = decayed(g[i], p[i], hp);
        m[i] = rd(fmaf(rd(hp->omb1, dt), x, rd(m[i] * hp->beta1, dt)), dt);   /* add_(alpha): dtype alpha */
        v[i] = rd(fmaf(hp->omb2 * x, x, rd(v[i] * hp->beta2, dt)), dt);       /* addcmul_(value): fp32 value */
        p[i] = adam_write(p[i], m[i], v[i], hp);
    }
}

/* full-resolution int8 moments, "quant_only" groups (spatial_8bit.py:263-277) */
int oracle_quant_only_step(float *p, const float *g, int8_t *mq, float *ms, int8_t *vq, float *vs,
                           int64_t n, int64_t B, const oracle_hyper *hp)
{
    float *m = malloc(sizeof(float) * n), *v = malloc(sizeof(float) * n);
    if (!m || !v) { free(m); free(v); return 1; }
    const int dt = hp->dtype;
    oracle_dequantize_dt(mq, ms, n, B, m, dt);
    oracle_dequantize_dt(vq, vs, n, B, v, dt);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        float x = decayed(g[i], p[i], hp);
        m[i] = rd(fmaf(rd(hp->omb1, dt), x, rd(m[i] * hp->beta1, dt)), dt);
        v[i] = rd(fmaf(hp->omb2 * x, x, rd(v[i] * hp->beta2, dt)), dt);
    }
    oracle_quantize_dt(m, n, B, mq, ms, dt);
    oracle_quantize_dt(v, n, B, vq, vs, dt);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++)
        p[i] = adam_write(p[i], m[i], v[i], hp);
    free(m); free(v);
    return 0;
}

int oracle_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
