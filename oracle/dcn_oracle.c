/*
 * CPU oracle for modulated deformable convolution (DCNv2) -- TEST INFRASTRUCTURE.
 *
 * This file restates, in plain C, the arithmetic of the reference operator
 * (TseLin-Liu/DCNv2) so that the CUDA product can be checked against it.  It is
 * used only by tests/, by __graft_entry__.smoke() as the checker, and by
 * bench.py's CPU-baseline leg.  It is never on the product path.
 *
 * Reference arithmetic followed (file:line in the reference project):
 *   bilinear sample with per-corner zero padding ..... com.cu:119-148
 *   sample position, validity rule (-1<h<H, -1<w<W),
 *   mask multiply, tap order k = i*kw + j .............. com.cu:151-195, 637-706
 *   output size (H - kh + 2p)/s + 1, bias add .......... com.cu:227-228, 114
 *   grad of the columns  gcol = W^T . gO ............... com.cu:789-793
 *   grad_offset / grad_mask (coordinate weights) ...... com.cu:388-429, 431-501
 *   grad_input scatter (gradient weights) ............. com.cu:526-550, 553-609
 *   grad_weight = gO . cols^T, grad_bias = gO . 1 ..... com.cu:818-835
 *
 * Extensions beyond the reference kernels (the reference stores but never
 * applies them, dcn_v2_mm.py:76-77): dilation enters the sample position as
 * i*dil_h / j*dil_w and the output size as (H + 2p - (dil*(k-1)+1))/s + 1;
 * deformable groups split the input channels into dg equal groups, group g
 * reading offset channels g*2*k*k + 2*t (+1) and mask channel g*k*k + t.  With
 * dil = 1 and dg = 1 both reduce exactly to the reference formulas.
 *
 * The reference's backward passes pad_h where pad_w is meant (com.cu:625); this
 * oracle uses pad_w, which equals the reference whenever pad_h == pad_w.
 *
 * Two instantiations: _f64 (double arithmetic; the parity oracle) and _f32
 * (float arithmetic, OpenMP-parallel; the CPU baseline timed by bench.py).
 *
 * Sample coordinates.  The reference forms every sample position in float32:
 * h = (h_in + i) + offset_h as one float addition (com.cu:184-185, 479-480,
 * 587-588, 688-689), and the cell (floor) and the one-sided coordinate weights
 * of the backward are discontinuous at integer positions, so the double oracle
 * forms the position the same way by default (dcn_oracle_set_coord_f32(1)):
 * a position within one float32 ulp of an integer then lands in the same cell
 * as in the reference.  dcn_oracle_set_coord_f32(0) adds in the arithmetic type
 * instead (how torchvision's double kernels do it; used for its fixtures).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
    int B, C, H, W, Co, kh, kw, sh, sw, ph, pw, dh, dw, dg;
    int Ho, Wo;
} dcn_oracle_shape;

static int out_size(int in, int k, int s, int p, int d) {
    return (in + 2 * p - (d * (k - 1) + 1)) / s + 1;
}

int dcn_oracle_out_h(int H, int kh, int sh, int ph, int dh) { return out_size(H, kh, sh, ph, dh); }
int dcn_oracle_out_w(int W, int kw, int sw, int pw, int dw) { return out_size(W, kw, sw, pw, dw); }

static int g_coord_f32 = 1;
void dcn_oracle_set_coord_f32(int on) { g_coord_f32 = on ? 1 : 0; }

/* sample position base + off, in float32 (the reference) or in the type T */
#define DCN_COORD(T, base, off) \
    (g_coord_f32 ? (T)((float)(base) + (float)(off)) : (T)(base) + (off))

int dcn_oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* threads of the CPU legs of the benchmark (a launcher may have set OMP_NUM_THREADS=1) */
void dcn_oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

#define DCN_ORACLE_DEFINE(T, SFX)                                                              \
/* bilinear value at (h, w) of one HxW plane; corners outside are 0 (com.cu:119-148) */       \
static T bilinear_##SFX(const T *im, int H, int W, T h, T w) {                                 \
    int hl = (int)floor(h), wl = (int)floor(w);                                                 \
    int hh_ = hl + 1, wh_ = wl + 1;                                                             \
    T lh = h - hl, lw = w - wl, hh = 1 - lh, hw = 1 - lw;                                       \
    T v1 = 0, v2 = 0, v3 = 0, v4 = 0;                                                           \
    if (hl >= 0 && wl >= 0) v1 = im[hl * W + wl];                                               \
    if (hl >= 0 && wh_ <= W - 1) v2 = im[hl * W + wh_];                                         \
    if (hh_ <= H - 1 && wl >= 0) v3 = im[hh_ * W + wl];                                         \
    if (hh_ <= H - 1 && wh_ <= W - 1) v4 = im[hh_ * W + wh_];                                    \
    return hh * hw * v1 + hh * lw * v2 + lh * hw * v3 + lh * lw * v4;                           \
}                                                                                              \
/* d bilinear / d h (dir 0) or d w (dir 1) (com.cu:388-429) */                                 \
static T coord_weight_##SFX(const T *im, int H, int W, T h, T w, int dir) {                     \
    if (h <= -1 || h >= H || w <= -1 || w >= W) return 0;                                       \
    int hl = (int)floor(h), wl = (int)floor(w);                                                 \
    int hh_ = hl + 1, wh_ = wl + 1;                                                             \
    T r = 0;                                                                                    \
    if (dir == 0) {                                                                             \
        if (hl >= 0 && wl >= 0) r += -(wl + 1 - w) * im[hl * W + wl];                           \
        if (hl >= 0 && wh_ <= W - 1) r += -(w - wl) * im[hl * W + wh_];                         \
        if (hh_ <= H - 1 && wl >= 0) r += (wl + 1 - w) * im[hh_ * W + wl];                      \
        if (hh_ <= H - 1 && wh_ <= W - 1) r += (w - wl) * im[hh_ * W + wh_];                    \
    } else {                                                                                    \
        if (hl >= 0 && wl >= 0) r += -(hl + 1 - h) * im[hl * W + wl];                           \
        if (hl >= 0 && wh_ <= W - 1) r += (hl + 1 - h) * im[hl * W + wh_];                      \
        if (hh_ <= H - 1 && wl >= 0) r += -(h - hl) * im[hh_ * W + wl];                         \
        if (hh_ <= H - 1 && wh_ <= W - 1) r += (h - hl) * im[hh_ * W + wh_];                    \
    }                                                                                           \
    return r;                                                                                   \
}                                                                                              \
/* cols[b][(c*kh*kw + t)][p] = mask * bilinear (com.cu:151-195); one sample b */              \
static void im2col_##SFX(const dcn_oracle_shape *s, const T *x, const T *off, const T *msk,     \
                          int b, T *cols) {                                                     \
    const int K2 = s->kh * s->kw, P = s->Ho * s->Wo, cpg = s->C / s->dg;                        \
    _Pragma("omp parallel for schedule(static)")                                               \
    for (int c = 0; c < s->C; ++c) {                                                            \
        const int g = c / cpg;                                                                  \
        const T *im = x + ((size_t)b * s->C + c) * s->H * s->W;                                 \
        const T *ob = off + ((size_t)b * s->dg + g) * 2 * K2 * P;                               \
        const T *mb = msk + ((size_t)b * s->dg + g) * K2 * P;                                   \
        for (int t = 0; t < K2; ++t) {                                                          \
            const int i = t / s->kw, j = t % s->kw;                                             \
            T *col = cols + ((size_t)c * K2 + t) * P;                                           \
            for (int p = 0; p < P; ++p) {                                                       \
                const int ho = p / s->Wo, wo = p % s->Wo;                                       \
                const T h = DCN_COORD(T, ho * s->sh - s->ph + i * s->dh, ob[(2 * t) * P + p]);          \
                const T w = DCN_COORD(T, wo * s->sw - s->pw + j * s->dw, ob[(2 * t + 1) * P + p]);      \
                T v = 0;                                                                        \
                if (h > -1 && w > -1 && h < s->H && w < s->W) v = bilinear_##SFX(im, s->H, s->W, h, w); \
                col[p] = v * mb[t * P + p];                                                     \
            }                                                                                   \
        }                                                                                       \
    }                                                                                           \
}                                                                                              \
void dcn_oracle_forward_##SFX(const T *x, const T *wt, const T *bias, const T *off,            \
                              const T *msk, T *y, const int *shape14) {                         \
    dcn_oracle_shape s;                                                                         \
    memcpy(&s, shape14, 14 * sizeof(int));                                                      \
    s.Ho = out_size(s.H, s.kh, s.sh, s.ph, s.dh);                                               \
    s.Wo = out_size(s.W, s.kw, s.sw, s.pw, s.dw);                                               \
    const int K = s.C * s.kh * s.kw, P = s.Ho * s.Wo;                                           \
    if (s.B <= 0 || P <= 0) return;                                                             \
    T *cols = (T *)malloc((size_t)K * P * sizeof(T));                                           \
    for (int b = 0; b < s.B; ++b) {                                                             \
        im2col_##SFX(&s, x, off, msk, b, cols);                                                 \
        _Pragma("omp parallel for schedule(static)")                                           \
        for (int co = 0; co < s.Co; ++co) {                                                     \
            T *yr = y + ((size_t)b * s.Co + co) * P;                                            \
            for (int p = 0; p < P; ++p) yr[p] = 0;                                              \
            const T *wr = wt + (size_t)co * K;                                                  \
            for (int k = 0; k < K; ++k) {                                                       \
                const T a = wr[k];                                                              \
                const T *cr = cols + (size_t)k * P;                                             \
                for (int p = 0; p < P; ++p) yr[p] += a * cr[p];                                 \
            }                                                                                   \
            const T bv = bias ? bias[co] : 0;                                                   \
            for (int p = 0; p < P; ++p) yr[p] += bv;                                            \
        }                                                                                       \
    }                                                                                           \
    free(cols);                                                                                 \
}                                                                                              \
void dcn_oracle_backward_##SFX(const T *x, const T *wt, const T *off, const T *msk,           \
                               const T *gy, T *gx, T *goff, T *gmask, T *gw, T *gb,             \
                               const int *shape14) {                                            \
    dcn_oracle_shape s;                                                                         \
    memcpy(&s, shape14, 14 * sizeof(int));                                                      \
    s.Ho = out_size(s.H, s.kh, s.sh, s.ph, s.dh);                                               \
    s.Wo = out_size(s.W, s.kw, s.sw, s.pw, s.dw);                                               \
    const int K2 = s.kh * s.kw, K = s.C * K2, P = s.Ho * s.Wo, cpg = s.C / s.dg;                \
    const size_t HW = (size_t)s.H * s.W;                                                        \
    memset(gx, 0, (size_t)s.B * s.C * HW * sizeof(T));                                          \
    memset(goff, 0, (size_t)s.B * s.dg * 2 * K2 * P * sizeof(T));                               \
    memset(gmask, 0, (size_t)s.B * s.dg * K2 * P * sizeof(T));                                  \
    memset(gw, 0, (size_t)s.Co * K * sizeof(T));                                                \
    if (gb) memset(gb, 0, (size_t)s.Co * sizeof(T));                                            \
    if (s.B <= 0 || P <= 0) return;                                                             \
    T *gcol = (T *)malloc((size_t)K * P * sizeof(T));                                           \
    for (int b = 0; b < s.B; ++b) {                                                             \
        const T *gyb = gy + (size_t)b * s.Co * P;                                               \
        /* gcol = W^T . gO_b  (com.cu:789-793) */                                               \
        _Pragma("omp parallel for schedule(static)")                                           \
        for (int k = 0; k < K; ++k) {                                                           \
            T *gr = gcol + (size_t)k * P;                                                       \
            for (int p = 0; p < P; ++p) gr[p] = 0;                                              \
            for (int co = 0; co < s.Co; ++co) {                                                 \
                const T a = wt[(size_t)co * K + k];                                             \
                const T *yr = gyb + (size_t)co * P;                                             \
                for (int p = 0; p < P; ++p) gr[p] += a * yr[p];                                 \
            }                                                                                   \
        }                                                                                       \
        /* grad_offset, grad_mask: sum over the channels of a group (com.cu:431-501) */        \
        _Pragma("omp parallel for schedule(static)")                                           \
        for (int gt = 0; gt < s.dg * K2; ++gt) {                                                \
            const int g = gt / K2, t = gt % K2, i = t / s.kw, j = t % s.kw;                     \
            const T *ob = off + ((size_t)b * s.dg + g) * 2 * K2 * P;                            \
            const T *mb = msk + ((size_t)b * s.dg + g) * K2 * P;                                \
            T *gob = goff + ((size_t)b * s.dg + g) * 2 * K2 * P;                                \
            T *gmb = gmask + ((size_t)b * s.dg + g) * K2 * P;                                   \
            for (int p = 0; p < P; ++p) {                                                       \
                const int ho = p / s.Wo, wo = p % s.Wo;                                         \
                const T h = DCN_COORD(T, ho * s.sh - s.ph + i * s.dh, ob[(2 * t) * P + p]);             \
                const T w = DCN_COORD(T, wo * s.sw - s.pw + j * s.dw, ob[(2 * t + 1) * P + p]);         \
                const T m = mb[t * P + p];                                                      \
                const int valid = (h > -1 && w > -1 && h < s.H && w < s.W);                     \
                T vh = 0, vw = 0, vm = 0;                                                       \
                for (int c = g * cpg; c < (g + 1) * cpg; ++c) {                                 \
                    const T gc = gcol[((size_t)c * K2 + t) * P + p];                            \
                    const T *im = x + ((size_t)b * s.C + c) * HW;                               \
                    if (valid) vm += gc * bilinear_##SFX(im, s.H, s.W, h, w);                   \
                    vh += coord_weight_##SFX(im, s.H, s.W, h, w, 0) * gc * m;                   \
                    vw += coord_weight_##SFX(im, s.H, s.W, h, w, 1) * gc * m;                   \
                }                                                                               \
                gob[(2 * t) * P + p] = vh;                                                      \
                gob[(2 * t + 1) * P + p] = vw;                                                  \
                gmb[t * P + p] = vm;                                                            \
            }                                                                                   \
        }                                                                                       \
        /* grad_input: scatter gcol * mask * corner weight (com.cu:553-609); channel planes  \
           are disjoint, so channels run in parallel without atomics */                         \
        _Pragma("omp parallel for schedule(static)")                                           \
        for (int c = 0; c < s.C; ++c) {                                                         \
            const int g = c / cpg;                                                              \
            const T *ob = off + ((size_t)b * s.dg + g) * 2 * K2 * P;                            \
            const T *mb = msk + ((size_t)b * s.dg + g) * K2 * P;                                \
            T *gim = gx + ((size_t)b * s.C + c) * HW;                                           \
            for (int t = 0; t < K2; ++t) {                                                      \
                const int i = t / s.kw, j = t % s.kw;                                           \
                for (int p = 0; p < P; ++p) {                                                   \
                    const int ho = p / s.Wo, wo = p % s.Wo;                                     \
                    const T h = DCN_COORD(T, ho * s.sh - s.ph + i * s.dh, ob[(2 * t) * P + p]);         \
                    const T w = DCN_COORD(T, wo * s.sw - s.pw + j * s.dw, ob[(2 * t + 1) * P + p]);     \
                    if (!(h > -1 && w > -1 && h < s.H && w < s.W)) continue;                    \
                    const T top = gcol[((size_t)c * K2 + t) * P + p] * mb[t * P + p];           \
                    const int hl = (int)floor(h), wl = (int)floor(w);                           \
                    const T lh = h - hl, lw = w - wl;                                           \
                    if (hl >= 0 && wl >= 0) gim[hl * s.W + wl] += (1 - lh) * (1 - lw) * top;    \
                    if (hl >= 0 && wl + 1 <= s.W - 1) gim[hl * s.W + wl + 1] += (1 - lh) * lw * top; \
                    if (hl + 1 <= s.H - 1 && wl >= 0) gim[(hl + 1) * s.W + wl] += lh * (1 - lw) * top; \
                    if (hl + 1 <= s.H - 1 && wl + 1 <= s.W - 1)                                 \
                        gim[(hl + 1) * s.W + wl + 1] += lh * lw * top;                          \
                }                                                                               \
            }                                                                                   \
        }                                                                                       \
        /* grad_weight += gO_b . cols^T, grad_bias += gO_b . 1 (com.cu:818-835) */              \
        im2col_##SFX(&s, x, off, msk, b, gcol);                                                 \
        _Pragma("omp parallel for schedule(static)")                                           \
        for (int co = 0; co < s.Co; ++co) {                                                     \
            const T *yr = gyb + (size_t)co * P;                                                 \
            for (int k = 0; k < K; ++k) {                                                       \
                const T *cr = gcol + (size_t)k * P;                                             \
                T acc = 0;                                                                      \
                for (int p = 0; p < P; ++p) acc += yr[p] * cr[p];                               \
                gw[(size_t)co * K + k] += acc;                                                  \
            }                                                                                   \
            if (gb) {                                                                           \
                T acc = 0;                                                                      \
                for (int p = 0; p < P; ++p) acc += yr[p];                                       \
                gb[co] += acc;                                                                  \
            }                                                                                   \
        }                                                                                       \
    }                                                                                           \
    free(gcol);                                                                                 \
}

DCN_ORACLE_DEFINE(double, f64)
DCN_ORACLE_DEFINE(float, f32)
