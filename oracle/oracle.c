/*
 * CPU oracle for the JPEG AI synthesis / analysis path — TEST INFRASTRUCTURE ONLY.
 * See oracle.h for what it restates and how it is pinned. Every function names the
 * reference file:line (paths inside the imazen/zenjpegai crate) whose behaviour it follows.
 *
 * Build: `-O3 -ffp-contract=off`: the contract's multiply-adds are explicit `fmaf` calls and
 * every other expression must round op by op, as Rust evaluates it (Rust never contracts).
 */
#include "oracle.h"

#include <malloc.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 1;
static int g_fast = 0;  /* 1: convolutions run the nn::fast restatement (fast.c) */
static zo_dump_fn g_dump = NULL;

void zo_set_threads(int n) { g_threads = n > 0 ? n : 1; }
int zo_get_threads(void) { return g_threads; }
void zo_set_dump(zo_dump_fn fn) { g_dump = fn; }
void zo_set_fast(int on) {
    g_fast = on != 0;
#ifdef __GLIBC__
    /* the per-layer buffers are large: keep freed memory in the heap instead of returning it
     * to the kernel, so the next layer's buffers do not take fresh page faults */
    if (g_fast) {
        mallopt(M_MMAP_THRESHOLD, 1 << 30);
        mallopt(M_TRIM_THRESHOLD, 1 << 30);
    }
#endif
}
int zo_get_fast(void) { return g_fast; }

/* Element-parallel loops in the baseline mode (the crate's math runs SIMD and threaded); each
 * element's arithmetic is the same as on one thread, so the result is the same bits. */
#define ZO_PAR_FOR _Pragma("omp parallel for schedule(static) if(g_fast) num_threads(g_threads)")

static float clampf(float v, float lo, float hi) {
    /* Rust f32::clamp: NaN passes through. */
    if (v < lo) return lo;
    if (v > hi) return hi;
    return v;
}

/* ======================================================================================= */
/* Convolution (reference.rs:16-133; layers.rs:100-115 for the extra zero border)            */
/* ======================================================================================= */

void zo_conv2d_out_size(int h, int w, int kh, int kw, int stride, int pad_h, int pad_w,
                        const int extra[4], int *oh, int *ow) {
    int et = extra ? extra[0] : 0, el = extra ? extra[1] : 0;
    int eb = extra ? extra[2] : 0, er = extra ? extra[3] : 0;
    *oh = (h + et + eb + 2 * pad_h - kh) / stride + 1;
    *ow = (w + el + er + 2 * pad_w - kw) / stride + 1;
}

int zo_conv2d(const float *x, int c, int h, int w, const float *weight, const float *bias,
              int oc, int kh, int kw, int stride, int pad_h, int pad_w, int groups,
              const int extra[4], float *out) {
    if (g_fast) {  /* the timed CPU baseline: same bits, blocked algorithm */
        int r = zf_conv2d(x, c, h, w, weight, bias, oc, kh, kw, stride, pad_h, pad_w, groups,
                          extra, out);
        if (r != 1) return r;
    }
    if (groups <= 0 || c % groups || oc % groups || stride <= 0 || kh <= 0 || kw <= 0)
        return -1;
    int et = extra ? extra[0] : 0, el = extra ? extra[1] : 0;
    int eb = extra ? extra[2] : 0, er = extra ? extra[3] : 0;
    int hh = h + et + eb, ww = w + el + er;
    if (hh + 2 * pad_h < kh || ww + 2 * pad_w < kw) return -1;
    int oh, ow;
    zo_conv2d_out_size(h, w, kh, kw, stride, pad_h, pad_w, extra, &oh, &ow);
    /* zero_pad (reference.rs:16-27) of the (extra-padded) input */
    int ph = hh + 2 * pad_h, pw = ww + 2 * pad_w;
    int top = et + pad_h, left = el + pad_w;
    float *xp = (float *)calloc((size_t)c * ph * pw, sizeof(float));
    if (!xp) return -2;
    for (int ci = 0; ci < c; ci++)
        for (int y = 0; y < h; y++)
            memcpy(xp + ((size_t)ci * ph + y + top) * pw + left, x + ((size_t)ci * h + y) * w,
                   sizeof(float) * w);
    int icg = c / groups, ocg = oc / groups;
    int wlen = icg * kh * kw;
    /* conv_plane (reference.rs:47-89): per output row, acc = bias, then for i, ky, kx the
     * contract's fma over the row. One output channel per task. */
#pragma omp parallel for schedule(dynamic) num_threads(g_threads)
    for (int o = 0; o < oc; o++) {
        float *acc = (float *)malloc(sizeof(float) * ow);
        int ic0 = (o / ocg) * icg;
        const float *wt = weight + (size_t)o * wlen;
        float b = bias ? bias[o] : 0.0f;
        for (int oy = 0; oy < oh; oy++) {
            for (int ox = 0; ox < ow; ox++) acc[ox] = b;
            for (int i = 0; i < icg; i++) {
                const float *plane = xp + (size_t)(ic0 + i) * ph * pw;
                for (int ky = 0; ky < kh; ky++) {
                    const float *row = plane + (size_t)(oy * stride + ky) * pw;
                    for (int kx = 0; kx < kw; kx++) {
                        float wv = wt[(i * kh + ky) * kw + kx];
                        if (stride == 1) {
                            const float *r = row + kx;
                            for (int ox = 0; ox < ow; ox++) acc[ox] = fmaf(wv, r[ox], acc[ox]);
                        } else {
                            for (int ox = 0; ox < ow; ox++)
                                acc[ox] = fmaf(wv, row[ox * stride + kx], acc[ox]);
                        }
                    }
                }
            }
            memcpy(out + ((size_t)o * oh + oy) * ow, acc, sizeof(float) * ow);
        }
        free(acc);
    }
    free(xp);
    return 0;
}

void zo_conv_transpose2d_out_size(int h, int w, int k, int stride, int pad, int out_pad,
                                  int *oh, int *ow) {
    *oh = (h - 1) * stride + k + out_pad - 2 * pad;
    *ow = (w - 1) * stride + k + out_pad - 2 * pad;
}

/* conv_transpose2d / conv_transpose_plane (reference.rs:155-236). The reference walks, per
 * output element, ic then ky then kx ascending over a copy zero-padded by `ext`, skipping the
 * taps whose stride parity does not reach the element. Here the loops are interchanged so
 * that each output plane is swept per (ic, ky, kx); every element still sees its taps in the
 * same (ic, ky, kx) order, so the result is the same bits. */
int zo_conv_transpose2d(const float *x, int c, int h, int w, const float *weight,
                        const float *bias, int oc, int k, int stride, int pad, int out_pad,
                        float *out) {
    if (g_fast) {
        int r = zf_conv_transpose2d(x, c, h, w, weight, bias, oc, k, stride, pad, out_pad, out);
        if (r != 1) return r;
    }
    if (stride <= 0 || k <= 0 || pad >= k || out_pad >= stride || h <= 0 || w <= 0) return -1;
    int oh, ow;
    zo_conv_transpose2d_out_size(h, w, k, stride, pad, out_pad, &oh, &ow);
    int ext = (k + stride - 1) / stride + 1;
    int ph = h + 2 * ext, pw = w + 2 * ext;
    float *xp = (float *)calloc((size_t)c * ph * pw, sizeof(float));
    if (!xp) return -2;
    for (int ci = 0; ci < c; ci++)
        for (int y = 0; y < h; y++)
            memcpy(xp + ((size_t)ci * ph + y + ext) * pw + ext, x + ((size_t)ci * h + y) * w,
                   sizeof(float) * w);
#pragma omp parallel for schedule(dynamic) num_threads(g_threads)
    for (int o = 0; o < oc; o++) {
        float *op = out + (size_t)o * oh * ow;
        float b = bias ? bias[o] : 0.0f;
        for (int64_t i = 0; i < (int64_t)oh * ow; i++) op[i] = b;
        for (int ic = 0; ic < c; ic++) {
            const float *plane = xp + (size_t)ic * ph * pw;
            const float *wb = weight + ((size_t)ic * oc + o) * k * k;
            for (int ky = 0; ky < k; ky++) {
                for (int kx = 0; kx < k; kx++) {
                    float wv = wb[ky * k + kx];
                    for (int oy = 0; oy < oh; oy++) {
                        int ty = oy + pad + ext * stride - ky;
                        if (ty % stride) continue;
                        const float *row = plane + (size_t)(ty / stride) * pw;
                        float *orow = op + (size_t)oy * ow;
                        /* first ox with matching column parity */
                        int ox0 = 0;
                        while (ox0 < ow && (ox0 + pad + ext * stride - kx) % stride) ox0++;
                        for (int ox = ox0; ox < ow; ox += stride) {
                            int tx = ox + pad + ext * stride - kx;
                            orow[ox] = fmaf(wv, row[tx / stride], orow[ox]);
                        }
                    }
                }
            }
        }
    }
    free(xp);
    return 0;
}

/* pixel_shuffle (reference.rs:353-375) */
int zo_pixel_shuffle(const float *x, int c4, int h, int w, int r, float *out) {
    if (r <= 0 || c4 % (r * r)) return -1;
    int c = c4 / (r * r);
    for (int oc = 0; oc < c; oc++)
        for (int dy = 0; dy < r; dy++)
            for (int dx = 0; dx < r; dx++) {
                const float *src = x + (size_t)(oc * r * r + dy * r + dx) * h * w;
                for (int y = 0; y < h; y++) {
                    float *dst = out + ((size_t)oc * h * r + (size_t)y * r + dy) * w * r;
                    for (int xi = 0; xi < w; xi++) dst[xi * r + dx] = src[y * w + xi];
                }
            }
    return 0;
}

/* ======================================================================================= */
/* Pointwise ops (layers.rs:174-229; math.rs:28-62, 371-397)                                 */
/* ======================================================================================= */

void zo_relu(float *x, int64_t n) {
    ZO_PAR_FOR
    for (int64_t i = 0; i < n; i++) x[i] = x[i] > 0.0f ? x[i] : 0.0f;
}
void zo_relu6(float *x, int64_t n) {
    ZO_PAR_FOR
    for (int64_t i = 0; i < n; i++) x[i] = clampf(x[i], 0.0f, 6.0f);
}
void zo_add(float *dst, const float *src, int64_t n) {
    ZO_PAR_FOR
    for (int64_t i = 0; i < n; i++) dst[i] += src[i];
}
/* `x *= 1 + m`: two IEEE operations, not an FMA (layers.rs:195-201) */
void zo_gate(float *x, const float *mask, int64_t n) {
    ZO_PAR_FOR
    for (int64_t i = 0; i < n; i++) x[i] *= 1.0f + mask[i];
}
void zo_mul(float *a, const float *b, int64_t n) {
    ZO_PAR_FOR
    for (int64_t i = 0; i < n; i++) a[i] *= b[i];
}

/* Cephes `expf` (math.rs:28-62): clamp to [-87, 88], n = floor(x log2e + 1/2), two-step
 * Cody-Waite reduction by ln 2, degree-5 polynomial evaluated with separate multiplies and
 * adds, then scaling by 2^n built from the exponent bits. Constants as Cephes prints them. */
float zo_exp(float x) {
    static const float LOG2E = 1.44269504088896340736f;
    static const float LN2_HI = 0.693359375f;
    static const float LN2_LO = -2.12194440e-4f;
    static const float P0 = 1.9875691500e-4f, P1 = 1.3981999507e-3f, P2 = 8.3334519073e-3f,
                       P3 = 4.1665795894e-2f, P4 = 1.6666665459e-1f, P5 = 5.0000001201e-1f;
    x = clampf(x, -87.0f, 88.0f);
    float n = floorf(x * LOG2E + 0.5f);
    float r = x - n * LN2_HI;
    r = r - n * LN2_LO;
    float p = P0;
    p = p * r + P1;
    p = p * r + P2;
    p = p * r + P3;
    p = p * r + P4;
    p = p * r + P5;
    float y = p * (r * r) + r + 1.0f;
    uint32_t bits = (uint32_t)((int32_t)n + 127) << 23;
    float scale;
    memcpy(&scale, &bits, 4);
    return y * scale;
}

void zo_sigmoid(float *x, int64_t n) {
    ZO_PAR_FOR
    for (int64_t i = 0; i < n; i++) x[i] = 1.0f / (1.0f + zo_exp(-x[i]));
}

/* elu(a) * b (math.rs:66-72) */
void zo_elu_gate(float *a, const float *b, int64_t n) {
    ZO_PAR_FOR
    for (int64_t i = 0; i < n; i++) {
        float e = zo_exp(a[i]) - 1.0f;
        float elu = a[i] > 0.0f ? a[i] : e;
        a[i] = elu * b[i];
    }
}

/* `x * 128 + 127.5` clamped to [0, 255] (synthesis.rs:188-192); without the clamp while
 * zo_set_output_clamp(0) (a diagnostic for comparing values the clamp would saturate) */
static int g_clamp = 1;
void zo_set_output_clamp(int on) { g_clamp = on != 0; }
void zo_denormalize(float *x, int64_t n) {
    ZO_PAR_FOR
    for (int64_t i = 0; i < n; i++) {
        float v = x[i] * 128.0f + 127.5f;
        x[i] = g_clamp ? clampf(v, 0.0f, 255.0f) : v;
    }
}

/* `(x - 127.5) / 128` (analysis.rs:36-39) */
void zo_normalize(const float *x, int64_t n, float *out) {
    ZO_PAR_FOR
    for (int64_t i = 0; i < n; i++) out[i] = (x[i] - 127.5f) / 128.0f;
}

int zo_pad_amount(int len, int divider) {
    return 2 * ((len + 2 * divider - 1) / (2 * divider)) - (len + divider - 1) / divider;
}

/* ======================================================================================= */
/* Layer norm and channel attention (math.rs:399-603)                                        */
/* ======================================================================================= */

int zo_layer_norm_channels(float *x, int c, int h, int w, const float *weight,
                           const float *bias) {
    if (c <= 0) return -1;
    int64_t n = (int64_t)h * w;
    /* per pixel: f64 mean and biased variance over the channels in channel order, then
     * (x - mean) / sqrt(var + 1e-5) * w + b in f32; pixel blocks are independent */
    const int64_t blk = 256;
    const int64_t nblk = (n + blk - 1) / blk;
#pragma omp parallel for schedule(static) if(g_fast) num_threads(g_threads)
    for (int64_t bi = 0; bi < nblk; bi++) {
        const int64_t i0 = bi * blk, i1 = i0 + blk < n ? i0 + blk : n;
        double mean[256], var[256];
        float mean32[256], denom[256];
        for (int64_t i = i0; i < i1; i++) mean[i - i0] = 0.0, var[i - i0] = 0.0;
        for (int ch = 0; ch < c; ch++) {
            const float *p = x + ch * n;
            for (int64_t i = i0; i < i1; i++) mean[i - i0] += (double)p[i];
        }
        for (int64_t i = i0; i < i1; i++) mean[i - i0] /= (double)c;
        for (int ch = 0; ch < c; ch++) {
            const float *p = x + ch * n;
            for (int64_t i = i0; i < i1; i++) {
                double d = (double)p[i] - mean[i - i0];
                var[i - i0] += d * d;
            }
        }
        for (int64_t i = i0; i < i1; i++) {
            mean32[i - i0] = (float)mean[i - i0];
            denom[i - i0] = sqrtf((float)(var[i - i0] / (double)c) + 1e-5f);
        }
        for (int ch = 0; ch < c; ch++) {
            float *p = x + ch * n;
            float wv = weight[ch], bv = bias[ch];
            for (int64_t i = i0; i < i1; i++)
                p[i] = (p[i] - mean32[i - i0]) / denom[i - i0] * wv + bv;
        }
    }
    return 0;
}

/* Eight interleaved f64 accumulators (index mod 8), combined pairwise (math.rs:452-465). */
double zo_dot8(const float *a, const float *b, int64_t n) {
    double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t full = n / 8 * 8;
    for (int64_t i = 0; i < full; i += 8)
        for (int l = 0; l < 8; l++) acc[l] += (double)a[i + l] * (double)b[i + l];
    for (int64_t i = full; i < n; i++) acc[i - full] += (double)a[i] * (double)b[i];
    return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

/* channel_attention_impl, exact (non-approximate) precision (math.rs:512-603):
 * q, k rows L2-normalised over the pixels (norm from dot8 in f64, eps 1e-12), per head the
 * c x c Gram q_i . k_j (dot8, narrowed to f32) times temperature[head], row softmax with the
 * max subtracted and Cephes exp, f64 sum, f32 divide; out_i = sum_j a_ij v_j in f64. */
int zo_channel_attention(const float *qkv, int c3, int h, int w, int heads,
                         const float *temperature, float *out) {
    if (heads <= 0 || c3 % (3 * heads)) return -1;
    int dim = c3 / 3, c = dim / heads;
    int64_t n = (int64_t)h * w;
    float *qk = (float *)malloc(sizeof(float) * 2 * dim * n);
    memcpy(qk, qkv, sizeof(float) * 2 * dim * n);
#pragma omp parallel for schedule(dynamic) num_threads(g_threads)
    for (int r = 0; r < 2 * dim; r++) {
        float *row = qk + (int64_t)r * n;
        float norm = (float)sqrt(zo_dot8(row, row, n));
        float d = norm > 1e-12f ? norm : 1e-12f;
        for (int64_t i = 0; i < n; i++) row[i] /= d;
    }
    const float *q = qk, *k = qk + (int64_t)dim * n, *v = qkv + (int64_t)2 * dim * n;
    float *attn = (float *)malloc(sizeof(float) * dim * c);
#pragma omp parallel for schedule(dynamic) num_threads(g_threads)
    for (int ri = 0; ri < dim; ri++) {
        int head = ri / c;
        float *row = attn + (int64_t)ri * c;
        const float *qi = q + (int64_t)ri * n;
        float mx = -INFINITY;
        for (int j = 0; j < c; j++) {
            const float *kj = k + (int64_t)(head * c + j) * n;
            row[j] = (float)zo_dot8(qi, kj, n) * temperature[head];
            mx = row[j] > mx ? row[j] : mx;
        }
        for (int j = 0; j < c; j++) row[j] = zo_exp(row[j] - mx);
        double sum = 0.0;
        for (int j = 0; j < c; j++) sum += (double)row[j];
        float s32 = (float)sum;
        for (int j = 0; j < c; j++) row[j] /= s32;
    }
#pragma omp parallel for schedule(dynamic) num_threads(g_threads)
    for (int ri = 0; ri < dim; ri++) {
        int head = ri / c;
        const float *wts = attn + (int64_t)ri * c;
        double *acc = (double *)calloc(n, sizeof(double));
        for (int j = 0; j < c; j++) {
            double a = (double)wts[j];
            const float *vj = v + (int64_t)(head * c + j) * n;
            for (int64_t i = 0; i < n; i++) acc[i] += a * (double)vj[i];
        }
        float *o = out + (int64_t)ri * n;
        for (int64_t i = 0; i < n; i++) o[i] = (float)acc[i];
        free(acc);
    }
    free(attn);
    free(qk);
    return 0;
}

/* ======================================================================================= */
/* Network plumbing: planar tensors and checkpoint lookups (model/load.rs:11-85)             */
/* ======================================================================================= */

typedef struct {
    int c, h, w;
    float *d;
} T;

static T t_new(int c, int h, int w) {
    T t = {c, h, w, (float *)calloc((size_t)c * h * w, sizeof(float))};
    return t;
}
static void t_free(T *t) {
    free(t->d);
    t->d = NULL;
}
static int64_t t_len(const T *t) { return (int64_t)t->c * t->h * t->w; }
static T t_clone(const T *t) {
    T o = t_new(t->c, t->h, t->w);
    memcpy(o.d, t->d, sizeof(float) * t_len(t));
    return o;
}
static void t_move(T *dst, T src) {
    t_free(dst);
    *dst = src;
}
static void dump(const char *name, const T *t) {
    if (g_dump) g_dump(name, t->d, t->c, t->h, t->w);
}

#define ZO_FAIL(msg)                                                \
    do {                                                            \
        fprintf(stderr, "oracle: %s\n", msg);                       \
        abort();                                                    \
    } while (0)

static const zo_param *find(const zo_ckpt *ck, const char *name) {
    for (int i = 0; i < ck->n; i++)
        if (strcmp(ck->params[i].name, name) == 0) return &ck->params[i];
    return NULL;
}

static const float *need(const zo_ckpt *ck, const char *prefix, const char *suffix, int n0,
                         int n1, int n2, int n3) {
    char name[256];
    snprintf(name, sizeof name, "%s.%s", prefix, suffix);
    const zo_param *p = find(ck, name);
    if (!p) {
        fprintf(stderr, "oracle: missing parameter %s\n", name);
        abort();
    }
    int want[4] = {n0, n1, n2, n3};
    int nd = n3 >= 0 ? 4 : n2 >= 0 ? 3 : n1 >= 0 ? 2 : 1;
    if (p->ndim != nd) {
        fprintf(stderr, "oracle: %s has ndim %d, expected %d\n", name, p->ndim, nd);
        abort();
    }
    for (int i = 0; i < nd; i++)
        if (p->shape[i] != want[i]) {
            fprintf(stderr, "oracle: %s dim %d is %d, expected %d\n", name, i, p->shape[i],
                    want[i]);
            abort();
        }
    return p->data;
}

/* load::conv (load.rs:11-40) + ConvLayer::forward */
static T conv_layer(const zo_ckpt *ck, const char *prefix, const T *x, int out_ch, int kh,
                    int kw, int stride, int pad, int groups, int bias, const int extra[4]) {
    if (x->c % groups) ZO_FAIL("groups");
    const float *w = need(ck, prefix, "weight", out_ch, x->c / groups, kh, kw);
    const float *b = bias ? need(ck, prefix, "bias", out_ch, -1, -1, -1) : NULL;
    int oh, ow;
    zo_conv2d_out_size(x->h, x->w, kh, kw, stride, pad, pad, extra, &oh, &ow);
    T o = t_new(out_ch, oh, ow);
    if (zo_conv2d(x->d, x->c, x->h, x->w, w, b, out_ch, kh, kw, stride, pad, pad, groups,
                  extra, o.d))
        ZO_FAIL("conv2d");
    return o;
}
static T conv3x3(const zo_ckpt *ck, const char *prefix, const T *x, int out_ch, int groups,
                 int bias) {
    return conv_layer(ck, prefix, x, out_ch, 3, 3, 1, 1, groups, bias, NULL);
}
static T conv1x1(const zo_ckpt *ck, const char *prefix, const T *x, int out_ch, int bias) {
    return conv_layer(ck, prefix, x, out_ch, 1, 1, 1, 0, 1, bias, NULL);
}
static T conv3x3_s2(const zo_ckpt *ck, const char *prefix, const T *x, int out_ch) {
    return conv_layer(ck, prefix, x, out_ch, 3, 3, 2, 1, 1, 1, NULL);
}
/* load::conv_transpose (load.rs:64-85): always with bias */
static T convt(const zo_ckpt *ck, const char *prefix, const T *x, int out_ch, int k,
               int stride, int pad, int out_pad) {
    const float *w = need(ck, prefix, "weight", x->c, out_ch, k, k);
    const float *b = need(ck, prefix, "bias", out_ch, -1, -1, -1);
    int oh, ow;
    zo_conv_transpose2d_out_size(x->h, x->w, k, stride, pad, out_pad, &oh, &ow);
    T o = t_new(out_ch, oh, ow);
    if (zo_conv_transpose2d(x->d, x->c, x->h, x->w, w, b, out_ch, k, stride, pad, out_pad,
                            o.d))
        ZO_FAIL("conv_transpose2d");
    return o;
}
/* conv3x3_t (attention.rs:80-91): k3 s2 p1 op1 */
static T convt3(const zo_ckpt *ck, const char *prefix, const T *x, int out_ch) {
    return convt(ck, prefix, x, out_ch, 3, 2, 1, 1);
}

static T crop(const T *x, int h, int w) {
    if (h > x->h || w > x->w) ZO_FAIL("crop larger than tensor");
    T o = t_new(x->c, h, w);
    for (int c = 0; c < x->c; c++)
        for (int y = 0; y < h; y++)
            memcpy(o.d + ((size_t)c * h + y) * w, x->d + ((size_t)c * x->h + y) * x->w,
                   sizeof(float) * w);
    return o;
}

static T pixel_shuffle_t(const T *x, int r) {
    T o = t_new(x->c / (r * r), x->h * r, x->w * r);
    if (zo_pixel_shuffle(x->d, x->c, x->h, x->w, r, o.d)) ZO_FAIL("pixel_shuffle");
    return o;
}

static int cdiv(int a, int b) { return (a + b - 1) / b; }

/* ResAu::load / forward (synthesis.rs:24-74): y = x * (1 + conv1x1(gconv3x3(relu6 x))) */
static void resau(const zo_ckpt *ck, const char *prefix, T *x) {
    char name[256];
    snprintf(name, sizeof name, "%s.conv.weight", prefix);
    const zo_param *p = find(ck, name);
    if (!p || p->ndim != 4 || p->shape[1] <= 0 || x->c % p->shape[1]) ZO_FAIL(name);
    int groups = x->c / p->shape[1];
    T act = t_clone(x);
    zo_relu6(act.d, t_len(&act));
    char pc[256], pc2[256];
    snprintf(pc, sizeof pc, "%s.conv", prefix);
    snprintf(pc2, sizeof pc2, "%s.conv2", prefix);
    T t = conv3x3(ck, pc, &act, x->c, groups, 0);
    t_free(&act);
    T mask = conv1x1(ck, pc2, &t, x->c, 0);
    t_free(&t);
    zo_gate(x->d, mask.d, t_len(x));
    t_free(&mask);
}

/* ResidualBlock::forward (attention.rs:36-43): conv2(relu(conv1 x)) + x */
static T residual_block(const zo_ckpt *ck, const char *prefix, const T *x) {
    char p1[256], p2[256];
    snprintf(p1, sizeof p1, "%s.conv1", prefix);
    snprintf(p2, sizeof p2, "%s.conv2", prefix);
    T t = conv3x3(ck, p1, x, x->c, 1, 1);
    zo_relu(t.d, t_len(&t));
    T out = conv3x3(ck, p2, &t, x->c, 1, 1);
    t_free(&t);
    zo_add(out.d, x->d, t_len(&out));
    return out;
}

/* Cab::forward (attention.rs:122-139): x + RB(RB(x)) * sigmoid(convT(RB(RB(conv_s2 x)))) */
static T cab(const zo_ckpt *ck, const char *prefix, const T *x) {
    char p[256];
    snprintf(p, sizeof p, "%s.residual_trunk.0", prefix);
    T trunk = residual_block(ck, p, x);
    snprintf(p, sizeof p, "%s.residual_trunk.1", prefix);
    t_move(&trunk, residual_block(ck, p, &trunk));
    snprintf(p, sizeof p, "%s.subscale", prefix);
    T m = conv3x3_s2(ck, p, x, x->c);
    snprintf(p, sizeof p, "%s.residual_mask2.0", prefix);
    t_move(&m, residual_block(ck, p, &m));
    snprintf(p, sizeof p, "%s.residual_mask3.0", prefix);
    t_move(&m, residual_block(ck, p, &m));
    snprintf(p, sizeof p, "%s.upscale", prefix);
    t_move(&m, convt3(ck, p, &m, x->c));
    if (m.h != trunk.h || m.w != trunk.w) ZO_FAIL("CAB: odd feature map size");
    zo_sigmoid(m.d, t_len(&m));
    zo_mul(trunk.d, m.d, t_len(&trunk));
    zo_add(trunk.d, x->d, t_len(&trunk));
    t_free(&m);
    return trunk;
}

/* TransformerBlock::forward (attention.rs:328-372); heads 4, FFN gamma 4 */
static void transformer_block(const zo_ckpt *ck, const char *prefix, T *x) {
    int dim = x->c, hidden = dim * 4;
    char p[256];
    /* x = x + project_out(attn(dw(conv1(LN(x))))) */
    snprintf(p, sizeof p, "%s.prep_data.norm1", prefix);
    T t = t_clone(x);
    zo_layer_norm_channels(t.d, t.c, t.h, t.w, need(ck, p, "weight", dim, -1, -1, -1),
                           need(ck, p, "bias", dim, -1, -1, -1));
    snprintf(p, sizeof p, "%s.prep_data.conv1", prefix);
    t_move(&t, conv1x1(ck, p, &t, 3 * dim, 0));
    snprintf(p, sizeof p, "%s.prep_data.conv2", prefix);
    t_move(&t, conv3x3(ck, p, &t, 3 * dim, 3 * dim, 0));
    snprintf(p, sizeof p, "%s.attn", prefix);
    const float *temp = need(ck, p, "temperature", 4, 1, 1, -1);
    T a = t_new(dim, x->h, x->w);
    zo_channel_attention(t.d, t.c, t.h, t.w, 4, temp, a.d);
    t_free(&t);
    snprintf(p, sizeof p, "%s.attn.project_out", prefix);
    t_move(&a, conv1x1(ck, p, &a, dim, 0));
    zo_add(x->d, a.d, t_len(x));
    t_free(&a);
    /* x = x + project_out(elu(first half) * second half of dw(project_in(LN(x)))) */
    snprintf(p, sizeof p, "%s.ffn.norm1", prefix);
    t = t_clone(x);
    zo_layer_norm_channels(t.d, t.c, t.h, t.w, need(ck, p, "weight", dim, -1, -1, -1),
                           need(ck, p, "bias", dim, -1, -1, -1));
    snprintf(p, sizeof p, "%s.ffn.project_in", prefix);
    t_move(&t, conv1x1(ck, p, &t, 2 * hidden, 0));
    snprintf(p, sizeof p, "%s.ffn.dwconv", prefix);
    t_move(&t, conv3x3(ck, p, &t, 2 * hidden, 2 * hidden, 0));
    int64_t n = (int64_t)hidden * t.h * t.w;
    zo_elu_gate(t.d, t.d + n, n);
    t.c = hidden;
    snprintf(p, sizeof p, "%s.ffn.project_out", prefix);
    T f = conv1x1(ck, p, &t, dim, 0);
    t_free(&t);
    zo_add(x->d, f.d, t_len(x));
    t_free(&f);
}

/* Tam::forward (attention.rs:530-545) */
static void tam(const zo_ckpt *ck, const char *prefix, T *x, int downsample) {
    char p[256];
    if (downsample) {
        snprintf(p, sizeof p, "%s.ds_conv", prefix);
        t_move(x, conv3x3_s2(ck, p, x, x->c));
    }
    snprintf(p, sizeof p, "%s.TABs.0", prefix);
    transformer_block(ck, p, x);
    snprintf(p, sizeof p, "%s.TABs.1", prefix);
    transformer_block(ck, p, x);
    if (downsample) {
        snprintf(p, sizeof p, "%s.us_conv", prefix);
        t_move(x, convt3(ck, p, x, x->c));
    }
}

/* Upsample (synthesis.rs:117-171): BOP convT 4x4 s2 p1; SOP pad(0,1,0,1) + conv2x2 + PS2 */
static T upsample(const zo_ckpt *ck, int op, const char *prefix, const T *x, int out_ch) {
    if (op == ZO_BOP) return convt(ck, prefix, x, out_ch, 4, 2, 1, 0);
    char p[256];
    snprintf(p, sizeof p, "%s.conv", prefix);
    static const int extra[4] = {0, 0, 1, 1};
    T t = conv_layer(ck, p, x, out_ch * 4, 2, 2, 1, 0, 1, 0, extra);
    T o = pixel_shuffle_t(&t, 2);
    t_free(&t);
    return o;
}

void zo_synth_out_size(int op, int secondary, int h, int w, int *oh, int *ow) {
    if (op == ZO_HOP && !secondary) {
        *oh = 2 * cdiv(h, 2);
        *ow = 2 * cdiv(w, 2);
    } else if (op == ZO_HOP) {
        *oh = 4 * cdiv(h, 4);
        *ow = 4 * cdiv(w, 4);
    } else if (!secondary) {
        *oh = 4 * cdiv(h, 4);
        *ow = 4 * cdiv(w, 4);
    } else {
        *oh = 8 * cdiv(h, 8);
        *ow = 8 * cdiv(w, 8);
    }
}

/* LightPrimary::forward (synthesis.rs:514-580); (c1, c2, c3) = SOP (64,32,32), BOP (64,64,96) */
static T light_primary(const zo_ckpt *ck, int op, const T *y, int h, int w) {
    int c1 = 64, c2 = op == ZO_SOP ? 32 : 64, c3 = op == ZO_SOP ? 32 : 96;
    T x = conv3x3(ck, "first_stage.0.0.conv1", y, 160, 1, 1);
    zo_relu(x.d, t_len(&x));
    zo_add(x.d, y->d, t_len(&x));
    dump("res", &x);
    t_move(&x, upsample(ck, op, "first_stage.1", &x, c1));
    dump("up1", &x);
    resau(ck, "first_stage.2", &x);
    t_move(&x, crop(&x, cdiv(h, 8), cdiv(w, 8)));
    dump("act1", &x);
    t_move(&x, upsample(ck, op, "conv2_t", &x, c2));
    t_move(&x, crop(&x, cdiv(h, 4), cdiv(w, 4)));
    dump("up2", &x);
    resau(ck, "iact2", &x);
    dump("act2", &x);
    t_move(&x, conv3x3(ck, "conv3", &x, c3, 1, 1));
    dump("conv3", &x);
    resau(ck, "iact3", &x);
    dump("act3", &x);
    t_move(&x, conv1x1(ck, "conv4", &x, 16, 0));
    t_move(&x, pixel_shuffle_t(&x, 4));
    zo_denormalize(x.d, t_len(&x));
    dump("out", &x);
    return x;
}

/* HopPrimary::forward (synthesis.rs:324-390) */
static T hop_primary(const zo_ckpt *ck, const T *y, int h, int w) {
    const int c = 128;
    T x = residual_block(ck, "first_stage.0.0", y);
    dump("res", &x);
    t_move(&x, convt3(ck, "first_stage.1", &x, c));
    dump("up1", &x);
    resau(ck, "first_stage.2", &x);
    t_move(&x, crop(&x, cdiv(h, 8), cdiv(w, 8)));
    dump("act1", &x);
    t_move(&x, convt3(ck, "conv2_t", &x, c));
    dump("up2", &x);
    t_move(&x, cab(ck, "CAB", &x));
    t_move(&x, crop(&x, cdiv(h, 4), cdiv(w, 4)));
    dump("cab", &x);
    resau(ck, "iact2", &x);
    dump("act2", &x);
    t_move(&x, conv1x1(ck, "conv3_t", &x, 4 * c, 1));
    t_move(&x, pixel_shuffle_t(&x, 2));
    dump("conv3", &x);
    tam(ck, "TAM", &x, 1);
    t_move(&x, crop(&x, cdiv(h, 2), cdiv(w, 2)));
    dump("tam", &x);
    resau(ck, "iact3", &x);
    dump("act3", &x);
    t_move(&x, convt3(ck, "conv4_t", &x, 1));
    zo_denormalize(x.d, t_len(&x));
    dump("out", &x);
    return x;
}

int zo_synthesis_primary(const zo_ckpt *ck, int op, const float *y_hat, int lh, int lw, int h,
                         int w, float *out) {
    T y = {160, lh, lw, (float *)y_hat};
    T x = op == ZO_HOP ? hop_primary(ck, &y, h, w) : light_primary(ck, op, &y, h, w);
    memcpy(out, x.d, sizeof(float) * t_len(&x));
    t_free(&x);
    return 0;
}

/* LightSecondary::forward (synthesis.rs:862-909); (c2, c3) = SOP (32,32), BOP (64,128) */
static T light_secondary(const zo_ckpt *ck, int op, const T *x0, int h, int w) {
    int c2 = op == ZO_SOP ? 32 : 64, c3 = op == ZO_SOP ? 32 : 128;
    T x = upsample(ck, op, "conv2_t", x0, c2);
    t_move(&x, crop(&x, cdiv(h, 8), cdiv(w, 8)));
    dump("uv.up", &x);
    resau(ck, "iact2", &x);
    dump("uv.act2", &x);
    t_move(&x, conv3x3(ck, "conv3", &x, c3, 1, 1));
    dump("uv.conv3", &x);
    resau(ck, "iact3", &x);
    dump("uv.act3", &x);
    t_move(&x, conv1x1(ck, "conv4", &x, 128, 0));
    t_move(&x, pixel_shuffle_t(&x, 8));
    return x;
}

/* HopSecondary::forward (synthesis.rs:723-773) */
static T hop_secondary(const zo_ckpt *ck, const T *x0, int h, int w) {
    const int c = 64;
    T x = convt3(ck, "conv2_t", x0, c);
    dump("uv.up", &x);
    t_move(&x, cab(ck, "CAB", &x));
    t_move(&x, crop(&x, cdiv(h, 8), cdiv(w, 8)));
    dump("uv.cab", &x);
    resau(ck, "iact2", &x);
    dump("uv.act2", &x);
    t_move(&x, conv1x1(ck, "conv3_t", &x, 4 * c, 1));
    t_move(&x, pixel_shuffle_t(&x, 2));
    dump("uv.conv3", &x);
    tam(ck, "TAM", &x, 0);
    t_move(&x, crop(&x, cdiv(h, 4), cdiv(w, 4)));
    dump("uv.tam", &x);
    resau(ck, "iact3", &x);
    dump("uv.act3", &x);
    t_move(&x, convt3(ck, "conv4_t", &x, 8));
    t_move(&x, pixel_shuffle_t(&x, 2));
    return x;
}

int zo_synthesis_secondary(const zo_ckpt *ck, int op, const float *y_hat_luma, int llh,
                           int llw, const float *y_hat_chroma, int lh, int lw, int h, int w,
                           float *out) {
    /* forward_with (synthesis.rs:1004-1038): the luma latent is cropped to the chroma one */
    if (lh > llh || lw > llw) return -1;
    T cat = t_new(256, lh, lw);
    for (int c = 0; c < 160; c++)
        for (int y = 0; y < lh; y++)
            memcpy(cat.d + ((size_t)c * lh + y) * lw, y_hat_luma + ((size_t)c * llh + y) * llw,
                   sizeof(float) * lw);
    memcpy(cat.d + (size_t)160 * lh * lw, y_hat_chroma, sizeof(float) * 96 * lh * lw);
    T info = conv3x3(ck, "first_stage.conv1", &cat, 48, 1, 1);
    t_free(&cat);
    dump("uv.combine", &info);
    T x = t_new(144, lh, lw);
    memcpy(x.d, info.d, sizeof(float) * t_len(&info));
    memcpy(x.d + t_len(&info), y_hat_chroma, sizeof(float) * 96 * lh * lw);
    t_free(&info);
    T o = op == ZO_HOP ? hop_secondary(ck, &x, h, w) : light_secondary(ck, op, &x, h, w);
    t_free(&x);
    zo_denormalize(o.d, t_len(&o));
    dump("uv.out", &o);
    memcpy(out, o.d, sizeof(float) * t_len(&o));
    t_free(&o);
    return 0;
}

/* ======================================================================================= */
/* Analysis (analysis.rs:96-311)                                                              */
/* ======================================================================================= */

/* replicate_pad (analysis.rs:48-71) */
static T replicate_pad(const T *x, int bottom, int right) {
    T o = t_new(x->c, x->h + bottom, x->w + right);
    for (int c = 0; c < x->c; c++)
        for (int y = 0; y < o.h; y++) {
            int sy = y < x->h ? y : x->h - 1;
            const float *src = x->d + ((size_t)c * x->h + sy) * x->w;
            float *dst = o.d + ((size_t)c * o.h + y) * o.w;
            memcpy(dst, src, sizeof(float) * x->w);
            for (int xx = x->w; xx < o.w; xx++) dst[xx] = src[x->w - 1];
        }
    return o;
}

/* pad_for (analysis.rs:74-83) */
static T pad_for(const T *x, int h, int w, int divider) {
    if (x->h != cdiv(h, divider) || x->w != cdiv(w, divider)) ZO_FAIL("analysis map size");
    return replicate_pad(x, zo_pad_amount(h, divider), zo_pad_amount(w, divider));
}

/* Trunk::forward (analysis.rs:157-206), clip off */
static T trunk(const zo_ckpt *ck, int op, const T *xin, int tam_ds) {
    int h = xin->h, w = xin->w;
    const int C = 128;
    T n = t_new(xin->c, h, w);
    zo_normalize(xin->d, t_len(xin), n.d);
    T p = pad_for(&n, h, w, 1);
    t_free(&n);
    T x = conv_layer(ck, "conv1", &p, C, 3, 3, 2, 1, 1, 1, NULL);
    t_free(&p);
    resau(ck, "act1", &x);
    dump("ana.act1", &x);
    t_move(&x, pad_for(&x, h, w, 2));
    if (op == ZO_HOP) tam(ck, "TAM", &x, tam_ds);
    t_move(&x, conv_layer(ck, "conv2", &x, C, 3, 3, 2, 1, 1, 1, NULL));
    resau(ck, "act2", &x);
    dump("ana.act2", &x);
    t_move(&x, pad_for(&x, h, w, 4));
    if (op == ZO_HOP) t_move(&x, cab(ck, "cab", &x));
    t_move(&x, conv_layer(ck, "conv3", &x, C, 3, 3, 2, 1, 1, 1, NULL));
    resau(ck, "act3", &x);
    dump("ana.act3", &x);
    return x;
}

/* One stage of the analysis transform of an h x w picture, from that stage's input (the
 * per-stage parity check: the engine's stage output is compared with this stage run on the
 * engine's own input). Stage 1: picture [1 or 12][h][w] in [0, 255] -> act1 (normalize, pad,
 * conv1 s2, ResAu act1); stage 2: act1 -> act2 (pad, HOP TAM, conv2 s2, ResAu act2); stage 3:
 * act2 -> act3 (pad, HOP CAB, conv3 s2, ResAu act3); stage 4: act3 -> the latent (primary:
 * pad, conv4 s2, conv5 1x1; secondary: conv5 1x1). Trunk::forward (analysis.rs:157-206),
 * AnalysisPrimary/Secondary::forward (:242-311). Returns -1 for a stage outside 1..4, a
 * malformed input extent or SOP. */
int zo_analysis_stage(const zo_ckpt *ck, int op, int secondary, int stage, const float *x, int c,
                      int h, int w, float *out) {
    if (op == ZO_SOP || stage < 1 || stage > 4) return -1;
    static const int div_in[5] = {0, 1, 2, 4, 8};
    const int d = div_in[stage];
    if (c != (stage == 1 ? (secondary ? 12 : 1) : 128)) return -1;
    T in = {c, cdiv(h, d), cdiv(w, d), (float *)x};
    const int C = 128;
    T t;
    if (stage == 1) {
        T n = t_new(in.c, in.h, in.w);
        zo_normalize(in.d, t_len(&in), n.d);
        t = pad_for(&n, h, w, 1);
        t_free(&n);
        t_move(&t, conv_layer(ck, "conv1", &t, C, 3, 3, 2, 1, 1, 1, NULL));
        resau(ck, "act1", &t);
    } else if (stage == 2) {
        t = pad_for(&in, h, w, 2);
        if (op == ZO_HOP) tam(ck, "TAM", &t, !secondary);
        t_move(&t, conv_layer(ck, "conv2", &t, C, 3, 3, 2, 1, 1, 1, NULL));
        resau(ck, "act2", &t);
    } else if (stage == 3) {
        t = pad_for(&in, h, w, 4);
        if (op == ZO_HOP) t_move(&t, cab(ck, "cab", &t));
        t_move(&t, conv_layer(ck, "conv3", &t, C, 3, 3, 2, 1, 1, 1, NULL));
        resau(ck, "act3", &t);
    } else if (secondary) {
        t = t_clone(&in);
        t_move(&t, conv1x1(ck, "conv5", &t, 96, 0));
    } else {
        t = pad_for(&in, h, w, 8);
        t_move(&t, conv_layer(ck, "conv4", &t, 160, 3, 3, 2, 1, 1, 1, NULL));
        t_move(&t, conv1x1(ck, "conv5", &t, 160, 0));
    }
    memcpy(out, t.d, sizeof(float) * t_len(&t));
    t_free(&t);
    return 0;
}

int zo_analysis_primary(const zo_ckpt *ck, int op, const float *xin, int h, int w,
                        float *out) {
    if (op == ZO_SOP) return -1;
    T in = {1, h, w, (float *)xin};
    T t = trunk(ck, op, &in, 1);
    t_move(&t, pad_for(&t, h, w, 8));
    t_move(&t, conv_layer(ck, "conv4", &t, 160, 3, 3, 2, 1, 1, 1, NULL));
    t_move(&t, conv1x1(ck, "conv5", &t, 160, 0));
    dump("ana.out", &t);
    memcpy(out, t.d, sizeof(float) * t_len(&t));
    t_free(&t);
    return 0;
}

int zo_analysis_secondary(const zo_ckpt *ck, int op, const float *xin, int h, int w,
                          float *out) {
    if (op == ZO_SOP) return -1;
    T in = {12, h, w, (float *)xin};
    T t = trunk(ck, op, &in, 0);
    t_move(&t, conv1x1(ck, "conv5", &t, 96, 0));
    dump("ana.uv.out", &t);
    memcpy(out, t.d, sizeof(float) * t_len(&t));
    t_free(&t);
    return 0;
}

/* ======================================================================================= */
/* Latent-domain networks: the hyper-decoder z_hat -> psi (hyper_decoder.rs) and the        */
/* multi-stage context model psi, residual -> y_hat (mcm.rs)                               */
/* ======================================================================================= */

/* HyperDecoder::forward_f32 (hyper_decoder.rs:94-113, layers :24-42): conv1x1 C -> C (no bias),
 * convT 4x4 s2 p1 C -> C (bias), crop to (out_h, out_w), ReLU6, conv3x3 C -> C (bias), ReLU6,
 * conv3x3 C -> 4C (bias). z [c][hz][wz] -> psi [4c][out_h][out_w]. Returns -1 when the crop
 * is larger than the upsampled map. */
int zo_hyper_decode(const zo_ckpt *ck, const float *z, int c, int hz, int wz, int out_h,
                    int out_w, float *psi) {
    if (c <= 0 || hz <= 0 || wz <= 0 || out_h <= 0 || out_w <= 0 || out_h > 2 * hz ||
        out_w > 2 * wz)
        return -1;
    T x = {c, hz, wz, (float *)z};
    T t = conv1x1(ck, "hyper_decoder.conv1", &x, c, 0);
    t_move(&t, convt(ck, "hyper_decoder.conv2", &t, c, 4, 2, 1, 0));
    if (t.h != out_h || t.w != out_w) t_move(&t, crop(&t, out_h, out_w));
    zo_relu6(t.d, t_len(&t));
    t_move(&t, conv3x3(ck, "hyper_decoder.conv3", &t, c, 1, 1));
    zo_relu6(t.d, t_len(&t));
    t_move(&t, conv3x3(ck, "hyper_decoder.conv4", &t, 4 * c, 1, 1));
    dump("hyper.psi", &t);
    memcpy(psi, t.d, sizeof(float) * t_len(&t));
    t_free(&t);
    return 0;
}

/* (row, column) of each context-model stage in a 2 x 2 cell (mcm.rs:25 STAGE_POSITIONS) */
static const int MCM_PY[4] = {0, 1, 0, 1}, MCM_PX[4] = {0, 1, 1, 0};

static T cat2(const T *a, const T *b) {
    if (a->h != b->h || a->w != b->w) ZO_FAIL("cat: extent mismatch");
    T o = t_new(a->c + b->c, a->h, a->w);
    memcpy(o.d, a->d, sizeof(float) * t_len(a));
    memcpy(o.d + t_len(a), b->d, sizeof(float) * t_len(b));
    return o;
}

/* FusionPredNet::forward (mcm.rs:59-65): three bias-free 1x1 convs, ReLU between them. */
static T fusion_pred(const zo_ckpt *ck, const char *prefix, const T *x, int c) {
    char n1[160], n2[160], n3[160];
    snprintf(n1, sizeof n1, "%s.conv1", prefix);
    snprintf(n2, sizeof n2, "%s.conv2", prefix);
    snprintf(n3, sizeof n3, "%s.conv3", prefix);
    T t = conv1x1(ck, n1, x, c, 0);
    zo_relu(t.d, t_len(&t));
    t_move(&t, conv1x1(ck, n2, &t, c, 0));
    zo_relu(t.d, t_len(&t));
    t_move(&t, conv1x1(ck, n3, &t, c, 0));
    return t;
}

/* The latent from psi and the dequantised residual (reconstruct.rs:200-212): with a context
 * model in the checkpoint (present iff "context.MCM.0.fusion_pred_net.conv1.weight" is,
 * common.rs:111-115), ContextModel::decompress (mcm.rs:161-257); without one,
 * upshuffle_psi (mcm.rs:742-760, stage of (y % 2, x % 2) from STAGE_LUT) plus the residual.
 * residual, y [c][h][w]; psi [4c][ceil(h/2)][ceil(w/2)]. Returns -1 on a shape the crate
 * rejects (a context model needs c a multiple of 32, mcm.rs:123-127). */
int zo_context_decompress(const zo_ckpt *ck, int c, const float *residual, int h, int w,
                          const float *psi, float *y) {
    if (c <= 0 || h <= 0 || w <= 0) return -1;
    const int hh = cdiv(h, 2), hw = cdiv(w, 2);
    const size_t qplane = (size_t)hh * hw, plane = (size_t)h * w;
    if (!find(ck, "context.MCM.0.fusion_pred_net.conv1.weight")) {
        static const int LUT[4] = {0, 2, 3, 1};
        for (int ch = 0; ch < c; ch++)
            for (int yy = 0; yy < h; yy++)
                for (int xx = 0; xx < w; xx++) {
                    const int s = LUT[(yy % 2) * 2 + xx % 2];
                    const float m = psi[((size_t)s * c + ch) * qplane + (size_t)(yy / 2) * hw +
                                        xx / 2];
                    const size_t i = ch * plane + (size_t)yy * w + xx;
                    y[i] = m + residual[i];
                }
        return 0;
    }
    if (c % 32) return -1;
    memset(y, 0, sizeof(float) * c * plane);
    T ctx = {0, hh, hw, NULL};
    for (int s = 0; s < 4; s++) {
        T psi_s = t_new(c, hh, hw);
        memcpy(psi_s.d, psi + (size_t)s * c * qplane, sizeof(float) * c * qplane);
        char pre[96], name[128];
        snprintf(pre, sizeof pre, "context.MCM.%d", s);
        T mean;
        if (s == 0) {
            snprintf(name, sizeof name, "%s.fusion_pred_net", pre);
            mean = fusion_pred(ck, name, &psi_s, c);
        } else {
            snprintf(name, sizeof name, "%s.conv.0", pre);
            T t = conv1x1(ck, name, &ctx, c, 0);
            snprintf(name, sizeof name, "%s.conv.1", pre);
            t_move(&t, conv3x3(ck, name, &t, c, c / 32, 1));
            T joined = cat2(&t, &psi_s);
            t_free(&t);
            snprintf(name, sizeof name, "%s.fusion_pred_net", pre);
            mean = fusion_pred(ck, name, &joined, c);
            t_free(&joined);
        }
        t_free(&psi_s);
        /* stage = mean + residual at (2y + py, 2x + px); padded positions keep the mean */
        const int py = MCM_PY[s], px = MCM_PX[s];
        for (int ch = 0; ch < c; ch++)
            for (int yy = 0; yy < hh; yy++) {
                const int sy = 2 * yy + py;
                if (sy >= h) continue;
                for (int xx = 0; xx < hw; xx++) {
                    const int sx = 2 * xx + px;
                    if (sx >= w) continue;
                    float *m = mean.d + ch * qplane + (size_t)yy * hw + xx;
                    const size_t i = ch * plane + (size_t)sy * w + sx;
                    *m = *m + residual[i];
                    y[i] = *m;
                }
            }
        if (s == 0)
            ctx = mean;
        else {
            T nc = cat2(&ctx, &mean);
            t_free(&mean);
            t_move(&ctx, nc);
        }
    }
    t_free(&ctx);
    return 0;
}

/* ======================================================================================= */
/* Tiling (tiles.rs:39-119, 220-229) and whole-picture synthesis (reconstruct.rs:274-464)   */
/* ======================================================================================= */

static int latent_extent(int pos, int len, int latent_len, int *out) {
    if (len % 16 && cdiv(pos + len, 16) < latent_len) return -1;
    *out = cdiv(len, 16);
    return 0;
}

int zo_synthesis_tiles(int height, int width, int latent_h, int latent_w, int tile_size,
                       int overlap, zo_tile *tiles, int max_tiles) {
    if (tile_size <= 0) {
        if (max_tiles >= 1) {
            zo_tile t = {0, 0, width, height, 0, 0, latent_w, latent_h,
                         0, 0, width, height, 0, 0};
            tiles[0] = t;
        }
        return 1;
    }
    int tile_h = tile_size < height ? tile_size : height;
    int tile_w = tile_size < width ? tile_size : width;
    int half = overlap / 2;
    if (tile_h <= overlap || tile_w <= overlap) return -1;
    int n = 0;
    for (int y = 0; y < height - overlap; y += tile_h - overlap)
        for (int x = 0; x < width - overlap; x += tile_w - overlap) {
            zo_tile t;
            t.img_x = x;
            t.img_y = y;
            t.img_w = tile_w < width - x ? tile_w : width - x;
            t.img_h = tile_h < height - y ? tile_h : height - y;
            t.lat_x = x / 16;
            t.lat_y = y / 16;
            if (latent_extent(t.img_x, t.img_w, latent_w, &t.lat_w)) return -1;
            if (latent_extent(t.img_y, t.img_h, latent_h, &t.lat_h)) return -1;
            if (t.lat_x + t.lat_w > latent_w || t.lat_y + t.lat_h > latent_h) return -1;
            int left = t.img_x == 0 ? 0 : half;
            int top = t.img_y == 0 ? 0 : half;
            int right = t.img_x + t.img_w >= width ? 0 : half;
            int bottom = t.img_y + t.img_h >= height ? 0 : half;
            if (t.img_w <= left + right || t.img_h <= top + bottom) return -1;
            t.core_x = t.img_x + left;
            t.core_y = t.img_y + top;
            t.core_w = t.img_w - left - right;
            t.core_h = t.img_h - top - bottom;
            t.off_x = left;
            t.off_y = top;
            if (n < max_tiles) tiles[n] = t;
            n++;
        }
    return n;
}

/* Tensor::window of a planar latent */
static T window(const float *src, int c, int h, int w, int x0, int y0, int ww, int hh) {
    T o = t_new(c, hh, ww);
    for (int ci = 0; ci < c; ci++)
        for (int y = 0; y < hh; y++)
            memcpy(o.d + ((size_t)ci * hh + y) * ww, src + ((size_t)ci * h + y0 + y) * w + x0,
                   sizeof(float) * ww);
    return o;
}

int zo_synthesize(const zo_ckpt *ck_y, const zo_ckpt *ck_uv, int op, const float *y_hat_y,
                  const float *y_hat_uv, int lh, int lw, int height, int width, int out_h,
                  int out_w, int tile_size, int overlap, int sv, int sh, float *rec_y,
                  float *rec_u, float *rec_v) {
    int nt = zo_synthesis_tiles(height, width, lh, lw, tile_size, overlap, NULL, 0);
    if (nt <= 0) return -1;
    zo_tile *tiles = (zo_tile *)malloc(sizeof(zo_tile) * nt);
    zo_synthesis_tiles(height, width, lh, lw, tile_size, overlap, tiles, nt);
    int cw = cdiv(out_w, sh);
    for (int i = 0; i < nt; i++) {
        zo_tile t = tiles[i];
        /* synthesize_luma_into (reconstruct.rs:379-411) */
        T ly = window(y_hat_y, 160, lh, lw, t.lat_x, t.lat_y, t.lat_w, t.lat_h);
        int oh, ow;
        zo_synth_out_size(op, 0, t.img_h, t.img_w, &oh, &ow);
        float *ty = (float *)malloc(sizeof(float) * oh * ow);
        zo_synthesis_primary(ck_y, op, ly.d, ly.h, ly.w, t.img_h, t.img_w, ty);
        if (oh < t.off_y + t.core_h || ow < t.off_x + t.core_w) return -1;
        int cols = t.core_w < out_w - t.core_x ? t.core_w : out_w - t.core_x;
        if (cols < 0) cols = 0;
        for (int y = 0; y < t.core_h && t.core_y + y < out_h; y++)
            memcpy(rec_y + (size_t)(t.core_y + y) * out_w + t.core_x,
                   ty + (size_t)(t.off_y + y) * ow + t.off_x, sizeof(float) * cols);
        free(ty);
        /* synthesize_chroma_into (reconstruct.rs:416-464) */
        T luv = window(y_hat_uv, 96, lh, lw, t.lat_x, t.lat_y, t.lat_w, t.lat_h);
        zo_synth_out_size(op, 1, t.img_h, t.img_w, &oh, &ow);
        float *tuv = (float *)malloc(sizeof(float) * 2 * oh * ow);
        zo_synthesis_secondary(ck_uv, op, ly.d, ly.h, ly.w, luv.d, luv.h, luv.w, t.img_h,
                               t.img_w, tuv);
        if (oh < t.off_y + t.core_h || ow < t.off_x + t.core_w) return -1;
        for (int c = 0; c < 2; c++) {
            const float *src = tuv + (size_t)c * oh * ow;
            float *dst = c == 0 ? rec_u : rec_v;
            int y_end = t.core_y + t.core_h < out_h ? t.core_y + t.core_h : out_h;
            int x_end = t.core_x + t.core_w < out_w ? t.core_x + t.core_w : out_w;
            for (int py = cdiv(t.core_y, sv) * sv; py < y_end; py += sv)
                for (int px = cdiv(t.core_x, sh) * sh; px < x_end; px += sh)
                    dst[(size_t)(py / sv) * cw + px / sh] =
                        src[(size_t)(t.off_y + py - t.core_y) * ow + t.off_x + px - t.core_x];
        }
        free(tuv);
        t_free(&ly);
        t_free(&luv);
    }
    free(tiles);
    return 0;
}

/* ======================================================================================= */
/* Output stage (output.rs:28-438)                                                            */
/* ======================================================================================= */

static float convert_range(float x, float in_max, float out_max) {
    return ((x - 0.0f) / in_max) * out_max + 0.0f;
}

/* quantize_plane_par (output.rs:330-342): clip, scale, round half to even, clip */
void zo_quantize_plane(const float *x, int64_t n, int bit_depth, uint16_t *out) {
    float mx = (float)((1u << bit_depth) - 1);
    for (int64_t i = 0; i < n; i++)
        out[i] = (uint16_t)clampf(rintf(convert_range(clampf(x[i], 0.0f, 255.0f), 255.0f, mx)),
                                  0.0f, mx);
}

static const float CUBIC_A = -0.75f;
static float cubic1(float x) {
    float p = fmaf(CUBIC_A + 2.0f, x, -(CUBIC_A + 3.0f));
    return fmaf(p * x, x, 1.0f);
}
static float cubic2(float x) {
    float p = fmaf(CUBIC_A, x, -5.0f * CUBIC_A);
    p = fmaf(p, x, 8.0f * CUBIC_A);
    return fmaf(p, x, -4.0f * CUBIC_A);
}
/* dot4 (output.rs:85-91): fma(x3,c3, fma(x2,c2, fma(x0,c0, x1*c1))) */
static float dot4(const float x[4], const float c[4]) {
    float acc = x[1] * c[1];
    acc = fmaf(x[0], c[0], acc);
    acc = fmaf(x[2], c[2], acc);
    return fmaf(x[3], c[3], acc);
}
static void cubic_taps(int dst, int in_len, int out_len, int idx[4], float wt[4]) {
    float scale = out_len > 1 ? (float)(in_len - 1) / (float)(out_len - 1) : 0.0f;
    float real = scale * (float)dst;
    float base = floorf(real);
    float t = real - base;
    int b = (int)base;
    for (int k = 0; k < 4; k++) {
        int v = b - 1 + k;
        idx[k] = v < 0 ? 0 : v > in_len - 1 ? in_len - 1 : v;
    }
    float u = 1.0f - t;
    wt[0] = cubic2(t + 1.0f);
    wt[1] = cubic1(t);
    wt[2] = cubic1(u);
    wt[3] = cubic2(u + 1.0f);
}

/* resize_bicubic_par (output.rs:103-151), align_corners = True */
int zo_resize_bicubic(const float *src, int c, int h, int w, int out_h, int out_w,
                      float *out) {
    if (h <= 0 || w <= 0) return -1;
    int *xi = (int *)malloc(sizeof(int) * 4 * out_w);
    float *xw = (float *)malloc(sizeof(float) * 4 * out_w);
    int *yi = (int *)malloc(sizeof(int) * 4 * out_h);
    float *yw = (float *)malloc(sizeof(float) * 4 * out_h);
    for (int x = 0; x < out_w; x++) cubic_taps(x, w, out_w, xi + 4 * x, xw + 4 * x);
    for (int y = 0; y < out_h; y++) cubic_taps(y, h, out_h, yi + 4 * y, yw + 4 * y);
    for (int ci = 0; ci < c; ci++) {
        const float *sp = src + (size_t)ci * h * w;
        float *op = out + (size_t)ci * out_h * out_w;
#pragma omp parallel for schedule(static) num_threads(g_threads)
        for (int y = 0; y < out_h; y++) {
            for (int x = 0; x < out_w; x++) {
                float rows[4];
                for (int k = 0; k < 4; k++) {
                    const float *row = sp + (size_t)yi[4 * y + k] * w;
                    float v[4] = {row[xi[4 * x]], row[xi[4 * x + 1]], row[xi[4 * x + 2]],
                                  row[xi[4 * x + 3]]};
                    rows[k] = dot4(v, xw + 4 * x);
                }
                op[(size_t)y * out_w + x] = dot4(rows, yw + 4 * y);
            }
        }
    }
    free(xi);
    free(xw);
    free(yi);
    free(yw);
    return 0;
}

/* to_rgb_planes_owned_par (output.rs:218-262) */
void zo_to_rgb_planes(float *py, float *pu, float *pv, int64_t n) {
    const double KR = 0.2126, KG = 0.7152, KB = 0.0722, KBY = 1.8556, KRY = 1.5748;
    float kry = (float)KRY, kby = (float)KBY;
    float gu = (float)(KB * KBY / KG), gv = (float)(KR * KRY / KG);
    for (int64_t i = 0; i < n; i++) {
        float y = convert_range(py[i], 255.0f, 1.0f);
        float u = convert_range(pu[i], 255.0f, 1.0f) - 0.5f;
        float v = convert_range(pv[i], 255.0f, 1.0f) - 0.5f;
        float rv = y + kry * v;
        float gvv = y - gu * u - gv * v;
        float bv = y + kby * u;
        py[i] = clampf(convert_range(rv, 1.0f, 255.0f), 0.0f, 255.0f);
        pu[i] = clampf(convert_range(gvv, 1.0f, 255.0f), 0.0f, 255.0f);
        pv[i] = clampf(convert_range(bv, 1.0f, 255.0f), 0.0f, 255.0f);
    }
}

/* quantize_par (output.rs:407-438) */
void zo_quantize_rgb(const float *r, const float *g, const float *b, int64_t n, int bit_depth,
                     uint16_t *out) {
    float mx = (float)((1u << bit_depth) - 1);
    for (int64_t i = 0; i < n; i++) {
        out[3 * i] = (uint16_t)clampf(rintf(convert_range(r[i], 255.0f, mx)), 0.0f, mx);
        out[3 * i + 1] = (uint16_t)clampf(rintf(convert_range(g[i], 255.0f, mx)), 0.0f, mx);
        out[3 * i + 2] = (uint16_t)clampf(rintf(convert_range(b[i], 255.0f, mx)), 0.0f, mx);
    }
}

/* ======================================================================================= */
/* Encoder front end: colour pre-processing (encoder/colour.rs) and analysis tiling         */
/* (encoder/tiles.rs, encoder/mod.rs)                                                        */
/* ======================================================================================= */

/* replicate_pad (colour.rs:331-342) to an even size, then unshuffle_into (colour.rs:316-329):
 * channel k = dy * 2 + dx of out takes sample (2y + dy, 2x + dx) of the padded plane */
static void unshuffle_padded(const float *plane, int h, int w, float *out) {
    int ph = h + h % 2, pw = w + w % 2, ch = ph / 2, cw = pw / 2;
    for (int k = 0; k < 4; k++) {
        int dy = k / 2, dx = k % 2;
        float *dst = out + (size_t)k * ch * cw;
        for (int y = 0; y < ch; y++) {
            int sy = 2 * y + dy < h ? 2 * y + dy : h - 1;
            for (int x = 0; x < cw; x++) {
                int sx = 2 * x + dx < w ? 2 * x + dx : w - 1;
                dst[(size_t)y * cw + x] = plane[(size_t)sy * w + sx];
            }
        }
    }
}

void zo_preprocess_rgb(const uint8_t *rgb, int h, int w, float *luma, float *chroma) {
    /* BT.709 weights and chroma denominators (colour.rs:26-30) */
    const float KR = 0.2126f, KG = 0.7152f, KB = 0.0722f, KBY = 1.8556f, KRY = 1.5748f;
    const float mx = 255.0f;
    size_t n = (size_t)h * w;
    float *u = (float *)malloc(sizeof(float) * n);
    float *v = (float *)malloc(sizeof(float) * n);
    for (size_t i = 0; i < n; i++) {
        /* to_YUV_ on [0, 1] (colour.rs:418-428), then * 255 (source_planes, :396-400); every
         * operation rounded on its own (Rust does not contract) */
        float r = (float)rgb[3 * i] / mx, g = (float)rgb[3 * i + 1] / mx,
              b = (float)rgb[3 * i + 2] / mx;
        float y = KR * r + KG * g + KB * b;
        luma[i] = y * 255.0f;
        u[i] = ((b - y) / KBY + 0.5f) * 255.0f;
        v[i] = ((r - y) / KRY + 0.5f) * 255.0f;
    }
    int ph = h + h % 2, pw = w + w % 2;
    size_t cplane = (size_t)(ph / 2) * (pw / 2);
    unshuffle_padded(luma, h, w, chroma);
    unshuffle_padded(u, h, w, chroma + 4 * cplane);
    unshuffle_padded(v, h, w, chroma + 8 * cplane);
    free(u);
    free(v);
}

/* cfg/CTC.json tile_manager_enc per component (encoder/tiles.rs:20-24) */
static const int ENC_SAMPLES_PER_TILE[2] = {1048576, 262144};
static const int ENC_TILE_OVERLAP[2] = {64, 32};
static const int ENC_LATENT_DOWNSCALE[2] = {16, 8};

/* `_get_latent_tile_from_image_tile` for one axis (encoder/tiles.rs:276-284) */
static int latent_len(int pos, int len, int down, int full, int *out) {
    if (len % down && cdiv(pos + len, down) < full) return -1;
    *out = cdiv(len, down);
    return 0;
}

int zo_analysis_tiles(int ccs, int h, int w, int lh, int lw, zo_atile *tiles, int max_tiles) {
    if (ccs < 0 || ccs > 1 || h <= 0 || w <= 0) return -1;
    const int nsamp = ENC_SAMPLES_PER_TILE[ccs], yd = ENC_LATENT_DOWNSCALE[ccs];
    if ((int64_t)nsamp >= (int64_t)h * w) {  /* tile_size: no tiling (tiles.rs:53-60) */
        if (max_tiles > 0 && tiles) {
            zo_atile t = {0, 0, w, h, 0, 0, lw, lh, 0, 0, lw, lh, 0, 0};
            tiles[0] = t;
        }
        return 1;
    }
    const int size = cdiv((int)floor(sqrt((double)nsamp)), yd) * yd;
    const int overlap = ENC_TILE_OVERLAP[ccs];
    const int tile_h = size < h ? size : h, tile_w = size < w ? size : w;
    if (tile_h <= overlap || tile_w <= overlap) return -1;
    const int o = overlap / 2 / yd;
    int n = 0;
    for (int y = 0; y < h - overlap; y += tile_h - overlap)
        for (int x = 0; x < w - overlap; x += tile_w - overlap) {
            zo_atile t;
            t.img_x = x;
            t.img_y = y;
            t.img_w = tile_w < w - x ? tile_w : w - x;
            t.img_h = tile_h < h - y ? tile_h : h - y;
            t.lat_x = x / yd;
            t.lat_y = y / yd;
            if (latent_len(t.img_x, t.img_w, yd, lw, &t.lat_w) ||
                latent_len(t.img_y, t.img_h, yd, lh, &t.lat_h))
                return -1;
            /* `_get_core_of_overlapping_tile`, picture-border branch (tiles.rs:127-139) */
            int left = x == 0 ? 0 : o, top = y == 0 ? 0 : o;
            int right = x + t.img_w >= w ? 0 : o, bottom = y + t.img_h >= h ? 0 : o;
            if (t.lat_w < left + right || t.lat_h < top + bottom) return -1;
            t.core_x = t.lat_x + left;
            t.core_y = t.lat_y + top;
            t.core_w = t.lat_w - left - right;
            t.core_h = t.lat_h - top - bottom;
            t.off_x = left;
            t.off_y = top;
            if (tiles && n < max_tiles) tiles[n] = t;
            n++;
        }
    return n;
}

int zo_analyze_tiled(const zo_ckpt *ck, int op, int ccs, const float *x, int h, int w,
                     float *out) {
    const int cin = ccs ? 12 : 1, cout = ccs ? 96 : 160, d = ENC_LATENT_DOWNSCALE[ccs];
    const int lh = cdiv(h, d), lw = cdiv(w, d);
    int nt = zo_analysis_tiles(ccs, h, w, lh, lw, NULL, 0);
    if (nt <= 0) return -1;
    zo_atile *tiles = (zo_atile *)malloc(sizeof(zo_atile) * nt);
    zo_analysis_tiles(ccs, h, w, lh, lw, tiles, nt);
    int rc = 0;
    for (int i = 0; i < nt && !rc; i++) {
        zo_atile t = tiles[i];
        float *win = (float *)malloc(sizeof(float) * cin * t.img_h * t.img_w);
        for (int c = 0; c < cin; c++)
            for (int y = 0; y < t.img_h; y++)
                memcpy(win + ((size_t)c * t.img_h + y) * t.img_w,
                       x + ((size_t)c * h + t.img_y + y) * w + t.img_x, sizeof(float) * t.img_w);
        float *lat = (float *)malloc(sizeof(float) * cout * t.lat_h * t.lat_w);
        rc = ccs ? zo_analysis_secondary(ck, op, win, t.img_h, t.img_w, lat)
                 : zo_analysis_primary(ck, op, win, t.img_h, t.img_w, lat);
        for (int c = 0; c < cout && !rc; c++)
            for (int y = 0; y < t.core_h; y++)
                memcpy(out + ((size_t)c * lh + t.core_y + y) * lw + t.core_x,
                       lat + ((size_t)c * t.lat_h + t.off_y + y) * t.lat_w + t.off_x,
                       sizeof(float) * t.core_w);
        free(win);
        free(lat);
    }
    free(tiles);
    return rc;
}

/* ======================================================================================= */
/* LEF luma edge filter (src/filters/lef.rs:67-171)                                         */
/* ======================================================================================= */

static const int LEF_THR[4][3] = {{600, 1200, 2000}, {800, 1400, 2400}, {1000, 1600, 2800},
                                  {1200, 2000, 3200}};
static const float LEF_MAG[4][3] = {{1.10f, 1.13f, 1.16f}, {1.07f, 1.09f, 1.11f},
                                    {1.03f, 1.04f, 1.05f}, {1.01f, 1.02f, 1.03f}};

/* torch nearest interpolation source index: min(floor(dst * (src / dst)), src - 1), f32 */
int zo_nearest_index(int i, int src, int dst) {
    const float scale = (float)src / (float)dst;
    const int v = (int)floorf((float)i * scale);
    return v < src - 1 ? v : src - 1;
}

static float clamp01(float v) { return v < 0.f ? 0.f : v > 1.f ? 1.f : v; }

/* LEF `sharpen`: luma [h][w] in [0, 255] filtered into out (out != luma); scale_log [c][sh][sw]
 * int32. Returns -1 for the inputs the crate rejects. */
int zo_lef(const float *luma, int h, int w, const int32_t *scale_log, int c, int sh, int sw,
           int channel, int model_id, int bit_depth, float *out) {
    if (model_id < 0 || model_id > 3 || channel < 0 || channel >= c) return -1;
    if (h <= 0 || w <= 0 || sh <= 0 || sw <= 0 || bit_depth < 1 || bit_depth > 16) return -1;
    const float range = 255.f, outer = 5.f / 64.f, centre = 24.f / 64.f;
    const int32_t *region = scale_log + (size_t)channel * sh * sw;
    float *x = (float *)malloc(sizeof(float) * (size_t)h * w);
    for (size_t i = 0; i < (size_t)h * w; i++) x[i] = luma[i] / range;
    for (int y = 0; y < h; y++) {
        const float *cur = x + (size_t)y * w;
        float *o = out + (size_t)y * w;
        if (y == 0 || y + 1 == h || w < 3) {
            for (int i = 0; i < w; i++) o[i] = clamp01(cur[i]) * range;
            continue;
        }
        const float *up = cur - w, *down = cur + w;
        const int32_t *rrow = region + (size_t)zo_nearest_index(y, sh, h) * sw;
        o[0] = clamp01(cur[0]) * range;
        o[w - 1] = clamp01(cur[w - 1]) * range;
        for (int i = 1; i < w - 1; i++) {
            const int s = rrow[zo_nearest_index(i, sw, w)];
            const int *t = LEF_THR[model_id];
            const float g = s >= t[2] ? LEF_MAG[model_id][2] : s >= t[1] ? LEF_MAG[model_id][1]
                            : s >= t[0] ? LEF_MAG[model_id][0] : 1.f;
            float acc = 0.f;
            acc = fmaf(up[i - 1], outer, acc);
            acc = fmaf(up[i], outer, acc);
            acc = fmaf(up[i + 1], outer, acc);
            acc = fmaf(cur[i - 1], outer, acc);
            acc = fmaf(cur[i], centre, acc);
            acc = fmaf(cur[i + 1], outer, acc);
            acc = fmaf(down[i - 1], outer, acc);
            acc = fmaf(down[i], outer, acc);
            acc = fmaf(down[i + 1], outer, acc);
            const float blur = clamp01(acc);
            const float diff = (cur[i] - blur) * g;
            o[i] = clamp01(blur + diff) * range;
        }
    }
    free(x);
    return 0;
}


/* ======================================================================================= */
/* eICCI post-filter (src/model/icci.rs, src/filters/icci.rs), 4:4:4 pictures               */
/* ======================================================================================= */

#define ICCI_NF 48
#define ICCI_BANDS 16

static double ck_scalar(const zo_ckpt *ck, const char *name) {
    const zo_param *p = find(ck, name);
    if (!p || p->ndim > 1 || (p->ndim == 1 && p->shape[0] != 1)) ZO_FAIL(name);
    return (double)p->data[0];
}

/* folded_conv (icci.rs:99-125): conv `prefix` then the per-channel affine map (a, shift):
 * w' = w * a, b' = b * a + shift in f64, rounded once; the conv runs in f32 */
typedef struct {
    int cin, cout, kh, kw;
    float *w, *b;
} FConv;

static FConv fold(const zo_ckpt *ck, const char *prefix, int cin, int cout, int kh, int kw,
                  const double *a, const double *shift) {
    FConv f = {cin, cout, kh, kw, NULL, NULL};
    const float *w = need(ck, prefix, "weight", cout, cin, kh, kw);
    const float *b = need(ck, prefix, "bias", cout, -1, -1, -1);
    const int per = cin * kh * kw;
    f.w = (float *)malloc(sizeof(float) * cout * per);
    f.b = (float *)malloc(sizeof(float) * cout);
    for (int o = 0; o < cout; o++) {
        for (int i = 0; i < per; i++) f.w[o * per + i] = (float)((double)w[o * per + i] * a[o]);
        f.b[o] = (float)((double)b[o] * a[o] + shift[o]);
    }
    return f;
}

/* batch_norm (icci.rs:64-87): (a s, (beta - mean a) s), a = gamma / sqrt(var + 1e-5) */
static void bn_affine(const zo_ckpt *ck, const char *prefix, double s, double *a, double *sh) {
    const float *g = need(ck, prefix, "weight", ICCI_NF, -1, -1, -1);
    const float *be = need(ck, prefix, "bias", ICCI_NF, -1, -1, -1);
    const float *m = need(ck, prefix, "running_mean", ICCI_NF, -1, -1, -1);
    const float *v = need(ck, prefix, "running_var", ICCI_NF, -1, -1, -1);
    for (int c = 0; c < ICCI_NF; c++) {
        const double k = (double)g[c] / sqrt((double)v[c] + 1e-5);
        a[c] = k * s;
        sh[c] = ((double)be[c] - (double)m[c] * k) * s;
    }
}

static T fconv(const FConv *f, const T *x) {
    T o = t_new(f->cout, x->h, x->w);
    if (zo_conv2d(x->d, x->c, x->h, x->w, f->w, f->b, f->cout, f->kh, f->kw, 1, f->kh / 2,
                  f->kw / 2, 1, NULL, o.d))
        ZO_FAIL("icci conv");
    return o;
}

static void ffree(FConv *f) {
    free(f->w);
    free(f->b);
}

/* Trunk::forward (icci.rs:168-178): relu(first(x)), then f += conv2(relu(conv1(f))) */
static T icci_trunk(const zo_ckpt *ck, const T *x, const char *first, const char *bn,
                    const char *hidden, int blocks) {
    double a[ICCI_NF], sh[ICCI_NF];
    char n1[128], n2[128];
    bn_affine(ck, bn, 1.0, a, sh);
    FConv f0 = fold(ck, first, 3 * ICCI_BANDS, ICCI_NF, 3, 3, a, sh);
    T f = fconv(&f0, x);
    ffree(&f0);
    zo_relu(f.d, t_len(&f));
    for (int i = 0; i < blocks; i++) {
        snprintf(n1, sizeof n1, "%s.%d.scale", hidden, i);
        const double s = ck_scalar(ck, n1);
        double a2[ICCI_NF], sh2[ICCI_NF];
        snprintf(n1, sizeof n1, "%s.%d.BN1", hidden, i);
        bn_affine(ck, n1, 1.0, a, sh);
        snprintf(n2, sizeof n2, "%s.%d.BN2", hidden, i);
        bn_affine(ck, n2, s, a2, sh2);
        snprintf(n1, sizeof n1, "%s.%d.conv1", hidden, i);
        snprintf(n2, sizeof n2, "%s.%d.conv2", hidden, i);
        FConv c1 = fold(ck, n1, ICCI_NF, ICCI_NF, 1, 3, a, sh);
        FConv c2 = fold(ck, n2, ICCI_NF, ICCI_NF, 3, 1, a2, sh2);
        T o = fconv(&c1, &f);
        zo_relu(o.d, t_len(&o));
        T r = fconv(&c2, &o);
        zo_add(f.d, r.d, t_len(&f));
        t_free(&o);
        t_free(&r);
        ffree(&c1);
        ffree(&c2);
    }
    return f;
}

/* the last conv of a plane: 48 -> 16 sub-band corrections times the plane's scale */
static T icci_last(const zo_ckpt *ck, const T *f, const char *conv, const char *scale) {
    double a[ICCI_BANDS], sh[ICCI_BANDS];
    const double s = ck_scalar(ck, scale);
    for (int i = 0; i < ICCI_BANDS; i++) {
        a[i] = s;
        sh[i] = 0.0;
    }
    FConv c = fold(ck, conv, ICCI_NF, ICCI_BANDS, 3, 3, a, sh);
    T o = fconv(&c, f);
    ffree(&c);
    return o;
}

static void haar4(float x1, float x2, float x3, float x4, float o[4]) {
    o[0] = x1 + x2 + x3 + x4;
    o[1] = -x1 - x2 + x3 + x4;
    o[2] = -x1 + x2 - x3 + x4;
    o[3] = x1 - x2 - x3 + x4;
}
static void ihaar4(float x1, float x2, float x3, float x4, float o[4]) {
    o[0] = x1 - x2 - x3 + x4;
    o[1] = x1 - x2 + x3 - x4;
    o[2] = x1 + x2 - x3 - x4;
    o[3] = x1 + x2 + x3 + x4;
}

/* dwt2_block (icci.rs:326-360): two Haar levels of a 4 x 4 block p[row][col] */
void zo_dwt2_block(const float p[16], float out[16]) {
    float l1[2][2][4];
    for (int by = 0; by < 2; by++)
        for (int bx = 0; bx < 2; bx++) {
            const int r = 2 * by, c = 2 * bx;
            haar4(p[r * 4 + c] / 2.f, p[(r + 1) * 4 + c] / 2.f, p[r * 4 + c + 1] / 2.f,
                  p[(r + 1) * 4 + c + 1] / 2.f, l1[by][bx]);
        }
    for (int k = 0; k < 4; k++)
        haar4(l1[0][0][k] / 2.f, l1[1][0][k] / 2.f, l1[0][1][k] / 2.f, l1[1][1][k] / 2.f,
              out + 4 * k);
}

/* idwt2_block (icci.rs:363-402) */
void zo_idwt2_block(const float s[16], float out[16]) {
    float q[4][2][2];
    for (int i = 0; i < 4; i++) {
        float r[4];
        ihaar4(s[4 * i] / 2.f, s[4 * i + 1] / 2.f, s[4 * i + 2] / 2.f, s[4 * i + 3] / 2.f, r);
        q[i][0][0] = r[0];
        q[i][0][1] = r[2];
        q[i][1][0] = r[1];
        q[i][1][1] = r[3];
    }
    for (int dy = 0; dy < 2; dy++)
        for (int dx = 0; dx < 2; dx++) {
            float r[4];
            ihaar4(q[0][dy][dx] / 2.f, q[1][dy][dx] / 2.f, q[2][dy][dx] / 2.f,
                   q[3][dy][dx] / 2.f, r);
            out[(2 * dy) * 4 + 2 * dx] = r[0];
            out[(2 * dy + 1) * 4 + 2 * dx] = r[1];
            out[(2 * dy) * 4 + 2 * dx + 1] = r[2];
            out[(2 * dy + 1) * 4 + 2 * dx + 1] = r[3];
        }
}

/* axis of the filter tiling (filters/icci.rs:68-96): starts / lengths; -1 when malformed */
#define ICCI_MIN_TILE 176
static int icci_axis(int len, int tile, int overlap, int *pos, int *sz, int max) {
    tile = tile < len ? tile : len;
    if (tile <= overlap || len <= overlap) return -1;
    int n = 0;
    for (int p = 0; p < len - overlap; p += tile - overlap) {
        if (n >= max) return -1;
        pos[n] = p;
        sz[n] = tile < len - p ? tile : len - p;
        n++;
    }
    if (sz[n - 1] < ICCI_MIN_TILE) {
        if (n < 2 || sz[n - 2] <= ICCI_MIN_TILE + overlap) return -1;
        sz[n - 2] -= ICCI_MIN_TILE;
        pos[n - 1] -= ICCI_MIN_TILE;
        sz[n - 1] += ICCI_MIN_TILE;
    }
    return n;
}

/* The eICCI filter (filters/icci.rs:175-325) of a 4:4:4 picture in place: planes y, u, v
 * [h][w] in [0, 255]; ck_y filters luma, ck_uv the chroma planes selected by use_u / use_v
 * (NULL: not filtered); tile_size 0: one tile. Tiles in raster order, each reading the cores
 * its predecessors wrote. Returns -1 for a malformed tiling. */
int zo_icci_filter(const zo_ckpt *ck_y, const zo_ckpt *ck_uv, int use_u, int use_v, float *y,
                   float *u, float *v, int h, int w, int tile_size, int overlap) {
    enum { MAXT = 256 };
    int ry[MAXT], rh[MAXT], cx[MAXT], cw[MAXT], nr = 1, nc = 1;
    if (h <= 0 || w <= 0) return -1;
    if (tile_size > 0) {
        nr = icci_axis(h, tile_size, overlap, ry, rh, MAXT);
        nc = icci_axis(w, tile_size, overlap, cx, cw, MAXT);
        if (nr < 0 || nc < 0) return -1;
    } else {
        ry[0] = cx[0] = 0;
        rh[0] = h;
        cw[0] = w;
        overlap = 0;
    }
    const int half = overlap / 2;
    float *planes[3] = {y, u, v};
    const size_t n = (size_t)h * w;
    for (int p = 0; p < 3; p++)
        for (size_t i = 0; i < n; i++) planes[p][i] = planes[p][i] / 255.f;
    for (int ti = 0; ti < nr; ti++)
        for (int tj = 0; tj < nc; tj++) {
            const int x0 = cx[tj], y0 = ry[ti], tw = cw[tj], th = rh[ti];
            const int left = x0 == 0 ? 0 : half, top = y0 == 0 ? 0 : half;
            const int right = x0 + tw >= w ? 0 : half, bottom = y0 + th >= h ? 0 : half;
            if (tw <= left + right || th <= top + bottom) return -1;
            if (!ck_y && !ck_uv) continue;
            const int bh = cdiv(th, 4), bw = cdiv(tw, 4);
            T in = t_new(3 * ICCI_BANDS, bh, bw);
            for (int p = 0; p < 3; p++)
                for (int by = 0; by < bh; by++)
                    for (int bx = 0; bx < bw; bx++) {
                        float blk[16], o[16];
                        for (int r = 0; r < 4; r++)
                            for (int c = 0; c < 4; c++) {
                                const int sy = y0 + (4 * by + r < th - 1 ? 4 * by + r : th - 1);
                                const int sx = x0 + (4 * bx + c < tw - 1 ? 4 * bx + c : tw - 1);
                                blk[r * 4 + c] = planes[p][(size_t)sy * w + sx];
                            }
                        zo_dwt2_block(blk, o);
                        for (int k = 0; k < 16; k++)
                            in.d[((size_t)(p * 16 + k) * bh + by) * bw + bx] = o[k];
                    }
            T corr[3] = {{0, 0, 0, NULL}, {0, 0, 0, NULL}, {0, 0, 0, NULL}};
            if (ck_y) {
                T f = icci_trunk(ck_y, &in, "conv_first_Y", "BNY", "hidden_layer_Y", 2);
                corr[0] = icci_last(ck_y, &f, "conv_last_Y", "scaleY");
                t_free(&f);
            }
            if (ck_uv && (use_u || use_v)) {
                T f = icci_trunk(ck_uv, &in, "conv_firstUV", "BNUV", "hidden_layer_UV", 4);
                if (use_u) corr[1] = icci_last(ck_uv, &f, "conv_last_u", "scaleU");
                if (use_v) corr[2] = icci_last(ck_uv, &f, "conv_last_v", "scaleV");
                t_free(&f);
            }
            for (int p = 0; p < 3; p++) {
                if (!corr[p].d) continue;
                for (int by = 0; by < bh; by++)
                    for (int bx = 0; bx < bw; bx++) {
                        float s[16], o[16];
                        for (int k = 0; k < 16; k++) {
                            const size_t i = ((size_t)k * bh + by) * bw + bx;
                            s[k] = corr[p].d[i] + in.d[((size_t)(p * 16 + k) * bh + by) * bw + bx];
                        }
                        zo_idwt2_block(s, o);
                        for (int r = 0; r < 4; r++)
                            for (int c = 0; c < 4; c++) {
                                const int fy = 4 * by + r, fx = 4 * bx + c;  /* padded tile */
                                if (fy < top || fy >= th - bottom || fx < left || fx >= tw - right)
                                    continue;
                                planes[p][(size_t)(y0 + fy) * w + x0 + fx] = o[r * 4 + c];
                            }
                    }
                t_free(&corr[p]);
            }
            t_free(&in);
        }
    for (int p = 0; p < 3; p++)
        for (size_t i = 0; i < n; i++) planes[p][i] = clamp01(planes[p][i]) * 255.f;
    return 0;
}


/* ======================================================================================= */
/* EFE post-filters (src/filters/efe_linear.rs, src/filters/efe_nonlinear.rs)              */
/* ======================================================================================= */

/* The candidate splits of a phase plane (efe_linear.rs:34-73, `EFElinear.cands`): regions as
 * fractions [row_start, row_end, col_start, col_end]; EFE_NSPLITS = header.rs:619. Constants of
 * the format, kept as the reference lists them. */
static const int EFE_NSPLITS[8] = {1, 2, 2, 3, 3, 4, 6, 6};
static const double EFE_SPLITS[8][6][4] = {
    {{0, 1, 0, 1}},
    {{0, .5, 0, 1}, {.5, 1, 0, 1}},
    {{0, 1, 0, .5}, {0, 1, .5, 1}},
    {{0, 1, 0, .33}, {0, 1, .33, .66}, {0, 1, .66, 1}},
    {{0, .33, 0, 1}, {.33, .66, 0, 1}, {.66, 1, 0, 1}},
    {{0, .5, 0, .5}, {0, .5, .5, 1}, {.5, 1, 0, .5}, {.5, 1, .5, 1}},
    {{0, .33, 0, .5}, {0, .33, .5, 1}, {.33, .66, 0, .5}, {.33, .66, .5, 1}, {.66, 1, 0, .5},
     {.66, 1, .5, 1}},
    {{0, .5, 0, .33}, {.5, 1, 0, .33}, {0, .5, .33, .66}, {.5, 1, .33, .66}, {0, .5, .66, 1},
     {.5, 1, .66, 1}},
};
/* DCT-IF 4-tap interpolation kernels of the sub-sampling phases 0..3 (efe_linear.rs:77-110),
 * unsignalled constants of the format: horizontal, vertical and diagonal half-sample taps. */
static const float EFE_DCT_IF[4][16] = {
    {0},
    {0, 0, 0, 0, -0.0625f, -0.4375f, 0.5625f, -0.0625f, 0, 0, 0, 0, 0, 0, 0, 0},
    {0, -0.0625f, 0, 0, 0, -0.4375f, 0, 0, 0, 0.5625f, 0, 0, 0, -0.0625f, 0, 0},
    {0.00390625f, -0.03515625f, -0.03515625f, 0.00390625f,
     -0.03515625f, -0.68359375f, 0.31640625f, -0.03515625f,
     -0.03515625f, 0.31640625f, 0.31640625f, -0.03515625f,
     0.00390625f, -0.03515625f, -0.03515625f, 0.00390625f},
};

/* `deinteger` (efe_linear.rs:113-115): (code - 32767) / 2^11 in f32 */
static float efe_deinteger(long long code) { return (float)(code - 32767) / 2048.0f; }

/* round(f * (s + 31) / 32) * 32, Python's round (half to even, rint) on doubles
 * (efe_linear.rs:128-131) */
int zo_efe_split_edge(double fraction, int s) {
    return (int)rint(fraction * (double)(s + 31) / 32.0) * 32;
}

typedef struct {
    int r0, r1, c0, c1, k, before;
    float chroma[4][16], luma[16];
} efe_region;

/* `regions` (efe_linear.rs:134-219): the non-empty regions of plane p with their kernels
 * (identity and, below the source's chroma resolution, DCT-IF taps included). */
static int efe_regions(const zo_efe_linear_set *set, int p, int coded_444, int s0, int s1,
                       efe_region *out, int *nout) {
    const int weighted = set->cand[p] >= 0;
    const int cand = weighted ? set->cand[p] : 0, fl = weighted ? set->filter_len[p] : 0;
    if (set->cand[p] < -1 || cand >= 8 || fl > 4 || fl < 0 || (weighted && fl == 0)) return 6;
    if (weighted && (!set->chroma_codes[p] || !set->luma_codes[p])) return 6;
    *nout = 0;
    for (int num = 0; num < EFE_NSPLITS[cand]; num++) {
        const double *sp = EFE_SPLITS[cand][num];
        const int r0 = zo_efe_split_edge(sp[0], s0), c0 = zo_efe_split_edge(sp[2], s1);
        int r1 = zo_efe_split_edge(sp[1], s0), c1 = zo_efe_split_edge(sp[3], s1);
        if (r1 > s0) r1 = s0;
        if (c1 > s1) c1 = s1;
        if (r0 >= r1 || c0 >= c1) continue;
        efe_region *r = &out[(*nout)++];
        memset(r, 0, sizeof *r);
        r->r0 = r0; r->r1 = r1; r->c0 = c0; r->c1 = c1;
        int off;
        if (coded_444) {
            r->k = fl;
            r->before = fl > 0 ? (fl - 1) / 2 : 0;
            off = 0;
        } else {
            r->k = 4;
            r->before = 1;
            off = 1 - ((fl > 1 ? fl : 1) - 1) / 2;
        }
        const int k = r->k, centre = coded_444 ? (fl - 1) / 2 : 1;
        if (weighted) {
            const int phases = coded_444 ? 1 : 4;
            const uint32_t *cw = set->chroma_codes[p] + (size_t)num * phases * fl * fl;
            const uint32_t *lw = set->luma_codes[p] + (size_t)num * fl * fl;
            for (int ky = 0; ky < fl; ky++)
                for (int kx = 0; kx < fl; kx++) {
                    const int dst = (off + ky) * k + off + kx;
                    r->luma[dst] = efe_deinteger((long long)lw[ky * fl + kx] + set->min_symbol);
                    for (int i = 0; i < 4; i++) {
                        const int ph = coded_444 ? 0 : i;
                        r->chroma[i][dst] = efe_deinteger(
                            (long long)cw[(ph * fl + ky) * fl + kx] + set->min_symbol);
                    }
                }
        }
        for (int i = 0; i < 4; i++) {
            if (!coded_444)
                for (int t = 0; t < k * k; t++) r->chroma[i][t] += EFE_DCT_IF[i][t];
            r->chroma[i][centre * k + centre] += 1.0f;
        }
    }
    return 0;
}

/* `phase_plane` (efe_linear.rs:238-275): phase (py, px) of src [h][w] sampled every (fv, fh)
 * samples as an s0 x s1 plane with a replicated border of 1 before and 2 after, `offset`
 * subtracted; stride s1 + 3. */
static float *efe_phase_plane(const float *src, int h, int w, int fv, int fh, int py, int px,
                              int s0, int s1, float offset) {
    const int stride = s1 + 3, rows = s0 + 3;
    float *d = (float *)calloc((size_t)rows * stride, sizeof(float));
    int direct = 0;
    if (w > px) {
        direct = (w - px + fh - 1) / fh;
        if (direct > s1) direct = s1;
    }
    for (int r = 0; r < rows; r++) {
        int sy = r > 0 ? r - 1 : 0;
        if (sy > s0 - 1) sy = s0 - 1;
        int row_i = sy * fv + py;
        if (row_i > h - 1) row_i = h - 1;
        const float *row = src + (size_t)row_i * w;
        float *dst = d + (size_t)r * stride;
        const int start = px < w - 1 ? px : w - 1;
        for (int i = 0; i < direct; i++) dst[1 + i] = row[start + i * fh] - offset;
        const float last = row[w - 1] - offset;
        const float edge = direct > 0 ? dst[direct] : last;
        const float fill = direct < s1 ? last : edge;
        for (int i = 1 + direct; i < stride; i++) dst[i] = fill;
        dst[0] = dst[1];
    }
    return d;
}

/* `filter_plane` (efe_linear.rs:308-359) for plane p; out [ch][cw] */
static int efe_filter_plane(int coded_444, const zo_efe_linear_set *set, int p, float mean,
                            int fv, int fh, int s0, int s1, float *const luma[4],
                            float *const chroma[4], int ch, int cw, float *out) {
    if (set->cand[p] < 0 && coded_444) return 2;
    efe_region reg[6];
    int nreg = 0;
    const int st = efe_regions(set, p, coded_444, s0, s1, reg, &nreg);
    if (st) return st;
    const int stride = s1 + 3;
    memset(out, 0, sizeof(float) * (size_t)ch * cw);
    float *acc = (float *)malloc(sizeof(float) * (size_t)(s1 + 1));
    float *lum = (float *)malloc(sizeof(float) * (size_t)(s1 + 1));
    for (int oy = 0; oy < ch; oy++) {
        const int py = oy % fv, yy = oy / fv;
        float *row = out + (size_t)oy * cw;
        for (int ri = 0; ri < nreg; ri++) {
            const efe_region *r = &reg[ri];
            if (!(r->r0 <= yy && yy < r->r1)) continue;
            const int n = r->c1 - r->c0;
            for (int px = 0; px < fh; px++) {
                const int group = py * 2 + px;
                const float *c = chroma[group], *l = luma[group];
                if (!c || !l) continue;
                for (int i = 0; i < n; i++) acc[i] = lum[i] = 0.f;
                for (int ky = 0; ky < r->k; ky++) {
                    const size_t line = (size_t)(yy + 1 + ky - r->before) * stride;
                    for (int kx = 0; kx < r->k; kx++) {
                        const size_t x0 = line + r->c0 + 1 + kx - r->before;
                        const float wc = r->chroma[group][ky * r->k + kx];
                        const float wl = r->luma[ky * r->k + kx];
                        if (wc != 0.f)
                            for (int i = 0; i < n; i++) acc[i] += wc * c[x0 + i];
                        if (wl != 0.f)
                            for (int i = 0; i < n; i++) lum[i] += wl * l[x0 + i];
                    }
                }
                for (int i = 0; i < n; i++) {
                    const int x = (r->c0 + i) * fh + px;
                    if (x >= cw) break;
                    row[x] = (acc[i] + mean) + lum[i];
                }
            }
        }
    }
    free(acc);
    free(lum);
    return 0;
}

/* `supported_format` (efe_linear.rs:364-379) */
static int efe_supported(int s_ver, int s_hor, int c_ver, int c_hor) {
    if (s_ver == 1 && s_hor == 1)
        return (c_ver == 1 && c_hor == 1) || (c_ver == 1 && c_hor == 2) ||
               (c_ver == 2 && c_hor == 2);
    if (s_ver == 1 && s_hor == 2) return c_ver == 1 && c_hor == 2;
    if (s_ver == 2 && s_hor == 2) return c_ver == 2 && c_hor == 2;
    return 0;
}

int zo_efe_linear(const float *y, int h, int w, const float *u, const float *v, int ch, int cw,
                  int s_ver, int s_hor, int c_ver, int c_hor, int mean_u, int mean_v,
                  const zo_efe_linear_set *set, float *out_u, float *out_v) {
    if (!efe_supported(s_ver, s_hor, c_ver, c_hor)) return 2;
    if (h <= 0 || w <= 0) return 1;
    const int fv = 3 - s_ver, fh = 3 - s_hor, s0 = (h + 1) / 2, s1 = (w + 1) / 2;
    if ((ch + fv - 1) / fv != s0 || (cw + fh - 1) / fh != s1) return 1;
    /* float(code) / 100 in doubles, narrowed to f32 (efe_linear.rs:427-429) */
    const float mean[2] = {(float)((double)mean_u / 100.0), (float)((double)mean_v / 100.0)};
    float *luma[4] = {0}, *chroma[2][4] = {{0}};
    for (int py = 0; py < fv; py++)
        for (int px = 0; px < fh; px++) {
            luma[py * 2 + px] = efe_phase_plane(y, h, w, 2, 2, py, px, s0, s1, 0.f);
            chroma[0][py * 2 + px] = efe_phase_plane(u, ch, cw, fv, fh, py, px, s0, s1, mean[0]);
            chroma[1][py * 2 + px] = efe_phase_plane(v, ch, cw, fv, fh, py, px, s0, s1, mean[1]);
        }
    const int coded_444 = c_ver == s_ver && c_hor == s_hor;
    int st = efe_filter_plane(coded_444, set, 0, mean[0], fv, fh, s0, s1, luma, chroma[0], ch,
                              cw, out_u);
    if (!st)
        st = efe_filter_plane(coded_444, set, 1, mean[1], fv, fh, s0, s1, luma, chroma[1], ch,
                              cw, out_v);
    for (int i = 0; i < 4; i++) {
        free(luma[i]);
        free(chroma[0][i]);
        free(chroma[1][i]);
    }
    return st;
}

#define EFE_BINS 8

/* `tile_edge` (efe_nonlinear.rs:50-53): round(float(a) / n * n) in doubles */
static int efe_tile_edge(long long a, long long n) {
    return (int)rint(((double)a / (double)n) * (double)n);
}

/* `filter_plane` (efe_nonlinear.rs:57-141), with the per-tile parameters of `tiles` */
static int efe_nl_plane(const zo_efe_nonlinear_params *t, int p, const float *y, int lw, int sv,
                        int sh, float *plane, int hh, int ww) {
    const int th = t->tile_height, tw = t->tile_width;
    if (th <= 0 || tw <= 0) return 6;
    const int ni = (hh + th - 1) / th, nj = (ww + tw - 1) / tw, count = ni * nj;
    if (t->ntiles < count || t->ncodes[p] < count * EFE_BINS || !t->luma_min || !t->luma_max)
        return 6;
    for (int i = 0; i < ni; i++)
        for (int j = 0; j < nj; j++) {
            const int idx = i * nj + j;
            const uint32_t *cd = t->codes[p] + (size_t)idx * EFE_BINS;
            float wv[EFE_BINS];
            for (int k = 0; k < EFE_BINS; k++)
                wv[k] = efe_deinteger((long long)cd[k] + t->min_symbol);
            const double minimum = (double)t->luma_min[idx] / 100.0;
            const double gap = ((double)t->luma_max[idx] / 100.0 - minimum) / EFE_BINS;
            float ceil_k[EFE_BINS];
            for (int k = 0; k < EFE_BINS; k++)
                ceil_k[k] = -(1.0f * (float)minimum + (float)k * (float)gap);
            const float w0 = wv[0], b0 = wv[0] * ceil_k[0];
            const int r0 = efe_tile_edge((long long)i * th, hh);
            const int r1 = efe_tile_edge((long long)((i + 1) * th < hh ? (i + 1) * th : hh), hh);
            const int c0 = efe_tile_edge((long long)j * tw, ww);
            int c1 = efe_tile_edge((long long)((j + 1) * tw < ww ? (j + 1) * tw : ww), ww);
            if (c1 > ww) c1 = ww;
            for (int r = r0; r < r1; r++) {
                const float *yrow = y + (size_t)r * sv * lw;
                float *row = plane + (size_t)r * ww;
                for (int x = c0; x < c1; x++) {
                    const float l = yrow[(size_t)x * sh];
                    float acc = fmaxf(w0 * l + row[x] + b0, 0.f);
                    for (int k = 0; k < EFE_BINS - 1; k++)
                        acc += wv[k + 1] * fmaxf(l + ceil_k[k + 1], 0.f);
                    row[x] = acc;
                }
            }
        }
    return 0;
}

/* `switch_plane` (efe_nonlinear.rs:145-187) */
static int efe_switch(int bs, int my, int mx, const uint8_t *mask, const float *alt,
                      float *plane, int h, int w) {
    if (bs <= 0 || my != (h + bs - 1) / bs || mx != (w + bs - 1) / bs) return 6;
    for (int y = 0; y < h; y++) {
        const uint8_t *mrow = mask + (size_t)(y / bs) * mx;
        for (int x = 0; x < w; x++) {
            const uint8_t m = mrow[x / bs];
            const size_t i = (size_t)y * w + x;
            if (m == 0) continue;
            plane[i] = m == 2 ? alt[i] : (alt[i] + plane[i]) / 2.0f;
        }
    }
    return 0;
}

int zo_efe_nonlinear(const float *y, int h, int w, float *u, float *v, int ch, int cw,
                     int s_ver, int s_hor, int c_ver, int c_hor,
                     const zo_efe_nonlinear_params *prm, const float *alt_u, const float *alt_v) {
    if (!efe_supported(s_ver, s_hor, c_ver, c_hor)) return 2;
    if (h < 0 || w < 0) return 1;
    const int hh = (h + s_ver - 1) / s_ver, ww = (w + s_hor - 1) / s_hor;
    if (ch != hh || cw != ww) return 1;
    float *planes[2] = {u, v};
    for (int p = 0; p < 2; p++)
        if (prm->codes[p] && hh > 0 && ww > 0) {
            const int st = efe_nl_plane(prm, p, y, w, s_ver, s_hor, planes[p], hh, ww);
            if (st) return st;
        }
    /* `has_first_mask` (efe_nonlinear.rs:31-33): the U mask decides; the alternative picture
     * (both planes) must then be there */
    if (prm->mask[0] && (prm->mask_h > 0 || prm->mask_w > 0)) {
        if (!alt_u || !alt_v) return 6;
        const float *alt[2] = {alt_u, alt_v};
        for (int p = 0; p < 2; p++) {
            if (!prm->mask[p]) continue;
            const int st = efe_switch(prm->mask_bs, prm->mask_h, prm->mask_w, prm->mask[p],
                                      alt[p], planes[p], hh, ww);
            if (st) return st;
        }
    }
    return 0;
}


/* ======================================================================================= */
/* RDLR layer VJPs: input gradients of the conv layers (src/nn/reference.rs:238-336,        */
/* src/nn/fast/layers.rs:72-90, 156-160)                                                    */
/* ======================================================================================= */

/* `conv2d_backward` (reference.rs:241-292) through `ConvLayer::backward` (layers.rs:72-90):
 * the gradient on the padded input (h + top + bottom) x (w + left + right), each d_out sample's
 * products `g_o * w` added in the crate's loop order (output channel, its group's input
 * channels, output row, column, ky, kx; zero d_out samples skipped), then the extra border
 * dropped. The input channels are independent, so they run in parallel. */
int zo_conv2d_backward(const float *dout, int oc, int oh, int ow, const float *weight, int c,
                       int kh, int kw, int stride, int pad_h, int pad_w, int groups,
                       const int extra[4], int h, int w, float *din) {
    if (oc <= 0 || c <= 0 || groups <= 0 || c % groups || oc % groups || h <= 0 || w <= 0 ||
        stride <= 0)
        return -1;
    const int pt = extra ? extra[0] : 0, pl = extra ? extra[1] : 0;
    const int pb = extra ? extra[2] : 0, pr = extra ? extra[3] : 0;
    const int H = h + pt + pb, W = w + pl + pr;
    const int icg = c / groups, ocg = oc / groups;
    float *full = (float *)calloc((size_t)c * H * W, sizeof(float));
    if (!full) return -1;
#pragma omp parallel for schedule(dynamic) num_threads(g_threads)
    for (int c_in = 0; c_in < c; c_in++) {
        const int g = c_in / icg, ci = c_in % icg;
        float *dst = full + (size_t)c_in * H * W;
        for (int co = g * ocg; co < (g + 1) * ocg; co++) {
            const float *wb = weight + ((size_t)co * icg + ci) * kh * kw;
            const float *d = dout + (size_t)co * oh * ow;
            for (int oy = 0; oy < oh; oy++)
                for (int ox = 0; ox < ow; ox++) {
                    const float g_o = d[(size_t)oy * ow + ox];
                    if (g_o == 0.0f) continue;
                    for (int ky = 0; ky < kh; ky++) {
                        const int y = oy * stride + ky;
                        if (y < pad_h || y - pad_h >= H) continue;
                        const int iy = y - pad_h;
                        for (int kx = 0; kx < kw; kx++) {
                            const int x = ox * stride + kx;
                            if (x < pad_w || x - pad_w >= W) continue;
                            dst[(size_t)iy * W + x - pad_w] += g_o * wb[ky * kw + kx];
                        }
                    }
                }
        }
    }
    for (int ch = 0; ch < c; ch++)
        for (int y = 0; y < h; y++)
            memcpy(din + ((size_t)ch * h + y) * w, full + ((size_t)ch * H + y + pt) * W + pl,
                   sizeof(float) * w);
    free(full);
    return 0;
}

/* `conv_transpose2d_backward` (reference.rs:294-336): per input channel, per output channel of
 * the transposed conv, per input position the taps' products summed in (ky, kx) order, then
 * added to the gradient (weight [c][oc][k][k]). */
int zo_conv_transpose2d_backward(const float *dout, int oc, int oh, int ow, const float *weight,
                                 int c, int k, int stride, int pad, int h, int w, float *din) {
    if (oc <= 0 || c <= 0 || k <= 0 || stride <= 0 || h <= 0 || w <= 0) return -1;
#pragma omp parallel for schedule(dynamic) num_threads(g_threads)
    for (int ic = 0; ic < c; ic++) {
        float *dst = din + (size_t)ic * h * w;
        memset(dst, 0, sizeof(float) * (size_t)h * w);
        const float *wb = weight + (size_t)ic * oc * k * k;
        for (int o = 0; o < oc; o++) {
            const float *d = dout + (size_t)o * oh * ow;
            for (int y = 0; y < h; y++)
                for (int x = 0; x < w; x++) {
                    float acc = 0.0f;
                    for (int ky = 0; ky < k; ky++) {
                        const int oy = y * stride + ky;
                        if (oy < pad || oy - pad >= oh) continue;
                        for (int kx = 0; kx < k; kx++) {
                            const int ox = x * stride + kx;
                            if (ox < pad || ox - pad >= ow) continue;
                            acc += d[(size_t)(oy - pad) * ow + ox - pad] *
                                   wb[(size_t)o * k * k + ky * k + kx];
                        }
                    }
                    dst[(size_t)y * w + x] += acc;
                }
        }
    }
    return 0;
}

/* `ResidualBlock::backward` (attention.rs:58-75): d = conv2^T d_out; d = 0 where the tape
 * conv1_out <= 0; din = conv1^T d + d_out (3x3 convs, padding 1, c -> c). */
int zo_residual_block_backward(const float *dout, const float *conv1_out, int c, int h, int w,
                               const float *w1, const float *w2, float *din) {
    const size_t n = (size_t)c * h * w;
    float *d = (float *)malloc(sizeof(float) * n);
    if (!d) return -1;
    int r = zo_conv2d_backward(dout, c, h, w, w2, c, 3, 3, 1, 1, 1, 1, NULL, h, w, d);
    if (!r) {
        for (size_t i = 0; i < n; i++)
            if (conv1_out[i] <= 0.0f) d[i] = 0.0f;
        r = zo_conv2d_backward(d, c, h, w, w1, c, 3, 3, 1, 1, 1, 1, NULL, h, w, din);
    }
    if (!r)
        for (size_t i = 0; i < n; i++) din[i] += dout[i];
    free(d);
    return r;
}

/* `Cab::backward` (attention.rs:182-223): tape t = {trunk_pre, sig, rb_c1[0], rb_c1[1]}
 * [c][h][w] and mask_c1[2] [c][h/2][w/2]; weights wt = {trunk0 conv1, conv2, trunk1 conv1,
 * conv2, subscale, mask2 conv1, conv2, mask3 conv1, conv2, upscale}, each [c][c][3][3]. */
int zo_cab_backward(const float *dout, int c, int h, int w, const float *const t[4],
                    const float *const mask_c1[2], const float *const wt[10], float *din) {
    if (c <= 0 || h <= 0 || w <= 0 || h % 2 || w % 2) return -1;
    const int mh = h / 2, mw = w / 2;
    const size_t n = (size_t)c * h * w, nm = (size_t)c * mh * mw;
    float *dtr = (float *)malloc(sizeof(float) * n), *dsg = (float *)malloc(sizeof(float) * n);
    float *t1 = (float *)malloc(sizeof(float) * n);
    float *m1 = (float *)malloc(sizeof(float) * nm), *m2 = (float *)malloc(sizeof(float) * nm);
    int r = (!dtr || !dsg || !t1 || !m1 || !m2) ? -1 : 0;
    if (!r) {
        for (size_t i = 0; i < n; i++) {
            const float s = t[1][i];
            dtr[i] = dout[i] * s;
            float ds = dout[i] * t[0][i];
            ds *= s * (1.0f - s);
            dsg[i] = ds;
        }
        r = zo_residual_block_backward(dtr, t[3], c, h, w, wt[2], wt[3], t1);
        if (!r) r = zo_residual_block_backward(t1, t[2], c, h, w, wt[0], wt[1], din);
        if (!r) r = zo_conv_transpose2d_backward(dsg, c, h, w, wt[9], c, 3, 2, 1, mh, mw, m1);
        if (!r) r = zo_residual_block_backward(m1, mask_c1[1], c, mh, mw, wt[7], wt[8], m2);
        if (!r) r = zo_residual_block_backward(m2, mask_c1[0], c, mh, mw, wt[5], wt[6], m1);
        if (!r) r = zo_conv2d_backward(m1, c, mh, mw, wt[4], c, 3, 3, 2, 1, 1, 1, NULL, h, w, t1);
        if (!r) {
            for (size_t i = 0; i < n; i++) din[i] += t1[i];
            for (size_t i = 0; i < n; i++) din[i] += dout[i];
        }
    }
    free(dtr); free(dsg); free(t1); free(m1); free(m2);
    return r;
}

/* `elu_gate_backward` (math.rs:838-858) of y = elu(a) . b: d_a = elu'(a) . b . d (elu' = 1 above
 * 0, exp(a) else) and d_b = elu(a) . d, with the crate's exp. */
void zo_elu_gate_backward(const float *d, const float *a, const float *b, int64_t n, float *d_a,
                          float *d_b) {
    for (int64_t i = 0; i < n; i++) {
        const float av = a[i];
        const float e = av > 0.0f ? 0.0f : zo_exp(av);
        const float elu = av > 0.0f ? av : e - 1.0f;
        const float delu = av > 0.0f ? 1.0f : e;
        d_a[i] = delu * b[i] * d[i];
        d_b[i] = elu * d[i];
    }
}

/* `layer_norm_channels_backward` (math.rs:860-913): per position, mean and variance over the
 * channels in f64 (channel order), the f32 deviation and normalised x as the forward makes them,
 * then d_x[c] = (dy[c] - s1 / c - xn[c] . s2 / c) / sigma with dy = d . w and the f64 sums
 * s1 = sum dy, s2 = sum dy . xn. */
int zo_layer_norm_backward(const float *d, const float *x, int c, int h, int w,
                           const float *weight, float *dx) {
    if (c <= 0 || h <= 0 || w <= 0) return -1;
    const int64_t n = (int64_t)h * w;
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int64_t i = 0; i < n; i++) {
        double mean = 0.0, var = 0.0;
        for (int ch = 0; ch < c; ch++) mean += (double)x[ch * n + i];
        mean /= c;
        for (int ch = 0; ch < c; ch++) {
            const double dv = (double)x[ch * n + i] - mean;
            var += dv * dv;
        }
        const float sig = sqrtf((float)(var / c) + 1e-5f);
        const float m = (float)mean;
        double s1 = 0.0, s2 = 0.0;
        for (int ch = 0; ch < c; ch++) {
            const float xn = (x[ch * n + i] - m) / sig;
            const float dy = d[ch * n + i] * weight[ch];
            s1 += (double)dy;
            s2 += (double)dy * (double)xn;
        }
        const float m1 = (float)s1 / (float)c, m2 = (float)s2 / (float)c;
        for (int ch = 0; ch < c; ch++) {
            const float xn = (x[ch * n + i] - m) / sig;
            const float dy = d[ch * n + i] * weight[ch];
            dx[ch * n + i] = (dy - m1 - xn * m2) / sig;
        }
    }
    return 0;
}

/* The softmax weights attn [dim][c] of `channel_attention` (math.rs:506-603), the tape
 * `channel_attention_backward` reads; computed as zo_channel_attention computes them. */
int zo_channel_attention_weights(const float *qkv, int c3, int h, int w, int heads,
                                 const float *temperature, float *attn) {
    if (heads <= 0 || c3 % (3 * heads)) return -1;
    const int dim = c3 / 3, c = dim / heads;
    const int64_t n = (int64_t)h * w;
    float *qk = (float *)malloc(sizeof(float) * 2 * dim * n);
    if (!qk) return -1;
    memcpy(qk, qkv, sizeof(float) * 2 * dim * n);
    for (int r = 0; r < 2 * dim; r++) {
        float *row = qk + (int64_t)r * n;
        const float norm = (float)sqrt(zo_dot8(row, row, n));
        const float d = norm > 1e-12f ? norm : 1e-12f;
        for (int64_t i = 0; i < n; i++) row[i] /= d;
    }
    const float *q = qk, *k = qk + (int64_t)dim * n;
    for (int ri = 0; ri < dim; ri++) {
        const int head = ri / c;
        float *row = attn + (int64_t)ri * c;
        float mx = -INFINITY;
        for (int j = 0; j < c; j++) {
            row[j] = (float)zo_dot8(q + (int64_t)ri * n, k + (int64_t)(head * c + j) * n, n) *
                     temperature[head];
            mx = row[j] > mx ? row[j] : mx;
        }
        for (int j = 0; j < c; j++) row[j] = zo_exp(row[j] - mx);
        double sum = 0.0;
        for (int j = 0; j < c; j++) sum += (double)row[j];
        const float s32 = (float)sum;
        for (int j = 0; j < c; j++) row[j] /= s32;
    }
    free(qk);
    return 0;
}

/* `channel_attention_backward` (math.rs:668-836, the exact path): d_out [dim][h][w] ->
 * dqkv [3 dim][h][w]. q, k re-normalised with their clamped L2 norms kept; d_attn = d_out . v^T
 * (dot8) and the row softmax VJP with an f64 row sum; dq = T . da . k, dk = T . da^T . q in f64
 * accumulators followed by the L2-norm backward ((s - <x, s> x) / |x|); dv = attn^T . d_out in
 * f64. */
int zo_channel_attention_backward(const float *qkv, int c3, int h, int w, int heads,
                                  const float *temperature, const float *attn,
                                  const float *dout, float *dqkv) {
    if (heads <= 0 || c3 % (3 * heads)) return -1;
    const int dim = c3 / 3, c = dim / heads;
    const int64_t n = (int64_t)h * w;
    float *qk = (float *)malloc(sizeof(float) * 2 * dim * n);
    float *norms = (float *)malloc(sizeof(float) * 2 * dim);
    float *da = (float *)malloc(sizeof(float) * dim * c);
    if (!qk || !norms || !da) {
        free(qk); free(norms); free(da);
        return -1;
    }
    memcpy(qk, qkv, sizeof(float) * 2 * dim * n);
    for (int r = 0; r < 2 * dim; r++) {
        float *row = qk + (int64_t)r * n;
        const float nv = (float)sqrt(zo_dot8(row, row, n));
        norms[r] = nv > 1e-12f ? nv : 1e-12f;
        for (int64_t i = 0; i < n; i++) row[i] /= norms[r];
    }
    const float *q = qk, *k = qk + (int64_t)dim * n, *v = qkv + (int64_t)2 * dim * n;
    for (int ri = 0; ri < dim; ri++) {
        const int head = ri / c;
        const float *a_row = attn + (int64_t)ri * c;
        float *row = da + (int64_t)ri * c;
        double sdot = 0.0;
        for (int j = 0; j < c; j++) {
            row[j] = (float)zo_dot8(dout + (int64_t)ri * n, v + (int64_t)(head * c + j) * n, n);
            sdot += (double)a_row[j] * (double)row[j];
        }
        for (int j = 0; j < c; j++) row[j] = a_row[j] * (row[j] - (float)sdot);
    }
#pragma omp parallel for schedule(dynamic) num_threads(g_threads)
    for (int ri = 0; ri < 3 * dim; ri++) {
        double *acc = (double *)calloc(n, sizeof(double));
        float *o = dqkv + (int64_t)ri * n;
        if (ri < 2 * dim) {
            const int is_k = ri >= dim;
            const int head = (ri - (is_k ? dim : 0)) / c, j = (ri - (is_k ? dim : 0)) % c;
            const float *x = is_k ? k + (int64_t)(head * c + j) * n : q + (int64_t)ri * n;
            for (int i = 0; i < c; i++) {
                /* dq: row ri of da against k_i; dk: column j of da against q_i */
                const float wv = is_k ? temperature[head] * da[(int64_t)(head * c + i) * c + j]
                                      : temperature[head] * da[(int64_t)ri * c + i];
                const float *src = is_k ? q + (int64_t)(head * c + i) * n
                                        : k + (int64_t)(head * c + i) * n;
                for (int64_t l = 0; l < n; l++) acc[l] += (double)wv * (double)src[l];
            }
            double proj = 0.0;
            for (int64_t l = 0; l < n; l++) proj += (double)x[l] * acc[l];
            const double inv = 1.0 / (double)norms[ri];
            for (int64_t l = 0; l < n; l++) o[l] = (float)((acc[l] - proj * (double)x[l]) * inv);
        } else {
            const int head = (ri - 2 * dim) / c, j = (ri - 2 * dim) % c;
            for (int i = 0; i < c; i++) {
                const double a = (double)attn[(int64_t)(head * c + i) * c + j];
                const float *d = dout + (int64_t)(head * c + i) * n;
                for (int64_t l = 0; l < n; l++) acc[l] += a * (double)d[l];
            }
            for (int64_t l = 0; l < n; l++) o[l] = (float)acc[l];
        }
        free(acc);
    }
    free(qk); free(norms); free(da);
    return 0;
}

/* `TransformerBlock::backward` (attention.rs:435-480) from its tape: the feed-forward branch
 * (project_out, ELU gate, depthwise, project_in, layer norm of x_mid) added to d_out gives
 * d_xmid; the attention branch (project_out, channel attention, depthwise, project_in, layer
 * norm of x_in) of d_xmid added to it gives d_x. Shapes: x_in, x_mid [dim][n], qkv [3 dim][n],
 * attn [dim][dim / heads], gate [2 hidden][n]; weights w[] = prep_norm.weight [dim], prep_conv1
 * [3 dim][dim], prep_conv2 [3 dim][1][3][3], temperature [heads], attn_out [dim][dim],
 * ffn_norm.weight [dim], ffn_in [2 hidden][dim], ffn_dw [2 hidden][1][3][3], ffn_out
 * [dim][hidden]. */
int zo_transformer_block_backward(const float *dout, int dim, int hidden, int heads, int h, int w,
                                  const float *const tape[5], const float *const wt[9],
                                  float *din) {
    const float *x_in = tape[0], *qkv = tape[1], *attn = tape[2], *x_mid = tape[3],
                *gate = tape[4];
    const int64_t n = (int64_t)h * w;
    float *df = (float *)malloc(sizeof(float) * hidden * n);
    float *dd = (float *)malloc(sizeof(float) * 2 * hidden * n);
    float *dd2 = (float *)malloc(sizeof(float) * 2 * hidden * n);
    float *dm = (float *)malloc(sizeof(float) * dim * n);
    float *d3 = (float *)malloc(sizeof(float) * 3 * dim * n);
    float *d3b = (float *)malloc(sizeof(float) * 3 * dim * n);
    float *da = (float *)malloc(sizeof(float) * dim * n);
    int r = (!df || !dd || !dd2 || !dm || !d3 || !d3b || !da) ? -1 : 0;
    /* feed-forward branch */
    if (!r) r = zo_conv2d_backward(dout, dim, h, w, wt[8], hidden, 1, 1, 1, 0, 0, 1, NULL, h, w, df);
    if (!r) {
        zo_elu_gate_backward(df, gate, gate + (int64_t)hidden * n, (int64_t)hidden * n, dd,
                             dd + (int64_t)hidden * n);
        r = zo_conv2d_backward(dd, 2 * hidden, h, w, wt[7], 2 * hidden, 3, 3, 1, 1, 1,
                               2 * hidden, NULL, h, w, dd2);
    }
    if (!r) r = zo_conv2d_backward(dd2, 2 * hidden, h, w, wt[6], dim, 1, 1, 1, 0, 0, 1, NULL, h, w, dm);
    if (!r) r = zo_layer_norm_backward(dm, x_mid, dim, h, w, wt[5], da);
    if (!r)
        for (int64_t i = 0; i < (int64_t)dim * n; i++) din[i] = dout[i] + da[i];  /* d_xmid */
    /* attention branch on d_xmid */
    if (!r) r = zo_conv2d_backward(din, dim, h, w, wt[4], dim, 1, 1, 1, 0, 0, 1, NULL, h, w, dm);
    if (!r) r = zo_channel_attention_backward(qkv, 3 * dim, h, w, heads, wt[3], attn, dm, d3);
    if (!r) r = zo_conv2d_backward(d3, 3 * dim, h, w, wt[2], 3 * dim, 3, 3, 1, 1, 1, 3 * dim,
                                   NULL, h, w, d3b);
    if (!r) r = zo_conv2d_backward(d3b, 3 * dim, h, w, wt[1], dim, 1, 1, 1, 0, 0, 1, NULL, h, w, dm);
    if (!r) r = zo_layer_norm_backward(dm, x_in, dim, h, w, wt[0], da);
    if (!r)
        for (int64_t i = 0; i < (int64_t)dim * n; i++) din[i] += da[i];
    free(df); free(dd); free(dd2); free(dm); free(d3); free(d3b); free(da);
    return r;
}

/* `Tam::backward` (attention.rs:578-600): d_out through us_conv's VJP when resampled, block 1,
 * block 0, then ds_conv's VJP. h x w: the TAM's input extent; with resample the blocks run at
 * (h + 1) / 2 x (w + 1) / 2 (ds_conv: 3x3 stride 2 padding 1; us_conv: 3x3 transposed, stride 2,
 * padding 1, output padding 1, weight [dim][dim][3][3]). tape0 / tape1, wt0 / wt1: the blocks'
 * tapes and weights as zo_transformer_block_backward takes them. */
int zo_tam_backward(const float *dout, int dim, int hidden, int heads, int h, int w, int resample,
                    const float *const tape0[5], const float *const tape1[5],
                    const float *const wt0[9], const float *const wt1[9], const float *ds_w,
                    const float *us_w, float *din) {
    const int bh = resample ? (h + 1) / 2 : h, bw = resample ? (w + 1) / 2 : w;
    const size_t nb = (size_t)dim * bh * bw;
    float *a = (float *)malloc(sizeof(float) * nb), *b = (float *)malloc(sizeof(float) * nb);
    int r = (!a || !b) ? -1 : 0;
    if (!r) {
        if (resample)
            r = zo_conv_transpose2d_backward(dout, dim, 2 * bh, 2 * bw, us_w, dim, 3, 2, 1, bh,
                                             bw, a);
        else
            memcpy(a, dout, sizeof(float) * nb);
    }
    if (!r) r = zo_transformer_block_backward(a, dim, hidden, heads, bh, bw, tape1, wt1, b);
    if (!r) {
        if (resample) {
            r = zo_transformer_block_backward(b, dim, hidden, heads, bh, bw, tape0, wt0, a);
            if (!r) r = zo_conv2d_backward(a, dim, bh, bw, ds_w, dim, 3, 3, 2, 1, 1, 1, NULL, h,
                                           w, din);
        } else {
            r = zo_transformer_block_backward(b, dim, hidden, heads, bh, bw, tape0, wt0, din);
        }
    }
    free(a);
    free(b);
    return r;
}
