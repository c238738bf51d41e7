/*
 * Restatement of the crate's `nn::fast` convolution algorithm — TEST INFRASTRUCTURE ONLY (the
 * timed CPU baseline of bench.py and the reference arm; never part of the GPU product path).
 *
 * What it follows (paths inside the imazen/zenjpegai crate):
 *  - `PackedConv::pack` (src/nn/fast/conv.rs:453-487, 521-545): weights repacked to
 *    [ocb][icb][V in][taps][V out], zero for channels beyond the real counts; grouped convs
 *    (group sizes a multiple of V) pack every group on its own.
 *  - `block` / `tap_loop_n` (conv.rs:187-335): a register tile of B output positions x V
 *    output channels; the bias goes straight into the accumulators, then for every input block
 *    icb, channel v and tap t one weight-vector load and B splat / fused multiply-add steps,
 *    stored once at the end. Per output element that is acc = bias, then fma over (ic, ky, kx)
 *    in ascending order: the same operations in the same order as `nn::reference::conv_plane`
 *    (reference.rs:47-89), so the result is the same bits (the crate pins this in
 *    tests/fast_vs_reference.rs; tests/test_fast_baseline.py pins it here).
 *  - `for_each_row` (conv.rs:434-452): one task per (output block, output row).
 *  - `PackedConvTranspose::forward` (conv.rs:1967-2028): stride-2 transposed convs as parity
 *    phases over an input zero-padded by EXT, each phase's live taps (ky, kx) ascending.
 *  - `PackedDepthwise::forward` (src/nn/fast/depthwise.rs:155-209): V channels per vector,
 *    acc = 0 then the nine taps in order.
 * Winograd (`Precision::Approximate`, conv.rs:620-625) is opt-in in the crate and not used.
 *
 * Layout here: the oracle's planar [c][h][w] tensors are converted to the blocked, zero-padded
 * NCHWc layout around each layer (the crate keeps the blocked layout between layers; the
 * conversions are memory passes next to compute-bound convolutions). V = 8 lanes (AVX2 + FMA,
 * the crate's x86-64-v3 tier), B = 8 positions.
 */
#include "oracle.h"

#include <immintrin.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define V 8
#define BT 8

static int cdivi(int a, int b) { return (a + b - 1) / b; }

/* planar [c][h][w] -> blocked [cb][h + pt + pb][w + pl + pr][V], zero elsewhere. One task per
 * (block, row): V contiguous plane rows in, one contiguous blocked row out. */
static float *to_blocked(const float *x, int c, int h, int w, int pt, int pl, int pb, int pr,
                         int *ph_out, int *pw_out) {
    int cb = cdivi(c, V), ph = h + pt + pb, pw = w + pl + pr;
    float *d = (float *)calloc((size_t)cb * ph * pw * V, sizeof(float));
    if (!d) return NULL;
#pragma omp parallel for schedule(static) num_threads(zo_get_threads())
    for (int row = 0; row < cb * h; row++) {
        const int b = row / h, y = row % h, nv = c - b * V < V ? c - b * V : V;
        float *dst = d + (((size_t)b * ph + y + pt) * pw + pl) * V;
        const float *src = x + ((size_t)b * V * h + y) * w;
        for (int v = 0; v < nv; v++) {
            const float *sv = src + (size_t)v * h * w;
            for (int xx = 0; xx < w; xx++) dst[(size_t)xx * V + v] = sv[xx];
        }
    }
    *ph_out = ph;
    *pw_out = pw;
    return d;
}

/* blocked [cb][h][w][V] -> planar [c][h][w] (the first c channels), per (block, row) */
static void from_blocked(const float *d, int c, int h, int w, float *out) {
    const int cb = cdivi(c, V);
#pragma omp parallel for schedule(static) num_threads(zo_get_threads())
    for (int row = 0; row < cb * h; row++) {
        const int b = row / h, y = row % h, nv = c - b * V < V ? c - b * V : V;
        const float *src = d + ((size_t)b * h + y) * w * V;
        float *dst = out + ((size_t)b * V * h + y) * w;
        for (int v = 0; v < nv; v++) {
            float *dv = dst + (size_t)v * h * w;
            for (int xx = 0; xx < w; xx++) dv[xx] = src[(size_t)xx * V + v];
        }
    }
}

/* The register tile: NB (<= BT) output positions x V output channels over the input blocks
 * icb0 .. icb0 + nicb. `rows[t]` points at the first position's input pixel of tap t in the
 * first input block (channel lane 0); positions are `step` pixels apart; input blocks are
 * `bstride` floats apart. Weights [nicb][V in][ntaps][V out]. */
static inline void tile_kernel(int nb, const float *const *rows, int ntaps, int step,
                               size_t bstride, int nicb, const float *w, const float *bias,
                               float *out, int ostep) {
    __m256 acc[BT];
    const __m256 b0 = _mm256_loadu_ps(bias);
    for (int b = 0; b < BT; b++) acc[b] = b0;
    const size_t ps = (size_t)step * V;
    if (nb == BT) {
        for (int icb = 0; icb < nicb; icb++) {
            const size_t xo = (size_t)icb * bstride;
            const float *wb = w + (size_t)icb * V * ntaps * V;
            for (int v = 0; v < V; v++)
                for (int t = 0; t < ntaps; t++) {
                    const __m256 wv = _mm256_loadu_ps(wb + ((size_t)v * ntaps + t) * V);
                    const float *r = rows[t] + xo + v;
                    acc[0] = _mm256_fmadd_ps(wv, _mm256_broadcast_ss(r), acc[0]);
                    acc[1] = _mm256_fmadd_ps(wv, _mm256_broadcast_ss(r + ps), acc[1]);
                    acc[2] = _mm256_fmadd_ps(wv, _mm256_broadcast_ss(r + 2 * ps), acc[2]);
                    acc[3] = _mm256_fmadd_ps(wv, _mm256_broadcast_ss(r + 3 * ps), acc[3]);
                    acc[4] = _mm256_fmadd_ps(wv, _mm256_broadcast_ss(r + 4 * ps), acc[4]);
                    acc[5] = _mm256_fmadd_ps(wv, _mm256_broadcast_ss(r + 5 * ps), acc[5]);
                    acc[6] = _mm256_fmadd_ps(wv, _mm256_broadcast_ss(r + 6 * ps), acc[6]);
                    acc[7] = _mm256_fmadd_ps(wv, _mm256_broadcast_ss(r + 7 * ps), acc[7]);
                }
        }
    } else {
        for (int icb = 0; icb < nicb; icb++) {
            const size_t xo = (size_t)icb * bstride;
            const float *wb = w + (size_t)icb * V * ntaps * V;
            for (int v = 0; v < V; v++)
                for (int t = 0; t < ntaps; t++) {
                    const __m256 wv = _mm256_loadu_ps(wb + ((size_t)v * ntaps + t) * V);
                    const float *r = rows[t] + xo + v;
                    for (int b = 0; b < nb; b++)
                        acc[b] = _mm256_fmadd_ps(wv, _mm256_broadcast_ss(r + b * ps), acc[b]);
                }
        }
    }
    for (int b = 0; b < nb; b++) _mm256_storeu_ps(out + (size_t)b * ostep * V, acc[b]);
}

/* Depthwise 3x3-class conv (groups == c == oc) on the blocked input: one vector of V channels
 * per output pixel, acc = bias then the taps in (ky, kx) order. */
static int depthwise(const float *x, int c, int h, int w, const float *weight, const float *bias,
                     int kh, int kw, int stride, int pt, int pl, int pb, int pr, int oh, int ow,
                     float *out) {
    int ph = 0, pw = 0;
    float *xb = to_blocked(x, c, h, w, pt, pl, pb, pr, &ph, &pw);
    int cb = cdivi(c, V), nt = kh * kw;
    float *wp = (float *)calloc((size_t)cb * nt * V, sizeof(float));
    float *bp = (float *)calloc((size_t)cb * V, sizeof(float));
    float *ob = (float *)malloc(sizeof(float) * (size_t)cb * oh * ow * V);
    if (!xb || !wp || !bp || !ob) {
        free(xb), free(wp), free(bp), free(ob);
        return -2;
    }
    for (int ci = 0; ci < c; ci++) {
        for (int t = 0; t < nt; t++) wp[((size_t)(ci / V) * nt + t) * V + ci % V] = weight[ci * nt + t];
        bp[ci] = bias ? bias[ci] : 0.0f;
    }
#pragma omp parallel for schedule(dynamic) num_threads(zo_get_threads())
    for (int row = 0; row < cb * oh; row++) {
        const int b = row / oh, oy = row % oh;
        const float *xc = xb + (size_t)b * ph * pw * V;
        float *orow = ob + ((size_t)b * oh + oy) * ow * V;
        const __m256 b0 = _mm256_loadu_ps(bp + (size_t)b * V);
        for (int ox = 0; ox < ow; ox++) {
            __m256 acc = b0;
            for (int ky = 0; ky < kh; ky++)
                for (int kx = 0; kx < kw; kx++)
                    acc = _mm256_fmadd_ps(
                        _mm256_loadu_ps(wp + ((size_t)b * nt + ky * kw + kx) * V),
                        _mm256_loadu_ps(xc + ((size_t)(oy * stride + ky) * pw + ox * stride + kx) * V),
                        acc);
            _mm256_storeu_ps(orow + (size_t)ox * V, acc);
        }
    }
    from_blocked(ob, c, oh, ow, out);
    free(xb), free(wp), free(bp), free(ob);
    return 0;
}

/* zo_conv2d on the nn::fast scheme. Returns 1 (not handled: the caller runs the reference
 * loop) for grouped convs whose group sizes are not a multiple of V, like the crate's
 * `Error::Unsupported` fallback (conv.rs:516-520). */
int zf_conv2d(const float *x, int c, int h, int w, const float *weight, const float *bias,
              int oc, int kh, int kw, int stride, int pad_h, int pad_w, int groups,
              const int extra[4], float *out) {
    if (groups <= 0 || c % groups || oc % groups || stride <= 0 || kh <= 0 || kw <= 0) return -1;
    const int et = extra ? extra[0] : 0, el = extra ? extra[1] : 0;
    const int eb = extra ? extra[2] : 0, er = extra ? extra[3] : 0;
    const int pt = et + pad_h, pl = el + pad_w, pb = eb + pad_h, pr = er + pad_w;
    int oh, ow;
    zo_conv2d_out_size(h, w, kh, kw, stride, pad_h, pad_w, extra, &oh, &ow);
    if (oh <= 0 || ow <= 0) return -1;
    const int icg = c / groups, ocg = oc / groups;
    if (groups > 1 && icg == 1 && ocg == 1)
        return depthwise(x, c, h, w, weight, bias, kh, kw, stride, pt, pl, pb, pr, oh, ow, out);
    if (groups > 1 && (icg % V || ocg % V)) return 1;
    const int nt = kh * kw;
    if (nt > 64) return 1;
    const int icb_g = cdivi(icg, V), ocb_g = cdivi(ocg, V), ocb = groups * ocb_g;
    int ph = 0, pw = 0;
    float *xb = to_blocked(x, c, h, w, pt, pl, pb, pr, &ph, &pw);
    /* pack (conv.rs:453-487): [g][ocb_g][icb_g][V in][taps][V out] */
    float *wp = (float *)calloc((size_t)ocb * icb_g * V * nt * V, sizeof(float));
    float *bp = (float *)calloc((size_t)ocb * V, sizeof(float));
    float *ob = (float *)malloc(sizeof(float) * (size_t)ocb * oh * ow * V);
    if (!xb || !wp || !bp || !ob) {
        free(xb), free(wp), free(bp), free(ob);
        return -2;
    }
    for (int g = 0; g < groups; g++)
        for (int o = 0; o < ocg; o++)
            for (int i = 0; i < icg; i++)
                for (int t = 0; t < nt; t++) {
                    const int blk = g * ocb_g + o / V;
                    wp[((((size_t)blk * icb_g + i / V) * V + i % V) * nt + t) * V + o % V] =
                        weight[((size_t)(g * ocg + o) * icg + i) * nt + t];
                }
    for (int g = 0; g < groups; g++)
        for (int o = 0; o < ocg; o++) bp[(size_t)(g * ocb_g + o / V) * V + o % V] = bias ? bias[g * ocg + o] : 0.0f;
    const size_t bstride = (size_t)ph * pw * V;
#pragma omp parallel for schedule(dynamic) num_threads(zo_get_threads())
    for (int row = 0; row < ocb * oh; row++) {
        const int blk = row / oh, oy = row % oh, g = blk / ocb_g;
        const float *xg = xb + (size_t)g * icb_g * bstride;  /* group g's first input block */
        const float *wb = wp + (size_t)blk * icb_g * V * nt * V;
        float *orow = ob + ((size_t)blk * oh + oy) * ow * V;
        const float *rows[64];
        for (int ox0 = 0; ox0 < ow; ox0 += BT) {
            for (int t = 0; t < nt; t++)
                rows[t] = xg + ((size_t)(oy * stride + t / kw) * pw + ox0 * stride + t % kw) * V;
            const int nb = ow - ox0 < BT ? ow - ox0 : BT;
            tile_kernel(nb, rows, nt, stride, bstride, icb_g, wb, bp + (size_t)blk * V,
                        orow + (size_t)ox0 * V, 1);
        }
    }
    /* block g * ocb_g + o / V holds channel g * ocg + o (ocg is a multiple of V when
     * groups > 1), so the blocks are in channel order */
    from_blocked(ob, oc, oh, ow, out);
    free(xb), free(wp), free(bp), free(ob);
    return 0;
}

/* zo_conv_transpose2d on the nn::fast scheme: parity phases (conv.rs:1967-2028). Output row oy
 * and column parity q: the live taps are ky = oy + pad (mod 2), kx = q + pad (mod 2), ascending;
 * output ox = 2 m + q reads padded input row (oy + pad - ky) / 2 + ext, column
 * m + (q + pad - kx) / 2 + ext. */
int zf_conv_transpose2d(const float *x, int c, int h, int w, const float *weight,
                        const float *bias, int oc, int k, int stride, int pad, int out_pad,
                        float *out) {
    if (stride != 2 || k > 4) return 1;
    if (k <= 0 || pad >= k || out_pad >= stride || h <= 0 || w <= 0) return -1;
    int oh, ow;
    zo_conv_transpose2d_out_size(h, w, k, stride, pad, out_pad, &oh, &ow);
    const int ext = (k + stride - 1) / stride + 1;
    int ph = 0, pw = 0;
    float *xb = to_blocked(x, c, h, w, ext, ext, ext, ext, &ph, &pw);
    const int icb = cdivi(c, V), ocb = cdivi(oc, V);
    /* per phase (py, px): taps and packed weights [ocb][icb][V in][nt][V out] */
    int nt[4], tky[4][16], tkx[4][16];
    float *wp[4];
    for (int p = 0; p < 4; p++) {
        const int py = p >> 1, px = p & 1;
        nt[p] = 0;
        for (int ky = 0; ky < k; ky++)
            for (int kx = 0; kx < k; kx++)
                if (((py + pad - ky) & 1) == 0 && ((px + pad - kx) & 1) == 0) {
                    tky[p][nt[p]] = ky;
                    tkx[p][nt[p]] = kx;
                    nt[p]++;
                }
        wp[p] = (float *)calloc((size_t)ocb * icb * V * (nt[p] ? nt[p] : 1) * V, sizeof(float));
    }
    float *bp = (float *)calloc((size_t)ocb * V, sizeof(float));
    float *ob = (float *)malloc(sizeof(float) * (size_t)ocb * oh * ow * V);
    int bad = !xb || !bp || !ob;
    for (int p = 0; p < 4; p++) bad |= !wp[p];
    if (bad) {
        free(xb), free(bp), free(ob);
        for (int p = 0; p < 4; p++) free(wp[p]);
        return -2;
    }
    for (int p = 0; p < 4; p++)
        for (int o = 0; o < oc; o++)
            for (int i = 0; i < c; i++)
                for (int t = 0; t < nt[p]; t++)
                    wp[p][((((size_t)(o / V) * icb + i / V) * V + i % V) * nt[p] + t) * V + o % V] =
                        weight[(((size_t)i * oc + o) * k + tky[p][t]) * k + tkx[p][t]];
    for (int o = 0; o < oc; o++) bp[o] = bias ? bias[o] : 0.0f;
    const size_t bstride = (size_t)ph * pw * V;
#pragma omp parallel for schedule(dynamic) num_threads(zo_get_threads())
    for (int row = 0; row < ocb * oh; row++) {
        const int blk = row / oh, oy = row % oh, py = oy & 1;
        float *orow = ob + ((size_t)blk * oh + oy) * ow * V;
        const float *rows[16];
        for (int q = 0; q < 2 && q < ow; q++) {
            const int p = py * 2 + q;
            const int n = (ow - q + 1) / 2;  /* outputs ox = q, q + 2, .. */
            const float *wb = wp[p] + (size_t)blk * icb * V * nt[p] * V;
            for (int m0 = 0; m0 < n; m0 += BT) {
                for (int t = 0; t < nt[p]; t++) {
                    const int iy = (oy + pad - tky[p][t]) / 2 + ext;
                    const int ix = m0 + (q + pad - tkx[p][t]) / 2 + ext;
                    rows[t] = xb + ((size_t)iy * pw + ix) * V;
                }
                const int nb = n - m0 < BT ? n - m0 : BT;
                tile_kernel(nb, rows, nt[p], 1, bstride, icb, wb, bp + (size_t)blk * V,
                            orow + (size_t)(2 * m0 + q) * V, 2);
            }
        }
    }
    from_blocked(ob, oc, oh, ow, out);
    free(xb), free(bp), free(ob);
    for (int p = 0; p < 4; p++) free(wp[p]);
    return 0;
}
