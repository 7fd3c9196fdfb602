/*
 * CPU oracle for the wgpu-ocr inference hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement (fp32 storage, fp32 arithmetic, NCHW layout) of the arithmetic of the
 * reference's WGSL kernels and of the ONNX operator semantics its executors implement.  Each
 * function cites the reference code it follows (paths inside huppiflupp/wgpu-ocr).  Only the
 * tests, the smoke check and the benchmark's CPU-baseline leg may load this library; the
 * product path (the CUDA library) never does.
 *
 * Parity pinning: the reference ships no golden vectors and cannot run here (Rust + wgpu over a
 * graphics API; its rten CPU path is an un-vendored crates.io dependency, rten =0.26.0).  The
 * oracle is therefore "parity unpinned" against the reference itself; it is cross-checked
 * against an independent implementation (PyTorch CPU: conv2d, conv_transpose2d, max/avg pool,
 * nn.GRU, layer_norm, softmax) in tests/test_oracle.py.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* Abramowitz & Stegun 7.1.26 erf, as the reference's kernels compute it
 * (src/gpu.rs:19-27, src/nd.rs:70-76). */
static float erf_as(float v) {
    float s = (v > 0.f) - (v < 0.f);
    float a = fabsf(v);
    float t = 1.0f / (1.0f + 0.3275911f * a);
    float poly = ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    return s * (1.0f - poly * expf(-a * a));
}

/* Activation codes of the reference's epilogue (src/gpu.rs:28-34):
 * 0 none, 1 Relu, 2 Sigmoid, 3 GELU (erf form), 4 SiLU. */
static float act_f(float v, int act) {
    switch (act) {
    case 1: return v > 0.f ? v : 0.f;
    case 2: return 1.0f / (1.0f + expf(-v));
    case 3: return 0.5f * v * (1.0f + erf_as(v * 0.70710678118654752f));
    case 4: return v / (1.0f + expf(-v));
    default: return v;
    }
}

float oracle_erf(float v) { return erf_as(v); }
float oracle_act(float v, int act) { return act_f(v, act); }

void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int oracle_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/*
 * Dense or grouped convolution, zero padding (pt, pl leading; pb, pr trailing), strides
 * (sh, sw), weights in ONNX order [cout][cin/group][kh][kw].  Epilogue as the reference's
 * `put` (src/gpu.rs:58-73): act(acc + b) then + res when given.  `insc` [n][cin] scales the
 * input before the multiply (squeeze-excitation input scale, src/gpu.rs:95-97, src/nd.rs:552-571).
 * Output size (h + pt + pb - kh) / sh + 1 (src/nd.rs:1279-1280).
 */
void oracle_conv2d(const float *x, int n, int cin, int h, int w,
                   const float *wt, const float *b, int cout, int group, int kh, int kw,
                   int sh, int sw, int pt, int pl, int pb, int pr, int act,
                   const float *res, const float *insc, float *y) {
    int oh = (h + pt + pb - kh) / sh + 1;
    int ow = (w + pl + pr - kw) / sw + 1;
    int cin_g = cin / group, cout_g = cout / group;
    long plane = (long)h * w, oplane = (long)oh * ow;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int nb = 0; nb < n; nb++) {
        for (int co = 0; co < cout; co++) {
            float *yp = y + ((long)nb * cout + co) * oplane;
            float bias = b ? b[co] : 0.f;
            for (long i = 0; i < oplane; i++) yp[i] = 0.f;
            int g = co / cout_g;
            for (int cg = 0; cg < cin_g; cg++) {
                int ci = g * cin_g + cg;
                const float *xp = x + ((long)nb * cin + ci) * plane;
                float sc = insc ? insc[(long)nb * cin + ci] : 1.f;
                for (int ky = 0; ky < kh; ky++) {
                    for (int kx = 0; kx < kw; kx++) {
                        float wv = wt[(((long)co * cin_g + cg) * kh + ky) * kw + kx];
                        /* ox range with 0 <= ox*sw + kx - pl < w */
                        int ox0 = 0, ox1 = ow;
                        while (ox0 < ow && ox0 * sw + kx - pl < 0) ox0++;
                        while (ox1 > ox0 && (ox1 - 1) * sw + kx - pl >= w) ox1--;
                        for (int oy = 0; oy < oh; oy++) {
                            int iy = oy * sh + ky - pt;
                            if (iy < 0 || iy >= h) continue;
                            const float *xr = xp + (long)iy * w + kx - pl;
                            float *yr = yp + (long)oy * ow;
                            if (insc) {
                                for (int ox = ox0; ox < ox1; ox++) yr[ox] += (xr[ox * sw] * sc) * wv;
                            } else if (sw == 1) {
                                for (int ox = ox0; ox < ox1; ox++) yr[ox] += xr[ox] * wv;
                            } else {
                                for (int ox = ox0; ox < ox1; ox++) yr[ox] += xr[ox * sw] * wv;
                            }
                        }
                    }
                }
            }
            const float *rp = res ? res + ((long)nb * cout + co) * oplane : NULL;
            for (long i = 0; i < oplane; i++) {
                float r = act_f(yp[i] + bias, act);
                if (rp) r += rp[i];
                yp[i] = r;
            }
        }
    }
}

/*
 * ConvTranspose, group 1, no pads/output_padding: out (h - 1) * s + k (src/gpu.rs:424-460,
 * src/nd.rs:874-886).  Weights [cin][cout][kh][kw]; y = act(b + sum of the taps).
 */
void oracle_convt(const float *x, int n, int cin, int h, int w, const float *wt, const float *b,
                  int cout, int kh, int kw, int s, int act, float *y) {
    int oh = (h - 1) * s + kh, ow = (w - 1) * s + kw;
    long plane = (long)h * w, oplane = (long)oh * ow;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int nb = 0; nb < n; nb++) {
        for (int co = 0; co < cout; co++) {
            float *yp = y + ((long)nb * cout + co) * oplane;
            for (long i = 0; i < oplane; i++) yp[i] = 0.f;
            for (int ci = 0; ci < cin; ci++) {
                const float *xp = x + ((long)nb * cin + ci) * plane;
                for (int ky = 0; ky < kh; ky++)
                    for (int kx = 0; kx < kw; kx++) {
                        float wv = wt[(((long)ci * cout + co) * kh + ky) * kw + kx];
                        for (int iy = 0; iy < h; iy++) {
                            float *yr = yp + (long)(iy * s + ky) * ow + kx;
                            const float *xr = xp + (long)iy * w;
                            for (int ix = 0; ix < w; ix++) yr[ix * s] += xr[ix] * wv;
                        }
                    }
            }
            float bias = b ? b[co] : 0.f;
            for (long i = 0; i < oplane; i++) yp[i] = act_f(yp[i] + bias, act);
        }
    }
}

/*
 * Max or average pooling with strides and leading padding; padding is never counted
 * (src/nd.rs:246-275, 1319-1349).  The ocrs MaxPool (kernel = stride, no pad, src/gpu.rs:462-482)
 * is the special case pt = pl = 0, sh = kh, sw = kw.  oh, ow given by the caller.
 */
void oracle_pool(const float *x, int nc, int h, int w, int oh, int ow, int kh, int kw, int sh, int sw,
                 int pt, int pl, int avg, float *y) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < nc; c++) {
        for (int oy = 0; oy < oh; oy++)
            for (int ox = 0; ox < ow; ox++) {
                float m = -3.4e38f, s = 0.f, cnt = 0.f;
                for (int ky = 0; ky < kh; ky++) {
                    int iy = oy * sh + ky - pt;
                    if (iy < 0 || iy >= h) continue;
                    for (int kx = 0; kx < kw; kx++) {
                        int ix = ox * sw + kx - pl;
                        if (ix < 0 || ix >= w) continue;
                        float v = x[((long)c * h + iy) * w + ix];
                        m = v > m ? v : m;
                        s += v;
                        cnt += 1.f;
                    }
                }
                y[((long)c * oh + oy) * ow + ox] = avg ? s / (cnt > 1.f ? cnt : 1.f) : m;
            }
    }
}

/* Linear interpolation as WGSL `mix(a, b, t)` = a * (1 - t) + b * t. */
static inline float mixf(float a, float b, float t) { return a * (1.0f - t) + b * t; }

static inline float byte_at(const uint8_t *rgb, long i) { return (float)rgb[i]; }

/* ocrs grey value of page pixel (x, y), -0.5 outside the page (src/gpu.rs:537-542). */
static inline float grey_px(const uint8_t *rgb, int w, int h, int x, int yy) {
    if (x >= w || yy >= h) return -0.5f;
    long i = ((long)yy * w + x) * 3;
    return -0.5f + byte_at(rgb, i) * (0.299f / 255.0f) + byte_at(rgb, i + 1) * (0.587f / 255.0f) +
           byte_at(rgb, i + 2) * (0.114f / 255.0f);
}

/*
 * Detector input: RGB page -> ocrs grey, padded with -0.5 to (ph, pw) = (max(h, oh), max(w, ow)),
 * half-pixel bilinear resize (clamped, x then y) to oh x ow (src/gpu.rs:530-561, 1394-1411).
 */
void oracle_grey_resize(const uint8_t *rgb, int w, int h, int ow, int oh, float *y) {
    int ph = h > oh ? h : oh, pw = w > ow ? w : ow;
    float sx = (float)pw / (float)ow, sy = (float)ph / (float)oh;
#pragma omp parallel for schedule(static)
    for (int oy = 0; oy < oh; oy++) {
        for (int ox = 0; ox < ow; ox++) {
            float iy = sy * ((float)oy + 0.5f) - 0.5f;
            float ix = sx * ((float)ox + 0.5f) - 0.5f;
            iy = iy < 0.f ? 0.f : (iy > (float)ph - 1.f ? (float)ph - 1.f : iy);
            ix = ix < 0.f ? 0.f : (ix > (float)pw - 1.f ? (float)pw - 1.f : ix);
            int y1 = (int)iy, x1 = (int)ix;
            int y2 = y1 + 1 < ph - 1 ? y1 + 1 : ph - 1;
            int x2 = x1 + 1 < pw - 1 ? x1 + 1 : pw - 1;
            float wy = iy - (float)y1, wx = ix - (float)x1;
            float top = mixf(grey_px(rgb, w, h, x1, y1), grey_px(rgb, w, h, x2, y1), wx);
            float bot = mixf(grey_px(rgb, w, h, x1, y2), grey_px(rgb, w, h, x2, y2), wx);
            y[(long)oy * ow + ox] = mixf(top, bot, wy);
        }
    }
}

/*
 * Detector output: the valid vh x vw part of the model's map (row stride `stride`), half-pixel
 * bilinear to the page (w x h), `> thr`, 32 pixels to a word, bit b = pixel 32 * wx + b
 * (src/gpu.rs:563-593, 1414-1418).  `prob` (nullable) receives the page-level interpolated
 * probabilities [h][w], for the threshold tie band of the parity tests.
 */
void oracle_mask_up(const float *m, int stride, int vw, int vh, int w, int h, float thr,
                    uint32_t *bits, float *prob) {
    int words = (w + 31) / 32;
    float sx = (float)vw / (float)w, sy = (float)vh / (float)h;
#pragma omp parallel for schedule(static)
    for (int oy = 0; oy < h; oy++) {
        float iy = sy * ((float)oy + 0.5f) - 0.5f;
        iy = iy < 0.f ? 0.f : (iy > (float)vh - 1.f ? (float)vh - 1.f : iy);
        int y1 = (int)iy;
        int y2 = y1 + 1 < vh - 1 ? y1 + 1 : vh - 1;
        float fy = iy - (float)y1;
        for (int wx = 0; wx < words; wx++) {
            uint32_t v = 0;
            for (int b = 0; b < 32; b++) {
                int ox = wx * 32 + b;
                if (ox >= w) break;
                float ix = sx * ((float)ox + 0.5f) - 0.5f;
                ix = ix < 0.f ? 0.f : (ix > (float)vw - 1.f ? (float)vw - 1.f : ix);
                int x1 = (int)ix;
                int x2 = x1 + 1 < vw - 1 ? x1 + 1 : vw - 1;
                float fx = ix - (float)x1;
                float top = mixf(m[(long)y1 * stride + x1], m[(long)y1 * stride + x2], fx);
                float bot = mixf(m[(long)y2 * stride + x1], m[(long)y2 * stride + x2], fx);
                float p = mixf(top, bot, fy);
                if (prob) prob[(long)oy * w + ox] = p;
                if (p > thr) v |= 1u << b;
            }
            bits[(long)oy * words + wx] = v;
        }
    }
}

/*
 * PP-OCR detection input: RGB page -> half-pixel bilinear to ow x oh (clamped), BGR planes,
 * (v / 255 - mean) / std with the ImageNet constants (src/nd.rs:172-204, 1353-1369).
 */
void oracle_det_prep(const uint8_t *rgb, int w, int h, int ow, int oh, float *y) {
    const float mean[3] = {0.485f, 0.456f, 0.406f};
    const float dev[3] = {0.229f, 0.224f, 0.225f};
    float sx = (float)w / (float)ow, sy = (float)h / (float)oh;
#pragma omp parallel for schedule(static)
    for (int oy = 0; oy < oh; oy++) {
        for (int ox = 0; ox < ow; ox++) {
            float ix = sx * ((float)ox + 0.5f) - 0.5f;
            float iy = sy * ((float)oy + 0.5f) - 0.5f;
            ix = ix < 0.f ? 0.f : (ix > (float)w - 1.f ? (float)w - 1.f : ix);
            iy = iy < 0.f ? 0.f : (iy > (float)h - 1.f ? (float)h - 1.f : iy);
            int x1 = (int)ix, y1 = (int)iy;
            int x2 = x1 + 1 < w - 1 ? x1 + 1 : w - 1;
            int y2 = y1 + 1 < h - 1 ? y1 + 1 : h - 1;
            float fx = ix - (float)x1, fy = iy - (float)y1;
            for (int c = 0; c < 3; c++) {
                int k = 2 - c; /* BGR: output channel 0 is blue, byte 2 */
                float a = mixf(byte_at(rgb, ((long)y1 * w + x1) * 3 + k), byte_at(rgb, ((long)y1 * w + x2) * 3 + k), fx);
                float bb = mixf(byte_at(rgb, ((long)y2 * w + x1) * 3 + k), byte_at(rgb, ((long)y2 * w + x2) * 3 + k), fx);
                y[((long)c * oh + oy) * ow + ox] = (mixf(a, bb, fy) / 255.0f - mean[c]) / dev[c];
            }
        }
    }
}

/* Nearest Resize, asymmetric, floor: in = min(floor(out / scale), size - 1) (src/nd.rs:155-170). */
void oracle_resize_nearest(const float *x, int nc, int h, int w, int oh, int ow, float sy, float sx,
                           float *y) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < nc; c++)
        for (int oy = 0; oy < oh; oy++) {
            int iy = (int)floorf((float)oy / sy);
            if (iy > h - 1) iy = h - 1;
            for (int ox = 0; ox < ow; ox++) {
                int ix = (int)floorf((float)ox / sx);
                if (ix > w - 1) ix = w - 1;
                y[((long)c * oh + oy) * ow + ox] = x[((long)c * h + iy) * w + ix];
            }
        }
}

/*
 * y[m, k] = x[m, :] . wt[:, k] + b[k], wt stored [i][k] (src/gpu.rs:616-678); with act
 * (src/nd.rs:291-358 with zero batch strides).
 */
void oracle_gemm(const float *x, const float *wt, const float *b, int m, int k, int i, int act, float *y) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < m; r++) {
        float *yr = y + (long)r * k;
        for (int c = 0; c < k; c++) yr[c] = 0.f;
        for (int j = 0; j < i; j++) {
            float xv = x[(long)r * i + j];
            const float *wr = wt + (long)j * k;
            for (int c = 0; c < k; c++) yr[c] += xv * wr[c];
        }
        for (int c = 0; c < k; c++) yr[c] = act_f(yr[c] + (b ? b[c] : 0.f), act);
    }
}

static inline float sigm(float v) { return 1.0f / (1.0f + expf(-v)); }

/*
 * ONNX GRU, linear_before_reset = 1, gate order z, r, h (src/gpu.rs:680-819).
 *   g  [tmax][ntot][2][768]  = W x + Wb   (input projection, both directions)
 *   r  [2][768][hid]         recurrent weights (rows z | r | h)
 *   rb [2][768]              recurrent bias
 *   lens[ntot]               each line's length; the backward direction starts at len - 1
 *   y  [tmax][ntot][2][hid]  only t < len is written
 * hid is 256 in the reference (hidden_size check, src/gpu.rs:1461).
 */
void oracle_gru(const float *g, const float *r, const float *rb, const int *lens, int tmax, int ntot,
                int hid, float *y) {
    int G = 3 * hid;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int dir = 0; dir < 2; dir++) {
        for (int line = 0; line < ntot; line++) {
            float *h = (float *)calloc((size_t)hid, sizeof(float));
            float *acc = (float *)malloc((size_t)G * sizeof(float));
            const float *R = r + (long)dir * G * hid;
            const float *RB = rb + (long)dir * G;
            int len = lens[line];
            for (int s = 0; s < len && s < tmax; s++) {
                int t = dir == 0 ? s : len - 1 - s;
                for (int row = 0; row < G; row++) {
                    const float *rr = R + (long)row * hid;
                    float a = 0.f;
                    for (int q = 0; q < hid; q++) a += rr[q] * h[q];
                    acc[row] = a;
                }
                const float *gb = g + ((long)t * ntot + line) * 2 * G + (long)dir * G;
                float *yo = y + ((long)t * ntot + line) * 2 * hid + (long)dir * hid;
                for (int j = 0; j < hid; j++) {
                    float z = sigm(gb[j] + acc[j] + RB[j]);
                    float rr = sigm(gb[hid + j] + acc[hid + j] + RB[hid + j]);
                    float c = tanhf(gb[2 * hid + j] + rr * (acc[2 * hid + j] + RB[2 * hid + j]));
                    yo[j] = (1.0f - z) * c + z * h[j];
                }
                for (int j = 0; j < hid; j++) h[j] = yo[j];
            }
            free(h);
            free(acc);
        }
    }
}

/* AvgPool (kh, 1) over the whole height to one row, time-major [t][ntot][c] at line offset
 * `noff` (src/gpu.rs:595-614). */
void oracle_avgpool_t(const float *x, int n, int c, int h, int w, int kh, int ntot, int noff, float *y) {
    for (int nb = 0; nb < n; nb++)
        for (int t = 0; t < w; t++)
            for (int ch = 0; ch < c; ch++) {
                float s = 0.f;
                for (int r = 0; r < kh; r++) s += x[(((long)nb * c + ch) * h + r) * w + t];
                y[((long)t * ntot + noff + nb) * c + ch] = s / (float)kh;
            }
}

/* LayerNorm over the last axis, two-pass (src/nd.rs:135-153). */
void oracle_layer_norm(const float *x, const float *gamma, const float *beta, long rows, int len, float eps,
                       float *y) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < rows; i++) {
        const float *xr = x + i * len;
        float m = 0.f, v = 0.f;
        for (int j = 0; j < len; j++) m += xr[j];
        m /= (float)len;
        for (int j = 0; j < len; j++) { float d = xr[j] - m; v += d * d; }
        float inv = 1.0f / sqrtf(v / (float)len + eps);
        for (int j = 0; j < len; j++) y[i * len + j] = (xr[j] - m) * inv * gamma[j] + beta[j];
    }
}

/* Row softmax (src/nd.rs:206-220). */
void oracle_softmax(const float *x, long rows, long len, float *y) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < rows; i++) {
        const float *xr = x + i * len;
        float m = -3.4e38f, s = 0.f;
        for (long j = 0; j < len; j++) m = xr[j] > m ? xr[j] : m;
        for (long j = 0; j < len; j++) s += expf(xr[j] - m);
        for (long j = 0; j < len; j++) y[i * len + j] = expf(xr[j] - m) / s;
    }
}

/*
 * Row arg-max; ties -> the lowest index (src/nd.rs:360-391).  Also, per row, the largest value,
 * the second largest (for the tie band) and log(sum(exp(v - max))) + max.
 */
void oracle_argmax(const float *x, long rows, long len, uint32_t *best, float *top1, float *top2, float *lse) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < rows; i++) {
        const float *xr = x + i * len;
        float m1 = -3.4e38f, m2 = -3.4e38f;
        long at = 0;
        for (long j = 0; j < len; j++) {
            float v = xr[j];
            if (v > m1) { m2 = m1; m1 = v; at = j; }
            else if (v > m2) m2 = v;
        }
        double s = 0.0;
        for (long j = 0; j < len; j++) s += exp((double)xr[j] - (double)m1);
        best[i] = (uint32_t)at;
        if (top1) top1[i] = m1;
        if (top2) top2[i] = m2;
        if (lse) lse[i] = (float)(log(s) + (double)m1);
    }
}

/* Mean over the trailing `inner` values of each of `outer` rows (src/nd.rs:98-133). */
void oracle_reduce_mean(const float *x, long outer, long inner, float *y) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < outer; i++) {
        float s = 0.f;
        for (long j = 0; j < inner; j++) s += x[i * inner + j];
        y[i] = s / (float)inner;
    }
}

/* Batched y[b] = a[b] (m x k) . c[b] (k x n), row-major, fp32 (src/nd.rs:947-962). */
void oracle_bmm(const float *a, const float *c, long batch, int m, int k, int n, float *y) {
#pragma omp parallel for collapse(2) schedule(static)
    for (long bt = 0; bt < batch; bt++)
        for (int r = 0; r < m; r++) {
            const float *ar = a + (bt * m + r) * (long)k;
            const float *cb = c + bt * (long)k * n;
            float *yr = y + (bt * m + r) * (long)n;
            for (int j = 0; j < n; j++) yr[j] = 0.f;
            for (int q = 0; q < k; q++) {
                float av = ar[q];
                const float *cr = cb + (long)q * n;
                for (int j = 0; j < n; j++) yr[j] += av * cr[j];
            }
        }
}

/* Elementwise unary ops of src/nd.rs:67-96: 1 Relu, 2 Sigmoid, 3 HardSigmoid(alpha, beta),
 * 4 Erf, 5 Sqrt. */
void oracle_unary(const float *x, long n, int op, float alpha, float beta, float *y) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < n; i++) {
        float v = x[i], r = v;
        switch (op) {
        case 1: r = v > 0.f ? v : 0.f; break;
        case 2: r = 1.0f / (1.0f + expf(-v)); break;
        case 3: r = alpha * v + beta; r = r < 0.f ? 0.f : (r > 1.f ? 1.f : r); break;
        case 4: r = erf_as(v); break;
        case 5: r = sqrtf(v); break;
        default: break;
        }
        y[i] = r;
    }
}

/*
 * PP-OCR recognition line (src/ppocr.rs:39-62).  The box [left, top, right, bottom] of an RGB
 * page is clamped to the page (v.max(0).min(size) as u32) and cut out as the reference cuts it:
 * crop row y is the cw * 3 bytes at ((top + y) * w + left) * 3, or zeros when that range leaves
 * the page buffer.  It is resized to height 48 keeping its aspect ratio,
 * out_w = clamp(ceil(48 cw / ch), 8, 3200), with the Triangle filter of the `image` crate's
 * imageops::resize (image =0.25.10, an un-vendored dependency; restated from its published
 * separable-resampling algorithm):
 *   - per axis: ratio = in / out, s = max(ratio, 1), support = s, c = (o + 0.5) ratio;
 *   - taps i in [clamp(floor(c - s), 0, in - 1), clamp(ceil(c + s), left + 1, in));
 *   - weight tri((i - (c - 0.5)) / s) / (sum of the weights), tri(x) = max(0, 1 - |x|);
 *   - a vertical pass into an f32 image, then a horizontal pass clamped to [0, 255] and rounded
 *     to u8 (half away from zero).
 * Then (v / 255 - 0.5) / 0.5, planar [3][48][out_w].  Returns out_w; with out == NULL it only
 * returns it.
 */
static float tri_kernel(float x) {
    x = fabsf(x);
    return x < 1.f ? 1.f - x : 0.f;
}

/* Taps of output coordinate o of one axis: first input index in *left, count returned, the
 * normalised weights in ws (at most `cap`). */
static int resample_taps(int in, int out, int o, int *left, float *ws, int cap) {
    float ratio = (float)in / (float)out;
    float sratio = ratio < 1.f ? 1.f : ratio;
    float support = 1.0f * sratio;
    float center = ((float)o + 0.5f) * ratio;
    long l = (long)floorf(center - support);
    l = l < 0 ? 0 : (l > in - 1 ? in - 1 : l);
    long r = (long)ceilf(center + support);
    r = r < l + 1 ? l + 1 : (r > in ? in : r);
    center = center - 0.5f;
    float sum = 0.f;
    int n = 0;
    for (long i = l; i < r && n < cap; i++, n++) {
        ws[n] = tri_kernel(((float)i - center) / sratio);
        sum = sum + ws[n];
    }
    for (int k = 0; k < n; k++) ws[k] = ws[k] / sum;
    *left = (int)l;
    return n;
}

static unsigned clamp_box(float v, int hi) {
    if (!(v > 0.f)) v = 0.f; /* Rust f32::max ignores NaN */
    if (v > (float)hi) v = (float)hi;
    return (unsigned)v;
}

int oracle_pp_line(const uint8_t *rgb, int w, int h, const float *rect, float *out) {
    unsigned l = clamp_box(rect[0], w), t = clamp_box(rect[1], h), r = clamp_box(rect[2], w), b = clamp_box(rect[3], h);
    int cw = r > l ? (int)(r - l) : 1, ch = b > t ? (int)(b - t) : 1;
    float fw = ceilf(48.f * (float)cw / (float)ch);
    int ow = fw < 8.f ? 8 : (fw > 3200.f ? 3200 : (int)fw);
    if (!out) return ow;
    const long total = (long)w * h * 3;
    int cap = 2 * (cw > ch ? cw : ch) + 8;
    float *wx = (float *)malloc(sizeof(float) * cap), *wy = (float *)malloc(sizeof(float) * cap);
    for (int y = 0; y < 48; y++) {
        int ly, ny = resample_taps(ch, 48, y, &ly, wy, cap);
        for (int x = 0; x < ow; x++) {
            int lx, nx = resample_taps(cw, ow, x, &lx, wx, cap);
            for (int c = 0; c < 3; c++) {
                float acc = 0.f;
                for (int j = 0; j < nx; j++) {
                    float v = 0.f;
                    for (int i = 0; i < ny; i++) {
                        long row = ((long)(t + ly + i) * w + l) * 3;
                        float px = 0.f;
                        if (row + (long)cw * 3 <= total) px = (float)rgb[row + (long)(lx + j) * 3 + c];
                        v = v + px * wy[i];
                    }
                    acc = acc + v * wx[j];
                }
                acc = acc < 0.f ? 0.f : (acc > 255.f ? 255.f : acc);
                float q = roundf(acc);
                out[((long)c * 48 + y) * ow + x] = (q / 255.f - 0.5f) / 0.5f;
            }
        }
    }
    free(wx);
    free(wy);
    return ow;
}

/*
 * DB box score (src/ppdet.rs:63-83): the mean of the probabilities (map `prob`, w x h) of the
 * pixels inside the rotated box rect = [cx, cy, up_x, up_y, width, height]:
 * |dx up_x + dy up_y| <= height / 2 and |dx (-up_y) + dy up_x| <= width / 2, dx = x - cx,
 * dy = y - cy, summed in f32 row by row.  The scan covers the box's bounding rectangle widened by
 * a pixel and clamped to the map (the inside test alone decides which pixels count).  0 when no
 * pixel is inside.
 */
/* Rust's `f32 as usize`: saturating, NaN to 0 */
static long db_idx(float v) { return v > 0.f ? (v < 4e9f ? (long)v : 4000000000L) : 0; }

float oracle_db_score(const float *prob, int w, int h, const float *r) {
    float cx = r[0], cy = r[1], ux = r[2], uy = r[3], hw = r[4] / 2.0f, hh = r[5] / 2.0f;
    float lo_x = INFINITY, hi_x = -INFINITY, lo_y = INFINITY, hi_y = -INFINITY;
    for (int sa = -1; sa <= 1; sa += 2)
        for (int sb = -1; sb <= 1; sb += 2) {
            float px = cx + sa * hh * ux + sb * hw * -uy;
            float py = cy + sa * hh * uy + sb * hw * ux;
            lo_x = px < lo_x ? px : lo_x;
            hi_x = px > hi_x ? px : hi_x;
            lo_y = py < lo_y ? py : lo_y;
            hi_y = py > hi_y ? py : hi_y;
        }
    float fx0 = floorf(lo_x) - 1.f, fy0 = floorf(lo_y) - 1.f, fx1 = ceilf(hi_x) + 1.f, fy1 = ceilf(hi_y) + 1.f;
    long x0 = db_idx(fx0), y0 = db_idx(fy0), x1 = db_idx(fx1), y1 = db_idx(fy1);
    if (x1 > w - 1) x1 = w - 1;
    if (y1 > h - 1) y1 = h - 1;
    float sum = 0.f;
    long n = 0;
    for (long y = y0; y <= y1; y++)
        for (long x = x0; x <= x1; x++) {
            float dx = (float)x - cx, dy = (float)y - cy;
            float along = dx * ux + dy * uy;
            float across = dx * -uy + dy * ux;
            if (fabsf(along) <= hh && fabsf(across) <= hw) {
                sum = sum + prob[y * w + x];
                n++;
            }
        }
    return n == 0 ? 0.f : sum / (float)n;
}

/*
 * Word rectangles of a binary detection mask: `word_rects` of src/bin/ocr-bench.rs:38-60 (ocrs'
 * find_connected_component_rects with expand 3, min area 100).  Its steps are rten-imageproc
 * =0.26.0 functions, an un-vendored crates.io dependency, restated here from the published
 * algorithms they name:
 *   find_contours(mask, External): Suzuki & Abe 1985, "Topological structural analysis of
 *     digitized binary images by border following", Algorithm 1 (8-connected foreground, the
 *     image framed by 0-pixels), keeping the outer borders whose parent is the frame;
 *   simplify_polygon(points, 2): Douglas-Peucker on the closed polyline (first point repeated at
 *     the end, dropped again afterwards); point-to-segment distance;
 *   min_area_rect: the convex hull (Andrew's monotone chain, collinear points dropped), then
 *     the exhaustive search over hull edges (each edge's direction and its normal, extents of
 *     the hull's projections, first strict minimum of the area);
 *   RotatedRect::resize(width + 2 (expand + expand_x), height + 2 expand), kept if area >=
 *     min_area.
 * A rectangle is [cx, cy, up_x, up_y, width, height] (the height is measured along up).
 */
typedef struct {
    int *x, *y;
    int n, cap;
} wr_pts;

static void wr_push(wr_pts *p, int x, int y) {
    if (p->n == p->cap) {
        p->cap = p->cap ? 2 * p->cap : 256;
        p->x = (int *)realloc(p->x, sizeof(int) * p->cap);
        p->y = (int *)realloc(p->y, sizeof(int) * p->cap);
    }
    p->x[p->n] = x;
    p->y[p->n] = y;
    p->n++;
}

/* 8-neighbourhood in clockwise order on the screen (y down), starting at the left neighbour */
static const int WR_DX[8] = {-1, -1, 0, 1, 1, 1, 0, -1};
static const int WR_DY[8] = {0, -1, -1, -1, 0, 1, 1, 1};

static int wr_dir(int dx, int dy) {
    for (int d = 0; d < 8; d++)
        if (WR_DX[d] == dx && WR_DY[d] == dy) return d;
    return -1;
}

/* Steps (3.1)-(3.5) of Algorithm 1: follow the border through (x, y) of the padded label image
 * f (row length W), entered from the 0-pixel in direction d2, labelling with nbd.  The border's
 * points (each (i3, j3) in turn) go to out in padded coordinates. */
static void wr_follow(int *f, int W, int x, int y, int d2, int nbd, wr_pts *out) {
    int d1 = -1;
    for (int k = 0; k < 8; k++) {
        int d = (d2 + k) & 7;
        if (f[(y + WR_DY[d]) * W + x + WR_DX[d]] != 0) {
            d1 = d;
            break;
        }
    }
    if (d1 < 0) {
        f[y * W + x] = -nbd;
        wr_push(out, x, y);
        return;
    }
    int x1 = x + WR_DX[d1], y1 = y + WR_DY[d1];
    int x2 = x1, y2 = y1, x3 = x, y3 = y;
    for (;;) {
        wr_push(out, x3, y3);
        int e = wr_dir(x2 - x3, y2 - y3), x4 = x3, y4 = y3, right_zero = 0;
        for (int k = 1; k <= 8; k++) {
            int d = (e - k) & 7, xx = x3 + WR_DX[d], yy = y3 + WR_DY[d];
            if (f[yy * W + xx] != 0) {
                x4 = xx;
                y4 = yy;
                break;
            }
            if (d == 4) right_zero = 1;
        }
        if (right_zero)
            f[y3 * W + x3] = -nbd;
        else if (f[y3 * W + x3] == 1)
            f[y3 * W + x3] = nbd;
        if (x4 == x && y4 == y && x3 == x1 && y3 == y1) break;
        x2 = x3;
        y2 = y3;
        x3 = x4;
        y3 = y4;
    }
}

/* point-to-segment distance (the comp.graphics.algorithms FAQ 1.02 method) */
static float wr_seg_dist(float px, float py, float ax, float ay, float bx, float by) {
    float abx = bx - ax, aby = by - ay, acx = px - ax, acy = py - ay;
    float l2 = abx * abx + aby * aby;
    if (l2 == 0.f) return sqrtf(acx * acx + acy * acy);
    float r = (acx * abx + acy * aby) / l2;
    if (r <= 0.f) return sqrtf(acx * acx + acy * acy);
    if (r >= 1.f) {
        float bcx = px - bx, bcy = py - by;
        return sqrtf(bcx * bcx + bcy * bcy);
    }
    float s = (abx * acy - aby * acx) / l2;
    return fabsf(s * sqrtf(l2));
}

/* Douglas-Peucker over points[lo..hi] (inclusive ends kept), recursion by an explicit stack */
static void wr_dp(const float *px, const float *py, int n, float eps, unsigned char *keep) {
    int *st = (int *)malloc(sizeof(int) * 2 * (size_t)(n + 1));
    int sp = 0;
    keep[0] = keep[n - 1] = 1;
    st[sp++] = 0;
    st[sp++] = n - 1;
    while (sp) {
        int hi = st[--sp], lo = st[--sp];
        float best = -1.f;
        int bi = -1;
        for (int i = lo + 1; i < hi; i++) {
            float d = wr_seg_dist(px[i], py[i], px[lo], py[lo], px[hi], py[hi]);
            if (d > best) {
                best = d;
                bi = i;
            }
        }
        if (bi >= 0 && best > eps) {
            keep[bi] = 1;
            st[sp++] = lo;
            st[sp++] = bi;
            st[sp++] = bi;
            st[sp++] = hi;
        }
    }
    free(st);
}

static int wr_cmp(const void *a, const void *b) {
    const int *p = (const int *)a, *q = (const int *)b;
    if (p[0] != q[0]) return p[0] < q[0] ? -1 : 1;
    return p[1] < q[1] ? -1 : p[1] > q[1];
}

static int64_t wr_cross(const int *o, const int *a, const int *b) {
    return (int64_t)(a[0] - o[0]) * (b[1] - o[1]) - (int64_t)(a[1] - o[1]) * (b[0] - o[0]);
}

/* The minimum-area rectangle of integer points xy[n][2] (sorted in place).  Returns 0 when the
 * points are fewer than two distinct ones. */
static int wr_min_rect(int *xy, int n, float *rect) {
    qsort(xy, (size_t)n, sizeof(int) * 2, wr_cmp);
    int m = 0;
    for (int i = 0; i < n; i++)
        if (m == 0 || xy[2 * i] != xy[2 * (m - 1)] || xy[2 * i + 1] != xy[2 * (m - 1) + 1]) {
            xy[2 * m] = xy[2 * i];
            xy[2 * m + 1] = xy[2 * i + 1];
            m++;
        }
    if (m < 2) return 0;
    int *hull = (int *)malloc(sizeof(int) * 2 * (size_t)(2 * m + 1));
    int k = 0;
    for (int i = 0; i < m; i++) {
        while (k >= 2 && wr_cross(hull + 2 * (k - 2), hull + 2 * (k - 1), xy + 2 * i) <= 0) k--;
        hull[2 * k] = xy[2 * i];
        hull[2 * k + 1] = xy[2 * i + 1];
        k++;
    }
    for (int i = m - 2, lo = k + 1; i >= 0; i--) {
        while (k >= lo && wr_cross(hull + 2 * (k - 2), hull + 2 * (k - 1), xy + 2 * i) <= 0) k--;
        hull[2 * k] = xy[2 * i];
        hull[2 * k + 1] = xy[2 * i + 1];
        k++;
    }
    int h = k - 1; /* the last point repeats the first */
    float best = INFINITY;
    for (int i = 0; i < h; i++) {
        const int *a = hull + 2 * i, *b = hull + 2 * ((i + 1) % h);
        float dx = (float)(b[0] - a[0]), dy = (float)(b[1] - a[1]);
        float len = sqrtf(dx * dx + dy * dy);
        float ux = dx / len, uy = dy / len;
        float s0 = INFINITY, s1 = -INFINITY, t0 = INFINITY, t1 = -INFINITY;
        for (int j = 0; j < h; j++) {
            float rx = (float)(hull[2 * j] - a[0]), ry = (float)(hull[2 * j + 1] - a[1]);
            float s = rx * ux + ry * uy, t = rx * -uy + ry * ux;
            s0 = s < s0 ? s : s0;
            s1 = s > s1 ? s : s1;
            t0 = t < t0 ? t : t0;
            t1 = t > t1 ? t : t1;
        }
        float area = (s1 - s0) * (t1 - t0);
        if (area < best) {
            best = area;
            float sc = (s0 + s1) * 0.5f, tc = (t0 + t1) * 0.5f;
            rect[0] = (float)a[0] + ux * sc + -uy * tc;
            rect[1] = (float)a[1] + uy * sc + ux * tc;
            rect[2] = -uy;
            rect[3] = ux;
            rect[4] = s1 - s0;
            rect[5] = t1 - t0;
        }
    }
    free(hull);
    return 1;
}

/* The rectangle of one contour (unpadded integer points), before resize: 0 when none. */
static int wr_contour_rect(const wr_pts *c, float *rect) {
    int n = c->n + 1; /* closed: the first point again at the end */
    float *px = (float *)malloc(sizeof(float) * (size_t)n), *py = (float *)malloc(sizeof(float) * (size_t)n);
    unsigned char *keep = (unsigned char *)calloc((size_t)n, 1);
    for (int i = 0; i < n; i++) {
        px[i] = (float)c->x[i % c->n];
        py[i] = (float)c->y[i % c->n];
    }
    wr_dp(px, py, n, 2.0f, keep);
    int *xy = (int *)malloc(sizeof(int) * 2 * (size_t)n), m = 0;
    for (int i = 0; i < n - 1; i++)
        if (keep[i]) {
            xy[2 * m] = c->x[i];
            xy[2 * m + 1] = c->y[i];
            m++;
        }
    int ok = wr_min_rect(xy, m, rect);
    free(px);
    free(py);
    free(keep);
    free(xy);
    return ok;
}

/* The external contours of mask (w x h bits, ceil(w / 32) words per row, bit b of word j =
 * pixel 32 j + b) in the order the raster scan meets them, as unpadded pixel coordinates, into
 * *out_c; returns their number. */
static int wr_contours(const uint32_t *mask, int w, int h, wr_pts **out_c) {
    const int W = w + 2, H = h + 2, words = (w + 31) / 32;
    int *f = (int *)calloc((size_t)W * H, sizeof(int));
    for (int y = 0; y < h; y++)
        for (int x = 0; x < w; x++) f[(y + 1) * W + x + 1] = (mask[(size_t)y * words + x / 32] >> (x % 32)) & 1u;
    int cap = 1024, nb = 1, nc = 0;
    int *type = (int *)malloc(sizeof(int) * cap), *parent = (int *)malloc(sizeof(int) * cap);
    wr_pts *cs = NULL;
    int ccap = 0;
    type[1] = 0; /* the frame: a hole border */
    parent[1] = 0;
    for (int y = 1; y < H - 1; y++) {
        int lnbd = 1;
        for (int x = 1; x < W - 1; x++) {
            int v = f[y * W + x];
            if (v == 0) continue;
            int outer = v == 1 && f[y * W + x - 1] == 0;
            int hole = !outer && v >= 1 && f[y * W + x + 1] == 0;
            if (outer || hole) {
                if (hole && v > 1) lnbd = v;
                nb++;
                if (nb >= cap) {
                    cap *= 2;
                    type = (int *)realloc(type, sizeof(int) * cap);
                    parent = (int *)realloc(parent, sizeof(int) * cap);
                }
                type[nb] = outer;
                if (outer)
                    parent[nb] = type[lnbd] ? parent[lnbd] : lnbd;
                else
                    parent[nb] = type[lnbd] ? lnbd : parent[lnbd];
                wr_pts pts = {0};
                wr_follow(f, W, x, y, outer ? 0 : 4, nb, &pts);
                if (outer && parent[nb] == 1) {
                    if (nc == ccap) {
                        ccap = ccap ? 2 * ccap : 64;
                        cs = (wr_pts *)realloc(cs, sizeof(wr_pts) * ccap);
                    }
                    for (int i = 0; i < pts.n; i++) {
                        pts.x[i] -= 1;
                        pts.y[i] -= 1;
                    }
                    cs[nc++] = pts;
                } else {
                    free(pts.x);
                    free(pts.y);
                }
            }
            v = f[y * W + x];
            if (v != 1) lnbd = v < 0 ? -v : v;
        }
    }
    free(f);
    free(type);
    free(parent);
    *out_c = cs;
    return nc;
}

/* The external contours, flattened: returns the number of contours; lens / xs / ys are filled
 * up to their capacities (cap_c contours, cap_p points); *n_points = the total length. */
int oracle_contours(const uint32_t *mask, int w, int h, int *lens, int cap_c, int *xs, int *ys, int64_t cap_p,
                    int64_t *n_points) {
    wr_pts *cs = NULL;
    int nc = wr_contours(mask, w, h, &cs);
    int64_t np = 0;
    for (int i = 0; i < nc; i++) {
        if (i < cap_c) lens[i] = cs[i].n;
        for (int j = 0; j < cs[i].n; j++, np++)
            if (np < cap_p) {
                xs[np] = cs[i].x[j];
                ys[np] = cs[i].y[j];
            }
        free(cs[i].x);
        free(cs[i].y);
    }
    free(cs);
    *n_points = np;
    return nc;
}

/* word_rects (src/bin/ocr-bench.rs:38-60): rectangles [cx, cy, up_x, up_y, width, height] of the
 * external contours, expanded and filtered by area; returns their number (rects filled up to
 * cap). */
int oracle_word_rects(const uint32_t *mask, int w, int h, float expand, float expand_x, float min_area, float *rects,
                      int cap) {
    wr_pts *cs = NULL;
    int nc = wr_contours(mask, w, h, &cs), n = 0;
    for (int i = 0; i < nc; i++) {
        float r[6] = {0};
        if (wr_contour_rect(&cs[i], r)) {
            r[4] = r[4] + 2.f * (expand + expand_x);
            r[5] = r[5] + 2.f * expand;
            if (r[4] * r[5] >= min_area) {
                if (n < cap) memcpy(rects + 6 * (size_t)n, r, sizeof r);
                n++;
            }
        }
        free(cs[i].x);
        free(cs[i].y);
    }
    free(cs);
    return n;
}

/* A box's bounding rectangle (its four corners: center +- up * height / 2 +- across * width / 2)
 * for the reading-order sort of src/ppdet.rs:117-130. */
static void db_bounds(const float *r, float *left, float *top) {
    float hw = r[4] / 2.0f, hh = r[5] / 2.0f, lx = INFINITY, ty = INFINITY;
    for (int sa = -1; sa <= 1; sa += 2)
        for (int sb = -1; sb <= 1; sb += 2) {
            float px = r[0] + sa * hh * r[2] + sb * hw * -r[3];
            float py = r[1] + sa * hh * r[3] + sb * hw * r[2];
            lx = px < lx ? px : lx;
            ty = py < ty ? py : ty;
        }
    *left = lx;
    *top = ty;
}

/*
 * `ppdet::boxes` (src/ppdet.rs:87-132): DB text boxes of a probability map (w x h) in page
 * coordinates, in reading order.  The mask is p > thresh; each external contour, simplified
 * (epsilon 2), gives its minimum-area rectangle (the word_rects restatement above, no expand);
 * it is kept when min(width, height) >= min_size and its `score` >= box_thresh, then unclipped
 * by d = w h unclip_ratio / max(2 (w + h), 1e-6) on every side, dropped when min side <
 * min_size + 2, and scaled to the page (center by to_page, sides by their mean).  Sorted by the
 * top of the bounding rectangle (stable), then boxes whose tops are within 10 px move left of
 * their predecessors by an insertion pass.  Returns the number of boxes (filled up to cap).
 */
int oracle_db_boxes(const float *prob, int w, int h, const float *to_page, float thresh, float box_thresh,
                    float unclip_ratio, float min_size, float *out, int cap) {
    const int words = (w + 31) / 32;
    uint32_t *bits = (uint32_t *)calloc((size_t)words * h, 4);
    for (int y = 0; y < h; y++)
        for (int x = 0; x < w; x++)
            if (prob[(size_t)y * w + x] > thresh) bits[(size_t)y * words + x / 32] |= 1u << (x % 32);
    int nr = oracle_word_rects(bits, w, h, 0.f, 0.f, -INFINITY, NULL, 0);
    float *rs = (float *)malloc(sizeof(float) * 6 * (size_t)(nr > 0 ? nr : 1));
    oracle_word_rects(bits, w, h, 0.f, 0.f, -INFINITY, rs, nr);
    free(bits);
    float *keep = (float *)malloc(sizeof(float) * 6 * (size_t)(nr > 0 ? nr : 1));
    int n = 0;
    const float s = (to_page[0] + to_page[1]) / 2.0f;
    for (int i = 0; i < nr; i++) {
        const float *r = rs + 6 * (size_t)i;
        float rw = r[4], rh = r[5];
        if ((rw < rh ? rw : rh) < min_size || oracle_db_score(prob, w, h, r) < box_thresh) continue;
        float per = 2.0f * (rw + rh);
        float d = rw * rh * unclip_ratio / (per > 1e-6f ? per : 1e-6f);
        float nw = rw + 2.0f * d, nh = rh + 2.0f * d;
        if ((nw < nh ? nw : nh) < min_size + 2.0f) continue;
        float *o = keep + 6 * (size_t)n++;
        o[0] = r[0] * to_page[0];
        o[1] = r[1] * to_page[1];
        o[2] = r[2];
        o[3] = r[3];
        o[4] = nw * s;
        o[5] = nh * s;
    }
    free(rs);
    /* stable sort by top (insertion sort keeps equal keys in order) */
    float *tops = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    float *lefts = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    for (int i = 0; i < n; i++) db_bounds(keep + 6 * (size_t)i, &lefts[i], &tops[i]);
    for (int i = 1; i < n; i++)
        for (int j = i; j > 0 && tops[j] < tops[j - 1]; j--) {
            float t[6];
            memcpy(t, keep + 6 * (size_t)j, sizeof t);
            memcpy(keep + 6 * (size_t)j, keep + 6 * (size_t)(j - 1), sizeof t);
            memcpy(keep + 6 * (size_t)(j - 1), t, sizeof t);
            float u = tops[j]; tops[j] = tops[j - 1]; tops[j - 1] = u;
            u = lefts[j]; lefts[j] = lefts[j - 1]; lefts[j - 1] = u;
        }
    for (int i = 0; i < n; i++)
        for (int j = i; j > 0 && fabsf(tops[j] - tops[j - 1]) < 10.0f && lefts[j] < lefts[j - 1]; j--) {
            float t[6];
            memcpy(t, keep + 6 * (size_t)j, sizeof t);
            memcpy(keep + 6 * (size_t)j, keep + 6 * (size_t)(j - 1), sizeof t);
            memcpy(keep + 6 * (size_t)(j - 1), t, sizeof t);
            float u = tops[j]; tops[j] = tops[j - 1]; tops[j - 1] = u;
            u = lefts[j]; lefts[j] = lefts[j - 1]; lefts[j - 1] = u;
        }
    if (out) memcpy(out, keep, sizeof(float) * 6 * (size_t)(n < cap ? n : cap));
    free(keep);
    free(tops);
    free(lefts);
    return n;
}

/*
 * ---- the ocrs page pipeline: text lines, line padding, line images -----------------------
 * The reference's ocrs path (src/bin/ocr-bench.rs:458-585 without DET / REC) turns the word
 * rectangles of a page mask (word_rects above) into text lines with ocrs' find_text_lines
 * (src/bin/ocr-bench.rs:516), pads them (src/bin/ocr-bench.rs:534-558, RELV 0.15, RELEND 0.1)
 * and cuts one 64-row line image per line with ocrs' prepare_recognition_input
 * (src/bin/ocr-bench.rs:365-408), batched by width.  ocrs =0.13.1 is an un-vendored crates.io
 * dependency, so its two functions are restated from their documented behaviour; PARITY
 * UNPINNED for them (no test of the reference pins either).  The rules, in full:
 *
 * Lines (group_into_lines): words sorted by the integer part of their bounding rectangle's left
 * edge (stable).  A line starts at the first remaining word and grows to the right: among the
 * remaining words whose bounding left edge is at least the last word's right edge minus 5 px and
 * whose bounding rectangles overlap the last word's vertically by at least 5 px, the one with the
 * smallest left edge (the first in sorted order on ties) joins, until none does.  Lines are put in
 * reading order by the top of their first word's bounding rectangle (stable).  ocrs also splits
 * lines at column separators found from empty page regions; the single-column synthetic pages
 * have none, and that step is not restated.
 *
 * Line image: the line's polygon is, word by word left to right, the two corners of each word's
 * top edge, then, right to left, the two corners of each bottom edge, each corner truncated to
 * integers (Rust's `as i32`).  A word's top edge is the side its most upward axis points to: of
 * up, -up, right = (-up.y, up.x) and -right (first on ties), the one with the smallest y
 * component.  The crop is the polygon's bounding rectangle clamped to the page (at least 1 x 1).
 * Each crop pixel whose centre is inside the polygon (even-odd rule) takes its grey value
 * (-0.5 + (0.299 r + 0.587 g + 0.114 b) / 255, the ocrs input normalisation the detector's grey
 * conversion also follows, src/gpu.rs:537-542); the others are BLACK (-0.5).  The crop is resized
 * to 64 x W, W = (int) clamp(64 cw / ch, 10, 800), by half-pixel bilinear interpolation with the
 * detector's resize arithmetic (src/gpu.rs:543-560).
 *
 * Batches (line_batches, src/bin/ocr-bench.rs:365-408): lines grouped by W rounded up to a
 * multiple of 50 (ascending), 20 lines a batch in line order, padded with BLACK.
 */

static void rr_corner(const float *r, int sa, int sb, float *x, float *y) {
    const float hw = r[4] / 2.0f, hh = r[5] / 2.0f;
    *x = r[0] + (float)sa * hh * r[2] + (float)sb * hw * -r[3];
    *y = r[1] + (float)sa * hh * r[3] + (float)sb * hw * r[2];
}

/* The bounding rectangle of a rotated rect [cx, cy, up_x, up_y, width, height]. */
static void rr_bounds(const float *r, float *l, float *t, float *rt, float *b) {
    *l = INFINITY, *t = INFINITY, *rt = -INFINITY, *b = -INFINITY;
    for (int sa = -1; sa <= 1; sa += 2)
        for (int sb = -1; sb <= 1; sb += 2) {
            float x, y;
            rr_corner(r, sa, sb, &x, &y);
            *l = x < *l ? x : *l;
            *rt = x > *rt ? x : *rt;
            *t = y < *t ? y : *t;
            *b = y > *b ? y : *b;
        }
}

int oracle_text_lines(const float *words, int n, int *order, int *line_len) {
    int *idx = (int *)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
    int *key = (int *)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
    float *bl = (float *)malloc(sizeof(float) * 4 * (size_t)(n > 0 ? n : 1));
    char *used = (char *)calloc((size_t)(n > 0 ? n : 1), 1);
    for (int i = 0; i < n; i++) {
        float *q = bl + 4 * (size_t)i;
        rr_bounds(words + 6 * (size_t)i, &q[0], &q[1], &q[2], &q[3]);
        key[i] = (int)q[0];
        idx[i] = i;
    }
    for (int i = 1; i < n; i++)  /* stable insertion sort by the truncated left edge */
        for (int j = i; j > 0 && key[idx[j]] < key[idx[j - 1]]; j--) {
            int u = idx[j];
            idx[j] = idx[j - 1];
            idx[j - 1] = u;
        }
    int nl = 0, o = 0;
    int *first = (int *)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
    int *tmp = (int *)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
    for (int s = 0; s < n; s++) {
        if (used[idx[s]]) continue;
        int last = idx[s], start = o, len = 1;
        used[last] = 1;
        tmp[o++] = last;
        for (;;) {
            const float *lb = bl + 4 * (size_t)last;
            int best = -1;
            for (int q = 0; q < n; q++) {
                const int c = idx[q];
                if (used[c]) continue;
                const float *cb = bl + 4 * (size_t)c;
                const float ov = (lb[3] < cb[3] ? lb[3] : cb[3]) - (lb[1] > cb[1] ? lb[1] : cb[1]);
                if (cb[0] >= lb[2] - 5.0f && ov >= 5.0f && (best < 0 || cb[0] < bl[4 * (size_t)best]))
                    best = c;
            }
            if (best < 0) break;
            used[best] = 1;
            tmp[o++] = best;
            last = best;
            len++;
        }
        first[nl] = start;
        line_len[nl] = len;
        nl++;
    }
    /* reading order: stable by the top of the first word's bounding rectangle */
    int *lo = (int *)malloc(sizeof(int) * (size_t)(nl > 0 ? nl : 1));
    for (int i = 0; i < nl; i++) lo[i] = i;
    for (int i = 1; i < nl; i++)
        for (int j = i; j > 0 && bl[4 * (size_t)tmp[first[lo[j]]] + 1] < bl[4 * (size_t)tmp[first[lo[j - 1]]] + 1];
             j--) {
            int u = lo[j];
            lo[j] = lo[j - 1];
            lo[j - 1] = u;
        }
    int *lens = (int *)malloc(sizeof(int) * (size_t)(nl > 0 ? nl : 1));
    memcpy(lens, line_len, sizeof(int) * (size_t)nl);
    o = 0;
    for (int i = 0; i < nl; i++) {
        line_len[i] = lens[lo[i]];
        for (int k = 0; k < lens[lo[i]]; k++) order[o++] = tmp[first[lo[i]] + k];
    }
    free(idx), free(key), free(bl), free(used), free(first), free(tmp), free(lo), free(lens);
    return nl;
}

/* Line padding of src/bin/ocr-bench.rs:534-558 on words[nw] of one line, in place: every word
 * relv x the line's median word height taller on both sides, the first and last relend x it
 * longer at their ends (height and width swap for a word whose up axis is nearer horizontal). */
void oracle_pad_line(float *words, int nw, float relv, float relend) {
    if (nw <= 0) return;
    float *hs = (float *)malloc(sizeof(float) * (size_t)nw);
    for (int i = 0; i < nw; i++) {
        const float *r = words + 6 * (size_t)i;
        hs[i] = fabsf(r[3]) >= fabsf(r[2]) ? r[5] : r[4];
    }
    for (int i = 1; i < nw; i++)
        for (int j = i; j > 0 && hs[j] < hs[j - 1]; j--) {
            float u = hs[j];
            hs[j] = hs[j - 1];
            hs[j - 1] = u;
        }
    const float med = hs[nw / 2];
    free(hs);
    for (int i = 0; i < nw; i++) {
        float *r = words + 6 * (size_t)i;
        const float along = (i == 0 || i + 1 == nw) ? relend * med : 0.0f, across = relv * med;
        if (fabsf(r[3]) >= fabsf(r[2])) {
            r[4] = r[4] + 2.0f * along;
            r[5] = r[5] + 2.0f * across;
        } else {
            r[4] = r[4] + 2.0f * across;
            r[5] = r[5] + 2.0f * along;
        }
    }
}

/* The integer polygon of a line (4 nw vertices, x then y). */
static void line_polygon(const float *words, int nw, int *px, int *py) {
    for (int i = 0; i < nw; i++) {
        const float *r = words + 6 * (size_t)i;
        const float hw = r[4] / 2.0f, hh = r[5] / 2.0f;
        /* candidates: up, -up, right = (-up.y, up.x), -right */
        const float cand[4][3] = {{r[2], r[3], hh}, {-r[2], -r[3], hh}, {-r[3], r[2], hw}, {r[3], -r[2], hw}};
        int k = 0;
        for (int q = 1; q < 4; q++)
            if (cand[q][1] < cand[k][1]) k = q;
        const float ux = cand[k][0], uy = cand[k][1], eu = cand[k][2], er = (k < 2) ? hw : hh;
        const float rx = -uy, ry = ux;
        const float tx = r[0] + eu * ux, ty = r[1] + eu * uy, bx = r[0] - eu * ux, by = r[1] - eu * uy;
        /* upper chain left to right: top-left, top-right */
        px[2 * i] = (int)(tx - er * rx);
        py[2 * i] = (int)(ty - er * ry);
        px[2 * i + 1] = (int)(tx + er * rx);
        py[2 * i + 1] = (int)(ty + er * ry);
        /* lower chain right to left: bottom-right, bottom-left */
        const int j = 4 * nw - 2 - 2 * i;
        px[j] = (int)(bx + er * rx);
        py[j] = (int)(by + er * ry);
        px[j + 1] = (int)(bx - er * rx);
        py[j + 1] = (int)(by - er * ry);
    }
}

static int poly_inside(const int *px, const int *py, int nv, float cx, float cy) {
    int in = 0;
    for (int k = 0, j = nv - 1; k < nv; j = k++) {
        const float yk = (float)py[k], yj = (float)py[j];
        if ((yk > cy) != (yj > cy)) {
            const float xc = (float)px[k] + (cy - yk) * (float)(px[j] - px[k]) / (yj - yk);
            if (cx < xc) in = !in;
        }
    }
    return in;
}

/* The 64-row image of one line (words[nw], padded); returns its width W and, with out, writes
 * [64][W]; crop (nullable) gets [left, top, width, height]. */
int oracle_ocrs_line(const uint8_t *rgb, int w, int h, const float *words, int nw, float *out, int *crop) {
    if (nw <= 0) return 0;
    int *px = (int *)malloc(sizeof(int) * 4 * (size_t)nw), *py = (int *)malloc(sizeof(int) * 4 * (size_t)nw);
    line_polygon(words, nw, px, py);
    int mnx = px[0], mxx = px[0], mny = py[0], mxy = py[0];
    for (int k = 1; k < 4 * nw; k++) {
        mnx = px[k] < mnx ? px[k] : mnx;
        mxx = px[k] > mxx ? px[k] : mxx;
        mny = py[k] < mny ? py[k] : mny;
        mxy = py[k] > mxy ? py[k] : mxy;
    }
    const int l = mnx < 0 ? 0 : (mnx > w - 1 ? w - 1 : mnx), t = mny < 0 ? 0 : (mny > h - 1 ? h - 1 : mny);
    const int r = mxx < l + 1 ? l + 1 : (mxx > w ? w : mxx), b = mxy < t + 1 ? t + 1 : (mxy > h ? h : mxy);
    const int cw = r - l, ch = b - t;
    float fw = 64.0f * (float)cw / (float)ch;
    fw = fw < 10.0f ? 10.0f : (fw > 800.0f ? 800.0f : fw);
    const int W = (int)fw;
    if (crop) {
        crop[0] = l;
        crop[1] = t;
        crop[2] = cw;
        crop[3] = ch;
    }
    if (out) {
        const float sx = (float)cw / (float)W, sy = (float)ch / 64.0f;
        for (int oy = 0; oy < 64; oy++) {
            float iy = sy * ((float)oy + 0.5f) - 0.5f;
            iy = iy < 0.f ? 0.f : (iy > (float)ch - 1.f ? (float)ch - 1.f : iy);
            const int y1 = (int)iy, y2 = y1 + 1 < ch ? y1 + 1 : ch - 1;
            const float wy = iy - (float)y1;
            for (int ox = 0; ox < W; ox++) {
                float ix = sx * ((float)ox + 0.5f) - 0.5f;
                ix = ix < 0.f ? 0.f : (ix > (float)cw - 1.f ? (float)cw - 1.f : ix);
                const int x1 = (int)ix, x2 = x1 + 1 < cw ? x1 + 1 : cw - 1;
                const float wx = ix - (float)x1;
                float v[2][2];
                for (int a = 0; a < 2; a++)
                    for (int c = 0; c < 2; c++) {
                        const int gx = l + (c ? x2 : x1), gy = t + (a ? y2 : y1);
                        v[a][c] = poly_inside(px, py, 4 * nw, (float)gx + 0.5f, (float)gy + 0.5f)
                                      ? grey_px(rgb, w, h, gx, gy)
                                      : -0.5f;
                    }
                const float top = mixf(v[0][0], v[0][1], wx), bot = mixf(v[1][0], v[1][1], wx);
                out[(size_t)oy * W + ox] = mixf(top, bot, wy);
            }
        }
    }
    free(px);
    free(py);
    return W;
}
