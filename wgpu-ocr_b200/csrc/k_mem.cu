// Memory-bound kernels of the hot path: page pre/post-processing, pooling, elementwise,
// row reductions.  Channels-last (NHWC) for 4-D image tensors; vectorised where the layout
// allows.  Grid sizes are multiples of the SM count with grid-stride loops.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>

#include "act.h"
#include "kernels.h"

namespace wocr {
namespace k {

namespace {

constexpr int kThreads = 256;

inline int grid_for(Ctx *c, int64_t work, int per_block = kThreads) {
    int64_t g = (work + per_block - 1) / per_block;
    int64_t cap = (int64_t)c->sm_count * 16;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (int)g;
}

// WGSL mix(a, b, t) = a * (1 - t) + b * t.
__device__ __forceinline__ float mixf(float a, float b, float t) { return a * (1.0f - t) + b * t; }

// ---------------------------------------------------------------------------------------
__global__ void k_grey_resize(const uint8_t *__restrict__ rgb, int64_t page_bytes, int w, int h, int ph, int pw,
                              int oh, int ow, float sx, float sy, float *__restrict__ y) {
    int page = blockIdx.y;
    const uint8_t *src = rgb + page * page_bytes;
    float *dst = y + (int64_t)page * oh * ow;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)oh * ow;
         i += (int64_t)gridDim.x * blockDim.x) {
        int ox = (int)(i % ow), oy = (int)(i / ow);
        float iy = fminf(fmaxf(sy * ((float)oy + 0.5f) - 0.5f, 0.f), (float)ph - 1.f);
        float ix = fminf(fmaxf(sx * ((float)ox + 0.5f) - 0.5f, 0.f), (float)pw - 1.f);
        int y1 = (int)iy, x1 = (int)ix;
        int y2 = min(y1 + 1, ph - 1), x2 = min(x1 + 1, pw - 1);
        float wy = iy - (float)y1, wx = ix - (float)x1;
        auto grey = [&](int x, int yy) -> float {
            if (x >= w || yy >= h) return -0.5f;
            const uint8_t *p = src + ((int64_t)yy * w + x) * 3;
            return -0.5f + (float)p[0] * (0.299f / 255.0f) + (float)p[1] * (0.587f / 255.0f) +
                   (float)p[2] * (0.114f / 255.0f);
        };
        float top = mixf(grey(x1, y1), grey(x2, y1), wx);
        float bot = mixf(grey(x1, y2), grey(x2, y2), wx);
        dst[i] = mixf(top, bot, wy);
    }
}

// k_grey_resize on a compacted page: only the two source rows each output row interpolates,
// rows 2 oy (top) and 2 oy + 1 (bottom) of `cmp`, uploaded by the host.  rows[oy] = {wy (float
// bits), flags}: the vertical weight, and bit 0 / bit 1 when the top / bottom row lies below the
// page (the padding value).  The column arithmetic is k_grey_resize's.
__global__ void k_grey_rows(const uint8_t *__restrict__ cmp, int64_t page_bytes, const int2 *__restrict__ rows, int w,
                            int pw, int oh, int ow, float sx, float *__restrict__ y) {
    int page = blockIdx.y;
    const uint8_t *src = cmp + page * page_bytes;
    float *dst = y + (int64_t)page * oh * ow;
    const int64_t rb = (int64_t)w * 3;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)oh * ow;
         i += (int64_t)gridDim.x * blockDim.x) {
        int ox = (int)(i % ow), oy = (int)(i / ow);
        const int2 rt = rows[oy];
        float wy = __int_as_float(rt.x);
        float ix = fminf(fmaxf(sx * ((float)ox + 0.5f) - 0.5f, 0.f), (float)pw - 1.f);
        int x1 = (int)ix;
        int x2 = min(x1 + 1, pw - 1);
        float wx = ix - (float)x1;
        auto grey = [&](int x, int r) -> float {
            if (x >= w || (rt.y >> r) & 1) return -0.5f;
            const uint8_t *p = src + (2 * oy + r) * rb + (int64_t)x * 3;
            return -0.5f + (float)p[0] * (0.299f / 255.0f) + (float)p[1] * (0.587f / 255.0f) +
                   (float)p[2] * (0.114f / 255.0f);
        };
        float top = mixf(grey(x1, 0), grey(x2, 0), wx);
        float bot = mixf(grey(x1, 1), grey(x2, 1), wx);
        dst[i] = mixf(top, bot, wy);
    }
}

// One warp builds 32 consecutive words of a page row: lane b thresholds pixel 32*wx + b, a
// ballot forms the word, lane j keeps word j and the warp stores its 32 words at once.
__global__ void k_mask_up(const float *__restrict__ m, int stride, int64_t plane, int vw, int vh, int w, int h,
                          int words, float sx, float sy, float thr, uint32_t *__restrict__ bits) {
    int page = blockIdx.z;
    const float *mp = m + page * plane;
    uint32_t *out = bits + (int64_t)page * words * h;
    int lane = threadIdx.x & 31;
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int oy = blockIdx.y;
    int wx0 = warp * 32;
    if (wx0 >= words) return;
    float iy = fminf(fmaxf(sy * ((float)oy + 0.5f) - 0.5f, 0.f), (float)vh - 1.f);
    int y1 = (int)iy;
    int y2 = min(y1 + 1, vh - 1);
    float fy = iy - (float)y1;
    const float *r1 = mp + (int64_t)y1 * stride, *r2 = mp + (int64_t)y2 * stride;
    uint32_t mine = 0;
    int nw = min(32, words - wx0);
    for (int j = 0; j < nw; j++) {
        int ox = (wx0 + j) * 32 + lane;
        bool on = false;
        if (ox < w) {
            float ix = fminf(fmaxf(sx * ((float)ox + 0.5f) - 0.5f, 0.f), (float)vw - 1.f);
            int x1 = (int)ix;
            int x2 = min(x1 + 1, vw - 1);
            float fx = ix - (float)x1;
            float top = mixf(r1[x1], r1[x2], fx);
            float bot = mixf(r2[x1], r2[x2], fx);
            on = mixf(top, bot, fy) > thr;
        }
        uint32_t word = __ballot_sync(0xffffffffu, on);
        if (lane == j) mine = word;
    }
    if (lane < nw) out[(int64_t)oy * words + wx0 + lane] = mine;
}

// k_mask_up for pages up to kMaskCols (3072) wide, a block per kMaskBlockRows page rows of a page.
// Shared memory holds each page column's (x1, fx) (once per block) and the horizontally
// interpolated top and bottom map rows of the current output row (recomputed only when the
// output row reads another pair of map rows, about every h / vh rows); per pixel that leaves two
// shared loads, one blend, a compare and a ballot.  Same arithmetic, in the same order, as
// k_mask_up.
constexpr int kMaskCols = 3072, kMaskBlockRows = 16;  // 43 KB of static shared memory

__global__ void __launch_bounds__(256) k_mask_up_rows(const float *__restrict__ m, int stride, int64_t plane, int vw,
                                                      int vh, int w, int h, int words, float sx, float sy, float thr,
                                                      uint32_t *__restrict__ bits) {
    __shared__ uint16_t xs1[kMaskCols];  // the map is narrower than 65536 columns (checked on the host)
    __shared__ float xfx[kMaskCols], top[kMaskCols], bot[kMaskCols];
    const int page = blockIdx.z;
    const float *mp = m + page * plane;
    uint32_t *out = bits + (int64_t)page * words * h;
    const int oy0 = blockIdx.x * kMaskBlockRows, oy1 = min(oy0 + kMaskBlockRows, h);
    for (int ox = threadIdx.x; ox < w; ox += blockDim.x) {
        const float ix = fminf(fmaxf(sx * ((float)ox + 0.5f) - 0.5f, 0.f), (float)vw - 1.f);
        const int x1 = (int)ix;
        xs1[ox] = (uint16_t)x1;
        xfx[ox] = ix - (float)x1;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    int cy = -1;
    for (int oy = oy0; oy < oy1; oy++) {
        const float iy = fminf(fmaxf(sy * ((float)oy + 0.5f) - 0.5f, 0.f), (float)vh - 1.f);
        const int y1 = (int)iy;
        const float fy = iy - (float)y1;
        if (y1 != cy) {
            __syncthreads();  // the column table is written; the previous rows' readers are done
            cy = y1;
            const int y2 = min(y1 + 1, vh - 1);
            const float *r1 = mp + (int64_t)y1 * stride, *r2 = mp + (int64_t)y2 * stride;
            for (int ox = threadIdx.x; ox < w; ox += blockDim.x) {
                const int x1 = xs1[ox], x2 = min(x1 + 1, vw - 1);
                const float fx = xfx[ox];
                top[ox] = mixf(r1[x1], r1[x2], fx);
                bot[ox] = mixf(r2[x1], r2[x2], fx);
            }
            __syncthreads();
        }
        // warp k takes words k, k + nwarps, ...: lane b thresholds pixel 32 word + b
        for (int wd0 = warp * 32; wd0 < words; wd0 += nwarps * 32) {
            uint32_t mine = 0;
            const int nw = min(32, words - wd0);
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int ox = (wd0 + j) * 32 + lane;
                const bool on = j < nw && ox < w && mixf(top[ox < w ? ox : 0], bot[ox < w ? ox : 0], fy) > thr;
                const uint32_t word = __ballot_sync(0xffffffffu, on);
                mine = lane == j ? word : mine;
            }
            if (lane < nw) out[(int64_t)oy * words + wd0 + lane] = mine;
        }
    }
}

__global__ void k_det_prep(const uint8_t *__restrict__ rgb, int w, int h, int ow, int oh, float sx, float sy,
                           int nchw, float *__restrict__ y) {
    const float mean[3] = {0.485f, 0.456f, 0.406f};
    const float dev[3] = {0.229f, 0.224f, 0.225f};
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)oh * ow;
         i += (int64_t)gridDim.x * blockDim.x) {
        int ox = (int)(i % ow), oy = (int)(i / ow);
        float ix = fminf(fmaxf(sx * ((float)ox + 0.5f) - 0.5f, 0.f), (float)w - 1.f);
        float iy = fminf(fmaxf(sy * ((float)oy + 0.5f) - 0.5f, 0.f), (float)h - 1.f);
        int x1 = (int)ix, y1 = (int)iy;
        int x2 = min(x1 + 1, w - 1), y2 = min(y1 + 1, h - 1);
        float fx = ix - (float)x1, fy = iy - (float)y1;
        const uint8_t *p11 = rgb + ((int64_t)y1 * w + x1) * 3, *p12 = rgb + ((int64_t)y1 * w + x2) * 3;
        const uint8_t *p21 = rgb + ((int64_t)y2 * w + x1) * 3, *p22 = rgb + ((int64_t)y2 * w + x2) * 3;
#pragma unroll
        for (int c = 0; c < 3; c++) {
            int kb = 2 - c;  // BGR: output channel 0 is blue, byte 2
            float a = mixf((float)p11[kb], (float)p12[kb], fx);
            float b = mixf((float)p21[kb], (float)p22[kb], fx);
            float v = (mixf(a, b, fy) / 255.0f - mean[c]) / dev[c];
            if (nchw) y[(int64_t)c * oh * ow + i] = v;
            else y[i * 3 + c] = v;
        }
    }
}

// ---------------------------------------------------------------------------------------
__global__ void k_pool(const float *__restrict__ x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch, int kh,
                       int kw, int sh, int sw, int pt, int pl, int oh, int ow, int avg, float *__restrict__ y,
                       int64_t y_n, int64_t y_pix) {
    int64_t total = (int64_t)n * oh * ow * ch;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int c = (int)(i % ch);
        int64_t pix = i / ch;
        int ox = (int)(pix % ow);
        int oy = (int)((pix / ow) % oh);
        int nb = (int)(pix / ((int64_t)ow * oh));
        const float *xb = x + nb * x_n + c;
        float m = -3.4e38f, s = 0.f, cnt = 0.f;
        for (int ky = 0; ky < kh; ky++) {
            int iy = oy * sh + ky - pt;
            if (iy < 0 || iy >= h) continue;
            for (int kx = 0; kx < kw; kx++) {
                int ix = ox * sw + kx - pl;
                if (ix < 0 || ix >= w) continue;
                float v = xb[((int64_t)iy * w + ix) * x_pix];
                m = fmaxf(m, v);
                s += v;
                cnt += 1.f;
            }
        }
        y[nb * y_n + ((int64_t)oy * ow + ox) * y_pix + c] = avg ? s / fmaxf(cnt, 1.f) : m;
    }
}

// ---- split activations -------------------------------------------------------------------
__device__ __forceinline__ float bf_f(uint32_t b) { return __uint_as_float(b << 16); }

__device__ __forceinline__ void split_f(float v, uint16_t &h, uint16_t &l) {
    __nv_bfloat16 hb = __float2bfloat16_rn(v);
    __nv_bfloat16 lb = __float2bfloat16_rn(v - __bfloat162float(hb));
    h = *reinterpret_cast<uint16_t *>(&hb);
    l = *reinterpret_cast<uint16_t *>(&lb);
}

// One thread per (output pixel, 8 channels) when VEC (16-byte aligned hi / lo vectors), else per
// channel.  The maximum is taken over hi + lo; its hi and lo parts are copied unchanged.
template <bool VEC>
__global__ void k_maxpool_split(const uint16_t *__restrict__ x, int64_t x_n, int64_t x_pix, int n, int h, int w,
                                int ch, int kh, int kw, int oh, int ow, void *__restrict__ y, int64_t y_n,
                                int64_t y_pix, int split_out) {
    const int cv = VEC ? ch / 8 : ch;
    const int64_t total = (int64_t)n * oh * ow * cv;
    const int64_t xlo = x_pix / 2, ylo = y_pix / 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int cq = (int)(i % cv);
        const int64_t pix = i / cv;
        const int ox = (int)(pix % ow);
        const int oy = (int)((pix / ow) % oh);
        const int nb = (int)(pix / ((int64_t)ow * oh));
        const uint16_t *xb = x + nb * x_n;
        const int64_t yoff = nb * y_n + ((int64_t)oy * ow + ox) * y_pix;
        if (VEC) {
            const int c = cq * 8;
            float best[8];
            uint32_t bh[8], bl[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                best[e] = -3.4e38f;
                bh[e] = bl[e] = 0;
            }
            for (int ky = 0; ky < kh; ky++)
                for (int kx = 0; kx < kw; kx++) {
                    const int iy = oy * kh + ky, ix = ox * kw + kx;
                    if (iy >= h || ix >= w) continue;
                    const uint16_t *src = xb + ((int64_t)iy * w + ix) * x_pix + c;
                    const uint4 hv = *reinterpret_cast<const uint4 *>(src);
                    const uint4 lv = *reinterpret_cast<const uint4 *>(src + xlo);
                    const uint32_t hw4[4] = {hv.x, hv.y, hv.z, hv.w}, lw4[4] = {lv.x, lv.y, lv.z, lv.w};
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const uint32_t hb = (hw4[e >> 1] >> ((e & 1) * 16)) & 0xffffu;
                        const uint32_t lb = (lw4[e >> 1] >> ((e & 1) * 16)) & 0xffffu;
                        const float v = bf_f(hb) + bf_f(lb);
                        if (v > best[e]) {
                            best[e] = v;
                            bh[e] = hb;
                            bl[e] = lb;
                        }
                    }
                }
            if (split_out) {
                uint16_t *yo = reinterpret_cast<uint16_t *>(y) + yoff + c;
                *reinterpret_cast<uint4 *>(yo) = make_uint4(bh[0] | bh[1] << 16, bh[2] | bh[3] << 16,
                                                            bh[4] | bh[5] << 16, bh[6] | bh[7] << 16);
                *reinterpret_cast<uint4 *>(yo + ylo) = make_uint4(bl[0] | bl[1] << 16, bl[2] | bl[3] << 16,
                                                                  bl[4] | bl[5] << 16, bl[6] | bl[7] << 16);
            } else {
                float *yo = reinterpret_cast<float *>(y) + yoff + c;
#pragma unroll
                for (int e = 0; e < 8; e++) yo[e] = best[e];
            }
        } else {
            const int c = cq;
            float best = -3.4e38f;
            uint16_t bh = 0, bl = 0;
            for (int ky = 0; ky < kh; ky++)
                for (int kx = 0; kx < kw; kx++) {
                    const int iy = oy * kh + ky, ix = ox * kw + kx;
                    if (iy >= h || ix >= w) continue;
                    const uint16_t *src = xb + ((int64_t)iy * w + ix) * x_pix + c;
                    const float v = bf_f(src[0]) + bf_f(src[xlo]);
                    if (v > best) {
                        best = v;
                        bh = src[0];
                        bl = src[xlo];
                    }
                }
            if (split_out) {
                uint16_t *yo = reinterpret_cast<uint16_t *>(y) + yoff + c;
                yo[0] = bh;
                yo[ylo] = bl;
            } else {
                reinterpret_cast<float *>(y)[yoff + c] = best;
            }
        }
    }
}

struct Dims4 {
    int64_t d[4], xs[4], ys[4];
};

__device__ __forceinline__ void index4(const Dims4 &g, int64_t i, int64_t &xo, int64_t &yo) {
    xo = yo = 0;
#pragma unroll
    for (int k = 3; k >= 0; k--) {
        const int64_t q = i % g.d[k];
        i /= g.d[k];
        xo += q * g.xs[k];
        yo += q * g.ys[k];
    }
}

__global__ void k_unsplit(const uint16_t *__restrict__ x, int64_t lo_off, float *__restrict__ y, Dims4 g,
                          int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t xo, yo;
        index4(g, i, xo, yo);
        y[yo] = bf_f(x[xo]) + bf_f(x[xo + lo_off]);
    }
}

__global__ void k_resplit(const float *__restrict__ x, uint16_t *__restrict__ y, int64_t lo_off, Dims4 g,
                          int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t xo, yo;
        index4(g, i, xo, yo);
        split_f(x[xo], y[yo], y[yo + lo_off]);
    }
}

// One warp per row: the tiles' maxima reduced over the lanes, the lowest tile reaching the
// maximum gives the column, the sums rescaled to the maximum.
__global__ void k_argmax_merge(const float *__restrict__ pmax, const float *__restrict__ psum,
                               const uint32_t *__restrict__ pidx, int64_t rows, int ntiles, uint32_t *best,
                               float *row_max, float *row_lse) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = wid; r < rows; r += nw) {
        const float *pm = pmax + r * ntiles;
        float m = -INFINITY;
        for (int t = lane; t < ntiles; t += 32) m = fmaxf(m, pm[t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        int first = ntiles;
        float s = 0.f;
        for (int t = lane; t < ntiles; t += 32) {
            const float v = pm[t];
            if (v == m && t < first) first = t;
            if (psum) s += psum[r * ntiles + t] * __expf(v - m);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
            s += __shfl_xor_sync(0xffffffffu, s, o);
        }
        if (lane == 0) {
            best[r] = first < ntiles ? pidx[r * ntiles + first] : 0u;
            if (row_max) row_max[r] = m;
            if (row_lse && psum) row_lse[r] = m + logf(s);
        }
    }
}

// One block per (image, 32-channel slab): threads stride over the pixels, then reduce.
__global__ void k_gap(const float *__restrict__ x, int64_t x_n, int64_t x_pix, int hw, int ch, float *__restrict__ y) {
    __shared__ float part[8][33];
    int nb = blockIdx.y;
    int c = blockIdx.x * 32 + (threadIdx.x & 31);
    int row = threadIdx.x >> 5;  // 8 pixel lanes
    float s = 0.f;
    if (c < ch)
        for (int p = row; p < hw; p += 8) s += x[nb * x_n + (int64_t)p * x_pix + c];
    part[row][threadIdx.x & 31] = s;
    __syncthreads();
    if (row == 0 && c < ch) {
        float t = 0.f;
#pragma unroll
        for (int r = 0; r < 8; r++) t += part[r][threadIdx.x & 31];
        y[(int64_t)nb * ch + c] = t / (float)hw;
    }
}

__global__ void k_resize_nearest(const float *__restrict__ x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch,
                                 int oh, int ow, float sy, float sx, float *__restrict__ y, int64_t y_n, int64_t y_pix) {
    int64_t total = (int64_t)n * oh * ow * ch;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int c = (int)(i % ch);
        int64_t pix = i / ch;
        int ox = (int)(pix % ow);
        int oy = (int)((pix / ow) % oh);
        int nb = (int)(pix / ((int64_t)ow * oh));
        int iy = min((int)floorf((float)oy / sy), h - 1);
        int ix = min((int)floorf((float)ox / sx), w - 1);
        y[nb * y_n + ((int64_t)oy * ow + ox) * y_pix + c] = x[nb * x_n + ((int64_t)iy * w + ix) * x_pix + c];
    }
}

// ---------------------------------------------------------------------------------------
// The element's coordinates from its linear index with 32-bit divisions (tensors below 2^31
// elements: 64-bit division is many times slower), its offsets in x, b and y from them.
__device__ __forceinline__ void strided_offsets32(uint32_t i, const Strided &s, int64_t &xi, int64_t &bi,
                                                  int64_t &yi) {
    uint32_t rem = i;
    xi = bi = yi = 0;
#pragma unroll
    for (int d = kMaxRank - 1; d >= 0; d--) {
        if (d >= s.rank) continue;
        const uint32_t dim = (uint32_t)s.dims[d], cdx = rem % dim;
        rem /= dim;
        xi += (int64_t)cdx * s.xs[d];
        bi += (int64_t)cdx * s.bs[d];
        yi += (int64_t)cdx * s.ys[d];
    }
}

__global__ void k_copy(const float *__restrict__ x, float *__restrict__ y, Strided s, int64_t total) {
    if (total < (int64_t)INT32_MAX) {
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < (uint32_t)total; i += gridDim.x * blockDim.x) {
            int64_t xi, bi, yi;
            strided_offsets32(i, s, xi, bi, yi);
            y[yi] = x[xi];
        }
        return;
    }
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = i, xi = 0, yi = 0;
#pragma unroll
        for (int d = kMaxRank - 1; d >= 0; d--) {
            if (d >= s.rank) continue;
            int64_t cdx = rem % s.dims[d];
            rem /= s.dims[d];
            xi += cdx * s.xs[d];
            yi += cdx * s.ys[d];
        }
        y[yi] = x[xi];
    }
}

__device__ __forceinline__ float binop(int op, float xv, float z) {
    switch (op) {
    case 0: return xv + z;
    case 1: return xv - z;
    case 2: return xv * z;
    case 3: return xv / z;
    default: return z == 2.0f ? xv * xv : (z == 0.5f ? sqrtf(xv) : powf(xv, z));
    }
}

__global__ void k_binary(int op, const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ y,
                         Strided s, int64_t total) {
    if (total < (int64_t)INT32_MAX) {
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < (uint32_t)total; i += gridDim.x * blockDim.x) {
            int64_t ai, bi, yi;
            strided_offsets32(i, s, ai, bi, yi);
            y[yi] = binop(op, a[ai], b[bi]);
        }
        return;
    }
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = i, ai = 0, bi = 0, yi = 0;
#pragma unroll
        for (int d = kMaxRank - 1; d >= 0; d--) {
            if (d >= s.rank) continue;
            int64_t cdx = rem % s.dims[d];
            rem /= s.dims[d];
            ai += cdx * s.xs[d];
            bi += cdx * s.bs[d];
            yi += cdx * s.ys[d];
        }
        y[yi] = binop(op, a[ai], b[bi]);
    }
}

__global__ void k_unary(int op, const float *__restrict__ x, float *__restrict__ y, int64_t n, float alpha, float beta) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float v = x[i], r = v;
        switch (op) {
        case 1: r = fmaxf(v, 0.f); break;
        case 2: r = 1.0f / (1.0f + expf(-v)); break;
        case 3: r = fminf(fmaxf(alpha * v + beta, 0.f), 1.f); break;
        case 4: r = erf_as(v); break;
        case 5: r = sqrtf(v); break;
        default: break;
        }
        y[i] = r;
    }
}

__global__ void k_affine(const float *__restrict__ x, float *__restrict__ y, int64_t n, int C, int64_t cdiv,
                         const float *__restrict__ st) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int c = (int)((i / cdiv) % C);
        y[i] = x[i] * st[c] + st[C + c];
    }
}

// One warp per row.
__global__ void k_reduce_mean(const float *__restrict__ x, float *__restrict__ y, int64_t outer, int64_t inner) {
    int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (row >= outer) return;
    float s = 0.f;
    for (int64_t j = lane; j < inner; j += 32) s += x[row * inner + j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) y[row] = s / (float)inner;
}

// One warp per row, two passes as the reference (src/nd.rs:143-150).
__global__ void k_layer_norm(const float *__restrict__ x, float *__restrict__ y, int64_t rows, int len,
                             const float *__restrict__ gb, float eps) {
    int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *xr = x + row * len;
    float s = 0.f;
    for (int j = lane; j < len; j += 32) s += xr[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    float m = s / (float)len;
    float v = 0.f;
    for (int j = lane; j < len; j += 32) {
        float d = xr[j] - m;
        v += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    float inv = 1.0f / sqrtf(v / (float)len + eps);
    for (int j = lane; j < len; j += 32) y[row * len + j] = (xr[j] - m) * inv * gb[j] + gb[len + j];
}

// One block per row.
__global__ void k_softmax(const float *__restrict__ x, float *__restrict__ y, int64_t rows, int64_t len) {
    __shared__ float red[32];
    int64_t row = blockIdx.x;
    if (row >= rows) return;
    const float *xr = x + row * len;
    float m = -3.4e38f;
    for (int64_t j = threadIdx.x; j < len; j += blockDim.x) m = fmaxf(m, xr[j]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -3.4e38f;
        for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    m = red[0];
    __syncthreads();
    float s = 0.f;
    for (int64_t j = threadIdx.x; j < len; j += blockDim.x) s += expf(xr[j] - m);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    s = red[0];
    for (int64_t j = threadIdx.x; j < len; j += blockDim.x) y[row * len + j] = expf(xr[j] - m) / s;
}

// Rows of at most 1024 values (attention scores): a warp per row, the row in registers, the
// maximum and the sum by shuffles (one block per row spends its time in block barriers).
constexpr int kSmRowWarps = 8;

__global__ void __launch_bounds__(kSmRowWarps * 32) k_softmax_warp(const float *__restrict__ x, float *__restrict__ y,
                                                                   int64_t rows, int len) {
    const int64_t row = (int64_t)blockIdx.x * kSmRowWarps + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *xr = x + row * len;
    float v[32];
    float m = -3.4e38f;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        const int j = lane + 32 * i;
        v[i] = j < len ? xr[j] : -3.4e38f;
        m = fmaxf(m, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++)
        if (lane + 32 * i < len) {
            v[i] = expf(v[i] - m);
            s += v[i];
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    float *yr = y + row * len;
#pragma unroll
    for (int i = 0; i < 32; i++)
        if (lane + 32 * i < len) yr[lane + 32 * i] = v[i] / s;
}

// One block per row: best index (tie rule per `tie_last`), row max and log-sum-exp.
// Lowest-index rule (K30, src/nd.rs:360-391): the search starts from (-3.4e38, index 0) and
// takes a value only when it is larger, so a row of NaN or -inf values gives 0, as there.
// Last-index rule: a row with no value above -3.4e38 gives its last index (Rust's max_by over
// equal keys returns the last).
__global__ void k_argmax(const float *__restrict__ x, int64_t rows, int64_t len, int64_t ld, uint32_t *__restrict__ best,
                         float *__restrict__ row_max, float *__restrict__ row_lse, int tie_last) {
    __shared__ float bv[32];
    __shared__ int64_t bi[32];
    __shared__ float ss[32];
    int64_t row = blockIdx.x;
    if (row >= rows) return;
    const float *xr = x + row * ld;
    float m = -3.4e38f;
    int64_t at = tie_last ? -1 : 0;
    for (int64_t j = threadIdx.x; j < len; j += blockDim.x) {
        float v = xr[j];
        if (v > m || (v == m && (tie_last ? j > at : j < at))) { m = v; at = j; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        float om = __shfl_xor_sync(0xffffffffu, m, o);
        int64_t oa = __shfl_xor_sync(0xffffffffu, at, o);
        if (om > m || (om == m && (tie_last ? oa > at : oa < at))) { m = om; at = oa; }
    }
    int wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) { bv[wid] = m; bi[wid] = at; }
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < nw ? bv[threadIdx.x] : -3.4e38f;
        int64_t ta = threadIdx.x < nw ? bi[threadIdx.x] : (tie_last ? -1 : INT64_MAX);
        for (int o = 16; o > 0; o >>= 1) {
            float om = __shfl_xor_sync(0xffffffffu, t, o);
            int64_t oa = __shfl_xor_sync(0xffffffffu, ta, o);
            if (om > t || (om == t && (tie_last ? oa > ta : oa < ta))) { t = om; ta = oa; }
        }
        if (threadIdx.x == 0) { bv[0] = t; bi[0] = ta; }
    }
    __syncthreads();
    m = bv[0];
    if (row_lse) {
        float s = 0.f;
        for (int64_t j = threadIdx.x; j < len; j += blockDim.x) s += expf(xr[j] - m);
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if ((threadIdx.x & 31) == 0) ss[wid] = s;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = 0.f;
            for (int q = 0; q < nw; q++) t += ss[q];
            row_lse[row] = logf(t) + m;
        }
    }
    if (threadIdx.x == 0) {
        best[row] = (uint32_t)(bi[0] < 0 ? len - 1 : bi[0]);
        if (row_max) row_max[row] = m;
    }
}

// Small batched matmul: 32 x 32 output tile per block, k in steps of 32 through shared memory.
__global__ void k_bmm(const float *__restrict__ a, const float *__restrict__ bm, float *__restrict__ y, int m, int kk,
                      int n) {
    __shared__ float As[32][33], Bs[32][33];
    int64_t bt = blockIdx.z;
    const float *ab = a + bt * (int64_t)m * kk;
    const float *bb = bm + bt * (int64_t)kk * n;
    int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
    int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads, 4 rows each
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < kk; k0 += 32) {
        for (int r = ty; r < 32; r += 8) {
            As[r][tx] = (r0 + r < m && k0 + tx < kk) ? ab[(int64_t)(r0 + r) * kk + k0 + tx] : 0.f;
            Bs[r][tx] = (k0 + r < kk && c0 + tx < n) ? bb[(int64_t)(k0 + r) * n + c0 + tx] : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int q = 0; q < 32; q++) {
            float bv = Bs[q][tx];
#pragma unroll
            for (int i = 0; i < 4; i++) acc[i] += As[ty + 8 * i][q] * bv;
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int r = r0 + ty + 8 * i, cc = c0 + tx;
        if (r < m && cc < n) y[bt * (int64_t)m * n + (int64_t)r * n + cc] = acc[i];
    }
}

__global__ void k_avgpool_t(const float *__restrict__ x, int64_t x_n, int64_t x_pix, int n, int ch, int h, int w,
                            int kh, int ntot, int noff, float *__restrict__ y) {
    int64_t total = (int64_t)n * w * ch;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int c = (int)(i % ch);
        int t = (int)((i / ch) % w);
        int nb = (int)(i / ((int64_t)ch * w));
        float s = 0.f;
        for (int r = 0; r < kh; r++) s += x[nb * x_n + ((int64_t)r * w + t) * x_pix + c];
        y[((int64_t)t * ntot + noff + nb) * ch + c] = s / (float)kh;
    }
}

}  // namespace

// ---------------------------------------------------------------------------------------
void grey_resize(Ctx *c, const uint8_t *rgb, int64_t page_bytes, int n, int w, int h, int oh, int ow, float *y) {
    Prof pf(c, "grey_resize", 0, (double)n * ((double)std::min(h, 2 * oh) * w * 3 + (double)oh * ow * 4));
    int ph = h > oh ? h : oh, pw = w > ow ? w : ow;
    float sx = (float)pw / (float)ow, sy = (float)ph / (float)oh;
    dim3 grid(grid_for(c, (int64_t)oh * ow), n);
    k_grey_resize<<<grid, kThreads, 0, c->stream>>>(rgb, page_bytes, w, h, ph, pw, oh, ow, sx, sy, y);
    WOCR_LAUNCHED(c);
}

void grey_resize_rows(Ctx *c, const uint8_t *cmp, const int2 *rows, int n, int w, int oh, int ow, float *y) {
    const int64_t page_bytes = 2LL * oh * w * 3;
    Prof pf(c, "grey_resize", 0, (double)n * ((double)page_bytes + (double)oh * ow * 4));
    const int pw = w > ow ? w : ow;
    dim3 grid(grid_for(c, (int64_t)oh * ow), n);
    k_grey_rows<<<grid, kThreads, 0, c->stream>>>(cmp, page_bytes, rows, w, pw, oh, ow, (float)pw / (float)ow, y);
    WOCR_LAUNCHED(c);
}

void mask_up(Ctx *c, const float *m, int stride, int64_t plane, int n, int vw, int vh, int w, int h, float thr,
             uint32_t *bits) {
    Prof pf(c, "mask_up", 0, (double)n * ((double)vh * vw * 4 + (double)h * ((w + 31) / 32) * 4));
    int words = (w + 31) / 32;
    int warps = (words + 31) / 32;
    // one block per page row: exactly the row's warps (3 for a 2550-pixel page), so no idle warps
    // hold block slots
    if (w <= kMaskCols && vw < 65536) {
        dim3 grid((unsigned)((h + kMaskBlockRows - 1) / kMaskBlockRows), 1, n);
        k_mask_up_rows<<<grid, 256, 0, c->stream>>>(m, stride, plane, vw, vh, w, h, words, (float)vw / (float)w,
                                                    (float)vh / (float)h, thr, bits);
        WOCR_LAUNCHED(c);
        return;
    }
    const int per_block = std::min(warps, 32);
    dim3 grid((warps + per_block - 1) / per_block, h, n);
    k_mask_up<<<grid, per_block * 32, 0, c->stream>>>(m, stride, plane, vw, vh, w, h, words, (float)vw / (float)w,
                                                  (float)vh / (float)h, thr, bits);
    WOCR_LAUNCHED(c);
}

void det_prep(Ctx *c, const uint8_t *rgb, int w, int h, int ow, int oh, int nchw, float *y) {
    Prof pf(c, "det_prep", 0, (double)std::min(h, 2 * oh) * w * 3 + 12.0 * oh * ow);
    k_det_prep<<<grid_for(c, (int64_t)oh * ow), kThreads, 0, c->stream>>>(rgb, w, h, ow, oh, (float)w / (float)ow,
                                                                           (float)h / (float)oh, nchw, y);
    WOCR_LAUNCHED(c);
}

void pool(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch, int kh, int kw, int sh,
          int sw, int pt, int pl, int oh, int ow, int avg, float *y, int64_t y_n, int64_t y_pix) {
    Prof pf(c, "pool", 0, 4.0 * n * ch * ((double)h * w + (double)oh * ow));
    int64_t total = (int64_t)n * oh * ow * ch;
    k_pool<<<grid_for(c, total), kThreads, 0, c->stream>>>(x, x_n, x_pix, n, h, w, ch, kh, kw, sh, sw, pt, pl, oh, ow,
                                                          avg, y, y_n, y_pix);
    WOCR_LAUNCHED(c);
}

void maxpool_split(Ctx *c, const uint16_t *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch, int kh, int kw,
                   int oh, int ow, void *y, int64_t y_n, int64_t y_pix, int split_out) {
    Prof pf(c, "maxpool_split", 0, 4.0 * n * ch * ((double)h * w + (double)oh * ow));
    const bool al = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
    const bool vec = al && ch % 8 == 0 && x_pix % 16 == 0 && x_n % 8 == 0 &&
                     (split_out ? (y_pix % 16 == 0 && y_n % 8 == 0) : true);
    const int64_t total = (int64_t)n * oh * ow * (vec ? ch / 8 : ch);
    if (total == 0) return;
    if (vec)
        k_maxpool_split<true><<<grid_for(c, total), kThreads, 0, c->stream>>>(x, x_n, x_pix, n, h, w, ch, kh, kw, oh,
                                                                              ow, y, y_n, y_pix, split_out);
    else
        k_maxpool_split<false><<<grid_for(c, total), kThreads, 0, c->stream>>>(x, x_n, x_pix, n, h, w, ch, kh, kw, oh,
                                                                               ow, y, y_n, y_pix, split_out);
    WOCR_LAUNCHED(c);
}

void unsplit(Ctx *c, const uint16_t *x, const int64_t (&xs)[4], int64_t lo_off, float *y, const int64_t (&ys)[4],
             const int64_t (&dims)[4]) {
    Dims4 g;
    int64_t total = 1;
    for (int k = 0; k < 4; k++) {
        g.d[k] = dims[k];
        g.xs[k] = xs[k];
        g.ys[k] = ys[k];
        total *= dims[k];
    }
    if (total == 0) return;
    Prof pf(c, "unsplit", 0, 8.0 * total);
    k_unsplit<<<grid_for(c, total), kThreads, 0, c->stream>>>(x, lo_off, y, g, total);
    WOCR_LAUNCHED(c);
}

void resplit(Ctx *c, const float *x, const int64_t (&xs)[4], uint16_t *y, const int64_t (&ys)[4], int64_t lo_off,
             const int64_t (&dims)[4]) {
    Dims4 g;
    int64_t total = 1;
    for (int k = 0; k < 4; k++) {
        g.d[k] = dims[k];
        g.xs[k] = xs[k];
        g.ys[k] = ys[k];
        total *= dims[k];
    }
    if (total == 0) return;
    Prof pf(c, "resplit", 0, 8.0 * total);
    k_resplit<<<grid_for(c, total), kThreads, 0, c->stream>>>(x, y, lo_off, g, total);
    WOCR_LAUNCHED(c);
}

void argmax_merge(Ctx *c, const float *pmax, const float *psum, const uint32_t *pidx, int64_t rows, int ntiles,
                  uint32_t *best, float *row_max, float *row_lse) {
    if (rows == 0) return;
    Prof pf(c, "argmax_merge", 0, 12.0 * (double)rows * ntiles);
    k_argmax_merge<<<grid_for(c, rows * 32), kThreads, 0, c->stream>>>(pmax, psum, pidx, rows, ntiles, best,
                                                                       row_max, row_lse);
    WOCR_LAUNCHED(c);
}

void gap(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int hw, int ch, float *y) {
    Prof pf(c, "gap", 0, 4.0 * n * ch * ((double)hw + 1));
    dim3 grid((ch + 31) / 32, n);
    k_gap<<<grid, kThreads, 0, c->stream>>>(x, x_n, x_pix, hw, ch, y);
    WOCR_LAUNCHED(c);
}

void resize_nearest(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch, int oh, int ow,
                    float sy, float sx, float *y, int64_t y_n, int64_t y_pix) {
    Prof pf(c, "resize_nearest", 0, 4.0 * n * ch * ((double)h * w + (double)oh * ow));
    int64_t total = (int64_t)n * oh * ow * ch;
    k_resize_nearest<<<grid_for(c, total), kThreads, 0, c->stream>>>(x, x_n, x_pix, n, h, w, ch, oh, ow, sy, sx, y,
                                                                    y_n, y_pix);
    WOCR_LAUNCHED(c);
}

void copy(Ctx *c, const float *x, float *y, const Strided &s) {
    int64_t total = 1;
    for (int d = 0; d < s.rank; d++) total *= s.dims[d];
    if (total == 0) return;
    Prof pf(c, "copy", 0, 8.0 * total);
    k_copy<<<grid_for(c, total), kThreads, 0, c->stream>>>(x, y, s, total);
    WOCR_LAUNCHED(c);
}

void binary(Ctx *c, int op, const float *a, const float *b, float *y, const Strided &s) {
    int64_t total = 1;
    for (int d = 0; d < s.rank; d++) total *= s.dims[d];
    if (total == 0) return;
    Prof pf(c, "binary", 0, 12.0 * total);
    k_binary<<<grid_for(c, total), kThreads, 0, c->stream>>>(op, a, b, y, s, total);
    WOCR_LAUNCHED(c);
}

void unary(Ctx *c, int op, const float *x, float *y, int64_t n, float alpha, float beta) {
    Prof pf(c, "unary", 0, 8.0 * n);
    if (n == 0) return;
    k_unary<<<grid_for(c, n), kThreads, 0, c->stream>>>(op, x, y, n, alpha, beta);
    WOCR_LAUNCHED(c);
}

void affine(Ctx *c, const float *x, float *y, int64_t n, int C, int64_t cdiv, const float *st) {
    Prof pf(c, "affine", 0, 8.0 * n);
    if (n == 0) return;
    k_affine<<<grid_for(c, n), kThreads, 0, c->stream>>>(x, y, n, C, cdiv, st);
    WOCR_LAUNCHED(c);
}

void reduce_mean(Ctx *c, const float *x, float *y, int64_t outer, int64_t inner) {
    Prof pf(c, "reduce_mean", 0, 4.0 * outer * (inner + 1));
    if (outer == 0) return;
    int64_t blocks = (outer * 32 + kThreads - 1) / kThreads;
    k_reduce_mean<<<(unsigned)blocks, kThreads, 0, c->stream>>>(x, y, outer, inner);
    WOCR_LAUNCHED(c);
}

void layer_norm(Ctx *c, const float *x, float *y, int64_t rows, int len, const float *gb, float eps) {
    Prof pf(c, "layer_norm", 0, 8.0 * rows * len);
    if (rows == 0) return;
    int64_t blocks = (rows * 32 + kThreads - 1) / kThreads;
    k_layer_norm<<<(unsigned)blocks, kThreads, 0, c->stream>>>(x, y, rows, len, gb, eps);
    WOCR_LAUNCHED(c);
}

void softmax(Ctx *c, const float *x, float *y, int64_t rows, int64_t len) {
    Prof pf(c, "softmax", 0, 8.0 * rows * len);
    if (rows == 0) return;
    if (len <= 1024) {
        k_softmax_warp<<<(unsigned)((rows + kSmRowWarps - 1) / kSmRowWarps), kSmRowWarps * 32, 0, c->stream>>>(
            x, y, rows, (int)len);
    } else {
        k_softmax<<<(unsigned)rows, kThreads, 0, c->stream>>>(x, y, rows, len);
    }
    WOCR_LAUNCHED(c);
}

void argmax(Ctx *c, const float *x, int64_t rows, int64_t len, int64_t ld, uint32_t *best, float *row_max,
            float *row_lse, int tie_last) {
    Prof pf(c, "argmax", 0, 4.0 * rows * len);
    if (rows == 0) return;
    int threads = len >= 4096 ? 512 : (len >= 512 ? 256 : 128);
    k_argmax<<<(unsigned)rows, threads, 0, c->stream>>>(x, rows, len, ld, best, row_max, row_lse, tie_last);
    WOCR_LAUNCHED(c);
}

void bmm(Ctx *c, const float *a, const float *bm, float *y, int64_t batch, int m, int kk, int n) {
    Prof pf(c, "bmm", 2.0 * batch * m * kk * n, 4.0 * batch * ((double)m * kk + (double)kk * n + (double)m * n));
    if (batch == 0) return;
    dim3 grid((n + 31) / 32, (m + 31) / 32, (unsigned)batch);
    k_bmm<<<grid, 256, 0, c->stream>>>(a, bm, y, m, kk, n);
    WOCR_LAUNCHED(c);
}

void avgpool_t(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int ch, int h, int w, int kh, int ntot,
               int noff, float *y) {
    Prof pf(c, "avgpool_t", 0, 4.0 * n * w * ch * (h + 1));
    int64_t total = (int64_t)n * w * ch;
    k_avgpool_t<<<grid_for(c, total), kThreads, 0, c->stream>>>(x, x_n, x_pix, n, ch, h, w, kh, ntot, noff, y);
    WOCR_LAUNCHED(c);
}

}  // namespace k
}  // namespace wocr
