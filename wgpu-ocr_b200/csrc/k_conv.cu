// Convolution family on channels-last tensors: implicit-GEMM dense conv / linear / strided
// ConvTranspose (CUDA-core fp32 path), Cin = 1 direct conv with fused MaxPool, depthwise conv,
// general ConvTranspose.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "act.h"
#include "kernels.h"

namespace wocr {
namespace k {

namespace {

constexpr int BM = 128, BN = 64, BK = 16;

// 256 threads; thread (tx, ty) = (tid % 16, tid / 16) owns pixels tx*8..+8 and channels
// ty*4..+4 of the 128 x 64 tile.  A tile is staged k-major so the FMA loop reads it as float4.
// VEC: cin % 8 == 0 and 16-byte aligned rows, so a thread's 8 consecutive k (one tap, 8 input
// channels) load as two float4.
template <bool VEC>
__global__ void __launch_bounds__(256) k_conv_gemm(ConvP p) {
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Bs[BK][BN];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t M = (int64_t)p.n * p.oh * p.ow;
    const int64_t m0 = (int64_t)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;
    const int K = p.kh * p.kw * p.cin;

    // A loader: pixel am of the tile, k slice ak .. ak + 8
    const int am = tid & (BM - 1);
    const int ak = (tid >> 7) * 8;
    const int64_t m = m0 + am;
    const bool mvalid = m < M;
    int ox = 0, oy = 0, nb = 0;
    if (mvalid) {
        ox = (int)(m % p.ow);
        int64_t t = m / p.ow;
        oy = (int)(t % p.oh);
        nb = (int)(t / p.oh);
    }
    const int iy0 = oy * p.sh - p.pt, ix0 = ox * p.sw - p.pl;
    const float *xb = p.x + (int64_t)nb * p.x_n;
    const float *scb = p.insc ? p.insc + (int64_t)nb * p.cin : nullptr;
    // B loader: k row tid / 16, channels (tid % 16) * 4 .. + 4
    const int bk = tid >> 4, bc = (tid & 15) * 4;

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.f;

    for (int k0 = 0; k0 < K; k0 += BK) {
        float av[8];
#pragma unroll
        for (int e = 0; e < 8; e++) av[e] = 0.f;
        if (VEC) {
            int kq = k0 + ak;
            if (mvalid && kq < K) {
                int tap = kq / p.cin, ci = kq - tap * p.cin;
                int ky = tap / p.kw, kx = tap - ky * p.kw;
                int iy = iy0 + ky, ix = ix0 + kx;
                if (iy >= 0 && iy < p.h && ix >= 0 && ix < p.w) {
                    const float4 *src = reinterpret_cast<const float4 *>(xb + ((int64_t)iy * p.w + ix) * p.x_pix + ci);
                    float4 v0 = src[0], v1 = src[1];
                    av[0] = v0.x; av[1] = v0.y; av[2] = v0.z; av[3] = v0.w;
                    av[4] = v1.x; av[5] = v1.y; av[6] = v1.z; av[7] = v1.w;
                    if (scb) {
#pragma unroll
                        for (int e = 0; e < 8; e++) av[e] *= scb[ci + e];
                    }
                }
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                int kq = k0 + ak + e;
                if (mvalid && kq < K) {
                    int tap = kq / p.cin, ci = kq - tap * p.cin;
                    int ky = tap / p.kw, kx = tap - ky * p.kw;
                    int iy = iy0 + ky, ix = ix0 + kx;
                    if (iy >= 0 && iy < p.h && ix >= 0 && ix < p.w) {
                        float v = xb[((int64_t)iy * p.w + ix) * p.x_pix + ci];
                        if (scb) v *= scb[ci];
                        av[e] = v;
                    }
                }
            }
        }
#pragma unroll
        for (int e = 0; e < 8; e++) As[ak + e][am] = av[e];
        {
            float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
            int kq = k0 + bk;
            if (kq < K && n0 + bc < p.ldw) bv = *reinterpret_cast<const float4 *>(p.wt + (int64_t)kq * p.ldw + n0 + bc);
            *reinterpret_cast<float4 *>(&Bs[bk][bc]) = bv;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float4 a0 = *reinterpret_cast<const float4 *>(&As[kk][tx * 8]);
            float4 a1 = *reinterpret_cast<const float4 *>(&As[kk][tx * 8 + 4]);
            float4 b = *reinterpret_cast<const float4 *>(&Bs[kk][ty * 4]);
            float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            float bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] += a[i] * bb[j];
        }
        __syncthreads();
    }

    // epilogue: bias, activation, residual; channels-last stores
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int64_t mm = m0 + tx * 8 + i;
        if (mm >= M) continue;
        int eox = (int)(mm % p.ow);
        int64_t t = mm / p.ow;
        int eoy = (int)(t % p.oh);
        int enb = (int)(t / p.oh);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int col = n0 + ty * 4 + j;
            if (col >= p.cout) continue;
            if (p.scatter) {
                int s = p.scatter;
                int co = col % p.scat_cout, tap = col / p.scat_cout;
                int ky = tap / s, kx = tap % s;
                int yy = eoy * s + ky, xx = eox * s + kx;
                int ow2 = p.ow * s;
                float v = act_f(acc[i][j] + (p.bias ? p.bias[co] : 0.f), p.act);
                p.y[(int64_t)enb * p.y_n + ((int64_t)yy * ow2 + xx) * p.y_pix + co] = v;
            } else {
                float v = act_f(acc[i][j] + (p.bias ? p.bias[col] : 0.f), p.act);
                int64_t pix = (int64_t)eoy * p.ow + eox;
                if (p.res) v += p.res[(int64_t)enb * p.res_n + pix * p.res_pix + col];
                p.y[(int64_t)enb * p.y_n + pix * p.y_pix + col] = v;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// Cin = 1 direct conv: one thread per output pixel (after the fused pool), all channels.
// Split activations (bf16 hi = bf16(v), lo = bf16(v - hi)) as the tap-convolution kernel reads them.
__device__ __forceinline__ void split1(float v, uint16_t &h, uint16_t &l) {
    __nv_bfloat16 hb = __float2bfloat16_rn(v);
    __nv_bfloat16 lb = __float2bfloat16_rn(v - __bfloat162float(hb));
    h = *reinterpret_cast<uint16_t *>(&hb);
    l = *reinterpret_cast<uint16_t *>(&lb);
}

__device__ __forceinline__ void split8v(const float *v, uint4 &hi, uint4 &lo) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint16_t h0, l0, h1, l1;
        split1(v[2 * i], h0, l0);
        split1(v[2 * i + 1], h1, l1);
        hw[i] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        lw[i] = (uint32_t)l0 | ((uint32_t)l1 << 16);
    }
    hi = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    lo = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

__device__ __forceinline__ float unsplit1(const uint16_t *hp, int64_t lo_off) {
    return __uint_as_float((uint32_t)hp[0] << 16) + __uint_as_float((uint32_t)hp[lo_off] << 16);
}

template <int COUT, int SPLIT>
__global__ void k_conv_direct(const float *__restrict__ x, int64_t x_n, int64_t x_pix, int n, int h, int w,
                              const float *__restrict__ wt, const float *__restrict__ bias, int kh, int kw, int pad,
                              int act, int ph, int pw, void *__restrict__ yv, int64_t y_n, int64_t y_pix, int oh,
                              int ow, int vec) {
    __shared__ float ws[7 * 7 * COUT];
    __shared__ float bs[COUT];
    for (int i = threadIdx.x; i < kh * kw * COUT; i += blockDim.x) ws[i] = wt[i];
    for (int i = threadIdx.x; i < COUT; i += blockDim.x) bs[i] = bias[i];
    __syncthreads();
    int64_t total = (int64_t)n * oh * ow;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int ox = (int)(i % ow);
        int oy = (int)((i / ow) % oh);
        int nb = (int)(i / ((int64_t)ow * oh));
        const float *xb = x + nb * x_n;
        float best[COUT];
#pragma unroll
        for (int c = 0; c < COUT; c++) best[c] = -3.4e38f;
        for (int py = 0; py < ph; py++)
            for (int px = 0; px < pw; px++) {
                int cy = oy * ph + py, cx = ox * pw + px;
                float acc[COUT];
#pragma unroll
                for (int c = 0; c < COUT; c++) acc[c] = bs[c];
                for (int ky = 0; ky < kh; ky++) {
                    int iy = cy + ky - pad;
                    if (iy < 0 || iy >= h) continue;
                    for (int kx = 0; kx < kw; kx++) {
                        int ix = cx + kx - pad;
                        if (ix < 0 || ix >= w) continue;
                        float v = xb[((int64_t)iy * w + ix) * x_pix];
                        const float *wr = ws + (ky * kw + kx) * COUT;
#pragma unroll
                        for (int c = 0; c < COUT; c++) acc[c] += v * wr[c];
                    }
                }
                act_n(acc, act);
#pragma unroll
                for (int c = 0; c < COUT; c++) best[c] = fmaxf(best[c], acc[c]);
            }
        const int64_t off = nb * y_n + ((int64_t)oy * ow + ox) * y_pix;
        if (SPLIT) {
            // split activations: bf16 hi parts of the pixel's channels, lo parts y_pix / 2 later
            uint16_t *yo = reinterpret_cast<uint16_t *>(yv) + off;
            if (vec) {
#pragma unroll
                for (int c = 0; c < COUT; c += 8) {
                    uint4 hi, lo;
                    split8v(best + c, hi, lo);
                    *reinterpret_cast<uint4 *>(yo + c) = hi;
                    *reinterpret_cast<uint4 *>(yo + y_pix / 2 + c) = lo;
                }
            } else {
#pragma unroll
                for (int c = 0; c < COUT; c++) split1(best[c], yo[c], yo[y_pix / 2 + c]);
            }
        } else {
            float *yo = reinterpret_cast<float *>(yv) + off;
#pragma unroll
            for (int c = 0; c < COUT; c++) yo[c] = best[c];
        }
    }
}

// 3 x 3, Cin = 1 convolution on 16 x 16 tiles of conv outputs (one per block): the input halo
// in shared memory, weights read 4 output channels at a time; POOL 2 fuses a 2 x 2 MaxPool.
template <int COUT, int SPLIT, int POOL>
__global__ void __launch_bounds__(256) k_conv3_cin1(const float *__restrict__ x, int64_t x_n, int64_t x_pix, int n,
                                                    int h, int w, const float *__restrict__ wt,
                                                    const float *__restrict__ bias, int pad, int act,
                                                    void *__restrict__ yv, int64_t y_n, int64_t y_pix, int oh, int ow,
                                                    int ch, int cw, int tiles_x, int tiles_y, int vec) {
    __shared__ __align__(16) float ws[9 * COUT];
    __shared__ float bs[COUT];
    __shared__ float tile[18][19];
    __shared__ __align__(16) float pooled[POOL == 2 ? 256 * COUT : 1];
    for (int i = threadIdx.x; i < 9 * COUT; i += 256) ws[i] = wt[i];
    for (int i = threadIdx.x; i < COUT; i += 256) bs[i] = bias[i];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    for (int64_t b = blockIdx.x; b < (int64_t)n * tiles_y * tiles_x; b += gridDim.x) {
        const int bx = (int)(b % tiles_x);
        const int64_t r = b / tiles_x;
        const int by = (int)(r % tiles_y), nb = (int)(r / tiles_y);
        const int cy0 = by * 16, cx0 = bx * 16;
        const float *xb = x + nb * x_n;
        __syncthreads();  // the previous tile's readers are done
        for (int i = threadIdx.x; i < 18 * 18; i += 256) {
            const int yy = i / 18, xx = i - (i / 18) * 18;
            const int iy = cy0 + yy - pad, ix = cx0 + xx - pad;
            tile[yy][xx] = iy >= 0 && iy < h && ix >= 0 && ix < w ? xb[((int64_t)iy * w + ix) * x_pix] : 0.f;
        }
        __syncthreads();
        float acc[COUT];
#pragma unroll
        for (int c = 0; c < COUT; c++) acc[c] = bs[c];
#pragma unroll
        for (int ky = 0; ky < 3; ky++)
#pragma unroll
            for (int kx = 0; kx < 3; kx++) {
                const float v = tile[ty + ky][tx + kx];
                const float4 *w4 = reinterpret_cast<const float4 *>(ws + (ky * 3 + kx) * COUT);
#pragma unroll
                for (int c4 = 0; c4 < COUT / 4; c4++) {
                    const float4 q = w4[c4];
                    acc[4 * c4] += v * q.x;
                    acc[4 * c4 + 1] += v * q.y;
                    acc[4 * c4 + 2] += v * q.z;
                    acc[4 * c4 + 3] += v * q.w;
                }
            }
        act_n(acc, act);
        int oy = cy0 + ty, ox = cx0 + tx;
        bool store = oy < ch && ox < cw;
        if (POOL == 2) {
            float4 *ps = reinterpret_cast<float4 *>(pooled + threadIdx.x * COUT);
#pragma unroll
            for (int c4 = 0; c4 < COUT / 4; c4++)
                ps[c4] = make_float4(acc[4 * c4], acc[4 * c4 + 1], acc[4 * c4 + 2], acc[4 * c4 + 3]);
            __syncthreads();
            store = false;
            if (threadIdx.x < 64) {
                const int py = threadIdx.x >> 3, px = threadIdx.x & 7;
                oy = by * 8 + py;
                ox = bx * 8 + px;
                store = oy < oh && ox < ow;
                const float *q0 = pooled + ((2 * py) * 16 + 2 * px) * COUT;
#pragma unroll
                for (int c = 0; c < COUT; c++)
                    acc[c] = fmaxf(fmaxf(q0[c], q0[COUT + c]), fmaxf(q0[16 * COUT + c], q0[17 * COUT + c]));
            }
        }
        if (!store) continue;
        const int64_t off = nb * y_n + ((int64_t)oy * ow + ox) * y_pix;
        if (SPLIT) {
            uint16_t *yo = reinterpret_cast<uint16_t *>(yv) + off;
            if (vec) {
#pragma unroll
                for (int c = 0; c < COUT; c += 8) {
                    uint4 hi, lo;
                    split8v(acc + c, hi, lo);
                    *reinterpret_cast<uint4 *>(yo + c) = hi;
                    *reinterpret_cast<uint4 *>(yo + y_pix / 2 + c) = lo;
                }
            } else {
#pragma unroll
                for (int c = 0; c < COUT; c++) split1(acc[c], yo[c], yo[y_pix / 2 + c]);
            }
        } else {
            float *yo = reinterpret_cast<float *>(yv) + off;
#pragma unroll
            for (int c = 0; c < COUT; c++) yo[c] = acc[c];
        }
    }
}

// Generic-cout direct conv: one thread per (output pixel, channel).
__global__ void k_conv_direct_any(const float *__restrict__ x, int64_t x_n, int64_t x_pix, int n, int h, int w,
                                  const float *__restrict__ wt, const float *__restrict__ bias, int cout, int kh,
                                  int kw, int pad, int act, int ph, int pw, float *__restrict__ y, int64_t y_n,
                                  int64_t y_pix, int oh, int ow) {
    int64_t total = (int64_t)n * oh * ow * cout;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int c = (int)(i % cout);
        int64_t pix = i / cout;
        int ox = (int)(pix % ow);
        int oy = (int)((pix / ow) % oh);
        int nb = (int)(pix / ((int64_t)ow * oh));
        const float *xb = x + nb * x_n;
        float best = -3.4e38f;
        for (int py = 0; py < ph; py++)
            for (int px = 0; px < pw; px++) {
                int cy = oy * ph + py, cx = ox * pw + px;
                float acc = bias[c];
                for (int ky = 0; ky < kh; ky++) {
                    int iy = cy + ky - pad;
                    if (iy < 0 || iy >= h) continue;
                    for (int kx = 0; kx < kw; kx++) {
                        int ix = cx + kx - pad;
                        if (ix < 0 || ix >= w) continue;
                        acc += xb[((int64_t)iy * w + ix) * x_pix] * wt[(ky * kw + kx) * cout + c];
                    }
                }
                best = fmaxf(best, act_f(acc, act));
            }
        y[nb * y_n + ((int64_t)oy * ow + ox) * y_pix + c] = best;
    }
}

// Depthwise: one thread per (output pixel, 4 channels) when c % 4 == 0, else per channel.
template <bool VEC4>
__global__ void k_depthwise(const float *__restrict__ x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch,
                            const float *__restrict__ wt, const float *__restrict__ bias, int kh, int kw, int sh, int sw,
                            int pt, int pl, int oh, int ow, int act, float *__restrict__ y, int64_t y_n, int64_t y_pix) {
    const int cv = VEC4 ? ch / 4 : ch;
    int64_t total = (int64_t)n * oh * ow * cv;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int cq = (int)(i % cv);
        int64_t pix = i / cv;
        int ox = (int)(pix % ow);
        int oy = (int)((pix / ow) % oh);
        int nb = (int)(pix / ((int64_t)ow * oh));
        const float *xb = x + nb * x_n;
        if (VEC4) {
            int c = cq * 4;
            float4 acc = *reinterpret_cast<const float4 *>(bias + c);
            for (int ky = 0; ky < kh; ky++) {
                int iy = oy * sh + ky - pt;
                if (iy < 0 || iy >= h) continue;
                for (int kx = 0; kx < kw; kx++) {
                    int ix = ox * sw + kx - pl;
                    if (ix < 0 || ix >= w) continue;
                    float4 v = *reinterpret_cast<const float4 *>(xb + ((int64_t)iy * w + ix) * x_pix + c);
                    float4 wv = *reinterpret_cast<const float4 *>(wt + (int64_t)(ky * kw + kx) * ch + c);
                    acc.x += v.x * wv.x; acc.y += v.y * wv.y; acc.z += v.z * wv.z; acc.w += v.w * wv.w;
                }
            }
            float4 o = make_float4(act_f(acc.x, act), act_f(acc.y, act), act_f(acc.z, act), act_f(acc.w, act));
            *reinterpret_cast<float4 *>(y + nb * y_n + ((int64_t)oy * ow + ox) * y_pix + c) = o;
        } else {
            int c = cq;
            float acc = bias[c];
            for (int ky = 0; ky < kh; ky++) {
                int iy = oy * sh + ky - pt;
                if (iy < 0 || iy >= h) continue;
                for (int kx = 0; kx < kw; kx++) {
                    int ix = ox * sw + kx - pl;
                    if (ix < 0 || ix >= w) continue;
                    acc += xb[((int64_t)iy * w + ix) * x_pix + c] * wt[(int64_t)(ky * kw + kx) * ch + c];
                }
            }
            y[nb * y_n + ((int64_t)oy * ow + ox) * y_pix + c] = act_f(acc, act);
        }
    }
}

// General ConvTranspose: each output gathers only the taps of its parity (src/gpu.rs:443-456).
__global__ void k_convt_gather(const float *__restrict__ x, int64_t x_n, int64_t x_pix, int n, int h, int w, int cin,
                               const float *__restrict__ wt, const float *__restrict__ bias, int cout, int kh, int kw,
                               int s, int act, float *__restrict__ y, int64_t y_n, int64_t y_pix, int oh, int ow) {
    int64_t total = (int64_t)n * oh * ow * cout;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int co = (int)(i % cout);
        int64_t pix = i / cout;
        int ox = (int)(pix % ow);
        int oy = (int)((pix / ow) % oh);
        int nb = (int)(pix / ((int64_t)ow * oh));
        float acc = bias ? bias[co] : 0.f;
        for (int ky = oy % s; ky < kh && ky <= oy; ky += s) {
            int iy = (oy - ky) / s;
            if (iy >= h) continue;
            for (int kx = ox % s; kx < kw && kx <= ox; kx += s) {
                int ix = (ox - kx) / s;
                if (ix >= w) continue;
                const float *xr = x + nb * x_n + ((int64_t)iy * w + ix) * x_pix;
                for (int ci = 0; ci < cin; ci++) acc += xr[ci] * wt[(((int64_t)ci * cout + co) * kh + ky) * kw + kx];
            }
        }
        y[nb * y_n + ((int64_t)oy * ow + ox) * y_pix + co] = act_f(acc, act);
    }
}


// 1 x 1 convolution with few output channels (< 16, e.g. a detector head): memory-bound, one
// thread per pixel, weights [cin][cout] in shared memory.  The tensor-core tile would be mostly
// empty for such an N.
template <int COUT, bool VEC, bool SPLIT_IN>
__global__ void k_pointwise(const void *__restrict__ xv, int64_t x_n, int64_t x_pix, int64_t hw, int n, int cin,
                            const float *__restrict__ wt, int ldw, const float *__restrict__ bias, int cout, int act,
                            float *__restrict__ y, int64_t y_n, int64_t y_pix) {
    extern __shared__ float ws[];  // [cin][COUT]
    for (int i = threadIdx.x; i < cin * COUT; i += blockDim.x) {
        int ci = i / COUT, co = i % COUT;
        ws[i] = co < cout ? wt[(int64_t)ci * ldw + co] : 0.f;
    }
    __syncthreads();
    const int64_t total = (int64_t)n * hw;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t nb = i / hw, pix = i - nb * hw;
        float acc[COUT];
#pragma unroll
        for (int co = 0; co < COUT; co++) acc[co] = co < cout ? bias[co] : 0.f;
        if (SPLIT_IN) {
            const uint16_t *xp = reinterpret_cast<const uint16_t *>(xv) + nb * x_n + pix * x_pix;
            const int64_t lo = x_pix / 2;
            if (VEC) {
                for (int ci = 0; ci < cin; ci += 8) {
                    uint4 h = __ldg(reinterpret_cast<const uint4 *>(xp + ci));
                    uint4 l = __ldg(reinterpret_cast<const uint4 *>(xp + lo + ci));
                    const uint32_t hw4[4] = {h.x, h.y, h.z, h.w}, lw4[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const uint32_t hb = (hw4[e >> 1] >> ((e & 1) * 16)) & 0xffffu;
                        const uint32_t lb = (lw4[e >> 1] >> ((e & 1) * 16)) & 0xffffu;
                        const float v = __uint_as_float(hb << 16) + __uint_as_float(lb << 16);
                        const float *w0 = ws + (ci + e) * COUT;
#pragma unroll
                        for (int co = 0; co < COUT; co++) acc[co] += v * w0[co];
                    }
                }
            } else {
                for (int ci = 0; ci < cin; ci++) {
                    float v = unsplit1(xp + ci, lo);
#pragma unroll
                    for (int co = 0; co < COUT; co++) acc[co] += v * ws[ci * COUT + co];
                }
            }
        } else if (VEC) {
            const float *xp = reinterpret_cast<const float *>(xv) + nb * x_n + pix * x_pix;
            for (int ci = 0; ci < cin; ci += 4) {
                float4 v = __ldg(reinterpret_cast<const float4 *>(xp + ci));
                const float *w0 = ws + ci * COUT;
#pragma unroll
                for (int co = 0; co < COUT; co++)
                    acc[co] += v.x * w0[co] + v.y * w0[COUT + co] + v.z * w0[2 * COUT + co] + v.w * w0[3 * COUT + co];
            }
        } else {
            const float *xp = reinterpret_cast<const float *>(xv) + nb * x_n + pix * x_pix;
            for (int ci = 0; ci < cin; ci++) {
                float v = xp[ci];
#pragma unroll
                for (int co = 0; co < COUT; co++) acc[co] += v * ws[ci * COUT + co];
            }
        }
        float *yp = y + nb * y_n + pix * y_pix;
        act_n(acc, act);
#pragma unroll
        for (int co = 0; co < COUT; co++)
            if (co < cout) yp[co] = acc[co];
    }
}

inline int grid_for(Ctx *c, int64_t work, int per_block = 256) {
    int64_t g = (work + per_block - 1) / per_block;
    int64_t cap = (int64_t)c->sm_count * 16;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace

void conv_gemm(Ctx *c, const ConvP &p) {
    int64_t M = (int64_t)p.n * p.oh * p.ow;
    if (M == 0 || p.cout == 0) return;
    dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((p.cout + BN - 1) / BN));
    Prof pf(c, p.scatter ? "convt_gemm" : "conv_gemm", 2.0 * (double)M * p.cout * p.kh * p.kw * p.cin,
            4.0 * ((double)p.n * p.h * p.w * p.cin + (double)p.kh * p.kw * p.cin * p.cout + (double)M * p.cout));
    bool vec = (p.cin % 8 == 0) && (p.x_pix % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) &&
               (p.x_n % 4 == 0);
    if (vec) k_conv_gemm<true><<<grid, 256, 0, c->stream>>>(p);
    else k_conv_gemm<false><<<grid, 256, 0, c->stream>>>(p);
    WOCR_LAUNCHED(c);
    c->flops += 2.0 * (double)M * p.cout * p.kh * p.kw * p.cin;
}

// Narrow convolutions: at most 64 output channels and at most kNarrowMacs multiply-adds per
// output pixel.  Their arithmetic intensity is far below the tensor cores' ridge, so they are
// bound by the activations' bytes, and a tensor-core tile (128 pixels x 64 + channels, an
// implicit-GEMM A tile split into bf16 parts) would spend its time on tiles mostly of padding.
// CUDA cores in fp32 instead: a thread per output pixel keeps its output channels in registers;
// the weights [K][CO] sit in shared memory and every read of them is a warp-wide broadcast.  The
// K order (ky, kx, ci) and the epilogue (bias, activation, then the residual) are those of
// k_conv_gemm.
template <int CO, bool VEC, bool VEC4>
__global__ void __launch_bounds__(256) k_conv_narrow(ConvP p) {
    extern __shared__ float ws[];  // [K][CO]
    const int K = p.kh * p.kw * p.cin;
    for (int i = threadIdx.x; i < K * CO; i += blockDim.x) {
        const int k = i / CO, co = i - k * CO;
        ws[i] = co < p.cout ? p.wt[(int64_t)k * p.ldw + co] : 0.f;
    }
    __syncthreads();
    const int64_t M = (int64_t)p.n * p.oh * p.ow;
    for (int64_t m = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; m < M; m += (int64_t)gridDim.x * blockDim.x) {
        const int ox = (int)(m % p.ow);
        const int64_t t = m / p.ow;
        const int oy = (int)(t % p.oh), nb = (int)(t / p.oh);
        float acc[CO];
#pragma unroll
        for (int co = 0; co < CO; co++) acc[co] = 0.f;
        const float *xb = p.x + (int64_t)nb * p.x_n;
        const float *scb = p.insc ? p.insc + (int64_t)nb * p.cin : nullptr;
        for (int ky = 0; ky < p.kh; ky++) {
            const int iy = oy * p.sh - p.pt + ky;
            if (iy < 0 || iy >= p.h) continue;
            for (int kx = 0; kx < p.kw; kx++) {
                const int ix = ox * p.sw - p.pl + kx;
                if (ix < 0 || ix >= p.w) continue;
                const float *xp = xb + ((int64_t)iy * p.w + ix) * p.x_pix;
                const float *wk = ws + (ky * p.kw + kx) * p.cin * CO;
                if (VEC) {
                    for (int ci = 0; ci < p.cin; ci += 4) {
                        float4 v4 = *reinterpret_cast<const float4 *>(xp + ci);
                        float v[4] = {v4.x, v4.y, v4.z, v4.w};
                        if (scb) {
#pragma unroll
                            for (int e = 0; e < 4; e++) v[e] *= scb[ci + e];
                        }
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const float4 *w4 = reinterpret_cast<const float4 *>(wk + (ci + e) * CO);
#pragma unroll
                            for (int q = 0; q < CO / 4; q++) {
                                const float4 w = w4[q];
                                acc[4 * q] += v[e] * w.x;
                                acc[4 * q + 1] += v[e] * w.y;
                                acc[4 * q + 2] += v[e] * w.z;
                                acc[4 * q + 3] += v[e] * w.w;
                            }
                        }
                    }
                } else {
                    for (int ci = 0; ci < p.cin; ci++) {
                        float v = xp[ci];
                        if (scb) v *= scb[ci];
                        const float4 *w4 = reinterpret_cast<const float4 *>(wk + ci * CO);
#pragma unroll
                        for (int q = 0; q < CO / 4; q++) {
                            const float4 w = w4[q];
                            acc[4 * q] += v * w.x;
                            acc[4 * q + 1] += v * w.y;
                            acc[4 * q + 2] += v * w.z;
                            acc[4 * q + 3] += v * w.w;
                        }
                    }
                }
            }
        }
        const int64_t pix = (int64_t)oy * p.ow + ox;
        float *yp = p.y + (int64_t)nb * p.y_n + pix * p.y_pix;
        const float *rp = p.res ? p.res + (int64_t)nb * p.res_n + pix * p.res_pix : nullptr;
#pragma unroll
        for (int co = 0; co < CO; co++) acc[co] += p.bias && co < p.cout ? p.bias[co] : 0.f;
        act_n(acc, p.act);
        if (rp) {
#pragma unroll
            for (int co = 0; co < CO; co++)
                if (co < p.cout) acc[co] += rp[co];
        }
        if (VEC4) {  // whole output pixels of 16-byte aligned float4s
#pragma unroll
            for (int q = 0; q < CO / 4; q++)
                if (4 * q < p.cout)
                    *reinterpret_cast<float4 *>(yp + 4 * q) =
                        make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
        } else {
#pragma unroll
            for (int co = 0; co < CO; co++)
                if (co < p.cout) yp[co] = acc[co];
        }
    }
}

template <int CO>
void launch_narrow(Ctx *c, const ConvP &p, bool vec) {
    const int K = p.kh * p.kw * p.cin;
    const size_t smem = (size_t)K * CO * 4;
    const int64_t M = (int64_t)p.n * p.oh * p.ow;
    // a few blocks per SM, each over many pixels: the weights are staged once per block
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((M + 255) / 256, (int64_t)c->sm_count * 4));
    const bool vec4 = p.cout % 4 == 0 && p.y_pix % 4 == 0 && p.y_n % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(p.y) & 15) == 0;
    if (vec && vec4) k_conv_narrow<CO, true, true><<<grid, 256, smem, c->stream>>>(p);
    else if (vec) k_conv_narrow<CO, true, false><<<grid, 256, smem, c->stream>>>(p);
    else if (vec4) k_conv_narrow<CO, false, true><<<grid, 256, smem, c->stream>>>(p);
    else k_conv_narrow<CO, false, false><<<grid, 256, smem, c->stream>>>(p);
    WOCR_LAUNCHED(c);
}

bool conv_narrow_ok(const ConvP &p) {
    const int K = p.kh * p.kw * p.cin;
    const int co = p.cout <= 16 ? 16 : (p.cout <= 32 ? 32 : 64);  // the instance launch_narrow picks
    return p.scatter == 0 && p.cout > 0 && p.cout <= 64 && (int64_t)K * p.cout <= kNarrowMacs &&
           (int64_t)K * co * 4 <= 48 * 1024;
}

void conv_narrow(Ctx *c, const ConvP &p) {
    const int64_t M = (int64_t)p.n * p.oh * p.ow;
    if (M == 0) return;
    Prof pf(c, "conv_narrow", 2.0 * (double)M * p.cout * p.kh * p.kw * p.cin,
            4.0 * ((double)p.n * p.h * p.w * p.cin + (double)M * p.cout * (p.res ? 2 : 1)));
    const bool vec = (p.cin % 4 == 0) && (p.x_pix % 4 == 0) && (p.x_n % 4 == 0) &&
                     ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0);
    if (p.cout <= 16) launch_narrow<16>(c, p, vec);
    else if (p.cout <= 32) launch_narrow<32>(c, p, vec);
    else launch_narrow<64>(c, p, vec);
    c->flops += 2.0 * (double)M * p.cout * p.kh * p.kw * p.cin;
}

void pointwise(Ctx *c, const void *x, int64_t x_n, int64_t x_pix, int64_t hw, int n, int cin, const float *wt, int ldw,
               const float *bias, int cout, int act, float *y, int64_t y_n, int64_t y_pix, int split_in) {
    const int64_t total = (int64_t)n * hw;
    if (total == 0) return;
    Prof pf(c, "pointwise", 2.0 * (double)total * cin * cout, 4.0 * (double)total * (cin + cout));
    const bool al = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const bool vec = split_in ? (al && cin % 8 == 0 && x_pix % 16 == 0 && x_n % 8 == 0)
                              : (al && cin % 4 == 0 && x_pix % 4 == 0 && x_n % 4 == 0);
    const int grid = grid_for(c, total);
    auto go = [&](auto cout_tag) {
        constexpr int CO = decltype(cout_tag)::value;
        const size_t smem = sizeof(float) * cin * CO;
        if (split_in && vec)
            k_pointwise<CO, true, true><<<grid, 256, smem, c->stream>>>(x, x_n, x_pix, hw, n, cin, wt, ldw, bias, cout,
                                                                         act, y, y_n, y_pix);
        else if (split_in)
            k_pointwise<CO, false, true><<<grid, 256, smem, c->stream>>>(x, x_n, x_pix, hw, n, cin, wt, ldw, bias, cout,
                                                                          act, y, y_n, y_pix);
        else if (vec)
            k_pointwise<CO, true, false><<<grid, 256, smem, c->stream>>>(x, x_n, x_pix, hw, n, cin, wt, ldw, bias, cout,
                                                                          act, y, y_n, y_pix);
        else
            k_pointwise<CO, false, false><<<grid, 256, smem, c->stream>>>(x, x_n, x_pix, hw, n, cin, wt, ldw, bias,
                                                                           cout, act, y, y_n, y_pix);
    };
    if (cout <= 1) go(std::integral_constant<int, 1>());
    else if (cout <= 2) go(std::integral_constant<int, 2>());
    else if (cout <= 4) go(std::integral_constant<int, 4>());
    else if (cout <= 8) go(std::integral_constant<int, 8>());
    else go(std::integral_constant<int, 16>());
    WOCR_LAUNCHED(c);
    c->flops += 2.0 * (double)total * cin * cout;
}

void conv_direct(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, const float *wt,
                 const float *bias, int cout, int kh, int kw, int pad, int act, int ph, int pw, void *yv,
                 int64_t y_n, int64_t y_pix, int oh, int ow, int split_out) {
    int64_t pix = (int64_t)n * oh * ow;
    if (pix == 0) return;
    Prof pf(c, "conv_direct", 2.0 * (double)pix * ph * pw * cout * kh * kw,
            4.0 * ((double)n * h * w + (double)pix * cout));
    if (kh == 3 && kw == 3 && (cout == 16 || cout == 32) && ph == pw && (ph == 1 || ph == 2)) {
        // 16 x 16 conv-output tiles in shared memory
        const int vec = (reinterpret_cast<uintptr_t>(yv) & 15) == 0 && y_pix % 16 == 0 && y_n % 8 == 0;
        const int cch = h + 2 * pad - 2, ccw = w + 2 * pad - 2;  // conv output before the pool
        const int tiles_x = (ccw + 15) / 16, tiles_y = (cch + 15) / 16;
        const int64_t blocks = (int64_t)n * tiles_x * tiles_y;
        const int grid = (int)std::min<int64_t>(blocks, (int64_t)c->sm_count * 8);
        auto go = [&](auto co_tag, auto split_tag, auto pool_tag) {
            constexpr int CO = decltype(co_tag)::value, SP = decltype(split_tag)::value,
                          PL = decltype(pool_tag)::value;
            k_conv3_cin1<CO, SP, PL><<<grid, 256, 0, c->stream>>>(x, x_n, x_pix, n, h, w, wt, bias, pad, act, yv, y_n,
                                                                  y_pix, oh, ow, cch, ccw, tiles_x, tiles_y, vec);
        };
        using I1 = std::integral_constant<int, 1>;
        using I0 = std::integral_constant<int, 0>;
        using I2 = std::integral_constant<int, 2>;
        using C16 = std::integral_constant<int, 16>;
        using C32 = std::integral_constant<int, 32>;
        if (cout == 16) {
            if (ph == 1) split_out ? go(C16(), I1(), I1()) : go(C16(), I0(), I1());
            else split_out ? go(C16(), I1(), I2()) : go(C16(), I0(), I2());
        } else {
            if (ph == 1) split_out ? go(C32(), I1(), I1()) : go(C32(), I0(), I1());
            else split_out ? go(C32(), I1(), I2()) : go(C32(), I0(), I2());
        }
    } else if (kh * kw <= 49 && (cout == 16 || cout == 32)) {
        const int vec = (reinterpret_cast<uintptr_t>(yv) & 15) == 0 && y_pix % 16 == 0 && y_n % 8 == 0;
        auto go = [&](auto co_tag, auto split_tag) {
            constexpr int CO = decltype(co_tag)::value, SP = decltype(split_tag)::value;
            k_conv_direct<CO, SP><<<grid_for(c, pix), 256, 0, c->stream>>>(x, x_n, x_pix, n, h, w, wt, bias, kh, kw,
                                                                           pad, act, ph, pw, yv, y_n, y_pix, oh, ow,
                                                                           vec);
        };
        if (cout == 16 && split_out) go(std::integral_constant<int, 16>(), std::integral_constant<int, 1>());
        else if (cout == 16) go(std::integral_constant<int, 16>(), std::integral_constant<int, 0>());
        else if (split_out) go(std::integral_constant<int, 32>(), std::integral_constant<int, 1>());
        else go(std::integral_constant<int, 32>(), std::integral_constant<int, 0>());
    } else {
        if (split_out) fail(WOCR_ERR_UNSUPPORTED, "split output of a direct conv with " + std::to_string(cout) + " channels");
        float *y = reinterpret_cast<float *>(yv);
        k_conv_direct_any<<<grid_for(c, pix * cout), 256, 0, c->stream>>>(x, x_n, x_pix, n, h, w, wt, bias, cout, kh,
                                                                          kw, pad, act, ph, pw, y, y_n, y_pix, oh, ow);
    }
    WOCR_LAUNCHED(c);
    c->flops += 2.0 * (double)pix * ph * pw * cout * kh * kw;
}

void depthwise(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch, const float *wt,
               const float *bias, int kh, int kw, int sh, int sw, int pt, int pl, int oh, int ow, int act, float *y,
               int64_t y_n, int64_t y_pix) {
    int64_t pix = (int64_t)n * oh * ow;
    if (pix == 0) return;
    Prof pf(c, "depthwise", 2.0 * (double)pix * ch * kh * kw, 4.0 * ch * ((double)n * h * w + (double)pix));
    bool vec = ch % 4 == 0 && x_pix % 4 == 0 && y_pix % 4 == 0 && x_n % 4 == 0 && y_n % 4 == 0 &&
               ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
    if (vec)
        k_depthwise<true><<<grid_for(c, pix * ch / 4), 256, 0, c->stream>>>(x, x_n, x_pix, n, h, w, ch, wt, bias, kh,
                                                                            kw, sh, sw, pt, pl, oh, ow, act, y, y_n, y_pix);
    else
        k_depthwise<false><<<grid_for(c, pix * ch), 256, 0, c->stream>>>(x, x_n, x_pix, n, h, w, ch, wt, bias, kh, kw,
                                                                         sh, sw, pt, pl, oh, ow, act, y, y_n, y_pix);
    WOCR_LAUNCHED(c);
    c->flops += 2.0 * (double)pix * ch * kh * kw;
}

void convt_gather(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int cin, const float *wt,
                  const float *bias, int cout, int kh, int kw, int s, int act, float *y, int64_t y_n, int64_t y_pix,
                  int oh, int ow) {
    int64_t total = (int64_t)n * oh * ow * cout;
    if (total == 0) return;
    Prof pf(c, "convt_gather", 2.0 * (double)n * h * w * cin * cout * kh * kw,
            4.0 * ((double)n * h * w * cin + (double)total));
    k_convt_gather<<<grid_for(c, total), 256, 0, c->stream>>>(x, x_n, x_pix, n, h, w, cin, wt, bias, cout, kh, kw, s,
                                                             act, y, y_n, y_pix, oh, ow);
    WOCR_LAUNCHED(c);
    c->flops += 2.0 * (double)n * h * w * cin * cout * kh * kw;
}

}  // namespace k
}  // namespace wocr
