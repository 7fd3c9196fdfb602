// Recognition line extraction on the device: PP-OCR lines cut from a device-resident RGB page,
// resized to height 48 with the Triangle filter of the `image` crate's imageops::resize and
// normalised to [-1, 1], written straight into the padded batch layout the recogniser reads
// (src/ppocr.rs:39-78, src/bin/ocr-bench.rs:312-345).  This replaces the host crop/resize and
// the upload of the line batches.
//
// Resampling (image =0.25.10, separable): per axis ratio = in / out, s = max(ratio, 1), the taps
// of output o are i in [clamp(floor(c - s), 0, in - 1), clamp(ceil(c + s), left + 1, in)) with
// c = (o + 0.5) ratio, weights tri((i - c + 0.5) / s) normalised by their sum.  A vertical pass
// makes an f32 image, a horizontal pass clamps to [0, 255] and rounds to u8.  A thread computes
// one output pixel: for each horizontal tap it forms that column's vertical sum, then the
// horizontal sum, in the same order and with the same single roundings (no contraction) as the
// two passes, so the u8 values are those of the two-pass resize without its intermediate image.
#include "kernels.h"

namespace wocr {
namespace k {

namespace {

__device__ __forceinline__ float tri(float x) {
    x = fabsf(x);
    return x < 1.f ? 1.f - x : 0.f;
}

// taps of output coordinate o: first index and count; weights are tri(...) / sum
struct Taps {
    int left, n;
    float center, sratio, sum;
};

__device__ __forceinline__ Taps taps(int in, int out, int o) {
    Taps t;
    const float ratio = __fdiv_rn((float)in, (float)out);
    t.sratio = ratio < 1.f ? 1.f : ratio;
    const float support = t.sratio;
    float c = __fmul_rn(__fadd_rn((float)o, 0.5f), ratio);
    long long l = (long long)floorf(__fsub_rn(c, support));
    l = l < 0 ? 0 : (l > in - 1 ? in - 1 : l);
    long long r = (long long)ceilf(__fadd_rn(c, support));
    r = r < l + 1 ? l + 1 : (r > in ? in : r);
    t.center = __fsub_rn(c, 0.5f);
    t.left = (int)l;
    t.n = (int)(r - l);
    float sum = 0.f;
    for (int k = 0; k < t.n; k++) sum = __fadd_rn(sum, tri(__fdiv_rn(__fsub_rn((float)(t.left + k), t.center), t.sratio)));
    t.sum = sum;
    return t;
}

__device__ __forceinline__ float weight(const Taps &t, int k) {
    return __fdiv_rn(tri(__fdiv_rn(__fsub_rn((float)(t.left + k), t.center), t.sratio)), t.sum);
}

constexpr int kRowTaps = 16;  // vertical taps per row kept in shared memory (more: computed per use)
constexpr int kMaxXTaps = 8;  // horizontal taps kept in registers (more: computed per use)

// A block: 128 output columns of one line, all 48 rows.  The rows' vertical taps are computed
// once per block (thread y: row y, its sum in order, then its weights), each thread's horizontal
// taps once per thread.
__global__ void __launch_bounds__(128) k_pp_lines(const uint8_t *__restrict__ rgb, int w, int h,
                                                  const PpLine *__restrict__ lines, float *__restrict__ out) {
    __shared__ Taps ty_s[48];
    __shared__ float wy_s[48][kRowTaps];
    const PpLine L = lines[blockIdx.y];
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    if (blockIdx.x * blockDim.x >= L.width) return;  // the whole block is past this line's batch width
    if (threadIdx.x < 48) {
        const Taps t = taps(L.ch, 48, threadIdx.x);
        ty_s[threadIdx.x] = t;
        for (int k = 0; k < t.n && k < kRowTaps; k++) wy_s[threadIdx.x][k] = weight(t, k);
    }
    __syncthreads();
    if (x >= L.width) return;
    float *o = out + L.off;
    const int64_t plane = (int64_t)48 * L.width;
    if (x >= L.ow) {
        for (int y = 0; y < 48; y++)
            for (int c = 0; c < 3; c++) o[c * plane + (int64_t)y * L.width + x] = 0.f;
        return;
    }
    const int64_t total = (int64_t)w * h * 3;
    const Taps tx = taps(L.cw, L.ow, x);
    float wxr[kMaxXTaps];
#pragma unroll
    for (int k = 0; k < kMaxXTaps; k++) wxr[k] = k < tx.n ? weight(tx, k) : 0.f;
    for (int y = 0; y < 48; y++) {
        const Taps ty = ty_s[y];
        float acc[3] = {0.f, 0.f, 0.f};
        for (int j = 0; j < tx.n; j++) {
            float wx = 0.f;
#pragma unroll
            for (int k = 0; k < kMaxXTaps; k++)
                if (k == j) wx = wxr[k];
            if (j >= kMaxXTaps) wx = weight(tx, j);
            float v[3] = {0.f, 0.f, 0.f};
            for (int i = 0; i < ty.n; i++) {
                const float wy = i < kRowTaps ? wy_s[y][i] : weight(ty, i);
                // crop row: cw * 3 bytes at ((top + row) * w + left) * 3, zeros when they leave the page
                const int64_t row = ((int64_t)(L.t + ty.left + i) * w + L.l) * 3;
                const bool in = row + (int64_t)L.cw * 3 <= total;
                const uint8_t *p = rgb + row + (int64_t)(tx.left + j) * 3;
#pragma unroll
                for (int c = 0; c < 3; c++) v[c] = __fadd_rn(v[c], __fmul_rn(in ? (float)p[c] : 0.f, wy));
            }
#pragma unroll
            for (int c = 0; c < 3; c++) acc[c] = __fadd_rn(acc[c], __fmul_rn(v[c], wx));
        }
#pragma unroll
        for (int c = 0; c < 3; c++) {
            const float a = acc[c] < 0.f ? 0.f : (acc[c] > 255.f ? 255.f : acc[c]);
            const float q = roundf(a);
            o[c * plane + (int64_t)y * L.width + x] = __fdiv_rn(__fsub_rn(__fdiv_rn(q, 255.f), 0.5f), 0.5f);
        }
    }
}

// Tall crops (many vertical taps: a downscale of 8 or more) in two passes, as the `image` crate
// runs them: the vertical pass into an f32 image [48][cw][3] per line (a thread per crop column
// and output row), then the horizontal pass (a thread per output pixel).  The sums are the
// one-pass kernel's, in the same order, so the values are identical; the work is linear in the
// taps of each axis instead of their product, and spread over the whole crop width.
constexpr int kTallTaps = 1024;  // vertical weights kept in shared memory (more: computed per use)

__global__ void __launch_bounds__(128) k_pp_vert(const uint8_t *__restrict__ rgb, int w, int h,
                                                 const PpLine *__restrict__ lines, const int64_t *__restrict__ tmp_off,
                                                 float *__restrict__ tmp) {
    __shared__ Taps ty_s;
    __shared__ float wy_s[kTallTaps];
    const PpLine L = lines[blockIdx.z];
    const int y = blockIdx.y, col = blockIdx.x * blockDim.x + threadIdx.x;
    if (blockIdx.x * blockDim.x >= L.cw) return;  // the whole block is past this crop's width
    if (threadIdx.x == 0) ty_s = taps(L.ch, 48, y);
    __syncthreads();
    const Taps ty = ty_s;
    for (int i = threadIdx.x; i < ty.n && i < kTallTaps; i += blockDim.x) wy_s[i] = weight(ty, i);
    __syncthreads();
    if (col >= L.cw) return;
    const int64_t total = (int64_t)w * h * 3;
    float v[3] = {0.f, 0.f, 0.f};
    for (int i = 0; i < ty.n; i++) {
        const float wy = i < kTallTaps ? wy_s[i] : weight(ty, i);
        // crop row: cw * 3 bytes at ((top + row) * w + left) * 3, zeros when they leave the page
        const int64_t row = ((int64_t)(L.t + ty.left + i) * w + L.l) * 3;
        const bool in = row + (int64_t)L.cw * 3 <= total;
        const uint8_t *p = rgb + row + (int64_t)col * 3;
#pragma unroll
        for (int c = 0; c < 3; c++) v[c] = __fadd_rn(v[c], __fmul_rn(in ? (float)p[c] : 0.f, wy));
    }
    float *t = tmp + tmp_off[blockIdx.z] + ((int64_t)y * L.cw + col) * 3;
#pragma unroll
    for (int c = 0; c < 3; c++) t[c] = v[c];
}

__global__ void __launch_bounds__(128) k_pp_horz(const PpLine *__restrict__ lines, const int64_t *__restrict__ tmp_off,
                                                 const float *__restrict__ tmp, float *__restrict__ out) {
    const PpLine L = lines[blockIdx.z];
    const int y = blockIdx.y, x = blockIdx.x * blockDim.x + threadIdx.x;
    if (x >= L.width) return;
    float *o = out + L.off;
    const int64_t plane = (int64_t)48 * L.width;
    if (x >= L.ow) {
        for (int c = 0; c < 3; c++) o[c * plane + (int64_t)y * L.width + x] = 0.f;
        return;
    }
    const Taps tx = taps(L.cw, L.ow, x);
    const float *t = tmp + tmp_off[blockIdx.z] + (int64_t)y * L.cw * 3;
    float acc[3] = {0.f, 0.f, 0.f};
    for (int j = 0; j < tx.n; j++) {
        const float wx = weight(tx, j);
        const float *v = t + (int64_t)(tx.left + j) * 3;
#pragma unroll
        for (int c = 0; c < 3; c++) acc[c] = __fadd_rn(acc[c], __fmul_rn(v[c], wx));
    }
#pragma unroll
    for (int c = 0; c < 3; c++) {
        const float a = acc[c] < 0.f ? 0.f : (acc[c] > 255.f ? 255.f : acc[c]);
        const float q = roundf(a);
        o[c * plane + (int64_t)y * L.width + x] = __fdiv_rn(__fsub_rn(__fdiv_rn(q, 255.f), 0.5f), 0.5f);
    }
}

}  // namespace

void pp_lines(Ctx *c, const uint8_t *rgb, int w, int h, const PpLine *lines, int n, int max_width, float *out,
              double bytes) {
    if (n <= 0) return;
    Prof pf(c, "pp_lines", 0, bytes);
    dim3 grid((unsigned)((max_width + 127) / 128), (unsigned)n);
    k_pp_lines<<<grid, 128, 0, c->stream>>>(rgb, w, h, lines, out);
    WOCR_LAUNCHED(c);
}

void pp_lines_tall(Ctx *c, const uint8_t *rgb, int w, int h, const PpLine *lines, int n, int max_cw, int max_width,
                   const int64_t *tmp_off, float *tmp, float *out, double bytes) {
    if (n <= 0) return;
    Prof pf(c, "pp_lines_tall", 0, bytes);
    k_pp_vert<<<dim3((unsigned)((max_cw + 127) / 128), 48, (unsigned)n), 128, 0, c->stream>>>(rgb, w, h, lines, tmp_off,
                                                                                              tmp);
    WOCR_LAUNCHED(c);
    k_pp_horz<<<dim3((unsigned)((max_width + 127) / 128), 48, (unsigned)n), 128, 0, c->stream>>>(lines, tmp_off, tmp,
                                                                                                 out);
    WOCR_LAUNCHED(c);
}

}  // namespace k
}  // namespace wocr
