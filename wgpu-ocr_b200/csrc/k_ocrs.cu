// ocrs recognition line images on the device (ocrs' prepare_recognition_input, called by the
// reference's line_batches at src/bin/ocr-bench.rs:365-408, which runs it on the host): each line
// cut from the device-resident page at its polygon's bounding rectangle, pixels outside the
// polygon BLACK (-0.5), the others the page's grey value, resized to 64 rows by half-pixel
// bilinear interpolation and written straight into its slot of the padded batch the recogniser
// reads (BLACK past the line's width).
//
// A block computes one output row of one line.  The row interpolates two crop rows; two warps
// find where those rows' pixel centres cross the polygon's edges (each edge tested once), so
// a pixel's inside test is the parity of the crossings to its right, as the even-odd rule
// counts them.  Every operation that feeds a value is an explicitly rounded single-precision
// operation in the order the oracle evaluates it (no contraction), so the images are the
// oracle's bit for bit.
#include "kernels.h"

namespace wocr {
namespace k {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxCross = 2048;  // crossings kept per crop row (a line has at most 2048 vertices)

__device__ __forceinline__ float mixr(float a, float b, float t) {
    return __fadd_rn(__fmul_rn(a, __fsub_rn(1.0f, t)), __fmul_rn(b, t));
}

__device__ __forceinline__ float grey_at(const uint8_t *page, int pw, int x, int y) {
    const uint8_t *p = page + ((int64_t)y * pw + x) * 3;
    return __fadd_rn(__fadd_rn(__fadd_rn(-0.5f, __fmul_rn((float)p[0], 0.299f / 255.0f)),
                               __fmul_rn((float)p[1], 0.587f / 255.0f)),
                     __fmul_rn((float)p[2], 0.114f / 255.0f));
}

// The x coordinates where the horizontal line y = cy crosses the polygon's edges (edge k runs from
// vertex k - 1 to vertex k; the crossing is computed from vertex k, as the oracle computes it).
__device__ void row_crossings(const int2 *v, int nv, float cy, float *xs, int *count) {
    const int lane = threadIdx.x & 31;
    int base = 0;
    for (int k0 = 0; k0 < nv; k0 += 32) {
        const int k = k0 + lane;
        bool hit = false;
        float xc = 0.f;
        if (k < nv) {
            const int2 a = v[k], b = v[k == 0 ? nv - 1 : k - 1];
            const float ya = (float)a.y, yb = (float)b.y;
            if ((ya > cy) != (yb > cy)) {
                hit = true;
                xc = __fadd_rn((float)a.x,
                               __fdiv_rn(__fmul_rn(__fsub_rn(cy, ya), (float)(b.x - a.x)), __fsub_rn(yb, ya)));
            }
        }
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        if (hit) {
            const int at = base + __popc(m & ((1u << lane) - 1u));
            if (at < kMaxCross) xs[at] = xc;
        }
        base += __popc(m);
    }
    if (lane == 0) *count = base < kMaxCross ? base : kMaxCross;
}

__device__ __forceinline__ bool inside(const float *xs, int n, float cx) {
    int c = 0;
    for (int i = 0; i < n; i++) c += cx < xs[i];
    return c & 1;
}

__global__ void __launch_bounds__(kThreads) k_ocrs_lines(const OcrsLine *__restrict__ lines, const int2 *__restrict__ verts,
                                                         float *__restrict__ out) {
    __shared__ float xs[2][kMaxCross];
    __shared__ int nx[2];
    const OcrsLine L = lines[blockIdx.y];
    const int oy = blockIdx.x;
    const float sy = __fdiv_rn((float)L.ch, 64.0f), sx = __fdiv_rn((float)L.cw, (float)L.W);
    float iy = __fsub_rn(__fmul_rn(sy, __fadd_rn((float)oy, 0.5f)), 0.5f);
    iy = fminf(fmaxf(iy, 0.f), __fsub_rn((float)L.ch, 1.f));
    const int y1 = (int)iy, y2 = min(y1 + 1, L.ch - 1);
    const float wy = __fsub_rn(iy, (float)y1);
    const int warp = threadIdx.x >> 5;
    if (warp < 2) {
        const int gy = L.t + (warp ? y2 : y1);
        row_crossings(verts + L.v0, L.nv, __fadd_rn((float)gy, 0.5f), xs[warp], &nx[warp]);
    }
    __syncthreads();
    float *row = out + L.off + (int64_t)oy * L.bw;
    const int gy1 = L.t + y1, gy2 = L.t + y2;
    for (int ox = threadIdx.x; ox < L.bw; ox += kThreads) {
        float v = -0.5f;
        if (ox < L.W) {
            float ix = __fsub_rn(__fmul_rn(sx, __fadd_rn((float)ox, 0.5f)), 0.5f);
            ix = fminf(fmaxf(ix, 0.f), __fsub_rn((float)L.cw, 1.f));
            const int x1 = (int)ix, x2 = min(x1 + 1, L.cw - 1);
            const float wx = __fsub_rn(ix, (float)x1);
            const int gx1 = L.l + x1, gx2 = L.l + x2;
            const float cx1 = __fadd_rn((float)gx1, 0.5f), cx2 = __fadd_rn((float)gx2, 0.5f);
            const float a = inside(xs[0], nx[0], cx1) ? grey_at(L.page, L.pw, gx1, gy1) : -0.5f;
            const float b = inside(xs[0], nx[0], cx2) ? grey_at(L.page, L.pw, gx2, gy1) : -0.5f;
            const float c = inside(xs[1], nx[1], cx1) ? grey_at(L.page, L.pw, gx1, gy2) : -0.5f;
            const float d = inside(xs[1], nx[1], cx2) ? grey_at(L.page, L.pw, gx2, gy2) : -0.5f;
            v = mixr(mixr(a, b, wx), mixr(c, d, wx), wy);
        }
        row[ox] = v;
    }
}

}  // namespace

void ocrs_lines(Ctx *c, const OcrsLine *lines, int n, const int2 *verts, float *out, double bytes) {
    if (n <= 0) return;
    Prof pf(c, "ocrs_lines", 0, bytes);
    k_ocrs_lines<<<dim3(64, (unsigned)n), kThreads, 0, c->stream>>>(lines, verts, out);
    WOCR_LAUNCHED(c);
}

}  // namespace k
}  // namespace wocr
