// DB post-processing on the device (src/ppdet.rs:63-92): the detector's probability map
// thresholded into a bit mask for the host's contour search, and the mean probability inside
// each box the host found (`score`), so that only the bits and one float per box cross PCIe
// instead of the probability map.
#include "kernels.h"

namespace wocr {
namespace k {

namespace {

// One warp makes 32 consecutive words of a row: lane b thresholds pixel 32 word + b, a ballot
// forms the word, lane j keeps word j (bit b of word j = pixel 32 j + b).
__global__ void k_db_mask(const float *__restrict__ prob, int w, int h, int words, float thr,
                          uint32_t *__restrict__ bits) {
    const int y = blockIdx.y, lane = threadIdx.x & 31;
    const int wd0 = (blockIdx.x * blockDim.x + threadIdx.x) / 32 * 32;
    if (wd0 >= words) return;
    const float *row = prob + (int64_t)y * w;
    uint32_t mine = 0;
    const int nw = min(32, words - wd0);
    for (int j = 0; j < nw; j++) {
        const int x = (wd0 + j) * 32 + lane;
        const uint32_t word = __ballot_sync(0xffffffffu, x < w && row[x] > thr);
        if (lane == j) mine = word;
    }
    if (lane < nw) bits[(int64_t)y * words + wd0 + lane] = mine;
}

// `score` of src/ppdet.rs:63-83 with the reference's order of additions (a sequential f32 sum
// over the rows, then the columns, of the pixels inside the box), so the result is the
// reference's to the bit.  A warp per box walks the box's bounding rectangle in rounds of 8 x 32
// pixels (row by row, left to right): the lanes test and load a round (8 loads in flight per
// lane) and stage it in shared memory, lane 0 adds the inside values in column order.  The next
// round's loads are issued before lane 0's chain of adds, so they arrive while it runs.  The
// inside test alone decides which pixels count.
constexpr int kDbWarps = 8, kDbChunks = 8, kDbRound = kDbChunks * 32;

struct DbRound {
    float v[kDbChunks];
    uint32_t m[kDbChunks];
};

// round r of box b: row y0 + r / per_row, columns from x0 + (r % per_row) * kDbRound
__device__ __forceinline__ void db_load(const float *prob, int w, const DbBox &b, int per_row, int r, int lane,
                                        DbRound &o) {
    const int y = b.y0 + r / per_row, xs = b.x0 + (r % per_row) * kDbRound;
    const float dy = __fsub_rn((float)y, b.cy);
    const float *row = prob + b.map + (int64_t)y * w;
#pragma unroll
    for (int q = 0; q < kDbChunks; q++) {
        const int x = xs + q * 32 + lane;
        bool in = false;
        o.v[q] = 0.f;
        if (x <= b.x1) {
            const float dx = __fsub_rn((float)x, b.cx);
            const float along = __fadd_rn(__fmul_rn(dx, b.ux), __fmul_rn(dy, b.uy));
            const float across = __fadd_rn(__fmul_rn(dx, -b.uy), __fmul_rn(dy, b.ux));
            in = fabsf(along) <= b.hh && fabsf(across) <= b.hw;
            if (in) o.v[q] = row[x];
        }
        o.m[q] = __ballot_sync(0xffffffffu, in);
    }
}

__global__ void __launch_bounds__(kDbWarps * 32) k_db_scores(const float *__restrict__ prob, int w, int h,
                                                             const DbBox *__restrict__ boxes, int n,
                                                             float *__restrict__ scores) {
    __shared__ float stage[kDbWarps][kDbRound];
    const int wi = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int k = blockIdx.x * kDbWarps + wi;
    if (k >= n) return;
    const DbBox b = boxes[k];
    float sum = 0.f;
    int64_t cnt = 0;
    const int per_row = b.x1 >= b.x0 ? (b.x1 - b.x0) / kDbRound + 1 : 0;
    const int rounds = b.y1 >= b.y0 ? per_row * (b.y1 - b.y0 + 1) : 0;
    DbRound cur;
    if (rounds > 0) db_load(prob, w, b, per_row, 0, lane, cur);
    for (int r = 0; r < rounds; r++) {
        bool any = false;
#pragma unroll
        for (int q = 0; q < kDbChunks; q++) any |= cur.m[q] != 0u;
        if (any) {
#pragma unroll
            for (int q = 0; q < kDbChunks; q++) stage[wi][q * 32 + lane] = cur.v[q];
        }
        const DbRound now = cur;
        if (r + 1 < rounds) db_load(prob, w, b, per_row, r + 1, lane, cur);  // in flight during the adds
        if (!any) continue;
        __syncwarp();
        if (lane == 0) {
#pragma unroll
            for (int q = 0; q < kDbChunks; q++) {
                const uint32_t mq = now.m[q];
                if (mq == 0u) continue;
                float t[32];
#pragma unroll
                for (int j = 0; j < 32; j++) t[j] = stage[wi][q * 32 + j];
                if (mq == 0xffffffffu) {  // all 32 inside: a plain chain of adds
#pragma unroll
                    for (int j = 0; j < 32; j++) sum = __fadd_rn(sum, t[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if ((mq >> j) & 1u) sum = __fadd_rn(sum, t[j]);
                }
                cnt += __popc(mq);
            }
        }
        __syncwarp();
    }
    if (lane == 0) scores[k] = cnt == 0 ? 0.f : __fdiv_rn(sum, (float)cnt);
}

// Per box, the inside pixels' count, their sum in double and the sum of their magnitudes, in
// any order (a block per box over its bounding rectangle, the same inside test as above): enough
// to bound the ordered f32 score without forming it.
constexpr int kDbBoundT = 256;

constexpr int kDbBoundRows = 8;  // box rows per block (blockIdx.y picks the slice)

__global__ void __launch_bounds__(kDbBoundT) k_db_bounds(const float *__restrict__ prob, int w,
                                                         const DbBox *__restrict__ boxes, double *__restrict__ sums,
                                                         long long *__restrict__ counts) {
    __shared__ double s_s[kDbBoundT / 32], s_a[kDbBoundT / 32];
    __shared__ long long s_c[kDbBoundT / 32];
    const DbBox b = boxes[blockIdx.x];
    const int ya = b.y0 + (int)blockIdx.y * kDbBoundRows, yb = min(b.y1, ya + kDbBoundRows - 1);
    if (ya > b.y1 || b.x1 < b.x0) return;  // past this box (the grid covers the tallest box)
    double sum = 0.0, mag = 0.0;
    long long cnt = 0;
    {
        // a warp per row, lanes along it (coalesced)
        for (int y = ya + (int)(threadIdx.x >> 5); y <= yb; y += kDbBoundT / 32) {
            const float dy = __fsub_rn((float)y, b.cy);
            const float *row = prob + b.map + (int64_t)y * w;
            for (int x = b.x0 + (int)(threadIdx.x & 31); x <= b.x1; x += 32) {
                const float dx = __fsub_rn((float)x, b.cx);
                const float along = __fadd_rn(__fmul_rn(dx, b.ux), __fmul_rn(dy, b.uy));
                const float across = __fadd_rn(__fmul_rn(dx, -b.uy), __fmul_rn(dy, b.ux));
                if (fabsf(along) <= b.hh && fabsf(across) <= b.hw) {
                    const double v = (double)row[x];
                    sum += v;
                    mag += fabs(v);
                    cnt++;
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
        mag += __shfl_xor_sync(0xffffffffu, mag, o);
        cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    }
    const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
    if (lane == 0) {
        s_s[wi] = sum;
        s_a[wi] = mag;
        s_c[wi] = cnt;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < kDbBoundT / 32; i++) {
            sum += s_s[i];
            mag += s_a[i];
            cnt += s_c[i];
        }
        // slices of one box add up in any order: the bound on the ordered sum allows for that
        atomicAdd(&sums[2 * blockIdx.x], sum);
        atomicAdd(&sums[2 * blockIdx.x + 1], mag);
        atomicAdd(reinterpret_cast<unsigned long long *>(&counts[blockIdx.x]), (unsigned long long)cnt);
    }
}

}  // namespace

void db_bounds(Ctx *c, const float *prob, int w, const DbBox *boxes, int n, int max_rows, double *sums,
               long long *counts) {
    if (n <= 0) return;
    Prof pf(c, "db_bounds", 0, 0);
    WOCR_CUDA(cudaMemsetAsync(sums, 0, (size_t)n * 16, c->stream));
    WOCR_CUDA(cudaMemsetAsync(counts, 0, (size_t)n * 8, c->stream));
    const dim3 grid((unsigned)n, (unsigned)std::max(1, (max_rows + kDbBoundRows - 1) / kDbBoundRows));
    k_db_bounds<<<grid, kDbBoundT, 0, c->stream>>>(prob, w, boxes, sums, counts);
    WOCR_LAUNCHED(c);
}

void db_mask(Ctx *c, const float *prob, int w, int h, float thr, uint32_t *bits) {
    const int words = (w + 31) / 32;
    Prof pf(c, "db_mask", 0, (double)w * h * 4 + (double)words * h * 4);
    dim3 grid((unsigned)((((words + 31) / 32) * 32 + 127) / 128), (unsigned)h);
    k_db_mask<<<grid, 128, 0, c->stream>>>(prob, w, h, words, thr, bits);
    WOCR_LAUNCHED(c);
}

void db_scores(Ctx *c, const float *prob, int w, int h, const DbBox *boxes, int n, float *scores) {
    if (n <= 0) return;
    Prof pf(c, "db_scores", 0, 0);
    k_db_scores<<<(n + kDbWarps - 1) / kDbWarps, kDbWarps * 32, 0, c->stream>>>(prob, w, h, boxes, n, scores);
    WOCR_LAUNCHED(c);
}

}  // namespace k
}  // namespace wocr
