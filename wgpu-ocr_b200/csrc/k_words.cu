// Word rectangles of detection masks on the device: `word_rects` (src/bin/ocr-bench.rs:38-60),
// i.e. rten-imageproc's find_contours(mask, External), simplify_polygon(2), min_area_rect, then
// resize by the expand distances and an area filter, for a batch of page masks that never
// leave HBM.
//
// The raster scan of Suzuki & Abe's border following is sequential; the same contours come
// from a parallel labelling instead:
//   1. every row of the bit mask is cut into runs of equal pixels (a warp per row);
//   2. a union-find over the runs joins 8-connected foreground runs and 4-connected background
//      runs of adjacent rows, and every background run on the page's edge with the page's frame
//      node.  Union by smaller index makes a component's root its first run in raster order, so
//      the root run starts at the pixel where the raster scan would meet the component;
//   3. a foreground component is external (its outer border's parent is the frame) exactly when
//      the background left of that pixel belongs to the frame's component (or the pixel is in
//      column 0);
//   4. one warp per external component follows its outer border from that pixel with
//      Algorithm 1's steps (3.1)-(3.5) (count, then write); a block per component then runs
//      Douglas-Peucker, the convex hull and the minimum-area rectangle on its points.
// Every floating-point step uses the round-to-nearest intrinsics in the order of the C
// restatement, so the rectangles are bit-identical to it.
#include "kernels.h"

namespace wocr {
namespace k {

namespace {

// (dx + 1) and (dy + 1) of the 8 neighbours, 2 bits each, clockwise on the screen (y down) from
// the left neighbour: left, up-left, up, up-right, right, down-right, down, down-left.
constexpr uint32_t kNbX = 6800, kNbY = 43265;
__device__ __forceinline__ int nb_dx(int d) { return (int)((kNbX >> (2 * d)) & 3u) - 1; }
__device__ __forceinline__ int nb_dy(int d) { return (int)((kNbY >> (2 * d)) & 3u) - 1; }

// transitions between pixel x - 1 and x for the 32 pixels of word j (bit b = x = 32 j + b),
// none at x = 0 or at x >= w
__device__ __forceinline__ uint32_t row_edges(const uint32_t *row, int j, int w) {
    const uint32_t cur = row[j], prev = j ? row[j - 1] : 0u;
    uint32_t d = cur ^ ((cur << 1) | (prev >> 31));
    if (j == 0) d &= ~1u;
    const int valid = w - 32 * j;
    if (valid < 32) d &= (1u << valid) - 1u;
    return d;
}

// ---- scans ---------------------------------------------------------------------------------

constexpr int kScanT = 1024, kScanItems = 4, kScanBlock = kScanT * kScanItems;

// exclusive scan of each 4096-item block (in place allowed); the block's total to sums[block]
__global__ void __launch_bounds__(kScanT) k_scan_blocks(const int *in, int n, int *out, int *sums) {
    __shared__ int ws[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t base = (int64_t)blockIdx.x * kScanBlock + threadIdx.x * kScanItems;
    int v[kScanItems], s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; i++) {
        v[i] = base + i < n ? in[base + i] : 0;
        s += v[i];
    }
    int x = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) ws[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int t = ws[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        ws[lane] = t;
    }
    __syncthreads();
    int pre = x - s + (warp ? ws[warp - 1] : 0);
#pragma unroll
    for (int i = 0; i < kScanItems; i++) {
        if (base + i < n) out[base + i] = pre;
        pre += v[i];
    }
    if (threadIdx.x == kScanT - 1) sums[blockIdx.x] = pre;
}

__global__ void __launch_bounds__(kScanT) k_scan_add(int *out, int n, const int *sums) {
    const int64_t base = (int64_t)blockIdx.x * kScanBlock + threadIdx.x * kScanItems;
    const int add = sums[blockIdx.x];
#pragma unroll
    for (int i = 0; i < kScanItems; i++)
        if (base + i < n) out[base + i] += add;
}

// ---- runs ----------------------------------------------------------------------------------

constexpr int kRowWarps = 8;

// runs per row = transitions + 1 (a warp per row)
__global__ void __launch_bounds__(kRowWarps * 32) k_run_count(const uint32_t *__restrict__ mask, int words, int w,
                                                              int rows, int *__restrict__ cnt) {
    const int row = blockIdx.x * kRowWarps + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (row >= rows) return;
    const uint32_t *m = mask + (int64_t)row * words;
    int t = 0;
    for (int j = lane; j < words; j += 32) t += __popc(row_edges(m, j, w));
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) cnt[row] = t + 1;
}

// run starts (x), colours and rows; run 0 of a row starts at x = 0
__global__ void __launch_bounds__(kRowWarps * 32) k_run_write(const uint32_t *__restrict__ mask, int words, int w,
                                                              int rows, const int *__restrict__ off,
                                                              int *__restrict__ run_x, uint8_t *__restrict__ run_c,
                                                              int *__restrict__ run_row) {
    const int row = blockIdx.x * kRowWarps + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (row >= rows) return;
    const uint32_t *m = mask + (int64_t)row * words;
    const int o = off[row];
    if (lane == 0) {
        run_x[o] = 0;
        run_c[o] = (uint8_t)(m[0] & 1u);
        run_row[o] = row;
    }
    int done = 1;
    for (int j0 = 0; j0 < words; j0 += 32) {
        const int j = j0 + lane;
        const uint32_t d = j < words ? row_edges(m, j, w) : 0u;
        const uint32_t cur = j < words ? m[j] : 0u;
        const int c = __popc(d);
        int x = c;
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, s);
            if (lane >= s) x += y;
        }
        int k = o + done + x - c;
        for (uint32_t b = d; b; b &= b - 1, k++) {
            const int bit = __ffs(b) - 1;
            run_x[k] = 32 * j + bit;
            run_c[k] = (uint8_t)((cur >> bit) & 1u);
            run_row[k] = row;
        }
        done += __shfl_sync(0xffffffffu, x, 31);
    }
}

// ---- union-find over runs (node p < pages: page p's frame; node pages + r: run r) ------------

__device__ __forceinline__ int uf_find(int *P, int x) {
    for (;;) {
        const int p = __ldcg(P + x);
        if (p == x) return x;
        const int g = __ldcg(P + p);
        if (g != p) __stcg(P + x, g);
        x = p;
    }
}

__device__ __forceinline__ void uf_unite(int *P, int a, int b) {
    a = uf_find(P, a);
    b = uf_find(P, b);
    while (a != b) {
        if (a > b) {
            const int t = a;
            a = b;
            b = t;
        }
        const int old = atomicCAS(P + b, b, a);
        if (old == b) return;
        b = uf_find(P, old);
        a = uf_find(P, a);
    }
}

__global__ void k_uf_init(int *P, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) P[i] = i;
}

__device__ __forceinline__ int run_end(const int *run_x, int r, int row_end, int w) {
    return r + 1 < row_end ? run_x[r + 1] - 1 : w - 1;
}

// Band-local union-find: block b takes the runs of rows [b kBandRows, (b + 1) kBandRows).  Their
// unions with runs of the band's own rows happen in shared memory (local indices, smaller root
// wins), then every run's global parent is its band-local root.  Unions that leave the band (a
// band's first row with the row above, background runs touching the page frame) are left to
// k_uf_cross, after every band has written its parents.  Linking always points a root to a
// smaller index, so whatever the order of the unions, a component's final root is its smallest
// node.  A band with more than kBandRuns runs writes P[r] = r and leaves all of its unions to
// k_uf_cross.
constexpr int kBandRows = 16, kBandRuns = 8192;

__device__ __forceinline__ int band_find(int *L, int x) {
    for (;;) {
        const int p = L[x];
        if (p == x) return x;
        const int g = L[p];
        if (g != p) L[x] = g;
        x = p;
    }
}

__device__ __forceinline__ void band_unite(int *L, int a, int b) {
    a = band_find(L, a);
    b = band_find(L, b);
    while (a != b) {
        if (a > b) {
            const int t = a;
            a = b;
            b = t;
        }
        const int old = atomicCAS(L + b, b, a);
        if (old == b) return;
        b = band_find(L, old);
        a = band_find(L, a);
    }
}

__global__ void __launch_bounds__(512) k_uf_band(const int *__restrict__ run_x, const uint8_t *__restrict__ run_c,
                                                 const int *__restrict__ off, const int *__restrict__ cnt, int rows,
                                                 int w, int h, int pages, int *__restrict__ P, int *__restrict__ big) {
    __shared__ int L[kBandRuns];
    const int row0 = blockIdx.x * kBandRows, row1 = min(rows, row0 + kBandRows);
    const int r0 = off[row0], r1 = off[row1 - 1] + cnt[row1 - 1], nr = r1 - r0;
    if (nr > kBandRuns) {  // too many runs for shared memory: k_uf_union unites these rows
        for (int i = threadIdx.x; i < nr; i += blockDim.x) P[pages + r0 + i] = pages + r0 + i;
        if (threadIdx.x == 0) big[blockIdx.x] = 1;
        return;
    }
    if (threadIdx.x == 0) big[blockIdx.x] = 0;
    for (int i = threadIdx.x; i < nr; i += blockDim.x) L[i] = i;
    __syncthreads();
    for (int i = threadIdx.x; i < nr; i += blockDim.x) {
        const int r = r0 + i;
        // this run's row: the last band row whose first run is at or before r
        int row = row0;
        while (row + 1 < row1 && off[row + 1] <= r) row++;
        if (row == row0 || row % h == 0) continue;  // the row above is another band's (or page's)
        const int a = run_x[r], c = run_c[r], b = run_end(run_x, r, off[row] + cnt[row], w);
        const int q0 = off[row - 1], q1 = q0 + cnt[row - 1];
        const int lo = c ? max(a - 1, 0) : a, hi = c ? min(b + 1, w - 1) : b;
        int l = q0, u = q1 - 1;  // the last run of the row above starting at or before lo
        while (l < u) {
            const int mid = (l + u + 1) >> 1;
            if (run_x[mid] <= lo)
                l = mid;
            else
                u = mid - 1;
        }
        for (int q = l; q < q1 && run_x[q] <= hi; q++)
            if (run_c[q] == c) band_unite(L, i, q - r0);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nr; i += blockDim.x) P[pages + r0 + i] = pages + r0 + band_find(L, i);
}

// The unions k_uf_band left: a band's first row with the row above, background runs on the page's
// edge with the frame node, and every union of an oversized band's runs.
__global__ void k_uf_cross(const int *__restrict__ run_x, const uint8_t *__restrict__ run_c,
                           const int *__restrict__ run_row, const int *__restrict__ off, const int *__restrict__ cnt,
                           int R, int w, int h, int pages, const int *__restrict__ big, int *P) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    const int row = run_row[r], y = row % h, page = row / h;
    const int a = run_x[r], c = run_c[r], b = run_end(run_x, r, off[row] + cnt[row], w);
    const int node = pages + r;
    if (!c && (y == 0 || y == h - 1 || a == 0 || b == w - 1)) uf_unite(P, node, page);
    if (y == 0) return;
    if (row % kBandRows != 0 && !big[row / kBandRows]) return;  // united inside its band
    const int q0 = off[row - 1], q1 = q0 + cnt[row - 1];
    const int lo = c ? max(a - 1, 0) : a, hi = c ? min(b + 1, w - 1) : b;
    int l = q0, u = q1 - 1;
    while (l < u) {
        const int mid = (l + u + 1) >> 1;
        if (run_x[mid] <= lo)
            l = mid;
        else
            u = mid - 1;
    }
    for (int q = l; q < q1 && run_x[q] <= hi; q++)
        if (run_c[q] == c) uf_unite(P, node, pages + q);
}

__global__ void k_uf_flatten(int *P, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) P[i] = uf_find(P, i);
}

// 1 for the root run of an external foreground component
__device__ __forceinline__ int is_ext_root(const int *run_x, const uint8_t *run_c, const int *run_row, const int *P,
                                           int r, int h, int pages) {
    if (!run_c[r] || P[pages + r] != pages + r) return 0;
    return run_x[r] == 0 || P[pages + r - 1] == run_row[r] / h;
}

__global__ void k_ext_flag(const int *__restrict__ run_x, const uint8_t *__restrict__ run_c,
                           const int *__restrict__ run_row, const int *__restrict__ P, int R, int h, int pages,
                           int *__restrict__ flag) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < R) flag[r] = is_ext_root(run_x, run_c, run_row, P, r, h, pages);
}

__global__ void k_ext_list(const int *__restrict__ run_x, const uint8_t *__restrict__ run_c,
                           const int *__restrict__ run_row, const int *__restrict__ P, int R, int h, int pages,
                           const int *__restrict__ pos, int *__restrict__ comp_run) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < R && is_ext_root(run_x, run_c, run_row, P, r, h, pages)) comp_run[pos[r]] = r;
}

// ---- border following ------------------------------------------------------------------------

// Columns wx0 .. wx0 + 63 of row y as bits (pixels off the page read 0).
__device__ __forceinline__ uint64_t row_win64(const uint32_t *m, int words, int w, int h, int y, int wx0) {
    if ((unsigned)y >= (unsigned)h) return 0ull;
    const uint32_t *row = m + (int64_t)y * words;
    const int j = wx0 >> 5;  // floor, also for wx0 < 0
    const uint32_t a = (unsigned)j < (unsigned)words ? __ldg(row + j) : 0u;
    const uint32_t b = (unsigned)(j + 1) < (unsigned)words ? __ldg(row + j + 1) : 0u;
    const uint32_t c = (unsigned)(j + 2) < (unsigned)words ? __ldg(row + j + 2) : 0u;
    uint64_t v = ((uint64_t)__funnelshift_r(b, c, wx0 & 31) << 32) | __funnelshift_r(a, b, wx0 & 31);
    const int valid = w - wx0;
    if (valid < 64) v &= valid <= 0 ? 0ull : (1ull << valid) - 1ull;
    return v;
}

// Step (3.3)-(3.4) of Algorithm 1 as a table: for the direction e from the current point back to
// the previous one and the 3 x 3 block around the current point (bits 0-2 the row above, 3-5 its
// own row, 6-8 the row below, each left to right), the first set neighbour counterclockwise from
// e - 1: (dx + 1) | (dy + 1) << 2 | (its direction back to the current point) << 4, or 0x80 when
// no neighbour is set.
struct StepLut {
    uint8_t v[8 * 512];
};

constexpr StepLut make_step_lut() {
    StepLut t{};
    for (int e = 0; e < 8; e++)
        for (int b = 0; b < 512; b++) {
            const uint32_t u = b & 7, c = b >> 3 & 7, d = b >> 6 & 7;
            const uint32_t nb = (c & 1u) | (u & 1u) << 1 | (u >> 1 & 1u) << 2 | (u >> 2 & 1u) << 3 |
                                (c >> 2 & 1u) << 4 | (d >> 2 & 1u) << 5 | (d >> 1 & 1u) << 6 | (d & 1u) << 7;
            int d4 = -1;
            for (int k = 1; k <= 8 && d4 < 0; k++)
                if (nb >> ((e - k) & 7) & 1u) d4 = (e - k) & 7;
            t.v[e * 512 + b] = d4 < 0 ? (uint8_t)0x80
                                      : (uint8_t)((kNbX >> (2 * d4) & 3u) | (kNbY >> (2 * d4) & 3u) << 2 |
                                                  (uint32_t)((d4 + 4) & 7) << 4);
        }
    return t;
}

__constant__ StepLut kStep = make_step_lut();

// Algorithm 1 (3.1)-(3.5) from the outer-border start (x, y) entered from its left neighbour,
// run by a whole warp: the number of border points, the points written to out while their index
// is below wcap (0: count only).  The warp holds a 32-row x 64-column window of the mask, lane l
// row wy0 + l, in registers; every lane runs the same steps, and the three neighbour rows of the
// current point come from their lanes by shuffles, so a step reads no memory until the point
// leaves the window (then every lane loads its row of a window re-centred on it, in parallel).
// (3.1) takes the first set neighbour clockwise from the left one, (3.3) the first
// counterclockwise from the one after the previous point (StepLut).  A border is at most 4 points
// a pixel; past that the status word is set and the trace stops.  Must be called by all 32 lanes
// of a warp.
__device__ int follow_warp(const uint32_t *m, int words, int w, int h, int x, int y, short2 *out, int wcap,
                           int *status) {
    const int lane = threadIdx.x & 31;
    int wx0 = x - 32, wy0 = y - 16;
    uint64_t win = row_win64(m, words, w, h, wy0 + lane, wx0);
    // the 3 x 3 block around (xx, yy) (StepLut's bit order): xx - 1 - wx0 in 0 .. 61, yy - wy0 in 1 .. 30
    auto block = [&](int xx, int yy) -> uint32_t {
        const uint32_t t = (uint32_t)(win >> (xx - 1 - wx0)) & 7u;
        const int r = yy - wy0;
        const uint32_t u = __shfl_sync(0xffffffffu, t, r - 1), c = __shfl_sync(0xffffffffu, t, r),
                       d = __shfl_sync(0xffffffffu, t, r + 1);
        return u | c << 3 | d << 6;
    };
    uint32_t blk = block(x, y);
    // (3.1): the first set neighbour clockwise from the left one (bit d = neighbour d)
    const uint32_t nb0 = (blk >> 3 & 1u) | (blk & 1u) << 1 | (blk >> 1 & 1u) << 2 | (blk >> 2 & 1u) << 3 |
                         (blk >> 5 & 1u) << 4 | (blk >> 8 & 1u) << 5 | (blk >> 7 & 1u) << 6 | (blk >> 6 & 1u) << 7;
    if (nb0 == 0) {
        if (wcap > 0 && lane == 0) out[0] = make_short2((short)x, (short)y);
        return 1;
    }
    const int d1 = __ffs(nb0) - 1;
    const int x1 = x + nb_dx(d1), y1 = y + nb_dy(d1);
    int x3 = x, y3 = y, e = d1, n = 0;
    const int64_t cap = 4 * (int64_t)w * h + 8;
    for (;;) {
        if (lane == 0 && n < wcap) out[n] = make_short2((short)x3, (short)y3);
        n++;
        const uint32_t v = kStep.v[e << 9 | blk];
        if ((v & 0x80u) || n >= cap) {  // the previous point is always set: a broken mask read
            if (lane == 0) atomicExch(status, 40);
            break;
        }
        const int x4 = x3 + (int)(v & 3u) - 1, y4 = y3 + (int)(v >> 2 & 3u) - 1;
        if (x4 == x && y4 == y && x3 == x1 && y3 == y1) break;
        e = (int)(v >> 4);  // from the new (i3, j3) back to the old one
        if (x4 - 1 < wx0 || x4 + 1 > wx0 + 63 || y4 - 1 < wy0 || y4 + 1 > wy0 + 31) {
            wx0 = x4 - 32;
            wy0 = y4 - 16;
            win = row_win64(m, words, w, h, wy0 + lane, wx0);
        }
        x3 = x4;
        y3 = y4;
        blk = block(x3, y3);
    }
    return n;
}

// A warp per component.  The first cache_cap points go to the component's cache slot, so borders
// no longer than that are not followed a second time.
__global__ void __launch_bounds__(32) k_trace_len(const uint32_t *__restrict__ mask, int words, int w, int h,
                                                  const int *__restrict__ run_x, const int *__restrict__ run_row,
                                                  const int *__restrict__ comp_run, int C, int *__restrict__ len,
                                                  short2 *__restrict__ cache, int cache_cap, int *status) {
    const int k = blockIdx.x;
    if (k >= C) return;
    const int r = comp_run[k], row = run_row[r];
    const uint32_t *m = mask + (int64_t)(row / h) * h * words;
    const int n = follow_warp(m, words, w, h, run_x[r], row % h, cache + (int64_t)k * cache_cap, cache_cap, status);
    if (threadIdx.x == 0) len[k] = n;
}

// Block sizes of k_word_rect: components of more than kBigLen border points get kWTBig threads.
// A Douglas-Peucker level of at most kFewSegs open segments runs each segment with the whole
// block (a shuffle and shared-memory argmax) instead of the flat scan over all of them.
constexpr int kWT = 128, kWTBig = 1024, kBigLen = 4096, kSortCap = 2048, kFewSegs = 4;

// the components whose border is longer than kBigLen, for the wide instance of k_word_rect
__global__ void k_big_list(const int *__restrict__ len, int C, int *__restrict__ big, int *__restrict__ nbig) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k < C && len[k] > kBigLen) big[atomicAdd(nbig, 1)] = k;
}

// ---- per-component geometry ------------------------------------------------------------------

__device__ __forceinline__ float sq_len(float x, float y) { return __fadd_rn(__fmul_rn(x, x), __fmul_rn(y, y)); }

// point-to-segment distance (comp.graphics.algorithms FAQ 1.02): r = dot / l2 picks the nearer
// end or the perpendicular, s = cross / l2, distance |s| sqrt(l2).  The tests on r are made on
// dot itself (SegC holds the segment's terms), which takes the same branch
// with one division less: l2 > 0 and dot are integer-valued floats here (page coordinates), so
// fl(dot / l2) <= 0 exactly when dot <= 0, and fl(dot / l2) >= 1 exactly when dot >= l2 (for
// positive normal a < b, a / b <= 1 - 2^-24 (the float below 1) before rounding, so it never
// rounds up to 1).  The distance is therefore the C restatement's to the bit.
// (b = a + ab exactly: integer-valued coordinates below 2^24)
struct SegC {
    float ax, ay, abx, aby, l2, sl2;
};

__device__ __forceinline__ SegC seg_c(float ax, float ay, float bx, float by) {
    SegC c;
    c.ax = ax;
    c.ay = ay;
    c.abx = __fsub_rn(bx, ax);
    c.aby = __fsub_rn(by, ay);
    c.l2 = sq_len(c.abx, c.aby);
    c.sl2 = __fsqrt_rn(c.l2);
    return c;
}

__device__ __forceinline__ float seg_dist(const SegC &c, float px, float py) {
    const float acx = __fsub_rn(px, c.ax), acy = __fsub_rn(py, c.ay);
    if (c.l2 == 0.f) return __fsqrt_rn(sq_len(acx, acy));
    const float dot = __fadd_rn(__fmul_rn(acx, c.abx), __fmul_rn(acy, c.aby));
    if (dot <= 0.f) return __fsqrt_rn(sq_len(acx, acy));
    if (dot >= c.l2)
        return __fsqrt_rn(sq_len(__fsub_rn(px, __fadd_rn(c.ax, c.abx)), __fsub_rn(py, __fadd_rn(c.ay, c.aby))));
    const float s = __fdiv_rn(__fsub_rn(__fmul_rn(c.abx, acy), __fmul_rn(c.aby, acx)), c.l2);
    return fabsf(__fmul_rn(s, c.sl2));
}

__device__ __forceinline__ int key_x(uint32_t k) { return (int)(k >> 16); }
__device__ __forceinline__ int key_y(uint32_t k) { return (int)(k & 0xffffu); }

__device__ __forceinline__ int64_t cross3(uint32_t o, uint32_t a, uint32_t b) {
    return (int64_t)(key_x(a) - key_x(o)) * (key_y(b) - key_y(o)) -
           (int64_t)(key_y(a) - key_y(o)) * (key_x(b) - key_x(o));
}

__device__ void heap_sort(uint32_t *a, int n) {
    auto sift = [&](int i, int end) {
        for (;;) {
            int c = 2 * i + 1;
            if (c >= end) return;
            if (c + 1 < end && a[c + 1] > a[c]) c++;
            if (a[c] <= a[i]) return;
            const uint32_t t = a[c];
            a[c] = a[i];
            a[i] = t;
            i = c;
        }
    };
    for (int i = n / 2 - 1; i >= 0; i--) sift(i, n);
    for (int end = n - 1; end > 0; end--) {
        const uint32_t t = a[0];
        a[0] = a[end];
        a[end] = t;
        sift(0, end);
    }
}

struct WordP {
    const uint32_t *mask;
    int words, w, h;
    const int *run_x, *run_row, *comp_run, *pt_off, *len;
    const short2 *cache;  // the length pass's first cache_cap points of each border
    int cache_cap;
    const int *big;       // for the kWTBig instance: the components of more than kBigLen points
    int C;
    // per component, n + 1 slots each (n border points; slot base = pt_off[k] + k)
    short2 *pts;       // its border, then the first point again
    uint8_t *keep;     // Douglas-Peucker marks
    int2 *seg_a, *seg_b;  // segments of the current and the next level
    int *pref;         // exclusive prefix of the current level's interior sizes
    unsigned long long *best;  // per segment: (distance bits << 32) | ~index, the level's argmax
    uint32_t *keys;    // kept points as (x << 16) | y
    uint32_t *hull;    // 2 (n + 1) + 1 slots per component (base 2 base + k)
    float *rect;       // 6 per component
    int *valid;
    float expand, expand_x, min_area;
    int *status;
};


// exclusive prefix of size(i) for i < n into out; returns the total (all threads)
template <int T, typename F>
__device__ int block_scan(int n, int *out, F size, int *warp_tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int carry = 0;
    for (int c0 = 0; c0 < n; c0 += T) {
        const int i = c0 + threadIdx.x;
        const int v = i < n ? size(i) : 0;
        int x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_tot[warp] = x;
        __syncthreads();
        int before = carry;
        for (int q = 0; q < warp; q++) before += warp_tot[q];
        int all = carry;
        for (int q = 0; q < T / 32; q++) all += warp_tot[q];
        if (i < n) out[i] = before + x - v;
        __syncthreads();
        carry = all;
    }
    return carry;
}

__device__ __forceinline__ unsigned long long dp_key(float d, int i) {
    return ((unsigned long long)__float_as_uint(d) << 32) | (0xffffffffu - (uint32_t)i);
}

// The octagon of extreme points (in x, y, x + y, x - y) has points of the set on the hull as its
// vertices, so a point of the closed octagon that is not one of its vertices lies strictly inside
// the hull or on a hull edge strictly between two hull points, and the monotone chain (which
// drops collinear points) never returns it.  (A degenerate, collinear octagon keeps its two ends.)
__device__ __forceinline__ bool in_octagon(const uint32_t *oct, int noct, uint32_t q) {
    if (noct < 3) return false;
    for (int i = 0; i < 8; i++) {
        const uint32_t a = oct[i], b = oct[(i + 1) & 7];
        if (q == a) return false;
        if (a == b) continue;
        if (cross3(a, b, q) < 0) return false;
    }
    return true;
}

// One block per external component: border following (one warp, when the length pass could not
// keep the border), Douglas-Peucker by levels
// (every point of every open segment at once, argmax per segment by a 64-bit atomicMax: the
// largest distance, then the smallest index, as the sequential search finds it), the hull of
// the kept points (octagon filter, sort, monotone chain) and the minimum-area rectangle (an
// argmin over the hull's edges, first edge on ties).
template <int T>
__global__ void __launch_bounds__(T) k_word_rect(WordP p) {
    __shared__ int s_n, s_nseg, s_next, s_tot, s_m, s_ns, s_hc, s_noct;
    __shared__ int warp_tot[T / 32];
    __shared__ uint32_t s_oct[8];
    __shared__ unsigned long long s_ext[8], s_best;
    __shared__ uint32_t s_sort[kSortCap];
    __shared__ int2 s_few[2][kFewSegs];                   // a level's segments when few (by parity)
    __shared__ unsigned long long s_wbest[kFewSegs][T / 32];
    const int k = T == kWTBig ? p.big[blockIdx.x] : (int)blockIdx.x, tid = threadIdx.x, lane = tid & 31,
              warp = tid >> 5;
    if (k >= p.C || (p.len[k] > kBigLen) != (T == kWTBig)) return;  // the other instance's component
    const int r = p.comp_run[k], row = p.run_row[r];
    const int64_t base = (int64_t)p.pt_off[k] + k;
    short2 *pts = p.pts + base;
    const int L = p.len[k];
    if (L <= p.cache_cap) {  // the border is in the cache: copy it
        const short2 *src = p.cache + (int64_t)k * p.cache_cap;
        for (int i = tid; i < L; i += T) pts[i] = src[i];
    }
    if (warp == 0) {
        int nb = L;
        if (L > p.cache_cap) {
            const uint32_t *m = p.mask + (int64_t)(row / p.h) * p.h * p.words;
            nb = follow_warp(m, p.words, p.w, p.h, p.run_x[r], row % p.h, pts, 0x7fffffff, p.status);
        }
        if (lane == 0) {
            pts[nb] = L > p.cache_cap ? pts[0] : p.cache[(int64_t)k * p.cache_cap];
            s_n = nb + 1;
            s_nseg = 0;
            if (nb + 1 > 2) {
                p.seg_a[base] = make_int2(0, nb);
                s_few[0][0] = make_int2(0, nb);
                s_nseg = 1;
            }
        }
    }
    __syncthreads();
    const int n = s_n;
    uint8_t *keep = p.keep + base;
    for (int i = tid; i < n; i += T) keep[i] = (i == 0 || i == n - 1);
    int2 *sa = p.seg_a + base, *sb = p.seg_b + base;
    int *pref = p.pref + base;
    unsigned long long *best = p.best + base;
    __syncthreads();
    // Douglas-Peucker, epsilon 2, on the closed polyline
    int par = 0;
    while (s_nseg > 0) {
        const int nseg = s_nseg;
        if (nseg <= kFewSegs) {
            // few open segments (deep, narrow levels): one pass of the block over all of them,
            // each thread keeping a maximum per segment, then a warp and a block reduction
            int2 sg[kFewSegs];
            int pre[kFewSegs + 1];
            pre[0] = 0;
#pragma unroll
            for (int u = 0; u < kFewSegs; u++) {
                sg[u] = u < nseg ? s_few[par][u] : make_int2(0, 1);
                pre[u + 1] = pre[u] + (u < nseg ? sg[u].y - sg[u].x - 1 : 0);
            }
            unsigned long long bk[kFewSegs];
#pragma unroll
            for (int u = 0; u < kFewSegs; u++) bk[u] = 0ull;
            for (int g = tid; g < pre[kFewSegs]; g += T) {
#pragma unroll
                for (int u = 0; u < kFewSegs; u++)
                    if (g >= pre[u] && g < pre[u + 1]) {
                        const int i = sg[u].x + 1 + (g - pre[u]);
                        const SegC c = seg_c((float)pts[sg[u].x].x, (float)pts[sg[u].x].y, (float)pts[sg[u].y].x,
                                             (float)pts[sg[u].y].y);
                        const unsigned long long key = dp_key(seg_dist(c, (float)pts[i].x, (float)pts[i].y), i);
                        bk[u] = key > bk[u] ? key : bk[u];
                    }
            }
            // (only the level's nseg segments are reduced: nseg is the same for the whole block)
#pragma unroll
            for (int u = 0; u < kFewSegs; u++) {
                if (u >= nseg) break;
#pragma unroll
                for (int o = 16; o; o >>= 1) {
                    const unsigned long long ot = __shfl_xor_sync(0xffffffffu, bk[u], o);
                    bk[u] = ot > bk[u] ? ot : bk[u];
                }
                if (lane == 0) s_wbest[u][warp] = bk[u];
            }
            __syncthreads();
            if (warp == 0) {
#pragma unroll
                for (int u = 0; u < kFewSegs; u++) {
                    if (u >= nseg) break;
                    unsigned long long v = lane < T / 32 ? s_wbest[u][lane] : 0ull;
#pragma unroll
                    for (int o = 16; o; o >>= 1) {
                        const unsigned long long ot = __shfl_xor_sync(0xffffffffu, v, o);
                        v = ot > v ? ot : v;
                    }
                    bk[u] = v;
                }
                if (tid == 0) {
                    int nx = 0;
#pragma unroll
                    for (int u = 0; u < kFewSegs; u++) {
                        if (u >= nseg) break;
                        const float d = __uint_as_float((uint32_t)(bk[u] >> 32));
                        const int i = (int)(0xffffffffu - (uint32_t)bk[u]);
                        if (d > 2.0f) {
                            keep[i] = 1;
                            if (i - sg[u].x > 1) {
                                if (nx < kFewSegs) s_few[par ^ 1][nx] = make_int2(sg[u].x, i);
                                sb[nx++] = make_int2(sg[u].x, i);
                            }
                            if (sg[u].y - i > 1) {
                                if (nx < kFewSegs) s_few[par ^ 1][nx] = make_int2(i, sg[u].y);
                                sb[nx++] = make_int2(i, sg[u].y);
                            }
                        }
                    }
                    s_nseg = nx;
                }
            }
            int2 *t = sa;
            sa = sb;
            sb = t;
            par ^= 1;
            __syncthreads();
            continue;
        }
        for (int q = tid; q < nseg; q += T) best[q] = 0ull;
        const int tot = block_scan<T>(nseg, pref, [&](int q) { return sa[q].y - sa[q].x - 1; }, warp_tot);
        for (int g = tid; g < tot; g += T) {
            int lo = 0, hi = nseg - 1;  // the last segment whose prefix is <= g
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (pref[mid] <= g)
                    lo = mid;
                else
                    hi = mid - 1;
            }
            const int2 sg = sa[lo];
            const int i = sg.x + 1 + (g - pref[lo]);
            const SegC c = seg_c((float)pts[sg.x].x, (float)pts[sg.x].y, (float)pts[sg.y].x, (float)pts[sg.y].y);
            const float d = seg_dist(c, (float)pts[i].x, (float)pts[i].y);
            atomicMax(best + lo, dp_key(d, i));
        }
        if (tid == 0) s_next = 0;
        __syncthreads();
        for (int q = tid; q < nseg; q += T) {
            const unsigned long long b = best[q];
            const float d = __uint_as_float((uint32_t)(b >> 32));
            const int i = (int)(0xffffffffu - (uint32_t)b);
            const int2 sg = sa[q];
            if (d > 2.0f) {
                keep[i] = 1;
                if (i - sg.x > 1) {
                    const int j = atomicAdd(&s_next, 1);
                    sb[j] = make_int2(sg.x, i);
                    if (j < kFewSegs) s_few[par ^ 1][j] = make_int2(sg.x, i);
                }
                if (sg.y - i > 1) {
                    const int j = atomicAdd(&s_next, 1);
                    sb[j] = make_int2(i, sg.y);
                    if (j < kFewSegs) s_few[par ^ 1][j] = make_int2(i, sg.y);
                }
            }
        }
        __syncthreads();
        if (tid == 0) s_nseg = s_next;
        int2 *t = sa;
        sa = sb;
        sb = t;
        par ^= 1;
        __syncthreads();
    }
    // the kept points (the closing copy excluded), and their extremes
    uint32_t *keys = p.keys + base;
    if (tid == 0) s_m = 0;
    if (tid < 8) s_ext[tid] = (tid & 1) ? 0ull : ~0ull;
    __syncthreads();
    for (int i = tid; i < n - 1; i += T)
        if (keep[i]) {
            const uint32_t kk = ((uint32_t)pts[i].x << 16) | (uint32_t)pts[i].y;
            keys[atomicAdd(&s_m, 1)] = kk;
            const int x = pts[i].x, y = pts[i].y;
            // (value, key) pairs: even slots take the minimum, odd ones the maximum
            const int v[4] = {x, y, x + y, x - y + 65536};
            for (int e = 0; e < 4; e++) {
                const unsigned long long pk = ((unsigned long long)(uint32_t)v[e] << 32) | kk;
                atomicMin(&s_ext[2 * e], pk);
                atomicMax(&s_ext[2 * e + 1], pk);
            }
        }
    __syncthreads();
    const int m = s_m;
    if (tid == 0) {
        // octagon in order: min x, min x+y, min y, max x-y, max x, max x+y, max y, min x-y
        const int ord[8] = {0, 4, 2, 7, 1, 5, 3, 6};
        int distinct = 0;
        for (int i = 0; i < 8; i++) {
            s_oct[i] = (uint32_t)s_ext[ord[i]];
            bool seen = false;
            for (int j = 0; j < i; j++) seen |= s_oct[j] == s_oct[i];
            distinct += !seen;
        }
        s_noct = m > 0 ? distinct : 0;
        s_ns = 0;
    }
    __syncthreads();
    // survivors of the octagon filter (into the free segment slots), sorted in shared memory
    // when they fit
    uint32_t *surv = (uint32_t *)sb;
    for (int i = tid; i < m; i += T)
        if (!in_octagon(s_oct, s_noct, keys[i])) surv[atomicAdd(&s_ns, 1)] = keys[i];
    __syncthreads();
    const bool small = s_ns <= kSortCap;
    uint32_t *sv = small ? s_sort : surv;
    if (small) {
        const int ns = s_ns;
        for (int i = tid; i < ns; i += T) s_sort[i] = surv[i];
        int np2 = 1;
        while (np2 < ns) np2 <<= 1;
        for (int i = ns + tid; i < np2; i += T) s_sort[i] = 0xffffffffu;
        __syncthreads();
        for (int len = 2; len <= np2; len <<= 1)
            for (int j = len >> 1; j > 0; j >>= 1) {
                for (int i = tid; i < np2; i += T) {
                    const int l = i ^ j;
                    if (l > i) {
                        const uint32_t a = s_sort[i], b = s_sort[l];
                        const bool up = (i & len) == 0;
                        if ((a > b) == up) {
                            s_sort[i] = b;
                            s_sort[l] = a;
                        }
                    }
                }
                __syncthreads();
            }
    } else if (tid == 0) {
        heap_sort(surv, s_ns);
    }
    __syncthreads();
    uint32_t *hl = p.hull + 2 * base + k;
    if (tid == 0) {
        const int ns = s_ns;
        int u = 0;
        for (int i = 0; i < ns; i++)
            if (u == 0 || sv[i] != sv[u - 1]) sv[u++] = sv[i];
        int hn = 0;
        if (u >= 2) {
            for (int i = 0; i < u; i++) {
                while (hn >= 2 && cross3(hl[hn - 2], hl[hn - 1], sv[i]) <= 0) hn--;
                hl[hn++] = sv[i];
            }
            for (int i = u - 2, lo = hn + 1; i >= 0; i--) {
                while (hn >= lo && cross3(hl[hn - 2], hl[hn - 1], sv[i]) <= 0) hn--;
                hl[hn++] = sv[i];
            }
        }
        s_hc = u >= 2 ? hn - 1 : 0;
        s_best = ~0ull;
    }
    __syncthreads();
    const int hc = s_hc;
    if (hc == 0) {
        if (tid == 0) p.valid[k] = 0;
        return;
    }
    // the edge of least area (first on ties)
    auto edge = [&](int i, float *rc) -> float {
        const uint32_t a = hl[i], b = hl[(i + 1) % hc];
        const float dx = (float)(key_x(b) - key_x(a)), dy = (float)(key_y(b) - key_y(a));
        const float len = __fsqrt_rn(sq_len(dx, dy));
        const float ux = __fdiv_rn(dx, len), uy = __fdiv_rn(dy, len);
        float s0 = __int_as_float(0x7f800000), s1 = -s0, t0 = s0, t1 = -s0;
        for (int j = 0; j < hc; j++) {
            const float rx = (float)(key_x(hl[j]) - key_x(a)), ry = (float)(key_y(hl[j]) - key_y(a));
            const float s = __fadd_rn(__fmul_rn(rx, ux), __fmul_rn(ry, uy));
            const float t = __fadd_rn(__fmul_rn(rx, -uy), __fmul_rn(ry, ux));
            s0 = s < s0 ? s : s0;
            s1 = s > s1 ? s : s1;
            t0 = t < t0 ? t : t0;
            t1 = t > t1 ? t : t1;
        }
        if (rc) {
            const float sc = __fmul_rn(__fadd_rn(s0, s1), 0.5f), tc = __fmul_rn(__fadd_rn(t0, t1), 0.5f);
            rc[0] = __fadd_rn(__fadd_rn((float)key_x(a), __fmul_rn(ux, sc)), __fmul_rn(-uy, tc));
            rc[1] = __fadd_rn(__fadd_rn((float)key_y(a), __fmul_rn(uy, sc)), __fmul_rn(ux, tc));
            rc[2] = -uy;
            rc[3] = ux;
            rc[4] = __fsub_rn(s1, s0);
            rc[5] = __fsub_rn(t1, t0);
        }
        return __fmul_rn(__fsub_rn(s1, s0), __fsub_rn(t1, t0));
    };
    for (int i = tid; i < hc; i += T)
        atomicMin(&s_best, ((unsigned long long)__float_as_uint(edge(i, nullptr)) << 32) | (uint32_t)i);
    __syncthreads();
    if (tid == 0) {
        float rc[6];
        edge((int)(uint32_t)s_best, rc);
        rc[4] = __fadd_rn(rc[4], __fmul_rn(2.f, __fadd_rn(p.expand, p.expand_x)));
        rc[5] = __fadd_rn(rc[5], __fmul_rn(2.f, p.expand));
        float *out = p.rect + 6 * (int64_t)k;
#pragma unroll
        for (int i = 0; i < 6; i++) out[i] = rc[i];
        p.valid[k] = __fmul_rn(rc[4], rc[5]) >= p.min_area;
    }
}

__global__ void k_word_pack(const float *__restrict__ rect, const int *__restrict__ valid, const int *__restrict__ pos,
                            const int *__restrict__ comp_run, const int *__restrict__ run_row, int h, int C,
                            float *__restrict__ out, int *__restrict__ page_cnt) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= C || !valid[k]) return;
#pragma unroll
    for (int i = 0; i < 6; i++) out[6 * (int64_t)pos[k] + i] = rect[6 * (int64_t)k + i];
    atomicAdd(page_cnt + run_row[comp_run[k]] / h, 1);
}

inline unsigned blocks(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

void scan_i32(Ctx *c, const int *in, int n, int *out, int *total) {
    if (n <= 0) {
        WOCR_CUDA(cudaMemsetAsync(total, 0, sizeof(int), c->stream));
        return;
    }
    const int nb = (n + kScanBlock - 1) / kScanBlock;
    if (nb == 1) {
        k_scan_blocks<<<1, kScanT, 0, c->stream>>>(in, n, out, total);
        WOCR_LAUNCHED(c);
        return;
    }
    BufP sums = alloc(c, (size_t)nb * sizeof(int));
    int *s = (int *)sums->p;
    k_scan_blocks<<<nb, kScanT, 0, c->stream>>>(in, n, out, s);
    WOCR_LAUNCHED(c);
    scan_i32(c, s, nb, s, total);
    k_scan_add<<<nb, kScanT, 0, c->stream>>>(out, n, s);
    WOCR_LAUNCHED(c);
}

namespace {
int read_int(Ctx *c, const int *d) {
    int v = 0;
    WOCR_CUDA(cudaMemcpyAsync(&v, d, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    wait_stream(c);
    return v;
}
}  // namespace

WordRects word_rects(Ctx *c, const uint32_t *mask, int pages, int w, int h, float expand, float expand_x,
                     float min_area) {
    WordRects res;
    res.page_count = alloc(c, (size_t)pages * sizeof(int));
    WOCR_CUDA(cudaMemsetAsync(res.page_count->p, 0, (size_t)pages * sizeof(int), c->stream));
    const int words = (w + 31) / 32, rows = pages * h;
    BufP cnt = alloc(c, (size_t)rows * 4), off = alloc(c, (size_t)rows * 4), tot = alloc(c, 4);
    int *d_cnt = (int *)cnt->p, *d_off = (int *)off->p, *d_tot = (int *)tot->p;
    {
        Prof pf(c, "word_runs", 0, (double)rows * words * 4);
        k_run_count<<<blocks(rows, kRowWarps), kRowWarps * 32, 0, c->stream>>>(mask, words, w, rows, d_cnt);
        WOCR_LAUNCHED(c);
    }
    scan_i32(c, d_cnt, rows, d_off, d_tot);
    const int R = read_int(c, d_tot);
    BufP rx = alloc(c, (size_t)R * 4), rc = alloc(c, (size_t)R), rr = alloc(c, (size_t)R * 4);
    BufP par = alloc(c, (size_t)(R + pages) * 4), flag = alloc(c, (size_t)R * 4), pos = alloc(c, (size_t)R * 4);
    int *run_x = (int *)rx->p, *run_row = (int *)rr->p, *P = (int *)par->p;
    uint8_t *run_c = (uint8_t *)rc->p;
    {
        Prof pf(c, "word_runs", 0, (double)rows * words * 4 + (double)R * 9);
        k_run_write<<<blocks(rows, kRowWarps), kRowWarps * 32, 0, c->stream>>>(mask, words, w, rows, d_off, run_x,
                                                                                 run_c, run_row);
        WOCR_LAUNCHED(c);
    }
    {
        Prof pf(c, "word_label", 0, (double)R * 30);
        const int bands = (rows + kBandRows - 1) / kBandRows;
        BufP bigb = alloc(c, (size_t)bands * 4);
        k_uf_init<<<blocks(pages, 256), 256, 0, c->stream>>>(P, pages);  // the frame nodes
        WOCR_LAUNCHED(c);
        k_uf_band<<<bands, 512, 0, c->stream>>>(run_x, run_c, d_off, d_cnt, rows, w, h, pages, P, (int *)bigb->p);
        WOCR_LAUNCHED(c);
        k_uf_cross<<<blocks(R, 256), 256, 0, c->stream>>>(run_x, run_c, run_row, d_off, d_cnt, R, w, h, pages,
                                                          (const int *)bigb->p, P);
        WOCR_LAUNCHED(c);
        k_uf_flatten<<<blocks(R + pages, 256), 256, 0, c->stream>>>(P, R + pages);
        WOCR_LAUNCHED(c);
        k_ext_flag<<<blocks(R, 256), 256, 0, c->stream>>>(run_x, run_c, run_row, P, R, h, pages, (int *)flag->p);
        WOCR_LAUNCHED(c);
    }
    scan_i32(c, (const int *)flag->p, R, (int *)pos->p, d_tot);
    const int C = read_int(c, d_tot);
    res.n = 0;
    if (C == 0) {
        res.rects = alloc(c, 4);
        return res;
    }
    BufP crun = alloc(c, (size_t)C * 4), len = alloc(c, (size_t)C * 4), ptoff = alloc(c, (size_t)C * 4);
    // border cache of the length pass: 256 MiB shared by the components, 64 .. 16384 points each
    const int cache_cap = (int)std::min<int64_t>(16384, std::max<int64_t>(64, ((int64_t)64 << 20) / C));
    BufP cache = alloc(c, (size_t)C * cache_cap * 4);
    k_ext_list<<<blocks(R, 256), 256, 0, c->stream>>>(run_x, run_c, run_row, P, R, h, pages, (const int *)pos->p,
                                                      (int *)crun->p);
    WOCR_LAUNCHED(c);
    {
        Prof pf(c, "word_trace", 0, 0);
        k_trace_len<<<C, 32, 0, c->stream>>>(mask, words, w, h, run_x, run_row, (const int *)crun->p, C,
                                             (int *)len->p, (short2 *)cache->p, cache_cap, c->status);
        WOCR_LAUNCHED(c);
    }
    BufP big = alloc(c, (size_t)C * 4), nbig = alloc(c, 4);
    WOCR_CUDA(cudaMemsetAsync(nbig->p, 0, 4, c->stream));
    k_big_list<<<blocks(C, 256), 256, 0, c->stream>>>((const int *)len->p, C, (int *)big->p, (int *)nbig->p);
    WOCR_LAUNCHED(c);
    scan_i32(c, (const int *)len->p, C, (int *)ptoff->p, d_tot);
    int n_big = 0;
    WOCR_CUDA(cudaMemcpyAsync(&n_big, nbig->p, 4, cudaMemcpyDeviceToHost, c->stream));
    const int64_t slots = (int64_t)read_int(c, d_tot) + C;  // (its sync also brings n_big)
    BufP pts = alloc(c, (size_t)slots * 4), keep = alloc(c, (size_t)slots), sega = alloc(c, (size_t)slots * 8);
    BufP segb = alloc(c, (size_t)slots * 8), pref = alloc(c, (size_t)slots * 4), best = alloc(c, (size_t)slots * 8);
    BufP keys = alloc(c, (size_t)slots * 4), hull = alloc(c, (size_t)(2 * slots + C) * 4);
    BufP rect = alloc(c, (size_t)C * 24), valid = alloc(c, (size_t)C * 4), vpos = alloc(c, (size_t)C * 4);
    WordP p;
    p.mask = mask;
    p.words = words;
    p.w = w;
    p.h = h;
    p.run_x = run_x;
    p.run_row = run_row;
    p.comp_run = (const int *)crun->p;
    p.pt_off = (const int *)ptoff->p;
    p.len = (const int *)len->p;
    p.cache = (const short2 *)cache->p;
    p.cache_cap = cache_cap;
    p.big = (const int *)big->p;
    p.C = C;
    p.pts = (short2 *)pts->p;
    p.keep = (uint8_t *)keep->p;
    p.seg_a = (int2 *)sega->p;
    p.seg_b = (int2 *)segb->p;
    p.pref = (int *)pref->p;
    p.best = (unsigned long long *)best->p;
    p.keys = (uint32_t *)keys->p;
    p.hull = (uint32_t *)hull->p;
    p.rect = (float *)rect->p;
    p.valid = (int *)valid->p;
    p.expand = expand;
    p.expand_x = expand_x;
    p.min_area = min_area;
    p.status = c->status;
    {
        // algorithmic bytes: every border point read from the cache and written once, its keep
        // flag, and the rectangles (the kernel is bound by the sequential Douglas-Peucker levels)
        Prof pf(c, "word_rect", 0, 9.0 * (double)slots + 24.0 * C);
        k_word_rect<kWT><<<C, kWT, 0, c->stream>>>(p);
        WOCR_LAUNCHED(c);
        if (n_big > 0) {
            k_word_rect<kWTBig><<<n_big, kWTBig, 0, c->stream>>>(p);
            WOCR_LAUNCHED(c);
        }
    }
    scan_i32(c, (const int *)valid->p, C, (int *)vpos->p, d_tot);
    res.n = read_int(c, d_tot);
    res.rects = alloc(c, (size_t)std::max(res.n, 1) * 24);
    k_word_pack<<<blocks(C, 256), 256, 0, c->stream>>>((const float *)rect->p, (const int *)valid->p,
                                                       (const int *)vpos->p, (const int *)crun->p, run_row, h, C,
                                                       (float *)res.rects->p, (int *)res.page_count->p);
    WOCR_LAUNCHED(c);
    return res;
}

}  // namespace k
}  // namespace wocr
