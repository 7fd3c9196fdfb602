// Launchers of the sm_100a kernels.  All run on the context stream; all tensors are device
// pointers.  Every launcher cites the reference kernel whose result it reproduces.
#pragma once

#include "common.h"

namespace wocr {
namespace k {

// Activation codes of the reference epilogue (src/gpu.rs:28-34): 0 none, 1 Relu, 2 Sigmoid,
// 3 GELU (erf), 4 SiLU.
enum Act { ACT_NONE = 0, ACT_RELU = 1, ACT_SIGMOID = 2, ACT_GELU = 3, ACT_SILU = 4 };

// Implicit-GEMM convolution on channels-last tensors (K1-K4, src/gpu.rs:37-350): M = output
// pixels, N = output channels, K = taps x input channels (order ky, kx, ci).  Also serves the
// row-major linear layers (1 x 1 over M "pixels", K15 src/gpu.rs:616-678, K29 src/nd.rs:291)
// and ConvTranspose with kernel == stride (one 1 x 1 GEMM with N = cout*s*s and a scatter
// epilogue, K7 src/gpu.rs:424-460).
struct ConvP {
    const float *x = nullptr;
    int64_t x_n = 0, x_pix = 0;      // batch and pixel strides of x (elements)
    int n = 0, h = 0, w = 0, cin = 0;
    const float *wt = nullptr;       // [K][ldw], K = kh*kw*cin, zero padded columns
    int ldw = 0;
    const float *bias = nullptr;     // [cout] (scatter: [scat_cout])
    int cout = 0;                    // GEMM N
    int kh = 1, kw = 1, sh = 1, sw = 1, pt = 0, pl = 0, oh = 0, ow = 0;
    float *y = nullptr;
    int64_t y_n = 0, y_pix = 0;      // output batch and pixel strides (y at channel offset)
    const float *res = nullptr;      // residual added after the activation (src/gpu.rs:64-65)
    int64_t res_n = 0, res_pix = 0;
    const float *insc = nullptr;     // [n][cin] input scale (squeeze-excitation)
    int act = 0;
    int scatter = 0;                 // ConvTranspose stride s (kernel == stride), 0 = plain conv
    int scat_cout = 0;
};
void conv_gemm(Ctx *c, const ConvP &p);
// Narrow convolutions on CUDA cores (k_conv.cu): at most 64 output channels and kNarrowMacs
// multiply-adds per output pixel; conv_narrow_ok says whether p qualifies.
constexpr int kNarrowMacs = 4096;
bool conv_narrow_ok(const ConvP &p);
void conv_narrow(Ctx *c, const ConvP &p);

// Cin = 1, stride 1 convolution with its activation and an optional fused MaxPool (ph, pw)
// (K6, src/gpu.rs:385-422).  wt [kh][kw][cout]; output NHWC with pixel stride y_pix.
// split_out: y is a split tensor (bf16 hi | lo per pixel, strides in bf16 elements; cout 16
// or 32 only).
void conv_direct(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, const float *wt,
                 const float *bias, int cout, int kh, int kw, int pad, int act, int ph, int pw, void *y,
                 int64_t y_n, int64_t y_pix, int oh, int ow, int split_out = 0);

// 1 x 1, stride 1 convolution with cout < 16 (a detector head), memory-bound; wt [cin][ldw].
// split_in: x is a split tensor (strides in bf16 elements).  y fp32 NHWC.
void pointwise(Ctx *c, const void *x, int64_t x_n, int64_t x_pix, int64_t hw, int n, int cin, const float *wt, int ldw,
               const float *bias, int cout, int act, float *y, int64_t y_n, int64_t y_pix, int split_in = 0);

// Split activations: per pixel the bf16 hi parts of the buffer's channels, then their lo parts
// (hi = bf16(v), lo = bf16(v - hi)); views carry strides in bf16 elements, and the lo part of a
// channel lies x_pix / 2 elements after its hi part.
// Max pool with kernel == stride, no padding (K8, src/gpu.rs:462), on a split input; the output
// is split (split_out) or fp32.
void maxpool_split(Ctx *c, const uint16_t *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch, int kh, int kw,
                   int oh, int ow, void *y, int64_t y_n, int64_t y_pix, int split_out);
// split <-> fp32 conversions of 4-D views [n][c][h][w] with any strides (xs, ys in elements of
// each side; a split side has channel stride 1 and its lo part at lo_off elements).
void unsplit(Ctx *c, const uint16_t *x, const int64_t (&xs)[4], int64_t lo_off, float *y, const int64_t (&ys)[4],
             const int64_t (&dims)[4]);
void resplit(Ctx *c, const float *x, const int64_t (&xs)[4], uint16_t *y, const int64_t (&ys)[4], int64_t lo_off,
             const int64_t (&dims)[4]);

// Depthwise convolution (K5, src/gpu.rs:356-383): wt [kh][kw][c], NHWC.
void depthwise(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch, const float *wt,
               const float *bias, int kh, int kw, int sh, int sw, int pt, int pl, int oh, int ow, int act, float *y,
               int64_t y_n, int64_t y_pix);

// General ConvTranspose by parity gather (K7, src/gpu.rs:424-460): wt [cin][cout][kh][kw].
void convt_gather(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int cin, const float *wt,
                  const float *bias, int cout, int kh, int kw, int s, int act, float *y, int64_t y_n, int64_t y_pix,
                  int oh, int ow);

// Max/average pooling with strides and leading pads, padding never counted (K8 src/gpu.rs:462,
// K27 src/nd.rs:246-275).  NHWC.
void pool(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch, int kh, int kw, int sh,
          int sw, int pt, int pl, int oh, int ow, int avg, float *y, int64_t y_n, int64_t y_pix);

// Global average pool over H x W of an NHWC tensor -> [n][c] (K20/K21, src/nd.rs:98-133).
void gap(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int hw, int ch, float *y);

// Nearest resize, asymmetric, floor (K23, src/nd.rs:155-170).  NHWC.
void resize_nearest(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int h, int w, int ch, int oh, int ow,
                    float sy, float sx, float *y, int64_t y_n, int64_t y_pix);

// Strided N-D copy (K26 src/nd.rs:222-244, K9 src/gpu.rs:484, K10 src/gpu.rs:501).
struct Strided {
    int rank = 0;
    int64_t dims[kMaxRank] = {0};
    int64_t xs[kMaxRank] = {0};
    int64_t ys[kMaxRank] = {0};
    int64_t bs[kMaxRank] = {0};
};
void copy(Ctx *c, const float *x, float *y, const Strided &s);

// Broadcast binary op (K18, src/nd.rs:32-65): 0 Add, 1 Sub, 2 Mul, 3 Div, 4 Pow (2 -> x*x,
// 0.5 -> sqrt).  Strides of a in xs, of b in bs, of y in ys.
void binary(Ctx *c, int op, const float *a, const float *b, float *y, const Strided &s);

// Unary op on n dense values (K19 src/nd.rs:67-96, K11 src/gpu.rs:517): 1 Relu, 2 Sigmoid,
// 3 HardSigmoid(alpha, beta), 4 Erf (A&S 7.1.26), 5 Sqrt.
void unary(Ctx *c, int op, const float *x, float *y, int64_t n, float alpha, float beta);

// y = x * scale[ch] + shift[ch] with ch = (i / cdiv) % C (K28, src/nd.rs:277-289).
void affine(Ctx *c, const float *x, float *y, int64_t n, int C, int64_t cdiv, const float *st);

// Mean of each row of `inner` contiguous values (K20/K21, src/nd.rs:98-133).
void reduce_mean(Ctx *c, const float *x, float *y, int64_t outer, int64_t inner);

// LayerNorm over the last axis (K22, src/nd.rs:135-153): gb = gamma[len] then beta[len].
void layer_norm(Ctx *c, const float *x, float *y, int64_t rows, int len, const float *gb, float eps);

// Row softmax (K25, src/nd.rs:206-220).
void softmax(Ctx *c, const float *x, float *y, int64_t rows, int64_t len);

// Row arg-max (K30, src/nd.rs:360-391): ties -> lowest index (tie_last = 0) or last (1, Rust
// max_by as in src/bin/ocr-bench.rs:67).  row_max / row_lse nullable.
void argmax(Ctx *c, const float *x, int64_t rows, int64_t len, int64_t ld, uint32_t *best, float *row_max,
            float *row_lse, int tie_last);

// Rows of arg-max partials [rows][ntiles] (per tile: maximum, its lowest column, sum of
// exp(value - maximum)) -> the row's arg-max (lowest column on ties, as K30), maximum and
// log-sum-exp.  row_max / row_lse nullable.
void argmax_merge(Ctx *c, const float *pmax, const float *psum, const uint32_t *pidx, int64_t rows, int ntiles,
                  uint32_t *best, float *row_max, float *row_lse);

// Batched row-major matmul y[b] = a[b] (m x k) . bm[b] (k x n) (K29 with two activations,
// src/nd.rs:947-962).
void bmm(Ctx *c, const float *a, const float *bm, float *y, int64_t batch, int m, int kk, int n);

// ocrs detector input (K13, src/gpu.rs:530-561): packed RGB pages -> grey, pad, half-pixel
// bilinear to oh x ow.  n pages at rgb + i * page_bytes; output [n][oh][ow].
void grey_resize(Ctx *c, const uint8_t *rgb, int64_t page_bytes, int n, int w, int h, int oh, int ow, float *y);

// DB post-processing (k_db.cu): a box for `score` (src/ppdet.rs:63-83): its center, up axis,
// half width and half height, and the map rectangle to scan ([x0, x1] x [y0, y1], inclusive).
struct DbBox {
    float cx, cy, ux, uy, hw, hh;
    int x0, y0, x1, y1;
    int64_t map;  // element offset of the box's map from `prob` (maps of several pages stacked)
};
void db_mask(Ctx *c, const float *prob, int w, int h, float thr, uint32_t *bits);
void db_scores(Ctx *c, const float *prob, int w, int h, const DbBox *boxes, int n, float *scores);
// Per box: sums[2 k] = the inside pixels' sum in double, sums[2 k + 1] = the sum of their
// magnitudes, counts[k] = their number (order-free: a bound on `score`, not its value).
// max_rows: the tallest box's scan rows (y1 - y0 + 1); blocks take 8-row slices of a box.
void db_bounds(Ctx *c, const float *prob, int w, const DbBox *boxes, int n, int max_rows, double *sums,
               long long *counts);

// Word rectangles of bit masks (k_words.cu, `word_rects` of src/bin/ocr-bench.rs:38-60): `pages`
// masks of h rows x ceil(w / 32) words at mask; rects [n][6] = [cx, cy, up_x, up_y, width,
// height] page after page in raster order of the contours, page_count[pages] per page.
// Synchronises the stream to size its buffers.
struct WordRects {
    BufP rects, page_count;
    int n = 0;
};
WordRects word_rects(Ctx *c, const uint32_t *mask, int pages, int w, int h, float expand, float expand_x,
                     float min_area);
// exclusive prefix sum of n ints (out may be in); the total to *total (device)
void scan_i32(Ctx *c, const int *in, int n, int *out, int *total);

// One PP-OCR recognition line of a batch (k_lines.cu): the clamped box (left, top, cw x ch), its
// resized width ow, the batch width (>= ow, zero padding past ow) and the float offset of its
// [3][48][width] block in the output.
struct PpLine {
    int l, t, cw, ch, ow, width;
    int64_t off;
};
// bytes: the algorithmic bytes (the boxes' page bytes read, the batches written), for the profile
void pp_lines(Ctx *c, const uint8_t *rgb, int w, int h, const PpLine *lines, int n, int max_width, float *out,
              double bytes);
// The same for tall crops (ch >= kPpTallRows: a vertical downscale of 8 or more) in two passes
// through tmp: line i's intermediate at tmp + tmp_off[i], 48 * cw * 3 floats; max_cw and
// max_width over the lines.
constexpr int kPpTallRows = 8 * 48;
void pp_lines_tall(Ctx *c, const uint8_t *rgb, int w, int h, const PpLine *lines, int n, int max_cw, int max_width,
                   const int64_t *tmp_off, float *tmp, float *out, double bytes);
// One ocrs recognition line (k_ocrs.cu): its page (device RGB, pw x ph), the crop (left, top,
// cw x ch) of its polygon (nv vertices from v0 in the vertex array, x, y pairs), its image width
// W, the batch width bw (>= W, BLACK past W) and the float offset of its [64][bw] block.
struct OcrsLine {
    const uint8_t *page;
    int pw, ph;
    int l, t, cw, ch;
    int W, bw;
    int v0, nv;
    int64_t off;
};
// The 64-row line images of n lines: polygon mask, grey, half-pixel bilinear resize to 64 x W.
// bytes: the algorithmic bytes (crops read, images written), for the profile.
void ocrs_lines(Ctx *c, const OcrsLine *lines, int n, const int2 *verts, float *out, double bytes);

// The same on compacted pages: per page 2 oh rows of w * 3 bytes (the top and bottom source rows
// of each output row), rows[oy] = {vertical weight (float bits), bit 0/1: top/bottom is padding}.
void grey_resize_rows(Ctx *c, const uint8_t *cmp, const int2 *rows, int n, int w, int oh, int ow, float *y);

// ocrs detector output (K14, src/gpu.rs:563-593): valid vh x vw part of the map (row stride
// `stride`, plane `plane` per page) -> page size, `> thr`, 32 pixels a word.
void mask_up(Ctx *c, const float *m, int stride, int64_t plane, int n, int vw, int vh, int w, int h, float thr,
             uint32_t *bits);

// PP detection input (K24, src/nd.rs:172-204): RGB -> bilinear ow x oh -> BGR -> ImageNet
// normalisation; output NHWC [oh][ow][3] (nchw = 0) or planar [3][oh][ow] (nchw = 1).
void det_prep(Ctx *c, const uint8_t *rgb, int w, int h, int ow, int oh, int nchw, float *y);

// AvgPool (kh, 1) to one row, time-major x[t][ntot][c] at line offset noff (K12,
// src/gpu.rs:595-614).  Input NHWC [n][h][w][c].
void avgpool_t(Ctx *c, const float *x, int64_t x_n, int64_t x_pix, int n, int ch, int h, int w, int kh, int ntot,
               int noff, float *y);

// GRU recurrence of one layer, both directions (K16/K17, src/gpu.rs:680-819), as a persistent
// cluster kernel: g [tmax][ntot][1536], r [2][768][256] (rows z | r | h), rb [2][768],
// lens [ntot], y [tmax][ntot][512].
void gru_layer(Ctx *c, const float *g, const float *r, const float *rb, const int *lens, int tmax, int ntot,
               float *y);

}  // namespace k
}  // namespace wocr
