// Tap convolution on split activations (k_tconv.cu): parameters and pre-split weights.
#pragma once

#include <cuda.h>

#include "common.h"

namespace wocr {
namespace k {

// Weights of a stride-1 convolution as tap-major GEMM operand: [Npad][taps][cin_pad] bf16,
// split into hi = bf16(w) and lo = bf16(w - hi), with TMA descriptors whose boxes are one tap's
// cg-channel chunk (cg = 16, 32 or 64, the swizzle span of its rows) of bn output channels.
struct TconvW {
    BufP hi, lo;
    CUtensorMap map_hi, map_lo;
    int N = 0, taps = 0, cin = 0, cin_pad = 0, cg = 0, bn = 0;
    // 3 x 3 kernels with N <= 32 and cin <= 64 also get the column-stacked operand of the row
    // kernel (k_tconv_rows): per kernel row dy and 8-channel plane, 6 x3_cout rows of 8 bf16, row
    // v 3 x3_cout + kx x3_cout + n holding the hi (v = 0) or lo (v = 1) part of w[n][dy][kx]
    BufP x3;
    int x3_cout = 0, x3_cg = 0;
    // x3_ct: the operand is that of a 2 x 2 / stride 2 ConvTranspose instead (taps 2 ky + kx
    // stacked along N the same way: row v 4 x3_cout + tap x3_cout + n, one plane set)
    int x3_ct = 0;
};

// The row kernel's operand of a 2 x 2 / stride 2 ConvTranspose (cout <= 32, cin <= 64) added to
// its tap-convolution weights; nk: [tap * cout + co][cin] (tap = 2 ky + kx).
void add_convt_rows(Ctx *c, TconvW &w, const std::vector<float> &nk, int cout, int cin);

// wnk: [N][taps][cin] fp32 (taps in (ky, kx) order).
TconvW make_tconv_weights(Ctx *c, const std::vector<float> &wnk, int N, int taps, int cin);

// One launch.  The input is a split NHWC tensor: per pixel the bf16 hi parts of all channels of
// its buffer, then their lo parts; x points at the hi part of channel 0 of this view, strides
// are in bf16 elements and the lo part of a channel sits x_pix / 2 elements after its hi part.
struct TconvP {
    const uint16_t *x = nullptr;
    int64_t x_n = 0, x_pix = 0;
    int n = 0, h = 0, w = 0, cin = 0;
    int kh = 1, kw = 1, pt = 0, pl = 0, oh = 0, ow = 0;  // stride 1
    const float *bias = nullptr;
    int act = 0;
    void *y = nullptr;
    int split_out = 0;               // 1: y split like x (bf16 elements); 0: fp32 NHWC
    int64_t y_n = 0, y_pix = 0;
    int scatter = 0, scat_cout = 0;  // ConvTranspose kernel == stride s: N = cout * s * s
    // fused 2 x 2 / stride 2 MaxPool of the output (null: none): [n][oh/2][ow/2] at pool_y,
    // split like x (pool_split) or fp32, strides in elements of its format
    void *pool_y = nullptr;
    int pool_split = 0;
    int64_t pool_n = 0, pool_pix = 0;
    // fused 1 x 1 head (null head_y: none): the output is not stored; instead
    // head_y[n][oh][ow][head_n] (fp32, strides in floats) = act(head_b + sum_c out_c head_w[c][co]),
    // head_w [cin][head_ldw], head_n <= 4.  Only the row kernel has it (tconv_rows_eligible).
    const float *head_w = nullptr, *head_b = nullptr;
    int head_ldw = 0, head_n = 0, head_act = 0;
    float *head_y = nullptr;
    int64_t head_y_n = 0, head_y_pix = 0;
};

// Whether tconv runs this launch on the row kernel (the only one with the fused head).
bool tconv_rows_eligible(const TconvW &w, const TconvP &p);

// The input view meets the TMA rules (16-byte aligned base, lo part and strides).
bool tconv_input_ok(const uint16_t *x, int64_t x_n, int64_t x_pix);
void tconv(Ctx *c, const TconvW &w, const TconvP &p);

}  // namespace k
}  // namespace wocr
