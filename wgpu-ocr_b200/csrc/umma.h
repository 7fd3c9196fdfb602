// The tcgen05 tensor-core GEMM (k_umma.cu): parameters and pre-split weights.
#pragma once

#include <cuda.h>

#include "common.h"

namespace wocr {
namespace k {

// Weights of one GEMM as the tensor cores read them: B = W^T, [N][Kpad] bf16 K-major, split into
// hi = bf16(w) and lo = bf16(w - hi), rows padded with zeros to a multiple of the N tile, with
// their TMA descriptors (128-byte swizzle, 64 x bn boxes).
struct UmmaW {
    BufP hi, lo;
    CUtensorMap map_hi, map_lo;
    // the same weights in 64- and 32-row boxes (when bn is wider): a launch with few row tiles
    // takes narrower N tiles, so more SMs share it
    CUtensorMap map_hi64, map_lo64, map_hi32, map_lo32;
    bool has64 = false, has32 = false;
    int N = 0, K = 0, Kpad = 0, bn = 0;
};

struct UmmaP {
    int mode = 0;                 // 0: A row-major [M][lda]; 1: implicit im2col of an NHWC tensor
    const float *x = nullptr;
    int64_t x_n = 0, x_pix = 0;
    int n = 0, h = 0, w = 0, cin = 0;
    int kh = 1, kw = 1, sh = 1, sw = 1, pt = 0, pl = 0, oh = 0, ow = 0;
    const float *insc = nullptr;  // [n][cin] squeeze-excitation input scale
    int64_t lda = 0;
    int vec = 0;                  // 8-wide aligned loads are valid
    int64_t M = 0;
    int K = 0, Kpad = 0, N = 0;
    const float *bias = nullptr;
    int act = 0;
    float *y = nullptr;
    int64_t y_n = 0, y_pix = 0, ldy = 0;
    int out_vec = 0;              // 16-byte aligned output rows: float4 stores
    int tma_y = 0;                // y rows (M x N, 16-byte aligned) written by TMA tensor stores
    int a_tma = 0;                // mode 0: A pre-split into bf16 hi / lo rows, loaded by the TMA warp
    uint32_t ntn_m = 1, ntn_l = 0;  // tile index / N tiles as a multiply-high and a shift (per launch)
    // tests of the bounded waits: a budget in clock cycles (0: the default of about 2 s) and a
    // first A stage whose producers do not arrive (its wait then runs out)
    long long budget = 0;
    int test_stall = 0;
    const float *res = nullptr;
    int64_t res_n = 0, res_pix = 0;
    int scatter = 0, scat_cout = 0;
    // mode 0 only: instead of storing y, each N tile writes its per-row arg-max partials at
    // [row][tile] (part_ld tiles a row): the maximum, the lowest column reaching it and the sum
    // of exp(value - maximum) over the tile's columns (part_sum null: no sums, maxima and
    // columns only)
    float *part_max = nullptr, *part_sum = nullptr;
    uint32_t *part_idx = nullptr;
    int part_ld = 0;
    int *status = nullptr;        // device error word (bounded waits that gave up)
};

int umma_bn(int N);
// wnk: [N][K] fp32, k in the order the A operand is produced (ky, kx, ci for convolutions).
// max_bn caps the N tile (a ConvTranspose with kernel == stride uses its cout, so each N tile
// is one tap and the scatter epilogue stores contiguous channels).
UmmaW make_umma_weights(Ctx *c, const std::vector<float> &wnk, int N, int K, int max_bn = 256);
void umma_gemm(Ctx *c, const UmmaW &w, UmmaP p);
inline int umma_ntiles(const UmmaW &w) { return (w.N + w.bn - 1) / w.bn; }
// arg-max partial slots per row of a fused arg-max launch: two per N tile (a slot per half tile)
inline int umma_part_slots(const UmmaW &w) { return 2 * umma_ntiles(w); }

}  // namespace k
}  // namespace wocr
