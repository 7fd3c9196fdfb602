// Tap convolution: a stride-1 convolution (or a ConvTranspose with kernel == stride, as a 1 x 1
// GEMM with a scatter epilogue) on tcgen05 tensor cores, for activations stored split: bf16 hi |
// lo parts written so by the producing kernel's epilogue, so filling the A operand is a plain
// copy.  A tile is 128 output pixels, 16 image rows of 8; its input is loaded ONCE as a halo of
// (16 + kh - 1) x (8 + kw - 1) pixels per cg-channel chunk (cg = 16 or 32), coalesced 16-byte
// cp.async copies into 8-channel planes (pixel p of a plane at 16 p bytes, zeros outside the
// image).  That is the tensor cores' unswizzled K-major layout: every tap (ky, kx) of the kernel
// is the same halo seen from another start address, (ky * halo_width + kx) * 16 bytes further,
// with the 8-row groups (the tile's image rows) one halo row apart.  So the halo is read once
// for all taps instead of once per tap.
//   B hi, B lo: the tap's chunk of the pre-split weights for bn output channels (128-byte or
//               smaller swizzle), by TMA, resident for the whole kernel when it fits, else
//               through a ring of per-tap stages.
// Per tap the MMA thread issues hi.hi + hi.lo + lo.hi per 16-channel step (fp32-accurate
// products, as in k_umma.cu) into tensor memory.  Reference kernels: the implicit-GEMM
// convolution K1-K4 (src/gpu.rs:37-350) and the ConvTranspose K7 (src/gpu.rs:424-460).
//
// Warp roles (448 threads, one CTA per SM, persistent over tiles):
//   warps 0-3   halo producers (cp.async, up to kLagMax stages in flight per thread);
//   warps 4-11  epilogue: tcgen05.ld (lane quadrant warp % 4, column half), bias, activation,
//               split (or fp32) stores, plain or ConvTranspose scatter;
//   warp 12     B by TMA;
//   warp 13     tensor-memory allocation and MMA issue.
// Every wait is bounded; on expiry the kernel records an error code, drains its own copies and
// MMAs, frees its tensor memory and returns.
#include <atomic>
#include "kernels.h"
#include "tc.h"
#include "tconv.h"

#include <algorithm>
#include <cstdlib>

namespace wocr {
namespace k {

namespace {

using namespace tc;

constexpr int kProd = 4, kEpi0 = 4, kEpiWarps = 8, kTmaW = 12, kMmaW = 13, kThreads = 448;
constexpr int kLagMax = 4;        // cp.async stages in flight per producer thread
constexpr int kSmemBudget = 212 * 1024;  // stages and B; barriers and bias after it
constexpr int TP = 8, TR = 16;    // an MMA block: TR image rows of TP pixels (an 8-row group per image row)

struct TcP {
    const uint16_t *x;
    int64_t x_n, x_pix;
    int h, w, cin;
    int n, oh, ow;              // GEMM output grid (ConvTranspose: its input grid)
    int tiles_x, tiles_y, ntn;
    int trows;                  // image rows of a tile: TR * MB
    int ntiles;                 // < 2^31 (checked on the host)
    FastDiv div_ntn, div_tx, div_ty;
    int N, nchunk, taps, kw, pt, pl, cin_pad;
    int two_acc;                // the tile's MMAs alternate between two accumulators
    int hw_w, halo_px;          // halo row length and pixel count
    uint32_t plane, a_stage;    // bytes of one 8-channel halo plane, of one A stage
    uint32_t b_stage;           // bytes of one B ring stage (every tap of a chunk)
    int SA, SB, lag, b_res;     // A stages, B ring stages, cp.async stages in flight, B resident
    uint32_t b_off, bar_off;    // shared-memory offsets of the B region and the barriers
    const float *bias;
    int bias_n;                 // bias values copied to shared memory at bias_off
    uint32_t bias_off;
    int act;
    void *y;
    int split_out, out_vec;
    int64_t y_n, y_pix;
    int ow_out;                 // pixels per output row
    int scatter, scat_cout;
    void *pool_y;               // fused 2 x 2 MaxPool output (null: none), oh / 2 x ow / 2
    int pool_split, pool_vec;
    int64_t pool_n, pool_pix;
    uint32_t stg_off;           // per-warp 2 KB store staging (transposed stores), 0: none
    // fused 1 x 1 head (row kernel): weights [N][4] at head_off in shared memory, bias after them
    const float *head_w, *head_b;
    int head_ldw, head_n, head_act;
    float *head_y;
    int64_t head_y_n, head_y_pix;
    uint32_t head_off;
    int tile_w;                 // row kernel: output columns a tile advances (RV, or RP for the ConvTranspose)
    int *status;
};

struct Tile {
    int nb, oy0, ox0, nt;
};

// tile t -> (image, tile row, tile column, N tile), N tile fastest
__device__ __forceinline__ Tile decode(const TcP &p, int t) {
    Tile r;
    const uint32_t q1 = p.div_ntn.div((uint32_t)t), q2 = p.div_tx.div(q1), q3 = p.div_ty.div(q2);
    r.nt = t - (int)(q1 * p.div_ntn.d);
    r.ox0 = (int)(q1 - q2 * p.div_tx.d) * TP;
    r.oy0 = (int)(q2 - q3 * p.div_ty.d) * p.trows;
    r.nb = (int)q3;
    return r;
}


__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait(int n) {
    switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    }
}

// 16 fp32 values -> bf16 hi and lo parts, 8 per uint4
__device__ __forceinline__ void split16(const float (&v)[16], uint4 (&hi)[2], uint4 (&lo)[2]) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
        float t[8];
#pragma unroll
        for (int j = 0; j < 8; j++) t[j] = v[8 * h + j];
        split8(t, hi[h], lo[h]);
    }
}

__device__ __forceinline__ void store1(const TcP &p, int64_t off, float o) {
    if (p.split_out) {
        uint16_t *y = reinterpret_cast<uint16_t *>(p.y);
        __nv_bfloat16 h = __float2bfloat16_rn(o);
        __nv_bfloat16 l = __float2bfloat16_rn(o - __bfloat162float(h));
        y[off] = *reinterpret_cast<uint16_t *>(&h);
        y[off + p.y_pix / 2] = *reinterpret_cast<uint16_t *>(&l);
    } else {
        reinterpret_cast<float *>(p.y)[off] = o;
    }
}

// 16 consecutive channels at element offset `off` (all valid)
__device__ __forceinline__ void store16(const TcP &p, int64_t off, const float (&v)[16]) {
    if (p.split_out) {
        uint16_t *y = reinterpret_cast<uint16_t *>(p.y);
        if (p.out_vec) {
            uint4 hi[2], lo[2];
            split16(v, hi, lo);
            uint4 *dh = reinterpret_cast<uint4 *>(y + off);
            uint4 *dl = reinterpret_cast<uint4 *>(y + off + p.y_pix / 2);
            dh[0] = hi[0];
            dh[1] = hi[1];
            dl[0] = lo[0];
            dl[1] = lo[1];
            return;
        }
    } else if (p.out_vec) {
        float4 *d4 = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.y) + off);
#pragma unroll
        for (int j = 0; j < 4; j++) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        return;
    }
#pragma unroll
    for (int j = 0; j < 16; j++) store1(p, off + j, v[j]);
}

// store16 for a whole warp (warp_store16 in tc.h: transposed through the warp's staging area).
// Needs p.out_vec; every lane of the warp takes part.
__device__ __forceinline__ void store16_t(const TcP &p, int64_t off, bool valid, const float (&v)[16], uint4 *stg,
                                         int lane) {
    warp_store16(p.y, p.split_out != 0, p.y_pix, off, valid, v, stg, lane);
}

// TAPS: 9 (3 x 3 kernel), 1 (1 x 1) or 0 (any kernel, taps counted at run time).
// MB: 128-pixel MMA blocks per tile (2 for the narrow layers: one halo, the per-tile waits and
// commits shared by 256 pixels).
// 16 pooled channels at element offset `off` of the MaxPool output
__device__ __forceinline__ void store_pool(const TcP &p, int64_t off, const float (&v)[16]) {
    if (p.pool_split) {
        uint16_t *y = reinterpret_cast<uint16_t *>(p.pool_y);
        if (p.pool_vec) {
            uint4 hi[2], lo[2];
            split16(v, hi, lo);
            uint4 *dh = reinterpret_cast<uint4 *>(y + off);
            uint4 *dl = reinterpret_cast<uint4 *>(y + off + p.pool_pix / 2);
            dh[0] = hi[0];
            dh[1] = hi[1];
            dl[0] = lo[0];
            dl[1] = lo[1];
            return;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
            __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
            __nv_bfloat16 l = __float2bfloat16_rn(v[j] - __bfloat162float(h));
            y[off + j] = *reinterpret_cast<uint16_t *>(&h);
            y[off + p.pool_pix / 2 + j] = *reinterpret_cast<uint16_t *>(&l);
        }
    } else {
        float *y = reinterpret_cast<float *>(p.pool_y) + off;
        if (p.pool_vec) {
            float4 *d4 = reinterpret_cast<float4 *>(y);
#pragma unroll
            for (int j = 0; j < 4; j++) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) y[j] = v[j];
        }
    }
}

template <int BN, int CG, int TAPS, int MB>
__global__ void __launch_bounds__(kThreads, 1)
    k_tconv(const __grid_constant__ CUtensorMap wb_hi, const __grid_constant__ CUtensorMap wb_lo, TcP p) {
    constexpr int RB = CG * 2;                 // bytes of one B row
    constexpr uint32_t B_BYTES = BN * RB;      // B hi (or lo) of one tap chunk
    constexpr int NPL = CG / 8;                // 8-channel planes per split part
    // BN = 16: one 16-column chunk per tile, so the two halves of the epilogue take alternate
    // tiles instead of alternate chunks
    constexpr bool TSPLIT = BN == 16 && MB == 1;
    // STACK (BN <= 64): B hi and lo are one 2 BN-row operand, so one MMA of N = 2 BN (no slower
    // than N = BN up to 128) gives hi.hi in columns [0, BN) and hi.lo in [BN, 2 BN), and a second
    // MMA adds lo.hi to [0, BN): two MMAs per 16-channel step instead of three.
    constexpr bool STACK = BN <= 64;
    constexpr int ACCW = STACK ? 2 * BN : BN;  // columns of one accumulator
    // accumulator buffers in tensor memory: NACC tiles of two accumulators each (the MMAs after a
    // commit inside a tile go to the other one, so they never wait on the committed ones)
    constexpr int TCOLS = MB * 2 * ACCW;
    constexpr int NACC = 512 / TCOLS < 8 ? 512 / TCOLS : 8;
    constexpr int KW = TAPS == 9 ? 3 : 1;       // kernel width when TAPS is fixed
    constexpr uint32_t kCols = NACC * TCOLS <= 32 ? 32 : (NACC * TCOLS <= 64 ? 64 : (NACC * TCOLS <= 128 ? 128 : (NACC * TCOLS <= 256 ? 256 : 512)));
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int SA = p.SA, SB = p.SB;
    uint8_t *bsm = smem + p.b_off;
    uint64_t *fullA = reinterpret_cast<uint64_t *>(smem + p.bar_off);
    uint64_t *emptyA = fullA + SA;
    uint64_t *fullB = emptyA + SA;
    uint64_t *emptyB = fullB + SB;
    uint64_t *tfull = emptyB + SB;
    uint64_t *tempty = tfull + NACC;
    uint64_t *drain = tempty + NACC;
    uint64_t *bres = drain + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bres + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    float *bias_s = reinterpret_cast<float *>(smem + p.bias_off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < p.bias_n; i += blockDim.x) bias_s[i] = p.bias[i];

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; s++) {
            mbar_init(&fullA[s], kProd);
            mbar_init(&emptyA[s], 1);
        }
        for (int s = 0; s < SB; s++) {
            mbar_init(&fullB[s], 1);
            mbar_init(&emptyB[s], 1);
        }
        for (int a = 0; a < NACC; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], TSPLIT ? kEpiWarps / 2 : kEpiWarps);
        }
        mbar_init(drain, 1);
        mbar_init(bres, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == kMmaW) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < kProd) {
        // ---------------- halo producers ----------------
        // thread: whole halo pixels hp = threadIdx.x + 128 i (all 2 NPL 16-byte pieces, hi then
        // lo, each to its plane); consecutive threads take consecutive pixels (coalesced), the
        // pixel slots' halo coordinates are fixed for the launch
        constexpr int kSlots = 4;  // halo pixels per thread (halo_px <= 512, checked on the host)
        int sy[kSlots], sx[kSlots];
#pragma unroll
        for (int i = 0; i < kSlots; i++) {
            const int hp = threadIdx.x + i * kProd * 32;
            sy[i] = hp < p.halo_px ? hp / p.hw_w : -1;  // -1: no pixel
            sx[i] = hp < p.halo_px ? hp - (hp / p.hw_w) * p.hw_w : 0;
        }
        const int64_t xlo = p.x_pix / 2;
        int s = 0, ph = 0, sa = 0, inflight = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
            const Tile tl = decode(p, t);
            const int iy0 = tl.oy0 - p.pt, ix0 = tl.ox0 - p.pl;
            const uint16_t *xb = p.x + (int64_t)tl.nb * p.x_n;
            for (int ch = 0; ch < p.nchunk; ch++) {
                if (!warp_wait(&emptyA[s], ph ^ 1, p.status, abort_flag, 21)) {
                    ok = false;
                    break;
                }
                uint8_t *a = smem + (uint32_t)s * p.a_stage;
#pragma unroll
                for (int i = 0; i < kSlots; i++) {
                    if (sy[i] < 0) continue;
                    const int iy = iy0 + sy[i], ix = ix0 + sx[i];
                    const bool v = iy >= 0 && iy < p.h && ix >= 0 && ix < p.w;
                    const uint16_t *src = v ? xb + ((int64_t)iy * p.w + ix) * p.x_pix + ch * CG : p.x;
                    uint8_t *dst = a + (uint32_t)(threadIdx.x + i * kProd * 32) * 16;
#pragma unroll
                    for (int j = 0; j < NPL; j++) {
                        const int left = (p.cin - (ch * CG + j * 8)) * 2;
                        const uint32_t nb = v && left > 0 ? (left < 16 ? (uint32_t)left : 16u) : 0u;
                        cp_async16(dst + (uint32_t)j * p.plane, nb ? src + j * 8 : p.x, nb);
                        cp_async16(dst + (uint32_t)(NPL + j) * p.plane, nb ? src + xlo + j * 8 : p.x, nb);
                    }
                }
                cp_async_commit();
                if (inflight == p.lag) {
                    // the oldest stage in flight has landed: publish it to the tensor cores
                    cp_async_wait(p.lag);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&fullA[sa]);
                    if (++sa == SA) sa = 0;
                } else {
                    inflight++;
                }
                if (++s == SA) {
                    s = 0;
                    ph ^= 1;
                }
            }
        }
        // the stages still in flight
        cp_async_wait(0);
        fence_async_smem();
        __syncwarp();
        for (; inflight > 0; inflight--) {
            if (lane == 0) mbar_arrive(&fullA[sa]);
            if (++sa == SA) sa = 0;
        }
    } else if (warp == kTmaW) {
        // ---------------- B loader ----------------
        if (lane == 0) {
            if (p.b_res) {
                // every (N tile, tap, chunk) of the weights, once
                mbar_expect_tx(bres, (uint32_t)p.ntn * p.taps * p.nchunk * 2 * B_BYTES);
                for (int nt = 0; nt < p.ntn; nt++)
                    for (int tap = 0; tap < p.taps; tap++)
                        for (int ch = 0; ch < p.nchunk; ch++) {
                            uint8_t *dst = bsm + (uint32_t)((nt * p.taps + tap) * p.nchunk + ch) * 2 * B_BYTES;
                            const int kx0 = tap * p.cin_pad + ch * CG;
                            tma_load_2d(dst, &wb_hi, bres, kx0, nt * BN);
                            tma_load_2d(dst + B_BYTES, &wb_lo, bres, kx0, nt * BN);
                        }
                long long t0 = clock64();
                while (!mbar_try(bres, 0) && clock64() - t0 < kWaitBudget) {
                }
            } else {
                int s = 0, ph = 0, issued = 0;
                bool ok = true;
                for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
                    const Tile tl = decode(p, t);
                    for (int ch = 0; ch < p.nchunk && ok; ch++, issued++) {
                        // one stage: every tap of the chunk, hi and lo
                        if (!mbar_wait_spin(&emptyB[s], ph ^ 1, p.status, abort_flag, 22)) {
                            ok = false;
                            break;
                        }
                        uint8_t *dst = bsm + (uint32_t)s * p.b_stage;
                        mbar_expect_tx(&fullB[s], (uint32_t)p.taps * 2 * B_BYTES);
                        for (int tap = 0; tap < p.taps; tap++) {
                            const int kx0 = tap * p.cin_pad + ch * CG;
                            tma_load_2d(dst + (uint32_t)tap * 2 * B_BYTES, &wb_hi, &fullB[s], kx0, tl.nt * BN);
                            tma_load_2d(dst + (uint32_t)tap * 2 * B_BYTES + B_BYTES, &wb_lo, &fullB[s], kx0, tl.nt * BN);
                        }
                        if (++s == SB) {
                            s = 0;
                            ph ^= 1;
                        }
                    }
                }
                // drain: the last SB issued loads land before the CTA may exit (bounded)
                for (int j = (issued > SB ? issued - SB : 0); j < issued; j++) {
                    long long t0 = clock64();
                    while (!mbar_try(&fullB[j % SB], (j / SB) & 1) && clock64() - t0 < kWaitBudget) {
                    }
                }
            }
        }
    } else if (warp == kMmaW) {
        // ---------------- MMA issue ----------------
        // Descriptors are built once per stage and advanced by adding 16-byte units to their start
        // address field; with TAPS fixed the tap loop unrolls into constant offsets.
        if (lane == 0) {
            const uint32_t idesc = instr_desc(BN), idesc2 = instr_desc(STACK ? 2 * BN : BN);
            const uint32_t plane16 = p.plane >> 4, b16 = B_BYTES >> 4;
            const uint32_t sbo = (uint32_t)p.hw_w * 16;  // one halo row per 8-row group
            const uint32_t blk16 = (uint32_t)(TR * p.hw_w);  // next MMA block: TR halo rows further
            const uint32_t bsm32 = smem_u32(bsm);
            const uint64_t tap_b16 = (uint64_t)p.nchunk * 2 * b16;  // resident B: next tap
            const int taps = TAPS ? TAPS : p.taps, kw = TAPS ? KW : p.kw, hw_w = TAPS ? KW + TP - 1 : p.hw_w;
            bool ok = !p.b_res || mbar_wait(bres, 0, p.status, abort_flag, 27);
            // A start offsets (16-byte units) of the hi and lo planes of each 16-channel step
            uint32_t ahi_off[CG / 16], alo_off[CG / 16];
#pragma unroll
            for (int kk = 0; kk < CG / 16; kk++) {
                ahi_off[kk] = 2 * kk * plane16;
                alo_off[kk] = (NPL + 2 * kk) * plane16;
            }
            int sa = 0, pha = 0, sb = 0, phb = 0, lt = 0;
            for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x, lt++) {
                const int ab = lt % NACC;
                const uint32_t dtile = tmem + ab * TCOLS;
                const int nt = t - (int)(p.div_ntn.div((uint32_t)t) * p.div_ntn.d);
                ok = mbar_wait_spin(&tempty[ab], ((lt / NACC) & 1) ^ 1, p.status, abort_flag, 26);
                if (!ok) break;
                tc_fence_after();
                if (p.b_res) {
                    // resident B: the only commits inside a tile end a chunk; chunks alternate
                    // between the two accumulators, the first two chunks start them
                    for (int ch = 0; ch < p.nchunk && ok; ch++) {
                        ok = mbar_wait_spin(&fullA[sa], pha, p.status, abort_flag, 23);
                        if (!ok) break;
                        tc_fence_after();
                        const uint64_t da0 = smem_desc_plain(smem_u32(smem + (uint32_t)sa * p.a_stage), p.plane, sbo);
                        uint64_t db = smem_desc_sw(bsm32 + (uint32_t)(nt * taps * p.nchunk + ch) * 2 * B_BYTES, RB);
                        const uint32_t d = dtile + (ch & 1) * ACCW;
                        const uint32_t acc0 = ch >= 2 ? 1u : 0u;
#pragma unroll
                        for (int tap = 0; tap < (TAPS ? TAPS : 64); tap++) {
                            if (!TAPS && tap >= taps) break;
#pragma unroll
                            for (int b = 0; b < MB; b++) {
                                const uint64_t da = da0 + (uint32_t)((tap / kw) * hw_w + tap % kw) + b * blk16;
                                const uint32_t db_d = d + b * 2 * ACCW;
#pragma unroll
                                for (int kk = 0; kk < CG / 16; kk++) {
                                    const uint32_t acc = tap == 0 && kk == 0 ? acc0 : 1u;
                                    if (STACK) {
                                        umma(db_d, da + ahi_off[kk], db + 2 * kk, idesc2, acc);  // hi . [hi; lo]
                                        umma(db_d, da + alo_off[kk], db + 2 * kk, idesc, 1u);    // lo . hi
                                    } else {
                                        umma(db_d, da + ahi_off[kk], db + 2 * kk, idesc, acc);
                                        umma(db_d, da + ahi_off[kk], db + b16 + 2 * kk, idesc, 1u);
                                        umma(db_d, da + alo_off[kk], db + 2 * kk, idesc, 1u);
                                    }
                                }
                            }
                            db += tap_b16;
                        }
                        umma_commit(&emptyA[sa]);
                        if (++sa == SA) {
                            sa = 0;
                            pha ^= 1;
                        }
                    }
                } else {
                    // B through the ring, a stage per chunk with all its taps: one wait and one
                    // commit per chunk; chunks alternate between the two accumulators
                    for (int ch = 0; ch < p.nchunk && ok; ch++) {
                        ok = mbar_wait_spin(&fullA[sa], pha, p.status, abort_flag, 23) &&
                             mbar_wait_spin(&fullB[sb], phb, p.status, abort_flag, 24);
                        if (!ok) break;
                        tc_fence_after();
                        const uint64_t da0 = smem_desc_plain(smem_u32(smem + (uint32_t)sa * p.a_stage), p.plane, sbo);
                        uint64_t db = smem_desc_sw(bsm32 + (uint32_t)sb * p.b_stage, RB);
                        const uint32_t d = dtile + (ch & 1) * ACCW;
                        const uint32_t acc0 = ch >= 2 ? 1u : 0u;
#pragma unroll
                        for (int tap = 0; tap < (TAPS ? TAPS : 64); tap++) {
                            if (!TAPS && tap >= taps) break;
#pragma unroll
                            for (int b = 0; b < MB; b++) {
                                const uint64_t da = da0 + (uint32_t)((tap / kw) * hw_w + tap % kw) + b * blk16;
                                const uint32_t db_d = d + b * 2 * ACCW;
#pragma unroll
                                for (int kk = 0; kk < CG / 16; kk++) {
                                    const uint32_t acc = tap == 0 && kk == 0 ? acc0 : 1u;
                                    if (STACK) {
                                        umma(db_d, da + ahi_off[kk], db + 2 * kk, idesc2, acc);
                                        umma(db_d, da + alo_off[kk], db + 2 * kk, idesc, 1u);
                                    } else {
                                        umma(db_d, da + ahi_off[kk], db + 2 * kk, idesc, acc);
                                        umma(db_d, da + ahi_off[kk], db + b16 + 2 * kk, idesc, 1u);
                                        umma(db_d, da + alo_off[kk], db + 2 * kk, idesc, 1u);
                                    }
                                }
                            }
                            db += 2 * b16;
                        }
                        umma_commit(&emptyB[sb]);
                        if (++sb == SB) {
                            sb = 0;
                            phb ^= 1;
                        }
                        umma_commit(&emptyA[sa]);
                        if (++sa == SA) {
                            sa = 0;
                            pha ^= 1;
                        }
                    }
                }
                if (ok) umma_commit(&tfull[ab]);
            }
            // every issued MMA completes before the shared and tensor memory go away (bounded)
            umma_commit(drain);
            long long t0 = clock64();
            while (!mbar_try(drain, 0) && clock64() - t0 < kWaitBudget) {
            }
        }
    } else {
        // ---------------- epilogue: warps 4-11, lane quadrant warp % 4, column half ----------------
        const int q = warp & 3, half = (warp - kEpi0) >> 2;
        const int row = q * 32 + lane;
        // MB = 2: half h takes MMA block h (image rows 16 h .. 16 h + 15 of the tile), all columns
        const int blk = MB == 2 ? half : 0;
        const int r = row / TP + TR * blk, pc = row % TP;
        uint4 *stg = reinterpret_cast<uint4 *>(smem + p.stg_off) + (warp - kEpi0) * 128;
        int lt = 0;
        for (int t = blockIdx.x; t < p.ntiles; t += gridDim.x, lt++) {
            if (TSPLIT && (lt & 1) != half) continue;
            const int ab = lt % NACC;
            if (!warp_wait(&tfull[ab], (lt / NACC) & 1, p.status, abort_flag, 25)) break;
            tc_fence_after();
            const Tile tl = decode(p, t);
            const int oy = tl.oy0 + r, ox = tl.ox0 + pc;
            const bool valid = oy < p.oh && ox < p.ow;
#pragma unroll 1
            for (int c0 = TSPLIT || MB == 2 ? 0 : half * 16; c0 < BN; c0 += TSPLIT || MB == 2 ? 16 : 32) {
                float v[16];
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * TCOLS + blk * 2 * ACCW + c0;
                if (STACK) {
                    if (p.two_acc) tmem_ld16_sum4(tbase, tbase + BN, tbase + ACCW, tbase + ACCW + BN, v);
                    else tmem_ld16_sum2(tbase, tbase + BN, v);
                } else {
                    if (p.two_acc) tmem_ld16_sum2(tbase, tbase + ACCW, v);
                    else tmem_ld16(tbase, v);
                }
                const int col = tl.nt * BN + c0;
                if (p.pool_y && col + 16 <= p.N) {
                    // plain store and the fused 2 x 2 MaxPool: every lane takes part in the
                    // shuffles (lanes l, l + 1, l + 8, l + 9 hold a window), the window's top-left
                    // lane stores the maximum
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) v[jj] += bias_s[col + jj];
                    act_n(v, p.act);
                    const int64_t off = (int64_t)tl.nb * p.y_n + ((int64_t)oy * p.ow_out + ox) * p.y_pix + col;
                    if (p.stg_off) store16_t(p, off, valid, v, stg, lane);
                    else if (valid) store16(p, off, v);
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) {
                        float a = fmaxf(v[jj], __shfl_down_sync(0xffffffffu, v[jj], 1));
                        v[jj] = fmaxf(a, __shfl_down_sync(0xffffffffu, a, 8));
                    }
                    if (valid && !(oy & 1) && !(ox & 1) && oy + 1 < p.oh && ox + 1 < p.ow)
                        store_pool(p, (int64_t)tl.nb * p.pool_n + ((int64_t)(oy >> 1) * (p.ow >> 1) + (ox >> 1)) * p.pool_pix +
                                          col,
                                   v);
                    continue;
                }
                if (p.stg_off && col + 16 <= p.N && (!p.scatter || p.scat_cout % 16 == 0)) {
                    // whole 16-channel chunk: every lane takes part in the transposed store
                    int64_t off;
                    int b0 = col;
                    if (p.scatter) {
                        // a 16-column chunk lies in one tap: 16 channels of pixel (s oy + ky, s ox + kx)
                        const int sc = p.scatter, tap = col / p.scat_cout;
                        b0 = col - tap * p.scat_cout;
                        off = (int64_t)tl.nb * p.y_n +
                              ((int64_t)(oy * sc + tap / sc) * p.ow_out + ox * sc + tap % sc) * p.y_pix + b0;
                    } else {
                        off = (int64_t)tl.nb * p.y_n + ((int64_t)oy * p.ow_out + ox) * p.y_pix + col;
                    }
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) v[jj] += bias_s[b0 + jj];
                    act_n(v, p.act);
                    store16_t(p, off, valid, v, stg, lane);
                    continue;
                }
                if (!valid || col >= p.N) continue;
                if (p.scatter) {
                    const int sc = p.scatter;
                    if (p.scat_cout % 16 == 0) {
                        // a 16-column chunk lies in one tap: 16 channels of pixel (s oy + ky, s ox + kx)
                        const int tap = col / p.scat_cout, co0 = col - tap * p.scat_cout;
                        const int yy = oy * sc + tap / sc, xx = ox * sc + tap % sc;
#pragma unroll
                        for (int jj = 0; jj < 16; jj++) v[jj] += bias_s[co0 + jj];
                        act_n(v, p.act);
                        store16(p, (int64_t)tl.nb * p.y_n + ((int64_t)yy * p.ow_out + xx) * p.y_pix + co0, v);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 16; jj++) {
                            const int cc = col + jj < p.N ? col + jj : p.N - 1;
                            v[jj] += bias_s[cc - cc / p.scat_cout * p.scat_cout];
                        }
                        act_n(v, p.act);
#pragma unroll
                        for (int jj = 0; jj < 16; jj++) {
                            if (col + jj >= p.N) continue;
                            const int cc = col + jj, tap = cc / p.scat_cout, co = cc - tap * p.scat_cout;
                            const int yy = oy * sc + tap / sc, xx = ox * sc + tap % sc;
                            store1(p, (int64_t)tl.nb * p.y_n + ((int64_t)yy * p.ow_out + xx) * p.y_pix + co, v[jj]);
                        }
                    }
                    continue;
                }
                const int64_t off = (int64_t)tl.nb * p.y_n + ((int64_t)oy * p.ow_out + ox) * p.y_pix + col;
                if (col + 16 <= p.N) {
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) v[jj] += bias_s[col + jj];
                    act_n(v, p.act);
                    store16(p, off, v);
                } else {
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) v[jj] += col + jj < p.N ? bias_s[col + jj] : 0.f;
                    act_n(v, p.act);
#pragma unroll
                    for (int jj = 0; jj < 16; jj++)
                        if (col + jj < p.N) store1(p, off + jj, v[jj]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[ab]);  // one arrival per warp
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaW) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
    }
}

// ---------------------------------------------------------------------------------------------
// Row kernel for the narrow 3 x 3 layers (N <= 32 output channels).  There k_tconv's MMAs are
// 128 x 16 (or 32) x 16, and the tensor core's fixed cost per instruction, not its arithmetic,
// sets the pace (18 MMAs per 128-pixel tile at 16 channels in).  Here the three kernel columns
// kx are stacked along N instead.  An MMA block is RX = 8 image rows of RP = 16 positions
// (M = 128, 8-position core-matrix groups, so one halo row is 256 bytes and kernel row dy is the
// same halo RP * dy 16-byte units further); B is [w_hi(kx = 0, 1, 2); w_lo(kx = 0, 1, 2)] for C =
// 16 or 32 output channels.  Per kernel row and 16-channel step:
//   LO (C = 16): hi . [hi; lo] (N = 6 C) and lo . hi (N = 3 C, into the hi columns), the
//                epilogue adding the hi and lo columns: 2 MMAs, 6 C accumulator columns;
//   else (C = 32): hi . hi, hi . lo and lo . hi into the same 3 C columns: 3 MMAs, 3 C columns.
// Position j of a row accumulates, per kx, the kernel-row sums for input column x0 + j; output
// column x0 + i is the sum over kx of those at position i + kx, gathered by the epilogue with two
// warp shuffles (a warp's 32 lanes are two rows of 16 positions).  Positions 14 and 15 only feed
// that sum, so tiles advance RV = 14 columns.  The fused 2 x 2 MaxPool is a reduce-scatter over
// each window's lanes l, l + 1, l + 16, l + 17, after which each of them stores 4 channels.
//
// The halo comes by TMA, one 4-D box (channels x RP positions x RX + 2 rows) per split part, in
// the K-major swizzled layout whose rows are pixels of CG channels (CG = 16, 32, 64: 32-, 64-,
// 128-byte swizzle): a kernel row is 16 pixel rows, two whole swizzle atoms, further; zeros
// outside the image and past cin come from the TMA bounds.  WHOLE: the view is its whole buffer
// (a pixel is cin hi parts then cin lo parts, cin = CG <= 32), so one box of whole pixels (64- or
// 128-byte rows) brings both parts, the lo part CG elements along the row: half the TMA lines,
// twice as long, whose rate bounds these layers.
//
// Warp roles (512 threads): warp 0 halo TMA, warp 1 tensor-memory allocation and MMA issue,
// warps 4-15 three epilogue groups of four (one per lane quadrant) taking every third tile.  B (at
// most 72 KB) is copied into shared memory once.  Every barrier check or commit on the MMA thread
// stalls its issue (an MMA is only accepted when the tensor core takes it, so the pipe drains
// meanwhile: about 100 cycles a check), so the thread has one of each per tile: the TMA thread
// loads a tile's halo only once the tile's accumulator buffer is free, making the stage's full
// barrier mean both, and the epilogue group that sees a tile's MMAs complete releases its stage.
constexpr int RX = 8, RP = 16, RV = 14;
constexpr int kRGroups = 3, kRTmaW = 0, kRMmaW = 1, kRThreads = 32 * (4 + 4 * kRGroups);

__device__ __forceinline__ Tile decode_rows(const TcP &p, int t) {
    Tile r;
    const uint32_t q1 = p.div_tx.div((uint32_t)t), q2 = p.div_ty.div(q1);
    r.nt = 0;
    r.ox0 = (t - (int)(q1 * p.div_tx.d)) * p.tile_w;
    r.oy0 = (int)(q1 - q2 * p.div_ty.d) * RX;
    r.nb = (int)q2;
    return r;
}

// fused 2 x 2 MaxPool of 16 channels held by the lanes of each window (l, l + 1, l + 16, l + 17,
// l even and below 16): after two exchange-and-max steps lane (odd, upper) holds the window's
// channels 8 odd + 4 upper .. + 3, which it stores
__device__ __forceinline__ void pool_rows(const TcP &p, const float (&v)[16], int lane, int64_t off, bool store) {
    const bool odd = lane & 1, up = lane & 16;
    float k8[8], k4[4];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float send = odd ? v[i] : v[8 + i];
        const float got = __shfl_xor_sync(0xffffffffu, send, 1);
        k8[i] = fmaxf(odd ? v[8 + i] : v[i], got);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float send = up ? k8[i] : k8[4 + i];
        const float got = __shfl_xor_sync(0xffffffffu, send, 16);
        k4[i] = fmaxf(up ? k8[4 + i] : k8[i], got);
    }
    if (!store) return;
    off += (odd ? 8 : 0) + (up ? 4 : 0);
    if (p.pool_split) {
        uint16_t *y = reinterpret_cast<uint16_t *>(p.pool_y);
        uint32_t h[2], l[2];
#pragma unroll
        for (int i = 0; i < 2; i++) {
            __nv_bfloat162 hv = __floats2bfloat162_rn(k4[2 * i], k4[2 * i + 1]);
            float2 hf = __bfloat1622float2(hv);
            __nv_bfloat162 lv = __floats2bfloat162_rn(k4[2 * i] - hf.x, k4[2 * i + 1] - hf.y);
            h[i] = *reinterpret_cast<uint32_t *>(&hv);
            l[i] = *reinterpret_cast<uint32_t *>(&lv);
        }
        if (p.pool_vec) {
            *reinterpret_cast<uint2 *>(y + off) = make_uint2(h[0], h[1]);
            *reinterpret_cast<uint2 *>(y + off + p.pool_pix / 2) = make_uint2(l[0], l[1]);
        } else {
            uint16_t *dh = y + off, *dl = y + off + p.pool_pix / 2;
#pragma unroll
            for (int i = 0; i < 2; i++) {
                dh[2 * i] = (uint16_t)(h[i] & 0xffffu);
                dh[2 * i + 1] = (uint16_t)(h[i] >> 16);
                dl[2 * i] = (uint16_t)(l[i] & 0xffffu);
                dl[2 * i + 1] = (uint16_t)(l[i] >> 16);
            }
        }
    } else {
        float *y = reinterpret_cast<float *>(p.pool_y) + off;
        if (p.pool_vec) {
            *reinterpret_cast<float4 *>(y) = make_float4(k4[0], k4[1], k4[2], k4[3]);
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) y[i] = k4[i];
        }
    }
}

// CT: the ConvTranspose with kernel == stride 2 instead, a 1 x 1 GEMM whose four taps (ky, kx)
// are stacked along N the way the kernel columns are (B rows v 4 C + (2 ky + kx) C + c): no halo
// (tiles of 8 rows x 16 pixels, all output), one MMA pair (or triple) per 16-channel step, and an
// epilogue that writes each tap's channels to output pixel (2 y + ky, 2 x + kx).
template <int C, int CG, bool LO, bool WHOLE, bool CT>
__global__ void __launch_bounds__(kRThreads, 1)
    k_tconv_rows(const __grid_constant__ CUtensorMap x_hi, const __grid_constant__ CUtensorMap x_lo,
                 const uint16_t *__restrict__ wx, TcP p) {
    constexpr int NPL = CG / 8;                 // 8-channel planes per split part
    constexpr int T = CT ? 4 : 3;               // kernel columns (or taps) stacked along N
    constexpr int DY = CT ? 1 : 3;              // kernel rows (MMA blocks shifted by a halo row)
    constexpr int NB = 2 * T * C;               // B rows
    constexpr int TCOLS = LO ? 2 * T * C : T * C;  // accumulator columns of a tile
    constexpr int NACC = 512 / TCOLS < 8 ? 512 / TCOLS : 8;
    constexpr uint32_t kCols = NACC * TCOLS <= 128 ? 128 : (NACC * TCOLS <= 256 ? 256 : 512);
    constexpr uint32_t B_BYTES = (uint32_t)DY * NPL * NB * 16;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int SA = p.SA;
    uint8_t *bsm = smem + p.b_off;
    uint64_t *fullA = reinterpret_cast<uint64_t *>(smem + p.bar_off);
    uint64_t *emptyA = fullA + SA;
    uint64_t *tfull = emptyA + SA;
    uint64_t *tempty = tfull + NACC;
    uint64_t *drain = tempty + NACC;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    float *bias_s = reinterpret_cast<float *>(smem + p.bias_off);
    float *head_s = reinterpret_cast<float *>(smem + p.head_off);  // [C][4] weights, then 4 biases
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < p.bias_n; i += blockDim.x) bias_s[i] = p.bias[i];
    if (p.head_y)
        for (int i = threadIdx.x; i < C * 4 + 4; i += blockDim.x) {
            const int c = i >> 2, co = i & 3;
            head_s[i] = c < C ? (c < p.N && co < p.head_n ? p.head_w[(int64_t)c * p.head_ldw + co] : 0.f)
                              : (co < p.head_n ? p.head_b[co] : 0.f);
        }
    {
        // the stacked weights, resident for the whole kernel: generic stores, made visible to
        // the tensor cores by each writer's proxy fence before the barrier
        const uint4 *src = reinterpret_cast<const uint4 *>(wx);
        uint4 *dst = reinterpret_cast<uint4 *>(bsm);
        for (int i = threadIdx.x; i < (int)(B_BYTES / 16); i += blockDim.x) dst[i] = src[i];
        fence_async_smem();
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; s++) {
            mbar_init(&fullA[s], 1);
            mbar_init(&emptyA[s], 1);
        }
        for (int a = 0; a < NACC; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == kRMmaW) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kRTmaW) {
        // ---------------- halo TMA: the hi and the lo part of a tile's halo per stage ----------------
        if (lane == 0) {
            const uint32_t part = p.a_stage / 2;
            int s = 0, ph = 0, issued = 0;
            for (int t = blockIdx.x; t < p.ntiles; t += gridDim.x) {
                const Tile tl = decode_rows(p, t);
                if (!mbar_wait_spin(&emptyA[s], ph ^ 1, p.status, abort_flag, 31)) break;
                // the tile's accumulator buffer is free (its previous tile's epilogue is done)
                if (!mbar_wait_spin(&tempty[issued % NACC], ((issued / NACC) & 1) ^ 1, p.status, abort_flag, 36)) break;
                uint8_t *a = smem + (uint32_t)s * p.a_stage;
                mbar_expect_tx(&fullA[s], p.a_stage);
                tma_load_4d(a, &x_hi, &fullA[s], 0, tl.ox0 - p.pl, tl.oy0 - p.pt, tl.nb);
                if (!WHOLE) tma_load_4d(a + part, &x_lo, &fullA[s], 0, tl.ox0 - p.pl, tl.oy0 - p.pt, tl.nb);
                issued++;
                if (++s == SA) {
                    s = 0;
                    ph ^= 1;
                }
            }
            // the loads still in flight land before the CTA may exit (bounded)
            for (int k = (issued > SA ? issued - SA : 0); k < issued; k++) {
                long long t0 = clock64();
                while (!mbar_try(&fullA[k % SA], (k / SA) & 1) && clock64() - t0 < kWaitBudget) {
                }
            }
        }
    } else if (warp == kRMmaW) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            constexpr uint32_t idesc_w = instr_desc(NB), idesc_3 = instr_desc(T * C);
            constexpr int ROWB = WHOLE ? 4 * CG : 2 * CG;  // bytes of a halo pixel row
            // the lo part: CG elements along the row, or half a stage further
            const uint32_t lo16 = WHOLE ? CG / 8 : p.a_stage >> 5;
            const uint64_t db0 = smem_desc_plain(smem_u32(bsm), NB * 16, 128);
            int sa = 0, pha = 0;
            bool ok = true;
            for (int t = blockIdx.x, lt = 0; t < p.ntiles && ok; t += gridDim.x, lt++) {
                const int ab = lt % NACC;
                // the halo has landed and the accumulator buffer is free
                ok = mbar_wait_spin(&fullA[sa], pha, p.status, abort_flag, 33);
                if (!ok) break;
                tc_fence_after();
                const uint64_t da0 = smem_desc_sw(smem_u32(smem + (uint32_t)sa * p.a_stage), ROWB);
                const uint32_t d = tmem + ab * TCOLS;
#pragma unroll
                for (int dy = 0; dy < DY; dy++)
#pragma unroll
                    for (int kk = 0; kk < CG / 16; kk++) {
                        // kernel row dy: RP pixel rows further; 16 channels: 32 bytes
                        const uint64_t da = da0 + (uint32_t)(dy * RP * ROWB / 16) + 2 * kk;
                        const uint64_t db = db0 + (uint32_t)((dy * NPL + 2 * kk) * NB);
                        const uint32_t acc = dy == 0 && kk == 0 ? 0u : 1u;
                        if (LO) {
                            umma(d, da, db, idesc_w, acc);                     // hi . [hi; lo]
                            umma(d, da + lo16, db, idesc_3, 1u);               // lo . hi
                        } else {
                            umma(d, da, db, idesc_3, acc);                     // hi . hi
                            umma(d, da, db + T * C, idesc_3, 1u);              // hi . lo
                            umma(d, da + lo16, db, idesc_3, 1u);               // lo . hi
                        }
                    }
                if (++sa == SA) {
                    sa = 0;
                    pha ^= 1;
                }
                umma_commit(&tfull[ab]);  // the epilogue group then releases the stage
            }
            umma_commit(drain);
            long long t0 = clock64();
            while (!mbar_try(drain, 0) && clock64() - t0 < kWaitBudget) {
            }
        }
    } else {
        // ---------------- epilogue group g: tiles lt = g (mod 3), lane quadrant warp % 4 ----------------
        const int q = warp & 3, g = (warp - 4) >> 2;
        const int r = 2 * q + (lane >> 4), j = lane & 15;
        uint4 *stg = reinterpret_cast<uint4 *>(smem + p.stg_off) + (warp - 4) * 128;
        int lt = 0;
        for (int t = blockIdx.x; t < p.ntiles; t += gridDim.x, lt++) {
            if (lt % kRGroups != g) continue;
            const int ab = lt % NACC;
            if (!warp_wait(&tfull[ab], (lt / NACC) & 1, p.status, abort_flag, 35)) break;
            tc_fence_after();
            // the tile's MMAs are complete: its halo stage may be refilled
            if (q == 0 && lane == 0) mbar_arrive(&emptyA[lt % SA]);
            const Tile tl = decode_rows(p, t);
            if constexpr (CT) {
                // ConvTranspose: tap tp = 2 ky + kx of input pixel (iy, ix) is output (2 iy + ky, 2 ix + kx)
                const int iy = tl.oy0 + r, ix = tl.ox0 + j;
                const bool in_ok = iy < p.oh && ix < p.ow;
#pragma unroll 1
                for (int tp = 0; tp < 4; tp++)
#pragma unroll 1
                    for (int c0 = 0; c0 < C; c0 += 16) {
                        const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + ab * TCOLS + tp * C + c0;
                        float v[16];
                        if (LO) tmem_ld16_sum2(tb, tb + T * C, v);  // hi + lo columns
                        else tmem_ld16(tb, v);
                        if (c0 >= p.scat_cout) continue;  // padding columns
#pragma unroll
                        for (int jj = 0; jj < 16; jj++) v[jj] += bias_s[c0 + jj];
                        act_n(v, p.act);
                        const int yy = 2 * iy + (tp >> 1), xx = 2 * ix + (tp & 1);
                        const int64_t off = (int64_t)tl.nb * p.y_n + ((int64_t)yy * p.ow_out + xx) * p.y_pix + c0;
                        if (p.stg_off && c0 + 16 <= p.scat_cout) {
                            store16_t(p, off, in_ok, v, stg, lane);
                        } else if (in_ok) {
#pragma unroll
                            for (int jj = 0; jj < 16; jj++)
                                if (c0 + jj < p.scat_cout) store1(p, off + jj, v[jj]);
                        }
                    }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[ab]);
                continue;
            }
            const int oy = tl.oy0 + r, ox = tl.ox0 + j;
            const bool valid = j < RV && oy < p.oh && ox < p.ow;
            float hacc[4];
#pragma unroll
            for (int co = 0; co < 4; co++) hacc[co] = head_s[C * 4 + co];
#pragma unroll 1
            for (int c0 = 0; c0 < C; c0 += 16) {
                const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + ab * TCOLS + c0;
                float v[16], s1[16], s2[16];
                if (LO) {
                    tmem_ld16_sum2(tb + C, tb + 4 * C, s1);      // kx = 1: hi + lo columns
                    tmem_ld16_sum2(tb + 2 * C, tb + 5 * C, s2);  // kx = 2
                    tmem_ld16_sum2(tb, tb + 3 * C, v);           // kx = 0
                } else {
                    tmem_ld16x3(tb, tb + C, tb + 2 * C, v, s1, s2);
                }
                const int col = c0;
                const float4 *b4 = reinterpret_cast<const float4 *>(bias_s + col);
#pragma unroll
                for (int jj = 0; jj < 16; jj += 2) {
                    const float2 sh = __fadd2_rn(make_float2(__shfl_down_sync(0xffffffffu, s1[jj], 1),
                                                             __shfl_down_sync(0xffffffffu, s1[jj + 1], 1)),
                                                 make_float2(__shfl_down_sync(0xffffffffu, s2[jj], 2),
                                                             __shfl_down_sync(0xffffffffu, s2[jj + 1], 2)));
                    const float4 bb = b4[jj >> 2];
                    const float2 bj = (jj & 2) ? make_float2(bb.z, bb.w) : make_float2(bb.x, bb.y);
                    const float2 o = __fadd2_rn(__fadd2_rn(make_float2(v[jj], v[jj + 1]), sh), bj);
                    v[jj] = o.x;
                    v[jj + 1] = o.y;
                }
                act_n(v, p.act);
                if (p.head_y) {
                    // the 1 x 1 head, channels in order as k_pointwise sums them; no output stored
#pragma unroll
                    for (int jj = 0; jj < 16; jj++)
                        if (c0 + jj < p.N)  // past N: padding columns, not channels
#pragma unroll
                            for (int co = 0; co < 4; co++) hacc[co] += v[jj] * head_s[(c0 + jj) * 4 + co];
                    continue;
                }
                const int64_t off = (int64_t)tl.nb * p.y_n + ((int64_t)oy * p.ow_out + ox) * p.y_pix + col;
                if (p.stg_off && col + 16 <= p.N) {
                    store16_t(p, off, valid, v, stg, lane);
                    if (!p.pool_y) continue;
                }
                if (p.pool_y) {
                    // N % 16 == 0 (checked on the host): every chunk is whole
                    if (!p.stg_off && valid) store16(p, off, v);
                    const bool wv = j < RV && (oy | 1) < p.oh && (ox | 1) < p.ow;
                    pool_rows(p, v, lane,
                              (int64_t)tl.nb * p.pool_n + ((int64_t)(oy >> 1) * (p.ow >> 1) + (ox >> 1)) * p.pool_pix + col,
                              wv);
                    continue;
                }
                if (!valid || col >= p.N) continue;
                if (col + 16 <= p.N) {
                    store16(p, off, v);
                } else {
#pragma unroll
                    for (int jj = 0; jj < 16; jj++)
                        if (col + jj < p.N) store1(p, off + jj, v[jj]);
                }
            }
            if (p.head_y && valid) {
                float *hy = p.head_y + (int64_t)tl.nb * p.head_y_n + ((int64_t)oy * p.ow + ox) * p.head_y_pix;
#pragma unroll
                for (int co = 0; co < 4; co++)
                    if (co < p.head_n) hy[co] = act_f(hacc[co], p.head_act);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[ab]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kRMmaW) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
    }
}

CUtensorMapSwizzle swizzle_of(int cg) {
    return cg == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : (cg == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
}

void encode(CUtensorMap *map, int rank, void *base, const cuuint64_t *dims, const cuuint64_t *strides,
            const cuuint32_t *box, int cg) {
    auto fn = encode_fn();
    if (!fn) fail(WOCR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_of(cg), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(WOCR_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

template <int BN, int CG, int TAPS, int MB>
void launch(Ctx *c, const TconvW &w, const TcP &p, int smem) {
    static std::atomic<bool> set[64];
    if (!set[c->device]) {
        WOCR_CUDA(cudaFuncSetAttribute(k_tconv<BN, CG, TAPS, MB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       227 * 1024));
        set[c->device] = true;
    }
    unsigned grid = (unsigned)std::min<int64_t>(p.ntiles, c->sm_count);
    k_tconv<BN, CG, TAPS, MB><<<grid, kThreads, smem, c->stream>>>(w.map_hi, w.map_lo, p);
    WOCR_LAUNCHED(c);
}

template <int CG, int TAPS>
void launch_bn(Ctx *c, const TconvW &w, const TcP &p, int smem) {
    const bool two = p.trows == 2 * TR;
    switch (w.bn) {
    case 16: two ? launch<16, CG, TAPS, 2>(c, w, p, smem) : launch<16, CG, TAPS, 1>(c, w, p, smem); break;
    case 32: two ? launch<32, CG, TAPS, 2>(c, w, p, smem) : launch<32, CG, TAPS, 1>(c, w, p, smem); break;
    case 64: launch<64, CG, TAPS, 1>(c, w, p, smem); break;
    default: launch<128, CG, TAPS, 1>(c, w, p, smem); break;
    }
}

template <int CG>
void launch_taps(Ctx *c, const TconvW &w, const TcP &p, int smem, int kh, int kw) {
    if (kh == 3 && kw == 3) launch_bn<CG, 9>(c, w, p, smem);
    else if (kh == 1 && kw == 1) launch_bn<CG, 1>(c, w, p, smem);
    else launch_bn<CG, 0>(c, w, p, smem);
}

int tconv_bn(int N) { return N <= 16 ? 16 : N <= 32 ? 32 : N <= 64 ? 64 : 128; }

template <int C, int CG, bool WHOLE, bool CT>
void launch_rows(Ctx *c, const TconvW &w, const TcP &p, int smem, const CUtensorMap *xm) {
    constexpr bool LO = C == 16;  // 2 MMAs over 2 T C columns; C = 32: 3 MMAs over T C columns
    static std::atomic<bool> set[64];
    if (!set[c->device]) {
        WOCR_CUDA(cudaFuncSetAttribute(k_tconv_rows<C, CG, LO, WHOLE, CT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        set[c->device] = true;
    }
    unsigned grid = (unsigned)std::min<int64_t>(p.ntiles, c->sm_count);
    k_tconv_rows<C, CG, LO, WHOLE, CT><<<grid, kRThreads, smem, c->stream>>>(
        xm[0], xm[1], reinterpret_cast<const uint16_t *>(w.x3->p), p);
    WOCR_LAUNCHED(c);
}

template <bool CT>
void launch_rows_ct(Ctx *c, const TconvW &w, const TcP &p, int smem, const CUtensorMap *xm, bool whole) {
    if (w.x3_cout == 16) {
        if (w.x3_cg == 16)
            whole ? launch_rows<16, 16, true, CT>(c, w, p, smem, xm) : launch_rows<16, 16, false, CT>(c, w, p, smem, xm);
        else if (w.x3_cg == 32)
            whole ? launch_rows<16, 32, true, CT>(c, w, p, smem, xm) : launch_rows<16, 32, false, CT>(c, w, p, smem, xm);
        else launch_rows<16, 64, false, CT>(c, w, p, smem, xm);
    } else {
        if (w.x3_cg == 16)
            whole ? launch_rows<32, 16, true, CT>(c, w, p, smem, xm) : launch_rows<32, 16, false, CT>(c, w, p, smem, xm);
        else if (w.x3_cg == 32)
            whole ? launch_rows<32, 32, true, CT>(c, w, p, smem, xm) : launch_rows<32, 32, false, CT>(c, w, p, smem, xm);
        else launch_rows<32, 64, false, CT>(c, w, p, smem, xm);
    }
}

void launch_rows_any(Ctx *c, const TconvW &w, const TcP &p, int smem, const CUtensorMap *xm, bool whole) {
    if (w.x3_ct) launch_rows_ct<true>(c, w, p, smem, xm, whole);
    else launch_rows_ct<false>(c, w, p, smem, xm, whole);
}

// The row kernel's shared memory: A stages, B, barriers, bias, head, store staging (p.out_vec and
// p.bias_n set); false when it does not fit.
bool plan_rows_smem(const TconvW &w, TcP &p, int &smem) {
    const int C = w.x3_cout, CG = w.x3_cg;
    const int T = w.x3_ct ? 4 : 3, DY = w.x3_ct ? 1 : 3, HR = w.x3_ct ? RX : RX + 2;
    p.hw_w = RP;
    p.halo_px = HR * RP;
    p.plane = 0;
    p.a_stage = (uint32_t)(2 * p.halo_px * CG * 2);  // hi part, lo part: multiples of 1024 bytes
    const int b_region = (DY * (CG / 8) * 2 * T * C * 16 + 1023) / 1024 * 1024;
    // transposed-store staging: 2 KB per epilogue warp when the stores are 16-byte aligned
    const int stg = p.out_vec ? kRGroups * 4 * 2048 : 0;
    const int SA = std::min(8, (kSmemBudget - b_region - stg) / (int)p.a_stage);
    if (SA < 2) return false;
    p.SA = SA;
    p.SB = 0;
    p.lag = std::min(kLagMax, SA - 2);
    p.b_off = (uint32_t)SA * p.a_stage;
    p.bar_off = p.b_off + (uint32_t)b_region;
    p.bias_off = p.bar_off + 1024;
    p.head_off = p.bias_off + (uint32_t)((p.bias_n * 4 + 15) / 16 * 16);
    const int head_bytes = (C * 4 + 4) * 4;
    p.stg_off = stg ? p.head_off + (uint32_t)head_bytes : 0;
    smem = (int)p.head_off + head_bytes + stg + 1024;
    return smem <= 227 * 1024;
}

// The row kernel's launch parameters (geometry, tensor maps of the halo, shared memory); false
// when it does not fit.
bool plan_rows(const TconvW &w, const TconvP &q, TcP &p, int &smem, CUtensorMap *xm, bool &whole) {
    const int CG = w.x3_cg, HR = w.x3_ct ? RX : RX + 2;
    p.trows = RX;
    p.tile_w = w.x3_ct ? RP : RV;  // a ConvTranspose tile has no halo: all 16 positions are output
    p.tiles_x = (q.ow + p.tile_w - 1) / p.tile_w;
    p.tiles_y = (q.oh + RX - 1) / RX;
    p.ntn = 1;
    const int64_t ntiles = (int64_t)q.n * p.tiles_x * p.tiles_y;
    if (ntiles >= (int64_t)INT32_MAX) return false;
    p.ntiles = (int)ntiles;
    p.div_ntn = FastDiv(1);
    p.div_tx = FastDiv((uint32_t)p.tiles_x);
    p.div_ty = FastDiv((uint32_t)p.tiles_y);
    if (!plan_rows_smem(w, p, smem)) return false;
    // the halo boxes: [n][h][w][channels < cin] of the hi and of the lo parts, zeros outside
    const cuuint64_t dims[4] = {(cuuint64_t)q.cin, (cuuint64_t)q.w, (cuuint64_t)q.h, (cuuint64_t)q.n};
    const cuuint64_t strides[3] = {(cuuint64_t)q.x_pix * 2, (cuuint64_t)q.w * q.x_pix * 2, (cuuint64_t)q.x_n * 2};
    const cuuint32_t box[4] = {(cuuint32_t)CG, (cuuint32_t)RP, (cuuint32_t)HR, 1};
    whole = CG <= 32 && q.cin == CG && q.x_pix == 2 * CG;
    if (whole) {
        // whole pixels: [n][h][w][2 CG] (the hi and the lo parts), rows of 4 CG bytes
        const cuuint64_t dw[4] = {(cuuint64_t)q.x_pix, (cuuint64_t)q.w, (cuuint64_t)q.h, (cuuint64_t)q.n};
        const cuuint32_t bw[4] = {(cuuint32_t)(2 * CG), (cuuint32_t)RP, (cuuint32_t)HR, 1};
        encode(&xm[0], 4, const_cast<uint16_t *>(q.x), dw, strides, bw, 2 * CG);
        xm[1] = xm[0];
    } else {
        encode(&xm[0], 4, const_cast<uint16_t *>(q.x), dims, strides, box, CG);
        encode(&xm[1], 4, const_cast<uint16_t *>(q.x + q.x_pix / 2), dims, strides, box, CG);
    }
    return true;
}

}  // namespace

TconvW make_tconv_weights(Ctx *c, const std::vector<float> &wnk, int N, int taps, int cin) {
    TconvW w;
    w.N = N;
    w.taps = taps;
    w.cin = cin;
    // the widest chunk that fits in cin (a last partial chunk reads zeros past cin)
    if (cin < 16) fail(WOCR_ERR_UNSUPPORTED, "tap convolution with fewer than 16 input channels");
    w.bn = tconv_bn(N);
    // B through the ring (over 96 KB) with several taps: 16-channel chunks, so a ring stage (every
    // tap of a chunk) stays near 36 KB (N tile 64) or 72 KB (128)
    const int64_t b_all16 = (int64_t)((N + w.bn - 1) / w.bn) * taps * ((cin + 15) / 16 * 16) * w.bn * 4;
    w.cg = cin >= 32 && !(taps > 1 && b_all16 > 96 * 1024) ? 32 : 16;
    w.cin_pad = (cin + w.cg - 1) / w.cg * w.cg;
    const int Npad = (N + w.bn - 1) / w.bn * w.bn;  // every TMA box lies inside the tensor
    const int64_t K = (int64_t)taps * w.cin_pad;
    std::vector<__nv_bfloat16> hi((size_t)Npad * K, __float2bfloat16_rn(0.f)), lo = hi;
    for (int n = 0; n < N; n++)
        for (int t = 0; t < taps; t++)
            for (int ci = 0; ci < cin; ci++) {
                float v = wnk[((size_t)n * taps + t) * cin + ci];
                __nv_bfloat16 h = __float2bfloat16_rn(v);
                size_t o = (size_t)n * K + (size_t)t * w.cin_pad + ci;
                hi[o] = h;
                lo[o] = __float2bfloat16_rn(v - __bfloat162float(h));
            }
    size_t bytes = (size_t)Npad * K * 2;
    w.hi = alloc(c, bytes);
    w.lo = alloc(c, bytes);
    WOCR_CUDA(cudaMemcpyAsync(w.hi->p, hi.data(), bytes, cudaMemcpyHostToDevice, c->stream));
    WOCR_CUDA(cudaMemcpyAsync(w.lo->p, lo.data(), bytes, cudaMemcpyHostToDevice, c->stream));
    WOCR_CUDA(cudaStreamSynchronize(c->stream));
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)Npad};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {(cuuint32_t)w.cg, (cuuint32_t)w.bn};
    encode(&w.map_hi, 2, w.hi->p, dims, strides, box, w.cg);
    encode(&w.map_lo, 2, w.lo->p, dims, strides, box, w.cg);
    if (taps == 9 && N <= 32 && cin <= 64) {
        // the row kernel's operand: [dy][8-channel plane][v 3 C + kx C + n][8], zeros past N
        // and cin, copied verbatim into shared memory
        const int C = N <= 16 ? 16 : 32, CG = cin <= 16 ? 16 : (cin <= 32 ? 32 : 64), NPL = CG / 8, NB = 6 * C;
        std::vector<__nv_bfloat16> b((size_t)3 * NPL * NB * 8, __float2bfloat16_rn(0.f));
        for (int dy = 0; dy < 3; dy++)
            for (int kx = 0; kx < 3; kx++)
                for (int n = 0; n < N; n++)
                    for (int ci = 0; ci < cin; ci++) {
                        const float v = wnk[((size_t)n * taps + dy * 3 + kx) * cin + ci];
                        const __nv_bfloat16 h = __float2bfloat16_rn(v);
                        const size_t o = ((size_t)(dy * NPL + ci / 8) * NB + kx * C + n) * 8 + ci % 8;
                        b[o] = h;
                        b[o + (size_t)3 * C * 8] = __float2bfloat16_rn(v - __bfloat162float(h));
                    }
        w.x3 = alloc(c, b.size() * 2);
        WOCR_CUDA(cudaMemcpyAsync(w.x3->p, b.data(), b.size() * 2, cudaMemcpyHostToDevice, c->stream));
        WOCR_CUDA(cudaStreamSynchronize(c->stream));
        w.x3_cout = C;
        w.x3_cg = CG;
    }
    return w;
}

void add_convt_rows(Ctx *c, TconvW &w, const std::vector<float> &nk, int cout, int cin) {
    if (cout > 32 || cin > 64 || w.taps != 1 || w.N != 4 * cout) return;
    // [8-channel plane][v 4 C + tap C + n][8], zeros past cout and cin, copied verbatim into
    // shared memory by the row kernel
    const int C = cout <= 16 ? 16 : 32, CG = cin <= 16 ? 16 : (cin <= 32 ? 32 : 64), NPL = CG / 8, NB = 8 * C;
    std::vector<__nv_bfloat16> b((size_t)NPL * NB * 8, __float2bfloat16_rn(0.f));
    for (int tap = 0; tap < 4; tap++)
        for (int n = 0; n < cout; n++)
            for (int ci = 0; ci < cin; ci++) {
                const float v = nk[(size_t)(tap * cout + n) * cin + ci];
                const __nv_bfloat16 h = __float2bfloat16_rn(v);
                const size_t o = ((size_t)(ci / 8) * NB + tap * C + n) * 8 + ci % 8;
                b[o] = h;
                b[o + (size_t)4 * C * 8] = __float2bfloat16_rn(v - __bfloat162float(h));
            }
    w.x3 = alloc(c, b.size() * 2);
    WOCR_CUDA(cudaMemcpyAsync(w.x3->p, b.data(), b.size() * 2, cudaMemcpyHostToDevice, c->stream));
    WOCR_CUDA(cudaStreamSynchronize(c->stream));
    w.x3_cout = C;
    w.x3_cg = CG;
    w.x3_ct = 1;
}

bool tconv_input_ok(const uint16_t *x, int64_t x_n, int64_t x_pix) {
    // 16-byte copies: base, lo part and pixel / image strides 16-byte aligned
    return (reinterpret_cast<uintptr_t>(x) & 15) == 0 && x_pix % 16 == 0 && x_n % 8 == 0;
}

// the row kernel's operand fits this launch: a 3 x 3 convolution, or the 2 x 2 / s2 ConvTranspose
static bool rows_kind_ok(const TconvW &w, const TconvP &q) {
    if (!w.x3 || std::getenv("WOCR_NO_ROWS")) return false;
    return w.x3_ct ? q.scatter == 2 && q.kh == 1 && q.kw == 1 && q.scat_cout == w.N / 4
                   : q.kh == 3 && q.kw == 3 && !q.scatter;
}

bool tconv_rows_eligible(const TconvW &w, const TconvP &q) {
    if (!rows_kind_ok(w, q)) return false;
    if ((int64_t)q.n * ((q.ow + RV - 1) / RV) * ((q.oh + RX - 1) / RX) >= (int64_t)INT32_MAX) return false;
    TcP p{};
    const bool al = (reinterpret_cast<uintptr_t>(q.y) & 15) == 0;
    p.out_vec = q.split_out ? (al && q.y_pix % 16 == 0 && q.y_n % 8 == 0) : (al && q.y_pix % 4 == 0 && q.y_n % 4 == 0);
    p.bias_n = w.N;
    int smem = 0;
    return plan_rows_smem(w, p, smem);
}

void tconv(Ctx *c, const TconvW &w, const TconvP &q) {
    const int64_t M = (int64_t)q.n * q.oh * q.ow;
    if (M == 0 || w.N == 0) return;
    if (q.cin != w.cin || q.kh * q.kw != w.taps) fail(WOCR_ERR_SHAPE, "tap convolution weights do not match");
    if (!tconv_input_ok(q.x, q.x_n, q.x_pix)) fail(WOCR_ERR_UNSUPPORTED, "tap convolution input not 16-byte aligned");
    if (q.scatter && (q.kh != 1 || q.kw != 1)) fail(WOCR_ERR_UNSUPPORTED, "scatter tap convolution with a kernel");
    if (!c->status) {
        c->status_buf = alloc(c, 16);
        c->status = (int *)c->status_buf->p;
        WOCR_CUDA(cudaMemsetAsync(c->status, 0, 16, c->stream));
    }
    TcP p{};
    p.x = q.x;
    p.x_n = q.x_n;
    p.x_pix = q.x_pix;
    p.h = q.h;
    p.w = q.w;
    p.cin = q.cin;
    p.n = q.n;
    p.oh = q.oh;
    p.ow = q.ow;
    p.N = w.N;
    p.pt = q.pt;
    p.pl = q.pl;
    p.bias_n = q.scatter ? q.scat_cout : w.N;
    p.bias = q.bias;
    p.act = q.act;
    p.y = q.y;
    p.split_out = q.split_out;
    const bool al = (reinterpret_cast<uintptr_t>(q.y) & 15) == 0;
    p.out_vec = q.split_out ? (al && q.y_pix % 16 == 0 && q.y_n % 8 == 0) : (al && q.y_pix % 4 == 0 && q.y_n % 4 == 0);
    p.y_n = q.y_n;
    p.y_pix = q.y_pix;
    p.scatter = q.scatter;
    p.scat_cout = q.scat_cout;
    p.ow_out = q.scatter ? q.ow * q.scatter : q.ow;
    p.pool_y = q.pool_y;
    p.pool_split = q.pool_split;
    p.pool_n = q.pool_n;
    p.pool_pix = q.pool_pix;
    if (q.pool_y) {
        if (q.scatter || w.N % 16) fail(WOCR_ERR_UNSUPPORTED, "fused MaxPool needs a plain output of 16-channel chunks");
        const bool pal = (reinterpret_cast<uintptr_t>(q.pool_y) & 15) == 0;
        p.pool_vec = q.pool_split ? (pal && q.pool_pix % 16 == 0 && q.pool_n % 8 == 0)
                                  : (pal && q.pool_pix % 4 == 0 && q.pool_n % 4 == 0);
    }
    p.status = c->status;
    if (q.head_y) {
        if (q.head_n < 1 || q.head_n > 4 || q.pool_y || q.scatter)
            fail(WOCR_ERR_UNSUPPORTED, "fused head: 1 to 4 outputs, no pool, no scatter");
        p.head_w = q.head_w;
        p.head_b = q.head_b;
        p.head_ldw = q.head_ldw;
        p.head_n = q.head_n;
        p.head_act = q.head_act;
        p.head_y = q.head_y;
        p.head_y_n = q.head_y_n;
        p.head_y_pix = q.head_y_pix;
    }
    const double flops = 2.0 * (double)M * w.N * w.taps * w.cin;
    const double bytes = 4.0 * ((double)q.n * q.h * q.w * q.cin + (double)M * w.N) + 4.0 * (double)w.N * w.taps * w.cin;
    if (q.head_y && !tconv_rows_eligible(w, q)) fail(WOCR_ERR_UNSUPPORTED, "fused head without the row kernel");
    // the narrow 3 x 3 layers and 2 x 2 ConvTransposes: taps stacked along N (k_tconv_rows)
    if (rows_kind_ok(w, q)) {
        TcP pr = p;
        int smem = 0;
        CUtensorMap xm[2];
        bool whole = false;
        if (plan_rows(w, q, pr, smem, xm, whole)) {
            Prof pf(c, q.scatter ? "tconv_convt" : "tconv", flops, bytes);
            launch_rows_any(c, w, pr, smem, xm, whole);
            c->flops += flops;
            return;
        }
    }
    // two MMA blocks per tile for the narrow layers when there are tiles to spare
    const int mb = w.bn <= 32 && (int64_t)q.n * q.oh * q.ow >= (int64_t)c->sm_count * 256 * 8 ? 2 : 1;
    p.trows = TR * mb;
    p.tiles_x = (q.ow + TP - 1) / TP;
    p.tiles_y = (q.oh + p.trows - 1) / p.trows;
    p.ntn = (w.N + w.bn - 1) / w.bn;
    const int64_t ntiles = (int64_t)q.n * p.tiles_x * p.tiles_y * p.ntn;
    if (ntiles >= (int64_t)INT32_MAX) fail(WOCR_ERR_UNSUPPORTED, "tap convolution with 2^31 tiles or more");
    p.ntiles = (int)ntiles;
    p.div_ntn = FastDiv((uint32_t)p.ntn);
    p.div_tx = FastDiv((uint32_t)p.tiles_x);
    p.div_ty = FastDiv((uint32_t)p.tiles_y);
    p.nchunk = w.cin_pad / w.cg;
    p.taps = w.taps;
    p.kw = q.kw;
    p.cin_pad = w.cin_pad;
    p.hw_w = TP + q.kw - 1;
    if ((p.trows + q.kh - 1) * p.hw_w > 512) fail(WOCR_ERR_UNSUPPORTED, "tap convolution kernel too large");
    p.halo_px = (p.trows + q.kh - 1) * p.hw_w;
    p.plane = (uint32_t)p.halo_px * 16;
    p.a_stage = (2 * (w.cg / 8) * p.plane + 1023) / 1024 * 1024;

    // shared memory: A stages, then B (resident or a ring of tap chunks), then the barriers, the
    // bias and the transposed-store staging (2 KB per epilogue warp, when stores are 16-byte aligned)
    const int stg = p.out_vec ? kEpiWarps * 2048 : 0;
    const int budget = kSmemBudget - stg;
    const int b_half = w.bn * w.cg * 2;
    const int b_all = p.ntn * w.taps * p.nchunk * 2 * b_half;
    int SA, SB;
    if (b_all <= 96 * 1024) {
        p.b_res = 1;
        SB = 1;
        const int b_region = (b_all + 1023) / 1024 * 1024;
        SA = std::min(8, (budget - b_region) / (int)p.a_stage);
        p.b_off = (uint32_t)SA * p.a_stage;
        p.bar_off = p.b_off + (uint32_t)b_region;
    } else {
        p.b_res = 0;
        p.b_stage = (uint32_t)(w.taps * 2 * b_half);
        SB = std::min(8, std::max(2, (budget / 2) / (int)p.b_stage));
        SA = std::min(8, (budget - SB * (int)p.b_stage) / (int)p.a_stage);
        p.b_off = (uint32_t)SA * p.a_stage;
        p.bar_off = p.b_off + (uint32_t)((SB * p.b_stage + 1023) / 1024 * 1024);
    }
    if (SA < 2) fail(WOCR_ERR_UNSUPPORTED, "tap convolution halo does not fit twice");
    // a second accumulator is written when a tile has a commit before its last MMA
    p.two_acc = p.nchunk > 1;
    p.SA = SA;
    p.SB = SB;
    p.lag = std::min(kLagMax, SA - 2);
    p.bias_off = p.bar_off + 1024;
    p.stg_off = stg ? p.bias_off + (uint32_t)((p.bias_n * 4 + 15) / 16 * 16) : 0;
    const int smem = (int)p.bias_off + (p.bias_n * 4 + 15) / 16 * 16 + stg + 1024;  // + alignment slack
    if (smem > 227 * 1024) fail(WOCR_ERR_UNSUPPORTED, "tap convolution bias too large");

    Prof pf(c, q.scatter ? "tconv_convt" : "tconv", flops, bytes);
    if (w.cg == 16) launch_taps<16>(c, w, p, smem, q.kh, q.kw);
    else launch_taps<32>(c, w, p, smem, q.kh, q.kw);
    c->flops += flops;
}

}  // namespace k
}  // namespace wocr
