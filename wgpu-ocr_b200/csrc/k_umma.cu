// Tensor-core GEMM / implicit-GEMM convolution on the 5th-generation tensor cores (tcgen05,
// sm_100a): the B200 path of the reference's dense conv (K1-K4, src/gpu.rs:37-350), its GEMM
// (K15, src/gpu.rs:616-678), the linear layers of nd_bgemm (K29, src/nd.rs:291-358) and the
// kernel == stride ConvTranspose (K7, src/gpu.rs:424-460).
//
// Precision: the reference computes in fp32.  Each operand is split into two bf16 parts,
// x = hi + lo (hi = bf16(x), lo = bf16(x - hi)), and the product is accumulated in fp32 in
// tensor memory as hi*hi + hi*lo + lo*hi: three kind::f16 MMAs per K step, relative error of a
// product about 2^-16 (the dropped lo*lo term and the rounding of lo), against 2^-8 for plain
// bf16 and 2^-11 for tf32.
//
// Persistent: one CTA per SM loops over 128 x BN output tiles; the shared-memory stage ring runs
// on across tile boundaries and the fp32 accumulators in tensor memory are multi-buffered (up to
// 8 tiles), so loads of the next tiles and the epilogues of earlier ones overlap the MMAs.
//   warps 0-15  produce A: four threads per tile row, 64 k per stage, fp32 loads (implicit
//               im2col for convolutions, zero padding, SE input scale), split to bf16 hi/lo,
//               written in the 128-byte-swizzled K-major layout the MMA reads;
//   warp 20     issues the TMA loads of the pre-split weight tiles (B hi/lo, BN x 64 each);
//   warp 21     allocates tensor memory and (one thread) issues tcgen05.mma + tcgen05.commit;
//   warps 16-19 the epilogue: tcgen05.ld of the accumulator, bias, activation, residual,
//               channels-last stores (or the ConvTranspose scatter), then hand the accumulator
//               buffer back to the MMA warp.
// Stages are handed over with mbarriers.  Every wait is bounded by a clock budget; on expiry
// the kernel records an error code in `status`, drains its own TMA loads and MMAs, frees its
// tensor memory and returns.
#include <atomic>
#include <cstdlib>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "kernels.h"
#include "tc.h"
#include "umma.h"

namespace wocr {
namespace k {

namespace {

constexpr int BK = 64;
constexpr int kTapTable = 1024;  // 8-wide k chunks described in shared memory (K <= 8192)
constexpr int kEpiWarps = 8;      // epilogue warps: two per TMEM lane quadrant
using namespace tc;

struct Smem {
    // per stage: A hi, A lo (128 x 64 bf16 = 16 KB each), B hi, B lo (BN x 64 bf16 each)
    static constexpr int a_bytes = BM * BK * 2;
};

template <int BN, int STAGES>
struct Layout {
    static constexpr int b_bytes = BN * BK * 2;
    static constexpr int stage_bytes = 2 * Smem::a_bytes + 2 * b_bytes;
    static constexpr int bar_off = STAGES * stage_bytes;
    static constexpr int tab_off = bar_off + 1024;   // barriers and tmem slot first
    // per epilogue warp, two tiles' bias columns of its half (each warp stages its own: no
    // cross-warp barrier)
    static constexpr int ecols = (BN / 16 + 1) / 2 * 16;
    static constexpr int ebias_off = tab_off + 4 * kTapTable;
    // per epilogue warp, a 32-row x 16-column output chunk for the TMA tensor store (64-byte
    // swizzle; 1024-byte aligned like every region above)
    static constexpr int ystage_off = ebias_off + kEpiWarps * 2 * ecols * 4;
    static constexpr int total = ystage_off + kEpiWarps * 2048 + 1024;  // + alignment slack
    static_assert(total <= 232448, "shared memory of one CTA");
};

// The fp32 source of one row of A (an output pixel of a convolution, or a row of x).
struct ARow {
    bool valid;
    int iy0, ix0;
    const float *xb;
    const float *scb;
};

__device__ __forceinline__ ARow a_row(const UmmaP &p, int64_t m) {
    ARow r;
    r.valid = m < p.M;
    r.iy0 = r.ix0 = 0;
    r.xb = p.x;
    r.scb = nullptr;
    if (r.valid) {
        if (p.mode == 0) {
            r.xb = p.x + m * p.lda;
        } else {
            const int mi = (int)m;  // M < 2^31 (checked on the host)
            const int ox = mi % p.ow;
            const int t = mi / p.ow;
            const int oy = t % p.oh;
            const int nb = t / p.oh;
            r.iy0 = oy * p.sh - p.pt;
            r.ix0 = ox * p.sw - p.pl;
            r.xb = p.x + (int64_t)nb * p.x_n;
            r.scb = p.insc ? p.insc + (int64_t)nb * p.cin : nullptr;
        }
    }
    return r;
}

// Loads 8 consecutive k values of one row of A (fp32) for k0 .. k0 + 8; zeros outside.
__device__ __forceinline__ void load8(const UmmaP &p, const ARow &r, int k0, float (&v)[8]) {
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = 0.f;
    if (!r.valid || k0 >= p.K) return;
    if (p.mode == 0) {  // row-major A
        const float *src = r.xb + k0;
        if (p.vec && k0 + 8 <= p.K) {
            float4 a = __ldg(reinterpret_cast<const float4 *>(src));
            float4 b = __ldg(reinterpret_cast<const float4 *>(src + 4));
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++)
                if (k0 + i < p.K) v[i] = src[i];
        }
        return;
    }
    if (p.vec) {  // cin % 8 == 0: one tap, 8 consecutive channels
        int tap = k0 / p.cin, ci = k0 - tap * p.cin;
        int ky = tap / p.kw, kx = tap - ky * p.kw;
        int iy = r.iy0 + ky, ix = r.ix0 + kx;
        if (iy < 0 || iy >= p.h || ix < 0 || ix >= p.w) return;
        const float4 *src = reinterpret_cast<const float4 *>(r.xb + ((int64_t)iy * p.w + ix) * p.x_pix + ci);
        float4 a = __ldg(src), b = __ldg(src + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        if (r.scb) {
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] *= r.scb[ci + i];
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int k = k0 + i;
        if (k >= p.K) break;
        int tap = k / p.cin, ci = k - tap * p.cin;
        int ky = tap / p.kw, kx = tap - ky * p.kw;
        int iy = r.iy0 + ky, ix = r.ix0 + kx;
        if (iy < 0 || iy >= p.h || ix < 0 || ix >= p.w) continue;
        float x = r.xb[((int64_t)iy * p.w + ix) * p.x_pix + ci];
        if (r.scb) x *= r.scb[ci];
        v[i] = x;
    }
}

// Warp roles of the persistent kernel (832 threads):
constexpr int kProdWarps = 16;  // warps 0-15: A producers, four threads per tile row
constexpr int kEpiWarp0 = 16;   // warps 16-19: epilogue, a tile's first half of columns
constexpr int kTmaWarp = 20;    // warp 20: B tiles by TMA
constexpr int kMmaWarp = 21;    // warp 21: TMEM allocation, MMA issue
constexpr int kEpiWarp1 = 22;   // warps 22-25: epilogue, the second half (lane quadrant = warp % 4)
constexpr int kAllThreads = 26 * 32;


// The im2col source of one 8-wide k chunk of a convolution, precomputed per CTA: tap row (bits
// 24-31), tap column (16-23) and first input channel (0-15); 0xffffffff past K.
__device__ __forceinline__ uint32_t tap_entry(const UmmaP &p, int g) {
    const int k0 = g * 8;
    if (k0 >= p.K) return 0xffffffffu;
    const int tap = k0 / p.cin, ci = k0 - tap * p.cin;
    const int ky = tap / p.kw, kx = tap - ky * p.kw;
    return ((uint32_t)ky << 24) | ((uint32_t)kx << 16) | (uint32_t)ci;
}

// load8 for convolutions with cin % 8 == 0 through the tap table: no divisions.
__device__ __forceinline__ void load8_tab(const UmmaP &p, const ARow &r, uint32_t e, float (&v)[8]) {
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = 0.f;
    if (!r.valid || e == 0xffffffffu) return;
    const int iy = r.iy0 + (int)(e >> 24), ix = r.ix0 + (int)((e >> 16) & 0xff), ci = (int)(e & 0xffff);
    if (iy < 0 || iy >= p.h || ix < 0 || ix >= p.w) return;
    const float4 *src = reinterpret_cast<const float4 *>(r.xb + ((int64_t)iy * p.w + ix) * p.x_pix + ci);
    float4 a = __ldg(src), b = __ldg(src + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    if (r.scb) {
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] *= r.scb[ci + i];
    }
}

// v[j] += b[j] for a chunk's 16 bias columns staged 64-byte aligned: four 16-byte loads
__device__ __forceinline__ void add_bias16(float (&v)[16], const float *b) {
    const float4 *b4 = reinterpret_cast<const float4 *>(b);
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const float4 t = b4[u];
        v[4 * u] += t.x;
        v[4 * u + 1] += t.y;
        v[4 * u + 2] += t.z;
        v[4 * u + 3] += t.w;
    }
}

// 2^x by the tensor unit's base-2 exponential (inputs <= 0 here, results in [0, 1])
__device__ __forceinline__ float ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// A tile index t (< 2^31) as (row tile, N tile): t / ntn by the launch's multiply-high divisor.
__device__ __forceinline__ uint32_t tile_row(const UmmaP &p, int64_t t) {
    const uint32_t x = (uint32_t)t;
    return (__umulhi(x, p.ntn_m) + x) >> p.ntn_l;
}

template <int BN, int STAGES, int CHAINS>
__global__ void __launch_bounds__(kAllThreads, 1)
    k_umma(const __grid_constant__ CUtensorMap tm_hi, const __grid_constant__ CUtensorMap tm_lo,
           const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_ahi,
           const __grid_constant__ CUtensorMap tm_alo, UmmaP p) {
    using Lay = Layout<BN, STAGES>;
    // CHAINS: accumulation chains per tile (0: Acc<BN>'s choice); one chain sums in the order of
    // the 128- and 256-column tiles, so a narrowed launch gives their results to the bit
    constexpr int NCH = CHAINS ? CHAINS : Acc<BN>::chains, TCOLS = BN * NCH;
    constexpr int NACC = 512 / TCOLS < 8 ? 512 / TCOLS : 8;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *afull = reinterpret_cast<uint64_t *>(smem + Lay::bar_off);
    uint64_t *bfull = afull + STAGES;
    uint64_t *empty = bfull + STAGES;
    uint64_t *tfull = empty + STAGES;   // [NACC] accumulator ready (tcgen05.commit)
    uint64_t *tempty = tfull + NACC;    // [NACC] accumulator drained by the epilogue (8 warps)
    uint64_t *drain = tempty + NACC;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long bud = p.budget > 0 ? p.budget : kWaitBudget;  // every wait's clock budget
    const int nk = p.Kpad / BK;
    const int ntn = (p.N + BN - 1) / BN;
    const int64_t ntiles = ((p.M + BM - 1) / BM) * ntn;
    // two accumulators of BN fp32 columns each
    constexpr uint32_t kCols = NACC * TCOLS <= 32 ? 32 : (NACC * TCOLS <= 64 ? 64 : (NACC * TCOLS <= 128 ? 128 : (NACC * TCOLS <= 256 ? 256 : 512)));

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&afull[s], kProdWarps);
            mbar_init(&bfull[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < NACC; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    uint32_t *taps = reinterpret_cast<uint32_t *>(smem + Lay::tab_off);
    const bool use_tab = p.mode == 1 && p.vec && p.Kpad / 8 <= kTapTable;
    if (use_tab)
        for (int g = threadIdx.x; g < p.Kpad / 8; g += blockDim.x) taps[g] = tap_entry(p, g);
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < kProdWarps) {
        if (p.a_tma) {
            // A arrives pre-split with the weights (the TMA warp): nothing to build
        } else {
        // ---------------- A producers: four threads per tile row, 2 chunks of 8 k each ----------------
        // Software-pipelined: the loads of the next k block are issued before waiting for a free
        // stage and converting the current one, so two k blocks of loads are in flight.
        const int row = threadIdx.x & (BM - 1);
        const int quarter = threadIdx.x >> 7;  // chunks 2 quarter, 2 quarter + 1
        const int sw = row & 7;
        int64_t t = blockIdx.x;
        int kb = 0, it = 0;
        auto load_pair = [&](const ARow &r, int kbl, float (&v)[2][8]) {
#pragma unroll
            for (int c = 0; c < 2; c++) {
                const int g = kbl * (BK / 8) + quarter * 2 + c;
                if (use_tab) load8_tab(p, r, taps[g], v[c]);
                else load8(p, r, g * 8, v[c]);
            }
        };
        if (t < ntiles) {
            ARow r = a_row(p, (int64_t)tile_row(p, t) * BM + row);
            float cur[2][8], nxt[2][8];
            load_pair(r, 0, cur);
            while (true) {
                // the (tile, k block) after this one
                int64_t t2 = t;
                int kb2 = kb + 1;
                if (kb2 == nk) {
                    kb2 = 0;
                    t2 = t + gridDim.x;
                }
                const bool more = t2 < ntiles;
                if (more) {
                    if (t2 != t) r = a_row(p, (int64_t)tile_row(p, t2) * BM + row);
                    load_pair(r, kb2, nxt);
                }
                const int s = it % STAGES;
                if (!warp_wait(&empty[s], ((it / STAGES) & 1) ^ 1, p.status, abort_flag, 11, bud)) break;
                uint8_t *rhi = smem + s * Lay::stage_bytes + (row >> 3) * 1024 + (row & 7) * 128;
                uint8_t *rlo = rhi + Smem::a_bytes;
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    uint4 hi, lo;
                    split8(cur[c], hi, lo);
                    const int ch = quarter * 2 + c;
                    *reinterpret_cast<uint4 *>(rhi + ((ch ^ sw) << 4)) = hi;
                    *reinterpret_cast<uint4 *>(rlo + ((ch ^ sw) << 4)) = lo;
                }
                fence_async_smem();
                __syncwarp();
                // (a wait test leaves the first stage without its arrivals)
                if (lane == 0 && !(p.test_stall && it == 0)) mbar_arrive(&afull[s]);  // one arrival per warp
                it++;
                if (!more) break;
                t = t2;
                kb = kb2;
#pragma unroll
                for (int c = 0; c < 2; c++)
#pragma unroll
                    for (int e = 0; e < 8; e++) cur[c][e] = nxt[c][e];
            }
        }
        }
    } else if (warp == kTmaWarp) {
        // ---------------- B loader: TMA of the pre-split weight tiles (and of A, pre-split) ----------------
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int n0 = (int)((uint32_t)t - tile_row(p, t) * (uint32_t)ntn) * BN;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait_spin(&empty[s], ((it / STAGES) & 1) ^ 1, p.status, abort_flag, 12, bud)) {
                        ok = false;
                        break;
                    }
                    uint8_t *bhi = smem + s * Lay::stage_bytes + 2 * Smem::a_bytes;
                    uint8_t *blo = bhi + Lay::b_bytes;
                    mbar_expect_tx(&bfull[s], 2 * Lay::b_bytes + (p.a_tma ? 2 * Smem::a_bytes : 0));
                    tma_load_2d(bhi, &tm_hi, &bfull[s], kb * BK, n0);
                    tma_load_2d(blo, &tm_lo, &bfull[s], kb * BK, n0);
                    if (p.a_tma) {  // the tile's rows, in the layout the producers would write
                        uint8_t *ahi = smem + s * Lay::stage_bytes;
                        const int m0 = (int)(tile_row(p, t) * BM);
                        tma_load_2d(ahi, &tm_ahi, &bfull[s], kb * BK, m0);
                        tma_load_2d(ahi + Smem::a_bytes, &tm_alo, &bfull[s], kb * BK, m0);
                    }
                }
            }
            // drain: the last STAGES issued copies land before the CTA may exit (bounded)
            for (int j = (it > STAGES ? it - STAGES : 0); j < it; j++) {
                long long t0 = clock64();
                while (!mbar_try(&bfull[j % STAGES], (j / STAGES) & 1) && clock64() - t0 < bud) {
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = instr_desc(BN);
            bool ok = true;
            int it = 0, lt = 0;
            for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, lt++) {
                const int ab = lt % NACC;
                const uint32_t dcol = tmem + ab * TCOLS;
                ok = mbar_wait_spin(&tempty[ab], ((lt / NACC) & 1) ^ 1, p.status, abort_flag, 16, bud);
                if (!ok) break;
                tc_fence_after();
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    const uint32_t par = (it / STAGES) & 1;
                    ok = (p.a_tma || mbar_wait_spin(&afull[s], par, p.status, abort_flag, 13, bud)) &&
                         mbar_wait_spin(&bfull[s], par, p.status, abort_flag, 14, bud);
                    if (!ok) break;
                    tc_fence_after();
                    uint8_t *base = smem + s * Lay::stage_bytes;
                    const uint32_t ahi = smem_u32(base), alo = ahi + Smem::a_bytes;
                    const uint32_t bhi = alo + Smem::a_bytes, blo = bhi + Lay::b_bytes;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++) {
                        const uint32_t off = kk * 32;
                        // MMA number j = 3 kk + {0, 1, 2} goes to chain j % NCH; a chain's first
                        // MMA of the tile overwrites, the others accumulate
                        const int j0 = 3 * kk;
                        const uint32_t d0 = dcol + ((j0 + 0) % NCH) * BN;
                        const uint32_t d1 = dcol + ((j0 + 1) % NCH) * BN;
                        const uint32_t d2 = dcol + ((j0 + 2) % NCH) * BN;
                        umma(d0, smem_desc(ahi + off), smem_desc(bhi + off), idesc, kb > 0 || j0 + 0 >= NCH);
                        umma(d1, smem_desc(ahi + off), smem_desc(blo + off), idesc, kb > 0 || j0 + 1 >= NCH);
                        umma(d2, smem_desc(alo + off), smem_desc(bhi + off), idesc, kb > 0 || j0 + 2 >= NCH);
                    }
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&tfull[ab]);
            }
            // every issued MMA completes before the shared and tensor memory go away (bounded)
            umma_commit(drain);
            long long t0 = clock64();
            while (!mbar_try(drain, 0) && clock64() - t0 < bud) {
            }
        }
    } else {
        // ---------- epilogue: warps 16-19 and 22-25, TMEM lanes 32 * (warp % 4) ----------
        // The two warps of a lane quadrant split each tile's 16-column chunks (the first
        // ceil(NCK / 2) to warps 16-19), so two warps a scheduler hide each other's latencies.
        constexpr int NCK = BN / 16, HCK = (NCK + 1) / 2;
        const int q = warp & 3, h = warp >= kEpiWarp1 ? 1 : 0;
        const int ck0 = h * HCK, nck = h ? NCK - HCK : HCK;  // this warp's chunks of a tile
        const int row = q * 32 + lane;
        float *ebias = reinterpret_cast<float *>(smem + Lay::ebias_off) + (q + 4 * h) * 2 * Lay::ecols;
        float *ystage = reinterpret_cast<float *>(smem + Lay::ystage_off) + (q + 4 * h) * 512;
        // row-major stores of whole 32-row chunks by the TMA engine (the host's map of y): the
        // lanes only write the warp's staging chunk in shared memory, instead of 32 rows' 16-byte
        // pieces through the load/store unit (which bounds the epilogue)
        const bool tma_y = p.tma_y && !p.part_max && !p.scatter;
        int lt = 0;
        int eb_n0_0 = -1, eb_n0_1 = -1;  // the N tile whose bias columns each slot holds
        for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, lt++) {
            const int ab = lt % NACC;
            const uint32_t trow_i = tile_row(p, t);
            const int64_t m = (int64_t)trow_i * BM + row, qrow0 = m - lane;  // qrow0: the quadrant's first row
            const int n0 = (int)((uint32_t)t - trow_i * (uint32_t)ntn) * BN;
            // the tile's bias columns (scatter tiles: per output channel) into this warp's slot while
            // the MMAs run, so no chunk below waits on a global load.  A slot that already holds
            // this N tile's columns is kept (a CTA whose tiles step by a multiple of the N tile
            // count, as 148 CTAs over 74 N tiles, keeps one N tile): when the epilogue is what
            // bounds the kernel, these loads would otherwise sit on every tile's path.
            float *eb = ebias + (lt & 1) * Lay::ecols;
            int &eb_n0 = (lt & 1) ? eb_n0_1 : eb_n0_0;
            if (eb_n0 != n0) {
                eb_n0 = n0;
#pragma unroll 4
                for (int j = lane; j < nck * 16; j += 32) {
                    const int col = n0 + ck0 * 16 + j;
                    const int bc = p.scatter ? col % p.scat_cout : col;
                    eb[j] = p.bias && col < p.N ? p.bias[bc] : 0.f;
                }
            }
            __syncwarp();
            if (!warp_wait(&tfull[ab], (lt / NACC) & 1, p.status, abort_flag, 15, bud)) break;
            tc_fence_after();
            int ox = 0, oy = 0, nb = 0;
            int64_t pix = 0;
            if (p.mode == 1 && m < p.M) {
                const int mi = (int)m;  // M < 2^31 (checked on the host)
                ox = mi % p.ow;
                const int tt = mi / p.ow;
                oy = tt % p.oh;
                nb = tt / p.oh;
                pix = (int64_t)oy * p.ow + ox;
            }
            // arg-max partials of this row over the warp's half of the tile: the maximum and its
            // first column, then the exponentials' sum against that maximum in four partial sums
            float amx = -INFINITY, as4[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t aidx = 0;
            const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + ab * TCOLS;
            // A chunk's accumulator: one load and wait (tensor-memory loads take tens of cycles
            // once no store still reads the registers they overwrite, and the other epilogue
            // warp of the scheduler runs meanwhile); several chains summed in chain order, the
            // first two in one wait.  The arg-max epilogue reads the accumulator twice (pass
            // chunk i is the warp's chunk i mod nck), a second pass cheaper than the serial chain
            // of an online maximum it replaces.
            const bool amax = BN >= 64 && p.part_max;  // arg-max partials (64-column tiles or wider)
            const int nck_all = amax && p.part_sum ? 2 * nck : nck;  // no sums wanted: pass 1 only
            const bool full_tile = n0 + BN <= p.N;
            // a chunk's maximum by a tree of fmaxf (NaN never wins, as K30's search from -inf); only a
            // chunk that beats the row's maximum so far looks for its first column holding that value
            // (an earlier column keeps a tie)
            auto amax_tree = [&](const float (&o)[16], int c0) {
                float m8[8];
#pragma unroll
                for (int t = 0; t < 8; t++) m8[t] = fmaxf(o[2 * t], o[2 * t + 1]);
#pragma unroll
                for (int w = 4; w >= 1; w >>= 1) {
#pragma unroll
                    for (int t = 0; t < w; t++) m8[t] = fmaxf(m8[2 * t], m8[2 * t + 1]);
                }
                if (m8[0] > amx) {
                    int first = 15;
                    float fv = o[15];  // the value itself (a zero keeps its sign)
#pragma unroll
                    for (int j = 14; j >= 0; j--)
                        if (o[j] == m8[0]) {
                            first = j;
                            fv = o[j];
                        }
                    amx = fv;
                    aidx = (uint32_t)(n0 + c0 + first);
                }
            };
            auto amax_chunk = [&](float (&o)[16], int c0) {
                if (m >= p.M || n0 + c0 >= p.N) return;
                add_bias16(o, eb + (c0 - ck0 * 16));
                if (!full_tile) {
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (n0 + c0 + j >= p.N) o[j] = -INFINITY;
                }
                amax_tree(o, c0);
            };
            if (amax && !p.part_sum && NCH == 1) {
                // classes and maxima only, one accumulation chain: two chunks' loads before one
                // wait (a load and its wait are a round trip that the scheduler's two epilogue
                // warps cannot hide)
#pragma unroll 1
                for (int ci = 0; ci < nck; ci += 2) {
                    const int c0 = (ck0 + ci) * 16;
                    uint32_t a[16], b[16];
                    float va[16];
                    tmem_ld16_async(trow + c0, a);
                    if (ci + 1 < nck) {  // (warp-uniform)
                        tmem_ld16_async(trow + c0 + 16, b);
                        tmem_wait16x2(a, b);
                    } else {
                        tmem_wait16(a);
                    }
#pragma unroll
                    for (int j = 0; j < 16; j++) va[j] = __uint_as_float(a[j]);
                    amax_chunk(va, c0);
                    if (ci + 1 < nck) {
#pragma unroll
                        for (int j = 0; j < 16; j++) va[j] = __uint_as_float(b[j]);
                        amax_chunk(va, c0 + 16);
                    }
                }
            } else
#pragma unroll 1
            for (int ci = 0; ci < nck_all; ci++) {
                float v[16];
                const int c0 = (ck0 + (ci < nck ? ci : ci - nck)) * 16;  // ci < 2 nck
                const float *ebc = eb + (c0 - ck0 * 16);  // the chunk's bias columns
                const uint32_t tbase = trow + c0;
                if (NCH == 1) {
                    tmem_ld16(tbase, v);
                } else {
                    uint32_t a[16], b[16];
                    tmem_ld16_async(tbase, a);
                    tmem_ld16_async(tbase + BN, b);
                    tmem_wait16x2(a, b);
#pragma unroll
                    for (int j = 0; j < 16; j++) v[j] = __uint_as_float(a[j]) + __uint_as_float(b[j]);
#pragma unroll 1
                    for (int ch = 2; ch < NCH; ch++) {  // one chain a wait: fewer live registers
                        tmem_ld16_async(tbase + ch * BN, b);
                        tmem_wait16(b);
#pragma unroll
                        for (int j = 0; j < 16; j++) v[j] += __uint_as_float(b[j]);
                    }
                }
                // (a TMA chunk is the warp's: only a chunk past N or past M for every lane is skipped)
                if (tma_y ? (n0 + c0 >= p.N || qrow0 >= p.M) : (m >= p.M || n0 + c0 >= p.N)) continue;
                if (amax) {
                    // the logits are v + bias, as the unfused GEMM stores them (columns past N:
                    // -inf); a scheduler has only two epilogue warps, so the chunk's work is
                    // short independent chains
                    float *o = v;
                    add_bias16(v, ebc);
                    if (!full_tile) {
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            if (n0 + c0 + j >= p.N) o[j] = -INFINITY;
                    }
                    if (ci < nck) {
                        amax_tree(v, c0);  // pass 1
                    } else {
                        // pass 2: exponentials against the row's maximum, e^(o - max) as
                        // 2^(o log2(e) - max log2(e)) (exp(-inf) = 0 past N)
                        const float nl = -amx * 1.4426950408889634f;
#pragma unroll
                        for (int j = 0; j < 16; j++) as4[j & 3] += ex2_approx(fmaf(o[j], 1.4426950408889634f, nl));
                    }
                    continue;
                }
                if (p.scatter && p.scat_cout % 16 == 0) {
                    // a 16-column chunk lies in one tap: 16 consecutive channels of output pixel
                    // (s oy + ky, s ox + kx)
                    const int s = p.scatter, col = n0 + c0;
                    const int tap = col / p.scat_cout, co0 = col - tap * p.scat_cout;
                    const int yy = oy * s + tap / s, xx = ox * s + tap % s;
                    float *dst = p.y + (int64_t)nb * p.y_n + ((int64_t)yy * p.ow * s + xx) * p.y_pix + co0;
                    add_bias16(v, ebc);
                    act_n(v, p.act);
                    if (p.out_vec) {
                        float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; j++) dst[j] = v[j];
                    }
                    continue;
                }
                if (p.scatter) {
                    const int s = p.scatter;
                    add_bias16(v, ebc);
                    act_n(v, p.act);
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int col = n0 + c0 + j;
                        if (col >= p.N) break;
                        const int co = col % p.scat_cout, tap = col / p.scat_cout;
                        const int yy = oy * s + tap / s, xx = ox * s + tap % s;
                        p.y[(int64_t)nb * p.y_n + ((int64_t)yy * p.ow * s + xx) * p.y_pix + co] = v[j];
                    }
                    continue;
                }
                float *dst;
                const float *rsrc = nullptr;
                if (p.mode == 1) {
                    dst = p.y + (int64_t)nb * p.y_n + pix * p.y_pix + n0 + c0;
                    if (p.res && m < p.M) rsrc = p.res + (int64_t)nb * p.res_n + pix * p.res_pix + n0 + c0;
                } else {
                    dst = p.y + m * p.ldy + n0 + c0;
                }
                add_bias16(v, ebc);
                act_n(v, p.act);
                if (rsrc) {
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (n0 + c0 + j < p.N) v[j] += rsrc[j];
                }
                if (tma_y) {
                    // the previous chunk's store has read the staging chunk; then row `lane`'s 16
                    // values in the 64-byte swizzle (16-byte piece u at u ^ ((lane >> 1) & 3)), and
                    // one store of the 32 x 16 box (the engine clips rows past M, columns past N)
                    if (lane == 0) bulk_wait_read0();
                    __syncwarp();
#pragma unroll
                    for (int u = 0; u < 4; u++)
                        *reinterpret_cast<float4 *>(ystage + lane * 16 + 4 * (u ^ ((lane >> 1) & 3))) =
                            make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) tma_store_2d(&tm_y, ystage, n0 + c0, (int)qrow0);
                    continue;
                }
                const bool full = n0 + c0 + 16 <= p.N && p.out_vec;
                if (full) {
                    float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
                    for (int j = 0; j < 4; j++) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (n0 + c0 + j < p.N) dst[j] = v[j];
                }
            }
            if (amax && m < p.M) {
                const int64_t o = m * p.part_ld + 2 * (n0 / BN) + h;  // two slots a tile
                p.part_max[o] = amx;
                if (p.part_sum) p.part_sum[o] = (as4[0] + as4[1]) + (as4[2] + as4[3]);
                p.part_idx[o] = aidx;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[ab]);  // one arrival per warp
        }
        if (tma_y && lane == 0) bulk_wait_all();  // the warp's tensor stores are done
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
    }
}

// A (mode 0, fp32 [M][lda]) as the producers split it: per row, bf16 hi = bf16(v) and lo =
// bf16(v - hi) of the first K values, zeros up to Kpad; a thread per 8 values.
__global__ void k_split_rows(const float *__restrict__ x, int64_t lda, int64_t M, int K, int Kpad,
                             uint4 *__restrict__ hi, uint4 *__restrict__ lo) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, per = Kpad / 8;
    if (g >= M * per) return;
    const int64_t m = g / per;
    const int k0 = (int)(g - m * per) * 8;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = k0 + i < K ? __ldg(x + m * lda + k0 + i) : 0.f;
    uint4 h, l;
    split8(v, h, l);
    hi[g] = h;
    lo[g] = l;
}

// ---- host side ------------------------------------------------------------------------------

// The output map of a TMA-store epilogue: fp32 [M][N] rows `stride` floats apart, 16 x 32 boxes
// (16 columns of the quadrant's 32 rows) in the 64-byte swizzle.
void make_ymap(CUtensorMap *map, float *y, int N, int64_t M, int64_t stride) {
    auto fn = encode_fn();
    if (!fn) fail(WOCR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)stride * 4};
    cuuint32_t box[2] = {16, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(WOCR_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed: " + std::to_string((int)r));
}

void make_map(CUtensorMap *map, void *base, int N, int Kpad, int bn) {
    auto fn = encode_fn();
    if (!fn) fail(WOCR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)Kpad, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)Kpad * 2};
    cuuint32_t box[2] = {BK, (cuuint32_t)bn};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(WOCR_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

template <int BN, int STAGES, int CHAINS = 0>
void launch(Ctx *c, const CUtensorMap &map_hi, const CUtensorMap &map_lo, const CUtensorMap &map_y, const UmmaP &p,
            const CUtensorMap &map_ahi = CUtensorMap{}, const CUtensorMap &map_alo = CUtensorMap{}) {
    using Lay = Layout<BN, STAGES>;
    static std::atomic<bool> set[64];
    if (!set[c->device]) {
        WOCR_CUDA(cudaFuncSetAttribute(k_umma<BN, STAGES, CHAINS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Lay::total));
        set[c->device] = true;
    }
    int64_t tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
    if (tiles >= ((int64_t)1 << 31)) fail(WOCR_ERR_UNSUPPORTED, "GEMM with 2^31 tiles or more");
    UmmaP q = p;
    const FastDiv fd((uint32_t)((p.N + BN - 1) / BN));
    q.ntn_m = fd.m;
    q.ntn_l = fd.l;
    unsigned grid = (unsigned)std::min<int64_t>(tiles, c->sm_count);
    k_umma<BN, STAGES, CHAINS><<<grid, kAllThreads, Lay::total, c->stream>>>(map_hi, map_lo, map_y, map_ahi, map_alo, q);
    WOCR_LAUNCHED(c);
}

}  // namespace

int umma_bn(int N) {
    if (N <= 16) return 16;
    if (N <= 32) return 32;
    if (N <= 64) return 64;
    if (N <= 128) return 128;
    return 256;
}

UmmaW make_umma_weights(Ctx *c, const std::vector<float> &wnk, int N, int K, int max_bn) {
    // wnk: [N][K] fp32 (row n = output channel, k in the A operand's order)
    UmmaW w;
    w.N = N;
    w.K = K;
    w.Kpad = (K + BK - 1) / BK * BK;
    w.bn = umma_bn(std::min(N, max_bn));
    const int Npad = (N + w.bn - 1) / w.bn * w.bn;  // every TMA box lies inside the tensor
    std::vector<__nv_bfloat16> hi((size_t)Npad * w.Kpad, __float2bfloat16_rn(0.f)), lo = hi;
    for (int n = 0; n < N; n++)
        for (int k = 0; k < K; k++) {
            float v = wnk[(size_t)n * K + k];
            __nv_bfloat16 h = __float2bfloat16_rn(v);
            hi[(size_t)n * w.Kpad + k] = h;
            lo[(size_t)n * w.Kpad + k] = __float2bfloat16_rn(v - __bfloat162float(h));
        }
    size_t bytes = (size_t)Npad * w.Kpad * 2;
    w.hi = alloc(c, bytes);
    w.lo = alloc(c, bytes);
    WOCR_CUDA(cudaMemcpyAsync(w.hi->p, hi.data(), bytes, cudaMemcpyHostToDevice, c->stream));
    WOCR_CUDA(cudaMemcpyAsync(w.lo->p, lo.data(), bytes, cudaMemcpyHostToDevice, c->stream));
    WOCR_CUDA(cudaStreamSynchronize(c->stream));
    make_map(&w.map_hi, w.hi->p, Npad, w.Kpad, w.bn);
    make_map(&w.map_lo, w.lo->p, Npad, w.Kpad, w.bn);
    if (w.bn > 64) {
        make_map(&w.map_hi64, w.hi->p, Npad, w.Kpad, 64);
        make_map(&w.map_lo64, w.lo->p, Npad, w.Kpad, 64);
        w.has64 = true;
    }
    if (w.bn > 32) {
        make_map(&w.map_hi32, w.hi->p, Npad, w.Kpad, 32);
        make_map(&w.map_lo32, w.lo->p, Npad, w.Kpad, 32);
        w.has32 = true;
    }
    return w;
}

void umma_gemm(Ctx *c, const UmmaW &w, UmmaP p) {
    if (p.M == 0 || w.N == 0) return;
    if (p.M >= (int64_t)INT32_MAX - BM) fail(WOCR_ERR_UNSUPPORTED, "GEMM with 2^31 rows or more");
    if (p.part_max && (p.mode != 0 || p.part_ld != umma_part_slots(w) || w.bn < 64))
        fail(WOCR_ERR_INVALID, "arg-max partials need a row-major GEMM of 64-column tiles and two slots per N tile");
    if (!c->status) {
        c->status_buf = alloc(c, 16);
        c->status = (int *)c->status_buf->p;
        WOCR_CUDA(cudaMemsetAsync(c->status, 0, 16, c->stream));
    }
    p.status = c->status;
    if (const char *b = std::getenv("WOCR_WAIT_BUDGET")) p.budget = std::atoll(b);
    p.test_stall = std::getenv("WOCR_TEST_STALL_FIRST_STAGE") != nullptr;
    const bool al = (reinterpret_cast<uintptr_t>(p.y) & 15) == 0;
    p.out_vec = p.mode == 1 ? (al && p.y_pix % 4 == 0 && p.y_n % 4 == 0) : (al && p.ldy % 4 == 0);
    // TMA tensor stores of the output: rows of y at a fixed stride (a convolution's pixels
    // consecutive over the batch), 16-byte aligned; the arg-max and scatter epilogues store
    // otherwise
    CUtensorMap my{};
    const int64_t ystride = p.mode == 1 ? p.y_pix : p.ldy;
    p.tma_y = !p.part_max && !p.scatter && p.out_vec &&
              (p.mode == 0 || p.n == 1 || p.y_n == (int64_t)p.oh * p.ow * p.y_pix) && !std::getenv("WOCR_NO_TMA_STORE");
    if (p.tma_y) make_ymap(&my, p.y, w.N, p.M, ystride);
    p.K = w.K;
    p.Kpad = w.Kpad;
    p.N = w.N;
    double flops = 2.0 * (double)p.M * w.N * w.K;
    // fp32 A (its pixels once for a convolution), the output (or the arg-max partials: 12 bytes a
    // slot), the split weights (4 bytes a weight)
    const double out_bytes = p.part_max ? 12.0 * (double)p.M * p.part_ld : 4.0 * (double)p.M * w.N;
    double bytes = 4.0 * (double)p.M * w.K / (p.mode == 1 ? (double)p.kh * p.kw : 1.0) + out_bytes +
                   4.0 * (double)w.N * w.Kpad;
    Prof pf(c, p.scatter ? "umma_convt" : (p.mode == 1 ? "umma_conv" : "umma_linear"), flops, bytes);
    // few row tiles (short inputs): 64- or 32-column tiles put more SMs on the launch, with the
    // accumulation chains of the weights' own tile width (so the same sums); the arg-max partials
    // keep one slot per weight tile, and the scatter epilogue keeps its tile width
    const int64_t mt = (p.M + BM - 1) / BM;
    auto fills_half = [&](int bn) { return 2 * mt * ((w.N + bn - 1) / bn) > c->sm_count; };
    if (!p.part_max && !p.scatter && !fills_half(w.bn)) {
        const bool wide = w.bn > 64;  // one chain (128 / 256 columns), else two (64)
        if (w.has32 && !fills_half(64)) {
            if (wide)
                launch<32, 5, 1>(c, w.map_hi32, w.map_lo32, my, p);
            else
                launch<32, 5, 2>(c, w.map_hi32, w.map_lo32, my, p);
            c->flops += flops;
            return;
        }
        if (w.has64) {
            launch<64, 4, 1>(c, w.map_hi64, w.map_lo64, my, p);
            c->flops += flops;
            return;
        }
    }
    // Many N tiles over the same rows (the CTC head: 74): the producers would split each A tile
    // once per N tile; instead A is split once into bf16 hi / lo rows and the TMA warp loads the
    // tiles with the weights' (same 128-byte swizzled K-major layout, zeros past M and K)
    CUtensorMap mahi{}, malo{};
    BufP ahi, alo;
    if (p.mode == 0 && !p.test_stall && umma_ntiles(w) >= 8 && p.M >= BM && !std::getenv("WOCR_NO_A_TMA")) {
        const size_t abytes = (size_t)p.M * w.Kpad * 2;
        ahi = alloc(c, abytes);
        alo = alloc(c, abytes);
        const int64_t n8 = p.M * (w.Kpad / 8);
        k_split_rows<<<(unsigned)((n8 + 255) / 256), 256, 0, c->stream>>>(p.x, p.lda, p.M, w.K, w.Kpad,
                                                                          (uint4 *)ahi->p, (uint4 *)alo->p);
        WOCR_LAUNCHED(c);
        make_map(&mahi, ahi->p, (int)p.M, w.Kpad, BM);
        make_map(&malo, alo->p, (int)p.M, w.Kpad, BM);
        p.a_tma = 1;
    }
    switch (w.bn) {
    case 16: launch<16, 5>(c, w.map_hi, w.map_lo, my, p, mahi, malo); break;
    case 32: launch<32, 5>(c, w.map_hi, w.map_lo, my, p, mahi, malo); break;
    case 64: launch<64, 4>(c, w.map_hi, w.map_lo, my, p, mahi, malo); break;
    case 128: launch<128, 3>(c, w.map_hi, w.map_lo, my, p, mahi, malo); break;
    default: launch<256, 2>(c, w.map_hi, w.map_lo, my, p, mahi, malo); break;
    }
    c->flops += flops;
}

}  // namespace k
}  // namespace wocr
