// Device helpers shared by the tcgen05 kernels (k_umma.cu, k_tconv.cu): mbarriers with bounded
// waits, TMA loads, shared-memory matrix descriptors, tcgen05.mma / commit / ld, the bf16 hi/lo
// split (the epilogue activations are in act.h).  All inline PTX for sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "act.h"

namespace wocr {
namespace k {
namespace tc {

constexpr int BM = 128;  // rows of every tensor-core tile (one TMEM lane each)

// Division of 0 <= x < 2^31 by a divisor fixed at launch, as a multiply-high, an add and a shift
// (Granlund and Montgomery, "Division by invariant integers using multiplication", 1994):
// l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1, x / d = (mulhi(x, m) + x) >> l.
struct FastDiv {
    uint32_t d = 1, m = 1, l = 0;
    FastDiv() = default;
    explicit FastDiv(uint32_t dv) : d(dv) {
        while ((1ull << l) < d) l++;
        m = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
    }
    __host__ __device__ __forceinline__ uint32_t div(uint32_t x) const {
#ifdef __CUDA_ARCH__
        return (__umulhi(x, m) + x) >> l;
#else
        return (uint32_t)((((uint64_t)x * m) >> 32) + x) >> l;
#endif
    }
};
constexpr long long kWaitBudget = 4000000000LL;  // clock cycles (about 2 s) per wait

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// The same, but the thread is suspended (not spinning, so it leaves the issue slots to the warps
// doing work) until the phase completes or about 0.5 ms pass.
__device__ __forceinline__ bool mbar_try_sleep(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(500000u)
        : "memory");
    return ok != 0;
}

// Bounded wait: false (and an error code in *status) when the budget runs out or another role
// has already given up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *status, volatile int *abort_flag,
                                          int code, long long budget = kWaitBudget) {
    long long t0 = clock64();
    while (!mbar_try_sleep(bar, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > budget) {
            *abort_flag = 1;
            atomicCAS(status, 0, code);
            return false;
        }
    }
    return true;
}

// Non-blocking test of a phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait for the single threads that issue MMAs or TMA copies: a test first, then try_wait
// without a time hint, which parks the thread in hardware until the phase completes (or a short
// limit passes) instead of a test_wait spin whose instructions take issue slots from the
// epilogue warps on the same scheduler; bounded alike.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t *bar, uint32_t parity, int *status, volatile int *abort_flag,
                                               int code, long long budget = kWaitBudget) {
    if (mbar_test(bar, parity)) return true;
    long long t0 = clock64();
    while (!mbar_try(bar, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > budget) {
            *abort_flag = 1;
            atomicCAS(status, 0, code);
            return false;
        }
    }
    return true;
}

// One lane polls, the warp follows: a warp-uniform outcome for warp-wide code after the wait.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, int *status, volatile int *abort_flag,
                                          int code, long long budget = kWaitBudget) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, status, abort_flag, code, budget);
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// Tensor store of a shared-memory box to the map's (x, y) (its own bulk group) by one thread;
// x * 4 bytes is a multiple of 16 and x, y >= 0 at every call site.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(src))
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// The thread's bulk stores have read their shared memory (the source may be rewritten).
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// The thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// K-major operand tile in the 128-byte swizzle: rows of 128 bytes, 8-row atoms of 1024 bytes.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16, D fp32, A and B bf16, both K-major, M = 128, N = bn.
__host__ __device__ constexpr uint32_t instr_desc(int bn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// A 16-column load without its wait (the registers are valid after tmem_wait16 on them).
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Waits for the thread's outstanding tensor-memory loads; the registers are passed through so
// that no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_wait16(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

__device__ __forceinline__ void tmem_wait16x2(uint32_t (&r)[16], uint32_t (&u)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(u[0]), "+r"(u[1]), "+r"(u[2]), "+r"(u[3]), "+r"(u[4]), "+r"(u[5]), "+r"(u[6]),
                   "+r"(u[7]), "+r"(u[8]), "+r"(u[9]), "+r"(u[10]), "+r"(u[11]), "+r"(u[12]), "+r"(u[13]),
                   "+r"(u[14]), "+r"(u[15])
                 :
                 : "memory");
}

// Two 16-column loads, one wait: v = columns at a0 + columns at a1.
__device__ __forceinline__ void tmem_ld16_sum2(uint32_t a0, uint32_t a1, float (&v)[16]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%32];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31}, [%33];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(a0), "r"(a1)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
        const float2 a = __fadd2_rn(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])),
                                    make_float2(__uint_as_float(r[16 + i]), __uint_as_float(r[17 + i])));
        v[i] = a.x;
        v[i + 1] = a.y;
    }
}

// Three 16-column loads, one wait.
__device__ __forceinline__ void tmem_ld16x3(uint32_t a0, uint32_t a1, uint32_t a2, float (&v0)[16], float (&v1)[16],
                                            float (&v2)[16]) {
    uint32_t r[48];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%48];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31}, [%49];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, "
        "%45, %46, %47}, [%50];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47])
        : "r"(a0), "r"(a1), "r"(a2)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) {
        v0[i] = __uint_as_float(r[i]);
        v1[i] = __uint_as_float(r[16 + i]);
        v2[i] = __uint_as_float(r[32 + i]);
    }
}

// Four 16-column loads, one wait: v = the sum of the four.
__device__ __forceinline__ void tmem_ld16_sum4(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, float (&v)[16]) {
    float u[16], w[16];
    tmem_ld16_sum2(a0, a1, u);
    tmem_ld16_sum2(a2, a3, w);
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = u[i] + w[i];
}

// Split 8 fp32 values into bf16 hi and lo parts, packed 2 per word.
__device__ __forceinline__ void split8(const float (&v)[8], uint4 &hi, uint4 &lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        __nv_bfloat162 hv = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        float2 hf = __bfloat1622float2(hv);
        __nv_bfloat162 lv = __floats2bfloat162_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
        h[i] = *reinterpret_cast<uint32_t *>(&hv);
        l[i] = *reinterpret_cast<uint32_t *>(&lv);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// 16 channels a lane stored for a whole warp, transposed through the warp's 2 KB staging area
// (`stg`, 128 uint4) so that each store instruction covers 8 pixels x 4 pieces instead of 32
// pixels x 1 piece (fewer lines per instruction).  A lane's channels are 4 pieces of 16 bytes:
// split (y bf16 elements): hi 0-7, hi 8-15 at off, lo 0-7, lo 8-15 at off + y_pix / 2; fp32: 4
// float4 at off.  They are written to the staging area (piece index XORed with bits 1-2 of the
// lane: conflict-free), then lane l stores piece l % 4 of pixel 8 k + l / 4 for k = 0..3.  `off`
// and `valid` are each lane's own pixel; the destination is 16-byte aligned.  Every lane of the
// warp takes part.
__device__ __forceinline__ void warp_store16(void *y, bool split, int64_t y_pix, int64_t off, bool valid,
                                             const float (&v)[16], uint4 *stg, int lane) {
    uint4 q[4];
    if (split) {
        float t[8];
#pragma unroll
        for (int j = 0; j < 8; j++) t[j] = v[j];
        split8(t, q[0], q[2]);
#pragma unroll
        for (int j = 0; j < 8; j++) t[j] = v[8 + j];
        split8(t, q[1], q[3]);
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++)
            q[i] = make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]), __float_as_uint(v[4 * i + 2]),
                              __float_as_uint(v[4 * i + 3]));
    }
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int i = 0; i < 4; i++) stg[lane * 4 + (i ^ sw)] = q[i];
    __syncwarp();
    const int pc = lane & 3;
    // piece pc of a pixel: element offset from its channel 0 (bf16 or fp32 elements)
    const int64_t poff = split ? (int64_t)(pc & 1) * 8 + (pc >> 1) * (y_pix / 2) : (int64_t)pc * 4;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int P = 8 * k + (lane >> 2);
        const int64_t o = __shfl_sync(0xffffffffu, off, P);
        const bool vv = __shfl_sync(0xffffffffu, (int)valid, P) != 0;
        const uint4 val = stg[P * 4 + (pc ^ ((P >> 1) & 3))];
        if (vv) {
            if (split) *reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(y) + o + poff) = val;
            else *reinterpret_cast<uint4 *>(reinterpret_cast<float *>(y) + o + poff) = val;
        }
    }
    __syncwarp();
}

// K-major operand tile with rows of `row_bytes` (32, 64 or 128) in the matching TMA swizzle:
// 8-row atoms of 8 * row_bytes bytes (the stride byte offset), layout codes 6 / 4 / 2.
__device__ __forceinline__ uint64_t smem_desc_sw(uint32_t addr, int row_bytes) {
    const uint64_t layout = row_bytes == 32 ? 6 : (row_bytes == 64 ? 4 : 2);
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)((8 * row_bytes) >> 4) << 32) |
           ((uint64_t)1 << 46) | (layout << 61);
}

// K-major operand without swizzle: 8 x 16-byte core matrices (8 rows of 8 bf16, 128 contiguous
// bytes); `lbo` bytes between the two core matrices of a 16-element K step, `sbo` bytes between
// consecutive 8-row groups.  Start, lbo and sbo are multiples of 16 bytes.
__device__ __forceinline__ uint64_t smem_desc_plain(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}

// Accumulator buffers in tensor memory: as many BN-column fp32 tiles as fit its 512 columns, at
// most 8, so the MMA warp can run that many tiles ahead of the epilogue.
template <int BN>
struct Acc {
    // Independent accumulation chains per tile: consecutive MMAs into one accumulator serialise
    // on its read-modify-write, so narrow tiles (whose MMAs are short) spread the 12 MMAs of a
    // stage over several accumulators and the epilogue adds them up.
    static constexpr int chains = BN <= 16 ? 6 : (BN <= 32 ? 4 : (BN <= 64 ? 2 : 1));
    static constexpr int cols = BN * chains;  // TMEM columns of one tile
    static constexpr int n = 512 / cols < 8 ? 512 / cols : 8;
};

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace tc
}  // namespace k
}  // namespace wocr
