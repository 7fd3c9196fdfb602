// GRU recurrence (ONNX, linear_before_reset = 1, hidden 256, gate order z, r, h) for all lines
// and both directions in one launch per layer -- the reference's K16/K17 (src/gpu.rs:680-819).
//
// The recurrent weights are fp16, as the reference's GPU path keeps them (src/gpu.rs:1478-1487:
// R converted to f16 when the device has shader-f16), with fp32 accumulation.
//
// B200 design: one thread-block cluster of 4 CTAs per (direction, group of L = 8 or 16 lines).
// CTA c of the cluster owns hidden units 64c .. 64c + 64, i.e. 192 rows of R (64 units x 3 gates),
// and holds them for the whole sequence in registers, as the A fragments of m16n8k16 tensor-core
// products: warp w < 12 owns the 16 rows (gate w / 4, units 16 (w % 4) ..) over all 256 k, 16
// fragments of 4 registers.  Every step:
//   1. each of the 12 warps multiplies its rows with h, the B operand read from shared memory as
//      fp16 hi and lo parts (h = hi + lo to about 2^-22, so the products are those of fp16 R with
//      the fp32 h: two products per k tile, accumulated in fp32), and leaves its 16 x L
//      pre-activations in shared memory;
//   2. one thread per (pair of units, line) applies the gates (the step's input-gate values were
//      fetched during the previous step), keeps its fp32 h in registers and stores the new h's
//      hi / lo parts into every CTA of the cluster through distributed shared memory;
//   3. `barrier.cluster` (hardware co-scheduled CTAs, no global-memory spin waits) publishes h:
//      arrive right after the stores, wait before the next step reads it.
// Each line runs for its own length; the backward direction starts at len - 1 (src/gpu.rs:797-800).
#include <atomic>
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"

namespace cg = cooperative_groups;

namespace wocr {
namespace k {

namespace {

constexpr int kHid = 256;
constexpr int kCluster = 4;
constexpr int kUnits = kHid / kCluster;  // 64 hidden units per CTA
constexpr int kKT = kHid / 16;           // k tiles of the m16n8k16 products
constexpr int kMatWarps = 12;            // 3 gates x 4 tiles of 16 units
constexpr int kThreadsG = 512;
constexpr int kHS = kHid + 8;            // halves per line row of h (pads the banks apart)

__device__ __forceinline__ float sigm(float v) { return 1.0f / (1.0f + expf(-v)); }

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// shared memory: h [2 buffers][hi, lo][L lines][kHS halves], pre-activations [3][L][64] floats
template <int L>
constexpr size_t gru_smem() {
    return sizeof(__half) * 2 * 2 * L * kHS + sizeof(float) * 3 * L * kUnits;
}

template <int NT>
__global__ void __launch_bounds__(kThreadsG, 1) k_gru(const float *__restrict__ g, const float *__restrict__ r,
                                                      const float *__restrict__ rb, const int *__restrict__ lens,
                                                      int tmax, int ntot, float *__restrict__ y) {
    constexpr int L = 8 * NT;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half *hs = reinterpret_cast<__half *>(smem_raw);                                     // [2][2][L][kHS]
    float *pre = reinterpret_cast<float *>(smem_raw + sizeof(__half) * 2 * 2 * L * kHS);  // [3][L][64]

    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int dir = blockIdx.y;
    const int line0 = (blockIdx.x / kCluster) * L;
    const int u0 = crank * kUnits;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane >> 2, tig = lane & 3;

    // the A fragments of this warp's 16 rows, fp16, for the whole sequence
    uint32_t a[kKT][4];
    const int gate = warp / 4, ut = warp % 4;
    if (warp < kMatWarps) {
        const float *Rd = r + (size_t)dir * 3 * kHid * kHid;
        const float *r0 = Rd + (size_t)(gate * kHid + u0 + ut * 16 + grp) * kHid;
        const float *r8 = r0 + (size_t)8 * kHid;
#pragma unroll
        for (int kt = 0; kt < kKT; kt++) {
            const int k0 = kt * 16 + 2 * tig;
            a[kt][0] = pack2(r0[k0], r0[k0 + 1]);
            a[kt][1] = pack2(r8[k0], r8[k0 + 1]);
            a[kt][2] = pack2(r0[k0 + 8], r0[k0 + 9]);
            a[kt][3] = pack2(r8[k0 + 8], r8[k0 + 9]);
        }
    }
    for (int i = tid; i < 2 * 2 * L * kHS / 2; i += kThreadsG) reinterpret_cast<uint32_t *>(hs)[i] = 0u;

    int steps = 0;
#pragma unroll
    for (int l = 0; l < L; l++) {
        const int len = line0 + l < ntot ? lens[line0 + l] : 0;
        steps = max(steps, min(len, tmax));
    }
    // gate role: a pair of units (2 up, 2 up + 1 of this CTA) of one line
    const int up = tid % 32, gl = tid / 32;
    const bool gater = gl < L;
    const int line = line0 + gl;
    const bool owner = gater && line < ntot;
    const int mylen = owner ? min(lens[line], tmax) : 0;
    const int j0 = u0 + 2 * up;  // the pair's first unit in the layer
    float bz[2] = {0.f, 0.f}, br[2] = {0.f, 0.f}, bh[2] = {0.f, 0.f};
    float hold[2] = {0.f, 0.f};
    float gz[2] = {0.f, 0.f}, gr[2] = {0.f, 0.f}, gh[2] = {0.f, 0.f};
    auto gate_ptr = [&](int s) {
        const int t = dir == 0 ? s : mylen - 1 - s;
        return g + ((size_t)t * ntot + line) * 1536 + dir * 768;
    };
    if (owner) {
#pragma unroll
        for (int q = 0; q < 2; q++) {
            bz[q] = rb[dir * 768 + j0 + q];
            br[q] = rb[dir * 768 + 256 + j0 + q];
            bh[q] = rb[dir * 768 + 512 + j0 + q];
        }
        if (mylen > 0) {
            const float *gb = gate_ptr(0);
#pragma unroll
            for (int q = 0; q < 2; q++) {
                gz[q] = gb[j0 + q];
                gr[q] = gb[256 + j0 + q];
                gh[q] = gb[512 + j0 + q];
            }
        }
    }
    cluster.sync();

    for (int s = 0; s < steps; s++) {
        const __half *hc = hs + (size_t)(s & 1) * 2 * L * kHS;
        __half *hn_buf = hs + (size_t)((s + 1) & 1) * 2 * L * kHS;
        if (warp < kMatWarps) {
            float acc[2][NT][4];
#pragma unroll
            for (int c = 0; c < 2; c++)
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                    for (int q = 0; q < 4; q++) acc[c][nt][q] = 0.f;
#pragma unroll
            for (int kt = 0; kt < kKT; kt++) {
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const __half *hi = hc + (size_t)(nt * 8 + grp) * kHS + kt * 16 + 2 * tig;
                    const __half *lo = hi + (size_t)L * kHS;
                    const uint32_t h0 = *reinterpret_cast<const uint32_t *>(hi);
                    const uint32_t h1 = *reinterpret_cast<const uint32_t *>(hi + 8);
                    const uint32_t l0 = *reinterpret_cast<const uint32_t *>(lo);
                    const uint32_t l1 = *reinterpret_cast<const uint32_t *>(lo + 8);
                    mma16816(acc[kt & 1][nt], a[kt], h0, h1);
                    mma16816(acc[kt & 1][nt], a[kt], l0, l1);
                }
            }
            // rows = units (grp, grp + 8), columns = lines (2 tig, 2 tig + 1)
            float *pg = pre + (size_t)gate * L * kUnits;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int ln = nt * 8 + 2 * tig, u = ut * 16 + grp;
                pg[(size_t)ln * kUnits + u] = acc[0][nt][0] + acc[1][nt][0];
                pg[(size_t)(ln + 1) * kUnits + u] = acc[0][nt][1] + acc[1][nt][1];
                pg[(size_t)ln * kUnits + u + 8] = acc[0][nt][2] + acc[1][nt][2];
                pg[(size_t)(ln + 1) * kUnits + u + 8] = acc[0][nt][3] + acc[1][nt][3];
            }
        }
        __syncthreads();
        bool wrote = false;
        float hn[2] = {hold[0], hold[1]};
        if (gater) {
            if (owner && s < mylen) {
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const int u = 2 * up + q;
                    const float pz = pre[(size_t)(0 * L + gl) * kUnits + u];
                    const float pr = pre[(size_t)(1 * L + gl) * kUnits + u];
                    const float ph = pre[(size_t)(2 * L + gl) * kUnits + u];
                    const float z = sigm(gz[q] + pz + bz[q]);
                    const float rr = sigm(gr[q] + pr + br[q]);
                    const float cc = tanhf(gh[q] + rr * (ph + bh[q]));
                    hn[q] = (1.0f - z) * cc + z * hold[q];
                }
                wrote = true;
            }
            hold[0] = hn[0];
            hold[1] = hn[1];
            const __half hi0 = __float2half_rn(hn[0]), hi1 = __float2half_rn(hn[1]);
            const __half2 hi2 = __halves2half2(hi0, hi1);
            const __half2 lo2 = __floats2half2_rn(hn[0] - __half2float(hi0), hn[1] - __half2float(hi1));
            const uint32_t hv = *reinterpret_cast<const uint32_t *>(&hi2), lv = *reinterpret_cast<const uint32_t *>(&lo2);
            __half *dst_hi = hn_buf + (size_t)gl * kHS + j0, *dst_lo = dst_hi + (size_t)L * kHS;
#pragma unroll
            for (int q = 0; q < kCluster; q++) {
                *reinterpret_cast<uint32_t *>(cluster.map_shared_rank(dst_hi, q)) = hv;
                *reinterpret_cast<uint32_t *>(cluster.map_shared_rank(dst_lo, q)) = lv;
            }
        }
        // publish h (release), then store y and fetch the next step's gates while the other
        // CTAs catch up, then wait for theirs (acquire)
        cluster_arrive();
        if (wrote) {
            const int t = dir == 0 ? s : mylen - 1 - s;
            float *yo = y + ((size_t)t * ntot + line) * 512 + dir * 256 + j0;
            *reinterpret_cast<float2 *>(yo) = make_float2(hn[0], hn[1]);
            if (s + 1 < mylen) {
                const float *gb = gate_ptr(s + 1);
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    gz[q] = gb[j0 + q];
                    gr[q] = gb[256 + j0 + q];
                    gh[q] = gb[512 + j0 + q];
                }
            }
        }
        cluster_wait();
    }
}

template <int NT>
cudaLaunchConfig_t gru_config(Ctx *c, int clusters, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(clusters * kCluster, 2, 1);
    cfg.blockDim = dim3(kThreadsG, 1, 1);
    cfg.dynamicSmemBytes = gru_smem<8 * NT>();
    cfg.stream = c->stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

template <int NT>
void configure(Ctx *c) {
    static std::atomic<bool> configured[64];
    if (!configured[c->device]) {
        WOCR_CUDA(cudaFuncSetAttribute(k_gru<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)gru_smem<8 * NT>()));
        configured[c->device] = true;
    }
}

template <int NT>
void launch_gru(Ctx *c, const float *g, const float *r, const float *rb, const int *lens, int tmax, int ntot,
                float *y) {
    configure<NT>(c);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = gru_config<NT>(c, (ntot + 8 * NT - 1) / (8 * NT), attr);
    WOCR_CUDA(cudaLaunchKernelEx(&cfg, k_gru<NT>, g, r, rb, lens, tmax, ntot, y));
    WOCR_LAUNCHED(c);
}

// clusters of the NT instance resident at once (both directions count)
template <int NT>
int max_clusters(Ctx *c) {
    static std::atomic<int> cached[64];
    if (cached[c->device]) return cached[c->device];
    configure<NT>(c);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = gru_config<NT>(c, 32, attr);
    int n = 0;
    WOCR_CUDA(cudaOccupancyMaxActiveClusters(&n, k_gru<NT>, &cfg));
    cached[c->device] = n > 0 ? n : 1;
    return cached[c->device];
}

}  // namespace

void gru_layer(Ctx *c, const float *g, const float *r, const float *rb, const int *lens, int tmax, int ntot,
               float *y) {
    if (ntot == 0 || tmax == 0) return;
    Prof pf(c, "gru", 2.0 * 2.0 * ntot * (double)tmax * 768.0 * 256.0,
            4.0 * (double)tmax * ntot * (1536.0 + 512.0) + 4.0 * 2 * 768 * 256);
    // 8 lines a cluster while both directions' clusters are all resident at once, else 16
    if (2 * ((ntot + 7) / 8) <= max_clusters<1>(c))
        launch_gru<1>(c, g, r, rb, lens, tmax, ntot, y);
    else
        launch_gru<2>(c, g, r, rb, lens, tmax, ntot, y);
    c->flops += 2.0 * 2.0 * ntot * (double)tmax * 768.0 * 256.0;
}

}  // namespace k
}  // namespace wocr
