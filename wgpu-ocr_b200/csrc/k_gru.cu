// GRU recurrence (ONNX, linear_before_reset = 1, hidden 256, gate order z, r, h) for all lines
// and both directions in one launch per layer -- the reference's K16/K17 (src/gpu.rs:680-819).
//
// B200 design: one thread-block cluster of 8 CTAs per (direction, group of L lines).  CTA c of
// the cluster owns hidden units 32c .. 32c + 32 and keeps their three gate rows of R (3 x 32 x 256
// fp32 = 96 KB, padded to 128 KB) in shared memory for the whole sequence.  Every step:
//   1. each CTA computes its rows' dot products with h for its L lines (thread = unit x k-slice,
//      R read as one float4 of the unit's z/r/h weights, h broadcast as float4),
//   2. the 8 k-slices (one warp each) are summed, the gate nonlinearity gives the new h for its
//      32 units (the step's input gates were loaded during the previous step),
//   3. the new h is stored into every CTA's next-step buffer through distributed shared memory
//      and `barrier.cluster` (hardware co-scheduled CTAs: no global-memory spin waits) publishes
//      it: arrive right after the stores, wait before the next step reads h.
// Each line runs for its own length; the backward direction starts at len - 1 (src/gpu.rs:797-800).
#include <atomic>
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "kernels.h"

namespace cg = cooperative_groups;

namespace wocr {
namespace k {

namespace {

constexpr int kHid = 256;
constexpr int kCluster = 8;
constexpr int kUnits = kHid / kCluster;  // 32 hidden units per CTA
constexpr int kSlices = 8;               // k split over 8 warps
constexpr int kThreadsG = kSlices * 32;
constexpr int kSliceLen = kHid / kSlices;

__device__ __forceinline__ float sigm(float v) { return 1.0f / (1.0f + expf(-v)); }

// h of L lines at one k (L consecutive floats, 4 L-byte aligned) as vector loads
template <int L>
__device__ __forceinline__ void load_h(const float *p, float (&h)[L]) {
    if (L % 4 == 0) {
#pragma unroll
        for (int i = 0; i < L / 4; i++) {
            const float4 v = reinterpret_cast<const float4 *>(p)[i];
            h[4 * i] = v.x;
            h[4 * i + 1] = v.y;
            h[4 * i + 2] = v.z;
            h[4 * i + 3] = v.w;
        }
    } else if (L == 2) {
        const float2 v = *reinterpret_cast<const float2 *>(p);
        h[0] = v.x;
        h[L - 1] = v.y;
    } else {
        h[0] = p[0];
    }
}

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

template <int L>
__global__ void __launch_bounds__(kThreadsG) k_gru(const float *__restrict__ g, const float *__restrict__ r,
                                            const float *__restrict__ rb, const int *__restrict__ lens, int tmax,
                                            int ntot, float *__restrict__ y) {
    extern __shared__ __align__(16) float smem[];
    float4 *Rs = reinterpret_cast<float4 *>(smem);              // [256 k][32 u] (z, r, h, 0)
    float *hbuf = smem + kHid * kUnits * 4;                       // [2][256 k][L]
    float *red = hbuf + 2 * kHid * L;                             // [8 slices][3][L][32 u]

    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int dir = blockIdx.y;
    const int group = blockIdx.x / kCluster;
    const int line0 = group * L;
    const int u0 = crank * kUnits;
    const int tid = threadIdx.x;

    // R rows of this CTA's units, k-major
    const float *Rd = r + (size_t)dir * 3 * kHid * kHid;
    for (int i = tid; i < kHid * kUnits; i += blockDim.x) {
        int u = i % kUnits, kk = i / kUnits;
        float4 v;
        v.x = Rd[(size_t)(0 * kHid + u0 + u) * kHid + kk];
        v.y = Rd[(size_t)(1 * kHid + u0 + u) * kHid + kk];
        v.z = Rd[(size_t)(2 * kHid + u0 + u) * kHid + kk];
        v.w = 0.f;
        Rs[kk * kUnits + u] = v;
    }
    for (int i = tid; i < 2 * kHid * L; i += blockDim.x) hbuf[i] = 0.f;

    int steps = 0;
#pragma unroll
    for (int l = 0; l < L; l++) {
        int len = line0 + l < ntot ? lens[line0 + l] : 0;
        steps = max(steps, min(len, tmax));
    }
    // phase-2 role of this thread: unit u2, line l2
    const int u2 = tid % kUnits, l2 = tid / kUnits;
    const int j = u0 + u2;
    const int line = line0 + l2;
    const bool owner = l2 < L && line < ntot;
    const int mylen = owner ? min(lens[line], tmax) : 0;
    float bz = 0.f, br = 0.f, bh = 0.f;
    if (owner) {
        bz = rb[dir * 768 + j];
        br = rb[dir * 768 + 256 + j];
        bh = rb[dir * 768 + 512 + j];
    }
    // phase-1 role: unit u1, k-slice sl
    const int u1 = tid % kUnits, sl = tid / kUnits;
    // the input-gate values of this thread's (unit, line) for the next step, loaded a step ahead
    auto gate_ptr = [&](int s) {
        const int t = dir == 0 ? s : mylen - 1 - s;
        return g + ((size_t)t * ntot + line) * 1536 + dir * 768;
    };
    float gz = 0.f, gr = 0.f, gh = 0.f;
    if (owner && mylen > 0) {
        const float *gb = gate_ptr(0);
        gz = gb[j];
        gr = gb[256 + j];
        gh = gb[512 + j];
    }
    cluster.sync();

    for (int s = 0; s < steps; s++) {
        const float *hc = hbuf + (s & 1) * kHid * L;
        float *hn_buf = hbuf + ((s + 1) & 1) * kHid * L;
        float az[L], ar[L], ah[L];
#pragma unroll
        for (int l = 0; l < L; l++) az[l] = ar[l] = ah[l] = 0.f;
#pragma unroll 4
        for (int kk = 0; kk < kSliceLen; kk++) {
            int k = sl * kSliceLen + kk;
            float4 w = Rs[k * kUnits + u1];
            float hv[L];
            load_h<L>(hc + k * L, hv);
#pragma unroll
            for (int l = 0; l < L; l++) {
                az[l] += w.x * hv[l];
                ar[l] += w.y * hv[l];
                ah[l] += w.z * hv[l];
            }
        }
        float *rd = red + (size_t)sl * 3 * L * kUnits + u1;
#pragma unroll
        for (int l = 0; l < L; l++) {
            rd[l * kUnits] = az[l];
            rd[(L + l) * kUnits] = ar[l];
            rd[(2 * L + l) * kUnits] = ah[l];
        }
        __syncthreads();
        float hn = 0.f;
        bool wrote = false;
        if (l2 < L) {
            float hold = hc[j * L + l2];
            hn = hold;
            if (owner && s < mylen) {
                float pz = 0.f, pr = 0.f, ph = 0.f;
#pragma unroll
                for (int q = 0; q < kSlices; q++) {
                    const float *rq = red + (size_t)q * 3 * L * kUnits + u2;
                    pz += rq[l2 * kUnits];
                    pr += rq[(L + l2) * kUnits];
                    ph += rq[(2 * L + l2) * kUnits];
                }
                float z = sigm(gz + pz + bz);
                float rr = sigm(gr + pr + br);
                float c = tanhf(gh + rr * (ph + bh));
                hn = (1.0f - z) * c + z * hold;
                wrote = true;
            }
#pragma unroll
            for (int q = 0; q < kCluster; q++) {
                float *dst = cluster.map_shared_rank(hn_buf + j * L + l2, q);
                *dst = hn;
            }
        }
        // publish h (release), then store y and fetch the next step's gates while the other
        // CTAs catch up, then wait for theirs (acquire)
        cluster_arrive();
        if (wrote) {
            const int t = dir == 0 ? s : mylen - 1 - s;
            y[((size_t)t * ntot + line) * 512 + dir * 256 + j] = hn;
            if (s + 1 < mylen) {
                const float *gb = gate_ptr(s + 1);
                gz = gb[j];
                gr = gb[256 + j];
                gh = gb[512 + j];
            }
        }
        cluster_wait();
    }
}

template <int L>
size_t gru_smem() {
    return sizeof(float) * ((size_t)kHid * kUnits * 4 + 2 * kHid * L + (size_t)kSlices * kUnits * 3 * L);
}

template <int L>
void launch_gru(Ctx *c, const float *g, const float *r, const float *rb, const int *lens, int tmax, int ntot,
                float *y) {
    size_t smem = gru_smem<L>();
    static std::atomic<bool> configured[64];
    if (!configured[c->device]) {
        WOCR_CUDA(cudaFuncSetAttribute(k_gru<L>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured[c->device] = true;
    }
    int groups = (ntot + L - 1) / L;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(groups * kCluster, 2, 1);
    cfg.blockDim = dim3(kThreadsG, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    WOCR_CUDA(cudaLaunchKernelEx(&cfg, k_gru<L>, g, r, rb, lens, tmax, ntot, y));
    WOCR_LAUNCHED(c);
}

template <int L>
int max_clusters(Ctx *c) {
    static std::atomic<int> cached[64];
    if (cached[c->device]) return cached[c->device];
    size_t smem = gru_smem<L>();
    WOCR_CUDA(cudaFuncSetAttribute(k_gru<L>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCluster * 64, 2, 1);
    cfg.blockDim = dim3(kThreadsG, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    WOCR_CUDA(cudaOccupancyMaxActiveClusters(&n, k_gru<L>, &cfg));
    cached[c->device] = n > 0 ? n : 1;
    return cached[c->device];
}

}  // namespace

void gru_layer(Ctx *c, const float *g, const float *r, const float *rb, const int *lens, int tmax, int ntot,
               float *y) {
    if (ntot == 0 || tmax == 0) return;
    Prof pf(c, "gru", 2.0 * 2.0 * ntot * (double)tmax * 768.0 * 256.0,
            4.0 * (double)tmax * ntot * (1536.0 + 512.0) + 4.0 * 2 * 768 * 256);
    // The fewest lines per cluster that still fit all clusters of both directions at once.
    auto fits = [&](int L, int maxc) { return 2 * ((ntot + L - 1) / L) <= maxc; };
    if (fits(1, max_clusters<1>(c))) launch_gru<1>(c, g, r, rb, lens, tmax, ntot, y);
    else if (fits(2, max_clusters<2>(c))) launch_gru<2>(c, g, r, rb, lens, tmax, ntot, y);
    else if (fits(4, max_clusters<4>(c))) launch_gru<4>(c, g, r, rb, lens, tmax, ntot, y);
    else launch_gru<8>(c, g, r, rb, lens, tmax, ntot, y);
    c->flops += 2.0 * 2.0 * ntot * (double)tmax * 768.0 * 256.0;
}

}  // namespace k
}  // namespace wocr
