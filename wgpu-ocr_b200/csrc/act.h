// The activations the fused epilogues apply (codes of the graph builder: 0 none, 1 ReLU,
// 2 sigmoid, 3 GELU with the erf below, 4 SiLU), shared by every kernel that fuses one.
#pragma once

#include <cuda_runtime.h>

namespace wocr {
namespace k {

// Abramowitz & Stegun 7.1.26, the erf of the reference's epilogue (src/gpu.rs:19-27).
__device__ __forceinline__ float erf_as(float v) {
    float s = (v > 0.f) - (v < 0.f);
    float a = fabsf(v);
    float t = 1.0f / (1.0f + 0.3275911f * a);
    float poly = ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    return s * (1.0f - poly * expf(-a * a));
}

__device__ __forceinline__ float act_f(float v, int act) {
    switch (act) {
    case 1: return fmaxf(v, 0.f);
    case 2: return 1.0f / (1.0f + expf(-v));
    case 3: return 0.5f * v * (1.0f + erf_as(v * 0.70710678118654752f));
    case 4: return v / (1.0f + expf(-v));
    default: return v;
    }
}

// act_f of N values with the code tested once.  Each case is its own unrolled loop, so a launch
// runs one short straight stretch of code; N inlined act_f calls would put N dispatches over
// the code of every case in the loop, and with the sigmoid / GELU / SiLU bodies such a loop no
// longer fits the instruction cache, so every pass over it stalls on instruction fetch.
template <int N>
__device__ __forceinline__ void act_n(float (&v)[N], int act) {
    switch (act) {
    case 1:
#pragma unroll
        for (int j = 0; j < N; j++) v[j] = fmaxf(v[j], 0.f);
        break;
    case 2:
#pragma unroll
        for (int j = 0; j < N; j++) v[j] = 1.0f / (1.0f + expf(-v[j]));
        break;
    case 3:
#pragma unroll
        for (int j = 0; j < N; j++) v[j] = 0.5f * v[j] * (1.0f + erf_as(v[j] * 0.70710678118654752f));
        break;
    case 4:
#pragma unroll
        for (int j = 0; j < N; j++) v[j] = v[j] / (1.0f + expf(-v[j]));
        break;
    default: break;
    }
}

}  // namespace k
}  // namespace wocr
