// Warp-level reductions used by the scan kernels.
#pragma once

#include <cuda_runtime.h>

namespace ssm {

// Reduce-scatter of V per-lane values across the R adjacent lanes whose lane-id bits
// 0..log2(R)-1 differ (R a power of two, R <= 32).  With RR = min(R, V): afterwards slot
// j of lane g (j a multiple of RR) holds the R-lane sum of index j + (g & (RR - 1)).  When
// R > V the last log2(R/V) levels are an all-reduce, so lanes that differ only in those
// bits hold the same sums.  Uses a select + one shuffle per exchanged value.
template <int R, int V>
__device__ __forceinline__ void reduce_scatter(float (&v)[V], int g) {
    constexpr int RR = R < V ? R : V;
#pragma unroll
    for (int m = RR / 2; m >= 1; m >>= 1) {
        const bool hi = (g & m) != 0;
#pragma unroll
        for (int j = 0; j < V; j++) {
            if ((j & (RR - 1) & ~(m - 1)) != 0) continue;
            const float send = hi ? v[j] : v[j + m];
            const float keep = hi ? v[j + m] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
    }
#pragma unroll
    for (int m = RR; m < R; m *= 2) {
#pragma unroll
        for (int j = 0; j < V; j += RR) v[j] += __shfl_xor_sync(0xffffffffu, v[j], m);
    }
}

// Reduce-scatter of V = R * Rl per-lane values across the R adjacent lanes (lane-id bits
// 0..log2(R)-1), leaving lane g with the R-lane sums of the CONTIGUOUS indices
// [g*Rl, g*Rl + Rl) in slots 0..Rl-1.  Stage m (lane bit m) pairs index j with j + m*Rl.
template <int R, int V>
__device__ __forceinline__ void reduce_scatter_contig(float (&v)[V], int g) {
    constexpr int Rl = V / R;
    static_assert(V % R == 0, "values must split evenly over the lanes");
#pragma unroll
    for (int m = R / 2; m >= 1; m >>= 1) {
        const bool hi = (g & m) != 0;
#pragma unroll
        for (int j = 0; j < m * Rl; j++) {
            const float send = hi ? v[j] : v[j + m * Rl];
            const float keep = hi ? v[j + m * Rl] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
    }
}

// All-reduce of one value across the R adjacent lanes (R a power of two).
template <int R>
__device__ __forceinline__ float allreduce(float x) {
#pragma unroll
    for (int m = 1; m < R; m *= 2) x += __shfl_xor_sync(0xffffffffu, x, m);
    return x;
}

}  // namespace ssm
