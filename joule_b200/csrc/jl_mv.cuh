// Matvec helpers in the reference's 8-lane FMA order, shared by the decode
// step (jl_decode.cu) and the bf16 expert tier (jl_bf16.cu).
//
// Weight layout (coalesced 16-byte loads): matrix W [N, K] is stored as
// W'[c][n][j][u] = W[n][j + 8*(U*c + u)] with U = 8 values per 16 bytes for
// bf16 (4 for fp32); thread (row n, lane j) reads chunk c as one 16-byte load
// and lane j's accumulator takes the products of columns j, j+8, j+16, ... in
// column order by fused multiply-add, as one lane of the reference's AVX2
// accumulator does (decode_kernel.c:693-718, 969-995, 934-957).
#pragma once

#include "jl_common.cuh"

namespace jl {

template <typename WT>
struct mv_traits;
template <>
struct mv_traits<uint16_t> {
    static constexpr int U = 8;  // values per 16-byte chunk
};
template <>
struct mv_traits<float> {
    static constexpr int U = 4;
};

__device__ __forceinline__ void fma_chunk(const uint4 w, const float* xp, float& acc, uint16_t) {
    const float4 x0 = *reinterpret_cast<const float4*>(xp);
    const float4 x1 = *reinterpret_cast<const float4*>(xp + 4);
    acc = __fmaf_rn(__uint_as_float(w.x << 16), x0.x, acc);
    acc = __fmaf_rn(__uint_as_float(w.x & 0xFFFF0000u), x0.y, acc);
    acc = __fmaf_rn(__uint_as_float(w.y << 16), x0.z, acc);
    acc = __fmaf_rn(__uint_as_float(w.y & 0xFFFF0000u), x0.w, acc);
    acc = __fmaf_rn(__uint_as_float(w.z << 16), x1.x, acc);
    acc = __fmaf_rn(__uint_as_float(w.z & 0xFFFF0000u), x1.y, acc);
    acc = __fmaf_rn(__uint_as_float(w.w << 16), x1.z, acc);
    acc = __fmaf_rn(__uint_as_float(w.w & 0xFFFF0000u), x1.w, acc);
}
__device__ __forceinline__ void fma_chunk(const uint4 w, const float* xp, float& acc, float) {
    const float4 x0 = *reinterpret_cast<const float4*>(xp);
    acc = __fmaf_rn(__uint_as_float(w.x), x0.x, acc);
    acc = __fmaf_rn(__uint_as_float(w.y), x0.y, acc);
    acc = __fmaf_rn(__uint_as_float(w.z), x0.z, acc);
    acc = __fmaf_rn(__uint_as_float(w.w), x0.w, acc);
}

__host__ __device__ inline int mv_xstride(int K) { return K / 8 + 4; }

// W [N, K] (row-major, device) -> the chunked lane-major layout.
template <typename WT>
__global__ void k_repack_mv(const WT* __restrict__ src, WT* __restrict__ dst, int N, int K) {
    constexpr int U = mv_traits<WT>::U;
    const size_t total = (size_t)N * K;
    for (size_t o = blockIdx.x * (size_t)blockDim.x + threadIdx.x; o < total; o += (size_t)gridDim.x * blockDim.x) {
        // o = ((c * N + n) * 8 + j) * U + u
        const int u = (int)(o % U);
        const int j = (int)((o / U) % 8);
        const size_t cn = o / (8 * U);
        const int n = (int)(cn % N);
        const int c = (int)(cn / N);
        dst[o] = src[(size_t)n * K + j + 8 * (U * c + u)];
    }
}

}  // namespace jl
