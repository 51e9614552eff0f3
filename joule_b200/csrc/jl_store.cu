// Q4 store: on-device quantiser, repack into the device tile layout, and the
// standalone Q4 GEMV/GEMM over the reference's row-major record layout.
#include <cuda_fp16.h>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

// ---------------------------------------------------------------------------
// Quantiser: one thread per 64-value group, restating _quantize_tensor
// (q4_store.py:40-55): absmax in fp32, scale = fp16_rne(max(absmax,1e-12)/7),
// q = clip(rint(v / fp32(scale)), -8, 7) stored +8, even element low nibble.
// A NaN quotient (0/0 when the scale underflows to 0) becomes q = 0, which is
// what numpy's float->int8 cast yields on x86. Values past n (the padded
// tail of the last group) are stored as nibble 0, as the reference does.
__global__ void k_quantize(const float* __restrict__ x, long long n, uint16_t* __restrict__ scales,
                           uint8_t* __restrict__ packed, long long ngroups) {
    const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= ngroups) return;
    const long long base = g * kGroup;
    const int cnt = (int)min((long long)kGroup, n - base);
    float v[kGroup];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kGroup; i++) {
        v[i] = (i < cnt) ? x[base + i] : 0.0f;
        amax = fmaxf(amax, fabsf(v[i]));
    }
    amax = fmaxf(amax, 1e-12f);
    const __half sh = __float2half_rn(__fdiv_rn(amax, 7.0f));
    const float s = __half2float(sh);
    scales[g] = __half_as_ushort(sh);
    uint32_t words[8];
#pragma unroll
    for (int w = 0; w < 8; w++) {
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = w * 8 + j;
            float q = rintf(__fdiv_rn(v[i], s));
            int qi;
            if (q != q) qi = 0;                       // NaN
            else qi = (int)fminf(fmaxf(q, -8.0f), 7.0f);
            uint32_t nib = (uint32_t)(qi + 8);
            if (i >= cnt) nib = 0u;
            word |= nib << (4 * j);
        }
        words[w] = word;
    }
    uint4* dst = reinterpret_cast<uint4*>(packed + g * kGroupBytes);
    dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
    dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
}

// ---------------------------------------------------------------------------
// Repack one part matrix from the reference layout (packed [R, C/2] u8,
// scales [R, C/64] fp16, row-major) into the device tile records of one
// expert record. Thread = (tile, row t, half h): one 16-byte move; half 0
// also moves the row's scale.
__global__ void k_repack(const uint8_t* __restrict__ pk, const uint16_t* __restrict__ sc, int p,
                         jl_layout L, uint8_t* __restrict__ rec) {
    const int R = p < 2 ? L.m : L.d, C = p < 2 ? L.d : L.m;
    const int ng = C / kGroup;
    const long long ntiles = (long long)(R / kTileRows) * ng;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // tile*64 + h*32 + t
    if (idx >= ntiles * 64) return;
    const long long tile = idx >> 6;
    const int h = (int)(idx >> 5) & 1;
    const int t = (int)idx & 31;
    const int rb = (int)(tile / ng), g = (int)(tile % ng);
    const int row = rb * kTileRows + t;
    uint8_t* dst = rec + L.tile_off(p, rb, g);
    const uint4 v = *reinterpret_cast<const uint4*>(pk + (size_t)row * (C / 2) + (size_t)g * kGroupBytes + h * 16);
    *reinterpret_cast<uint4*>(dst + h * 512 + t * 16) = v;
    if (h == 0) reinterpret_cast<uint16_t*>(dst + kTileBytes)[t] = sc[(size_t)row * ng + g];
}

// ---------------------------------------------------------------------------
// Router weights, lane-major: the reference's row e of gate_w [E, d] becomes
// 8 runs dst[e][j][t] = src[e][j + 8t] (t < d/8), one per lane j of its 8-wide
// accumulator (decode_kernel.c:234-256), each followed by 8 halves of zero
// padding, so the router reads a lane's next 8 steps with one 16-byte load
// and a CTA's experts with one bulk copy. Thread = one destination half.
__global__ void k_repack_router(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int E,
                                int d) {
    const int c8 = d / 8, rh = router_row_halves(d);
    const long long n = (long long)E * 8 * rh;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const long long row = i / rh;
    const int t = (int)(i % rh), j = (int)(row % 8);
    const long long e = row / 8;
    dst[i] = t < c8 ? src[e * d + j + 8 * t] : (uint16_t)0;
}

// ---------------------------------------------------------------------------
// Standalone exact Q4 GEMM over the reference layout: thread = one row, all
// groups in order, up to 8 activation rows per pass staged in shared memory.
// The per-row sum follows decode_kernel.c:770-858 exactly.
constexpr int kGemvRows = 128;
constexpr int kGemvTok = 8;

template <int NT>
__device__ __forceinline__ void gemv_row(const uint8_t* __restrict__ row,
                                         const uint16_t* __restrict__ sc, const float* xs, int d,
                                         float (&acc)[kGemvTok]) {
    const int ng = d / kGroup;
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t] = 0.0f;
    for (int g = 0; g < ng; g++) {
        const uint4 q0 = __ldg(reinterpret_cast<const uint4*>(row + g * kGroupBytes));
        const uint4 q1 = __ldg(reinterpret_cast<const uint4*>(row + g * kGroupBytes + 16));
        const float s = fp16_to_f32(__ldg(sc + g));
        const uint32_t wq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        float lane[NT][8];
#pragma unroll
        for (int t = 0; t < NT; t++)
#pragma unroll
            for (int j = 0; j < 8; j++) lane[t][j] = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) {
            float a[8];
            dequant8(wq[w], a);
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float4 x0 = *reinterpret_cast<const float4*>(xs + t * d + g * kGroup + w * 8);
                const float4 x1 = *reinterpret_cast<const float4*>(xs + t * d + g * kGroup + w * 8 + 4);
                lane[t][0] = __fmaf_rn(a[0], x0.x, lane[t][0]);
                lane[t][1] = __fmaf_rn(a[1], x0.y, lane[t][1]);
                lane[t][2] = __fmaf_rn(a[2], x0.z, lane[t][2]);
                lane[t][3] = __fmaf_rn(a[3], x0.w, lane[t][3]);
                lane[t][4] = __fmaf_rn(a[4], x1.x, lane[t][4]);
                lane[t][5] = __fmaf_rn(a[5], x1.y, lane[t][5]);
                lane[t][6] = __fmaf_rn(a[6], x1.z, lane[t][6]);
                lane[t][7] = __fmaf_rn(a[7], x1.w, lane[t][7]);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = __fadd_rn(acc[t], __fmul_rn(hsum8(lane[t]), s));
    }
}

__global__ void __launch_bounds__(kGemvRows) k_q4_gemm_ref(float* __restrict__ out,
                                                           const float* __restrict__ X, int T,
                                                           const uint8_t* __restrict__ pk,
                                                           const uint16_t* __restrict__ sc, int m,
                                                           int d) {
    extern __shared__ __align__(16) float xs[];  // [kGemvTok, d]
    const int t0 = blockIdx.y * kGemvTok;
    const int nt = min(kGemvTok, T - t0);
    for (int i = threadIdx.x; i < nt * d / 4; i += blockDim.x)
        reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(X + (size_t)t0 * d)[i];
    __syncthreads();
    const int row = blockIdx.x * kGemvRows + threadIdx.x;
    if (row >= m) return;
    const uint8_t* r = pk + (size_t)row * (d / 2);
    const uint16_t* s = sc + (size_t)row * (d / kGroup);
    float acc[kGemvTok];
    switch (nt) {
        case 1: gemv_row<1>(r, s, xs, d, acc); break;
        case 2: gemv_row<2>(r, s, xs, d, acc); break;
        case 3: gemv_row<3>(r, s, xs, d, acc); break;
        case 4: gemv_row<4>(r, s, xs, d, acc); break;
        case 5: gemv_row<5>(r, s, xs, d, acc); break;
        case 6: gemv_row<6>(r, s, xs, d, acc); break;
        case 7: gemv_row<7>(r, s, xs, d, acc); break;
        default: gemv_row<8>(r, s, xs, d, acc); break;
    }
    for (int t = 0; t < nt; t++) out[(size_t)(t0 + t) * m + row] = acc[t];
}

}  // namespace jl

// ---------------------------------------------------------------------------
// Host entry points.

extern "C" int jl_q4_quantize(const float* x, long long n, unsigned short* scales,
                              unsigned char* packed, void* stream) {
    if (!x || !scales || !packed || n <= 0) return JL_ERR_INVALID;
    const long long ng = (n + jl::kGroup - 1) / jl::kGroup;
    const int tpb = 128;
    const long long blocks = (ng + tpb - 1) / tpb;
    if (blocks > 0x7FFFFFFFll) return JL_ERR_INVALID;
    jl::k_quantize<<<(unsigned)blocks, tpb, 0, (cudaStream_t)stream>>>(x, n, scales, packed, ng);
    JL_LAUNCH_CHECK();
    return JL_OK;
}

int jl_launch_repack_part(const uint8_t* pk_ref, const uint16_t* sc_ref, int p, const jl_layout& L,
                          uint8_t* rec, cudaStream_t s) {
    const int R = p < 2 ? L.m : L.d, C = p < 2 ? L.d : L.m;
    if (R % jl::kTileRows || C % jl::kGroup) return JL_ERR_INVALID;
    const long long threads = (long long)(R / jl::kTileRows) * (C / jl::kGroup) * 64;
    const int tpb = 256;
    jl::k_repack<<<(unsigned)((threads + tpb - 1) / tpb), tpb, 0, s>>>(pk_ref, sc_ref, p, L, rec);
    JL_LAUNCH_CHECK();
    return JL_OK;
}

int jl_launch_repack_router(const uint16_t* src, uint16_t* dst, int E, int d, cudaStream_t s) {
    if (E < 1 || d < 8 || d % 8) return JL_ERR_INVALID;
    const long long n = (long long)E * router_expert_halves(d);
    const int tpb = 256;
    jl::k_repack_router<<<(unsigned)((n + tpb - 1) / tpb), tpb, 0, s>>>(src, dst, E, d);
    JL_LAUNCH_CHECK();
    return JL_OK;
}

static int q4_gemm_common(float* out, const float* X, int T, const unsigned char* packed,
                          const unsigned short* scales, int m, int d, int group, void* stream) {
    if (!out || !X || !packed || !scales) return JL_ERR_INVALID;
    if (group != jl::kGroup || d <= 0 || d % jl::kGroup || m <= 0 || T <= 0) return JL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(X)) & 15)
        return JL_ERR_INVALID;
    const size_t smem = (size_t)jl::kGemvTok * d * sizeof(float);
    if (smem > 200 * 1024) return JL_ERR_INVALID;
    const int rc = jl_device_once(kOnceGemm, [] {
        JL_CUDA(cudaFuncSetAttribute(jl::k_q4_gemm_ref, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024));
        return JL_OK;
    });
    if (rc) return rc;
    dim3 grid((m + jl::kGemvRows - 1) / jl::kGemvRows, (T + jl::kGemvTok - 1) / jl::kGemvTok);
    jl::k_q4_gemm_ref<<<grid, jl::kGemvRows, smem, (cudaStream_t)stream>>>(out, X, T, packed,
                                                                          scales, m, d);
    JL_LAUNCH_CHECK();
    return JL_OK;
}

extern "C" int jl_q4_gemv_f32(float* out, const float* x, const unsigned char* packed,
                              const unsigned short* scales, int m, int d, int group, void* stream) {
    return q4_gemm_common(out, x, 1, packed, scales, m, d, group, stream);
}

extern "C" int jl_q4_gemm_f32(float* out, const float* X, int T, const unsigned char* packed,
                              const unsigned short* scales, int m, int d, int group, void* stream) {
    return q4_gemm_common(out, X, T, packed, scales, m, d, group, stream);
}
