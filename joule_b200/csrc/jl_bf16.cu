// The bf16 expert tier (KernelCfg.expert_bf16): gate, up and down of every
// expert as bf16 matrices, no quantisation (decode_kernel.c:1276-1301, the
// reference's drift-free tier). Each expert row is dotted with its tokens by
// bf16_row_dot_B's arithmetic (decode_kernel.c:934-957): eight FMA lanes over
// the columns in order, then the AVX tree, so act, y and the layer output are
// the reference's bits.
//
// Store: per expert record [gate'][up'][down'], each matrix in the chunked
// lane-major layout of jl_mv.cuh (gate/up [m, d], down [d, m]).
// Kernels: k_bf16_gateup (block = 16 rows of one union expert's gate and up
// matrices against the expert's tokens, SwiGLU in the epilogue) and
// k_bf16_down (16 rows of the down matrix against the expert's act rows,
// y = 0 + w * dot); the existing combine adds the slots in union order.
#include <algorithm>

#include "jl_common.cuh"
#include "jl_internal.h"
#include "jl_mv.cuh"

namespace jl {

constexpr int kBfRows = 16;  // rows per block (x 8 lanes = 128 threads)
constexpr int kBfTok = 8;    // tokens per pass

// Token rows x_rows[t] (t < nt, K floats each) into lane-major shared rows.
__device__ __forceinline__ void stage_rows(float* x_s, const float* const* rows, int nt, int K) {
    const int xs = mv_xstride(K), k4 = K / 4;
    for (int i = threadIdx.x; i < nt * k4; i += blockDim.x) {
        const int t = i / k4, c = (i - t * k4) * 4;
        const float4 v = reinterpret_cast<const float4*>(rows[t])[c / 4];
        float* dst = x_s + (size_t)(t * 8 + (c & 7)) * xs + (c >> 3);
        dst[0] = v.x;
        dst[xs] = v.y;
        dst[2 * xs] = v.z;
        dst[3 * xs] = v.w;
    }
}

// Lane j's chain of row n of W' ([N, K] chunked bf16) against nt staged rows.
template <int NT>
__device__ __forceinline__ void row_chains(const uint16_t* W, int N, int K, int n, int j, const float* x_s, int nt,
                                           float (&acc)[NT]) {
    const int nc = K / 64, xs = mv_xstride(K);
    const uint4* wp = reinterpret_cast<const uint4*>(W) + (size_t)n * 8 + j;
    const size_t cstride = (size_t)N * 8;
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t] = 0.0f;
    constexpr int P = 8;
    uint4 cur[P], nxt[P];
#pragma unroll
    for (int i = 0; i < P; i++) cur[i] = i < nc ? __ldg(wp + (size_t)i * cstride) : make_uint4(0, 0, 0, 0);
    for (int c0 = 0; c0 < nc; c0 += P) {
#pragma unroll
        for (int i = 0; i < P; i++)
            nxt[i] = c0 + P + i < nc ? __ldg(wp + (size_t)(c0 + P + i) * cstride) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < P; i++)
            if (c0 + i < nc)
#pragma unroll
                for (int t = 0; t < NT; t++)
                    if (t < nt) fma_chunk(cur[i], x_s + (size_t)(t * 8 + j) * xs + (c0 + i) * 8, acc[t], uint16_t());
#pragma unroll
        for (int i = 0; i < P; i++) cur[i] = nxt[i];
    }
#pragma unroll
    for (int t = 0; t < NT; t++) {  // the AVX tree: ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7))
        float a = acc[t];
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 2));
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
        acc[t] = a;
    }
}

__global__ void __launch_bounds__(kBfRows * 8) k_bf16_gateup(const uint8_t* __restrict__ store_l, size_t rec_bytes,
                                                             int d, int m, int k, const float* __restrict__ x,
                                                             jl_ws ws) {
    extern __shared__ __align__(16) float x_s[];  // [kBfTok][8][d/8 + 4]
    __shared__ const float* rows[kBfTok];
    griddep_wait();
    griddep_launch_dependents();
    const int u = blockIdx.y;
    if (u >= *ws.U) return;
    const int e = ws.sel[u], s0 = ws.uh[u], n = ws.uh[u + 1] - s0;
    const int tid = threadIdx.x, j = tid & 7, row = blockIdx.x * kBfRows + (tid >> 3);
    const uint16_t* Wg = reinterpret_cast<const uint16_t*>(store_l + (size_t)e * rec_bytes);
    const uint16_t* Wu = Wg + (size_t)m * d;
    for (int c0 = 0; c0 < n; c0 += kBfTok) {
        const int nt = min(kBfTok, n - c0);
        __syncthreads();
        if (tid < nt) rows[tid] = x + (size_t)(ws.uidx[s0 + c0 + tid] / k) * d;
        __syncthreads();
        stage_rows(x_s, rows, nt, d);
        __syncthreads();
        float g[kBfTok], up[kBfTok];
        row_chains<kBfTok>(Wg, m, d, min(row, m - 1), j, x_s, nt, g);
        row_chains<kBfTok>(Wu, m, d, min(row, m - 1), j, x_s, nt, up);
        if (j == 0 && row < m) {
#pragma unroll
            for (int t = 0; t < kBfTok; t++)
                if (t < nt) ws.act[(size_t)ws.uidx[s0 + c0 + t] * m + row] = silu_mul(g[t], up[t]);
        }
    }
}

__global__ void __launch_bounds__(kBfRows * 8) k_bf16_down(const uint8_t* __restrict__ store_l, size_t rec_bytes,
                                                           int d, int m, jl_ws ws) {
    extern __shared__ __align__(16) float a_s[];  // [kBfTok][8][m/8 + 4]
    __shared__ const float* rows[kBfTok];
    griddep_wait();
    griddep_launch_dependents();
    const int u = blockIdx.y;
    if (u >= *ws.U) return;
    const int e = ws.sel[u], s0 = ws.uh[u], n = ws.uh[u + 1] - s0;
    const int tid = threadIdx.x, j = tid & 7, row = blockIdx.x * kBfRows + (tid >> 3);
    const uint16_t* Wd = reinterpret_cast<const uint16_t*>(store_l + (size_t)e * rec_bytes) + (size_t)2 * m * d;
    for (int c0 = 0; c0 < n; c0 += kBfTok) {
        const int nt = min(kBfTok, n - c0);
        __syncthreads();
        if (tid < nt) rows[tid] = ws.act + (size_t)ws.uidx[s0 + c0 + tid] * m;
        __syncthreads();
        stage_rows(a_s, rows, nt, m);
        __syncthreads();
        float acc[kBfTok];
        row_chains<kBfTok>(Wd, d, m, min(row, d - 1), j, a_s, nt, acc);
        if (j == 0 && row < d) {
#pragma unroll
            for (int t = 0; t < kBfTok; t++)
                if (t < nt) {
                    const int pos = s0 + c0 + t;
                    ws.y[(size_t)ws.uidx[pos] * d + row] = __fadd_rn(0.0f, __fmul_rn(ws.uw[pos], acc[t]));
                }
        }
    }
}

}  // namespace jl

int jl_launch_bf16_ffn(const jl_moe* h, const uint8_t* store_l, const float* x, int B, cudaStream_t s) {
    using namespace jl;
    const int umax = std::min(h->E, B * h->k);
    const size_t sg = (size_t)kBfTok * 8 * mv_xstride(h->d) * 4, sd = (size_t)kBfTok * 8 * mv_xstride(h->m) * 4;
    if (sg > 200 * 1024 || sd > 200 * 1024) return JL_ERR_INVALID;
    int rc = jl_device_once(kOnceBf16, [] {
        JL_CUDA(cudaFuncSetAttribute(jl::k_bf16_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        JL_CUDA(cudaFuncSetAttribute(jl::k_bf16_down, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        return JL_OK;
    });
    if (rc) return rc;
    rc = launch(k_bf16_gateup, dim3((h->m + kBfRows - 1) / kBfRows, umax), dim3(kBfRows * 8), sg, s, store_l,
                h->lay.rec_bytes, h->d, h->m, h->k, x, h->ws);
    if (rc) return rc;
    return launch(k_bf16_down, dim3((h->d + kBfRows - 1) / kBfRows, umax), dim3(kBfRows * 8), sd, s, store_l,
                  h->lay.rec_bytes, h->d, h->m, h->ws);
}

int jl_repack_bf16_part(const uint16_t* src, int p, const jl_moe* h, uint8_t* rec, cudaStream_t s) {
    const int R = p < 2 ? h->m : h->d, C = p < 2 ? h->d : h->m;
    uint16_t* dst = reinterpret_cast<uint16_t*>(rec) + (size_t)p * h->m * h->d;
    const size_t total = (size_t)R * C;
    const int tpb = 256;
    const unsigned blocks = (unsigned)std::min<size_t>((total + tpb - 1) / tpb, 65535u * 16);
    jl::k_repack_mv<uint16_t><<<blocks, tpb, 0, s>>>(src, dst, R, C);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? JL_OK : jl_note_cuda(e);
}
