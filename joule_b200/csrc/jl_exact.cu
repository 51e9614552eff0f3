// Expert FFN on CUDA cores in the reference's FP32 arithmetic order
// (ffn_expert_worker Q4 branch, decode_kernel.c:1365-1384, with the row dot
// q4_row_dot_B, decode_kernel.c:770-858), so the layer output is
// bit-identical to the reference's for the same inputs.
//
// Work decomposition: the product p = hsum8(...) * scale of one (row, 64-value
// group) is independent of every other; only the per-row sum over groups is a
// sequential chain. A block takes one 32-row block of an expert's matrices;
// each warp stages its share of the tiles with 1-D bulk copies on its own
// mbarrier, every lane computes p for its row (lane = row) of each tile, and
// one warp per part then runs the per-row chains from shared memory. The
// products use Blackwell's packed FP32x2 FMA (__ffma2_rn), which rounds each
// lane exactly like the scalar FMA, so lane pairs of the reference's 8-wide
// accumulator advance in one instruction. Tokens routed to the expert are
// staged in shared memory and read as warp-uniform broadcasts.
#include <algorithm>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

constexpr int kGuWarpsPerPart = 8;  // gate/up block: warps 0-7 gate, 8-15 up
constexpr int kGuWarps = 2 * kGuWarpsPerPart;
constexpr int kGuTok = 2;           // tokens per pass (gate/up)
constexpr int kDnWarps = 4;
constexpr int kDnTok = 4;           // tokens per pass (down)

// p for NT tokens of one tile row: q0/q1 = the row's 32 bytes, xs = token
// rows (stride `xstride`) starting at this group's first column.
template <int NT>
__device__ __forceinline__ void tile_row_products(uint4 q0, uint4 q1, float s, const float* xs,
                                                  int xstride, float (&p)[NT]) {
    const uint32_t wq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    float2 lane[NT][4];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int j = 0; j < 4; j++) lane[t][j] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int w = 0; w < 8; w++) {
        float2 a[4];
        dequant8x2(wq[w], a);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float4 x0 = *reinterpret_cast<const float4*>(xs + t * xstride + w * 8);
            const float4 x1 = *reinterpret_cast<const float4*>(xs + t * xstride + w * 8 + 4);
            lane[t][0] = __ffma2_rn(a[0], make_float2(x0.x, x0.y), lane[t][0]);
            lane[t][1] = __ffma2_rn(a[1], make_float2(x0.z, x0.w), lane[t][1]);
            lane[t][2] = __ffma2_rn(a[2], make_float2(x1.x, x1.y), lane[t][2]);
            lane[t][3] = __ffma2_rn(a[3], make_float2(x1.z, x1.w), lane[t][3]);
        }
    }
#pragma unroll
    for (int t = 0; t < NT; t++) p[t] = __fmul_rn(hsum8x2(lane[t]), s);
}

// Products for tiles [g_lo, g_hi) of part `pi` (smem tile index pi*ng + g) for
// `nt` (<= NTMAX) tokens; p_s layout [(pi*NTMAX + t)*ng + g][32].
template <int NTMAX>
__device__ __forceinline__ bool warp_tiles(const uint8_t* w_s, const float* x_s, int xstride,
                                           float* p_s, int pi,
                                           int ng, int g_lo, int g_hi, int nt, uint64_t* bars,
                                           bool wait, int* err) {
    const int lane = threadIdx.x & 31;
    for (int g = g_lo; g < g_hi; g++) {
        // first pass: tile g may still be in flight; compute overlaps the rest
        if (wait && !mbar_wait_bounded(&bars[g - g_lo], 0, err)) return false;
        const uint8_t* tile = w_s + (size_t)(pi * ng + g) * kTileRec;
        const uint4 q0 = *reinterpret_cast<const uint4*>(tile + lane * 16);
        const uint4 q1 = *reinterpret_cast<const uint4*>(tile + 512 + lane * 16);
        const float s = half_bits_to_f32(reinterpret_cast<const uint16_t*>(tile + kTileBytes)[lane]);
        const float* xg = x_s + g * kGroup;
        float* pp = p_s + ((size_t)(pi * NTMAX) * ng + g) * 32 + lane;
        const size_t tstride = (size_t)ng * 32;
        if (nt == 1) {
            float p[1];
            tile_row_products<1>(q0, q1, s, xg, xstride, p);
            pp[0] = p[0];
        } else if (NTMAX >= 2 && nt == 2) {
            float p[2];
            tile_row_products<2>(q0, q1, s, xg, xstride, p);
            pp[0] = p[0];
            pp[tstride] = p[1];
        } else if (NTMAX >= 3 && nt == 3) {
            float p[3];
            tile_row_products<3>(q0, q1, s, xg, xstride, p);
#pragma unroll
            for (int t = 0; t < 3; t++) pp[t * tstride] = p[t];
        } else if (NTMAX >= 4) {
            float p[4];
            tile_row_products<4>(q0, q1, s, xg, xstride, p);
#pragma unroll
            for (int t = 0; t < 4; t++) pp[t * tstride] = p[t];
        }
    }
    return true;
}

constexpr int kMaxTilesPerWarp = 8;

// Issue this warp's bulk copies: tile record i (1088 B: packed + scales) on
// mbarrier bars[i], so the warp can start on tile 0 while later tiles are in
// flight. Tiles g in [g_lo, g_hi) of part p, row block rb.
__device__ __forceinline__ void warp_stage(uint8_t* w_dst, const uint8_t* rec, const jl_layout& L,
                                           int p, int rb, int g_lo, int g_hi, uint64_t* bars) {
    if ((threadIdx.x & 31) == 0) {
        const int ntiles = g_hi - g_lo;
        for (int i = 0; i < ntiles; i++) mbar_init(&bars[i], 1);
        mbar_fence_init();
        for (int i = 0; i < ntiles; i++) {
            mbar_expect_tx(&bars[i], kTileRec);
            bulk_g2s(w_dst + (size_t)i * kTileRec, rec + L.tile_off(p, rb, g_lo + i), kTileRec, &bars[i]);
        }
    }
    __syncwarp();
}

// Wait (bounded) for every tile copy of this warp: a block must not exit
// while its bulk copies are still landing in shared memory.
__device__ __forceinline__ void warp_drain(uint64_t* bars, int ntiles, int* err) {
    for (int i = 0; i < ntiles; i++) mbar_wait_bounded(&bars[i], 0, err);
}

// Sequential per-row sum over ng group products (lane = row).
__device__ __forceinline__ float row_chain(const float* pp, int ng) {
    float acc = 0.0f;
    int g = 0;
    for (; g + 4 <= ng; g += 4) {
        const float a = pp[(g + 0) * 32], b = pp[(g + 1) * 32];
        const float c = pp[(g + 2) * 32], d = pp[(g + 3) * 32];
        acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, a), b), c), d);
    }
    for (; g < ng; g++) acc = __fadd_rn(acc, pp[g * 32]);
    return acc;
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU. grid = (m/32 row blocks, max union size); block (rb, u)
// handles rows 32rb..32rb+31 of expert sel[u]'s gate (warps 0-7) and up
// (warps 8-15) for all of its tokens and writes act[slot][row] = silu(g) * u.
__global__ void __launch_bounds__(kGuWarps * 32) k_gateup_exact(
    const uint8_t* __restrict__ store_l, jl_layout L, int k, const float* __restrict__ x,
    jl_ws ws) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int d = L.d, m = L.m, ng = d / kGroup;
    const int rb = blockIdx.x, u = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* w_s = smem;                                                   // [2*ng] tile records
    float* x_s = reinterpret_cast<float*>(w_s + (size_t)2 * ng * kTileRec);  // [kGuTok, d]
    float* p_s = x_s + kGuTok * d;                                         // [2, kGuTok, ng, 32]
    float* gu_s = p_s + 2 * kGuTok * ng * 32;                              // [kGuTok, 32] up sums
    uint64_t* bars = reinterpret_cast<uint64_t*>(gu_s + kGuTok * 32) + warp * kMaxTilesPerWarp;
    long long* tr = (rb == 0 && u == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceGateup, 0);
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceGateup, 1);
    if (u >= *ws.U) return;
    const int e = ws.sel[u];
    const int s0 = ws.uh[u], n = ws.uh[u + 1] - s0;
    const uint8_t* rec = store_l + (size_t)e * L.rec_bytes;
    const int pi = warp / kGuWarpsPerPart, q = warp % kGuWarpsPerPart;
    const int g_lo = q * ng / kGuWarpsPerPart, g_hi = (q + 1) * ng / kGuWarpsPerPart;
    warp_stage(w_s + (size_t)(pi * ng + g_lo) * kTileRec, rec, L, pi, rb, g_lo, g_hi, bars);
    bool ok = true;
    for (int c0 = 0; c0 < n; c0 += kGuTok) {
        const int nt = min(kGuTok, n - c0);
        for (int i = threadIdx.x; i < nt * d / 4; i += blockDim.x) {
            const int t = i / (d / 4), c = i % (d / 4);
            const int b = ws.uidx[s0 + c0 + t] / k;
            reinterpret_cast<float4*>(x_s + t * d)[c] =
                reinterpret_cast<const float4*>(x + (size_t)b * d)[c];
        }
        __syncthreads();
        if (c0 == 0) trace_point(tr, kTraceGateup, 2);
        if (ok) ok = warp_tiles<kGuTok>(w_s, x_s, d, p_s, pi, ng, g_lo, g_hi, nt, bars, c0 == 0,
                                        ws.err);
        __syncthreads();
        if (c0 == 0) trace_point(tr, kTraceGateup, 3);
        if (warp == 1)  // up chains
            for (int t = 0; t < nt; t++)
                gu_s[t * 32 + lane] = row_chain(p_s + (size_t)((1 * kGuTok + t) * ng) * 32 + lane, ng);
        __syncthreads();
        if (warp == 0)  // gate chains + SwiGLU
            for (int t = 0; t < nt; t++) {
                const float ga = row_chain(p_s + (size_t)((0 * kGuTok + t) * ng) * 32 + lane, ng);
                const int slot = ws.uidx[s0 + c0 + t];
                ws.act[(size_t)slot * m + rb * kTileRows + lane] = silu_mul(ga, gu_s[t * 32 + lane]);
            }
        __syncthreads();
    }
    trace_point(tr, kTraceGateup, 4);
    if (n == 0 || !ok) warp_drain(bars, g_hi - g_lo, ws.err);  // never leave copies in flight
}

// ---------------------------------------------------------------------------
// down. grid = (d/32 row blocks, max union size); block (rb, u) handles rows
// 32rb..32rb+31 of expert sel[u]'s down matrix for all of its tokens and
// writes y[slot][row] = 0 + w * dacc (the reference's `ye += uw * dacc`
// onto a zeroed ye).
__global__ void __launch_bounds__(kDnWarps * 32) k_down_exact(const uint8_t* __restrict__ store_l,
                                                              jl_layout L, jl_ws ws) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int d = L.d, m = L.m, ng = m / kGroup;
    const int rb = blockIdx.x, u = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* w_s = smem;                                                // [ng] tile records
    float* a_s = reinterpret_cast<float*>(w_s + (size_t)ng * kTileRec);  // [kDnTok, m]
    float* p_s = a_s + kDnTok * m;                                 // [kDnTok, ng, 32]
    uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + kDnTok * ng * 32) + warp * kMaxTilesPerWarp;
    // The routing (U, sel, uh) was written by the router, which completed
    // before the gate/up kernel's blocks passed their wait and released this
    // grid; only act (gate/up's output) needs griddep_wait. So this block's
    // down weights are fetched while gate/up is still running.
    long long* tr = (rb == 0 && u == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceDown, 0);
    const int U = *ws.U;
    if (u >= U) return;
    const int e = ws.sel[u];
    const int s0 = ws.uh[u], n = ws.uh[u + 1] - s0;
    const uint8_t* rec = store_l + (size_t)e * L.rec_bytes;
    const int g_lo = warp * ng / kDnWarps, g_hi = (warp + 1) * ng / kDnWarps;
    warp_stage(w_s + (size_t)g_lo * kTileRec, rec, L, 2, rb, g_lo, g_hi, bars);
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceDown, 1);
    bool ok = true;
    for (int c0 = 0; c0 < n; c0 += kDnTok) {
        const int nt = min(kDnTok, n - c0);
        for (int i = threadIdx.x; i < nt * m / 4; i += blockDim.x) {
            const int t = i / (m / 4), c = i % (m / 4);
            const int slot = ws.uidx[s0 + c0 + t];
            reinterpret_cast<float4*>(a_s + t * m)[c] =
                reinterpret_cast<const float4*>(ws.act + (size_t)slot * m)[c];
        }
        __syncthreads();
        if (c0 == 0) trace_point(tr, kTraceDown, 2);
        if (ok) ok = warp_tiles<kDnTok>(w_s, a_s, m, p_s, 0, ng, g_lo, g_hi, nt, bars, c0 == 0,
                                        ws.err);
        __syncthreads();
        if (warp < nt) {  // one warp per token
            const int t = warp;
            const float acc = row_chain(p_s + (size_t)(t * ng) * 32 + lane, ng);
            const int pos = s0 + c0 + t;
            const int slot = ws.uidx[pos];
            ws.y[(size_t)slot * d + rb * kTileRows + lane] =
                __fadd_rn(0.0f, __fmul_rn(ws.uw[pos], acc));
        }
        __syncthreads();
    }
    trace_point(tr, kTraceDown, 3);
    if (n == 0 || !ok) warp_drain(bars, g_hi - g_lo, ws.err);
}

// ---------------------------------------------------------------------------
// Combine (decode_kernel.c:1490-1507): out[b] = 0 + y of b's experts in union
// order (experts b did not choose contribute +0 in the reference, which
// leaves every nonzero partial sum unchanged). Also copies top/tw out.
__global__ void k_combine(int B, int k, int d, jl_ws ws, float* __restrict__ out,
                          int* __restrict__ top, float* __restrict__ tw) {
    long long* tr = (blockIdx.x == 0 && blockIdx.y == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceCombine, 0);
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceCombine, 1);
    const int b = blockIdx.y;
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (c < d) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < k; j++) {
            const int slot = ws.comb[b * k + j];
            const float4 v = *reinterpret_cast<const float4*>(ws.y + (size_t)slot * d + c);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        *reinterpret_cast<float4*>(out + (size_t)b * d + c) = acc;
    }
    if (blockIdx.x == 0 && threadIdx.x < k) {
        if (top) top[b * k + threadIdx.x] = ws.top[b * k + threadIdx.x];
        if (tw) tw[b * k + threadIdx.x] = ws.tw[b * k + threadIdx.x];
    }
    __syncthreads();
    trace_point(tr, kTraceCombine, 2);
}

size_t gateup_smem(int d) {
    const int ng = d / kGroup;
    return (size_t)2 * ng * kTileRec + (size_t)kGuTok * d * 4 +
           (size_t)2 * kGuTok * ng * 32 * 4 + (size_t)kGuTok * 32 * 4 +
           (size_t)kGuWarps * kMaxTilesPerWarp * 8;
}
size_t down_smem(int m) {
    const int ng = m / kGroup;
    return (size_t)ng * kTileRec + (size_t)kDnTok * m * 4 +
           (size_t)kDnTok * ng * 32 * 4 + (size_t)kDnWarps * kMaxTilesPerWarp * 8;
}

}  // namespace jl

static int exact_attrs() {
    using namespace jl;
    static bool attr = false;
    if (!attr) {
        JL_CUDA(cudaFuncSetAttribute(k_gateup_exact, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        JL_CUDA(cudaFuncSetAttribute(k_down_exact, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        attr = true;
    }
    return JL_OK;
}

int jl_launch_gateup_exact(const jl_moe* h, const uint8_t* store_l, const float* x, int B,
                           cudaStream_t s) {
    using namespace jl;
    const int umax = std::min(h->E, B * h->k);
    const size_t gsm = gateup_smem(h->d);
    if (gsm > 220 * 1024) return JL_ERR_INVALID;
    if ((h->d / kGroup + kGuWarpsPerPart - 1) / kGuWarpsPerPart > kMaxTilesPerWarp) return JL_ERR_INVALID;
    int rc = exact_attrs();
    if (rc) return rc;
    return launch(k_gateup_exact, dim3(h->m / kTileRows, umax), dim3(kGuWarps * 32), gsm, s,
                  store_l, h->lay, h->k, x, h->ws);
}

int jl_launch_down_exact(const jl_moe* h, const uint8_t* store_l, int B, cudaStream_t s) {
    using namespace jl;
    const int umax = std::min(h->E, B * h->k);
    const size_t dsm = down_smem(h->m);
    if (dsm > 220 * 1024) return JL_ERR_INVALID;
    if ((h->m / kGroup + kDnWarps - 1) / kDnWarps > kMaxTilesPerWarp) return JL_ERR_INVALID;
    int rc = exact_attrs();
    if (rc) return rc;
    return launch(k_down_exact, dim3(h->d / kTileRows, umax), dim3(kDnWarps * 32), dsm, s, store_l,
                  h->lay, h->ws);
}

int jl_launch_combine(const jl_moe* h, int B, float* out, int* top, float* tw, cudaStream_t s) {
    using namespace jl;
    const int tpb = 128;
    dim3 grid((h->d / 4 + tpb - 1) / tpb, B);
    return launch(k_combine, grid, dim3(tpb), 0, s, B, h->k, h->d, h->ws, out, top, tw);
}
