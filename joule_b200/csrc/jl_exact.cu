// Expert FFN on CUDA cores in the reference's FP32 arithmetic order
// (ffn_expert_worker Q4 branch, decode_kernel.c:1365-1384, with the row dot
// q4_row_dot_B, decode_kernel.c:770-858), so the layer output is
// bit-identical to the reference's for the same inputs.
//
// Work decomposition: the product p = hsum8(...) * scale of one (row, 64-value
// group) is independent of every other; only the per-row sum over groups is a
// sequential chain. A block takes one row block of one expert (gate/up: 64
// gate + 64 up rows; down: 128 rows), whose tile records are one contiguous
// region of the store, and stages it with a few large 1-D bulk copies issued
// by different lanes (a bulk copy costs its issuing thread a few hundred
// nanoseconds whatever its size, so small per-tile copies cannot keep an SM's
// share of HBM busy). Every lane computes p for its row (lane = row) of each
// tile of its warp, and one warp per (row block, token) then runs the per-row
// chain from shared memory. The products use Blackwell's packed FP32x2 FMA
// (__ffma2_rn), which rounds each lane exactly like the scalar FMA, so lane
// pairs of the reference's 8-wide accumulator advance in one instruction.
// Tokens routed to the expert are staged in shared memory and read as
// warp-uniform broadcasts.
#include <algorithm>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

constexpr int kXWarps = 16;   // 4 row blocks of 32 rows x 4 group ranges
constexpr int kXRB = 4;       // row blocks per block (gate/up: gate 0, gate 1, up 0, up 1)
constexpr int kXChunks = 8;   // bulk copies per block (up to)
constexpr int kGuTok = 2;     // tokens per pass (gate/up)
constexpr int kDnTok = 4;     // tokens per pass (down)

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

// Products of this warp's tiles: row block j (32 rows) for groups [g_lo,
// g_hi) of the staged region, whose group g holds kXRB consecutive tile
// records (record j at g * kXRB + j). nt <= NTMAX tokens; p_s layout
// [(j * NTMAX + t) * ng + g][32]. On the first pass the warp waits for the
// chunk holding each group (chunk = g / gpc, barrier bars[chunk]).
template <int NTMAX>
__device__ __forceinline__ bool warp_tiles(const uint8_t* w_s, const float* x_s, int xstride,
                                           float* p_s, int j, int ng, int g_lo, int g_hi, int nt,
                                           uint64_t* bars, int gpc, bool wait, int* err) {
    const int lane = threadIdx.x & 31;
    for (int g = g_lo; g < g_hi; g++) {
        // first pass: later chunks may still be in flight; compute overlaps them
        if (wait && (g == g_lo || g % gpc == 0) && !mbar_wait_bounded(&bars[g / gpc], 0, err))
            return false;
        const uint8_t* tile = w_s + ((size_t)g * kXRB + j) * kTileRec;
        const uint4 q0 = *reinterpret_cast<const uint4*>(tile + lane * 16);
        const uint4 q1 = *reinterpret_cast<const uint4*>(tile + 512 + lane * 16);
        const float s = half_bits_to_f32(reinterpret_cast<const uint16_t*>(tile + kTileBytes)[lane]);
        const float* xg = x_s + g * kGroup;
        float* pp = p_s + ((size_t)(j * NTMAX) * ng + g) * 32 + lane;
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

// Stage the block's contiguous region (ng groups of kXRB tile records) with
// nchunks bulk copies of gpc groups each, issued by lanes 0..nchunks-1 of
// warp 0 in parallel, chunk c completing on bars[c].
__device__ __forceinline__ void stage_region(uint8_t* w_s, const uint8_t* src, int ng, int gpc,
                                             int nchunks, uint64_t* bars) {
    const int tid = threadIdx.x;
    if (tid < 32) {
        if (tid < nchunks) {
            const int g0 = tid * gpc, gn = min(gpc, ng - g0);
            const uint32_t bytes = (uint32_t)gn * kXRB * kTileRec;
            mbar_init(&bars[tid], 1);
            mbar_fence_init();
            mbar_expect_tx(&bars[tid], bytes);
            bulk_g2s_hint(w_s + (size_t)g0 * kXRB * kTileRec, src + (size_t)g0 * kXRB * kTileRec, bytes,
                          &bars[tid], l2_policy_evict_first());
        }
    }
}

// Wait (bounded) for every chunk: a block must not exit while its bulk
// copies are still landing in shared memory.
__device__ __forceinline__ void region_drain(uint64_t* bars, int nchunks, int* err) {
    if (threadIdx.x < nchunks) mbar_wait_bounded(&bars[threadIdx.x], 0, err);
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

// groups per bulk copy: at least 4 (a 17 KB copy), at most kXChunks copies
__host__ __device__ inline int region_gpc(int ng) { return max(4, (ng + kXChunks - 1) / kXChunks); }

// ---------------------------------------------------------------------------
// gate/up + SwiGLU. grid = (m/64 row blocks, max union size); block (mt, u)
// handles gate rows and up rows 64mt..64mt+63 of expert sel[u] (row blocks j
// = gate 0, gate 1, up 0, up 1; warp = j * 4 + group range) for all of its
// tokens and writes act[slot][row] = silu(g) * u.
__global__ void __launch_bounds__(kXWarps * 32) k_gateup_exact(
    const uint8_t* __restrict__ store_l, jl_layout L, int k, const float* __restrict__ x,
    jl_ws ws) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[kXChunks];
    const int d = L.d, m = L.m, ng = d / kGroup, gpc = region_gpc(ng);
    const int nchunks = (ng + gpc - 1) / gpc;
    const int mt = blockIdx.x, u = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* w_s = smem;                                                          // [ng][4] records
    float* x_s = reinterpret_cast<float*>(w_s + (size_t)ng * kXRB * kTileRec);   // [kGuTok, d]
    float* p_s = x_s + kGuTok * d;                                                // [4, kGuTok, ng, 32]
    float* gu_s = p_s + kXRB * kGuTok * ng * 32;                                  // [2, kGuTok, 32] up sums
    long long* tr = (mt == 0 && u == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceGateup, 0);
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceGateup, 1);
    if (u >= *ws.U) return;
    const int e = ws.sel[u];
    const int s0 = ws.uh[u], n = ws.uh[u + 1] - s0;
    const uint8_t* rec = store_l + (size_t)e * L.rec_bytes;
    stage_region(w_s, rec + L.tile_off(0, 2 * mt, 0), ng, gpc, nchunks, bars);
    const int j = warp >> 2, q = warp & 3;
    const int g_lo = q * ng / 4, g_hi = (q + 1) * ng / 4;
    bool ok = true;
    for (int c0 = 0; c0 < n; c0 += kGuTok) {
        const int nt = min(kGuTok, n - c0);
        for (int i = threadIdx.x; i < nt * d / 4; i += blockDim.x) {
            const int t = i / (d / 4), c = i % (d / 4);
            const int b = ws.uidx[s0 + c0 + t] / k;
            reinterpret_cast<float4*>(x_s + t * d)[c] =
                reinterpret_cast<const float4*>(x + (size_t)b * d)[c];
        }
        __syncthreads();  // also publishes the barrier initialisation of stage_region
        if (c0 == 0) trace_point(tr, kTraceGateup, 2);
        if (ok) ok = warp_tiles<kGuTok>(w_s, x_s, d, p_s, j, ng, g_lo, g_hi, nt, bars, gpc, c0 == 0,
                                        ws.err);
        __syncthreads();
        if (c0 == 0) trace_point(tr, kTraceGateup, 3);
        // chains: warp (jj, t) for row block jj in {up 0, up 1} first, then gate
        const int jj = warp >> 1, t = warp & 1;
        if (warp < 4 && t < nt)  // up chains (row blocks 2, 3)
            gu_s[((jj) * kGuTok + t) * 32 + lane] =
                row_chain(p_s + (size_t)(((2 + jj) * kGuTok + t) * ng) * 32 + lane, ng);
        __syncthreads();
        if (warp >= 4 && warp < 8) {  // gate chains (row blocks 0, 1) + SwiGLU
            const int gj = (warp - 4) >> 1, gt = warp & 1;
            if (gt < nt) {
                const float ga = row_chain(p_s + (size_t)((gj * kGuTok + gt) * ng) * 32 + lane, ng);
                const int slot = ws.uidx[s0 + c0 + gt];
                ws.act[(size_t)slot * m + mt * 64 + gj * 32 + lane] =
                    silu_mul(ga, gu_s[(gj * kGuTok + gt) * 32 + lane]);
            }
        }
        __syncthreads();
    }
    trace_point(tr, kTraceGateup, 4);
    if (n == 0 || !ok) region_drain(bars, nchunks, ws.err);  // never leave copies in flight
}

// ---------------------------------------------------------------------------
// down. grid = (d/128 row blocks, max union size); block (mt, u) handles rows
// 128mt..128mt+127 of expert sel[u]'s down matrix (row blocks j = 0..3; warp
// = j * 4 + group range) for all of its tokens and writes y[slot][row] = 0 +
// w * dacc (the reference's `ye += uw * dacc` onto a zeroed ye).
__global__ void __launch_bounds__(kXWarps * 32) k_down_exact(const uint8_t* __restrict__ store_l,
                                                             jl_layout L, jl_ws ws) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[kXChunks];
    const int d = L.d, m = L.m, ng = m / kGroup, gpc = region_gpc(ng);
    const int nchunks = (ng + gpc - 1) / gpc;
    const int mt = blockIdx.x, u = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* w_s = smem;                                                          // [ng][4] records
    float* a_s = reinterpret_cast<float*>(w_s + (size_t)ng * kXRB * kTileRec);   // [kDnTok, m]
    float* p_s = a_s + kDnTok * m;                                                // [4, kDnTok, ng, 32]
    // The routing (U, sel, uh) was written by the router, which completed
    // before the gate/up kernel's blocks passed their wait and released this
    // grid; only act (gate/up's output) needs griddep_wait. So this block's
    // down weights are fetched while gate/up is still running.
    long long* tr = (mt == 0 && u == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceDown, 0);
    const int U = *ws.U;
    if (u >= U) return;
    const int e = ws.sel[u];
    const int s0 = ws.uh[u], n = ws.uh[u + 1] - s0;
    const uint8_t* rec = store_l + (size_t)e * L.rec_bytes;
    stage_region(w_s, rec + L.tile_off(2, 4 * mt, 0), ng, gpc, nchunks, bars);
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceDown, 1);
    const int j = warp >> 2, q = warp & 3;
    const int g_lo = q * ng / 4, g_hi = (q + 1) * ng / 4;
    bool ok = true;
    for (int c0 = 0; c0 < n; c0 += kDnTok) {
        const int nt = min(kDnTok, n - c0);
        for (int i = threadIdx.x; i < nt * m / 4; i += blockDim.x) {
            const int t = i / (m / 4), c = i % (m / 4);
            const int slot = ws.uidx[s0 + c0 + t];
            reinterpret_cast<float4*>(a_s + t * m)[c] =
                reinterpret_cast<const float4*>(ws.act + (size_t)slot * m)[c];
        }
        __syncthreads();  // also publishes the barrier initialisation of stage_region
        if (c0 == 0) trace_point(tr, kTraceDown, 2);
        if (ok) ok = warp_tiles<kDnTok>(w_s, a_s, m, p_s, j, ng, g_lo, g_hi, nt, bars, gpc, c0 == 0,
                                        ws.err);
        __syncthreads();
        {  // warp (row block jj, token t)
            const int jj = warp >> 2, t = warp & 3;
            if (t < nt) {
                const float acc = row_chain(p_s + (size_t)((jj * kDnTok + t) * ng) * 32 + lane, ng);
                const int pos = s0 + c0 + t;
                const int slot = ws.uidx[pos];
                ws.y[(size_t)slot * d + mt * 128 + jj * 32 + lane] =
                    __fadd_rn(0.0f, __fmul_rn(ws.uw[pos], acc));
            }
        }
        __syncthreads();
    }
    trace_point(tr, kTraceDown, 3);
    if (n == 0 || !ok) region_drain(bars, nchunks, ws.err);
}

// ---------------------------------------------------------------------------
// Combine (decode_kernel.c:1490-1507): out[b] = 0 + y of b's experts in union
// order (experts b did not choose contribute +0 in the reference, which
// leaves every nonzero partial sum unchanged). Also copies top/tw out.
// With tokorder = 1 a token adds its slots in its own top-k order (b*k + j),
// the union order it has when it is routed alone (B = 1): a batch of
// positions of one sequence then gives each position the bits of a one-token
// call (prefill_layers, decode_kernel.c:1606-1615, runs one position per call).
__global__ void k_combine(int B, int k, int d, jl_ws ws, float* __restrict__ out,
                          int* __restrict__ top, float* __restrict__ tw, int tokorder) {
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
            const int slot = tokorder ? b * k + j : ws.comb[b * k + j];
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
    return (size_t)ng * kXRB * kTileRec + (size_t)kGuTok * d * 4 + (size_t)kXRB * kGuTok * ng * 32 * 4 +
           (size_t)2 * kGuTok * 32 * 4;
}
size_t down_smem(int m) {
    const int ng = m / kGroup;
    return (size_t)ng * kXRB * kTileRec + (size_t)kDnTok * m * 4 + (size_t)kXRB * kDnTok * ng * 32 * 4;
}

}  // namespace jl

static int exact_attrs() {
    return jl_device_once(kOnceExact, [] {
        JL_CUDA(cudaFuncSetAttribute(jl::k_gateup_exact, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        JL_CUDA(cudaFuncSetAttribute(jl::k_down_exact, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        return JL_OK;
    });
}

int jl_launch_gateup_exact(const jl_moe* h, const uint8_t* store_l, const float* x, int B,
                           cudaStream_t s) {
    using namespace jl;
    const int umax = std::min(h->E, B * h->k);
    const size_t gsm = gateup_smem(h->d);
    if (gsm > 220 * 1024 || h->m % 64) return JL_ERR_INVALID;
    int rc = exact_attrs();
    if (rc) return rc;
    return launch(k_gateup_exact, dim3(h->m / 64, umax), dim3(kXWarps * 32), gsm, s, store_l, h->lay,
                  h->k, x, h->ws);
}

int jl_launch_down_exact(const jl_moe* h, const uint8_t* store_l, int B, cudaStream_t s) {
    using namespace jl;
    const int umax = std::min(h->E, B * h->k);
    const size_t dsm = down_smem(h->m);
    if (dsm > 220 * 1024 || h->d % 128) return JL_ERR_INVALID;
    int rc = exact_attrs();
    if (rc) return rc;
    return launch(k_down_exact, dim3(h->d / 128, umax), dim3(kXWarps * 32), dsm, s, store_l, h->lay,
                  h->ws);
}

int jl_launch_combine(const jl_moe* h, int B, float* out, int* top, float* tw, cudaStream_t s) {
    using namespace jl;
    const int tpb = 128;
    dim3 grid((h->d / 4 + tpb - 1) / tpb, B);
    return launch(k_combine, grid, dim3(tpb), 0, s, B, h->k, h->d, h->ws, out, top, tw, h->comb_token_order);
}
