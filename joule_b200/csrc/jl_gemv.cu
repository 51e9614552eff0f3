// Small-batch expert FFN (B <= 4) as warp-per-row GEMVs over every SM,
// judged by HBM bandwidth. Same math as the reference's expert worker
// (decode_kernel.c:1251-1275, 1365-1384: gate and up rows of each union
// expert against its tokens, SwiGLU, down rows, weighted per-slot outputs),
// summed in another order in FP32: results agree with the reference within
// the 1e-3 row-relative bar; routing stays bit-exact (the router is shared
// with the other paths).
//
// gate/up: a unit is 32 gate rows and the matching 32 up rows of one union
// expert over all d columns (the 64-value groups g of tile records
// (gate, rb, g) and (up, rb, g): 2 x 32 x 1088 bytes). One block per unit
// (persistent over units); its 8 warps take the groups g = w, w + 8, ...,
// lane t owning row t: every record of the warp is requested with 128-bit
// loads before any arithmetic, dequantised in registers and dotted with the
// token rows held in shared memory. The 8 warps' partial sums are added in
// warp order through shared memory, SwiGLU applied, and act written: no
// cross-block reduction, no atomics, deterministic.
//
// down: a unit is 32 rows of the down matrix of one union expert over all m
// columns (12 tile records at m = 768): one warp per unit, all records
// requested before the dependent-grid wait (the routing is known by then;
// only act is the previous kernel's output), act staged in shared memory,
// y[slot][row] = 0 + w * (row . act) written per slot. The existing combine
// adds the slots in the reference's union order.
#include <algorithm>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

constexpr int kGvWarps = 8;    // warps per block
constexpr int kGvMaxTok = 4;   // B <= 4
constexpr int kMaxUnion = 256;
constexpr int kGuBatch = 4;  // gate/up: groups (x 2 records) one warp holds in registers at a time
constexpr int kDnBatch = 6;  // down: records one warp holds in registers at a time

struct rec1 {
    uint4 a, b;      // bytes 0-15 and 16-31 of this lane's row group
    uint32_t s;      // its fp16 scale
};

__device__ __forceinline__ void load_rec(const uint8_t* rec, int lane, rec1& r) {
    r.a = __ldg(reinterpret_cast<const uint4*>(rec + lane * 16));
    r.b = __ldg(reinterpret_cast<const uint4*>(rec + 512 + lane * 16));
    r.s = __ldg(reinterpret_cast<const uint16_t*>(rec + kTileBytes) + lane);
}

// (row . x[0..64)) for one record row and NT tokens at base + xo[t]
// (shared memory), fp32, pairs of lanes of the 8-value words in FFMA2.
template <int NT>
__device__ __forceinline__ void rec_dot(const rec1& r, const float* base, const int (&xo)[NT], int nt,
                                        float (&dot)[NT]) {
    float2 part[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) part[t] = make_float2(0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const uint4& q = w < 4 ? r.a : r.b;
        const uint32_t word = (w & 3) == 0 ? q.x : (w & 3) == 1 ? q.y : (w & 3) == 2 ? q.z : q.w;
        float2 a[4];
        dequant8x2(word, a);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            if (t < nt) {
                const float4 x0 = *reinterpret_cast<const float4*>(base + xo[t] + 8 * w);
                const float4 x1 = *reinterpret_cast<const float4*>(base + xo[t] + 8 * w + 4);
                part[t] = __ffma2_rn(a[0], make_float2(x0.x, x0.y), part[t]);
                part[t] = __ffma2_rn(a[1], make_float2(x0.z, x0.w), part[t]);
                part[t] = __ffma2_rn(a[2], make_float2(x1.x, x1.y), part[t]);
                part[t] = __ffma2_rn(a[3], make_float2(x1.z, x1.w), part[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NT; t++) dot[t] = __fadd_rn(part[t].x, part[t].y);
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU. Block = one unit (32 gate + 32 up rows of one union
// expert); warp w holds groups g = w + 8 i in batches of kGuBatch.
template <int NT>
__global__ void __launch_bounds__(kGvWarps * 32, 2) k_gateup_gemv(const uint8_t* __restrict__ store_l,
                                                                  jl_layout L, int k,
                                                                  const float* __restrict__ x, int B, jl_ws ws) {
    extern __shared__ __align__(16) float x_s[];  // [B][d]
    __shared__ float red[kGvWarps][2][NT][32];
    __shared__ int sel_s[kMaxUnion], uh_s[kMaxUnion + 1], tok_s[kGvMaxTok * 16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = L.d, m = L.m, ngd = L.ngd, RB = m / 32;
    long long* tr = blockIdx.x == 0 ? ws.trace : nullptr;
    trace_point(tr, kTraceGateup, 0);
    // x is the router's input: complete before the router released this grid
    for (int i = threadIdx.x; i < B * d / 4; i += blockDim.x)
        reinterpret_cast<float4*>(x_s)[i] = reinterpret_cast<const float4*>(x)[i];
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceGateup, 1);
    const int U = *ws.U;
    for (int i = threadIdx.x; i < U; i += blockDim.x) sel_s[i] = ws.sel[i];
    for (int i = threadIdx.x; i <= U; i += blockDim.x) uh_s[i] = ws.uh[i];
    for (int i = threadIdx.x; i < B * k; i += blockDim.x) tok_s[i] = ws.uidx[i];
    __syncthreads();
    trace_point(tr, kTraceGateup, 2);
    const size_t rec_bytes = L.rec_bytes;
    const int units = U * RB;
    for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
        const int u = unit / RB, rb = unit - u * RB;
        const uint8_t* base = store_l + (size_t)sel_s[u] * rec_bytes;
        const int s0 = uh_s[u], nt = min(NT, uh_s[u + 1] - s0);
        int xo[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) xo[t] = (t < nt ? tok_s[s0 + t] / k : 0) * d;
        float ag[NT], au[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) ag[t] = au[t] = 0.0f;
        for (int g0 = warp; g0 < ngd; g0 += kGvWarps * kGuBatch) {
            rec1 gr[kGuBatch], ur[kGuBatch];  // every record of the batch requested before any arithmetic
#pragma unroll
            for (int i = 0; i < kGuBatch; i++) {
                const int g = g0 + kGvWarps * i;
                if (g < ngd) {
                    const size_t t0 = ((size_t)((rb >> 1) * ngd + g) * 4 + (rb & 1)) * kTileRec;  // gate rb, group g
                    load_rec(base + t0, lane, gr[i]);
                    load_rec(base + t0 + 2 * kTileRec, lane, ur[i]);  // up rb, group g
                }
            }
#pragma unroll
            for (int i = 0; i < kGuBatch; i++) {
                const int g = g0 + kGvWarps * i;
                if (g < ngd) {
                    float dg[NT], du[NT];
                    rec_dot<NT>(gr[i], x_s + g * 64, xo, nt, dg);
                    rec_dot<NT>(ur[i], x_s + g * 64, xo, nt, du);
                    const float sg = half_bits_to_f32((uint16_t)gr[i].s), su = half_bits_to_f32((uint16_t)ur[i].s);
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        ag[t] = __fmaf_rn(dg[t], sg, ag[t]);
                        au[t] = __fmaf_rn(du[t], su, au[t]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            red[warp][0][t][lane] = ag[t];
            red[warp][1][t][lane] = au[t];
        }
        __syncthreads();
        if (warp < nt) {  // warp t finishes token t: partial sums in warp order, SwiGLU
            float g = 0.0f, up = 0.0f;
#pragma unroll
            for (int w = 0; w < kGvWarps; w++) {
                g = __fadd_rn(g, red[w][0][warp][lane]);
                up = __fadd_rn(up, red[w][1][warp][lane]);
            }
            ws.act[(size_t)tok_s[s0 + warp] * m + rb * 32 + lane] = silu_mul(g, up);
        }
        __syncthreads();
    }
    trace_point(tr, kTraceGateup, 3);
}

// ---------------------------------------------------------------------------
// down. Block = one unit (128 rows of one union expert's down matrix: the
// four 32-row records of each group); warp w takes record rb4 = w % 4 of the
// groups g = w / 4 + 2 i, in batches of kDnBatch (the first batch requested
// before the dependent-grid wait: the routing is known by then, only act is
// gate/up's output). The two warps of a record add their sums in order.
template <int NT>
__global__ void __launch_bounds__(kGvWarps * 32, 2) k_down_gemv(const uint8_t* __restrict__ store_l, jl_layout L,
                                                                int B, int k, jl_ws ws) {
    extern __shared__ __align__(16) float a_s[];  // [B*k slots][m] act
    __shared__ float red[2][4][NT][32];
    __shared__ int sel_s[kMaxUnion], uh_s[kMaxUnion + 1], slot_s[kGvMaxTok * 16];
    __shared__ float w_s[kGvMaxTok * 16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rb4 = warp & 3, half = warp >> 2;
    const int d = L.d, m = L.m, ngm = L.ngm, MT = d / 128;
    long long* tr = blockIdx.x == 0 ? ws.trace : nullptr;
    trace_point(tr, kTraceDown, 0);
    const int U = *ws.U;
    const int units = U * MT;
    const size_t rec_bytes = L.rec_bytes, dn_off = L.dn_off;
    const int* sel_g = ws.sel;
    rec1 r[kDnBatch];
    auto rec_at = [=](int e, int mt, int g) {
        return store_l + (size_t)e * rec_bytes + dn_off + ((size_t)(mt * ngm + g) * 4 + rb4) * kTileRec;
    };
    if ((int)blockIdx.x < units) {  // this block's first unit, first batch
        const int u = blockIdx.x / MT, mt = blockIdx.x - u * MT, e = sel_g[u];
#pragma unroll
        for (int i = 0; i < kDnBatch; i++) {
            const int g = half + 2 * i;
            if (g < ngm) load_rec(rec_at(e, mt, g), lane, r[i]);
        }
    }
    for (int i = threadIdx.x; i < U; i += blockDim.x) sel_s[i] = ws.sel[i];
    for (int i = threadIdx.x; i <= U; i += blockDim.x) uh_s[i] = ws.uh[i];
    const int S = B * k;
    for (int i = threadIdx.x; i < S; i += blockDim.x) {
        slot_s[i] = ws.uidx[i];
        w_s[i] = ws.uw[i];
    }
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceDown, 1);
    for (int i = threadIdx.x; i < S * m / 4; i += blockDim.x)  // act of every slot (gate/up's output)
        reinterpret_cast<float4*>(a_s)[i] = reinterpret_cast<const float4*>(ws.act)[i];
    __syncthreads();
    bool first = true;
    for (int unit = blockIdx.x; unit < units; unit += gridDim.x) {
        const int u = unit / MT, mt = unit - u * MT, e = sel_s[u];
        const int s0 = uh_s[u], nt = min(NT, uh_s[u + 1] - s0);
        int ao[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) ao[t] = (t < nt ? slot_s[s0 + t] : 0) * m;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.0f;
        for (int g0 = half; g0 < ngm; g0 += 2 * kDnBatch) {
            if (!first) {
#pragma unroll
                for (int i = 0; i < kDnBatch; i++) {
                    const int g = g0 + 2 * i;
                    if (g < ngm) load_rec(rec_at(e, mt, g), lane, r[i]);
                }
            }
            first = false;
#pragma unroll
            for (int i = 0; i < kDnBatch; i++) {
                const int g = g0 + 2 * i;
                if (g < ngm) {
                    float dt[NT];
                    rec_dot<NT>(r[i], a_s + g * 64, ao, nt, dt);
                    const float sc = half_bits_to_f32((uint16_t)r[i].s);
#pragma unroll
                    for (int t = 0; t < NT; t++) acc[t] = __fmaf_rn(dt[t], sc, acc[t]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) red[half][rb4][t][lane] = acc[t];
        __syncthreads();
        if (half == 0) {
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < nt) {
                    const float v = __fadd_rn(red[0][rb4][t][lane], red[1][rb4][t][lane]);
                    ws.y[(size_t)slot_s[s0 + t] * d + mt * 128 + rb4 * 32 + lane] =
                        __fadd_rn(0.0f, __fmul_rn(w_s[s0 + t], v));
                }
            }
        }
        __syncthreads();
    }
    trace_point(tr, kTraceDown, 3);
}

}  // namespace jl

bool jl_gemv_ok(const jl_moe* h, int B) {
    using namespace jl;
    return B >= 1 && B <= kGvMaxTok && h->d % 128 == 0 && h->m % 64 == 0 &&
           (size_t)B * h->k * h->m * sizeof(float) <= 96 * 1024 && B * h->k <= kGvMaxTok * 16 &&
           (size_t)B * h->d * sizeof(float) <= 96 * 1024;
}

static int gemv_attrs() {
    return jl_device_once(kOnceGemv, [] {
        using namespace jl;
        const int big = 100 * 1024;
        JL_CUDA(cudaFuncSetAttribute(k_gateup_gemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_gateup_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_gateup_gemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_down_gemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_down_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_down_gemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        return JL_OK;
    });
}

int jl_launch_gateup_gemv(const jl_moe* h, const uint8_t* store_l, const float* x, int B, cudaStream_t s) {
    using namespace jl;
    if (!jl_gemv_ok(h, B)) return JL_ERR_INVALID;
    int rc = gemv_attrs();
    if (rc) return rc;
    const size_t smem = (size_t)B * h->d * sizeof(float);
    // units: union experts x (m / 32); two blocks per SM, persistent beyond that
    const int units = std::min(h->E, B * h->k) * (h->m / 32);
    const dim3 grid(std::min(units, 2 * h->sm_count)), block(kGvWarps * 32);
    if (B == 1) return launch(k_gateup_gemv<1>, grid, block, smem, s, store_l, h->lay, h->k, x, B, h->ws);
    if (B == 2) return launch(k_gateup_gemv<2>, grid, block, smem, s, store_l, h->lay, h->k, x, B, h->ws);
    return launch(k_gateup_gemv<4>, grid, block, smem, s, store_l, h->lay, h->k, x, B, h->ws);
}

int jl_launch_down_gemv(const jl_moe* h, const uint8_t* store_l, int B, cudaStream_t s) {
    using namespace jl;
    if (!jl_gemv_ok(h, B)) return JL_ERR_INVALID;
    int rc = gemv_attrs();
    if (rc) return rc;
    const size_t smem = (size_t)B * h->k * h->m * sizeof(float);
    const int units = std::min(h->E, B * h->k) * (h->d / 128);
    const dim3 grid(std::min(units, 2 * h->sm_count)), block(kGvWarps * 32);
    if (B == 1) return launch(k_down_gemv<1>, grid, block, smem, s, store_l, h->lay, B, h->k, h->ws);
    if (B == 2) return launch(k_down_gemv<2>, grid, block, smem, s, store_l, h->lay, B, h->k, h->ws);
    return launch(k_down_gemv<4>, grid, block, smem, s, store_l, h->lay, B, h->k, h->ws);
}
