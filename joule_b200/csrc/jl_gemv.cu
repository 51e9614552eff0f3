// Small-batch expert FFN (B <= 4) as warp-per-row GEMVs balanced over every
// warp of the GPU, judged by HBM bandwidth. Same math as the reference's
// expert worker (decode_kernel.c:1251-1275, 1365-1384: gate and up rows of
// each union expert against its tokens, SwiGLU, down rows, weighted
// per-slot outputs), summed in another order in FP32: results agree with the
// reference within the 1e-3 row-relative bar, routing stays bit-exact (the
// router is shared with the other paths).
//
// Work decomposition ("stream-K"). A K-step is one 64-value group of one
// 64-row M-tile of an expert's gate and up matrices: four tile records
// (gate rows 0-31, 32-63, up rows 0-31, 32-63; 4352 contiguous bytes). The
// layer's Q = U * (m/64) * (d/64) K-steps, ordered (expert, M-tile, group),
// are cut into equal contiguous ranges, one per warp of the grid, so every
// warp streams the same number of bytes whatever U is. Lane t of a warp owns
// row t of each of the four records: it loads its 2 x 16 bytes of each
// record (128-bit loads, the next K-step's in flight while one is used),
// dequantises in registers and accumulates per token. Where a warp's range
// ends inside an M-tile it stores its partial sums; the warp that finishes
// an M-tile's last piece (a counter per M-tile) adds the pieces in range
// order, applies SwiGLU and writes act. The down projection works the same
// way over 128-row M-tiles of the down matrix and writes y = w * (down . act)
// per slot; the existing combine adds the slots in the reference's union
// order. No bulk copies, no mbarriers: nothing waits on another block except
// through the counters, whose last arrival is the only reader.
#include <algorithm>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

constexpr int kGvWarps = 8;     // warps per block
constexpr int kGvMaxTok = 4;    // B <= 4
constexpr int kGvPiece = 4 * kGvMaxTok * 32;  // floats per stored piece: [4 records][tokens][32 lanes]
constexpr int kMaxUnion = 256;  // union experts (E <= 256)

// B*k: the slots of the batch (uh[U])
__device__ __forceinline__ int uh_s_total(const jl_ws& ws, int U) { return ws.uh[U]; }

// Owner warp of K-step q when Q steps are cut into NW contiguous ranges
// [w*Q/NW, (w+1)*Q/NW) (NW <= Q, so every range is non-empty).
__device__ __forceinline__ int owner(int q, int Q, int NW) {
    return (int)(((long long)(q + 1) * NW - 1) / Q);
}
__device__ __forceinline__ int range_start(int w, int Q, int NW) { return (int)((long long)w * Q / NW); }

struct rec4 {
    uint4 a[4][2];   // record r: bytes 0-15 and 16-31 of this lane's row group
    uint32_t s[2];   // the four fp16 scales, two per word
};

__device__ __forceinline__ void load_rec4(const uint8_t* p, int lane, rec4& r) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint8_t* rec = p + (size_t)i * kTileRec;
        r.a[i][0] = __ldg(reinterpret_cast<const uint4*>(rec + lane * 16));
        r.a[i][1] = __ldg(reinterpret_cast<const uint4*>(rec + 512 + lane * 16));
    }
    const uint16_t s0 = __ldg(reinterpret_cast<const uint16_t*>(p + 0 * kTileRec + kTileBytes) + lane);
    const uint16_t s1 = __ldg(reinterpret_cast<const uint16_t*>(p + 1 * kTileRec + kTileBytes) + lane);
    const uint16_t s2 = __ldg(reinterpret_cast<const uint16_t*>(p + 2 * kTileRec + kTileBytes) + lane);
    const uint16_t s3 = __ldg(reinterpret_cast<const uint16_t*>(p + 3 * kTileRec + kTileBytes) + lane);
    r.s[0] = (uint32_t)s0 | ((uint32_t)s1 << 16);
    r.s[1] = (uint32_t)s2 | ((uint32_t)s3 << 16);
}

// acc[i][t] += scale_i * (row . xs_t) over one 64-value group for the four
// records i of one K-step; xs_t (shared memory) is token t's 64 inputs.
template <int NT>
__device__ __forceinline__ void step_dot(const rec4& r, const float* const (&xs)[NT], int nt,
                                         float (&acc)[4][NT]) {
    float2 part[4][NT];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int t = 0; t < NT; t++) part[i][t] = make_float2(0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 8; w++) {
        float4 x0[NT], x1[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) {
            if (t < nt) {
                x0[t] = *reinterpret_cast<const float4*>(xs[t] + 8 * w);
                x1[t] = *reinterpret_cast<const float4*>(xs[t] + 8 * w + 4);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint4& q = r.a[i][w >> 2];
            const uint32_t word = (w & 3) == 0 ? q.x : (w & 3) == 1 ? q.y : (w & 3) == 2 ? q.z : q.w;
            float2 a[4];
            dequant8x2(word, a);
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < nt) {
                    part[i][t] = __ffma2_rn(a[0], make_float2(x0[t].x, x0[t].y), part[i][t]);
                    part[i][t] = __ffma2_rn(a[1], make_float2(x0[t].z, x0[t].w), part[i][t]);
                    part[i][t] = __ffma2_rn(a[2], make_float2(x1[t].x, x1[t].y), part[i][t]);
                    part[i][t] = __ffma2_rn(a[3], make_float2(x1[t].z, x1[t].w), part[i][t]);
                }
            }
        }
    }
    const float sc[4] = {half_bits_to_f32((uint16_t)(r.s[0] & 0xFFFFu)), half_bits_to_f32((uint16_t)(r.s[0] >> 16)),
                         half_bits_to_f32((uint16_t)(r.s[1] & 0xFFFFu)), half_bits_to_f32((uint16_t)(r.s[1] >> 16))};
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[i][t] = __fmaf_rn(__fadd_rn(part[i][t].x, part[i][t].y), sc[i], acc[i][t]);
}

// Store this warp's partial of M-tile `unit` as piece p; the warp whose
// arrival completes the M-tile's np pieces gets true and the pieces' sum (in
// piece order) in acc.
template <int NT>
__device__ __forceinline__ bool piece_done(float (&acc)[4][NT], int nt, int unit, int p, int np, float* parts,
                                           int* counters) {
    const int lane = threadIdx.x & 31;
    if (np == 1) return true;
    float* mine = parts + ((size_t)unit * 64 + p) * kGvPiece;  // at most 64 pieces per M-tile
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int t = 0; t < NT; t++)
            if (t < nt) mine[(i * kGvMaxTok + t) * 32 + lane] = acc[i][t];
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(counters + unit, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != np - 1) return false;
    __threadfence();
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[i][t] = 0.0f;
    // pieces in order; loads of 8 pieces are in flight before their adds
    for (int q0 = 0; q0 < np; q0 += 8) {
        float v[8][4][NT];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float* pp = parts + ((size_t)unit * 64 + q0 + j) * kGvPiece;
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int t = 0; t < NT; t++)
                    v[j][i][t] = (q0 + j < np && t < nt) ? __ldcg(pp + (i * kGvMaxTok + t) * 32 + lane) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (q0 + j < np)
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int t = 0; t < NT; t++) acc[i][t] = __fadd_rn(acc[i][t], v[j][i][t]);
    }
    if (lane == 0) counters[unit] = 0;  // every piece has arrived: ready for the next launch
    return true;
}

// ---------------------------------------------------------------------------
// gate/up + SwiGLU. grid = SMs x kGvWarps warps.
template <int NT>
__global__ void __launch_bounds__(kGvWarps * 32) k_gateup_gemv(const uint8_t* __restrict__ store_l, jl_layout L,
                                                               int k, const float* __restrict__ x, int B,
                                                               jl_ws ws) {
    extern __shared__ __align__(16) float x_s[];  // [B][d]
    __shared__ int sel_s[kMaxUnion], uh_s[kMaxUnion + 1], tok_s[kGvMaxTok * 16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = L.d, m = L.m, ngd = L.ngd, MT = m / 64;
    long long* tr = blockIdx.x == 0 ? ws.trace : nullptr;
    trace_point(tr, kTraceGateup, 0);
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceGateup, 1);
    const int U = *ws.U;
    const int Q = U * MT * ngd;
    const int NW = min((int)gridDim.x * kGvWarps, Q);
    const int wg = blockIdx.x * kGvWarps + warp;
    // this warp's first K-step: its weights go out before anything else
    const int q0 = wg < NW ? range_start(wg, Q, NW) : 0, q1 = wg < NW ? range_start(wg + 1, Q, NW) : 0;
    auto addr = [&](int q, const int* sel) {
        const int unit = q / ngd, g = q - unit * ngd;
        const int u = unit / MT, mt = unit - u * MT;
        return store_l + (size_t)sel[u] * L.rec_bytes + L.tile_off(0, 2 * mt, g);
    };
    rec4 cur, nxt;
    if (wg < NW) load_rec4(addr(q0, ws.sel), lane, cur);
    for (int i = threadIdx.x; i < U; i += blockDim.x) sel_s[i] = ws.sel[i];
    for (int i = threadIdx.x; i <= U; i += blockDim.x) uh_s[i] = ws.uh[i];
    for (int i = threadIdx.x; i < B * k; i += blockDim.x) tok_s[i] = ws.uidx[i];
    for (int i = threadIdx.x; i < B * d / 4; i += blockDim.x)
        reinterpret_cast<float4*>(x_s)[i] = reinterpret_cast<const float4*>(x)[i];
    __syncthreads();
    trace_point(tr, kTraceGateup, 2);
    if (wg >= NW) return;
    float acc[4][NT];
    int unit = -1, nt = 0, s0 = 0;
    const float* xs[NT];
    for (int q = q0; q < q1; q++) {
        const int qu = q / ngd, g = q - qu * ngd;
        if (qu != unit) {
            unit = qu;
            const int u = unit / MT;
            s0 = uh_s[u];
            nt = min(NT, uh_s[u + 1] - s0);
#pragma unroll
            for (int t = 0; t < NT; t++) {
                acc[0][t] = acc[1][t] = acc[2][t] = acc[3][t] = 0.0f;
                xs[t] = x_s + (size_t)(t < nt ? tok_s[s0 + t] / k : 0) * d;
            }
        }
        if (q + 1 < q1) load_rec4(addr(q + 1, sel_s), lane, nxt);
        const float* xg[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) xg[t] = xs[t] + g * 64;
        step_dot<NT>(cur, xg, nt, acc);
        cur = nxt;
        if (q + 1 == q1 || g == ngd - 1) {
            const int fq = unit * ngd;
            const int pw0 = owner(fq, Q, NW), pw1 = owner(fq + ngd - 1, Q, NW);
            if (piece_done<NT>(acc, nt, unit, wg - pw0, pw1 - pw0 + 1, ws.gv_parts, ws.gv_count)) {
                const int mt = unit % MT;
                for (int t = 0; t < nt; t++) {
                    float* a = ws.act + (size_t)tok_s[s0 + t] * m + mt * 64 + lane;
                    a[0] = silu_mul(acc[0][t], acc[2][t]);
                    a[32] = silu_mul(acc[1][t], acc[3][t]);
                }
            }
        }
    }
    if (warp == 0) trace_point(tr, kTraceGateup, 3);
}

// ---------------------------------------------------------------------------
// down: K-steps are (expert, 128-row M-tile of d, group of m): four records
// (rows 0-31, ..., 96-127) = 4352 contiguous bytes. y[slot][row] = 0 + w * sum.
// Each block stages the act rows of the union experts its warps touch.
template <int NT>
__global__ void __launch_bounds__(kGvWarps * 32) k_down_gemv(const uint8_t* __restrict__ store_l, jl_layout L,
                                                             jl_ws ws, int span) {
    extern __shared__ __align__(16) float a_s[];  // [span experts][NT][m]
    __shared__ int sel_s[kMaxUnion], uh_s[kMaxUnion + 1], slot_s[kGvMaxTok * 16];
    __shared__ float w_s[kGvMaxTok * 16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = L.d, m = L.m, ngm = L.ngm, MT = d / 128;
    // The routing is the router's output, complete before gate/up released
    // this grid: read it (and this warp's first weights) before the wait.
    const int U = *ws.U;
    const int Q = U * MT * ngm;
    const int NW = min((int)gridDim.x * kGvWarps, Q);
    const int wg = blockIdx.x * kGvWarps + warp;
    const bool active = wg < NW;
    const int q0 = active ? range_start(wg, Q, NW) : 0, q1 = active ? range_start(wg + 1, Q, NW) : 0;
    auto addr = [&](int q, const int* sel) {
        const int unit = q / ngm, g = q - unit * ngm;
        const int u = unit / MT, mt = unit - u * MT;
        return store_l + (size_t)sel[u] * L.rec_bytes + L.tile_off(2, 4 * mt, g);
    };
    long long* tr = blockIdx.x == 0 ? ws.trace : nullptr;
    trace_point(tr, kTraceDown, 0);
    rec4 cur, nxt;
    if (active) load_rec4(addr(q0, ws.sel), lane, cur);
    for (int i = threadIdx.x; i < U; i += blockDim.x) sel_s[i] = ws.sel[i];
    for (int i = threadIdx.x; i <= U; i += blockDim.x) uh_s[i] = ws.uh[i];
    const int S = uh_s_total(ws, U);
    for (int i = threadIdx.x; i < S; i += blockDim.x) {
        slot_s[i] = ws.uidx[i];
        w_s[i] = ws.uw[i];
    }
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceDown, 1);
    // the block's experts: union positions from its first warp's to its last warp's
    const int wb0 = blockIdx.x * kGvWarps;
    if (wb0 >= NW) return;
    const int wb1 = min(wb0 + kGvWarps, NW) - 1;
    const int bq0 = range_start(wb0, Q, NW), bq1 = range_start(wb1 + 1, Q, NW) - 1;
    const int u_lo = (bq0 / ngm) / MT, u_hi = (bq1 / ngm) / MT;
    if (u_hi - u_lo + 1 > span) {  // more experts than the staging area holds (host bound violated)
        if (threadIdx.x == 0) atomicOr(ws.err, kErrCapacity);
        return;
    }
    __syncthreads();
    for (int uu = u_lo; uu <= u_hi; uu++) {
        const int s0 = uh_s[uu], nt = min(NT, uh_s[uu + 1] - s0);
        float* dst = a_s + (size_t)(uu - u_lo) * NT * m;
        for (int i = threadIdx.x; i < nt * m / 4; i += blockDim.x) {
            const int t = i / (m / 4), c = i % (m / 4);
            reinterpret_cast<float4*>(dst + (size_t)t * m)[c] =
                reinterpret_cast<const float4*>(ws.act + (size_t)slot_s[s0 + t] * m)[c];
        }
    }
    __syncthreads();
    if (!active) return;
    float acc[4][NT];
    int unit = -1, nt = 0, s0 = 0;
    const float* as[NT];
    for (int q = q0; q < q1; q++) {
        const int qu = q / ngm, g = q - qu * ngm;
        if (qu != unit) {
            unit = qu;
            const int u = unit / MT;
            s0 = uh_s[u];
            nt = min(NT, uh_s[u + 1] - s0);
#pragma unroll
            for (int t = 0; t < NT; t++) {
                acc[0][t] = acc[1][t] = acc[2][t] = acc[3][t] = 0.0f;
                as[t] = a_s + ((size_t)(u - u_lo) * NT + (t < nt ? t : 0)) * m;
            }
        }
        if (q + 1 < q1) load_rec4(addr(q + 1, sel_s), lane, nxt);
        const float* ag[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) ag[t] = as[t] + g * 64;
        step_dot<NT>(cur, ag, nt, acc);
        cur = nxt;
        if (q + 1 == q1 || g == ngm - 1) {
            const int fq = unit * ngm;
            const int pw0 = owner(fq, Q, NW), pw1 = owner(fq + ngm - 1, Q, NW);
            if (piece_done<NT>(acc, nt, unit, wg - pw0, pw1 - pw0 + 1, ws.gv_parts_dn, ws.gv_count_dn)) {
                const int mt = unit % MT;
                for (int t = 0; t < nt; t++) {
                    const int slot = slot_s[s0 + t];
                    const float w = w_s[s0 + t];
                    float* y = ws.y + (size_t)slot * d + mt * 128 + lane;
#pragma unroll
                    for (int i = 0; i < 4; i++) y[32 * i] = __fadd_rn(0.0f, __fmul_rn(w, acc[i][t]));
                }
            }
        }
    }
    if (warp == 0) trace_point(tr, kTraceDown, 3);
}

}  // namespace jl

size_t jl_gemv_ws_floats(int E, int k, int d, int m, size_t* dn_off, size_t* count_off) {
    const int U = std::min(E, jl::kGvMaxTok * k);
    const size_t gu = (size_t)U * (m / 64) * 64 * jl::kGvPiece;
    const size_t dn = (size_t)U * (d / 128) * 64 * jl::kGvPiece;
    *dn_off = gu;
    *count_off = gu + dn;
    return gu + dn + (size_t)U * ((m / 64) + (d / 128));
}

bool jl_gemv_ok(const jl_moe* h, int B) {
    return h->ws.gv_parts && B >= 1 && B <= jl::kGvMaxTok && h->d % 128 == 0 && h->m % 64 == 0 &&
           h->d / 64 <= 64 && h->m / 64 <= 64;
}

static int gemv_attrs() {
    return jl_device_once(kOnceGemv, [] {
        using namespace jl;
        const int big = 200 * 1024;
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
    const dim3 grid(h->sm_count), block(kGvWarps * 32);
    if (B == 1) return launch(k_gateup_gemv<1>, grid, block, smem, s, store_l, h->lay, h->k, x, B, h->ws);
    if (B == 2) return launch(k_gateup_gemv<2>, grid, block, smem, s, store_l, h->lay, h->k, x, B, h->ws);
    return launch(k_gateup_gemv<4>, grid, block, smem, s, store_l, h->lay, h->k, x, B, h->ws);
}

int jl_launch_down_gemv(const jl_moe* h, const uint8_t* store_l, int B, cudaStream_t s) {
    using namespace jl;
    if (!jl_gemv_ok(h, B)) return JL_ERR_INVALID;
    int rc = gemv_attrs();
    if (rc) return rc;
    const int nt = B == 1 ? 1 : B == 2 ? 2 : 4;
    // Experts one block's warps can touch: with U <= Umax union experts of spe
    // K-steps each and NW = min(grid warps, Q) ranges, a warp holds at most
    // spw = ceil(Qmax / grid warps) steps (1 when Q < grid warps), a block
    // 8 * spw contiguous steps, which meet at most (8 spw - 1) / spe + 2 experts.
    const long long spe = (long long)(h->m / 64) * (h->d / 128);
    const int Umax = std::min(h->E, B * h->k);
    const long long Qmax = Umax * spe, NWg = (long long)h->sm_count * kGvWarps;
    const long long spw = Qmax <= NWg ? 1 : (Qmax + NWg - 1) / NWg;
    const int span = (int)std::min<long long>(Umax, (kGvWarps * spw - 1) / spe + 2);
    const size_t smem = (size_t)span * nt * h->m * sizeof(float);
    if (smem > 200 * 1024) return JL_ERR_INVALID;
    const dim3 grid(h->sm_count), block(kGvWarps * 32);
    if (nt == 1) return launch(k_down_gemv<1>, grid, block, smem, s, store_l, h->lay, h->ws, span);
    if (nt == 2) return launch(k_down_gemv<2>, grid, block, smem, s, store_l, h->lay, h->ws, span);
    return launch(k_down_gemv<4>, grid, block, smem, s, store_l, h->lay, h->ws, span);
}
