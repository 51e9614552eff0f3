// Routing device code of the router kernels (jl_router.cu): per-token
// softmax / top-k / renorm and the warp-level dispatch for up to 128 slots.
#pragma once

#include <climits>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

constexpr int kMaxK = 16;         // top-k capacity (the reference caps topk at 16, ws_init)
constexpr int kMaxE = 256;

__device__ __forceinline__ int clamp_e(int e, int E) { return (e < 0 || e >= E) ? 0 : e; }

// comb: token b's slots in the union order of their experts (stable for
// equal positions). Slot s goes to position #{i2 : (u[i2], i2) < (u[i], i)}
// of its token's k-slot list.
__device__ __forceinline__ void comb_slot(const int* top, const int* upos, int s, int k, int E,
                                          int* comb) {
    const int b = s / k, i = s - b * k;
    const int u = upos[clamp_e(top[s], E)];
    int r = 0;
    for (int i2 = 0; i2 < k; i2++) {
        const int u2 = upos[clamp_e(top[b * k + i2], E)];
        r += (u2 < u) || (u2 == u && i2 < i);
    }
    comb[b * k + r] = s;
}

// Dispatch for S = B*k <= 128 slots by warp 0 alone (no block barriers):
// union positions in first-appearance order from __match_any_sync leaders,
// offsets by a warp scan, ranks inside an expert by running counts.
// Same outputs as dispatch_block. `sm` holds 4*E + 2 ints.
__device__ __forceinline__ void dispatch_warp_small(const int* top, const float* tw, int B, int k, int E,
                                    const jl_ws& ws, int* sm) {
    const int lane = threadIdx.x & 31, S = B * k;
    const unsigned lt = (1u << lane) - 1u;
    int* upos = sm;          // [E]
    int* cnt = upos + E;     // [E]
    int* run = cnt + E;      // [E]
    int* sel_s = run + E;    // [E]
    for (int e = lane; e < E; e += 32) {
        upos[e] = -1;
        cnt[e] = 0;
        run[e] = 0;
    }
    __syncwarp();
    int U = 0;
    for (int c0 = 0; c0 < S; c0 += 32) {
        const int s = c0 + lane;
        const bool valid = s < S;
        int e = valid ? top[s] : -1 - lane;
        if (valid && (e < 0 || e >= E)) {
            atomicOr(ws.err, kErrBadExpert);
            e = 0;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const bool leader = valid && lane == __ffs(peers) - 1;
        const bool fresh = leader && upos[e] < 0;
        const unsigned bal = __ballot_sync(0xffffffffu, fresh);
        if (fresh) {
            const int u = U + __popc(bal & lt);
            upos[e] = u;
            sel_s[u] = e;
            ws.sel[u] = e;
        }
        if (leader) cnt[e] += __popc(peers);
        U += __popc(bal);
        __syncwarp();
    }
    int acc = 0;
    for (int u0 = 0; u0 < U; u0 += 32) {
        const int u = u0 + lane;
        const int c = u < U ? cnt[sel_s[u]] : 0;
        int inc = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += t;
        }
        if (u < U) {
            ws.uh[u] = acc + inc - c;
            run[sel_s[u]] = acc + inc - c;  // start offset; ranks are added below
        }
        acc += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) {
        ws.uh[U] = acc;
        *ws.U = U;
    }
    __syncwarp();
    for (int c0 = 0; c0 < S; c0 += 32) {
        const int s = c0 + lane;
        const bool valid = s < S;
        int e = valid ? top[s] : -1 - lane;
        if (valid && (e < 0 || e >= E)) e = 0;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (valid) {
            const int pos = run[e] + __popc(peers & lt);
            ws.uidx[pos] = s;
            ws.uw[pos] = tw[s];
            ws.slot_pos[s] = pos;
        }
        __syncwarp();
        if (valid && lane == __ffs(peers) - 1) run[e] += __popc(peers);
        __syncwarp();
    }
    for (int s = lane; s < S; s += 32) comb_slot(top, upos, s, k, E, ws.comb);
}

// Shared-memory rows of the cluster router: router row (expert ee, lane j)
// holds that lane's d/8 bf16 weights plus 8 halves of padding, exactly as the
// lane-major HBM layout keeps them (one bulk copy per CTA); token row (tb, j)
// holds x[tb][j + 8t] for t < d/8, padded by 4 floats. With rows 16 bytes
// apart modulo 128, the 8 lanes x 4 experts of a warp read distinct banks.
__host__ __device__ inline int router_gstride(int d) { return router_row_halves(d); }  // halves
__host__ __device__ inline int router_xstride(int d) { return d / 8 + 4; }             // floats

// Thread t < ne*8 owns lane j = t % 8 of expert ee = t / 8 for all NB tokens
// of the cluster (nb <= NB live; the rest recompute token 0 and are not
// stored). Each step reads the lane's next 8 weights (one 16-byte load,
// shared by the NB tokens) and 8 activations per token (two), and the loads
// of step t + 8 are issued before the FMAs of step t: the dependent FMA chain
// of each (token, lane), in k order as the reference's lane j, sets the pace.
template <int NB>
__device__ __forceinline__ void cluster_logits(const uint16_t* g_s, const float* x_s, int d, int nb,
                                               int E, int e0, int ne, int b0, float* lg_lead,
                                               float* lg_glob) {
    const int tid = threadIdx.x;
    if ((tid & ~31) >= ne * 8) return;  // whole warp idle (warp-uniform)
    const int gs = router_gstride(d), xs = router_xstride(d), c8 = d / 8;
    const int live = tid < ne * 8;
    const int j = tid & 7, ee = live ? tid >> 3 : 0;
    const uint16_t* gp = g_s + (size_t)(ee * 8 + j) * gs;
    const float* xp[NB];
#pragma unroll
    for (int r = 0; r < NB; r++) xp[r] = x_s + (size_t)((r < nb ? r : 0) * 8 + j) * xs;
    float acc[NB];
    float4 xc0[NB], xc1[NB];
    uint4 gc = *reinterpret_cast<const uint4*>(gp);
#pragma unroll
    for (int r = 0; r < NB; r++) {
        acc[r] = 0.0f;
        xc0[r] = *reinterpret_cast<const float4*>(xp[r]);
        xc1[r] = *reinterpret_cast<const float4*>(xp[r] + 4);
    }
    for (int t0 = 0; t0 < c8; t0 += 8) {
        const int tn = (t0 + 8 < c8) ? t0 + 8 : t0;
        const uint4 gn = *reinterpret_cast<const uint4*>(gp + tn);
        float4 xn0[NB], xn1[NB];
#pragma unroll
        for (int r = 0; r < NB; r++) {
            xn0[r] = *reinterpret_cast<const float4*>(xp[r] + tn);
            xn1[r] = *reinterpret_cast<const float4*>(xp[r] + tn + 4);
        }
        const uint32_t w[4] = {gc.x, gc.y, gc.z, gc.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float lo = __uint_as_float(w[q] << 16), hi = __uint_as_float(w[q] & 0xFFFF0000u);
#pragma unroll
            for (int r = 0; r < NB; r++) {
                const float x0 = q == 0 ? xc0[r].x : q == 1 ? xc0[r].z : q == 2 ? xc1[r].x : xc1[r].z;
                const float x1 = q == 0 ? xc0[r].y : q == 1 ? xc0[r].w : q == 2 ? xc1[r].y : xc1[r].w;
                acc[r] = __fmaf_rn(lo, x0, acc[r]);
                acc[r] = __fmaf_rn(hi, x1, acc[r]);
            }
        }
        gc = gn;
#pragma unroll
        for (int r = 0; r < NB; r++) {
            xc0[r] = xn0[r];
            xc1[r] = xn1[r];
        }
    }
#pragma unroll
    for (int r = 0; r < NB; r++) {
        float a = acc[r];
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 2));
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
        if (live && j == 0 && r < nb) {
            if (lg_lead) lg_lead[r * E + e0 + ee] = a;
            lg_glob[(size_t)(b0 + r) * E + e0 + ee] = a;
        }
    }
}


// ---------------------------------------------------------------------------
// Routing of one token by one warp (decode_kernel.c:1425-1448) with the
// top-k as k rounds of a warp argmax (two warp reductions a round). Lane l
// holds experts l + 32 i.
//  - smax: max over experts; p_e = expf_fast(s_e - smax), summed
//    SEQUENTIALLY in expert order by lane 0 from `p_s` (32 * EPL floats of
//    this warp's shared memory; zeros past E leave the sum unchanged)
//  - p_e /= sum
//  - round r picks the unused expert with the largest p, the lowest index
//    among equal p: the expert the reference's r-th strict-'>' argmax pass
//    over ascending e picks
//  - optional renorm: sequential sum of the k weights in pick order, then
//    divide.
template <int EPL>
__device__ __forceinline__ void route_token_warp_argmax(const float* logits_b, int E, int k, int norm,
                                                        int* top_b, float* tw_b, float* p_s) {
    const int lane = threadIdx.x & 31;
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; i++) {
        const int e = lane + 32 * i;
        v[i] = (e < E) ? logits_b[e] : 0.0f;
    }
    float mx = -1e30f;
#pragma unroll
    for (int i = 0; i < EPL; i++)
        if (lane + 32 * i < E && v[i] > mx) mx = v[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float p[EPL];
#pragma unroll
    for (int i = 0; i < EPL; i++) {
        const int e = lane + 32 * i;
        p[i] = (e < E) ? expf_fast(__fsub_rn(v[i], mx)) : 0.0f;
        p_s[e] = p[i];
    }
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0) {  // 8 float4 ahead of the dependent adds
        const float4* q4 = reinterpret_cast<const float4*>(p_s);
        float4 cur[8];
#pragma unroll
        for (int c = 0; c < 8; c++) cur[c] = q4[c];
#pragma unroll
        for (int c0 = 0; c0 < EPL * 8; c0 += 8) {
            float4 nxt[8];
#pragma unroll
            for (int c = 0; c < 8; c++) nxt[c] = c0 + 8 + c < EPL * 8 ? q4[c0 + 8 + c] : cur[c];
#pragma unroll
            for (int c = 0; c < 8; c++) {
                sum = __fadd_rn(sum, cur[c].x);
                sum = __fadd_rn(sum, cur[c].y);
                sum = __fadd_rn(sum, cur[c].z);
                sum = __fadd_rn(sum, cur[c].w);
            }
#pragma unroll
            for (int c = 0; c < 8; c++) cur[c] = nxt[c];
        }
    }
    sum = __shfl_sync(0xffffffffu, sum, 0);
#pragma unroll
    for (int i = 0; i < EPL; i++) p[i] = __fdiv_rn(p[i], sum);
    // Each round: key = float bits of p + 1 for unused experts (p >= 0, so keys
    // order like p; 0 marks a picked expert), the lane's best key over its
    // experts in ascending order (strict '>': the lowest index among equals;
    // NaN never wins, as under the reference's '>'),
    // the warp's largest key by one redux, then the lowest expert index among
    // the lanes holding it by a second.
    unsigned used = 0;  // bit i: expert lane + 32 i already picked
    float ssum = 0.0f, mine = 0.0f;
    for (int r = 0; r < k; r++) {
        uint32_t bk = 0;
        int be = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < EPL; i++) {
            const int e = lane + 32 * i;
            const uint32_t key = (e < E && !((used >> i) & 1u) && p[i] == p[i]) ? __float_as_uint(p[i]) + 1u : 0u;
            if (key > bk) {
                bk = key;
                be = e;
            }
        }
        const uint32_t wk = __reduce_max_sync(0xffffffffu, bk);
        const int we = (int)__reduce_min_sync(0xffffffffu, bk == wk ? (uint32_t)be : 0x7fffffffu);
        const float bv = __uint_as_float(wk - 1u);
        if ((we & 31) == lane) used |= 1u << (we >> 5);
        if (lane == r) mine = bv;
        if (lane == 0) top_b[r] = we;
        ssum = __fadd_rn(ssum, bv);
    }
    if (lane < k) tw_b[lane] = norm ? __fdiv_rn(mine, ssum) : mine;
    __syncwarp();
}

__device__ __forceinline__ void route_token_lean(const float* logits_b, int E, int k, int norm, int* top_b,
                                                 float* tw_b, float* p_s) {
    if (E <= 32) route_token_warp_argmax<1>(logits_b, E, k, norm, top_b, tw_b, p_s);
    else if (E <= 64) route_token_warp_argmax<2>(logits_b, E, k, norm, top_b, tw_b, p_s);
    else if (E <= 128) route_token_warp_argmax<4>(logits_b, E, k, norm, top_b, tw_b, p_s);
    else route_token_warp_argmax<8>(logits_b, E, k, norm, top_b, tw_b, p_s);
}

}  // namespace jl
