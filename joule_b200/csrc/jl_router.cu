// Router: logits (bit-exact with the reference), softmax / top-k / renorm,
// and the token-to-expert dispatch (union of experts + slot map).
#include <climits>

#include <cooperative_groups.h>

#include "jl_common.cuh"
#include "jl_internal.h"
#include "jl_tiles.cuh"

#include <algorithm>

namespace jl {

constexpr int kRouteEPB = 4;      // experts per router block
constexpr int kRouteTB = 8;       // tokens per router block (one warp each)
constexpr int kFuseTailMaxB = 8;  // B up to which the last router block routes + dispatches
constexpr int kMaxK = 16;         // top-k capacity (the reference caps topk at 16, ws_init)
constexpr int kMaxE = 256;

// ---------------------------------------------------------------------------
// Per-token softmax / top-k / renorm by one warp (decode_kernel.c:1425-1448).
// `p_s` is 32*EPL floats of shared memory private to this warp.
//  - smax: max over experts (the reference scans with strict '>' from -1e30)
//  - p_e = expf_fast(s_e - smax), summed SEQUENTIALLY in expert order (lane 0,
//    vector loads issued up front, one dependent add per expert)
//  - p_e /= sum
//  - top-k: the reference's k argmax passes (strict '>', ascending scan) pick
//    experts in order of (p descending, index ascending); here each lane ranks
//    its experts against all E by that order and the ones ranked < k are
//    written at their rank: same ids, same order, no dependent passes.
//  - optional renorm: sequential sum of the k weights, then divide.
template <int EPL>
__device__ void route_token_warp_t(const float* logits_b, int E, int k, int norm, int* top_b,
                                   float* tw_b, float* p_s) {
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
        p_s[e] = p[i];  // zero past E: adding +0 to a positive sum leaves it unchanged
    }
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0) {
        float4 q[EPL * 8];
#pragma unroll
        for (int c = 0; c < EPL * 8; c++) q[c] = reinterpret_cast<const float4*>(p_s)[c];
#pragma unroll
        for (int c = 0; c < EPL * 8; c++) {
            sum = __fadd_rn(sum, q[c].x);
            sum = __fadd_rn(sum, q[c].y);
            sum = __fadd_rn(sum, q[c].z);
            sum = __fadd_rn(sum, q[c].w);
        }
    }
    sum = __shfl_sync(0xffffffffu, sum, 0);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < EPL; i++) {
        p[i] = __fdiv_rn(p[i], sum);
        p_s[lane + 32 * i] = p[i];
    }
    __syncwarp();
    int rank[EPL];
#pragma unroll
    for (int i = 0; i < EPL; i++) rank[i] = 0;
    for (int c = 0; c < (E + 3) / 4; c++) {
        const float4 q = reinterpret_cast<const float4*>(p_s)[c];
        const float qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const int e2 = 4 * c + t;
            if (e2 >= E) break;
#pragma unroll
            for (int i = 0; i < EPL; i++) {
                const int e = lane + 32 * i;
                rank[i] += (qq[t] > p[i]) || (qq[t] == p[i] && e2 < e);
            }
        }
    }
    __syncwarp();
    // p_s reused: [k] selected weights for the renorm
#pragma unroll
    for (int i = 0; i < EPL; i++) {
        const int e = lane + 32 * i;
        if (e < E && rank[i] < k) {
            top_b[rank[i]] = e;
            p_s[rank[i]] = p[i];
        }
    }
    __syncwarp();
    if (lane < k) {
        float w = p_s[lane];
        if (norm) {
            float ssum = 0.0f;
            for (int i = 0; i < k; i++) ssum = __fadd_rn(ssum, p_s[i]);
            w = __fdiv_rn(w, ssum);
        }
        tw_b[lane] = w;
    }
    __syncwarp();
}

__device__ void route_token_warp(const float* logits_b, int E, int k, int norm, int* top_b,
                                 float* tw_b, float* p_s) {
    if (E <= 32) route_token_warp_t<1>(logits_b, E, k, norm, top_b, tw_b, p_s);
    else if (E <= 64) route_token_warp_t<2>(logits_b, E, k, norm, top_b, tw_b, p_s);
    else if (E <= 128) route_token_warp_t<4>(logits_b, E, k, norm, top_b, tw_b, p_s);
    else route_token_warp_t<8>(logits_b, E, k, norm, top_b, tw_b, p_s);
}

// ---------------------------------------------------------------------------
// Dispatch by one block (decode_kernel.c:1449-1485, same outputs):
//   sel[u]      experts in first-appearance order over the slots s = b*k + i
//   uh[u]       exclusive prefix of per-expert slot counts, uh[U] = B*k
//   uidx/uw     slots grouped by union position, increasing slot order inside
//   slot_pos[s] index of slot s in uidx
//   comb[b*k+j] token b's slots ordered by the union position of their expert
// Union positions come from a block-wide scan of "first slot of its expert"
// flags, offsets from a warp scan over the union, and ranks inside an expert
// from per-warp slot ranges (count prefix + __match_any_sync in 32-slot
// chunks): O(B*k / threads + E) work, no quadratic search.
__host__ __device__ inline int dispatch_smem_ints(int E, int W) { return 6 * E + 36 + W * E; }

__device__ __forceinline__ int clamp_e(int e, int E) { return (e < 0 || e >= E) ? 0 : e; }

__device__ void dispatch_block(const int* top, const float* tw, int B, int k, int E,
                               const jl_ws& ws, int* sm) {
    const int S = B * k;
    const int T = blockDim.x, tid = threadIdx.x, W = T >> 5, warp = tid >> 5, lane = tid & 31;
    const unsigned lt = (1u << lane) - 1u;
    int* first = sm;            // [E] first slot of expert e
    int* cnt = first + E;       // [E] slots of expert e
    int* upos = cnt + E;        // [E] union position of e (-1: unused)
    int* base = upos + E;       // [E] first uidx index of e
    int* sel_s = base + E;      // [E] union position -> expert
    int* ustart = sel_s + E;    // [E] union position -> first uidx index
    int* wtot = ustart + E;     // [32] per-warp totals (scans)
    int* misc = wtot + 32;      // [4]
    int* wrun = misc + 4;       // [W, E]
    for (int e = tid; e < E; e += T) {
        first[e] = INT_MAX;
        cnt[e] = 0;
        upos[e] = -1;
    }
    for (int i = tid; i < W * E; i += T) wrun[i] = 0;
    __syncthreads();
    const int per = (S + W - 1) / W;
    const int s_lo = min(S, warp * per), s_hi = min(S, s_lo + per);
    for (int s = s_lo + lane; s < s_hi; s += 32) {
        const int e0 = top[s];
        if (e0 < 0 || e0 >= E) atomicOr(ws.err, kErrBadExpert);
        const int e = clamp_e(e0, E);
        atomicMin(&first[e], s);
        atomicAdd(&cnt[e], 1);
        atomicAdd(&wrun[warp * E + e], 1);
    }
    __syncthreads();
    // union positions: exclusive scan over slots of "s is the first slot of its expert"
    int carry = 0;
    for (int c0 = 0; c0 < S; c0 += T) {
        const int s = c0 + tid;
        const int e = (s < S) ? clamp_e(top[s], E) : 0;
        const bool f = (s < S) && first[e] == s;
        const unsigned bal = __ballot_sync(0xffffffffu, f);
        if (lane == 0) wtot[warp] = __popc(bal);
        __syncthreads();
        if (warp == 0) {
            const int v = lane < W ? wtot[lane] : 0;
            int inc = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += t;
            }
            if (lane < W) wtot[lane] = inc - v;
            if (lane == 31) misc[0] = inc;
        }
        __syncthreads();
        if (f) {
            const int u = carry + wtot[warp] + __popc(bal & lt);
            upos[e] = u;
            sel_s[u] = e;
            ws.sel[u] = e;
        }
        carry += misc[0];
        __syncthreads();
    }
    const int U = carry;
    // slot offsets per union position (warp 0 scans cnt in union order)
    if (warp == 0) {
        int run = 0;
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
                ustart[u] = run + inc - c;
                ws.uh[u] = run + inc - c;
            }
            run += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) {
            ws.uh[U] = run;
            *ws.U = U;
        }
    }
    __syncthreads();
    for (int e = tid; e < E; e += T) {
        base[e] = (upos[e] >= 0) ? ustart[upos[e]] : 0;
        int run = 0;
        for (int w = 0; w < W; w++) {
            const int c = wrun[w * E + e];
            wrun[w * E + e] = run;
            run += c;
        }
    }
    __syncthreads();
    for (int c0 = s_lo; c0 < s_hi; c0 += 32) {
        const int s = c0 + lane;
        const bool valid = s < s_hi;
        const int e = valid ? clamp_e(top[s], E) : -1 - lane;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (valid) {
            const int pos = base[e] + wrun[warp * E + e] + __popc(peers & lt);
            ws.uidx[pos] = s;
            ws.uw[pos] = tw[s];
            ws.slot_pos[s] = pos;
        }
        __syncwarp();
        if (valid && lane == __ffs(peers) - 1) wrun[warp * E + e] += __popc(peers);
        __syncwarp();
    }
    for (int b = tid; b < B; b += T) {
        int us[kMaxK], ss[kMaxK];
        for (int i = 0; i < k; i++) {
            const int u = upos[clamp_e(top[b * k + i], E)];
            int j = i;
            while (j > 0 && us[j - 1] > u) {
                us[j] = us[j - 1];
                ss[j] = ss[j - 1];
                j--;
            }
            us[j] = u;
            ss[j] = b * k + i;
        }
        for (int i = 0; i < k; i++) ws.comb[b * k + i] = ss[i];
    }
}

// ---------------------------------------------------------------------------
// Router logits, bit-exact with matvec_f32[_B] (decode_kernel.c:234-256,
// 693-718): lane j of an 8-wide accumulator sums k = j (mod 8) by FMA in k
// order; the 8 lanes are reduced in the AVX order. One thread per (token,
// expert, lane j); 4 experts x up to 8 tokens per block. The 4 router rows
// are staged by bulk copies issued before waiting on the previous kernel
// (they do not depend on it), then the token rows. With `fuse_tail`, the
// last block to finish also routes every token and builds the dispatch.
__global__ void k_router(const uint16_t* __restrict__ gate_w, const float* __restrict__ x, int B,
                         int E, int d, int k, int norm, jl_ws ws, int fuse_tail) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar[2];
    __shared__ int is_last;
    const int tid = threadIdx.x, TB = blockDim.x >> 5;
    const int e0 = blockIdx.x * kRouteEPB, b0 = blockIdx.y * TB;
    const int nb = min(TB, B - b0), ne = min(kRouteEPB, E - e0);
    const int grow = d * 2 + 16;  // padded router row: lanes of 4 experts hit distinct banks
    uint8_t* g_s = smem;
    float* x_s = reinterpret_cast<float*>(smem + kRouteEPB * grow);
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_fence_init();
        mbar_expect_tx(&bar[0], (uint32_t)(ne * d * 2));
        for (int r = 0; r < ne; r++)
            bulk_g2s(g_s + r * grow, gate_w + (size_t)(e0 + r) * d, (uint32_t)(d * 2), &bar[0]);
    }
    griddep_wait();  // x is the previous kernel's output
    griddep_launch_dependents();
    if (tid == 0) {
        mbar_expect_tx(&bar[1], (uint32_t)(nb * d * 4));
        bulk_g2s(x_s, x + (size_t)b0 * d, (uint32_t)(nb * d * 4), &bar[1]);
    }
    __syncthreads();
    const bool ok0 = mbar_wait_bounded(&bar[0], 0, ws.err);
    const bool ok1 = mbar_wait_bounded(&bar[1], 0, ws.err);
    const int tb = tid >> 5, ee = (tid >> 3) & 3, j = tid & 7;
    const bool live = ok0 && ok1 && tb < nb && ee < ne;
    float acc = 0.0f;
    if (live) {
        const uint16_t* gr = reinterpret_cast<const uint16_t*>(g_s + ee * grow) + j;
        const float* xr = x_s + tb * d + j;
        const int c8 = d / 8;
#pragma unroll 8
        for (int t = 0; t < c8; t++) acc = __fmaf_rn(bf16_to_f32(gr[8 * t]), xr[8 * t], acc);
    }
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
    if (live && j == 0) ws.logits[(size_t)(b0 + tb) * E + e0 + ee] = acc;
    if (!fuse_tail) return;

    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = (atomicAdd(ws.counter, 1) == (int)(gridDim.x * gridDim.y) - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (tid == 0) *ws.counter = 0;
    float* p_s = reinterpret_cast<float*>(smem);  // [TB, kMaxE]; staging no longer needed
    for (int b = tb; b < B; b += TB)
        route_token_warp(ws.logits + (size_t)b * E, E, k, norm, ws.top + b * k, ws.tw + b * k,
                         p_s + tb * kMaxE);
    __syncthreads();
    dispatch_block(ws.top, ws.tw, B, k, E, ws, reinterpret_cast<int*>(smem) + TB * kMaxE);
}

// ---------------------------------------------------------------------------
// Small-batch routing tail, run by one whole CTA (B <= 8). G = blockDim /
// next_pow2(B) threads share a token (G >= 32) and synchronise on named
// barrier 1 + token. Same arithmetic as route_token_warp: max, expf_fast,
// sequential sum (one thread, vector loads), division, rank-based top-k in
// (p desc, index asc) order, sequential renorm.
__device__ __forceinline__ void named_barrier(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ void route_tokens_cta(const float* lg_s, int B, int E, int k, int norm, const jl_ws& ws,
                                 float* scratch) {
    const int T = blockDim.x, tid = threadIdx.x;
    const int Bp = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : 8;
    const int G = T / Bp, b = tid / G, gl = tid % G;
    const int Ep = (E + 3) & ~3;
    float* p_s = scratch + b * (Ep + 64);  // [Ep] probabilities, then 64 floats of misc
    float* misc = p_s + Ep;                // [0..31] warp maxima, [32] max, [33] sum, [40..55] top-k weights
    const bool active = b < B;
    const int bar_id = 1 + b;
    if (active) {
        const float* lg = lg_s + b * E;
        float mx = -1e30f;
        for (int e = gl; e < E; e += G) {
            const float v = lg[e];
            if (v > mx) mx = v;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((gl & 31) == 0) misc[gl >> 5] = mx;
        named_barrier(bar_id, G);
        mx = misc[0];
        for (int w = 1; w < G / 32; w++) mx = fmaxf(mx, misc[w]);
        for (int e = gl; e < Ep; e += G) p_s[e] = (e < E) ? expf_fast(__fsub_rn(lg[e], mx)) : 0.0f;
        named_barrier(bar_id, G);
        if (gl == 0) {  // the sum runs sequentially in expert order
            float sum = 0.0f;
            for (int c = 0; c < Ep / 4; c += 8) {
                float4 q[8];
#pragma unroll
                for (int i = 0; i < 8; i++)
                    q[i] = (c + i < Ep / 4) ? reinterpret_cast<const float4*>(p_s)[c + i]
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    sum = __fadd_rn(sum, q[i].x);
                    sum = __fadd_rn(sum, q[i].y);
                    sum = __fadd_rn(sum, q[i].z);
                    sum = __fadd_rn(sum, q[i].w);
                }
            }
            misc[33] = sum;
        }
        named_barrier(bar_id, G);
        const float sum = misc[33];
        for (int e = gl; e < E; e += G) p_s[e] = __fdiv_rn(p_s[e], sum);
        named_barrier(bar_id, G);
        for (int e = gl; e < E; e += G) {
            const float pe = p_s[e];
            int rank = 0;
            for (int c = 0; c < Ep / 4; c++) {
                const float4 q = reinterpret_cast<const float4*>(p_s)[c];
                const int e2 = 4 * c;
                rank += (q.x > pe) || (q.x == pe && e2 + 0 < e);
                rank += (e2 + 1 < E) && ((q.y > pe) || (q.y == pe && e2 + 1 < e));
                rank += (e2 + 2 < E) && ((q.z > pe) || (q.z == pe && e2 + 2 < e));
                rank += (e2 + 3 < E) && ((q.w > pe) || (q.w == pe && e2 + 3 < e));
            }
            if (rank < k) {
                ws.top[b * k + rank] = e;
                misc[40 + rank] = pe;
            }
        }
        named_barrier(bar_id, G);
        if (gl < k) {
            float w = misc[40 + gl];
            if (norm) {
                float ssum = 0.0f;
                for (int i = 0; i < k; i++) ssum = __fadd_rn(ssum, misc[40 + i]);
                w = __fdiv_rn(w, ssum);
            }
            ws.tw[b * k + gl] = w;
        }
    }
    __syncthreads();
}

// Dispatch for S = B*k <= 128 slots by warp 0 alone (no block barriers):
// union positions in first-appearance order from __match_any_sync leaders,
// offsets by a warp scan, ranks inside an expert by running counts.
// Same outputs as dispatch_block. `sm` holds 4*E + 2 ints.
__device__ void dispatch_warp_small(const int* top, const float* tw, int B, int k, int E,
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
    if (lane < B) {
        const int b = lane;
        int us[kMaxK], ss[kMaxK];
        for (int i = 0; i < k; i++) {
            const int u = upos[clamp_e(top[b * k + i], E)];
            int j = i;
            while (j > 0 && us[j - 1] > u) {
                us[j] = us[j - 1];
                ss[j] = ss[j - 1];
                j--;
            }
            us[j] = u;
            ss[j] = b * k + i;
        }
        for (int i = 0; i < k; i++) ws.comb[b * k + i] = ss[i];
    }
}

// B == 1: the union is the top-k list itself (distinct experts in slot order).
__device__ void dispatch_one(int k, const jl_ws& ws) {
    const int i = threadIdx.x;
    if (i < k) {
        ws.sel[i] = ws.top[i];
        ws.uh[i] = i;
        ws.uidx[i] = i;
        ws.uw[i] = ws.tw[i];
        ws.slot_pos[i] = i;
        ws.comb[i] = i;
    }
    if (i == 0) {
        ws.uh[k] = k;
        *ws.U = k;
    }
}

// ---------------------------------------------------------------------------
// Small-batch router (B <= 8) on one 8-CTA thread-block cluster. CTA r stages
// router rows [r*EPC, (r+1)*EPC) (bulk copies issued before waiting on the
// previous kernel) and the B token rows, computes its logits in the
// reference's order (up to 4 independent chains per thread), and stores them
// into the leader CTA's shared memory over DSMEM; after the cluster barrier
// the leader routes every token (one warp each) and builds the dispatch.
constexpr int kClusterCTAs = 8;
constexpr int kClusterThreads = 256;

template <int R>
__device__ __forceinline__ void cluster_logits(const uint8_t* g_s, int grow, const float* x_s,
                                               int d, int B, int E, int e0, int ne, float* lg_lead,
                                               float* lg_glob) {
    const int tid = threadIdx.x;
    float acc[R];
    int idx[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        acc[r] = 0.0f;
        idx[r] = tid + r * kClusterThreads;
    }
    const int items = ne * B * 8;
    const uint16_t* gr[R];
    const float* xr[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int it = idx[r] < items ? idx[r] : 0;
        const int j = it & 7, L = it >> 3, ee = L / B, tb = L % B;
        gr[r] = reinterpret_cast<const uint16_t*>(g_s + ee * grow) + j;
        xr[r] = x_s + tb * d + j;
    }
    const int c8 = d / 8;
#pragma unroll 16
    for (int t = 0; t < c8; t++)
#pragma unroll
        for (int r = 0; r < R; r++)
            acc[r] = __fmaf_rn(bf16_to_f32(gr[r][8 * t]), xr[r][8 * t], acc[r]);
#pragma unroll
    for (int r = 0; r < R; r++) {
        float a = acc[r];
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 2));
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
        const int it = idx[r];
        if (it < items && (it & 7) == 0) {
            const int L = it >> 3, ee = L / B, tb = L % B;
            lg_lead[tb * E + e0 + ee] = a;
            lg_glob[(size_t)tb * E + e0 + ee] = a;
        }
    }
}

__global__ void __cluster_dims__(kClusterCTAs, 1, 1) __launch_bounds__(kClusterThreads)
    k_router_cluster(const uint16_t* __restrict__ gate_w, const float* __restrict__ x, int B, int E,
                     int d, int k, int norm, jl_ws ws, int lg_off) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar[2];
    const int tid = threadIdx.x;
    const int rank = (int)cluster.block_rank();
    const int EPC = (E + kClusterCTAs - 1) / kClusterCTAs;
    const int e0 = rank * EPC, ne = max(0, min(EPC, E - e0));
    const int grow = d * 2 + 16;  // padded router row: the 4 experts of a warp hit distinct banks
    uint8_t* g_s = smem;
    float* x_s = reinterpret_cast<float*>(smem + (size_t)EPC * grow);
    float* lg_s = reinterpret_cast<float*>(smem + lg_off);  // [B, E] logits (leader CTA's are read)
    long long* tr = (blockIdx.x == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceRouter, 0);
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_fence_init();
        mbar_expect_tx(&bar[0], (uint32_t)(ne * d * 2));
        for (int r = 0; r < ne; r++)
            bulk_g2s(g_s + (size_t)r * grow, gate_w + (size_t)(e0 + r) * d, (uint32_t)(d * 2), &bar[0]);
        if (ne == 0) mbar_arrive(&bar[0]);
    }
    griddep_wait();  // x is the previous kernel's output
    griddep_launch_dependents();
    trace_point(tr, kTraceRouter, 1);
    if (tid == 0) {
        mbar_expect_tx(&bar[1], (uint32_t)(B * d * 4));
        bulk_g2s(x_s, x, (uint32_t)(B * d * 4), &bar[1]);
    }
    __syncthreads();
    const bool ok = mbar_wait_bounded(&bar[0], 0, ws.err) & mbar_wait_bounded(&bar[1], 0, ws.err);
    trace_point(tr, kTraceRouter, 2);
    float* lg_lead = cluster.map_shared_rank(lg_s, 0);
    if (ok && ne > 0) {
        const int items = ne * B * 8;
        if (items <= kClusterThreads)
            cluster_logits<1>(g_s, grow, x_s, d, B, E, e0, ne, lg_lead, ws.logits);
        else if (items <= 2 * kClusterThreads)
            cluster_logits<2>(g_s, grow, x_s, d, B, E, e0, ne, lg_lead, ws.logits);
        else
            cluster_logits<4>(g_s, grow, x_s, d, B, E, e0, ne, lg_lead, ws.logits);
    }
    trace_point(tr, kTraceRouter, 3);
    cluster.sync();
    if (rank != 0) return;
    trace_point(tr, kTraceRouter, 4);
    // leader: staging no longer needed; scratch [8][kMaxE + 64] floats, then dispatch ints
    float* scratch = reinterpret_cast<float*>(smem);
    route_tokens_cta(lg_s, B, E, k, norm, ws, scratch);
    trace_point(tr, kTraceRouter, 5);
    if (B == 1) {
        dispatch_one(k, ws);
    } else if (tid < 32) {
        dispatch_warp_small(ws.top, ws.tw, B, k, E, ws,
                            reinterpret_cast<int*>(scratch + kRouteTB * (kMaxE + 64)));
    }
    __syncthreads();
    if (tid < 32) tc_build_tiles(ws);
    trace_point(tr, kTraceRouter, 6);
}

__global__ void k_topk(const float* __restrict__ logits, int B, int E, int k, int norm,
                       jl_ws ws) {
    extern __shared__ __align__(16) float p_all[];
    griddep_wait();
    griddep_launch_dependents();
    const int warp = threadIdx.x >> 5;
    const int b = blockIdx.x * (blockDim.x >> 5) + warp;
    if (b >= B) return;
    route_token_warp(logits + (size_t)b * E, E, k, norm, ws.top + b * k, ws.tw + b * k,
                     p_all + warp * kMaxE);
}

__global__ void k_dispatch(int B, int k, int E, jl_ws ws) {
    extern __shared__ __align__(16) int dsm[];
    griddep_wait();
    griddep_launch_dependents();
    dispatch_block(ws.top, ws.tw, B, k, E, ws, dsm);
    __syncthreads();
    if (threadIdx.x < 32) tc_build_tiles(ws);
}

}  // namespace jl

int jl_launch_route(const jl_moe* h, const unsigned short* gate_w_l, const float* x, int B,
                    cudaStream_t s) {
    using namespace jl;
    const int E = h->E, d = h->d, k = h->k;
    if (E > kMaxE || k > kMaxK || k < 1 || E < k) return JL_ERR_INVALID;
    static bool attr = false;
    if (!attr) {
        JL_CUDA(cudaFuncSetAttribute(k_router, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        JL_CUDA(cudaFuncSetAttribute(k_dispatch, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        JL_CUDA(cudaFuncSetAttribute(k_router_cluster, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        attr = true;
    }
    if (B <= kFuseTailMaxB) {
        const int EPC = (E + kClusterCTAs - 1) / kClusterCTAs;
        // [router rows | token rows] staging, reused by the leader's tail; logits after both
        const size_t stage = (size_t)EPC * (d * 2 + 16) + (size_t)kRouteTB * d * 4;
        const size_t tail = ((size_t)kRouteTB * (kMaxE + 64) + 4 * E + 2) * 4;
        const size_t lg_off = (std::max(stage, tail) + 127) / 128 * 128;
        const size_t smem = lg_off + (size_t)kRouteTB * E * 4;
        if (smem > 220 * 1024) return JL_ERR_INVALID;
        return launch(k_router_cluster, dim3(kClusterCTAs), dim3(kClusterThreads), smem, s, gate_w_l,
                      x, B, E, d, k, h->norm, h->ws, (int)lg_off);
    }
    const int TB = kRouteTB;
    const int threads = 32 * TB;
    const size_t smem = (size_t)kRouteEPB * (d * 2 + 16) + (size_t)TB * d * 4;
    if (smem > 220 * 1024) return JL_ERR_INVALID;
    dim3 grid((E + kRouteEPB - 1) / kRouteEPB, (B + TB - 1) / TB);
    int rc = launch(k_router, grid, dim3(threads), smem, s, gate_w_l, x, B, E, d, k, h->norm,
                    h->ws, 0);
    if (rc) return rc;
    const int wpb = 8;
    rc = launch(k_topk, dim3((B + wpb - 1) / wpb), dim3(32 * wpb), (size_t)wpb * kMaxE * 4, s,
                (const float*)h->ws.logits, B, E, k, h->norm, h->ws);
    if (rc) return rc;
    const int T = 1024;
    const size_t dsm = (size_t)dispatch_smem_ints(E, T / 32) * 4;
    return launch(k_dispatch, dim3(1), dim3(T), dsm, s, B, k, E, h->ws);
}

// Routing only, into buffers the caller chooses: k_router (no fused tail)
// then k_topk. ws.logits ([B, E] fp32 scratch), ws.top / ws.tw (the outputs)
// and ws.err are the only workspace fields these two kernels touch.
int jl_router_topk_prepare() {
    JL_CUDA(cudaFuncSetAttribute(jl::k_router, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
    return JL_OK;
}

int jl_launch_router_topk(const jl_ws& ws, const unsigned short* gate_w, const float* x, int B, int E,
                          int d, int k, int norm, cudaStream_t s) {
    using namespace jl;
    if (E > kMaxE || k > kMaxK || k < 1 || E < k || B < 1 || d < 8 || d % 8) return JL_ERR_INVALID;
    const int TB = kRouteTB;
    const size_t smem = (size_t)kRouteEPB * (d * 2 + 16) + (size_t)TB * d * 4;
    if (smem > 220 * 1024) return JL_ERR_INVALID;
    dim3 grid((E + kRouteEPB - 1) / kRouteEPB, (B + TB - 1) / TB);
    int rc = launch(k_router, grid, dim3(32 * TB), smem, s, gate_w, x, B, E, d, k, norm, ws, 0);
    if (rc) return rc;
    const int wpb = 8;
    return launch(k_topk, dim3((B + wpb - 1) / wpb), dim3(32 * wpb), (size_t)wpb * kMaxE * 4, s,
                  (const float*)ws.logits, B, E, k, norm, ws);
}
