// Router: logits (bit-exact with the reference), softmax / top-k / renorm,
// and the token-to-expert dispatch (union of experts + slot map).
#include <climits>

#include <cooperative_groups.h>

#include "jl_common.cuh"
#include "jl_internal.h"
#include "jl_route.cuh"
#include "jl_tiles.cuh"

#include <algorithm>

namespace jl {

constexpr int kRouteEPB = 4;      // experts per router block
constexpr int kRouteTB = 8;       // tokens per router block (one warp each)

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
// Dispatch by one block (decode_kernel.c:1449-1485, same outputs). A slot
// whose expert id is -1 is padding: it takes no place in the union or the
// slot map (batches received by expert parallelism are padded).
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


__device__ __forceinline__ void dispatch_block(const int* top, const float* tw, int B, int k, int E,
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
        if (e0 == -1) continue;  // padding slot (expert-parallel receive batches)
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
        const bool valid = s < s_hi && top[s] != -1;
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
    for (int s = tid; s < S; s += T) comb_slot(top, upos, s, k, E, ws.comb);
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
// Router on 8-CTA thread-block clusters, one cluster per group of TPC tokens
// (TPC = route_tpc(B), so up to 32 clusters run at once). CTA r of a cluster
// stages router rows [r*EPC, (r+1)*EPC) by bulk copies issued before waiting
// on the previous kernel (they do not depend on it), then the cluster's token
// rows; it computes their logits in the reference's order (8 lane chains of
// FMAs in k order plus the AVX tree) and stores them into the leader CTA's
// shared memory over DSMEM. After the cluster barrier the leader routes its
// tokens. The last leader to finish (a global arrival counter) builds the
// dispatch for all B tokens and the tensor-core tile table.
constexpr int kClusterCTAs = 8;
constexpr int kClusterThreads = 256;
constexpr int kMaxTPC = 8;

__host__ __device__ inline int route_tpc(int B) {  // tokens per cluster: 1, 2, 4 or 8
    const int t = (B + 31) / 32;
    return t <= 1 ? 1 : t <= 2 ? 2 : t <= 4 ? 4 : kMaxTPC;
}

__host__ __device__ inline int dispatch_smem_bytes(int B, int k, int E) {
    return B * k * 8 + dispatch_smem_ints(E, kClusterThreads / 32) * 4;
}

__global__ void __cluster_dims__(kClusterCTAs, 1, 1) __launch_bounds__(kClusterThreads)
    k_router_cluster(const uint16_t* __restrict__ gate_w, const float* __restrict__ x, int B, int E,
                     int d, int k, int norm, jl_ws ws, int tpc, int lg_off, int fuse_dispatch,
                     int tiles) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int is_last;
    const int tid = threadIdx.x;
    const int rank = (int)cluster.block_rank();
    const int nclusters = gridDim.x / kClusterCTAs;
    const int cl = blockIdx.x / kClusterCTAs;
    const int b0 = cl * tpc, nb = min(tpc, B - b0);
    const int EPC = (E + kClusterCTAs - 1) / kClusterCTAs;
    const int e0 = rank * EPC, ne = max(0, min(EPC, E - e0));
    const int gs = router_gstride(d), xs = router_xstride(d);
    uint16_t* g_s = reinterpret_cast<uint16_t*>(smem);                         // [EPC * 8][gs]
    float* x_s = reinterpret_cast<float*>(smem + (size_t)EPC * 8 * gs * 2);   // [tpc * 8][xs]
    float* lg_s = reinterpret_cast<float*>(smem + lg_off);  // [tpc, E] logits (the leader's are read)
    long long* tr = (blockIdx.x == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceRouter, 0);
    if (tid == 0) {  // router rows do not depend on the previous kernel: fetch them first
        mbar_init(&bar, 1);
        mbar_fence_init();
        if (ne > 0) {
            const uint32_t bytes = (uint32_t)(ne * router_expert_halves(d) * 2);
            mbar_expect_tx(&bar, bytes);
            bulk_g2s_hint(g_s, gate_w + (size_t)e0 * router_expert_halves(d), bytes, &bar, l2_policy_evict_last());
        } else {
            mbar_arrive(&bar);
        }
    }
    griddep_wait();  // x is the previous kernel's output
    griddep_launch_dependents();
    trace_point(tr, kTraceRouter, 1);
    // token rows, transposed into lane rows
    for (int q = tid; q < nb * d / 4; q += kClusterThreads) {
        const int tb = q / (d / 4), i = (q % (d / 4)) * 4;
        const float4 v = *reinterpret_cast<const float4*>(x + (size_t)(b0 + tb) * d + i);
        float* row = x_s + (size_t)(tb * 8 + (i & 7)) * xs + (i >> 3);
        row[0] = v.x;
        row[xs] = v.y;
        row[2 * xs] = v.z;
        row[3 * xs] = v.w;
    }
    __syncthreads();
    const bool ok = mbar_wait_bounded(&bar, 0, ws.err);
    trace_point(tr, kTraceRouter, 2);
    float* lg_lead = cluster.map_shared_rank(lg_s, 0);
    if (ok && ne > 0) {
        if (tpc == 1) cluster_logits<1>(g_s, x_s, d, nb, E, e0, ne, b0, lg_lead, ws.logits);
        else if (tpc == 2) cluster_logits<2>(g_s, x_s, d, nb, E, e0, ne, b0, lg_lead, ws.logits);
        else if (tpc == 4) cluster_logits<4>(g_s, x_s, d, nb, E, e0, ne, b0, lg_lead, ws.logits);
        else cluster_logits<8>(g_s, x_s, d, nb, E, e0, ne, b0, lg_lead, ws.logits);
    }
    trace_point(tr, kTraceRouter, 3);
    cluster.sync();
    if (rank != 0) return;
    trace_point(tr, kTraceRouter, 4);
    // leader: the staging area is free; routing scratch, then dispatch scratch
    if ((int)(threadIdx.x >> 5) < nb) {  // one warp per token
        const int w = threadIdx.x >> 5;
        route_token_lean(lg_s + (size_t)w * E, E, k, norm, ws.top + (b0 + w) * k, ws.tw + (b0 + w) * k,
                         reinterpret_cast<float*>(smem) + w * kMaxE);
    }
    __syncthreads();
    trace_point(tr, kTraceRouter, 5);
    if (!fuse_dispatch) return;  // k_dispatch follows
    if (nclusters > 1) {
        if (tid == 0) {
            __threadfence();
            is_last = atomicAdd(ws.counter, 1) == nclusters - 1;
        }
        __syncthreads();
        if (!is_last) return;
        __threadfence();
        if (tid == 0) *ws.counter = 0;
        tr = ws.trace;  // the last leader stamps the dispatch
    }
    trace_point(tr, kTraceRouter, 6);
    // every token's ids and weights, read through L2 (other clusters wrote them)
    const int S = B * k;
    if (B == 1) {  // this CTA routed the only token (its stores are visible after the barrier)
        trace_point(tr, kTraceRouter, 7);
        if (tid < k) {
            ws.sel[tid] = ws.top[tid];
            ws.uh[tid] = tid;
            ws.uidx[tid] = tid;
            ws.uw[tid] = ws.tw[tid];
            ws.slot_pos[tid] = tid;
            ws.comb[tid] = tid;
        }
        if (tid == 0) {
            ws.uh[k] = k;
            *ws.U = k;
        }
        trace_point(tr, kTraceRouter, 8);
        if (tiles) {
            __syncthreads();
            if (tid < 32) tc_build_tiles(ws);
            trace_point(tr, kTraceRouter, 9);
        }
        return;
    }
    int* top_s = reinterpret_cast<int*>(smem);
    float* tw_s = reinterpret_cast<float*>(top_s + S);
    int* dsm = reinterpret_cast<int*>(tw_s + S);
    for (int i = tid; i < S; i += kClusterThreads) {
        top_s[i] = __ldcg(ws.top + i);
        tw_s[i] = __ldcg(ws.tw + i);
    }
    __syncthreads();
    trace_point(tr, kTraceRouter, 7);
    if (B == 1) {
        if (tid < k) {
            ws.sel[tid] = top_s[tid];
            ws.uh[tid] = tid;
            ws.uidx[tid] = tid;
            ws.uw[tid] = tw_s[tid];
            ws.slot_pos[tid] = tid;
            ws.comb[tid] = tid;
        }
        if (tid == 0) {
            ws.uh[k] = k;
            *ws.U = k;
        }
    } else if (S <= 128 && B <= 32) {
        if (tid < 32) dispatch_warp_small(top_s, tw_s, B, k, E, ws, dsm);
    } else {
        dispatch_block(top_s, tw_s, B, k, E, ws, dsm);
    }
    trace_point(tr, kTraceRouter, 8);
    if (tiles) {
        __syncthreads();
        if (tid < 32) tc_build_tiles(ws);
        trace_point(tr, kTraceRouter, 9);
    }
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

__global__ void k_dispatch(int B, int k, int E, jl_ws ws, int stage) {
    extern __shared__ __align__(16) int dsm[];
    trace_point(ws.trace, kTraceRouter, 10);
    griddep_wait();
    griddep_launch_dependents();
    trace_point(ws.trace, kTraceRouter, 11);
    if (stage) {  // the routing in shared memory: the dispatch reads each slot several times
        const int S = B * k;
        int* top_s = dsm;
        float* tw_s = reinterpret_cast<float*>(top_s + S);
        for (int i = threadIdx.x; i < S; i += blockDim.x) {
            top_s[i] = __ldcg(ws.top + i);
            tw_s[i] = __ldcg(ws.tw + i);
        }
        __syncthreads();
        dispatch_block(top_s, tw_s, B, k, E, ws, reinterpret_cast<int*>(tw_s + S));
    } else {
        dispatch_block(ws.top, ws.tw, B, k, E, ws, dsm);
    }
    trace_point(ws.trace, kTraceRouter, 12);
    __syncthreads();
    if (threadIdx.x < 32) tc_build_tiles(ws);
    trace_point(ws.trace, kTraceRouter, 13);
}

// ---------------------------------------------------------------------------
// Dispatch of router output (every token's k experts distinct) by one block
// in a few barrier-separated steps, same outputs as dispatch_block plus the
// tensor-core tile table (tc_build_tiles):
//   1. per slot: first slot and slot count of its expert (shared atomics),
//      and the token's bit in its expert's token mask
//   2. per expert with slots: its first slot's bit in a slot mask; per
//      expert, prefix popcounts of its token mask words
//   3. prefix popcounts of the slot mask words: a union position is the
//      number of experts whose first slot comes earlier (first appearance)
//   4. one block scan over union positions of (slots, tiles, padded rows)
//   5. per slot: its rank inside its expert = earlier tokens that chose the
//      same expert (slot order, since each token holds an expert at most once)
constexpr int kDfThreads = 512;

__host__ __device__ inline size_t dispatch_fast_smem(int B, int k, int E) {
    const size_t S = (size_t)B * k, NW = (B + 31) / 32, NF = (S + 31) / 32;
    return (2 * S + 5 * (size_t)E + 2 * NF + 2 * (size_t)E * NW + 3 * 32 + 4) * 4;
}

__global__ void __launch_bounds__(kDfThreads) k_dispatch_fast(int B, int k, int E, jl_ws ws) {
    extern __shared__ __align__(16) int sm[];
    trace_point(ws.trace, kTraceRouter, 10);
    griddep_wait();
    griddep_launch_dependents();
    trace_point(ws.trace, kTraceRouter, 11);
    const int S = B * k, NW = (B + 31) >> 5, NF = (S + 31) >> 5;
    const int T = blockDim.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int* top = sm;
    float* tw = reinterpret_cast<float*>(top + S);
    int* first = reinterpret_cast<int*>(tw + S);
    int* cnt = first + E;
    int* upos = cnt + E;
    int* sel = upos + E;
    int* ustart = sel + E;
    unsigned* fflag = reinterpret_cast<unsigned*>(ustart + E);
    int* fpre = reinterpret_cast<int*>(fflag + NF);
    unsigned* tmask = reinterpret_cast<unsigned*>(fpre + NF);
    int* tpre = reinterpret_cast<int*>(tmask + (size_t)E * NW);
    int* wsum = tpre + (size_t)E * NW;  // [3][32]
    int* misc = wsum + 96;
    for (int i = tid; i < S; i += T) {
        top[i] = __ldcg(ws.top + i);
        tw[i] = __ldcg(ws.tw + i);
    }
    for (int e = tid; e < E; e += T) {
        first[e] = INT_MAX;
        cnt[e] = 0;
    }
    for (int i = tid; i < NF; i += T) fflag[i] = 0u;
    for (int i = tid; i < E * NW; i += T) tmask[i] = 0u;
    __syncthreads();
    for (int s = tid; s < S; s += T) {
        int e = top[s];
        if (e < 0 || e >= E) {
            atomicOr(ws.err, kErrBadExpert);
            e = 0;
            top[s] = 0;
        }
        const int b = s / k;
        atomicMin(&first[e], s);
        atomicAdd(&cnt[e], 1);
        atomicOr(&tmask[e * NW + (b >> 5)], 1u << (b & 31));
    }
    __syncthreads();
    for (int e = tid; e < E; e += T) {
        if (cnt[e] > 0) atomicOr(&fflag[first[e] >> 5], 1u << (first[e] & 31));
        int run = 0;
        for (int w = 0; w < NW; w++) {
            tpre[e * NW + w] = run;
            run += __popc(tmask[e * NW + w]);
        }
    }
    __syncthreads();
    if (warp == 0) {
        int run = 0;
        for (int w0 = 0; w0 < NF; w0 += 32) {
            const int w = w0 + lane;
            const int c = w < NF ? __popc(fflag[w]) : 0;
            int inc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += a;
            }
            if (w < NF) fpre[w] = run + inc - c;
            run += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) misc[0] = run;
    }
    __syncthreads();
    const int U = misc[0];
    for (int e = tid; e < E; e += T) {
        if (cnt[e] > 0) {
            const int f = first[e];
            const int u = fpre[f >> 5] + __popc(fflag[f >> 5] & ((1u << (f & 31)) - 1u));
            upos[e] = u;
            sel[u] = e;
            ws.sel[u] = e;
        } else {
            upos[e] = -1;
        }
    }
    __syncthreads();
    // union-order scans (U <= E <= 256: warps 0..7 hold one position each)
    {
        const int u = tid;
        int n = 0, t = 0, r = 0;
        if (u < U) {
            n = cnt[sel[u]];
            t = (n + kTcNT - 1) / kTcNT;
            r = tc_rows(n);
        }
        int ni = n, ti = t, ri = r;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, ni, o);
            const int b2 = __shfl_up_sync(0xffffffffu, ti, o);
            const int c2 = __shfl_up_sync(0xffffffffu, ri, o);
            if (lane >= o) {
                ni += a;
                ti += b2;
                ri += c2;
            }
        }
        if (warp < 8 && lane == 31) {
            wsum[warp] = ni;
            wsum[32 + warp] = ti;
            wsum[64 + warp] = ri;
        }
        __syncthreads();
        if (warp == 0) {
#pragma unroll
            for (int q = 0; q < 3; q++) {
                const int v = lane < 8 ? wsum[32 * q + lane] : 0;
                int inc = v;
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    const int a = __shfl_up_sync(0xffffffffu, inc, o);
                    if (lane >= o) inc += a;
                }
                if (lane < 8) wsum[32 * q + lane] = inc - v;
                if (lane == 7) misc[1 + q] = inc;
            }
        }
        __syncthreads();
        if (u < U) {
            const int nex = wsum[warp] + ni - n, tex = wsum[32 + warp] + ti - t, rex = wsum[64 + warp] + ri - r;
            ustart[u] = nex;
            ws.uh[u] = nex;
            const int e = sel[u];
            for (int j = 0; j < t; j++) {
                int* tt = ws.tc_tile + (size_t)(tex + j) * 4;
                tt[0] = e;
                tt[1] = min(kTcNT, n - j * kTcNT);
                tt[2] = nex + j * kTcNT;
                tt[3] = rex + j * kTcNT;
            }
        }
        if (tid == 0) {
            ws.uh[U] = misc[1];
            *ws.U = U;
            *ws.tc_ntiles = misc[2];
        }
    }
    __syncthreads();
    for (int s = tid; s < S; s += T) {
        const int e = top[s], b = s / k, w = b >> 5;
        const int rank = tpre[e * NW + w] + __popc(tmask[e * NW + w] & ((1u << (b & 31)) - 1u));
        const int pos = ustart[upos[e]] + rank;
        ws.uidx[pos] = s;
        ws.uw[pos] = tw[s];
        ws.slot_pos[s] = pos;
        comb_slot(top, upos, s, k, E, ws.comb);
    }
    trace_point(ws.trace, kTraceRouter, 13);
}

}  // namespace jl

// k_dispatch with the routing staged in shared memory when it fits.
static int launch_dispatch(const jl_ws& ws, int B, int k, int E, cudaStream_t s) {
    using namespace jl;
    const int T = 1024;
    const size_t base = (size_t)dispatch_smem_ints(E, T / 32) * 4, staged = base + (size_t)B * k * 8;
    const int stage = staged <= 220 * 1024;
    return launch(k_dispatch, dim3(1), dim3(T), stage ? staged : base, s, B, k, E, ws, stage);
}

int jl_launch_route(const jl_moe* h, const unsigned short* gate_w_l, const float* x, int B,
                    bool tiles, cudaStream_t s) {
    using namespace jl;
    const int E = h->E, d = h->d, k = h->k;
    if (E > kMaxE || k > kMaxK || k < 1 || E < k) return JL_ERR_INVALID;
    int rc0 = jl_device_once(kOnceRouter, [] {
        JL_CUDA(cudaFuncSetAttribute(jl::k_dispatch, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        JL_CUDA(cudaFuncSetAttribute(jl::k_router_cluster, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        return JL_OK;
    });
    if (rc0) return rc0;
    if (d % 128) return JL_ERR_INVALID;
    const int tpc = route_tpc(B);
    const int ncl = (B + tpc - 1) / tpc;
    const int EPC = (E + kClusterCTAs - 1) / kClusterCTAs;
    const size_t stage = (size_t)EPC * 8 * router_gstride(d) * 2 + (size_t)tpc * 8 * router_xstride(d) * 4;
    // the dispatch runs in the last leader when its scratch fits, else in k_dispatch
    const size_t dsp = (size_t)dispatch_smem_bytes(B, k, E);
    const int fuse = dsp <= 64 * 1024 && B <= 32;
    const size_t tail = std::max((size_t)kMaxTPC * kMaxE * 4, fuse ? dsp : (size_t)0);
    const size_t lg_off = (std::max(stage, tail) + 127) / 128 * 128;
    const size_t smem = lg_off + (size_t)tpc * E * 4;
    if (smem > 220 * 1024) return JL_ERR_INVALID;
    int rc = launch(k_router_cluster, dim3(kClusterCTAs * ncl), dim3(kClusterThreads), smem, s, gate_w_l,
                    x, B, E, d, k, h->norm, h->ws, tpc, (int)lg_off, fuse, tiles ? 1 : 0);
    if (rc || fuse) return rc;
    const size_t fsm = dispatch_fast_smem(B, k, E);
    if (fsm <= 200 * 1024) {
        rc = jl_device_once(kOnceRouterFast, [] {
            JL_CUDA(cudaFuncSetAttribute(jl::k_dispatch_fast, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
            return JL_OK;
        });
        if (rc) return rc;
        return launch(k_dispatch_fast, dim3(1), dim3(kDfThreads), fsm, s, B, k, E, h->ws);
    }
    return launch_dispatch(h->ws, B, k, E, s);
}

int jl_launch_dispatch(const jl_moe* h, int B, cudaStream_t s) {
    using namespace jl;
    if (h->E > kMaxE || h->k > kMaxK) return JL_ERR_INVALID;
    const int rc = jl_device_once(kOnceDispatch, [] {
        JL_CUDA(cudaFuncSetAttribute(jl::k_dispatch, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        return JL_OK;
    });
    if (rc) return rc;
    return launch_dispatch(h->ws, B, h->k, h->E, s);
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
