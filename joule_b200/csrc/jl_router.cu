// Router: logits (bit-exact with the reference), softmax / top-k / renorm,
// and the token-to-expert dispatch (union of experts + slot map).
#include <climits>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

constexpr int kRouteEPB = 4;      // experts per router block
constexpr int kRouteTB = 8;       // tokens per router block (one warp each)
constexpr int kFuseTailMaxB = 8;  // B up to which the last router block routes + dispatches
constexpr int kMaxK = 16;         // top-k capacity (the reference caps topk at 16, ws_init)
constexpr int kMaxE = 256;

// ---------------------------------------------------------------------------
// Per-token softmax / top-k / renorm by one warp (decode_kernel.c:1425-1448).
// `p_s` is E floats of shared memory private to this warp.
__device__ void route_token_warp(const float* logits_b, int E, int k, int norm, int* top_b,
                                 float* tw_b, float* p_s) {
    const int lane = threadIdx.x & 31;
    constexpr int EPL = kMaxE / 32;
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; i++) {
        const int e = lane + 32 * i;
        v[i] = (e < E) ? __ldcg(logits_b + e) : 0.0f;
    }
    // smax: the reference scans with strict '>' from -1e30
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
        if (e < E) p_s[e] = p[i];
    }
    __syncwarp();
    // the sum runs sequentially in expert order
    float sum = 0.0f;
    if (lane == 0)
        for (int e = 0; e < E; e++) sum = __fadd_rn(sum, p_s[e]);
    sum = __shfl_sync(0xffffffffu, sum, 0);
#pragma unroll
    for (int i = 0; i < EPL; i++) p[i] = __fdiv_rn(p[i], sum);
    // k passes of argmax over unused experts, ties -> lowest index
    uint32_t used = 0;
    float wsel[kMaxK];
    int esel[kMaxK];
    for (int it = 0; it < k; it++) {
        float bv = -1e30f;
        int be = -1;
#pragma unroll
        for (int i = 0; i < EPL; i++) {
            const int e = lane + 32 * i;
            if (e < E && !((used >> i) & 1u) && p[i] > bv) {
                bv = p[i];
                be = e;
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ov > bv || (ov == bv && oe >= 0 && (be < 0 || oe < be))) {
                bv = ov;
                be = oe;
            }
        }
        if (be >= 0 && (be & 31) == lane) used |= 1u << (be >> 5);
        wsel[it] = bv;
        esel[it] = be;
    }
    if (lane == 0) {
        if (norm) {
            float ssum = 0.0f;
            for (int it = 0; it < k; it++) ssum = __fadd_rn(ssum, wsel[it]);
            for (int it = 0; it < k; it++) wsel[it] = __fdiv_rn(wsel[it], ssum);
        }
        for (int it = 0; it < k; it++) {
            top_b[it] = esel[it];
            tw_b[it] = wsel[it];
        }
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// Dispatch by one block (decode_kernel.c:1449-1485, same outputs):
//   sel[u]      experts in first-appearance order over the slots s = b*k + i
//   uh[u]       exclusive prefix of per-expert slot counts, uh[U] = B*k
//   uidx/uw     slots grouped by union position, increasing slot order inside
//   slot_pos[s] index of slot s in uidx
//   comb[b*k+j] token b's slots ordered by the union position of their expert
// Each warp owns a contiguous slot range; ranks inside an expert come from a
// per-warp count prefix plus __match_any_sync within 32-slot chunks, so the
// cost is O(B*k / threads + E^2 / threads).
__host__ __device__ inline int dispatch_smem_ints(int E, int W) { return 6 * E + W * E + 2; }

__device__ void dispatch_block(const int* top, const float* tw, int B, int k, int E,
                               const jl_ws& ws, int* sm) {
    const int S = B * k;
    const int T = blockDim.x, tid = threadIdx.x, W = T >> 5, warp = tid >> 5, lane = tid & 31;
    int* first = sm;            // [E]
    int* cnt = first + E;       // [E]
    int* upos = cnt + E;        // [E]
    int* base = upos + E;       // [E]
    int* ucnt = base + E;       // [E] count by union position
    int* ustart = ucnt + E;     // [E]
    int* wrun = ustart + E;     // [W, E]
    int* Ush = wrun + W * E;    // [1]
    for (int e = tid; e < E; e += T) {
        first[e] = INT_MAX;
        cnt[e] = 0;
    }
    for (int i = tid; i < W * E; i += T) wrun[i] = 0;
    if (tid == 0) *Ush = 0;
    __syncthreads();
    const int per = (S + W - 1) / W;
    const int s_lo = min(S, warp * per), s_hi = min(S, s_lo + per);
    for (int s = s_lo + lane; s < s_hi; s += 32) {
        int e = top[s];
        if (e < 0 || e >= E) {
            atomicOr(ws.err, kErrBadExpert);
            e = 0;
        }
        atomicMin(&first[e], s);
        atomicAdd(&cnt[e], 1);
        atomicAdd(&wrun[warp * E + e], 1);
    }
    __syncthreads();
    for (int e = tid; e < E; e += T) {
        int r = -1;
        if (first[e] != INT_MAX) {
            r = 0;
            const int f = first[e];
            for (int e2 = 0; e2 < E; e2++) r += (first[e2] < f);
            atomicAdd(Ush, 1);
        }
        upos[e] = r;
        int run = 0;
        for (int w = 0; w < W; w++) {
            const int c = wrun[w * E + e];
            wrun[w * E + e] = run;
            run += c;
        }
    }
    __syncthreads();
    for (int e = tid; e < E; e += T)
        if (upos[e] >= 0) {
            ws.sel[upos[e]] = e;
            ucnt[upos[e]] = cnt[e];
        }
    __syncthreads();
    const int U = *Ush;
    if (tid == 0) {
        int acc = 0;
        for (int u = 0; u < U; u++) {
            ustart[u] = acc;
            ws.uh[u] = acc;
            acc += ucnt[u];
        }
        ws.uh[U] = acc;
        *ws.U = U;
    }
    __syncthreads();
    for (int e = tid; e < E; e += T) base[e] = (upos[e] >= 0) ? ustart[upos[e]] : 0;
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
    for (int c0 = s_lo; c0 < s_hi; c0 += 32) {
        const int s = c0 + lane;
        const bool valid = s < s_hi;
        int e = valid ? top[s] : -1 - lane;
        if (valid && (e < 0 || e >= E)) e = 0;
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
            int e = top[b * k + i];
            if (e < 0 || e >= E) e = 0;
            const int u = upos[e];
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
// expert, lane j); 4 experts x up to 8 tokens per block, staged in shared
// memory. With `fuse_tail`, the last block to finish also routes every token
// and builds the dispatch (B <= kFuseTailMaxB).
__global__ void k_router(const uint16_t* __restrict__ gate_w, const float* __restrict__ x, int B,
                         int E, int d, int k, int norm, jl_ws ws, int fuse_tail) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int tid = threadIdx.x, TB = blockDim.x >> 5;
    const int e0 = blockIdx.x * kRouteEPB, b0 = blockIdx.y * TB;
    const int nb = min(TB, B - b0);
    const int grow = d * 2 + 16;  // padded gate row (bytes): conflict-free lane reads
    uint8_t* g_s = smem;
    float* x_s = reinterpret_cast<float*>(smem + kRouteEPB * grow);
    griddep_wait();
    const int c8 = d / 8;
    for (int i = tid; i < kRouteEPB * c8; i += blockDim.x) {
        const int r = i / c8, c = i % c8, e = e0 + r;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (e < E) v = __ldg(reinterpret_cast<const uint4*>(gate_w + (size_t)e * d) + c);
        *reinterpret_cast<uint4*>(g_s + r * grow + c * 16) = v;
    }
    for (int i = tid; i < nb * d / 4; i += blockDim.x)
        reinterpret_cast<float4*>(x_s)[i] = reinterpret_cast<const float4*>(x + (size_t)b0 * d)[i];
    __syncthreads();
    const int tb = tid >> 5, ee = (tid >> 3) & 3, j = tid & 7;
    const bool live = tb < nb && e0 + ee < E;
    float acc = 0.0f;
    if (live) {
        const uint16_t* gr = reinterpret_cast<const uint16_t*>(g_s + ee * grow) + j;
        const float* xr = x_s + tb * d + j;
#pragma unroll 8
        for (int t = 0; t < c8; t++) acc = __fmaf_rn(bf16_to_f32(gr[8 * t]), xr[8 * t], acc);
    }
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
    if (live && j == 0) ws.logits[(size_t)(b0 + tb) * E + e0 + ee] = acc;
    if (!fuse_tail) return;

    __shared__ int is_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = (atomicAdd(ws.counter, 1) == (int)(gridDim.x * gridDim.y) - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (tid == 0) *ws.counter = 0;
    float* p_s = reinterpret_cast<float*>(smem);  // [TB, E]; staging no longer needed
    for (int b = tb; b < B; b += TB)
        route_token_warp(ws.logits + (size_t)b * E, E, k, norm, ws.top + b * k, ws.tw + b * k,
                         p_s + tb * E);
    __syncthreads();
    dispatch_block(ws.top, ws.tw, B, k, E, ws, reinterpret_cast<int*>(smem) + TB * E);
}

__global__ void k_topk(const float* __restrict__ logits, int B, int E, int k, int norm,
                       jl_ws ws) {
    extern __shared__ __align__(16) float p_all[];
    griddep_wait();
    const int warp = threadIdx.x >> 5;
    const int b = blockIdx.x * (blockDim.x >> 5) + warp;
    if (b >= B) return;
    route_token_warp(logits + (size_t)b * E, E, k, norm, ws.top + b * k, ws.tw + b * k,
                     p_all + warp * E);
}

__global__ void k_dispatch(int B, int k, int E, jl_ws ws) {
    extern __shared__ __align__(16) int dsm[];
    griddep_wait();
    dispatch_block(ws.top, ws.tw, B, k, E, ws, dsm);
}

}  // namespace jl

int jl_launch_route(const jl_moe* h, const unsigned short* gate_w_l, const float* x, int B,
                    cudaStream_t s) {
    using namespace jl;
    const int E = h->E, d = h->d, k = h->k;
    if (E > kMaxE || k > kMaxK || k < 1 || E < k) return JL_ERR_INVALID;
    const int TB = B < kRouteTB ? B : kRouteTB;
    const bool fuse = B <= kFuseTailMaxB;
    const int threads = 32 * TB;
    size_t smem = (size_t)kRouteEPB * (d * 2 + 16) + (size_t)TB * d * 4;
    if (fuse) {
        const size_t tail = ((size_t)TB * E + dispatch_smem_ints(E, TB)) * 4;
        if (tail > smem) smem = tail;
    }
    static bool attr = false;
    if (!attr) {
        JL_CUDA(cudaFuncSetAttribute(k_router, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        JL_CUDA(cudaFuncSetAttribute(k_dispatch, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr = true;
    }
    if (smem > 200 * 1024) return JL_ERR_INVALID;
    dim3 grid((E + kRouteEPB - 1) / kRouteEPB, (B + TB - 1) / TB);
    k_router<<<grid, threads, smem, s>>>(gate_w_l, x, B, E, d, k, h->norm, h->ws, fuse ? 1 : 0);
    JL_LAUNCH_CHECK();
    if (!fuse) {
        const int wpb = 8;
        k_topk<<<(B + wpb - 1) / wpb, 32 * wpb, (size_t)wpb * E * 4, s>>>(h->ws.logits, B, E, k,
                                                                          h->norm, h->ws);
        JL_LAUNCH_CHECK();
        const int T = 1024;
        const size_t dsm = (size_t)dispatch_smem_ints(E, T / 32) * 4;
        k_dispatch<<<1, T, dsm, s>>>(B, k, E, h->ws);
        JL_LAUNCH_CHECK();
    }
    return JL_OK;
}
