// Single-launch MoE layer for small batches (B <= 8): router logits, softmax /
// top-k / renorm, dispatch, gate/up + SwiGLU, down and combine in ONE
// persistent grid of one CTA per SM, in the reference's FP32 arithmetic order
// (layer_ffn_batch, decode_kernel.c:1387-1508), so the output is
// bit-identical to the reference's and to the three-kernel exact path.
//
// At decode batch sizes a layer moves tens of MB and its phases depend on one
// another (the router picks which expert rows the FFN reads). As separate
// kernels each phase pays a launch, a ramp-up and a tail; here the phases
// hand over through counters in global memory instead:
//   1. CTA c (< E) computes the logits of experts c, c + G, ... for all B
//      tokens; its router rows are fetched before the dependent-grid wait.
//      Each router CTA bumps an arrival counter; every CTA waits (bounded)
//      for all of them, then routes all B tokens and builds the dispatch in
//      its own shared memory (the same deterministic result in every CTA).
//   2. Work units: gate/up unit (u, mt) = 64 gate + 64 up rows of union
//      expert u; down unit (u, mt) = 128 down rows. The grid splits into
//      gate/up CTAs and down CTAs in proportion to the bytes of the two
//      matrices; each walks its units with stride (so experts finish in
//      order) and streams their tile records through a shared-memory ring
//      of 17 KB bulk copies issued by a producer warp that runs ahead across
//      units. Down CTAs prefetch their weights while they wait for the
//      activations of their expert (a per-expert counter of finished gate/up
//      units).
//   3. Each down unit bumps a counter of its 128-row block; the CTA that
//      completes a block's last expert sums y over the union in the
//      reference's order (combine) for those rows of every token.
// The last CTA to leave resets the counters for the next launch.
//
// Products are computed per (row, 64-value group) exactly as the reference's
// q4_row_dot_B does (8 lane chains of FMAs, AVX reduction tree, times the
// scale), spread over all 16 compute warps, and the per-row chain over groups
// (one add per group, in group order) advances chunk by chunk.
//
// Every wait is bounded (~2 s of SM clock); a timeout sets the handle's
// error word and an abort flag after which the CTA skips the rest of its
// work (still executing the same barrier sequence) and leaves once its bulk
// copies have landed.
#include <algorithm>
#include <mutex>

#include "jl_common.cuh"
#include "jl_internal.h"
#include "jl_route.cuh"

namespace jl {

constexpr int kFWarps = 16;                        // compute warps
constexpr int kFThreads = (kFWarps + 1) * 32;      // + one producer warp
constexpr int kFChunkGroups = 4;                   // groups per bulk copy
constexpr int kFChunkBytes = kFChunkGroups * 4 * kTileRec;  // 17,408 B: 4 records per group
constexpr int kFMaxStages = 16;
constexpr int kFMaxB = 8;
constexpr int kFMaxS = kFMaxB * kMaxK;             // slots
constexpr int kFBar = 15;                          // named barrier of the compute warps
// fsync words: [0] router arrivals, [1] CTA exits, [8, 8 + E) finished
// gate/up units per union expert, [8 + kMaxE, ...) finished down units per
// 128-row block
constexpr int kFSyncLg = 0, kFSyncExit = 1, kFSyncGu = 8, kFSyncRb = 8 + kMaxE;
static_assert(kMaxE == 256, "fsync layout (jl_internal.h)");

struct FShared {
    uint64_t full[kFMaxStages], empty[kFMaxStages];
    uint64_t rbar;
    int abort;
    int U;
    int last;
    int xoff[kFMaxB];  // per token of the current unit: float offset of its input row
    int top[kFMaxS];
    float tw[kFMaxS];
    int sel[kMaxE];
    int uh[kMaxE + 1];
    int uidx[kFMaxS];
    float uw[kFMaxS];
    int comb[kFMaxS];
    int slot_pos[kFMaxS];
};

// Shared-memory plan of one launch (host-computed; byte offsets into the
// dynamic shared memory).
struct FPlan {
    int S;         // ring stages
    int xs;        // x row stride (floats)
    int ps_off, ups_off, ring_off;
    int xt_off, lg_off, rs_off, ds_off;  // routing scratch inside the ring (before the ring is used)
};

__device__ __forceinline__ void named_barrier(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *p >= target (acquire), giving up when the CTA aborted.
__device__ __noinline__ bool f_wait_count(const int* p, int target, int* err, volatile int* abort) {
    if (ld_acquire_gpu(p) >= target) return true;
    const long long t0 = clock64();
    for (int i = 1;; i++) {
        if (ld_acquire_gpu(p) >= target) return true;
        if ((i & 15) == 0) {
            if (*abort) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                atomicOr(err, kErrTimeout);
                *abort = 1;
                return false;
            }
        }
    }
}

// Bounded mbarrier wait that also gives up when the CTA aborted.
__device__ __forceinline__ bool f_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (int i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*abort) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                atomicOr(err, kErrTimeout);
                *abort = 1;
                return false;
            }
        }
    }
}

// p = hsum8(8 lane chains) * s for NT token rows of one tile row (lane =
// row): the same operations, in the same order, as tile_row_products and the
// reference's q4_row_dot_B group step. xr[t] + off = the group's first input.
template <int NT>
__device__ __forceinline__ void rec_products(const uint32_t (&wq)[8], float s, const float* const* xr,
                                             int off, float (&p)[NT]) {
    float2 acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[t][j] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int w = 0; w < 8; w++) {
        float2 a[4];
        dequant8x2(wq[w], a);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float4 x0 = *reinterpret_cast<const float4*>(xr[t] + off + w * 8);
            const float4 x1 = *reinterpret_cast<const float4*>(xr[t] + off + w * 8 + 4);
            acc[t][0] = __ffma2_rn(a[0], make_float2(x0.x, x0.y), acc[t][0]);
            acc[t][1] = __ffma2_rn(a[1], make_float2(x0.z, x0.w), acc[t][1]);
            acc[t][2] = __ffma2_rn(a[2], make_float2(x1.x, x1.y), acc[t][2]);
            acc[t][3] = __ffma2_rn(a[3], make_float2(x1.z, x1.w), acc[t][3]);
        }
    }
#pragma unroll
    for (int t = 0; t < NT; t++) p[t] = __fmul_rn(hsum8x2(acc[t]), s);
}

// Products of one tile record (in shared memory) for the n tokens whose input
// rows start at base + xoff[t]; p_t = p_s + t * tstride.
__device__ __forceinline__ void record_products(const uint8_t* tile, const float* base, const int* xoff,
                                                int n, int off, float* pp, int tstride) {
    const int lane = threadIdx.x & 31;
    const uint4 q0 = *reinterpret_cast<const uint4*>(tile + lane * 16);
    const uint4 q1 = *reinterpret_cast<const uint4*>(tile + 512 + lane * 16);
    const float s = half_bits_to_f32(reinterpret_cast<const uint16_t*>(tile + kTileBytes)[lane]);
    const uint32_t wq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    for (int t0 = 0; t0 < n; t0 += 4) {
        const int nt = min(4, n - t0);
        const float* xr[4];
#pragma unroll
        for (int t = 0; t < 4; t++) xr[t] = base + xoff[t0 + (t < nt ? t : 0)];
        float* q = pp + (size_t)t0 * tstride;
        if (nt == 1) {
            float p[1];
            rec_products<1>(wq, s, xr, off, p);
            q[0] = p[0];
        } else if (nt == 2) {
            float p[2];
            rec_products<2>(wq, s, xr, off, p);
            q[0] = p[0];
            q[tstride] = p[1];
        } else if (nt == 3) {
            float p[3];
            rec_products<3>(wq, s, xr, off, p);
#pragma unroll
            for (int t = 0; t < 3; t++) q[t * tstride] = p[t];
        } else {
            float p[4];
            rec_products<4>(wq, s, xr, off, p);
#pragma unroll
            for (int t = 0; t < 4; t++) q[t * tstride] = p[t];
        }
    }
}

// Unit walk of CTA c, identical in every CTA (they all hold the same U):
// gate/up unit i goes to CTA i % G, down unit j to CTA G - 1 - j % G (so the
// CTAs with the fewest gate/up units take the first down units). A CTA runs
// its gate/up units, then its down units; unit list position i < ngu is
// gate/up unit c + i G, else down unit (G - 1 - c) + (i - ngu) G.
struct FWork {
    int ngu, ndn;
};
__device__ __forceinline__ FWork f_work(int U, int G, int c, int MTg, int MTd) {
    const int NGU = U * MTg, ND = U * MTd, cd = G - 1 - c;
    FWork w;
    w.ngu = c < NGU ? (NGU - c + G - 1) / G : 0;
    w.ndn = cd < ND ? (ND - cd + G - 1) / G : 0;
    return w;
}

__global__ void __launch_bounds__(kFThreads, 1)
    k_layer_small(const uint16_t* __restrict__ gate_w_l, const uint8_t* __restrict__ store_l, jl_layout L,
                  int E, int k, int norm, const float* __restrict__ x, int B, float* __restrict__ out,
                  int* __restrict__ top_out, float* __restrict__ tw_out, jl_ws ws, FPlan P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ FShared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int d = L.d, m = L.m;
    const int xs = P.xs;
    float* x_s = reinterpret_cast<float*>(smem);  // [B][xs] token rows; down CTAs: [n][m] act rows
    float* p_s = reinterpret_cast<float*>(smem + P.ps_off);   // [2][B][4][128] group products
    float* up_s = reinterpret_cast<float*>(smem + P.ups_off);  // [B][64] up-row sums
    uint8_t* ring = smem + P.ring_off;
    uint16_t* g_s = reinterpret_cast<uint16_t*>(ring);  // router rows (before the ring is used)
    float* xt_s = reinterpret_cast<float*>(ring + P.xt_off);  // token rows as lane rows (router)
    float* lg_s = reinterpret_cast<float*>(ring + P.lg_off);
    uint8_t* rscr = ring + P.rs_off;
    int* dsm = reinterpret_cast<int*>(ring + P.ds_off);
    int* fs = ws.fsync;
    volatile int* abort = &sh.abort;
    long long* tr = ws.trace == nullptr ? nullptr : c == 0 ? ws.trace : c == G - 1 ? ws.trace + 16 : nullptr;
    trace_point(tr, kTraceRouter, 0);

    const int reh = (int)router_expert_halves(d);
    const int nexp = (c < E) ? (E - 1 - c) / G + 1 : 0;  // router experts c, c + G, ...
    if (tid == 0) {
        sh.abort = 0;
        for (int s = 0; s < P.S; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], kFWarps);
        }
        mbar_init(&sh.rbar, 1);
        mbar_fence_init();
        // router rows do not depend on the previous kernel: fetch them first
        if (nexp > 0) {
            const uint32_t eb = (uint32_t)reh * 2;
            mbar_expect_tx(&sh.rbar, eb * nexp);
            for (int i = 0; i < nexp; i++)
                bulk_g2s_hint(g_s + (size_t)i * reh, gate_w_l + (size_t)(c + i * G) * reh, eb, &sh.rbar,
                              l2_policy_evict_last());
        }
    }
    griddep_wait();  // x is the previous kernel's output
    griddep_launch_dependents();
    trace_point(tr, kTraceRouter, 1);
    {
        // token rows, plain (expert products) and as lane rows: lane row (b, j)
        // holds x[b][j + 8t], t < d/8 (the router's 8 FMA chains)
        const int xr = router_xstride(d);
        for (int q = tid; q < B * (d / 4); q += kFThreads) {
            const int b = q / (d / 4), i = q - b * (d / 4);
            const float4 v = __ldcg(reinterpret_cast<const float4*>(x + (size_t)b * d) + i);
            *reinterpret_cast<float4*>(x_s + (size_t)b * xs + 4 * i) = v;
            float* row = xt_s + (size_t)(b * 8 + ((4 * i) & 7)) * xr + ((4 * i) >> 3);
            row[0] = v.x;
            row[xr] = v.y;
            row[2 * xr] = v.z;
            row[3 * xr] = v.w;
        }
    }
    __syncthreads();

    // ---- 1. logits of this CTA's experts (decode_kernel.c:693-718 order)
    if (nexp > 0 && warp < kFWarps) {
        if (f_wait(&sh.rbar, 0, ws.err, abort)) {
            for (int i = 0; i < nexp; i++) {
                const uint16_t* gi = g_s + (size_t)i * reh;
                const int e0 = c + i * G;
                if (B == 1) cluster_logits<1>(gi, xt_s, d, B, E, e0, 1, 0, nullptr, ws.logits);
                else if (B == 2) cluster_logits<2>(gi, xt_s, d, B, E, e0, 1, 0, nullptr, ws.logits);
                else if (B <= 4) cluster_logits<4>(gi, xt_s, d, B, E, e0, 1, 0, nullptr, ws.logits);
                else cluster_logits<8>(gi, xt_s, d, B, E, e0, 1, 0, nullptr, ws.logits);
            }
        }
        __threadfence();
    }
    __syncthreads();
    trace_point(tr, kTraceRouter, 6);
    if (tid == 0) {
        if (nexp > 0) red_release_add(fs + kFSyncLg, 1);
        f_wait_count(fs + kFSyncLg, min(E, G), ws.err, abort);
    }
    __syncthreads();
    trace_point(tr, kTraceRouter, 2);

    // ---- routing of all B tokens, then the dispatch, in every CTA
    for (int i = tid; i < B * E; i += kFThreads) lg_s[i] = __ldcg(ws.logits + i);
    __syncthreads();
    if (warp < B)
        route_token_lean(lg_s + (size_t)warp * E, E, k, norm, sh.top + warp * k, sh.tw + warp * k,
                         reinterpret_cast<float*>(rscr) + warp * kMaxE);
    __syncthreads();
    if (warp == 0) {
        jl_ws wl;
        memset(&wl, 0, sizeof(wl));
        wl.sel = sh.sel;
        wl.uh = sh.uh;
        wl.uidx = sh.uidx;
        wl.uw = sh.uw;
        wl.comb = sh.comb;
        wl.slot_pos = sh.slot_pos;
        wl.U = &sh.U;
        wl.err = ws.err;
        dispatch_warp_small(sh.top, sh.tw, B, k, E, wl, dsm);
    }
    // the routing scratch shares bytes with the ring: order these generic
    // writes before the producer's bulk copies into the same bytes
    fence_proxy_async_smem();
    __syncthreads();
    trace_point(tr, kTraceRouter, 3);
    const int U = sh.U, S = B * k;
    if (c == 0) {  // publish the routing (top-k outputs, debug_routing)
        for (int i = tid; i < S; i += kFThreads) {
            ws.top[i] = sh.top[i];
            ws.tw[i] = sh.tw[i];
            ws.uidx[i] = sh.uidx[i];
            ws.uw[i] = sh.uw[i];
            ws.comb[i] = sh.comb[i];
            ws.slot_pos[i] = sh.slot_pos[i];
            if (top_out) top_out[i] = sh.top[i];
            if (tw_out) tw_out[i] = sh.tw[i];
        }
        for (int i = tid; i <= U; i += kFThreads) {
            if (i < U) ws.sel[i] = sh.sel[i];
            ws.uh[i] = sh.uh[i];
        }
        if (tid == 0) *ws.U = U;
    }

    // ---- 2. expert units
    const int MTg = m / 64, MTd = d / 128, ngd = d / kGroup, ngm = m / kGroup;
    const FWork W = f_work(U, G, c, MTg, MTd);
    const int nunits = W.ngu + W.ndn;
    if (warp == kFWarps) {
        // ---------------- producer: chunks of every unit, in order
        if (lane == 0) {
            int Gi = 0;
            bool ok = !*abort;
            for (int i = 0; ok && i < nunits; i++) {
                const bool dn = i >= W.ngu;
                const int MT = dn ? MTd : MTg, ng = dn ? ngm : ngd;
                const int unit = dn ? (G - 1 - c) + (i - W.ngu) * G : c + i * G;
                const int u = unit / MT, mt = unit - u * MT;
                const int nch = (ng + kFChunkGroups - 1) / kFChunkGroups;
                const uint8_t* base = store_l + (size_t)sh.sel[u] * L.rec_bytes +
                                      (dn ? L.tile_off(2, 4 * mt, 0) : L.tile_off(0, 2 * mt, 0));
                for (int ch = 0; ch < nch; ch++, Gi++) {
                    const int s = Gi % P.S;
                    if (Gi >= P.S && !f_wait(&sh.empty[s], ((Gi / P.S) - 1) & 1, ws.err, abort)) {
                        ok = false;
                        break;
                    }
                    const int gn = min(kFChunkGroups, ng - ch * kFChunkGroups);
                    const uint32_t bytes = (uint32_t)gn * 4 * kTileRec;
                    mbar_expect_tx(&sh.full[s], bytes);
                    bulk_g2s_hint(ring + (size_t)s * kFChunkBytes, base + (size_t)ch * kFChunkBytes, bytes, &sh.full[s],
                                  l2_policy_evict_first());
                }
            }
            // no copy may still be landing when the CTA leaves
            for (int q = max(0, Gi - P.S); q < Gi; q++)
                mbar_wait_bounded(&sh.full[q % P.S], (q / P.S) & 1, ws.err);
        }
    } else {
        // ---------------- compute warps
        const int ur = tid & 127, tq = tid >> 7;  // chain pairs (unit row ur, tokens tq, tq + 4)
        int Gi = 0;
        for (int i = 0; i < nunits; i++) {
            const bool dn = i >= W.ngu;
            const int MT = dn ? MTd : MTg, ng = dn ? ngm : ngd;
            const int unit = dn ? (G - 1 - c) + (i - W.ngu) * G : c + i * G;
            const int u = unit / MT, mt = unit - u * MT;
            const int nch = (ng + kFChunkGroups - 1) / kFChunkGroups;
            const int s0 = sh.uh[u], n = sh.uh[u + 1] - s0;
            if (dn) {
                // activations of expert u: wait for all its gate/up units
                if (tid == 0) f_wait_count(fs + kFSyncGu + u, MTg, ws.err, abort);
                named_barrier(kFBar, kFWarps * 32);
                if (i == W.ngu) trace_point(tr, kTraceRouter, 8);
                for (int q = tid; q < n * (m / 4); q += kFWarps * 32) {
                    const int t = q / (m / 4), cc = q - t * (m / 4);
                    const float4 v =
                        __ldcg(reinterpret_cast<const float4*>(ws.act + (size_t)sh.uidx[s0 + t] * m) + cc);
                    *reinterpret_cast<float4*>(x_s + (size_t)t * m + 4 * cc) = v;
                }
                if (tid < n) sh.xoff[tid] = tid * m;
            } else {
                if (tid < n) sh.xoff[tid] = (sh.uidx[s0 + tid] / k) * xs;
            }
            named_barrier(kFBar, kFWarps * 32);
            float acc0 = 0.0f, acc1 = 0.0f;
            for (int ch = 0; ch < nch; ch++, Gi++) {
                const int s = Gi % P.S, buf = Gi & 1;
                const int gn = min(kFChunkGroups, ng - ch * kFChunkGroups);
                const bool ok = f_wait(&sh.full[s], (Gi / P.S) & 1, ws.err, abort);
                if (Gi == 0) trace_point(tr, kTraceRouter, 7);
                if (ok && warp < gn * 4) {
                    const int gl = warp >> 2, j = warp & 3;
                    const uint8_t* tile = ring + (size_t)s * kFChunkBytes + (size_t)(gl * 4 + j) * kTileRec;
                    float* pp = p_s + ((size_t)(buf * B) * 4 + gl) * 128 + 32 * j + lane;
                    record_products(tile, x_s, sh.xoff, n, (ch * kFChunkGroups + gl) * kGroup, pp, 4 * 128);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.empty[s]);
                named_barrier(kFBar, kFWarps * 32);
                // per-row chains advance over this chunk's groups, in group order
                if (tq < n) {
                    const float* pc = p_s + ((size_t)(buf * B + tq) * 4) * 128 + ur;
                    for (int gl = 0; gl < gn; gl++) acc0 = __fadd_rn(acc0, pc[gl * 128]);
                }
                if (tq + 4 < n) {
                    const float* pc = p_s + ((size_t)(buf * B + tq + 4) * 4) * 128 + ur;
                    for (int gl = 0; gl < gn; gl++) acc1 = __fadd_rn(acc1, pc[gl * 128]);
                }
            }
            if (!dn) {
                // SwiGLU: unit rows 0..63 are gate rows, 64..127 the matching up rows
                if (ur >= 64) {
                    if (tq < n) up_s[tq * 64 + ur - 64] = acc0;
                    if (tq + 4 < n) up_s[(tq + 4) * 64 + ur - 64] = acc1;
                }
                named_barrier(kFBar, kFWarps * 32);
                if (ur < 64) {
                    if (tq < n)
                        ws.act[(size_t)sh.uidx[s0 + tq] * m + mt * 64 + ur] = silu_mul(acc0, up_s[tq * 64 + ur]);
                    if (tq + 4 < n)
                        ws.act[(size_t)sh.uidx[s0 + tq + 4] * m + mt * 64 + ur] =
                            silu_mul(acc1, up_s[(tq + 4) * 64 + ur]);
                }
                __threadfence();
                named_barrier(kFBar, kFWarps * 32);
                if (tid == 0) red_release_add(fs + kFSyncGu + u, 1);
            } else {
                // y[slot] = 0 + w * dacc (the reference's `ye += uw * dacc` onto a zeroed ye)
                if (tq < n)
                    ws.y[(size_t)sh.uidx[s0 + tq] * d + mt * 128 + ur] =
                        __fadd_rn(0.0f, __fmul_rn(sh.uw[s0 + tq], acc0));
                if (tq + 4 < n)
                    ws.y[(size_t)sh.uidx[s0 + tq + 4] * d + mt * 128 + ur] =
                        __fadd_rn(0.0f, __fmul_rn(sh.uw[s0 + tq + 4], acc1));
                __threadfence();
                named_barrier(kFBar, kFWarps * 32);
                if (tid == 0) sh.last = atomicAdd(fs + kFSyncRb + mt, 1) == U - 1;
                named_barrier(kFBar, kFWarps * 32);
                if (sh.last) {
                    // ---- 3. combine of rows [128 mt, 128 mt + 128) (decode_kernel.c:1490-1507)
                    __threadfence();
                    for (int q = tid; q < B * 128; q += kFWarps * 32) {
                        const int b = q >> 7, r = mt * 128 + (q & 127);
                        float v[kMaxK];
#pragma unroll
                        for (int j = 0; j < kMaxK; j++)
                            v[j] = j < k ? __ldcg(ws.y + (size_t)sh.comb[b * k + j] * d + r) : 0.0f;
                        float a = 0.0f;
#pragma unroll
                        for (int j = 0; j < kMaxK; j++)
                            if (j < k) a = __fadd_rn(a, v[j]);
                        out[(size_t)b * d + r] = a;
                    }
                    if (tid == 0) fs[kFSyncRb + mt] = 0;
                }
            }
        }
        if (tid == 0) trace_point(tr, kTraceRouter, 4);
    }
    __syncthreads();
    trace_point(tr, kTraceRouter, 5);
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(fs + kFSyncExit, 1) == G - 1) {
            // every CTA has passed all its waits: reset the counters for the next launch
            fs[kFSyncLg] = 0;
            for (int u = 0; u < U; u++) fs[kFSyncGu + u] = 0;
            fs[kFSyncExit] = 0;
            __threadfence();
        }
    }
}

}  // namespace jl

// Per-device limits of k_layer_small: the opt-in shared memory per block
// minus the kernel's own static shared memory (read from the compiled
// function, which holds more than FShared alone).
namespace {
struct FLimits {
    int dev = -1;
    size_t dyn_max = 0;  // dynamic shared memory the kernel may request
    bool ok = false;
};
FLimits g_flimits[64];
std::mutex g_flimits_mu;

const FLimits* fused_limits(int dev) {
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_flimits_mu);
    FLimits& f = g_flimits[dev];
    if (f.dev == dev) return &f;
    int optin = 0;
    cudaFuncAttributes fa{};
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaFuncGetAttributes(&fa, jl::k_layer_small) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    f.dev = dev;
    f.ok = false;
    if ((size_t)optin > fa.sharedSizeBytes + 1024) {
        f.dyn_max = (size_t)optin - fa.sharedSizeBytes;
        f.ok = cudaFuncSetAttribute(jl::k_layer_small, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)f.dyn_max) == cudaSuccess;
        if (!f.ok) cudaGetLastError();
    }
    return &f;
}
}  // namespace

// Shared-memory plan for batch B; false when the shape does not fit.
static bool plan_small(const jl_moe* h, int B, jl::FPlan* P, size_t* smem_bytes) {
    using namespace jl;
    const int d = h->d, m = h->m, E = h->E, k = h->k;
    if (B < 1 || B > kFMaxB || k > kMaxK || E > kMaxE || E < k) return false;
    if (d % 128 || m % 64 || h->sm_count < 2) return false;
    const FLimits* lim = fused_limits(h->device);
    if (!lim || !lim->ok) return false;
    auto al = [](size_t v) { return (v + 127) / 128 * 128; };
    FPlan p{};
    p.xs = d + 8;  // 8-float pad: the router's 4 tokens x 8 lanes of a warp hit distinct banks
    const size_t xa = al(std::max((size_t)B * p.xs * 4, (size_t)B * m * 4));
    const size_t ps = al((size_t)2 * B * 4 * 128 * 4);
    const size_t ups = al((size_t)B * 64 * 4);
    p.ps_off = (int)xa;
    p.ups_off = (int)(xa + ps);
    p.ring_off = (int)(xa + ps + ups);
    const size_t cap = lim->dyn_max;
    if ((size_t)p.ring_off + 3 * kFChunkBytes > cap) return false;
    p.S = (int)std::min<size_t>(kFMaxStages, (cap - p.ring_off) / kFChunkBytes);
    // routing scratch inside the ring: router rows, logits, per-token scratch, dispatch scratch
    const int nexp_max = (E + h->sm_count - 1) / h->sm_count;
    p.xt_off = (int)al((size_t)nexp_max * router_expert_halves(d) * 2);
    p.lg_off = p.xt_off + (int)al((size_t)B * 8 * router_xstride(d) * 4);
    p.rs_off = p.lg_off + (int)al((size_t)B * E * 4);
    p.ds_off = p.rs_off + (int)al((size_t)B * kMaxE * 4);
    if ((size_t)p.ds_off + (size_t)(4 * E + 2) * 4 > (size_t)p.S * kFChunkBytes) return false;
    *P = p;
    *smem_bytes = (size_t)p.ring_off + (size_t)p.S * kFChunkBytes;
    return true;
}

size_t jl_fsync_bytes(int d) { return (size_t)(jl::kFSyncRb + d / 128 + 8) * sizeof(int); }

bool jl_layer_small_ok(const jl_moe* h, int B) {
    jl::FPlan P;
    size_t smem = 0;
    return plan_small(h, B, &P, &smem);
}

int jl_launch_layer_small(const jl_moe* h, const unsigned short* gate_w_l, const uint8_t* store_l,
                          const float* x, int B, float* out, int* top, float* tw, cudaStream_t s) {
    using namespace jl;
    FPlan P;
    size_t smem = 0;
    if (!plan_small(h, B, &P, &smem)) return JL_ERR_INVALID;
    return launch(k_layer_small, dim3(h->sm_count), dim3(kFThreads), smem, s, (const uint16_t*)gate_w_l,
                  store_l, h->lay, h->E, h->k, h->norm, x, B, out, top, tw, h->ws, P);
}
