// Expert parallelism on the device. Two forms of the per-layer exchange:
//  - with NCCL (the caller runs the all-to-alls): k_ep_order / k_ep_gather
//    pack a rank's routed slots by owner rank, k_ep_combine adds the rows
//    that come back (jl_ep_pack, jl_ep_combine);
//  - over NVLink peer memory, no host round trip (jl_ep_forward): the
//    kernels below the second banner store token rows into the owners'
//    exported buffers and the weighted rows back, synchronised by epoch
//    flags.
#include <algorithm>
#include <cstring>
#include <new>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

constexpr int kEpThreads = 1024;
constexpr int kEpMaxWorld = 64;

// Stable grouping of the S = B*k slots by owner rank dest = top / E_local:
// pos[s] = start of dest's block + #{s' < s : dest(s') == dest(s)}.
// One block; per owner w a block-wide exclusive scan of (dest == w) flags.
__global__ void __launch_bounds__(kEpThreads) k_ep_order(const int* __restrict__ top, int S, int E_local,
                                                         int world, int* __restrict__ pos,
                                                         int* __restrict__ counts, int* err) {
    __shared__ int wsum[kEpThreads / 32];
    __shared__ int base[kEpMaxWorld];
    __shared__ int cnt[kEpMaxWorld];
    __shared__ int chunk_total;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, W = blockDim.x >> 5;
    griddep_wait();
    griddep_launch_dependents();
    if (tid < world) cnt[tid] = 0;
    __syncthreads();
    for (int s = tid; s < S; s += blockDim.x) {
        const int e = top[s];
        int w = e / E_local;
        if (e < 0 || w >= world) {
            atomicOr(err, kErrBadExpert);
            w = 0;
        }
        atomicAdd(&cnt[w], 1);
    }
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
        for (int w = 0; w < world; w++) {
            base[w] = acc;
            counts[w] = cnt[w];
            acc += cnt[w];
        }
    }
    __syncthreads();
    for (int w = 0; w < world; w++) {
        int carry = 0;
        for (int c0 = 0; c0 < S; c0 += blockDim.x) {
            const int s = c0 + tid;
            int e = s < S ? top[s] : -1;
            int dw = (e < 0) ? 0 : e / E_local;
            if (dw >= world) dw = 0;
            const bool f = s < S && dw == w;
            const unsigned bal = __ballot_sync(0xffffffffu, f);
            if (lane == 0) wsum[warp] = __popc(bal);
            __syncthreads();
            if (warp == 0) {
                const int v = lane < W ? wsum[lane] : 0;
                int inc = v;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, inc, o);
                    if (lane >= o) inc += t;
                }
                if (lane < W) wsum[lane] = inc - v;
                if (lane == 31) chunk_total = inc;
            }
            __syncthreads();
            if (f) pos[s] = base[w] + carry + wsum[warp] + __popc(bal & ((1u << lane) - 1u));
            carry += chunk_total;
            __syncthreads();
        }
    }
}

// Row gather into send order: block = one slot (its d floats) plus its
// (local expert, weight bits) pair.
__global__ void k_ep_gather(const float* __restrict__ x, const int* __restrict__ top,
                            const float* __restrict__ tw, const int* __restrict__ pos, int k, int d,
                            int E_local, float* __restrict__ rows, int* __restrict__ meta) {
    griddep_wait();
    griddep_launch_dependents();
    const int s = blockIdx.x, p = pos[s];
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)(s / k) * d);
    float4* dst = reinterpret_cast<float4*>(rows + (size_t)p * d);
    for (int i = threadIdx.x; i < d / 4; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) {
        meta[2 * p] = top[s] % E_local;
        meta[2 * p + 1] = __float_as_int(tw[s]);
    }
}

// out[b] = 0 + back[pos[comb[b*k]]] + back[pos[comb[b*k+1]]] + ... in order
// (the reference's union-order combine, decode_kernel.c:1490-1507).
__global__ void k_ep_combine(const float* __restrict__ back, const int* __restrict__ pos,
                             const int* __restrict__ comb, int k, int d, float* __restrict__ out) {
    griddep_wait();
    griddep_launch_dependents();
    const int b = blockIdx.y;
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (c >= d) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; j++) {
        const int p = pos[comb[b * k + j]];
        const float4 v = *reinterpret_cast<const float4*>(back + (size_t)p * d + c);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    *reinterpret_cast<float4*>(out + (size_t)b * d + c) = acc;
}

}  // namespace jl

extern "C" int jl_ep_pack(const int* top, const float* tw, const float* x, int B, int k, int d,
                          int E_local, int world, float* rows, int* meta, int* pos, int* counts,
                          int* dev_status, void* stream) {
    using namespace jl;
    if (!top || !tw || !x || !rows || !meta || !pos || !counts || !dev_status) return JL_ERR_INVALID;
    if (B < 1 || k < 1 || d < 4 || d % 4 || E_local < 1 || world < 1 || world > kEpMaxWorld)
        return JL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(rows)) & 15) return JL_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    const int S = B * k;
    int rc = launch(k_ep_order, dim3(1), dim3(kEpThreads), 0, s, top, S, E_local, world, pos, counts,
                    dev_status);
    if (rc) return rc;
    return launch(k_ep_gather, dim3(S), dim3(128), 0, s, x, top, tw, (const int*)pos, k, d, E_local,
                  rows, meta);
}

extern "C" int jl_ep_combine(const float* back, const int* pos, const int* comb, int B, int k, int d,
                             float* out, void* stream) {
    using namespace jl;
    if (!back || !pos || !comb || !out || B < 1 || k < 1 || d < 4 || d % 4) return JL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(back) | reinterpret_cast<uintptr_t>(out)) & 15) return JL_ERR_INVALID;
    const int tpb = 128;
    dim3 grid((d / 4 + tpb - 1) / tpb, B);
    return launch(k_ep_combine, grid, dim3(tpb), 0, (cudaStream_t)stream, back, pos, comb, k, d, out);
}

// ---------------------------------------------------------------------------
// Expert-parallel layer over NVLink peer memory (no host round trip).
//
// Every rank exports one buffer (CUDA IPC) with the same layout:
//   recv_rows [world][cap][d]  token rows sent to this rank by rank r
//   recv_meta [world][cap][2]  their (local expert, weight bits)
//   recv_cnt  [world]          rows rank r sent here this layer
//   ret_rows  [world][cap][d]  weighted expert rows owner q sent back
//   flags     [2][world]       epoch stamps: [0][r] rows from r landed,
//                              [1][q] returns from q landed
// where cap = max tokens x topk (the most slots one rank can send to one
// owner). A layer: route -> order by owner -> send (peer stores) -> owner
// waits for every sender, runs its experts on the padded receive batch ->
// return (peer stores) -> sender waits for every owner and combines. Flags
// carry a per-call epoch, so nothing is ever reset; every wait is bounded
// and reports kErrTimeout instead of hanging.

namespace jl {

struct ep_layout {
    size_t rr, rm, rc, ret, fl, bytes;
};

__host__ __device__ inline ep_layout ep_offsets(int world, int cap, int d) {
    ep_layout o;
    size_t off = 0;
    auto take = [&](size_t n) {
        const size_t at = off;
        off = (off + n + 255) / 256 * 256;
        return at;
    };
    o.rr = take((size_t)world * cap * d * 4);
    o.rm = take((size_t)world * cap * 2 * 4);
    o.rc = take((size_t)world * 4);
    o.ret = take((size_t)world * cap * d * 4);
    o.fl = take((size_t)2 * world * 8);
    o.bytes = off;
    return o;
}

struct ep_peers {
    uint8_t* p[kEpMaxWorld];
};

__device__ __forceinline__ void st_release_sys(unsigned long long* a, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* a) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}

// Bounded wait until flags[f][0..world) all reached `epoch`; gives up after
// `limit` SM clock cycles in total.
__device__ bool ep_wait_flags(const uint8_t* buf, ep_layout o, int world, int f,
                              unsigned long long epoch, long long limit, int* err) {
    const unsigned long long* fl = reinterpret_cast<const unsigned long long*>(buf + o.fl) + f * world;
    const long long t0 = clock64();
    for (int r = 0; r < world; r++) {
        while (ld_acquire_sys(fl + r) < epoch) {
            if (clock64() - t0 > limit) {
                atomicOr(err, kErrTimeout);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

// Slot s -> owner q's recv_rows[rank][pos[s] - base[q]] (+ meta); the last
// block to finish publishes the counts and stamps flags[0][rank] on every
// owner.
__global__ void k_ep_send(const float* __restrict__ x, const int* __restrict__ top,
                          const float* __restrict__ tw, const int* __restrict__ pos,
                          const int* __restrict__ counts, int S, int k, int d, int E_local, int rank,
                          int world, int cap, ep_peers peers, ep_layout o, unsigned long long epoch,
                          int* done) {
    __shared__ int is_last;
    griddep_wait();
    griddep_launch_dependents();
    for (int s = blockIdx.x; s < S; s += gridDim.x) {
        const int e = top[s], q = e / E_local;
        if (e < 0 || q >= world) continue;  // k_ep_order flagged it; store nothing
        int base = 0;
        for (int w = 0; w < q; w++) base += counts[w];
        const int i = pos[s] - base;
        uint8_t* pb = peers.p[q];
        float4* dst = reinterpret_cast<float4*>(pb + o.rr + ((size_t)rank * cap + i) * d * 4);
        const float4* src = reinterpret_cast<const float4*>(x + (size_t)(s / k) * d);
        for (int c = threadIdx.x; c < d / 4; c += blockDim.x) dst[c] = src[c];
        if (threadIdx.x == 0) {
            int* m = reinterpret_cast<int*>(pb + o.rm) + ((size_t)rank * cap + i) * 2;
            m[0] = e - q * E_local;
            m[1] = __float_as_int(tw[s]);
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(done, 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!is_last) return;
    if (threadIdx.x < world) {
        const int q = threadIdx.x;
        reinterpret_cast<int*>(peers.p[q] + o.rc)[rank] = counts[q];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < world) {
        const int q = threadIdx.x;
        st_release_sys(reinterpret_cast<unsigned long long*>(peers.p[q] + o.fl) + rank, epoch);
    }
    if (threadIdx.x == 0) *done = 0;
}

// Owner side: wait for every sender, then turn the received rows into a
// padded routed batch for the topk = 1 expert handle: slot r*cap + i is row
// i from rank r (expert id -1 past that rank's count).
// stats[0] accumulates the rows received, stats[1] the calls.
__global__ void k_ep_recv(const uint8_t* __restrict__ buf, ep_layout o, int world, int cap,
                          unsigned long long epoch, long long limit, int* __restrict__ top,
                          float* __restrict__ tw, unsigned long long* stats, int* err) {
    __shared__ int ok;
    griddep_wait();
    griddep_launch_dependents();
    if (threadIdx.x == 0) ok = ep_wait_flags(buf, o, world, 0, epoch, limit, err);
    __syncthreads();
    // peers wrote these: read them past L1 (__ldcv)
    const int* cnt = reinterpret_cast<const int*>(buf + o.rc);
    const int* meta = reinterpret_cast<const int*>(buf + o.rm);
    if (threadIdx.x == 0 && ok) {
        unsigned long long n = 0;
        for (int r = 0; r < world; r++) n += (unsigned long long)min(max(__ldcv(cnt + r), 0), cap);
        atomicAdd(stats, n);
        atomicAdd(stats + 1, 1ull);
    }
    for (int s = threadIdx.x; s < world * cap; s += blockDim.x) {
        const int r = s / cap, i = s % cap;
        const bool valid = ok && i < __ldcv(cnt + r);
        top[s] = valid ? __ldcv(meta + 2 * s) : -1;
        tw[s] = valid ? __int_as_float(__ldcv(meta + 2 * s + 1)) : 0.0f;
    }
}

// Owner side: row i from rank r (weighted expert output y[slot]) goes back
// to rank r's ret_rows[rank][i]; the last block stamps flags[1][rank] there.
__global__ void k_ep_return(const uint8_t* __restrict__ buf, const float* __restrict__ y, int d,
                            int rank, int world, int cap, ep_peers peers, ep_layout o,
                            unsigned long long epoch, int* done) {
    __shared__ int is_last;
    griddep_wait();
    griddep_launch_dependents();
    const int* cnt = reinterpret_cast<const int*>(buf + o.rc);
    for (int s = blockIdx.x; s < world * cap; s += gridDim.x) {
        const int r = s / cap, i = s % cap;
        if (i >= __ldcv(cnt + r)) continue;
        float4* dst = reinterpret_cast<float4*>(peers.p[r] + o.ret + ((size_t)rank * cap + i) * d * 4);
        const float4* src = reinterpret_cast<const float4*>(y + (size_t)s * d);
        for (int c = threadIdx.x; c < d / 4; c += blockDim.x) dst[c] = src[c];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(done, 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!is_last) return;
    if (threadIdx.x < world)
        st_release_sys(reinterpret_cast<unsigned long long*>(peers.p[threadIdx.x] + o.fl) + world + rank,
                       epoch);
    if (threadIdx.x == 0) *done = 0;
}

// Sender side: wait for every owner, then out[b] = 0 + the k returned rows
// of token b in union order.
__global__ void k_ep_gather_out(const uint8_t* __restrict__ buf, ep_layout o, const int* __restrict__ top,
                                const int* __restrict__ pos, const int* __restrict__ counts,
                                const int* __restrict__ comb, int k, int d, int E_local, int world,
                                int cap, unsigned long long epoch, long long limit, float* __restrict__ out,
                                int* err) {
    __shared__ int ok;
    griddep_wait();
    griddep_launch_dependents();
    if (threadIdx.x == 0) ok = ep_wait_flags(buf, o, world, 1, epoch, limit, err);
    __syncthreads();
    if (!ok) return;
    const int b = blockIdx.y;
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (c >= d) return;
    const float* ret = reinterpret_cast<const float*>(buf + o.ret);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; j++) {
        const int s = comb[b * k + j], e = top[s], q = e / E_local;
        if (e < 0 || q >= world) continue;  // k_ep_order flagged it; the term is dropped
        int base = 0;
        for (int w = 0; w < q; w++) base += counts[w];
        const float4 v = __ldcv(reinterpret_cast<const float4*>(ret + ((size_t)q * cap + pos[s] - base) * d + c));
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    *reinterpret_cast<float4*>(out + (size_t)b * d + c) = acc;
}

}  // namespace jl

struct jl_ep {
    int device, rank, world, cap, d, k, max_tokens;
    jl::ep_layout o;
    uint8_t* buf;
    uint8_t* peer[jl::kEpMaxWorld];
    bool opened[jl::kEpMaxWorld];
    int* scratch;  // pos [cap], counts [world], done [2], err [1]
    unsigned long long* stats;  // [2] rows received, calls (k_ep_recv)
    unsigned long long epoch;
    long long wait_cycles;  // bound of each wait on other ranks, SM clock cycles
    jl_moe* local;
    cudaEvent_t ev[9];  // optional phase events (jl_ep_set_phase_events)
    int n_ev;
};

extern "C" int jl_ep_create(jl_moe* local, int rank, int world, int max_tokens, int topk, jl_ep** out) {
    using namespace jl;
    if (!out || !local || world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world || max_tokens < 1 ||
        topk < 1 || local->k != 1 || local->router_only || local->staged || local->bf16)
        return JL_ERR_INVALID;
    *out = nullptr;
    const int cap = max_tokens * topk;
    if ((long long)world * cap > local->max_tokens) return JL_ERR_CAPACITY;
    jl_ep* ep = new (std::nothrow) jl_ep();
    if (!ep) return JL_ERR_OOM;
    memset(ep, 0, sizeof(*ep));
    ep->device = local->device;
    ep->rank = rank;
    ep->world = world;
    ep->cap = cap;
    ep->d = local->d;
    ep->k = topk;
    ep->max_tokens = max_tokens;
    ep->local = local;
    ep->o = ep_offsets(world, cap, local->d);
    ep->wait_cycles = kWaitLimitCycles;
    if (cudaMalloc(&ep->buf, ep->o.bytes) != cudaSuccess ||
        cudaMalloc(&ep->scratch, ((size_t)cap + world + 3) * sizeof(int)) != cudaSuccess ||
        cudaMalloc(&ep->stats, 2 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(ep->stats, 0, 2 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(ep->buf, 0, ep->o.bytes) != cudaSuccess ||
        cudaMemset(ep->scratch, 0, ((size_t)cap + world + 3) * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        if (ep->buf) cudaFree(ep->buf);
        if (ep->scratch) cudaFree(ep->scratch);
        if (ep->stats) cudaFree(ep->stats);
        delete ep;
        return JL_ERR_OOM;
    }
    ep->peer[rank] = ep->buf;
    ep->epoch = 0;
    *out = ep;
    return JL_OK;
}

extern "C" int jl_ep_ipc_handle(jl_ep* ep, void* handle) {
    if (!ep || !handle) return JL_ERR_INVALID;
    cudaIpcMemHandle_t h;
    JL_CUDA(cudaIpcGetMemHandle(&h, ep->buf));
    memcpy(handle, &h, sizeof(h));
    return JL_OK;
}

extern "C" int jl_ep_open_peers(jl_ep* ep, const void* handles) {
    if (!ep || !handles) return JL_ERR_INVALID;
    const cudaIpcMemHandle_t* hs = reinterpret_cast<const cudaIpcMemHandle_t*>(handles);
    for (int r = 0; r < ep->world; r++) {
        if (r == ep->rank || ep->opened[r]) continue;
        void* p = nullptr;
        JL_CUDA(cudaIpcOpenMemHandle(&p, hs[r], cudaIpcMemLazyEnablePeerAccess));
        ep->peer[r] = (uint8_t*)p;
        ep->opened[r] = true;
    }
    return JL_OK;
}

extern "C" int jl_ep_attach(jl_ep* ep, int r, jl_ep* peer) {
    if (!ep || !peer || r < 0 || r >= ep->world || r == ep->rank || ep->opened[r]) return JL_ERR_INVALID;
    if (peer->rank != r || peer->world != ep->world || peer->cap != ep->cap || peer->d != ep->d)
        return JL_ERR_INVALID;
    if (peer->device != ep->device) {
        int can = 0;
        JL_CUDA(cudaDeviceCanAccessPeer(&can, ep->device, peer->device));
        if (!can) return JL_ERR_INVALID;
        const cudaError_t e = cudaDeviceEnablePeerAccess(peer->device, 0);
        if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return jl_note_cuda(e);
        cudaGetLastError();
    }
    ep->peer[r] = peer->buf;
    return JL_OK;
}

extern "C" int jl_ep_set_wait_limit(jl_ep* ep, long long ns) {
    if (!ep || ns < 1) return JL_ERR_INVALID;
    // clock64 counts SM cycles; 2 cycles per ns bounds the wait by at least
    // `ns` at any SM clock up to 2 GHz (a B200 runs at most 1.965 GHz)
    ep->wait_cycles = ns > (1ll << 61) ? (1ll << 62) : 2 * ns;
    return JL_OK;
}

extern "C" int jl_ep_set_phase_events(jl_ep* ep, void* const* events, int n) {
    if (!ep || n < 0 || n > 9 || (n > 0 && !events)) return JL_ERR_INVALID;
    for (int i = 0; i < n; i++)
        if (!events[i]) return JL_ERR_INVALID;
    for (int i = 0; i < n; i++) ep->ev[i] = (cudaEvent_t)events[i];
    ep->n_ev = n;
    return JL_OK;
}

extern "C" int jl_ep_stats(jl_ep* ep, long long* rows, long long* calls, void* stream) {
    if (!ep || !rows || !calls) return JL_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long h[2] = {0, 0};
    JL_CUDA(cudaMemcpyAsync(h, ep->stats, sizeof(h), cudaMemcpyDeviceToHost, s));
    JL_CUDA(cudaMemsetAsync(ep->stats, 0, sizeof(h), s));
    JL_CUDA(cudaStreamSynchronize(s));
    *rows = (long long)h[0];
    *calls = (long long)h[1];
    return JL_OK;
}

extern "C" int jl_ep_destroy(jl_ep* ep) {
    if (!ep) return JL_OK;
    for (int r = 0; r < ep->world; r++)
        if (ep->opened[r]) cudaIpcCloseMemHandle(ep->peer[r]);
    if (ep->buf) cudaFree(ep->buf);
    if (ep->scratch) cudaFree(ep->scratch);
    if (ep->stats) cudaFree(ep->stats);
    delete ep;
    return JL_OK;
}

extern "C" int jl_ep_forward(jl_ep* ep, jl_moe* router, int l, const float* x, int B, float* out,
                             void* stream) {
    using namespace jl;
    if (!ep || !router || !x || !out || l < 0 || l >= router->L || B < 1) return JL_ERR_INVALID;
    if (B > ep->max_tokens || B > router->max_tokens) return JL_ERR_CAPACITY;
    if (router->k != ep->k || router->d != ep->d || router->E != ep->local->E * ep->world) return JL_ERR_INVALID;
    if (!router->uploaded[l] || !ep->local->uploaded[l]) return JL_ERR_NOT_READY;
    for (int r = 0; r < ep->world; r++)
        if (!ep->peer[r]) return JL_ERR_INVALID;  // jl_ep_open_peers first
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) return JL_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    jl_moe* h = ep->local;
    const int S = B * ep->k, E_local = h->E, world = ep->world, cap = ep->cap;
    const unsigned long long epoch = ++ep->epoch;
    int* pos = ep->scratch;
    int* counts = pos + cap;
    int* done = counts + world;
    int* err = h->ws.err;
    ep_peers peers;
    for (int r = 0; r < kEpMaxWorld; r++) peers.p[r] = r < world ? ep->peer[r] : nullptr;
    // optional phase events (an event record inside stream capture must be an
    // external node to be timed when the graph replays)
    cudaStreamCaptureStatus cap_st = cudaStreamCaptureStatusNone;
    if (ep->n_ev > 0 && cudaStreamIsCapturing(s, &cap_st) != cudaSuccess) return JL_ERR_CUDA;
    auto mark = [&](int i) -> int {
        if (i >= ep->n_ev) return JL_OK;
        const cudaError_t e = (cap_st == cudaStreamCaptureStatusActive)
                                  ? cudaEventRecordWithFlags(ep->ev[i], s, cudaEventRecordExternal)
                                  : cudaEventRecord(ep->ev[i], s);
        return e == cudaSuccess ? JL_OK : jl_note_cuda(e);
    };
    // 1. route this rank's tokens (all E experts)
    const unsigned short* gw = router->gate_w + (size_t)l * router->E * router_expert_halves(router->d);
    int rc = mark(0);
    if (!rc) rc = jl_launch_route(router, gw, x, B, false, s);
    if (!rc) rc = mark(1);
    if (rc) return rc;
    // 2. group the slots by owner, 3. send them
    rc = launch(k_ep_order, dim3(1), dim3(kEpThreads), 0, s, (const int*)router->ws.top, S, E_local, world, pos,
                counts, err);
    if (!rc)
        rc = launch(k_ep_send, dim3(std::min(S, 4 * h->sm_count)), dim3(128), 0, s, x, (const int*)router->ws.top,
                    (const float*)router->ws.tw, (const int*)pos, (const int*)counts, S, ep->k, ep->d, E_local,
                    ep->rank, world, cap, peers, ep->o, epoch, done);
    if (!rc) rc = mark(2);
    // 4. owner: receive, run the local experts on the padded batch
    const int Bpad = world * cap;
    if (!rc)
        rc = launch(k_ep_recv, dim3(1), dim3(1024), 0, s, (const uint8_t*)ep->buf, ep->o, world, cap, epoch,
                    ep->wait_cycles, h->ws.top, h->ws.tw, ep->stats, err);
    if (!rc) rc = mark(3);
    const uint8_t* store_l = h->store + (size_t)l * h->E * h->lay.rec_bytes;
    const float* xr = reinterpret_cast<const float*>(ep->buf + ep->o.rr);
    const bool tc_ok = h->d % 512 == 0 && h->m % 256 == 0;
    const bool tc = h->path == JL_PATH_TC || (h->path == JL_PATH_AUTO && Bpad > 8 && tc_ok);
    if (!rc) rc = jl_launch_dispatch(h, Bpad, s);
    if (!rc) rc = mark(4);
    if (!rc) rc = tc ? jl_launch_gateup_tc(h, store_l, xr, Bpad, s) : jl_launch_gateup_exact(h, store_l, xr, Bpad, s);
    if (!rc) rc = mark(5);
    if (!rc) rc = tc ? jl_launch_down_tc(h, store_l, Bpad, s) : jl_launch_down_exact(h, store_l, Bpad, s);
    if (!rc) rc = mark(6);
    // 5. return the weighted rows, 6. combine
    if (!rc)
        rc = launch(k_ep_return, dim3(std::min(Bpad, 4 * h->sm_count)), dim3(128), 0, s, (const uint8_t*)ep->buf,
                    (const float*)h->ws.y, ep->d, ep->rank, world, cap, peers, ep->o, epoch, done + 1);
    if (!rc) rc = mark(7);
    if (!rc) {
        const int tpb = 128;
        rc = launch(k_ep_gather_out, dim3((ep->d / 4 + tpb - 1) / tpb, B), dim3(tpb), 0, s,
                    (const uint8_t*)ep->buf, ep->o, (const int*)router->ws.top, (const int*)pos,
                    (const int*)counts, (const int*)router->ws.comb, ep->k, ep->d, E_local, world, cap, epoch,
                    ep->wait_cycles, out, err);
    }
    if (!rc) rc = mark(8);
    return rc;
}
