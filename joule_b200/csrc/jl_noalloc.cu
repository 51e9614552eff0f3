// Router + top-k entry point that allocates no device memory.
//
// Every other entry point works out of a handle whose workspace was
// cudaMalloc'ed at creation. This one is for callers that cannot take that
// route: a host that reserves its whole device budget at start-up and must not
// grow it per request (an allocation there can fail under load, and
// cudaMalloc/cudaFree may synchronise the device and stall the other streams),
// and code that must stay off the allocator entirely (for instance code
// running inside a caching allocator's own hooks). Its only scratch, the
// [B, E] fp32 router logits, lives in a file-scope device array of fixed size;
// the top-k ids and weights go straight to the caller's buffers.
//
// Limits and rules:
//  - at most kNoAllocMaxB = 64 tokens and kNoAllocMaxE = 256 experts per call
//    (64 x 256 x 4 B = 64 KiB of static scratch); larger sizes are rejected
//    with JL_ERR_CAPACITY (B) or JL_ERR_INVALID (E), before any CUDA call;
//  - the first call on each device does a one-time setup: it looks up the
//    scratch array's device address (cudaGetSymbolAddress) and sets the
//    router kernel's shared-memory limit. That first call must come before any
//    stream capture is begun on the device;
//  - the scratch needs no clearing: every logit the top-k step reads was
//    written earlier in the same call. The caller-owned status word is
//    required (a bounded wait that runs out leaves this call's logits
//    unwritten, and the status word is the only place that says so); it must
//    hold zero before the call, and the kernels only OR error bits into it;
//  - one scratch array per device is shared by all callers, so two calls on
//    the same device must not overlap in time: issue them on one stream, or
//    order them with events. Overlapping calls race on the logits.
#include <atomic>
#include <mutex>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace {

constexpr int kNoAllocMaxB = 64;
constexpr int kNoAllocMaxE = 256;
constexpr int kNoAllocMaxK = 16;
constexpr int kNoAllocDevices = 64;
constexpr int kNoAllocLogits = kNoAllocMaxB * kNoAllocMaxE;

// [kNoAllocLogits] fp32 router logits.
__device__ __align__(256) float g_noalloc_scratch[kNoAllocLogits];

std::atomic<float*> g_scratch_dev[kNoAllocDevices];
std::mutex g_setup_mu;

// One-time per-device setup (symbol lookup; kernel attribute). Allocates
// nothing.
int scratch_for_device(int dev, float** out) {
    float* p = g_scratch_dev[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lk(g_setup_mu);
        p = g_scratch_dev[dev].load(std::memory_order_relaxed);
        if (!p) {
            void* sym = nullptr;
            if (cudaGetSymbolAddress(&sym, g_noalloc_scratch) != cudaSuccess || !sym) {
                cudaGetLastError();
                return JL_ERR_CUDA;
            }
            const int rc = jl_router_topk_prepare();
            if (rc) return rc;
            p = static_cast<float*>(sym);
            g_scratch_dev[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    return JL_OK;
}

}  // namespace

extern "C" int jl_route_noalloc(const unsigned short* gate_w, const float* x, int B, int E, int d,
                                int topk, int norm_topk_prob, int* top, float* tw, int* dev_status,
                                void* stream) {
    if (B < 0) return JL_ERR_INVALID;
    if (B == 0) return JL_OK;  // empty batch: nothing to route
    if (!gate_w || !x || !top || !tw || !dev_status) return JL_ERR_INVALID;
    if (B > kNoAllocMaxB) return JL_ERR_CAPACITY;
    if (E < 1 || E > kNoAllocMaxE || topk < 1 || topk > kNoAllocMaxK || topk > E) return JL_ERR_INVALID;
    if (d < 8 || d % 8) return JL_ERR_INVALID;
    // rows are moved by 16-byte bulk copies
    if ((reinterpret_cast<uintptr_t>(gate_w) | reinterpret_cast<uintptr_t>(x)) & 15) return JL_ERR_INVALID;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return JL_ERR_CUDA;
    }
    if (dev < 0 || dev >= kNoAllocDevices) return JL_ERR_INVALID;
    float* scratch = nullptr;
    int rc = scratch_for_device(dev, &scratch);
    if (rc) return rc;
    jl_ws ws;
    memset(&ws, 0, sizeof(ws));
    ws.logits = scratch;
    ws.top = top;
    ws.tw = tw;
    ws.err = dev_status;
    return jl_launch_router_topk(ws, gate_w, x, B, E, d, topk, norm_topk_prob ? 1 : 0,
                                 (cudaStream_t)stream);
}
