// Internal declarations shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "joule_moe.h"

#include <cuda_fp16.h>

// Device layout of the Q4 store. A tile is 32 rows x one 64-value group of a
// part matrix, stored as a 1088-byte record: [half h][row t][16 B] (bytes
// 16h..16h+15 of row t's group; 1024 B) followed by the 32 fp16 scales. A
// warp reading one tile (lane t = row t) issues two fully coalesced 512-byte
// loads and one 64-byte load.
//
// Tiles are grouped so that every K step of the tensor-core path is ONE
// contiguous 4352-byte copy:
//   gate/up: for M-tile mt (gate rows and up rows 64mt..64mt+63), for group g:
//            [gate rb=2mt][gate rb=2mt+1][up rb=2mt][up rb=2mt+1]
//   down:    for M-tile mt (rows 128mt..128mt+127 of d), for group g:
//            [rb=4mt][rb=4mt+1][rb=4mt+2][rb=4mt+3]
// One expert record (per layer, per expert) = all gate/up tiles, then all
// down tiles; its size equals the reference's three Q4 records together
// (q4_store.py:150-158).
struct jl_layout {
    int d, m, E;
    int ngd, ngm;      // groups per row: d/64 (gate, up), m/64 (down)
    size_t dn_off;     // byte offset of the down tiles inside a record
    size_t rec_bytes;  // bytes per expert record
    // byte offset of tile (part p in gate/up/down, row block rb, group g)
    __host__ __device__ size_t tile_off(int p, int rb, int g) const {
        if (p < 2) return ((size_t)((rb >> 1) * ngd + g) * 4 + p * 2 + (rb & 1)) * 1088u;
        return dn_off + ((size_t)((rb >> 2) * ngm + g) * 4 + (rb & 3)) * 1088u;
    }
};

// Device workspace of one handle (all device pointers).
struct jl_ws {
    float* logits;   // [Bmax, E]
    int* top;        // [Bmax, k]
    float* tw;       // [Bmax, k]
    int* U;          // [1] union size
    int* sel;        // [E] union position -> expert
    int* uh;         // [E+1] union position -> first index into uidx/uw
    int* uidx;       // [Bmax*k] slots grouped by union position (slot order inside)
    float* uw;       // [Bmax*k] routing weight of uidx[i]
    int* comb;       // [Bmax*k] per token, its slots in union order
    int* slot_pos;   // [Bmax*k] slot -> index into uidx
    float* act;      // [Bmax*k, m] SwiGLU output per slot
    float* y;        // [Bmax*k, d] weighted expert output per slot
    int* counter;    // [1] last-block counter of the router kernel
    int* err;        // [1] device error word (jl::kErr* bits)
    long long* trace;  // [kTraceSlots] phase timestamps, nullptr when tracing is off
    // tensor-core path
    int* tc_ntiles;    // [1] token tiles of the current layer
    int* tc_tile;      // [max tiles][4]: expert, tokens, first uidx position, padded row offset
    __half* xc;        // token tiles: per tile [d/8][2N rows: hi, lo][8] fp16 (UMMA core layout)
    __half* ac;        // SwiGLU activations of the tiles, same layout over m
    size_t xc_plane, ac_plane;  // halves per plane
};

// Trace buffer layout: per kernel kind a row of 16 slots of %globaltimer
// stamps (ns) taken by thread 0 of one chosen block.
constexpr int kTraceRouter = 0, kTraceGateup = 1, kTraceDown = 2, kTraceCombine = 3;
constexpr int kTraceSlots = 8 * 16;  // rows 4, 5: wait-cycle counters of the tensor-core kernels

struct jl_moe {
    int device;
    int sm_count;  // streaming multiprocessors of the device (persistent grids)
    int router_only;  // JL_CREATE_ROUTER_ONLY: router weights and workspace, no expert store
    int L, d, E, k, m, norm;
    int bf16;                 // bf16 expert tier (KernelCfg.expert_bf16): bf16 matrices, no Q4
    int max_tokens;
    int path;
    jl_layout lay;
    unsigned short* gate_w;   // [L, E, 8, d/8 + 8] bf16, lane-major rows (jl_launch_repack_router)
    uint8_t* store;           // [L, E] records
    unsigned char* uploaded;  // host flags [L]
    jl_ws ws;
    void* ws_base;
    size_t ws_bytes;
    size_t store_bytes;
    int last_B;
    int comb_token_order;     // combine each token's slots in its own top-k order (batched prefill)
    long long* trace_buf;     // trace buffer: kept until destroy (captured graphs hold it)
    cudaEvent_t phase_ev[5];  // optional phase timing events
    int n_phase_ev;
    // host staging for uploads from host memory
    void* pinned;
    size_t pinned_bytes;
    uint8_t* dev_stage;       // device staging: one expert's reference records, or one layer's router rows
    size_t dev_stage_bytes;
    // staged store (jl_moe_create_staged): all L layers in pinned host memory,
    // `resident` of them in HBM slots, copied in on a side stream
    int staged;
    int resident;
    uint8_t* host_store;      // [L, E] records, pinned host memory
    uint8_t* dev_rec;         // one repacked expert record on its way to host_store
    int* slot_layer;          // [resident] layer held by each slot (-1: none)
    int* layer_slot;          // [L] slot holding each layer (-1: not resident)
    long long* slot_used;     // [resident] last use (least recently used slot is refilled)
    long long use_clock;
    cudaEvent_t* ev_ready;    // [resident] copy into the slot finished
    cudaEvent_t* ev_free;     // [resident] last kernel reading the slot finished
    cudaStream_t side;        // the copy stream
};

// The device records of layer l for a forward on stream s: for a staged
// store, the layer's slot (its copy enqueued on the side stream first when
// it is not resident; s then waits for it). jl_moe_layer_done records the
// slot's release after the forward's kernels and prefetches the next layer.
int jl_moe_layer_store(jl_moe* h, int l, cudaStream_t s, const uint8_t** out);
int jl_moe_layer_done(jl_moe* h, int l, cudaStream_t s);

// ---- launchers (return JL_OK or JL_ERR_*) --------------------------------

// Runs `setup` once per (current device, key) and returns its status (JL_OK
// on later calls). Kernel attributes such as the dynamic shared-memory limit
// are per device, so a process that drives several GPUs sets them on each;
// callers from several host threads are serialised. key < 32.
enum {
    kOnceExact = 0, kOnceRouter, kOnceRouterFast, kOnceDispatch, kOnceGemm, kOnceTc, kOnceGemv,
    kOnceDecode, kOnceEp, kOnceBf16, kOnceMmBf16, kOnceMmF32, kOnceAttn
};
int jl_device_once(int key, int (*setup)());

// Decode-step matvecs on the register-tiled kernel (jl_mm.cu): the
// reference's 8-lane FMA order; W in the chunked lane-major layout
// (jl_mv.cuh), the tokens column-major xT [K][Bp] (Bp a multiple of 4, >= B).
// From 16 tokens for every matrix; from kMmMinB tokens (its 16-token tiles
// part empty) for matrices too large for the small-batch kernel's L2
// prefetch (> 64 MB, the lm_head): at B = 8 the lm_head takes 379 us there
// against 572 us, while the prefetched projections are faster on the
// small-batch kernel inside the decode step's graph.
constexpr int kMmMinB = 8;
bool jl_mm_ok(int N, int K, int B, int min_b);
template <typename WT>
int jl_launch_mm(const WT* W, const float* xT, int Bp, int N, int K, int B, const float* bias, float* out,
                 int sm_count, cudaStream_t s);

// Fingerprint of the host weights a (cfg, W) pair points at: leading bytes of
// the router rows and of the first and last expert records, the expert
// pointer tables' first and last entries, and with `dense` the embedding, the
// first q projection and the lm_head. The host-buffer drop-ins cache a device
// copy per (cfg, W) and compare it on every call, so a model loaded into
// reused addresses is not mistaken for the cached one.
uint64_t jl_weights_fingerprint(const KernelCfg* c, const KernelW* W, bool dense);

// jl_store.cu
int jl_launch_repack_part(const uint8_t* pk_ref, const uint16_t* sc_ref, int p, const jl_layout& L,
                          uint8_t* rec, cudaStream_t s);

// Router weights [E, d] bf16 (reference layout, device) -> lane-major rows
// [E][8][d/8 + 8] (what jl_moe keeps in gate_w): lane j of expert e holds
// src[e][j + 8t], t < d/8, then 8 halves of padding, so the rows of one
// expert (and of consecutive experts) are one contiguous block whose rows
// start 16 bytes apart modulo 128: shared-memory rows without bank conflicts.
__host__ __device__ inline int router_row_halves(int d) { return d / 8 + 8; }
__host__ __device__ inline size_t router_expert_halves(int d) { return (size_t)8 * router_row_halves(d); }
int jl_launch_repack_router(const uint16_t* src, uint16_t* dst, int E, int d, cudaStream_t s);

// jl_router.cu: logits, softmax/top-k and dispatch on thread-block clusters;
// `tiles` also builds the tensor-core tile table.
int jl_launch_route(const jl_moe* h, const unsigned short* gate_w_l, const float* x, int B,
                    bool tiles, cudaStream_t s);

// jl_router.cu: routing only (logits -> top-k) with a caller-built ws; used by
// the entry point that allocates nothing (jl_noalloc.cu).
int jl_router_topk_prepare();
int jl_launch_router_topk(const jl_ws& ws, const unsigned short* gate_w, const float* x, int B, int E,
                          int d, int k, int norm, cudaStream_t s);

// Dispatch (union, slot map, tile table) from the top/tw already in the
// workspace, for callers that bring their own routing.
int jl_launch_dispatch(const jl_moe* h, int B, cudaStream_t s);

// jl_exact.cu: CUDA-core expert FFN in the reference's arithmetic order.
int jl_launch_gateup_exact(const jl_moe* h, const uint8_t* store_l, const float* x, int B,
                           cudaStream_t s);
int jl_launch_down_exact(const jl_moe* h, const uint8_t* store_l, int B, cudaStream_t s);
int jl_launch_combine(const jl_moe* h, int B, float* out, int* top, float* tw, cudaStream_t s);

// jl_gemv.cu: small-batch (B <= 4) expert FFN, warp-per-row GEMVs over all SMs.
bool jl_gemv_ok(const jl_moe* h, int B);
int jl_launch_gateup_gemv(const jl_moe* h, const uint8_t* store_l, const float* x, int B, cudaStream_t s);
int jl_launch_down_gemv(const jl_moe* h, const uint8_t* store_l, int B, cudaStream_t s);

// jl_bf16.cu: the bf16 expert tier (gate/up + SwiGLU, down; the combine follows).
int jl_launch_bf16_ffn(const jl_moe* h, const uint8_t* store_l, const float* x, int B, cudaStream_t s);
int jl_repack_bf16_part(const uint16_t* src, int p, const jl_moe* h, uint8_t* rec, cudaStream_t s);

// jl_tc.cu: tensor-core expert FFN (permute -> gate/up+SwiGLU -> down).
// The tile table is built at the end of the dispatch step (jl_tiles.cuh).
size_t jl_tc_ws_bytes(int Bmax, int E, int k, int d, int m, size_t* xc_plane, size_t* ac_plane);
int jl_launch_gateup_tc(const jl_moe* h, const uint8_t* store_l, const float* x, int B, cudaStream_t s);
int jl_launch_down_tc(const jl_moe* h, const uint8_t* store_l, int B, cudaStream_t s);
