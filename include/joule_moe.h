/* joule_moe.h — C ABI of the B200 (sm_100a) MoE decode hot path.
 *
 * One MoE FFN layer at decode: router softmax/top-k -> token-to-expert
 * dispatch -> grouped per-expert gate/up -> SwiGLU -> down over the Q4 expert
 * store -> weighted combine. This library replaces the reference's CPU DLL
 * for that path; every entry point below names the reference interface it
 * replaces (paths relative to the reference project root).
 *
 * Conventions
 *  - Plain C types only. `stream` is a cudaStream_t passed as void*
 *    (NULL = the legacy default stream).
 *  - Every function returns an int status: JL_OK (0) or a negative JL_ERR_*.
 *    The reference's functions return void and clamp silently
 *    (decode_kernel.c:1522); here a bad argument is an error instead.
 *  - Pointers documented "device" must be CUDA device (or managed) memory;
 *    "host" pointers are ordinary CPU memory.
 *  - A jl_moe handle is not reentrant: calls on one handle must be issued
 *    from one host thread at a time (the reference serialises its global
 *    workspace the same way, session_manager.py:78-87). Different handles
 *    are independent.
 */
#ifndef JOULE_MOE_H
#define JOULE_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define JL_OK 0
#define JL_ERR_INVALID (-1)  /* bad argument or unsupported shape */
#define JL_ERR_OOM (-2)      /* device or pinned-host allocation failed */
#define JL_ERR_CUDA (-3)     /* a CUDA runtime call failed */
#define JL_ERR_TIMEOUT (-4)  /* a bounded device-side wait ran out */
#define JL_ERR_CAPACITY (-5) /* B (or B*topk) above the handle's capacity */
#define JL_ERR_NOT_READY (-6)/* layer weights not uploaded yet */
#define JL_ERR_DEVICE (-7)   /* a kernel reported a bad index / state */

/* Same field order and types as the reference's KernelCfg
 * (decode_kernel.c:269-286, decoder3.py:35-46): a caller's existing struct
 * can be passed unchanged. Only d, E, topk, intermediate, norm_topk_prob
 * and L are read by this library. */
typedef struct {
    int L, d, n_heads, n_kv, hd, E, topk, V;
    float eps;
    int maxT;
    int intermediate;
    int qk_norm_type;
    int bias_qkv;
    int norm_topk_prob;
    int expert_i8;
    int expert_bf16;
} KernelCfg;

/* Same layout as the reference's KernelW (decode_kernel.c:288-325,
 * decoder3.py:49-69). Only gate_w ([L, E, d] bf16) and the Q4 pointer tables
 * expert_pk[p][l*E+e] / expert_sc[p][l*E+e] (p = gate, up, down; the tables
 * built by decoder3.py:329-367) are read, and only as HOST memory. */
typedef struct {
    const unsigned short* embed;
    const unsigned short* lm_head;
    const unsigned short* final_norm;
    const unsigned short* norm1;
    const unsigned short* norm2;
    const unsigned short* wq;
    const unsigned short* wk;
    const unsigned short* wv;
    const unsigned short* wo;
    const float* bq;
    const float* bk;
    const float* bv;
    const unsigned short* qn;
    const unsigned short* kn;
    const unsigned short* gate_w;
    const unsigned short* w1;
    const unsigned short* w2;
    const unsigned short* w3;
    const unsigned char* wq_i8;
    const float* wq_i8s;
    const unsigned char* wk_i8;
    const float* wk_i8s;
    const unsigned char* wv_i8;
    const float* wv_i8s;
    const unsigned char* wo_i8;
    const float* wo_i8s;
    const unsigned char* lm_i8;
    const float* lm_i8s;
    const unsigned char* const* expert_pk[3];
    const unsigned short* const* expert_sc[3];
    const float* cos;
    const float* sin;
    int use_i8;
} KernelW;

/* ------------------------------------------------------------------ */
/* Q4 GEMV / GEMM over the reference's record layout (device pointers). */

/* out[m] = dequant(packed, scales)[m, d] @ x[d].
 * Replaces q4_gemv_f32 (src/jouleai/native/quant_gemv.c:35-57, bound by
 * kernel.py:24-44 and backend.py:92-103). packed: [m, d/2] u8, scales:
 * [m, d/group] fp16 bits, x: [d] fp32, out: [m] fp32 — all device memory.
 * group must be 64 and d a multiple of 64. The sum follows the reference's
 * AVX2 row dot exactly (decode_kernel.c:770-858), so the result is
 * bit-identical to expert_ffn.c's q4_gemv_f32 built for AVX2. */
int jl_q4_gemv_f32(float* out, const float* x, const unsigned char* packed,
                   const unsigned short* scales, int m, int d, int group,
                   void* stream);

/* out[T, m] = X[T, d] @ dequant(W)^T. Replaces q4_gemm_f32
 * (src/jouleai/native/expert_ffn.c:200-215, bound by kernel.py:47-62 and
 * backend.py:119-129). Device pointers; same arithmetic as jl_q4_gemv_f32. */
int jl_q4_gemm_f32(float* out, const float* X, int T,
                   const unsigned char* packed, const unsigned short* scales,
                   int m, int d, int group, void* stream);

/* ------------------------------------------------------------------ */
/* The reference's own symbols, with its signatures (host pointers, void,
 * synchronous), so that its unmodified Python binds this library through
 * get_dll (src/jouleai/native/backend.py:32-42). Inputs are copied to device
 * buffers the library caches per device, the kernel runs on the current
 * device, and the result is back in `out` when the call returns. A failed
 * call (bad argument, no device, CUDA error) fills `out` with NaN and
 * jl_compat_status() returns its JL_ERR_* code. */

/* quant_gemv.c:35-57 (bound by kernel.py:15-41 and ScalarBackend,
 * backend.py:72-91): out[m] = dequant(packed, scales) @ x[d], the scalar
 * loop's order (per byte gacc += lo*x0 + hi*x1; acc += gacc*s per group).
 * group must be 64 and d a multiple of 64. */
void q4_gemv_f32(float* out, const float* x, const unsigned char* packed,
                 const unsigned short* scales, int m, int d, int group);

/* expert_ffn.c:200-215 (bound by kernel.py:43-62 and AVX2Backend,
 * backend.py:94-116): out[T, m] = X[T, d] @ dequant(W)^T in the AVX2 row
 * dot's order, as jl_q4_gemm_f32. T = 0 does nothing. */
void q4_gemm_f32(float* out, const float* X, int T, const unsigned char* packed,
                 const unsigned short* scales, int m, int d, int group);

/* Status of this thread's last q4_gemv_f32 / q4_gemm_f32 call (JL_OK or a
 * JL_ERR_* code). No counterpart in the reference, whose calls return void. */
int jl_compat_status(void);

/* ------------------------------------------------------------------ */
/* Q4 store: on-device quantiser and repack. */

/* Quantise n fp32 values (device) into the reference's Q4 record format:
 * scales [ceil(n/64)] fp16 bits and packed [ceil(n/64)*32] u8 (device).
 * Bit-identical to _quantize_tensor (src/jouleai/storage/q4_store.py:40-55),
 * which convert_experts_q4 (q4_store.py:125-166) applies per expert tensor. */
int jl_q4_quantize(const float* x, long long n, unsigned short* scales,
                   unsigned char* packed, void* stream);

/* ------------------------------------------------------------------ */
/* The MoE layer. */

typedef struct jl_moe jl_moe;

/* Create a handle for one model's MoE layers on the current device.
 * Reads cfg->L, d, E, topk, intermediate, norm_topk_prob. max_tokens is the
 * largest B one forward call may pass (no BMAX=16 clamp as in
 * decode_kernel.c:1522). Allocates the HBM expert store for all L layers and
 * the workspace. Replaces the expert part of NativeDecoder.__init__ /
 * _load_experts (decoder3.py:86-163, 329-367) and ws_init
 * (decode_kernel.c:382-424). */
int jl_moe_create(const KernelCfg* cfg, int max_tokens, jl_moe** out);
int jl_moe_destroy(jl_moe* h);

/* jl_moe_create with flags. JL_CREATE_ROUTER_ONLY allocates the router
 * weights and the workspace but no expert store: such a handle serves
 * jl_moe_upload_router and jl_moe_route only (the routing side of expert
 * parallelism, where each rank stores a slice of the experts in a second
 * handle). No counterpart in the reference, which runs on one host. */
#define JL_CREATE_ROUTER_ONLY 1
int jl_moe_create_ex(const KernelCfg* cfg, int max_tokens, int flags, jl_moe** out);

/* jl_moe_create for stores larger than HBM: all L layers' repacked records
 * live in pinned host memory and only `resident_layers` of them in HBM at a
 * time. A forward of a layer that is not resident first copies it in
 * (cudaMemcpyAsync on the handle's side stream, into the least recently used
 * slot once that slot's last reader has finished; the forward's stream waits
 * for the copy), and every forward prefetches the next layer into another
 * slot, so in-order decode overlaps the copy of layer l+1 with the kernels
 * of layer l. Results are identical to a resident store. Staged handles
 * cannot be captured into CUDA graphs (their copies run on a stream of their
 * own) and cannot serve jl_ep_create. Replaces the reference's on-demand
 * expert loading from its memory-mapped store (decoder3.py:329-367,
 * q4_store.py:169-200). */
int jl_moe_create_staged(const KernelCfg* cfg, int max_tokens, int resident_layers, jl_moe** out);

/* Upload layer l: router rows gate_w [E, d] bf16 and, for each part p in
 * (gate, up, down) and expert e, the Q4 record pk[p*E+e] / sc[p*E+e] in the
 * reference layout (the pointers decoder3.py:355-361 builds). Pointers may
 * be host or device memory (`src_on_device`). The records are repacked into
 * the device tile layout on `stream`; host sources are staged through a
 * pinned buffer. */
int jl_moe_upload_layer(jl_moe* h, int l, const unsigned short* gate_w,
                        const unsigned char* const* pk,
                        const unsigned short* const* sc, int src_on_device,
                        void* stream);

/* Quantise and upload layer l from fp32 weights already on the device:
 * gate_w [E, d] bf16; w_gate/w_up [E, m, d] and w_down [E, d, m] fp32. The
 * store then holds exactly what convert_experts_q4 would have written. */
int jl_moe_quantize_layer(jl_moe* h, int l, const unsigned short* gate_w,
                          const float* w_gate, const float* w_up,
                          const float* w_down, void* stream);

/* Path selection for jl_moe_forward. */
#define JL_PATH_AUTO 0  /* GEMV for B <= 4, tensor-core beyond (d % 512 == 0, m % 256 == 0), else exact */
#define JL_PATH_EXACT 1 /* CUDA-core FP32 in the reference's order (bit-identical outputs) */
#define JL_PATH_TC 2    /* tcgen05 grouped GEMM (fp16 operands, fp32 acc) */
#define JL_PATH_GEMV 3  /* B <= 4: dequantising GEMVs over every SM, exact fp16 (n - 8) weights x
                           fp16 hi + lo activations on mma.sync, fp32 accumulate and scale
                           (<= 1e-3 row-relative); larger B runs as JL_PATH_AUTO */
int jl_moe_set_path(jl_moe* h, int path);

/* One MoE FFN layer: out[B, d] = MoE(x[B, d]) for layer l (device fp32).
 * Replaces layer_ffn_batch (decode_kernel.c:1387-1508) as called from
 * decode_layers_batch[_argmax] (decode_kernel.c:1535, 1577). top/tw
 * (nullable, device) receive the router's top-k ids [B, topk] int32 and
 * weights [B, topk] fp32. Enqueued on `stream`; returns after launch.
 * B = 0 is an empty batch: JL_OK with nothing launched or written (x, out
 * may then be NULL), as the reference's loops run zero times; B < 0 is
 * JL_ERR_INVALID. jl_moe_forward_phases, jl_moe_route, jl_moe_forward_routed,
 * jl_layer_ffn_batch and jl_route_noalloc treat B = 0 the same way. */
int jl_moe_forward(jl_moe* h, int l, const float* x, int B, float* out,
                   int* top, float* tw, void* stream);

/* jl_moe_forward restricted to the phases in `mask` (1 = router + dispatch,
 * 2 = gate/up + SwiGLU, 4 = down + combine; 7 = the full layer). A phase
 * reads what the previous phase of the LAST call left in the workspace, so a
 * partial mask is for profiling one kernel in isolation. No counterpart in
 * the reference. */
int jl_moe_forward_phases(jl_moe* h, int l, const float* x, int B, float* out,
                          int* top, float* tw, int mask, void* stream);

/* Router weights of layer l only: gate_w [E, d] bf16, host or device
 * (`src_on_device`). Synchronises `stream`. For JL_CREATE_ROUTER_ONLY
 * handles this is the whole upload. */
int jl_moe_upload_router(jl_moe* h, int l, const unsigned short* gate_w,
                         int src_on_device, void* stream);

/* Routing of layer l alone (decode_kernel.c:1424-1485): top [B, topk] int32
 * expert ids, tw [B, topk] fp32 weights and, when comb is not NULL,
 * comb [B, topk]: token b's slots b*topk + i in the union order the
 * reference's combine adds them in (decode_kernel.c:1490-1507). Device
 * buffers; enqueued on `stream`. */
int jl_moe_route(jl_moe* h, int l, const float* x, int B, int* top, float* tw,
                 int* comb, void* stream);

/* The expert FFN and combine of layer l with routing supplied by the caller
 * instead of the router: top [B, topk] (expert ids of this handle) and tw
 * [B, topk] (device). out[b] = the combine of b's topk weighted expert
 * outputs, as jl_moe_forward computes it after its own routing. With a
 * topk = 1 handle holding a rank's slice of the experts, this is the
 * remote half of expert parallelism: out[i] = tw[i] * FFN_top[i](x[i]). */
int jl_moe_forward_routed(jl_moe* h, int l, const float* x, int B, const int* top,
                          const float* tw, float* out, void* stream);

/* Expert-parallel bookkeeping for one layer on one rank (no counterpart in
 * the reference, which runs on one host). The S = B*topk routed slots of
 * the rank's tokens (top/tw [B, topk] from jl_moe_route, global expert ids)
 * are grouped by owner rank top / E_local, keeping slot order within a
 * group: pos[s] is slot s's row in send order, counts[w] the rows for rank
 * w, rows [S, d] the token rows x[s / topk] in send order and meta [S, 2]
 * their (local expert id, weight bits). dev_status (device int, 0 before the
 * call) receives error bits for expert ids outside [0, E_local * world).
 * Device buffers; x and rows 16-byte aligned. */
int jl_ep_pack(const int* top, const float* tw, const float* x, int B, int topk,
               int d, int E_local, int world, float* rows, int* meta, int* pos,
               int* counts, int* dev_status, void* stream);

/* out[b] = 0 + back[pos[comb[b*topk]]] + ... + back[pos[comb[b*topk+topk-1]]]
 * in that order: the reference's union-order combine
 * (decode_kernel.c:1490-1507) over rows that came back in send order. */
int jl_ep_combine(const float* back, const int* pos, const int* comb, int B,
                  int topk, int d, float* out, void* stream);

/* Expert parallelism over NVLink peer memory, with no host round trip per
 * layer (no counterpart in the reference). A jl_ep pairs this rank's
 * topk = 1 expert handle `local` (experts [rank*E_local, (rank+1)*E_local),
 * max_tokens >= world * max_tokens_per_rank * topk) with one exported
 * device buffer. Set-up: jl_ep_create on every rank, exchange the 64-byte
 * jl_ep_ipc_handle of every rank (rank order), then jl_ep_open_peers.
 * jl_ep_forward(ep, router, l, x, B, out) runs layer l for this rank's B
 * tokens: route (router: all E experts), send each routed slot's row to
 * its owner's buffer, wait for every sender, run the local experts, return
 * the weighted rows to their senders, wait for every owner, and combine in
 * the batch's union order: out equals a single GPU's jl_moe_forward on the
 * same tokens. Every rank must make the same sequence of calls. Waits on
 * other ranks are bounded; jl_moe_check(local) reports JL_ERR_TIMEOUT.
 * B >= 1 on every rank: a rank takes part in the exchange even when no
 * token of its own routes anywhere, so unlike jl_moe_forward an empty batch
 * is JL_ERR_INVALID here (the caller pads it with one token). */
typedef struct jl_ep jl_ep;
int jl_ep_create(jl_moe* local, int rank, int world, int max_tokens_per_rank,
                 int topk, jl_ep** out);
int jl_ep_ipc_handle(jl_ep* ep, void* handle64);
int jl_ep_open_peers(jl_ep* ep, const void* handles64);
int jl_ep_forward(jl_ep* ep, jl_moe* router, int l, const float* x, int B,
                  float* out, void* stream);
int jl_ep_destroy(jl_ep* ep);

/* Peer r of `ep` is `peer`, a jl_ep of the same world created in this
 * process (ranks driven from one process: no IPC handle; on another device
 * peer access is enabled). In place of jl_ep_open_peers for that rank. */
int jl_ep_attach(jl_ep* ep, int r, jl_ep* peer);

/* Bound of each device-side wait on other ranks, in nanoseconds (default
 * about 2 s). A wait that runs out sets JL_ERR_TIMEOUT on the local expert
 * handle (jl_moe_check), the layer's output is then not valid, and the
 * rank's epochs no longer match its peers': destroy and recreate every
 * rank's jl_ep before the next layer. */
int jl_ep_set_wait_limit(jl_ep* ep, long long ns);

/* Phase timing of jl_ep_forward: events (cudaEvent_t, n <= 9) recorded on
 * the call's stream before routing, then after routing, the send, the
 * receive (its wait included), the dispatch, gate/up, down, the return and
 * the final combine (its wait included). n = 0 turns it off. */
int jl_ep_set_phase_events(jl_ep* ep, void* const* events, int n);

/* Rows this rank received as an owner (summed over calls) and the number of
 * calls, since the previous jl_ep_stats; resets both. Synchronises
 * `stream`. */
int jl_ep_stats(jl_ep* ep, long long* rows, long long* calls, void* stream);

/* Debug / parity: copies (device) the router logits [B, E], the union
 * experts sel [U], offsets uh [U+1] and the slot map uidx/uw [B*topk] built
 * by the last jl_moe_forward (decode_kernel.c:1424-1485). *U_out (host)
 * receives U. Synchronises `stream`. */
int jl_moe_debug_routing(jl_moe* h, int B, float* logits, int* sel, int* uh,
                         int* uidx, float* uw, int* U_out, void* stream);

/* Read and clear the handle's device error word (bounded waits that ran
 * out, bad expert ids). Synchronises `stream`. Returns JL_OK or the error. */
int jl_moe_check(jl_moe* h, void* stream);

/* Host-buffer drop-in for layer_ffn_batch(c, W, l, x, B, out)
 * (decode_kernel.c:1387): x and out are HOST fp32 [B, d]. On first use of a
 * (c, W) pair the L layers of W's expert tables are uploaded to a cached
 * handle; each call copies x to the device, runs jl_moe_forward and copies
 * out back (synchronous). */
int jl_layer_ffn_batch(const KernelCfg* c, const KernelW* W, int l,
                       const float* x, int B, float* out);

/* Device-side trace (the counterpart of the reference's g_trace breadcrumbs,
 * decode_kernel.c:22-28): with enable = 1 the kernels of later forwards stamp
 * %globaltimer (ns) at phase boundaries into a 128-slot device buffer: rows
 * of 16 slots for the router, gate/up, down and combine kernels (thread 0 of
 * one block), then rows 4 and 5 with the SM-clock cycles that block 0 of the
 * tensor-core gate/up and down kernels spent in each role's waits, MMA issue
 * and dequantisation, and each role's total (they add
 * up over launches). out (host, n slots) receives the buffer (synchronises
 * `stream`); enable = 1 with n = 0 zeroes it; enable = 0 stops later launches
 * from tracing. The buffer stays allocated until jl_moe_destroy, because CUDA
 * graphs captured while tracing keep writing to it. */
int jl_moe_trace(jl_moe* h, int enable, long long* out, int n, void* stream);

/* Phase timing: when n > 0, each jl_moe_forward[_phases] records events[0]
 * before the router, events[1] after it, events[2] after gate/up+SwiGLU and
 * events[3] after down+combine (n < 4 records the first n), on the forward's
 * stream; under stream capture they become external event-record nodes.
 * events are cudaEvent_t handles; n = 0 turns it off. No counterpart in the
 * reference (its profiling is wall-clock, batch_bench.py:58-68). */
int jl_moe_set_phase_events(jl_moe* h, void* const* events, int n);

/* Router + softmax/top-k (+ optional renorm) for B <= 64 tokens with no
 * device allocation and no handle. No counterpart in the reference.
 * gate_w [E, d] bf16 and x [B, d] fp32 are device memory, 16-byte aligned;
 * top [B, topk] int32 and tw [B, topk] fp32 (device) receive the same ids
 * and weights as jl_moe_forward's top/tw. The [B, E] logits go to a static
 * 64 KiB device array (64 tokens x 256 experts), one per device, so:
 * B > 64 returns JL_ERR_CAPACITY and E > 256 JL_ERR_INVALID; calls on one
 * device must not overlap (one stream, or ordered by events); the first call
 * on a device performs a one-time setup that must precede any stream
 * capture. dev_status (device int, required; NULL is JL_ERR_INVALID) must
 * hold 0 before the call; the kernels OR bit 1 into it when a bounded wait
 * runs out, and top/tw are then not valid. For hosts that must not allocate
 * per request. */
int jl_route_noalloc(const unsigned short* gate_w, const float* x, int B, int E,
                     int d, int topk, int norm_topk_prob, int* top, float* tw,
                     int* dev_status, void* stream);

/* ------------------------------------------------------------------ */
/* The whole decode step on the GPU: norms, attention, the MoE layers, the
 * lm_head and the argmax, in the reference's arithmetic order. */

/* The reference's KV cache entry (decode_kernel.c:328-331): kv[b*L + l] holds
 * sequence b's layer-l keys and values, each [maxT, n_kv, hd] fp32. */
typedef struct {
    float* k;
    float* v;
} KVCache;

typedef struct jl_dec jl_dec;

/* A decoder on the current device: uploads every weight KernelW names (host
 * memory, or device memory when src_on_device; lm_head is fp32 [V, d] as
 * decoder3.py:218-230 stores it) into the device layout, creates the MoE
 * handle (its Q4 layers from W's expert tables; when expert_pk[0] is NULL
 * they are left for jl_dec_moe + jl_moe_upload_layer / jl_moe_quantize_layer)
 * and KV caches of `slots` sequences x L layers x maxT rows. max_batch is the
 * most sequences one step may run. Replaces what NativeDecoder.__init__
 * (decoder3.py:86-163) and ws_init (decode_kernel.c:382-424) set up. */
int jl_dec_create(const KernelCfg* c, const KernelW* W, int max_batch, int slots,
                  int src_on_device, jl_dec** out);
int jl_dec_destroy(jl_dec* h);

/* The decoder's MoE handle (to upload experts, or set its path). */
int jl_dec_moe(jl_dec* h, jl_moe** moe);

/* Device base pointers of the K and V caches, [slots][L][maxT][n_kv*hd] fp32. */
int jl_dec_kv(jl_dec* h, float** k, float** v);

/* x[b] = bf16 embed[tokens[b]] as fp32 (embed_lookup, decode_kernel.c:1597-1600);
 * tokens [B] and x [B, d] device. */
int jl_dec_embed(jl_dec* h, const int* tokens, int B, float* x, void* stream);

/* One batched decode step (decode_layers_batch[_argmax], decode_kernel.c:
 * 1518-1586) for B sequences: sequence b is KV slot slots[b] at position
 * positions[b] (its rows [0, positions[b]) already in the cache; this step
 * appends row positions[b] of every layer), input x[b] (embedded, fp32 [d]).
 * logits [B, V] and tok [B] (argmax, lowest index on ties) are nullable
 * device outputs. All pointers device; enqueued on `stream`. With the MoE
 * handle on JL_PATH_EXACT the logits equal the reference's bit for bit. */
int jl_dec_step(jl_dec* h, const int* slots, const int* positions, const float* x, int B,
                float* logits, int* tok, void* stream);

/* Batched prefill of one sequence: tokens [T] (device ids) at positions
 * pos0 .. pos0+T-1 of KV slot `slot`, max_batch positions per pass (each
 * pass appends its K/V rows before its attention reads them; the MoE
 * layers add each token's experts in its own top-k order). The logits [V]
 * and argmax tok [1] (nullable, device) are the last position's. With the
 * MoE handle on JL_PATH_EXACT every position gets the bits of the
 * reference's one-position steps (prefill_layers, decode_kernel.c:
 * 1606-1615); decoder3.py:512-571 (prefill_batch) runs prompts this way. */
int jl_dec_prefill(jl_dec* h, int slot, const int* tokens, int T, int pos0, float* logits,
                   int* tok, void* stream);

/* Read and clear the decoder's error word and its MoE handle's
 * (synchronises): JL_ERR_INVALID for a position outside [0, maxT). */
int jl_dec_check(jl_dec* h, void* stream);

/* The reference's own decode entry points with its signatures (host
 * buffers, void, synchronous), bound through get_dll("decode_kernel") by
 * NativeDecoder (decoder3.py:32, 490-629). One decoder per (cfg, W) is
 * created on first use (weights uploaded from W, MoE on the exact path) for
 * up to 32 sequences per call. The library keeps a device copy of each
 * sequence's KV cache (a sequence is identified by its kv[b*L].k pointer):
 * a call at position p uses that copy when it holds exactly p rows, and
 * otherwise first copies the host rows [0, p) of every layer over; after
 * the step the new row of every layer is written back to the host caches.
 * A failed call fills logits with NaN (out_tok with -1) and
 * jl_decode_status() returns its JL_ERR_* code.
 *   decode_layers_batch: decode_kernel.c:1518-1556 (logits [B, V] host)
 *   decode_layers_batch_argmax: decode_kernel.c:1560-1586 (out_tok [B]; the
 *     argmax of the logits, lowest index on ties)
 *   decode_layers: decode_kernel.c:1588-1595 (B = 1)
 *   embed_lookup: decode_kernel.c:1597-1600 */
void decode_layers_batch(const KernelCfg* c, const KernelW* W, KVCache* kv,
                         const int* positions, const float* xin, int B, float* logits);
void decode_layers_batch_argmax(const KernelCfg* c, const KernelW* W, KVCache* kv,
                                const int* positions, const float* xin, int B, int* out_tok);
void decode_layers(const KernelCfg* c, const KernelW* W, KVCache* kv, int pos,
                   const float* xin, float* logits);
void embed_lookup(const KernelW* W, const KernelCfg* c, int token, float* out);

/* prefill_layers (decode_kernel.c:1606-1615): one B = 1 step per position
 * 0..T-1 of one sequence; logits [V] (host) of the last position. */
void prefill_layers(const KernelCfg* c, const KernelW* W, KVCache* kv, const int* tokens,
                    int T, float* logits);

/* debug_decode_layers (decode_kernel.c:1764-1790): one B = 1 step at pos;
 * out (host) receives per layer 7 rows of max(E, d) floats: norm1 output,
 * attention output, h after attention, norm2 output, router logits, MoE
 * output, h after the MoE layer. */
void debug_decode_layers(const KernelCfg* c, const KernelW* W, KVCache* kv, int pos,
                         const float* xin, float* out);

/* The reference's host thread-pool controls (decode_kernel.c:631, 1843),
 * called by NativeDecoder at start-up (decoder3.py:133-145). This library
 * has no host pool: spin_pool_init returns 1 (success) and set_lm_threads
 * does nothing. */
int spin_pool_init(int n_workers);
void set_lm_threads(int n);

/* Status of this thread's last reference-signature decode call. No
 * counterpart in the reference. */
int jl_decode_status(void);

/* Bytes of device memory the handle holds (store + workspace). */
long long jl_moe_device_bytes(const jl_moe* h);

/* Library version string, e.g. "joule_b200 0.1 sm_100a". */
const char* jl_version(void);

/* Text of the CUDA runtime error behind the most recent JL_ERR_CUDA of any
 * call in this process ("" when none). No counterpart in the reference,
 * whose calls return void. */
const char* jl_last_cuda_error(void);

#ifdef __cplusplus
}
#endif
#endif
