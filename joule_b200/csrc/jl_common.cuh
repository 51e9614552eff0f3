// Shared device helpers for the sm_100a MoE kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "joule_moe.h"

// Records a failed CUDA runtime call (jl_last_cuda_error) and returns JL_ERR_CUDA.
int jl_note_cuda(cudaError_t e);

#define JL_CUDA(call)                                   \
    do {                                                \
        cudaError_t _e = (call);                        \
        if (_e != cudaSuccess) return jl_note_cuda(_e); \
    } while (0)

#define JL_LAUNCH_CHECK()                                   \
    do {                                                    \
        if (cudaGetLastError() != cudaSuccess) return JL_ERR_CUDA; \
    } while (0)

namespace jl {

constexpr int kGroup = 64;        // Q4 group (q4_store.py:23)
constexpr int kGroupBytes = 32;   // packed bytes per group
constexpr int kTileRows = 32;     // rows per device tile
constexpr int kTileBytes = kTileRows * kGroupBytes;  // 1024 packed bytes per tile
constexpr int kTileRec = kTileBytes + kTileRows * 2;  // 1088: a tile's packed bytes + its 32 scales

// Device error codes written into a handle's error word.
constexpr int kErrTimeout = 1;
constexpr int kErrBadExpert = 2;
constexpr int kErrCapacity = 4;

// ---------------------------------------------------------------------------
// Exact scalar conversions and the reference's expf_fast.

// bf16 bits -> fp32 (decode_kernel.c:47-53): the bits are the top half.
__device__ __forceinline__ float bf16_to_f32(uint32_t h) {
    return __uint_as_float(h << 16);
}

// fp16 bits -> fp32, exactly as decode_kernel.c:64-85 (subnormals
// normalised, inf/NaN payload kept).
__device__ __forceinline__ float fp16_to_f32(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1Fu;
    const uint32_t man = h & 0x3FFu;
    if (ex == 0u) {
        // man * 2^-24 is exact in fp32 for man < 1024
        const float v = __fmul_rn(__uint2float_rn(man), 5.9604644775390625e-8f);
        return __uint_as_float(__float_as_uint(v) | sign);
    }
    if (ex == 31u) return __uint_as_float(sign | 0x7F800000u | (man << 13));
    return __uint_as_float(sign | ((ex + 112u) << 23) | (man << 13));
}

// The reference's own expf approximation (decode_kernel.c:94-108), with every
// product and sum rounded separately as in its C source. Written without
// branches (its early returns become selects, same results for every input,
// NaN included), so that several calls interleave in one thread.
__device__ __forceinline__ float expf_fast(float v) {
    const bool under = v < -17.0f;
    v = v > 88.0f ? 88.0f : v;
    const float y = __fmul_rn(v, 1.4426950408889634f);
    const int k = __float2int_rz(__fadd_rn(y, y >= 0.0f ? 0.5f : -0.5f));
    const float f = __fsub_rn(y, __int2float_rn(k));
    float p = 0.0013330f;
    p = __fadd_rn(0.0096181f, __fmul_rn(f, p));
    p = __fadd_rn(0.0555041f, __fmul_rn(f, p));
    p = __fadd_rn(0.2402265f, __fmul_rn(f, p));
    p = __fadd_rn(0.6931472f, __fmul_rn(f, p));
    p = __fadd_rn(1.0f, __fmul_rn(f, p));
    const int kk = k + 127;
    const float r = __fmul_rn(p, __uint_as_float((uint32_t)min(max(kk, 0), 254) << 23));
    return (under || kk < 0) ? 0.0f : r;
}

// silu(g) * u as the reference writes it: (g / (1 + expf_fast(-g))) * u.
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float den = __fadd_rn(1.0f, expf_fast(-g));
    return __fmul_rn(__fdiv_rn(g, den), u);
}

// The same with the division by __fdividef (within 2 ulp for den <= 2^126; den
// >= 1, and above 2^126 it returns 0 where the exact quotient is below 1e-36),
// for the tensor-core path, whose results are held to a relative tolerance.
__device__ __forceinline__ float silu_mul_approx_div(float g, float u) {
    const float den = __fadd_rn(1.0f, expf_fast(-g));
    return __fmul_rn(__fdividef(g, den), u);
}

// Horizontal sum of an 8-lane AVX accumulator in the reference's order
// (decode_kernel.c:843-846): ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)).
__device__ __forceinline__ float hsum8(const float (&l)[8]) {
    const float s0 = __fadd_rn(l[0], l[4]), s1 = __fadd_rn(l[1], l[5]);
    const float s2 = __fadd_rn(l[2], l[6]), s3 = __fadd_rn(l[3], l[7]);
    return __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
}

// Eight Q4 values of one 32-bit word as exact floats (nib - 8), as four
// float2 pairs (elements 2i, 2i+1). Element j of the word is nibble j (bits
// 4j..4j+3): byte j/2, low nibble first (q4_store.py:53). Each nibble is
// OR-ed into the mantissa of 2^23 at its own bit position and rescaled by an
// exact packed FMA (v * 2^-4j - (2^(23-4j) + 8) is exact), so only one shift
// per word is needed.
__device__ __forceinline__ void dequant8x2(uint32_t w, float2 (&a)[4]) {
    const uint32_t M = 0x4B000000u;  // 2^23
    const uint32_t h = w >> 12;      // nibbles 5..7 -> bits 8..19
    const float2 v0 = make_float2(__uint_as_float((w & 0x0000000Fu) | M),
                                  __uint_as_float((w & 0x000000F0u) | M));
    const float2 v1 = make_float2(__uint_as_float((w & 0x00000F00u) | M),
                                  __uint_as_float((w & 0x0000F000u) | M));
    const float2 v2 = make_float2(__uint_as_float((w & 0x000F0000u) | M),
                                  __uint_as_float((h & 0x00000F00u) | M));
    const float2 v3 = make_float2(__uint_as_float((h & 0x0000F000u) | M),
                                  __uint_as_float((h & 0x000F0000u) | M));
    a[0] = __ffma2_rn(v0, make_float2(1.0f, 0.0625f), make_float2(-8388616.0f, -524296.0f));
    a[1] = __ffma2_rn(v1, make_float2(0.00390625f, 0.000244140625f), make_float2(-32776.0f, -2056.0f));
    a[2] = __ffma2_rn(v2, make_float2(1.52587890625e-05f, 0.00390625f), make_float2(-136.0f, -32776.0f));
    a[3] = __ffma2_rn(v3, make_float2(0.000244140625f, 1.52587890625e-05f), make_float2(-2056.0f, -136.0f));
}

// Scalar form of dequant8x2 (same values).
__device__ __forceinline__ void dequant8(uint32_t w, float (&a)[8]) {
    float2 p[4];
    dequant8x2(w, p);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        a[2 * i] = p[i].x;
        a[2 * i + 1] = p[i].y;
    }
}

// hsum8 over four float2 lane pairs {l0,l1},{l2,l3},{l4,l5},{l6,l7}.
__device__ __forceinline__ float hsum8x2(const float2 (&l)[4]) {
    const float2 s01 = __fadd2_rn(l[0], l[2]);  // (l0+l4, l1+l5)
    const float2 s23 = __fadd2_rn(l[1], l[3]);  // (l2+l6, l3+l7)
    const float2 t = __fadd2_rn(s01, s23);      // (s0+s2, s1+s3)
    return __fadd_rn(t.x, t.y);
}

// fp16 bits -> fp32 by the hardware conversion: exact for every finite half
// (subnormals included), equal to fp16_to_f32 except for NaN payloads.
__device__ __forceinline__ float half_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// ---------------------------------------------------------------------------
// Bounded waits, mbarriers and 1-D bulk copies (TMA, no multicast).

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of an mbarrier with a time bound. The bound is
// counted in SM clock cycles (clock64 is cheap to read; %globaltimer is not),
// checked every 64 polls: 4e9 cycles is at least 2 s at any B200 SM clock.
// On timeout the error word gets kErrTimeout and false is returned.
constexpr long long kWaitLimitCycles = 4000000000ll;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (int i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0 && clock64() - t0 > kWaitLimitCycles) {
            if (err) atomicOr(err, kErrTimeout);
            return false;
        }
    }
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy ones (bulk copies, tensor-core operand reads) on the same bytes:
// a consumer that read a ring stage with plain loads runs it before releasing
// the stage to the producer's next bulk copy.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Global -> shared bulk copy completing on `bar` (bytes % 16 == 0, both
// addresses 16-byte aligned). Source is this GPU's own memory; no multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 cache policies for bulk copies: expert weights stream through once per
// layer (evict first); router rows are re-read every decode step (evict last).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_g2s with an L2 cache policy (same address and size rules).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Prefetch [p, p + bytes) of this GPU's own memory into L2 (p 16-byte aligned,
// bytes a multiple of 16); no data is returned and no completion is tracked.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Per-thread asynchronous global -> shared copies (16 bytes, both addresses
// 16-byte aligned), completed by commit / wait groups.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// 4-byte form (both addresses 4-byte aligned), through L1 (.ca is the only form below 16 bytes).
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Phase stamp for the optional trace buffer (thread 0 of the calling block).
__device__ __forceinline__ void trace_point(long long* trace, int kind, int slot) {
    if (trace != nullptr && threadIdx.x == 0) trace[kind * 16 + slot] = (long long)globaltimer_ns();
}

__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch with programmatic dependent launch (PDL) enabled: the kernel may
// start while the previous kernel on the stream finishes; it must call
// griddep_wait() before touching that kernel's outputs.
template <typename... KArgs, typename... Args>
inline int launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                  Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    return e == cudaSuccess ? JL_OK : jl_note_cuda(e);
}

}  // namespace jl
