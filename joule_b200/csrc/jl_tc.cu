// Tensor-core (tcgen05) path of the expert FFN for larger batches.
//
// Per layer, after routing:
//   tc_build_tiles (end of the dispatch step) cuts every union expert's
//                 tokens into tiles of <= kTcNT = 32 (padded to 16 or 32).
//   k_tc_permute  gathers each tile's tokens and writes them as fp16 hi/lo
//                 pairs (x = hi + lo, ~22 significant bits) in the UMMA
//                 K-major "interleaved" core layout, hi rows then lo rows, so
//                 one MMA of N = 2 x tokens covers both (the epilogue adds the
//                 two accumulator halves). Pad rows are left unwritten.
//   k_expert_tc<false> (gate/up) a persistent grid, one CTA per SM walking
//                 items (tile, 64 gate rows + the matching 64 up rows): a
//                 producer warp streams the Q4 tiles (6-stage ring of 17 KB
//                 bulk copies), another the token tiles (2-stage ring); four
//                 dequant warpgroups turn each 64-value group into fp16
//                 (n - 8) * scale (correctly rounded) and store it straight
//                 into tensor memory as the MMA's A operand (lane = weight
//                 row); two issuer warps run tcgen05.mma (M=128, N=2 x tokens,
//                 K=16, fp32 accumulate in TMEM). The epilogue reads the
//                 accumulators with tcgen05.ld, applies SwiGLU and writes the
//                 activations (hi/lo, same core layout) for down.
//   k_expert_tc<true> (down) the same pipeline over the down matrix (M=128
//                 rows of d, K = intermediate); the epilogue writes
//                 y[slot] = w * acc.
//   k_combine     (jl_exact.cu) sums y in the reference's union order.
//
// K order inside each 8-value chunk is permuted identically in A and B
// (position p holds element kPerm[p]) so that the fp16 pairs produced by the
// dequantiser land in TMEM columns without shuffles; a dot product does not
// depend on the order of its terms' pairing, only its rounding does.
//
// Every mbarrier wait is bounded; a timeout sets the handle's error word and
// an abort flag that makes every role leave its loop, after which the CTA
// frees its tensor memory and exits.
#include <algorithm>

#include "jl_common.cuh"
#include "jl_internal.h"
#include "jl_tiles.cuh"

namespace jl {

constexpr int kTcQ4Stage = 4 * kTileRec;  // the 4 contiguous tile records of one K step
// position p of an 8-value K chunk holds element kPerm[p] = {0,4,1,5,2,6,3,7}[p]

__host__ __device__ inline int tc_max_tiles(int S, int E) { return S / kTcNT + E + 1; }

// ---------------------------------------------------------------------------
// small PTX helpers

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
        "}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
        "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]),
        "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),
        "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
        "%12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// 16 tokens' results from the two issuers' accumulators (each: hi columns
// [0, N), lo columns [N, 2N)), added in a fixed order: (hi0 + hi1) + (lo0 +
// lo1). The four loads are issued before one wait.
__device__ __forceinline__ void tc_ld_acc16(uint32_t acc0, uint32_t acc1, int N, int t0, float (&v)[16]) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%64];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%65];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47}, [%66];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%67];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(acc0 + t0), "r"(acc1 + t0), "r"(acc0 + N + t0), "r"(acc1 + N + t0)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++)
        v[i] = (__uint_as_float(r[i]) + __uint_as_float(r[16 + i])) +
               (__uint_as_float(r[32 + i]) + __uint_as_float(r[48 + i]));
}

// UMMA shared-memory descriptor, K-major, no swizzle: core matrices of 8 rows
// x 16 bytes; `lbo` = bytes between the two 8-value K halves of one MMA,
// `sbo` = bytes between 8-row groups.
__device__ __forceinline__ uint64_t umma_desc(const void* smem, uint32_t lbo, uint32_t sbo) {
    const uint64_t a = (uint64_t)((smem_u32(smem) >> 4) & 0x3FFF);
    return a | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) | ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) |
           (1ull << 46);  // descriptor version 1 (sm_100); layout type 0 = no swizzle
}

// kind::f16 instruction descriptor: fp16 A and B (K-major), fp32 D, M=128.
__device__ __forceinline__ uint32_t umma_idesc_f16(int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// Role wait counters of CTA 0 when the device trace is on (rows 4 / 5 of
// the trace buffer for gate/up / down): cycles spent in each wait, summed in
// registers (dgl) and written once when the role ends, so that the counting
// adds no memory round trip to the role it times. Only the kTrace instance of
// the kernel (launched while tracing) reads the clock; the other instance
// compiles the plain wait.
#define TC_TIMED(slot, expr)                                              \
    ([&]() {                                                              \
        if constexpr (kTrace) {                                           \
            const long long _c0 = clock64();                              \
            const bool _r = (expr);                                       \
            dgl[slot] += clock64() - _c0;                                 \
            return _r;                                                    \
        } else {                                                          \
            return (bool)(expr);                                          \
        }                                                                 \
    }())

// Bounded mbarrier wait that also gives up when another role aborted.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int* err,
                                        volatile int* abort) {
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

// Bounded wait for roles off the critical path (the epilogue waits a whole
// item for its accumulators): polls are spaced by a short sleep so the
// waiting warp leaves the issue slots to the dequant warps.
__device__ __forceinline__ bool tc_wait_relaxed(uint64_t* bar, uint32_t parity, int* err,
                                                volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (int i = 1;; i++) {
        __nanosleep(128);
        if (mbar_try_wait(bar, parity)) return true;
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

// Warp-wide form for the warps that go on to tcgen05.ld / tcgen05.st: those
// are .sync.aligned, so every lane must leave the spin together and agree on
// the outcome (each lane polls on its own and may exit at another iteration).
__device__ __forceinline__ bool tc_wait_warp(uint64_t* bar, uint32_t parity, int* err,
                                             volatile int* abort) {
    return __all_sync(0xffffffffu, tc_wait(bar, parity, err, abort));
}

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\telect.sync r|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// 64 Q4 values of one row (32 bytes) -> 32 words of fp16 pairs (n - 8) * s,
// pair order per 8-value chunk: (e0,e4) (e1,e5) (e2,e6) (e3,e7) = kPerm.
__device__ __forceinline__ void dequant_row_f16(uint4 q0, uint4 q1, __half s, uint32_t (&out)[32]) {
    const uint32_t wq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const __half2 s2 = __halves2half2(s, s);
    const __half2 c1032 = __float2half2_rn(-1032.0f);
    const __half2 c16 = __float2half2_rn(0.0625f);
    const __half2 c72 = __float2half2_rn(-72.0f);
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const uint32_t v = wq[w], v8 = v >> 8;
        // halves: low half holds nibble j, high half nibble j+4 (element order within the word)
        const __half2 h0 = u32_as_h2((v & 0x000F000Fu) | 0x64006400u);   // (e0, e4) + 1024
        const __half2 h1 = u32_as_h2((v & 0x00F000F0u) | 0x64006400u);   // (e1, e5)*16 + 1024
        const __half2 h2 = u32_as_h2((v8 & 0x000F000Fu) | 0x64006400u);  // (e2, e6) + 1024
        const __half2 h3 = u32_as_h2((v8 & 0x00F000F0u) | 0x64006400u);  // (e3, e7)*16 + 1024
        out[4 * w + 0] = h2_as_u32(__hmul2(__hadd2(h0, c1032), s2));
        out[4 * w + 1] = h2_as_u32(__hmul2(__hfma2(h1, c16, c72), s2));
        out[4 * w + 2] = h2_as_u32(__hmul2(__hadd2(h2, c1032), s2));
        out[4 * w + 3] = h2_as_u32(__hmul2(__hfma2(h3, c16, c72), s2));
    }
}

// Split 8 fp32 values (one K chunk, natural order) into hi/lo fp16 chunks in
// kPerm order: position p holds element kPerm[p] = {0,4,1,5,2,6,3,7}[p].
__device__ __forceinline__ void split_chunk(const float (&x)[8], uint4& hi, uint4& lo) {
    const int perm[8] = {0, 4, 1, 5, 2, 6, 3, 7};
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float a = x[perm[2 * i]], b = x[perm[2 * i + 1]];
        const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
        const __half la = __float2half_rn(a - __half2float(ha));
        const __half lb = __float2half_rn(b - __half2float(hb));
        h[i] = h2_as_u32(__halves2half2(ha, hb));
        l[i] = h2_as_u32(__halves2half2(la, lb));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// ---------------------------------------------------------------------------
// Activation gather: grid = (max tiles, d / 512), block 256. Block (t, y)
// writes K chunks [64y, 64y + 64) of tile t's n token rows as fp16 hi/lo in
// core layout. The pad rows n..N-1 are not written: an MMA column depends
// only on its own B row, and the epilogues drop the pad columns, so whatever
// the pad rows hold (left from earlier tiles) never reaches a result.
__global__ void __launch_bounds__(256) k_tc_permute(const float* __restrict__ x, int d, int k,
                                                    jl_ws ws) {
    long long* tr = (blockIdx.x == 0 && blockIdx.y == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceCombine, 8);
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceCombine, 9);
    const int ti = blockIdx.x;
    if (ti >= *ws.tc_ntiles) return;
    const int n = ws.tc_tile[ti * 4 + 1], N = (n + 15) & ~15;
    const int pos0 = ws.tc_tile[ti * 4 + 2], row0 = ws.tc_tile[ti * 4 + 3];
    const int kc0 = blockIdx.y * 64, kcn = min(64, d / 8 - kc0);
    // the tile's token rows (at most kTcNT), read once
    __shared__ int brow[kTcNT];
    if (threadIdx.x < n) brow[threadIdx.x] = ws.uidx[pos0 + threadIdx.x] / k;
    __syncthreads();
    // tile layout: [kc][2N rows: hi rows 0..N-1, lo rows N..2N-1][8 halves].
    // Each thread loads all of its chunks before converting and storing any,
    // so the loads of one thread overlap.
    __half* base = ws.xc + (size_t)2 * row0 * d;
    constexpr int kPer = kTcNT * 64 / 256;  // chunks per thread at the largest tile (N = kTcNT)
    float4 va[kPer], vc[kPer];
#pragma unroll
    for (int q = 0; q < kPer; q++) {
        const int i = threadIdx.x + q * 256;
        const int r = i % N, kc = kc0 + i / N;
        va[q] = vc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < N * kcn && r < n) {
            const float* src = x + (size_t)brow[r] * d + kc * 8;
            va[q] = __ldg(reinterpret_cast<const float4*>(src));
            vc[q] = __ldg(reinterpret_cast<const float4*>(src + 4));
        }
    }
#pragma unroll
    for (int q = 0; q < kPer; q++) {
        const int i = threadIdx.x + q * 256;
        const int r = i % N, kc = kc0 + i / N;
        if (i < N * kcn && r < n) {
            uint4 vh, vl;
            const float v[8] = {va[q].x, va[q].y, va[q].z, va[q].w, vc[q].x, vc[q].y, vc[q].z, vc[q].w};
            split_chunk(v, vh, vl);
            __half* blk = base + (size_t)kc * 2 * N * 8;
            *reinterpret_cast<uint4*>(blk + r * 8) = vh;
            *reinterpret_cast<uint4*>(blk + (N + r) * 8) = vl;
        }
    }
    trace_point(tr, kTraceCombine, 10);
}

// ---------------------------------------------------------------------------
// Persistent grouped GEMM (gate/up and down). One CTA per SM walks the work
// items blockIdx.x, blockIdx.x + gridDim.x, ... where an item is one token
// tile x one block of 128 weight rows (gate/up: 64 gate + 64 up rows). Each
// role walks the same item sequence, so the rings run on across items. Roles:
//   warps 0-3   epilogue: thread = accumulator row = TMEM lane
//   warps 4-19  dequant warpgroups 0-3: warpgroup g dequantises the K-step
//               pairs P = g (mod 4) into TMEM A buffer g
//   warp 20     weight producer: 6 stages of 4 K steps (17,408 B, one bulk copy)
//   warp 21     activation producer: 2 stages of 32 KB (one bulk copy each)
//   warps 22-23 MMA issuers: issuer w takes the K-step pairs of parity w into
//               its own accumulator; the epilogue adds the two in a fixed order
// TMEM (512 columns): 4 A buffers of 64 columns (one pair of 64-value K steps),
// then accumulators [issuer][buffer] of 2 x kTcNT columns; items alternate
// buffers, so the epilogue of item i overlaps the main loop of item i + 1.
// Two costs shape this: a bulk copy costs its issuing thread a few hundred
// nanoseconds whatever its size (4 KB copies cap an SM near 20 GB/s; 16 KB
// and larger reach its HBM share), and a tcgen05.mma costs its issuing
// thread tens of cycles whatever N is (issued from a converged warp through
// elect.sync: a lone diverged lane issues about half as fast), while the
// tensor core takes several issuers' MMAs at once. The hand-off from the
// dequant warps (TMEM store, wait, fence, arrive) costs a few hundred cycles,
// so it runs once per pair of K steps. A buffer b always serves the pairs
// P = b (mod 4), i.e. one warpgroup and one issuer (b % 2). Each dequant warp
// arrives once on a barrier (after __syncwarp), not once per thread: 256
// arrivals on one mbarrier per stage serialise in the shared-memory atomics.
constexpr int kPQK = 4;    // K steps per weight stage: one 17,408-byte bulk copy
constexpr int kPQ = 6;     // weight stages
constexpr int kPBBytes = 32 * 1024;  // activation stage: 8 / (N/16) K steps of 2N rows
constexpr int kPB = 2;     // activation stages
constexpr int kPA = 4;     // TMEM A buffers (one K-step pair, 64 columns, each)
constexpr int kPI = 2;     // MMA issuers
constexpr int kPDq = 4;    // dequant warpgroups: warpgroup g fills TMEM A buffer g
constexpr int kPAccCols = 2 * kTcNT;  // accumulator columns (hi + lo rows of a tile)
constexpr int kWProd = 4 + 4 * kPDq;  // weight producer warp
constexpr int kWAct = kWProd + 1;     // activation producer warp
constexpr int kWMma = kWProd + 2;     // first MMA issuer warp (it also owns the TMEM allocation)
constexpr int kPWarps = kWMma + kPI;
static_assert(kPA == kPDq && kPA % kPI == 0, "A buffer g belongs to warpgroup g and issuer g % kPI");
constexpr int kPThreads = kPWarps * 32;
constexpr int kPStage = kPQK * kTcQ4Stage;
// TMEM column of accumulator (issuer w, buffer b): after the A buffers
__host__ __device__ constexpr int p_acc_col(int w, int b) { return kPA * 64 + (2 * w + b) * kPAccCols; }
static_assert(p_acc_col(kPI - 1, 1) + kPAccCols <= 512, "TMEM columns");

struct PSmem {
    uint64_t q4_full[kPQ], q4_empty[kPQ];
    uint64_t b_full[kPB], b_empty[kPB];
    uint64_t a_full[kPA], a_empty[kPA];
    uint64_t acc_full[kPI][2], acc_empty[2];
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(PSmem) <= 512, "barrier block");
constexpr size_t kPQ4Off = 512;
constexpr size_t kPBOff = kPQ4Off + (size_t)kPQ * kPStage;
constexpr size_t kPScrOff = kPBOff + (size_t)kPB * kPBBytes;
constexpr size_t kPScratch = 32 * 1024;  // gate/up epilogue: gate + up rows fp32 [128][33] + act hi/lo [2][32][64]
constexpr size_t kPSmemBytes = kPScrOff + kPScratch;

// K steps per activation stage for a tile of N (16 or 32) token rows: a
// multiple of kPI, so every issuer has steps in every stage
__device__ __forceinline__ int p_bsteps(int N) { return 8 / (N >> 4); }
__device__ __forceinline__ int p_lbsteps(int N) { return N == 16 ? 3 : 2; }  // log2(p_bsteps(N))
static_assert(128 * (kTcNT + 1) * 4 + 2 * kTcNT * 64 * 2 <= kPScratch, "epilogue scratch");
static_assert(kTcNT == 32 && kPA == 4 && kPB == 2, "tile N is 16 or 32; ring sizes are powers of two");

struct PItem {
    int e, n, N, pos0, row0, mt;
};
__device__ __forceinline__ PItem p_item(const int* tc_tile, int item, int MT) {
    const int ti = item / MT;
    const int4 t = *reinterpret_cast<const int4*>(tc_tile + ti * 4);
    PItem it;
    it.mt = item - ti * MT;
    it.e = t.x;
    it.n = t.y;
    it.N = (t.y + 15) & ~15;
    it.pos0 = t.z;
    it.row0 = t.w;
    return it;
}

template <bool is_down, bool kTrace>
__global__ void __launch_bounds__(kPThreads, 1)
    k_expert_tc(const uint8_t* __restrict__ store_l, jl_layout L, jl_ws ws) {
    extern __shared__ __align__(1024) uint8_t smem[];
    PSmem& sh = *reinterpret_cast<PSmem*>(smem);
    uint8_t* q4_ring = smem + kPQ4Off;
    uint8_t* b_ring = smem + kPBOff;
    uint8_t* scr = smem + kPScrOff;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = L.d, m = L.m;
    const int MT = is_down ? d / 128 : m / 64;
    const int nk = (is_down ? m : d) / kGroup;  // K steps per item
    long long* tr = (blockIdx.x == 0) ? ws.trace : nullptr;
    const int tk = is_down ? kTraceDown : kTraceGateup;
    trace_point(tr, tk, 0);
    // Only the activation producer reads the previous kernel's output (the
    // token tiles of k_tc_permute, or gate/up's activations for down) and
    // waits for it. The tile list is the dispatch step's, two or three
    // launches back and complete once the previous kernel runs (it waited
    // for its own predecessor before releasing this grid), so the weights
    // stream and dequantise meanwhile.
    const int n_items = *ws.tc_ntiles * MT;
    if ((int)blockIdx.x >= n_items) return;
    const int my_items = (n_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const int my_steps = my_items * nk;
    trace_point(tr, tk, 1);
    if (threadIdx.x == 0) {
        sh.abort = 0;
        for (int s = 0; s < kPQ; s++) {
            mbar_init(&sh.q4_full[s], 1);
            mbar_init(&sh.q4_empty[s], 8);  // one arrival per dequant warp (both warpgroups)
        }
        for (int s = 0; s < kPB; s++) {
            mbar_init(&sh.b_full[s], 1);
            mbar_init(&sh.b_empty[s], kPI);  // every issuer releases a stage
        }
        for (int b = 0; b < kPA; b++) {
            mbar_init(&sh.a_full[b], 4);  // one arrival per warp of a dequant warpgroup
            mbar_init(&sh.a_empty[b], 1);
        }
        for (int b = 0; b < 2; b++) {
            for (int w = 0; w < kPI; w++) mbar_init(&sh.acc_full[w][b], 1);
            mbar_init(&sh.acc_empty[b], 4);  // one arrival per epilogue warp
        }
        mbar_fence_init();
    }
    if (warp == kWMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sh.tmem_base)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;
    // wait counters: [0] dequant q4_full, [1] dequant a_empty, [2] dequant TMEM store,
    // [3] dequant total, [4] issuer a_full, [5] issuer b_full, [6] issuer acc_empty,
    // [7] issuer total, [8] producer q4_empty, [9] producer total, [10] activation
    // producer b_empty, [11] epilogue acc_full, [12] epilogue total, [13] items,
    // [14] issuer MMA issue (elected lane's block), [15] dequant of the first row
    long long* dg = (kTrace && blockIdx.x == 0 && ws.trace != nullptr) ? ws.trace + (is_down ? 5 : 4) * 16 : nullptr;
    const long long t_role = kTrace ? clock64() : 0;
    if (dg && threadIdx.x == 0) dg[13] = my_items;
    long long dgl[16] = {};  // this thread's counters (kTrace only)
    // lane 0 of the role's timed warp writes its slots [lo, hi) and the role total
    auto dg_flush = [&](int wid, int lo, int hi, int total) {
        if (kTrace && dg && lane == 0 && warp == wid) {
            for (int i = lo; i < hi; i++) dg[i] += dgl[i];
            dg[total] = clock64() - t_role;
        }
    };

    if (warp == kWProd) {
        // ---------------- weight producer: stage G = K steps [4G, 4G + 4) of the stream
        if (lane == 0) {
            const uint64_t wpol = l2_policy_evict_first();  // expert weights: read once per layer
            const int nq = nk / kPQK;
            int G = 0;
            bool ok = true;
            PItem nx = p_item(ws.tc_tile, (int)blockIdx.x, MT);  // the next item's record, loaded one item ahead
            for (int i = 0; ok && i < my_items; i++) {
                const PItem it = nx;
                if (i + 1 < my_items) nx = p_item(ws.tc_tile, (int)blockIdx.x + (i + 1) * (int)gridDim.x, MT);
                const uint8_t* rec = store_l + (size_t)it.e * L.rec_bytes;
                for (int j = 0; j < nq; j++, G++) {
                    const int s = G % kPQ;
                    if (G >= kPQ && !TC_TIMED(8, tc_wait_relaxed(&sh.q4_empty[s], ((G / kPQ) - 1) & 1, ws.err, &sh.abort))) {
                        ok = false;
                        break;
                    }
                    // the records of consecutive K steps of one row block are contiguous
                    const size_t off = is_down ? L.tile_off(2, it.mt * 4, j * kPQK) : L.tile_off(0, it.mt * 2, j * kPQK);
                    mbar_expect_tx(&sh.q4_full[s], kPStage);
                    bulk_g2s_hint(q4_ring + (size_t)s * kPStage, rec + off, kPStage, &sh.q4_full[s], wpol);
                }
            }
            dg_flush(kWProd, 8, 9, 9);
            for (int c = max(0, G - kPQ); c < G; c++)  // no copies left in flight
                mbar_wait_bounded(&sh.q4_full[c % kPQ], (c / kPQ) & 1, ws.err);
        }
    } else if (warp == kWAct) {
        // ---------------- activation producer: stage = kb K steps of one item's tile
        griddep_wait();
        griddep_launch_dependents();
        if (lane == 0) {
            int G = 0;
            bool ok = true;
            PItem nx = p_item(ws.tc_tile, (int)blockIdx.x, MT);  // the next item's record, loaded one item ahead
            for (int i = 0; ok && i < my_items; i++) {
                const PItem it = nx;
                if (i + 1 < my_items) nx = p_item(ws.tc_tile, (int)blockIdx.x + (i + 1) * (int)gridDim.x, MT);
                const __half* bsrc = is_down ? ws.ac + (size_t)2 * it.row0 * m : ws.xc + (size_t)2 * it.row0 * d;
                const int kb = p_bsteps(it.N);
                for (int c0 = 0; c0 < nk; c0 += kb, G++) {
                    const int s = G % kPB;
                    if (G >= kPB && !TC_TIMED(10, tc_wait_relaxed(&sh.b_empty[s], ((G / kPB) - 1) & 1, ws.err, &sh.abort))) {
                        ok = false;
                        break;
                    }
                    // K step c: 8 chunks x 2N rows (hi, lo) x 16 B = N * 256 bytes
                    const uint32_t bytes = (uint32_t)(min(kb, nk - c0) * it.N * 256);
                    mbar_expect_tx(&sh.b_full[s], bytes);
                    bulk_g2s(b_ring + (size_t)s * kPBBytes, bsrc + (size_t)c0 * 16 * it.N * 8, bytes, &sh.b_full[s]);
                }
            }
            if (kTrace && dg && warp == kWAct) dg[10] += dgl[10];
            for (int c = max(0, G - kPB); c < G; c++)
                mbar_wait_bounded(&sh.b_full[c % kPB], (c / kPB) & 1, ws.err);
        }
    } else if (warp >= kWMma) {
        // ---------------- MMA issuers (whole warps; one elected lane issues):
        // issuer w runs the K-step pairs of parity w of every item, 8 MMAs (K = 16
        // each) of N = 2 x tokens (hi rows -> accumulator columns [0, N), lo
        // rows -> [N, 2N)) into accumulator (w, i % 2)
        const int w = warp - kWMma;
        const int np = nk / 2;  // pairs per item (even: nk % 4 == 0)
        int G = 0;  // activation stages before the current item
        bool ok = true;
        PItem nx = p_item(ws.tc_tile, (int)blockIdx.x, MT);  // the next item's record, loaded one item ahead
        for (int i = 0; ok && i < my_items; i++) {
            const PItem it = nx;
            if (i + 1 < my_items) nx = p_item(ws.tc_tile, (int)blockIdx.x + (i + 1) * (int)gridDim.x, MT);
            const int ib = i & 1;
            if (i >= 2 && !TC_TIMED(6, tc_wait_warp(&sh.acc_empty[ib], ((i >> 1) - 1) & 1, ws.err, &sh.abort)))
                break;
            tc_fence_after();
            const int lkb = p_lbsteps(it.N), kb = 1 << lkb;  // K steps per activation stage: 4 or 8
            const uint32_t idesc = umma_idesc_f16(2 * it.N);
            const uint64_t desc0 = umma_desc(b_ring, (uint32_t)it.N * 32, 128);
            const uint64_t kstep = (uint64_t)((2 * it.N * 32) >> 4);   // 16 K values of 2N rows
            const uint64_t cstep = (uint64_t)((it.N * 256) >> 4);      // one K step
            const uint32_t dacc = tmem + p_acc_col(w, ib);
            for (int pl = w; pl < np; pl += kPI) {
                const int P = i * np + pl, ab = P % kPA;
                const int c = 2 * pl, cb = c & (kb - 1), Gs = G + (c >> lkb), sb = Gs % kPB;
                const int ns = min(kb, nk - (c - cb));  // K steps in this stage (a multiple of 4)
                if (cb == 2 * w && !TC_TIMED(5, tc_wait_warp(&sh.b_full[sb], (Gs / kPB) & 1, ws.err, &sh.abort))) {
                    ok = false;
                    break;
                }
                if (!TC_TIMED(4, tc_wait_warp(&sh.a_full[ab], (P / kPA) & 1, ws.err, &sh.abort))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t dsb = desc0 + (uint64_t)sb * (kPBBytes >> 4) + (uint64_t)cb * cstep;
                const long long c_mma = kTrace ? clock64() : 0;
                if (elect_one()) {
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int ks = 0; ks < 4; ks++)
                            tc_mma_ts(dacc, tmem + ab * 64 + h * 32 + ks * 8, dsb + h * cstep + ks * kstep, idesc,
                                      (pl >= kPI || h || ks) ? 1u : 0u);
                    tc_commit(&sh.a_empty[ab]);
                    if (cb >= ns - 4) tc_commit(&sh.b_empty[sb]);  // this issuer's last pair of the stage
                }
                __syncwarp();
                if (kTrace) dgl[14] += clock64() - c_mma;
            }
            G += (nk + kb - 1) >> lkb;
            if (ok) {
                if (elect_one()) tc_commit(&sh.acc_full[w][ib]);
                __syncwarp();
            }
        }
        dg_flush(kWMma, 4, 7, 7);
        if (kTrace && dg && lane == 0 && warp == kWMma) dg[14] += dgl[14];
    } else if (warp >= 4) {
        // ---------------- dequant warpgroups: thread = A row (TMEM lane). Stage G
        // holds K steps 4G .. 4G+3 = pairs 2G and 2G + 1; pair P goes to warpgroup
        // P % kPDq and TMEM buffer P % kPA (the same number), so warpgroup g only
        // sees stages G = g / 2 (mod 2) and one buffer: every barrier it waits on
        // is released by itself or by a role that walks the same sequence, which
        // keeps its phases at most one apart.
        const int wg = (warp - 4) >> 2, wl = warp & 3, h = wg & 1;
        const int n_stages = my_steps / kPQK;
        for (int G = wg >> 1; G < n_stages; G += 2) {
            const int s = G % kPQ, P = 2 * G + h, ab = wg;
            if (!TC_TIMED(0, tc_wait_warp(&sh.q4_full[s], (G / kPQ) & 1, ws.err, &sh.abort))) break;
            const uint8_t* q = q4_ring + (size_t)s * kPStage + (2 * h) * kTcQ4Stage + wl * kTileRec;
            const uint4 q0 = *reinterpret_cast<const uint4*>(q + lane * 16);
            const uint4 q1 = *reinterpret_cast<const uint4*>(q + 512 + lane * 16);
            const uint16_t sc0 = reinterpret_cast<const uint16_t*>(q + kTileBytes)[lane];
            const uint4 q2 = *reinterpret_cast<const uint4*>(q + kTcQ4Stage + lane * 16);
            const uint4 q3 = *reinterpret_cast<const uint4*>(q + kTcQ4Stage + 512 + lane * 16);
            const uint16_t sc1 = reinterpret_cast<const uint16_t*>(q + kTcQ4Stage + kTileBytes)[lane];
            // this thread's reads of the stage are done; the next bulk copy into it is
            // an async-proxy write, ordered after these plain loads by the proxy fence
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.q4_empty[s]);
            const long long c_dq = kTrace ? clock64() : 0;
            uint32_t a0[32];
            dequant_row_f16(q0, q1, __ushort_as_half(sc0), a0);
            if (kTrace) dgl[15] += clock64() - c_dq;
            if (P >= kPA && !TC_TIMED(1, tc_wait_warp(&sh.a_empty[ab], ((P / kPA) - 1) & 1, ws.err, &sh.abort))) break;
            // order these TMEM writes after the MMAs that read the buffer (released by a_empty)
            tc_fence_after();
            const uint32_t ta = tmem + ((uint32_t)(wl * 32) << 16) + ab * 64;
            const long long c_st = kTrace ? clock64() : 0;
            tc_st32(ta, a0);
            uint32_t a1[32];
            dequant_row_f16(q2, q3, __ushort_as_half(sc1), a1);
            tc_st32(ta + 32, a1);
            tc_wait_st();
            if (kTrace) dgl[2] += clock64() - c_st;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.a_full[ab]);
        }
        dg_flush(4, 0, 3, 3);
        if (kTrace && dg && lane == 0 && warp == 4) dg[15] += dgl[15];
    } else {
        // ---------------- epilogue warps 0-3: thread = accumulator row
        const int row = warp * 32 + lane;
        float* gu_s = reinterpret_cast<float*>(scr);  // [128 rows][kTcNT + 1] (odd stride: no bank conflicts)
        __half* act_s = reinterpret_cast<__half*>(scr + 128 * (kTcNT + 1) * sizeof(float));  // [2][kTcNT][64]
        PItem nx = p_item(ws.tc_tile, (int)blockIdx.x, MT);  // the next item's record, loaded one item ahead
        for (int i = 0; i < my_items; i++) {
            const PItem it = nx;
            if (i + 1 < my_items) nx = p_item(ws.tc_tile, (int)blockIdx.x + (i + 1) * (int)gridDim.x, MT);
            const int ib = i & 1;
            // down: the tile's token slots and weights, one token per lane (n <= 32),
            // loaded before the wait so that the stores below never wait on them
            int t_slot = 0;
            float t_w = 0.0f;
            if (is_down && lane < it.n) {
                t_slot = ws.uidx[it.pos0 + lane];
                t_w = ws.uw[it.pos0 + lane];
            }
            bool got = true;
            for (int w = 0; got && w < kPI; w++)
                got = TC_TIMED(11, __all_sync(0xffffffffu, tc_wait_relaxed(&sh.acc_full[w][ib], (i >> 1) & 1, ws.err, &sh.abort)));
            if (!got) break;
            tc_fence_after();
            if (i == 0) trace_point(tr, tk, 10);
            const uint32_t lanes = (uint32_t)(warp * 32) << 16;
            const uint32_t acc0 = tmem + lanes + p_acc_col(0, ib), acc1 = tmem + lanes + p_acc_col(1, ib);
            const int N = it.N, n = it.n;
            if (is_down) {
                for (int t0 = 0; t0 < N; t0 += 16) {
                    float v[16];
                    tc_ld_acc16(acc0, acc1, N, t0, v);
                    if (t0 + 16 >= N) {  // last TMEM read: hand the accumulators back before storing
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&sh.acc_empty[ib]);
                    }
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int u = __shfl_sync(0xffffffffu, t_slot, t0 + j);
                        const float wj = __shfl_sync(0xffffffffu, t_w, t0 + j);
                        if (t0 + j < n) ws.y[(size_t)u * d + it.mt * 128 + row] = wj * v[j];
                    }
                }
            } else {
                // gate rows (warps 0, 1) and up rows (warps 2, 3) -> smem; the
                // accumulators go back to the MMA as soon as they are read
                for (int t0 = 0; t0 < N; t0 += 16) {
                    float v[16];
                    tc_ld_acc16(acc0, acc1, N, t0, v);
#pragma unroll
                    for (int j = 0; j < 16; j++) gu_s[row * (kTcNT + 1) + t0 + j] = v[j];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.acc_empty[ib]);
                asm volatile("bar.sync 1, 128;" ::: "memory");
                // SwiGLU on all four warps: thread = (intermediate row r, half of the tokens)
                {
                    const int r = row & 63, j8 = r & 7, kc = r >> 3;
                    const int pp = j8 < 4 ? 2 * j8 : 2 * (j8 - 4) + 1;  // position of element j8 (kPerm inverse)
                    const int th = N >> 1, tb = (row >> 6) * th;  // th = 8 or 16
                    for (int t8 = tb; t8 < tb + th; t8 += 8) {
                        // 8 independent SwiGLU chains in flight
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const int t = t8 + j;
                            const float a = silu_mul_approx_div(gu_s[r * (kTcNT + 1) + t], gu_s[(64 + r) * (kTcNT + 1) + t]);
                            const __half h = __float2half_rn(a);
                            const __half l = __float2half_rn(a - __half2float(h));
                            act_s[t * 64 + kc * 8 + pp] = h;
                            act_s[kTcNT * 64 + t * 64 + kc * 8 + pp] = l;
                        }
                    }
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
                // copy out: chunk (t, kc) of 8 halves -> ac tile layout [kc][2N][8]
                __half* abase = ws.ac + (size_t)2 * it.row0 * m;
                const int lN = N == 16 ? 4 : 5;  // log2(N)
                for (int q = row; q < N * 8; q += 128) {
                    const int t = q & (N - 1), kcl = q >> lN;
                    if (t >= n) continue;  // pad rows: never read into a kept result
                    __half* blk = abase + (size_t)(it.mt * 8 + kcl) * 2 * N * 8;
                    *reinterpret_cast<uint4*>(blk + t * 8) = *reinterpret_cast<const uint4*>(act_s + t * 64 + kcl * 8);
                    *reinterpret_cast<uint4*>(blk + (N + t) * 8) =
                        *reinterpret_cast<const uint4*>(act_s + kTcNT * 64 + t * 64 + kcl * 8);
                }
            }
        }
        trace_point(tr, tk, 11);
        dg_flush(0, 11, 12, 12);
    }
    trace_point(tr, tk, 12);
    tc_fence_before();
    __syncthreads();
    if (warp == kWMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

}  // namespace jl

// ---------------------------------------------------------------------------

size_t jl_tc_ws_bytes(int Bmax, int E, int k, int d, int m, size_t* xc_plane, size_t* ac_plane) {
    const int S = Bmax * k;
    const int tiles = jl::tc_max_tiles(S, E);
    const size_t rows = (size_t)S + 15 * (size_t)tiles;
    *xc_plane = rows * d;  // halves per hi (or lo) plane; tiles interleave both
    *ac_plane = rows * m;
    return (*xc_plane + *ac_plane) * 2 * sizeof(__half) + (size_t)tiles * 4 * sizeof(int) + 16;
}

static int tc_attrs() {
    return jl_device_once(kOnceTc, [] {
        using namespace jl;
        JL_CUDA(cudaFuncSetAttribute(k_expert_tc<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kPSmemBytes));
        JL_CUDA(cudaFuncSetAttribute(k_expert_tc<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kPSmemBytes));
        JL_CUDA(cudaFuncSetAttribute(k_expert_tc<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kPSmemBytes));
        JL_CUDA(cudaFuncSetAttribute(k_expert_tc<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kPSmemBytes));
        return JL_OK;
    });
}

int jl_launch_gateup_tc(const jl_moe* h, const uint8_t* store_l, const float* x, int B, cudaStream_t s) {
    using namespace jl;
    int rc = tc_attrs();
    if (rc) return rc;
    if (h->d % 512 || h->m % 256 || !h->ws.xc) return JL_ERR_INVALID;
    const int tiles = tc_max_tiles(B * h->k, h->E);
    rc = launch(k_tc_permute, dim3(tiles, h->d / 512), dim3(256), 0, s, x, h->d, h->k, h->ws);
    if (rc) return rc;
    const int items = tiles * (h->m / 64);
    return launch(h->ws.trace ? k_expert_tc<false, true> : k_expert_tc<false, false>,
                  dim3(std::min(h->sm_count, items)), dim3(kPThreads), kPSmemBytes, s, store_l, h->lay, h->ws);
}

int jl_launch_down_tc(const jl_moe* h, const uint8_t* store_l, int B, cudaStream_t s) {
    using namespace jl;
    int rc = tc_attrs();
    if (rc) return rc;
    if (h->d % 512 || h->m % 256 || !h->ws.xc) return JL_ERR_INVALID;
    const int items = tc_max_tiles(B * h->k, h->E) * (h->d / 128);
    return launch(h->ws.trace ? k_expert_tc<true, true> : k_expert_tc<true, false>,
                  dim3(std::min(h->sm_count, items)), dim3(kPThreads), kPSmemBytes, s, store_l, h->lay, h->ws);
}
