// Tensor-core (tcgen05) path of the expert FFN for larger batches.
//
// Per layer, after routing:
//   tc_build_tiles (end of the dispatch step) cuts every union expert's
//                 tokens into tiles of <= 64 (padded to a multiple of 16).
//   k_tc_permute  gathers each tile's tokens and writes them as fp16 hi/lo
//                 pairs (x = hi + lo, ~22 significant bits) in the UMMA
//                 K-major "interleaved" core layout, hi rows then lo rows, so
//                 one MMA of N = 2 x tokens covers both (the epilogue adds the
//                 two accumulator halves).
//   k_gateup_tc   one CTA per (tile, 64 gate rows + the matching 64 up rows):
//                 two producer warps stream the Q4 tiles (8-stage ring) and
//                 the token tiles (4-stage ring) with 1-D bulk copies;
//                 4 dequant warps turn each 64-value group into fp16
//                 (n - 8) * scale (correctly rounded) and store it straight
//                 into tensor memory as the MMA's A operand (lane = weight
//                 row); one thread issues tcgen05.mma (M=128, N=2 x tokens,
//                 K=16, fp32 accumulate in TMEM). The epilogue
//                 reads the accumulator with tcgen05.ld, applies SwiGLU and
//                 writes the activations (hi/lo, same core layout) for down.
//   k_down_tc     the same pipeline over the down matrix (M=128 rows of d,
//                 K = intermediate); the epilogue writes y[slot] = w * acc.
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

constexpr int kTcDqWarps = 4;        // dequant/epilogue warps = TMEM lanes 0..127
constexpr int kTcQ4Stage = 4 * kTileRec;  // the 4 contiguous tile records of one K step
constexpr int kTcBStage = 2 * kTcNT * 128;  // 8 K chunks x (hi + lo rows) x 16 B, 64 K values
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

// hi + lo accumulator columns of 16 tokens
__device__ __forceinline__ void tc_ld_sum16(uint32_t taddr_hi, uint32_t taddr_lo, float (&v)[16]) {
    float a[16], b[16];
    tc_ld16(taddr_hi, a);
    tc_ld16(taddr_lo, b);
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = a[i] + b[i];
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

// Warp-wide form for the warps that go on to tcgen05.ld / tcgen05.st: those
// are .sync.aligned, so every lane must leave the spin together and agree on
// the outcome (each lane polls on its own and may exit at another iteration).
__device__ __forceinline__ bool tc_wait_warp(uint64_t* bar, uint32_t parity, int* err,
                                             volatile int* abort) {
    return __all_sync(0xffffffffu, tc_wait(bar, parity, err, abort));
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
// writes K chunks [64y, 64y + 64) of tile t as fp16 hi/lo in core layout.
__global__ void __launch_bounds__(256) k_tc_permute(const float* __restrict__ x, int d, int k,
                                                    jl_ws ws) {
    griddep_wait();
    griddep_launch_dependents();
    const int ti = blockIdx.x;
    if (ti >= *ws.tc_ntiles) return;
    const int n = ws.tc_tile[ti * 4 + 1], N = (n + 15) & ~15;
    const int pos0 = ws.tc_tile[ti * 4 + 2], row0 = ws.tc_tile[ti * 4 + 3];
    const int kc0 = blockIdx.y * 64, kcn = min(64, d / 8 - kc0);
    // tile layout: [kc][2N rows: hi rows 0..N-1, lo rows N..2N-1][8 halves]
    __half* base = ws.xc + (size_t)2 * row0 * d;
    for (int i = threadIdx.x; i < N * kcn; i += blockDim.x) {
        const int r = i % N, kc = kc0 + i / N;
        uint4 vh = make_uint4(0, 0, 0, 0), vl = make_uint4(0, 0, 0, 0);
        if (r < n) {
            const int b = ws.uidx[pos0 + r] / k;
            const float4 a = *reinterpret_cast<const float4*>(x + (size_t)b * d + kc * 8);
            const float4 c = *reinterpret_cast<const float4*>(x + (size_t)b * d + kc * 8 + 4);
            const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
            split_chunk(v, vh, vl);
        }
        __half* blk = base + (size_t)kc * 2 * N * 8;
        *reinterpret_cast<uint4*>(blk + r * 8) = vh;
        *reinterpret_cast<uint4*>(blk + (N + r) * 8) = vl;
    }
}

// ---------------------------------------------------------------------------
// The grouped GEMM CTA (shared by gate/up and down). Roles:
//   warps 0-3  dequant (thread = A row = TMEM lane) and epilogue
//   warp 4     Q4 producer: weight tiles + scales, 8-stage ring
//   warp 5     activation producer: hi/lo K chunks, 4-stage ring
//   warp 6     MMA issuer; TMEM allocation
// The weight ring is released as soon as the dequant warps have the bytes in
// registers, so the weight stream runs up to 8 chunks ahead of the MMAs; the
// 4 TMEM A buffers let dequant run 4 chunks ahead.

constexpr int kTcQS = 8;   // weight stages
constexpr int kTcBS = 4;   // activation stages
constexpr int kTcAB = 4;   // TMEM A buffers (32 columns each)
constexpr int kTcAcc = kTcAB * 32;  // accumulator column
constexpr int kTcCols = 256;
constexpr int kTcWarps = 7;

struct TcSmem {
    uint64_t q4_full[kTcQS], q4_empty[kTcQS];
    uint64_t b_full[kTcBS], b_empty[kTcBS];
    uint64_t a_full[kTcAB], a_empty[kTcAB];
    uint64_t acc_full;
    uint32_t tmem_base;
    int abort;
    int info[4];  // expert, tokens, first uidx position, row offset
};

constexpr size_t kTcSmemQ4Off = 512;
constexpr size_t kTcSmemBOff = kTcSmemQ4Off + (size_t)kTcQS * kTcQ4Stage;
constexpr size_t kTcSmemBytes = kTcSmemBOff + (size_t)kTcBS * kTcBStage;

// is_down: A = down rows [mt*128, +128) of d (4 tiles of 32 rows), K = m,
//          B = activations; epilogue y = w * acc.
// else:    A = gate rows [mt*64, +64) then up rows [mt*64, +64), K = d,
//          B = tokens; epilogue act = silu(g) * u.
template <bool is_down>
__global__ void __launch_bounds__(kTcWarps * 32, 1)
    k_expert_tc(const uint8_t* __restrict__ store_l, jl_layout L, jl_ws ws) {
    extern __shared__ __align__(1024) uint8_t smem[];
    TcSmem& sh = *reinterpret_cast<TcSmem*>(smem);
    uint8_t* q4_ring = smem + kTcSmemQ4Off;
    uint8_t* b_ring = smem + kTcSmemBOff;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = L.d, m = L.m;
    const int MT = is_down ? d / 128 : m / 64;
    const int ti = blockIdx.x / MT, mt = blockIdx.x % MT;
    const int K = is_down ? m : d;
    const int nchunks = K / kGroup;
    long long* tr = (blockIdx.x == 0) ? ws.trace : nullptr;
    const int tk = is_down ? kTraceDown : kTraceGateup;
    trace_point(tr, tk, 0);
    griddep_wait();
    griddep_launch_dependents();
    if (ti >= *ws.tc_ntiles) return;
    trace_point(tr, tk, 1);
    if (threadIdx.x == 0) {
        sh.info[0] = ws.tc_tile[ti * 4 + 0];
        sh.info[1] = ws.tc_tile[ti * 4 + 1];
        sh.info[2] = ws.tc_tile[ti * 4 + 2];
        sh.info[3] = ws.tc_tile[ti * 4 + 3];
        sh.abort = 0;
        for (int s = 0; s < kTcQS; s++) {
            mbar_init(&sh.q4_full[s], 1);
            mbar_init(&sh.q4_empty[s], kTcDqWarps * 32);
        }
        for (int s = 0; s < kTcBS; s++) {
            mbar_init(&sh.b_full[s], 1);
            mbar_init(&sh.b_empty[s], 1);
        }
        for (int b = 0; b < kTcAB; b++) {
            mbar_init(&sh.a_full[b], kTcDqWarps * 32);
            mbar_init(&sh.a_empty[b], 1);
        }
        mbar_init(&sh.acc_full, 1);
        mbar_fence_init();
    }
    if (warp == 6) {  // TMEM allocation by one full warp
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sh.tmem_base)),
                     "r"(kTcCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;
    const int e = sh.info[0], n = sh.info[1], N = (n + 15) & ~15, pos0 = sh.info[2], row0 = sh.info[3];
    const uint8_t* rec = store_l + (size_t)e * L.rec_bytes;
    const uint32_t b_stage = (uint32_t)N * 256;  // 8 K-chunks x 2N rows (hi, lo) x 16 B

    if (warp == 4) {
        // ---------------- weight producer
        if (lane == 0) {
            int issued = 0;
            for (int c = 0; c < nchunks; c++) {
                const int s = c % kTcQS;
                if (c >= kTcQS && !tc_wait(&sh.q4_empty[s], ((c / kTcQS) - 1) & 1, ws.err, &sh.abort))
                    break;
                uint8_t* q = q4_ring + (size_t)s * kTcQ4Stage;
                mbar_expect_tx(&sh.q4_full[s], kTcQ4Stage);
                // gate/up: [gate 2mt][gate 2mt+1][up 2mt][up 2mt+1]; down: rb 4mt..4mt+3
                const size_t off = is_down ? L.tile_off(2, mt * 4, c) : L.tile_off(0, mt * 2, c);
                bulk_g2s(q, rec + off, kTcQ4Stage, &sh.q4_full[s]);
                issued = c + 1;
            }
            for (int c = std::max(0, issued - kTcQS); c < issued; c++)  // no copies left in flight
                mbar_wait_bounded(&sh.q4_full[c % kTcQS], (c / kTcQS) & 1, ws.err);
        }
    } else if (warp == 5) {
        // ---------------- activation producer
        if (lane == 0) {
            const __half* bsrc = is_down ? ws.ac + (size_t)2 * row0 * m : ws.xc + (size_t)2 * row0 * d;
            int issued = 0;
            for (int c = 0; c < nchunks; c++) {
                const int s = c % kTcBS;
                if (c >= kTcBS && !tc_wait(&sh.b_empty[s], ((c / kTcBS) - 1) & 1, ws.err, &sh.abort))
                    break;
                uint8_t* bb = b_ring + (size_t)s * kTcBStage;
                mbar_expect_tx(&sh.b_full[s], b_stage);
                bulk_g2s(bb, bsrc + (size_t)c * 8 * 2 * N * 8, b_stage, &sh.b_full[s]);
                issued = c + 1;
            }
            for (int c = std::max(0, issued - kTcBS); c < issued; c++)
                mbar_wait_bounded(&sh.b_full[c % kTcBS], (c / kTcBS) & 1, ws.err);
        }
    } else if (warp == 6) {
        // ---------------- MMA issuer: per K step one MMA over 2N columns
        // (hi rows -> accumulator columns [0, N), lo rows -> [N, 2N))
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(2 * N);
            const uint64_t desc0 = umma_desc(b_ring, (uint32_t)N * 32, 128);
            const uint64_t kstep = (uint64_t)((2 * N * 32) >> 4);      // 2 K chunks of 2N rows
            const uint64_t sstep = (uint64_t)(kTcBStage >> 4);
            for (int c = 0; c < nchunks; c++) {
                const int ab = c % kTcAB, sb = c % kTcBS;
                if (!tc_wait(&sh.a_full[ab], (c / kTcAB) & 1, ws.err, &sh.abort)) break;
                if (!tc_wait(&sh.b_full[sb], (c / kTcBS) & 1, ws.err, &sh.abort)) break;
                tc_fence_after();
                const uint64_t dsb = desc0 + sb * sstep;
#pragma unroll
                for (int ks = 0; ks < 4; ks++)
                    tc_mma_ts(tmem + kTcAcc, tmem + ab * 32 + ks * 8, dsb + ks * kstep, idesc,
                              (c | ks) ? 1u : 0u);
                tc_commit(&sh.a_empty[ab]);
                tc_commit(&sh.b_empty[sb]);
            }
            tc_commit(&sh.acc_full);
        }
    } else {
        // ---------------- dequant warps: thread = A row (TMEM lane)
        const int row = warp * 32 + lane;
        for (int c = 0; c < nchunks; c++) {
            const int s = c % kTcQS, ab = c % kTcAB;
            if (!tc_wait_warp(&sh.q4_full[s], (c / kTcQS) & 1, ws.err, &sh.abort)) break;
            if (c < 8) trace_point(tr, tk, 2 + c);
            const uint8_t* q = q4_ring + (size_t)s * kTcQ4Stage + warp * kTileRec;
            const uint4 q0 = *reinterpret_cast<const uint4*>(q + lane * 16);
            const uint4 q1 = *reinterpret_cast<const uint4*>(q + 512 + lane * 16);
            const uint16_t sb = reinterpret_cast<const uint16_t*>(q + kTileBytes)[lane];
            // the stage's bytes are in registers; the next bulk copy into it is an
            // async-proxy write, ordered after these plain loads by the proxy fence
            fence_proxy_async_smem();
            mbar_arrive(&sh.q4_empty[s]);
            uint32_t a[32];
            dequant_row_f16(q0, q1, __ushort_as_half(sb), a);
            if (c >= kTcAB && !tc_wait_warp(&sh.a_empty[ab], ((c / kTcAB) - 1) & 1, ws.err, &sh.abort))
                break;
            // order this TMEM write after the MMAs that read the buffer (released by a_empty)
            tc_fence_after();
            tc_st32(tmem + ((uint32_t)(warp * 32) << 16) + ab * 32, a);
            tc_wait_st();
            tc_fence_before();
            mbar_arrive(&sh.a_full[ab]);
        }
        // ---------------- epilogue
        trace_point(tr, tk, 10);
        const bool ok = tc_wait_warp(&sh.acc_full, 0, ws.err, &sh.abort);
        tc_fence_after();
        trace_point(tr, tk, 11);
        // the activation ring is idle once acc_full completed (every bulk copy into it
        // landed and every MMA read of it finished); reuse it as epilogue scratch
        fence_proxy_async_smem();
        float* scr = reinterpret_cast<float*>(b_ring);
        if (ok) {
            const uint32_t tacc = tmem + ((uint32_t)(warp * 32) << 16) + kTcAcc;
            if (is_down) {
                for (int t0 = 0; t0 < N; t0 += 16) {
                    float v[16];
                    tc_ld_sum16(tacc + t0, tacc + N + t0, v);
                    for (int i = 0; i < 16 && t0 + i < n; i++) {
                        const int pos = pos0 + t0 + i;
                        const int slot = ws.uidx[pos];
                        ws.y[(size_t)slot * d + mt * 128 + row] = ws.uw[pos] * v[i];
                    }
                }
            } else {
                // up rows (warps 2,3) -> smem; gate rows (warps 0,1) apply SwiGLU
                float* up_s = scr;                                            // [64 rows][kTcNT]
                __half* act_s = reinterpret_cast<__half*>(scr + 64 * kTcNT);  // [2][kTcNT][64]
                if (warp >= 2)
                    for (int t0 = 0; t0 < N; t0 += 16) {
                        float v[16];
                        tc_ld_sum16(tacc + t0, tacc + N + t0, v);
#pragma unroll
                        for (int i = 0; i < 16; i++) up_s[(row - 64) * kTcNT + t0 + i] = v[i];
                    }
                asm volatile("bar.sync 1, %0;" ::"r"(kTcDqWarps * 32) : "memory");
                if (warp < 2) {
                    const int j = row & 7, kc = row >> 3;
                    const int pp = j < 4 ? 2 * j : 2 * (j - 4) + 1;  // position of element j (kPerm inverse)
                    for (int t0 = 0; t0 < N; t0 += 16) {
                        float v[16];
                        tc_ld_sum16(tacc + t0, tacc + N + t0, v);
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            const float a = silu_mul(v[i], up_s[row * kTcNT + t0 + i]);
                            const __half h = __float2half_rn(a);
                            const __half l = __float2half_rn(a - __half2float(h));
                            act_s[(t0 + i) * 64 + kc * 8 + pp] = h;
                            act_s[kTcNT * 64 + (t0 + i) * 64 + kc * 8 + pp] = l;
                        }
                    }
                }
                asm volatile("bar.sync 1, %0;" ::"r"(kTcDqWarps * 32) : "memory");
                // copy out: chunk (t, kc) of 8 halves -> ac tile layout [kc][2N][8]
                __half* abase = ws.ac + (size_t)2 * row0 * m;
                for (int i = row; i < N * 8; i += kTcDqWarps * 32) {
                    const int t = i % N, kcl = i / N;
                    __half* blk = abase + (size_t)(mt * 8 + kcl) * 2 * N * 8;
                    uint4 vh = make_uint4(0, 0, 0, 0), vl = make_uint4(0, 0, 0, 0);
                    if (t < n) {
                        vh = *reinterpret_cast<const uint4*>(act_s + t * 64 + kcl * 8);
                        vl = *reinterpret_cast<const uint4*>(act_s + kTcNT * 64 + t * 64 + kcl * 8);
                    }
                    *reinterpret_cast<uint4*>(blk + t * 8) = vh;
                    *reinterpret_cast<uint4*>(blk + (N + t) * 8) = vl;
                }
            }
        }
    }
    trace_point(tr, tk, 12);
    tc_fence_before();
    __syncthreads();
    if (warp == 6) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols));
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

int jl_launch_experts_tc(const jl_moe* h, const uint8_t* store_l, const float* x, int B,
                         cudaStream_t s) {
    using namespace jl;
    static bool attr = false;
    if (!attr) {
        JL_CUDA(cudaFuncSetAttribute(k_expert_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kTcSmemBytes));
        JL_CUDA(cudaFuncSetAttribute(k_expert_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kTcSmemBytes));
        attr = true;
    }
    if (h->d % 512 || h->m % 64 || h->d % 128 || !h->ws.xc) return JL_ERR_INVALID;
    const int tiles = tc_max_tiles(B * h->k, h->E);
    int rc = launch(k_tc_permute, dim3(tiles, h->d / 512), dim3(256), 0, s, x, h->d, h->k, h->ws);
    if (rc) return rc;
    rc = launch(k_expert_tc<false>, dim3(tiles * (h->m / 64)), dim3(kTcWarps * 32), kTcSmemBytes, s,
                store_l, h->lay, h->ws);
    if (rc) return rc;
    return launch(k_expert_tc<true>, dim3(tiles * (h->d / 128)), dim3(kTcWarps * 32), kTcSmemBytes, s,
                  store_l, h->lay, h->ws);
}
