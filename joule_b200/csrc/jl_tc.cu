// Tensor-core (tcgen05) path of the expert FFN for larger batches.
//
// Per layer, after routing:
//   k_tc_permute  gathers the tokens of every union expert into token tiles
//                 (<= 64 tokens, padded to a multiple of 16) and writes them
//                 as fp16 hi/lo pairs (x = hi + lo, ~22 significant bits) in
//                 the UMMA K-major "interleaved" core layout; it also writes
//                 the tile table (expert, tile, tokens, row offsets).
//   k_gateup_tc   one CTA per (tile, 64 gate rows + the matching 64 up rows):
//                 a producer warp streams the Q4 tiles and the token tiles
//                 through a 4-stage shared-memory ring with 1-D bulk copies;
//                 4 dequant warps turn each 64-value group into fp16
//                 (n - 8) * scale (correctly rounded) and store it straight
//                 into tensor memory as the MMA's A operand (lane = weight
//                 row); one thread issues tcgen05.mma (M=128, N=tokens,
//                 K=16, fp32 accumulate in TMEM) for hi and lo. The epilogue
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

namespace jl {

constexpr int kTcNT = 64;            // max tokens per tile (MMA N <= 64)
constexpr int kTcStages = 4;         // shared-memory ring depth
constexpr int kTcDqWarps = 4;        // dequant/epilogue warps = TMEM lanes 0..127
constexpr int kTcThreads = (kTcDqWarps + 2) * 32;  // + producer warp + MMA warp
constexpr int kTcTmemCols = 128;     // A double buffer (2 x 32) + accumulator (<= 64)
constexpr int kTcAccCol = 64;
constexpr int kTcQ4Stage = 4 * kTileBytes + 4 * kTileRows * 2;  // 4 tiles + their scales
constexpr int kTcBStage = 2 * kTcNT * 128;                         // hi + lo, 64 K values
// position p of an 8-value K chunk holds element kPerm[p]; kPermInv is its inverse
__constant__ int kPermInvC[8] = {0, 2, 4, 6, 1, 3, 5, 7};

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
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(err, kErrTimeout);
            *abort = 1;
            return false;
        }
    }
    return true;
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
// Tile table + activation gather. grid = (max tiles, d / 512); block 256.

// rows of expert with n tokens in the padded tile space: full 64-token tiles
// plus the last tile rounded up to 16.
__device__ __forceinline__ int tc_rows(int n) { return (n / kTcNT) * kTcNT + ((n % kTcNT + 15) & ~15); }

// Locate tile `ti`: its expert u, tile j, first uidx position and row offset.
// Warp 0 scans the union (U <= 256) in chunks of 32. Returns false past the end.
__device__ bool tc_find_tile(const jl_ws& ws, int ti, int* info /* smem [6] */) {
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const int U = *ws.U;
        int tiles_before = 0, rows_before = 0, found = 0;
        for (int u0 = 0; u0 < U; u0 += 32) {  // full scan: tiles_before ends as the total
            const int u = u0 + lane;
            const int n = (u < U) ? ws.uh[u + 1] - ws.uh[u] : 0;
            const int t = (n + kTcNT - 1) / kTcNT, r = tc_rows(n);
            int ti_inc = t, r_inc = r;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, ti_inc, o);
                const int b = __shfl_up_sync(0xffffffffu, r_inc, o);
                if (lane >= o) {
                    ti_inc += a;
                    r_inc += b;
                }
            }
            const int t_ex = tiles_before + ti_inc - t, r_ex = rows_before + r_inc - r;
            const bool mine = u < U && ti >= t_ex && ti < t_ex + t;
            const unsigned bal = __ballot_sync(0xffffffffu, mine);
            if (mine) {
                const int j = ti - t_ex;
                info[0] = 1;
                info[1] = u;
                info[2] = j;
                info[3] = min(kTcNT, n - j * kTcNT);     // tokens in the tile
                info[4] = ws.uh[u] + j * kTcNT;          // first uidx position
                info[5] = r_ex + j * kTcNT;              // padded row offset
            }
            found |= bal != 0;
            tiles_before += __shfl_sync(0xffffffffu, ti_inc, 31);
            rows_before += __shfl_sync(0xffffffffu, r_inc, 31);
        }
        if (!found && lane == 0) info[0] = 0;
        if (lane == 0 && ti == 0 && blockIdx.y == 0) ws.tc_ntiles[0] = tiles_before;
    }
    __syncthreads();
    return info[0] != 0;
}

__global__ void __launch_bounds__(256) k_tc_permute(const float* __restrict__ x, int d, int k,
                                                    jl_ws ws) {
    __shared__ int info[6];
    griddep_wait();
    griddep_launch_dependents();
    const int ti = blockIdx.x;
    // the total tile count is written by tile 0's block even when it has work
    if (!tc_find_tile(ws, ti, info)) return;
    const int n = info[3], N = (n + 15) & ~15, pos0 = info[4], row0 = info[5];
    if (blockIdx.y == 0 && threadIdx.x == 0) {
        ws.tc_tile[ti * 4 + 0] = ws.sel[info[1]];  // expert id of union position u
        ws.tc_tile[ti * 4 + 1] = n;
        ws.tc_tile[ti * 4 + 2] = pos0;
        ws.tc_tile[ti * 4 + 3] = row0;
    }
    // K slice of this block: chunks kc in [kc0, kc0 + 64)
    const int kc0 = blockIdx.y * 64, kcn = min(64, d / 8 - kc0);
    __half* hi = ws.xc + (size_t)row0 * d;
    __half* lo = ws.xc + ws.xc_plane + (size_t)row0 * d;
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
        *reinterpret_cast<uint4*>(hi + (size_t)kc * N * 8 + r * 8) = vh;
        *reinterpret_cast<uint4*>(lo + (size_t)kc * N * 8 + r * 8) = vl;
    }
}

// ---------------------------------------------------------------------------
// The grouped GEMM CTA (shared by gate/up and down).

struct TcSmem {
    uint64_t full[kTcStages], empty[kTcStages], a_full[2], a_empty[2], acc_full;
    uint32_t tmem_base;
    int abort;
    int info[4];  // expert, tokens, first uidx position, row offset
};

// smem: [TcSmem][q4 ring][b ring]; the b ring is reused by the epilogue
constexpr size_t kTcSmemQ4Off = 256;
constexpr size_t kTcSmemBOff = kTcSmemQ4Off + (size_t)kTcStages * kTcQ4Stage;
constexpr size_t kTcSmemBytes = kTcSmemBOff + (size_t)kTcStages * kTcBStage;

// is_down: A = down rows [mt*128, +128) of d (4 tiles of 32 rows), K = m,
//          B = activations; epilogue y = w * acc.
// else:    A = gate rows [mt*64, +64) then up rows [mt*64, +64), K = d,
//          B = tokens; epilogue act = silu(g) * u.
template <bool is_down>
__global__ void __launch_bounds__(kTcThreads, 1)
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
    griddep_wait();
    griddep_launch_dependents();
    if (ti >= *ws.tc_ntiles) return;
    if (threadIdx.x == 0) {
        sh.info[0] = ws.tc_tile[ti * 4 + 0];
        sh.info[1] = ws.tc_tile[ti * 4 + 1];
        sh.info[2] = ws.tc_tile[ti * 4 + 2];
        sh.info[3] = ws.tc_tile[ti * 4 + 3];
        sh.abort = 0;
        for (int s = 0; s < kTcStages; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], kTcDqWarps * 32 + 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&sh.a_full[b], kTcDqWarps * 32);
            mbar_init(&sh.a_empty[b], 1);
        }
        mbar_init(&sh.acc_full, 1);
        mbar_fence_init();
    }
    if (warp == kTcDqWarps + 1) {  // TMEM allocation by one full warp
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sh.tmem_base)),
                     "r"(kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;
    const int e = sh.info[0], n = sh.info[1], N = (n + 15) & ~15, pos0 = sh.info[2], row0 = sh.info[3];
    const uint8_t* rec = store_l + (size_t)e * L.rec_bytes;
    const int ngK = K / kGroup;  // groups per weight row
    const uint32_t b_part = (uint32_t)N * 128;  // bytes of one hi or lo chunk (8 K-chunks x N rows x 16 B)

    if (warp == kTcDqWarps) {
        // ---------------- producer: Q4 tiles + token chunks
        if (lane == 0) {
            const __half* bsrc = is_down ? ws.ac + (size_t)row0 * m : ws.xc + (size_t)row0 * d;
            const size_t plane = is_down ? ws.ac_plane : ws.xc_plane;
            int issued = 0;
            for (int c = 0; c < nchunks; c++) {
                const int s = c % kTcStages;
                if (c >= kTcStages &&
                    !tc_wait(&sh.empty[s], ((c / kTcStages) - 1) & 1, ws.err, &sh.abort))
                    break;
                uint8_t* q = q4_ring + (size_t)s * kTcQ4Stage;
                uint8_t* bb = b_ring + (size_t)s * kTcBStage;
                mbar_expect_tx(&sh.full[s], kTcQ4Stage + 2 * b_part);
                for (int t = 0; t < 4; t++) {
                    int p, rb;
                    if (is_down) {
                        p = 2;
                        rb = mt * 4 + t;
                    } else {
                        p = t >> 1;
                        rb = mt * 2 + (t & 1);
                    }
                    const size_t tile = (size_t)rb * ngK + c;
                    bulk_g2s(q + t * kTileBytes, rec + L.tiles_off(p) + tile * kTileBytes, kTileBytes,
                             &sh.full[s]);
                    bulk_g2s(q + 4 * kTileBytes + t * kTileRows * 2,
                             rec + L.scales_off(p) + tile * kTileRows * 2, kTileRows * 2, &sh.full[s]);
                }
                const size_t koff = (size_t)c * 8 * N * 8;  // halves: 8 K-chunks of N rows x 8
                bulk_g2s(bb, bsrc + koff, b_part, &sh.full[s]);
                bulk_g2s(bb + b_part, bsrc + plane + koff, b_part, &sh.full[s]);
                issued = c + 1;
            }
            // never leave bulk copies landing in a CTA that is about to exit
            for (int c = std::max(0, issued - kTcStages); c < issued; c++)
                mbar_wait_bounded(&sh.full[c % kTcStages], (c / kTcStages) & 1, ws.err);
        }
    } else if (warp == kTcDqWarps + 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(N);
            for (int c = 0; c < nchunks; c++) {
                const int s = c % kTcStages, ab = c & 1;
                if (!tc_wait(&sh.a_full[ab], (c >> 1) & 1, ws.err, &sh.abort)) break;
                if (!tc_wait(&sh.full[s], (c / kTcStages) & 1, ws.err, &sh.abort)) break;
                tc_fence_after();
                const uint8_t* bb = b_ring + (size_t)s * kTcBStage;
#pragma unroll
                for (int ks = 0; ks < 4; ks++)
#pragma unroll
                    for (int part = 0; part < 2; part++) {
                        const uint64_t desc =
                            umma_desc(bb + part * b_part + (size_t)ks * 2 * N * 16, (uint32_t)N * 16, 128);
                        tc_mma_ts(tmem + kTcAccCol, tmem + ab * 32 + ks * 8, desc, idesc,
                                  (c | ks | part) ? 1u : 0u);
                    }
                tc_commit(&sh.a_empty[ab]);
                tc_commit(&sh.empty[s]);
            }
            tc_commit(&sh.acc_full);
        }
    } else {
        // ---------------- dequant warps: thread = A row (TMEM lane)
        const int row = warp * 32 + lane;
        for (int c = 0; c < nchunks; c++) {
            const int s = c % kTcStages, ab = c & 1;
            if (!tc_wait(&sh.full[s], (c / kTcStages) & 1, ws.err, &sh.abort)) break;
            const uint8_t* q = q4_ring + (size_t)s * kTcQ4Stage + warp * kTileBytes;
            const uint4 q0 = *reinterpret_cast<const uint4*>(q + lane * 16);
            const uint4 q1 = *reinterpret_cast<const uint4*>(q + 512 + lane * 16);
            const uint16_t sb = reinterpret_cast<const uint16_t*>(
                q4_ring + (size_t)s * kTcQ4Stage + 4 * kTileBytes)[warp * kTileRows + lane];
            mbar_arrive(&sh.empty[s]);  // this stage's Q4 bytes are in registers
            uint32_t a[32];
            dequant_row_f16(q0, q1, __ushort_as_half(sb), a);
            if (c >= 2 && !tc_wait(&sh.a_empty[ab], ((c >> 1) - 1) & 1, ws.err, &sh.abort)) break;
            tc_st32(tmem + ((uint32_t)(warp * 32) << 16) + ab * 32, a);
            tc_wait_st();
            tc_fence_before();
            mbar_arrive(&sh.a_full[ab]);
        }
        // ---------------- epilogue
        const bool ok = tc_wait(&sh.acc_full, 0, ws.err, &sh.abort);
        tc_fence_after();
        float* scr = reinterpret_cast<float*>(b_ring);  // ring is idle once acc_full completed
        if (ok) {
            const uint32_t tacc = tmem + ((uint32_t)(warp * 32) << 16) + kTcAccCol;
            if (is_down) {
                for (int t0 = 0; t0 < N; t0 += 16) {
                    float v[16];
                    tc_ld16(tacc + t0, v);
                    for (int i = 0; i < 16 && t0 + i < n; i++) {
                        const int pos = pos0 + t0 + i;
                        const int slot = ws.uidx[pos];
                        ws.y[(size_t)slot * d + mt * 128 + row] = ws.uw[pos] * v[i];
                    }
                }
            } else {
                // up rows (warps 2,3) -> smem; gate rows (warps 0,1) combine
                float* up_s = scr;                                            // [64 rows][kTcNT]
                __half* act_s = reinterpret_cast<__half*>(scr + 64 * kTcNT);  // [2][kTcNT][64]
                if (warp >= 2)
                    for (int t0 = 0; t0 < N; t0 += 16) {
                        float v[16];
                        tc_ld16(tacc + t0, v);
#pragma unroll
                        for (int i = 0; i < 16; i++) up_s[(row - 64) * kTcNT + t0 + i] = v[i];
                    }
                asm volatile("bar.sync 1, %0;" ::"r"(kTcDqWarps * 32) : "memory");
                if (warp < 2) {
                    const int kc = row >> 3, pp = kPermInvC[row & 7];
                    for (int t0 = 0; t0 < N; t0 += 16) {
                        float v[16];
                        tc_ld16(tacc + t0, v);
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
                // copy out: chunk (t, kc) of 8 halves -> ac core layout
                __half* ahi = ws.ac + (size_t)row0 * m;
                __half* alo = ws.ac + ws.ac_plane + (size_t)row0 * m;
                for (int i = row; i < N * 8; i += kTcDqWarps * 32) {
                    const int t = i % N, kcl = i / N;
                    const size_t dst = (size_t)(mt * 8 + kcl) * N * 8 + (size_t)t * 8;
                    uint4 vh = make_uint4(0, 0, 0, 0), vl = make_uint4(0, 0, 0, 0);
                    if (t < n) {
                        vh = *reinterpret_cast<const uint4*>(act_s + t * 64 + kcl * 8);
                        vl = *reinterpret_cast<const uint4*>(act_s + kTcNT * 64 + t * 64 + kcl * 8);
                    }
                    *reinterpret_cast<uint4*>(ahi + dst) = vh;
                    *reinterpret_cast<uint4*>(alo + dst) = vl;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcDqWarps + 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTcTmemCols));
    }
}

}  // namespace jl

// ---------------------------------------------------------------------------

size_t jl_tc_ws_bytes(int Bmax, int E, int k, int d, int m, size_t* xc_plane, size_t* ac_plane) {
    const int S = Bmax * k;
    const int tiles = jl::tc_max_tiles(S, E);
    const size_t rows = (size_t)S + 15 * (size_t)tiles;
    *xc_plane = rows * d;  // halves per hi/lo plane
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
    rc = launch(k_expert_tc<false>, dim3(tiles * (h->m / 64)), dim3(kTcThreads), kTcSmemBytes, s,
                store_l, h->lay, h->ws);
    if (rc) return rc;
    return launch(k_expert_tc<true>, dim3(tiles * (h->d / 128)), dim3(kTcThreads), kTcSmemBytes, s,
                  store_l, h->lay, h->ws);
}
