// Matvecs of the decode step for batches of 16 tokens and more (QKV, o_proj,
// lm_head; the lm_head from 8 tokens, see jl_mm_ok in jl_internal.h): out[b][n] = hsum8_j( chain over s of fma(W[n][8s + j], x[b][8s + j]) )
// (+ bias[n]), the reference's 8-lane FMA order (decode_kernel.c:693-718,
// 969-995) with the AVX tree at the end, bit for bit.
//
// At these batch sizes the work is FP32-FMA bound (the order forbids tensor
// cores), so the kernel is register-tiled like an SGEMM: block = BN rows x BT
// tokens; warp j is lane j of the reference's accumulator, and its thread
// (rg, tg) holds RN x RT chains (rows rg*RN + r, tokens mm_token(tg, q)): per
// 8-column step it reads RN weights and RT token values (RN/4 and RT/4 16-byte
// shared loads) and issues RN*RT/2 packed fp32-pair FMAs (each lane rounds as
// fmaf; the pairs are 2 x 2 blocks of chains, diagonal and anti-diagonal). Each block reads its weight rows once.
// The token rows come column-major ([K][Bp], written by the producer kernel
// beside its row-major output), so a step's RT tokens are contiguous.
//
// Stages of 64 columns flow through a ring of 3 to 6 slots of 16-byte cp.async copies:
// the weight rows (the chunked lane-major layout of jl_mv.cuh, so a block's
// rows of one chunk are one contiguous run) and the token rows. Each stage's
// weights are widened to fp32 into [step][lane][row] once, one stage ahead
// of use; one barrier per stage. The 8 lanes' sums meet in shared memory and
// the AVX tree adds them.
#include <algorithm>

#include "jl_common.cuh"
#include "jl_internal.h"
#include "jl_mv.cuh"

namespace jl {

constexpr int kMmThreads = 256;
constexpr int kMmXPad = 4;  // floats of padding per staged column (16-byte rows)
// shared memory per block: three blocks per SM for the shapes whose registers
// allow three (RN x RT <= 16), two for the others
constexpr size_t kMmSmemCap3 = 72 * 1024, kMmSmemCap2 = 110 * 1024;

template <typename WT, int RN, int RT>
struct mm_shape {
    static constexpr int BN = 4 * RN, BT = 8 * RT;
    static constexpr int U = mv_traits<WT>::U;
    static constexpr int CPS = 8 / U;                 // weight chunks per 64-column stage
    static constexpr int WSS = BN + 4;                // fp32 weight row stride [step][lane][row]
    static constexpr int XS = BT + kMmXPad;           // floats per staged column of tokens
    static constexpr int X_F = 64 * XS;               // floats per token stage [64 columns][XS]
    static constexpr int WR_B = CPS * BN * 8 * 16;    // raw weight bytes per stage
    static constexpr int WS_F = 8 * 8 * WSS;          // floats per widened weight stage
    // ring depth: as many 64-column stages as fit the blocks per SM (3 to 6)
    static constexpr size_t stage_bytes = (size_t)X_F * 4 + WR_B;
    static constexpr size_t cap = RN * RT <= 16 ? kMmSmemCap3 : kMmSmemCap2;
    static constexpr int NS_fit = (int)((cap - (size_t)2 * WS_F * 4) / stage_bytes);
    static constexpr int NS = NS_fit < 3 ? 3 : NS_fit > 6 ? 6 : NS_fit;
    static constexpr size_t ring_bytes = (size_t)NS * stage_bytes + (size_t)2 * WS_F * 4;
    // lanes' sums [j][token][row]: rows in 4 groups of RN + 1 (one pad float
    // each), tokens RS = 4 (RN + 1) + 1 floats apart, so a warp's 32 stores
    // (8 token runs x 4 row groups) fall in distinct banks
    static constexpr int RS = 4 * (RN + 1) + 1;
    static constexpr size_t red_bytes = (size_t)8 * BT * RS * 4;
    static constexpr size_t smem = ring_bytes > red_bytes ? ring_bytes : red_bytes;
};

// Token (within the block's tile) of chain q of thread tg: runs of four
// consecutive tokens per lane, the lanes' runs side by side (tile tokens
// 4 tg .. 4 tg + 3, then 32 + 4 tg .., ...), so a warp's 16-byte loads of one
// run cover 128 contiguous bytes; two per lane when RT = 2.
__host__ __device__ constexpr int mm_token(int tg, int q, int RT) {
    return RT >= 4 ? (q / 4) * 32 + 4 * tg + q % 4 : RT * tg + q;
}

__device__ __forceinline__ void widen(uint4 v, float* dst, int stride, uint16_t) {  // 8 bf16 -> rows of dst
    dst[0] = __uint_as_float(v.x << 16);
    dst[stride] = __uint_as_float(v.x & 0xFFFF0000u);
    dst[2 * stride] = __uint_as_float(v.y << 16);
    dst[3 * stride] = __uint_as_float(v.y & 0xFFFF0000u);
    dst[4 * stride] = __uint_as_float(v.z << 16);
    dst[5 * stride] = __uint_as_float(v.z & 0xFFFF0000u);
    dst[6 * stride] = __uint_as_float(v.w << 16);
    dst[7 * stride] = __uint_as_float(v.w & 0xFFFF0000u);
}
__device__ __forceinline__ void widen(uint4 v, float* dst, int stride, float) {  // 4 fp32
    dst[0] = __uint_as_float(v.x);
    dst[stride] = __uint_as_float(v.y);
    dst[2 * stride] = __uint_as_float(v.z);
    dst[3 * stride] = __uint_as_float(v.w);
}

template <typename WT, int RN, int RT>
__global__ void __launch_bounds__(kMmThreads, RN * RT <= 16 ? 3 : 2) k_mm(const WT* __restrict__ W, const float* __restrict__ xT, int Bp,
                                                      int N, int K, int B, const float* __restrict__ bias,
                                                      float* __restrict__ out) {
    using S = mm_shape<WT, RN, RT>;
    constexpr int BN = S::BN, BT = S::BT, U = S::U, CPS = S::CPS, WSS = S::WSS, NS = S::NS, XS = S::XS;
    extern __shared__ __align__(16) float sm[];
    float* xr = sm;                                                      // [NS][64][XS]
    uint8_t* wr = reinterpret_cast<uint8_t*>(sm + NS * S::X_F);         // [NS][CPS][BN][8][U] raw
    float* ws = reinterpret_cast<float*>(wr + NS * S::WR_B);            // [2][8 steps][8 lanes][WSS]
    const int tid = threadIdx.x, j = tid >> 5, lane = tid & 31, rg = lane >> 3, tg = lane & 7;
    const int n0 = blockIdx.x * BN, t0 = blockIdx.y * BT;
    const int nst = K / 64;
    const size_t cstride = (size_t)N * 8 * U;  // elements per chunk of W'

    // Per-thread copy and widen assignments are the same at every stage: their
    // offsets are computed once (the stage adds a constant).
    constexpr int PW = CPS * BN * 8;            // 16-byte weight pieces per stage
    constexpr int KW = (PW + kMmThreads - 1) / kMmThreads;
    constexpr int PX = 64 * (BT / 4);           // 16-byte token pieces per stage
    constexpr int KX = (PX + kMmThreads - 1) / kMmThreads;
    // element offsets (32-bit: a stage adds CPS * N * 8U for the weights, 64 Bp
    // for the tokens, both far below 2^31 here)
    const WT* wbase = W + (size_t)(n0 * 8) * U;
    const float* xbase = xT + t0;
    int wsrc[KW], wst[KW], xsrc[KX], xdst[KX];  // wst: widened offset (floats), -1: no piece
    unsigned wlive = 0, xlive = 0;               // bit k: piece k exists and is in range
#pragma unroll
    for (int k = 0; k < KW; k++) {
        const int p = tid + k * kMmThreads;
        const int cc = p / (BN * 8), r = (p >> 3) % BN, jj = p & 7;
        if (p < PW && n0 + r < N) wlive |= 1u << k;
        wsrc[k] = cc * (int)cstride + (p % (BN * 8)) * U;
        wst[k] = p < PW ? ((cc * U) * 8 + jj) * WSS + r : -1;
    }
#pragma unroll
    for (int k = 0; k < KX; k++) {
        const int p = tid + k * kMmThreads;
        const int c = p / (BT / 4), q4 = (p % (BT / 4)) * 4;
        if (p < PX && t0 + q4 < B) xlive |= 1u << k;
        xsrc[k] = c * Bp + q4;
        xdst[k] = c * XS + q4;
    }
    const int wstep = CPS * (int)cstride, xstep = 64 * Bp;
    auto issue_w = [&](int st) {  // this stage's weight rows: CPS runs of BN * 128 bytes
        uint8_t* dst = wr + (st % NS) * S::WR_B;
#pragma unroll
        for (int k = 0; k < KW; k++)
            if ((wlive >> k) & 1u) cp_async16(dst + (tid + k * kMmThreads) * 16, wbase + wsrc[k] + st * wstep);
    };
    auto issue_x = [&](int st) {  // this stage's 64 columns of the token tile, 4 tokens per copy
        float* dst = xr + (st % NS) * S::X_F;
#pragma unroll
        for (int k = 0; k < KX; k++)
            if ((xlive >> k) & 1u) cp_async16(dst + xdst[k], xbase + xsrc[k] + st * xstep);
    };
    auto widen_stage = [&](int st) {  // raw weights of stage st -> ws[st & 1][s][j][row]
        const uint4* src = reinterpret_cast<const uint4*>(wr + (st % NS) * S::WR_B);
        float* dst = ws + (st & 1) * S::WS_F;
#pragma unroll
        for (int k = 0; k < KW; k++)
            if (wst[k] >= 0) widen(src[tid + k * kMmThreads], dst + wst[k], 8 * WSS, WT());
    };

    // weights do not depend on the previous kernel: their first NS - 1 stages
    // go out before the wait. Groups: G0 = {w0..w(NS-2), x0}, Gi = {xi} up to
    // G(NS-2); the loop's iteration st adds G(st+NS-1) = {w, x of stage st+NS-1}.
    for (int st = 0; st < NS - 1 && st < nst; st++) issue_w(st);
    griddep_wait();
    griddep_launch_dependents();
    for (int st = 0; st < NS - 1; st++) {
        if (st < nst) issue_x(st);
        cp_async_commit();
    }
    cp_async_wait<NS - 2>();  // G0
    __syncthreads();
    widen_stage(0);

    // chains in 2 x 2 blocks (rows 2i, 2i+1; tokens 2k, 2k+1), two packed FMAs
    // per block and step: dg[i][k] = {(2i, 2k), (2i+1, 2k+1)} takes the weight
    // pair times the token pair, an[i][k] = {(2i, 2k+1), (2i+1, 2k)} the weight
    // pair times the swapped token pair. Each lane is fmaf(w, x, acc).
    float2 dg[RN / 2][RT / 2], an[RN / 2][RT / 2];
#pragma unroll
    for (int i = 0; i < RN / 2; i++)
#pragma unroll
        for (int k = 0; k < RT / 2; k++) dg[i][k] = an[i][k] = make_float2(0.0f, 0.0f);

    for (int st = 0; st < nst; st++) {
        cp_async_wait<NS - 3>();  // this thread's copies up to stage st + 1 have landed
        __syncthreads();          // everyone's have; stage st - 1 is consumed; ws[st & 1] is complete
        if (st + NS - 1 < nst) {
            issue_w(st + NS - 1);
            issue_x(st + NS - 1);
        }
        cp_async_commit();
        if (st + 1 < nst) widen_stage(st + 1);
        const float* wsb = ws + (st & 1) * S::WS_F + j * WSS + rg * RN;
        const float* xb = xr + (st % NS) * S::X_F + j * XS + (RT >= 4 ? 4 : RT) * tg;
#pragma unroll
        for (int s = 0; s < 8; s++) {
            float w[RN], xv[RT];
#pragma unroll
            for (int r4 = 0; r4 < RN / 4; r4++) {
                const float4 v = *reinterpret_cast<const float4*>(wsb + s * 8 * WSS + r4 * 4);
                w[4 * r4] = v.x;
                w[4 * r4 + 1] = v.y;
                w[4 * r4 + 2] = v.z;
                w[4 * r4 + 3] = v.w;
            }
            if constexpr (RT % 4 == 0) {
#pragma unroll
                for (int q4 = 0; q4 < RT / 4; q4++) {
                    const float4 v = *reinterpret_cast<const float4*>(xb + s * 8 * XS + q4 * 32);
                    xv[4 * q4] = v.x;
                    xv[4 * q4 + 1] = v.y;
                    xv[4 * q4 + 2] = v.z;
                    xv[4 * q4 + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int q2 = 0; q2 < RT / 2; q2++) {
                    const float2 v = *reinterpret_cast<const float2*>(xb + s * 8 * XS + q2 * 2);
                    xv[2 * q2] = v.x;
                    xv[2 * q2 + 1] = v.y;
                }
            }
#pragma unroll
            for (int k = 0; k < RT / 2; k++) {
                const float2 xp = make_float2(xv[2 * k], xv[2 * k + 1]), xs = make_float2(xv[2 * k + 1], xv[2 * k]);
#pragma unroll
                for (int i = 0; i < RN / 2; i++) {
                    const float2 wp = make_float2(w[2 * i], w[2 * i + 1]);
                    dg[i][k] = __ffma2_rn(wp, xp, dg[i][k]);
                    an[i][k] = __ffma2_rn(wp, xs, an[i][k]);
                }
            }
        }
    }
    float acc[RN][RT];
#pragma unroll
    for (int i = 0; i < RN / 2; i++)
#pragma unroll
        for (int k = 0; k < RT / 2; k++) {
            acc[2 * i][2 * k] = dg[i][k].x;
            acc[2 * i + 1][2 * k + 1] = dg[i][k].y;
            acc[2 * i][2 * k + 1] = an[i][k].x;
            acc[2 * i + 1][2 * k] = an[i][k].y;
        }
    cp_async_wait<0>();
    __syncthreads();  // the ring is free: it becomes the lanes' reduction area [j][token][row]
    float* red = sm;
#pragma unroll
    for (int r = 0; r < RN; r++)
#pragma unroll
        for (int q = 0; q < RT; q++) red[(j * BT + mm_token(tg, q, RT)) * S::RS + rg * (RN + 1) + r] = acc[r][q];
    __syncthreads();
    for (int o = tid; o < BN * BT; o += kMmThreads) {
        const int r = o % BN, t = o / BN;
        if (n0 + r >= N || t0 + t >= B) continue;
        float l[8];
#pragma unroll
        for (int jj = 0; jj < 8; jj++) l[jj] = red[(jj * BT + t) * S::RS + (r / RN) * (RN + 1) + r % RN];
        float v = hsum8(l);
        if (bias) v = __fadd_rn(v, bias[n0 + r]);
        out[(size_t)(t0 + t) * N + n0 + r] = v;
    }
}

template <typename WT, int RN, int RT>
int launch_mm_shape(const WT* W, const float* xT, int Bp, int N, int K, int B, const float* bias, float* out,
                    cudaStream_t s) {
    using S = mm_shape<WT, RN, RT>;
    const dim3 grid((N + S::BN - 1) / S::BN, (B + S::BT - 1) / S::BT);
    return launch(k_mm<WT, RN, RT>, grid, dim3(kMmThreads), S::smem, s, W, xT, Bp, N, K, B, bias, out);
}

template <typename WT, int RN, int RT>
int mm_attr() {
    JL_CUDA(cudaFuncSetAttribute(k_mm<WT, RN, RT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)mm_shape<WT, RN, RT>::smem));
    return JL_OK;
}

template <typename WT>
int mm_attrs_for() {
    int rc = mm_attr<WT, 8, 8>();
    if (!rc) rc = mm_attr<WT, 8, 4>();
    if (!rc) rc = mm_attr<WT, 8, 2>();
    if (!rc) rc = mm_attr<WT, 4, 4>();
    if (!rc) rc = mm_attr<WT, 4, 2>();
    return rc;
}

}  // namespace jl

// (the kernel's per-thread copy offsets are 32-bit: the matrix stays below 2^31 elements)
bool jl_mm_ok(int N, int K, int B, int min_b) {
    return B >= min_b && B >= kMmMinB && K % 64 == 0 && N >= 1 && (long long)N * K < (1ll << 31);
}

// Tile choice (BN x BT = 4 RN x 8 RT), from timings of every shape on the
// decode step's matrices on a B200 (QKV 5120 x 2048, o_proj 2048 x 4096,
// lm_head 151936 x 2048 at B = 16, 32, 64; microseconds, best shape first):
//   QKV     B=16: 32x16 26.7, 16x16 26.8 | B=32: 16x32 37.7 | B=64: 16x32 59.5
//   o_proj  B=16: 16x16 22.7 | B=32: 32x16 30.0 | B=64: 32x32 48.1
//   lm_head B=16: 32x16 442 | B=32: 32x32 688 | B=64: 32x64 1146
// Token tiles no wider than the batch; for large N the widest such tile; for
// projection-sized N, 16-row tiles (more blocks) except at long K, where the
// per-block work is large anyway.
template <typename WT>
int jl_launch_mm(const WT* W, const float* xT, int Bp, int N, int K, int B, const float* bias, float* out,
                 int sm_count, cudaStream_t s) {
    using namespace jl;
    if (!jl_mm_ok(N, K, B, kMmMinB) || Bp % 4 || Bp < B || (long long)K * Bp >= (1ll << 31)) return JL_ERR_INVALID;
    const int rc = jl_device_once(sizeof(WT) == 2 ? kOnceMmBf16 : kOnceMmF32, [] { return mm_attrs_for<WT>(); });
    if (rc) return rc;
    const long rows32 = (N + 31) / 32;
    if (rows32 >= 8L * sm_count) {  // lm_head-sized
        if (B <= 16) return launch_mm_shape<WT, 8, 2>(W, xT, Bp, N, K, B, bias, out, s);
        if (B <= 32) return launch_mm_shape<WT, 8, 4>(W, xT, Bp, N, K, B, bias, out, s);
        return launch_mm_shape<WT, 8, 8>(W, xT, Bp, N, K, B, bias, out, s);
    }
    if (B <= 16) return launch_mm_shape<WT, 4, 2>(W, xT, Bp, N, K, B, bias, out, s);
    if (K >= 4096) {
        if (B <= 32) return launch_mm_shape<WT, 8, 2>(W, xT, Bp, N, K, B, bias, out, s);
        return launch_mm_shape<WT, 8, 4>(W, xT, Bp, N, K, B, bias, out, s);
    }
    return launch_mm_shape<WT, 4, 4>(W, xT, Bp, N, K, B, bias, out, s);
}

template int jl_launch_mm<uint16_t>(const uint16_t*, const float*, int, int, int, int, const float*, float*, int,
                                    cudaStream_t);
template int jl_launch_mm<float>(const float*, const float*, int, int, int, int, const float*, float*, int,
                                 cudaStream_t);
