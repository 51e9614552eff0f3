// Small-batch expert FFN (B <= 4), judged by HBM bandwidth. Same math as the
// reference's expert worker (decode_kernel.c:1251-1275, 1365-1384: gate and
// up rows of each union expert against its tokens, SwiGLU, down rows,
// weighted per-slot outputs), summed in another order: results agree with the
// reference within the 1e-3 row-relative bar; routing stays bit-exact (the
// router is shared with the other paths).
//
// At B <= 4 the cost per weight is the issue slots of its dequantisation and
// multiply, not the multiply's throughput, so the products run on mma.sync
// m16n8k16 (fp16 x fp16 -> fp32) used as a 256-MAC dot-product instruction:
// A = 16 weight rows x 16 values, dequantised in registers to the exact fp16
// (n - 8) (one lop3 and one packed subtract per two values); B = 8 columns,
// the up-to-4 tokens' activations split into fp16 hi and lo parts (x = hi +
// lo keeps ~22 bits); C accumulates in fp32 per 64-value group and is scaled
// by the group's fp16 scale in fp32. Lane (g, t) of a warp ends with token
// t's dot products (hi + lo columns) for rows g and g + 8: no shuffles.
//
// Value order inside a group: lane t owns bytes [8t, 8t + 8) of each of its
// two rows (values 16t .. 16t + 15); k-step ks takes word ks / 2 of them and
// its nibble pairs (i, i + 4), (i + 1, i + 5) with i = 2 (ks % 2). The token
// fragments are built in the same order (gv_frag_fill), so A and B agree.
//
// gate/up: block = (16-row strip of m, union expert); warp w takes the 64-value
// groups w, w + 8, ... of the strip's gate and up rows (every load of a batch
// issued before any arithmetic), the 8 warps' sums meet in shared memory in
// warp order, SwiGLU, act written per slot. The token fragments are built
// before the dependent-grid wait (x is the router's input).
// down: block = (64 rows of d, union expert); warp w takes 16 rows (w % 4)
// over half of the groups (w / 4), its records requested before the wait;
// the two halves' sums meet in shared memory; y[slot] = 0 + w * (row . act)
// per slot. The existing combine adds the slots in the reference's union order.
#include <algorithm>

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

constexpr int kGvWarps = 8;    // warps per block
constexpr int kGvMaxTok = 4;   // B <= 4: 4 tokens x (hi, lo) = the 8 mma columns
constexpr int kGuBatch = 2;    // gate/up: groups one warp holds in registers at a time
constexpr int kDnBatch = 6;    // down: groups one warp holds in registers at a time

// The 8 bytes lane t owns of row r of a tile record, and the row's scale.
struct q4row {
    uint2 v;
    uint32_t s;  // fp16 scale bits
};

__device__ __forceinline__ void load_row(const uint8_t* rec, int r, int t, q4row& q) {
    const uint8_t* p = rec + (t < 2 ? r * 16 + 8 * t : 512 + r * 16 + 8 * (t - 2));
    q.v = __ldg(reinterpret_cast<const uint2*>(p));
    q.s = __ldg(reinterpret_cast<const uint16_t*>(rec + kTileBytes) + r);
}

// half2 (1024 + n_lo, 1024 + n_hi) from the nibbles at bits 0-3 and 16-19.
__device__ __forceinline__ uint32_t nib_half2(uint32_t w) {
    uint32_t d;
    asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(d) : "r"(w));
    return d;
}
// h - (1032, 1032): exact, giving (n - 8) for both halves.
__device__ __forceinline__ uint32_t sub1032(uint32_t h) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(h), "r"(0x64086408u));
    return d;
}
// Word w (values v0..v7 at bits 4j) -> (v0, v4), (v1, v5), (v2, v6), (v3, v7) as fp16 (n - 8).
__device__ __forceinline__ void dq_word(uint32_t w, uint32_t (&h)[4]) {
    h[0] = sub1032(nib_half2(w));
    h[1] = sub1032(nib_half2(w >> 4));
    h[2] = sub1032(nib_half2(w >> 8));
    h[3] = sub1032(nib_half2(w >> 12));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One 64-value group of a 16-row strip: rows (r0 = g, r1 = g + 8) of this
// lane, against the token fragments xf[ks * 32 + lane]; acc += s_row * (row . x).
__device__ __forceinline__ void group_mma(const q4row& r0, const q4row& r1, const uint2* xf, int lane,
                                          float (&acc)[4]) {
    uint32_t a00[4], a01[4], a10[4], a11[4];  // row 0 words 0, 1; row 1 words 0, 1
    dq_word(r0.v.x, a00);
    dq_word(r0.v.y, a01);
    dq_word(r1.v.x, a10);
    dq_word(r1.v.y, a11);
    float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < 4; ks++) {
        const int i = 2 * (ks & 1);
        const uint32_t a[4] = {ks < 2 ? a00[i] : a01[i], ks < 2 ? a10[i] : a11[i], ks < 2 ? a00[i + 1] : a01[i + 1],
                               ks < 2 ? a10[i + 1] : a11[i + 1]};
        const uint2 b = xf[ks * 32 + lane];
        mma16816(c, a, b.x, b.y);
    }
    const float s0 = half_bits_to_f32((uint16_t)r0.s), s1 = half_bits_to_f32((uint16_t)r1.s);
    acc[0] = __fmaf_rn(s0, c[0], acc[0]);
    acc[1] = __fmaf_rn(s0, c[1], acc[1]);
    acc[2] = __fmaf_rn(s1, c[2], acc[2]);
    acc[3] = __fmaf_rn(s1, c[3], acc[3]);
}

// Token fragments for the mma B operand, entry (group g, k-step ks, lane =
// 4 gid + t) of a [ngroups][4][32] table: column gid = 2 * token + part (part
// 0 the fp16 hi part, 1 the lo part); k rows (2t, 2t + 1) and (2t + 8, 2t + 9)
// hold the values base + i + {0, 4} and base + i + {1, 5}. One call fills the
// 8 entries of one (g, ks, t) for every column; rows[j] is token j's row of
// floats, j < nt (the other columns are zero).
__device__ __forceinline__ void gv_frag_fill(uint2* tab, int g, int ks, int t, const float* const* rows, int nt) {
    const int base = 64 * g + 16 * t + 8 * (ks >> 1) + 2 * (ks & 1);
    uint2* e = tab + (g * 4 + ks) * 32 + t;
#pragma unroll
    for (int j = 0; j < kGvMaxTok; j++) {
        uint2 hi2 = make_uint2(0u, 0u), lo2 = make_uint2(0u, 0u);
        if (j < nt) {
            const float* row = rows[j];
            const float v[4] = {row[base], row[base + 4], row[base + 1], row[base + 5]};
            uint32_t h[4], l[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const __half hh = __float2half_rn(v[i]);
                h[i] = __half_as_ushort(hh);
                l[i] = __half_as_ushort(__float2half_rn(__fsub_rn(v[i], __half2float(hh))));
            }
            hi2 = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
            lo2 = make_uint2(l[0] | (l[1] << 16), l[2] | (l[3] << 16));
        }
        e[(2 * j) * 4] = hi2;
        e[(2 * j + 1) * 4] = lo2;
    }
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kGvWarps * 32, 3) k_gateup_gemv(const uint8_t* __restrict__ store_l,
                                                                  jl_layout L, int k,
                                                                  const float* __restrict__ x, int B, jl_ws ws) {
    extern __shared__ __align__(16) uint2 xf[];  // [ngd][4][32] token fragments
    __shared__ float red[kGvWarps][32][8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = lane & 3;
    const int d = L.d, m = L.m, ngd = L.ngd;
    const int strip = blockIdx.x, u = blockIdx.y;
    long long* tr = (blockIdx.x == 0 && blockIdx.y == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceGateup, 0);
    // x is the router's input: complete before the router released this grid
    {
        const float* rows[kGvMaxTok];
#pragma unroll
        for (int j = 0; j < kGvMaxTok; j++) rows[j] = x + (size_t)min(j, B - 1) * d;
        for (int q = threadIdx.x; q < ngd * 16; q += blockDim.x) gv_frag_fill(xf, q >> 4, (q >> 2) & 3, q & 3, rows, B);
    }
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceGateup, 1);
    if (u >= *ws.U) return;
    const uint8_t* base = store_l + (size_t)ws.sel[u] * L.rec_bytes;
    const int rb = strip >> 1, r0 = 16 * (strip & 1) + (lane >> 2);
    __syncthreads();  // the fragments
    trace_point(tr, kTraceGateup, 2);
    float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g0 = warp; g0 < ngd; g0 += kGvWarps * kGuBatch) {
        q4row gr[kGuBatch][2], ur[kGuBatch][2];  // every record of the batch requested before any arithmetic
#pragma unroll
        for (int i = 0; i < kGuBatch; i++) {
            const int g = g0 + kGvWarps * i;
            if (g < ngd) {
                const uint8_t* rg = base + L.tile_off(0, rb, g);
                const uint8_t* ru = base + L.tile_off(1, rb, g);
                load_row(rg, r0, t, gr[i][0]);
                load_row(rg, r0 + 8, t, gr[i][1]);
                load_row(ru, r0, t, ur[i][0]);
                load_row(ru, r0 + 8, t, ur[i][1]);
            }
        }
#pragma unroll
        for (int i = 0; i < kGuBatch; i++) {
            const int g = g0 + kGvWarps * i;
            if (g < ngd) {
                group_mma(gr[i][0], gr[i][1], xf + g * 128, lane, ag);
                group_mma(ur[i][0], ur[i][1], xf + g * 128, lane, au);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        red[warp][lane][i] = ag[i];
        red[warp][lane][4 + i] = au[i];
    }
    __syncthreads();
    if (warp == 0 && t < B) {  // lane (g, t): token t, rows r0 and r0 + 8 of the strip; sums in warp order
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = red[0][lane][i];
        for (int w = 1; w < kGvWarps; w++)
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = __fadd_rn(v[i], red[w][lane][i]);
        const int s0 = ws.uh[u], s1 = ws.uh[u + 1];
        for (int pos = s0; pos < s1; pos++) {
            const int slot = ws.uidx[pos];
            if (slot / k != t) continue;
            const int row = 16 * strip + (lane >> 2);
            ws.act[(size_t)slot * m + row] = silu_mul(__fadd_rn(v[0], v[1]), __fadd_rn(v[4], v[5]));
            ws.act[(size_t)slot * m + row + 8] = silu_mul(__fadd_rn(v[2], v[3]), __fadd_rn(v[6], v[7]));
        }
    }
    trace_point(tr, kTraceGateup, 3);
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kGvWarps * 32, 3) k_down_gemv(const uint8_t* __restrict__ store_l, jl_layout L,
                                                                int k, jl_ws ws) {
    extern __shared__ __align__(16) uint2 af[];  // [ngm][4][32] the expert's act fragments
    __shared__ float red[4][32][4];
    __shared__ int slot_s[kGvMaxTok];
    __shared__ float w_s[kGvMaxTok];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = lane & 3;
    const int d = L.d, m = L.m, ngm = L.ngm;
    const int mt = blockIdx.x, u = blockIdx.y;
    const int strip = warp & 3, half = warp >> 2;  // 4 strips of 16 rows; two halves of the groups
    long long* tr = (blockIdx.x == 0 && blockIdx.y == 0) ? ws.trace : nullptr;
    trace_point(tr, kTraceDown, 0);
    // the routing is known before the wait (only act is gate/up's output)
    if (u >= *ws.U) {
        griddep_wait();
        griddep_launch_dependents();
        return;
    }
    const uint8_t* base = store_l + (size_t)ws.sel[u] * L.rec_bytes;
    const int rb = 2 * mt + (strip >> 1), r0 = 16 * (strip & 1) + (lane >> 2);
    q4row rr[kDnBatch][2];
#pragma unroll
    for (int i = 0; i < kDnBatch; i++) {
        const int g = half + 2 * i;
        if (g < ngm) {
            const uint8_t* rec = base + L.tile_off(2, rb, g);
            load_row(rec, r0, t, rr[i][0]);
            load_row(rec, r0 + 8, t, rr[i][1]);
        }
    }
    const int s0 = ws.uh[u], nt = min(kGvMaxTok, ws.uh[u + 1] - s0);
    if (threadIdx.x < nt) {
        slot_s[threadIdx.x] = ws.uidx[s0 + threadIdx.x];
        w_s[threadIdx.x] = ws.uw[s0 + threadIdx.x];
    }
    griddep_wait();
    griddep_launch_dependents();
    trace_point(tr, kTraceDown, 1);
    __syncthreads();  // slot_s
    {
        const float* rows[kGvMaxTok];
#pragma unroll
        for (int j = 0; j < kGvMaxTok; j++) rows[j] = ws.act + (size_t)slot_s[min(j, nt - 1)] * m;
        for (int q = threadIdx.x; q < ngm * 16; q += blockDim.x) gv_frag_fill(af, q >> 4, (q >> 2) & 3, q & 3, rows, nt);
    }
    __syncthreads();
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g0 = half; g0 < ngm; g0 += 2 * kDnBatch) {
        if (g0 > half) {
#pragma unroll
            for (int i = 0; i < kDnBatch; i++) {
                const int g = g0 + 2 * i;
                if (g < ngm) {
                    const uint8_t* rec = base + L.tile_off(2, rb, g);
                    load_row(rec, r0, t, rr[i][0]);
                    load_row(rec, r0 + 8, t, rr[i][1]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kDnBatch; i++) {
            const int g = g0 + 2 * i;
            if (g < ngm) group_mma(rr[i][0], rr[i][1], af + g * 128, lane, acc);
        }
    }
    if (half == 1)
#pragma unroll
        for (int i = 0; i < 4; i++) red[strip][lane][i] = acc[i];
    __syncthreads();
    if (half == 0 && t < nt) {  // lane (g, t): the expert's token t, rows r0 and r0 + 8; halves in order
        const int row = 64 * mt + 16 * strip + (lane >> 2);
        const float w = w_s[t];
        float* y = ws.y + (size_t)slot_s[t] * d;
        const float v0 = __fadd_rn(__fadd_rn(acc[0], red[strip][lane][0]), __fadd_rn(acc[1], red[strip][lane][1]));
        const float v1 = __fadd_rn(__fadd_rn(acc[2], red[strip][lane][2]), __fadd_rn(acc[3], red[strip][lane][3]));
        y[row] = __fadd_rn(0.0f, __fmul_rn(w, v0));
        y[row + 8] = __fadd_rn(0.0f, __fmul_rn(w, v1));
    }
    trace_point(tr, kTraceDown, 3);
}

}  // namespace jl

bool jl_gemv_ok(const jl_moe* h, int B) {
    using namespace jl;
    return B >= 1 && B <= kGvMaxTok && h->d % 128 == 0 && h->m % 64 == 0 && h->lay.ngd <= 96 && h->lay.ngm <= 96;
}

static int gemv_attrs() {
    return jl_device_once(kOnceGemv, [] {
        using namespace jl;
        const int big = 100 * 1024;
        JL_CUDA(cudaFuncSetAttribute(k_gateup_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_down_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        return JL_OK;
    });
}

int jl_launch_gateup_gemv(const jl_moe* h, const uint8_t* store_l, const float* x, int B, cudaStream_t s) {
    using namespace jl;
    if (!jl_gemv_ok(h, B)) return JL_ERR_INVALID;
    int rc = gemv_attrs();
    if (rc) return rc;
    const size_t smem = (size_t)h->lay.ngd * 4 * 32 * sizeof(uint2);
    const dim3 grid(h->m / 16, std::min(h->E, B * h->k)), block(kGvWarps * 32);
    return launch(k_gateup_gemv, grid, block, smem, s, store_l, h->lay, h->k, x, B, h->ws);
}

int jl_launch_down_gemv(const jl_moe* h, const uint8_t* store_l, int B, cudaStream_t s) {
    using namespace jl;
    if (!jl_gemv_ok(h, B)) return JL_ERR_INVALID;
    int rc = gemv_attrs();
    if (rc) return rc;
    const size_t smem = (size_t)h->lay.ngm * 4 * 32 * sizeof(uint2);
    const dim3 grid(h->d / 64, std::min(h->E, B * h->k)), block(kGvWarps * 32);
    return launch(k_down_gemv, grid, block, smem, s, store_l, h->lay, h->k, h->ws);
}
