// The decode step around the MoE layer on the GPU: RMSNorm, bf16 QKV and
// o_proj, QKV bias, QK-norm (per head or whole vector), RoPE, attention over
// per-sequence KV caches, the fp32 lm_head and the argmax, in the reference's
// arithmetic order (decode_layers_batch, decode_kernel.c:1518-1556, with
// layer_attn_batch 1120-1234, rms_norm 224-230, rope_apply 259-266,
// sqrtf_fast 88-93, matvec_B_worker 693-718, lm_B_worker 969-995), so that a
// decode step gives the reference's logits bit for bit when the MoE layer runs
// on its exact path.
//
// Per layer: k_rms (h += previous residual, norm1) -> k_mv (QKV, + bias) ->
// k_attn_qk (QK-norm, RoPE, KV append, scores) -> k_attn_pv (softmax, values)
// -> k_mv (o_proj) ->
// k_rms (h += o, norm2) -> the MoE layer (jl_moe_forward) -> next layer.
// Then k_rms (final norm) -> k_mv (fp32 lm_head) -> k_argmax.
//
// Every sum the reference forms sequentially stays one sequential chain here
// (the norms' sums of squares, the attention's score, softmax and value sums);
// the parallelism is across rows, heads, positions and sequences. The matvecs
// use the reference's 8-lane FMA order: lane j of a row sums the products of
// columns j, j+8, j+16, ... by fused multiply-add, then the AVX tree
// ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7)).
//
// Weight layout for the matvecs (coalesced 16-byte loads): matrix W [N, K] is
// stored as W'[c][n][j][u] = W[n][j + 8*(U*c + u)] with U = 8 values per
// 16 bytes for bf16 (4 for fp32); thread (row n, lane j) reads chunk c as one
// 16-byte load and a warp (4 rows x 8 lanes) reads 512 contiguous bytes.
#include <algorithm>
#include <climits>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "jl_common.cuh"
#include "jl_internal.h"
#include "jl_mv.cuh"

namespace jl {

constexpr int kMvRows = 16;           // rows per matvec block (x 8 lanes = 128 threads)
constexpr int kMvTok = 8;             // tokens per pass of a matvec block
constexpr int kAttnThreads = 128;     // attention block (head dim <= 128)
constexpr int kNormThreads = 256;
constexpr int kErrPosition = 8;       // a position outside [0, maxT) (error word bit)

// decode_kernel.c:88-93: halve the exponent for a first estimate, then one
// Newton step 0.5 * (y + x / y).
__device__ __forceinline__ float sqrtf_fast(float x) {
    const float y = __uint_as_float((__float_as_uint(x) + 0x3F800000u) >> 1);
    return __fmul_rn(0.5f, __fadd_rn(y, __fdiv_rn(x, y)));
}

// 1 / sqrtf_fast(ss / n + eps) (decode_kernel.c:227, 1168, 1181)
__device__ __forceinline__ float rms_inv(float ss, int n, float eps) {
    return __fdiv_rn(1.0f, sqrtf_fast(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// Sequential sum of v[0..n) in index order by the calling thread (n % 4 == 0,
// v 16-byte aligned): loads run ahead of the one dependent add chain.
__device__ __forceinline__ float chain_sum(const float* v, int n) {
    float s = 0.0f;
    const float4* v4 = reinterpret_cast<const float4*>(v);
#pragma unroll 8
    for (int i = 0; i < n / 4; i++) {
        const float4 q = v4[i];
        s = __fadd_rn(s, q.x);
        s = __fadd_rn(s, q.y);
        s = __fadd_rn(s, q.z);
        s = __fadd_rn(s, q.w);
    }
    return s;
}

// ---------------------------------------------------------------------------
// Residual add + RMSNorm (decode_kernel.c:224-230, 1528-1535). One block per
// sequence b: h[b] += add[b] (when add != null), then t[b] = (h * inv) * w
// with inv from the sum of squares in index order.
__global__ void __launch_bounds__(kNormThreads) k_rms(float* __restrict__ h, const float* __restrict__ add,
                                                      const uint16_t* __restrict__ w, float eps, int d,
                                                      float* __restrict__ t, float* __restrict__ tT, int Bp) {
    extern __shared__ __align__(16) float sm[];  // v [d], squares [d]
    float* v_s = sm;
    float* sq = sm + d;
    __shared__ float inv_s;
    griddep_wait();
    griddep_launch_dependents();
    const int b = blockIdx.x, n4 = d / 4;
    float4* h4 = reinterpret_cast<float4*>(h + (size_t)b * d);
    const float4* a4 = add ? reinterpret_cast<const float4*>(add + (size_t)b * d) : nullptr;
    for (int i0 = threadIdx.x; i0 < n4; i0 += 4 * blockDim.x) {  // four float4 loads in flight
        float4 hv[4], av[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = i0 + j * blockDim.x;
            if (i < n4) {
                hv[j] = h4[i];
                if (a4) av[j] = a4[i];
            }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = i0 + j * blockDim.x;
            if (i >= n4) continue;
            float4 v = hv[j];
            if (a4) {
                v = make_float4(__fadd_rn(v.x, av[j].x), __fadd_rn(v.y, av[j].y), __fadd_rn(v.z, av[j].z),
                                __fadd_rn(v.w, av[j].w));
                h4[i] = v;
            }
            reinterpret_cast<float4*>(v_s)[i] = v;
            reinterpret_cast<float4*>(sq)[i] =
                make_float4(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y), __fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w));
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) inv_s = rms_inv(chain_sum(sq, d), d, eps);
    __syncthreads();
    const float inv = inv_s;
    const uint2* w4 = reinterpret_cast<const uint2*>(w);  // 4 bf16 per load
    float4* t4 = reinterpret_cast<float4*>(t + (size_t)b * d);
    for (int i0 = threadIdx.x; i0 < n4; i0 += 4 * blockDim.x) {
        uint2 wv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = i0 + j * blockDim.x;
            if (i < n4) wv[j] = __ldg(w4 + i);
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = i0 + j * blockDim.x;
            if (i >= n4) continue;
            const float4 v = reinterpret_cast<const float4*>(v_s)[i];
            const float4 o = make_float4(__fmul_rn(__fmul_rn(v.x, inv), bf16_to_f32(wv[j].x & 0xFFFFu)),
                                __fmul_rn(__fmul_rn(v.y, inv), bf16_to_f32(wv[j].x >> 16)),
                                __fmul_rn(__fmul_rn(v.z, inv), bf16_to_f32(wv[j].y & 0xFFFFu)),
                                __fmul_rn(__fmul_rn(v.w, inv), bf16_to_f32(wv[j].y >> 16)));
            t4[i] = o;
            if (tT) {  // column-major copy [d][Bp] for the large-batch matvec
                tT[(size_t)(4 * i) * Bp + b] = o.x;
                tT[(size_t)(4 * i + 1) * Bp + b] = o.y;
                tT[(size_t)(4 * i + 2) * Bp + b] = o.z;
                tT[(size_t)(4 * i + 3) * Bp + b] = o.w;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// out[b, n] = W[n, :] . x[b, :] (+ bias[n], a separate add as the reference's
// `q[i] += bq[i]`), W in the chunked lane-major layout above. Block: 32 rows x
// 8 lanes; it runs the B tokens in passes of kMvTok, with the pass's token
// rows staged lane-major in shared memory (x_s[t][j][i] = x[b0+t][j + 8i], rows
// padded by 4 floats so the 8 lanes' float4 reads hit distinct banks). The
// block's weight rows are re-read from L2 on later passes.

// Block (token group blockIdx.x, row blocks blockIdx.y) stages the NT token
// rows of its group once, then runs RT consecutive tiles of kMvRows rows
// against them. The token group varies fastest in the grid, so the blocks
// that read the same weight rows run at about the same time and all but the
// first find them in L2.
template <typename WT, int NT>
__global__ void __launch_bounds__(kMvRows * 8) k_mv(const WT* __restrict__ W, const float* __restrict__ x,
                                                    int N, int K, int B, const float* __restrict__ bias,
                                                    float* __restrict__ out, int RT, int pf) {
    constexpr int U = mv_traits<WT>::U;
    constexpr int P = 8;  // chunks per load group; the next group is in flight while one is used
    extern __shared__ __align__(16) float x_s[];  // [NT][8][K/8 + 4]
    const int tid = threadIdx.x, j = tid & 7;
    const int nc = K / (8 * U), xs = mv_xstride(K);
    const size_t cstride = (size_t)N * 8;  // uint4 per chunk
    const int tile0 = blockIdx.y * RT;
    auto row_of = [=](int rt) { return (tile0 + rt) * kMvRows + (tid >> 3); };
    auto load_group = [=](int n, int c0, uint4 (&w)[P]) {
        const bool live = n < N;
        const uint4* wp = reinterpret_cast<const uint4*>(W) + (size_t)(live ? n : 0) * 8 + j;
#pragma unroll
        for (int i = 0; i < P; i++)
            w[i] = (live && c0 + i < nc) ? __ldg(wp + (size_t)(c0 + i) * cstride) : make_uint4(0, 0, 0, 0);
    };
    uint4 cur[P], nxt[P];
    load_group(row_of(0), 0, cur);  // weights do not depend on the previous kernel: fetch before the wait
    if (pf && blockIdx.x == 0) {  // and the rest of this block's rows into L2 while the producer runs
        const int r0 = tile0 * kMvRows, r1 = min(N, (tile0 + RT) * kMvRows);
        for (int c = tid; c < nc && r1 > r0; c += blockDim.x)
            prefetch_l2(W + ((size_t)c * N + r0) * 8 * U, (uint32_t)(r1 - r0) * 128u);
    }
    griddep_wait();
    griddep_launch_dependents();
    const int b0 = blockIdx.x * NT, nt = min(NT, B - b0);
    {  // the group's token rows into lane-major rows; float4 loads, four in flight per thread
        const int n4 = nt * K / 4, k4 = K / 4;
        for (int i0 = tid; i0 < n4; i0 += 4 * blockDim.x) {
            float4 r[4];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const int i = i0 + jj * blockDim.x;
                if (i < n4) r[jj] = reinterpret_cast<const float4*>(x + (size_t)b0 * K)[i];
            }
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const int i = i0 + jj * blockDim.x;
                if (i >= n4) continue;
                const int t = i / k4, c = (i - t * k4) * 4;  // c % 8 is 0 or 4
                float* dst = x_s + (size_t)(t * 8 + (c & 7)) * xs + (c >> 3);
                dst[0] = r[jj].x;
                dst[xs] = r[jj].y;
                dst[2 * xs] = r[jj].z;
                dst[3 * xs] = r[jj].w;
            }
        }
    }
    __syncthreads();
    for (int rt = 0; rt < RT; rt++) {
        const int n = row_of(rt);
        if ((tile0 + rt) * kMvRows >= N) break;  // whole block: past the last row tile
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.0f;
        for (int c0 = 0; c0 < nc; c0 += P) {
            // the next group of this tile, or the first group of the next tile
            if (c0 + P < nc) load_group(n, c0 + P, nxt);
            else if (rt + 1 < RT) load_group(row_of(rt + 1), 0, nxt);
#pragma unroll
            for (int i = 0; i < P; i++) {
                if (c0 + i < nc) {
#pragma unroll
                    for (int t = 0; t < NT; t++)
                        if (t < nt) fma_chunk(cur[i], x_s + (size_t)(t * 8 + j) * xs + (c0 + i) * U, acc[t], WT());
                }
            }
#pragma unroll
            for (int i = 0; i < P; i++) cur[i] = nxt[i];
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            float a = acc[t];
            a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
            a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 2));
            a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
            if (n < N && j == 0 && t < nt) {
                if (bias) a = __fadd_rn(a, bias[n]);
                out[(size_t)(b0 + t) * N + n] = a;
            }
        }
    }
}


// ---------------------------------------------------------------------------
// Attention (decode_kernel.c:1150-1231) in two launches.
//
// k_attn_qk, block (KV head g, sequence b, position split p): QK-norm and RoPE
// of the group's q heads and of k, the KV append (split 0), then the scores
// q.k_t / sqrtf_fast(hd) of the group's heads for the split's positions, each
// a sequential sum over the head dimension (two chains per thread), into a
// [B][H][maxT] score buffer. The block that holds
// position pos uses the k row it computed itself, so no block reads a row
// another block is writing.
//
// k_attn_pv, block (heads h0..h0+hpb of one KV group, sequence b, dimension
// slice z): per head (one warp each) max over t, p_t = expf_fast(s_t - max),
// their sum in t order by one lane, p_t /= sum; then att[i] = 0 + p_0 v_0[i]
// + p_1 v_1[i] + ... in t order for the slice's dimensions of every head, V
// tiles by 16-byte cp.async, read once for the block's heads (hpb = the group
// size at large batches; one head per block at small ones, for more blocks).
//
// Parallelism is across (group, sequence, positions) and (head, sequence,
// dimensions); every sum the reference forms sequentially stays one chain.
struct attn_args {
    const float* qkv;        // [B][qn + 2 kn] (bias added)
    float* att;              // [B][qn]
    float* attT;             // [qn][Bp] column-major copy for the large-batch matvec, or null
    int Bp;
    const int* positions;    // [B]
    const int* slots;        // [B] KV cache slot of each sequence
    float* kc;               // [slots][L][maxT][kn]
    float* vc;
    const uint16_t* qnw;     // QK-norm weights of this layer (per head [hd] or whole [qn]/[kn])
    const uint16_t* knw;
    const float* cosb;       // [maxT][hd]
    const float* sinb;
    int l, L, H, KH, hd, maxT, qk_type;
    int nslots;              // KV cache slots held
    int from_cache;          // 1: this position's K/V rows are already in the cache (k_kv_append ran)
    int sqn;                 // floats per squares buffer of k_kv_append: max(qn, kn) for whole-vector norms, else hd
    float eps;
    int* err;
    float* qr;               // [B][H][hd] q after QK-norm and RoPE (register-tiled attention)
};

// Squares of v[0..n) into sq (n % 4 == 0, 16-byte aligned), loads batched.
__device__ __forceinline__ void squares(const float* __restrict__ v, int n, float* sq) {
    const float4* v4 = reinterpret_cast<const float4*>(v);
    float4* s4 = reinterpret_cast<float4*>(sq);
    for (int i0 = threadIdx.x; i0 < n / 4; i0 += 4 * blockDim.x) {
        float4 r[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = i0 + j * blockDim.x;
            if (i < n / 4) r[j] = v4[i];
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = i0 + j * blockDim.x;
            if (i < n / 4)
                s4[i] = make_float4(__fmul_rn(r[j].x, r[j].x), __fmul_rn(r[j].y, r[j].y), __fmul_rn(r[j].z, r[j].z),
                                    __fmul_rn(r[j].w, r[j].w));
        }
    }
}

// Sum of squares of v[0..n) in index order by the calling thread (n % 4 == 0,
// v 16-byte aligned): each square rounded, then added (decode_kernel.c:1181).
__device__ __forceinline__ float chain_sumsq(const float* v, int n) {
    float s = 0.0f;
    const float4* v4 = reinterpret_cast<const float4*>(v);
#pragma unroll 8
    for (int i = 0; i < n / 4; i++) {
        const float4 q = v4[i];
        s = __fadd_rn(s, __fmul_rn(q.x, q.x));
        s = __fadd_rn(s, __fmul_rn(q.y, q.y));
        s = __fadd_rn(s, __fmul_rn(q.z, q.z));
        s = __fadd_rn(s, __fmul_rn(q.w, q.w));
    }
    return s;
}

// The score kernels' prologue for KV group g of sequence b at position pos:
// the group's q heads into q_s [gsz][qs], the k and v rows into k_s, v_s
// [hd], then QK-norm and RoPE of q_s and k_s (decode_kernel.c:1162-1199).
// The rows and this position's RoPE tables (cs_s, sn_s [hd]) arrive as one
// batch of 16-byte copies with a single wait (the caller's earlier copy
// groups complete with it). sq holds the squares of the whole-vector norm
// (qk_type 2; qn + kn floats, each part padded to 4), inv gsz + 1 floats.
// Every thread of the block calls it; it ends with a barrier.
__device__ void qk_prepare(const attn_args& a, int g, int b, int pos, float* q_s, int qs, float* k_s, float* v_s,
                           float* cs_s, float* sn_s, float* sq, float* inv) {
    const int hd = a.hd, qn = a.H * hd, kn = a.KH * hd, gsz = a.H / a.KH, h0 = g * gsz, tid = threadIdx.x;
    const int c4 = hd / 4;
    const float* row = a.qkv + (size_t)b * (qn + 2 * kn);
    for (int r = 0; r < gsz + 4; r++) {  // q rows, k, v, cos, sin (all 16-byte aligned: hd % 4 == 0)
        float* dst = r < gsz ? q_s + r * qs : r == gsz ? k_s : r == gsz + 1 ? v_s : r == gsz + 2 ? cs_s : sn_s;
        const float* src = r < gsz         ? row + (h0 + r) * hd
                           : r == gsz      ? row + qn + g * hd
                           : r == gsz + 1  ? row + qn + kn + g * hd
                           : r == gsz + 2  ? a.cosb + (size_t)pos * hd
                                           : a.sinb + (size_t)pos * hd;
        for (int c = tid; c < c4; c += blockDim.x) cp_async16(dst + 4 * c, src + 4 * c);
    }
    cp_async_commit();
    if (a.qk_type == 2) {  // whole vectors q [qn], k [kn] (decode_kernel.c:1162-1174)
        const int qn4 = (qn + 3) / 4 * 4;
        squares(row, qn, sq);
        squares(row + qn, kn, sq + qn4);
        cp_async_wait<0>();
        __syncthreads();
        if (tid == 0) inv[0] = rms_inv(chain_sum(sq, qn), qn, a.eps);
        if (tid == (blockDim.x > 32 ? 32 : 1)) inv[1] = rms_inv(chain_sum(sq + qn4, kn), kn, a.eps);
        __syncthreads();
        for (int c = tid; c < hd; c += blockDim.x) {
            for (int hh = 0; hh < gsz; hh++) {
                float* q = q_s + hh * qs + c;
                *q = __fmul_rn(__fmul_rn(*q, inv[0]), bf16_to_f32(a.qnw[(h0 + hh) * hd + c]));
            }
            k_s[c] = __fmul_rn(__fmul_rn(k_s[c], inv[1]), bf16_to_f32(a.knw[g * hd + c]));
        }
    } else {
        cp_async_wait<0>();
        __syncthreads();
        if (a.qk_type == 1) {  // per head, weights [hd] (decode_kernel.c:1180-1193)
            if (tid <= gsz) inv[tid] = rms_inv(chain_sumsq(tid < gsz ? q_s + tid * qs : k_s, hd), hd, a.eps);
            __syncthreads();
            for (int c = tid; c < hd; c += blockDim.x) {
                const float wq = bf16_to_f32(a.qnw[c]);
                for (int hh = 0; hh < gsz; hh++) {
                    float* q = q_s + hh * qs + c;
                    *q = __fmul_rn(__fmul_rn(*q, inv[hh]), wq);
                }
                k_s[c] = __fmul_rn(__fmul_rn(k_s[c], inv[gsz]), bf16_to_f32(a.knw[c]));
            }
        }
    }
    __syncthreads();
    // RoPE, rotate-half (decode_kernel.c:259-266, 1195-1199); each item owns its pair
    const int half = hd / 2;
    for (int i = tid; i < half; i += blockDim.x) {
        const float cs = cs_s[i], sn = sn_s[i];
        for (int hh = 0; hh <= gsz; hh++) {
            float* v = hh < gsz ? q_s + hh * qs : k_s;
            const float x0 = v[i], x1 = v[i + half];
            v[i] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            v[i + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
    }
    __syncthreads();
}

constexpr int kQkThreads = 256;
constexpr int kQkTile = 64;   // positions per K tile
constexpr int kQkRing = 3;    // K tiles in the ring (two in flight while one is used)
constexpr int kPvThreads = 256;
constexpr int kPvTile = 16;   // positions per V tile
constexpr int kPvRing = 8;    // V tiles in the ring (seven in flight while one is used)
constexpr int kPvItems = 4;   // (head, four dimensions) items per thread at most (NI of k_attn_pv)

// Shared-memory layout of k_attn_qk (floats): q [gsz][hd + 4], k [hd],
// v [hd], cos [hd], sin [hd], squares (whole-vector QK-norm only), inverse norms [gsz + 1]
// (padded to 4), K tiles [kQkTile][hd + 4] x kQkRing.
struct qk_layout {
    int qs, sq, inv, tiles, total;
    __host__ __device__ qk_layout(int qk_type, int H, int KH, int hd) {
        const int gsz = H / KH, qrow = hd + 4;
        qs = qrow;
        sq = gsz * qrow + 4 * hd;
        const int nsq = qk_type == 2 ? (H * hd + 3) / 4 * 4 + (KH * hd + 3) / 4 * 4 : 0;
        inv = sq + (nsq + 3) / 4 * 4;
        tiles = inv + (gsz + 4) / 4 * 4;
        total = tiles + kQkRing * kQkTile * qrow;
    }
};

__global__ void __launch_bounds__(kQkThreads) k_attn_qk(attn_args a, float* __restrict__ scores, int tp) {
    extern __shared__ __align__(16) float sm[];
    const int g = blockIdx.x, b = blockIdx.y, split = blockIdx.z, tid = threadIdx.x;
    const int hd = a.hd, qn = a.H * hd, kn = a.KH * hd, gsz = a.H / a.KH, h0 = g * gsz;
    const qk_layout lay(a.qk_type, a.H, a.KH, hd);
    const int QS = lay.qs, KP = hd + 4;
    float* q_s = sm;                 // [gsz][QS]
    float* k_s = sm + gsz * QS;      // [hd]
    float* v_s = k_s + hd;           // [hd]
    float* cs_s = v_s + hd;          // [hd]
    float* sn_s = cs_s + hd;         // [hd]
    float* sq = sm + lay.sq;
    float* inv = sm + lay.inv;
    float* tb0 = sm + lay.tiles;     // tile j at tb0 + (j % kQkRing) * kQkTile * KP
    griddep_wait();
    griddep_launch_dependents();
    const int pos = a.positions[b];
    const int slot = a.slots[b];
    if (pos < 0 || pos >= a.maxT || slot < 0 || slot >= a.nslots) {
        if (tid == 0) atomicOr(a.err, kErrPosition);
        return;
    }
    const int T = pos + 1, t_lo = split * tp, t_hi = min(T, t_lo + tp);
    if (t_lo >= T) return;  // split 0 always has positions (and appends the rows)
    const size_t cache_off = ((size_t)slot * a.L + a.l) * a.maxT * kn;
    const float* K = a.kc + cache_off;
    const int own = a.from_cache ? -1 : pos;  // the row this block takes from k_s
    // tile copies: thread (row r0 + i * rstep, column c) with c fixed per thread
    const int c4 = hd / 4, rstep = kQkThreads / c4, kr0 = tid / c4, kc = (tid - kr0 * c4) * 4;
    auto issue_k = [&](int t0, float* buf) {
        const int nt = min(kQkTile, t_hi - t0);
        if (kr0 < rstep)
            for (int r = kr0; r < nt; r += rstep)
                if (t0 + r != own) cp_async16(buf + r * KP + kc, K + (size_t)(t0 + r) * kn + g * hd + kc);
        cp_async_commit();
    };
    // scores (decode_kernel.c:1212-1218): chains (position, head) in pairs
    const float scale = sqrtf_fast((float)hd);
    float* out = scores + ((size_t)b * a.H + h0) * a.maxT;
    const int ntiles = (t_hi - t_lo + kQkTile - 1) / kQkTile;
    const int npairs = kQkTile * gsz / 2 + (kQkTile * gsz) % 2;
    // a ring of kQkRing tiles, kQkRing - 1 in flight: one commit group per tile (empty past the
    // end). The first ones go out before the norms: they depend only on the position.
    for (int jt = 0; jt < kQkRing - 1; jt++) {
        if (jt < ntiles) issue_k(t_lo + jt * kQkTile, tb0 + jt * kQkTile * KP);
        else cp_async_commit();
    }
    qk_prepare(a, g, b, pos, q_s, QS, k_s, v_s, cs_s, sn_s, sq, inv);
    if (!a.from_cache && split == 0) {        // KV append (decode_kernel.c:1200-1205)
        for (int i = tid; i < hd; i += blockDim.x) {
            a.kc[cache_off + (size_t)pos * kn + g * hd + i] = k_s[i];
            a.vc[cache_off + (size_t)pos * kn + g * hd + i] = v_s[i];
        }
    }
    for (int jt = 0; jt < ntiles; jt++) {
        const int t0 = t_lo + jt * kQkTile, nt = min(kQkTile, t_hi - t0);
        float* buf = tb0 + (jt % kQkRing) * kQkTile * KP;
        const int jn = jt + kQkRing - 1;  // refills the slot tile jt - 1 used
        if (jn < ntiles) issue_k(t_lo + jn * kQkTile, tb0 + (jn % kQkRing) * kQkTile * KP);
        else cp_async_commit();
        cp_async_wait<kQkRing - 1>();
        if (own >= t0 && own < t0 + nt)
            for (int i = tid; i < hd; i += blockDim.x) buf[(own - t0) * KP + i] = k_s[i];
        __syncthreads();
        for (int pi = tid; pi < npairs; pi += blockDim.x) {
            const int ca = 2 * pi, cb = min(2 * pi + 1, kQkTile * gsz - 1);
            const int ta = ca / gsz, ha = ca - ta * gsz, tb = cb / gsz, hb = cb - tb * gsz;
            if (ta >= nt) continue;
            const int tbc = tb < nt ? tb : ta;
            const float* qa = q_s + ha * QS;
            const float* qb = q_s + hb * QS;
            const float* ka = buf + ta * KP;
            const float* kb = buf + tbc * KP;
            float s0 = 0.0f, s1 = 0.0f;  // two chains, each a product then a sum per element
            if (ka == kb) {              // two heads of one position (even group sizes): one k row
#pragma unroll 4
                for (int i = 0; i < hd; i += 4) {
                    const float4 x = *reinterpret_cast<const float4*>(qa + i);
                    const float4 y = *reinterpret_cast<const float4*>(qb + i);
                    const float4 u = *reinterpret_cast<const float4*>(ka + i);
                    s0 = __fadd_rn(s0, __fmul_rn(x.x, u.x));
                    s1 = __fadd_rn(s1, __fmul_rn(y.x, u.x));
                    s0 = __fadd_rn(s0, __fmul_rn(x.y, u.y));
                    s1 = __fadd_rn(s1, __fmul_rn(y.y, u.y));
                    s0 = __fadd_rn(s0, __fmul_rn(x.z, u.z));
                    s1 = __fadd_rn(s1, __fmul_rn(y.z, u.z));
                    s0 = __fadd_rn(s0, __fmul_rn(x.w, u.w));
                    s1 = __fadd_rn(s1, __fmul_rn(y.w, u.w));
                }
            } else {
#pragma unroll 4
                for (int i = 0; i < hd; i += 4) {
                    const float4 x = *reinterpret_cast<const float4*>(qa + i);
                    const float4 y = *reinterpret_cast<const float4*>(qb + i);
                    const float4 u = *reinterpret_cast<const float4*>(ka + i);
                    const float4 w = *reinterpret_cast<const float4*>(kb + i);
                    s0 = __fadd_rn(s0, __fmul_rn(x.x, u.x));
                    s1 = __fadd_rn(s1, __fmul_rn(y.x, w.x));
                    s0 = __fadd_rn(s0, __fmul_rn(x.y, u.y));
                    s1 = __fadd_rn(s1, __fmul_rn(y.y, w.y));
                    s0 = __fadd_rn(s0, __fmul_rn(x.z, u.z));
                    s1 = __fadd_rn(s1, __fmul_rn(y.z, w.z));
                    s0 = __fadd_rn(s0, __fmul_rn(x.w, u.w));
                    s1 = __fadd_rn(s1, __fmul_rn(y.w, w.w));
                }
            }
            out[(size_t)ha * a.maxT + t0 + ta] = __fdiv_rn(s0, scale);
            if (tb < nt && cb != ca) out[(size_t)hb * a.maxT + t0 + tb] = __fdiv_rn(s1, scale);
        }
        __syncthreads();  // the slot is refilled in the next iteration
    }
}

template <int NI>
__global__ void __launch_bounds__(kPvThreads) k_attn_pv(attn_args a, const float* __restrict__ scores, int hpb,
                                                         int dw, int whole) {
    extern __shared__ __align__(16) float sm[];
    const int hb = blockIdx.x, b = blockIdx.y, z = blockIdx.z, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int hd = a.hd, qn = a.H * hd, kn = a.KH * hd, h0 = hb * hpb, g = h0 / (a.H / a.KH);
    const int maxT4 = (a.maxT + 3) / 4 * 4;
    float* p_s = sm;                 // [hpb][maxT4]
    float* vt0 = sm + hpb * maxT4;   // whole: all rows [maxT][dw]; else a ring of kPvRing tiles [kPvTile][dw]
    __shared__ float red[kPvThreads / 32];
    __shared__ float stat[kPvThreads / 32];
    griddep_wait();
    griddep_launch_dependents();
    const int pos = a.positions[b];
    const int slot = a.slots[b];
    if (pos < 0 || pos >= a.maxT || slot < 0 || slot >= a.nslots) return;  // k_attn_qk flagged it
    const int T = pos + 1, T4 = (T + 3) / 4 * 4;
    const float* V = a.vc + ((size_t)slot * a.L + a.l) * a.maxT * kn + g * hd + z * dw;
    const int c4 = dw / 4, rstep = kPvThreads / c4, vr0 = tid / c4, vc = (tid - vr0 * c4) * 4;
    auto issue_v = [&](int t0, float* buf) {
        const int nt = min(kPvTile, T - t0);
        if (vr0 < rstep)
            for (int r = vr0; r < nt; r += rstep) cp_async16(buf + r * dw + vc, V + (size_t)(t0 + r) * kn + vc);
        cp_async_commit();
    };
    // the values do not depend on the softmax: all rows (whole) or the ring's
    // first kPvRing - 1 tiles go out now
    const int ntiles = (T + kPvTile - 1) / kPvTile;
    if (whole) {
        if (vr0 < rstep)
            for (int r = vr0; r < T; r += rstep) cp_async16(vt0 + r * dw + vc, V + (size_t)r * kn + vc);
        cp_async_commit();
    } else {
        for (int j = 0; j < kPvRing - 1; j++) {
            if (j < ntiles) issue_v(j * kPvTile, vt0 + j * kPvTile * dw);
            else cp_async_commit();
        }
    }
    // softmax: head hh by the wph warps [hh * wph, (hh + 1) * wph) (hpb <= 8)
    const int wph = kPvThreads / 32 / hpb, hh = warp / wph, sub = (warp - hh * wph) * 32 + lane, nsub = wph * 32;
    float* p = p_s + hh * maxT4;
    const float* src = scores + ((size_t)b * a.H + h0 + hh) * a.maxT;
    float mx = -1e30f;
    for (int t = sub; t < T4; t += nsub) {
        const float v = t < T ? src[t] : 0.0f;  // pads are +0 for the sum
        p[t] = v;
        if (t < T && v > mx) mx = v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[hh * wph];
    for (int w = 1; w < wph; w++) mx = fmaxf(mx, red[hh * wph + w]);
    for (int t = sub; t < T; t += nsub) p[t] = expf_fast(__fsub_rn(p[t], mx));
    __syncthreads();
    if (sub == 0) stat[hh] = chain_sum(p, T4);  // sequential over t (decode_kernel.c:1220)
    __syncthreads();
    const float sum = stat[hh];
    for (int t = sub; t < T; t += nsub) p[t] = __fdiv_rn(p[t], sum);
    // att[i] = 0 + p_0 v_0[i] + p_1 v_1[i] + ... (decode_kernel.c:1222-1229): items (head, four
    // dimensions), NI per thread, their chains interleaved
    const int nq = dw / 4, items = hpb * nq;  // items: (head, four consecutive dimensions)
    int ih[NI], ii[NI];
    float4 o[NI];  // the item's four chains, scalar products and sums (a packed fp32-pair
                   // multiply and add measured different bits from the reference here)
#pragma unroll
    for (int k = 0; k < NI; k++) {
        const int it = min(tid + k * kPvThreads, items - 1);
        ih[k] = it / nq;
        ii[k] = it - ih[k] * nq;
        o[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    const bool live = tid < items;  // the last item's thread set is complete (items <= NI * threads)
    auto rows = [&](const float* vbuf, int t0, int nt) {
#pragma unroll 4
        for (int r = 0; r < nt; r++) {
#pragma unroll
            for (int k = 0; k < NI; k++) {
                const float pp = p_s[ih[k] * maxT4 + t0 + r];
                const float4 v = *reinterpret_cast<const float4*>(vbuf + r * dw + 4 * ii[k]);
                o[k].x = __fadd_rn(o[k].x, __fmul_rn(pp, v.x));
                o[k].y = __fadd_rn(o[k].y, __fmul_rn(pp, v.y));
                o[k].z = __fadd_rn(o[k].z, __fmul_rn(pp, v.z));
                o[k].w = __fadd_rn(o[k].w, __fmul_rn(pp, v.w));
            }
        }
    };
    if (whole) {  // one wait, then the chains over every row without a barrier
        cp_async_wait<0>();
        __syncthreads();
        if (live) rows(vt0, 0, T);
    }
    for (int j = 0; j < (whole ? 0 : ntiles); j++) {
        const int t0 = j * kPvTile, nt = min(kPvTile, T - t0);
        float* buf = vt0 + (j % kPvRing) * kPvTile * dw;
        const int jn = j + kPvRing - 1;  // refills the slot tile j - 1 used
        if (jn < ntiles) issue_v(jn * kPvTile, vt0 + (jn % kPvRing) * kPvTile * dw);
        else cp_async_commit();
        cp_async_wait<kPvRing - 1>();
        __syncthreads();
        if (live) rows(buf, t0, nt);
        __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < NI; k++)
        if (tid + k * kPvThreads < items) {
            const int col = (h0 + ih[k]) * hd + z * dw + 4 * ii[k];
            *reinterpret_cast<float4*>(a.att + (size_t)b * qn + col) = o[k];
            if (a.attT) {
                a.attT[(size_t)col * a.Bp + b] = o[k].x;
                a.attT[(size_t)(col + 1) * a.Bp + b] = o[k].y;
                a.attT[(size_t)(col + 2) * a.Bp + b] = o[k].z;
                a.attT[(size_t)(col + 3) * a.Bp + b] = o[k].w;
            }
        }
}

// ---------------------------------------------------------------------------
// Register-tiled attention for KV groups of an even number of heads and head
// dimensions 64 or 128 (the decode step at batches of 16 and more), in three
// launches: the same chains in the same order as k_attn_qk / k_attn_pv, each
// thread running several of them (8 scores, 4 values), so one shared-memory
// load feeds several chains and the loops unroll at compile time; two
// chains' sums share one packed add (add_prod2).
//
// k_qk_prep, block (KV group g, row b): the prologue once per (group, row):
// QK-norm and RoPE of the group's q heads, written to qr [B][H][hd], and of
// the k row, which goes into the cache at positions[b] with the v row
// (decode_kernel.c:1162-1205). The score kernel then reads q from qr and
// every K row from the cache.
//
// k_attn_qk_t<HD, PPT>, block (KV group g, sequence b, split p): the block's
// positions are split p of ceil(T / PT) even splits of [0, T) (PT = 32 PPT);
// their K rows of the group arrive whole in shared memory, one bulk copy per
// row on one mbarrier. Thread (head pair hp, position lane pq) owns heads 2hp,
// 2hp + 1 against positions pq, pq + 32, ... (2 x PPT chains): a 4-column
// step loads 2 q and PPT k float4s for 8 PPT products and sums.
//
// k_attn_pv_t<HD>, block (KV group g, sequence b, dimension slice z of dw):
// the softmax of the group's heads from their staged score rows (per head the
// max, p_t = expf_fast(s_t - max), their sum in t order by one thread,
// p_t /= sum; decode_kernel.c:1219-1221), then thread (head h, dimension
// quad dq) runs the 4 chains att[i] = 0 + p_0 v_0[i] + ... in t order of
// dimensions z dw + 4 dq .. + 3. V rows [t][dw] stream through a ring of
// kPvRingT tiles of kPvRowsT rows; per 4 rows a thread loads a p float4 (p
// rows padded to ps = 4 mod 32 floats, so the heads' rows sit in distinct
// banks) and 4 v float4s for 16 products and sums. The block is rounded up
// to whole warps; the extra threads only copy.

// Chain steps o += a * b for two chains at once: each product by the scalar
// multiply, the two sums by one packed add (each lane rounds as the scalar add
// does). A packed multiply feeding a packed add directly is not used: the
// assembler fuses that pair into a packed FMA (one rounding instead of two).
__device__ __forceinline__ float2 add_prod2(float2 o, float a0, float b0, float a1, float b1) {
    return __fadd2_rn(o, make_float2(__fmul_rn(a0, b0), __fmul_rn(a1, b1)));
}

__global__ void __launch_bounds__(kAttnThreads) k_qk_prep(attn_args a) {
    extern __shared__ __align__(16) float sm[];
    const int g = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int hd = a.hd, kn = a.KH * hd, gsz = a.H / a.KH, QS = hd + 4;
    float* q_s = sm;              // [gsz][QS]
    float* k_s = q_s + gsz * QS;  // [hd]
    float* v_s = k_s + hd;        // [hd]
    float* cs_s = v_s + hd;       // [hd]
    float* sn_s = cs_s + hd;      // [hd]
    float* inv = sn_s + hd;       // [gsz + 1], padded to 4
    float* sq = inv + (gsz + 4) / 4 * 4;
    griddep_wait();
    griddep_launch_dependents();
    const int pos = a.positions[b];
    const int slot = a.slots[b];
    if (pos < 0 || pos >= a.maxT || slot < 0 || slot >= a.nslots) {
        if (tid == 0) atomicOr(a.err, kErrPosition);
        return;
    }
    qk_prepare(a, g, b, pos, q_s, QS, k_s, v_s, cs_s, sn_s, sq, inv);
    float* dst = a.qr + ((size_t)b * a.H + g * gsz) * hd;
    for (int hh = 0; hh < gsz; hh++)
        for (int c = tid; c < hd / 4; c += blockDim.x)
            reinterpret_cast<float4*>(dst + hh * hd)[c] = reinterpret_cast<const float4*>(q_s + hh * QS)[c];
    const size_t off = (((size_t)slot * a.L + a.l) * a.maxT + pos) * kn + g * hd;
    for (int i = tid; i < hd; i += blockDim.x) {
        a.kc[off + i] = k_s[i];
        a.vc[off + i] = v_s[i];
    }
}

size_t qk_prep_smem(int qk_type, int H, int KH, int hd) {
    const int gsz = H / KH;
    return ((size_t)gsz * (hd + 4) + 4 * hd + (gsz + 4) / 4 * 4 +
            (qk_type == 2 ? (H * hd + 3) / 4 * 4 + (KH * hd + 3) / 4 * 4 : 0)) * sizeof(float);
}

// Shared memory of k_attn_qk_t (floats): the K rows [PT][HD + 4], then q
// [gsz][HD + 4] (rows padded by 16 bytes: the eight rows a warp reads at once
// fall in distinct banks).
template <int HD, int PPT>
struct qk_t_layout {
    static constexpr int PT = 32 * PPT, KS = HD + 4;
    static size_t bytes(int gsz) { return (size_t)(PT + gsz) * KS * sizeof(float); }
};

template <int HD, int PPT>
__global__ void __launch_bounds__(256) k_attn_qk_t(attn_args a, float* __restrict__ scores) {
    using LY = qk_t_layout<HD, PPT>;
    constexpr int PT = LY::PT, KS = LY::KS;
    extern __shared__ __align__(16) float sm[];
    __shared__ __align__(8) uint64_t bar;
    const int g = blockIdx.x, b = blockIdx.y, split = blockIdx.z, tid = threadIdx.x;
    const int gsz = a.H / a.KH, nhp = gsz / 2, h0 = g * gsz, kn = a.KH * HD;
    const int hp = tid % nhp, pq = tid / nhp;
    float* kt = sm;              // [PT][KS]
    float* q_s = sm + PT * KS;   // [gsz][KS]
    // Positions and slots are inputs of the step, written before its first
    // kernel: they, and the K rows of earlier steps, are read before the
    // dependent-grid wait, so the rows stream in while k_qk_prep runs. The
    // row it appends (and every row, for a prefill chunk) and q come after.
    const int pos = a.positions[b];
    const int slot = a.slots[b];
    if (pos < 0 || pos >= a.maxT || slot < 0 || slot >= a.nslots) return;  // k_qk_prep flags it
    const int T = pos + 1, ns = (T + PT - 1) / PT, tpb = (T + ns - 1) / ns, t_lo = split * tpb;
    if (split >= ns || t_lo >= T) return;
    const int n = min(T - t_lo, tpb);
    const int early = a.from_cache ? 0 : split == ns - 1 ? n - 1 : n;  // rows loaded before the wait
    const float* K = a.kc + ((size_t)slot * a.L + a.l) * a.maxT * kn + (size_t)t_lo * kn + g * HD;
    if (tid == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
        mbar_expect_tx(&bar, (uint32_t)((n + gsz) * HD * sizeof(float)));
    }
    __syncthreads();
    for (int r = tid; r < early; r += blockDim.x) bulk_g2s(kt + r * KS, K + (size_t)r * kn, HD * sizeof(float), &bar);
    griddep_wait();
    griddep_launch_dependents();
    for (int r = early + tid; r < n; r += blockDim.x)
        bulk_g2s(kt + r * KS, K + (size_t)r * kn, HD * sizeof(float), &bar);
    const float* qsrc = a.qr + ((size_t)b * a.H + h0) * HD;
    for (int r = tid; r < gsz; r += blockDim.x) bulk_g2s(q_s + r * KS, qsrc + r * HD, HD * sizeof(float), &bar);
    if (!mbar_wait_bounded(&bar, 0, a.err)) return;
    // scores (decode_kernel.c:1212-1218): acc[i] = the chains of heads 2hp, 2hp + 1 at position pq + 32 i
    float2 acc[PPT];
#pragma unroll
    for (int i = 0; i < PPT; i++) acc[i] = make_float2(0.0f, 0.0f);
    const float* qa = q_s + 2 * hp * KS;
    const float* qb = qa + KS;
    const float* kb = kt + pq * KS;
#pragma unroll 8
    for (int c = 0; c < HD / 4; c++) {
        const float4 x = *reinterpret_cast<const float4*>(qa + 4 * c);
        const float4 y = *reinterpret_cast<const float4*>(qb + 4 * c);
        float4 u[PPT];
#pragma unroll
        for (int i = 0; i < PPT; i++) u[i] = *reinterpret_cast<const float4*>(kb + 32 * i * KS + 4 * c);
#pragma unroll
        for (int i = 0; i < PPT; i++) acc[i] = add_prod2(acc[i], x.x, u[i].x, y.x, u[i].x);
#pragma unroll
        for (int i = 0; i < PPT; i++) acc[i] = add_prod2(acc[i], x.y, u[i].y, y.y, u[i].y);
#pragma unroll
        for (int i = 0; i < PPT; i++) acc[i] = add_prod2(acc[i], x.z, u[i].z, y.z, u[i].z);
#pragma unroll
        for (int i = 0; i < PPT; i++) acc[i] = add_prod2(acc[i], x.w, u[i].w, y.w, u[i].w);
    }
    const float scale = sqrtf_fast((float)HD);
    float* out = scores + ((size_t)b * a.H + h0 + 2 * hp) * a.maxT + t_lo;
#pragma unroll
    for (int i = 0; i < PPT; i++) {
        const int t = pq + 32 * i;
        if (t < n) {
            out[t] = __fdiv_rn(acc[i].x, scale);
            out[a.maxT + t] = __fdiv_rn(acc[i].y, scale);
        }
    }
}

constexpr int kPvRowsT = 32;
constexpr int kPvRingT = 4;

__device__ __forceinline__ void pv_step(float2& oxy, float2& ozw, float p, const float4& v) {
    oxy = add_prod2(oxy, p, v.x, p, v.y);
    ozw = add_prod2(ozw, p, v.z, p, v.w);
}

// four rows r .. r + 3 of a V tile into the thread's four chains
__device__ __forceinline__ void pv_rows4(float2& oxy, float2& ozw, const float* p, const float* vb, int dw) {
    const float4 pp = *reinterpret_cast<const float4*>(p);
    pv_step(oxy, ozw, pp.x, *reinterpret_cast<const float4*>(vb));
    pv_step(oxy, ozw, pp.y, *reinterpret_cast<const float4*>(vb + dw));
    pv_step(oxy, ozw, pp.z, *reinterpret_cast<const float4*>(vb + 2 * dw));
    pv_step(oxy, ozw, pp.w, *reinterpret_cast<const float4*>(vb + 3 * dw));
}

// Shared memory of k_attn_pv_t (floats): scores, then probabilities, [gsz][ps]
// (ps = 4 mod 32: the heads' rows in distinct banks), then the V ring.
struct pv_t_layout {
    int ps, vt, total;
    __host__ __device__ pv_t_layout(int gsz, int maxT, int dw) {
        ps = (maxT + 31) / 32 * 32 + 4;
        vt = gsz * ps;
        total = vt + kPvRingT * kPvRowsT * dw;
    }
};

template <int HD>
__global__ void __launch_bounds__(256) k_attn_pv_t(attn_args a, const float* __restrict__ scores, int dw) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float stat[16];
    const int g = blockIdx.x, b = blockIdx.y, z = blockIdx.z, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const int gsz = a.H / a.KH, h0 = g * gsz, qn = a.H * HD, kn = a.KH * HD;
    const int hh0 = tid % gsz, dq = tid / gsz, nq = dw / 4;  // the thread's head and dimension quad
    const bool live = dq < nq;
    const pv_t_layout lay(gsz, a.maxT, dw);
    const int ps = lay.ps;
    float* s_s = sm;           // [gsz][ps]
    float* vt = sm + lay.vt;   // [kPvRingT][kPvRowsT][dw]
    // Positions and slots are inputs of the step and the V rows are in the
    // cache once k_attn_qk_t runs (k_qk_prep appended this step's rows and
    // k_attn_qk_t waited for it before releasing this kernel): the ring's
    // first tiles go out before the dependent-grid wait, the scores after it.
    const int pos = a.positions[b];
    const int slot = a.slots[b];
    if (pos < 0 || pos >= a.maxT || slot < 0 || slot >= a.nslots) return;  // k_qk_prep flags it
    const int T = pos + 1, T4 = (T + 3) / 4 * 4;
    const float* V = a.vc + ((size_t)slot * a.L + a.l) * a.maxT * kn + g * HD + z * dw;
    const int ntiles = (T + kPvRowsT - 1) / kPvRowsT;
    // tile copies: thread (rows vr0, vr0 + rstep, ..., 16-byte column vc), fixed per thread
    const int rstep = blockDim.x / nq, vr0 = tid / nq, vc = 4 * (tid - vr0 * nq);
    auto issue_v = [&](int j) {  // tile j into slot j % kPvRingT
        const int t0 = j * kPvRowsT, nt = min(kPvRowsT, T - t0);
        float* buf = vt + (j % kPvRingT) * kPvRowsT * dw + vc;
        const float* src = V + (size_t)t0 * kn + vc;
        for (int r = vr0; r < nt; r += rstep) cp_async16(buf + r * dw, src + (size_t)r * kn);
    };
    for (int j = 0; j < kPvRingT - 1; j++) {
        if (j < ntiles) issue_v(j);
        cp_async_commit();
    }
    griddep_wait();
    griddep_launch_dependents();
    // the group's score rows (16-byte pieces when the rows are 16-byte aligned)
    const float* src = scores + ((size_t)b * a.H + h0) * a.maxT;
    if ((a.maxT & 3) == 0) {
        for (int hh = 0; hh < gsz; hh++)
            for (int c = tid; c < T4 / 4; c += blockDim.x) cp_async16(s_s + hh * ps + 4 * c, src + (size_t)hh * a.maxT + 4 * c);
    } else {
        for (int hh = 0; hh < gsz; hh++)
            for (int t = tid; t < T; t += blockDim.x) cp_async4(s_s + hh * ps + t, src + (size_t)hh * a.maxT + t);
    }
    cp_async_commit();
    // softmax (decode_kernel.c:1219-1221): per head the max, p_t = expf_fast(s_t - max), their sum
    // in t order by one thread, p_t /= sum
    cp_async_wait<0>();  // the scores (the newest group) have landed, and the ring's first tiles
    __syncthreads();
    for (int hh = warp; hh < gsz; hh += nwarps) {
        float* p = s_s + hh * ps;
        float mx = -1e30f;
        for (int t = lane; t < T; t += 32) {
            const float v = p[t];
            if (v > mx) mx = v;
        }
        if (lane < T4 - T) p[T + lane] = 0.0f;  // pads are +0 for the sum
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        for (int t = lane; t < T; t += 32) p[t] = expf_fast(__fsub_rn(p[t], mx));
    }
    __syncthreads();
    if (tid < gsz) stat[tid] = chain_sum(s_s + tid * ps, T4);  // sequential over t (decode_kernel.c:1220)
    __syncthreads();
    for (int hh = 0; hh < gsz; hh++) {
        const float sum = stat[hh];
        for (int t = tid; t < T; t += blockDim.x) s_s[hh * ps + t] = __fdiv_rn(s_s[hh * ps + t], sum);
    }
    // att[i] = 0 + p_0 v_0[i] + p_1 v_1[i] + ... (decode_kernel.c:1222-1229)
    float2 oxy = make_float2(0.0f, 0.0f), ozw = oxy;
    const float* pa = s_s + hh0 * ps;
    for (int j = 0; j < ntiles; j++) {
        const int t0 = j * kPvRowsT, nt = min(kPvRowsT, T - t0);
        const int jn = j + kPvRingT - 1;  // refills the slot tile j - 1 used
        if (jn < ntiles) issue_v(jn);
        cp_async_commit();
        cp_async_wait<kPvRingT - 1>();
        __syncthreads();
        const float* vb = vt + (j % kPvRingT) * kPvRowsT * dw + 4 * dq;
        if (live) {
            if (nt == kPvRowsT) {
#pragma unroll
                for (int r = 0; r < kPvRowsT; r += 4) pv_rows4(oxy, ozw, pa + t0 + r, vb + r * dw, dw);
            } else {
                int r = 0;
                for (; r + 4 <= nt; r += 4) pv_rows4(oxy, ozw, pa + t0 + r, vb + r * dw, dw);
                for (; r < nt; r++) pv_step(oxy, ozw, pa[t0 + r], *reinterpret_cast<const float4*>(vb + r * dw));
            }
        }
        __syncthreads();
    }
    if (!live) return;
    const int col = (h0 + hh0) * HD + z * dw + 4 * dq;
    *reinterpret_cast<float4*>(a.att + (size_t)b * qn + col) = make_float4(oxy.x, oxy.y, ozw.x, ozw.y);
    if (a.attT) {
        a.attT[(size_t)col * a.Bp + b] = oxy.x;
        a.attT[(size_t)(col + 1) * a.Bp + b] = oxy.y;
        a.attT[(size_t)(col + 2) * a.Bp + b] = ozw.x;
        a.attT[(size_t)(col + 3) * a.Bp + b] = ozw.y;
    }
}

// K/V append for a batch of positions of one or more sequences (batched
// prefill, where one launch's positions of a sequence attend to each other):
// per (KV head g, row b) the K row gets its QK-norm and RoPE exactly as in
// k_attn_qk, and both rows go into the cache at positions[b]. k_attn_qk then runs
// with from_cache = 1.
__global__ void __launch_bounds__(kAttnThreads) k_kv_append(attn_args a) {
    extern __shared__ __align__(16) float sm[];
    const int g = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int hd = a.hd, qn = a.H * hd, kn = a.KH * hd;
    float* k_s = sm;
    float* sq = sm + 128;  // [a.sqn]
    __shared__ float inv_k;
    griddep_wait();
    griddep_launch_dependents();
    const int pos = a.positions[b];
    const int slot = a.slots[b];
    if (pos < 0 || pos >= a.maxT || slot < 0 || slot >= a.nslots) {
        if (tid == 0) atomicOr(a.err, kErrPosition);
        return;
    }
    const float* row = a.qkv + (size_t)b * (qn + 2 * kn);
    if (tid < hd) k_s[tid] = row[qn + g * hd + tid];
    if (a.qk_type == 2) {
        squares(row + qn, kn, sq);
        __syncthreads();
        if (tid == 0) inv_k = rms_inv(chain_sum(sq, kn), kn, a.eps);
        __syncthreads();
        if (tid < hd) k_s[tid] = __fmul_rn(__fmul_rn(k_s[tid], inv_k), bf16_to_f32(a.knw[g * hd + tid]));
    } else if (a.qk_type == 1) {
        __syncthreads();
        if (tid < hd) sq[tid] = __fmul_rn(k_s[tid], k_s[tid]);
        __syncthreads();
        if (tid == 0) inv_k = rms_inv(chain_sum(sq, hd), hd, a.eps);
        __syncthreads();
        if (tid < hd) k_s[tid] = __fmul_rn(__fmul_rn(k_s[tid], inv_k), bf16_to_f32(a.knw[tid]));
    }
    __syncthreads();
    const int half = hd / 2;
    float ka = 0.f, kb = 0.f;
    if (tid < half) {
        const float cs = a.cosb[(size_t)pos * hd + tid], sn = a.sinb[(size_t)pos * hd + tid];
        const float y0 = k_s[tid], y1 = k_s[tid + half];
        ka = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
        kb = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
    }
    __syncthreads();
    if (tid < half) {
        k_s[tid] = ka;
        k_s[tid + half] = kb;
    }
    __syncthreads();
    const size_t off = (((size_t)slot * a.L + a.l) * a.maxT + pos) * kn + g * hd;
    if (tid < hd) {
        a.kc[off + tid] = k_s[tid];
        a.vc[off + tid] = row[qn + kn + g * hd + tid];
    }
}

// squares buffer size (floats, a multiple of 4) for the QK-norm of a type
int attn_sqn(int qk_type, int H, int KH, int hd) {
    const int n = qk_type == 2 ? std::max(H * hd, KH * hd) : hd;
    return (n + 3) / 4 * 4;
}


// ---------------------------------------------------------------------------
// argmax over each logits row, lowest index on ties (the first maximum of an
// ascending scan with strict '>', as the greedy pick over the reference's
// logits). Two launches: blocks (part, b) reduce slices of the row to a
// (value, index) pair (four float4 loads in flight per thread), then one
// warp per row reduces the pairs.
constexpr int kArgParts = 32;

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(256) k_argmax_part(const float* __restrict__ logits, int V, float* pv, int* pi) {
    __shared__ float sv[8];
    __shared__ int si[8];
    griddep_wait();
    griddep_launch_dependents();
    const int part = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int per = (V + kArgParts - 1) / kArgParts;
    const int lo = part * per, hi = min(V, lo + per);
    const float* r = logits + (size_t)b * V;
    float bv = -__int_as_float(0x7f800000);
    int bi = INT_MAX;
    for (int i0 = lo + tid; i0 < hi; i0 += 4 * blockDim.x) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = i0 + j * blockDim.x;
            v[j] = i < hi ? r[i] : bv;
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = i0 + j * blockDim.x;
            if (i < hi) better(bv, bi, v[j], i);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, ov, oi);
    }
    if ((tid & 31) == 0) {
        sv[tid >> 5] = bv;
        si[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) better(bv, bi, sv[w], si[w]);
        pv[b * kArgParts + part] = bv;
        pi[b * kArgParts + part] = bi;
    }
}

__global__ void k_argmax_fin(const float* __restrict__ pv, const int* __restrict__ pi, int* __restrict__ tok) {
    griddep_wait();
    griddep_launch_dependents();
    const int b = blockIdx.x, lane = threadIdx.x;
    float bv = pv[b * kArgParts + lane];
    int bi = pi[b * kArgParts + lane];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, ov, oi);
    }
    if (lane == 0) tok[b] = bi == INT_MAX ? 0 : bi;
}

// embed_lookup (decode_kernel.c:1597-1600): x[b] = bf16 embed[tok[b]] as fp32.
__global__ void k_embed(const uint16_t* __restrict__ embed, const int* __restrict__ tok, int V, int d,
                        float* __restrict__ x, int* err) {
    griddep_wait();
    griddep_launch_dependents();
    const int b = blockIdx.y;
    const int t = tok[b];
    if (t < 0 || t >= V) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, kErrBadExpert);
        return;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x)
        x[(size_t)b * d + i] = bf16_to_f32(embed[(size_t)t * d + i]);
}

}  // namespace jl

// ---------------------------------------------------------------------------
// The handle.

struct jl_dec {
    int device;
    int L, d, H, KH, hd, E, k, m, V, maxT, qk_type, bias;
    float eps;
    int qn, kn, nqkv;
    int max_batch, slots;
    jl_moe* moe;
    uint16_t* embed;   // [V, d]
    uint16_t* norm1;   // [L, d]
    uint16_t* norm2;   // [L, d]
    uint16_t* fnorm;   // [d]
    uint16_t* qnw;     // [L, hd] (per head) or [L, qn] (whole)
    uint16_t* knw;     // [L, hd] or [L, kn]
    uint16_t* wqkv;    // per layer: [nqkv, d] chunked lane-major
    uint16_t* wo;      // per layer: [d, qn] chunked lane-major
    float* bqkv;       // [L, nqkv] or null
    float* lm;         // [V, d] fp32 chunked lane-major
    float* cosb;       // [maxT, hd]
    float* sinb;
    float* kc;         // [slots][L][maxT][kn]
    float* vc;
    // workspace
    float* h;          // [max_batch, d]
    float* t;          // [max_batch, d]
    float* h2;         // [max_batch, d]
    float* qkv;        // [max_batch, nqkv]
    float* att;        // [max_batch, qn]
    float* tT;         // [d, Bp] column-major copies of the norm output and of att (large batches)
    float* attT;       // [qn, Bp]
    int Bp;            // max_batch rounded up to 8
    float* scores;     // [max_batch, H, maxT] attention scores
    float* qr;         // [max_batch, qn] prepared q of the register-tiled attention
    float* logits;     // [max_batch, V]
    int* tok;          // [max_batch]
    float* arg_v;      // [max_batch][kArgParts] argmax partials
    int* arg_i;
    int* pre_pos;      // [max_batch] positions of a prefill chunk
    int* pre_slot;     // [max_batch] its slot, repeated
    int* err;          // [1]
    void* stage;       // device staging for uploads
    size_t stage_bytes;
};

namespace {

int dec_attrs() {
    return jl_device_once(kOnceDecode, [] {
        using namespace jl;
        const int big = 200 * 1024;
        JL_CUDA(cudaFuncSetAttribute(k_mv<uint16_t, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_mv<uint16_t, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_mv<uint16_t, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_mv<uint16_t, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_mv<float, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_mv<float, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_mv<float, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_mv<float, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_attn_qk, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_attn_pv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_attn_pv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_attn_pv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_rms, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_attn_qk_t<64, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_attn_qk_t<128, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_attn_pv_t<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_attn_pv_t<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        JL_CUDA(cudaFuncSetAttribute(k_qk_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
        return JL_OK;
    });
}

// The register-tiled attention of one layer (head dims 64 and 128, even
// group sizes up to 16): k_qk_prep (which also appends the K/V rows), then
// k_attn_qk_t with 4 positions per thread, then k_attn_pv_t with one head per
// thread (4 chains) and the head dimension cut into slices of at least 32
// until there is about one value block per SM and at most 256 threads a
// block. Timed at B = 16 and 64 on the Qwen3 shape, 2 and 4 positions per
// score thread and 1 and 2 heads per value thread all took within 3 % of one
// another (latency-bound, about 50 % issue efficiency); the chosen pair was
// the fastest at B = 16.
bool attn_tiled_ok(int hd, int gsz) { return (hd == 64 || hd == 128) && gsz % 2 == 0 && gsz <= 16; }

template <int HD, int PPT>
int launch_qk_t(const jl::attn_args& aa, float* scores, int B, cudaStream_t s) {
    using namespace jl;
    using LY = qk_t_layout<HD, PPT>;
    const int gsz = aa.H / aa.KH;
    const size_t smem = LY::bytes(gsz);
    if (smem > 200 * 1024) return JL_ERR_INVALID;
    return launch(k_attn_qk_t<HD, PPT>, dim3(aa.KH, B, (aa.maxT + LY::PT - 1) / LY::PT), dim3(16 * gsz), smem, s, aa,
                  scores);
}

template <int HD>
int launch_attn_t(const jl::attn_args& aa, float* scores, int B, int sms, cudaStream_t s) {
    using namespace jl;
    const int gsz = aa.H / aa.KH;
    int rc = launch(k_qk_prep, dim3(aa.KH, B), dim3(kAttnThreads), qk_prep_smem(aa.qk_type, aa.H, aa.KH, HD), s, aa);
    if (!rc) rc = launch_qk_t<HD, 4>(aa, scores, B, s);
    if (rc) return rc;
    int ds = 1;
    while (ds < 4 && HD / (2 * ds) >= 32 && (aa.KH * B * ds < sms || gsz * (HD / ds / 4) > 256)) ds *= 2;
    const int dw = HD / ds;
    const int threads = (gsz * (dw / 4) + 31) / 32 * 32;
    if (threads > 256) return JL_ERR_INVALID;
    const size_t smem = (size_t)pv_t_layout(gsz, aa.maxT, dw).total * sizeof(float);
    if (smem > 200 * 1024) return JL_ERR_INVALID;
    return launch(k_attn_pv_t<HD>, dim3(aa.KH, B, ds), dim3(threads), smem, s, aa, (const float*)scores, dw);
}

// Row tiles per block: one for a single token group (the most blocks), more
// when the token rows are staged per block for several groups.
// x: [B][K] row-major; xT: the same as a column-major [K][Bp] copy (the
// register-tiled kernel at B >= kMmMinB reads that one).
template <typename WT>
int launch_mv(const WT* W, const float* x, const float* xT, int Bp, int N, int K, int B, const float* bias,
              float* out, int sm_count, cudaStream_t s) {
    using namespace jl;
    const bool big = (size_t)N * K * sizeof(WT) > ((size_t)64 << 20);  // beyond the L2 prefetch below
    if (jl_mm_ok(N, K, B, big ? kMmMinB : 16)) {
        if (!xT) return JL_ERR_INVALID;
        return jl_launch_mm<WT>(W, xT, Bp, N, K, B, bias, out, sm_count, s);
    }
    const int nt = B >= 8 ? 8 : B >= 4 ? 4 : B >= 2 ? 2 : 1;
    const size_t smem = (size_t)nt * 8 * mv_xstride(K) * sizeof(float);
    if (smem > 200 * 1024) return JL_ERR_INVALID;
    const int groups = (B + nt - 1) / nt, tiles = (N + kMvRows - 1) / kMvRows;
    const int RT = groups == 1 ? 1 : 4;
    const dim3 grid(groups, (tiles + RT - 1) / RT), block(kMvRows * 8);
    // matrices that fit comfortably in L2 are prefetched there before the
    // dependent-grid wait (the previous kernel is latency-bound at small B)
    const int pf = (size_t)N * K * sizeof(WT) <= ((size_t)64 << 20);
    switch (nt) {
        case 8: return launch(k_mv<WT, 8>, grid, block, smem, s, W, x, N, K, B, bias, out, RT, pf);
        case 4: return launch(k_mv<WT, 4>, grid, block, smem, s, W, x, N, K, B, bias, out, RT, pf);
        case 2: return launch(k_mv<WT, 2>, grid, block, smem, s, W, x, N, K, B, bias, out, RT, pf);
        default: return launch(k_mv<WT, 1>, grid, block, smem, s, W, x, N, K, B, bias, out, RT, pf);
    }
}

template <typename WT>
int repack_mv(const WT* src, WT* dst, int N, int K, cudaStream_t s) {
    const size_t total = (size_t)N * K;
    const int tpb = 256;
    const unsigned blocks = (unsigned)std::min<size_t>((total + tpb - 1) / tpb, 65535u * 16);
    jl::k_repack_mv<WT><<<blocks, tpb, 0, s>>>(src, dst, N, K);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? JL_OK : jl_note_cuda(e);
}

int check_dec_cfg(const KernelCfg* c) {
    if (!c || c->L < 1 || c->d < 64 || c->n_heads < 1 || c->n_kv < 1 || c->hd < 2 || c->V < 1 || c->maxT < 1)
        return JL_ERR_INVALID;
    if (c->n_heads % c->n_kv || c->hd > 128 || c->hd % 4) return JL_ERR_INVALID;
    if (c->d % 64 || (c->n_heads * c->hd) % 64 || (c->n_kv * c->hd) % 8) return JL_ERR_INVALID;
    if (c->qk_norm_type < 0 || c->qk_norm_type > 2) return JL_ERR_INVALID;
    return JL_OK;
}

// Copy `bytes` from src (host or device) into dst (device).
int put(void* dst, const void* src, size_t bytes, int on_dev, cudaStream_t s) {
    if (!src) return JL_ERR_INVALID;
    JL_CUDA(cudaMemcpyAsync(dst, src, bytes, on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
    return JL_OK;
}

}  // namespace

extern "C" int jl_dec_destroy(jl_dec* h) {
    if (!h) return JL_OK;
    if (h->moe) jl_moe_destroy(h->moe);
    void* ptrs[] = {h->embed, h->norm1, h->norm2, h->fnorm, h->qnw, h->knw, h->wqkv, h->wo, h->bqkv, h->lm,
                    h->cosb, h->sinb, h->kc, h->vc, h->h, h->t, h->h2, h->qkv, h->att, h->tT, h->attT, h->scores, h->qr,
                    h->logits, h->tok, h->arg_v, h->arg_i, h->pre_pos, h->pre_slot, h->err, h->stage};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    delete h;
    return JL_OK;
}

extern "C" int jl_dec_create(const KernelCfg* c, const KernelW* W, int max_batch, int slots, int src_on_device,
                             jl_dec** out) {
    using namespace jl;
    if (!out || !W || max_batch < 1 || slots < max_batch) return JL_ERR_INVALID;
    *out = nullptr;
    int rc = check_dec_cfg(c);
    if (rc) return rc;
    if (c->qk_norm_type && (!W->qn || !W->kn)) return JL_ERR_INVALID;
    if (c->bias_qkv && (!W->bq || !W->bk || !W->bv)) return JL_ERR_INVALID;
    if (!W->embed || !W->lm_head || !W->final_norm || !W->norm1 || !W->norm2 || !W->wq || !W->wk || !W->wv ||
        !W->wo || !W->gate_w || !W->cos || !W->sin)
        return JL_ERR_INVALID;
    rc = dec_attrs();
    if (rc) return rc;
    jl_dec* h = new (std::nothrow) jl_dec();
    if (!h) return JL_ERR_OOM;
    memset(h, 0, sizeof(*h));
    cudaGetDevice(&h->device);
    h->L = c->L, h->d = c->d, h->H = c->n_heads, h->KH = c->n_kv, h->hd = c->hd, h->E = c->E, h->k = c->topk;
    h->m = c->intermediate, h->V = c->V, h->maxT = c->maxT, h->qk_type = c->qk_norm_type, h->bias = c->bias_qkv;
    h->eps = c->eps;
    h->qn = h->H * h->hd, h->kn = h->KH * h->hd, h->nqkv = h->qn + 2 * h->kn;
    h->max_batch = max_batch, h->slots = slots;
    h->Bp = (max_batch + 7) / 8 * 8;
    rc = jl_moe_create(c, max_batch, &h->moe);
    if (rc) {
        delete h;
        return rc;
    }
    const size_t L = h->L, d = h->d, V = h->V;
    const size_t qnw_n = h->qk_type == 2 ? (size_t)h->qn : h->hd, knw_n = h->qk_type == 2 ? (size_t)h->kn : h->hd;
    const size_t kvb = (size_t)slots * L * h->maxT * h->kn * sizeof(float);
    h->stage_bytes = std::max({V * d * sizeof(float), (size_t)h->nqkv * d * 2, d * (size_t)h->qn * 2});
    struct alloc { void** p; size_t n; } al[] = {
        {(void**)&h->embed, V * d * 2},
        {(void**)&h->norm1, L * d * 2},
        {(void**)&h->norm2, L * d * 2},
        {(void**)&h->fnorm, d * 2},
        {(void**)&h->qnw, h->qk_type ? L * qnw_n * 2 : 0},
        {(void**)&h->knw, h->qk_type ? L * knw_n * 2 : 0},
        {(void**)&h->wqkv, L * h->nqkv * d * 2},
        {(void**)&h->wo, L * d * h->qn * 2},
        {(void**)&h->bqkv, h->bias ? L * h->nqkv * 4 : 0},
        {(void**)&h->lm, V * d * 4},
        {(void**)&h->cosb, (size_t)h->maxT * h->hd * 4},
        {(void**)&h->sinb, (size_t)h->maxT * h->hd * 4},
        {(void**)&h->kc, kvb},
        {(void**)&h->vc, kvb},
        {(void**)&h->h, (size_t)max_batch * d * 4},
        {(void**)&h->t, (size_t)max_batch * d * 4},
        {(void**)&h->h2, (size_t)max_batch * d * 4},
        {(void**)&h->qkv, (size_t)max_batch * h->nqkv * 4},
        {(void**)&h->att, (size_t)max_batch * h->qn * 4},
        {(void**)&h->scores, (size_t)max_batch * h->H * h->maxT * 4},
        {(void**)&h->qr, (size_t)max_batch * h->qn * 4},
        {(void**)&h->tT, max_batch >= kMmMinB ? (size_t)d * h->Bp * 4 : 0},
        {(void**)&h->attT, max_batch >= kMmMinB ? (size_t)h->qn * h->Bp * 4 : 0},
        {(void**)&h->logits, (size_t)max_batch * V * 4},
        {(void**)&h->tok, (size_t)max_batch * 4},
        {(void**)&h->arg_v, (size_t)max_batch * kArgParts * 4},
        {(void**)&h->arg_i, (size_t)max_batch * kArgParts * 4},
        {(void**)&h->pre_pos, (size_t)max_batch * 4},
        {(void**)&h->pre_slot, (size_t)max_batch * 4},
        {(void**)&h->err, 16},
        {&h->stage, h->stage_bytes},
    };
    for (auto& a : al) {
        if (!a.n) continue;
        if (cudaMalloc(a.p, a.n) != cudaSuccess) {
            cudaGetLastError();
            jl_dec_destroy(h);
            return JL_ERR_OOM;
        }
    }
    cudaStream_t s = nullptr;
    const int od = src_on_device;
    auto fail = [&](int r) {
        cudaStreamSynchronize(s);
        jl_dec_destroy(h);
        return r;
    };
    if (cudaMemsetAsync(h->err, 0, 16, s) != cudaSuccess || cudaMemsetAsync(h->kc, 0, kvb, s) != cudaSuccess ||
        cudaMemsetAsync(h->vc, 0, kvb, s) != cudaSuccess)
        return fail(JL_ERR_CUDA);
    if ((rc = put(h->embed, W->embed, V * d * 2, od, s)) || (rc = put(h->norm1, W->norm1, L * d * 2, od, s)) ||
        (rc = put(h->norm2, W->norm2, L * d * 2, od, s)) || (rc = put(h->fnorm, W->final_norm, d * 2, od, s)) ||
        (rc = put(h->cosb, W->cos, (size_t)h->maxT * h->hd * 4, od, s)) ||
        (rc = put(h->sinb, W->sin, (size_t)h->maxT * h->hd * 4, od, s)))
        return fail(rc);
    if (h->qk_type && ((rc = put(h->qnw, W->qn, L * qnw_n * 2, od, s)) || (rc = put(h->knw, W->kn, L * knw_n * 2, od, s))))
        return fail(rc);
    uint16_t* st16 = static_cast<uint16_t*>(h->stage);
    for (int l = 0; l < h->L; l++) {
        const size_t qrows = (size_t)h->qn * d, krows = (size_t)h->kn * d;
        if ((rc = put(st16, W->wq + l * qrows, qrows * 2, od, s)) ||
            (rc = put(st16 + qrows, W->wk + l * krows, krows * 2, od, s)) ||
            (rc = put(st16 + qrows + krows, W->wv + l * krows, krows * 2, od, s)) ||
            (rc = repack_mv<uint16_t>(st16, h->wqkv + (size_t)l * h->nqkv * d, h->nqkv, (int)d, s)))
            return fail(rc);
        if ((rc = put(st16, W->wo + (size_t)l * d * h->qn, d * h->qn * 2, od, s)) ||
            (rc = repack_mv<uint16_t>(st16, h->wo + (size_t)l * d * h->qn, (int)d, h->qn, s)))
            return fail(rc);
        if (h->bias) {
            float* bl = h->bqkv + (size_t)l * h->nqkv;
            if ((rc = put(bl, W->bq + (size_t)l * h->qn, h->qn * 4, od, s)) ||
                (rc = put(bl + h->qn, W->bk + (size_t)l * h->kn, h->kn * 4, od, s)) ||
                (rc = put(bl + h->qn + h->kn, W->bv + (size_t)l * h->kn, h->kn * 4, od, s)))
                return fail(rc);
        }
    }
    // lm_head: declared unsigned short* in KernelW but fp32 [V, d] (decoder3.py:218-230)
    if ((rc = put(h->stage, W->lm_head, V * d * 4, od, s)) ||
        (rc = repack_mv<float>(static_cast<float*>(h->stage), h->lm, (int)V, (int)d, s)))
        return fail(rc);
    if (cudaStreamSynchronize(s) != cudaSuccess) return fail(JL_ERR_CUDA);
    cudaFree(h->stage);  // the staging buffer is only needed while uploading
    h->stage = nullptr;
    // the MoE layers (expert tables may be absent: upload them later through jl_dec_moe)
    if (W->expert_pk[0] && W->expert_sc[0]) {
        std::vector<const unsigned char*> pk(3 * h->E);
        std::vector<const unsigned short*> sc(3 * h->E);
        for (int l = 0; l < h->L; l++) {
            for (int p = 0; p < 3; p++)
                for (int e = 0; e < h->E; e++) {
                    pk[p * h->E + e] = W->expert_pk[p][(size_t)l * h->E + e];
                    sc[p * h->E + e] = W->expert_sc[p][(size_t)l * h->E + e];
                }
            rc = jl_moe_upload_layer(h->moe, l, W->gate_w + (size_t)l * h->E * d, pk.data(), sc.data(), od, s);
            if (rc) return fail(rc);
        }
    }
    *out = h;
    return JL_OK;
}

extern "C" int jl_dec_moe(jl_dec* h, jl_moe** moe) {
    if (!h || !moe) return JL_ERR_INVALID;
    *moe = h->moe;
    return JL_OK;
}

extern "C" int jl_dec_kv(jl_dec* h, float** k, float** v) {
    if (!h || !k || !v) return JL_ERR_INVALID;
    *k = h->kc;
    *v = h->vc;
    return JL_OK;
}

extern "C" int jl_dec_embed(jl_dec* h, const int* tokens, int B, float* x, void* stream) {
    using namespace jl;
    if (!h || B < 0) return JL_ERR_INVALID;
    if (B == 0) return JL_OK;
    if (!tokens || !x) return JL_ERR_INVALID;
    return launch(k_embed, dim3((h->d + 255) / 256, B), dim3(256), 0, (cudaStream_t)stream, (const uint16_t*)h->embed,
                  tokens, h->V, h->d, x, h->err);
}

// dbg (device, B = 1 only): per layer 7 rows of max(E, d) floats, as the
// reference's debug_decode_layers (decode_kernel.c:1764-1790) writes them:
// norm1 output, attention output, h after attention, norm2 output, router
// logits, MoE output, h after the MoE layer.
// prefill = 1: the B rows are consecutive positions of one sequence (one
// launch's rows attend to each other: K/V rows are appended first, then the
// attention reads every row from the cache); the MoE layers combine in each
// token's own order; logits/tok are of the last row only.
static int dec_step(jl_dec* h, const int* slots, const int* positions, const float* x, int B, float* logits,
                    int* tok, float* dbg, cudaStream_t s, int prefill = 0);

extern "C" int jl_dec_step(jl_dec* h, const int* slots, const int* positions, const float* x, int B,
                           float* logits, int* tok, void* stream) {
    return dec_step(h, slots, positions, x, B, logits, tok, nullptr, (cudaStream_t)stream);
}

static int dec_step(jl_dec* h, const int* slots, const int* positions, const float* x, int B, float* logits,
                    int* tok, float* dbg, cudaStream_t s, int prefill) {
    using namespace jl;
    if (!h || B < 0) return JL_ERR_INVALID;
    if (B == 0) return JL_OK;
    if (!slots || !positions || !x) return JL_ERR_INVALID;
    if (B > h->max_batch) return JL_ERR_CAPACITY;
    if (dbg && B != 1) return JL_ERR_INVALID;
    int rc = dec_attrs();
    if (rc) return rc;
    const int d = h->d, sms = h->moe->sm_count;
    const size_t rowlen = (size_t)std::max(h->E, d);
    auto snap = [&](int l, int r, const float* src, int n) -> int {
        if (!dbg) return JL_OK;
        const cudaError_t e = cudaMemcpyAsync(dbg + ((size_t)l * 7 + r) * rowlen, src, (size_t)n * 4,
                                              cudaMemcpyDeviceToDevice, s);
        return e == cudaSuccess ? JL_OK : jl_note_cuda(e);
    };
    JL_CUDA(cudaMemcpyAsync(h->h, x, (size_t)B * d * 4, cudaMemcpyDeviceToDevice, s));
    const size_t nsm = (size_t)2 * d * sizeof(float);
    attn_args aa;
    aa.qkv = h->qkv, aa.att = h->att, aa.positions = positions, aa.slots = slots, aa.kc = h->kc, aa.vc = h->vc;
    aa.cosb = h->cosb, aa.sinb = h->sinb, aa.L = h->L, aa.H = h->H, aa.KH = h->KH, aa.hd = h->hd, aa.maxT = h->maxT;
    aa.qk_type = h->qk_type, aa.eps = h->eps, aa.err = h->err, aa.qr = h->qr;
    aa.sqn = attn_sqn(h->qk_type, h->H, h->KH, h->hd);
    aa.nslots = h->slots;
    // column-major copies of the matvec inputs for the register-tiled kernel (B >= kMmMinB)
    float* tT = B >= kMmMinB ? h->tT : nullptr;
    aa.attT = B >= kMmMinB ? h->attT : nullptr;
    aa.Bp = h->Bp;
    // attention work split: score blocks (group, sequence, position split) and
    // value blocks (head, sequence, dimension slice), about two blocks per SM
    const qk_layout qkl(h->qk_type, h->H, h->KH, h->hd);
    const size_t qk_smem = (size_t)qkl.total * sizeof(float);
    int splits = std::max(1, std::min((2 * sms + h->KH * B - 1) / (h->KH * B), (h->maxT + kQkTile - 1) / kQkTile));
    const int tp = ((h->maxT + splits - 1) / splits + kQkTile - 1) / kQkTile * kQkTile;
    splits = (h->maxT + tp - 1) / tp;
    // value blocks: whole KV groups when that still gives >= one block per SM
    // (V read once per group), else single heads; slices of the head
    // dimension (multiples of 4 floats) up to 4 per head
    const int gsz = h->H / h->KH, maxT4 = (h->maxT + 3) / 4 * 4;
    // the register-tiled kernels at batches of 16 and more, for contexts whose
    // score rows fit the value kernel's shared memory (longer ones take k_attn_pv)
    const bool attn_t = B >= 16 && attn_tiled_ok(h->hd, gsz) &&
                        (size_t)pv_t_layout(gsz, h->maxT, h->hd).total * sizeof(float) <= 200 * 1024;
    auto pick_slices = [&](int units, int target) {
        int ds = 1;
        while (ds < 4 && units * ds < target && h->hd % (8 * ds) == 0) ds *= 2;
        return ds;
    };
    int hpb = gsz, dslices = pick_slices(h->KH * B, sms);
    auto pv_bytes = [&](int hp, int ds) {
        return ((size_t)hp * maxT4 + (size_t)kPvRing * kPvTile * (h->hd / ds)) * sizeof(float);
    };
    // all of a block's V rows in shared memory when they fit (small batches:
    // one wait instead of a barrier per tile)
    auto pv_whole_bytes = [&](int hp, int ds) {
        return ((size_t)hp * maxT4 + (size_t)maxT4 * (h->hd / ds)) * sizeof(float);
    };
    if (gsz > 8 || 8 % gsz || h->KH * B * dslices < sms || hpb * (h->hd / dslices) / 4 > kPvItems * kPvThreads ||
        pv_bytes(hpb, dslices) > 200 * 1024) {
        hpb = 1;
        dslices = pick_slices(h->H * B, 2 * sms);
    }
    const int pv_items = (hpb * (h->hd / dslices) / 4 + kPvThreads - 1) / kPvThreads;
    const int dw = h->hd / dslices;
    const int pv_whole = pv_whole_bytes(hpb, dslices) <= 100 * 1024;
    const size_t pv_smem = pv_whole ? pv_whole_bytes(hpb, dslices) : pv_bytes(hpb, dslices);
    if (qk_smem > 200 * 1024 || pv_smem > 200 * 1024) return JL_ERR_INVALID;
    for (int l = 0; l < h->L; l++) {
        // norm1 (adding the previous layer's MoE output to the residual)
        rc = launch(k_rms, dim3(B), dim3(kNormThreads), nsm, s, h->h, (const float*)(l ? h->h2 : nullptr),
                    (const uint16_t*)(h->norm1 + (size_t)l * d), h->eps, d, h->t, tT, h->Bp);
        if (!rc && l > 0) rc = snap(l - 1, 6, h->h, d);
        if (!rc) rc = snap(l, 0, h->t, d);
        if (!rc)
            rc = launch_mv<uint16_t>(h->wqkv + (size_t)l * h->nqkv * d, h->t, tT, h->Bp, h->nqkv, d, B,
                                     h->bias ? h->bqkv + (size_t)l * h->nqkv : nullptr, h->qkv, sms, s);
        if (!rc) {
            aa.l = l;
            const size_t qs = h->qk_type == 2 ? (size_t)h->qn : h->hd, ks = h->qk_type == 2 ? (size_t)h->kn : h->hd;
            aa.qnw = h->qk_type ? h->qnw + l * qs : nullptr;
            aa.knw = h->qk_type ? h->knw + l * ks : nullptr;
            aa.from_cache = prefill;
            if (prefill && !attn_t)
                rc = launch(k_kv_append, dim3(h->KH, B), dim3(kAttnThreads), (size_t)(128 + aa.sqn) * sizeof(float),
                            s, aa);
            if (!rc && attn_t)
                rc = h->hd == 64 ? launch_attn_t<64>(aa, h->scores, B, sms, s)
                                 : launch_attn_t<128>(aa, h->scores, B, sms, s);
            else if (!rc) rc = launch(k_attn_qk, dim3(h->KH, B, splits), dim3(kQkThreads), qk_smem, s, aa, h->scores, tp);
            if (!rc && !attn_t) {
                auto kern = pv_items <= 1 ? k_attn_pv<1> : pv_items <= 2 ? k_attn_pv<2> : k_attn_pv<4>;
                rc = launch(kern, dim3(h->H / hpb, B, dslices), dim3(kPvThreads), pv_smem, s, aa,
                            (const float*)h->scores, hpb, dw, pv_whole);
            }
        }
        if (!rc)
            rc = launch_mv<uint16_t>(h->wo + (size_t)l * d * h->qn, h->att, aa.attT, h->Bp, d, h->qn, B, nullptr, h->h2,
                                     sms, s);
        if (!rc) rc = snap(l, 1, h->h2, d);
        // norm2 (adding the attention output to the residual), then the MoE layer
        if (!rc)
            rc = launch(k_rms, dim3(B), dim3(kNormThreads), nsm, s, h->h, (const float*)h->h2,
                        (const uint16_t*)(h->norm2 + (size_t)l * d), h->eps, d, h->t, (float*)nullptr, h->Bp);
        if (!rc) rc = snap(l, 2, h->h, d);
        if (!rc) rc = snap(l, 3, h->t, d);
        if (!rc) {
            h->moe->comb_token_order = prefill;
            rc = jl_moe_forward(h->moe, l, h->t, B, h->h2, nullptr, nullptr, s);
            h->moe->comb_token_order = 0;
        }
        if (!rc) rc = snap(l, 4, h->moe->ws.logits, h->E);
        if (!rc) rc = snap(l, 5, h->h2, d);
        if (rc) return rc;
    }
    rc = launch(k_rms, dim3(B), dim3(kNormThreads), nsm, s, h->h, (const float*)h->h2, (const uint16_t*)h->fnorm,
                h->eps, d, h->t, tT, h->Bp);
    if (!rc) rc = snap(h->L - 1, 6, h->h, d);
    if (rc) return rc;
    if (logits || tok) {
        const int nb = prefill ? 1 : B;
        const float* tx = prefill ? h->t + (size_t)(B - 1) * d : h->t;
        rc = launch_mv<float>(h->lm, tx, prefill ? nullptr : tT, h->Bp, h->V, d, nb, nullptr, h->logits, sms, s);
        if (!rc && tok)
            rc = launch(k_argmax_part, dim3(kArgParts, nb), dim3(256), 0, s, (const float*)h->logits, h->V,
                        h->arg_v, h->arg_i);
        if (!rc && tok) rc = launch(k_argmax_fin, dim3(nb), dim3(32), 0, s, (const float*)h->arg_v,
                                    (const int*)h->arg_i, tok);
        if (!rc && logits)
            rc = cudaMemcpyAsync(logits, h->logits, (size_t)nb * h->V * 4, cudaMemcpyDeviceToDevice, s) == cudaSuccess
                     ? JL_OK
                     : JL_ERR_CUDA;
    }
    return rc;
}

namespace jl {
__global__ void k_prefill_rows(int* pos, int* slot, int p0, int s, int n) {
    griddep_wait();
    griddep_launch_dependents();
    const int i = threadIdx.x + blockIdx.x * blockDim.x;
    if (i < n) {
        pos[i] = p0 + i;
        slot[i] = s;
    }
}
}  // namespace jl

extern "C" int jl_dec_prefill(jl_dec* h, int slot, const int* tokens, int T, int pos0, float* logits, int* tok,
                              void* stream) {
    using namespace jl;
    if (!h || T < 0 || slot < 0 || slot >= h->slots || pos0 < 0) return JL_ERR_INVALID;
    if (T == 0) return JL_OK;
    if (!tokens || pos0 + T > h->maxT) return JL_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    const int Bm = h->max_batch;
    for (int c0 = 0; c0 < T; c0 += Bm) {
        const int n = std::min(Bm, T - c0);
        const bool last = c0 + n == T;
        int rc = launch(k_prefill_rows, dim3((n + 127) / 128), dim3(128), 0, s, h->pre_pos, h->pre_slot, pos0 + c0,
                        slot, n);
        if (!rc) rc = jl_dec_embed(h, tokens + c0, n, h->t, s);
        if (!rc)
            rc = dec_step(h, h->pre_slot, h->pre_pos, h->t, n, last ? logits : nullptr, last ? tok : nullptr,
                          nullptr, s, 1);
        if (rc) return rc;
    }
    return JL_OK;
}

extern "C" int jl_dec_check(jl_dec* h, void* stream) {
    if (!h) return JL_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    int err = 0;
    JL_CUDA(cudaMemcpyAsync(&err, h->err, sizeof(int), cudaMemcpyDeviceToHost, s));
    JL_CUDA(cudaStreamSynchronize(s));
    if (err) JL_CUDA(cudaMemsetAsync(h->err, 0, sizeof(int), s));
    const int rc = jl_moe_check(h->moe, stream);
    if (err & jl::kErrPosition) return JL_ERR_INVALID;
    if (err) return JL_ERR_DEVICE;
    return rc;
}

// ---------------------------------------------------------------------------
// The reference's own decode entry points (decode_kernel.c:1518-1600), host
// buffers and KVCache pointers, backed by one cached jl_dec per (cfg, W).
//
// KV caches: the reference keeps them in the caller's host arrays
// (kv[b*L + l].k / .v, each [maxT, KH, hd] fp32). The library keeps a device
// copy of each sequence (identified by its layer-0 K pointer) and its row
// count n. A call at position p uses the device copy when p == n; otherwise it
// first copies the host rows [0, p) of every layer to the device. After the
// step the new row of every layer is written back to the host arrays, so the
// caller's caches hold what the reference would have written.

namespace {

struct dec_entry {
    KernelCfg cfg;
    const void* key_embed;
    const void* key_pk;
    uint64_t fp;  // jl_weights_fingerprint at upload
    jl_dec* h;
    cudaStream_t st;
    int* slots_d;
    int* pos_d;
    float* x_d;
    int* tok_d;
    float* k_pin;   // pinned staging of one step's new K/V rows [B][L][kn] x 2
    float* v_pin;
    std::unordered_map<const float*, int> seq_slot;  // layer-0 K pointer -> slot
    std::vector<int> slot_rows;                      // rows held per slot
    std::vector<const float*> slot_key;
    std::vector<long long> slot_used;                // last call that used the slot (eviction)
    long long calls;
};

std::mutex g_dec_mu;
std::vector<dec_entry*> g_decs;
thread_local int t_dec_status = JL_OK;

constexpr int kDropinBatch = 32;  // sequences per call and KV slots held (the reference caps a call at 16)

void dec_entry_free(dec_entry* e) {
    cudaStreamSynchronize(e->st);
    cudaFree(e->slots_d);
    cudaFree(e->pos_d);
    cudaFree(e->x_d);
    cudaFree(e->tok_d);
    cudaFreeHost(e->k_pin);
    cudaFreeHost(e->v_pin);
    cudaStreamDestroy(e->st);
    jl_dec_destroy(e->h);
    delete e;
}

dec_entry* dec_for(const KernelCfg* c, const KernelW* W, int* rc) {
    const uint64_t fp = jl_weights_fingerprint(c, W, true);
    for (size_t i = 0; i < g_decs.size(); i++) {
        dec_entry* e = g_decs[i];
        if (e->key_embed != W->embed || e->key_pk != W->expert_pk[0] || memcmp(&e->cfg, c, sizeof(*c))) continue;
        if (e->fp == fp) return e;
        dec_entry_free(e);  // same addresses, other weights: drop the stale copy
        g_decs.erase(g_decs.begin() + i);
        break;
    }
    auto* e = new (std::nothrow) dec_entry();
    if (!e) {
        *rc = JL_ERR_OOM;
        return nullptr;
    }
    e->cfg = *c;
    e->key_embed = W->embed;
    e->key_pk = W->expert_pk[0];
    e->fp = fp;
    e->calls = 0;
    const int slots = kDropinBatch;
    *rc = jl_dec_create(c, W, kDropinBatch, slots, 0, &e->h);
    if (*rc) {
        delete e;
        return nullptr;
    }
    jl_moe_set_path(e->h->moe, JL_PATH_EXACT);  // the reference's arithmetic: bit-identical layers
    const size_t rows = (size_t)kDropinBatch * c->L * e->h->kn;
    if (cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&e->slots_d, kDropinBatch * 4) != cudaSuccess || cudaMalloc(&e->pos_d, kDropinBatch * 4) != cudaSuccess ||
        cudaMalloc(&e->x_d, (size_t)kDropinBatch * c->d * 4) != cudaSuccess ||
        cudaMalloc(&e->tok_d, kDropinBatch * 4) != cudaSuccess ||
        cudaHostAlloc(&e->k_pin, rows * 4, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc(&e->v_pin, rows * 4, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        *rc = JL_ERR_OOM;
        jl_dec_destroy(e->h);
        delete e;
        return nullptr;
    }
    e->slot_rows.assign(slots, -1);
    e->slot_key.assign(slots, nullptr);
    e->slot_used.assign(slots, -1);
    g_decs.push_back(e);
    return e;
}

// The device slot of the sequence whose layer caches are kvb[0..L): found by
// its layer-0 K pointer, else a free slot or the least recently used one not
// in this call. Unless the slot holds exactly p rows, the host rows [0, p)
// of every layer are copied over first. Afterwards it counts rows_after rows.
int acquire_slot(dec_entry* e, const KVCache* kvb, int L, int p, int rows_after, int* out) {
    jl_dec* h = e->h;
    const int kn = h->kn;
    const size_t row_b = (size_t)kn * 4;
    if (p < 0 || rows_after > h->maxT) return JL_ERR_INVALID;
    const float* key = kvb[0].k;
    if (!key) return JL_ERR_INVALID;
    auto it = e->seq_slot.find(key);
    int sl;
    if (it != e->seq_slot.end()) {
        sl = it->second;
    } else {
        sl = -1;
        for (int i = 0; i < h->slots; i++)
            if (!e->slot_key[i]) {
                sl = i;
                break;
            }
        if (sl < 0) {
            long long best = LLONG_MAX;
            for (int i = 0; i < h->slots; i++)
                if (e->slot_used[i] < e->calls && e->slot_used[i] < best) {
                    best = e->slot_used[i];
                    sl = i;
                }
            if (sl < 0) return JL_ERR_CAPACITY;
            e->seq_slot.erase(e->slot_key[sl]);
        }
        e->seq_slot[key] = sl;
        e->slot_key[sl] = key;
        e->slot_rows[sl] = -1;
    }
    e->slot_used[sl] = e->calls;
    if (e->slot_rows[sl] != p) {  // bring the host rows [0, p) of every layer over
        for (int l = 0; l < L; l++) {
            const KVCache& cl = kvb[l];
            if (!cl.k || !cl.v) return JL_ERR_INVALID;
            const size_t off = ((size_t)sl * L + l) * h->maxT * kn;
            if (p > 0) {
                JL_CUDA(cudaMemcpyAsync(h->kc + off, cl.k, (size_t)p * row_b, cudaMemcpyHostToDevice, e->st));
                JL_CUDA(cudaMemcpyAsync(h->vc + off, cl.v, (size_t)p * row_b, cudaMemcpyHostToDevice, e->st));
            }
        }
    }
    e->slot_rows[sl] = rows_after;
    *out = sl;
    return JL_OK;
}

// One batched step through the drop-in: logits (host, [B, V]) and/or tokens.
int dropin_step(const KernelCfg* c, const KernelW* W, KVCache* kv, const int* positions, const float* xin,
                int B, float* logits, int* out_tok, float* dbg_host = nullptr) {
    if (!c || !W || !kv || !positions || !xin || B < 0) return JL_ERR_INVALID;
    if (B == 0) return JL_OK;
    std::lock_guard<std::mutex> lk(g_dec_mu);
    int rc = JL_OK;
    dec_entry* e = dec_for(c, W, &rc);
    if (!e) return rc;
    jl_dec* h = e->h;
    if (B > h->max_batch) return JL_ERR_CAPACITY;
    const int L = c->L, kn = h->kn;
    const size_t row_b = (size_t)kn * 4;
    e->calls++;
    std::vector<int> slot(B);
    for (int b = 0; b < B; b++) {
        rc = acquire_slot(e, kv + (size_t)b * L, L, positions[b], positions[b] + 1, &slot[b]);
        if (rc) return rc;
    }
    JL_CUDA(cudaMemcpyAsync(e->slots_d, slot.data(), (size_t)B * 4, cudaMemcpyHostToDevice, e->st));
    JL_CUDA(cudaMemcpyAsync(e->pos_d, positions, (size_t)B * 4, cudaMemcpyHostToDevice, e->st));
    JL_CUDA(cudaMemcpyAsync(e->x_d, xin, (size_t)B * c->d * 4, cudaMemcpyHostToDevice, e->st));
    float* dbg_d = nullptr;
    const size_t dbg_n = (size_t)L * 7 * std::max(h->E, c->d);
    if (dbg_host) {
        if (B != 1) return JL_ERR_INVALID;
        if (cudaMallocAsync(reinterpret_cast<void**>(&dbg_d), dbg_n * 4, e->st) != cudaSuccess) return JL_ERR_OOM;
        JL_CUDA(cudaMemsetAsync(dbg_d, 0, dbg_n * 4, e->st));
    }
    rc = dec_step(h, e->slots_d, e->pos_d, e->x_d, B, nullptr, out_tok ? e->tok_d : nullptr, dbg_d, e->st);
    if (dbg_d) {
        if (!rc && cudaMemcpyAsync(dbg_host, dbg_d, dbg_n * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess)
            rc = JL_ERR_CUDA;
        cudaFreeAsync(dbg_d, e->st);
    }
    if (!rc && logits)
        rc = launch_mv<float>(h->lm, h->t, B >= kMmMinB ? h->tT : nullptr, h->Bp, h->V, c->d, B, nullptr, h->logits,
                              h->moe->sm_count, e->st);
    if (rc) return rc;
    // the new K/V row of every layer back into the caller's caches
    for (int b = 0; b < B; b++)
        for (int l = 0; l < L; l++) {
            const size_t off = (((size_t)slot[b] * L + l) * h->maxT + positions[b]) * kn;
            JL_CUDA(cudaMemcpyAsync(e->k_pin + ((size_t)b * L + l) * kn, h->kc + off, row_b, cudaMemcpyDeviceToHost, e->st));
            JL_CUDA(cudaMemcpyAsync(e->v_pin + ((size_t)b * L + l) * kn, h->vc + off, row_b, cudaMemcpyDeviceToHost, e->st));
        }
    if (logits) JL_CUDA(cudaMemcpyAsync(logits, h->logits, (size_t)B * h->V * 4, cudaMemcpyDeviceToHost, e->st));
    if (out_tok) JL_CUDA(cudaMemcpyAsync(out_tok, e->tok_d, (size_t)B * 4, cudaMemcpyDeviceToHost, e->st));
    JL_CUDA(cudaStreamSynchronize(e->st));
    rc = jl_dec_check(h, e->st);
    if (rc) {
        for (int b = 0; b < B; b++) e->slot_rows[slot[b]] = -1;  // resync these sequences next time
        return rc;
    }
    for (int b = 0; b < B; b++)
        for (int l = 0; l < L; l++) {
            const KVCache& cl = kv[(size_t)b * L + l];
            memcpy(cl.k + (size_t)positions[b] * kn, e->k_pin + ((size_t)b * L + l) * kn, row_b);
            memcpy(cl.v + (size_t)positions[b] * kn, e->v_pin + ((size_t)b * L + l) * kn, row_b);
        }
    return JL_OK;
}

void nan_fill(float* p, size_t n) {
    if (!p) return;
    const float q = __builtin_nanf("");
    for (size_t i = 0; i < n; i++) p[i] = q;
}

}  // namespace

extern "C" void decode_layers_batch(const KernelCfg* c, const KernelW* W, KVCache* kv, const int* positions,
                                    const float* xin, int B, float* logits) {
    t_dec_status = dropin_step(c, W, kv, positions, xin, B, logits, nullptr);
    if (t_dec_status && c && B > 0) nan_fill(logits, (size_t)B * c->V);
}

extern "C" void decode_layers_batch_argmax(const KernelCfg* c, const KernelW* W, KVCache* kv,
                                           const int* positions, const float* xin, int B, int* out_tok) {
    t_dec_status = dropin_step(c, W, kv, positions, xin, B, nullptr, out_tok);
    if (t_dec_status && out_tok)
        for (int b = 0; b < B; b++) out_tok[b] = -1;
}

extern "C" void decode_layers(const KernelCfg* c, const KernelW* W, KVCache* kv, int pos, const float* xin,
                              float* logits) {
    const int p[1] = {pos};
    decode_layers_batch(c, W, kv, p, xin, 1, logits);
}

extern "C" void embed_lookup(const KernelW* W, const KernelCfg* c, int token, float* out) {
    t_dec_status = JL_ERR_INVALID;
    if (!W || !c || !out || !W->embed) return;
    if (token < 0 || token >= c->V) {
        nan_fill(out, (size_t)c->d);
        return;
    }
    std::lock_guard<std::mutex> lk(g_dec_mu);
    int rc = JL_OK;
    dec_entry* e = dec_for(c, W, &rc);
    if (e) {
        if (cudaMemcpyAsync(e->tok_d, &token, 4, cudaMemcpyHostToDevice, e->st) != cudaSuccess) rc = JL_ERR_CUDA;
        if (!rc) rc = jl_dec_embed(e->h, e->tok_d, 1, e->x_d, e->st);
        if (!rc && cudaMemcpyAsync(out, e->x_d, (size_t)c->d * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess)
            rc = JL_ERR_CUDA;
        if (!rc && cudaStreamSynchronize(e->st) != cudaSuccess) rc = JL_ERR_CUDA;
    }
    t_dec_status = rc;
    if (rc) nan_fill(out, (size_t)c->d);
}

// prefill_layers (decode_kernel.c:1606-1615) runs one B = 1 decode step per
// position; here the positions run as batches of one sequence (jl_dec_prefill:
// K/V rows appended before the attention, each token's own combine order),
// which gives every position the bits of the one-position step.
static int dropin_prefill(const KernelCfg* c, const KernelW* W, KVCache* kv, const int* tokens, int T,
                          float* logits) {
    if (!c || !W || !kv || !tokens || T < 0) return JL_ERR_INVALID;
    if (T == 0) return JL_OK;
    for (int t = 0; t < T; t++)
        if (tokens[t] < 0 || tokens[t] >= c->V) return JL_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_dec_mu);
    int rc = JL_OK;
    dec_entry* e = dec_for(c, W, &rc);
    if (!e) return rc;
    jl_dec* h = e->h;
    if (T > h->maxT) return JL_ERR_INVALID;
    const int L = c->L, kn = h->kn;
    e->calls++;
    int sl = 0;
    rc = acquire_slot(e, kv, L, 0, T, &sl);
    if (rc) return rc;
    int* tok_d = nullptr;
    float* lg_d = nullptr;
    if (cudaMallocAsync(reinterpret_cast<void**>(&tok_d), (size_t)T * 4, e->st) != cudaSuccess ||
        cudaMallocAsync(reinterpret_cast<void**>(&lg_d), (size_t)c->V * 4, e->st) != cudaSuccess) {
        cudaGetLastError();
        if (tok_d) cudaFreeAsync(tok_d, e->st);
        return JL_ERR_OOM;
    }
    rc = cudaMemcpyAsync(tok_d, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, e->st) == cudaSuccess ? JL_OK
                                                                                                  : JL_ERR_CUDA;
    if (!rc) rc = jl_dec_prefill(h, sl, tok_d, T, 0, logits ? lg_d : nullptr, nullptr, e->st);
    if (!rc && logits &&
        cudaMemcpyAsync(logits, lg_d, (size_t)c->V * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess)
        rc = JL_ERR_CUDA;
    // the rows [0, T) of every layer back into the caller's caches
    for (int l = 0; l < L && !rc; l++) {
        const size_t off = ((size_t)sl * L + l) * h->maxT * kn;
        if (cudaMemcpyAsync(kv[l].k, h->kc + off, (size_t)T * kn * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess ||
            cudaMemcpyAsync(kv[l].v, h->vc + off, (size_t)T * kn * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess)
            rc = JL_ERR_CUDA;
    }
    cudaFreeAsync(tok_d, e->st);
    cudaFreeAsync(lg_d, e->st);
    if (cudaStreamSynchronize(e->st) != cudaSuccess && !rc) rc = JL_ERR_CUDA;
    if (!rc) rc = jl_dec_check(h, e->st);
    if (rc) e->slot_rows[sl] = -1;
    return rc;
}

extern "C" void prefill_layers(const KernelCfg* c, const KernelW* W, KVCache* kv, const int* tokens, int T,
                               float* logits) {
    t_dec_status = dropin_prefill(c, W, kv, tokens, T, logits);
    if (t_dec_status && logits && c) nan_fill(logits, (size_t)c->V);
}

extern "C" void debug_decode_layers(const KernelCfg* c, const KernelW* W, KVCache* kv, int pos, const float* xin,
                                    float* out) {
    const int p[1] = {pos};
    t_dec_status = dropin_step(c, W, kv, p, xin, 1, nullptr, nullptr, out);
    if (t_dec_status && c && out) nan_fill(out, (size_t)c->L * 7 * std::max(c->E, c->d));
}

// The reference's CPU thread-pool controls, which its Python calls at start-up
// (decoder3.py:133-145): the GPU library has no host pool, so they only
// report success.
extern "C" int spin_pool_init(int n_workers) {
    (void)n_workers;
    return 1;
}
extern "C" void set_lm_threads(int n) { (void)n; }

extern "C" int jl_decode_status(void) { return t_dec_status; }
