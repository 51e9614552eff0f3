/* CPU restatement of the reference's MoE decode hot path (see joule_oracle.h).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA product. Build with
 * -ffp-contract=off (oracle/Makefile) so that every scalar product and sum
 * below rounds exactly where the reference's rounds; the reference's AVX2
 * `_mm256_fmadd_ps` chains are restated with explicit fmaf() calls.
 */
#include "joule_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef union {
    uint32_t u;
    float f;
} bits32;

/* decode_kernel.c:64-85: exact half -> float, subnormals normalised. */
float jo_fp16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int32_t e = (h >> 10) & 0x1F;
    uint32_t man = h & 0x3FFu;
    bits32 r;
    if (e == 0) {
        if (man == 0) {
            r.u = sign;
        } else {
            int32_t ex = 113; /* 127 - 15 + 1 */
            while (!(man & 0x400u)) {
                man <<= 1;
                ex--;
            }
            r.u = sign | ((uint32_t)ex << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        r.u = sign | 0x7F800000u | (man << 13);
    } else {
        r.u = sign | ((uint32_t)(e + 112) << 23) | (man << 13);
    }
    return r.f;
}

/* decode_kernel.c:47-53: bf16 is the top half of an fp32. */
float jo_bf16_to_f32(uint16_t h) {
    bits32 r;
    r.u = (uint32_t)h << 16;
    return r.f;
}

/* decode_kernel.c:94-108: the reference's own range-reduced degree-5
 * polynomial; every product and sum rounds separately (no contraction). */
float jo_expf_fast(float v) {
    if (v < -17.0f) return 0.0f;
    if (v > 88.0f) v = 88.0f;
    const float y = v * 1.4426950408889634f;
    const int k = (int)(y + (y >= 0 ? 0.5f : -0.5f));
    const float f = y - (float)k;
    float p = 0.0013330f;
    p = 0.0096181f + f * p;
    p = 0.0555041f + f * p;
    p = 0.2402265f + f * p;
    p = 0.6931472f + f * p;
    p = 1.0f + f * p;
    int kk = k + 127;
    if (kk < 0) return 0.0f;
    if (kk > 254) kk = 254;
    bits32 s;
    s.u = (uint32_t)kk << 23;
    return p * s.f;
}

/* Horizontal sum of an 8-lane AVX register in the reference's order
 * (decode_kernel.c:843-846): (lo128 + hi128) -> + movehl -> + lane 1. */
static inline float hsum8(const float l[8]) {
    const float s0 = l[0] + l[4], s1 = l[1] + l[5];
    const float s2 = l[2] + l[6], s3 = l[3] + l[7];
    return (s0 + s2) + (s1 + s3);
}

/* Value of element i (0..63) of a 32-byte Q4 group, as the float (nib - 8):
 * byte i/2, low nibble for even i (q4_store.py:53, decode_kernel.c:787-797). */
static inline float q4_val(const uint8_t* grp, int i) {
    const uint8_t byte = grp[i >> 1];
    const int nib = (i & 1) ? (byte >> 4) : (byte & 0x0F);
    return (float)(nib - 8);
}

/* decode_kernel.c:770-858 (AVX2): per 64-value group, lane j of an 8-lane
 * accumulator takes elements j, j+8, ..., j+56 by FMA in that order; the
 * lanes are summed by hsum8, then acc[b] += hsum * scale (mul, then add). */
void jo_q4_row_dot_B(const uint8_t* row, const uint16_t* sc, const float* x,
                     int B, int stride, int ncols, float* acc) {
    const int ng = ncols / 64;
    for (int b = 0; b < B; b++) acc[b] = 0.0f;
    for (int g = 0; g < ng; g++) {
        const uint8_t* grp = row + (size_t)g * 32;
        const float s = jo_fp16_to_f32(sc[g]);
        float a[64];
        for (int i = 0; i < 64; i++) a[i] = q4_val(grp, i);
        for (int b = 0; b < B; b++) {
            const float* xg = x + (size_t)b * stride + (size_t)g * 64;
            float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int w = 0; w < 8; w++)
                for (int j = 0; j < 8; j++)
                    lane[j] = fmaf(a[w * 8 + j], xg[w * 8 + j], lane[j]);
            const float h = hsum8(lane);
            const float t = h * s;
            acc[b] = acc[b] + t;
        }
    }
    /* ncols % 64 != 0 never occurs for the store's shapes (the reference's
     * scalar tail, decode_kernel.c:826-840, is not restated). */
}

void jo_q4_gemm(float* out, const float* X, int T, const uint8_t* packed,
                const uint16_t* scales, int m, int d) {
    const int nb = d / 2, ng = d / 64;
    for (int t = 0; t < T; t++)
        for (int i = 0; i < m; i++) {
            float acc;
            jo_q4_row_dot_B(packed + (size_t)i * nb, scales + (size_t)i * ng,
                            X + (size_t)t * d, 1, d, d, &acc);
            out[(size_t)t * m + i] = acc;
        }
}

/* quant_gemv.c:35-57 (the scalar GEMV that ScalarBackend and kernel.q4_gemv
 * bind): per group, a sequential per-byte chain gacc += lo*x0 + hi*x1 (each
 * product and sum rounded), then acc += gacc * s. */
void jo_q4_gemv_scalar(float* out, const float* x, const uint8_t* packed,
                       const uint16_t* scales, int m, int d) {
    const int nb = d / 2, ng = d / 64;
    for (int i = 0; i < m; i++) {
        const uint8_t* row = packed + (size_t)i * nb;
        float acc = 0.0f;
        for (int g = 0; g < ng; g++) {
            const float s = jo_fp16_to_f32(scales[(size_t)i * ng + g]);
            float gacc = 0.0f;
            for (int b = g * 32; b < g * 32 + 32; b++) {
                const float lo = (float)((int)(row[b] & 0x0Fu) - 8) * x[2 * b];
                const float hi = (float)((int)(row[b] >> 4) - 8) * x[2 * b + 1];
                const float t = lo + hi;
                gacc = gacc + t;
            }
            const float p = gacc * s;
            acc = acc + p;
        }
        out[i] = acc;
    }
}

/* decode_kernel.c:234-256 / 693-718: lane j sums k = j mod 8 by FMA in k
 * order, then hsum8; the scalar tail (d % 8) is a separate mul and add. */
void jo_router_logits(const uint16_t* gate_w, const float* x, int B, int E,
                      int d, float* scores) {
    for (int b = 0; b < B; b++) {
        const float* xb = x + (size_t)b * d;
        for (int e = 0; e < E; e++) {
            const uint16_t* row = gate_w + (size_t)e * d;
            float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int k = 0;
            for (; k + 8 <= d; k += 8)
                for (int j = 0; j < 8; j++)
                    lane[j] = fmaf(jo_bf16_to_f32(row[k + j]), xb[k + j], lane[j]);
            float acc = hsum8(lane);
            for (; k < d; k++) {
                const float t = jo_bf16_to_f32(row[k]) * xb[k];
                acc = acc + t;
            }
            scores[(size_t)b * E + e] = acc;
        }
    }
}

/* decode_kernel.c:1425-1448 */
void jo_route(const float* logits, int B, int E, int k, int norm_topk_prob,
              int* top, float* tw, float* probs) {
    float* p = (float*)malloc(sizeof(float) * (size_t)E);
    for (int b = 0; b < B; b++) {
        const float* sc = logits + (size_t)b * E;
        float smax = -1e30f;
        for (int e = 0; e < E; e++)
            if (sc[e] > smax) smax = sc[e];
        float sum = 0.0f;
        for (int e = 0; e < E; e++) {
            p[e] = jo_expf_fast(sc[e] - smax);
            sum = sum + p[e];
        }
        for (int e = 0; e < E; e++) p[e] = p[e] / sum;
        int* tb = top + (size_t)b * k;
        float* wb = tw + (size_t)b * k;
        for (int i = 0; i < k; i++) {
            int bi = -1;
            float bv = -1e30f;
            for (int e = 0; e < E; e++) {
                int used = 0;
                for (int j = 0; j < i; j++)
                    if (tb[j] == e) {
                        used = 1;
                        break;
                    }
                if (!used && p[e] > bv) {
                    bv = p[e];
                    bi = e;
                }
            }
            tb[i] = bi;
            wb[i] = bv;
        }
        if (norm_topk_prob) {
            float ssum = 0.0f;
            for (int i = 0; i < k; i++) ssum = ssum + wb[i];
            for (int i = 0; i < k; i++) wb[i] = wb[i] / ssum;
        }
        if (probs) memcpy(probs + (size_t)b * E, p, sizeof(float) * (size_t)E);
    }
    free(p);
}

/* decode_kernel.c:1449-1485: experts in first-appearance order over the
 * slots s = b*k + i; per expert, its slots in increasing s order. */
int jo_dispatch(const int* top, const float* tw, int B, int k, int E,
                int* sel, int* uh, int* uidx, float* uw) {
    int* upos = (int*)malloc(sizeof(int) * (size_t)E);
    int* cnt = (int*)calloc((size_t)E + 1, sizeof(int));
    for (int e = 0; e < E; e++) upos[e] = -1;
    int U = 0;
    for (int s = 0; s < B * k; s++) {
        const int e = top[s];
        if (upos[e] < 0 && U < E) {
            upos[e] = U;
            sel[U++] = e;
        }
    }
    for (int s = 0; s < B * k; s++) cnt[upos[top[s]]]++;
    int acc = 0;
    for (int u = 0; u < U; u++) {
        uh[u] = acc;
        acc += cnt[u];
    }
    uh[U] = acc;
    for (int u = 0; u < U; u++) cnt[u] = uh[u];
    for (int s = 0; s < B * k; s++) {
        const int u = upos[top[s]];
        uidx[cnt[u]] = s;
        uw[cnt[u]] = tw[s];
        cnt[u]++;
    }
    free(upos);
    free(cnt);
    return U;
}

static inline float silu_mul(float g, float u) {
    const float den = 1.0f + jo_expf_fast(-g);
    const float sg = g / den;
    return sg * u;
}

/* One expert row against one activation row: the Q4 row dot
 * (decode_kernel.c:770-858) or, for the bf16 tier, bf16_row_dot_B
 * (decode_kernel.c:934-963), whose 8 FMA lanes + hsum8 + scalar tail are the
 * order of jo_router_logits. */
static float expert_row_dot(int bf16, const void* w, const uint16_t* sc, int row, int ncols,
                            const float* x) {
    float acc;
    if (bf16) {
        jo_router_logits((const uint16_t*)w + (size_t)row * ncols, x, 1, 1, ncols, &acc);
    } else {
        jo_q4_row_dot_B((const uint8_t*)w + (size_t)row * (ncols / 2), sc + (size_t)row * (ncols / 64),
                        x, 1, ncols, ncols, &acc);
    }
    return acc;
}

static void moe_layer(int bf16, int d, int E, int k, int m, int norm_topk_prob,
                      const uint16_t* gate_w, const void* const* pk,
                      const uint16_t* const* sc, const float* x, int B,
                      float* out, int* top_out, float* tw_out) {
    const int S = B * k;
    float* logits = (float*)malloc(sizeof(float) * (size_t)B * E);
    int* top = (int*)malloc(sizeof(int) * (size_t)S);
    float* tw = (float*)malloc(sizeof(float) * (size_t)S);
    int* sel = (int*)malloc(sizeof(int) * (size_t)E);
    int* uh = (int*)malloc(sizeof(int) * ((size_t)E + 1));
    int* uidx = (int*)malloc(sizeof(int) * (size_t)S);
    float* uw = (float*)malloc(sizeof(float) * (size_t)S);
    float* act = (float*)malloc(sizeof(float) * (size_t)m);
    float* y = (float*)malloc(sizeof(float) * (size_t)S * d); /* per slot */
    int* slot_u = (int*)malloc(sizeof(int) * (size_t)S);      /* slot -> union pos */

    jo_router_logits(gate_w, x, B, E, d, logits);
    jo_route(logits, B, E, k, norm_topk_prob, top, tw, NULL);
    const int U = jo_dispatch(top, tw, B, k, E, sel, uh, uidx, uw);

    /* ffn_expert_worker, Q4 branch (decode_kernel.c:1365-1384) and bf16
     * branch (1276-1301): for each union expert and each of its slots
     * (token b = slot / k), the gate and up rows give act = silu(g) * u, then
     * down rows give y = w * dacc (the reference's `ye += uw * dacc` onto a
     * zeroed ye). */
    for (int u = 0; u < U; u++) {
        const int e = sel[u];
        const void* pkg = pk[0 * E + e];
        const void* pku = pk[1 * E + e];
        const void* pkd = pk[2 * E + e];
        const uint16_t* scg = bf16 ? NULL : sc[0 * E + e];
        const uint16_t* scu = bf16 ? NULL : sc[1 * E + e];
        const uint16_t* scd = bf16 ? NULL : sc[2 * E + e];
        for (int s = uh[u]; s < uh[u + 1]; s++) {
            const int slot = uidx[s];
            const int b = slot / k;
            const float* xb = x + (size_t)b * d;
            slot_u[slot] = u;
            for (int i = 0; i < m; i++) {
                const float g = expert_row_dot(bf16, pkg, scg, i, d, xb);
                const float up = expert_row_dot(bf16, pku, scu, i, d, xb);
                act[i] = silu_mul(g, up);
            }
            float* ys = y + (size_t)slot * d;
            for (int i = 0; i < d; i++) {
                const float dacc = expert_row_dot(bf16, pkd, scd, i, m, act);
                const float t = uw[s] * dacc;
                ys[i] = 0.0f + t;
            }
        }
    }
    /* combine (decode_kernel.c:1490-1507): out[b] = 0, then += y of every
     * union expert in union order; experts b did not choose add +0. */
    for (int b = 0; b < B; b++) {
        int pos[64]; /* union position -> slot of b, or -1 */
        float* ob = out + (size_t)b * d;
        for (int i = 0; i < d; i++) ob[i] = 0.0f;
        for (int u0 = 0; u0 < U; u0 += 64) {
            const int n = (U - u0 < 64) ? U - u0 : 64;
            for (int j = 0; j < n; j++) pos[j] = -1;
            for (int i = 0; i < k; i++) {
                const int slot = b * k + i;
                const int u = slot_u[slot];
                if (u >= u0 && u < u0 + n) pos[u - u0] = slot;
            }
            for (int j = 0; j < n; j++) {
                if (pos[j] < 0) {
                    for (int i = 0; i < d; i++) ob[i] = ob[i] + 0.0f;
                } else {
                    const float* ys = y + (size_t)pos[j] * d;
                    for (int i = 0; i < d; i++) ob[i] = ob[i] + ys[i];
                }
            }
        }
    }
    if (top_out) memcpy(top_out, top, sizeof(int) * (size_t)S);
    if (tw_out) memcpy(tw_out, tw, sizeof(float) * (size_t)S);
    free(logits);
    free(top);
    free(tw);
    free(sel);
    free(uh);
    free(uidx);
    free(uw);
    free(act);
    free(y);
    free(slot_u);
}

void jo_moe_layer(int d, int E, int k, int m, int norm_topk_prob,
                  const uint16_t* gate_w, const uint8_t* const* pk,
                  const uint16_t* const* sc, const float* x, int B,
                  float* out, int* top_out, float* tw_out) {
    moe_layer(0, d, E, k, m, norm_topk_prob, gate_w, (const void* const*)pk, sc, x, B, out,
              top_out, tw_out);
}

void jo_moe_layer_bf16(int d, int E, int k, int m, int norm_topk_prob,
                       const uint16_t* gate_w, const uint16_t* const* bw, const float* x, int B,
                       float* out, int* top_out, float* tw_out) {
    moe_layer(1, d, E, k, m, norm_topk_prob, gate_w, (const void* const*)bw, NULL, x, B, out,
              top_out, tw_out);
}

/* ------------------------------------------------------------------------
 * The rest of the decode step (attention, norms, lm_head) for the greedy
 * parity pin of a full decode step. Same rounding rules as above: every
 * scalar product and sum rounds on its own (-ffp-contract=off), the AVX2
 * dot products are 8 fmaf lanes plus hsum8.
 * ------------------------------------------------------------------------ */

/* decode_kernel.c:88-93: halve the exponent for a first estimate, then one
 * Newton step y' = (y + x / y) / 2. */
float jo_sqrtf_fast(float x) {
    bits32 v;
    v.f = x;
    v.u = (v.u + 0x3F800000u) >> 1;
    const float q = x / v.f;
    const float s = v.f + q;
    return 0.5f * s;
}

/* decode_kernel.c:224-230: sum of squares in index order, one reciprocal of
 * the root, then (x * inv) * w per element. */
void jo_rms_norm(float* out, const float* x, const uint16_t* w, int d, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < d; i++) {
        const float sq = x[i] * x[i];
        ss = ss + sq;
    }
    const float mean = ss / (float)d;
    const float inv = 1.0f / jo_sqrtf_fast(mean + eps);
    for (int i = 0; i < d; i++) {
        const float t = x[i] * inv;
        out[i] = t * jo_bf16_to_f32(w[i]);
    }
}

/* decode_kernel.c:259-266: rotate-half RoPE with the first hd/2 entries of
 * the position's cos / sin rows. */
void jo_rope(float* q, const float* cs, const float* sn, int hd) {
    const int h = hd / 2;
    for (int i = 0; i < h; i++) {
        const float a = q[i], b = q[i + h];
        const float ac = a * cs[i], bs = b * sn[i], as = a * sn[i], bc = b * cs[i];
        q[i] = ac - bs;
        q[i + h] = as + bc;
    }
}

/* decode_kernel.c:969-995 (lm_B_worker) and 1021-1047 (lm_A_worker): an fp32
 * weight row against B rows, 8 fmaf lanes + hsum8, scalar tail. */
void jo_matvec_f32w(const float* W, const float* x, int B, int n, int d, float* out) {
    for (int b = 0; b < B; b++) {
        const float* xb = x + (size_t)b * d;
        for (int i = 0; i < n; i++) {
            const float* row = W + (size_t)i * d;
            float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int k = 0;
            for (; k + 8 <= d; k += 8)
                for (int j = 0; j < 8; j++) lane[j] = fmaf(row[k + j], xb[k + j], lane[j]);
            float acc = hsum8(lane);
            for (; k < d; k++) {
                const float t = row[k] * xb[k];
                acc = acc + t;
            }
            out[(size_t)b * n + i] = acc;
        }
    }
}

/* Root-mean-square norm of a vector in place with bf16 weights, the QK-norm
 * form of decode_kernel.c:1155-1189 (n = H*hd whole-vector, or hd per head). */
static void qk_norm(float* v, const uint16_t* w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) {
        const float sq = v[i] * v[i];
        ss = ss + sq;
    }
    const float mean = ss / (float)n;
    const float inv = 1.0f / jo_sqrtf_fast(mean + eps);
    for (int i = 0; i < n; i++) {
        const float t = v[i] * inv;
        v[i] = t * jo_bf16_to_f32(w[i]);
    }
}

/* layer_attn_batch (decode_kernel.c:1120-1234), bf16 projections: q/k/v,
 * optional bias, QK-norm (1 = per head, 2 = whole vector), RoPE, append to
 * the KV cache, softmax attention over positions 0..pos, o_proj. */
static void attn_layer(const jo_decoder* M, int l, float* const* kc, float* const* vc,
                       const int* positions, const float* x, int B, float* out) {
    const int d = M->d, H = M->H, KH = M->KH, hd = M->hd;
    const int qn = H * hd, kn = KH * hd;
    float* q = (float*)malloc(sizeof(float) * (size_t)B * qn);
    float* kx = (float*)malloc(sizeof(float) * (size_t)B * kn);
    float* vx = (float*)malloc(sizeof(float) * (size_t)B * kn);
    float* att = (float*)malloc(sizeof(float) * (size_t)B * qn);
    float* sc = (float*)malloc(sizeof(float) * (size_t)M->maxT);
    jo_router_logits(M->wq + (size_t)l * qn * d, x, B, qn, d, q);
    jo_router_logits(M->wk + (size_t)l * kn * d, x, B, kn, d, kx);
    jo_router_logits(M->wv + (size_t)l * kn * d, x, B, kn, d, vx);
    if (M->bias_qkv)
        for (int b = 0; b < B; b++) {
            for (int i = 0; i < qn; i++) q[(size_t)b * qn + i] += M->bq[(size_t)l * qn + i];
            for (int i = 0; i < kn; i++) {
                kx[(size_t)b * kn + i] += M->bk[(size_t)l * kn + i];
                vx[(size_t)b * kn + i] += M->bv[(size_t)l * kn + i];
            }
        }
    if (M->qk_norm_type == 2)
        for (int b = 0; b < B; b++) {
            qk_norm(q + (size_t)b * qn, M->qn + (size_t)l * qn, qn, M->eps);
            qk_norm(kx + (size_t)b * kn, M->kn + (size_t)l * kn, kn, M->eps);
        }
    for (int b = 0; b < B; b++) {
        float* qb = q + (size_t)b * qn;
        float* kb = kx + (size_t)b * kn;
        const float* vb = vx + (size_t)b * kn;
        if (M->qk_norm_type == 1) {
            for (int h = 0; h < H; h++) qk_norm(qb + (size_t)h * hd, M->qn + (size_t)l * hd, hd, M->eps);
            for (int h = 0; h < KH; h++) qk_norm(kb + (size_t)h * hd, M->kn + (size_t)l * hd, hd, M->eps);
        }
        const int pos = positions[b];
        const float* cs = M->cos + (size_t)pos * hd;
        const float* sn = M->sin + (size_t)pos * hd;
        for (int h = 0; h < H; h++) jo_rope(qb + (size_t)h * hd, cs, sn, hd);
        for (int h = 0; h < KH; h++) jo_rope(kb + (size_t)h * hd, cs, sn, hd);
        float* K = kc[(size_t)b * M->L + l];
        float* V = vc[(size_t)b * M->L + l];
        memcpy(K + (size_t)pos * kn, kb, sizeof(float) * (size_t)kn);
        memcpy(V + (size_t)pos * kn, vb, sizeof(float) * (size_t)kn);
        const int T = pos + 1;
        const float scale = jo_sqrtf_fast((float)hd);
        for (int h = 0; h < H; h++) {
            const float* qh = qb + (size_t)h * hd;
            const int g = h / (H / KH);
            float smax = -1e30f;
            for (int t = 0; t < T; t++) {
                const float* kt = K + (size_t)t * kn + (size_t)g * hd;
                float s = 0.0f;
                for (int i = 0; i < hd; i++) {
                    const float p = qh[i] * kt[i];
                    s = s + p;
                }
                sc[t] = s / scale;
                if (sc[t] > smax) smax = sc[t];
            }
            float sum = 0.0f;
            for (int t = 0; t < T; t++) {
                sc[t] = jo_expf_fast(sc[t] - smax);
                sum = sum + sc[t];
            }
            float* oh = att + (size_t)b * qn + (size_t)h * hd;
            for (int i = 0; i < hd; i++) oh[i] = 0.0f;
            for (int t = 0; t < T; t++) {
                const float* vt = V + (size_t)t * kn + (size_t)g * hd;
                const float p = sc[t] / sum;
                for (int i = 0; i < hd; i++) {
                    const float pv = p * vt[i];
                    oh[i] = oh[i] + pv;
                }
            }
        }
    }
    jo_router_logits(M->wo + (size_t)l * d * qn, att, B, d, qn, out);
    free(q);
    free(kx);
    free(vx);
    free(att);
    free(sc);
}

/* decode_layers_batch / decode_layers_batch_argmax (decode_kernel.c:1518-1586)
 * on the Q4 MoE layers: per layer h += attn(norm1(h)), h += moe(norm2(h));
 * then the final norm and the fp32 lm_head. */
void jo_decode_step(const jo_decoder* M, float* const* kc, float* const* vc, const int* positions,
                    const float* x, int B, int* out_tok, float* logits) {
    const int d = M->d, E = M->E;
    float* h = (float*)malloc(sizeof(float) * (size_t)B * d);
    float* t = (float*)malloc(sizeof(float) * (size_t)B * d);
    float* h2 = (float*)malloc(sizeof(float) * (size_t)B * d);
    float* lg = (float*)malloc(sizeof(float) * (size_t)B * M->V);
    memcpy(h, x, sizeof(float) * (size_t)B * d);
    for (int l = 0; l < M->L; l++) {
        for (int b = 0; b < B; b++)
            jo_rms_norm(t + (size_t)b * d, h + (size_t)b * d, M->norm1 + (size_t)l * d, d, M->eps);
        attn_layer(M, l, kc, vc, positions, t, B, h2);
        for (size_t i = 0; i < (size_t)B * d; i++) h[i] = h[i] + h2[i];
        for (int b = 0; b < B; b++)
            jo_rms_norm(t + (size_t)b * d, h + (size_t)b * d, M->norm2 + (size_t)l * d, d, M->eps);
        jo_moe_layer(d, E, M->k, M->m, M->norm_topk_prob, M->gate_w + (size_t)l * E * d,
                     M->pk + (size_t)l * 3 * E, M->sc + (size_t)l * 3 * E, t, B, h2, NULL, NULL);
        for (size_t i = 0; i < (size_t)B * d; i++) h[i] = h[i] + h2[i];
    }
    for (int b = 0; b < B; b++)
        jo_rms_norm(t + (size_t)b * d, h + (size_t)b * d, M->final_norm, d, M->eps);
    jo_matvec_f32w(M->lm_head, t, B, M->V, d, lg);
    for (int b = 0; b < B; b++) {
        const float* r = lg + (size_t)b * M->V;
        int best = 0;
        float bv = -1e30f;
        for (int v = 0; v < M->V; v++)
            if (r[v] > bv) {
                bv = r[v];
                best = v;
            }
        if (out_tok) out_tok[b] = best;
    }
    if (logits) memcpy(logits, lg, sizeof(float) * (size_t)B * M->V);
    free(h);
    free(t);
    free(h2);
    free(lg);
}
