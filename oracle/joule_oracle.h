/* CPU restatement of the reference's MoE decode hot path (Q4 experts).
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker that the CUDA product is
 * compared against; the product never links, loads or calls it. Every
 * function cites the reference file:line whose arithmetic it restates
 * (paths are relative to the reference project root).
 *
 * Pinned against the reference itself: the reference C sources compiled
 * unmodified into _ref/ (see Makefile) produce the golden fixtures under
 * tests/golden/, and tests check this restatement against them bit for bit.
 */
#ifndef JOULE_ORACLE_H
#define JOULE_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* decode_kernel.c:64-85 */
float jo_fp16_to_f32(uint16_t h);
/* decode_kernel.c:47-53 */
float jo_bf16_to_f32(uint16_t h);
/* decode_kernel.c:94-108 */
float jo_expf_fast(float v);

/* One Q4 row (ncols values, group 64, fp16 scales) against B activation
 * rows of stride `stride`: decode_kernel.c:770-858 (AVX2 branch). */
void jo_q4_row_dot_B(const uint8_t* row, const uint16_t* sc, const float* x,
                     int B, int stride, int ncols, float* acc);

/* out[T, m] = X[T, d] @ dequant(W[m, d])^T: expert_ffn.c:200-215 with the
 * AVX2 row dot (expert_ffn.c:59-130, same order as decode_kernel.c:114-145). */
void jo_q4_gemm(float* out, const float* X, int T, const uint8_t* packed,
                const uint16_t* scales, int m, int d);

/* out[m] = dequant(W[m, d]) @ x[d] in quant_gemv.c:35-57's scalar order. */
void jo_q4_gemv_scalar(float* out, const float* x, const uint8_t* packed,
                       const uint16_t* scales, int m, int d);

/* scores[B, E] = bf16 gate[E, d] @ x[B, d]^T: decode_kernel.c:234-256 and
 * 693-718 (identical lane order for B == 1 and B > 1). */
void jo_router_logits(const uint16_t* gate_w, const float* x, int B, int E,
                      int d, float* scores);

/* softmax / top-k / optional renorm: decode_kernel.c:1425-1448.
 * probs (nullable) receives the normalised softmax [B, E]. */
void jo_route(const float* logits, int B, int E, int k, int norm_topk_prob,
              int* top, float* tw, float* probs);

/* union of experts + slot map: decode_kernel.c:1449-1485. Returns U. */
int jo_dispatch(const int* top, const float* tw, int B, int k, int E,
                int* sel, int* uh, int* uidx, float* uw);

/* One MoE FFN layer (layer_ffn_batch, decode_kernel.c:1387-1508, Q4 branch
 * of ffn_expert_worker 1365-1384).
 *   gate_w : [E, d] bf16 router rows of this layer
 *   pk, sc : 3*E pointers, index p*E + e, p in (gate, up, down): the Q4
 *            record of that part (packed u8 / fp16 scales), reference layout
 *   x      : [B, d]; out: [B, d]
 *   top/tw : optional [B, k] outputs (nullable) */
void jo_moe_layer(int d, int E, int k, int m, int norm_topk_prob,
                  const uint16_t* gate_w, const uint8_t* const* pk,
                  const uint16_t* const* sc, const float* x, int B,
                  float* out, int* top, float* tw);

/* The bf16 expert tier of the same layer (decode_kernel.c:1276-1301, taken
 * when KernelCfg.expert_bf16 is set): bw[p*E + e] points at expert e's part p
 * as a bf16 matrix, gate/up [m, d] and down [d, m]; no scales. */
void jo_moe_layer_bf16(int d, int E, int k, int m, int norm_topk_prob,
                       const uint16_t* gate_w, const uint16_t* const* bw, const float* x, int B,
                       float* out, int* top_out, float* tw_out);

/* ---- the rest of the decode step (greedy parity pin) ---- */

/* decode_kernel.c:88-93 */
float jo_sqrtf_fast(float x);
/* decode_kernel.c:224-230: out[d] = rms_norm(x) * bf16 w */
void jo_rms_norm(float* out, const float* x, const uint16_t* w, int d, float eps);
/* decode_kernel.c:259-266: rotate-half RoPE of one head in place */
void jo_rope(float* q, const float* cs, const float* sn, int hd);
/* out[B, n] = fp32 W[n, d] @ x[B, d]^T: decode_kernel.c:969-995, 1021-1047 */
void jo_matvec_f32w(const float* W, const float* x, int B, int n, int d, float* out);

/* A decoder in the reference's weight layout (KernelW, decode_kernel.c:288-325)
 * with Q4 MoE layers. bf16 weights: embed [V, d], norm1/norm2 [L, d],
 * final_norm [d], wq [L, H*hd, d], wk/wv [L, KH*hd, d], wo [L, d, H*hd],
 * qn/kn [L, hd] (qk_norm_type 1) or [L, H*hd] / [L, KH*hd] (type 2),
 * gate_w [L, E, d]. fp32: lm_head [V, d], bq/bk/bv [L, H*hd / KH*hd],
 * cos/sin [maxT, hd]. pk/sc: index (l*3 + p)*E + e, p = gate, up, down. */
typedef struct {
    int L, d, H, KH, hd, E, k, m, V, maxT, qk_norm_type, bias_qkv, norm_topk_prob;
    float eps;
    const uint16_t *embed, *final_norm, *norm1, *norm2, *wq, *wk, *wv, *wo, *qn, *kn, *gate_w;
    const float *lm_head, *bq, *bk, *bv, *cos, *sin;
    const uint8_t* const* pk;
    const uint16_t* const* sc;
} jo_decoder;

/* One batched decode step (decode_layers_batch[_argmax], decode_kernel.c:
 * 1518-1586): x [B, d] embedded inputs at positions[b]; kc/vc: B*L caches
 * kc[b*L + l] = [maxT, KH, hd] fp32 (the reference's kv[b*L + l]), appended
 * at positions[b]. out_tok [B] (argmax, lowest index on ties) and logits
 * [B, V] are nullable. */
void jo_decode_step(const jo_decoder* M, float* const* kc, float* const* vc, const int* positions,
                    const float* x, int B, int* out_tok, float* logits);

#ifdef __cplusplus
}
#endif
#endif
