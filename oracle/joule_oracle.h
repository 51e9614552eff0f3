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

#ifdef __cplusplus
}
#endif
#endif
