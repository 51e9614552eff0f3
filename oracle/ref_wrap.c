/* Wrapper translation unit that compiles the reference's UNMODIFIED
 * src/jouleai/native/decode_kernel.c (pulled in by #include from the
 * reference tree; nothing is copied) and exports its static MoE FFN entry
 * so the CPU oracle and the CPU baseline can call it directly.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline).
 *
 * Exports:
 *   oracle_ffn_batch      -> layer_ffn_batch      (decode_kernel.c:1387-1508)
 *   oracle_ffn_debug      -> layer_ffn_batch, then a copy of the routing and
 *                            union state it left in the global workspace
 *                            (g_ws: top/tw/sel/uh/uidx/uw, decode_kernel.c:344-356)
 *   oracle_router_logits  -> matvec_f32_B         (decode_kernel.c:720-725)
 *   oracle_q4_row_dot_B   -> q4_row_dot_B         (decode_kernel.c:770-858)
 *   oracle_expf_fast      -> expf_fast            (decode_kernel.c:94-108)
 *   oracle_fp16_to_f32    -> fp16_to_f32          (decode_kernel.c:64-85)
 */
#include "decode_kernel.c"

void oracle_ffn_batch(const KernelCfg* c, const KernelW* W, int l,
                      const float* x, int B, float* out) {
    layer_ffn_batch(c, W, l, x, B, out);
}

/* Same call; afterwards copies the routing/union arrays. `U` receives the
 * union size. Buffers: top/tw [B*topk], sel [E], uh [E+1], uidx/uw [B*topk]. */
void oracle_ffn_debug(const KernelCfg* c, const KernelW* W, int l,
                      const float* x, int B, float* out, int* top, float* tw,
                      int* sel, int* uh, int* uidx, float* uw, int* U) {
    layer_ffn_batch(c, W, l, x, B, out);
    const int k = c->topk, E = c->E;
    int u = 0;
    /* the union size is uh's last non-decreasing index: recount from top */
    {
        int seen[1024];
        for (int e = 0; e < E && e < 1024; e++) seen[e] = 0;
        for (int s = 0; s < B * k; s++) {
            int e = g_ws.top[s];
            if (e >= 0 && e < E && !seen[e]) { seen[e] = 1; u++; }
        }
    }
    *U = u;
    for (int s = 0; s < B * k; s++) {
        top[s] = g_ws.top[s];
        tw[s] = g_ws.tw[s];
        uidx[s] = g_ws.uidx[s];
        uw[s] = g_ws.uw[s];
    }
    for (int i = 0; i < u; i++) sel[i] = g_ws.sel[i];
    for (int i = 0; i <= u; i++) uh[i] = g_ws.uh[i];
}

void oracle_router_logits(const KernelCfg* c, const KernelW* W, int l,
                          const float* x, int B, float* scores) {
    matvec_f32_B(scores, W->gate_w + (size_t)l * c->E * c->d, x, c->E, c->d, B);
}

void oracle_q4_row_dot_B(const unsigned char* row, const unsigned short* sc,
                         const float* x, int B, float* acc, int ncols,
                         int stride) {
    q4_row_dot_B(row, sc, x, B, acc, ncols >> 1, 32, ncols / 64, stride);
}

float oracle_expf_fast(float v) { return expf_fast(v); }

float oracle_fp16_to_f32(unsigned short h) { return fp16_to_f32(h); }
