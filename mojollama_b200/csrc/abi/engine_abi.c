/* Reference-named entry points of the "engine" set (combined_engine.so,
 * quant_kernels_omp.so, cengine_batch_instr.so).  Each forwards to the mlq_* core
 * in libmojollama_b200.so; see include/mojollama_b200_ref_abi.h for the reference
 * definition each one replaces. */
#include <stddef.h>
#include <stdint.h>

#include "mojollama_b200.h"
#include "mojollama_b200_ref_abi.h"

void quant_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols, int quant_type) {
    mlq_matmul(W, quant_type, x, out, n_rows, n_cols, 1);
}

void f32_matmul_omp(const float *W, const float *x, float *out, int n_rows, int n_cols) {
    mlq_matmul(W, MLQ_F32, x, out, n_rows, n_cols, 1);
}

#define MLQ_GEMV1(name, qt) \
    void name(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols) { \
        mlq_matmul(W, qt, x, out, n_rows, n_cols, 1); \
    }
MLQ_GEMV1(q4_0_matmul_omp, MLQ_Q4_0)
MLQ_GEMV1(q4_1_matmul_omp, MLQ_Q4_1)
MLQ_GEMV1(q5_0_matmul_omp, MLQ_Q5_0)
MLQ_GEMV1(q8_0_matmul_omp, MLQ_Q8_0)
MLQ_GEMV1(q4_k_matmul_omp, MLQ_Q4_K)
MLQ_GEMV1(q5_k_matmul_omp, MLQ_Q5_K)
MLQ_GEMV1(q6_k_matmul_omp, MLQ_Q6_K)
MLQ_GEMV1(mxfp4_matmul_omp, MLQ_MXFP4)

#define MLQ_GEMVB(name, qt) \
    void name(const uint8_t *W, const float *x, float *out, int n_rows, int nc, int B) { \
        mlq_matmul(W, qt, x, out, n_rows, nc, B); \
    }
MLQ_GEMVB(q4_0_batch_matmul, MLQ_Q4_0)
MLQ_GEMVB(q8_0_batch_matmul, MLQ_Q8_0)
MLQ_GEMVB(q4_k_batch_matmul, MLQ_Q4_K)
MLQ_GEMVB(q5_k_batch_matmul, MLQ_Q5_K)
MLQ_GEMVB(q6_k_batch_matmul, MLQ_Q6_K)
MLQ_GEMVB(mxfp4_batch_matmul, MLQ_MXFP4)

void q8_0_q8_0_matmul_omp(const uint8_t *W, const uint8_t *x_q8, float *out, int n_rows, int n_cols, int B) {
    mlq_matmul_q8act(W, MLQ_Q8_0, x_q8, out, n_rows, n_cols, B);
}
void q4_0_q8_0_matmul_omp(const uint8_t *W, const uint8_t *x_q8, float *out, int n_rows, int n_cols,
                          int n_blocks_x) {
    (void)n_blocks_x;
    mlq_matmul_q8act(W, MLQ_Q4_0, x_q8, out, n_rows, n_cols, 1);
}
void q5_0_q8_0_matmul_omp(const uint8_t *W, const uint8_t *x_q8, float *out, int n_rows, int n_cols, int B) {
    mlq_matmul_q8act(W, MLQ_Q5_0, x_q8, out, n_rows, n_cols, B);
}
void q4_k_q8_0_matmul_omp(const uint8_t *W, const uint8_t *x_q8, float *out, int n_rows, int n_cols) {
    mlq_matmul_q8act(W, MLQ_Q4_K, x_q8, out, n_rows, n_cols, 1);
}

int quantize_row_q8_0(const float *x, uint8_t *q8, int n_cols) {
    mlq_quantize_q8_0(x, q8, n_cols);
    return n_cols / 32;
}

void q6_k_dequantize_row(const uint8_t *W, float *out, int n) { mlq_dequantize(W, MLQ_Q6_K, out, n); }
void q4_k_dequantize_row(const uint8_t *W, float *out, int n) { mlq_dequantize(W, MLQ_Q4_K, out, n); }
void q5_k_dequantize_row(const uint8_t *W, float *out, int n) { mlq_dequantize(W, MLQ_Q5_K, out, n); }
void q8_0_dequantize_row(const uint8_t *W, float *out, int n) { mlq_dequantize(W, MLQ_Q8_0, out, n); }

void batch_qkv_omp(const uint8_t *Wq, const uint8_t *Wk, const uint8_t *Wv, const float *x,
                   float *out_q, float *out_k, float *out_v, int nq, int nk, int nv, int n_cols,
                   int qtype_q, int qtype_k, int qtype_v) {
    mlq_matmul(Wq, qtype_q, x, out_q, nq, n_cols, 1);
    mlq_matmul(Wk, qtype_k, x, out_k, nk, n_cols, 1);
    mlq_matmul(Wv, qtype_v, x, out_v, nv, n_cols, 1);
}

void batch_gate_up_omp(const uint8_t *Wg, const uint8_t *Wu, const float *x, float *out_gate, float *out_up,
                       int ng, int nu, int n_cols, int qtype_g, int qtype_u) {
    mlq_matmul(Wg, qtype_g, x, out_gate, ng, n_cols, 1);
    mlq_matmul(Wu, qtype_u, x, out_up, nu, n_cols, 1);
}

void batch_matmul(const uint8_t *w[7], const float *x, float *out[7], int nrows[7], int ncols[7], int ts[7],
                  int n_proj) {
    for (int p = 0; p < n_proj && p < 7; p++)
        mlq_matmul(w[p], ts[p] == 20 ? MLQ_Q4_1 : MLQ_Q4_0, x, out[p], nrows[p], ncols[p], 1);
}

int get_max_threads(void) { return 1; }
void set_num_threads(int n) { (void)n; }

void rms_norm(const float *x, const float *weight, float *out, int n) {
    mlq_rms_norm(out, x, weight, 1, n, 1e-5f, 0, NULL);
}
void silu(float *x, int n) { mlq_silu(x, x, n, 0); }
void softmax(float *x, int n) { mlq_softmax(x, 1, n); }
void silu_omp(float *x, int n) { mlq_silu(x, x, n, 0); }
void rope_init(float *cos_table, float *sin_table, int max_ctx, int hd, int rope_dim) {
    /* the reference uses 10000^(2j/hd) with hd (not rope_dim) in the exponent */
    mlq_rope_init(cos_table, sin_table, max_ctx, hd, rope_dim, 10000.0);
}

/* PagedAttention (cengine_batch_instr.c:173-214) */
void page_table_init(PageTable *pt, int max_pages, int page_size, int nkh, int hd, int n_layers) {
    mlq_page_table_init(pt, max_pages, page_size, nkh, hd, n_layers);
}
int page_table_alloc(PageTable *pt) { return mlq_page_table_alloc(pt); }
void page_table_free(PageTable *pt, int page_id) { mlq_page_table_free(pt, page_id); }
void map_page(PageTable *pt, int logical_page, int physical_page) { mlq_map_page(pt, logical_page, physical_page); }
void kv_init(KVBlock *kv, int L, int NKH, int HD) { mlq_kv_init(kv, L, NKH, HD); }
int kv_alloc(KVBlock *kv) { return mlq_kv_alloc(kv); }

/* cengine_batch_instr.c:141 (static there): flat KV [sl][nkh*hd] */
void gqa(float *o, const float *q, const float *kc, const float *vc, int sl, int nh, int nkh, int hd) {
    mlq_attn_decode_flat(q, kc, vc, o, sl, nh, nkh, hd, 0);
}

/* quant_kernels_omp.c:2066; prealloc_buf / prealloc_q8 are not needed (the expert
   intermediates stay in device scratch) */
void moe_forward_omp(const uint8_t **gate_raw, const uint8_t **up_raw, const uint8_t **down_raw, const float *x_norm,
                     int n_ff_expert, int n_embd, int qt_gate, int qt_up, int qt_down, const int *top_indices,
                     const float *top_weights, int top_k, float *combined, float *prealloc_buf,
                     uint8_t *prealloc_q8) {
    (void)prealloc_buf;
    (void)prealloc_q8;
    mlq_moe_forward((const void *const *)gate_raw, (const void *const *)up_raw, (const void *const *)down_raw, x_norm,
                    n_ff_expert, n_embd, qt_gate, qt_up, qt_down, top_indices, top_weights, top_k, combined);
}

/* cengine_batch_instr.c:736, 803 */
void ssm_decode_step(const float *x, float *ssm_intermediate, const float *conv1d_w, const float *a_param,
                     const float *dt_bias, const float *alpha, const float *beta, const float *ssm_norm_w,
                     float *state, int B, int N, int inner, int groups, int state_size, int conv_kernel,
                     int dt_rank) {
    mlq_ssm_decode_step(x, ssm_intermediate, conv1d_w, a_param, dt_bias, alpha, beta, ssm_norm_w, state, B, N, inner,
                        groups, state_size, conv_kernel, dt_rank);
}
void ssm_layer_fused(const float *x, float *residual, float *output, const float *conv1d_w, const float *a_param,
                     const float *dt_bias, const float *alpha, const float *beta, const float *ssm_norm_w,
                     float *state, const uint8_t *gate_raw, int gate_nr, int gate_nc, int gate_qt,
                     const uint8_t *ssm_out_raw, int ssm_out_nr, int ssm_out_nc, int ssm_out_qt, int B, int N,
                     int inner, int groups, int state_size, int conv_kernel, int dt_rank) {
    mlq_ssm_layer_fused(x, residual, output, conv1d_w, a_param, dt_bias, alpha, beta, ssm_norm_w, state, gate_raw,
                        gate_nr, gate_nc, gate_qt, ssm_out_raw, ssm_out_nr, ssm_out_nc, ssm_out_qt, B, N, inner,
                        groups, state_size, conv_kernel, dt_rank);
}

/* cengine_batch_instr.c:1233: one decode step for B sequences (see mlq_batch_forward) */
void batch_forward(const BC *c, const int *tokens, int B, float *ws) { mlq_batch_forward(c, tokens, B, ws); }

/* cengine_batch_instr.c:591: gate_buf / up_buf are not needed */
void moe_ffn(const BC *c, int l, float *x, float *gate_buf, float *up_buf, float *ffn_buf, int B) {
    (void)gate_buf;
    (void)up_buf;
    mlq_moe_ffn(c, l, x, ffn_buf, B);
}

/* cengine_batch_instr.c:859: the 76 arguments, in order, into MlqQwen36Args */
void qwen36_batch_forward(
    int B, int L, int N, int NH, int n_kv_h, int HD, int FF, int n_experts, int top_k, int n_ff_expert, float eps,
    int rope_dim, int max_ctx, int ssm_inner, int ssm_groups, int ssm_state_size, int ssm_conv_kernel,
    int ssm_dt_rank, const float *emb, int emb_quant, const int *layer_types, const int *tokens, float *logits,
    const float **attn_norm_w, const float **ffn_norm_w, const uint8_t **attn_qkv_raw, const int *qkv_nr,
    const int *qkv_nc, const int *qkv_qt, const uint8_t **attn_gate_raw, const int *gate_nr, const int *gate_nc,
    const int *gate_qt, const uint8_t **ssm_out_raw, const int *ssm_out_nr, const int *ssm_out_nc,
    const int *ssm_out_qt, const uint8_t **attn_out_raw, const int *out_nr, const int *out_nc, const int *out_qt,
    uint8_t **gate_exp_raw, const int *gate_exp_qt, uint8_t **up_exp_raw, const int *up_exp_qt,
    uint8_t **down_exp_raw, const int *down_exp_qt, const float **shexp_gate_raw, const float **shexp_up_raw,
    const float **shexp_down_raw, const float **shexp_router, const int *shexp_int, const uint8_t **moe_router_raw,
    const int *moe_router_qt, const int *shexp_gate_qt, const int *shexp_up_qt, const int *shexp_down_qt,
    const float *out_norm_w, const uint8_t *out_w, int out_nr_final, int out_nc_final, int out_qt_final,
    const float **ssm_conv1d, const float **ssm_a, const float **ssm_dt_bias, const float **ssm_alpha,
    const float **ssm_beta, const float **ssm_norm, float *ssm_state, float *kv_k, float *kv_v, int *kv_lens,
    const float *cos_table, const float *sin_table, float *ws, uint8_t *q8_ws) {
    MlqQwen36Args a = {
        B, L, N, NH, n_kv_h, HD, FF, n_experts, top_k, n_ff_expert, eps,
        rope_dim, max_ctx, ssm_inner, ssm_groups, ssm_state_size, ssm_conv_kernel, ssm_dt_rank,
        emb, emb_quant, layer_types, tokens, logits,
        attn_norm_w, ffn_norm_w,
        attn_qkv_raw, qkv_nr, qkv_nc, qkv_qt,
        attn_gate_raw, gate_nr, gate_nc, gate_qt,
        ssm_out_raw, ssm_out_nr, ssm_out_nc, ssm_out_qt,
        attn_out_raw, out_nr, out_nc, out_qt,
        gate_exp_raw, gate_exp_qt, up_exp_raw, up_exp_qt, down_exp_raw, down_exp_qt,
        shexp_gate_raw, shexp_up_raw, shexp_down_raw, shexp_router, shexp_int,
        moe_router_raw, moe_router_qt, shexp_gate_qt, shexp_up_qt, shexp_down_qt,
        out_norm_w, out_w, out_nr_final, out_nc_final, out_qt_final,
        ssm_conv1d, ssm_a, ssm_dt_bias, ssm_alpha, ssm_beta, ssm_norm, ssm_state,
        kv_k, kv_v, kv_lens, cos_table, sin_table, ws, q8_ws};
    mlq_qwen36_batch_forward(&a);
}
