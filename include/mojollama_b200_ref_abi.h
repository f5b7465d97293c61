/* Reference-named drop-in entry points (C-ABI), exported by the alias libraries in
 * mojollama_b200/lib/: combined_engine.so, quant_kernels_omp.so and
 * cengine_batch_instr.so (the "engine" set below), simd_ops.so and gqa_attention.so.
 *
 * Signatures, argument meaning and buffer layouts are the reference's; each line
 * cites the reference definition it replaces (paths inside a730/MojoLlama).
 * Conventions kept from the reference: void return, caller-owned buffers, host
 * pointers accepted (device pointers too, see mojollama_b200.h), errors leave the
 * outputs untouched (the reference's `default:` case) and are readable through
 * mlq_last_error().  set_num_threads / get_max_threads keep their signatures but
 * have nothing to control on the GPU.
 */
#ifndef MOJOLLAMA_B200_REF_ABI_H
#define MOJOLLAMA_B200_REF_ABI_H

#include <stdint.h>

#include "mojollama_b200.h"

typedef MlqPageTable PageTable;   /* cengine_batch_instr.c:160-171 */
typedef MlqKVBlock KVBlock;       /* cengine_batch_instr.c:204-207 */

/* The batch engine's model description, field for field as cengine_batch_instr.c:536-589
 * defines it (the reference's Python mirrors it with ctypes, forward/zaya_bc.py:32-130),
 * so the same struct bytes drive this build.  Per-layer members are arrays of length L. */
typedef struct {
    int L, N, NH, NKH, HD, FF, V;
    float eps;
    const uint8_t **wQ, **wK, **wV, **wO, **wG, **wU, **wD;
    const float **wAN, **wFN;
    const int *nQ, *nK, *nV, *nO, *nG, *nU, *nD;
    int nc;
    const float *emb, *onw;
    const uint8_t *wOut;
    int outNR, outNC, outQuant;
    KVBlock **kv_array;
    float *logits;
    int n_experts, n_experts_per_tok, moe_intermediate;
    const float **w_gate_inp;
    const uint8_t **w_gate_exps;
    const uint8_t **w_up_exps;
    const uint8_t **w_down_exps;
    int gate_exp_quant, up_exp_quant, down_exp_quant;
    const int *q_quant, *k_quant, *v_quant, *o_quant;
    const int *g_quant, *u_quant, *d_quant;
    int emb_quant;
    const uint8_t **wQK;
    const int *qk_quant;
    float *cos_table;
    float *sin_table;
    int max_ctx;
    float *workspace;
    int ws_size;
    int rope_dim;
    int full_attn_interval;
    const uint8_t **wQKV;
    const int *qkv_quant;
    const uint8_t **wAttnG;
    const int *attnG_quant;
    const float **ssm_conv1d;
    const float **ssm_a;
    const float **ssm_dt_bias;
    const float **ssm_alpha;
    const float **ssm_beta;
    const float **ssm_norm;
    const uint8_t **wSsmOut;
    const int *ssm_out_quant;
    float *ssm_state;
    const uint8_t **wSHexpG, **wSHexpU, **wSHexpD;
    const int *shexp_g_quant, *shexp_u_quant, *shexp_d_quant;
    const float **wShexpRouter;
    const int *layer_types;
    int n_layers_actual;
    const uint8_t **w_zaya_ffn_gate_inp, **w_zaya_ffn_gate, **w_zaya_mlp2, **w_zaya_mlp4;
    const float **w_zaya_router_bias, **w_zaya_ffn_norm;
    const float **w_zaya_res_hs_w, **w_zaya_res_hs_b, **w_zaya_res_res_w, **w_zaya_res_res_b;
    int zaya_ffn_gate_inp_quant, zaya_ffn_gate_quant, zaya_mlp2_quant, zaya_mlp4_quant;
    int *has_moe_layer;
    int zaya_expert_n;
    int zaya_moe_intermediate;
    const uint8_t **w_cca_v1, **w_cca_v2, **w_ssm_conv1d;
    int cca_v1_quant, cca_v2_quant;
} BC;

#ifdef __cplusplus
extern "C" {
#endif

/* The reference ships rms_norm / silu / softmax twice with different signatures
 * (quant_kernels_omp.c vs simd_ops.c, in different .so files), so a translation
 * unit sees one set: define MLQ_REF_ABI_SIMD_OPS for the simd_ops.so signatures. */
#ifndef MLQ_REF_ABI_SIMD_OPS
/* ============================ engine set (combined_engine.so & co.) ============================ */

/* src/mojollama/kernels/quant_kernels_omp.c:1355  dispatch on GGUF type (0,2,3,6,8,12,13,14,39) */
void quant_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols, int quant_type);
/* quant_kernels_omp.c:884 */
void f32_matmul_omp(const float *W, const float *x, float *out, int n_rows, int n_cols);
/* quant_kernels_omp.c:135, 160, 1232-1242, 376, 199, 356, 734, 502 */
void q4_0_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols);
void q4_1_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols);
void q5_0_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols);
void q8_0_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols);
void q4_k_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols);
void q5_k_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols);
void q6_k_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols);
void mxfp4_matmul_omp(const uint8_t *W, const float *x, float *out, int n_rows, int n_cols);
/* cengine_batch_instr.c:68, 216, 256, 316, 381, 435   x [B][nc], out [B][n_rows] */
void q4_0_batch_matmul(const uint8_t *W, const float *x, float *out, int n_rows, int nc, int B);
void q8_0_batch_matmul(const uint8_t *W, const float *x, float *out, int n_rows, int nc, int B);
void q4_k_batch_matmul(const uint8_t *W, const float *x, float *out, int n_rows, int nc, int B);
void q5_k_batch_matmul(const uint8_t *W, const float *x, float *out, int n_rows, int nc, int B);
void q6_k_batch_matmul(const uint8_t *W, const float *x, float *out, int n_rows, int nc, int B);
void mxfp4_batch_matmul(const uint8_t *W, const float *x, float *out, int n_rows, int nc, int B);
/* quant_kernels_omp.c:428, 1524, 1311, 1751   Q8_0-quantized activations */
void q8_0_q8_0_matmul_omp(const uint8_t *W, const uint8_t *x_q8, float *out, int n_rows, int n_cols, int B);
void q4_0_q8_0_matmul_omp(const uint8_t *W, const uint8_t *x_q8, float *out, int n_rows, int n_cols, int n_blocks_x);
void q5_0_q8_0_matmul_omp(const uint8_t *W, const uint8_t *x_q8, float *out, int n_rows, int n_cols, int B);
void q4_k_q8_0_matmul_omp(const uint8_t *W, const uint8_t *x_q8, float *out, int n_rows, int n_cols);
/* quant_kernels_omp.c:1406   returns n_cols/32 */
int quantize_row_q8_0(const float *x, uint8_t *q8, int n_cols);
/* quant_kernels_omp.c:762, 804, 830, 868 */
void q6_k_dequantize_row(const uint8_t *W, float *out, int n_values);
void q4_k_dequantize_row(const uint8_t *W, float *out, int n_values);
void q5_k_dequantize_row(const uint8_t *W, float *out, int n_values);
void q8_0_dequantize_row(const uint8_t *W, float *out, int n_values);
/* quant_kernels_omp.c:1139, 1186   several projections of one activation in one launch set */
void batch_qkv_omp(const uint8_t *Wq, const uint8_t *Wk, const uint8_t *Wv, const float *x,
                   float *out_q, float *out_k, float *out_v, int nq, int nk, int nv, int n_cols,
                   int qtype_q, int qtype_k, int qtype_v);
void batch_gate_up_omp(const uint8_t *Wg, const uint8_t *Wu, const float *x, float *out_gate, float *out_up,
                       int ng, int nu, int n_cols, int qtype_g, int qtype_u);
/* quant_kernels_omp.c:938   Q4_0/Q4_1 (by block size ts[p] = 18 or 20), up to 7 projections */
void batch_matmul(const uint8_t *w[7], const float *x, float *out[7], int nrows[7], int ncols[7], int ts[7],
                  int n_proj);
/* quant_kernels_omp.c:1030-1031 (no threads to set on the GPU; kept for the ABI) */
int get_max_threads(void);
void set_num_threads(int n);
/* quant_kernels_omp.c:956 (eps 1e-5), 981, 1000, 1017 */
void rms_norm(const float *x, const float *weight, float *out, int n);
void silu(float *x, int n);
void softmax(float *x, int n);
void silu_omp(float *x, int n);
/* cengine_batch_instr.c:674 */
void rope_init(float *cos_table, float *sin_table, int max_ctx, int hd, int rope_dim);
/* cengine_batch_instr.c:173, 189, 194, 199, 208, 214 (pages / k / v in device memory here) */
void page_table_init(PageTable *pt, int max_pages, int page_size, int nkh, int hd, int n_layers);
int page_table_alloc(PageTable *pt);
void page_table_free(PageTable *pt, int page_id);
void map_page(PageTable *pt, int logical_page, int physical_page);
void kv_init(KVBlock *kv, int L, int NKH, int HD);
int kv_alloc(KVBlock *kv);
/* quant_kernels_omp.c:2066 */
void moe_forward_omp(const uint8_t **gate_raw, const uint8_t **up_raw, const uint8_t **down_raw, const float *x_norm,
                     int n_ff_expert, int n_embd, int qt_gate, int qt_up, int qt_down, const int *top_indices,
                     const float *top_weights, int top_k, float *combined, float *prealloc_buf,
                     uint8_t *prealloc_q8);
/* cengine_batch_instr.c:736, 803 */
void ssm_decode_step(const float *x, float *ssm_intermediate, const float *conv1d_w, const float *a_param,
                     const float *dt_bias, const float *alpha, const float *beta, const float *ssm_norm_w,
                     float *state, int B, int N, int inner, int groups, int state_size, int conv_kernel,
                     int dt_rank);
void ssm_layer_fused(const float *x, float *residual, float *output, const float *conv1d_w, const float *a_param,
                     const float *dt_bias, const float *alpha, const float *beta, const float *ssm_norm_w,
                     float *state, const uint8_t *gate_raw, int gate_nr, int gate_nc, int gate_qt,
                     const uint8_t *ssm_out_raw, int ssm_out_nr, int ssm_out_nc, int ssm_out_qt, int B, int N,
                     int inner, int groups, int state_size, int conv_kernel, int dt_rank);
/* cengine_batch_instr.c:1233 (computing the intended forward: see mojollama_b200.h) and :591 */
void batch_forward(const BC *c, const int *tokens, int B, float *ws);
void moe_ffn(const BC *c, int l, float *x, float *gate_buf, float *up_buf, float *ffn_buf, int B);
/* cengine_batch_instr.c:859-899 (the argument list of MlqQwen36Args, in order) */
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
    const float *cos_table, const float *sin_table, float *ws, uint8_t *q8_ws);
/* cengine_batch_instr.c:141 -- static in the reference, exported here */
void gqa(float *o, const float *q, const float *kc, const float *vc, int sl, int nh, int nkh, int hd);

#else  /* MLQ_REF_ABI_SIMD_OPS */
/* ================================== simd_ops.so set ================================== */
/* simd_ops.c:35, 56, 77, 88, 122, 218 */
void rms_norm(float *out, const float *x, const float *weight, int n, float eps);
void silu(float *out, const float *x, int n);
void residual_add(float *out, const float *a, const float *b, int n);
void softmax(float *x, int n);
void apply_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, int pos, float rope_base);
void set_num_threads(int n);
/* simd_ops.c:159, 209 */
void attention_forward(const float *q, const float *k_cache, const float *v_cache, float *out, int n_heads,
                       int n_kv_heads, int head_dim, int n_past, int max_seq);
void kv_cache_update(float *k_cache, float *v_cache, const float *k_new, const float *v_new, int layer,
                     int n_past, int max_seq, int n_kv_heads, int head_dim);
#endif /* MLQ_REF_ABI_SIMD_OPS */

/* ================================ gqa_attention.so set ================================ */
/* gqa_attention.c:93 */
void gqa_attention_decode(const float *q, const float *k_cache, const float *v_cache, float *out, int seq_len,
                          int n_head, int n_kv_head, int head_dim, float *workspace);
/* end of gqa_attention.so set */

#ifdef __cplusplus
}
#endif
#endif
