/* Reference-named entry points of simd_ops.so (src/mojollama/kernels/simd_ops.c of
 * the reference), forwarding to libmojollama_b200.so. */
#define MLQ_REF_ABI_SIMD_OPS 1
#include "mojollama_b200.h"
#include "mojollama_b200_ref_abi.h"

void rms_norm(float *out, const float *x, const float *weight, int n, float eps) {
    mlq_rms_norm(out, x, weight, 1, n, eps, 0, 0);
}
void silu(float *out, const float *x, int n) { mlq_silu(out, x, n, 1); }
void residual_add(float *out, const float *a, const float *b, int n) { mlq_add(out, a, b, n); }
void softmax(float *x, int n) { mlq_softmax(x, 1, n); }
void apply_rope(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, int pos, float rope_base) {
    mlq_rope_interleaved(q, k, n_heads, n_kv_heads, head_dim, pos, rope_base);
}
void set_num_threads(int n) { (void)n; }

/* simd_ops.c:159: k/v caches [max_seq][n_kv_heads][head_dim], n_past+1 positions */
void attention_forward(const float *q, const float *k_cache, const float *v_cache, float *out, int n_heads,
                       int n_kv_heads, int head_dim, int n_past, int max_seq) {
    (void)max_seq;
    mlq_attn_decode_flat(q, k_cache, v_cache, out, n_past + 1, n_heads, n_kv_heads, head_dim, 0);
}
void kv_cache_update(float *k_cache, float *v_cache, const float *k_new, const float *v_new, int layer,
                     int n_past, int max_seq, int n_kv_heads, int head_dim) {
    mlq_kv_cache_update(k_cache, v_cache, k_new, v_new, layer, n_past, max_seq, n_kv_heads, head_dim);
}
