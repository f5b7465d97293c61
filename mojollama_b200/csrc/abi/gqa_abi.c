/* Reference-named entry point of gqa_attention.so
 * (src/mojollama/kernels/gqa_attention.c of the reference), forwarding to
 * libmojollama_b200.so. */
#include "mojollama_b200.h"
#include "mojollama_b200_ref_abi.h"

/* gqa_attention.c:93; the workspace is not needed (scores never leave the chip) */
void gqa_attention_decode(const float *q, const float *k_cache, const float *v_cache, float *out, int seq_len,
                          int n_head, int n_kv_head, int head_dim, float *workspace) {
    (void)workspace;
    mlq_attn_decode_flat(q, k_cache, v_cache, out, seq_len, n_head, n_kv_head, head_dim, 0);
}
