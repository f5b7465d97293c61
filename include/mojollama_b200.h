/* mojollama_b200 -- core C-ABI of the B200 (sm_100a) engine.
 *
 * Every entry point takes plain pointers and sizes.  A pointer may be host
 * memory (pageable or pinned) or device memory of the current device; the
 * library classifies it with cudaPointerGetAttributes:
 *   - weights (const uint8_t *W) in host memory are copied to the device once and
 *     cached by (address, byte count); callers must treat a host weight buffer as
 *     immutable after its first use, or call mlq_cache_clear().
 *   - activations in host memory are copied in on every call, outputs in host
 *     memory are copied back, and the call returns when they are written.
 *   - when every pointer of a call is device memory the call is asynchronous on
 *     the library stream (mlq_set_stream / mlq_get_stream); mlq_sync() waits.
 * Errors never abort the process: the call returns with its outputs untouched
 * and records a code readable through mlq_last_error() (thread-local).
 *
 * The reference-named drop-in functions (quant_matmul_omp, moe_forward_omp, ...)
 * are declared in mojollama_b200_ref_abi.h and exported by the alias libraries
 * combined_engine.so / cengine_batch_instr.so / quant_kernels_omp.so /
 * gqa_attention.so / simd_ops.so, which forward to the functions below.
 */
#ifndef MOJOLLAMA_B200_H
#define MOJOLLAMA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- type codes: ggml/GGUF numbering (quant_kernels_omp.c:6-14 of the reference) ---- */
enum {
    MLQ_F32 = 0, MLQ_F16 = 1, MLQ_Q4_0 = 2, MLQ_Q4_1 = 3, MLQ_Q5_0 = 6, MLQ_Q8_0 = 8,
    MLQ_Q4_K = 12, MLQ_Q5_K = 13, MLQ_Q6_K = 14, MLQ_BF16 = 30, MLQ_MXFP4 = 39,
    /* the reference C decoder's own 17-byte MXFP4 layout {qs[16], e}, int4 mantissas
       (quant_kernels_omp.c:486-573); type 39 means GGUF MXFP4 {e, qs[16]}, E2M1 */
    MLQ_MXFP4_REF = 1039
};

/* ---- error codes ---- */
enum {
    MLQ_OK = 0,
    MLQ_ERR_ARG = 1,          /* null pointer, non-positive size, K not a multiple of the block */
    MLQ_ERR_TYPE = 2,         /* unsupported quant type (the reference silently skips these) */
    MLQ_ERR_CUDA = 3,         /* a CUDA runtime call failed */
    MLQ_ERR_NO_DEVICE = 4,    /* no CUDA device / library not initialised */
    MLQ_ERR_TIMEOUT = 5,      /* a device-side bounded wait gave up (see mlq_device_status) */
    MLQ_ERR_CAPACITY = 6,     /* size beyond a documented limit (page table full, K too large) */
    MLQ_ERR_UNSUPPORTED = 7
};

int         mlq_last_error(void);
const char *mlq_last_error_message(void);
void        mlq_clear_error(void);

/* ---- runtime ---- */
int   mlq_init(int device);               /* optional; first call otherwise initialises device 0 */
int   mlq_set_device(int device);
int   mlq_get_device(void);
void *mlq_get_stream(void);               /* cudaStream_t the library launches on */
/* launch on this cudaStream_t from now on (0 = the legacy default stream, e.g.
   torch.cuda.current_stream().cuda_stream); mlq_use_own_stream() goes back */
int   mlq_set_stream(void *cuda_stream);
int   mlq_use_own_stream(void);
int   mlq_sync(void);                     /* wait for the stream; also reports device-side errors */
int   mlq_device_status(void);            /* reads and clears the device error word */
/* Self-test of the device-side bounded-wait error path (no counterpart in the reference):
   one thread waits on a barrier nothing arrives on, gives up after limit_us (1..1e6)
   microseconds and reports it; returns what mlq_sync() then returns, MLQ_ERR_TIMEOUT.
   Nothing faults or hangs; the context stays usable. */
int   mlq_selftest_wait_timeout(int limit_us);
/* optional pre-residency of a whole host tensor (e.g. a 3-D expert tensor): every pointer
   inside it then maps to its device copy; unregister before freeing the host memory */
int   mlq_register_weights(const void *host_ptr, size_t bytes);
int   mlq_unregister_weights(const void *host_ptr);
int   mlq_cache_clear(void);              /* drop every cached device copy of host weights */
size_t mlq_cache_bytes(void);
int   mlq_num_sms(void);
/* number of kernels this library launched since load (all devices); for launch accounting */
unsigned long long mlq_launch_count(void);
/* 1 = reproduce the reference's quirks byte-for-byte where they differ from GGUF:
   type 39 decodes the reference MXFP4 layout, type 12 through the dispatcher follows
   the reference's Q8-activation dot, type 14 through the dispatcher reads ql low
   nibbles only.  0 (default) = GGUF-correct math. */
int   mlq_set_ref_compat(int on);
int   mlq_get_ref_compat(void);

/* ---- block formats ---- */
int    mlq_block_elems(int qt);            /* 32, 256 or 1; 0 if unknown */
int    mlq_block_bytes(int qt);
size_t mlq_row_bytes(int qt, int n_cols);  /* 0 if n_cols is not a multiple of the block */

/* ---- quantized matrix-vector / matrix-matrix products ----
 * W: n_rows x n_cols of type qt, row-major, rows are contiguous runs of blocks.
 * x: [B][n_cols] fp32, out: [B][n_rows] fp32 (the reference's batch layout,
 * cengine_batch_instr.c:251). */
int mlq_matmul(const void *W, int qt, const float *x, float *out, int n_rows, int n_cols, int B);

/* Decode GEMV of the batch engine's step (B <= 8) over n (1..4) matrices of one type that
   share the input x [B][K] (device pointers throughout): mode 0 out_i[B][n_rows_i] = x W_i^T;
   mode 1 out_i = res_i + x W_i^T (residual add folded in); mode 2 (n = 2, equal rows)
   out_0 = silu(x W_0^T) * (x W_1^T) (gate/up with the SiLU-mul).  The step's projections
   in batch_forward (cengine_batch_instr.c:1349-1351 q/k/v, :1409 o + residual add,
   :1463-1467 gate/up/silu/down + residual add, :1492 output head).
   MLQ_ERR_UNSUPPORTED when the shape or type is outside the kernel (the batch engine then
   uses mlq_matmul's path). */
int mlq_gemv_fused(int qt, int n, const void *const *W, const int *n_rows, float *const *out,
                   const float *const *res, int mode, const float *x, int B, int K);
/* dequantize n values of type qt to fp32, bit-identical to gguf-py / the reference */
int mlq_dequantize(const void *W, int qt, float *out, int64_t n);
/* the reference's Q8_0 activation quantizer, byte-identical (quant_kernels_omp.c:1406) */
int mlq_quantize_q8_0(const float *x, uint8_t *q8, int64_t n);
/* W (qt) times Q8_0-quantized activations x_q8 [B][n_cols/32 blocks] */
int mlq_matmul_q8act(const void *W, int qt, const uint8_t *x_q8, float *out, int n_rows, int n_cols, int B);
/* Same product for callers that cannot let the library allocate device memory (a
   process whose HBM is all owned by its own allocator, a decode loop that must not
   hit cudaMalloc/cudaFree).  No counterpart in the reference.  Allocates nothing: the
   fp32 activations go to a fixed 65536-element (256 KB) scratch array resident on
   every device that loads the library; B * n_cols beyond that is rejected with
   MLQ_ERR_CAPACITY.  W, x_q8 and out must be device memory; runs asynchronously on
   `stream` (a cudaStream_t, 0 = legacy default).  All calls on a device share the
   scratch, so calls that may overlap on the GPU race.  The first call on a device
   looks up the scratch address with that device current: make it before any stream
   capture. */
int mlq_matmul_q8act_noalloc(const void *W, int qt, const uint8_t *x_q8, float *out, int n_rows, int n_cols,
                             int B, void *stream);
/* Status of the mlq_matmul_q8act_noalloc calls on the current device (no counterpart in
   the reference): waits for `stream`, then reads and clears the status word their
   device-side bounded waits write.  MLQ_ERR_TIMEOUT when a wait gave up since the last
   query (that call's output is incomplete), else MLQ_OK.  Allocates nothing. */
int mlq_noalloc_status(void *stream);

/* ---- row / elementwise ops (out may equal x: in place) ---- */
/* out = x * w / sqrt(mean(x^2) + eps) per row (w may be NULL = ones).  sanitize = 1
   first maps NaN to 0 and clamps to +-1000 and, if res != NULL, stores that clamped
   input there (the batch engine's pre-norm, cengine_batch_instr.c:1258-1279). */
int mlq_rms_norm(float *out, const float *x, const float *w, int rows, int n, float eps, int sanitize, float *res);
/* mode 0: x / (1 + exp(-x)); mode 1: the simd_ops.c:56 Pade-tanh form on the first
   n - n%8 elements and the exact form on the tail, as the reference computes it */
int mlq_silu(float *out, const float *x, long long n, int mode);
/* h = silu(clamp(gate, -80, 80)) * up   (quant_kernels_omp.c:2157-2164) */
int mlq_swiglu(float *h, const float *gate, const float *up, long long n);
int mlq_add(float *out, const float *a, const float *b, long long n);
int mlq_softmax(float *x, int rows, int n);                    /* in place, per row */
/* interleaved-pair RoPE of simd_ops.c:122 on q [n_heads][hd] and k [n_kv_heads][hd] */
int mlq_rope_interleaved(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, int pos, float base);
/* cos/sin tables [max_ctx][rope_dim/2] of cengine_batch_instr.c:674 (base 10000 there) */
int mlq_rope_init(float *cos_t, float *sin_t, int max_ctx, int head_dim, int rope_dim, double base);
/* NeoX half-split RoPE of cengine_batch_instr.c:686 on `rows` rows of n_heads*head_dim
   (row_stride floats apart, 0 = packed); position per row from pos[] or pos_scalar */
int mlq_rope_neox(float *buf, int rows, int row_stride, int n_heads, int head_dim, const int *pos, int pos_scalar,
                  const float *cos_t, const float *sin_t, int rope_dim, int max_ctx);

/* ---- mixture of experts ---- */
/* moe_forward_omp (quant_kernels_omp.c:2066) semantics, GGUF-correct for every expert
   type: combined = sum_i top_w[i] * down[e] . (silu(clamp(gate[e] . x, +-80)) * (up[e] . x)),
   e = top_idx[i].  gate/up/down are arrays of per-expert pointers (host arrays; the
   pointers host or device), gate/up n_ff x n_embd, down n_embd x n_ff; top_k <= 16. */
int mlq_moe_forward(const void *const *gate, const void *const *up, const void *const *down, const float *x,
                    int n_ff, int n_embd, int qt_gate, int qt_up, int qt_down, const int *top_idx,
                    const float *top_w, int top_k, float *combined);
/* router: logits = W_r . x (E x N, type qt_r), softmax (1/(sum + 1e-10)), top-k with the
   reference's tie rule (lower expert index first), renorm = 1 rescales the k weights to
   sum 1 (cengine_batch_instr.c:1113-1152); x [B][N] -> idx, w [B][k]; E <= 256 */
int mlq_moe_router(const float *x, int B, int N, const void *W_r, int qt_r, int E, int k, int renorm, int *idx,
                   float *w);

/* ---- SSM decode step, the reference's semantics (cengine_batch_instr.c:736-849) ----
   x [B][N] -> interm [B][inner]; state [groups][state_size] shared by all B sequences and
   updated in sequence order.  ssm_norm_w and conv_kernel are accepted and unused, as there. */
int mlq_ssm_decode_step(const float *x, float *interm, const float *conv1d_w, const float *a_param,
                        const float *dt_bias, const float *alpha, const float *beta, const float *ssm_norm_w,
                        float *state, int B, int N, int inner, int groups, int state_size, int conv_kernel,
                        int dt_rank);
/* output_b = residual_b + W_out . ((W_gate . x_b) * interm_b);  W_gate inner x N, W_out N x inner */
int mlq_ssm_layer_fused(const float *x, const float *residual, float *output, const float *conv1d_w,
                        const float *a_param, const float *dt_bias, const float *alpha, const float *beta,
                        const float *ssm_norm_w, float *state, const void *gate_raw, int gate_nr, int gate_nc,
                        int gate_qt, const void *ssm_out_raw, int ssm_out_nr, int ssm_out_nc, int ssm_out_qt, int B,
                        int N, int inner, int groups, int state_size, int conv_kernel, int dt_rank);

/* ---- whole-model decode step over the reference's BC model description ----
   bc points to a BC struct (mojollama_b200_ref_abi.h, cengine_batch_instr.c:536-589);
   tokens [B] (B <= 64), one new token per sequence; c->logits [B][outNR] is written and
   every kv_array[b]->seq_len[0] advances by one.  ws is accepted and unused. */
int mlq_batch_forward(const void *bc, const int *tokens, int B, float *ws);
/* Sliding-window attention per layer for batch_forward on the model described by bc (no
   counterpart in the reference, whose engine attends to every position): layer l attends to
   its last windows[l] positions, 0 = all.  Kept per BC address; L = 0 clears it. */
int mlq_set_attention_windows(const void *bc, const int *windows, int L);

/* ---- GGUF reader and device weight loader ----
   Replaces the reference's gguf-py load path (turbo_engine_v7_moe.py:425-618: GGUFReader,
   numpy views of the mmapped file, host F32 copies).  The file is parsed natively (GGUF
   versions 2 and 3) and mapped; mlq_gguf_upload streams its whole data section into HBM
   unchanged (mmap -> two pinned buffers -> copy engine), so tensor i is at dev + its offset
   in GGUF block layout, ready for mlq_matmul / batch_forward device pointers. */
typedef struct {
    char name[128];
    int n_dims;
    int64_t dims[4];      /* as stored: dims[0] is the contiguous (fastest) dimension */
    int type;             /* ggml type code */
    uint64_t offset;      /* inside the data section */
    uint64_t bytes;       /* 0 when the type's block layout is not known to this library */
} MlqGgufTensor;
void *mlq_gguf_open(const char *path);      /* NULL on error (mlq_last_error_message) */
int mlq_gguf_close(void *h);
int mlq_gguf_version(void *h);
int64_t mlq_gguf_n_tensors(void *h);
int64_t mlq_gguf_n_kv(void *h);
uint64_t mlq_gguf_alignment(void *h);
uint64_t mlq_gguf_data_offset(void *h);     /* file offset of the data section */
uint64_t mlq_gguf_data_bytes(void *h);
int mlq_gguf_tensor(void *h, int64_t i, MlqGgufTensor *out);
int64_t mlq_gguf_find(void *h, const char *name);            /* -1 if absent */
int mlq_gguf_kv_type(void *h, const char *key);              /* GGUF value type 0..12, -1 if absent */
int mlq_gguf_kv_int(void *h, const char *key, int64_t *out); /* integer and bool values */
int mlq_gguf_kv_float(void *h, const char *key, double *out);
int64_t mlq_gguf_kv_str(void *h, const char *key, char *buf, size_t len);   /* full length, -1 if absent */
int64_t mlq_gguf_kv_array(void *h, const char *key, int *item_type);       /* count, -1 if not an array */
const void *mlq_gguf_tensor_data(void *h, int64_t i);        /* host view in the mapping */
int mlq_gguf_upload(void *h, void *dev, uint64_t dev_bytes);               /* whole data section */
int mlq_gguf_upload_tensor(void *h, int64_t i, void *dev, uint64_t dev_bytes);

/* ---- Mamba-2 decode step (no counterpart in the reference) ----
   The reference's ssm_decode_step (cengine_batch_instr.c:736-797) is a toy kept byte-
   compatible above; these are the published Mamba-2 recurrence (Dao & Gu 2024), one token
   per sequence, for config 5's hybrid model.  H heads of P channels, state size S, G groups
   of B/C (H % G == 0), conv width d_conv (<= 8).  Layouts: xbc [B][H*P + 2*G*S] (x | B | C),
   z [B][H*P] (NULL: no gate), dt [B][H], conv_state [B][conv_dim][d_conv] (last d_conv
   inputs, newest last), conv_w [conv_dim][d_conv], conv_b [conv_dim] (NULL: none), A_log /
   dt_bias / D [H] (A = -exp(A_log); D NULL: none), norm_w [H*P] (NULL: no norm), ssm_state
   [B][H][P][S]; both states are updated in place.  y [B][H*P] = norm_w * rmsnorm(y * silu(z))
   over groups of norm_group elements (0: the whole H*P).  P % 32 == 0; S in {16, 32, 64} or
   a multiple of 128. */
int mlq_mamba2_step(const float *xbc, const float *z, const float *dt, float *conv_state, const float *conv_w,
                    const float *conv_b, const float *A_log, const float *dt_bias, const float *D,
                    const float *norm_w, float *ssm_state, float *y, int B, int H, int P, int S, int G, int d_conv,
                    float eps, int norm_group);
/* the mixer: proj = W_in u (rows z | xBC | dt; W_in [H*P + conv_dim + H][hidden] of type
   qt_in), the step, out [B][hidden] = W_out y (W_out [hidden][H*P] of type qt_out) */
int mlq_mamba2_layer(const float *u, int B, int hidden, const void *W_in, int qt_in, const void *W_out, int qt_out,
                     float *conv_state, const float *conv_w, const float *conv_b, const float *A_log,
                     const float *dt_bias, const float *D, const float *norm_w, float *ssm_state, float *out, int H,
                     int P, int S, int G, int d_conv, float eps, int norm_group);

/* ---- next-token selection on the device ----
   The reference picks each next token on the host with np.argmax over the logits
   (turbo_engine_v7_moe.py:2101-2114); these keep logits and tokens on the device.
   mlq_sample: logits [B][V] -> tokens [B].  temperature <= 0: greedy, exactly np.argmax
   (first maximum; a NaN counts as the maximum).  temperature > 0: a draw from
   softmax(logits / temperature) by the Gumbel-max rule argmax(logit/T - log(-log u)),
   u from a counter-based generator keyed by (seed, step, row, index) -- reproducible,
   restated in numpy by oracle/sampling.py.  B <= 1024.  Calls on one device share a small
   per-device state: calls that may overlap on the GPU (unordered streams) race. */
int mlq_sample(const float *logits, int B, int V, float temperature, unsigned long long seed,
               unsigned long long step, int *tokens);
int mlq_argmax(const float *logits, int B, int V, int *tokens);   /* mlq_sample with temperature 0 */
/* one batch_forward step, then mlq_sample on its logits into next_tokens (which may be the
   tokens buffer itself); with device tokens / logits / next_tokens nothing reaches the host */
int mlq_batch_forward_sample(const void *bc, const int *tokens, int B, float *ws, float temperature,
                             unsigned long long seed, unsigned long long step, int *next_tokens);
/* moe_ffn: layer l's routed experts for x [B][N] -> ffn [B][N] (cengine_batch_instr.c:591) */
int mlq_moe_ffn(const void *bc, int l, const float *x, float *ffn, int B);
/* forget the cached per-model device plans (also done by mlq_cache_clear) */
void mlq_forget_model_plans(void);
/* sizeof(BC) as this library compiles it (layout check for ctypes mirrors) */
size_t mlq_sizeof_bc(void);

/* ---- qwen36_batch_forward (cengine_batch_instr.c:859-899): the reference's 76 arguments,
   field for field and in order, packed into one struct; the reference-named 76-argument
   function in mojollama_b200_ref_abi.h fills it.  Semantics in csrc/qwen36.cu. */
typedef struct {
    int B, L, N, NH, n_kv_h, HD, FF;
    int n_experts, top_k, n_ff_expert;
    float eps;
    int rope_dim, max_ctx, ssm_inner, ssm_groups, ssm_state_size, ssm_conv_kernel, ssm_dt_rank;
    const float *emb;
    int emb_quant;
    const int *layer_types;
    const int *tokens;
    float *logits;
    const float **attn_norm_w, **ffn_norm_w;
    const uint8_t **attn_qkv_raw; const int *qkv_nr, *qkv_nc, *qkv_qt;
    const uint8_t **attn_gate_raw; const int *gate_nr, *gate_nc, *gate_qt;
    const uint8_t **ssm_out_raw; const int *ssm_out_nr, *ssm_out_nc, *ssm_out_qt;
    const uint8_t **attn_out_raw; const int *out_nr, *out_nc, *out_qt;
    uint8_t **gate_exp_raw; const int *gate_exp_qt;
    uint8_t **up_exp_raw; const int *up_exp_qt;
    uint8_t **down_exp_raw; const int *down_exp_qt;
    const float **shexp_gate_raw, **shexp_up_raw, **shexp_down_raw;
    const float **shexp_router;
    const int *shexp_int;
    const uint8_t **moe_router_raw; const int *moe_router_qt;
    const int *shexp_gate_qt, *shexp_up_qt, *shexp_down_qt;
    const float *out_norm_w;
    const uint8_t *out_w; int out_nr_final, out_nc_final, out_qt_final;
    const float **ssm_conv1d, **ssm_a, **ssm_dt_bias, **ssm_alpha, **ssm_beta, **ssm_norm;
    float *ssm_state;
    float *kv_k, *kv_v; int *kv_lens;
    const float *cos_table, *sin_table;
    float *ws; uint8_t *q8_ws;
} MlqQwen36Args;
int mlq_qwen36_batch_forward(const MlqQwen36Args *args);

/* ---- expert parallelism (device pointers; the exchanges are the caller's collectives) ----
   A rank owns experts [rank*experts_per_rank, (rank+1)*experts_per_rank).
   mlq_ep_dispatch: idx [T][k] global expert ids -> counts[world] rows per destination rank,
     pos[T*k] row of slot t*k+i in the send buffer (grouped by destination, slot order kept),
     send_x [T*k][N] token rows, send_eid [T*k] local expert id at the destination (world <= 8).
   mlq_moe_rows: y[r] = down_e(silu(clamp(gate_e x_r, +-80)) * up_e x_r), e = eid[r] < n_experts,
     expert tensors [n_experts][rows][cols] at the given byte strides; rows are grouped by
     expert on the device and each active expert is streamed once (grouped GEMV).
   mlq_ep_combine: out[t] = residual[t] + sum_i w[t][i] * recv_y[pos[t*k+i]] (residual may be NULL). */
int mlq_ep_dispatch(const int *idx, int T, int k, int experts_per_rank, int world, const float *x, int N, int *counts,
                    int *pos, float *send_x, int *send_eid);
int mlq_moe_rows(int gqt, int uqt, int dqt, const void *gexp, const void *uexp, const void *dexp, long long gstride,
                 long long ustride, long long dstride, int n_experts, const int *eid, int R, int n_ff, int N,
                 const float *x, float *y);
/* Fixed-capacity forms for an exchange with equal splits (no count read back to the host):
   send / recv [world][cap][N + 4] floats, the destination-local expert id in-band at column
   N of each row (int bits; -1 = unused row).  Rows for destination d sit at d * cap + j in
   slot order; pos[t*k + i] = d * cap + j.  cap >= T * min(k, experts_per_rank). */
int mlq_ep_dispatch_packed(const int *idx, int T, int k, int experts_per_rank, int world, int cap, const float *x,
                           int N, int *pos, float *send);
int mlq_moe_rows_packed(int gqt, int uqt, int dqt, const void *gexp, const void *uexp, const void *dexp,
                        long long gstride, long long ustride, long long dstride, int n_experts, const float *recv,
                        int R, int n_ff, int N, float *y);
int mlq_ep_combine(const float *recv_y, const int *pos, const float *w, int T, int k, int N, const float *residual,
                   float *out);

/* ---- decode attention (one query per sequence), fp32 KV ---- */
/* flat KV k/v [seq_len][n_kv_head*head_dim] (gqa_attention.c:93, cengine_batch_instr.c:141);
   head h uses KV head h / (n_head / n_kv_head); window > 0 attends the last `window`
   positions only; q, out [n_head*head_dim] */
int mlq_attn_decode_flat(const float *q, const float *k_cache, const float *v_cache, float *out, int seq_len,
                         int n_head, int n_kv_head, int head_dim, int window);
/* paged KV: k_pages / v_pages [n_pages][page_size][n_kv_head*head_dim]; table [B][table_stride]
   logical -> physical page; seq_lens [B]; q, out [B][n_head*head_dim] */
int mlq_attn_decode_paged(const float *q, const float *k_pages, const float *v_pages, const int *table,
                          int table_stride, int page_size, int n_pages, const int *seq_lens, int B, int n_head,
                          int n_kv_head, int head_dim, int window, float *out);

/* ---- PagedAttention bookkeeping: the reference's structs, byte for byte
   (cengine_batch_instr.c:160-207).  pages / k / v are device memory in this build. ---- */
typedef struct {
    int page_size;     /* KV slots per page */
    int n_pages;       /* physical pages in the pool */
    float *pages;      /* [n_layers][n_pages][page_size][nkh*hd] K, then the same for V (device) */
    int *table;        /* [1024] logical page -> physical page, -1 = unmapped (host) */
    int *free_pages;   /* LIFO free list (host) */
    int free_count;
    int _nkh;
    int _hd;
    int _n_layers;
} MlqPageTable;

typedef struct {
    float *k, *v;      /* [L][1024][64][nkh*hd] each (device) */
    int n_blocks, seq_len[64], block_map[64][1024];
    MlqPageTable pt;
} MlqKVBlock;

int  mlq_page_table_init(MlqPageTable *pt, int max_pages, int page_size, int nkh, int hd, int n_layers);
int  mlq_page_table_alloc(MlqPageTable *pt);                 /* -1 when full */
void mlq_page_table_free(MlqPageTable *pt, int page_id);
void mlq_map_page(MlqPageTable *pt, int logical_page, int physical_page);
void mlq_page_table_destroy(MlqPageTable *pt);               /* frees pool, table, free list */
int  mlq_kv_init(MlqKVBlock *kv, int L, int nkh, int hd);
int  mlq_kv_alloc(MlqKVBlock *kv);
void mlq_kv_free(MlqKVBlock *kv);

/* ---- KV snapshots for the prefix cache (no counterpart in the C engine; the reference's
   Python prefix cache copies whole host KV arrays, prefix_cache.py:164-222) ----
   mlq_kv_snapshot: positions [0, len) (len <= seq_len) of every layer's K and V rows out of
   a KVBlock's page pool, packed as [2][n_layers][len][nkh*hd] floats at dst.
   mlq_kv_restore: the reverse; maps pages from the block's free list where its table has
   none, copies src in, sets seq_len = len.  dst / src may be device or host memory. */
int mlq_kv_snapshot(const MlqKVBlock *kv, int len, float *dst);
int mlq_kv_restore(MlqKVBlock *kv, int len, const float *src);

size_t mlq_sizeof_page_table(void);
size_t mlq_sizeof_kv_block(void);
/* simd_ops.c:209: copy one position's rows to offset n_past*nkh*hd (layer ignored) */
int  mlq_kv_cache_update(float *k_cache, float *v_cache, const float *k_new, const float *v_new, int layer,
                         int n_past, int max_seq, int nkh, int hd);

#ifdef __cplusplus
}
#endif
#endif
