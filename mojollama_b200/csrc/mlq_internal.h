// Internal runtime shared by the CUDA translation units of libmojollama_b200.so.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <vector>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "../../include/mojollama_b200.h"

namespace mlq {

// ---- errors ---------------------------------------------------------------------------
void set_error(int code, const char *fmt, ...);
inline bool cuda_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    set_error(MLQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return false;
}
#define MLQ_CUDA(call) ::mlq::cuda_ok((call), #call)

// ---- device context ------------------------------------------------------------------
struct Ctx {
    int device = -1;
    int num_sms = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;   // where launches go (own or user-bound)
    int *d_status = nullptr;         // device view of the error word (0 = ok), written by bounded waits
    volatile int *h_status = nullptr;  // the same word in mapped pinned host memory: read after a
                                       // synchronisation at no cost
};
Ctx *ctx();                          // current device's context (initialises on first use)

// What the kernel launchers need from the device: SM count and the device status word.
// Normally taken from ctx(); an entry point that must not allocate installs its own
// for the duration of its launches with LaunchEnvScope (ctx() allocates on first use).
struct LaunchEnv {
    int num_sms;
    int *d_status;
    bool no_alloc = false;           // launchers must not allocate (paths needing scratch step aside)
    bool out_host = false;           // outputs are host memory written over PCIe: kernels that can
                                     // gather a tile's outputs and write them as one run
};
const LaunchEnv *launch_env();
struct LaunchEnvScope {
    explicit LaunchEnvScope(const LaunchEnv *e);
    ~LaunchEnvScope();
    const LaunchEnv *prev;
};
cudaStream_t stream();
int *dev_status();
void count_launch(int n = 1);
// Programmatic dependent launch (MLQ_NO_PDL=1 turns it off): the kernel may be scheduled while
// the previous kernel on the stream drains; it must execute griddepcontrol.wait (pdl_wait())
// before it reads or writes any memory that kernel touches.  Counts the launch.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    count_launch();
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}
bool ref_compat();

// ---- pointer handling ------------------------------------------------------------------
bool is_device_ptr(const void *p);

// Per-call staging for host activations/outputs.  Reset by CallScope.
struct CallScope {
    CallScope();
    ~CallScope();
    // device view of an input; copies host data in when needed
    const void *in(const void *p, size_t bytes);
    // device view of an output; host outputs are copied back in finish()
    void *out(void *p, size_t bytes);
    // device view of an output that the kernels only store to, once per element, in
    // contiguous runs: pinned host memory the device can reach is written in place (no
    // staging copy); anything else as out()
    void *out_direct(void *p, size_t bytes, bool *host_mapped);
    // device view of an in/out buffer (copied in and back)
    void *inout(void *p, size_t bytes);
    // device scratch (uninitialised) for this call
    void *scratch(size_t bytes);
    // weights: device pointers pass through, host pointers go through the residency cache
    const void *weights(const void *p, size_t bytes);
    // copy host outputs back and synchronise when anything was host; returns MLQ_OK or error
    int finish();
    bool failed = false;
    bool any_host = false;

  private:
    struct Pending { void *host; void *dev; size_t bytes; };
    Pending pending_[64];
    int n_pending_ = 0;
    size_t arena_used_ = 0;
    void *stage(size_t bytes);
};

// ---- launchers implemented in the .cu files --------------------------------------------
int block_elems(int qt);
int block_bytes(int qt);
bool is_quant_type(int qt);

// W, x, out are device pointers here.
int launch_matmul(const uint8_t *W, int qt, const float *x, float *out, int n_rows, int n_cols,
                  int B, size_t w_bytes, cudaStream_t s);
int launch_dequantize(const uint8_t *W, int qt, float *out, int64_t n, cudaStream_t s);
// 16-bit float weights (bf16 = 1 / f16 = 0) times B fp32 activation rows through cuBLAS
// (blas.cu); MLQ_ERR_UNSUPPORTED when unavailable
int launch_gemm16(const void *W, int bf16, const float *x, float *out, int n_rows, int K, int B, cudaStream_t s);
// fp32 router rows and one extra fp32 row (a shared expert's gate score) in one launch (gemv.cu):
// out [B][n_rows], out_extra [B]
int launch_router_rows_f32(const float *W, const float *w_extra, const float *x, float *out, float *out_extra,
                           int n_rows, int K, int B, cudaStream_t s);
// tensor-core GEMM (gemm_tc.cu); MLQ_ERR_UNSUPPORTED for formats/shapes it does not cover
int launch_gemm_tc(const uint8_t *W, int qt, const float *x, float *out, int n_rows, int K, int M, cudaStream_t s);
// grouped experts on the tensor-core GEMM (csrc/gemm_tc.cu): sorted rows converted to fp16
// (xh [R][K rounded up to 256] halves, xs [R] power-of-two scales) by launch_rows_to_f16,
// then one launch per matrix list over k_group_plan's items of 128-row tiles
size_t tc_grouped_xh_bytes(int R, int K);
int launch_rows_to_f16(const float *x, const float *x2, const int *rows, int row_div, int x_stride, float clamp, int R,
                       int K, __half *xh, __half *xl, float *xs, cudaStream_t s);
bool tc_grouped_supported(int qt, const uint8_t *W, long long estride, int K);
int launch_gemm_tc_grouped(int qt, const uint8_t *W, long long estride, const uint8_t *W2, long long estride2,
                           int n_rows, int K, const void *items, const int *n_items_dev, int n_items_bound,
                           const __half *xh, const __half *xl, const float *xs, float *out, float *out2,
                           const int *out_rows, cudaStream_t s);
// grouped MXFP4 experts on the block-scaled tensor cores (moe_mxf4_tc.cu): sorted rows encoded
// once as E2M1 planes (launch_mxf4_planes_rows, mxf4_planes_bytes of scratch), then one launch
// per matrix list over k_group_plan's items of 128-row tiles; K % 32 == 0 (TMA tiles when K % 512 == 0 and the rows are 16-byte aligned, else 16-byte windows)
size_t mxf4_planes_bytes(int R, int K);
bool mxf4_grouped_supported(const uint8_t *W, long long estride, int E, int n_rows, int K);
bool mxf4_grouped_wanted(int R, int E, int item_tiles);
int launch_mxf4_planes_rows(const float *x, const float *x2, const int *rows, int row_div, int x_stride, float clamp,
                            int R, int K, uint8_t *planes, cudaStream_t s);
int launch_moe_mxf4_tc(const uint8_t *W, long long estride, const uint8_t *W2, long long estride2, int E, int n_rows,
                       int K, const void *items, const int *n_items_dev, int n_items_bound, const uint8_t *planes,
                       int R, float *out, float *out2, const int *out_rows, cudaStream_t s);
// one MXFP4 matrix (or a pair with the same shape: out2 = W2 x) times all R encoded rows, on the
// same kernel: out [R][n_rows]
bool mxf4_dense_supported(const uint8_t *W, int n_rows, int K);
int launch_mxf4_dense_tc(const uint8_t *W, const uint8_t *W2, int n_rows, int K, const uint8_t *planes, int R,
                         float *out, float *out2, cudaStream_t s);
int launch_quantize_q8_0(const float *x, uint8_t *q8, int64_t n, cudaStream_t s);
int launch_q8act_to_f32(const uint8_t *x_q8, float *x, int64_t n, cudaStream_t s);

// ops.cu
int launch_rms_norm(float *out, const float *x, const float *w, float *res, int rows, int n, float eps, int flags,
                    cudaStream_t s);
// x += y, then out = RMSNorm(x) (as launch_rms_norm with res null) in one launch
int launch_add_rms_norm(float *x, const float *y, const float *w, float *out, int rows, int n, float eps, int flags,
                        cudaStream_t s);
int launch_silu(float *out, const float *x, long long n, int mode, cudaStream_t s);
int launch_swiglu(float *h, const float *g, const float *u, long long n, cudaStream_t s);
int launch_add(float *out, const float *a, const float *b, long long n, cudaStream_t s);
int launch_softmax(float *x, int rows, int n, cudaStream_t s);
int launch_rope_init(float *cos_t, float *sin_t, int max_ctx, int hd, int rope_dim, double base, cudaStream_t s);
int launch_rope_neox(float *buf, int rows, int rows_stride, int nh, int hd, const int *pos_dev, int pos_host,
                     const float *cos_t, const float *sin_t, int rope_dim, cudaStream_t s);

// attention.cu: fp32 KV cache addressing
struct KVView {
    const float *k, *v;      // base of the K and V regions
    const int *table;        // [B][max_pages] physical page of each logical page, or null
    int table_stride;        // ints between sequences' tables
    long long page_stride;   // floats between pages
    int page_size;           // slots per page
    int row_stride;          // floats between slots (NKH * HD)
    // optional per-sequence page pools (one KVBlock per sequence): pool_seq[b] holds
    // [n_layers][n_pages][page_size][row] K then the same for V; K of layer `layer`
    // starts at layer * layer_stride, V at (n_layers + layer) * layer_stride
    float *const *pool_seq;
    long long layer_stride;
    int layer, n_layers;
    // optional own rows: position seq_len-1 of sequence b is read from tail_k/tail_v
    // [B][tail_stride] instead of the cache (sequences that share one cache slot)
    const float *tail_k = nullptr, *tail_v = nullptr;
    int tail_stride = 0;
    // physical pages in the pool (> 0: a table entry outside [0, n_pages) reads as zeros
    // and is never written, instead of addressing memory outside the pool; 0: unchecked)
    int n_pages = 0;
};

// The decode step's RoPE and KV store done by the attention kernel itself (instead of a
// k_rope_kv launch before it): q [B][nh][hd] and the new rows k_new / v_new [B][nkh*hd]
// arrive unrotated; each CTA rotates its own query heads and its KV head's new k row (NeoX
// halves of the first rope_dim dims at position pos[b]), and the CTA whose positions
// include pos[b] stores the new k / v rows of its head into the cache and, when mk / mv are
// given, into the KVBlock mirrors.  Requires per-sequence pools (kv.pool_seq).
struct AttnRope {
    const int *pos = nullptr;
    const float *cos_t = nullptr, *sin_t = nullptr;
    int rope_dim = 0;
    const float *k_new = nullptr, *v_new = nullptr;
    float *const *mk = nullptr;
    float *const *mv = nullptr;
};
// planes non-null: the output rows [B][nh*hd] also written as packed activation rows, when
// attn_packs_output(nh, nkh, hd) (otherwise planes is ignored); rope non-null: see AttnRope
// (MLQ_ERR_UNSUPPORTED when its requirements are not met; nothing is launched then)
int launch_attn_decode(const float *q, const KVView &kv, const int *seq_lens_dev, int seq_len_scalar,
                       int max_seq_len, int B, int nh, int nkh, int hd, int window, float scale, float *out,
                       float *scratch, size_t scratch_bytes, cudaStream_t s, uint8_t *planes = nullptr,
                       const AttnRope *rope = nullptr);
inline bool attn_packs_output(int nh, int nkh, int hd) { return nkh > 0 && (nh / nkh) * hd % 32 == 0 && hd % 32 == 0; }
int launch_kv_write(const KVView &kv, float *k_base, float *v_base, const float *k_new, const float *v_new,
                    const int *pos_dev, int pos_scalar, int B, int row, cudaStream_t s);
size_t attn_scratch_bytes(int B, int nh, int hd);
// decode step: RoPE of q and k in place, then k / v into the per-sequence page pools at pos[b]
// and (mk / mv non-null) the KVBlock mirror arrays; MLQ_ERR_UNSUPPORTED outside that case
int launch_rope_kv(float *q, float *k, const float *v, int B, int nh, int nkh, int hd, int rope_dim, const int *pos,
                   const float *cos_t, const float *sin_t, const KVView &kv, float *const *mk, float *const *mv,
                   cudaStream_t s);
// bytes of a KVBlock k or v array allocated by kv_init of this library (0 if unknown)
size_t kv_array_bytes(const void *p);

// ssm.cu
int launch_ssm_decode_step(const float *x, float *interm, const float *conv_w, const float *a_param,
                           const float *dt_bias, const float *alpha, const float *beta, float *state, int B, int N,
                           int inner, int groups, int state_size, int dt_rank, cudaStream_t s);
int launch_mul(float *a, const float *b, long long n, cudaStream_t s);

// moe.cu: mode 0 = SwiGLU pairs, 1 = weighted sum, 2 = store
int launch_moe_gemv(int mode, int qt, const uint8_t *const *W, const float *wgt, int G, int n_rows, int K,
                    const float *x, int nx, float *out, const float *residual, cudaStream_t s);
int launch_moe_indexed(int mode, int qt, const uint8_t *base_a, const uint8_t *base_b, long long expert_stride,
                       const int *d_idx, const float *d_w, int top_k, int n_tok, int n_rows, int K, const float *x,
                       float *out, const float *residual, cudaStream_t s, float swiglu_clamp = 80.0f);
int launch_moe_experts(int gqt, int uqt, int dqt, const uint8_t *gexp, const uint8_t *uexp, const uint8_t *dexp,
                       long long gs, long long us, long long ds, const int *idx, const float *w, int top_k,
                       int n_tok, int n_ff, int N, const float *x, float *h, float *h2, float *out,
                       const float *residual, float clamp, cudaStream_t s);
// grouped expert GEMV (gemv.cu): rows ordered by expert, each active expert streamed once
struct GroupedCall {
    int qt;
    const uint8_t *W;          // expert 0 of the first matrix; experts estride bytes apart
    long long estride;
    float *out;                // [rows][n_rows]
    const uint8_t *W2;         // optional second matrix of the same type and shape (tiles >= T)
    long long estride2;
    float *out2;
    const void *items;         // planner item list
    const int *n_items_dev;    // its length, on the device
    int n_items_bound;         // host bound of that length (grid size)
    const uint8_t *planes;     // packed activation rows in sorted order (launch_encode_packed)
    const int *out_rows;       // sorted position -> row of out / out2 (identity if null)
    int n_rows, K;             // of one expert's matrix
};
int grouped_tiles_per_expert(int qt, int n_rows, int K);
size_t grouped_packed_bytes(int R, int K);
int launch_grouped(const GroupedCall &gc, cudaStream_t s);
// packed activation rows p < R: x[rows[p] / row_div] (rows may be null: x[p / row_div]);
// with x2 set, silu(clamp(x, +-clamp)) * x2 of that row
int launch_encode_packed(const float *x, const float *x2, const int *rows, int R, int K, uint8_t *planes,
                         cudaStream_t s, int row_div = 1, float clamp = 80.0f, int x_stride = 0);
// Routed experts of R = T * k rows (row t * k + i: token t, slot i, expert eid[row]) over
// the grouped expert GEMV: a stable plan by expert, each active expert's gate / up / down
// matrices streamed once for all of its rows.  x holds one row per token when row_div = k
// (or one per row when row_div = 1); y [R][N] = down_e(silu(clamp(gate_e x)) * up_e x).
// Scratch: MoeGroupedScratch of moe_grouped_scratch_bytes.
struct MoeGroupedScratch {
    int *spos, *srow, *nitem;
    void *items[3];
    uint8_t *px, *ph;
    float *g, *u;
    __half *xg, *xd;   // tensor-core path: sorted fp16 input rows of gate/up and of down,
    __half *xgl, *xdl; // their fp16 rounding residuals
    float *sg, *sd;    // and their power-of-two scales
    uint8_t *bx, *bh;  // block-scaled (kind::mxf4) path: E2M1 planes of the gate/up and down inputs
};
size_t moe_grouped_scratch_bytes(int gqt, int uqt, int dqt, int R, int E, int n_ff, int N);
void moe_grouped_carve(MoeGroupedScratch &m, uint8_t *base, int gqt, int uqt, int dqt, int R, int E, int n_ff, int N);
// eid_stride / x_stride: ints / floats between rows of eid and x (packed exchange rows keep
// the expert id in-band at column N of an (N + 4)-float row); 0 = dense (1 / N)
int launch_moe_grouped(int gqt, int uqt, int dqt, const uint8_t *gexp, const uint8_t *uexp, const uint8_t *dexp,
                       long long gstride, long long ustride, long long dstride, int E, const int *eid, int R,
                       int row_div, int n_ff, int N, const float *x, float *y, float clamp, const MoeGroupedScratch &m,
                       cudaStream_t s, int eid_stride = 1, int x_stride = 0);
// out[t] = residual[t] (if set) + sum_i w[t * k + i] * y[pos[t * k + i]] (pos null: identity)
int launch_ep_combine(const float *y, const int *pos, const float *w, int T, int k, int N, const float *residual,
                      float *out, cudaStream_t s, const float *ys = nullptr, const float *score = nullptr);
// decode GEMV over up to 4 same-type matrices sharing packed activation rows [B <= 8]:
// out_i = (res_i +) W_i x, or with pair (2 matrices, same rows) out_0 = silu(W_0 x) * (W_1 x);
// MLQ_ERR_UNSUPPORTED when the shape or type does not suit it
int launch_gemv_seg(int qt, int n_seg, const uint8_t *const *W, const int *n_rows, float *const *out,
                    const float *const *res, int pair, const uint8_t *planes, int B, int K, cudaStream_t s);
size_t packed_rows_bytes(int rows, int K);
// RMSNorm of rows (as launch_rms_norm) that also writes the normalised rows as packed
// activation rows (out may be null when only the packed rows are needed)
int launch_rms_norm_encode(float *out, const float *x, const float *w, float *res, int rows, int n, float eps,
                           int flags, uint8_t *planes, cudaStream_t s);
// stable order of R rows by expert id (sorted_pos[r], src_row[p]) and the item lists of
// n_lists tilings (tiles[l] tiles per 8-row chunk; n_items[l] written on the device)
int launch_group_plan(const int *eid, int R, int E, int n_lists, void *const *items, const int *tiles,
                      int *sorted_pos, int *src_row, int *n_items, cudaStream_t s, int eid_stride = 1);
// batch-engine embedding rows (qwen36.cu)
int launch_embed(const void *emb, int emb_quant, const int *d_tok, const int *h_tok, float *x, int B, int N, int V,
                 cudaStream_t s);
size_t embed_bytes(int emb_quant, int N, int V);
bool host_tokens(const int *tokens, int B, std::vector<int> &out);
void forget_kv_mirrors();
void forget_tc_scratch();
// per-(device, stream) scratch of the tensor-core kernels, grown outside graph capture;
// null inside a capture that would need growth, or under a no-allocation LaunchEnv
void *tc_scratch(cudaStream_t s, size_t bytes);
// MXFP4 GEMV on the block-scaled tensor cores (gemv_mxf4_tc.cu), 1 <= M <= 8;
// MLQ_ERR_UNSUPPORTED when the shape / alignment is outside it
int launch_gemv_mxf4_tc(const uint8_t *W, const float *x, float *out, int n_rows, int K, int M, cudaStream_t s);
int launch_router_topk(const float *logits, int B, int E, int k, int renorm, int *idx, float *w, cudaStream_t s);

}  // namespace mlq
