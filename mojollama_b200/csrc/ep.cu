// Expert-parallel MoE building blocks (the MoE FFN of qwen36_batch_forward / moe_ffn,
// cengine_batch_instr.c:591-665 and :1113-1207, with the experts split over ranks).
//
// A rank owns experts [rank * E_local, (rank + 1) * E_local).  For T local tokens with
// top-k routing (idx [T][k] global expert ids, w [T][k]):
//   dispatch: slot s = t*k + i goes to rank idx[s] / E_local; the send buffer groups slots
//     by destination rank, and inside one destination keeps slot order (stable, so the
//     result does not depend on thread timing); it carries the token row x[t] and the
//     destination's local expert id;
//   experts:  every received row r is run through its one expert (no weight):
//     y[r] = down_e(silu(clamp(gate_e x_r)) * up_e x_r);
//   combine:  the rows come back in send order; out[t] = residual[t] + sum_i w[t][i] *
//     y[pos[t*k + i]], i = 0..k-1 in order.
// The exchanges themselves (all-to-all of counts, rows and ids) are NCCL collectives issued
// by the host (mojollama_b200/ep.py).
#include <cuda_runtime.h>

#include "mlq_internal.h"
#include "pipeline.cuh"

namespace mlq {

constexpr int kEpThreads = 1024;

// one CTA: counts[world], pos[T*k], send_eid[T*k] (stable by destination, then slot)
// cap > 0: fixed-capacity layout -- destination d's rows start at d * cap, and the slots
// beyond its count get id -1 (send_eid then has world * cap entries, eid_stride apart)
__global__ void __launch_bounds__(kEpThreads) k_ep_plan(const int *__restrict__ idx, int S, int e_local, int world,
                                                        int *__restrict__ counts, int *__restrict__ pos,
                                                        int *__restrict__ send_eid, int cap, int eid_stride) {
    __shared__ int warp_cnt[kEpThreads / 32][8];
    __shared__ int base[8];        // running start of each destination for the current chunk
    __shared__ int total[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    // pass 1: totals per destination
    if (tid < 8) total[tid] = 0;
    __syncthreads();
    for (int c0 = 0; c0 < S; c0 += blockDim.x) {
        const int s = c0 + tid;
        const int d = s < S ? idx[s] / e_local : -1;
        for (int r = 0; r < world; r++) {
            const unsigned m = __ballot_sync(0xffffffffu, d == r);
            if (lane == 0 && m) atomicAdd(&total[r], __popc(m));
        }
    }
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
        for (int r = 0; r < world; r++) {
            base[r] = cap > 0 ? r * cap : acc;
            if (counts) counts[r] = total[r];
            acc += total[r];
        }
    }
    __syncthreads();
    // pass 2: positions, chunk by chunk in slot order
    for (int c0 = 0; c0 < S; c0 += blockDim.x) {
        const int s = c0 + tid;
        const int g = s < S ? idx[s] : 0;
        const int d = s < S ? g / e_local : -1;
        int my_rank_in_warp = 0;
        for (int r = 0; r < world; r++) {
            const unsigned m = __ballot_sync(0xffffffffu, d == r);
            if (d == r) my_rank_in_warp = __popc(m & ((1u << lane) - 1u));
            if (lane == 0) warp_cnt[warp][r] = __popc(m);
        }
        __syncthreads();
        if (d >= 0) {
            int before = base[d] + my_rank_in_warp;
            for (int w2 = 0; w2 < warp; w2++) before += warp_cnt[w2][d];
            pos[s] = before;
            send_eid[(size_t)before * eid_stride] = g - d * e_local;
        }
        __syncthreads();
        if (tid < world) {
            int add = 0;
            for (int w2 = 0; w2 < nw; w2++) add += warp_cnt[w2][tid];
            base[tid] += add;
        }
        __syncthreads();
    }
    if (cap > 0) {   // unused rows of every destination: id -1 (the experts skip them)
        for (int r = 0; r < world; r++)
            for (int j = total[r] + tid; j < cap; j += blockDim.x) send_eid[((size_t)r * cap + j) * eid_stride] = -1;
    }
}

// send_x[pos[t*k + i]] = x[t]   (row stride `stride` floats in send_x)
__global__ void k_ep_gather(const float *__restrict__ x, const int *__restrict__ pos, int k, int N,
                            float *__restrict__ send_x, int stride) {
    const int s = blockIdx.x;
    const int t = s / k;
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * N);
    float4 *dst = reinterpret_cast<float4 *>(send_x + (size_t)pos[s] * stride);
    for (int i = threadIdx.x; i < N / 4; i += blockDim.x) dst[i] = src[i];
}

// out[t] = residual[t] + sum_i w[t][i] * y[pos[t*k + i]]   (i in order)
// out[t] = residual[t] + sum_i w[t k + i] y[pos[t k + i]]; with ys, then out[t] += score[t] ys[t]
// where score[t] > 0 (a shared expert's output, added after the routed ones as a separate step
// would add it)
__global__ void k_ep_combine(const float *__restrict__ y, const int *__restrict__ pos, const float *__restrict__ w,
                             int k, int N, const float *__restrict__ residual, float *__restrict__ out,
                             const float *__restrict__ ys, const float *__restrict__ score) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    const float sc = ys ? score[t] : 0.0f;
    for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < N; c += gridDim.y * blockDim.x) {
        float acc = residual ? residual[(size_t)t * N + c] : 0.0f;
        for (int i = 0; i < k; i++) {
            const int r = pos ? pos[t * k + i] : t * k + i;
            acc = fmaf(w[t * k + i], y[(size_t)r * N + c], acc);
        }
        if (ys && sc > 0.0f) acc = fmaf(sc, ys[(size_t)t * N + c], acc);
        out[(size_t)t * N + c] = acc;
    }
}

int launch_ep_combine(const float *y, const int *pos, const float *w, int T, int k, int N, const float *residual,
                      float *out, cudaStream_t s, const float *ys, const float *score) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(T, (N + 255) / 256);   // columns spread over CTAs: one token is 8 CTAs at N = 2048
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    count_launch();
    return MLQ_CUDA(cudaLaunchKernelEx(&cfg, k_ep_combine, y, pos, w, k, N, residual, out, ys, score)) ? MLQ_OK
                                                                                                      : MLQ_ERR_CUDA;
}

// ------------------------------------------------------------------ grouped routed experts
static void moe_grouped_tiles(int gqt, int uqt, int dqt, int n_ff, int N, int tiles[3], int &n_lists) {
    const int tg = grouped_tiles_per_expert(gqt, n_ff, N), tu = grouped_tiles_per_expert(uqt, n_ff, N);
    const int td = grouped_tiles_per_expert(dqt, N, n_ff);
    const bool pair = gqt == uqt;   // one type: one tiling, gate and up in one launch
    tiles[0] = pair ? tg + tu : tg;
    tiles[1] = pair ? td : tu;
    tiles[2] = td;
    n_lists = pair ? 2 : 3;
}

static size_t moe_grouped_layout(MoeGroupedScratch *m, uint8_t *base, int gqt, int uqt, int dqt, int R, int E,
                                 int n_ff, int N) {
    size_t o = 0;
    auto take = [&](size_t bytes) -> uint8_t * {
        uint8_t *p = base ? base + o : nullptr;
        o += (bytes + 255) & ~(size_t)255;
        return p;
    };
    int tiles[3], n_lists;
    moe_grouped_tiles(gqt, uqt, dqt, n_ff, N, tiles, n_lists);
    const int chunks = (R + 7) / 8 + (E < R ? E : R);
    MoeGroupedScratch t{};
    t.spos = (int *)take(sizeof(int) * (size_t)R);
    t.srow = (int *)take(sizeof(int) * (size_t)R);
    t.nitem = (int *)take(sizeof(int) * 4);
    for (int l = 0; l < 3; l++) t.items[l] = l < n_lists ? take(16 * (size_t)chunks * tiles[l]) : nullptr;
    t.px = take(grouped_packed_bytes(R, N));
    t.ph = take(grouped_packed_bytes(R, n_ff));
    t.g = (float *)take(sizeof(float) * (size_t)R * n_ff);
    t.u = (float *)take(sizeof(float) * (size_t)R * n_ff);
    t.xg = (__half *)take(tc_grouped_xh_bytes(R, N));
    t.xd = (__half *)take(tc_grouped_xh_bytes(R, n_ff));
    t.xgl = (__half *)take(tc_grouped_xh_bytes(R, N));
    t.xdl = (__half *)take(tc_grouped_xh_bytes(R, n_ff));
    t.sg = (float *)take(sizeof(float) * (size_t)R);
    t.sd = (float *)take(sizeof(float) * (size_t)R);
    if (gqt == MLQ_MXFP4 && uqt == MLQ_MXFP4 && dqt == MLQ_MXFP4) {
        t.bx = take(mxf4_planes_bytes(R, N));
        t.bh = take(mxf4_planes_bytes(R, n_ff));
    }
    if (m) *m = t;
    return o;
}

size_t moe_grouped_scratch_bytes(int gqt, int uqt, int dqt, int R, int E, int n_ff, int N) {
    return moe_grouped_layout(nullptr, nullptr, gqt, uqt, dqt, R, E, n_ff, N);
}

void moe_grouped_carve(MoeGroupedScratch &m, uint8_t *base, int gqt, int uqt, int dqt, int R, int E, int n_ff,
                       int N) {
    moe_grouped_layout(&m, base, gqt, uqt, dqt, R, E, n_ff, N);
}

// The tensor-core path for MXFP4 experts when the rows average at least MLQ_MOE_TC_ROWS per
// expert (default 0: off).  It is the more exact of the two (weights exact, activations as
// fp16 part + residual) but not yet the faster: at config 4, 64 tokens (8 rows per expert)
// its 128-row tiles ran at about the grouped GEMV's speed, 44.3 against 42.2 ms per step,
// bound like the dense tensor-core GEMM by the per-chunk decode / MMA / barrier sequence.
static bool moe_tc_wanted(int R, int E) {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("MLQ_MOE_TC_ROWS");
        v = e ? atoi(e) : 0;
    }
    return v > 0 && (long long)R >= (long long)v * E;
}

int launch_moe_grouped(int gqt, int uqt, int dqt, const uint8_t *gexp, const uint8_t *uexp, const uint8_t *dexp,
                       long long gstride, long long ustride, long long dstride, int E, const int *eid, int R,
                       int row_div, int n_ff, int N, const float *x, float *y, float clamp, const MoeGroupedScratch &m,
                       cudaStream_t s, int eid_stride, int x_stride) {
    if (R <= 0) return MLQ_OK;
    int tiles[3], n_lists;
    moe_grouped_tiles(gqt, uqt, dqt, n_ff, N, tiles, n_lists);
    if (!tiles[0] || !tiles[1] || !tiles[2]) {
        set_error(MLQ_ERR_UNSUPPORTED, "grouped experts: types %d/%d/%d with %d x %d", gqt, uqt, dqt, n_ff, N);
        return MLQ_ERR_UNSUPPORTED;
    }
    const bool pair = gqt == uqt;
    const int chunks = (R + 7) / 8 + (E < R ? E : R);
    void *items[3] = {m.items[0], m.items[1], m.items[2]};
    if (gqt == MLQ_MXFP4 && uqt == MLQ_MXFP4 && dqt == MLQ_MXFP4 && m.bx && m.bh) {
        // block-scaled tensor cores: 128-row tiles of E2M1 weights against the rows' E2M1 planes
        const int tg = (n_ff + 127) / 128, td = (N + 127) / 128;
        if (mxf4_grouped_wanted(R, E, 2 * tg) && mxf4_grouped_supported(gexp, gstride, E, n_ff, N) &&
            mxf4_grouped_supported(uexp, ustride, E, n_ff, N) && mxf4_grouped_supported(dexp, dstride, E, N, n_ff)) {
            int tt[2] = {2 * tg, td};
            int rc = launch_group_plan(eid, R, E, 2, items, tt, m.spos, m.srow, m.nitem, s, eid_stride);
            if (rc == MLQ_OK)
                rc = launch_mxf4_planes_rows(x, nullptr, m.srow, row_div, x_stride > 0 ? x_stride : N, 0.0f, R, N, m.bx,
                                             s);
            if (rc == MLQ_OK)
                rc = launch_moe_mxf4_tc(gexp, gstride, uexp, ustride, E, n_ff, N, items[0], m.nitem, chunks * tt[0], m.bx,
                                        R, m.g, m.u, nullptr, s);
            if (rc == MLQ_OK) rc = launch_mxf4_planes_rows(m.g, m.u, nullptr, 1, n_ff, clamp, R, n_ff, m.bh, s);
            if (rc == MLQ_OK)
                rc = launch_moe_mxf4_tc(dexp, dstride, nullptr, 0, E, N, n_ff, items[1], m.nitem + 1, chunks * tt[1],
                                        m.bh, R, y, nullptr, m.srow, s);
            return rc;
        }
    }
    // (MXFP4 experts only: their E2M1 x 2^e weights are exact in fp16 relative to each chunk's
    // largest block, and the activations enter as an fp16 part plus its fp16 residual, so the
    // products are as exact as fp32 sums make them; K-quant weights would be rounded to fp16)
    if (gqt == MLQ_MXFP4 && uqt == MLQ_MXFP4 && dqt == MLQ_MXFP4 && moe_tc_wanted(R, E) &&
        tc_grouped_supported(gqt, gexp, gstride, N) &&
        tc_grouped_supported(uqt, uexp, ustride, N) && tc_grouped_supported(dqt, dexp, dstride, n_ff)) {
        // many rows per expert: 128-row tiles on the tensor cores (fp16 operands, fp32 sums)
        const int tg = (n_ff + 127) / 128, td = (N + 127) / 128;
        int tt[3] = {pair ? 2 * tg : tg, pair ? td : tg, td};
        int rc = launch_group_plan(eid, R, E, n_lists, items, tt, m.spos, m.srow, m.nitem, s, eid_stride);
        if (rc == MLQ_OK) rc = launch_rows_to_f16(x, nullptr, m.srow, row_div, x_stride > 0 ? x_stride : N, 0.0f, R, N,
                                                  m.xg, m.xgl, m.sg, s);
        if (rc == MLQ_OK)
            rc = launch_gemm_tc_grouped(gqt, gexp, gstride, pair ? uexp : nullptr, ustride, n_ff, N, items[0], m.nitem,
                                        chunks * tt[0], m.xg, m.xgl, m.sg, m.g, pair ? m.u : nullptr, nullptr, s);
        if (rc == MLQ_OK && !pair)
            rc = launch_gemm_tc_grouped(uqt, uexp, ustride, nullptr, 0, n_ff, N, items[1], m.nitem + 1, chunks * tt[1],
                                        m.xg, m.xgl, m.sg, m.u, nullptr, nullptr, s);
        if (rc == MLQ_OK) rc = launch_rows_to_f16(m.g, m.u, nullptr, 1, n_ff, clamp, R, n_ff, m.xd, m.xdl, m.sd, s);
        if (rc == MLQ_OK)
            rc = launch_gemm_tc_grouped(dqt, dexp, dstride, nullptr, 0, N, n_ff, items[n_lists - 1],
                                        m.nitem + n_lists - 1, chunks * tt[n_lists - 1], m.xd, m.xdl, m.sd, y, nullptr,
                                        m.srow, s);
        return rc;
    }
    int rc = launch_group_plan(eid, R, E, n_lists, items, tiles, m.spos, m.srow, m.nitem, s, eid_stride);
    if (rc == MLQ_OK) rc = launch_encode_packed(x, nullptr, m.srow, R, N, m.px, s, row_div, 80.0f, x_stride);
    GroupedCall gc{};
    gc.planes = m.px;
    gc.n_rows = n_ff;
    gc.K = N;
    if (rc == MLQ_OK) {
        gc.qt = gqt; gc.W = gexp; gc.estride = gstride; gc.out = m.g;
        gc.items = items[0]; gc.n_items_dev = m.nitem; gc.n_items_bound = chunks * tiles[0];
        if (pair) { gc.W2 = uexp; gc.estride2 = ustride; gc.out2 = m.u; }
        rc = launch_grouped(gc, s);
    }
    if (rc == MLQ_OK && !pair) {
        gc.qt = uqt; gc.W = uexp; gc.estride = ustride; gc.out = m.u;
        gc.items = items[1]; gc.n_items_dev = m.nitem + 1; gc.n_items_bound = chunks * tiles[1];
        rc = launch_grouped(gc, s);
    }
    if (rc == MLQ_OK) rc = launch_encode_packed(m.g, m.u, nullptr, R, n_ff, m.ph, s, 1, clamp);
    if (rc == MLQ_OK) {
        GroupedCall dc{};
        dc.qt = dqt; dc.W = dexp; dc.estride = dstride; dc.out = y;
        dc.items = items[n_lists - 1]; dc.n_items_dev = m.nitem + n_lists - 1; dc.n_items_bound = chunks * tiles[n_lists - 1];
        dc.planes = m.ph; dc.out_rows = m.srow;
        dc.n_rows = N;
        dc.K = n_ff;
        rc = launch_grouped(dc, s);
    }
    return rc;
}

}  // namespace mlq

using namespace mlq;

extern "C" {

int mlq_ep_dispatch(const int *idx, int T, int k, int experts_per_rank, int world, const float *x, int N, int *counts,
                    int *pos, float *send_x, int *send_eid) {
    if (!idx || !x || !counts || !pos || !send_x || !send_eid || T <= 0 || k <= 0 || experts_per_rank <= 0 ||
        world <= 0 || world > 8 || N <= 0 || N % 4) {
        set_error(MLQ_ERR_ARG, "ep_dispatch: bad arguments (world 1..8, N %% 4 == 0)");
        return MLQ_ERR_ARG;
    }
    if (!is_device_ptr(idx) || !is_device_ptr(x) || !is_device_ptr(send_x)) {
        set_error(MLQ_ERR_ARG, "ep_dispatch: device pointers only");
        return MLQ_ERR_ARG;
    }
    cudaStream_t s = stream();
    const int S = T * k;
    k_ep_plan<<<1, kEpThreads, 0, s>>>(idx, S, experts_per_rank, world, counts, pos, send_eid, 0, 1);
    k_ep_gather<<<S, 128, 0, s>>>(x, pos, k, N, send_x, N);
    count_launch(2);
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

// Fixed-capacity dispatch for an exchange with equal splits (no count read back to the
// host): send [world][cap][N + 4] floats; the rows for destination d are at d * cap + j in
// slot order (stable), each row carries the destination-local expert id in-band at column
// N (as int bits), rows beyond d's count carry id -1.  pos[t*k + i] = d * cap + j, where the
// result of that slot comes back after the return exchange.  cap >= T * min(k, experts
// per rank) always suffices (a token sends at most one row per local expert of a peer).
int mlq_ep_dispatch_packed(const int *idx, int T, int k, int experts_per_rank, int world, int cap, const float *x,
                           int N, int *pos, float *send) {
    if (!idx || !x || !pos || !send || T <= 0 || k <= 0 || experts_per_rank <= 0 || world <= 0 || world > 8 ||
        N <= 0 || N % 4 || cap < T * (k < experts_per_rank ? k : experts_per_rank)) {
        set_error(MLQ_ERR_ARG, "ep_dispatch_packed: bad arguments (world 1..8, N %% 4 == 0, cap >= T * min(k, E/world))");
        return MLQ_ERR_ARG;
    }
    if (!is_device_ptr(idx) || !is_device_ptr(x) || !is_device_ptr(send)) {
        set_error(MLQ_ERR_ARG, "ep_dispatch_packed: device pointers only");
        return MLQ_ERR_ARG;
    }
    cudaStream_t s = stream();
    const int S = T * k, stride = N + 4;
    k_ep_plan<<<1, kEpThreads, 0, s>>>(idx, S, experts_per_rank, world, nullptr, pos,
                                       reinterpret_cast<int *>(send) + N, cap, stride);
    k_ep_gather<<<S, 128, 0, s>>>(x, pos, k, N, send, stride);
    count_launch(2);
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

int mlq_ep_combine(const float *recv_y, const int *pos, const float *w, int T, int k, int N, const float *residual,
                   float *out) {
    if (!recv_y || !pos || !w || !out || T <= 0 || k <= 0 || N <= 0) {
        set_error(MLQ_ERR_ARG, "ep_combine: bad arguments");
        return MLQ_ERR_ARG;
    }
    return launch_ep_combine(recv_y, pos, w, T, k, N, residual, out, stream());
}

// y[r] = down_e(silu(clamp(gate_e x_r, +-80)) * up_e x_r) for the local expert e = eid[r]
// (0 <= e < n_experts <= 1024; rows with another id are left unwritten); expert tensors
// are [n_experts][rows][cols] at the given byte strides (device memory).  The planner
// orders the rows by expert (stable) and lists the work items; the rows of x are encoded
// once in that order; the gate and up matrices of every active expert are streamed once
// for all of its rows (one launch when they share a type); silu(clamp(g)) * u is encoded
// the same way; the down matrices then write y in the callers' row order.
int mlq_moe_rows(int gqt, int uqt, int dqt, const void *gexp, const void *uexp, const void *dexp, long long gstride,
                 long long ustride, long long dstride, int n_experts, const int *eid, int R, int n_ff, int N,
                 const float *x, float *y) {
    if (R < 0 || !eid || !x || !y || !gexp || !uexp || !dexp || n_ff <= 0 || N <= 0 || n_experts <= 0 || N % 32 ||
        n_ff % 32) {
        set_error(MLQ_ERR_ARG, "moe_rows: bad arguments");
        return MLQ_ERR_ARG;
    }
    if (R == 0) return MLQ_OK;
    if (!grouped_tiles_per_expert(gqt, n_ff, N) || !grouped_tiles_per_expert(uqt, n_ff, N) ||
        !grouped_tiles_per_expert(dqt, N, n_ff)) {
        set_error(MLQ_ERR_TYPE, "moe_rows: expert types %d/%d/%d", gqt, uqt, dqt);
        return MLQ_ERR_TYPE;
    }
    CallScope cs;
    uint8_t *scr = (uint8_t *)cs.scratch(moe_grouped_scratch_bytes(gqt, uqt, dqt, R, n_experts, n_ff, N));
    if (cs.failed) return cs.finish();
    MoeGroupedScratch m;
    moe_grouped_carve(m, scr, gqt, uqt, dqt, R, n_experts, n_ff, N);
    int rc = launch_moe_grouped(gqt, uqt, dqt, (const uint8_t *)gexp, (const uint8_t *)uexp, (const uint8_t *)dexp,
                                gstride, ustride, dstride, n_experts, eid, R, 1, n_ff, N, x, y, 80.0f, m, stream());
    if (rc != MLQ_OK) {
        cs.failed = true;
        cs.finish();
        return rc;
    }
    return cs.finish();
}

// mlq_moe_rows over packed exchange rows: recv [R][N + 4] floats, the local expert id
// in-band at column N (rows with id -1, or any id outside [0, n_experts), are skipped).
int mlq_moe_rows_packed(int gqt, int uqt, int dqt, const void *gexp, const void *uexp, const void *dexp,
                        long long gstride, long long ustride, long long dstride, int n_experts, const float *recv,
                        int R, int n_ff, int N, float *y) {
    if (R < 0 || !recv || !y || !gexp || !uexp || !dexp || n_ff <= 0 || N <= 0 || n_experts <= 0 || N % 32 ||
        n_ff % 32) {
        set_error(MLQ_ERR_ARG, "moe_rows_packed: bad arguments");
        return MLQ_ERR_ARG;
    }
    if (R == 0) return MLQ_OK;
    if (!grouped_tiles_per_expert(gqt, n_ff, N) || !grouped_tiles_per_expert(uqt, n_ff, N) ||
        !grouped_tiles_per_expert(dqt, N, n_ff)) {
        set_error(MLQ_ERR_TYPE, "moe_rows_packed: expert types %d/%d/%d", gqt, uqt, dqt);
        return MLQ_ERR_TYPE;
    }
    CallScope cs;
    uint8_t *scr = (uint8_t *)cs.scratch(moe_grouped_scratch_bytes(gqt, uqt, dqt, R, n_experts, n_ff, N));
    if (cs.failed) return cs.finish();
    MoeGroupedScratch m;
    moe_grouped_carve(m, scr, gqt, uqt, dqt, R, n_experts, n_ff, N);
    const int stride = N + 4;
    int rc = launch_moe_grouped(gqt, uqt, dqt, (const uint8_t *)gexp, (const uint8_t *)uexp, (const uint8_t *)dexp,
                                gstride, ustride, dstride, n_experts, reinterpret_cast<const int *>(recv) + N, R, 1,
                                n_ff, N, recv, y, 80.0f, m, stream(), stride, stride);
    if (rc != MLQ_OK) {
        cs.failed = true;
        cs.finish();
        return rc;
    }
    return cs.finish();
}

}  // extern "C"
