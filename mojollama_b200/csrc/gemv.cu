// Quantized GEMV / skinny GEMM (B <= 8 activation rows per launch) for sm_100a.
//
// Replaces the reference's per-format OpenMP row loops
// (quant_kernels_omp.c:135-734 *_matmul_omp, 1355-1388 quant_matmul_omp;
//  cengine_batch_instr.c:68-534 *_batch_matmul).
//
// Data layout in HBM: W is the GGUF tensor as-is, rows of K/BE blocks back to back,
// so the whole matrix is one contiguous byte stream of N*row_bytes.  A persistent
// CTA walks tiles of `rpt` rows; each tile is a contiguous byte range.
//
// CTA = 9 warps, one CTA per SM.  Warp 8 is the producer: it streams each tile's
// 16-byte-aligned interior into a shared-memory ring of up to 8 stages (as many as
// fit in ~220 KB) with one cp.async.bulk (TMA engine, L2 evict_first) per tile and
// fetches the <=15-byte ragged head/tail with plain loads; full/empty mbarriers hand
// stages to the 8 decode warps.  The decode warps first encode the activation rows
// as int8 "x planes" (formats.cuh) in shared memory, then decode weight blocks
// straight from the staged bytes into packed int8 and reduce with dp4a, fp32
// per-block scaling and warp shuffles.
//   k_gemv_q1  (M = 1, many rows): 16 decode warps, 1-2 rows each per tile; each
//              lane keeps its activation slices in registers for the whole kernel.
//   k_gemv_q   (any M <= 8): activation slices from shared memory; when a tile holds
//              fewer than 8 rows, 8/rpt warps split each row and combine through smem.
//
// Roofline: HBM-bound.  Algorithmic bytes per launch = N*row_bytes + B*K*4 + B*N*4.
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "formats.cuh"
#include "mlq_internal.h"
#include "pipeline.cuh"
#include <stdlib.h>

namespace mlq {

static constexpr int kMaxStages = 8;
static constexpr int kConsumerWarps = 8;
static constexpr int kThreads = (kConsumerWarps + 1) * 32;
static constexpr int kMaxSmem = 232448;      // 227 KB opt-in per CTA on sm_100
static constexpr int kSmemBudget = 220 * 1024;
static constexpr int kStageTarget = 24576;   // bytes of weights per stage (generic path)
static constexpr int kFastWarps = 16;        // decode warps of the M=1 kernel (1 row each per tile)
static constexpr int kFastThreads = (kFastWarps + 1) * 32;

int block_elems(int qt) {
    switch (qt) {
        case MLQ_F32: case MLQ_F16: case MLQ_BF16: return 1;
        case MLQ_Q4_0: case MLQ_Q4_1: case MLQ_Q5_0: case MLQ_Q8_0: case MLQ_MXFP4: case MLQ_MXFP4_REF: return 32;
        case MLQ_Q4_K: case MLQ_Q5_K: case MLQ_Q6_K: return 256;
        default: return 0;
    }
}

int block_bytes(int qt) {
    switch (qt) {
        case MLQ_F32: return 4;
        case MLQ_F16: case MLQ_BF16: return 2;
        case MLQ_Q4_0: return 18;
        case MLQ_Q4_1: return 20;
        case MLQ_Q5_0: return 22;
        case MLQ_Q8_0: return 34;
        case MLQ_MXFP4: case MLQ_MXFP4_REF: return 17;
        case MLQ_Q4_K: return 144;
        case MLQ_Q5_K: return 176;
        case MLQ_Q6_K: return 210;
        default: return 0;
    }
}

bool is_quant_type(int qt) { return block_elems(qt) > 1; }

struct GemvArgs {
    const uint8_t *W;
    const float *x;
    float *out;
    int n_rows, K, nb_x;
    long long row_bytes, total_bytes;
    int rpt, wpr, n_tiles, stage_bytes, n_stages;
    int *status;
};

struct GemvLayout {
    int off_bar, off_flag, off_xh, off_xl, off_xs, off_xsum, off_red, off_stage, total;
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline GemvLayout gemv_layout(int M, int K, int stage_bytes, int n_stages) {
    GemvLayout L;
    int o = 0;
    L.off_bar = o;  o += 2 * kMaxStages * 8;
    L.off_flag = o; o += 16;
    o = align_up(o, 128);
    L.off_xh = o;   o = align_up(o + M * K, 16);
    L.off_xl = o;   o = align_up(o + M * K, 16);
    L.off_xs = o;   o += M * (K / 32) * 4;
    L.off_xsum = o; o = align_up(o + M * (K / 32) * 4, 16);
    L.off_red = o;  o = align_up(o + 2 * kConsumerWarps * M * 4, 128);
    L.off_stage = o; o += n_stages * stage_bytes;
    L.total = o;
    return L;
}

__device__ __forceinline__ void raise_status(int *status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// Producer warp: stream tile it of this CTA into stage it % n_stages.  The tile's
// 16-byte-aligned interior goes through one cp.async.bulk (TMA engine, L2
// evict_first); the <= 15-byte ragged head and tail are plain loads by the lanes.
__device__ __forceinline__ void produce_tiles(const GemvArgs &a, uint8_t *stages, uint64_t *full, uint64_t *empty,
                                              volatile int *abort_flag, int n_iter, int lane) {
    const uint64_t pol = policy_evict_first();
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    for (int it = 0; it < n_iter; ++it) {
        const int s = it % a.n_stages;
        if (it >= a.n_stages) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait_bounded(&empty[s], ((it / a.n_stages) - 1) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *abort_flag) {
                if (lane == 0) { *abort_flag = 1; raise_status(a.status, DEV_ST_WAIT_EMPTY); }
                return;
            }
        }
        const long long tile = (long long)blockIdx.x + (long long)it * gridDim.x;
        const long long b0 = tile * tile_bytes;
        const long long b1 = min(b0 + tile_bytes, a.total_bytes);
        const uintptr_t g0 = reinterpret_cast<uintptr_t>(a.W) + (uintptr_t)b0;
        const uintptr_t g1 = reinterpret_cast<uintptr_t>(a.W) + (uintptr_t)b1;
        const uintptr_t gd = g0 & ~uintptr_t(15);
        const uintptr_t i0 = (g0 + 15) & ~uintptr_t(15);
        const uintptr_t i1 = g1 & ~uintptr_t(15);
        uint8_t *st = stages + (size_t)s * a.stage_bytes;
        if (i1 > i0) {
            if (g0 + lane < i0) st[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
            if (i1 + lane < g1) st[i1 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(i1 + lane));
        } else {
            if (g0 + lane < g1) st[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
        }
        __syncwarp();
        if (lane == 0) {
            if (i1 > i0) {
                mbar_arrive_expect_tx(&full[s], (uint32_t)(i1 - i0));
                bulk_g2s(st + (i0 - gd), reinterpret_cast<const void *>(i0), (uint32_t)(i1 - i0), &full[s], pol);
            } else {
                mbar_arrive(&full[s]);
            }
        }
    }
}

// Before waiting on the previous kernel (programmatic dependent launch), the producer
// warp prefetches this CTA's first tiles into L2: the bytes are only read later, after
// the wait, so a tile the previous kernel is still writing is read correctly.
__device__ __forceinline__ void prefetch_first_tiles(const GemvArgs &a, int n_iter, int lane) {
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    const int n = n_iter < a.n_stages ? n_iter : a.n_stages;
    if (lane < n) {
        const long long tile = (long long)blockIdx.x + (long long)lane * gridDim.x;
        const long long b0 = tile * tile_bytes, b1 = min(b0 + tile_bytes, a.total_bytes);
        const uintptr_t g0 = reinterpret_cast<uintptr_t>(a.W) + (uintptr_t)b0;
        const uintptr_t g1 = reinterpret_cast<uintptr_t>(a.W) + (uintptr_t)b1;
        const uintptr_t i0 = (g0 + 15) & ~uintptr_t(15), i1 = g1 & ~uintptr_t(15);
        if (i1 > i0) prefetch_l2(reinterpret_cast<const void *>(i0), (uint32_t)(i1 - i0));
    }
}

// decode warps: bounded wait for stage s of iteration it; false on timeout/abort
__device__ __forceinline__ bool consume_wait(const GemvArgs &a, uint64_t *full, volatile int *abort_flag, int it,
                                             int lane) {
    if (*abort_flag) return false;
    bool ok = true;
    if (lane == 0) ok = mbar_wait_bounded(&full[it % a.n_stages], (it / a.n_stages) & 1);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok && lane == 0) { *abort_flag = 1; raise_status(a.status, DEV_ST_WAIT_FULL); }
    return ok;
}

__device__ __forceinline__ void init_barriers(uint64_t *full, uint64_t *empty, volatile int *abort_flag, int n_stages,
                                              int n_consumers) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < n_stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], n_consumers);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
}

// ---------------------------------------------------------------- generic kernel (any M <= 8)
// 8/rpt decode warps share each row of a tile when the matrix has few rows.
template <int QT, int M>
__global__ void __launch_bounds__(kThreads, 1) k_gemv_q(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvLayout L = gemv_layout(M, a.K, a.stage_bytes, a.n_stages);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kMaxStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.off_flag);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_iter = (a.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    if (warp == kConsumerWarps) prefetch_first_tiles(a, n_iter, lane);
    init_barriers(full, empty, abort_flag, a.n_stages, kConsumerWarps);
    pdl_wait();
    pdl_trigger();
    if (warp == kConsumerWarps) {
        produce_tiles(a, smem + L.off_stage, full, empty, abort_flag, n_iter, lane);
        return;
    }
    int8_t *xh = reinterpret_cast<int8_t *>(smem + L.off_xh);
    int8_t *xl = reinterpret_cast<int8_t *>(smem + L.off_xl);
    float *xs = reinterpret_cast<float *>(smem + L.off_xs);
    float *xsum = reinterpret_cast<float *>(smem + L.off_xsum);
    float *red = reinterpret_cast<float *>(smem + L.off_red);
    encode_x_planes<M>(a.x, a.nb_x, a.K, xh, xl, xs, xsum, warp, lane, kConsumerWarps);
    named_bar_sync(1, kConsumerWarps * 32);

    XPlanes xp{xh, xl, xs, xsum, a.K};
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    const int rr = warp / a.wpr, part = warp - rr * a.wpr;
    const int U = a.K / Fmt<QT>::UE;
    for (int it = 0; it < n_iter; ++it) {
        const int s = it % a.n_stages;
        const bool ok = consume_wait(a, full, abort_flag, it, lane);
        const long long tile = (long long)blockIdx.x + (long long)it * gridDim.x;
        const int row0 = (int)(tile * a.rpt);
        const int row = row0 + rr;
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; m++) acc[m] = 0.0f;
        if (ok && row < a.n_rows) {
            const uintptr_t g0 = reinterpret_cast<uintptr_t>(a.W) + (uintptr_t)(tile * tile_bytes);
            const uint8_t *rowp = smem + L.off_stage + (size_t)s * a.stage_bytes + (g0 & 15) + (size_t)rr * a.row_bytes;
            for (int u = part * 32 + lane; u < U; u += 32 * a.wpr) Unit<QT, M>::dot(rowp, u, xp, acc);
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(&empty[s]);
        if (a.wpr == 1) {
            if (lane == 0 && ok && row < a.n_rows) {
#pragma unroll
                for (int m = 0; m < M; m++)
                    if (m < a.nb_x) a.out[(size_t)m * a.n_rows + row] = acc[m];
            }
        } else {
            float *rd = red + (it & 1) * kConsumerWarps * M;
            if (lane == 0) {
#pragma unroll
                for (int m = 0; m < M; m++) rd[warp * M + m] = acc[m];
            }
            named_bar_sync(1, kConsumerWarps * 32);
            if ((int)threadIdx.x < a.rpt * M && ok) {
                const int r = threadIdx.x / M, m = threadIdx.x - r * M;
                float sum = 0.0f;
                for (int p = 0; p < a.wpr; p++) sum += rd[(r * a.wpr + p) * M + m];
                if (row0 + r < a.n_rows && m < a.nb_x) a.out[(size_t)m * a.n_rows + row0 + r] = sum;
            }
        }
    }
}

// ---------------------------------------------------------------- M = 1 decode kernel
// kFastWarps decode warps each own RW rows of every tile (rows w, w+16, ...), and
// each lane always handles units lane, lane+32, ... of a row, so the lane's
// activation slices XU are loaded into registers once and reused for every row the
// CTA streams.  UPL = units per lane (ceil(K/UE/32)); A16 = rows start on 16-byte
// boundaries in shared memory (Q4_K/Q5_K then use 128-bit loads); RW = rows per
// warp per tile (independent decode chains for latency hiding).
template <int QT, int UPL, bool A16, int RW>
__global__ void __launch_bounds__(kFastThreads, 1) k_gemv_q1(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvLayout L = gemv_layout(1, a.K, a.stage_bytes, a.n_stages);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kMaxStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.off_flag);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_iter = (a.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    if (warp == kFastWarps) prefetch_first_tiles(a, n_iter, lane);
    init_barriers(full, empty, abort_flag, a.n_stages, kFastWarps);
    pdl_wait();
    pdl_trigger();
    if (warp == kFastWarps) {
        produce_tiles(a, smem + L.off_stage, full, empty, abort_flag, n_iter, lane);
        return;
    }
    int8_t *xh = reinterpret_cast<int8_t *>(smem + L.off_xh);
    int8_t *xl = reinterpret_cast<int8_t *>(smem + L.off_xl);
    float *xs = reinterpret_cast<float *>(smem + L.off_xs);
    float *xsum = reinterpret_cast<float *>(smem + L.off_xsum);
    encode_x_planes<1>(a.x, 1, a.K, xh, xl, xs, xsum, warp, lane, kFastWarps);
    named_bar_sync(1, kFastWarps * 32);
    const XPlanes xp{xh, xl, xs, xsum, a.K};
    const int U = a.K / Fmt<QT>::UE;
    XU<QT> xu[UPL];
#pragma unroll
    for (int j = 0; j < UPL; j++) {
        const int u = lane + 32 * j;
        if (u < U) load_xu<QT>(xp, 0, u, xu[j]);
    }
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    for (int it = 0; it < n_iter; ++it) {
        const int s = it % a.n_stages;
        const bool ok = consume_wait(a, full, abort_flag, it, lane);
        const long long tile = (long long)blockIdx.x + (long long)it * gridDim.x;
        const int row0 = (int)(tile * a.rpt) + warp;
        const uintptr_t g0 = reinterpret_cast<uintptr_t>(a.W) + (uintptr_t)(tile * tile_bytes);
        const uint8_t *st = smem + L.off_stage + (size_t)s * a.stage_bytes + (g0 & 15);
        float acc[RW];
#pragma unroll
        for (int r = 0; r < RW; r++) acc[r] = 0.0f;
        if (ok) {
#pragma unroll
            for (int j = 0; j < UPL; j++) {
                const int u = lane + 32 * j;
                if (u < U) {
#pragma unroll
                    for (int r = 0; r < RW; r++) {
                        // rows warp, warp + 16, ...: row r of this warp within the tile
                        if (row0 + kFastWarps * r < a.n_rows) {
                            const uint8_t *rowp = st + (size_t)(warp + kFastWarps * r) * a.row_bytes;
                            W<QT> w;
                            if constexpr (A16) w.decode_a16(rowp, u);
                            else w.decode(rowp, u);
                            acc[r] += w.dot(xu[j]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RW; r++) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        }
        __syncwarp();
        if (lane == 0 && ok) {
            mbar_arrive(&empty[s]);
#pragma unroll
            for (int r = 0; r < RW; r++)
                if (row0 + kFastWarps * r < a.n_rows) a.out[row0 + kFastWarps * r] = acc[r];
        }
    }
}

// fp32 / fp16 / bf16 weights: one warp per row, 16-byte vector loads.
template <typename WT> __device__ __forceinline__ float to_f(WT v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename WT, int M>
__global__ void __launch_bounds__(256) k_gemv_float(const WT *__restrict__ W, const float *__restrict__ x,
                                                    float *__restrict__ out, int n_rows, int K, int nb_x,
                                                    int vec_ok) {
    constexpr int V = 16 / sizeof(WT);
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int row = gw; row < n_rows; row += nw) {
        const WT *wr = W + (size_t)row * K;
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; m++) acc[m] = 0.0f;
        if (vec_ok) {
            for (int k0 = lane * V; k0 < K; k0 += 32 * V) {
                union { int4 v; WT e[V]; } wv;
                wv.v = __ldcs(reinterpret_cast<const int4 *>(wr + k0));
#pragma unroll
                for (int m = 0; m < M; m++) {
                    if (m < nb_x) {
                        const float *xr = x + (size_t)m * K + k0;
#pragma unroll
                        for (int j = 0; j < V; j += 4) {
                            const float4 xv = __ldg(reinterpret_cast<const float4 *>(xr + j));
                            acc[m] = fmaf(to_f<WT>(wv.e[j + 0]), xv.x, acc[m]);
                            acc[m] = fmaf(to_f<WT>(wv.e[j + 1]), xv.y, acc[m]);
                            acc[m] = fmaf(to_f<WT>(wv.e[j + 2]), xv.z, acc[m]);
                            acc[m] = fmaf(to_f<WT>(wv.e[j + 3]), xv.w, acc[m]);
                        }
                    }
                }
            }
        } else {
            for (int k = lane; k < K; k += 32) {
                const float wv = to_f<WT>(wr[k]);
#pragma unroll
                for (int m = 0; m < M; m++)
                    if (m < nb_x) acc[m] = fmaf(wv, __ldg(x + (size_t)m * K + k), acc[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
        }
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < M; m++)
                if (m < nb_x) out[(size_t)m * n_rows + row] = acc[m];
        }
    }
}

// ------------------------------------------------------------------------------ launchers
// Launch with programmatic stream serialization: the kernel may start while the previous
// kernel on the stream finishes; it calls pdl_wait() before touching anything that kernel
// writes.  MLQ_NO_PDL=1 launches normally.
static bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("MLQ_NO_PDL");
        v = (e && atoi(e) != 0) ? 0 : 1;
    }
    return v == 1;
}

template <typename Kern, typename Args>
static cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, int smem, cudaStream_t s, const Args &args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args);
}

static int stages_for(int fixed, int stage_bytes) {
    int n = (kSmemBudget - fixed) / stage_bytes;
    return n > kMaxStages ? kMaxStages : n;
}

template <typename Kern>
static int launch_gemv_kernel(Kern kern, GemvArgs &a, int smem, cudaStream_t s, bool &attr_set,
                              int threads = kThreads) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    if (!attr_set) {
        if (!MLQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem)))
            return MLQ_ERR_CUDA;
        attr_set = true;
    }
    int per_sm = 0;
    if (!MLQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem))) return MLQ_ERR_CUDA;
    if (per_sm < 1) per_sm = 1;
    a.status = c->d_status;
    const int grid = a.n_tiles < per_sm * c->num_sms ? a.n_tiles : per_sm * c->num_sms;
    count_launch();
    return MLQ_CUDA(launch_pdl(kern, dim3(grid), dim3(threads), smem, s, a)) ? MLQ_OK : MLQ_ERR_CUDA;
}

template <int QT, int M>
static int launch_q_m(const uint8_t *W, const float *x, float *out, int n_rows, int K, int nb_x, cudaStream_t s) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    const long long rb = (long long)(K / Fmt<QT>::BE) * Fmt<QT>::BB;
    int rpt = (int)(kStageTarget / rb);
    rpt = rpt < 1 ? 1 : (rpt > 8 ? 8 : rpt);
    rpt = rpt >= 8 ? 8 : rpt >= 4 ? 4 : rpt >= 2 ? 2 : 1;
    while (rpt > 1 && (n_rows + rpt - 1) / rpt < 2 * c->num_sms) rpt >>= 1;
    const int stage_bytes = align_up((int)(rpt * rb), 16) + 48;
    const int fixed = gemv_layout(M, K, stage_bytes, 0).total;
    const int n_stages = stages_for(fixed, stage_bytes);
    if (n_stages < 2) return MLQ_ERR_CAPACITY;
    GemvArgs a{};
    a.W = W; a.x = x; a.out = out; a.n_rows = n_rows; a.K = K; a.nb_x = nb_x;
    a.row_bytes = rb; a.total_bytes = rb * n_rows; a.rpt = rpt; a.wpr = kConsumerWarps / rpt;
    a.n_tiles = (n_rows + rpt - 1) / rpt; a.stage_bytes = stage_bytes; a.n_stages = n_stages;
    static bool attr_set = false;
    return launch_gemv_kernel(k_gemv_q<QT, M>, a, fixed + n_stages * stage_bytes, s, attr_set);
}

// rows per decode warp per tile of the M=1 kernel, per format (MLQ_GEMV_RW overrides)
template <int QT> static int fast_rw() {
    const char *e = getenv("MLQ_GEMV_RW");
    if (e && (atoi(e) == 1 || atoi(e) == 2)) return atoi(e);
    return 2;
}

template <int QT, int UPL, int RW>
static int launch_q1_rw(const uint8_t *W, const float *x, float *out, int n_rows, int K, cudaStream_t s) {
    const long long rb = (long long)(K / Fmt<QT>::BE) * Fmt<QT>::BB;
    const int rpt = kFastWarps * RW;
    const int stage_bytes = align_up((int)(rpt * rb), 16) + 48;
    const int fixed = gemv_layout(1, K, stage_bytes, 0).total;
    const int n_stages = stages_for(fixed, stage_bytes);
    if (n_stages < 3) return MLQ_ERR_CAPACITY;
    GemvArgs a{};
    a.W = W; a.x = x; a.out = out; a.n_rows = n_rows; a.K = K; a.nb_x = 1;
    a.row_bytes = rb; a.total_bytes = rb * n_rows; a.rpt = rpt; a.wpr = 1;
    a.n_tiles = (n_rows + rpt - 1) / rpt; a.stage_bytes = stage_bytes; a.n_stages = n_stages;
    const int smem = fixed + n_stages * stage_bytes;
    constexpr bool kCanAlign = (QT == MLQ_Q4_K || QT == MLQ_Q5_K);
    if constexpr (kCanAlign) {
        if (rb % 16 == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0) {
            static bool attr_a = false;
            return launch_gemv_kernel(k_gemv_q1<QT, UPL, true, RW>, a, smem, s, attr_a, kFastThreads);
        }
    }
    static bool attr_set = false;
    return launch_gemv_kernel(k_gemv_q1<QT, UPL, false, RW>, a, smem, s, attr_set, kFastThreads);
}

template <int QT, int UPL>
static int launch_q1_fast(const uint8_t *W, const float *x, float *out, int n_rows, int K, cudaStream_t s) {
    if (fast_rw<QT>() == 2) return launch_q1_rw<QT, UPL, 2>(W, x, out, n_rows, K, s);
    return launch_q1_rw<QT, UPL, 1>(W, x, out, n_rows, K, s);
}

// M = 1 over many rows: the register-resident kernel; returns MLQ_ERR_UNSUPPORTED
// when the shape does not suit it (few rows, or too many units per lane).
template <int QT>
static int launch_q1(const uint8_t *W, const float *x, float *out, int n_rows, int K, cudaStream_t s) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    const int U = K / Fmt<QT>::UE;
    const int upl = (U + 31) / 32;
    if (n_rows < 8 * c->num_sms * kFastWarps || getenv("MLQ_GEMV_GENERIC")) return MLQ_ERR_UNSUPPORTED;
    // only the variants that stay inside the 96 registers a 544-thread CTA allows:
    // 64-element units at 1 per lane (K <= 2048), 32-element units at <= 3 (K <= 3072)
    if constexpr (Fmt<QT>::UE == 64) {
        if (upl == 1) return launch_q1_fast<QT, 1>(W, x, out, n_rows, K, s);
        return MLQ_ERR_UNSUPPORTED;
    } else {
        switch (upl) {
            case 1: return launch_q1_fast<QT, 1>(W, x, out, n_rows, K, s);
            case 2: return launch_q1_fast<QT, 2>(W, x, out, n_rows, K, s);
            case 3: return launch_q1_fast<QT, 3>(W, x, out, n_rows, K, s);
            default: return MLQ_ERR_UNSUPPORTED;
        }
    }
}

static bool fits(int M, int K) {
    return gemv_layout(M, K, 0, 0).total + 2 * (kStageTarget + 64) <= kSmemBudget;
}

// batch size from which the tensor-core GEMM takes over (MLQ_TC_MIN_M overrides; 0 = never)
static int tc_min_m() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("MLQ_TC_MIN_M");
        v = e ? atoi(e) : 16;
        if (v < 0) v = 0;
    }
    return v;
}

template <int QT>
static int launch_q(const uint8_t *W, const float *x, float *out, int n_rows, int K, int B, cudaStream_t s) {
    if (tc_min_m() > 0 && B >= tc_min_m()) {
        const int rc = launch_gemm_tc(W, QT, x, out, n_rows, K, B, s);
        if (rc != MLQ_ERR_UNSUPPORTED) return rc;
    }
    if (B == 1) {
        const int rc = launch_q1<QT>(W, x, out, n_rows, K, s);
        if (rc != MLQ_ERR_UNSUPPORTED) return rc;
    }
    for (int b = 0; b < B;) {
        const int left = B - b;
        const float *xb = x + (size_t)b * K;
        float *ob = out + (size_t)b * n_rows;
        int rc, take;
        if (left >= 5 && fits(8, K)) {
            take = left < 8 ? left : 8;
            rc = launch_q_m<QT, 8>(W, xb, ob, n_rows, K, take, s);
        } else if (left >= 4 && fits(4, K)) {
            take = 4;
            rc = launch_q_m<QT, 4>(W, xb, ob, n_rows, K, take, s);
        } else if (left == 3 && fits(3, K)) {
            take = 3;
            rc = launch_q_m<QT, 3>(W, xb, ob, n_rows, K, take, s);
        } else if (left >= 2 && fits(2, K)) {
            take = 2;
            rc = launch_q_m<QT, 2>(W, xb, ob, n_rows, K, take, s);
        } else {
            take = 1;
            rc = launch_q_m<QT, 1>(W, xb, ob, n_rows, K, take, s);
        }
        if (rc != MLQ_OK) {
            if (rc == MLQ_ERR_CAPACITY) set_error(rc, "K=%d too large for the shared-memory stage ring", K);
            return rc;
        }
        b += take;
    }
    return MLQ_OK;
}

template <typename WT>
static int launch_float(const uint8_t *W, const float *x, float *out, int n_rows, int K, int B, cudaStream_t s) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    const WT *w = reinterpret_cast<const WT *>(W);
    const int V = 16 / sizeof(WT);
    const int vec_ok = (K % V == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0) &&
                       ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && ((K * 4) % 16 == 0);
    const int warps = n_rows;
    int grid = (warps * 32 + 255) / 256;
    const int cap = c->num_sms * 8;
    if (grid > cap) grid = cap;
    for (int b = 0; b < B; b += 4) {
        const int take = (B - b) < 4 ? (B - b) : 4;
        const float *xb = x + (size_t)b * K;
        float *ob = out + (size_t)b * n_rows;
        if (take == 1) k_gemv_float<WT, 1><<<grid, 256, 0, s>>>(w, xb, ob, n_rows, K, take, vec_ok);
        else if (take == 2) k_gemv_float<WT, 2><<<grid, 256, 0, s>>>(w, xb, ob, n_rows, K, take, vec_ok);
        else k_gemv_float<WT, 4><<<grid, 256, 0, s>>>(w, xb, ob, n_rows, K, take, vec_ok);
        count_launch();
    }
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_matmul(const uint8_t *W, int qt, const float *x, float *out, int n_rows, int K, int B,
                  size_t w_bytes, cudaStream_t s) {
    (void)w_bytes;
    switch (qt) {
        case MLQ_F32: return launch_float<float>(W, x, out, n_rows, K, B, s);
        case MLQ_F16: return launch_float<__half>(W, x, out, n_rows, K, B, s);
        case MLQ_BF16: return launch_float<__nv_bfloat16>(W, x, out, n_rows, K, B, s);
        case MLQ_Q4_0: return launch_q<MLQ_Q4_0>(W, x, out, n_rows, K, B, s);
        case MLQ_Q4_1: return launch_q<MLQ_Q4_1>(W, x, out, n_rows, K, B, s);
        case MLQ_Q5_0: return launch_q<MLQ_Q5_0>(W, x, out, n_rows, K, B, s);
        case MLQ_Q8_0: return launch_q<MLQ_Q8_0>(W, x, out, n_rows, K, B, s);
        case MLQ_Q4_K: return launch_q<MLQ_Q4_K>(W, x, out, n_rows, K, B, s);
        case MLQ_Q5_K: return launch_q<MLQ_Q5_K>(W, x, out, n_rows, K, B, s);
        case MLQ_Q6_K: return launch_q<MLQ_Q6_K>(W, x, out, n_rows, K, B, s);
        case MLQ_MXFP4: return launch_q<MLQ_MXFP4>(W, x, out, n_rows, K, B, s);
        case MLQ_MXFP4_REF: return launch_q<MLQ_MXFP4_REF>(W, x, out, n_rows, K, B, s);
        default:
            set_error(MLQ_ERR_TYPE, "unsupported quant type %d", qt);
            return MLQ_ERR_TYPE;
    }
}

// ------------------------------------------------------------------------------ grouped experts
// Grouped expert GEMV: rows sorted by expert; every active expert's matrix is streamed once
// for all of its rows (up to 8 per pass).  Work items (expert e, first sorted row m0, row
// count mc <= 8, row tile t) are listed expert-major; a CTA takes a contiguous range of
// items, so it re-encodes its activation rows only when (e, m0) changes.  Tiles are the
// same contiguous byte ranges as in k_gemv_q, at base + e * estride.
struct GroupItem { int e, m0, mc, tile; };

// Item it of a warp's range, fetched 32 at a time (lane i loads item base + i) and
// broadcast with shuffles: one global round trip per 32 items.  Call warp-uniformly.
struct ItemFetcher {
    GroupItem mine;
    __device__ __forceinline__ GroupItem get(const GroupItem *items, int i0, int n, int it, int lane) {
        if ((it & 31) == 0) mine = (it + lane < n) ? items[i0 + it + lane] : GroupItem{0, 0, 0, 0};
        const int src = it & 31;
        return GroupItem{__shfl_sync(0xffffffffu, mine.e, src), __shfl_sync(0xffffffffu, mine.m0, src),
                         __shfl_sync(0xffffffffu, mine.mc, src), __shfl_sync(0xffffffffu, mine.tile, src)};
    }
};

struct GroupArgs {
    GemvArgs g;                 // W = expert 0, n_rows / K / row_bytes of one expert, rpt, wpr, stages
    long long estride;          // bytes between experts
    const GroupItem *items;
    const int *n_items;         // item count, written on the device by the planner
    int tiles_per_expert;
};

__device__ __forceinline__ void produce_group_tiles(const GroupArgs &ga, uint8_t *stages, uint64_t *full,
                                                    uint64_t *empty, volatile int *abort_flag, int i0, int n_iter,
                                                    int lane) {
    const GemvArgs &a = ga.g;
    const uint64_t pol = policy_evict_first();
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    const long long mat_bytes = (long long)a.n_rows * a.row_bytes;
    ItemFetcher fetch;
    for (int it = 0; it < n_iter; ++it) {
        const GroupItem item = fetch.get(ga.items, i0, n_iter, it, lane);
        const int s = it % a.n_stages;
        if (it >= a.n_stages) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait_bounded(&empty[s], ((it / a.n_stages) - 1) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *abort_flag) {
                if (lane == 0) { *abort_flag = 1; raise_status(a.status, DEV_ST_WAIT_EMPTY); }
                return;
            }
        }
        const long long b0 = (long long)item.tile * tile_bytes;
        const long long b1 = min(b0 + tile_bytes, mat_bytes);
        const uintptr_t base = reinterpret_cast<uintptr_t>(a.W) + (uintptr_t)(item.e * ga.estride);
        const uintptr_t g0 = base + (uintptr_t)b0, g1 = base + (uintptr_t)b1;
        const uintptr_t gd = g0 & ~uintptr_t(15);
        const uintptr_t j0 = (g0 + 15) & ~uintptr_t(15);
        const uintptr_t j1 = g1 & ~uintptr_t(15);
        uint8_t *st = stages + (size_t)s * a.stage_bytes;
        if (j1 > j0) {
            if (g0 + lane < j0) st[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
            if (j1 + lane < g1) st[j1 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(j1 + lane));
        } else {
            if (g0 + lane < g1) st[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
        }
        __syncwarp();
        if (lane == 0) {
            if (j1 > j0) {
                mbar_arrive_expect_tx(&full[s], (uint32_t)(j1 - j0));
                bulk_g2s(st + (j0 - gd), reinterpret_cast<const void *>(j0), (uint32_t)(j1 - j0), &full[s], pol);
            } else {
                mbar_arrive(&full[s]);
            }
        }
    }
}

template <int QT>
__global__ void __launch_bounds__(kThreads, 1) k_gemv_grouped(GroupArgs ga) {
    constexpr int M = 8;
    const GemvArgs &a = ga.g;
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvLayout L = gemv_layout(M, a.K, a.stage_bytes, a.n_stages);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kMaxStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.off_flag);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();   // the item list is the previous kernel's output
    pdl_trigger();
    const int n_items = *ga.n_items;
    const int per_cta = (n_items + (int)gridDim.x - 1) / (int)gridDim.x;
    const int i0 = blockIdx.x * per_cta;
    const int n_iter = max(0, min(n_items, i0 + per_cta) - i0);
    init_barriers(full, empty, abort_flag, a.n_stages, kConsumerWarps);
    if (warp == kConsumerWarps) {
        produce_group_tiles(ga, smem + L.off_stage, full, empty, abort_flag, i0, n_iter, lane);
        return;
    }
    int8_t *xh = reinterpret_cast<int8_t *>(smem + L.off_xh);
    int8_t *xl = reinterpret_cast<int8_t *>(smem + L.off_xl);
    float *xs = reinterpret_cast<float *>(smem + L.off_xs);
    float *xsum = reinterpret_cast<float *>(smem + L.off_xsum);
    XPlanes xp{xh, xl, xs, xsum, a.K};
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    const int U = a.K / Fmt<QT>::UE;
    int cur_e = -1, cur_m0 = -1;
    ItemFetcher fetch;
    for (int it = 0; it < n_iter; ++it) {
        const GroupItem item = fetch.get(ga.items, i0, n_iter, it, lane);
        if (item.e != cur_e || item.m0 != cur_m0) {
            named_bar_sync(1, kConsumerWarps * 32);   // every warp is done with the old rows
            encode_x_planes<M>(a.x + (size_t)item.m0 * a.K, item.mc, a.K, xh, xl, xs, xsum, warp, lane,
                               kConsumerWarps);
            named_bar_sync(1, kConsumerWarps * 32);
            cur_e = item.e;
            cur_m0 = item.m0;
        }
        const int s = it % a.n_stages;
        const bool ok = consume_wait(a, full, abort_flag, it, lane);
        const int row0 = item.tile * a.rpt;
        const uintptr_t g0 = reinterpret_cast<uintptr_t>(a.W) + (uintptr_t)(item.e * ga.estride) +
                             (uintptr_t)((long long)item.tile * tile_bytes);
        const uint8_t *stage = smem + L.off_stage + (size_t)s * a.stage_bytes + (g0 & 15);
        float *out = a.out + (size_t)item.m0 * a.n_rows;
        // warp w takes rows w, w + 8, ... of the tile
        for (int rr = warp; rr < a.rpt; rr += kConsumerWarps) {
            const int row = row0 + rr;
            float acc[M];
#pragma unroll
            for (int m = 0; m < M; m++) acc[m] = 0.0f;
            if (ok && row < a.n_rows) {
                const uint8_t *rowp = stage + (size_t)rr * a.row_bytes;
                for (int u = lane; u < U; u += 32) {
                    W<QT> w;
                    w.decode(rowp, u);
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        if (m < item.mc) {
                            XU<QT> xu;
                            load_xu<QT>(xp, m, u, xu);
                            acc[m] += w.dot(xu);
                        }
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < M; m++) {
                if (m < item.mc) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
                }
            }
            if (lane == 0 && ok && row < a.n_rows) {
#pragma unroll
                for (int m = 0; m < M; m++)
                    if (m < item.mc) out[(size_t)m * a.n_rows + row] = acc[m];
            }
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(&empty[s]);
    }
}

// Host-free grouping: counts per expert, stable sorted order and the work-item lists for
// two tilings (the gate/up matrices and the down matrix).  Thread 0 counts and orders
// (deterministic, small loops over rows and experts); the item lists are written in
// parallel, one expert per thread.
__global__ void k_group_plan(const int *__restrict__ eid, int R, int E, int tiles_a, int tiles_b,
                             int *__restrict__ offs, int *__restrict__ sorted_pos, GroupItem *__restrict__ items_a,
                             GroupItem *__restrict__ items_b, int *__restrict__ n_items) {
    extern __shared__ int sm_plan[];
    int *so = sm_plan;              // [E + 1] row offsets
    int *sc = so + E + 1;           // [E] running positions
    int *si = sc + E;               // [E + 1] first row-chunk index of each expert
    int *se = si + E + 1;           // [R] expert ids (read once from global memory)
    for (int e = threadIdx.x; e <= E; e += blockDim.x) so[e] = 0;
    for (int r = threadIdx.x; r < R; r += blockDim.x) se[r] = eid[r];
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        const int e = se[r];
        if (e >= 0 && e < E) atomicAdd(&so[e + 1], 1);   // counts: order-free
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int e = 0; e < E; e++) so[e + 1] += so[e];
        si[0] = 0;
        for (int e = 0; e < E; e++) si[e + 1] = si[e] + (so[e + 1] - so[e] + 7) / 8;
        n_items[0] = si[E] * tiles_a;
        n_items[1] = si[E] * tiles_b;
        for (int e = 0; e < E; e++) sc[e] = so[e];
        for (int r = 0; r < R; r++) {   // stable positions in arrival order
            const int e = se[r];
            sorted_pos[r] = (e >= 0 && e < E) ? sc[e]++ : -1;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e <= E; e += blockDim.x) offs[e] = so[e];
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int n = so[e + 1] - so[e];
        const int *offs_s = so;
        int c = si[e];
        for (int m0 = 0; m0 < n; m0 += 8, c++) {
            const int mc = min(8, n - m0);
            for (int t = 0; t < tiles_a; t++) items_a[(size_t)c * tiles_a + t] = GroupItem{e, offs_s[e] + m0, mc, t};
            for (int t = 0; t < tiles_b; t++) items_b[(size_t)c * tiles_b + t] = GroupItem{e, offs_s[e] + m0, mc, t};
        }
    }
}

__global__ void k_rows_permute(const float *__restrict__ src, const int *__restrict__ pos, int K, int to_sorted,
                               float *__restrict__ dst) {
    const int r = blockIdx.x;
    const int p = pos[r];
    if (p < 0) return;
    const float *s = src + (size_t)(to_sorted ? r : p) * K;
    float *d = dst + (size_t)(to_sorted ? p : r) * K;
    for (int i = threadIdx.x; i < K; i += blockDim.x) d[i] = s[i];
}

// rows per grouped tile: a multiple of the 8 decode warps, about kStageTarget bytes, <= 64
static int grouped_rpt(long long rb) {
    long long r = kStageTarget / rb;
    r = r < 8 ? 8 : (r > 64 ? 64 : r);
    return (int)(r / 8 * 8);
}

template <int QT>
static int launch_grouped_t(const uint8_t *W, long long estride, const GroupItem *items, const int *n_items_dev,
                            int n_items_bound, const float *x_sorted, float *y_sorted, int n_rows, int K,
                            cudaStream_t s) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    constexpr int M = 8;
    const long long rb = (long long)(K / Fmt<QT>::BE) * Fmt<QT>::BB;
    const int rpt = grouped_rpt(rb);
    const int stage_bytes = align_up((int)(rpt * rb), 16) + 48;
    const int fixed = gemv_layout(M, K, stage_bytes, 0).total;
    const int n_stages = stages_for(fixed, stage_bytes);
    if (n_stages < 2) {
        set_error(MLQ_ERR_CAPACITY, "grouped experts: K=%d too large for the stage ring", K);
        return MLQ_ERR_CAPACITY;
    }
    GroupArgs ga{};
    GemvArgs &a = ga.g;
    a.W = W; a.x = x_sorted; a.out = y_sorted; a.n_rows = n_rows; a.K = K; a.nb_x = M;
    a.row_bytes = rb; a.total_bytes = rb * n_rows; a.rpt = rpt; a.wpr = 1;
    a.stage_bytes = stage_bytes; a.n_stages = n_stages; a.status = c->d_status;
    ga.estride = estride;
    ga.items = items;
    ga.tiles_per_expert = (n_rows + rpt - 1) / rpt;
    // the item count is only known on the device: the grid covers the bound and every CTA
    // takes a contiguous share of the real count
    ga.n_items = n_items_dev;
    const int grid = n_items_bound < c->num_sms ? (n_items_bound > 0 ? n_items_bound : 1) : c->num_sms;
    static bool attr = false;
    if (!attr) {
        if (!MLQ_CUDA(cudaFuncSetAttribute(k_gemv_grouped<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem)))
            return MLQ_ERR_CUDA;
        attr = true;
    }
    count_launch();
    return MLQ_CUDA(launch_pdl(k_gemv_grouped<QT>, dim3(grid), dim3(kThreads), fixed + n_stages * stage_bytes, s, ga))
               ? MLQ_OK
               : MLQ_ERR_CUDA;
}

int grouped_tiles_per_expert(int qt, int n_rows, int K) {
    const long long rb = (long long)(K / block_elems(qt)) * block_bytes(qt);
    if (rb <= 0) return 0;
    const int rpt = grouped_rpt(rb);
    return (n_rows + rpt - 1) / rpt;
}

int launch_grouped(int qt, const uint8_t *W, long long estride, const void *items, const int *n_items_dev,
                   int n_items_bound, const float *x_sorted, float *y_sorted, int n_rows, int K, cudaStream_t s) {
    const GroupItem *it = (const GroupItem *)items;
    switch (qt) {
        case MLQ_Q4_0: return launch_grouped_t<MLQ_Q4_0>(W, estride, it, n_items_dev, n_items_bound, x_sorted, y_sorted, n_rows, K, s);
        case MLQ_Q4_1: return launch_grouped_t<MLQ_Q4_1>(W, estride, it, n_items_dev, n_items_bound, x_sorted, y_sorted, n_rows, K, s);
        case MLQ_Q5_0: return launch_grouped_t<MLQ_Q5_0>(W, estride, it, n_items_dev, n_items_bound, x_sorted, y_sorted, n_rows, K, s);
        case MLQ_Q8_0: return launch_grouped_t<MLQ_Q8_0>(W, estride, it, n_items_dev, n_items_bound, x_sorted, y_sorted, n_rows, K, s);
        case MLQ_Q4_K: return launch_grouped_t<MLQ_Q4_K>(W, estride, it, n_items_dev, n_items_bound, x_sorted, y_sorted, n_rows, K, s);
        case MLQ_Q5_K: return launch_grouped_t<MLQ_Q5_K>(W, estride, it, n_items_dev, n_items_bound, x_sorted, y_sorted, n_rows, K, s);
        case MLQ_Q6_K: return launch_grouped_t<MLQ_Q6_K>(W, estride, it, n_items_dev, n_items_bound, x_sorted, y_sorted, n_rows, K, s);
        case MLQ_MXFP4: return launch_grouped_t<MLQ_MXFP4>(W, estride, it, n_items_dev, n_items_bound, x_sorted, y_sorted, n_rows, K, s);
        case MLQ_MXFP4_REF: return launch_grouped_t<MLQ_MXFP4_REF>(W, estride, it, n_items_dev, n_items_bound, x_sorted, y_sorted, n_rows, K, s);
        default:
            set_error(MLQ_ERR_TYPE, "grouped experts: type %d", qt);
            return MLQ_ERR_TYPE;
    }
}

int launch_group_plan(const int *eid, int R, int E, int tiles_a, int tiles_b, int *offs, int *sorted_pos,
                      void *items_a, void *items_b, int *n_items, cudaStream_t s) {
    const size_t sm = sizeof(int) * (3 * (size_t)E + 2 + (size_t)R);
    if (sm > 48 * 1024) {
        set_error(MLQ_ERR_CAPACITY, "grouped experts: %d experts / %d rows per call", E, R);
        return MLQ_ERR_CAPACITY;
    }
    k_group_plan<<<1, 256, sm, s>>>(eid, R, E, tiles_a, tiles_b, offs, sorted_pos, (GroupItem *)items_a,
                                    (GroupItem *)items_b, n_items);
    count_launch();
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_rows_permute(const float *src, const int *pos, int R, int K, int to_sorted, float *dst, cudaStream_t s) {
    if (R <= 0) return MLQ_OK;
    k_rows_permute<<<R, 256, 0, s>>>(src, pos, K, to_sorted, dst);
    count_launch();
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

// ------------------------------------------------------------------------------ dequantize
// One thread per output element, bit-exact with the reference's *_dequantize_row and
// gguf-py: every product/difference is rounded separately (no FMA contraction).
__device__ __forceinline__ float f16_g(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

__global__ void k_dequant(const uint8_t *__restrict__ W, int qt, float *__restrict__ out, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float v = 0.0f;
        switch (qt) {
            case MLQ_F32: v = reinterpret_cast<const float *>(W)[i]; break;
            case MLQ_F16: v = __half2float(reinterpret_cast<const __half *>(W)[i]); break;
            case MLQ_BF16: v = __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(W)[i]); break;
            case MLQ_Q8_0: {
                const uint8_t *bp = W + (i >> 5) * 34;
                v = __fmul_rn((float)(int8_t)bp[2 + (i & 31)], f16_g(bp));
            } break;
            case MLQ_Q4_0: case MLQ_Q4_1: case MLQ_Q5_0: {
                const int bb = qt == MLQ_Q4_0 ? 18 : qt == MLQ_Q4_1 ? 20 : 22;
                const int hdr = qt == MLQ_Q4_0 ? 2 : qt == MLQ_Q4_1 ? 4 : 6;
                const uint8_t *bp = W + (i >> 5) * bb;
                const int j = (int)(i & 31);
                int q = (j < 16) ? (bp[hdr + j] & 0xF) : (bp[hdr + j - 16] >> 4);
                const float d = f16_g(bp);
                if (qt == MLQ_Q4_0) v = __fmul_rn((float)(q - 8), d);
                else if (qt == MLQ_Q4_1) v = __fadd_rn(__fmul_rn((float)q, d), f16_g(bp + 2));
                else {
                    const uint32_t qh = bp[2] | (bp[3] << 8) | (bp[4] << 16) | ((uint32_t)bp[5] << 24);
                    q |= ((qh >> j) & 1) << 4;
                    v = __fmul_rn((float)(q - 16), d);
                }
            } break;
            case MLQ_Q4_K: case MLQ_Q5_K: {
                const int bb = qt == MLQ_Q4_K ? 144 : 176;
                const uint8_t *bp = W + (i >> 8) * bb;
                const int e = (int)(i & 255), sub = e >> 5, l = e & 31, g = sub >> 1;
                const uint8_t *sc = bp + 4;
                uint32_t s, m;
                if (sub < 4) { s = sc[sub] & 63; m = sc[sub + 4] & 63; }
                else { s = (sc[sub + 4] & 0xF) | ((sc[sub - 4] >> 6) << 4); m = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4); }
                const uint8_t *qs = bp + (qt == MLQ_Q4_K ? 16 : 48) + 32 * g;
                int q = (sub & 1) ? (qs[l] >> 4) : (qs[l] & 0xF);
                if (qt == MLQ_Q5_K) q += ((bp[16 + l] >> sub) & 1) << 4;
                const float ds = __fmul_rn(f16_g(bp), (float)s);
                const float dm = __fmul_rn(f16_g(bp + 2), (float)m);
                v = __fsub_rn(__fmul_rn(ds, (float)q), dm);
            } break;
            case MLQ_Q6_K: {
                const uint8_t *bp = W + (i >> 8) * 210;
                const int e = (int)(i & 255), h = e >> 7, r = e & 127, quad = r >> 5, l = r & 31;
                const uint8_t qlb = bp[64 * h + l + ((quad & 1) ? 32 : 0)];
                const int lo = (quad < 2) ? (qlb & 0xF) : (qlb >> 4);
                const int hi = (bp[128 + 32 * h + l] >> (2 * quad)) & 3;
                const float ds = __fmul_rn(f16_g(bp + 208), (float)(int8_t)bp[192 + (e >> 4)]);
                v = __fmul_rn(ds, (float)((lo | (hi << 4)) - 32));
            } break;
            case MLQ_MXFP4: {
                const uint8_t *bp = W + (i >> 5) * 17;
                const int j = (int)(i & 31);
                const int nib = (j < 16) ? (bp[1 + j] & 0xF) : (bp[1 + j - 16] >> 4);
                const int kv[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
                v = __fmul_rn((float)kv[nib], e8m0_half(bp[0]));
            } break;
            case MLQ_MXFP4_REF: {
                const uint8_t *bp = W + (i >> 5) * 17;
                const int j = (int)(i & 31);
                int nib = (j & 1) ? (bp[j >> 1] >> 4) : (bp[j >> 1] & 0xF);
                if (nib > 7) nib -= 16;
                v = __fmul_rn((float)nib, __uint_as_float((uint32_t)bp[16] << 23));
            } break;
            default: break;
        }
        out[i] = v;
    }
}

int launch_dequantize(const uint8_t *W, int qt, float *out, int64_t n, cudaStream_t s) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    long long blocks = (n + 255) / 256;
    if (blocks > (long long)c->num_sms * 32) blocks = (long long)c->num_sms * 32;
    if (blocks < 1) blocks = 1;
    k_dequant<<<(int)blocks, 256, 0, s>>>(W, qt, out, n);
    count_launch();
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

// ------------------------------------------------------------------------------ Q8_0 quantizer
// quantize_row_q8_0 (quant_kernels_omp.c:1406-1455): d = amax/127 (1 if 0), id = 1/d,
// q = round-half-even(clamp(x*id, -127, 127)), d as f16 (round to nearest even).
__global__ void k_quantize_q8_0(const float *__restrict__ x, uint8_t *__restrict__ q8, long long nblk) {
    const int lane = threadIdx.x & 31;
    for (long long b = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; b < nblk;
         b += ((long long)gridDim.x * blockDim.x) >> 5) {
        const float v = x[b * 32 + lane];
        float amax = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        float d = __fdiv_rn(amax, 127.0f);
        if (d == 0.0f) d = 1.0f;
        const float id = __fdiv_rn(1.0f, d);
        const float t = fminf(fmaxf(__fmul_rn(v, id), -127.0f), 127.0f);
        const uint32_t qb = (uint32_t)__float2int_rn(t) & 0xFFu;
        unsigned short d16;
        asm("cvt.rn.f16.f32 %0, %1;" : "=h"(d16) : "f"(d));
        // the 34-byte block as 17 little-endian 16-bit words: word 0 = d, word i = (q[2i-2], q[2i-1])
        const uint32_t qlo = __shfl_sync(0xffffffffu, qb, (2 * lane - 2) & 31);
        const uint32_t qhi = __shfl_sync(0xffffffffu, qb, (2 * lane - 1) & 31);
        unsigned short *dst = reinterpret_cast<unsigned short *>(q8 + b * 34);
        if (lane == 0) dst[0] = d16;
        else if (lane <= 16) dst[lane] = (unsigned short)(qlo | (qhi << 8));
    }
}

int launch_quantize_q8_0(const float *x, uint8_t *q8, int64_t n, cudaStream_t s) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    const long long nblk = n / 32;
    long long blocks = (nblk * 32 + 255) / 256;
    if (blocks > (long long)c->num_sms * 16) blocks = (long long)c->num_sms * 16;
    if (blocks < 1) blocks = 1;
    k_quantize_q8_0<<<(int)blocks, 256, 0, s>>>(x, q8, nblk);
    count_launch();
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_q8act_to_f32(const uint8_t *x_q8, float *x, int64_t n, cudaStream_t s) {
    return launch_dequantize(x_q8, MLQ_Q8_0, x, n, s);
}

}  // namespace mlq
