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
#include <type_traits>
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
    int out_host;               // M=1 kernel: out is host memory (row sums leave in runs per tile)
};

struct GemvLayout {
    int off_bar, off_flag, off_xh, off_xl, off_xs, off_xsum, off_red, off_out, off_stage, total;
};

// row sums of one tile of the M=1 kernel, before the producer writes them out: two slots
// per stage, alternating with the stage's use count
static constexpr int kTileOutRows = 64;

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
    L.off_out = o;  o += M == 1 ? 2 * kMaxStages * kTileOutRows * 4 : 0;
    L.off_stage = o; o += n_stages * stage_bytes;
    L.total = o;
    return L;
}

__device__ __forceinline__ void raise_status(int *status, int code) {
    report_status(status, code);
}

struct NoFlush {
    static constexpr bool kActive = false;
    bool on = false;
    __device__ void operator()(int, int) const {}
};

// Row sums of the M=1 kernel when `out` is host memory: the decode warps leave each
// tile's sums in shared memory and the producer warp, once every decode warp has
// released the tile's stage, writes them to `out` as one contiguous run per tile, so the
// caller's pinned buffer is written in a few full PCIe packets per tile instead of
// 4-byte stores.  (Device outputs are stored by the decode warps directly: routing them
// through the producer measured ~8 % slower, the refills waiting behind the writes.)  Tile it uses
// slot tile_sum_slot(it): the producer writes tile it's sums out after it has issued the
// copy of tile it + n_stages into the same stage, whose decode warps fill the other slot.
__device__ __forceinline__ int tile_sum_slot(int it, int n_stages) {
    return (2 * (it % n_stages) + ((it / n_stages) & 1)) * kTileOutRows;
}

struct TileOutFlush {
    static constexpr bool kActive = true;
    bool on;
    const float *sums;   // shared: [kMaxStages][2][kTileOutRows]
    float *out;
    int rpt, n_rows, n_stages;
    __device__ void operator()(int it, int lane) const {
        const long long row0 = ((long long)blockIdx.x + (long long)it * gridDim.x) * rpt;
        const float *src = sums + tile_sum_slot(it, n_stages);
        for (int r = lane; r < rpt; r += 32)
            if (row0 + r < n_rows) out[row0 + r] = src[r];
    }
};

// producer lane 0: bounded wait until every decode warp released stage s (for tile it);
// broadcast to the warp, which then sees the decode warps' shared-memory writes
__device__ __forceinline__ bool producer_wait_empty(const GemvArgs &a, uint64_t *empty, volatile int *abort_flag,
                                                    int it, int lane) {
    bool ok = true;
    if (lane == 0) ok = mbar_wait_bounded(&empty[it % a.n_stages], (it / a.n_stages) & 1);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    if (!ok || *abort_flag) {
        if (lane == 0) { *abort_flag = 1; raise_status(a.status, DEV_ST_WAIT_EMPTY); }
        return false;
    }
    return true;
}

// Producer warp: stream tile it of this CTA into stage it % n_stages.  The tile's
// 16-byte-aligned interior goes through one cp.async.bulk (TMA engine, L2
// evict_first); the <= 15-byte ragged head and tail are plain loads by the lanes.
// With an active Flush, the row sums of tile it - n_stages are written out once its
// stage is released and tile it's copy is under way, and those of the last n_stages
// tiles after the loop.
template <typename Flush = NoFlush>
__device__ __forceinline__ void produce_tiles(const GemvArgs &a, uint8_t *stages, uint64_t *full, uint64_t *empty,
                                              volatile int *abort_flag, int n_iter, int lane,
                                              const Flush &flush = Flush()) {
    const uint64_t pol = policy_evict_first();
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    for (int it = 0; it < n_iter; ++it) {
        const int s = it % a.n_stages;
        if (it >= a.n_stages) {
            if (!producer_wait_empty(a, empty, abort_flag, it - a.n_stages, lane)) return;
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
        if constexpr (Flush::kActive) {
            if (flush.on && it >= a.n_stages) flush(it - a.n_stages, lane);
        }
    }
    if (flush.on) {
        for (int j = n_iter > a.n_stages ? n_iter - a.n_stages : 0; j < n_iter; ++j) {
            if (*abort_flag) return;   // a decode warp gave up: its stages are never released
            if (!producer_wait_empty(a, empty, abort_flag, j, lane)) return;
            flush(j, lane);
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

    XPlanes xp{xh, xl, xs, xsum, a.K, a.K, a.K / 32};
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
// NW decode warps each own RW rows of every tile (rows w, w+NW, ...), and each lane
// always handles units lane, lane+32, ... of a row, so the lane's activation slices XU
// are loaded into registers once and reused for every row the CTA streams.  UPL = units
// per lane (ceil(K/UE/32)); A16 = rows start on 16-byte boundaries in shared memory
// (Q4_K/Q5_K then use 128-bit loads); RW = rows per warp per tile (independent decode
// chains for latency hiding).  With RW = 2 the two row sums are reduced together: one
// exchange across the half-warps leaves each half with one row, then four levels.
template <int QT, int UPL, bool A16, int RW, int NW, bool OH>
__global__ void __launch_bounds__((NW + 1) * 32, 1) k_gemv_q1(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvLayout L = gemv_layout(1, a.K, a.stage_bytes, a.n_stages);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kMaxStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.off_flag);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_iter = (a.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    if (warp == NW) prefetch_first_tiles(a, n_iter, lane);
    init_barriers(full, empty, abort_flag, a.n_stages, NW);
    pdl_wait();
    pdl_trigger();
    float *sums = reinterpret_cast<float *>(smem + L.off_out);
    if (warp == NW) {
        produce_tiles(a, smem + L.off_stage, full, empty, abort_flag, n_iter, lane,
                      TileOutFlush{OH, sums, a.out, a.rpt, a.n_rows, a.n_stages});
        return;
    }
    int8_t *xh = reinterpret_cast<int8_t *>(smem + L.off_xh);
    int8_t *xl = reinterpret_cast<int8_t *>(smem + L.off_xl);
    float *xs = reinterpret_cast<float *>(smem + L.off_xs);
    float *xsum = reinterpret_cast<float *>(smem + L.off_xsum);
    encode_x_planes<1>(a.x, 1, a.K, xh, xl, xs, xsum, warp, lane, NW);
    named_bar_sync(1, NW * 32);
    const XPlanes xp{xh, xl, xs, xsum, a.K, a.K, a.K / 32};
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
                        // rows warp, warp + NW, ...: row r of this warp within the tile
                        if (row0 + NW * r < a.n_rows) {
                            const uint8_t *rowp = st + (size_t)(warp + NW * r) * a.row_bytes;
                            W<QT> w;
                            if constexpr (A16) w.decode_a16(rowp, u);
                            else w.decode(rowp, u);
                            acc[r] += w.dot(xu[j]);
                        }
                    }
                }
            }
        }
        if constexpr (RW == 2) {
            const bool up = (lane & 16) != 0;
            float v = (up ? acc[1] : acc[0]) + __shfl_xor_sync(0xffffffffu, up ? acc[0] : acc[1], 16);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            const int r = lane >> 4;
            if constexpr (OH) {
                if ((lane & 15) == 0) sums[tile_sum_slot(it, a.n_stages) + warp + NW * r] = v;
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(&empty[s]);   // releases the stage and its sums
            } else {
                // release the stage before the global store: an arrive after it would wait
                // for the store (release ordering)
                __syncwarp();
                if (ok) {
                    if (lane == 0) mbar_arrive(&empty[s]);
                    if ((lane & 15) == 0 && row0 + NW * r < a.n_rows) a.out[row0 + NW * r] = v;
                }
            }
        } else {
#pragma unroll
            for (int r = 0; r < RW; r++) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
            }
            if (OH && lane == 0) {
#pragma unroll
                for (int r = 0; r < RW; r++) sums[tile_sum_slot(it, a.n_stages) + warp + NW * r] = acc[r];
            }
            __syncwarp();
            if (lane == 0 && ok) {
                mbar_arrive(&empty[s]);
                if constexpr (!OH) {
#pragma unroll
                    for (int r = 0; r < RW; r++)
                        if (row0 + NW * r < a.n_rows) a.out[row0 + NW * r] = acc[r];
                }
            }
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

// fp32 / fp16 / bf16 weights, few rows (a router): one CTA per row, the row split over
// its 8 warps, up to 16 activation rows per launch; the row is read once for all of them
// and the per-warp partial sums meet in shared memory
constexpr int kFewRowsMaxB = 16;

template <typename WT>
__global__ void __launch_bounds__(256) k_gemv_float_rows(const WT *__restrict__ W, const float *__restrict__ x,
                                                         float *__restrict__ out, int n_rows, int K, int nb_x,
                                                         int vec_ok, const WT *__restrict__ w_extra,
                                                         float *__restrict__ out_extra) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    constexpr int V = 16 / sizeof(WT);
    __shared__ float part[8][kFewRowsMaxB];
    const int row = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // CTA n_rows (when w_extra is given): one more row from its own pointer, out_extra[m]
    const bool extra = row == n_rows;
    const WT *wr = extra ? w_extra : W + (size_t)row * K;
    float acc[kFewRowsMaxB];
#pragma unroll
    for (int m = 0; m < kFewRowsMaxB; m++) acc[m] = 0.0f;
    if (vec_ok) {
        for (int k0 = threadIdx.x * V; k0 < K; k0 += 256 * V) {
            union { int4 v; WT e[V]; } wv;
            wv.v = __ldg(reinterpret_cast<const int4 *>(wr + k0));
            float wf[V];
#pragma unroll
            for (int j = 0; j < V; j++) wf[j] = to_f<WT>(wv.e[j]);
#pragma unroll
            for (int m = 0; m < kFewRowsMaxB; m++) {
                if (m < nb_x) {
                    const float *xr = x + (size_t)m * K + k0;
#pragma unroll
                    for (int j = 0; j < V; j += 4) {
                        const float4 xv = __ldg(reinterpret_cast<const float4 *>(xr + j));
                        acc[m] = fmaf(wf[j + 0], xv.x, acc[m]);
                        acc[m] = fmaf(wf[j + 1], xv.y, acc[m]);
                        acc[m] = fmaf(wf[j + 2], xv.z, acc[m]);
                        acc[m] = fmaf(wf[j + 3], xv.w, acc[m]);
                    }
                }
            }
        }
    } else {
        for (int k = threadIdx.x; k < K; k += 256) {
            const float wv = to_f<WT>(wr[k]);
#pragma unroll
            for (int m = 0; m < kFewRowsMaxB; m++)
                if (m < nb_x) acc[m] = fmaf(wv, __ldg(x + (size_t)m * K + k), acc[m]);
        }
    }
#pragma unroll
    for (int m = 0; m < kFewRowsMaxB; m++) {
        if (m < nb_x) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int m = 0; m < kFewRowsMaxB; m++) part[warp][m] = acc[m];
    }
    __syncthreads();
    if (threadIdx.x < nb_x) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) sum += part[w][threadIdx.x];
        if (extra) out_extra[threadIdx.x] = sum;
        else out[(size_t)threadIdx.x * n_rows + row] = sum;
    }
}

// ------------------------------------------------------------------------------ launchers
// Launch with programmatic stream serialization: the kernel may start while the previous
// kernel on the stream finishes; it calls pdl_wait() before touching anything that kernel
// writes.  MLQ_NO_PDL=1 launches normally.
bool pdl_enabled() {
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

// the same for a kernel of several parameters
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl_n(void (*kern)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t s,
                                Args... args) {
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
    return cudaLaunchKernelEx(&cfg, kern, args...);
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
    // more than half the shared memory of an SM: one CTA per SM, no occupancy query
    int per_sm = 1;
    if (2 * smem <= kMaxSmem &&
        !MLQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem)))
        return MLQ_ERR_CUDA;
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

// decode warps of the M=1 kernel (MLQ_GEMV_WARPS = 16, 20 or 24 overrides); more warps
// hide more of the dp4a / shared-load latency but cap the registers per thread
// (20 warps + producer: 96, 24 + producer: 80).  Per format, the fastest measured at
// 151936 x 2048 on B200.
template <int QT> static int fast_nw() {
    const char *e = getenv("MLQ_GEMV_WARPS");
    if (e && (atoi(e) == 16 || atoi(e) == 20 || atoi(e) == 24)) return atoi(e);
    if constexpr (QT == kQ4_0Pair) return 24;   // Q8_0 pairs: 16 (larger tiles leave < 3 stages)
    if constexpr (QT == MLQ_Q4_K || QT == MLQ_Q5_K || QT == MLQ_Q6_K || QT == MLQ_Q8_0) return 20;
    return kFastWarps;
}

template <int QT, int UPL, int RW, int NW>
static int launch_q1_rw(const uint8_t *W, const float *x, float *out, int n_rows, int K, cudaStream_t s) {
    static_assert(NW * RW <= kTileOutRows, "a tile's row sums must fit their shared-memory slot");
    const long long rb = (long long)(K / Fmt<QT>::BE) * Fmt<QT>::BB;
    const int rpt = NW * RW;
    const int stage_bytes = align_up((int)(rpt * rb), 16) + 48;
    const int fixed = gemv_layout(1, K, stage_bytes, 0).total;
    const int n_stages = stages_for(fixed, stage_bytes);
    if (n_stages < 3) return MLQ_ERR_CAPACITY;
    GemvArgs a{};
    a.W = W; a.x = x; a.out = out; a.n_rows = n_rows; a.K = K; a.nb_x = 1;
    a.row_bytes = rb; a.total_bytes = rb * n_rows; a.rpt = rpt; a.wpr = 1;
    a.n_tiles = (n_rows + rpt - 1) / rpt; a.stage_bytes = stage_bytes; a.n_stages = n_stages;
    a.out_host = launch_env() && launch_env()->out_host ? 1 : 0;
    const int smem = fixed + n_stages * stage_bytes;
    constexpr int kThr = (NW + 1) * 32;
    constexpr bool kCanAlign = (QT == MLQ_Q4_K || QT == MLQ_Q5_K);
    if constexpr (kCanAlign) {
        if (rb % 16 == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0) {
            static bool attr_a = false, attr_ah = false;
            if (a.out_host) return launch_gemv_kernel(k_gemv_q1<QT, UPL, true, RW, NW, true>, a, smem, s, attr_ah, kThr);
            return launch_gemv_kernel(k_gemv_q1<QT, UPL, true, RW, NW, false>, a, smem, s, attr_a, kThr);
        }
    }
    static bool attr_set = false, attr_h = false;
    if (a.out_host) return launch_gemv_kernel(k_gemv_q1<QT, UPL, false, RW, NW, true>, a, smem, s, attr_h, kThr);
    return launch_gemv_kernel(k_gemv_q1<QT, UPL, false, RW, NW, false>, a, smem, s, attr_set, kThr);
}

// formats whose M=1 kernel is built with 20 and 24 decode warps as well as 16
template <int QT> constexpr bool kWarpVariants = QT == kQ4_0Pair || QT == MLQ_Q4_K || QT == MLQ_Q5_K ||
                                                 QT == MLQ_Q6_K || QT == MLQ_Q8_0 || QT == kQ8_0Pair;

// Q8_0 as block pairs where rows allow it (MLQ_Q8_0_PAIRS=0: single blocks)
static bool q8_0_pairs() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("MLQ_Q8_0_PAIRS");
        v = (e && atoi(e) == 0) ? 0 : 1;
    }
    return v == 1;
}

template <int QT, int UPL>
static int launch_q1_fast(const uint8_t *W, const float *x, float *out, int n_rows, int K, cudaStream_t s) {
    const int rw = fast_rw<QT>();
    if constexpr (kWarpVariants<QT>) {
        // a tile of NW * RW rows that leaves fewer than 3 stages falls back to 16 warps
        const int nw = fast_nw<QT>();
        int rc = MLQ_ERR_CAPACITY;
        if (nw == 24) rc = rw == 2 ? launch_q1_rw<QT, UPL, 2, 24>(W, x, out, n_rows, K, s)
                                   : launch_q1_rw<QT, UPL, 1, 24>(W, x, out, n_rows, K, s);
        else if (nw == 20) rc = rw == 2 ? launch_q1_rw<QT, UPL, 2, 20>(W, x, out, n_rows, K, s)
                                        : launch_q1_rw<QT, UPL, 1, 20>(W, x, out, n_rows, K, s);
        if (rc != MLQ_ERR_CAPACITY) return rc;
    }
    if (rw == 2) return launch_q1_rw<QT, UPL, 2, kFastWarps>(W, x, out, n_rows, K, s);
    return launch_q1_rw<QT, UPL, 1, kFastWarps>(W, x, out, n_rows, K, s);
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
    if constexpr (QT == MLQ_Q4_0) {
        // block pairs: rows of 36-byte pairs on 4-byte boundaries
        if (K % 64 == 0 && K <= 2048 && (reinterpret_cast<uintptr_t>(W) & 3) == 0)
            return launch_q1<kQ4_0Pair>(W, x, out, n_rows, K, s);
    }
    if constexpr (QT == MLQ_Q8_0) {
        if (q8_0_pairs() && K % 64 == 0 && K <= 2048 && (reinterpret_cast<uintptr_t>(W) & 3) == 0)
            return launch_q1<kQ8_0Pair>(W, x, out, n_rows, K, s);
    }
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

// batch size from which the tensor-core GEMM takes over (MLQ_TC_MIN_M overrides; 0 = never).
// From 5 rows its one weight pass beats the GEMV's passes of up to 8 rows on every format
// and shape of the sweep (2048 x 2048 Q8_0 at 10 rows: 36.3 -> 20.5 us; 151936 x 2048 Q4_K
// at 8 rows: 306 -> 253 us); at 4 rows the packed GEMV is still ahead (15.5 against ~20 us).
static int tc_min_m() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("MLQ_TC_MIN_M");
        v = e ? atoi(e) : 5;
        if (v < 0) v = 0;
    }
    return v;
}

template <int QT>
static int launch_q(const uint8_t *W, const float *x, float *out, int n_rows, int K, int B, cudaStream_t s) {
    // every format the tensor-core GEMM takes, from tc_min_m() rows (Q6_K included since its
    // decode packs four codes to a word: 2048 x 2048 at 16 rows 65 -> 21 us against two
    // passes of the 8-row GEMV; config-3 step at 16 tokens 20.3 -> 16.3 ms).  MXFP4 on a
    // large matrix keeps its block-scaled passes below 32 rows (151936 x 2048 at 16 rows:
    // 147 us in four passes, 318 us through the fp16 decode of the GEMM)
    int tc_from = tc_min_m();
    if (QT == MLQ_MXFP4 && n_rows >= 16384 && tc_from > 0 && tc_from < 32) tc_from = 32;
    // MXFP4 rows that fit one pass of the block-scaled GEMV (up to 8 at K <= 1024) stay there:
    // one launch, against the GEMM's activation conversion plus its own launch
    const int mx_pass = K <= 1024 ? 8 : K <= 2048 ? 4 : K <= 4096 ? 2 : 1;
    if (QT == MLQ_MXFP4 && B <= mx_pass) tc_from = 0;
    if constexpr (QT == MLQ_MXFP4) {
        // more rows than one block-scaled GEMV pass: the rows encoded once as E2M1 planes, then
        // 128-row tiles of the weights against up to 8 rows each, on the same kind::mxf4 tensor
        // cores (the grouped expert kernel in dense mode)
        // (from 5 rows at every size; rows that are not TMA tiles -- K % 512 != 0 or an
        // unaligned base -- only up to 64 rows: above, their windowed copies lose to the fp16
        // GEMM, 2880 x 2880 at 256 rows 93 against 71 us)
        const bool tiles = K % 512 == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0;
        const int from = tc_min_m();
        if (from > 0 && B > mx_pass && B >= from && (tiles || B <= 64) && mxf4_dense_supported(W, n_rows, K)) {
            uint8_t *planes = static_cast<uint8_t *>(tc_scratch(s, mxf4_planes_bytes(B, K)));
            if (planes) {
                int rc = launch_mxf4_planes_rows(x, nullptr, nullptr, 1, K, 0.0f, B, K, planes, s);
                if (rc == MLQ_OK) rc = launch_mxf4_dense_tc(W, nullptr, n_rows, K, planes, B, out, nullptr, s);
                if (rc != MLQ_ERR_UNSUPPORTED) return rc;
            }
        }
    }
    if (tc_from > 0 && B >= tc_from) {
        const int rc = launch_gemm_tc(W, QT, x, out, n_rows, K, B, s);
        if (rc != MLQ_ERR_UNSUPPORTED) return rc;
    }
    if constexpr (QT == MLQ_MXFP4) {
        // block-scaled tensor cores: groups of up to 8 activation rows per weight pass
        int b = 0, rc = MLQ_OK;
        const int g = mx_pass;
        for (; b < B && rc == MLQ_OK; b += g) {
            const int take = B - b < g ? B - b : g;
            rc = launch_gemv_mxf4_tc(W, x + (size_t)b * K, out + (size_t)b * n_rows, n_rows, K, take, s);
            if (rc == MLQ_ERR_UNSUPPORTED && b == 0) break;
        }
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
    if constexpr (sizeof(WT) == 2) {
        // more than four activation rows: one GEMM instead of passes of four over the matrix
        if (B > 4 && !getenv("MLQ_NO_GEMM16")) {
            const int rc = launch_gemm16(W, std::is_same<WT, __nv_bfloat16>::value ? 1 : 0, x, out, n_rows, K, B, s);
            if (rc != MLQ_ERR_UNSUPPORTED) return rc;
        }
    }
    const WT *w = reinterpret_cast<const WT *>(W);
    const int V = 16 / sizeof(WT);
    const int vec_ok = (K % V == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0) &&
                       ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && ((K * 4) % 16 == 0);
    if (n_rows < c->num_sms * 8) {
        // too few rows for a warp each to fill the GPU: a CTA per row
        for (int b = 0; b < B; b += kFewRowsMaxB) {
            const int take = (B - b) < kFewRowsMaxB ? (B - b) : kFewRowsMaxB;
            const WT *none = nullptr;
            float *none_out = nullptr;
            if (!MLQ_CUDA(launch_pdl_k(k_gemv_float_rows<WT>, dim3(n_rows), dim3(256), 0, s, w, x + (size_t)b * K,
                                       out + (size_t)b * n_rows, n_rows, K, take, vec_ok, none, none_out)))
                return MLQ_ERR_CUDA;
        }
        return MLQ_OK;
    }
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

// fp32 router rows plus one more fp32 row from its own pointer in the same launch (a MoE
// layer's router and its shared expert's gate score): out [B][n_rows], out_extra [B]
int launch_router_rows_f32(const float *W, const float *w_extra, const float *x, float *out, float *out_extra,
                           int n_rows, int K, int B, cudaStream_t s) {
    const int vec_ok = (K % 4 == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0) &&
                       ((reinterpret_cast<uintptr_t>(w_extra) & 15) == 0) &&
                       ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    for (int b = 0; b < B; b += kFewRowsMaxB) {
        const int take = (B - b) < kFewRowsMaxB ? (B - b) : kFewRowsMaxB;
        if (!MLQ_CUDA(launch_pdl_k(k_gemv_float_rows<float>, dim3(n_rows + 1), dim3(256), 0, s, W, x + (size_t)b * K,
                                   out + (size_t)b * n_rows, n_rows, K, take, vec_ok, w_extra, out_extra + b)))
            return MLQ_ERR_CUDA;
    }
    return MLQ_OK;
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
// Grouped expert GEMV: the rows of one call are ordered by expert (stable) and every
// active expert's matrix is streamed once for all of its rows, up to 8 rows per pass.
// Work items (expert e, first sorted position m0, row count mc <= 8, tile t) are listed
// expert-major by the planner.  Tiles are the same contiguous byte ranges as in k_gemv_q,
// at base + e * estride.  One launch can stream two matrices of one type and shape (gate
// and up): tiles [0, T) of an item address the first and [T, 2T) the second.
//
// The activation rows are encoded once, before the launch, into packed rows in global
// memory (k_encode_packed); the producer warp bulk-copies an item's mc rows into one of
// two shared-memory activation slots when (e, m0) changes, next to the weight tiles, so
// no decode warp ever waits on an encode.  CTAs take groups of G consecutive items
// round-robin (group g -> CTA g % grid), which spreads the costlier many-row items over
// all SMs.  The producer hands every tile's item to the decode warps in the stage itself.
struct GroupItem { int e, m0, mc, tile; };

struct GroupArgs {
    GemvArgs g;                 // W / out: first matrix; n_rows / K / row_bytes of one expert
    long long estride;          // bytes between experts of the first matrix
    const uint8_t *W2;          // second matrix (tiles >= tiles_per_expert), or null
    long long estride2;
    float *out2;
    const GroupItem *items;
    const int *n_items;         // item count, written on the device by the planner
    int tiles_per_expert;
    const uint8_t *planes;      // packed activation rows in sorted order
    int n_xslots;               // shared-memory activation slots (2, or 1 for very long rows)
    int xslot_bytes;            // 8 packed rows
    int group;                  // items per round-robin group
    int lane_group_log;         // log2 of the lanes per weight row (>= min(units per row, 32))
    const int *out_rows;        // result of sorted position p -> row out_rows[p] (identity if null)
};

struct GroupLayout {
    int off_bar, off_flag, off_x, off_stage, total;
};

__host__ __device__ inline GroupLayout group_layout(int xslot_bytes, int n_xslots, int stage_bytes, int n_stages) {
    GroupLayout L;
    int o = 0;
    L.off_bar = o;   o += (2 * kMaxStages + 4) * 8;   // full, empty, x_full[2], x_empty[2]
    L.off_flag = o;  o += 16;
    o = align_up(o, 128);
    L.off_x = o;     o = align_up(o + n_xslots * xslot_bytes, 128);
    L.off_stage = o; o += n_stages * stage_bytes;
    L.total = o;
    return L;
}

// item index of a CTA's it-th tile (round-robin groups of G)
__device__ __forceinline__ int group_item_index(int it, int G) {
    return ((it / G) * (int)gridDim.x + (int)blockIdx.x) * G + it % G;
}

// first byte, matrix-local tile and output base of an item's tile
struct ItemTile {
    uintptr_t g0;
    float *out;
    int tile;
};
__device__ __forceinline__ ItemTile item_tile(const GroupArgs &ga, const GroupItem &item, long long tile_bytes) {
    const bool second = item.tile >= ga.tiles_per_expert;
    ItemTile t;
    t.tile = second ? item.tile - ga.tiles_per_expert : item.tile;
    const uint8_t *W = second ? ga.W2 : ga.g.W;
    const long long es = second ? ga.estride2 : ga.estride;
    t.g0 = reinterpret_cast<uintptr_t>(W) + (uintptr_t)((long long)item.e * es) +
           (uintptr_t)((long long)t.tile * tile_bytes);
    t.out = second ? ga.out2 : ga.g.out;
    return t;
}

// the item travels in the last 16 bytes of its stage (past the tile and the decode slack)
__device__ __forceinline__ GroupItem *stage_item(uint8_t *stage, int stage_bytes) {
    return reinterpret_cast<GroupItem *>(stage + stage_bytes - 16);
}

__device__ __forceinline__ void produce_group_tiles(const GroupArgs &ga, uint8_t *stages, uint8_t *xslots,
                                                    uint64_t *full, uint64_t *empty, uint64_t *xfull,
                                                    uint64_t *xempty, volatile int *abort_flag, int n_items,
                                                    int lane) {
    const GemvArgs &a = ga.g;
    const uint64_t pol = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    const long long mat_bytes = (long long)a.n_rows * a.row_bytes;
    const int G = ga.group;
    const int prb = packed_row_bytes(a.K);
    int run = 0, cur_e = -1, cur_m0 = -1;
    GroupItem mine{-1, 0, 0, 0};
    for (int it = 0;; ++it) {
        const int j = it % G;
        if (j == 0) {   // lane i < G holds item i of the group
            const int li = group_item_index(it, G) + lane;
            mine = (lane < G && li < n_items) ? ga.items[li] : GroupItem{-1, 0, 0, 0};
        }
        const GroupItem item{__shfl_sync(0xffffffffu, mine.e, j), __shfl_sync(0xffffffffu, mine.m0, j),
                             __shfl_sync(0xffffffffu, mine.mc, j), __shfl_sync(0xffffffffu, mine.tile, j)};
        const int s = it % a.n_stages;
        if (it >= a.n_stages) {
            if (!producer_wait_empty(a, empty, abort_flag, it - a.n_stages, lane)) return;
        }
        uint8_t *st = stages + (size_t)s * a.stage_bytes;
        if (item.e < 0) {   // end of this CTA's items
            if (lane == 0) {
                *stage_item(st, a.stage_bytes) = GroupItem{-1, 0, 0, 0};
                mbar_arrive(&full[s]);
            }
            return;
        }
        const ItemTile t = item_tile(ga, item, tile_bytes);
        const long long b0 = (long long)t.tile * tile_bytes;
        const long long b1 = min(b0 + tile_bytes, mat_bytes);
        const uintptr_t g0 = t.g0, g1 = t.g0 + (uintptr_t)(b1 - b0);
        const uintptr_t gd = g0 & ~uintptr_t(15);
        const uintptr_t j0 = (g0 + 15) & ~uintptr_t(15);
        const uintptr_t j1 = g1 & ~uintptr_t(15);
        if (j1 > j0) {
            if (g0 + lane < j0) st[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
            if (j1 + lane < g1) st[j1 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(j1 + lane));
        } else {
            if (g0 + lane < g1) st[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
        }
        __syncwarp();
        if (lane == 0) {
            *stage_item(st, a.stage_bytes) = item;
            if (j1 > j0) {
                mbar_arrive_expect_tx(&full[s], (uint32_t)(j1 - j0));
                bulk_g2s(st + (j0 - gd), reinterpret_cast<const void *>(j0), (uint32_t)(j1 - j0), &full[s], pol);
            } else {
                mbar_arrive(&full[s]);
            }
        }
        // a new activation run: its rows into the next slot once the decode warps are done
        // with the run that used it (issued after the tile, which they need to see first)
        if (item.e != cur_e || item.m0 != cur_m0) {
            const int xs = run % ga.n_xslots;
            bool ok = true;
            if (run >= ga.n_xslots && lane == 0) ok = mbar_wait_bounded(&xempty[xs], ((run / ga.n_xslots) - 1) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *abort_flag) {
                if (lane == 0) { *abort_flag = 1; raise_status(a.status, DEV_ST_WAIT_EMPTY); }
                return;
            }
            if (lane == 0) {
                const uint32_t bytes = (uint32_t)(item.mc * prb);
                mbar_arrive_expect_tx(&xfull[xs], bytes);
                bulk_g2s(xslots + (size_t)xs * ga.xslot_bytes, ga.planes + (size_t)item.m0 * prb, bytes, &xfull[xs],
                         pol_x);
            }
            ++run;
            cur_e = item.e;
            cur_m0 = item.m0;
        }
    }
}

// Lanes form groups of GS = 2^gs_log (the units of one weight row, stepping by GS); warp
// w takes rows w + 16 (j * RPW + gi) of a tile, RPW = 32 / GS rows per pass.
struct LaneMap {
    int gs_log, rpw, gi, gl, U;
};

// One staged tile against MC (>= mc) activation rows: each unit is decoded once and
// dotted with every activation row from shared memory (conflict-free swizzled planes).
template <int QT, int MC, bool A16>
__device__ __forceinline__ void group_tile_rows(const GroupArgs &ga, const uint8_t *stage, const XPlanes &xp,
                                                const GroupItem &item, const ItemTile &t, const LaneMap &lm,
                                                int warp) {
    const GemvArgs &a = ga.g;
    const int GS = 1 << lm.gs_log;
    const int row0 = t.tile * a.rpt;
    const int mc = item.mc;
    for (int base = 0; warp + kFastWarps * base < a.rpt; base += lm.rpw) {
        const int r = warp + kFastWarps * (base + lm.gi);
        const bool v = r < a.rpt && row0 + r < a.n_rows;
        float acc[MC];
#pragma unroll
        for (int m = 0; m < MC; m++) acc[m] = 0.0f;
        if (v) {
            const uint8_t *pr = stage + (size_t)r * a.row_bytes;
            for (int u = lm.gl; u < lm.U; u += GS) {
                W<QT> w;
                if constexpr (A16) w.decode_a16(pr, u);
                else w.decode(pr, u);
#pragma unroll
                for (int m = 0; m < MC; m++) {
                    if (m < mc) {
                        XU<QT> xu;
                        load_xu<QT>(xp, m, u, xu);
                        acc[m] += w.dot(xu);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MC; m++) {
            if (m < mc) {
                for (int o = GS >> 1; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
            }
        }
        if (lm.gl == 0 && v) {
#pragma unroll
            for (int m = 0; m < MC; m++) {
                if (m < mc) {
                    const int p = item.m0 + m;
                    t.out[(size_t)(ga.out_rows ? __ldg(ga.out_rows + p) : p) * a.n_rows + row0 + r] = acc[m];
                }
            }
        }
    }
}

template <int QT, bool A16>
__global__ void __launch_bounds__(kFastThreads, 1) k_gemv_grouped(GroupArgs ga) {
    const GemvArgs &a = ga.g;
    extern __shared__ __align__(128) uint8_t smem[];
    const GroupLayout L = group_layout(ga.xslot_bytes, ga.n_xslots, a.stage_bytes, a.n_stages);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kMaxStages;
    uint64_t *xfull = empty + kMaxStages;
    uint64_t *xempty = xfull + 2;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.off_flag);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.n_stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kFastWarps);
        }
        for (int j = 0; j < 2; j++) {
            mbar_init(&xfull[j], 1);
            mbar_init(&xempty[j], kFastWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();   // the item list and the activation rows are earlier kernels' outputs
    pdl_trigger();
    if (warp == kFastWarps) {
        produce_group_tiles(ga, smem + L.off_stage, smem + L.off_x, full, empty, xfull, xempty, abort_flag,
                            *ga.n_items, lane);
        return;
    }
    int run = 0, cur_e = -1, cur_m0 = -1, xs = 0;
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    LaneMap lm;
    lm.gs_log = ga.lane_group_log;
    lm.rpw = 32 >> lm.gs_log;
    lm.gi = lane >> lm.gs_log;
    lm.gl = lane & ((1 << lm.gs_log) - 1);
    lm.U = a.K / Fmt<QT>::UE;
    for (int it = 0;; ++it) {
        const int s = it % a.n_stages;
        if (!consume_wait(a, full, abort_flag, it, lane)) break;
        uint8_t *st = smem + L.off_stage + (size_t)s * a.stage_bytes;
        GroupItem v;
        if (lane == 0) v = *stage_item(st, a.stage_bytes);
        GroupItem item;
        item.e = __shfl_sync(0xffffffffu, v.e, 0);
        item.m0 = __shfl_sync(0xffffffffu, v.m0, 0);
        item.mc = __shfl_sync(0xffffffffu, v.mc, 0);
        item.tile = __shfl_sync(0xffffffffu, v.tile, 0);
        if (item.e < 0) break;
        if (item.e != cur_e || item.m0 != cur_m0) {
            // a new run: release the previous run's activation slot, wait for this one's
            if (run > 0 && lane == 0) mbar_arrive(&xempty[(run - 1) % ga.n_xslots]);
            xs = run % ga.n_xslots;
            bool ok = true;
            if (lane == 0) ok = mbar_wait_bounded(&xfull[xs], (run / ga.n_xslots) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) { *abort_flag = 1; raise_status(a.status, DEV_ST_WAIT_FULL); }
                break;
            }
            ++run;
            cur_e = item.e;
            cur_m0 = item.m0;
        }
        const XPlanes xp = packed_planes(smem + L.off_x + (size_t)xs * ga.xslot_bytes, a.K);
        const ItemTile t = item_tile(ga, item, tile_bytes);
        const uint8_t *stage = st + (t.g0 & 15);
        if (item.mc == 1) group_tile_rows<QT, 1, A16>(ga, stage, xp, item, t, lm, warp);
        else if (item.mc == 2) group_tile_rows<QT, 2, A16>(ga, stage, xp, item, t, lm, warp);
        else if (item.mc <= 4) group_tile_rows<QT, 4, A16>(ga, stage, xp, item, t, lm, warp);
        else group_tile_rows<QT, 8, A16>(ga, stage, xp, item, t, lm, warp);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// activation element k of sorted row p: x[rows[p]] (or x[p]), or silu(clamp(g, +-80)) * u
// of rows p of g = x and u = x2 (k_swiglu, quant_kernels_omp.c:2157-2164)
struct GroupRows {
    const float *x, *x2;
    const int *rows;
    int K;
    int row_div;      // source row = rows[p] / row_div (several rows reading one token's activations)
    float clamp;      // silu(clamp(x, +-clamp)) * x2 when x2 is set (HUGE_VALF: no clamp)
    int stride;       // floats between source rows (K for dense rows)
    __device__ __forceinline__ float operator()(int p, int k) const {
        int r = rows ? __ldg(rows + p) : p;
        if (row_div > 1) r /= row_div;
        const size_t o = (size_t)r * stride + k;
        float v = __ldg(x + o);
        if (x2) {
            const float g = fminf(fmaxf(v, -clamp), clamp);
            v = (g / (1.0f + expf(-g))) * __ldg(x2 + o);
        }
        return v;
    }
};

// R packed activation rows: one warp per 32-element block (many independent warps: the
// kernel is latency-bound on its loads, not on work)
__global__ void __launch_bounds__(256) k_encode_packed(GroupRows src, int R, int K, uint8_t *__restrict__ planes) {
    pdl_wait();   // the rows are an earlier kernel's output
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int kbr = K / 32;
    const long long blk = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (blk >= (long long)R * kbr) return;   // warp-uniform
    const int p = (int)(blk / kbr), kb = (int)(blk - (long long)p * kbr);
    encode_block_packed(src(p, 32 * kb + lane), p, kb, K, planes, lane);
}

// Host-free grouping: a stable order of the rows by expert and the work-item lists of up
// to three tilings.  Deterministic and parallel: counts per expert (order-free atomics),
// block-wide exclusive scans of the row and 8-row-chunk counts, then positions
// kPlanThreads rows at a time (rank among the warp's rows of the same expert from
// __match_any_sync, plus the counts of earlier warps and earlier row groups).
constexpr int kPlanThreads = 256;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kPlanMaxE = 1024;

struct PlanLists {
    GroupItem *items[3];
    int tiles[3];
    int n;
};

__global__ void __launch_bounds__(kPlanThreads) k_group_plan(const int *__restrict__ eid, int eid_stride, int R, int E,
                                                             PlanLists pl, int *__restrict__ sorted_pos,
                                                             int *__restrict__ src_row, int *__restrict__ n_items) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    extern __shared__ int sm_plan[];
    int *run = sm_plan;          // [E] counts, then running positions
    int *so = run + E;           // [E + 1] first sorted position of each expert
    int *si = so + E + 1;        // [E + 1] first 8-row chunk of each expert
    int *wc = si + E + 1;        // [kPlanWarps][E] counts of the current row group, then bases
    __shared__ int wsum[2][kPlanWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < E; e += kPlanThreads) run[e] = 0;
    __syncthreads();
    for (int r = tid; r < R; r += kPlanThreads) {
        const int e = eid[(size_t)r * eid_stride];
        if (e >= 0 && e < E) atomicAdd(&run[e], 1);
    }
    __syncthreads();
    // exclusive scans; thread tid owns experts [tid * ept, (tid + 1) * ept)
    const int ept = (E + kPlanThreads - 1) / kPlanThreads;
    const int e0 = min(E, tid * ept), e1 = min(E, e0 + ept);
    int own_r = 0, own_c = 0;
    for (int e = e0; e < e1; e++) {
        own_r += run[e];
        own_c += (run[e] + 7) / 8;
    }
    int inc_r = own_r, inc_c = own_c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, inc_r, o), b = __shfl_up_sync(0xffffffffu, inc_c, o);
        if (lane >= o) {
            inc_r += a;
            inc_c += b;
        }
    }
    if (lane == 31) {
        wsum[0][warp] = inc_r;
        wsum[1][warp] = inc_c;
    }
    __syncthreads();
    int pr = inc_r - own_r, pc = inc_c - own_c;
    for (int w = 0; w < warp; w++) {
        pr += wsum[0][w];
        pc += wsum[1][w];
    }
    for (int e = e0; e < e1; e++) {
        so[e] = pr;
        si[e] = pc;
        pr += run[e];
        pc += (run[e] + 7) / 8;
    }
    if (tid == kPlanThreads - 1) {   // the last thread's running sums are the totals
        so[E] = pr;
        si[E] = pc;
    }
    __syncthreads();
    if (tid < pl.n) n_items[tid] = si[E] * pl.tiles[tid];
    for (int e = tid; e < E; e += kPlanThreads) run[e] = so[e];
    __syncthreads();
    // stable positions
    for (int c0 = 0; c0 < R; c0 += kPlanThreads) {
        const int r = c0 + tid;
        const int e = r < R ? eid[(size_t)r * eid_stride] : -1;
        const bool valid = e >= 0 && e < E;
        const unsigned same = __match_any_sync(0xffffffffu, valid ? e : -1);
        const int rank = __popc(same & ((1u << lane) - 1u));
        for (int i = tid; i < kPlanWarps * E; i += kPlanThreads) wc[i] = 0;
        __syncthreads();
        if (valid && rank == 0) wc[warp * E + e] = __popc(same);
        __syncthreads();
        for (int x = tid; x < E; x += kPlanThreads) {
            int acc = run[x];
            for (int w = 0; w < kPlanWarps; w++) {
                const int n = wc[w * E + x];
                wc[w * E + x] = acc;
                acc += n;
            }
            run[x] = acc;
        }
        __syncthreads();
        if (valid) {
            const int p = wc[warp * E + e] + rank;
            sorted_pos[r] = p;
            src_row[p] = r;
        } else if (r < R) {
            sorted_pos[r] = -1;
        }
        __syncthreads();
    }
    // positions past the valid rows (rows with an id outside [0, E)) read row 0, so that
    // consumers of src_row stay in bounds
    for (int p = so[E] + tid; p < R; p += kPlanThreads) src_row[p] = 0;
    // items: warp per chunk (ascending), lanes over the tiles; the chunk's expert is found
    // by advancing over si 32 experts per ballot (si is non-decreasing)
    const int n_chunks = si[E];
    int e = 0;
    for (int c = warp; c < n_chunks; c += kPlanWarps) {
        for (;;) {
            const int x = e + 1 + lane;
            const unsigned b = __ballot_sync(0xffffffffu, x < E && si[x] <= c);
            e += __popc(b);
            if (b != 0xffffffffu) break;
        }
        const int m0 = (c - si[e]) * 8;
        const int mc = min(8, so[e + 1] - so[e] - m0);
        for (int l = 0; l < pl.n; l++) {
            const int T = pl.tiles[l];
            GroupItem *dst = pl.items[l] + (size_t)c * T;
            for (int t = lane; t < T; t += 32) dst[t] = GroupItem{e, so[e] + m0, mc, t};
        }
    }
}

// rows per grouped tile: a multiple of the 16 decode warps, about 48 KB (every item then
// gives each warp several whole rows to amortise its bookkeeping over), <= 64.  Config-3
// MoE layers (16 tokens) measured 12.7 ms per 48-layer step at 36 KB tiles and 128 KB
// groups, 10.85 ms at 48 KB tiles and 64 KB groups (MLQ_GROUP_TILE_KB, MLQ_GROUP_KB override)
static int grouped_rpt(long long rb) {
    static int tile_kb = -1;
    if (tile_kb < 0) {
        const char *e = getenv("MLQ_GROUP_TILE_KB");
        tile_kb = e && atoi(e) > 0 ? atoi(e) : 48;
    }
    long long r = (long long)tile_kb * 1024 / rb;
    r = r < 16 ? 16 : (r > 64 ? 64 : r);
    return (int)(r / 16 * 16);
}

template <int QT, bool A16>
static int launch_grouped_t(const GroupedCall &gc, cudaStream_t s) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    const long long rb = (long long)(gc.K / Fmt<QT>::BE) * Fmt<QT>::BB;
    const int rpt = grouped_rpt(rb);
    const int stage_bytes = align_up((int)(rpt * rb), 16) + 48;
    const int xslot_bytes = 8 * packed_row_bytes(gc.K);
    const int n_xslots = group_layout(xslot_bytes, 2, stage_bytes, 3).total <= kSmemBudget ? 2 : 1;
    const int fixed = group_layout(xslot_bytes, n_xslots, stage_bytes, 0).total;
    const int n_stages = fixed < kSmemBudget ? stages_for(fixed, stage_bytes) : 0;
    if (n_stages < 2) {
        set_error(MLQ_ERR_CAPACITY, "grouped experts: K=%d too large for the stage ring", gc.K);
        return MLQ_ERR_CAPACITY;
    }
    const int U = gc.K / Fmt<QT>::UE;
    int gs_log = 0;
    while ((1 << gs_log) < U && gs_log < 5) gs_log++;
    // items per round-robin group: about 64 KB of weights, fewer when the call is small
    // enough that every SM should still get a couple of groups
    const long long tb = (long long)rpt * rb;
    static int group_kb = -1;
    if (group_kb < 0) {
        const char *e = getenv("MLQ_GROUP_KB");
        group_kb = e && atoi(e) > 0 ? atoi(e) : 64;
    }
    long long G = (long long)group_kb * 1024 / tb;
    const long long spread = (long long)gc.n_items_bound / (2LL * c->num_sms);
    if (spread < G) G = spread;
    G = G < 1 ? 1 : (G > 32 ? 32 : G);
    GroupArgs ga{};
    GemvArgs &a = ga.g;
    a.W = gc.W; a.x = nullptr; a.out = gc.out; a.n_rows = gc.n_rows; a.K = gc.K; a.nb_x = 8;
    a.row_bytes = rb; a.total_bytes = rb * gc.n_rows; a.rpt = rpt; a.wpr = 1;
    a.stage_bytes = stage_bytes; a.n_stages = n_stages; a.status = c->d_status;
    ga.estride = gc.estride;
    ga.W2 = gc.W2; ga.estride2 = gc.estride2; ga.out2 = gc.out2;
    ga.items = (const GroupItem *)gc.items;
    ga.n_items = gc.n_items_dev;
    ga.tiles_per_expert = (gc.n_rows + rpt - 1) / rpt;
    ga.planes = gc.planes;
    ga.n_xslots = n_xslots;
    ga.xslot_bytes = xslot_bytes;
    ga.group = (int)G;
    ga.lane_group_log = gs_log;
    ga.out_rows = gc.out_rows;
    // the item count is only known on the device: the grid covers the bound
    const int groups = (int)((gc.n_items_bound + G - 1) / G);
    const int grid = groups < c->num_sms ? (groups > 0 ? groups : 1) : c->num_sms;
    static bool attr = false;
    if (!attr) {
        if (!MLQ_CUDA(cudaFuncSetAttribute(k_gemv_grouped<QT, A16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kMaxSmem)))
            return MLQ_ERR_CUDA;
        attr = true;
    }
    count_launch();
    return MLQ_CUDA(launch_pdl(k_gemv_grouped<QT, A16>, dim3(grid), dim3(kFastThreads),
                               fixed + n_stages * stage_bytes, s, ga))
               ? MLQ_OK
               : MLQ_ERR_CUDA;
}

// Q4_K / Q5_K rows on 16-byte boundaries (row bytes, expert strides and bases all
// multiples of 16) decode with 128-bit shared-memory loads
template <int QT>
static int launch_grouped_a(const GroupedCall &gc, cudaStream_t s) {
    if constexpr (QT == MLQ_Q4_K || QT == MLQ_Q5_K) {
        const long long rb = (long long)(gc.K / Fmt<QT>::BE) * Fmt<QT>::BB;
        const bool al = rb % 16 == 0 && (reinterpret_cast<uintptr_t>(gc.W) & 15) == 0 && gc.estride % 16 == 0 &&
                        (!gc.W2 || ((reinterpret_cast<uintptr_t>(gc.W2) & 15) == 0 && gc.estride2 % 16 == 0));
        if (al) return launch_grouped_t<QT, true>(gc, s);
    }
    return launch_grouped_t<QT, false>(gc, s);
}

int grouped_tiles_per_expert(int qt, int n_rows, int K) {
    const long long rb = (long long)(K / block_elems(qt)) * block_bytes(qt);
    if (rb <= 0) return 0;
    const int rpt = grouped_rpt(rb);
    return (n_rows + rpt - 1) / rpt;
}

size_t grouped_packed_bytes(int R, int K) { return (size_t)R * packed_row_bytes(K); }

int launch_grouped(const GroupedCall &gc, cudaStream_t s) {
    if (!gc.planes || (reinterpret_cast<uintptr_t>(gc.planes) & 15) || gc.K % 32) {
        set_error(MLQ_ERR_ARG, "grouped experts: packed rows must be 16-byte aligned, K %% 32 == 0");
        return MLQ_ERR_ARG;
    }
    switch (gc.qt) {
        case MLQ_Q4_0: return launch_grouped_a<MLQ_Q4_0>(gc, s);
        case MLQ_Q4_1: return launch_grouped_a<MLQ_Q4_1>(gc, s);
        case MLQ_Q5_0: return launch_grouped_a<MLQ_Q5_0>(gc, s);
        case MLQ_Q8_0: return launch_grouped_a<MLQ_Q8_0>(gc, s);
        case MLQ_Q4_K: return launch_grouped_a<MLQ_Q4_K>(gc, s);
        case MLQ_Q5_K: return launch_grouped_a<MLQ_Q5_K>(gc, s);
        case MLQ_Q6_K: return launch_grouped_a<MLQ_Q6_K>(gc, s);
        case MLQ_MXFP4: return launch_grouped_a<MLQ_MXFP4>(gc, s);
        case MLQ_MXFP4_REF: return launch_grouped_a<MLQ_MXFP4_REF>(gc, s);
        default:
            set_error(MLQ_ERR_TYPE, "grouped experts: type %d", gc.qt);
            return MLQ_ERR_TYPE;
    }
}

int launch_encode_packed(const float *x, const float *x2, const int *rows, int R, int K, uint8_t *planes,
                         cudaStream_t s, int row_div, float clamp, int x_stride) {
    if (R <= 0) return MLQ_OK;
    const long long blocks = ((long long)R * (K / 32) + 7) / 8;
    count_launch();
    return MLQ_CUDA(launch_pdl_n(k_encode_packed, dim3((unsigned)blocks), dim3(256), 0, s,
                                 GroupRows{x, x2, rows, K, row_div, clamp, x_stride > 0 ? x_stride : K},
                                 R, K, planes))
               ? MLQ_OK
               : MLQ_ERR_CUDA;
}

int launch_group_plan(const int *eid, int R, int E, int n_lists, void *const *items, const int *tiles,
                      int *sorted_pos, int *src_row, int *n_items, cudaStream_t s, int eid_stride) {
    if (E <= 0 || E > kPlanMaxE || n_lists < 1 || n_lists > 3) {
        set_error(MLQ_ERR_CAPACITY, "grouped experts: %d experts (1..%d), %d item lists", E, kPlanMaxE, n_lists);
        return MLQ_ERR_CAPACITY;
    }
    PlanLists pl{};
    pl.n = n_lists;
    for (int l = 0; l < n_lists; l++) {
        pl.items[l] = (GroupItem *)items[l];
        pl.tiles[l] = tiles[l];
    }
    const size_t sm = sizeof(int) * (3 * (size_t)E + 2 + (size_t)kPlanWarps * E);
    return MLQ_CUDA(launch_pdl_k(k_group_plan, dim3(1), dim3(kPlanThreads), sm, s, eid, eid_stride, R, E, pl,
                                 sorted_pos, src_row, n_items))
               ? MLQ_OK
               : MLQ_ERR_CUDA;
}

// ------------------------------------------------------------------------------ decode GEMV
// Segmented decode GEMV for the batch engine's B <= 8 step: up to four matrices of one
// type sharing one input (Q, K and V; gate and up) in one launch, the input read as
// packed activation rows that an earlier kernel encoded once (the RMSNorm, or
// k_encode_packed), and the step's elementwise neighbours folded into the store:
//   plain     out_s[m][r] = W_s[r] . x_m
//   residual  out_s[m][r] = res_s[m][r] + W_s[r] . x_m          (o / down + residual add)
//   pair      out[m][r] = silu(G[r] . x_m) * (U[r] . x_m)        (gate / up + SiLU-mul)
// The producer warp streams the weight tiles it will need before waiting for the previous
// kernel (programmatic dependent launch: weights do not depend on it), then bulk-copies the
// activation rows once; 16 decode warps take the rows of every tile (lane groups for short
// rows) with each unit decoded once and dotted with all B rows.
constexpr int kSegMax = 4;

struct SegArgs {
    const uint8_t *W[kSegMax];
    float *out[kSegMax];
    const float *res[kSegMax];    // residual of each segment (null: plain store)
    int n_rows[kSegMax];
    int tile0[kSegMax + 1];       // first tile of each segment; tile0[n_seg] = all tiles
    int n_seg;
    int pair;                     // segments 0 / 1 are gate / up of one shape; tiles cover both
    const uint8_t *planes;        // packed activation rows [B]
    int B, K;
    long long row_bytes;
    int rpt, region_bytes, stage_bytes, n_stages, gs_log;
    int *status;
};

struct SegLayout {
    int off_bar, off_flag, off_x, off_stage, total;
};

__host__ __device__ inline SegLayout seg_layout(int x_bytes, int stage_bytes, int n_stages) {
    SegLayout L;
    int o = 0;
    L.off_bar = o;   o += (2 * kMaxStages + 1) * 8;   // full, empty, x_full
    L.off_flag = o;  o += 16;
    o = align_up(o, 128);
    L.off_x = o;     o = align_up(o + x_bytes, 128);
    L.off_stage = o; o += n_stages * stage_bytes;
    L.total = o;
    return L;
}

__device__ __forceinline__ int seg_of(const SegArgs &a, int tile) {
    int s = 0;
    while (s + 1 < a.n_seg && tile >= a.tile0[s + 1]) s++;
    return s;
}

// Stage the byte range of local tile lt of matrix W (n_rows rows) into a region: lanes
// copy the ragged head / tail, the 16-byte-aligned interior is returned for one bulk copy.
struct BulkPart {
    uint8_t *dst;
    const void *src;
    uint32_t bytes;
};
__device__ __forceinline__ BulkPart stage_tile_bytes(const SegArgs &a, const uint8_t *W, int n_rows, int lt,
                                                     uint8_t *region, int lane) {
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    const long long b0 = (long long)lt * tile_bytes;
    const long long b1 = min(b0 + tile_bytes, (long long)n_rows * a.row_bytes);
    const uintptr_t g0 = reinterpret_cast<uintptr_t>(W) + (uintptr_t)b0;
    const uintptr_t g1 = reinterpret_cast<uintptr_t>(W) + (uintptr_t)b1;
    const uintptr_t gd = g0 & ~uintptr_t(15);
    const uintptr_t j0 = (g0 + 15) & ~uintptr_t(15);
    const uintptr_t j1 = g1 & ~uintptr_t(15);
    if (j1 > j0) {
        if (g0 + lane < j0) region[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
        if (j1 + lane < g1) region[j1 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(j1 + lane));
        return BulkPart{region + (j0 - gd), reinterpret_cast<const void *>(j0), (uint32_t)(j1 - j0)};
    }
    if (g0 + lane < g1) region[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
    return BulkPart{nullptr, nullptr, 0};
}

__device__ __forceinline__ void seg_issue(const SegArgs &a, int tile, uint8_t *st, uint64_t *full, uint64_t pol,
                                          int lane) {
    BulkPart p0, p1{nullptr, nullptr, 0};
    if (a.pair) {
        p0 = stage_tile_bytes(a, a.W[0], a.n_rows[0], tile, st, lane);
        p1 = stage_tile_bytes(a, a.W[1], a.n_rows[1], tile, st + a.region_bytes, lane);
    } else {
        const int s = seg_of(a, tile);
        p0 = stage_tile_bytes(a, a.W[s], a.n_rows[s], tile - a.tile0[s], st, lane);
    }
    __syncwarp();
    if (lane == 0) {
        const uint32_t tx = p0.bytes + p1.bytes;
        if (tx) {
            mbar_arrive_expect_tx(full, tx);
            if (p0.bytes) bulk_g2s(p0.dst, p0.src, p0.bytes, full, pol);
            if (p1.bytes) bulk_g2s(p1.dst, p1.src, p1.bytes, full, pol);
        } else {
            mbar_arrive(full);
        }
    }
}

// dot of staged row r (region base + its head offset) with the B activation rows
template <int QT, int MC, bool A16>
__device__ __forceinline__ void seg_row_dot(const uint8_t *row, const XPlanes &xp, int B, int U, int GS, int gl,
                                            float (&acc)[MC]) {
    for (int u = gl; u < U; u += GS) {
        W<QT> w;
        if constexpr (A16) w.decode_a16(row, u);
        else w.decode(row, u);
#pragma unroll
        for (int m = 0; m < MC; m++) {
            if (m < B) {
                XU<QT> xu;
                load_xu<QT>(xp, m, u, xu);
                acc[m] += w.dot(xu);
            }
        }
    }
}

// the same for a gate row and an up row at once: each activation slice is loaded once
// for both (the pair's rows share their input)
template <int QT, int MC, bool A16>
__device__ __forceinline__ void seg_row_dot2(const uint8_t *row_a, const uint8_t *row_b, const XPlanes &xp, int B,
                                             int U, int GS, int gl, float (&acc)[MC], float (&acc2)[MC]) {
    for (int u = gl; u < U; u += GS) {
        W<QT> wa, wb;
        if constexpr (A16) {
            wa.decode_a16(row_a, u);
            wb.decode_a16(row_b, u);
        } else {
            wa.decode(row_a, u);
            wb.decode(row_b, u);
        }
#pragma unroll
        for (int m = 0; m < MC; m++) {
            if (m < B) {
                XU<QT> xu;
                load_xu<QT>(xp, m, u, xu);
                acc[m] += wa.dot(xu);
                acc2[m] += wb.dot(xu);
            }
        }
    }
}

template <int QT, int MC, bool A16>
__global__ void __launch_bounds__(kFastThreads, 1) k_gemv_seg(SegArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int prb = packed_row_bytes(a.K);
    const SegLayout L = seg_layout(a.B * prb, a.stage_bytes, a.n_stages);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kMaxStages;
    uint64_t *xfull = empty + kMaxStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.off_flag);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = a.tile0[a.n_seg];
    const int n_iter = (n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.n_stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kFastWarps);
        }
        mbar_init(xfull, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    uint8_t *stages = smem + L.off_stage;
    if (warp == kFastWarps) {
        const uint64_t pol = policy_evict_first();
        // the first stages' weights before the wait: they do not depend on the previous kernel
        const int pre = n_iter < a.n_stages ? n_iter : a.n_stages;
        for (int it = 0; it < pre; ++it)
            seg_issue(a, (int)blockIdx.x + it * (int)gridDim.x, stages + (size_t)it * a.stage_bytes, &full[it], pol,
                      lane);
        pdl_wait();
        pdl_trigger();
        if (lane == 0) {
            const uint32_t xb = (uint32_t)(a.B * prb);
            mbar_arrive_expect_tx(xfull, xb);
            bulk_g2s(smem + L.off_x, a.planes, xb, xfull, policy_evict_last());
        }
        for (int it = pre; it < n_iter; ++it) {
            const int s = it % a.n_stages;
            bool ok = true;
            if (lane == 0) ok = mbar_wait_bounded(&empty[s], ((it / a.n_stages) - 1) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *abort_flag) {
                if (lane == 0) { *abort_flag = 1; raise_status(a.status, DEV_ST_WAIT_EMPTY); }
                return;
            }
            seg_issue(a, (int)blockIdx.x + it * (int)gridDim.x, stages + (size_t)s * a.stage_bytes, &full[s], pol,
                      lane);
        }
        return;
    }
    pdl_wait();   // the residual rows are an earlier kernel's output too
    pdl_trigger();
    {
        bool ok = true;
        if (lane == 0) ok = mbar_wait_bounded(xfull, 0);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            if (lane == 0) { *abort_flag = 1; raise_status(a.status, DEV_ST_WAIT_FULL); }
            return;
        }
    }
    const XPlanes xp = packed_planes(smem + L.off_x, a.K);
    const int GS = 1 << a.gs_log, RPW = 32 >> a.gs_log;
    const int gi = lane >> a.gs_log, gl = lane & (GS - 1);
    const int U = a.K / Fmt<QT>::UE;
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    for (int it = 0; it < n_iter; ++it) {
        const int s = it % a.n_stages;
        bool ok = !*abort_flag;
        if (ok && lane == 0) ok = mbar_wait_bounded(&full[s], (it / a.n_stages) & 1);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            if (lane == 0) { *abort_flag = 1; raise_status(a.status, DEV_ST_WAIT_FULL); }
            return;
        }
        const int tile = (int)blockIdx.x + it * (int)gridDim.x;
        const int sg = a.pair ? 0 : seg_of(a, tile);
        const int lt = a.pair ? tile : tile - a.tile0[sg];
        const int nr = a.n_rows[sg];
        const uint8_t *st = stages + (size_t)s * a.stage_bytes;
        const uint8_t *ra = st + ((reinterpret_cast<uintptr_t>(a.W[sg]) + (uintptr_t)(lt * tile_bytes)) & 15);
        const uint8_t *rb2 = st + a.region_bytes +
                             ((reinterpret_cast<uintptr_t>(a.W[1]) + (uintptr_t)(lt * tile_bytes)) & 15);
        for (int base = 0; warp + kFastWarps * base < a.rpt; base += RPW) {
            const int r = warp + kFastWarps * (base + gi);
            const int row = lt * a.rpt + r;
            const bool v = r < a.rpt && row < nr;
            float acc[MC];
#pragma unroll
            for (int m = 0; m < MC; m++) acc[m] = 0.0f;
            if (a.pair) {
                float acc2[MC];
#pragma unroll
                for (int m = 0; m < MC; m++) acc2[m] = 0.0f;
                if (v)
                    seg_row_dot2<QT, MC, A16>(ra + (size_t)r * a.row_bytes, rb2 + (size_t)r * a.row_bytes, xp, a.B,
                                              U, GS, gl, acc, acc2);
#pragma unroll
                for (int m = 0; m < MC; m++) {
                    if (m < a.B) {
                        for (int o = GS >> 1; o > 0; o >>= 1) {
                            acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
                            acc2[m] += __shfl_xor_sync(0xffffffffu, acc2[m], o);
                        }
                    }
                }
                if (gl == 0 && v) {   // h = silu(g) * u, exact (cengine_batch_instr.c:1465)
#pragma unroll
                    for (int m = 0; m < MC; m++) {
                        if (m < a.B) {
                            const float gv = acc[m];
                            a.out[0][(size_t)m * nr + row] = (gv / (1.0f + expf(-gv))) * acc2[m];
                        }
                    }
                }
            } else {
                if (v) seg_row_dot<QT, MC, A16>(ra + (size_t)r * a.row_bytes, xp, a.B, U, GS, gl, acc);
#pragma unroll
                for (int m = 0; m < MC; m++) {
                    if (m < a.B) {
                        for (int o = GS >> 1; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
                    }
                }
            }
            if (!a.pair && gl == 0 && v) {
                const float *res = a.res[sg];
                float *out = a.out[sg];
#pragma unroll
                for (int m = 0; m < MC; m++) {
                    if (m < a.B) {
                        const size_t o = (size_t)m * nr + row;
                        out[o] = res ? res[o] + acc[m] : acc[m];
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

template <int QT, int MC, bool A16>
static int launch_seg_t(const SegArgs &a, int smem, cudaStream_t s) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    static bool attr = false;
    if (!attr) {
        if (!MLQ_CUDA(cudaFuncSetAttribute(k_gemv_seg<QT, MC, A16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kMaxSmem)))
            return MLQ_ERR_CUDA;
        attr = true;
    }
    const int n_tiles = a.tile0[a.n_seg];
    const int grid = n_tiles < c->num_sms ? n_tiles : c->num_sms;
    count_launch();
    return MLQ_CUDA(launch_pdl(k_gemv_seg<QT, MC, A16>, dim3(grid), dim3(kFastThreads), smem, s, a)) ? MLQ_OK
                                                                                                      : MLQ_ERR_CUDA;
}

template <int QT>
static int launch_seg_q(SegArgs &a, cudaStream_t s) {
    const LaunchEnv *c = launch_env();
    if (!c) return MLQ_ERR_NO_DEVICE;
    if (a.K % Fmt<QT>::BE || a.K % 32) return MLQ_ERR_UNSUPPORTED;
    const long long rb = (long long)(a.K / Fmt<QT>::BE) * Fmt<QT>::BB;
    const int mats = a.pair ? 2 : 1;
    long long rpt = 24576 / (rb * mats);
    rpt = rpt < 16 ? 16 : (rpt > 64 ? 64 : rpt);
    a.rpt = (int)(rpt / 16 * 16);
    a.row_bytes = rb;
    const int x_bytes = a.B * packed_row_bytes(a.K);
    int fixed = 0, n_stages = 0;
    // long rows: fewer rows per tile (down to 4, the other decode warps idle) until two
    // stages fit (more stages through smaller tiles measured slower: the kernel is bound by
    // its decode warps, and smaller tiles leave some of them idle)
    for (;; a.rpt >>= 1) {
        a.region_bytes = align_up((int)(a.rpt * rb), 16) + 32;
        a.stage_bytes = mats * a.region_bytes;
        fixed = seg_layout(x_bytes, a.stage_bytes, 0).total;
        n_stages = fixed < kSmemBudget ? stages_for(fixed, a.stage_bytes) : 0;
        if (n_stages >= 2 || a.rpt <= 4) break;
    }
    if (n_stages < 2) return MLQ_ERR_UNSUPPORTED;
    a.n_stages = n_stages;
    const int U = a.K / Fmt<QT>::UE;
    int gs_log = 0;
    while ((1 << gs_log) < U && gs_log < 5) gs_log++;
    a.gs_log = gs_log;
    a.status = c->d_status;
    int t = 0;
    for (int i = 0; i < a.n_seg; i++) {
        a.tile0[i] = t;
        if (!a.pair || i == 0) t += (a.n_rows[i] + a.rpt - 1) / a.rpt;
    }
    a.tile0[a.n_seg] = t;   // (pair: one tile list covers both matrices)
    const int smem = fixed + n_stages * a.stage_bytes;
    bool a16 = false;
    if constexpr (QT == MLQ_Q4_K || QT == MLQ_Q5_K) {
        a16 = rb % 16 == 0;
        for (int i = 0; i < a.n_seg; i++) a16 = a16 && (reinterpret_cast<uintptr_t>(a.W[i]) & 15) == 0;
    }
#define MLQ_SEG(MC)                                                                 \
    do {                                                                            \
        if constexpr (QT == MLQ_Q4_K || QT == MLQ_Q5_K) {                           \
            if (a16) return launch_seg_t<QT, MC, true>(a, smem, s);                 \
        }                                                                           \
        return launch_seg_t<QT, MC, false>(a, smem, s);                            \
    } while (0)
    if (a.B == 1) MLQ_SEG(1);
    if (a.B == 2) MLQ_SEG(2);
    if (a.B <= 4) MLQ_SEG(4);
    MLQ_SEG(8);
#undef MLQ_SEG
}

// MLQ_ERR_UNSUPPORTED when the shape or type does not suit the kernel (the caller then
// uses the plain GEMV path)
int launch_gemv_seg(int qt, int n_seg, const uint8_t *const *W, const int *n_rows, float *const *out,
                    const float *const *res, int pair, const uint8_t *planes, int B, int K, cudaStream_t s) {
    if (n_seg < 1 || n_seg > kSegMax || B < 1 || B > 8 || !planes || (reinterpret_cast<uintptr_t>(planes) & 15) ||
        (pair && (n_seg != 2 || n_rows[0] != n_rows[1])))
        return MLQ_ERR_UNSUPPORTED;
    SegArgs a{};
    a.n_seg = n_seg;
    a.pair = pair;
    a.planes = planes;
    a.B = B;
    a.K = K;
    for (int i = 0; i < n_seg; i++) {
        if (!W[i] || !out[i] || n_rows[i] <= 0) return MLQ_ERR_UNSUPPORTED;
        a.W[i] = W[i];
        a.out[i] = out[i];
        a.res[i] = res ? res[i] : nullptr;
        a.n_rows[i] = n_rows[i];
    }
    switch (qt) {
        case MLQ_Q4_0: return launch_seg_q<MLQ_Q4_0>(a, s);
        case MLQ_Q4_1: return launch_seg_q<MLQ_Q4_1>(a, s);
        case MLQ_Q5_0: return launch_seg_q<MLQ_Q5_0>(a, s);
        case MLQ_Q8_0: {
            bool pairs = q8_0_pairs() && K % 64 == 0;
            for (int i = 0; i < n_seg; i++) pairs = pairs && (reinterpret_cast<uintptr_t>(W[i]) & 3) == 0;
            return pairs ? launch_seg_q<kQ8_0Pair>(a, s) : launch_seg_q<MLQ_Q8_0>(a, s);
        }
        case MLQ_Q4_K: return launch_seg_q<MLQ_Q4_K>(a, s);
        case MLQ_Q5_K: return launch_seg_q<MLQ_Q5_K>(a, s);
        case MLQ_Q6_K: return launch_seg_q<MLQ_Q6_K>(a, s);
        case MLQ_MXFP4: return launch_seg_q<MLQ_MXFP4>(a, s);
        case MLQ_MXFP4_REF: return launch_seg_q<MLQ_MXFP4_REF>(a, s);
        default: return MLQ_ERR_UNSUPPORTED;
    }
}

size_t packed_rows_bytes(int rows, int K) { return (size_t)rows * packed_row_bytes(K); }


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
