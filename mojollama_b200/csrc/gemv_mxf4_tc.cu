// MXFP4 GEMV / skinny GEMM (1 <= M <= 8 activation rows) on the block-scaled tensor cores:
// tcgen05.mma kind::mxf4 with E8M0 block scales, the weights' own bytes as the A operand.
//
// Replaces, for GGUF MXFP4 weights, the reference's mxfp4_matmul_omp / mxfp4_batch_matmul
// (quant_kernels_omp.c:502-732, cengine_batch_instr.c:427-534) under quant_matmul_omp type 39.
//
// Why: a CUDA-core decode of E2M1 codes costs ~2.6 instructions per weight (sign split,
// table lookup, two int8 planes); at 0.53 bytes per weight that caps the GEMV near 40 %
// of HBM bandwidth.  Here the tensor core does the decode, the block scaling and the
// multiply-accumulate; the CUDA cores only move bytes (~0.25 instructions per weight).
//
// Operands (M = 128 weight rows per MMA, N = 8 columns per activation row, K = 64 per MMA):
//   A  weight tile, K-major, 128-byte swizzled: a GGUF MXFP4 block is {e, qs[16]} and qs
//      is exactly 32 packed E2M1 codes, so every block's 16 qs bytes are copied unchanged
//      into the operand (element j in the low nibble of byte j, j+16 in the high nibble),
//      and its E8M0 byte e becomes the block's A scale factor in tensor memory.
//   B  the activation row as 8 E2M1 "planes" with per-32-element E8M0 scales:
//      x = sum_p s_p q_p, each plane quantizing the residual the previous ones left
//      (exact fp32 residuals, the error shrinks ~4x per plane: |x - sum| <~ 4^-8 amax of
//      the block).  Plane p is column 8m + p of B; its byte j pairs x[j] (low nibble) with
//      x[j+16] (high nibble), the same element order as the weights' qs bytes.
//   D  fp32 [128 rows][8 M] in tensor memory; y[m][row] = sum_p D[row][8m + p].
// Products of E2M1 codes and power-of-two scales are exact; the MMA accumulates in fp32.
//
// Pipeline (one persistent CTA per SM, K in chunks of 512):
//   all warps but two  after the dependency wait, encode the activation planes into shared
//                memory (every CTA its own copy; hardware E2M1 rounding, ~2 us) while the
//                TMA warp already streams weights;
//   warp 12      TMA producer: 2-D tensor loads of [128 rows][272 bytes] (16 blocks per row,
//                the row pitch of the GGUF tensor) into a ring of raw stages;
//   warps 0-7    repack, two groups of 4 taking alternate chunks: thread = row; 16-byte qs
//                copies into the swizzled A chunk (one buffer per group), scale bytes gathered
//                per 128-row quarter and stored to tensor memory in the layout the MMA reads
//                (tcgen05.st, replicated per lane quarter, 4 columns per 128-K group);
//   warp 13      one thread issues the 8 MMAs of a chunk (operand descriptors precomputed: this
//                thread is on the critical path) and commits them to mbarriers;
//   warps 8-11   epilogue: tcgen05.ld of the double-buffered accumulator, plane sums, stores.
// Work split: whole 128-row tiles round-robin when there are at least as many tiles as SMs;
// otherwise the 512-K chunks are split evenly over up to one CTA per SM and the parts of a tile
// are added in chunk order by the last of its CTAs to finish (deterministic).
// Every mbarrier wait is bounded (%globaltimer, 2 s); a timeout sets the device status word
// and the CTA drains its copies and MMAs before it frees tensor memory and exits.
//
// Roofline: HBM-bound.  Algorithmic bytes per launch = N*row_bytes + M*K*4 + M*N*4.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include <map>
#include <mutex>
#include <vector>

#include "mlq_internal.h"
#include "mxf4.cuh"
#include "pipeline.cuh"
#include "tcgen05.cuh"
#include "tc_work.cuh"

namespace mlq {

namespace {

constexpr int kRows = 128;                 // MMA M: weight rows per tile
constexpr int kChunkK = 512;               // K elements per chunk (16 MXFP4 blocks per row)
constexpr int kRawRow = 272;               // bytes of one row's chunk: 16 x 17
constexpr int kRawBytes = kRows * kRawRow; // one raw stage
constexpr int kABytes = kRows * 256;       // packed E2M1 A chunk: two 128-byte-wide atom columns
constexpr int kAAtom = kRows * 128;        // one atom column (16 KB)
constexpr int kPlanes = kMxf4Planes;       // E2M1 planes per activation row
constexpr int kMaxM = 8;
constexpr int kThreads = 448;              // warps 0-7 repack, 8-11 epilogue, 12 TMA, 13 MMA
constexpr int kWarpTma = 12, kWarpMma = 13;
constexpr int kMaxStages = 6;
constexpr int kAccCol = 0;                 // 2 accumulator buffers x 64 columns
constexpr int kSfaCol = 128;               // 2 chunk buffers x 16 columns
constexpr int kSfbCol = 160;               // 4 columns per 128-K group (K <= 8192)
constexpr int kSmemMax = 232448;
constexpr int kMaxTailTiles = 160;         // tail tiles < grid <= SM count

struct Mxf4Args {
    const float *x;        // [M][K] activations (encoded into planes by every CTA)
    float *out;            // [M][n_rows]
    int n_rows, K, M, N;
    int n_tiles, n_chunks, n_stages;
    int tmem_cols;         // 256 or 512 (scale columns grow with K)
    // work split: whole tiles round-robin for floor(n_tiles / grid) rounds, then the chunks of
    // the remaining tiles split evenly over the grid (stream-K tail).  A tail tile whose chunks
    // fall to several CTAs leaves partial sums in part[tile][first chunk of the part][M][128]
    // and the last of its CTAs to finish (counter[tile], reset to 0 by that CTA) adds them in
    // chunk order
    int dp_rounds, tail_units;
    uint16_t tail_mask[kMaxTailTiles];   // per tail tile: bit c set when a CTA's part starts at chunk c
    float *part;
    int *counter;
    int off_b, off_sfb, off_sfx, off_raw, off_bar;
    int *status;
};

// barriers: raw_full[6], raw_empty[6], a_full[2], a_free[2], acc_full[2], acc_empty[2], drain
constexpr int kBarRawFull = 0, kBarRawEmpty = 6, kBarAFull = 12, kBarAFree = 14, kBarAccFull = 16,
              kBarAccEmpty = 18, kBarDrain = 20, kNumBars = 21;
constexpr int kBarBytes = kNumBars * 8 + 32;   // + TMEM base slot + flags

// ---------------------------------------------------------------- activation planes
// Activation planes, computed by every CTA into its own shared memory (B operand image and
// scale bytes).  One 4-lane group per (activation row m, 32-element block kb): lane j holds
// x[4j..4j+3] and x[16+4j..16+4j+3] and writes bytes 4j..4j+3 of the block's 16 bytes (byte i
// pairs x[i], low nibble, with x[i+16]) in each plane (mxf4_block_planes).
__device__ void encode_planes(const float *__restrict__ x, int M, int K, uint8_t *sB, uint8_t *sSfb, int tid,
                              int nthreads) {
    const int nb = K / 32, n_groups = nthreads >> 2, j = tid & 3;
    const int n_blocks = M * nb;
    const uint32_t gmask = 0xFu << (tid & 28);   // this 4-lane group within the warp
    for (int g0 = 0; g0 < n_blocks; g0 += n_groups) {
        const int gg = g0 + (tid >> 2);
        const bool live = gg < n_blocks;
        const int m = live ? gg / nb : 0, kb = live ? gg - m * nb : 0;
        float r[8];
        if (live) {
            const float4 lo = *reinterpret_cast<const float4 *>(x + (size_t)m * K + 32 * kb + 4 * j);
            const float4 hi = *reinterpret_cast<const float4 *>(x + (size_t)m * K + 32 * kb + 16 + 4 * j);
            r[0] = lo.x; r[1] = lo.y; r[2] = lo.z; r[3] = lo.w;
            r[4] = hi.x; r[5] = hi.y; r[6] = hi.z; r[7] = hi.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) r[e] = 0.0f;
        }
        uint32_t words[kPlanes], codes[kPlanes];
        mxf4_block_planes(r, gmask, words, codes);
        if (!live) continue;
#pragma unroll
        for (int p = 0; p < kPlanes; p++) {
            const uint32_t word = words[p], code = codes[p];
            const int n = kPlanes * m + p;
            *reinterpret_cast<uint32_t *>(sB + bimg_off(n, 16 * kb + 4 * j, kPlanes * M)) = word;
            if (j == 0) sSfb[(size_t)n * nb + kb] = (uint8_t)code;
        }
    }
}

// ---------------------------------------------------------------- the GEMV kernel
__global__ void __launch_bounds__(kThreads, 1) k_gemv_mxf4_tc(const __grid_constant__ CUtensorMap tmap,
                                                              Mxf4Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = sm;                                           // 2 x kABytes
    uint8_t *sB = sm + a.off_b;
    uint8_t *sSfb = sm + a.off_sfb;
    uint32_t *sfx = reinterpret_cast<uint32_t *>(sm + a.off_sfx);   // [2][4][128] scale words
    uint8_t *sRaw = sm + a.off_raw;
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm + a.off_bar);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + a.off_bar + kNumBars * 8);
    volatile int *rp_abort = reinterpret_cast<volatile int *>(sm + a.off_bar + kNumBars * 8 + 4);   // [2]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.n_stages, nc = a.n_chunks;
    const WorkMap wm(nc, a.n_tiles, a.dp_rounds, a.tail_units);
    const int total = wm.total();   // chunks of this CTA

    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&bar[kBarRawFull + s], 1);
            mbar_init(&bar[kBarRawEmpty + s], 4);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&bar[kBarAFull + b], 4);
            mbar_init(&bar[kBarAFree + b], 1);
            mbar_init(&bar[kBarAccFull + b], 1);
            mbar_init(&bar[kBarAccEmpty + b], 4);
        }
        mbar_init(&bar[kBarDrain], 1);
        rp_abort[0] = 0;
        rp_abort[1] = 0;
        rp_abort[2] = 0;   // epilogue abort
        rp_abort[3] = 0;   // epilogue: last part of a split tile
        fence_mbar_init();
    }
    if (warp == kWarpTma && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
        // weights are only read after the dependency wait: before it, just warm L2
        for (int g = 0; g < S && g < total; g++)
            tma_prefetch_2d(&tmap, (wm.unit(g) % nc) * (kRawRow / 2), (wm.unit(g) / nc) * kRows);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int tmem_cols = a.tmem_cols;
    pdl_wait();
    pdl_trigger();
    // the activation planes: every warp but the TMA and MMA ones (the TMA warp starts the
    // weight stream meanwhile); the repack warps need them in tensor memory / shared memory
    // before their first chunk, the MMA before its first instruction (ordered by a_full)
    if (warp < kWarpTma) {
        encode_planes(a.x, a.M, a.K, sB, sSfb, threadIdx.x, kWarpTma * 32);
        fence_async_smem();
        named_bar_sync(4, kWarpTma * 32);
    }

    if (warp == kWarpTma) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            const uint64_t once = policy_evict_first();
            int g = 0;
            UnitWalk uw(wm);
            for (int s = 0, ph = 0; g < total; ++g, uw.next()) {
                if (g >= S && !mbar_wait_bounded(&bar[kBarRawEmpty + s], ph ^ 1)) {
                    set_status(a.status, DEV_ST_WAIT_EMPTY);
                    break;
                }
                mbar_arrive_expect_tx(&bar[kBarRawFull + s], (uint32_t)kRawBytes);
                tma_load_2d(sRaw + (size_t)s * kRawBytes, &tmap, uw.c * (kRawRow / 2), uw.tile * kRows,
                            &bar[kBarRawFull + s], once);
                if (++s == S) { s = 0; ph ^= 1; }
            }
            // nothing may land in this CTA's shared memory after it exits
            for (int h = g - S < 0 ? 0 : g - S; h < g; ++h)
                if (!mbar_wait_bounded(&bar[kBarRawFull + h % S], (h / S) & 1)) set_status(a.status, DEV_ST_WAIT_DRAIN);
        }
    } else if (warp == kWarpMma) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            // operand descriptors and scale addresses as bases plus compile-time steps: this
            // thread's issue latency is on the pipeline's critical path
            const uint64_t ad0 = umma_desc_sw128(smem_u32(sA)), bd0 = umma_desc_sw128(smem_u32(sB));
            const uint32_t bstep = (uint32_t)(a.N * 128) >> 4;         // B atom column, descriptor units
            const uint32_t id0 = idesc_mxf4(a.N, 0, 0), id2 = idesc_mxf4(a.N, 2, 2);
            UnitWalk uw(wm);
            int sidx = -1;   // accumulation segment
            for (int g = 0; g < total; ++g, uw.next()) {
                const int ab = g & 1;
                const bool seg_start = uw.seg_start(), seg_end = uw.seg_end(total);
                if (seg_start) sidx++;
                const int accb = sidx & 1;
                if (seg_start && sidx >= 2 &&
                    !mbar_wait_bounded(&bar[kBarAccEmpty + accb], ((sidx >> 1) - 1) & 1)) {
                    set_status(a.status, DEV_ST_WAIT_EMPTY);
                    break;
                }
                if (!mbar_wait_bounded(&bar[kBarAFull + ab], (g >> 1) & 1)) {
                    set_status(a.status, DEV_ST_WAIT_FULL);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(kAccCol + 64 * accb);
                const uint64_t ad = ad0 + (uint64_t)(ab * (kABytes >> 4));
                const uint64_t bd = bd0 + (uint64_t)(2 * uw.c * bstep);   // 8 K steps = 2 atom columns
                const uint32_t sfa0 = tmem + (uint32_t)(kSfaCol + 16 * ab);
                const uint32_t sfb0 = tmem + (uint32_t)(kSfbCol + 16 * uw.c);
                // K step j: A atom column j/4 at +32 B per step; scale bytes 2(j%2) of the
                // 128-K group j/2 (the same byte id for A and B)
#pragma unroll
                for (int j = 0; j < kChunkK / 64; j++) {
                    const uint32_t hi = (j & 1) ? 0x80000000u : 0u;
                    umma_mxf4(d, ad + (uint64_t)((j >> 2) * (kAAtom >> 4) + (j & 3) * 2),
                              bd + (uint64_t)((j >> 2) * bstep + (j & 3) * 2), (j & 1) ? id2 : id0,
                              (sfa0 + 4 * (j >> 1)) | hi, (sfb0 + 4 * (j >> 1)) | hi,
                              (!seg_start || j) ? 1u : 0u);
                }
                umma_commit(&bar[kBarAFree + ab]);
                if (seg_end) umma_commit(&bar[kBarAccFull + accb]);
            }
            // every MMA issued above has finished before tensor memory is freed
            umma_commit(&bar[kBarDrain]);
            if (!mbar_wait_bounded(&bar[kBarDrain], 0)) set_status(a.status, DEV_ST_WAIT_DRAIN);
        }
        __syncwarp();
    } else if (warp < 8) {
        // ---------------------------------------------------------------- repack (thread = row)
        // two groups of 4 warps take alternate chunks (group G: chunks g = G mod 2, A buffer G)
        const int G = warp >> 2, q = warp & 3;
        const int m = threadIdx.x & 127;   // row of the tile
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
        // plane scales into tensor memory once, in the layout the MMA reads (the same as
        // for A): column 4 g + j (g = 128-K group, j = column quarter) of lane r in every
        // lane quarter holds the 4 scale bytes of B column n = r + 32 j
        bool ok = true;
        if (G == 0) {
            for (int g = 0; g < a.K / 128; g++) {
                uint32_t v[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int n = lane + 32 * j;
                    v[j] = n < a.N ? reinterpret_cast<const uint32_t *>(sSfb + (size_t)n * (a.K / 32))[g]
                                   : 0x7F7F7F7Fu;
                }
                tmem_st4(tq + (uint32_t)(kSfbCol + 4 * g), v);
            }
        }
        const int m8 = m & 7;
        const int rowoff = (m >> 3) * 1024 + m8 * 128;
        for (int g = G; g < total; g += 2) {
            const int s = g % S, ab = G;
            ok = !rp_abort[G];
            if (ok && !warp_wait(&bar[kBarRawFull + s], (g / S) & 1, lane)) ok = false;
            uint32_t R[68];
            if (ok) {
                const uint4 *src = reinterpret_cast<const uint4 *>(sRaw + (size_t)s * kRawBytes + m * kRawRow);
#pragma unroll
                for (int i = 0; i < 17; i++) {
                    const uint4 v = src[i];
                    R[4 * i] = v.x; R[4 * i + 1] = v.y; R[4 * i + 2] = v.z; R[4 * i + 3] = v.w;
                }
            }
            if (ok && g >= 2 && !warp_wait(&bar[kBarAFree + ab], ((g >> 1) - 1) & 1, lane)) ok = false;
            if (ok) {
                uint8_t *dstA = sA + ab * kABytes + rowoff;
#pragma unroll
                for (int b = 0; b < 16; b++) {
                    const int o = 17 * b + 1, w = o >> 2, sh = (o & 3) * 8;
                    uint4 q;
                    if (sh == 0) {
                        q = make_uint4(R[w], R[w + 1], R[w + 2], R[w + 3]);
                    } else {
                        q.x = __funnelshift_r(R[w], R[w + 1], sh);
                        q.y = __funnelshift_r(R[w + 1], R[w + 2], sh);
                        q.z = __funnelshift_r(R[w + 2], R[w + 3], sh);
                        q.w = __funnelshift_r(R[w + 3], R[w + 4], sh);
                    }
                    *reinterpret_cast<uint4 *>(dstA + (b >> 3) * kAAtom + (((b & 7) ^ m8) << 4)) = q;
                }
                // scale bytes e(b) at byte 17b of the row chunk, four per word (one 128-K group)
#pragma unroll
                for (int gi = 0; gi < 4; gi++) {
                    const int o0 = 17 * (4 * gi), o1 = o0 + 17, o2 = o0 + 34, o3 = o0 + 51;
                    const uint32_t t01 = __byte_perm(R[o0 >> 2], R[o1 >> 2], (uint32_t)((o0 & 3) | ((4 + (o1 & 3)) << 4)));
                    const uint32_t t23 = __byte_perm(R[o2 >> 2], R[o3 >> 2], (uint32_t)((o2 & 3) | ((4 + (o3 & 3)) << 4)));
                    sfx[(ab * 4 + gi) * kRows + m] = __byte_perm(t01, t23, 0x5410);
                }
                // the raw stage is released only now, after its rows were used above.  Released
                // right after the loads were issued, the stage's next TMA box (which fills rows 0,
                // 1, ... first) overwrote rows 0-15 before some of those loads had read them: about
                // one call in 30 had 1-3 wrong rows among a tile's first 16
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar[kBarRawEmpty + s]);
            } else {
                rp_abort[G] = 1;
            }
            named_bar_sync(1 + G, 128);
            if (rp_abort[G]) break;   // set before the barrier by a warp of this group: uniform
            // tensor-memory scale layout read by the MMA: lane r of every lane quarter, column
            // 4 * (128-K group) + (row quarter j) holds the 4 scale bytes of row r + 32 j
            uint32_t v[16];
#pragma unroll
            for (int gi = 0; gi < 4; gi++)
#pragma unroll
                for (int j = 0; j < 4; j++) v[4 * gi + j] = sfx[(ab * 4 + gi) * kRows + lane + 32 * j];
            tmem_st16(tq + (uint32_t)(kSfaCol + 16 * ab), v);
            tmem_st_wait();
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar[kBarAFull + ab]);
        }
        if (rp_abort[G]) set_status(a.status, DEV_ST_WAIT_FULL);
    } else {
        // ---------------------------------------------------------------- epilogue
        // one accumulation segment = one tile's chunks within this CTA; a whole tile is
        // stored directly, a split tile goes through the partial-sum slots
        const int q = warp & 3, rl = 32 * q + lane;
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
        volatile int *ep_flag = reinterpret_cast<volatile int *>(sm + a.off_bar + kNumBars * 8 + 12);   // [2]
        int sidx = -1, c0 = 0;
        UnitWalk uw(wm);
        for (int g = 0; g < total; ++g, uw.next()) {
            const int tile = uw.tile, c = uw.c;
            if (uw.seg_start()) { sidx++; c0 = c; }
            if (!uw.seg_end(total)) continue;
            const int accb = sidx & 1;
            const bool ok = warp_wait(&bar[kBarAccFull + accb], (sidx >> 1) & 1, lane);
            float y[kMaxM];
#pragma unroll
            for (int t = 0; t < kMaxM; t++) y[t] = 0.0f;
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int t = 0; t < kMaxM; t++) {
                    if (t < a.M) {
                        float v[8];
                        tmem_ld8(tq + (uint32_t)(kAccCol + 64 * accb + 8 * t), v);
#pragma unroll
                        for (int p = kPlanes - 1; p >= 0; p--) y[t] += v[p];
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar[kBarAccEmpty + accb]);
            } else if (lane == 0) {
                ep_flag[0] = 1;
                set_status(a.status, DEV_ST_WAIT_FULL);
            }
            named_bar_sync(3, 128);
            if (ep_flag[0]) break;   // set before the barrier by an epilogue warp: uniform
            const int row = tile * kRows + rl;
            if (c0 == 0 && c == nc - 1) {
                if (row < a.n_rows) {
#pragma unroll
                    for (int t = 0; t < kMaxM; t++)
                        if (t < a.M) a.out[(size_t)t * a.n_rows + row] = y[t];
                }
                continue;
            }
            // split tiles are tail tiles: one slot per part, indexed by the part's first chunk;
            // bit c of the tile's mask marks a part starting at chunk c
            const uint32_t pmask = a.tail_mask[tile - wm.dp_rounds_all];
            const int parts = __popc(pmask);
            const size_t slot = (size_t)a.M * kRows;
            float *mine = a.part + ((size_t)tile * nc + c0) * slot;
#pragma unroll
            for (int t = 0; t < kMaxM; t++)
                if (t < a.M) mine[(size_t)t * kRows + rl] = y[t];
            __threadfence();
            named_bar_sync(3, 128);
            if (threadIdx.x == 8 * 32) {
                const int last = atomicAdd(a.counter + tile, 1) == parts - 1 ? 1 : 0;
                if (last) a.counter[tile] = 0;   // ready for the next launch
                ep_flag[1] = last;
            }
            named_bar_sync(3, 128);
            if (ep_flag[1]) {   // the last part of this tile to land: add all parts in order
                __threadfence();
                const float *p0 = a.part + (size_t)tile * nc * slot;
                if (row < a.n_rows) {
#pragma unroll
                    for (int t = 0; t < kMaxM; t++) {
                        if (t < a.M) {
                            float acc = 0.0f;
                            for (int cc = 0; cc < nc; cc++)
                                if (pmask >> cc & 1u) acc += __ldcg(p0 + cc * slot + (size_t)t * kRows + rl);
                            a.out[(size_t)t * a.n_rows + row] = acc;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
    }
}

int tc_mxf4_enabled() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("MLQ_MXF4_TC");
        v = (e && atoi(e) == 0) ? 0 : 1;
    }
    return v;
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library does not
// link libcuda, so it still loads on a machine without a driver)
PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static bool looked = false;
    if (!looked) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
        looked = true;
    }
    return fn;
}

// Per-device arrival counters of split tiles, zeroed once when (re)allocated and left at zero
// by every launch.  Grown only outside stream capture and never under a no-allocation launch
// environment; a grown-out buffer is kept (a captured graph may still hold its address).
std::mutex g_cnt_mu;
std::map<int, std::pair<int *, int>> g_cnt;
std::vector<int *> g_cnt_retired;

int *tc_counters(int n, cudaStream_t s) {
    const LaunchEnv *env = launch_env();
    if (!env || env->no_alloc) return nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    std::lock_guard<std::mutex> lk(g_cnt_mu);
    auto &e = g_cnt[dev];
    if (e.second >= n) return e.first;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return nullptr;
    }
    int *p = nullptr;
    const int want = n < 4096 ? 4096 : n;
    if (cudaMalloc(&p, sizeof(int) * (size_t)want) != cudaSuccess || cudaMemset(p, 0, sizeof(int) * (size_t)want) != cudaSuccess) {
        cudaGetLastError();
        if (p) cudaFree(p);
        return nullptr;
    }
    if (e.first) g_cnt_retired.push_back(e.first);
    e = {p, want};
    return p;
}

// 2-D tensor map of a row-major byte matrix viewed as 16-bit elements: [rows][row_bytes / 2]
// with boxes of box_rows x box_bytes (row_bytes and box_bytes multiples of 16, base 16-aligned)
bool tc_tensor_map_rows(CUtensorMap *tmap, const void *base, long long rows, long long row_bytes, int box_bytes,
                        int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = encode_tiled_fn();
    if (!encode || row_bytes % 16 || box_bytes % 16 || ((uintptr_t)base & 15)) return false;
    const cuuint64_t gdim[2] = {(cuuint64_t)(row_bytes / 2), (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(box_bytes / 2), (cuuint32_t)box_rows};
    const cuuint32_t estride[2] = {1, 1};
    return encode(tmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Work split shared by the tensor-core GEMVs: with at least one 128-row tile per SM, whole
// tiles round-robin (tile b, b + grid, ...); splitting the last uneven round's chunks over
// all CTAs measured slower (the partial-sum hand-off at the end of a CTA costs more than the
// imbalance it removes).  With fewer tiles than SMs the chunks are split evenly over up to
// one CTA per SM, and a split tile's parts are added by the last of its CTAs to finish;
// mask[t] marks (bit c) the chunks that start a part of tile t.
bool tc_plan(int n_rows, int nc, int num_sms, TcPlan &p, uint16_t *mask, int max_tiles) {
    p.n_tiles = (n_rows + 127) / 128;
    p.nc = nc;
    const long long n_units = (long long)p.n_tiles * nc;
    if (n_units >= (1ll << 30) || nc > 16) return false;
    p.grid = p.n_tiles >= num_sms ? num_sms : (n_units < num_sms ? (int)n_units : num_sms);
    p.dp_rounds = p.n_tiles >= p.grid ? (p.n_tiles + p.grid - 1) / p.grid : 0;
    p.tail_units = p.dp_rounds ? 0 : (int)n_units;
    if (p.tail_units) {
        if (p.n_tiles > max_tiles) return false;
        auto owner = [&](long long u) { return (int)(((u + 1) * p.grid - 1) / p.tail_units); };
        for (int t = 0; t < p.n_tiles; t++) {
            uint32_t m = 1u;
            for (int c = 1; c < nc; c++)
                if (owner((long long)t * nc + c) != owner((long long)t * nc + c - 1)) m |= 1u << c;
            mask[t] = (uint16_t)m;
        }
    }
    return true;
}

// out [M][n_rows] = x [M][K] . W^T for GGUF MXFP4 W; MLQ_ERR_UNSUPPORTED outside the kernel's
// shapes (K % 512, 16-byte-aligned W, 8M * K / 2 bytes of planes in shared memory), under a
// no-allocation launch environment, or with MLQ_MXF4_TC=0
int launch_gemv_mxf4_tc(const uint8_t *W, const float *x, float *out, int n_rows, int K, int M, cudaStream_t s) {
    if (!tc_mxf4_enabled() || M < 1 || M > kMaxM || K <= 0 || K % kChunkK || n_rows <= 0 ||
        ((uintptr_t)W & 15))
        return MLQ_ERR_UNSUPPORTED;
    const LaunchEnv *env = launch_env();
    if (!env) return MLQ_ERR_NO_DEVICE;
    const int N = kPlanes * M;
    const int bimg = N * K / 2, sfb = N * (K / 32);
    if (bimg > 32768 || kSfbCol + 4 * (K / 128) > 512) return MLQ_ERR_UNSUPPORTED;
    const int tmem_cols = kSfbCol + 4 * (K / 128) <= 256 ? 256 : 512;
    const long long row_bytes = (long long)(K / 32) * 17;
    const int off_b = 2 * kABytes;
    const int off_sfb = off_b + bimg;
    const int off_sfx = (off_sfb + sfb + 15) / 16 * 16;
    const int off_bar = off_sfx + 2 * 4 * kRows * 4;
    const int off_raw = (off_bar + kBarBytes + 1023) / 1024 * 1024;
    int n_stages = (kSmemMax - 1024 - off_raw) / kRawBytes;
    if (n_stages > kMaxStages) n_stages = kMaxStages;
    if (n_stages < 2) return MLQ_ERR_UNSUPPORTED;
    const int smem = 1024 + off_raw + n_stages * kRawBytes;

    TcPlan plan;
    Mxf4Args a{};
    if (!tc_plan(n_rows, K / kChunkK, env->num_sms, plan, a.tail_mask, kMaxTailTiles)) return MLQ_ERR_UNSUPPORTED;
    const int n_tiles = plan.n_tiles, nc = plan.nc, grid = plan.grid;
    // partial sums of split tiles (written and read within one launch) and the per-tile
    // arrival counters (zero between launches: each launch's last arrival resets its tile)
    float *part = plan.tail_units ? (float *)tc_scratch(s, (size_t)n_tiles * nc * M * kRows * sizeof(float)) : nullptr;
    int *counter = plan.tail_units ? tc_counters(n_tiles, s) : nullptr;
    if (plan.tail_units && (!part || !counter)) return MLQ_ERR_UNSUPPORTED;
    // the weights as 16-bit elements [n_rows][row_bytes / 2], boxes of 128 rows x 272 bytes
    CUtensorMap tmap;
    if (!tc_tensor_map_rows(&tmap, W, n_rows, row_bytes, kRawRow, kRows)) return MLQ_ERR_UNSUPPORTED;

    static bool attr = false;
    if (!attr) {
        if (!MLQ_CUDA(cudaFuncSetAttribute(k_gemv_mxf4_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax)))
            return MLQ_ERR_CUDA;
        attr = true;
    }
    a.x = x;
    a.out = out;
    a.n_rows = n_rows; a.K = K; a.M = M; a.N = N;
    a.n_tiles = n_tiles;
    a.n_chunks = nc;
    a.dp_rounds = plan.dp_rounds;
    a.tail_units = plan.tail_units;
    a.part = part;
    a.counter = counter;
    a.n_stages = n_stages;
    a.tmem_cols = tmem_cols;
    a.off_b = off_b; a.off_sfb = off_sfb; a.off_sfx = off_sfx; a.off_raw = off_raw; a.off_bar = off_bar;
    a.status = env->d_status;

    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = getenv("MLQ_NO_PDL") ? 0 : 1;
    cfg.stream = s;
    cfg.blockDim = dim3(kThreads);
    cfg.gridDim = dim3(grid);
    cfg.dynamicSmemBytes = (size_t)smem;
    count_launch();
    return MLQ_CUDA(cudaLaunchKernelEx(&cfg, k_gemv_mxf4_tc, tmap, a)) ? MLQ_OK : MLQ_ERR_CUDA;
}

}  // namespace mlq
