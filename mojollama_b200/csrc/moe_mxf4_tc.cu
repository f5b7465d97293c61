// Grouped MXFP4 experts on the block-scaled tensor cores (tcgen05.mma kind::mxf4): the
// routed-expert products of a MoE layer, each active expert's weights streamed once for all of
// its rows.
//
// Replaces, for GGUF MXFP4 expert tensors, the per-expert MXFP4 matmuls of the reference's
// batched MoE layer (cengine_batch_instr.c:1113-1207, mxfp4_batch_matmul at :435-534), as
// launch_moe_grouped's dp4a expert GEMV does, over the same plan: k_group_plan's items
// {expert e, first sorted row m0, rows mc <= 8, 128-row tile}.
//
// Operands (as in gemv_mxf4_tc.cu; M = 128 weight rows, K = 64 per MMA):
//   A  128 rows of one expert's matrix: each GGUF MXFP4 block's 16 qs bytes copied unchanged
//      into the K-major 128-byte-swizzled operand, its E8M0 byte the A scale factor (TMEM).
//   B  the item's mc activation rows as 8 E2M1 planes each (N = 8 mc columns, n = 8 m + p),
//      with per-32-element E8M0 scales (TMEM).
//   D  fp32 [128][N] in TMEM; y[m][row] = sum_p D[row][8m + p].
// Weight tiles: one 2-D TMA box when K is a multiple of 512 and the rows are 16-byte aligned;
// otherwise (GPT-OSS: K = 2880, 1530-byte rows) each repack thread copies its own row's chunk
// as the 16-byte-aligned windows that cover it (cp.async, completion on the stage's mbarrier)
// one unit ahead -- two stages, one per repack group -- and shifts its row out of its window
// slot; a last partial chunk's missing blocks enter as zero codes with scale 1 (the planes past
// K are zero too).
// Unlike the one-matrix kernel, whose every CTA encodes the activation planes itself, the
// rows are encoded once per layer (k_mxf4_planes_rows) into global memory, already in the B
// operand's swizzled layout: planes [chunk][sorted row][2 atom columns x 1 KB], scale bytes
// [chunk][sorted row][plane][16 blocks].  A work unit (item, 512-K chunk) then brings its
// weight tile by one 2-D TMA load (no multicast) and its rows' planes and scales by two 1-D
// bulk copies into one stage; the MMA reads B from the stage itself (8-row groups 2 KB apart).
//
// Warps: 0-7 repack (two groups of 4 take alternate units: thread = weight row, qs bytes into
// the swizzled A buffer, A and B scale words into TMEM), 8-11 epilogue (TMEM -> plane sums ->
// rows of the output), 12 TMA / bulk-copy producer, 13 MMA issuer (one thread).  CTAs take
// items round-robin, all K chunks of an item in a row (one accumulation per item).  Every
// mbarrier wait is bounded (2 s of %globaltimer); a wait that gives up sets the device status
// word and the CTA drains its copies and MMAs before it frees tensor memory and exits.
//
// Roofline: HBM-bound.  Algorithmic bytes per launch = the active experts' matrices
// (rows x K / 32 x 17 each) + the planes read per item.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "mlq_internal.h"
#include "mxf4.cuh"
#include "pipeline.cuh"
#include "tc_work.cuh"
#include "tcgen05.cuh"

namespace mlq {

namespace {

constexpr int kRows = 128;                       // MMA M: weight rows per tile
constexpr int kChunkK = 512;                     // K per unit (16 MXFP4 blocks per row)
constexpr int kRawRow = 272;                     // one row's chunk: 16 x 17 bytes
constexpr int kRawBytes = kRows * kRawRow;       // 34816: the weight tile of a stage
constexpr int kBRowBytes = 2048;                 // one activation row's planes per chunk (2 atom columns)
constexpr int kMaxRows = 8;                      // activation rows per item
constexpr int kBBytes = kMaxRows * kBRowBytes;   // 16384
constexpr int kSfRowBytes = 128;                 // one row's scale bytes per chunk: 8 planes x 16
constexpr int kStage = kRawBytes + kBBytes + kMaxRows * kSfRowBytes;   // 52224 = 51 KB
constexpr int kABytes = kRows * 256;             // packed E2M1 A chunk: two 128-byte atom columns
constexpr int kAAtom = kRows * 128;
constexpr int kThreads = 448;
constexpr int kWarpTma = 12, kWarpMma = 13;
constexpr int kMaxStages = 4;
constexpr int kAccCol = 0;                       // 2 accumulators x 64 columns
constexpr int kSfaCol = 128;                     // 2 x 16 columns (per unit: 4 groups x 4 row quarters)
constexpr int kSfbCol = 160;                     // 2 x 16 columns
constexpr int kTmemCols = 256;
constexpr int kSmemMax = 232448;

constexpr int kBarRawFull = 0, kBarRawEmpty = 4, kBarAFull = 8, kBarAFree = 10, kBarAccFull = 12,
              kBarAccEmpty = 14, kBarDrain = 16, kNumBars = 17;
// after the barriers: TMEM base slot + flags, then each stage's work item, written by the producer
// before the stage's copies are armed (the MMA thread and the repack warps read it from here
// after the stage's full-barrier wait, instead of loading it from global memory per unit)
constexpr int kItemOff = 192;
constexpr int kDepOff = kItemOff + 16 * kMaxStages;   // windowed: one word per repack thread
constexpr int kBarBytes = kDepOff + 4 * 256;
static_assert(kNumBars * 8 + 16 <= kItemOff, "item records follow the barriers and flags");

// Rows that cannot be TMA tiles (a row pitch that is not a multiple of 16 bytes, K not a
// multiple of 512): each row's chunk arrives as the 16-byte-aligned windows that cover it
// (at most 18), one 288-byte slot per row (a 304-byte pitch with 16-byte reads, free of bank
// conflicts, measured the same)
constexpr int kWinRow = 288;
template <bool kWin> struct StageLayout {
    static constexpr int raw = kRows * (kWin ? kWinRow : kRawRow);        // weight part
    static constexpr int bytes = raw + kBBytes + kMaxRows * kSfRowBytes;   // 51 / 53 KB
};
static_assert(kRawBytes % 1024 == 0 && kStage % 1024 == 0 && StageLayout<true>::bytes % 1024 == 0 &&
                  StageLayout<true>::raw % 1024 == 0,
              "stage parts stay on 1 KB (swizzle atom) boundaries");

struct GroupMxf4Args {
    const int4 *items;        // {e, m0, mc, tile}
    const int *n_items;       // written on the device by the planner
    const uint8_t *planes;    // [nc][R][2048]
    const uint8_t *scales;    // [nc][R][128]
    float *out, *out2;        // [R][n_rows] (sorted rows); out2: tiles >= T1 (second matrix)
    const int *out_rows;      // with it: out[out_rows[p]][n_rows] instead
    int n_rows, nc, R, T1;
    int erows, erows2;        // tensor-map rows between consecutive experts
    int n_stages;
    int off_sfx, off_bar, off_raw;
    int dense_T;              // > 0: no item list; dense_T tiles x ceil(R / 8) row chunks (item_at)
    // windowed copies: the matrices' base addresses, expert strides, row pitch and K
    const uint8_t *W, *W2;
    long long estride, estride2;
    int row_bytes, K;
    int *status;
};

// work item it: from the planner's list, or in dense mode (one matrix pair, every row) computed,
// tile-major: the 8-row chunks of one tile are consecutive items, taken by neighbouring CTAs at
// about the same time, so the tile comes from DRAM once and from L2 for the other chunks
__device__ __forceinline__ int4 item_at(const GroupMxf4Args &a, int it) {
    if (a.dense_T) {
        const int nch = (a.R + 7) / 8, tile = it / nch, m0 = 8 * (it - tile * nch);
        return make_int4(0, m0, min(8, a.R - m0), tile);
    }
    return __ldg(a.items + it);
}

// ---------------------------------------------------------------- activation planes
// One 4-lane group per (sorted row p, 32-element block kb).  Row p is x[rows[p] / row_div]
// (rows null: row p), or with x2 the SwiGLU of the sorted gate and up rows,
// silu(clamp(x[p], +-clamp)) * x2[p] (the grouped GEMV's activation arithmetic).
// Blocks from K / 32 up to the last 512-K chunk's end are encoded as zeros (codes 0, scale 1).
__global__ void __launch_bounds__(256) k_mxf4_planes_rows(const float *__restrict__ x, const float *__restrict__ x2,
                                                          const int *__restrict__ rows, int row_div, int x_stride,
                                                          float clamp, int R, int K, uint8_t *__restrict__ planes,
                                                          uint8_t *__restrict__ scales) {
    pdl_wait();   // the rows are an earlier kernel's output
    pdl_trigger();
    const int nb = K / 32, nbp = (K + kChunkK - 1) / kChunkK * (kChunkK / 32), j = threadIdx.x & 3;
    const long long gid = (long long)blockIdx.x * 64 + (threadIdx.x >> 2);
    const bool live = gid < (long long)R * nbp;
    const int p = live ? (int)(gid / nbp) : 0, kb = live ? (int)(gid - (long long)p * nbp) : 0;
    float r[8];
#pragma unroll
    for (int e = 0; e < 8; e++) r[e] = 0.0f;
    if (live && kb < nb) {
        int src = rows ? __ldg(rows + p) : p;
        if (rows && row_div > 1) src /= row_div;
        const float *xr = x + (size_t)src * x_stride + 32 * kb;
        const float *x2r = x2 ? x2 + (size_t)p * x_stride + 32 * kb : nullptr;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int k = (e < 4 ? 0 : 16) + 4 * j + (e & 3);
            float v = __ldg(xr + k);
            if (x2r) {
                const float g = fminf(fmaxf(v, -clamp), clamp);
                v = (g / (1.0f + expf(-g))) * __ldg(x2r + k);
            }
            r[e] = v;
        }
    }
    uint32_t words[kMxf4Planes], codes[kMxf4Planes];
    mxf4_block_planes(r, 0xFu << (threadIdx.x & 28), words, codes);
    if (!live) return;
    const int c = kb >> 4, b = 16 * (kb & 15) + 4 * j, ac = b >> 7, o = b & 127;
    uint8_t *dst = planes + ((size_t)c * R + p) * kBRowBytes + ac * 1024;
#pragma unroll
    for (int pl = 0; pl < kMxf4Planes; pl++)
        *reinterpret_cast<uint32_t *>(dst + pl * 128 + ((((o >> 4) ^ pl) << 4) | (o & 15))) = words[pl];
    if (j == 0) {
        uint8_t *sd = scales + ((size_t)c * R + p) * kSfRowBytes + (kb & 15);
#pragma unroll
        for (int pl = 0; pl < kMxf4Planes; pl++) sd[pl * 16] = (uint8_t)codes[pl];
    }
}

// This CTA's units in order: local unit g -> (item index, chunk c), items b, b + G, ...
struct ItemWalk {
    int it, c, nc, G;
    __device__ ItemWalk(int nc_) : it(blockIdx.x), c(0), nc(nc_), G(gridDim.x) {}
    __device__ void next() {
        if (++c == nc) { c = 0; it += G; }
    }
};

// Windowed mode: this thread's weight row of unit (item, chunk c) as the 16-byte-aligned windows
// that cover it, into its 288-byte slot of the stage (the last window holds at least one byte of
// the row, so it stays inside the row's allocation)
__device__ __forceinline__ void copy_row_windows(const GroupMxf4Args &a, int4 item, int c, int m, uint8_t *st) {
    const bool second = item.w >= a.T1;
    const int row = (second ? item.w - a.T1 : item.w) * kRows + m;
    if (row >= a.n_rows) return;
    const uintptr_t start = reinterpret_cast<uintptr_t>(second ? a.W2 : a.W) +
                            (uintptr_t)item.x * (uintptr_t)(second ? a.estride2 : a.estride) + (uintptr_t)c * kRawRow +
                            (uintptr_t)row * (uintptr_t)a.row_bytes;
    const uintptr_t end = start + (uintptr_t)min(kRawRow, a.row_bytes - c * kRawRow);
    uint8_t *dst = st + m * kWinRow;
    for (uintptr_t p = start & ~(uintptr_t)15; p < end; p += 16, dst += 16) cp_async16(dst, reinterpret_cast<const void *>(p));
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------- the grouped kernel
template <bool kWin>
__global__ void __launch_bounds__(kThreads, 1) k_moe_mxf4_tc(const __grid_constant__ CUtensorMap tmap,
                                                             const __grid_constant__ CUtensorMap tmap2,
                                                             GroupMxf4Args a) {
    constexpr int RB = StageLayout<kWin>::raw, ST = StageLayout<kWin>::bytes;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = sm;                                                 // 2 x kABytes
    uint32_t *sfx = reinterpret_cast<uint32_t *>(sm + a.off_sfx);    // [2][4][128] A scale words
    uint8_t *sRaw = sm + a.off_raw;                                   // stages of ST bytes
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm + a.off_bar);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + a.off_bar + kNumBars * 8);
    volatile int *flag = reinterpret_cast<volatile int *>(sm + a.off_bar + kNumBars * 8 + 4);   // [3]
    int4 *s_item = reinterpret_cast<int4 *>(sm + a.off_bar + kItemOff);                       // [kMaxStages]
    uint32_t *s_dep = reinterpret_cast<uint32_t *>(sm + a.off_bar + kDepOff);                 // [256]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.n_stages, nc = a.nc;

    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&bar[kBarRawFull + s], kWin ? 129 : 1);   // windowed: the repack group's 128 rows + the producer
            mbar_init(&bar[kBarRawEmpty + s], 5);   // 4 repack warps + the MMAs that read B
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&bar[kBarAFull + b], 4);
            mbar_init(&bar[kBarAFree + b], 1);
            mbar_init(&bar[kBarAccFull + b], 1);
            mbar_init(&bar[kBarAccEmpty + b], 4);
        }
        mbar_init(&bar[kBarDrain], 1);
        flag[0] = 0;   // repack group 0 gave up
        flag[1] = 0;   // repack group 1 gave up
        flag[2] = 0;   // epilogue gave up
        fence_mbar_init();
    }
    if (!kWin && warp == kWarpTma && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap2) : "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();   // items, their count and the planes come from earlier kernels
    pdl_trigger();
    const int n_items = a.dense_T ? (a.R + 7) / 8 * a.dense_T : __ldg(a.n_items);
    const int G = gridDim.x;
    const int mine = n_items > (int)blockIdx.x ? (n_items - (int)blockIdx.x + G - 1) / G : 0;
    const int total = mine * nc;   // units of this CTA

    if (warp == kWarpTma) {
        // ---------------------------------------------------------------- producer
        // TMA mode: the weight tile (2-D TMA box) and the rows' planes and scales (1-D bulk
        // copies).  Windowed mode: the planes and scales only; the repack threads copy their
        // own rows' windows (copy_row_windows)
        if (lane == 0) {
            const uint64_t once = policy_evict_first(), keep = policy_evict_last();
            ItemWalk w(nc);
            int4 item = total ? item_at(a, w.it) : make_int4(0, 0, 0, 0);
            int4 nxt = w.it + G < n_items ? item_at(a, w.it + G) : item;
            int g = 0;
            for (int s = 0, ph = 0; g < total; ++g, w.next()) {
                if (g >= S && !mbar_wait_bounded(&bar[kBarRawEmpty + s], ph ^ 1)) {
                    set_status(a.status, DEV_ST_WAIT_EMPTY);
                    break;
                }
                const bool second = item.w >= a.T1;
                const int row0 = item.x * (second ? a.erows2 : a.erows) + (second ? item.w - a.T1 : item.w) * kRows;
                const uint32_t mc = (uint32_t)item.z;
                uint8_t *st = sRaw + (size_t)s * ST;
                const size_t pr = (size_t)w.c * a.R + item.y;
                s_item[s] = item;
                mbar_arrive_expect_tx(&bar[kBarRawFull + s], (kWin ? 0u : (uint32_t)RB) + mc * (kBRowBytes + kSfRowBytes));
                if (!kWin) tma_load_2d(st, second ? &tmap2 : &tmap, w.c * (kRawRow / 2), row0, &bar[kBarRawFull + s], once);
                bulk_g2s(st + RB, a.planes + pr * kBRowBytes, mc * kBRowBytes, &bar[kBarRawFull + s], keep);
                bulk_g2s(st + RB + kBBytes, a.scales + pr * kSfRowBytes, mc * kSfRowBytes, &bar[kBarRawFull + s], keep);
                if (w.c == nc - 1) {
                    item = nxt;
                    if (w.it + 2 * G < n_items) nxt = item_at(a, w.it + 2 * G);
                }
                if (++s == S) { s = 0; ph ^= 1; }
            }
            // nothing may land in this CTA's shared memory after it exits
            for (int h = g - S < 0 ? 0 : g - S; h < g; ++h)
                if (!mbar_wait_bounded(&bar[kBarRawFull + h % S], (h / S) & 1)) set_status(a.status, DEV_ST_WAIT_DRAIN);
        }
    } else if (warp == kWarpMma) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint64_t ad0 = umma_desc_sw128(smem_u32(sA));
            ItemWalk w(nc);
            int sidx = -1;   // item (accumulation) index of this CTA
            for (int g = 0; g < total; ++g, w.next()) {
                const int ab = g & 1, s = g % S;
                const bool seg_start = w.c == 0, seg_end = w.c == nc - 1;
                if (seg_start) sidx++;
                const int accb = sidx & 1;
                if (seg_start && sidx >= 2 && !mbar_wait_bounded(&bar[kBarAccEmpty + accb], ((sidx >> 1) - 1) & 1)) {
                    set_status(a.status, DEV_ST_WAIT_EMPTY);
                    break;
                }
                // the repack of this unit is done (A, scales); its B planes have landed
                if (!mbar_wait_bounded(&bar[kBarAFull + ab], (g >> 1) & 1) ||
                    !mbar_wait_bounded(&bar[kBarRawFull + s], (g / S) & 1)) {
                    set_status(a.status, DEV_ST_WAIT_FULL);
                    break;
                }
                tc_fence_after();
                const int n = kMxf4Planes * s_item[s].z;
                const uint32_t id0 = idesc_mxf4(n, 0, 0), id2 = idesc_mxf4(n, 2, 2);
                const uint32_t d = tmem + (uint32_t)(kAccCol + 64 * accb);
                const uint64_t ad = ad0 + (uint64_t)(ab * (kABytes >> 4));
                const uint64_t bd = umma_desc_sw128_sbo(smem_u32(sRaw + (size_t)s * ST + RB), kBRowBytes);
                const uint32_t sfa0 = tmem + (uint32_t)(kSfaCol + 16 * ab), sfb0 = tmem + (uint32_t)(kSfbCol + 16 * ab);
                // K step j: atom column j / 4 (A: +16 KB, B: +1 KB) at +32 B per step; scale
                // bytes 2 (j % 2) of the 128-K group j / 2 (the same byte id for A and B)
#pragma unroll
                for (int j = 0; j < kChunkK / 64; j++) {
                    const uint32_t hi = (j & 1) ? 0x80000000u : 0u;
                    umma_mxf4(d, ad + (uint64_t)((j >> 2) * (kAAtom >> 4) + (j & 3) * 2),
                              bd + (uint64_t)((j >> 2) * (1024 >> 4) + (j & 3) * 2), (j & 1) ? id2 : id0,
                              (sfa0 + 4 * (j >> 1)) | hi, (sfb0 + 4 * (j >> 1)) | hi, (!seg_start || j) ? 1u : 0u);
                }
                umma_commit(&bar[kBarAFree + ab]);
                umma_commit(&bar[kBarRawEmpty + s]);   // the stage's B planes are read
                if (seg_end) umma_commit(&bar[kBarAccFull + accb]);
            }
            // every MMA issued above has finished before tensor memory is freed
            umma_commit(&bar[kBarDrain]);
            if (!mbar_wait_bounded(&bar[kBarDrain], 0)) set_status(a.status, DEV_ST_WAIT_DRAIN);
        }
        __syncwarp();
    } else if (warp < 8) {
        // ---------------------------------------------------------------- repack (thread = row)
        // group G takes units g = G mod 2 into A buffer G and scale columns G
        const int G2 = warp >> 2, q = warp & 3;
        const int m = threadIdx.x & 127;
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
        const int m8 = m & 7;
        const int rowoff = (m >> 3) * 1024 + m8 * 128;
        ItemWalk w(nc);
        if (G2) w.next();
        // windowed mode (two stages, stage G2 always this group's): the group copies its own rows,
        // one unit ahead -- the first unit here, each next one once the current unit's rows have
        // been read
        if (kWin && G2 < total) {
            copy_row_windows(a, item_at(a, w.it), w.c, m, sRaw + (size_t)G2 * ST);
            cp_async_arrive_noinc(&bar[kBarRawFull + G2]);
        }
        for (int g = G2; g < total; g += 2, w.next(), w.next()) {
            const int s = g % S, ab = G2;
            ItemWalk wn = w;   // this group's next unit, g + 2
            wn.next();
            wn.next();
            const int4 nitem = kWin && g + 2 < total ? item_at(a, wn.it) : make_int4(0, 0, 0, 0);
            bool ok = !flag[G2];
            if (ok && !warp_wait(&bar[kBarRawFull + s], (g / S) & 1, lane)) ok = false;
            uint32_t R[68];
            const uint8_t *st = sRaw + (size_t)s * ST;
            // valid 32-element blocks of this chunk: the last chunk of a K that is not a multiple
            // of 512 has fewer, and its other blocks enter as zero codes with scale 1
            const int nvalid = min(16, a.K / 32 - 16 * w.c);
            if (ok) {
                if constexpr (kWin) {
                    // this row's chunk starts (start mod 16) bytes into its window slot
                    const int4 item = s_item[s];
                    const bool second = item.w >= a.T1;
                    const int row = (second ? item.w - a.T1 : item.w) * kRows + m;
                    const uintptr_t start = reinterpret_cast<uintptr_t>(second ? a.W2 : a.W) +
                                            (uintptr_t)item.x * (uintptr_t)(second ? a.estride2 : a.estride) +
                                            (uintptr_t)w.c * kRawRow + (uintptr_t)row * (uintptr_t)a.row_bytes;
                    const int off = (int)(start & 15), sh = (off & 3) * 8;
                    const uint32_t *wp = reinterpret_cast<const uint32_t *>(st + m * kWinRow + (off & ~3));
                    uint32_t prev = wp[0];
#pragma unroll
                    for (int i = 0; i < 68; i++) {
                        const uint32_t nxt = wp[i + 1];
                        R[i] = __funnelshift_r(prev, nxt, sh);
                        prev = nxt;
                    }
                    if (g + 2 < total) {
                        // this thread's row of the group's next unit, into the slot just read.  The
                        // copies must not land before this row's loads have read the slot: the XOR
                        // of the row's words (it needs every load's data) is stored first and the
                        // warp synchronises, so the copies issue only after all the loads returned
                        uint32_t dep = 0;
#pragma unroll
                        for (int i = 0; i < 68; i++) dep ^= R[i];
                        s_dep[threadIdx.x] = dep;
                        __syncwarp();
                        copy_row_windows(a, nitem, wn.c, m, const_cast<uint8_t *>(st));
                        cp_async_arrive_noinc(&bar[kBarRawFull + s]);
                    }
                } else {
                    const uint4 *src = reinterpret_cast<const uint4 *>(st + m * kRawRow);
#pragma unroll
                    for (int i = 0; i < 17; i++) {
                        const uint4 v = src[i];
                        R[4 * i] = v.x; R[4 * i + 1] = v.y; R[4 * i + 2] = v.z; R[4 * i + 3] = v.w;
                    }
                }
            }
            uint32_t *sx = sfx + ab * 4 * kRows;
            if (ok && g >= 2 && !warp_wait(&bar[kBarAFree + ab], ((g >> 1) - 1) & 1, lane)) ok = false;
            if (ok) {
                uint8_t *dstA = sA + ab * kABytes + rowoff;
#pragma unroll
                for (int b = 0; b < 16; b++) {
                    const int o = 17 * b + 1, wd = o >> 2, sh = (o & 3) * 8;
                    uint4 v;
                    if (sh == 0) {
                        v = make_uint4(R[wd], R[wd + 1], R[wd + 2], R[wd + 3]);
                    } else {
                        v.x = __funnelshift_r(R[wd], R[wd + 1], sh);
                        v.y = __funnelshift_r(R[wd + 1], R[wd + 2], sh);
                        v.z = __funnelshift_r(R[wd + 2], R[wd + 3], sh);
                        v.w = __funnelshift_r(R[wd + 3], R[wd + 4], sh);
                    }
                    if (b >= nvalid) v = make_uint4(0u, 0u, 0u, 0u);
                    *reinterpret_cast<uint4 *>(dstA + (b >> 3) * kAAtom + (((b & 7) ^ m8) << 4)) = v;
                }
                // A scale bytes e(b) at byte 17 b of the row chunk, four per word (one 128-K group)
#pragma unroll
                for (int gi = 0; gi < 4; gi++) {
                    const int o0 = 17 * (4 * gi), o1 = o0 + 17, o2 = o0 + 34, o3 = o0 + 51;
                    const uint32_t t01 = __byte_perm(R[o0 >> 2], R[o1 >> 2], (uint32_t)((o0 & 3) | ((4 + (o1 & 3)) << 4)));
                    const uint32_t t23 = __byte_perm(R[o2 >> 2], R[o3 >> 2], (uint32_t)((o2 & 3) | ((4 + (o3 & 3)) << 4)));
                    uint32_t wd = __byte_perm(t01, t23, 0x5410);
                    if (4 * gi + 4 > nvalid) {
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            if (4 * gi + j >= nvalid) wd = (wd & ~(0xFFu << (8 * j))) | (0x7Fu << (8 * j));
                    }
                    sx[gi * kRows + m] = wd;
                }
            } else {
                flag[G2] = 1;
            }
            named_bar_sync(1 + G2, 128);
            if (flag[G2]) break;   // set before the barrier by a warp of this group: uniform
            // A scale layout read by the MMA: lane r of every lane quarter, column 4 gi + j holds
            // the 4 scale bytes of weight row r + 32 j
            uint32_t v[16];
#pragma unroll
            for (int gi = 0; gi < 4; gi++)
#pragma unroll
                for (int j = 0; j < 4; j++) v[4 * gi + j] = sx[gi * kRows + lane + 32 * j];
            tmem_st16(tq + (uint32_t)(kSfaCol + 16 * ab), v);
            // B scale words, in the same layout: column 4 gi + j of lane r = the 4 scale bytes
            // of 128-K group gi of B column n = r + 32 j; columns past N carry scale 1 (their B
            // rows are never read)
            const int n_cols = kMxf4Planes * s_item[s].z;
            const uint8_t *sf = st + RB + kBBytes;
            uint32_t vb[16];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int n = lane + 32 * j;
#pragma unroll
                for (int gi = 0; gi < 4; gi++)
                    vb[4 * gi + j] = n < n_cols ? *reinterpret_cast<const uint32_t *>(sf + n * 16 + 4 * gi) : 0x7F7F7F7Fu;
            }
            tmem_st16(tq + (uint32_t)(kSfbCol + 16 * ab), vb);
            tmem_st_wait();
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            // the stage is released (its B planes stay until the MMAs that read them commit: the
            // fifth arrival) and the A buffer handed to the MMA
            if (lane == 0) {
                mbar_arrive(&bar[kBarRawEmpty + s]);
                mbar_arrive(&bar[kBarAFull + ab]);
            }
        }
        if (flag[G2]) set_status(a.status, DEV_ST_WAIT_FULL);
    } else {
        // ---------------------------------------------------------------- epilogue
        const int q = warp & 3, rl = 32 * q + lane;
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
        ItemWalk w(nc);
        int sidx = -1;
        for (int g = 0; g < total; ++g, w.next()) {
            if (w.c == 0) sidx++;
            if (w.c != nc - 1) continue;
            const int accb = sidx & 1;
            const int4 item = item_at(a, w.it);
            const bool ok = warp_wait(&bar[kBarAccFull + accb], (sidx >> 1) & 1, lane);
            float y[kMaxRows];
#pragma unroll
            for (int t = 0; t < kMaxRows; t++) y[t] = 0.0f;
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int t = 0; t < kMaxRows; t++) {
                    if (t < item.z) {
                        float v[8];
                        tmem_ld8(tq + (uint32_t)(kAccCol + 64 * accb + 8 * t), v);
#pragma unroll
                        for (int p = kMxf4Planes - 1; p >= 0; p--) y[t] += v[p];
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar[kBarAccEmpty + accb]);
            } else if (lane == 0) {
                flag[2] = 1;
                set_status(a.status, DEV_ST_WAIT_FULL);
            }
            named_bar_sync(3, 128);
            if (flag[2]) break;   // set before the barrier by an epilogue warp: uniform
            const bool second = item.w >= a.T1;
            const int row = (second ? item.w - a.T1 : item.w) * kRows + rl;
            if (row < a.n_rows) {
                float *dst = second ? a.out2 : a.out;
#pragma unroll
                for (int t = 0; t < kMaxRows; t++) {
                    if (t < item.z) {
                        const int p = item.y + t;
                        const int orow = a.out_rows ? __ldg(a.out_rows + p) : p;
                        dst[(size_t)orow * a.n_rows + row] = y[t];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// MLQ_MOE_MXF4_TC: 0 off, 1 (default) when the items fill the GPU at least twice, 2 always
int mxf4_group_mode() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("MLQ_MOE_MXF4_TC");
        v = e ? atoi(e) : 1;
        if (v < 0) v = 0;
    }
    return v;
}

}  // namespace

// at least two items per SM, estimated as min(R, E) active (expert, 8-row chunk) pairs x tiles
// per chunk: with fewer, the SMs that get a second item set the time (config 4 at one token,
// 4 experts x 46 tiles = 184 items: 4.69 ms per step against 4.15 on the grouped GEMV)
bool mxf4_grouped_wanted(int R, int E, int item_tiles) {
    const int mode = mxf4_group_mode();
    if (mode == 0) return false;
    if (mode >= 2) return true;
    const LaunchEnv *env = launch_env();
    return env && (long long)(R < E ? R : E) * item_tiles >= 2ll * env->num_sms;
}

size_t mxf4_planes_bytes(int R, int K) {
    const size_t nc = (size_t)(K + kChunkK - 1) / kChunkK;
    return nc * (size_t)R * (kBRowBytes + kSfRowBytes);
}

// Whether the expert matrices can be TMA tiles: K a multiple of 512 (rows of whole 272-byte
// chunks, a row pitch that is a multiple of 16 bytes), a 16-byte-aligned base, experts a whole
// number of rows apart, and every row index inside int range.  Otherwise the kernel copies each
// row's chunks as 16-byte windows (any K % 32 == 0, any alignment).
static bool mxf4_tma_ok(const uint8_t *W, long long estride, int E, int n_rows, int K) {
    if (K % kChunkK || ((uintptr_t)W & 15)) return false;
    const long long row_bytes = (long long)(K / 32) * 17;
    if (estride % row_bytes) return false;
    return (long long)(E - 1) * (estride / row_bytes) + n_rows < (1ll << 31);
}

bool mxf4_grouped_supported(const uint8_t *W, long long estride, int E, int n_rows, int K) {
    if (!mxf4_group_mode() || !W || K <= 0 || K % 32 || n_rows <= 0 || E <= 0) return false;
    return estride >= (long long)(K / 32) * 17 * n_rows;
}

int launch_mxf4_planes_rows(const float *x, const float *x2, const int *rows, int row_div, int x_stride, float clamp,
                            int R, int K, uint8_t *planes, cudaStream_t s) {
    if (R <= 0) return MLQ_OK;
    if (K <= 0 || K % 32) return MLQ_ERR_UNSUPPORTED;
    const int nc = (K + kChunkK - 1) / kChunkK;
    const long long groups = (long long)R * nc * (kChunkK / 32);
    uint8_t *scales = planes + (size_t)nc * R * kBRowBytes;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = getenv("MLQ_NO_PDL") ? 0 : 1;
    cfg.stream = s;
    cfg.blockDim = dim3(256);
    cfg.gridDim = dim3((unsigned)((groups + 63) / 64));
    count_launch();
    return MLQ_CUDA(cudaLaunchKernelEx(&cfg, k_mxf4_planes_rows, x, x2, rows, row_div, x_stride, clamp, R, K, planes,
                                       scales))
               ? MLQ_OK
               : MLQ_ERR_CUDA;
}

static int launch_mxf4_tc(const uint8_t *W, long long estride, const uint8_t *W2, long long estride2, int E,
                          int n_rows, int K, const void *items, const int *n_items_dev, int n_items_bound, int dense_T,
                          const uint8_t *planes, int R, float *out, float *out2, const int *out_rows, cudaStream_t s) {
    if (n_items_bound <= 0 || R <= 0) return MLQ_OK;
    if (!mxf4_grouped_supported(W, estride, E, n_rows, K) || (W2 && !mxf4_grouped_supported(W2, estride2, E, n_rows, K)))
        return MLQ_ERR_UNSUPPORTED;
    const LaunchEnv *env = launch_env();
    if (!env) return MLQ_ERR_NO_DEVICE;
    const int nc = (K + kChunkK - 1) / kChunkK;
    const long long row_bytes = (long long)(K / 32) * 17;
    const bool tma = mxf4_tma_ok(W, estride, E, n_rows, K) && (!W2 || mxf4_tma_ok(W2, estride2, E, n_rows, K));
    const long long erows = tma ? estride / row_bytes : 0, erows2 = tma && W2 ? estride2 / row_bytes : 0;
    CUtensorMap tmap{}, tmap2{};
    if (tma) {
        if (!tc_tensor_map_rows(&tmap, W, (E - 1) * erows + n_rows, row_bytes, kRawRow, kRows) ||
            !tc_tensor_map_rows(&tmap2, W2 ? W2 : W, W2 ? (E - 1) * erows2 + n_rows : (E - 1) * erows + n_rows,
                                row_bytes, kRawRow, kRows))
            return MLQ_ERR_UNSUPPORTED;
    }
    // shared memory: 2 A buffers, the A scale words, barriers, then the stages
    const int stage = tma ? StageLayout<false>::bytes : StageLayout<true>::bytes;
    const int off_sfx = 2 * kABytes;
    const int off_bar = off_sfx + 2 * 4 * kRows * 4;
    const int off_raw = (off_bar + kBarBytes + 1023) / 1024 * 1024;
    int n_stages = (kSmemMax - 1024 - off_raw) / stage;
    if (n_stages > kMaxStages) n_stages = kMaxStages;
    if (!tma) n_stages = 2;   // windowed: one stage per repack group (each group refills its own)
    if (n_stages < 2) return MLQ_ERR_UNSUPPORTED;
    const int smem = 1024 + off_raw + n_stages * stage;
    static bool attr[2] = {false, false};
    if (!attr[tma]) {
        if (!MLQ_CUDA(cudaFuncSetAttribute(tma ? k_moe_mxf4_tc<false> : k_moe_mxf4_tc<true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax)))
            return MLQ_ERR_CUDA;
        attr[tma] = true;
    }
    GroupMxf4Args a{};
    a.W = W;
    a.W2 = W2 ? W2 : W;
    a.estride = estride;
    a.estride2 = W2 ? estride2 : estride;
    a.row_bytes = (int)row_bytes;
    a.K = K;
    a.items = reinterpret_cast<const int4 *>(items);
    a.n_items = n_items_dev;
    a.planes = planes;
    a.scales = planes + (size_t)nc * R * kBRowBytes;
    a.out = out;
    a.out2 = out2;
    a.out_rows = out_rows;
    a.n_rows = n_rows;
    a.nc = nc;
    a.R = R;
    a.T1 = (n_rows + kRows - 1) / kRows;
    a.erows = (int)erows;
    a.erows2 = (int)erows2;
    a.n_stages = n_stages;
    a.off_sfx = off_sfx;
    a.off_bar = off_bar;
    a.off_raw = off_raw;
    a.dense_T = dense_T;
    a.status = env->d_status;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = getenv("MLQ_NO_PDL") ? 0 : 1;
    cfg.stream = s;
    cfg.blockDim = dim3(kThreads);
    cfg.gridDim = dim3((unsigned)(n_items_bound < env->num_sms ? n_items_bound : env->num_sms));
    cfg.dynamicSmemBytes = (size_t)smem;
    count_launch();
    return MLQ_CUDA(cudaLaunchKernelEx(&cfg, tma ? k_moe_mxf4_tc<false> : k_moe_mxf4_tc<true>, tmap, tmap2, a))
               ? MLQ_OK
               : MLQ_ERR_CUDA;
}

int launch_moe_mxf4_tc(const uint8_t *W, long long estride, const uint8_t *W2, long long estride2, int E, int n_rows,
                       int K, const void *items, const int *n_items_dev, int n_items_bound, const uint8_t *planes,
                       int R, float *out, float *out2, const int *out_rows, cudaStream_t s) {
    return launch_mxf4_tc(W, estride, W2, estride2, E, n_rows, K, items, n_items_dev, n_items_bound, 0, planes, R, out,
                          out2, out_rows, s);
}

bool mxf4_dense_supported(const uint8_t *W, int n_rows, int K) {
    return mxf4_grouped_supported(W, (long long)(K / 32) * 17 * n_rows, 1, n_rows, K);
}

int launch_mxf4_dense_tc(const uint8_t *W, const uint8_t *W2, int n_rows, int K, const uint8_t *planes, int R,
                         float *out, float *out2, cudaStream_t s) {
    const long long st = (long long)(K / 32) * 17 * n_rows;
    const int T = (W2 ? 2 : 1) * ((n_rows + kRows - 1) / kRows);
    return launch_mxf4_tc(W, st, W2, st, 1, n_rows, K, nullptr, nullptr, (R + 7) / 8 * T, T, planes, R, out, out2,
                          nullptr, s);
}

}  // namespace mlq
