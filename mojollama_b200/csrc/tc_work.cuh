// Work distribution and small helpers shared by the persistent tensor-core GEMV kernels
// (gemv_mxf4_tc.cu): the chunks a CTA processes, bounded warp waits, and the
// byte layout of a K-major 128-byte-swizzled B operand image.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pipeline.cuh"

namespace mlq {

// host side (gemv_mxf4_tc.cu)
struct TcPlan { int n_tiles, nc, grid, dp_rounds, tail_units; };
bool tc_plan(int n_rows, int nc, int num_sms, TcPlan &p, uint16_t *mask, int max_tiles);
bool tc_tensor_map_rows(CUtensorMap *tmap, const void *base, long long rows, long long row_bytes, int box_bytes,
                        int box_rows);
int *tc_counters(int n, cudaStream_t s);   // zeroed per-tile arrival counters (see gemv_mxf4_tc.cu)

__device__ __forceinline__ void set_status(int *status, int code) {
    report_status(status, code);
}

// lane 0 waits (bounded), the verdict is shared by the warp
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, int lane) {
    bool ok = true;
    if (lane == 0) ok = mbar_wait_bounded(bar, parity);
    return __shfl_sync(0xffffffffu, ok, 0);
}

// byte offset of byte kb of plane row n in the swizzled B image (n_pad rows, 128-byte atoms)
__device__ __forceinline__ int bimg_off(int n, int kb, int n_pad) {
    const int ac = kb >> 7, o = kb & 127, c = o >> 4;
    return ac * (n_pad * 128) + (n >> 3) * 1024 + (n & 7) * 128 + ((c ^ (n & 7)) << 4) + (o & 15);
}

// This CTA's chunks in processing order: local index g -> unit u = tile * nc + chunk.
struct WorkMap {
    int nc, G, b, dp_rounds, tail_base, tail_units, t0, t1;
    int dp_rounds_all;   // first tail tile = rounds of whole tiles x grid
    __device__ WorkMap(int nc_, int n_tiles, int dp, int tail) : nc(nc_), G(gridDim.x), b(blockIdx.x),
        dp_rounds(dp), tail_base(dp * (int)gridDim.x * nc_), tail_units(tail) {
        dp_rounds_all = dp * G;
        const int mine = (n_tiles - b + G - 1) / G;   // round-robin tiles this CTA has at all
        if (dp_rounds > mine) dp_rounds = mine;
        t0 = (int)((long long)b * tail / G);
        t1 = (int)((long long)(b + 1) * tail / G);
    }
    __device__ int total() const { return dp_rounds * nc + t1 - t0; }
    __device__ int unit(int g) const {
        const int d = dp_rounds * nc;
        if (g < d) {
            const int r = g / nc;
            return (b + r * G) * nc + (g - r * nc);
        }
        return tail_base + t0 + (g - d);
    }
};

// Walks this CTA's chunks in order without divisions: (tile, chunk c) of local chunk g and
// whether g starts / ends an accumulation segment (one tile's chunks within this CTA).
struct UnitWalk {
    const WorkMap &w;
    int g = 0, tile, c, d;
    __device__ explicit UnitWalk(const WorkMap &wm) : w(wm), d(wm.dp_rounds * wm.nc) { at(0); }
    __device__ void at(int gg) {
        g = gg;
        const int u = w.unit(gg);
        tile = u / w.nc;
        c = u - tile * w.nc;
    }
    __device__ bool seg_start() const { return g == 0 || c == 0 || g == d; }
    __device__ bool seg_end(int total) const { return g == total - 1 || c == w.nc - 1; }
    __device__ void next() {
        if (++g == d) { at(g); return; }   // first tail chunk
        if (++c == w.nc) {
            c = 0;
            tile += g < d ? w.G : 1;
        }
    }
};

}  // namespace mlq
