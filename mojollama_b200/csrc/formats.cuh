// Device decode of GGUF blocks, fused with the dot product against activations.
//
// Activation encoding ("x planes").  Each 32-element block b of an fp32 activation
// row is split into two int8 planes with one fp32 scale:
//     s_b = amax_b / 127,  h = rint(x / s_b),  l = rint((x / s_b - h) * 254)
//     x  ~=  (s_b / 254) * (254 h + l)          (|error| <= amax_b / 64516)
// so the dot of a block of integer weight codes q with x is
//     sum q x  ~=  xs_b * (254 * dp4a(q, h) + dp4a(q, l)),   xs_b = s_b / 254,
// computed exactly in int32 by two dp4a per 4 elements.  The relative error of
// the activation encoding is below 1.6e-5, far inside the 1e-3 relative-L2 bar.
// Block minima (Q4_K/Q5_K) and code offsets (Q4_0 -8, Q5_0 -16, reference-MXFP4
// sign) use the exact fp32 block sum xsum_b instead of the planes.
//
// Weight codes are turned into packed int8 (4 per 32-bit word, element order) with
// a handful of LOP3/PRMT per word; no int->float conversion per element.
//
// Per-format "units" (the work of one lane per step):
//   32-element formats (Q4_0, Q4_1, Q5_0, Q8_0, MXFP4, MXFP4_REF): one block.
//   Q4_K, Q5_K: a pair of 32-element sub-blocks sharing 32 bytes of qs (64 elements).
//   Q6_K: 16 consecutive l of one 128-element half, all four quadrants (64 elements).
// Layout citations are in the oracle (oracle/formats.py) and the reference:
// quant_kernels_omp.c:62-70, 77-113, 762-879, 486-573; cengine_batch_instr.c:26-51.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/mojollama_b200.h"

namespace mlq {

template <int QT> struct Fmt;
template <> struct Fmt<MLQ_Q4_0>      { static constexpr int BE = 32,  BB = 18,  UE = 32; };
template <> struct Fmt<MLQ_Q4_1>      { static constexpr int BE = 32,  BB = 20,  UE = 32; };
template <> struct Fmt<MLQ_Q5_0>      { static constexpr int BE = 32,  BB = 22,  UE = 32; };
template <> struct Fmt<MLQ_Q8_0>      { static constexpr int BE = 32,  BB = 34,  UE = 32; };
template <> struct Fmt<MLQ_MXFP4>     { static constexpr int BE = 32,  BB = 17,  UE = 32; };
template <> struct Fmt<MLQ_MXFP4_REF> { static constexpr int BE = 32,  BB = 17,  UE = 32; };
template <> struct Fmt<MLQ_Q4_K>      { static constexpr int BE = 256, BB = 144, UE = 64; };
template <> struct Fmt<MLQ_Q5_K>      { static constexpr int BE = 256, BB = 176, UE = 64; };
template <> struct Fmt<MLQ_Q6_K>      { static constexpr int BE = 256, BB = 210, UE = 64; };

// ---------------------------------------------------------------------------------- loads
// NW consecutive 32-bit words starting at any byte address p (shared memory).  Reads
// one aligned word past the end, so every staging buffer carries slack.
template <int NW>
__device__ __forceinline__ void load_words(const uint8_t *p, uint32_t (&w)[NW]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *q = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3) * 8u;
    uint32_t r[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; i++) r[i] = q[i];
#pragma unroll
    for (int i = 0; i < NW; i++) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}

__device__ __forceinline__ uint32_t load_u16(const uint8_t *p) {
    uint32_t w[1];
    load_words<1>(p, w);
    return w[0] & 0xFFFFu;
}

__device__ __forceinline__ float f16_at(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)load_u16(p)));
}

// 2^(e-128) exactly, including the denormal range (e < 2): gguf-py e8m0_to_fp32_half
__device__ __forceinline__ float e8m0_half(uint32_t e) {
    return __uint_as_float(e < 2 ? (0x00200000u << e) : ((e - 1u) << 23));
}

// signed byte idx (0..15) of a 16-byte array held in 4 words
__device__ __forceinline__ int sbyte16(const uint32_t (&w)[4], int idx) {
    const uint32_t word = (idx < 4) ? w[0] : (idx < 8) ? w[1] : (idx < 12) ? w[2] : w[3];
    return (int)(int8_t)(__byte_perm(word, 0, (unsigned)(idx & 3)) & 0xFF);
}
__device__ __forceinline__ uint32_t ubyte12(const uint32_t (&w)[3], int idx) {
    const uint32_t word = (idx < 4) ? w[0] : (idx < 8) ? w[1] : w[2];
    return __byte_perm(word, 0, (unsigned)(idx & 3)) & 0xFF;
}

// K-quant 6-bit (scale, min) pair j of the 12 packed bytes (get_scale_min_k4)
__device__ __forceinline__ void scale_min_k4(const uint32_t (&s)[3], int j, uint32_t &sc, uint32_t &m) {
    if (j < 4) {
        sc = ubyte12(s, j) & 63u;
        m = ubyte12(s, j + 4) & 63u;
    } else {
        sc = (ubyte12(s, j + 4) & 0xFu) | ((ubyte12(s, j - 4) >> 6) << 4);
        m = (ubyte12(s, j + 4) >> 4) | ((ubyte12(s, j) >> 6) << 4);
    }
}

// spread 4 bits (t & 0xF) to bit 4 of each byte: element i gets +16 when bit i is set
__device__ __forceinline__ uint32_t spread4_to_bit4(uint32_t t) {
    return (((t & 0xFu) * 0x00204081u) & 0x01010101u) << 4;
}

// doubled-E2M1 code of each byte's low nibble (GGUF MXFP4), as signed int8 bytes
__device__ __forceinline__ uint32_t e2m1x2_lut(uint32_t v /* low nibbles, bytes 0x0? */) {
    const uint32_t idx = v & 0x07070707u;
    const uint32_t t = idx | (idx >> 4);                  // nibble-compact bytes 0/1 and 2/3
    const uint32_t sel = __byte_perm(t, 0, 0x0020);         // 4 selector nibbles
    const uint32_t mag = __byte_perm(0x03020100u, 0x0C080604u, sel);   // {0,1,2,3,4,6,8,12}
    const uint32_t neg = ((v & 0x08080808u) >> 3) * 0xFFu;  // 0xFF where the sign bit is set
    return __vsub4(mag ^ neg, neg);
}

// ---------------------------------------------------------------------------------- x planes
struct XPlanes {
    const int8_t *h;      // [M][K]
    const int8_t *l;      // [M][K]
    const float *s;       // [M][K/32]   s_b / 254
    const float *sum;     // [M][K/32]   exact fp32 block sums
    int K;
};

// 254 * dp4a(q, h) + dp4a(q, l) over NW words; xh/xl 16-byte aligned
template <int NW>
__device__ __forceinline__ int dot_planes(const uint32_t (&q)[NW], const int8_t *xh, const int8_t *xl) {
    static_assert(NW % 4 == 0, "NW multiple of 4");
    int a = 0, b = 0;
#pragma unroll
    for (int i = 0; i < NW / 4; i++) {
        const int4 h = reinterpret_cast<const int4 *>(xh)[i];
        const int4 l = reinterpret_cast<const int4 *>(xl)[i];
        a = __dp4a((int)q[4 * i + 0], h.x, a);
        a = __dp4a((int)q[4 * i + 1], h.y, a);
        a = __dp4a((int)q[4 * i + 2], h.z, a);
        a = __dp4a((int)q[4 * i + 3], h.w, a);
        b = __dp4a((int)q[4 * i + 0], l.x, b);
        b = __dp4a((int)q[4 * i + 1], l.y, b);
        b = __dp4a((int)q[4 * i + 2], l.z, b);
        b = __dp4a((int)q[4 * i + 3], l.w, b);
    }
    return a * 254 + b;
}

// ---------------------------------------------------------------------------------- units
// acc[m] += dot(unit u of the row at `row`, x row m)
template <int QT, int M> struct Unit;

template <int M> struct Unit<MLQ_Q8_0, M> {
    static __device__ __forceinline__ void dot(const uint8_t *row, int u, const XPlanes &xp, float (&acc)[M]) {
        const uint8_t *bp = row + 34 * u;
        const float d = f16_at(bp);
        uint32_t q[8];
        load_words<8>(bp + 2, q);
#pragma unroll
        for (int m = 0; m < M; m++) {
            const size_t xo = (size_t)m * xp.K + 32 * u;
            const int c = dot_planes<8>(q, xp.h + xo, xp.l + xo);
            acc[m] = fmaf(d * xp.s[(size_t)m * (xp.K / 32) + u], (float)c, acc[m]);
        }
    }
};

template <int M> struct Unit<MLQ_Q4_0, M> {
    static __device__ __forceinline__ void dot(const uint8_t *row, int u, const XPlanes &xp, float (&acc)[M]) {
        const uint8_t *bp = row + 18 * u;
        const float d = f16_at(bp);
        uint32_t w[4], q[8];
        load_words<4>(bp + 2, w);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = w[i] & 0x0F0F0F0Fu;
            q[4 + i] = (w[i] >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            const size_t xo = (size_t)m * xp.K + 32 * u;
            const size_t so = (size_t)m * (xp.K / 32) + u;
            const int c = dot_planes<8>(q, xp.h + xo, xp.l + xo);
            acc[m] = fmaf(d, fmaf(xp.s[so], (float)c, -8.0f * xp.sum[so]), acc[m]);
        }
    }
};

template <int M> struct Unit<MLQ_Q4_1, M> {
    static __device__ __forceinline__ void dot(const uint8_t *row, int u, const XPlanes &xp, float (&acc)[M]) {
        const uint8_t *bp = row + 20 * u;
        const float d = f16_at(bp);
        const float mn = f16_at(bp + 2);
        uint32_t w[4], q[8];
        load_words<4>(bp + 4, w);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = w[i] & 0x0F0F0F0Fu;
            q[4 + i] = (w[i] >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            const size_t xo = (size_t)m * xp.K + 32 * u;
            const size_t so = (size_t)m * (xp.K / 32) + u;
            const int c = dot_planes<8>(q, xp.h + xo, xp.l + xo);
            acc[m] = fmaf(d * xp.s[so], (float)c, fmaf(mn, xp.sum[so], acc[m]));
        }
    }
};

template <int M> struct Unit<MLQ_Q5_0, M> {
    static __device__ __forceinline__ void dot(const uint8_t *row, int u, const XPlanes &xp, float (&acc)[M]) {
        const uint8_t *bp = row + 22 * u;
        const float d = f16_at(bp);
        uint32_t qh[1], w[4], q[8];
        load_words<1>(bp + 2, qh);
        load_words<4>(bp + 6, w);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = (w[i] & 0x0F0F0F0Fu) | spread4_to_bit4(qh[0] >> (4 * i));
            q[4 + i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | spread4_to_bit4(qh[0] >> (16 + 4 * i));
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            const size_t xo = (size_t)m * xp.K + 32 * u;
            const size_t so = (size_t)m * (xp.K / 32) + u;
            const int c = dot_planes<8>(q, xp.h + xo, xp.l + xo);
            acc[m] = fmaf(d, fmaf(xp.s[so], (float)c, -16.0f * xp.sum[so]), acc[m]);
        }
    }
};

template <int M> struct Unit<MLQ_MXFP4, M> {
    static __device__ __forceinline__ void dot(const uint8_t *row, int u, const XPlanes &xp, float (&acc)[M]) {
        const uint8_t *bp = row + 17 * u;
        uint32_t w[5], q[8];
        load_words<5>(bp, w);   // byte 0 = e, bytes 1..16 = qs
        const float sc = e8m0_half(w[0] & 0xFFu);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t qs = __funnelshift_r(w[i], w[i + 1], 8);   // qs bytes 4i..4i+3
            q[i] = e2m1x2_lut(qs & 0x0F0F0F0Fu);
            q[4 + i] = e2m1x2_lut((qs >> 4) & 0x0F0F0F0Fu);
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            const size_t xo = (size_t)m * xp.K + 32 * u;
            const int c = dot_planes<8>(q, xp.h + xo, xp.l + xo);
            acc[m] = fmaf(sc * xp.s[(size_t)m * (xp.K / 32) + u], (float)c, acc[m]);
        }
    }
};

template <int M> struct Unit<MLQ_MXFP4_REF, M> {
    static __device__ __forceinline__ void dot(const uint8_t *row, int u, const XPlanes &xp, float (&acc)[M]) {
        const uint8_t *bp = row + 17 * u;
        uint32_t w[5], q[8];
        load_words<5>(bp, w);   // bytes 0..15 = qs, byte 16 = e
        const float sc = __uint_as_float((w[4] & 0xFFu) << 23);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
            // element 2j = lo nibble of byte j, 2j+1 = hi nibble; offset-binary via ^8
            q[2 * i] = __byte_perm(lo, hi, 0x5140) ^ 0x08080808u;
            q[2 * i + 1] = __byte_perm(lo, hi, 0x7362) ^ 0x08080808u;
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            const size_t xo = (size_t)m * xp.K + 32 * u;
            const size_t so = (size_t)m * (xp.K / 32) + u;
            const int c = dot_planes<8>(q, xp.h + xo, xp.l + xo);
            acc[m] = fmaf(sc, fmaf(xp.s[so], (float)c, -8.0f * xp.sum[so]), acc[m]);
        }
    }
};

template <int QT, int M> struct UnitK45 {
    // Q4_K (QT=12) / Q5_K (QT=13): unit u = sub-block pair g of super-block sb
    static __device__ __forceinline__ void dot(const uint8_t *row, int u, const XPlanes &xp, float (&acc)[M]) {
        constexpr int BB = Fmt<QT>::BB;
        const int sb = u >> 2, g = u & 3;
        const uint8_t *blk = row + BB * sb;
        uint32_t hdr[4];
        load_words<4>(blk, hdr);   // d, dmin, scales[12]
        const float d = __half2float(__ushort_as_half((unsigned short)(hdr[0] & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr[0] >> 16)));
        const uint32_t sw[3] = {hdr[1], hdr[2], hdr[3]};
        uint32_t sc0, m0, sc1, m1;
        scale_min_k4(sw, 2 * g, sc0, m0);
        scale_min_k4(sw, 2 * g + 1, sc1, m1);
        uint32_t w[8], q0[8], q1[8];
        if (QT == MLQ_Q4_K) {
            load_words<8>(blk + 16 + 32 * g, w);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                q0[i] = w[i] & 0x0F0F0F0Fu;
                q1[i] = (w[i] >> 4) & 0x0F0F0F0Fu;
            }
        } else {
            uint32_t qh[8];
            load_words<8>(blk + 16, qh);
            load_words<8>(blk + 48 + 32 * g, w);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                q0[i] = (w[i] & 0x0F0F0F0Fu) | (((qh[i] >> (2 * g)) & 0x01010101u) << 4);
                q1[i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * g + 1)) & 0x01010101u) << 4);
            }
        }
        const float ds0 = d * (float)sc0, dm0 = dmin * (float)m0;
        const float ds1 = d * (float)sc1, dm1 = dmin * (float)m1;
        const int xb0 = 8 * sb + 2 * g;
#pragma unroll
        for (int m = 0; m < M; m++) {
            const size_t xo = (size_t)m * xp.K + 32 * xb0;
            const size_t so = (size_t)m * (xp.K / 32) + xb0;
            const int c0 = dot_planes<8>(q0, xp.h + xo, xp.l + xo);
            const int c1 = dot_planes<8>(q1, xp.h + xo + 32, xp.l + xo + 32);
            float a = acc[m];
            a = fmaf(ds0 * xp.s[so], (float)c0, a);
            a = fmaf(-dm0, xp.sum[so], a);
            a = fmaf(ds1 * xp.s[so + 1], (float)c1, a);
            a = fmaf(-dm1, xp.sum[so + 1], a);
            acc[m] = a;
        }
    }
};
template <int M> struct Unit<MLQ_Q4_K, M> : UnitK45<MLQ_Q4_K, M> {};
template <int M> struct Unit<MLQ_Q5_K, M> : UnitK45<MLQ_Q5_K, M> {};

template <int M> struct Unit<MLQ_Q6_K, M> {
    // unit u: super-block sb = u/4, half h = (u%4)/2, l range [16*(u%2), +16)
    static __device__ __forceinline__ void dot(const uint8_t *row, int u, const XPlanes &xp, float (&acc)[M]) {
        const int sb = u >> 2, h = (u >> 1) & 1, lr = u & 1, l0 = 16 * lr;
        const uint8_t *blk = row + 210 * sb;
        uint32_t a[4], b[4], qh[4], scw[4];
        load_words<4>(blk + 64 * h + l0, a);
        load_words<4>(blk + 64 * h + 32 + l0, b);
        load_words<4>(blk + 128 + 32 * h + l0, qh);
        load_words<4>(blk + 192, scw);
        const float d = f16_at(blk + 208);
        uint32_t q[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[0][i] = __vsub4((a[i] & 0x0F0F0F0Fu) | ((qh[i] & 0x03030303u) << 4), 0x20202020u);
            q[1][i] = __vsub4((b[i] & 0x0F0F0F0Fu) | (((qh[i] >> 2) & 0x03030303u) << 4), 0x20202020u);
            q[2][i] = __vsub4(((a[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 4) & 0x03030303u) << 4), 0x20202020u);
            q[3][i] = __vsub4(((b[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 6) & 0x03030303u) << 4), 0x20202020u);
        }
        float ds[4];
#pragma unroll
        for (int k = 0; k < 4; k++) ds[k] = d * (float)sbyte16(scw, 8 * h + lr + 2 * k);
#pragma unroll
        for (int m = 0; m < M; m++) {
            float acc_m = acc[m];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int xb = 8 * sb + 4 * h + k;
                const size_t xo = (size_t)m * xp.K + 32 * xb + l0;
                const int c = dot_planes<4>(q[k], xp.h + xo, xp.l + xo);
                acc_m = fmaf(ds[k] * xp.s[(size_t)m * (xp.K / 32) + xb], (float)c, acc_m);
            }
            acc[m] = acc_m;
        }
    }
};

}  // namespace mlq
