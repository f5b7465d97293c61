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
// Q4_0 read as block pairs (64 elements, 36 bytes) where rows start on 4-byte boundaries:
// an internal unit variant of MLQ_Q4_0, not an ABI type id
constexpr int kQ4_0Pair = 2002;
template <> struct Fmt<kQ4_0Pair>     { static constexpr int BE = 32,  BB = 18,  UE = 64; };
// Q8_0 read as block pairs (64 elements, 68 bytes = 17 aligned words) likewise
constexpr int kQ8_0Pair = 2008;
template <> struct Fmt<kQ8_0Pair>     { static constexpr int BE = 32,  BB = 34,  UE = 64; };
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

// (scale, min) of sub-blocks 2g and 2g+1 (get_scale_min_k4 for j = 2g, 2g+1) as floats.
// All eight pairs are built bytewise at once: j < 4 from the low 6 bits of bytes j and
// j+4; j >= 4 from the nibbles of byte j+4 and the top 2 bits of bytes j-4 and j.  The
// chosen byte becomes the float 2^23 + b (PRMT into 0x4B000000) minus 2^23, exactly.
__device__ __forceinline__ void scale_min_pair_k4(const uint32_t (&s)[3], int g, float &sc0, float &m0, float &sc1,
                                                  float &m1) {
    const uint32_t sc = g < 2 ? (s[0] & 0x3F3F3F3Fu) : ((s[2] & 0x0F0F0F0Fu) | ((s[0] >> 2) & 0x30303030u));
    const uint32_t mn = g < 2 ? (s[1] & 0x3F3F3F3Fu) : (((s[2] >> 4) & 0x0F0F0F0Fu) | ((s[1] >> 2) & 0x30303030u));
    const uint32_t k0 = 0x7540u | (uint32_t)(2 * (g & 1)), k1 = k0 + 1u;
    sc0 = __uint_as_float(__byte_perm(sc, 0x4B000000u, k0)) - 8388608.0f;
    sc1 = __uint_as_float(__byte_perm(sc, 0x4B000000u, k1)) - 8388608.0f;
    m0 = __uint_as_float(__byte_perm(mn, 0x4B000000u, k0)) - 8388608.0f;
    m1 = __uint_as_float(__byte_perm(mn, 0x4B000000u, k1)) - 8388608.0f;
}

// spread 4 bits (t & 0xF) to bit 4 of each byte: element i gets +16 when bit i is set
__device__ __forceinline__ uint32_t spread4_to_bit4(uint32_t t) {
    return (((t & 0xFu) * 0x00204081u) & 0x01010101u) << 4;
}

// PTX prmt.b32, default mode: each selector nibble picks one of the 8 bytes of {b:a}
// with its low 3 bits; when its bit 3 is set the picked byte's sign bit is replicated
// over the whole result byte instead.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// Doubled-E2M1 magnitudes (GGUF MXFP4) of the four nibbles in the low 16 bits of
// `sel`, split by sign, in nibble order.  With P = {0,1,2,3,4,6,8,12} in {b:a}:
// prmt(P, nib) gives the magnitude for a positive code and 0 for a negative one
// (sign-replicate of a positive byte); prmt(P, nib ^ 8) the reverse.  The dot
// product takes the two words as separate dp4a streams and subtracts.
__device__ __forceinline__ void e2m1x2_split(uint32_t sel, uint32_t &pos, uint32_t &neg) {
    pos = prmt(0x03020100u, 0x0C080604u, sel);
    neg = prmt(0x03020100u, 0x0C080604u, sel ^ 0x8888u);
}

// ---------------------------------------------------------------------------------- x planes
// Row m of the h / l planes starts at h + m * hs (bytes); its scales and sums at
// s + m * ss (floats).  Inside a row, the 16-byte chunks of every complete 128-byte
// group are permuted (plane_swz) so that the three unit load patterns -- lane u reading
// chunks 2u + i (32-element units), 4u + i (Q4_K/Q5_K) and 8(u/2) + u%2 + 2k (Q6_K) --
// hit eight different bank groups in each quarter-warp phase of a 128-bit load.
struct XPlanes {
    const int8_t *h;      // [M] rows of K int8, row stride hs
    const int8_t *l;
    const float *s;       // [M] rows of K/32: s_b / 254, row stride ss
    const float *sum;     // [M] rows of K/32: exact fp32 block sums
    int K;
    int hs, ss;
};

// byte offset of the 16-byte chunk holding logical byte k (a multiple of 16) of a row of
// K bytes: chunk c of 128-byte group a -> c ^ f(a & 7), f(a) = a ^ 2a (mod 8); a group
// cut short by the end of the row keeps its order
__device__ __forceinline__ int plane_swz(int k, int K) {
    const int a = (k >> 7) & 7;
    return ((k | 127) < K) ? (k ^ (((a ^ (a << 1)) & 7) << 4)) : k;
}

// NW words (NW % 4 == 0, at most 64 bytes) of a plane row from logical byte k (a multiple
// of 16 with the NW words inside one 128-byte group): one permutation term for all chunks
template <int NW>
__device__ __forceinline__ void lds_plane(const int8_t *row, int k, int K, uint32_t *w) {
    const int sw = plane_swz(k, K) ^ k;
#pragma unroll
    for (int i = 0; i < NW / 4; i++) {
        const int4 v = *reinterpret_cast<const int4 *>(row + ((k + 16 * i) ^ sw));
        w[4 * i + 0] = (uint32_t)v.x;
        w[4 * i + 1] = (uint32_t)v.y;
        w[4 * i + 2] = (uint32_t)v.z;
        w[4 * i + 3] = (uint32_t)v.w;
    }
}

// 254 * dp4a(q, h) + dp4a(q, l) over NW words held in registers
template <int NW>
__device__ __forceinline__ int dot_words(const uint32_t *q, const uint32_t *h, const uint32_t *l) {
    int a = 0, b = 0;
#pragma unroll
    for (int i = 0; i < NW; i++) {
        a = __dp4a((int)q[i], (int)h[i], a);
        b = __dp4a((int)q[i], (int)l[i], b);
    }
    return a * 254 + b;
}

// ---------------------------------------------------------------------------------- units
// A unit is decoded once into W<QT> (packed int8 codes + per-group fp32 scales) and
// then dotted with the activation slice XU<QT> of every activation row.  XU comes
// from shared memory (generic path) or stays in registers for the whole kernel
// (M = 1 decode path: each lane always sees the same units of every row).
//   Fmt<QT>::UE      elements per unit
//   XU<QT>           the unit's activation words: h[], l[] (element order of the
//                    decoded words), s[] / sum[] per 32-element x block touched
template <int QT> struct W;
template <int QT> struct XU;

// ---- 32-element block formats: one block per unit
struct XU32 {
    uint32_t h[8], l[8];
    float s, sum;
};
template <> struct XU<MLQ_Q8_0> : XU32 {};
template <> struct XU<MLQ_Q4_0> : XU32 {};
template <> struct XU<MLQ_Q4_1> : XU32 {};
template <> struct XU<MLQ_Q5_0> : XU32 {};
template <> struct XU<MLQ_MXFP4> : XU32 {};
template <> struct XU<MLQ_MXFP4_REF> : XU32 {};

template <int QT>
__device__ __forceinline__ void load_xu32(const XPlanes &xp, int m, int u, XU32 &x) {
    lds_plane<8>(xp.h + (size_t)m * xp.hs, 32 * u, xp.K, x.h);
    lds_plane<8>(xp.l + (size_t)m * xp.hs, 32 * u, xp.K, x.l);
    const size_t so = (size_t)m * xp.ss + u;
    x.s = xp.s[so];
    x.sum = xp.sum[so];
}

template <> struct W<MLQ_Q8_0> {
    uint32_t q[8];
    float d;
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        const uint8_t *bp = row + 34 * u;
        d = f16_at(bp);
        load_words<8>(bp + 2, q);
    }
    __device__ __forceinline__ float dot(const XU<MLQ_Q8_0> &x) const {
        return d * x.s * (float)dot_words<8>(q, x.h, x.l);
    }
};

template <> struct W<MLQ_Q4_0> {
    uint32_t q[8];
    float d;
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        const uint8_t *bp = row + 18 * u;
        d = f16_at(bp);
        uint32_t w[4];
        load_words<4>(bp + 2, w);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = w[i] & 0x0F0F0F0Fu;               // elements 4i..4i+3
            q[4 + i] = (w[i] >> 4) & 0x0F0F0F0Fu;    // elements 16+4i..
        }
    }
    __device__ __forceinline__ float dot(const XU<MLQ_Q4_0> &x) const {
        return d * fmaf(x.s, (float)dot_words<8>(q, x.h, x.l), -8.0f * x.sum);
    }
};

template <> struct W<MLQ_Q4_1> {
    uint32_t q[8];
    float d, m;
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        const uint8_t *bp = row + 20 * u;
        d = f16_at(bp);
        m = f16_at(bp + 2);
        uint32_t w[4];
        load_words<4>(bp + 4, w);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = w[i] & 0x0F0F0F0Fu;
            q[4 + i] = (w[i] >> 4) & 0x0F0F0F0Fu;
        }
    }
    __device__ __forceinline__ float dot(const XU<MLQ_Q4_1> &x) const {
        return fmaf(d * x.s, (float)dot_words<8>(q, x.h, x.l), m * x.sum);
    }
};

template <> struct W<MLQ_Q5_0> {
    uint32_t q[8];
    float d;
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        const uint8_t *bp = row + 22 * u;
        d = f16_at(bp);
        uint32_t qh[1], w[4];
        load_words<1>(bp + 2, qh);
        load_words<4>(bp + 6, w);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = (w[i] & 0x0F0F0F0Fu) | spread4_to_bit4(qh[0] >> (4 * i));
            q[4 + i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | spread4_to_bit4(qh[0] >> (16 + 4 * i));
        }
    }
    __device__ __forceinline__ float dot(const XU<MLQ_Q5_0> &x) const {
        return d * fmaf(x.s, (float)dot_words<8>(q, x.h, x.l), -16.0f * x.sum);
    }
};

// MXFP4 decodes in nibble order: word 2k holds elements (4k, 4k+16, 4k+1, 4k+17) and
// word 2k+1 holds (4k+2, 4k+18, 4k+3, 4k+19) -- qs byte j carries element j in its
// low nibble and j+16 in its high nibble -- so its activation words are permuted to
// the same order when they are loaded (load_xu).
template <> struct W<MLQ_MXFP4> {
    uint32_t qp[8], qn[8];   // magnitudes of the positive / negative codes
    float sc;
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        const uint8_t *bp = row + 17 * u;
        uint32_t w[5];
        load_words<5>(bp, w);   // byte 0 = e, bytes 1..16 = qs
        sc = e8m0_half(w[0] & 0xFFu);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t qs = __funnelshift_r(w[i], w[i + 1], 8);   // qs bytes 4i..4i+3
            e2m1x2_split(qs, qp[2 * i], qn[2 * i]);
            e2m1x2_split(qs >> 16, qp[2 * i + 1], qn[2 * i + 1]);
        }
    }
    __device__ __forceinline__ float dot(const XU<MLQ_MXFP4> &x) const {
        int a = 0, b = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            a = __dp4a((int)qp[i], (int)x.h[i], a);
            b = __dp4a((int)qp[i], (int)x.l[i], b);
        }
        int an = 0, bn = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            an = __dp4a((int)qn[i], (int)x.h[i], an);
            bn = __dp4a((int)qn[i], (int)x.l[i], bn);
        }
        return sc * x.s * (float)((a - an) * 254 + (b - bn));
    }
};

template <> struct W<MLQ_MXFP4_REF> {
    uint32_t q[8];
    float sc;
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        const uint8_t *bp = row + 17 * u;
        uint32_t w[5];
        load_words<5>(bp, w);   // bytes 0..15 = qs, byte 16 = e
        sc = __uint_as_float((w[4] & 0xFFu) << 23);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
            // element 2j = lo nibble of byte j, 2j+1 = hi nibble; offset-binary via ^8
            q[2 * i] = __byte_perm(lo, hi, 0x5140) ^ 0x08080808u;
            q[2 * i + 1] = __byte_perm(lo, hi, 0x7362) ^ 0x08080808u;
        }
    }
    __device__ __forceinline__ float dot(const XU<MLQ_MXFP4_REF> &x) const {
        return sc * fmaf(x.s, (float)dot_words<8>(q, x.h, x.l), -8.0f * x.sum);
    }
};

// ---- Q4_K / Q5_K: unit u = sub-block pair g = u%4 of super-block u/4 (64 elements)
struct XU64 {
    uint32_t h[16], l[16];
    float s[2], sum[2];
};
template <> struct XU<MLQ_Q4_K> : XU64 {};
template <> struct XU<kQ4_0Pair> : XU64 {};
template <> struct XU<kQ8_0Pair> : XU64 {};
template <> struct XU<MLQ_Q5_K> : XU64 {};

__device__ __forceinline__ void load_xu64(const XPlanes &xp, int m, int u, XU64 &x) {
    const int xb0 = 2 * u;                       // = 8*(u/4) + 2*(u%4)
    lds_plane<16>(xp.h + (size_t)m * xp.hs, 32 * xb0, xp.K, x.h);
    lds_plane<16>(xp.l + (size_t)m * xp.hs, 32 * xb0, xp.K, x.l);
    const size_t so = (size_t)m * xp.ss + xb0;
    x.s[0] = xp.s[so];
    x.s[1] = xp.s[so + 1];
    x.sum[0] = xp.sum[so];
    x.sum[1] = xp.sum[so + 1];
}

// Q4_0 block pair u (blocks 2u, 2u+1) of a row that starts on a 4-byte boundary: the
// pair's 9 words are aligned, so they load without shifts, and lanes reading
// consecutive pairs (9 words apart) touch 32 different banks.
template <> struct W<kQ4_0Pair> {
    uint32_t q[16];          // words 0..7 block 2u, 8..15 block 2u+1 (element order)
    float d0, d1;
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        const uint32_t *p = reinterpret_cast<const uint32_t *>(row + 36 * u);
        uint32_t w[9];
#pragma unroll
        for (int i = 0; i < 9; i++) w[i] = p[i];
        d0 = __half2float(__ushort_as_half((unsigned short)(w[0] & 0xFFFFu)));
        d1 = __half2float(__ushort_as_half((unsigned short)(w[4] >> 16)));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t qa = __byte_perm(w[i], w[i + 1], 0x5432);   // block 2u bytes 2+4i..5+4i
            q[i] = qa & 0x0F0F0F0Fu;
            q[4 + i] = (qa >> 4) & 0x0F0F0F0Fu;
            q[8 + i] = w[5 + i] & 0x0F0F0F0Fu;
            q[12 + i] = (w[5 + i] >> 4) & 0x0F0F0F0Fu;
        }
    }
    __device__ __forceinline__ float dot(const XU64 &x) const {
        const int c0 = dot_words<8>(q, x.h, x.l);
        const int c1 = dot_words<8>(q + 8, x.h + 8, x.l + 8);
        return fmaf(d0, fmaf(x.s[0], (float)c0, -8.0f * x.sum[0]), d1 * fmaf(x.s[1], (float)c1, -8.0f * x.sum[1]));
    }
};

// Q8_0 block pair u (blocks 2u, 2u+1) of a row that starts on a 4-byte boundary: 17
// aligned words, an odd stride between lanes (conflict-free shared loads); the first
// block's codes are bytes 2..33 (one PRMT per word), the second's words 9..16 as they are.
template <> struct W<kQ8_0Pair> {
    uint32_t q[16];
    float d0, d1;
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        const uint32_t *p = reinterpret_cast<const uint32_t *>(row + 68 * u);
        uint32_t w[17];
#pragma unroll
        for (int i = 0; i < 17; i++) w[i] = p[i];
        d0 = __half2float(__ushort_as_half((unsigned short)(w[0] & 0xFFFFu)));
        d1 = __half2float(__ushort_as_half((unsigned short)(w[8] >> 16)));
#pragma unroll
        for (int i = 0; i < 8; i++) {
            q[i] = __byte_perm(w[i], w[i + 1], 0x5432);
            q[8 + i] = w[9 + i];
        }
    }
    __device__ __forceinline__ float dot(const XU64 &x) const {
        const int c0 = dot_words<8>(q, x.h, x.l);
        const int c1 = dot_words<8>(q + 8, x.h + 8, x.l + 8);
        return fmaf(d0 * x.s[0], (float)c0, d1 * x.s[1] * (float)c1);
    }
};

template <int QT> struct WK45 {
    uint32_t q[16];          // words 0..7 sub-block 2g (lo nibbles), 8..15 sub-block 2g+1
    float ds0, dm0, ds1, dm1;
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        constexpr int BB = (QT == MLQ_Q4_K) ? 144 : 176;
        const int sb = u >> 2, g = u & 3;
        const uint8_t *blk = row + BB * sb;
        uint32_t hdr[4];
        load_words<4>(blk, hdr);   // d, dmin, scales[12]
        const float d = __half2float(__ushort_as_half((unsigned short)(hdr[0] & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr[0] >> 16)));
        const uint32_t sw[3] = {hdr[1], hdr[2], hdr[3]};
        float sc0, m0, sc1, m1;
        scale_min_pair_k4(sw, g, sc0, m0, sc1, m1);
        uint32_t w[8];
        if (QT == MLQ_Q4_K) {
            load_words<8>(blk + 16 + 32 * g, w);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                q[i] = w[i] & 0x0F0F0F0Fu;
                q[8 + i] = (w[i] >> 4) & 0x0F0F0F0Fu;
            }
        } else {
            uint32_t qh[8];
            load_words<8>(blk + 16, qh);
            load_words<8>(blk + 48 + 32 * g, w);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                q[i] = (w[i] & 0x0F0F0F0Fu) | (((qh[i] >> (2 * g)) & 0x01010101u) << 4);
                q[8 + i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * g + 1)) & 0x01010101u) << 4);
            }
        }
        ds0 = d * sc0;
        dm0 = dmin * m0;
        ds1 = d * sc1;
        dm1 = dmin * m1;
    }
    // same, for a row that starts on a 16-byte boundary of shared memory: the block
    // header and qs/qh are then 16-byte aligned (144 and 176 are multiples of 16),
    // so they come in with conflict-free 128-bit loads
    __device__ __forceinline__ void decode_a16(const uint8_t *row, int u) {
        constexpr int BB = (QT == MLQ_Q4_K) ? 144 : 176;
        const int sb = u >> 2, g = u & 3;
        const uint8_t *blk = row + BB * sb;
        const uint4 hv = *reinterpret_cast<const uint4 *>(blk);
        const float d = __half2float(__ushort_as_half((unsigned short)(hv.x & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hv.x >> 16)));
        const uint32_t sw[3] = {hv.y, hv.z, hv.w};
        float sc0, m0, sc1, m1;
        scale_min_pair_k4(sw, g, sc0, m0, sc1, m1);
        const uint4 *qp = reinterpret_cast<const uint4 *>(blk + (QT == MLQ_Q4_K ? 16 : 48) + 32 * g);
        const uint4 v0 = qp[0], v1 = qp[1];
        const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        if (QT == MLQ_Q4_K) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                q[i] = w[i] & 0x0F0F0F0Fu;
                q[8 + i] = (w[i] >> 4) & 0x0F0F0F0Fu;
            }
        } else {
            const uint4 *hp = reinterpret_cast<const uint4 *>(blk + 16);
            const uint4 h0 = hp[0], h1 = hp[1];
            const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                q[i] = (w[i] & 0x0F0F0F0Fu) | (((qh[i] >> (2 * g)) & 0x01010101u) << 4);
                q[8 + i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * g + 1)) & 0x01010101u) << 4);
            }
        }
        ds0 = d * sc0;
        dm0 = dmin * m0;
        ds1 = d * sc1;
        dm1 = dmin * m1;
    }
    __device__ __forceinline__ float dot(const XU64 &x) const {
        const int c0 = dot_words<8>(q, x.h, x.l);
        const int c1 = dot_words<8>(q + 8, x.h + 8, x.l + 8);
        float a = ds0 * x.s[0] * (float)c0;
        a = fmaf(-dm0, x.sum[0], a);
        a = fmaf(ds1 * x.s[1], (float)c1, a);
        return fmaf(-dm1, x.sum[1], a);
    }
};
template <> struct W<MLQ_Q4_K> : WK45<MLQ_Q4_K> {};
template <> struct W<MLQ_Q5_K> : WK45<MLQ_Q5_K> {};

// ---- Q6_K: unit u = super-block u/4, half h = (u%4)/2, l in [16*(u%2), +16):
// elements 128h + l0 + i + 32k (k = quadrant 0..3, i = 0..15)
template <> struct XU<MLQ_Q6_K> {
    uint32_t h[16], l[16];       // words 4k..4k+3 = quadrant k
    float s[4];
    int off[4];                  // 32 * (254 * sum(h) + sum(l)) over each quadrant's 16 elements
};

__device__ __forceinline__ void load_xu_q6k(const XPlanes &xp, int m, int u, XU<MLQ_Q6_K> &x) {
    const int sb = u >> 2, hh = (u >> 1) & 1, l0 = 16 * (u & 1);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int xb = 8 * sb + 4 * hh + k;
        lds_plane<4>(xp.h + (size_t)m * xp.hs, 32 * xb + l0, xp.K, x.h + 4 * k);
        lds_plane<4>(xp.l + (size_t)m * xp.hs, 32 * xb + l0, xp.K, x.l + 4 * k);
        x.s[k] = xp.s[(size_t)m * xp.ss + xb];
        int hs = 0, ls = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            hs = __dp4a(0x01010101, (int)x.h[4 * k + i], hs);
            ls = __dp4a(0x01010101, (int)x.l[4 * k + i], ls);
        }
        x.off[k] = 32 * (254 * hs + ls);
    }
}

// codes stay unsigned (0..63); the -32 offset is applied through XU::off.  The unit's
// eight scale bytes (8h..8h+7) and d come from one aligned window of the 18-byte
// scales + d tail; the signed scales become floats exactly through the 2^23 trick on
// the sign-flipped bytes, and d multiplies the unit's sum once.
template <> struct W<MLQ_Q6_K> {
    uint32_t q[16];
    float d, sc[4];
    __device__ __forceinline__ void decode(const uint8_t *row, int u) {
        const int sb = u >> 2, h = (u >> 1) & 1, lr = u & 1, l0 = 16 * lr;
        const uint8_t *blk = row + 210 * sb;
        uint32_t a[4], b[4], qh[4];
        load_words<4>(blk + 64 * h + l0, a);
        load_words<4>(blk + 64 * h + 32 + l0, b);
        load_words<4>(blk + 128 + 32 * h + l0, qh);
        const uintptr_t ta = reinterpret_cast<uintptr_t>(blk + 192);
        const uint32_t *tw = reinterpret_cast<const uint32_t *>(ta & ~uintptr_t(3));
        const uint32_t sh = (uint32_t)(ta & 3) * 8u;
        const uint32_t r0 = tw[2 * h], r1 = tw[2 * h + 1], r2 = tw[2 * h + 2];
        const uint32_t dw = __funnelshift_r(tw[4], tw[5], sh);   // tail bytes 16, 17 = d
        d = __half2float(__ushort_as_half((unsigned short)(dw & 0xFFFFu)));
        const uint32_t wa = __funnelshift_r(r0, r1, sh) ^ 0x80808080u;   // scales 8h..8h+3
        const uint32_t wb = __funnelshift_r(r1, r2, sh) ^ 0x80808080u;   // scales 8h+4..8h+7
        const uint32_t k0 = 0x7540u | (uint32_t)lr, k1 = k0 + 2u;
        sc[0] = __uint_as_float(__byte_perm(wa, 0x4B000000u, k0)) - 8388736.0f;
        sc[1] = __uint_as_float(__byte_perm(wa, 0x4B000000u, k1)) - 8388736.0f;
        sc[2] = __uint_as_float(__byte_perm(wb, 0x4B000000u, k0)) - 8388736.0f;
        sc[3] = __uint_as_float(__byte_perm(wb, 0x4B000000u, k1)) - 8388736.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = (a[i] & 0x0F0F0F0Fu) | ((qh[i] & 0x03030303u) << 4);
            q[4 + i] = (b[i] & 0x0F0F0F0Fu) | (((qh[i] >> 2) & 0x03030303u) << 4);
            q[8 + i] = ((a[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 4) & 0x03030303u) << 4);
            q[12 + i] = ((b[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 6) & 0x03030303u) << 4);
        }
    }
    __device__ __forceinline__ float dot(const XU<MLQ_Q6_K> &x) const {
        float a = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            int hi = 0, lo = -x.off[k];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                hi = __dp4a((int)q[4 * k + i], (int)x.h[4 * k + i], hi);
                lo = __dp4a((int)q[4 * k + i], (int)x.l[4 * k + i], lo);
            }
            a = fmaf(sc[k], x.s[k] * (float)(hi * 254 + lo), a);
        }
        return d * a;
    }
};

// natural element order -> the MXFP4 nibble order of W<MLQ_MXFP4>
__device__ __forceinline__ void permute_mxfp4_words(uint32_t (&w)[8]) {
    uint32_t n[8];
#pragma unroll
    for (int i = 0; i < 8; i++) n[i] = w[i];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        w[2 * k] = __byte_perm(n[k], n[k + 4], 0x5140);
        w[2 * k + 1] = __byte_perm(n[k], n[k + 4], 0x7362);
    }
}

template <int QT>
__device__ __forceinline__ void load_xu(const XPlanes &xp, int m, int u, XU<QT> &x) {
    if constexpr (QT == MLQ_Q6_K) {
        load_xu_q6k(xp, m, u, x);
    } else if constexpr (QT == MLQ_Q4_K || QT == MLQ_Q5_K || QT == kQ4_0Pair || QT == kQ8_0Pair) {
        load_xu64(xp, m, u, x);
    } else {
        load_xu32<QT>(xp, m, u, x);
        if constexpr (QT == MLQ_MXFP4) {
            permute_mxfp4_words(x.h);
            permute_mxfp4_words(x.l);
        }
    }
}

// Encode activation rows into the int8 planes + scales described at the top of this
// file; one warp per 32-element block.  src(m, k) gives element k of row m; only rows
// m < n_rows are written.  Each warp takes kEncBatch blocks at a time and issues all
// their loads before the reductions, so the L2 latency is paid once per batch rather
// than once per block.
constexpr int kEncBatch = 8;

// Packed activation row (the x planes of one row in global memory, copied to shared memory
// as a whole): [K int8 h][K int8 l][K/32 f32 s][K/32 f32 sum], padded to 16 bytes.
__host__ __device__ inline int packed_row_bytes(int K) { return (2 * K + (K / 32) * 8 + 15) / 16 * 16; }

__device__ __forceinline__ XPlanes packed_planes(const uint8_t *base, int K) {
    const int rb = packed_row_bytes(K);
    const float *s = reinterpret_cast<const float *>(base + 2 * K);
    return XPlanes{reinterpret_cast<const int8_t *>(base), reinterpret_cast<const int8_t *>(base + K), s, s + K / 32,
                   K, rb, rb / 4};
}

// encode one 32-element block into row m of a packed buffer
__device__ __forceinline__ void encode_block_packed(float v, int m, int kb, int K, uint8_t *planes, int lane);

// Block kb of row m from its 32 values (one per lane).
__device__ __forceinline__ void encode_block(float v, int m, int kb, int K, int8_t *xh, int8_t *xl, float *xs,
                                             float *xsum, int hs, int ss, int lane) {
    float amax = fabsf(v), sum = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    int h = 0, l = 0;
    float scale;
    if (amax > 0.0f && amax <= 3.402823466e38f) {
        const float sc = amax / 127.0f;
        const float t = v / sc;
        const float hh = rintf(t);
        h = (int)hh;
        l = (int)rintf((t - hh) * 254.0f);
        scale = sc / 254.0f;
    } else {
        scale = (amax == 0.0f) ? 0.0f : __int_as_float(0x7fc00000);   // NaN/inf block -> NaN
    }
    const int k = 32 * kb + lane;
    const size_t o = (size_t)m * hs + plane_swz(k & ~15, K) + (k & 15);
    xh[o] = (int8_t)h;
    xl[o] = (int8_t)l;
    if (lane == 0) {
        xs[(size_t)m * ss + kb] = scale;
        xsum[(size_t)m * ss + kb] = sum;
    }
}

__device__ __forceinline__ void encode_block_packed(float v, int m, int kb, int K, uint8_t *planes, int lane) {
    const int prb = packed_row_bytes(K);
    float *s = reinterpret_cast<float *>(planes + 2 * K);
    encode_block(v, m, kb, K, reinterpret_cast<int8_t *>(planes), reinterpret_cast<int8_t *>(planes + K), s,
                 s + K / 32, prb, prb / 4, lane);
}

template <typename Src>
__device__ void encode_blocks(const Src &src, int n_rows, int K, int8_t *xh, int8_t *xl, float *xs, float *xsum,
                              int hs, int ss, int warp, int lane, int nwarps) {
    const int kb_per_row = K / 32;
    const int total = n_rows * kb_per_row;
    for (int blk0 = warp * kEncBatch; blk0 < total; blk0 += nwarps * kEncBatch) {
        float v[kEncBatch];
#pragma unroll
        for (int i = 0; i < kEncBatch; i++) {
            const int blk = blk0 + i;
            const int m = blk / kb_per_row, kb = blk - m * kb_per_row;
            v[i] = blk < total ? src(m, 32 * kb + lane) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kEncBatch; i++) {
            const int blk = blk0 + i;
            if (blk >= total) break;
            const int m = blk / kb_per_row, kb = blk - m * kb_per_row;
            encode_block(v[i], m, kb, K, xh, xl, xs, xsum, hs, ss, lane);
        }
    }
}

// rows [nb_x][K] of x; rows nb_x..M-1 read as zero
struct PlainRows {
    const float *x;
    int K, nb;
    __device__ __forceinline__ float operator()(int m, int k) const {
        return m < nb ? __ldg(x + (size_t)m * K + k) : 0.0f;
    }
};

template <int M>
__device__ void encode_x_planes(const float *__restrict__ x, int nb_x, int K, int8_t *xh, int8_t *xl, float *xs,
                                float *xsum, int warp, int lane, int nwarps) {
    encode_blocks(PlainRows{x, K, nb_x}, M, K, xh, xl, xs, xsum, K, K / 32, warp, lane, nwarps);
}

// generic path: acc[m] += dot(unit u, x row m), activations from shared memory
template <int QT, int M> struct Unit {
    static __device__ __forceinline__ void dot(const uint8_t *row, int u, const XPlanes &xp, float (&acc)[M]) {
        W<QT> w;
        w.decode(row, u);
#pragma unroll
        for (int m = 0; m < M; m++) {
            XU<QT> x;
            load_xu<QT>(xp, m, u, x);
            acc[m] += w.dot(x);
        }
    }
};

}  // namespace mlq
