// Tensor-core quantized GEMM for many tokens: out[t][r] = sum_k W[r][k] * x[t][k]
// (the math of the reference's *_batch_matmul, cengine_batch_instr.c:68-534, at B >= 16).
//
// tcgen05 (5th-generation tensor cores) with the weights on the MMA's M side:
//   * a CTA owns 128 weight rows x NT tokens; the fp32 accumulator tile [128][NT] lives in
//     TMEM (NT columns), allocated once per CTA;
//   * K advances in chunks of 256 elements.  The raw GGUF bytes of the 128 rows' chunk are
//     copied into shared memory with cp.async (16-byte pieces, two stages), every thread
//     then decodes 8-element groups to fp16 and stores them in the canonical K-major
//     128-byte-swizzled operand layout (8-row x 128-byte atoms, 16-byte chunk c of row r at
//     c ^ (r & 7));
//   * the activations were converted once per call to fp16 with a power-of-two scale per
//     token (|x/s| <= 1, so fp16 keeps 11 significant bits and never overflows); their
//     chunk is copied straight into the same swizzled layout (two stages);
//   * one thread issues 16 tcgen05.mma.kind::f16 (K = 16 each) per chunk and commits them
//     to an mbarrier; the next chunk's decode waits on that barrier before it overwrites
//     the A operand;
//   * the epilogue reads the accumulators with tcgen05.ld (warp w reads TMEM lanes
//     32*(w%4).. = weight rows), multiplies by the token scale and writes fp32.
// Error model: weights rounded once to fp16 (relative 2^-11), activations once (2^-11),
// products and sums exact / fp32 -- relative L2 of the outputs ~3e-4.
// Formats: Q8_0, Q4_0, Q4_1, Q5_0, Q4_K, Q5_K with K % 256 == 0 and 16-byte aligned rows
// and chunks; Q6_K (210-byte super-blocks, only 2-byte aligned) with K % 256 == 0, copied
// in 4-byte pieces from the 4-byte boundary at or below each super-block; MXFP4 and odd K
// stay on their GEMV kernels.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <vector>

#include "formats.cuh"
#include "mlq_internal.h"
#include "pipeline.cuh"
#include "tcgen05.cuh"

namespace mlq {

constexpr int kTcRows = 128;      // MMA M
constexpr int kTcThreads = 512;   // 16 warps decode; warps 0-7 also read the accumulators out
constexpr int kTcKC = 256;        // K elements per chunk
constexpr int kTcAtomBytes = 16384;   // one 64-wide K atom of the A tile: 128 rows x 128 B

// ---------------------------------------------------------------- activations
// x [M][K] fp32 -> xh [Mp][K] fp16 of x / s_t, s_t = 2^ceil(log2(max|x_t|)) (1 for a zero
// row); rows M..Mp-1 are zero with scale 0.
__global__ void k_x_to_f16(const float *__restrict__ x, __half *__restrict__ xh, float *__restrict__ scale, int M,
                           int K, int Kp) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    __shared__ float sh[32];
    const int t = blockIdx.x;
    __half *dst = xh + (size_t)t * Kp;
    for (int i = K + threadIdx.x; i < Kp; i += blockDim.x) dst[i] = __float2half_rn(0.0f);   // K padding
    if (t >= M) {
        for (int i = threadIdx.x; i < K; i += blockDim.x) dst[i] = __float2half_rn(0.0f);
        if (threadIdx.x == 0) scale[t] = 0.0f;
        return;
    }
    const float *src = x + (size_t)t * K;
    float amax = 0.0f;
#pragma unroll 4
    for (int i = threadIdx.x; i < K; i += blockDim.x) amax = fmaxf(amax, fabsf(src[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) sh[0] = v;
    }
    __syncthreads();
    amax = sh[0];
    float s;
    if (!(amax <= 3.402823466e38f)) s = __int_as_float(0x7fc00000);   // inf / NaN row -> NaN outputs
    else if (amax == 0.0f) s = 1.0f;
    else {
        int e;
        frexpf(amax, &e);            // amax = f * 2^e, f in [0.5, 1)
        s = ldexpf(1.0f, e);         // amax / s in [0.5, 1)
    }
    const float inv = 1.0f / s;      // exact: s is a power of two
#pragma unroll 4
    for (int i = threadIdx.x; i < K; i += blockDim.x) dst[i] = __float2half_rn(src[i] * inv);
    if (threadIdx.x == 0) scale[t] = s;
}

// Sorted row p of grouped experts' input as fp16 / s_p, s_p a power of two as in k_x_to_f16:
// x[rows[p] / row_div] (row pitch x_stride; rows null: row p), or with x2 the SwiGLU of
// sorted gate and up rows, silu(clamp(x[p], +-clamp)) * x2[p] (the grouped GEMV's GroupRows
// arithmetic).  Columns K..Kp-1 are zero.
__global__ void k_rows_to_f16(const float *__restrict__ x, const float *__restrict__ x2, const int *__restrict__ rows,
                              int row_div, int x_stride, float clamp, int K, int Kp, __half *__restrict__ xh,
                              __half *__restrict__ xl, float *__restrict__ scale) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    __shared__ float sh[32];
    const int p = blockIdx.x;
    int r = rows ? __ldg(rows + p) : p;
    if (rows && row_div > 1) r /= row_div;
    const float *src = x + (size_t)r * x_stride;
    const float *src2 = x2 ? x2 + (size_t)p * x_stride : nullptr;
    auto val = [&](int k) {
        float v = __ldg(src + k);
        if (src2) {
            const float g = fminf(fmaxf(v, -clamp), clamp);
            v = (g / (1.0f + expf(-g))) * __ldg(src2 + k);
        }
        return v;
    };
    __half *dst = xh + (size_t)p * Kp;
    __half *dlo = xl ? xl + (size_t)p * Kp : nullptr;
    for (int i = K + threadIdx.x; i < Kp; i += blockDim.x) {
        dst[i] = __float2half_rn(0.0f);
        if (dlo) dlo[i] = __float2half_rn(0.0f);
    }
    float amax = 0.0f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) amax = fmaxf(amax, fabsf(val(i)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) sh[0] = v;
    }
    __syncthreads();
    amax = sh[0];
    float sc;
    if (!(amax <= 3.402823466e38f)) sc = __int_as_float(0x7fc00000);
    else if (amax == 0.0f) sc = 1.0f;
    else {
        int e;
        frexpf(amax, &e);
        sc = ldexpf(1.0f, e);
    }
    const float inv = 1.0f / sc;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float v = val(i) * inv;
        const __half h = __float2half_rn(v);
        dst[i] = h;
        if (dlo) dlo[i] = __float2half_rn(v - __half2float(h));   // the rounding residual
    }
    if (threadIdx.x == 0) scale[p] = sc;
}

// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, N = nt, M = 128
__host__ __device__ constexpr uint32_t umma_idesc_f16(int nt) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(nt >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// ---------------------------------------------------------------- decode of 8 weights
template <int QT> struct TcFmt;
//   chunk_bytes  GGUF bytes of one row's 256-element chunk
//   raw_row      shared-memory bytes per row of a raw stage
template <int QT> struct TcFmt { static constexpr int chunk_bytes = 0, raw_row = 0; };
// (32-element block formats: the 16-byte-aligned window around the chunk's blocks, whose
// rows need not start on 16 bytes and whose last chunk may hold fewer than 8 blocks)
template <> struct TcFmt<MLQ_Q8_0> { static constexpr int chunk_bytes = 8 * 34, raw_row = 288; };
template <> struct TcFmt<MLQ_Q4_0> { static constexpr int chunk_bytes = 8 * 18, raw_row = 160; };
template <> struct TcFmt<MLQ_Q4_1> { static constexpr int chunk_bytes = 8 * 20, raw_row = 176; };
template <> struct TcFmt<MLQ_Q5_0> { static constexpr int chunk_bytes = 8 * 22, raw_row = 192; };
template <> struct TcFmt<MLQ_MXFP4> { static constexpr int chunk_bytes = 8 * 17, raw_row = 160; };
template <int QT> constexpr bool tc_block32() {
    return QT == MLQ_Q8_0 || QT == MLQ_Q4_0 || QT == MLQ_Q4_1 || QT == MLQ_Q5_0 || QT == MLQ_MXFP4;
}
template <> struct TcFmt<MLQ_Q4_K> { static constexpr int chunk_bytes = 144, raw_row = chunk_bytes; };
template <> struct TcFmt<MLQ_Q5_K> { static constexpr int chunk_bytes = 176, raw_row = chunk_bytes; };
// a super-block and the 2 bytes before it when it starts 2 bytes past a 4-byte boundary
// (Q6_K: the 16-byte-aligned window around the super-block, at most 240 bytes)
template <> struct TcFmt<MLQ_Q6_K> { static constexpr int chunk_bytes = 210, raw_row = 240; };

__device__ __forceinline__ __half2 u2h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }
__device__ __forceinline__ uint32_t h22u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// Two codes of the packed bytes q (selector 0x5140: bytes 0, 1; 0x7362: bytes 2, 3) made
// exact fp16 integers by placing them under the exponent byte 0x64 (1024 + code), less
// `off`, then ds * v - dm in fp32 and rounded to fp16: the same arithmetic as the scalar
// form, at 3.5 instructions per weight instead of a byte load, shifts and a conversion each.
__device__ __forceinline__ uint32_t codes_h2(uint32_t q, uint32_t sel, __half2 off, float ds, float dm) {
    const float2 f = __half22float2(__hsub2(u2h2(__byte_perm(q, 0x64646464u, sel)), off));
    return h22u(__floats2half2_rn(ds * f.x - dm, ds * f.y - dm));
}
__device__ __forceinline__ uint32_t codes_h2(uint32_t q, uint32_t sel, __half2 off, float ds) {
    const float2 f = __half22float2(__hsub2(u2h2(__byte_perm(q, 0x64646464u, sel)), off));
    return h22u(__floats2half2_rn(ds * f.x, ds * f.y));
}

// elements 8j .. 8j+7 of a 256-element row chunk (raw bytes `c`), the GGUF dequantization
// of each format in fp32, rounded to fp16
template <int QT>
__device__ __forceinline__ uint4 deq8(const uint8_t *c, int j) {
    float v[8];
    if constexpr (QT == MLQ_Q8_0) {
        const uint8_t *bp = c + (j >> 2) * 34;
        const int o = (j & 3) * 8;
        const float d = f16_at(bp);
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = d * (float)(int8_t)bp[2 + o + i];
    } else if constexpr (QT == MLQ_Q4_0 || QT == MLQ_Q4_1 || QT == MLQ_Q5_0) {
        constexpr int bb = QT == MLQ_Q4_0 ? 18 : QT == MLQ_Q4_1 ? 20 : 22;
        constexpr int hdr = QT == MLQ_Q4_0 ? 2 : QT == MLQ_Q4_1 ? 4 : 6;
        const uint8_t *bp = c + (j >> 2) * bb;
        const int o = (j & 3) * 8;
        const float d = f16_at(bp);
        uint32_t qh = 0;
        if constexpr (QT == MLQ_Q5_0) qh = bp[2] | (bp[3] << 8) | (bp[4] << 16) | ((uint32_t)bp[5] << 24);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int e = o + i;
            int q = e < 16 ? (bp[hdr + e] & 0xF) : (bp[hdr + e - 16] >> 4);
            if constexpr (QT == MLQ_Q4_0) v[i] = d * (float)(q - 8);
            else if constexpr (QT == MLQ_Q4_1) v[i] = d * (float)q + f16_at(bp + 2);
            else v[i] = d * (float)((q | (int)(((qh >> e) & 1u) << 4)) - 16);
        }
    } else if constexpr (QT == MLQ_Q6_K) {
        // ggml's dequantize_row_q6_K: element n = 128h + 32k + l (l < 32) is
        // d * sc[8h + l/16 + 2k] * ((ql nibble | qh bits 2k..2k+1 << 4) - 32), the ql byte
        // being ql[64h + l + 32(k & 1)] (low nibble for k < 2) and the qh byte qh[32h + l];
        // the 8 elements' codes are assembled four to a word
        const int n0 = 8 * j, h = n0 >> 7, k = (n0 >> 5) & 3, l0 = n0 & 31;
        const float ds = f16_at(c + 208) * (float)(int8_t)c[192 + 8 * h + (l0 >> 4) + 2 * k];
        uint32_t ql[2], qh[2];
        load_words<2>(c + 64 * h + 32 * (k & 1) + l0, ql);
        load_words<2>(c + 128 + 32 * h + l0, qh);
        const __half2 off = u2h2(0x64206420u);   // 1056 = 1024 + 32
        uint32_t o[4];
#pragma unroll
        for (int w = 0; w < 2; w++) {
            const uint32_t lo = (k < 2 ? ql[w] : ql[w] >> 4) & 0x0F0F0F0Fu;
            const uint32_t q = lo | (((qh[w] >> (2 * k)) & 0x03030303u) << 4);
            o[2 * w] = codes_h2(q, 0x5140u, off, ds);
            o[2 * w + 1] = codes_h2(q, 0x7362u, off, ds);
        }
        return make_uint4(o[0], o[1], o[2], o[3]);
    } else {   // Q4_K, Q5_K: one 256-element super-block per chunk (16-byte aligned)
        const int sub = j >> 2, g = sub >> 1, l0 = (j & 3) * 8;
        const uint8_t *sc = c + 4;
        int s, m;
        if (sub < 4) {
            s = sc[sub] & 63;
            m = sc[sub + 4] & 63;
        } else {
            s = (sc[sub + 4] & 0xF) | ((sc[sub - 4] >> 6) << 4);
            m = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
        }
        const float ds = f16_at(c) * (float)s, dm = f16_at(c + 2) * (float)m;
        const uint2 qs = *reinterpret_cast<const uint2 *>(c + (QT == MLQ_Q4_K ? 16 : 48) + 32 * g + l0);
        uint32_t qw[2] = {qs.x, qs.y};
        if constexpr (QT == MLQ_Q5_K) {
            const uint2 qh = *reinterpret_cast<const uint2 *>(c + 16 + l0);
            qw[0] = ((sub & 1 ? qw[0] >> 4 : qw[0]) & 0x0F0F0F0Fu) | (((qh.x >> sub) & 0x01010101u) << 4);
            qw[1] = ((sub & 1 ? qw[1] >> 4 : qw[1]) & 0x0F0F0F0Fu) | (((qh.y >> sub) & 0x01010101u) << 4);
        } else {
            qw[0] = (sub & 1 ? qw[0] >> 4 : qw[0]) & 0x0F0F0F0Fu;
            qw[1] = (sub & 1 ? qw[1] >> 4 : qw[1]) & 0x0F0F0F0Fu;
        }
        const __half2 off = u2h2(0x64006400u);   // 1024
        return make_uint4(codes_h2(qw[0], 0x5140u, off, ds, dm), codes_h2(qw[0], 0x7362u, off, ds, dm),
                          codes_h2(qw[1], 0x5140u, off, ds, dm), codes_h2(qw[1], 0x7362u, off, ds, dm));
    }
    __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
    __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
    uint4 r;
    r.x = *reinterpret_cast<uint32_t *>(&h0);
    r.y = *reinterpret_cast<uint32_t *>(&h1);
    r.z = *reinterpret_cast<uint32_t *>(&h2);
    r.w = *reinterpret_cast<uint32_t *>(&h3);
    return r;
}

// Packed decode of one whole 32-element block (Q8_0 / Q4_0) into four 16-byte fp16 chunks.
// An integer code c in 0..255 becomes the fp16 value 1024 + c by placing it under the
// exponent byte 0x64 (PRMT); subtracting 1024 + bias (HSUB2) is exact, and the one HMUL2
// by the block scale rounds the exact product once -- the same fp16 as rounding d*q.

__device__ __forceinline__ void bytes_to_h2(uint32_t u, __half2 bias, __half2 d, uint32_t &lo, uint32_t &hi) {
    lo = h22u(__hmul2(__hsub2(u2h2(__byte_perm(u, 0x64646464u, 0x5140)), bias), d));
    hi = h22u(__hmul2(__hsub2(u2h2(__byte_perm(u, 0x64646464u, 0x7362)), bias), d));
}

// Four E2M1 codes (one per byte, 0..15) as fp16 values of gguf's doubled table
// {0, 1, 2, 3, 4, 6, 8, 12} with the sign bit 3: only the high byte of each fp16 value is
// nonzero, built bytewise: magnitude m >= 2 is (1 + m % 2 / 2) * 2^(m / 2) -> exponent byte
// 0x3C + 4 (m / 2) + 2 (m % 2); m = 1 -> 0x3C; m = 0 -> 0 (+0 for code 8 too, as the table).
__device__ __forceinline__ void e2m1_codes_h2(uint32_t c, float scale, uint32_t &h01, uint32_t &h23) {
    const uint32_t m = c & 0x07070707u;
    const uint32_t e = (m >> 1) & 0x03030303u, man = m & 0x01010101u;
    uint32_t hb = ((e << 2) | (man << 1)) + 0x3C3C3C3Cu;
    const uint32_t small = __vcmpeq4(e, 0u), zero = __vcmpeq4(m, 0u);
    hb = (hb & ~small) | (small & (man * 0x3Cu));
    hb |= ((c & 0x08080808u) << 4) & ~zero;
    const float2 f01 = __half22float2(u2h2(__byte_perm(hb, 0u, 0x1404u)));
    const float2 f23 = __half22float2(u2h2(__byte_perm(hb, 0u, 0x3424u)));
    h01 = h22u(__floats2half2_rn(f01.x * scale, f01.y * scale));
    h23 = h22u(__floats2half2_rn(f23.x * scale, f23.y * scale));
}

template <int QT>
__device__ __forceinline__ void deq_block32(const uint8_t *bp, uint4 (&o)[4], int emax = -1) {
    if constexpr (QT == MLQ_MXFP4) {
        // GGUF MXFP4 block {e, qs[16]}: element j < 16 is the low nibble of qs[j], j >= 16 the
        // high nibble of qs[j-16]; value table[code] * 2^(e - 128) (gguf-py e8m0_to_fp32_half).
        // With emax, the largest block exponent of the row within the chunk, the block is stored
        // as table[code] * 2^(e - emax) (at most 12; fp16 holds it exactly down to 2^-24 of the
        // chunk's largest block) and the chunk's product is scaled by 2^(emax - 128) in fp32
        // after the MMAs, so no block scale leaves fp16's range (a block more than 2^126 below
        // the chunk's largest is flushed to zero)
        const int e = bp[0];
        float sc;
        if (emax < 0) sc = e8m0_half((uint32_t)e);
        else sc = e - emax < -126 ? 0.0f : __uint_as_float((uint32_t)(127 + e - emax) << 23);
        uint32_t w[4];
        load_words<4>(bp + 1, w);
        uint32_t l[8], h[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            e2m1_codes_h2(w[i] & 0x0F0F0F0Fu, sc, l[2 * i], l[2 * i + 1]);
            e2m1_codes_h2((w[i] >> 4) & 0x0F0F0F0Fu, sc, h[2 * i], h[2 * i + 1]);
        }
        o[0] = make_uint4(l[0], l[1], l[2], l[3]);
        o[1] = make_uint4(l[4], l[5], l[6], l[7]);
        o[2] = make_uint4(h[0], h[1], h[2], h[3]);
        o[3] = make_uint4(h[4], h[5], h[6], h[7]);
        return;
    }
    const __half2 d = __half2half2(*reinterpret_cast<const __half *>(bp));   // 2-byte aligned
    if constexpr (QT == MLQ_Q8_0) {
        uint32_t w[8];
        load_words<8>(bp + 2, w);
        const __half2 bias = u2h2(0x64806480u);   // 1152 = 1024 + 128
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            uint32_t a0, a1, b0, b1;
            bytes_to_h2(w[i] ^ 0x80808080u, bias, d, a0, a1);
            bytes_to_h2(w[i + 1] ^ 0x80808080u, bias, d, b0, b1);
            o[i >> 1] = make_uint4(a0, a1, b0, b1);
        }
    } else {   // Q4_0: element j < 16 is the low nibble of qs[j], j >= 16 the high nibble of qs[j-16]
        uint32_t w[4];
        load_words<4>(bp + 2, w);
        const __half2 bias = u2h2(0x64086408u);   // 1032 = 1024 + 8
        uint32_t l[8], h[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            bytes_to_h2(w[i] & 0x0F0F0F0Fu, bias, d, l[2 * i], l[2 * i + 1]);
            bytes_to_h2((w[i] >> 4) & 0x0F0F0F0Fu, bias, d, h[2 * i], h[2 * i + 1]);
        }
        o[0] = make_uint4(l[0], l[1], l[2], l[3]);
        o[1] = make_uint4(l[4], l[5], l[6], l[7]);
        o[2] = make_uint4(h[0], h[1], h[2], h[3]);
        o[3] = make_uint4(h[4], h[5], h[6], h[7]);
    }
}

// Elements 32t .. 32t+31 of a K-quant super-block (chunk bytes `c`) into four 16-byte fp16
// chunks: the sub-block's scales are unpacked once for its 32 weights (deq8 unpacks them
// for every 8), the codes come in as whole words.  Same arithmetic as deq8.
//   Q4_K / Q5_K: t is the 32-element sub-block (one scale / min pair); c 16-byte aligned
//   Q6_K: t = 4h + k, elements 128h + 32k + l (l < 32), two scales (l < 16, l >= 16);
//         c 2-byte aligned at worst
template <int QT>
__device__ __forceinline__ void deq32_k(const uint8_t *c, int t, uint4 (&o)[4]) {
    if constexpr (QT == MLQ_Q6_K) {
        const int h = t >> 2, k = t & 3;
        const float d = f16_at(c + 208);
        const float ds0 = d * (float)(int8_t)c[192 + 8 * h + 2 * k];
        const float ds1 = d * (float)(int8_t)c[192 + 8 * h + 1 + 2 * k];
        uint32_t ql[8], qh[8];
        load_words<8>(c + 64 * h + 32 * (k & 1), ql);
        load_words<8>(c + 128 + 32 * h, qh);
        const __half2 off = u2h2(0x64206420u);   // 1056 = 1024 + 32
#pragma unroll
        for (int w = 0; w < 8; w++) {
            const uint32_t lo = (k < 2 ? ql[w] : ql[w] >> 4) & 0x0F0F0F0Fu;
            const uint32_t q = lo | (((qh[w] >> (2 * k)) & 0x03030303u) << 4);
            const float ds = w < 4 ? ds0 : ds1;
            const uint32_t a0 = codes_h2(q, 0x5140u, off, ds), a1 = codes_h2(q, 0x7362u, off, ds);
            if (w & 1) {
                o[w >> 1].z = a0;
                o[w >> 1].w = a1;
            } else {
                o[w >> 1].x = a0;
                o[w >> 1].y = a1;
            }
        }
    } else {   // Q4_K, Q5_K
        const int sub = t, g = sub >> 1;
        const uint8_t *sc = c + 4;
        int s, m;
        if (sub < 4) {
            s = sc[sub] & 63;
            m = sc[sub + 4] & 63;
        } else {
            s = (sc[sub + 4] & 0xF) | ((sc[sub - 4] >> 6) << 4);
            m = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
        }
        const float ds = f16_at(c) * (float)s, dm = f16_at(c + 2) * (float)m;
        const uint4 *qp = reinterpret_cast<const uint4 *>(c + (QT == MLQ_Q4_K ? 16 : 48) + 32 * g);
        const uint4 q0 = qp[0], q1 = qp[1];
        uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint32_t hw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if constexpr (QT == MLQ_Q5_K) {
            const uint4 h0 = *reinterpret_cast<const uint4 *>(c + 16), h1 = *reinterpret_cast<const uint4 *>(c + 32);
            const uint32_t hh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
            for (int w = 0; w < 8; w++) hw[w] = ((hh[w] >> sub) & 0x01010101u) << 4;
        }
        const __half2 off = u2h2(0x64006400u);   // 1024
#pragma unroll
        for (int w = 0; w < 8; w++) {
            const uint32_t q = ((sub & 1 ? qw[w] >> 4 : qw[w]) & 0x0F0F0F0Fu) | hw[w];
            const uint32_t a0 = codes_h2(q, 0x5140u, off, ds, dm), a1 = codes_h2(q, 0x7362u, off, ds, dm);
            if (w & 1) {
                o[w >> 1].z = a0;
                o[w >> 1].w = a1;
            } else {
                o[w >> 1].x = a0;
                o[w >> 1].y = a1;
            }
        }
    }
}

// byte offset of the 16-byte chunk (row r, K group j of 8) in a [rows][256] fp16 operand
// stored as four 64-wide K atoms of `atom_bytes` each
__device__ __forceinline__ uint32_t sw128_off(int r, int j, int atom_bytes) {
    const int kb = j >> 3, c = j & 7;
    return (uint32_t)(kb * atom_bytes + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

struct TcArgs {
    const uint8_t *W;
    const __half *xh;
    const float *xs;
    float *out;
    int n_rows, K, M;
    long long row_bytes;
    int n_row_tiles;
    int Kp;                // K rounded up to whole 256-element chunks (the activation row pitch)
    int win;               // block formats: rows not on 16 bytes or K % 256 != 0 (windowed copies)
    int *status;
    // split-K: work item w = (row tile w / n_splits, K slice w % n_splits of chunks_per_split
    // chunks); with n_splits > 1 each item leaves its partial tile in part and the last item
    // of a tile to finish (counters) adds the slices in order and writes the outputs
    int n_splits, chunks_per_split;
    float *part;
    int *counters;
    // grouped experts (items set): work item = one 128-row tile of one expert's matrix against
    // up to 8 of its sorted activation rows (k_group_plan's items {e, m0, mc, tile}); tiles from
    // tiles_per_expert on are the second matrix (W2 / out2); xh / xs are indexed by sorted row,
    // results go to row out_rows[p] (identity if null) of out; no K split
    const int4 *items;
    const int *n_items_dev;
    long long estride, estride2;
    const uint8_t *W2;
    float *out2;
    int tiles_per_expert;
    const int *out_rows;
    // grouped: the activation rows' fp16 residuals (x / s - hi); token-tile rows 0-7 take the
    // item's rows from xh, rows 8-15 the same rows from xlo, and the two sums are added
    const __half *xlo;
};

template <int QT, int NT>
struct TcSmem {
    static constexpr int a_bytes = 4 * kTcAtomBytes;                          // 64 KB
    static constexpr int b_atom = NT * 128;
    static constexpr int b_bytes = 4 * b_atom;                                // NT * 512
    static constexpr int raw_bytes = kTcRows * TcFmt<QT>::raw_row;
    // copy stages (raw weights + activation atoms): as many as fit beside the A operand, up
    // to 4, so that the copies run up to 3 chunks ahead of the decode
    static constexpr int stage_pair = b_bytes + raw_bytes;
    static constexpr int n_st_fit = (227 * 1024 - a_bytes - 64 - 1024 - 4096 - 1024 - 16) / stage_pair;
    static constexpr int n_st = n_st_fit > 4 ? 4 : n_st_fit;
    static constexpr int off_a = 0;
    static constexpr int off_b = a_bytes;                                     // n_st stages
    static constexpr int off_raw = off_b + n_st * b_bytes;                    // n_st stages
    static constexpr int off_bar = (off_raw + n_st * raw_bytes + 15) / 16 * 16;
    static constexpr int off_cx = off_bar + 64;                               // [2][128] ints
    static constexpr int off_lo = off_cx + 1024;                              // [128][8] floats
    static constexpr int total = off_lo + 4096 + 1024;                        // + alignment slack
};

template <int QT, int NT>
__global__ void __launch_bounds__(kTcThreads, 1) k_gemm_tc(TcArgs a) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    using S = TcSmem<QT, NT>;
    extern __shared__ uint8_t smem_raw[];
    // operand atoms must start on 1024-byte boundaries
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sa = smem + S::off_a;
    uint64_t *mma_bar = reinterpret_cast<uint64_t *>(smem + S::off_bar);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + S::off_bar + 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + S::off_bar + 16);
    volatile int *flag_last = reinterpret_cast<volatile int *>(smem + S::off_bar + 20);
    const int tid = threadIdx.x, warp = tid >> 5;
    // MXFP4: per-chunk products (two accumulator buffers) scaled into fp32 registers
    constexpr bool kPerChunk = QT == MLQ_MXFP4;
    constexpr int ncols = kPerChunk ? (2 * NT < 32 ? 32 : 2 * NT) : (NT < 32 ? 32 : NT);
    int *cx = reinterpret_cast<int *>(smem + S::off_cx);   // [2][128] chunk row exponents
    float *lo_tile = reinterpret_cast<float *>(smem + S::off_lo);   // grouped: residual sums [128][8]
    float accr[kPerChunk ? NT / 2 : 1];                     // warps 0-7: row rl, their NT/2 columns
    constexpr int chunk_bytes = TcFmt<QT>::chunk_bytes;
    constexpr int pieces = chunk_bytes / 16;
    int tok0 = blockIdx.y * NT;        // first activation row of the work item
    int mtok = NT;                     // grouped: the item's rows (the rest of the tile: zeros)
    const uint8_t *Wb = a.W;           // the item's weight matrix
    float *outp = a.out;
    const bool grouped = a.items != nullptr;
    const int n_chunks = (a.K + kTcKC - 1) / kTcKC;
    (void)n_chunks;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(mma_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    uint32_t issued = 0, waited = 0;   // MMA groups committed (all threads) / seen complete (thread 0)
    constexpr uint32_t idesc = umma_idesc_f16(NT);

    // every committed MMA group has completed; thread 0 waits (bounded) and the verdict
    // reaches all threads through the barrier, so control flow stays uniform
    auto wait_mma = [&]() -> bool {
        if (tid == 0 && !*abort_flag) {
            while (waited < issued) {
                if (!mbar_wait_bounded(mma_bar, waited & 1)) {
                    *abort_flag = 1;
                    report_status(a.status, DEV_ST_WAIT_FULL);
                    break;
                }
                waited++;
            }
        }
        __syncthreads();
        return !*abort_flag;
    };
    // chunk ci of row tile rt: raw weights and activation atoms into stage st
    auto issue_copies = [&](int rt, int ci, int st) {
        const int r0 = rt * kTcRows;
        uint8_t *raw = smem + S::off_raw + st * S::raw_bytes;
        if constexpr (QT == MLQ_Q6_K) {
            // 16-byte pieces of the aligned window around the super-block (row pitches are
            // multiples of 16, the super-blocks only 2-byte aligned); a piece past the end of
            // the matrix (the last row's last super-block) is copied byte by byte up to it
            const uint8_t *w_end = Wb + (size_t)a.n_rows * a.row_bytes;
            for (int p = tid; p < kTcRows * 15; p += kTcThreads) {
                const int r = p / 15, i = p - r * 15;
                if (r0 + r >= a.n_rows) continue;
                const uint8_t *src = Wb + (size_t)(r0 + r) * a.row_bytes + (size_t)ci * 210;
                const uintptr_t off = reinterpret_cast<uintptr_t>(src) & 15;
                if (16 * i >= (int)off + 210) continue;   // the window needs ceil((off + 210) / 16) pieces
                const uint8_t *piece = src - off + 16 * i;
                uint8_t *dst = raw + r * 240 + 16 * i;
                if (piece + 16 <= w_end) cp_async16(dst, piece);
                else
                    for (int b = 0; b < 16 && piece + b < w_end; b++) dst[b] = piece[b];
            }
        } else if (tc_block32<QT>() && a.win) {
            // the chunk's (up to 8) blocks through 16-byte pieces of their aligned window
            constexpr int bb = chunk_bytes / 8, np = TcFmt<QT>::raw_row / 16;
            const int nbc = min(8, a.K / 32 - 8 * ci);
            const uint8_t *w_end = Wb + (size_t)a.n_rows * a.row_bytes;
            for (int p = tid; p < kTcRows * np; p += kTcThreads) {
                const int r = p / np, i = p - r * np;
                if (r0 + r >= a.n_rows) continue;
                const uint8_t *src = Wb + (size_t)(r0 + r) * a.row_bytes + (size_t)ci * chunk_bytes;
                const uintptr_t off = reinterpret_cast<uintptr_t>(src) & 15;
                if (16 * i >= (int)off + nbc * bb) continue;
                const uint8_t *piece = src - off + 16 * i;
                uint8_t *dst = raw + r * TcFmt<QT>::raw_row + 16 * i;
                if (piece + 16 <= w_end) cp_async16(dst, piece);
                else
                    for (int b = 0; b < 16 && piece + b < w_end; b++) dst[b] = piece[b];
            }
        } else {
            for (int p = tid; p < kTcRows * pieces; p += kTcThreads) {
                const int r = p / pieces, i = p - r * pieces;
                if (r0 + r < a.n_rows)
                    cp_async16(raw + r * TcFmt<QT>::raw_row + 16 * i,
                               Wb + (size_t)(r0 + r) * a.row_bytes + (size_t)ci * chunk_bytes + 16 * i);
            }
        }
        uint8_t *sb = smem + S::off_b + st * S::b_bytes;
        for (int p = tid; p < NT * 32; p += kTcThreads) {
            const int n = p >> 5, j = p & 31;
            const bool lo = grouped && n >= 8;
            const int nr = lo ? n - 8 : n;
            if (nr < mtok)
                cp_async16(sb + sw128_off(n, j, S::b_atom),
                           (lo ? a.xlo : a.xh) + (size_t)(tok0 + nr) * a.Kp + (size_t)ci * kTcKC + 8 * j);
            else   // grouped: rows past the item's own are zeros
                *reinterpret_cast<uint4 *>(sb + sw128_off(n, j, S::b_atom)) = make_uint4(0, 0, 0, 0);
        }
        cp_async_commit();
    };

    // MXFP4: add chunk c's product (its accumulator buffer, complete) times 2^(emax - 128) of
    // each row into the registers of warps 0-7 (same lane / column split as the epilogue)
    auto fold_chunk = [&](int c) {
        if constexpr (kPerChunk) {
            if (warp < 8) {
                tc_fence_after();
                const int q = warp & 3, half = (warp >> 2) & 1, rl = 32 * q + (tid & 31);
                const float sc = e8m0_half((uint32_t)cx[(c & 1) * kTcRows + rl]);
#pragma unroll
                for (int c0 = 0; c0 < NT / 2; c0 += 8) {
                    float v[8];
                    tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((c & 1) * NT + half * (NT / 2) + c0), v);
#pragma unroll
                    for (int i = 0; i < 8; i++) accr[c0 + i] = fmaf(v[i], sc, accr[c0 + i]);
                }
            }
        }
    };
    const int n_items = grouped ? *a.n_items_dev : a.n_row_tiles * a.n_splits;
    for (int wi = blockIdx.x; wi < n_items && !*abort_flag; wi += gridDim.x) {
        int rt = wi / a.n_splits, sp = wi - rt * a.n_splits;
        if (grouped) {
            const int4 it = a.items[wi];   // {expert, first sorted row, rows, tile}
            const bool second = it.w >= a.tiles_per_expert;
            rt = second ? it.w - a.tiles_per_expert : it.w;
            sp = 0;
            Wb = (second ? a.W2 : a.W) + (size_t)it.x * (size_t)(second ? a.estride2 : a.estride);
            outp = second ? a.out2 : a.out;
            tok0 = it.y;
            mtok = it.z;
        }
        const int r0 = rt * kTcRows;
        const int c_begin = sp * a.chunks_per_split;
        const int c_end = min(n_chunks, c_begin + a.chunks_per_split);
        constexpr int NS = S::n_st;
        static_assert(NS >= 2, "two copy stages must fit");
        // chunks c_begin .. c_begin + NS - 2 in flight before the first decode (one commit
        // group each, empty past the end)
        for (int c = 0; c < NS - 1; c++) {
            if (c_begin + c < c_end) issue_copies(rt, c_begin + c, c);
            else cp_async_commit();
        }
#pragma unroll
        for (int i = 0; i < (kPerChunk ? NT / 2 : 1); i++) accr[i] = 0.0f;
        for (int ci = c_begin; ci < c_end; ci++) {
            const int st = (ci - c_begin) % NS;
            // the previous chunk's MMAs read A and the stage refilled next: wait before reuse
            if (!wait_mma()) break;
            if (ci > c_begin) fold_chunk(ci - 1);
            if (ci + NS - 1 < c_end) issue_copies(rt, ci + NS - 1, (ci + NS - 1 - c_begin) % NS);
            else cp_async_commit();
            cp_async_wait<NS - 1>();   // chunk ci's group is complete
            __syncthreads();
            // decode this chunk's raw weights into the swizzled fp16 A operand
            const uint8_t *raw = smem + S::off_raw + st * S::raw_bytes;
            if constexpr (QT == MLQ_Q8_0 || QT == MLQ_Q4_0 || QT == MLQ_MXFP4) {
                constexpr int bb = chunk_bytes / 8;
                const int nbc = min(8, a.K / 32 - 8 * ci);   // blocks in this chunk (the rest: zeros)
                for (int p = tid; p < kTcRows * 8; p += kTcThreads) {
                    const int r = p >> 3, b = p & 7;
                    uint4 o[4];
                    const bool valid = r0 + r < a.n_rows && b < nbc;
                    const uintptr_t src = reinterpret_cast<uintptr_t>(Wb) +
                                          (uintptr_t)((size_t)(r0 + r) * a.row_bytes + (size_t)ci * chunk_bytes);
                    const uint8_t *bp = raw + r * TcFmt<QT>::raw_row + (a.win ? (src & 15) : 0) + b * bb;
                    int cmax = -1;
                    if constexpr (QT == MLQ_MXFP4) {
                        // the row's largest block exponent in this chunk: lanes 8j..8j+7 hold one row
                        cmax = valid ? (int)bp[0] : 0;
#pragma unroll
                        for (int o2 = 1; o2 < 8; o2 <<= 1) cmax = max(cmax, __shfl_xor_sync(0xffffffffu, cmax, o2));
                        if (b == 0) cx[(ci & 1) * kTcRows + r] = cmax;
                    }
                    if (valid) {
                        deq_block32<QT>(bp, o, cmax);
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; c++) o[c] = make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int c = 0; c < 4; c++) *reinterpret_cast<uint4 *>(sa + sw128_off(r, 4 * b + c, kTcAtomBytes)) = o[c];
                }
            } else if constexpr (QT == MLQ_Q4_K || QT == MLQ_Q5_K || QT == MLQ_Q6_K) {
                // thread item (row r, 32-element group t): lanes of a warp take 4 rows x 8 groups
                for (int p = tid; p < kTcRows * 8; p += kTcThreads) {
                    const int r = p >> 3, t = p & 7;
                    uint4 o[4];
                    if (r0 + r < a.n_rows) {
                        if constexpr (QT == MLQ_Q6_K) {
                            const uintptr_t src = reinterpret_cast<uintptr_t>(Wb) +
                                                  (uintptr_t)((size_t)(r0 + r) * a.row_bytes + (size_t)ci * 210);
                            deq32_k<QT>(raw + r * 240 + (src & 15), t, o);
                        } else {
                            deq32_k<QT>(raw + r * chunk_bytes, t, o);
                        }
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; c++) o[c] = make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int c = 0; c < 4; c++) *reinterpret_cast<uint4 *>(sa + sw128_off(r, 4 * t + c, kTcAtomBytes)) = o[c];
                }
            } else {
                for (int p = tid; p < kTcRows * 32; p += kTcThreads) {
                    const int r = p >> 5, j = p & 31;
                    uint4 h = make_uint4(0, 0, 0, 0);
                    if (r0 + r < a.n_rows) {
                        if constexpr (QT == MLQ_Q6_K) {
                            const uintptr_t src = reinterpret_cast<uintptr_t>(Wb) +
                                                  (uintptr_t)((size_t)(r0 + r) * a.row_bytes + (size_t)ci * 210);
                            h = deq8<QT>(raw + r * 240 + (src & 15), j);
                        } else if constexpr (tc_block32<QT>()) {   // Q4_1, Q5_0
                            const uintptr_t src = reinterpret_cast<uintptr_t>(Wb) +
                                                  (uintptr_t)((size_t)(r0 + r) * a.row_bytes + (size_t)ci * chunk_bytes);
                            if ((j >> 2) < a.K / 32 - 8 * ci)
                                h = deq8<QT>(raw + r * TcFmt<QT>::raw_row + (a.win ? (src & 15) : 0), j);
                        } else {
                            h = deq8<QT>(raw + r * chunk_bytes, j);
                        }
                    }
                    *reinterpret_cast<uint4 *>(sa + sw128_off(r, j, kTcAtomBytes)) = h;
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const uint32_t a0 = smem_u32(sa), b0 = smem_u32(smem + S::off_b + st * S::b_bytes);
#pragma unroll
                for (int k = 0; k < kTcKC / 16; k++) {
                    const int kb = k >> 2, k16 = k & 3;
                    // MXFP4: each chunk into its own accumulator buffer (scaled and added in fp32)
                    umma_f16(kPerChunk ? tmem + (uint32_t)((ci & 1) * NT) : tmem,
                             umma_desc_sw128(a0 + kb * kTcAtomBytes + k16 * 32),
                             umma_desc_sw128(b0 + kb * S::b_atom + k16 * 32), idesc,
                             ((!kPerChunk && ci > c_begin) || k > 0) ? 1u : 0u);
                }
                umma_commit(mma_bar);
            }
            issued++;
        }
        // epilogue: accumulators -> scaled fp32 outputs
        if (!wait_mma()) break;
        fold_chunk(c_end - 1);
        tc_fence_after();
        // warps 0-7: TMEM lane quarter warp % 4 (weight rows), column half warp / 4
        const int q = warp & 3, half = (warp >> 2) & 1;
        const bool reader = warp < 8;
        const int rl = 32 * q + (tid & 31), row = r0 + rl;
        constexpr int per = NT / 2;   // columns per warp
        if (grouped) {
            // token columns 0-7 (warps 0-3) hold the rows' sums of the fp16 parts, columns 8-15
            // (warps 4-7) those of the residuals: the latter pass through shared memory
            float v[8];
            if (reader) {
                if constexpr (kPerChunk) {
#pragma unroll
                    for (int i = 0; i < 8; i++) v[i] = accr[i];
                } else {
                    tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(half * 8), v);
                }
                if (half == 1) {
#pragma unroll
                    for (int i = 0; i < 8; i++) lo_tile[rl * 8 + i] = v[i];
                }
            }
            __syncthreads();
            if (reader && half == 0) {
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int t = tok0 + i;
                    if (i < mtok && row < a.n_rows) {
                        const int o = a.out_rows ? __ldg(a.out_rows + t) : t;
                        outp[(size_t)o * a.n_rows + row] = (v[i] + lo_tile[rl * 8 + i]) * a.xs[t];
                    }
                }
            }
            tc_fence_before();
            __syncthreads();
        } else if (a.n_splits == 1) {
#pragma unroll
            for (int c0 = 0; c0 < per && reader; c0 += 8) {
                float v[8];
                if constexpr (kPerChunk) {
#pragma unroll
                    for (int i = 0; i < 8; i++) v[i] = accr[c0 + i];
                } else {
                    tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(half * per + c0), v);
                }
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int c = half * per + c0 + i, t = tok0 + c;
                    if (t < a.M && row < a.n_rows) a.out[(size_t)t * a.n_rows + row] = v[i] * a.xs[t];
                }
            }
            tc_fence_before();
            __syncthreads();
        } else {
            // partial tile [NT][128] of this K slice; the last slice to land reduces in order
            const size_t tile = (size_t)rt * gridDim.y + blockIdx.y;
            float *pt = a.part + (tile * a.n_splits + sp) * (size_t)(NT * kTcRows);
#pragma unroll
            for (int c0 = 0; c0 < per && reader; c0 += 8) {
                float v[8];
                if constexpr (kPerChunk) {
#pragma unroll
                    for (int i = 0; i < 8; i++) v[i] = accr[c0 + i];
                } else {
                    tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(half * per + c0), v);
                }
#pragma unroll
                for (int i = 0; i < 8; i++) pt[(size_t)(half * per + c0 + i) * kTcRows + rl] = v[i];
            }
            tc_fence_before();
            __threadfence();
            __syncthreads();
            if (tid == 0) *flag_last = (atomicAdd(a.counters + tile, 1) == a.n_splits - 1) ? 1 : 0;
            __syncthreads();
            if (*flag_last && reader) {
                __threadfence();
                const float *p0 = a.part + tile * a.n_splits * (size_t)(NT * kTcRows);
                for (int c = half * per; c < half * per + per; c++) {
                    float acc = 0.0f;
                    for (int k = 0; k < a.n_splits; k++) acc += __ldcg(p0 + ((size_t)k * NT + c) * kTcRows + rl);
                    const int t = tok0 + c;
                    if (t < a.M && row < a.n_rows) a.out[(size_t)t * a.n_rows + row] = acc * a.xs[t];
                }
                if (tid == 0) a.counters[tile] = 0;
            }
            __syncthreads();
        }
    }
    // drain: no copy or MMA may still target this CTA's memory when it exits
    cp_async_wait<0>();
    if (tid == 0) {   // one more bounded wait for MMAs still in flight after an abort
        while (waited < issued && mbar_wait_bounded(mma_bar, waited & 1)) waited++;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}

// ---------------------------------------------------------------- host side
// per-(device, stream) fp16 activation / split-K buffer, grown on demand outside graph
// capture.  A grown-out buffer is retired, not freed: a captured graph may still hold its
// address.  Retired buffers are freed with the graphs (forget_tc_scratch, after the
// plans and their graphs are destroyed).
struct TcScratch { void *p = nullptr; size_t bytes = 0; };
static std::mutex g_tc_mu;
static std::map<std::pair<int, cudaStream_t>, TcScratch> g_tc_scratch;
static std::vector<void *> g_tc_retired;

void forget_tc_scratch() {
    std::lock_guard<std::mutex> lk(g_tc_mu);
    cudaDeviceSynchronize();
    for (auto &kv : g_tc_scratch)
        if (kv.second.p) cudaFree(kv.second.p);
    for (void *p : g_tc_retired) cudaFree(p);
    g_tc_scratch.clear();
    g_tc_retired.clear();
}

void *tc_scratch(cudaStream_t s, size_t bytes) {
    const LaunchEnv *env = launch_env();
    if (!env || env->no_alloc) return nullptr;   // a caller that allocates nothing: fall back
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_tc_mu);
    TcScratch &t = g_tc_scratch[std::make_pair(dev, s)];
    if (t.bytes >= bytes) return t.p;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return nullptr;   // no allocation inside a capture: the caller falls back
    }
    if (t.p) g_tc_retired.push_back(t.p);
    t.p = nullptr;
    t.bytes = 0;
    if (cudaMalloc(&t.p, bytes) != cudaSuccess) {
        cudaGetLastError();
        t.p = nullptr;
        return nullptr;
    }
    t.bytes = bytes;
    return t.p;
}

bool tc_supported(int qt, const uint8_t *W, int K, long long row_bytes) {
    int cb = 0;
    switch (qt) {
        case MLQ_Q8_0: cb = TcFmt<MLQ_Q8_0>::chunk_bytes; break;
        case MLQ_Q4_0: cb = TcFmt<MLQ_Q4_0>::chunk_bytes; break;
        case MLQ_Q4_1: cb = TcFmt<MLQ_Q4_1>::chunk_bytes; break;
        case MLQ_Q5_0: cb = TcFmt<MLQ_Q5_0>::chunk_bytes; break;
        case MLQ_Q4_K: cb = TcFmt<MLQ_Q4_K>::chunk_bytes; break;
        case MLQ_Q5_K: cb = TcFmt<MLQ_Q5_K>::chunk_bytes; break;
        case MLQ_MXFP4: cb = TcFmt<MLQ_MXFP4>::chunk_bytes; break;
        case MLQ_Q6_K: return K % kTcKC == 0 && ((uintptr_t)W & 3) == 0;
        default: return false;
    }
    if (qt == MLQ_Q8_0 || qt == MLQ_Q4_0 || qt == MLQ_Q4_1 || qt == MLQ_Q5_0)   // any K % 32, 2-byte aligned
        return K % 32 == 0 && K > 0 && ((uintptr_t)W & 1) == 0;
    if (qt == MLQ_MXFP4) return K % 32 == 0 && K > 0;   // read bytewise: no alignment
    return K % kTcKC == 0 && cb % 16 == 0 && row_bytes % 16 == 0 && ((uintptr_t)W & 15) == 0;
}

template <int QT, int NT>
static int launch_tc_t(const TcArgs &a, int n_tok_tiles, cudaStream_t s) {
    using S = TcSmem<QT, NT>;
    const LaunchEnv *env = launch_env();
    if (!env) return MLQ_ERR_NO_DEVICE;
    static bool attr = false;
    if (!attr) {
        if (!MLQ_CUDA(cudaFuncSetAttribute(k_gemm_tc<QT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::total)))
            return MLQ_ERR_CUDA;
        attr = true;
    }
    int gx = env->num_sms / n_tok_tiles;
    if (gx < 1) gx = 1;
    if (gx > a.n_row_tiles * a.n_splits) gx = a.n_row_tiles * a.n_splits;
    return MLQ_CUDA(launch_pdl_k(k_gemm_tc<QT, NT>, dim3(gx, n_tok_tiles), dim3(kTcThreads), S::total, s, a)) ? MLQ_OK
                                                                                                             : MLQ_ERR_CUDA;
}

template <int QT>
static int launch_tc_q(const TcArgs &a, int NT, int n_tok_tiles, cudaStream_t s) {
    if (NT == 16) return launch_tc_t<QT, 16>(a, n_tok_tiles, s);
    if (NT == 32) return launch_tc_t<QT, 32>(a, n_tok_tiles, s);
    return launch_tc_t<QT, 64>(a, n_tok_tiles, s);
}

// out [M][n_rows] = x [M][K] . W^T on the tensor cores; MLQ_ERR_UNSUPPORTED when the
// format / shape / alignment is not covered (the caller then uses the dp4a kernels)
int launch_gemm_tc(const uint8_t *W, int qt, const float *x, float *out, int n_rows, int K, int M, cudaStream_t s) {
    const long long rb = (long long)(K / block_elems(qt)) * block_bytes(qt);
    if (!tc_supported(qt, W, K, rb) || M < 1) return MLQ_ERR_UNSUPPORTED;
    const int NT = M <= 16 ? 16 : M <= 32 ? 32 : 64;
    const int n_tok_tiles = (M + NT - 1) / NT;
    const int Mp = n_tok_tiles * NT;
    const LaunchEnv *env = launch_env();
    if (!env) return MLQ_ERR_NO_DEVICE;
    // split K over CTAs when the row tiles alone cannot fill the SMs
    const int n_row_tiles = (n_rows + kTcRows - 1) / kTcRows, n_chunks = (K + kTcKC - 1) / kTcKC;
    const int Kp = n_chunks * kTcKC;
    int n_splits = 1;
    if (n_row_tiles * n_tok_tiles < env->num_sms) {
        n_splits = env->num_sms / (n_row_tiles * n_tok_tiles);
        if (n_splits > n_chunks) n_splits = n_chunks;
        if (n_splits < 1) n_splits = 1;
    }
    const int cps = (n_chunks + n_splits - 1) / n_splits;
    n_splits = (n_chunks + cps - 1) / cps;
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t xh_bytes = al((size_t)Mp * Kp * sizeof(__half));
    const size_t xs_bytes = al((size_t)Mp * sizeof(float));
    const size_t n_tiles = (size_t)n_row_tiles * n_tok_tiles;
    const size_t cnt_bytes = n_splits > 1 ? al(n_tiles * sizeof(int)) : 0;
    const size_t part_bytes = n_splits > 1 ? n_tiles * n_splits * NT * kTcRows * sizeof(float) : 0;
    uint8_t *scr = (uint8_t *)tc_scratch(s, xh_bytes + xs_bytes + cnt_bytes + part_bytes);
    if (!scr) return MLQ_ERR_UNSUPPORTED;
    __half *xh = (__half *)scr;
    float *xs = (float *)(scr + xh_bytes);
    int *counters = n_splits > 1 ? (int *)(scr + xh_bytes + xs_bytes) : nullptr;
    float *part = n_splits > 1 ? (float *)(scr + xh_bytes + xs_bytes + cnt_bytes) : nullptr;
    if (counters && !MLQ_CUDA(cudaMemsetAsync(counters, 0, n_tiles * sizeof(int), s))) return MLQ_ERR_CUDA;
    if (!MLQ_CUDA(launch_pdl_k(k_x_to_f16, dim3(Mp), dim3(256), 0, s, x, xh, xs, M, K, Kp))) return MLQ_ERR_CUDA;
    const bool block32 = qt == MLQ_Q8_0 || qt == MLQ_Q4_0 || qt == MLQ_Q4_1 || qt == MLQ_Q5_0 || qt == MLQ_MXFP4;
    // (MXFP4 chunks are 136 bytes: never all on 16-byte boundaries)
    const int win = block32 && (qt == MLQ_MXFP4 || K % kTcKC != 0 || rb % 16 != 0 || ((uintptr_t)W & 15) != 0);
    TcArgs a{W, xh, xs, out, n_rows, K, M, rb, n_row_tiles, Kp, win, env->d_status, n_splits, cps, part, counters};
    switch (qt) {
        case MLQ_Q8_0: return launch_tc_q<MLQ_Q8_0>(a, NT, n_tok_tiles, s);
        case MLQ_Q4_0: return launch_tc_q<MLQ_Q4_0>(a, NT, n_tok_tiles, s);
        case MLQ_Q4_1: return launch_tc_q<MLQ_Q4_1>(a, NT, n_tok_tiles, s);
        case MLQ_Q5_0: return launch_tc_q<MLQ_Q5_0>(a, NT, n_tok_tiles, s);
        case MLQ_Q4_K: return launch_tc_q<MLQ_Q4_K>(a, NT, n_tok_tiles, s);
        case MLQ_Q5_K: return launch_tc_q<MLQ_Q5_K>(a, NT, n_tok_tiles, s);
        case MLQ_Q6_K: return launch_tc_q<MLQ_Q6_K>(a, NT, n_tok_tiles, s);
        case MLQ_MXFP4: return launch_tc_q<MLQ_MXFP4>(a, NT, n_tok_tiles, s);
        default: return MLQ_ERR_UNSUPPORTED;
    }
}


static int tc_kp(int K) { return (K + kTcKC - 1) / kTcKC * kTcKC; }

size_t tc_grouped_xh_bytes(int R, int K) { return (size_t)R * tc_kp(K) * sizeof(__half); }

int launch_rows_to_f16(const float *x, const float *x2, const int *rows, int row_div, int x_stride, float clamp, int R,
                       int K, __half *xh, __half *xl, float *xs, cudaStream_t s) {
    if (R <= 0) return MLQ_OK;
    return MLQ_CUDA(launch_pdl_k(k_rows_to_f16, dim3(R), dim3(256), 0, s, x, x2, rows, row_div, x_stride > 0 ? x_stride : K, clamp, K, tc_kp(K), xh, xl,
                                    xs)) ? MLQ_OK : MLQ_ERR_CUDA;
}

bool tc_grouped_supported(int qt, const uint8_t *W, long long estride, int K) {
    const long long rb = (long long)(K / block_elems(qt)) * block_bytes(qt);
    if (!tc_supported(qt, W, K, rb)) return false;
    const bool block32 = qt == MLQ_Q8_0 || qt == MLQ_Q4_0 || qt == MLQ_Q4_1 || qt == MLQ_Q5_0 || qt == MLQ_MXFP4;
    if (block32) return qt == MLQ_MXFP4 || estride % 2 == 0;
    return qt == MLQ_Q6_K ? estride % 4 == 0 : estride % 16 == 0;
}

template <int QT>
static int launch_tc_grouped_q(const TcArgs &a, int grid, cudaStream_t s) {
    using S = TcSmem<QT, 16>;
    static bool attr = false;
    if (!attr) {
        if (!MLQ_CUDA(cudaFuncSetAttribute(k_gemm_tc<QT, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::total)))
            return MLQ_ERR_CUDA;
        attr = true;
    }
    return MLQ_CUDA(launch_pdl_k(k_gemm_tc<QT, 16>, dim3(grid, 1), dim3(kTcThreads), S::total, s, a)) ? MLQ_OK
                                                                                                       : MLQ_ERR_CUDA;
}

// Grouped experts on the tensor cores: k_group_plan's items (tiles of 128 rows, chunks of up
// to 8 sorted rows) against sorted fp16 rows xh [R][Kp] with scales xs [R]
int launch_gemm_tc_grouped(int qt, const uint8_t *W, long long estride, const uint8_t *W2, long long estride2,
                           int n_rows, int K, const void *items, const int *n_items_dev, int n_items_bound,
                           const __half *xh, const __half *xl, const float *xs, float *out, float *out2,
                           const int *out_rows, cudaStream_t s) {
    const LaunchEnv *env = launch_env();
    if (!xl) return MLQ_ERR_UNSUPPORTED;
    if (!env) return MLQ_ERR_NO_DEVICE;
    if (!tc_grouped_supported(qt, W, estride, K) || (W2 && !tc_grouped_supported(qt, W2, estride2, K)))
        return MLQ_ERR_UNSUPPORTED;
    const long long rb = (long long)(K / block_elems(qt)) * block_bytes(qt);
    const int n_row_tiles = (n_rows + kTcRows - 1) / kTcRows, n_chunks = (K + kTcKC - 1) / kTcKC;
    const bool block32 = qt == MLQ_Q8_0 || qt == MLQ_Q4_0 || qt == MLQ_Q4_1 || qt == MLQ_Q5_0 || qt == MLQ_MXFP4;
    const int win = block32 && (qt == MLQ_MXFP4 || K % kTcKC != 0 || rb % 16 != 0 || ((uintptr_t)W & 15) != 0 ||
                                estride % 16 != 0 || (W2 && (((uintptr_t)W2 & 15) != 0 || estride2 % 16 != 0)));
    TcArgs a{W, xh, xs, out, n_rows, K, 0, rb, n_row_tiles, tc_kp(K), win, env->d_status, 1, n_chunks, nullptr, nullptr,
             (const int4 *)items, n_items_dev, estride, estride2, W2, out2, n_row_tiles, out_rows, xl};
    int grid = env->num_sms < n_items_bound ? env->num_sms : n_items_bound;
    if (grid < 1) grid = 1;
    switch (qt) {
        case MLQ_Q8_0: return launch_tc_grouped_q<MLQ_Q8_0>(a, grid, s);
        case MLQ_Q4_0: return launch_tc_grouped_q<MLQ_Q4_0>(a, grid, s);
        case MLQ_Q4_1: return launch_tc_grouped_q<MLQ_Q4_1>(a, grid, s);
        case MLQ_Q5_0: return launch_tc_grouped_q<MLQ_Q5_0>(a, grid, s);
        case MLQ_Q4_K: return launch_tc_grouped_q<MLQ_Q4_K>(a, grid, s);
        case MLQ_Q5_K: return launch_tc_grouped_q<MLQ_Q5_K>(a, grid, s);
        case MLQ_Q6_K: return launch_tc_grouped_q<MLQ_Q6_K>(a, grid, s);
        case MLQ_MXFP4: return launch_tc_grouped_q<MLQ_MXFP4>(a, grid, s);
        default: return MLQ_ERR_UNSUPPORTED;
    }
}

}  // namespace mlq
