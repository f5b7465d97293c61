// Block-scaled E2M1 (kind::mxf4) pieces shared by the MXFP4 tensor-core kernels
// (gemv_mxf4_tc.cu: one weight matrix; moe_mxf4_tc.cu: grouped experts): the instruction
// descriptor, the MMA, and the encoding of fp32 activations as 8 E2M1 "planes" with
// per-32-element E8M0 scales.
#pragma once

#include <stdint.h>

namespace mlq {

constexpr int kMxf4Planes = 8;   // E2M1 planes per activation row

// kind::mxf4 block-scaled instruction descriptor: A and B E2M1, K-major, UE8M0 scales,
// M = 128, N = n; the scale-factor byte ids of this MMA
__device__ __forceinline__ uint32_t idesc_mxf4(int n, uint32_t sfa_id, uint32_t sfb_id) {
    return (sfb_id << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) |
           ((uint32_t)(128 >> 4) << 24) | (sfa_id << 29);
}

__device__ __forceinline__ void umma_mxf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %6, 0;\n"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%4], [%5], p;\n}\n" ::"r"(
            tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
        : "memory");
}

// 2^e as a float for -127 <= e <= 127 (2^-127 is subnormal)
__device__ __forceinline__ float pow2f(int e) {
    return e >= -126 ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(0x00400000u);
}

// The 8 planes of one 32-element block, held by a 4-lane group of the warp (gmask: the group's
// lanes; every lane of the warp calls this): lane j holds r[0..3] = x[4j..4j+3] and
// r[4..7] = x[16+4j..16+4j+3].  words[p] = bytes 4j..4j+3 of plane p's 16 bytes (byte i pairs
// x[i], low nibble, with x[i+16]); codes[p] = plane p's E8M0 scale byte.
// x = sum_p 2^e_p q_p: plane 0 takes the smallest 2^e0 with amax / 2^e0 <= 6, plane p uses
// 2^(e0 - 2p); after plane 0 the residual is at most 2^e0 (half the widest E2M1 gap), after
// plane p >= 1 at most a quarter of plane p's scale, so no plane saturates and one
// max-reduction per block is enough.  A non-finite element gives NaN scales (code 255); a
// zero block gives code 127 and zero codes.
__device__ __forceinline__ void mxf4_block_planes(float (&r)[8], uint32_t gmask, uint32_t (&words)[kMxf4Planes],
                                                  uint32_t (&codes)[kMxf4Planes]) {
    float a = 0.0f;
    bool bad = false;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        a = fmaxf(a, fabsf(r[e]));
        bad |= !(fabsf(r[e]) <= 3.402823466e38f);
    }
    const bool finite = (__ballot_sync(0xffffffffu, bad) & gmask) == 0;
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2, 4));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1, 4));
    const uint32_t ab = __float_as_uint(a), E = ab >> 23;
    const bool zero = ab == 0u;
    // smallest 2^e0 with amax / 2^e0 <= 6: e0 = E - 2 when the significand is <= 1.5
    const int e0 = E == 0u ? -127 : (int)E - 127 - ((ab & 0x7FFFFFu) <= 0x400000u ? 2 : 1);
#pragma unroll
    for (int p = 0; p < kMxf4Planes; p++) {
        uint32_t code = 127, word = 0;
        if (!finite) {
            code = 255;   // NaN scale: a non-finite activation makes every product NaN
        } else if (!zero) {
            const int e = max(e0 - 2 * p, -127);
            code = (uint32_t)(e + 127);
            const float inv = __uint_as_float((uint32_t)(127 - e) << 23), sc = pow2f(e);
            // hardware E2M1 rounding (nearest, ties to even, saturating) of 8 elements, and
            // the codes' values back as f16 pairs (E2M1 values are exact in f16).  Every byte
            // goes through a 16-bit register of its own: 4-byte vector moves of 8-bit
            // registers dropped bytes 2 and 3 in a probe of this toolchain.
#pragma unroll
            for (int q = 0; q < 4; q++) {
                unsigned short b;
                uint32_t h;
                asm("{\n.reg .b8 t;\ncvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\nmov.b16 %0, {t, t};\n}"
                    : "=h"(b)
                    : "f"(r[4 + q] * inv), "f"(r[q] * inv));
                asm("{\n.reg .b8 lo, hi;\nmov.b16 {lo, hi}, %1;\ncvt.rn.f16x2.e2m1x2 %0, lo;\n}"
                    : "=r"(h)
                    : "h"(b));
                word |= (uint32_t)(b & 0xFFu) << (8 * q);
                const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&h));
                r[q] = fmaf(-v.x, sc, r[q]);          // exact: exact product, exact difference
                r[4 + q] = fmaf(-v.y, sc, r[4 + q]);
            }
        }
        words[p] = word;
        codes[p] = code;
    }
}

}  // namespace mlq
