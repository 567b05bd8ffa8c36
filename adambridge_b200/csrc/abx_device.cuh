// abx_device.cuh -- device-side element formats and update arithmetic of libabx.
//
// Every floating-point operation is written with an explicit round-to-nearest
// intrinsic (__fmul_rn, __fadd_rn, __fmaf_rn, __fdiv_rn, __fsqrt_rn) so that
// which operations are fused -- and therefore every result bit -- is fixed by
// this source and not by the compiler.  The reference fuses three multiply-adds
// per AdamW element in the vector loop of its SIMD kernels and none in its ISO-C
// scalar tail (adambridge/csrc/adambridge_kernels.c:171-178 vs :446-455); the
// FUSED template parameter selects between the two.  Lion is fused everywhere
// (:1107-1120).  The library is compiled with -ftz=false, so subnormals are
// kept exactly as the host's SSE/AVX arithmetic keeps them.
#pragma once

#include <cstdint>

namespace abx {

__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// lowbias32 integer hash: the stateless per-element random stream (csrc:100-106).
__device__ __forceinline__ uint32_t hash32(uint32_t x)
{
    x = (x ^ (x >> 16)) * 0x7feb352dU;
    x = (x ^ (x >> 15)) * 0x846ca68bU;
    return x ^ (x >> 16);
}

// bf16 bits of x (in the high half), nearest-even; NaN quieted (csrc:108-112).
__device__ __forceinline__ uint32_t bf16_rne(uint32_t b)
{
    const uint32_t r = b + 0x7fffU + ((b >> 16) & 1U);
    return (b & 0x7fffffffU) > 0x7f800000U ? (b | 0x00400000U) : r;
}

// A bf16 moment: stochastic -- add 16 random bits below the kept half and truncate --
// or nearest-even (csrc:120-126).  Returns the 16 stored bits.
__device__ __forceinline__ uint32_t bf16_store_bits(float x, bool sr, uint32_t r)
{
    const uint32_t b = f2u(x);
    return (sr ? b + (r & 0xffffU) : bf16_rne(b)) >> 16;
}

// The fp24 master's 24 kept bits (csrc:140-146): stochastic or nearest-even in the
// low byte, which is then cleared; a NaN is quieted and kept whole.
__device__ __forceinline__ uint32_t f24_bits(uint32_t b, bool sr, uint32_t r)
{
    const uint32_t k = (b + (sr ? (r & 0xffU) : 0x7fU + ((b >> 8) & 1U))) & ~0xffU;
    return (b & 0x7fffffffU) > 0x7f800000U ? (b | 0x00400000U) : k;
}

// ---- FP8 codec ---------------------------------------------------------------------
// E4M3fn (m; max 448, NaN = S.1111.111, no inf) and E5M2 (sqrt(v); max 57344, IEEE
// inf/NaN).  Decoding shifts the code's exponent and mantissa into an fp32 bit
// pattern with exponent field e (a normal or, for e = 0, a subnormal fp32 of the
// same significand) and rescales by a power of two; the product is exact.

__device__ __forceinline__ float dec_e4m3(uint32_t c)
{
    const uint32_t mag = c & 0x7fU;
    float a = __fmul_rn(u2f(mag << 20), 0x1p120f);   // 2^(e-127) * 1.m  ->  2^(e-7) * 1.m
    a = mag == 0x7fU ? __uint_as_float(0x7fc00000U) : a;
    return u2f(f2u(a) | ((c & 0x80U) << 24));
}

__device__ __forceinline__ float dec_e5m2(uint32_t c)
{
    const uint32_t mag = c & 0x7fU;
    float a = __fmul_rn(u2f(mag << 21), 0x1p112f);   // 2^(e-127) * 1.m  ->  2^(e-15) * 1.m
    a = (mag & 0x7cU) == 0x7cU ? ((mag & 3U) ? __uint_as_float(0x7fc00000U) : __uint_as_float(0x7f800000U)) : a;
    return u2f(f2u(a) | ((c & 0x80U) << 24));
}

// fp32 -> code (csrc:857-876): optional stochastic truncation of the fp32
// significand to the format's width, saturation at the format's max, then
// nearest-even -- in the exponent/mantissa fields for normals, as an integer
// multiple of the smallest subnormal below the normal range (an fp32 add of 2^23
// rounds that multiple to an integer).
template <int MBITS, int BIAS>
__device__ __forceinline__ uint32_t enc_fp8(float x, bool sr, uint32_t r, float fmax, uint32_t nan_code)
{
    constexpr int drop = 23 - MBITS;
    constexpr uint32_t low = (1U << drop) - 1U;
    const uint32_t b = f2u(x);
    const uint32_t sign = (b >> 24) & 0x80U;
    const bool is_nan = (b & 0x7fffffffU) > 0x7f800000U;
    const uint32_t t = sr ? ((b + (r & low)) & ~low) : b;
    float a = u2f(t & 0x7fffffffU);
    a = a > fmax ? fmax : a;
    const uint32_t ab = f2u(a);
    const uint32_t rn = sr ? ab : ab + (low >> 1) + ((ab >> drop) & 1U);
    const uint32_t normal = ((((rn >> 23) & 0xffU) + (uint32_t)(BIAS - 127)) << MBITS) | ((rn >> drop) & ((1U << MBITS) - 1U));
    const float sub_scale = u2f((uint32_t)(127 + BIAS + MBITS - 1) << 23);
    const uint32_t sub = f2u(__fadd_rn(__fmul_rn(a, sub_scale), 8388608.0f)) - 0x4b000000U;
    const float min_normal = u2f((uint32_t)(127 + 1 - BIAS) << 23);
    const uint32_t code = a >= min_normal ? normal : sub;
    return (sign | (is_nan ? nan_code : code)) & 0xffU;
}

__device__ __forceinline__ uint32_t enc_e4m3(float x, bool sr, uint32_t r) { return enc_fp8<3, 7>(x, sr, r, 448.0f, 0x7fU); }
__device__ __forceinline__ uint32_t enc_e5m2(float x, bool sr, uint32_t r) { return enc_fp8<2, 15>(x, sr, r, 57344.0f, 0x7eU); }

// ---- update arithmetic -------------------------------------------------------------

struct Coef {
    float b1, b2, omb1, omb2, decay, step, isbc2, eps;
};

// AdamW on one element in torch.optim.AdamW's order; m and v updated in fp32.
// Returns the new master value before storage rounding.
template <bool FUSED>
__device__ __forceinline__ float adamw_elem(float p, float g, float& m, float& v, const Coef& c)
{
    p = __fmul_rn(p, c.decay);
    if (FUSED) {
        m = __fmaf_rn(c.b1, m, __fmul_rn(c.omb1, g));
        v = __fmaf_rn(c.b2, v, __fmul_rn(c.omb2, __fmul_rn(g, g)));
        const float denom = __fmaf_rn(__fsqrt_rn(v), c.isbc2, c.eps);
        return __fmaf_rn(-c.step, __fdiv_rn(m, denom), p);
    } else {
        m = __fadd_rn(__fmul_rn(c.b1, m), __fmul_rn(c.omb1, g));
        v = __fadd_rn(__fmul_rn(c.b2, v), __fmul_rn(c.omb2, __fmul_rn(g, g)));
        const float denom = __fadd_rn(__fmul_rn(__fsqrt_rn(v), c.isbc2), c.eps);
        return __fsub_rn(p, __fmul_rn(c.step, __fdiv_rn(m, denom)));
    }
}

__device__ __forceinline__ float adamw_elem_sel(float p, float g, float& m, float& v, const Coef& c, bool fused)
{
    return fused ? adamw_elem<true>(p, g, m, v, c) : adamw_elem<false>(p, g, m, v, c);
}

// The same, also returning sqrt(new v): the FP8 path re-encodes v as sqrt(v), and for v >= 0 that is the
// square root the update already took (the reference takes it twice, csrc:454 and :1000).
template <bool FUSED>
__device__ __forceinline__ float adamw_elem_sq(float p, float g, float& m, float& v, float& sq, const Coef& c)
{
    p = __fmul_rn(p, c.decay);
    if (FUSED) {
        m = __fmaf_rn(c.b1, m, __fmul_rn(c.omb1, g));
        v = __fmaf_rn(c.b2, v, __fmul_rn(c.omb2, __fmul_rn(g, g)));
        sq = __fsqrt_rn(v);
        return __fmaf_rn(-c.step, __fdiv_rn(m, __fmaf_rn(sq, c.isbc2, c.eps)), p);
    } else {
        m = __fadd_rn(__fmul_rn(c.b1, m), __fmul_rn(c.omb1, g));
        v = __fadd_rn(__fmul_rn(c.b2, v), __fmul_rn(c.omb2, __fmul_rn(g, g)));
        sq = __fsqrt_rn(v);
        return __fsub_rn(p, __fmul_rn(c.step, __fdiv_rn(m, __fadd_rn(__fmul_rn(sq, c.isbc2), c.eps))));
    }
}

// Two floats -> packed bf16 pair (lo in the low half), round-to-nearest-even by the hardware conversion.
// Identical to bf16_rne for every non-NaN input; every NaN reaching it was produced by GPU arithmetic
// (the canonical 0x7fffffff), which both map to 0x7fff.
__device__ __forceinline__ uint32_t pack_bf16_rne(float lo, float hi)
{
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

// High halves of two 32-bit words -> one word (lo's half in the low 16 bits).
__device__ __forceinline__ uint32_t pack_hi16(uint32_t lo, uint32_t hi) { return __byte_perm(lo, hi, 0x7632); }

// Lion on one element: c = b1 m + (1-b1) g; p = p decay - lr sign(c); m = b2 m + (1-b2) g,
// each multiply-add fused; sign(0) = sign(NaN) = 0.
__device__ __forceinline__ float lion_elem(float p, float g, float& m, const Coef& c)
{
    const float cm = __fmaf_rn(c.b1, m, __fmul_rn(c.omb1, g));
    const float u = cm > 0.0f ? c.step : (cm < 0.0f ? -c.step : 0.0f);
    m = __fmaf_rn(c.b2, m, __fmul_rn(c.omb2, g));
    return __fmaf_rn(p, c.decay, -u);
}

}  // namespace abx
