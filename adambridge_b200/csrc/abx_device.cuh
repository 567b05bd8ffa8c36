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

// The per-step coefficients of one segment (abx_hparams without the seed).
struct Coef {
    float b1, b2, omb1, omb2, decay, step, isbc2, eps;
};

__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// lowbias32 integer hash: the stateless per-element random stream (csrc:100-106).
__device__ __forceinline__ uint32_t hash32(uint32_t x)
{
    x = (x ^ (x >> 16)) * 0x7feb352dU;
    x = (x ^ (x >> 15)) * 0x846ca68bU;
    return x ^ (x >> 16);
}

// The hash words of elements idx0 .. idx0+3 of one stream.  When idx0 is a multiple of 4 (a
// segment whose offset is), the inputs (idx0 + k) ^ seed = X ^ k differ only in their two low
// bits, so the first xor-shift is shared: (X ^ k) ^ ((X ^ k) >> 16) = (X ^ (X >> 16)) ^ k.
__device__ __forceinline__ void hash4(uint32_t idx0, uint32_t seed, uint32_t (&r)[4])
{
    if ((idx0 & 3U) == 0) {
        const uint32_t x0 = idx0 ^ seed;
        const uint32_t s = x0 ^ (x0 >> 16);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t x = (s ^ (uint32_t)k) * 0x7feb352dU;
            x = (x ^ (x >> 15)) * 0x846ca68bU;
            r[k] = x ^ (x >> 16);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) r[k] = hash32((idx0 + (uint32_t)k) ^ seed);
    }
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

// ---- FP8 codec on the hardware converters, 2 or 4 elements at a time ------------------
// Decoding: the e4m3 / e5m2 -> f16 conversions and f16 -> f32 are exact for every finite
// code, so they equal the reference's table lookups (NaN codes give a NaN).
// Encoding: after the stochastic truncation of the fp32 significand (the reference's first
// step), cvt.rn.satfinite rounds |x| to nearest even in the format and saturates at its
// largest finite value -- what the reference's normal and subnormal branches compute -- for
// every non-NaN input; a NaN input takes the reference's NaN code.  The sign is reattached
// from x, so -0 keeps its sign as in the reference.

// 4 codes (byte k = element k) -> 4 floats.
template <bool E4M3>
__device__ __forceinline__ void dec4_fp8(uint32_t w, float (&x)[4])
{
    uint32_t h01, h23;
    if (E4M3)
        asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; cvt.rn.f16x2.e4m3x2 %0, lo; cvt.rn.f16x2.e4m3x2 %1, hi; }"
            : "=r"(h01), "=r"(h23) : "r"(w));
    else
        asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %2; cvt.rn.f16x2.e5m2x2 %0, lo; cvt.rn.f16x2.e5m2x2 %1, hi; }"
            : "=r"(h01), "=r"(h23) : "r"(w));
    asm("{ .reg .b16 a, b; mov.b32 {a, b}, %2; cvt.f32.f16 %0, a; cvt.f32.f16 %1, b; }" : "=f"(x[0]), "=f"(x[1]) : "r"(h01));
    asm("{ .reg .b16 a, b; mov.b32 {a, b}, %2; cvt.f32.f16 %0, a; cvt.f32.f16 %1, b; }" : "=f"(x[2]), "=f"(x[3]) : "r"(h23));
}

// The reference's stochastic truncation of x's significand to MBITS bits, then |.|.
template <int MBITS, bool SR>
__device__ __forceinline__ float fp8_trunc_abs(float x, uint32_t r)
{
    constexpr uint32_t low = (1U << (23 - MBITS)) - 1U;
    const uint32_t b = f2u(x);
    const uint32_t t = SR ? ((b + (r & low)) & ~low) : b;
    return u2f(t & 0x7fffffffU);
}

// Sign and NaN handling around a hardware code: sign | (NaN ? nan_code : code).
__device__ __forceinline__ uint32_t fp8_finish(float x, uint32_t code, uint32_t nan_code)
{
    const uint32_t b = f2u(x);
    return ((b >> 24) & 0x80U) | ((b & 0x7fffffffU) > 0x7f800000U ? nan_code : code);
}

// 4 floats -> 4 codes (byte k = element k); r[k] are the elements' random bits (SR only).
template <bool E4M3, bool SR>
__device__ __forceinline__ uint32_t enc4_fp8(const float (&x)[4], const uint32_t (&r)[4])
{
    constexpr int MB = E4M3 ? 3 : 2;
    constexpr uint32_t NAN_CODE = E4M3 ? 0x7fU : 0x7eU;
    float a[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) a[k] = fp8_trunc_abs<MB, SR>(x[k], r[k]);
    uint16_t c01, c23;
    if (E4M3) {
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(c01) : "f"(a[1]), "f"(a[0]));
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(c23) : "f"(a[3]), "f"(a[2]));
    } else {
        asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(c01) : "f"(a[1]), "f"(a[0]));
        asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(c23) : "f"(a[3]), "f"(a[2]));
    }
    const uint32_t c[4] = {(uint32_t)c01 & 0xffU, (uint32_t)c01 >> 8, (uint32_t)c23 & 0xffU, (uint32_t)c23 >> 8};
    return fp8_finish(x[0], c[0], NAN_CODE) | (fp8_finish(x[1], c[1], NAN_CODE) << 8) |
           (fp8_finish(x[2], c[2], NAN_CODE) << 16) | (fp8_finish(x[3], c[3], NAN_CODE) << 24);
}

// ---- packed pairs: sm_100a f32x2 arithmetic ---------------------------------------------
// fma/mul/add.rn.f32x2 round each lane exactly as the scalar instruction does, so a pair of
// elements costs one FP32 instruction per operation instead of two.
typedef unsigned long long f2x;

__device__ __forceinline__ f2x pk2(float a, float b)
{
    f2x r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ void up2(f2x r, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r)); }

__device__ __forceinline__ f2x fma2(f2x a, f2x b, f2x c)
{
    f2x d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ f2x mul2(f2x a, f2x b)
{
    f2x d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// x / s for a pair, correctly rounded, by Markstein's correction (see div_by_scale below):
// Y = (RN(1/s), RN(1/s)), NS = (-s, -s).  Valid for the same range of s and x; signed x gives the
// negated quotient of |x| (every step rounds symmetrically) except that -0 comes out +0.
__device__ __forceinline__ f2x div2(f2x X, f2x Y, f2x NS)
{
    const f2x Q0 = mul2(X, Y);
    return fma2(fma2(Q0, NS, X), Y, Q0);
}

// The update's coefficients as pairs (both lanes equal).
struct Coef2 {
    f2x b1, b2, omb1, omb2, decay, nstep, isbc2, eps;
};

__device__ __forceinline__ Coef2 coef2(const Coef& c)
{
    return Coef2{pk2(c.b1, c.b1), pk2(c.b2, c.b2), pk2(c.omb1, c.omb1), pk2(c.omb2, c.omb2),
                 pk2(c.decay, c.decay), pk2(-c.step, -c.step), pk2(c.isbc2, c.isbc2), pk2(c.eps, c.eps)};
}

// Fused AdamW on elements (2j, 2j+1) -- the vector-loop arithmetic of adamw_elem<true>, pairwise.
// (s0, s1) receive sqrt(new v).
__device__ __forceinline__ void adamw2_fused(float& p0, float& p1, float g0, float g1, float& m0, float& m1,
                                             float& v0, float& v1, const Coef2& c, float& s0, float& s1)
{
    const f2x G = pk2(g0, g1);
    const f2x P = mul2(pk2(p0, p1), c.decay);
    const f2x M = fma2(c.b1, pk2(m0, m1), mul2(c.omb1, G));
    const f2x V = fma2(c.b2, pk2(v0, v1), mul2(c.omb2, mul2(G, G)));
    up2(M, m0, m1);
    up2(V, v0, v1);
    s0 = __fsqrt_rn(v0);
    s1 = __fsqrt_rn(v1);
    float d0, d1;
    up2(fma2(pk2(s0, s1), c.isbc2, c.eps), d0, d1);
    up2(fma2(c.nstep, pk2(__fdiv_rn(m0, d0), __fdiv_rn(m1, d1)), P), p0, p1);
}

// Lion on elements (2j, 2j+1), pairwise.
__device__ __forceinline__ void lion2(float& p0, float& p1, float g0, float g1, float& m0, float& m1,
                                      const Coef2& c, float step)
{
    const f2x G = pk2(g0, g1);
    const f2x Mo = pk2(m0, m1);
    float c0, c1;
    up2(fma2(c.b1, Mo, mul2(c.omb1, G)), c0, c1);
    const float u0 = c0 > 0.0f ? step : (c0 < 0.0f ? -step : 0.0f);
    const float u1 = c1 > 0.0f ? step : (c1 < 0.0f ? -step : 0.0f);
    up2(fma2(pk2(p0, p1), c.decay, pk2(-u0, -u1)), p0, p1);
    up2(fma2(c.b2, Mo, mul2(c.omb2, G)), m0, m1);
}

// Block scale absmax / fmax, correctly rounded: the constant reciprocal of fmax with Markstein's
// correction (exact remainder for finite amax >= 2^-100), else IEEE division (tiny or infinite
// amax: inf / fmax = inf, as the reference divides).  amax > 0.
__device__ __forceinline__ float scale_fmt(float amax, float fmax, float y)
{
    if (!(amax >= 0x1p-100f && amax <= 0x1p127f)) return __fdiv_rn(amax, fmax);
    const float q0 = __fmul_rn(amax, y);
    return __fmaf_rn(__fmaf_rn(-q0, fmax, amax), y, q0);
}

template <bool E4M3>
__device__ __forceinline__ float scale_of(float amax)
{
    // RN(1/448), RN(1/57344)
    return E4M3 ? scale_fmt(amax, 448.0f, 0x1.24924ap-9f) : scale_fmt(amax, 57344.0f, 0x1.24924ap-16f);
}

// Out-of-line copy of enc4_fp8 for the rare groups holding a NaN (kept out of the hot path's code).
template <bool E4M3, bool SR>
__device__ __noinline__ uint32_t enc4_fp8_slow(float x0, float x1, float x2, float x3, uint32_t r0, uint32_t r1,
                                               uint32_t r2, uint32_t r3)
{
    const float x[4] = {x0, x1, x2, x3};     // scalar arguments: passed in registers, no local copies
    const uint32_t r[4] = {r0, r1, r2, r3};
    return enc4_fp8<E4M3, SR>(x, r);
}

// 4 non-NaN floats -> 4 codes (byte k = element k), the sign handled by the converter: the
// stochastic truncation only touches significand bits (a carry out of them ends in the exponent,
// never in the sign bit, for any non-NaN value), and cvt.rn.satfinite is symmetric in the sign,
// so sign | code(|t|) == cvt(t).  Callers route groups that may hold a NaN to enc4_fp8.
template <bool E4M3, bool SR>
__device__ __forceinline__ uint32_t enc4_plain(const float (&x)[4], const uint32_t (&r)[4])
{
    constexpr uint32_t low = (1U << (23 - (E4M3 ? 3 : 2))) - 1U;
    float a[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t b = f2u(x[k]);
        a[k] = u2f(SR ? ((b + (r[k] & low)) & ~low) : b);
    }
    uint16_t c01, c23;
    if (E4M3) {
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(c01) : "f"(a[1]), "f"(a[0]));
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(c23) : "f"(a[3]), "f"(a[2]));
    } else {
        asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(c01) : "f"(a[1]), "f"(a[0]));
        asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(c23) : "f"(a[3]), "f"(a[2]));
    }
    return (uint32_t)c01 | ((uint32_t)c23 << 16);
}

// ---- division by a block scale -------------------------------------------------------
// x / s, correctly rounded, for a block-constant s > 0: with y = RN(1/s), q0 = RN(|x| y) is within
// one ulp of |x|/s, the remainder |x| - s q0 is exact in one FMA, and RN(q0 + remainder * y) is the
// correctly rounded quotient (P. Markstein, IBM J. Res. Dev. 34(1), 1990; the correction theorem
// for division).  Exactness of the remainder needs its quantum above the subnormal range: it holds
// for |x| >= 2^-100, and below that the quotient (|x| / s < 2^-20 when s >= 2^-80) encodes to a
// zero code whatever its last bits.  `fast_scale` tells whether s is in that range; otherwise the
// caller divides with __fdiv_rn.
__device__ __forceinline__ bool fast_scale(float s) { return s >= 0x1p-80f && s <= 0x1p100f; }

// IEEE quotients for blocks whose scale is outside the fast range (out of line: rare).
static __device__ __noinline__ float4 div4_ieee(float4 x, float s)
{
    return make_float4(__fdiv_rn(x.x, s), __fdiv_rn(x.y, s), __fdiv_rn(x.z, s), __fdiv_rn(x.w, s));
}

__device__ __forceinline__ float div_by_scale(float x, float s, float y)
{
    const float a = fabsf(x);
    const float q0 = __fmul_rn(a, y);
    const float q = __fmaf_rn(__fmaf_rn(-q0, s, a), y, q0);
    return copysignf(q, x);
}

// ---- update arithmetic -------------------------------------------------------------

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
