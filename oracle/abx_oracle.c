/*
 * abx_oracle.c -- TEST INFRASTRUCTURE ONLY: the CPU checker for libabx.
 *
 * A plain-C, single-threaded restatement of the fused AdamW / Lion update of
 * adambridge (adambridge/csrc/adambridge_kernels.c), written to state the
 * reference's arithmetic as explicitly as possible so the CUDA kernels can be
 * compared against it bit for bit.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it; the product never does.
 *
 * Build: `make -C oracle` (gcc -O2 -std=c11: ISO C mode turns floating-point
 * contraction off, so every multiply and add written separately below is
 * rounded separately, and fmaf() is the only fused operation).
 *
 * What the reference computes, element by element (each function cites the
 * reference lines it restates):
 *   - The vector loop of its AVX-512 / AVX2 / NEON kernels fuses three
 *     multiply-adds per AdamW element and runs over whole vectors; the last
 *     n % lanes elements of each piece go through the scalar function, whose
 *     ISO-C build fuses nothing.  Pieces start on 128-element boundaries, so for
 *     a segment of n elements, element i is "fused" iff i < n - n % lanes
 *     (lanes 16 / 8 / 4; the scalar level has lanes 0: nothing fused).
 *   - Lion is written with fmaf everywhere, so every level gives the same bits.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/abx.h"

#if defined(_WIN32)
#  define ORACLE_API __declspec(dllexport)
#else
#  define ORACLE_API __attribute__((visibility("default")))
#endif

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---- random bits: lowbias32 of (element index ^ stream seed) (csrc:100-106) ---- */
ORACLE_API uint32_t abxo_hash32(uint32_t x)
{
    x = (x ^ (x >> 16)) * 0x7feb352dU;
    x = (x ^ (x >> 15)) * 0x846ca68bU;
    return x ^ (x >> 16);
}

/* The three rounding streams of one (param, step) seed (csrc:164-165; precision.py:131-137). */
static uint32_t stream_v(uint32_t seed) { return abxo_hash32(seed ^ 0xA511E9B3U); }
static uint32_t stream_p(uint32_t seed) { return abxo_hash32(seed ^ 0x6C8E9CF5U); }

/* ---- per-step seed: three splitmix64-style rounds over (base, index, step) (csrc:773-790) ---- */
static uint64_t mix_round(uint64_t h, uint64_t v)
{
    h = (h ^ v) * 0xBF58476D1CE4E5B9ULL;
    h = (h ^ (h >> 31)) * 0x94D049BB133111EBULL;
    return h ^ (h >> 29);
}

ORACLE_API uint32_t abxo_step_seed(uint64_t base, uint64_t index, int64_t step)
{
    uint64_t h = 0x9E3779B97F4A7C15ULL;
    h = mix_round(h, base);
    h = mix_round(h, index);
    h = mix_round(h, (uint64_t)step);
    return (uint32_t)h;
}

/* ---- per-segment coefficients, in double, then narrowed (csrc:793-809) ---- */
ORACLE_API void abxo_hparams_for(const abx_segment* s, abx_hparams* h)
{
    const abx_group* G = s->group;
    const double t = (double)s->step;
    const double bc1 = 1.0 - pow(G->beta1, t);
    const double bc2 = 1.0 - pow(G->beta2, t);
    h->beta1 = (float)G->beta1;
    h->beta2 = (float)G->beta2;
    h->one_minus_beta1 = (float)(1.0 - G->beta1);
    h->one_minus_beta2 = (float)(1.0 - G->beta2);
    h->decay = (float)(1.0 - G->lr * G->weight_decay);
    h->step_size = (float)(s->algorithm == ABX_ALGO_LION ? G->lr : G->lr / bc1);
    h->inv_sqrt_bc2 = (float)(1.0 / sqrt(bc2));
    h->eps = (float)G->eps;
    h->seed = abxo_step_seed(G->seed, s->index, s->step);
    h->stochastic = G->stochastic;
}

/* ---- element formats ---- */

/* bf16 by round-to-nearest-even of the fp32 bits; NaN stays NaN, made quiet (csrc:108-112). */
static uint32_t bf16_rne_bits(uint32_t b)
{
    if ((b & 0x7fffffffU) > 0x7f800000U) return b | 0x00400000U;
    return b + 0x7fffU + ((b >> 16) & 1U);
}

static float load_elem(const void* base, int dt, int64_t i)
{
    if (dt == ABX_DT_BF16) return u2f((uint32_t)((const uint16_t*)base)[i] << 16);
    return ((const float*)base)[i];
}

/* A bf16 moment: stochastic = add 16 random bits below the kept ones and truncate (csrc:120-126). */
static void store_moment(void* base, int dt, int64_t i, float x, int sr, uint32_t r)
{
    if (dt == ABX_DT_F32) { ((float*)base)[i] = x; return; }
    const uint32_t b = sr ? f2u(x) + (r & 0xffffU) : bf16_rne_bits(f2u(x));
    ((uint16_t*)base)[i] = (uint16_t)(b >> 16);
}

/* fp24 master = bf16 hi plane + the next byte (csrc:132-159; precision.py:421-480). */
static float load_master(const abx_segment* s, int64_t i)
{
    if (s->p_dtype == ABX_DT_F24)
        return u2f(((uint32_t)((const uint16_t*)s->p)[i] << 16) | ((uint32_t)s->p_lo[i] << 8));
    return ((const float*)s->p)[i];
}

static uint32_t f24_bits(uint32_t b, int sr, uint32_t r)
{
    if ((b & 0x7fffffffU) > 0x7f800000U) return b | 0x00400000U;   /* NaN: quiet, low byte kept */
    b += sr ? (r & 0xffU) : 0x7fU + ((b >> 8) & 1U);
    return b & ~0xffU;
}

/* Store the new master value; returns the value actually stored. */
static float store_master(const abx_segment* s, int64_t i, float x, int sr, uint32_t r)
{
    if (s->p_dtype == ABX_DT_F24) {
        const uint32_t b = f24_bits(f2u(x), sr, r);
        ((uint16_t*)s->p)[i] = (uint16_t)(b >> 16);
        s->p_lo[i] = (uint8_t)(b >> 8);
        return u2f(b);
    }
    ((float*)s->p)[i] = x;
    return x;
}

static void store_out(const abx_segment* s, int64_t i, float stored)
{
    if (s->out_dtype == ABX_DT_F32) ((float*)s->out)[i] = stored;
    else if (s->out_dtype == ABX_DT_BF16) ((uint16_t*)s->out)[i] = (uint16_t)(bf16_rne_bits(f2u(stored)) >> 16);
}

/* ---- FP8 codec (csrc:811-876; precision.py:341-418) ---- */

/* Value of an 8-bit code with `mbits` mantissa bits and exponent bias `bias`.
 * E4M3fn (ieee = 0): no infinities, only S.1111.111 is NaN.  E5M2 (ieee = 1):
 * the top exponent holds inf and NaN. */
ORACLE_API float abxo_fp8_decode(uint32_t code, int mbits, int bias, int ieee)
{
    const int ebits = 7 - mbits;
    const uint32_t emax = (1u << ebits) - 1u;
    const uint32_t e = (code >> mbits) & emax, mant = code & ((1u << mbits) - 1u);
    const float sign = (code & 0x80u) ? -1.0f : 1.0f;
    if (ieee && e == emax) return mant ? sign * NAN : sign * INFINITY;
    if (!ieee && e == emax && mant == (1u << mbits) - 1u) return sign * NAN;
    if (e == 0) return sign * ldexpf((float)mant, 1 - bias - mbits);
    return sign * ldexpf((float)((1u << mbits) | mant), (int)e - bias - mbits);
}

/* fp32 -> code: optional stochastic truncation of the fp32 mantissa to the
 * format's width (random bits added below it), saturation at the format's
 * largest finite value, then round to nearest even -- in the exponent/mantissa
 * fields for normals, as an integer multiple of the smallest subnormal below
 * the normal range. */
ORACLE_API uint32_t abxo_fp8_encode(float x, int sr, uint32_t r, int mbits, int bias, float fmax, uint32_t nan_code)
{
    const uint32_t b = f2u(x);
    const uint32_t sign = (b >> 24) & 0x80u;
    if ((b & 0x7fffffffU) > 0x7f800000U) return sign | nan_code;
    const int drop = 23 - mbits;
    const uint32_t low = (1u << drop) - 1u;
    const uint32_t t = sr ? (b + (r & low)) & ~low : b;
    float a = u2f(t & 0x7fffffffU);
    if (a > fmax) a = fmax;
    if (a >= ldexpf(1.0f, 1 - bias)) {
        uint32_t ab = f2u(a);
        if (!sr) ab += (low >> 1) + ((ab >> drop) & 1u);
        const uint32_t e = ((ab >> 23) & 0xffu) - 127u + (uint32_t)bias;
        return sign | (e << mbits) | ((ab >> drop) & ((1u << mbits) - 1u));
    }
    return sign | (uint32_t)nearbyintf(a * ldexpf(1.0f, bias + mbits - 1));   /* exact product; RNE */
}

static float dec_m(uint8_t c) { return abxo_fp8_decode(c, 3, 7, 0); }
static float dec_u(uint8_t c) { return abxo_fp8_decode(c, 2, 15, 1); }
static uint8_t enc_m(float x, int sr, uint32_t r) { return (uint8_t)abxo_fp8_encode(x, sr, r, 3, 7, 448.0f, 0x7fu); }
static uint8_t enc_u(float x, int sr, uint32_t r) { return (uint8_t)abxo_fp8_encode(x, sr, r, 2, 15, 57344.0f, 0x7eu); }

/* ---- the element updates ---- */

/* Elements [0, fused_end) of a segment take the vector loop's fused arithmetic. */
static int64_t fused_end(int64_t n, int lanes) { return lanes > 0 ? n - n % lanes : 0; }

/* AdamW on one element, torch.optim.AdamW's operation order (csrc:171-178 unfused, :446-455 fused).
 * Updates *m and *v in fp32; returns the new master value before storage rounding. */
static float adamw_elem(float p, float g, float* m, float* v, const abx_hparams* h, int fused)
{
    p = p * h->decay;
    if (fused) {
        *m = fmaf(h->beta1, *m, h->one_minus_beta1 * g);
        *v = fmaf(h->beta2, *v, h->one_minus_beta2 * (g * g));
        const float denom = fmaf(sqrtf(*v), h->inv_sqrt_bc2, h->eps);
        return fmaf(-h->step_size, *m / denom, p);
    }
    *m = h->beta1 * *m + h->one_minus_beta1 * g;
    *v = h->beta2 * *v + h->one_minus_beta2 * (g * g);
    return p - h->step_size * (*m / (sqrtf(*v) * h->inv_sqrt_bc2 + h->eps));
}

/* Lion on one element, every multiply-add fused (csrc:1107-1120).  sign(c) is 0 for 0 and NaN. */
static float lion_elem(float p, float g, float* m, const abx_hparams* h)
{
    const float c = fmaf(h->beta1, *m, h->one_minus_beta1 * g);
    const float u = c > 0.0f ? h->step_size : (c < 0.0f ? -h->step_size : 0.0f);
    *m = fmaf(h->beta2, *m, h->one_minus_beta2 * g);
    return fmaf(p, h->decay, -u);
}

/* The gradient as the update sees it: optionally multiplied by a clip / unscale
 * factor as torch's in-place multiply of a CUDA tensor by an fp32 scalar tensor
 * does it -- for a bf16 gradient, by the factor rounded to bf16, and the product
 * rounded back to bf16. */
static float grad_elem(const abx_segment* s, int64_t i, const float* g_scale)
{
    float g = load_elem(s->g, s->g_dtype, i);
    if (g_scale) {
        if (s->g_dtype == ABX_DT_BF16) {
            const float f = u2f(bf16_rne_bits(f2u(*g_scale)) & 0xffff0000U);
            g = u2f(bf16_rne_bits(f2u(g * f)) & 0xffff0000U);
        } else {
            g = g * *g_scale;
        }
    }
    return g;
}

static void adamw_dense(const abx_segment* s, const abx_hparams* h, int lanes, const float* gs)
{
    const int64_t fe = fused_end(s->n, lanes);
    const uint32_t s_m = h->seed, s_v = stream_v(h->seed), s_p = stream_p(h->seed);
    const int sr = h->stochastic;
    for (int64_t i = 0; i < s->n; ++i) {
        float m = load_elem(s->m, s->mv_dtype, i), v = load_elem(s->v, s->mv_dtype, i);
        const float pn = adamw_elem(load_master(s, i), grad_elem(s, i, gs), &m, &v, h, i < fe);
        const uint32_t idx = (uint32_t)((uint64_t)s->offset + (uint64_t)i);
        const float stored = store_master(s, i, pn, sr, s->p_dtype == ABX_DT_F24 ? abxo_hash32(idx ^ s_p) : 0u);
        store_moment(s->m, s->mv_dtype, i, m, sr, abxo_hash32(idx ^ s_m));
        store_moment(s->v, s->mv_dtype, i, v, sr, abxo_hash32(idx ^ s_v));
        store_out(s, i, stored);
    }
}

static void lion_dense(const abx_segment* s, const abx_hparams* h, const float* gs)
{
    const uint32_t s_p = stream_p(h->seed);
    const int sr = h->stochastic;
    for (int64_t i = 0; i < s->n; ++i) {
        float m = load_elem(s->m, s->mv_dtype, i);
        const float pn = lion_elem(load_master(s, i), grad_elem(s, i, gs), &m, h);
        const uint32_t idx = (uint32_t)((uint64_t)s->offset + (uint64_t)i);
        const float stored = store_master(s, i, pn, sr, s->p_dtype == ABX_DT_F24 ? abxo_hash32(idx ^ s_p) : 0u);
        store_moment(s->m, s->mv_dtype, i, m, sr, abxo_hash32(idx ^ h->seed));
        store_out(s, i, stored);
    }
}

/* Block scale: absmax / format max, or 1 for an all-zero block (csrc:1048-1049). */
static float block_scale(float amax, float fmax) { return amax > 0.0f ? amax / fmax : 1.0f; }

/* FP8 moments, one 128-element block at a time (the FP8_RANGE_BODY, csrc:1034-1059):
 * decode with the block's scales (v kept as sqrt(v)), update in fp32, new block
 * maxima over the valid elements (NaN ignored), re-encode, zero the padding. */
static void adamw_fp8(const abx_segment* s, const abx_hparams* h, int lanes, const float* gs)
{
    uint8_t* mq = (uint8_t*)s->m;
    uint8_t* vq = (uint8_t*)s->v;
    const int64_t fe = fused_end(s->n, lanes);
    const uint32_t s_m = h->seed, s_v = stream_v(h->seed), s_p = stream_p(h->seed);
    const int sr = h->stochastic;
    float mt[ABX_FP8_BLOCK], ut[ABX_FP8_BLOCK];
    for (int64_t b0 = 0; b0 < s->n; b0 += ABX_FP8_BLOCK) {
        const int64_t blk = b0 / ABX_FP8_BLOCK;
        const int nb = (int)(s->n - b0 < ABX_FP8_BLOCK ? s->n - b0 : ABX_FP8_BLOCK);
        const float sm = s->m_scale[blk], su = s->v_scale[blk];
        float am = 0.0f, au = 0.0f;
        for (int k = 0; k < nb; ++k) {
            const int64_t i = b0 + k;
            float m = dec_m(mq[i]) * sm;
            const float u0 = dec_u(vq[i]) * su;
            float v = u0 * u0;
            const float pn = adamw_elem(load_master(s, i), grad_elem(s, i, gs), &m, &v, h, i < fe);
            const uint32_t idx = (uint32_t)((uint64_t)s->offset + (uint64_t)i);
            store_out(s, i, store_master(s, i, pn, sr, s->p_dtype == ABX_DT_F24 ? abxo_hash32(idx ^ s_p) : 0u));
            const float u = sqrtf(v > 0.0f ? v : 0.0f);
            mt[k] = m;
            ut[k] = u;
            if (fabsf(m) > am) am = fabsf(m);
            if (u > au) au = u;
        }
        const float scm = block_scale(am, 448.0f), scu = block_scale(au, 57344.0f);
        for (int k = 0; k < ABX_FP8_BLOCK; ++k) {
            const int64_t i = b0 + k;
            const uint32_t idx = (uint32_t)((uint64_t)s->offset + (uint64_t)i);
            mq[i] = k < nb ? enc_m(mt[k] / scm, sr, abxo_hash32(idx ^ s_m)) : 0;
            vq[i] = k < nb ? enc_u(ut[k] / scu, sr, abxo_hash32(idx ^ s_v)) : 0;
        }
        s->m_scale[blk] = scm;
        s->v_scale[blk] = scu;
    }
}

/* Lion with an FP8 moment: same block layout and codec as AdamW's m (csrc:1246-1266). */
static void lion_fp8(const abx_segment* s, const abx_hparams* h, const float* gs)
{
    uint8_t* mq = (uint8_t*)s->m;
    const uint32_t s_p = stream_p(h->seed);
    const int sr = h->stochastic;
    float mt[ABX_FP8_BLOCK];
    for (int64_t b0 = 0; b0 < s->n; b0 += ABX_FP8_BLOCK) {
        const int64_t blk = b0 / ABX_FP8_BLOCK;
        const int nb = (int)(s->n - b0 < ABX_FP8_BLOCK ? s->n - b0 : ABX_FP8_BLOCK);
        const float sm = s->m_scale[blk];
        float am = 0.0f;
        for (int k = 0; k < nb; ++k) {
            const int64_t i = b0 + k;
            float m = dec_m(mq[i]) * sm;
            const float pn = lion_elem(load_master(s, i), grad_elem(s, i, gs), &m, h);
            const uint32_t idx = (uint32_t)((uint64_t)s->offset + (uint64_t)i);
            store_out(s, i, store_master(s, i, pn, sr, s->p_dtype == ABX_DT_F24 ? abxo_hash32(idx ^ s_p) : 0u));
            mt[k] = m;
            if (fabsf(m) > am) am = fabsf(m);
        }
        const float scm = block_scale(am, 448.0f);
        for (int k = 0; k < ABX_FP8_BLOCK; ++k) {
            const uint32_t idx = (uint32_t)((uint64_t)s->offset + (uint64_t)(b0 + k));
            mq[b0 + k] = k < nb ? enc_m(mt[k] / scm, sr, abxo_hash32(idx ^ h->seed)) : 0;
        }
        s->m_scale[blk] = scm;
    }
}

/* ---- validation (csrc:1537-1553): same checks, same order, same codes ---- */
ORACLE_API int abxo_check_segment(const abx_segment* s, int need_group)
{
    if (!s || s->n < 0) return ABX_E_ARG;
    if (s->algorithm != ABX_ALGO_ADAMW && s->algorithm != ABX_ALGO_LION) return ABX_E_ALGO;
    if (s->n == 0) return ABX_OK;
    const int lion = s->algorithm == ABX_ALGO_LION;
    if (s->p_dtype != ABX_DT_NONE && s->p_dtype != ABX_DT_F32 && s->p_dtype != ABX_DT_F24) return ABX_E_P_DTYPE;
    if (!s->p || !s->g || !s->m || (!lion && !s->v) || (s->p_dtype == ABX_DT_F24 && !s->p_lo)) return ABX_E_NULL_PTR;
    if (s->g_dtype != ABX_DT_F32 && s->g_dtype != ABX_DT_BF16) return ABX_E_G_DTYPE;
    if (s->mv_dtype != ABX_DT_F32 && s->mv_dtype != ABX_DT_BF16 && s->mv_dtype != ABX_DT_FP8) return ABX_E_MV_DTYPE;
    if (s->out_dtype != ABX_DT_NONE && s->out_dtype != ABX_DT_F32 && s->out_dtype != ABX_DT_BF16) return ABX_E_OUT_DTYPE;
    if (s->out_dtype != ABX_DT_NONE && !s->out) return ABX_E_OUT_NULL;
    if (s->mv_dtype == ABX_DT_FP8 && (!s->m_scale || (!lion && !s->v_scale))) return ABX_E_SCALE_NULL;
    if (need_group && !s->group) return ABX_E_GROUP_NULL;
    if (s->offset < 0 || (s->mv_dtype == ABX_DT_FP8 && s->offset % ABX_FP8_BLOCK)) return ABX_E_OFFSET;
    return ABX_OK;
}

static void update_segment(const abx_segment* s, const abx_hparams* h, int lanes, const float* gs)
{
    if (s->n <= 0) return;
    if (s->algorithm == ABX_ALGO_LION) {
        if (s->mv_dtype == ABX_DT_FP8) lion_fp8(s, h, gs);
        else lion_dense(s, h, gs);
    } else if (s->mv_dtype == ABX_DT_FP8) {
        adamw_fp8(s, h, lanes, gs);
    } else {
        adamw_dense(s, h, lanes, gs);
    }
}

/* Lane width of a SIMD level's vector loop (0: nothing fused). */
ORACLE_API int abxo_lanes(int level)
{
    switch (level) {
    case ABX_SIMD_AVX512: return 16;
    case ABX_SIMD_AVX2: return 8;
    case ABX_SIMD_NEON: return 4;
    default: return 0;
    }
}

/* adambridge_multi_apply (csrc:1630-1641) at SIMD level `level`; g_scale may be NULL. */
ORACLE_API int abxo_multi_apply(abx_segment* const* segs, const abx_hparams* hps, int32_t nsegs, int level,
                                const float* g_scale)
{
    if (nsegs <= 0) return ABX_OK;
    if (!segs || !hps) return ABX_E_ARG;
    for (int32_t i = 0; i < nsegs; ++i) {
        const int rc = abxo_check_segment(segs[i], 0);
        if (rc) return rc;
    }
    for (int32_t i = 0; i < nsegs; ++i) update_segment(segs[i], &hps[i], abxo_lanes(level), g_scale);
    return ABX_OK;
}

/* adambridge_multi_step (csrc:1611-1626) at SIMD level `level`; g_scale may be NULL. */
ORACLE_API int abxo_multi_step(abx_segment* const* segs, int32_t nsegs, int level, const float* g_scale)
{
    if (nsegs <= 0) return ABX_OK;
    if (!segs) return ABX_E_ARG;
    for (int32_t i = 0; i < nsegs; ++i) {
        const int rc = abxo_check_segment(segs[i], 1);
        if (rc) return rc;
    }
    for (int32_t i = 0; i < nsegs; ++i) {
        abx_hparams h;
        abxo_hparams_for(segs[i], &h);
        update_segment(segs[i], &h, abxo_lanes(level), g_scale);
    }
    return ABX_OK;
}

ORACLE_API int abxo_segment_size(void) { return (int)sizeof(abx_segment); }
