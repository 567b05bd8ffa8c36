// abx_kernels.cu -- libabx: fused AdamW / Lion optimizer updates on HBM-resident
// state for B200 (sm_100a), behind the C ABI declared in include/abx.h.
//
// Design (one pass over HBM, bandwidth-bound; no tensor cores):
//   * A launch covers up to kMaxSegs segments of one (algorithm, moment format,
//     master format) combination.  Their descriptors travel by value in the
//     kernel parameters (__grid_constant__), so a launch needs no device-side
//     table, no host->device copy and no allocation.
//   * Each segment is cut into tiles of kTile = 2048 elements; the tiles of all
//     segments form one index space that a persistent grid (one wave of resident
//     CTAs on every SM) walks with a grid stride.  A CTA finds a tile's segment by
//     a binary search over the descriptors' first-tile indices.
//   * A thread owns 8 consecutive elements of a tile: 16-byte vector loads and
//     stores for every fp32/bf16 array (two for fp32), 8-byte ones for byte
//     arrays, so each warp moves whole 512-byte (bf16) or 1 KB (fp32) lines.
//   * FP8 moments: a 128-element block is exactly 16 threads (half a warp); the
//     block maxima for the new scales are reduced with four xor-shuffles.
//
// Bit-exactness with the reference (adambridge/csrc/adambridge_kernels.c) is
// obtained by restating every operation with an explicit rounding intrinsic and
// by reproducing which elements the reference's SIMD build runs fused (see
// abx_device.cuh and fused_end below).
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/abx.h"
#include "abx_device.cuh"

#define ABX_API extern "C" __attribute__((visibility("default")))

namespace abx {

constexpr int kThreads = 256;
constexpr int kVec = 8;                  // elements per thread per tile
constexpr int kTile = kThreads * kVec;   // elements per CTA per tile
constexpr int kMaxSegs = 64;             // segments per launch (parameter block ~9.8 KB)

// Device copy of one segment with its per-step coefficients (152 bytes).
struct KSeg {
    const void* g;
    void* p;
    uint8_t* p_lo;
    void* m;
    void* v;
    float* m_scale;
    float* v_scale;
    void* out;
    int64_t n;
    int64_t fused_end;    // elements [0, fused_end) take the fused (vector-loop) arithmetic
    int64_t tile_begin;   // first tile of this segment in the launch's tile space
    Coef c;
    uint32_t s_m, s_v, s_p;   // rounding streams of m, v and the fp24 master
    uint32_t off32;           // (uint32) element offset of p[0] within its parameter
    int32_t g_dt, out_dt;
    int32_t sr;
    int32_t vec_ok;           // every buffer aligned for 16-byte (8-byte for bytes) vector access
};

template <int NSEG>
struct KArgs {
    int32_t nseg;
    int32_t pad;
    int64_t total_tiles;
    const float* g_scale;     // optional device scalar multiplying every gradient element
    KSeg seg[NSEG];
};

// ---- 8-element loads and stores -----------------------------------------------------
// Vector path when the thread's 8 elements are all valid and the segment is aligned;
// otherwise element by element (tails and unaligned callers).

__device__ __forceinline__ void ld8_f32(const float* p, int cnt, bool vec, float (&x)[8])
{
    if (vec && cnt == 8) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        const float4 b = *reinterpret_cast<const float4*>(p + 4);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = k < cnt ? p[k] : 0.0f;
    }
}

__device__ __forceinline__ void ld8_bf16(const uint16_t* p, int cnt, bool vec, float (&x)[8])
{
    if (vec && cnt == 8) {
        const uint4 a = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) { x[2 * j] = u2f(w[j] << 16); x[2 * j + 1] = u2f(w[j] & 0xffff0000U); }
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = k < cnt ? u2f((uint32_t)p[k] << 16) : 0.0f;
    }
}

// Gradient in its own dtype, read through the non-coherent path (read-only during the kernel).
__device__ __forceinline__ void ld8_grad(const void* g, int dt, int cnt, bool vec, float (&x)[8])
{
    if (dt == ABX_DT_BF16) {
        const uint16_t* p = static_cast<const uint16_t*>(g);
        if (vec && cnt == 8) {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
            const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) { x[2 * j] = u2f(w[j] << 16); x[2 * j + 1] = u2f(w[j] & 0xffff0000U); }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = k < cnt ? u2f((uint32_t)__ldg(p + k) << 16) : 0.0f;
        }
    } else {
        const float* p = static_cast<const float*>(g);
        if (vec && cnt == 8) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(p));
            const float4 b = __ldg(reinterpret_cast<const float4*>(p + 4));
            x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = k < cnt ? __ldg(p + k) : 0.0f;
        }
    }
}

__device__ __forceinline__ void st8_f32(float* p, int cnt, bool vec, const float (&x)[8])
{
    if (vec && cnt == 8) {
        *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
        *reinterpret_cast<float4*>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) if (k < cnt) p[k] = x[k];
    }
}

// Stores 8 16-bit values given in the low halves of h[].
__device__ __forceinline__ void st8_u16(uint16_t* p, int cnt, bool vec, const uint32_t (&h)[8])
{
    if (vec && cnt == 8) {
        *reinterpret_cast<uint4*>(p) = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16),
                                                  h[6] | (h[7] << 16));
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) if (k < cnt) p[k] = (uint16_t)h[k];
    }
}

__device__ __forceinline__ void ld8_u8(const uint8_t* p, int cnt, bool vec, uint32_t (&c)[8])
{
    if (vec && cnt == 8) {
        const uint2 a = *reinterpret_cast<const uint2*>(p);
#pragma unroll
        for (int k = 0; k < 4; ++k) { c[k] = (a.x >> (8 * k)) & 0xffU; c[4 + k] = (a.y >> (8 * k)) & 0xffU; }
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) c[k] = k < cnt ? p[k] : 0U;
    }
}

__device__ __forceinline__ void st8_u8(uint8_t* p, int cnt, bool vec, const uint32_t (&c)[8])
{
    if (vec && cnt == 8) {
        *reinterpret_cast<uint2*>(p) = make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24),
                                                  c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) if (k < cnt) p[k] = (uint8_t)c[k];
    }
}

// ---- master and out ---------------------------------------------------------------

template <int PT>
__device__ __forceinline__ void ld8_master(const KSeg& S, int64_t i0, int cnt, bool vec, float (&p)[8])
{
    if constexpr (PT == ABX_DT_F24) {
        float hi[8];
        uint32_t lo[8];
        ld8_bf16(static_cast<const uint16_t*>(S.p) + i0, cnt, vec, hi);
        ld8_u8(S.p_lo + i0, cnt, vec, lo);
#pragma unroll
        for (int k = 0; k < 8; ++k) p[k] = u2f(f2u(hi[k]) | (lo[k] << 8));
    } else {
        ld8_f32(static_cast<const float*>(S.p) + i0, cnt, vec, p);
    }
}

// Round (fp24) and store the new master values; p[] becomes the values stored.
template <int PT>
__device__ __forceinline__ void st8_master(const KSeg& S, int64_t i0, int cnt, bool vec, float (&p)[8])
{
    if constexpr (PT == ABX_DT_F24) {
        uint32_t hi[8], lo[8];
        const bool sr = S.sr != 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t r = sr ? hash32((S.off32 + (uint32_t)(i0 + k)) ^ S.s_p) : 0U;
            const uint32_t b = f24_bits(f2u(p[k]), sr, r);
            hi[k] = b >> 16;
            lo[k] = (b >> 8) & 0xffU;
            p[k] = u2f(b);
        }
        st8_u16(static_cast<uint16_t*>(S.p) + i0, cnt, vec, hi);
        st8_u8(S.p_lo + i0, cnt, vec, lo);
    } else {
        st8_f32(static_cast<float*>(S.p) + i0, cnt, vec, p);
    }
}

__device__ __forceinline__ void st8_out(const KSeg& S, int64_t i0, int cnt, bool vec, const float (&p)[8])
{
    if (S.out_dt == ABX_DT_BF16) {
        uint32_t h[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) h[k] = bf16_rne(f2u(p[k])) >> 16;
        st8_u16(static_cast<uint16_t*>(S.out) + i0, cnt, vec, h);
    } else if (S.out_dt == ABX_DT_F32) {
        st8_f32(static_cast<float*>(S.out) + i0, cnt, vec, p);
    }
}

// Gradient with the optional clip / unscale factor (a bf16 gradient is rounded back
// to bf16, as torch's in-place multiply of a bf16 tensor leaves it).
__device__ __forceinline__ void ld8_scaled_grad(const KSeg& S, int64_t i0, int cnt, bool vec, const float* gs,
                                                float (&g)[8])
{
    const int elem = S.g_dt == ABX_DT_BF16 ? 2 : 4;
    ld8_grad(static_cast<const char*>(S.g) + i0 * elem, S.g_dt, cnt, vec, g);
    if (gs != nullptr) {
        const float s = *gs;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            g[k] = __fmul_rn(g[k], s);
            if (S.g_dt == ABX_DT_BF16) g[k] = u2f(bf16_rne(f2u(g[k])) & 0xffff0000U);
        }
    }
}

// Moments in fp32 or bf16 (dense layouts).
template <int MV>
__device__ __forceinline__ void ld8_moment(const void* base, int64_t i0, int cnt, bool vec, float (&x)[8])
{
    if constexpr (MV == ABX_DT_BF16) ld8_bf16(static_cast<const uint16_t*>(base) + i0, cnt, vec, x);
    else ld8_f32(static_cast<const float*>(base) + i0, cnt, vec, x);
}

template <int MV>
__device__ __forceinline__ void st8_moment(void* base, int64_t i0, int cnt, bool vec, const float (&x)[8], bool sr,
                                           uint32_t seed, uint32_t idx0)
{
    if constexpr (MV == ABX_DT_BF16) {
        uint32_t h[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) h[k] = bf16_store_bits(x[k], sr, sr ? hash32((idx0 + (uint32_t)k) ^ seed) : 0U);
        st8_u16(static_cast<uint16_t*>(base) + i0, cnt, vec, h);
    } else {
        st8_f32(static_cast<float*>(base) + i0, cnt, vec, x);
    }
}

// ---- one thread's 8 elements ---------------------------------------------------------

template <int ALGO, int MV, int PT>
__device__ __forceinline__ void update8_dense(const KSeg& S, int64_t i0, const float* gs)
{
    const int64_t left = S.n - i0;
    if (left <= 0) return;
    const int cnt = left < kVec ? (int)left : kVec;
    const bool vec = S.vec_ok != 0;
    float g[8], p[8], m[8];
    ld8_scaled_grad(S, i0, cnt, vec, gs, g);
    ld8_master<PT>(S, i0, cnt, vec, p);
    ld8_moment<MV>(S.m, i0, cnt, vec, m);
    const Coef c = S.c;
    const bool sr = S.sr != 0;
    const uint32_t idx0 = S.off32 + (uint32_t)i0;
    if constexpr (ALGO == ABX_ALGO_LION) {
#pragma unroll
        for (int k = 0; k < 8; ++k) p[k] = lion_elem(p[k], g[k], m[k], c);
        st8_master<PT>(S, i0, cnt, vec, p);
        st8_moment<MV>(S.m, i0, cnt, vec, m, sr, S.s_m, idx0);
    } else {
        float v[8];
        ld8_moment<MV>(S.v, i0, cnt, vec, v);
        if (i0 + kVec <= S.fused_end) {
#pragma unroll
            for (int k = 0; k < 8; ++k) p[k] = adamw_elem<true>(p[k], g[k], m[k], v[k], c);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) p[k] = adamw_elem_sel(p[k], g[k], m[k], v[k], c, i0 + k < S.fused_end);
        }
        st8_master<PT>(S, i0, cnt, vec, p);
        st8_moment<MV>(S.m, i0, cnt, vec, m, sr, S.s_m, idx0);
        st8_moment<MV>(S.v, i0, cnt, vec, v, sr, S.s_v, idx0);
    }
    st8_out(S, i0, cnt, vec, p);
}

// Max over the 16 lanes holding one 128-element block (lanes 0-15 or 16-31 of a warp).
__device__ __forceinline__ float block_max16(float x)
{
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffU, x, o));
    return x;
}

// FP8 moments.  Called by every lane of a warp whose first element is inside the
// segment (the shuffles need the whole warp); lanes of a half-warp whose block
// starts past the end touch no memory.
template <int ALGO, int PT>
__device__ __forceinline__ void update8_fp8(const KSeg& S, int64_t i0, const float* gs)
{
    const int lane16 = threadIdx.x & 15;
    const int64_t b0 = i0 - lane16 * kVec;          // start of this half-warp's block
    const bool blk_ok = b0 < S.n;
    const int64_t left = S.n - i0;
    const int cnt = left <= 0 ? 0 : (left < kVec ? (int)left : kVec);
    const bool vec = S.vec_ok != 0;
    const int64_t blk = b0 >> 7;
    const Coef c = S.c;
    const bool sr = S.sr != 0;
    const uint32_t idx0 = S.off32 + (uint32_t)i0;

    float g[8], p[8], mt[8];
    uint32_t mc[8];
    const float sm = blk_ok ? S.m_scale[blk] : 1.0f;
    ld8_u8(static_cast<const uint8_t*>(S.m) + i0, blk_ok ? 8 : 0, vec, mc);
#pragma unroll
    for (int k = 0; k < 8; ++k) mt[k] = __fmul_rn(dec_e4m3(mc[k]), sm);
    ld8_scaled_grad(S, i0, cnt, vec, gs, g);
    ld8_master<PT>(S, i0, cnt, vec, p);

    if constexpr (ALGO == ABX_ALGO_LION) {
#pragma unroll
        for (int k = 0; k < 8; ++k) p[k] = lion_elem(p[k], g[k], mt[k], c);
        st8_master<PT>(S, i0, cnt, vec, p);
        st8_out(S, i0, cnt, vec, p);
        float am = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) { const float a = fabsf(mt[k]); am = (k < cnt && a > am) ? a : am; }
        am = block_max16(am);
        const float scm = am > 0.0f ? __fdiv_rn(am, 448.0f) : 1.0f;
        if (blk_ok) {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                mc[k] = k < cnt ? enc_e4m3(__fdiv_rn(mt[k], scm), sr, sr ? hash32((idx0 + (uint32_t)k) ^ S.s_m) : 0U) : 0U;
            st8_u8(static_cast<uint8_t*>(S.m) + i0, 8, vec, mc);
            if (lane16 == 0) S.m_scale[blk] = scm;
        }
        return;
    }

    float vt[8];
    uint32_t vc[8];
    const float su = blk_ok ? S.v_scale[blk] : 1.0f;
    ld8_u8(static_cast<const uint8_t*>(S.v) + i0, blk_ok ? 8 : 0, vec, vc);
#pragma unroll
    for (int k = 0; k < 8; ++k) { const float u = __fmul_rn(dec_e5m2(vc[k]), su); vt[k] = __fmul_rn(u, u); }
    if (i0 + kVec <= S.fused_end) {
#pragma unroll
        for (int k = 0; k < 8; ++k) p[k] = adamw_elem<true>(p[k], g[k], mt[k], vt[k], c);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) p[k] = adamw_elem_sel(p[k], g[k], mt[k], vt[k], c, i0 + k < S.fused_end);
    }
    st8_master<PT>(S, i0, cnt, vec, p);
    st8_out(S, i0, cnt, vec, p);
    float am = 0.0f, au = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float u = __fsqrt_rn(vt[k] > 0.0f ? vt[k] : 0.0f);
        vt[k] = u;
        const float a = fabsf(mt[k]);
        am = (k < cnt && a > am) ? a : am;
        au = (k < cnt && u > au) ? u : au;
    }
    am = block_max16(am);
    au = block_max16(au);
    const float scm = am > 0.0f ? __fdiv_rn(am, 448.0f) : 1.0f;
    const float scu = au > 0.0f ? __fdiv_rn(au, 57344.0f) : 1.0f;
    if (blk_ok) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t idx = idx0 + (uint32_t)k;
            mc[k] = k < cnt ? enc_e4m3(__fdiv_rn(mt[k], scm), sr, sr ? hash32(idx ^ S.s_m) : 0U) : 0U;
            vc[k] = k < cnt ? enc_e5m2(__fdiv_rn(vt[k], scu), sr, sr ? hash32(idx ^ S.s_v) : 0U) : 0U;
        }
        st8_u8(static_cast<uint8_t*>(S.m) + i0, 8, vec, mc);
        st8_u8(static_cast<uint8_t*>(S.v) + i0, 8, vec, vc);
        if (lane16 == 0) { S.m_scale[blk] = scm; S.v_scale[blk] = scu; }
    }
}

template <int NSEG>
__device__ __forceinline__ int find_segment(const KArgs<NSEG>& a, int64_t t)
{
    if (NSEG == 1) return 0;
    int lo = 0, hi = a.nseg - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.seg[mid].tile_begin <= t) lo = mid; else hi = mid - 1;
    }
    return lo;
}

template <int ALGO, int MV, int PT, int NSEG>
__global__ void __launch_bounds__(kThreads) update_kernel(const __grid_constant__ KArgs<NSEG> a)
{
    for (int64_t t = blockIdx.x; t < a.total_tiles; t += gridDim.x) {
        const KSeg& S = a.seg[find_segment(a, t)];
        const int64_t base = (t - S.tile_begin) * kTile;
        const int64_t i0 = base + threadIdx.x * kVec;
        if constexpr (MV == ABX_DT_FP8) {
            if (base + (threadIdx.x & ~31) * kVec < S.n) update8_fp8<ALGO, PT>(S, i0, a.g_scale);
        } else {
            update8_dense<ALGO, MV, PT>(S, i0, a.g_scale);
        }
    }
}

// ---- host side ---------------------------------------------------------------------------

thread_local char g_err[512] = "";
std::atomic<int> g_simd_level{ABX_SIMD_AVX512};
std::atomic<uint64_t> g_launches{0};

int set_error(const char* what, cudaError_t e)
{
    snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
    return ABX_E_CUDA;
}

int lanes_of(int level)
{
    switch (level) {
    case ABX_SIMD_AVX512: return 16;
    case ABX_SIMD_AVX2: return 8;
    case ABX_SIMD_NEON: return 4;
    default: return 0;
    }
}

// Kernel table: index = ((algo * 3) + mv_index) * 2 + f24, mv_index 0/1/2 = F32/BF16/FP8.
constexpr int kKinds = 12;
using LaunchOne = cudaError_t (*)(const KArgs<1>&, int, cudaStream_t);
using LaunchMany = cudaError_t (*)(const KArgs<kMaxSegs>&, int, cudaStream_t);

template <int A, int M, int P, int N>
cudaError_t launch(const KArgs<N>& a, int grid, cudaStream_t st)
{
    update_kernel<A, M, P, N><<<grid, kThreads, 0, st>>>(a);
    return cudaGetLastError();
}

template <int N>
const void* kernel_ptr(int kind);

#define ABX_KIND_LIST(N)                                                                                  \
    {(const void*)update_kernel<0, ABX_DT_F32, ABX_DT_F32, N>, (const void*)update_kernel<0, ABX_DT_F32, ABX_DT_F24, N>, \
     (const void*)update_kernel<0, ABX_DT_BF16, ABX_DT_F32, N>, (const void*)update_kernel<0, ABX_DT_BF16, ABX_DT_F24, N>, \
     (const void*)update_kernel<0, ABX_DT_FP8, ABX_DT_F32, N>, (const void*)update_kernel<0, ABX_DT_FP8, ABX_DT_F24, N>, \
     (const void*)update_kernel<1, ABX_DT_F32, ABX_DT_F32, N>, (const void*)update_kernel<1, ABX_DT_F32, ABX_DT_F24, N>, \
     (const void*)update_kernel<1, ABX_DT_BF16, ABX_DT_F32, N>, (const void*)update_kernel<1, ABX_DT_BF16, ABX_DT_F24, N>, \
     (const void*)update_kernel<1, ABX_DT_FP8, ABX_DT_F32, N>, (const void*)update_kernel<1, ABX_DT_FP8, ABX_DT_F24, N>}

#define ABX_LAUNCH_LIST(N)                                                                                         \
    {launch<0, ABX_DT_F32, ABX_DT_F32, N>, launch<0, ABX_DT_F32, ABX_DT_F24, N>, launch<0, ABX_DT_BF16, ABX_DT_F32, N>, \
     launch<0, ABX_DT_BF16, ABX_DT_F24, N>, launch<0, ABX_DT_FP8, ABX_DT_F32, N>, launch<0, ABX_DT_FP8, ABX_DT_F24, N>,  \
     launch<1, ABX_DT_F32, ABX_DT_F32, N>, launch<1, ABX_DT_F32, ABX_DT_F24, N>, launch<1, ABX_DT_BF16, ABX_DT_F32, N>,   \
     launch<1, ABX_DT_BF16, ABX_DT_F24, N>, launch<1, ABX_DT_FP8, ABX_DT_F32, N>, launch<1, ABX_DT_FP8, ABX_DT_F24, N>}

const void* const kKernelsOne[kKinds] = ABX_KIND_LIST(1);
const void* const kKernelsMany[kKinds] = ABX_KIND_LIST(kMaxSegs);
const LaunchOne kLaunchOne[kKinds] = ABX_LAUNCH_LIST(1);
const LaunchMany kLaunchMany[kKinds] = ABX_LAUNCH_LIST(kMaxSegs);

// Per-device launch geometry: SM count and resident CTAs per SM of each kernel.
constexpr int kMaxDevices = 64;
struct DeviceInfo {
    std::once_flag once;
    int sms = 0;
    int blocks_one[kKinds] = {};
    int blocks_many[kKinds] = {};
    cudaError_t err = cudaSuccess;
};
DeviceInfo g_dev[kMaxDevices];

DeviceInfo* device_info(int* rc)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { *rc = set_error("cudaGetDevice", e); return nullptr; }
    if (dev < 0 || dev >= kMaxDevices) { *rc = set_error("device index out of range", cudaErrorInvalidDevice); return nullptr; }
    DeviceInfo& d = g_dev[dev];
    std::call_once(d.once, [&d, dev] {
        cudaError_t err = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        for (int k = 0; k < kKinds && err == cudaSuccess; ++k) {
            err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.blocks_one[k], kKernelsOne[k], kThreads, 0);
            if (err == cudaSuccess)
                err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.blocks_many[k], kKernelsMany[k], kThreads, 0);
        }
        d.err = err;
    });
    if (d.err != cudaSuccess) { *rc = set_error("querying the device", d.err); return nullptr; }
    return &d;
}

uint32_t step_seed(uint64_t base, uint64_t index, int64_t step);

// Same checks, order and codes as the reference's check_segment (csrc:1537-1553).
int check_segment(const abx_segment* s, bool need_group)
{
    if (!s || s->n < 0) return ABX_E_ARG;
    if (s->algorithm != ABX_ALGO_ADAMW && s->algorithm != ABX_ALGO_LION) return ABX_E_ALGO;
    if (s->n == 0) return ABX_OK;
    const bool lion = s->algorithm == ABX_ALGO_LION;
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

bool aligned(const void* p, uintptr_t a) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Device accesses need natural alignment (the reference's host loads do not);
// vector access additionally needs 16-byte (8-byte for byte arrays) alignment.
int check_alignment(const abx_segment* s, bool* vec_ok)
{
    const bool lion = s->algorithm == ABX_ALGO_LION;
    const bool f24 = s->p_dtype == ABX_DT_F24;
    const uintptr_t pe = f24 ? 2 : 4, ge = s->g_dtype == ABX_DT_BF16 ? 2 : 4;
    const uintptr_t me = s->mv_dtype == ABX_DT_F32 ? 4 : (s->mv_dtype == ABX_DT_BF16 ? 2 : 1);
    const uintptr_t oe = s->out_dtype == ABX_DT_F32 ? 4 : 2;
    const void* out = s->out_dtype != ABX_DT_NONE ? s->out : nullptr;
    const void* v = lion ? nullptr : s->v;
    const bool fp8 = s->mv_dtype == ABX_DT_FP8;
    if (!aligned(s->p, pe) || !aligned(s->g, ge) || !aligned(s->m, me) || !aligned(v, me) || !aligned(out, oe) ||
        (fp8 && (!aligned(s->m_scale, 4) || (!lion && !aligned(s->v_scale, 4))))) {
        snprintf(g_err, sizeof g_err, "segment buffer not aligned to its element size");
        return ABX_E_ALIGN;
    }
    const uintptr_t mv = fp8 ? 8 : 16;
    *vec_ok = aligned(s->p, 16) && aligned(f24 ? s->p_lo : nullptr, 8) && aligned(s->g, 16) && aligned(s->m, mv) &&
              aligned(v, mv) && aligned(out, 16);
    return ABX_OK;
}

uint32_t hash32_host(uint32_t x)
{
    x = (x ^ (x >> 16)) * 0x7feb352dU;
    x = (x ^ (x >> 15)) * 0x846ca68bU;
    return x ^ (x >> 16);
}

void fill_kseg(KSeg& k, const abx_segment* s, const abx_hparams* h, int lanes, bool vec_ok, int64_t tile_begin)
{
    const bool lion = s->algorithm == ABX_ALGO_LION;
    k.g = s->g;
    k.p = s->p;
    k.p_lo = s->p_dtype == ABX_DT_F24 ? s->p_lo : nullptr;
    k.m = s->m;
    k.v = lion ? nullptr : s->v;
    k.m_scale = s->mv_dtype == ABX_DT_FP8 ? s->m_scale : nullptr;
    k.v_scale = s->mv_dtype == ABX_DT_FP8 && !lion ? s->v_scale : nullptr;
    k.out = s->out_dtype != ABX_DT_NONE ? s->out : nullptr;
    k.n = s->n;
    k.fused_end = lanes > 0 ? s->n - s->n % lanes : 0;
    k.tile_begin = tile_begin;
    k.c = Coef{h->beta1, h->beta2, h->one_minus_beta1, h->one_minus_beta2, h->decay, h->step_size, h->inv_sqrt_bc2, h->eps};
    k.s_m = h->seed;
    k.s_v = hash32_host(h->seed ^ 0xA511E9B3U);
    k.s_p = hash32_host(h->seed ^ 0x6C8E9CF5U);
    k.off32 = (uint32_t)(uint64_t)s->offset;
    k.g_dt = s->g_dtype;
    k.out_dt = s->out_dtype;
    k.sr = h->stochastic != 0;
    k.vec_ok = vec_ok ? 1 : 0;
}

int kind_of(const abx_segment* s)
{
    const int mv = s->mv_dtype == ABX_DT_F32 ? 0 : (s->mv_dtype == ABX_DT_BF16 ? 1 : 2);
    return ((s->algorithm == ABX_ALGO_LION ? 1 : 0) * 3 + mv) * 2 + (s->p_dtype == ABX_DT_F24 ? 1 : 0);
}

int64_t tiles_of(int64_t n) { return (n + kTile - 1) / kTile; }

int grid_for(int64_t tiles, int blocks_per_sm, int sms, int32_t max_ctas)
{
    int64_t grid = (int64_t)(blocks_per_sm > 0 ? blocks_per_sm : 1) * sms;
    if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
    return (int)(tiles < grid ? tiles : grid);
}

// Validate everything, then launch kind by kind in batches of up to kMaxSegs.
int run(void* stream, abx_segment* const* segs, const abx_hparams* hps, int32_t nsegs, int32_t max_ctas,
        const float* g_scale)
{
    if (nsegs <= 0) return ABX_OK;
    if (!segs) return ABX_E_ARG;
    const bool from_groups = hps == nullptr;
    std::vector<char> vec_ok(nsegs);
    for (int32_t i = 0; i < nsegs; ++i) {
        const int rc = check_segment(segs[i], from_groups);
        if (rc) return rc;
    }
    for (int32_t i = 0; i < nsegs; ++i) {
        if (segs[i]->n == 0) continue;
        bool ok = false;
        const int rc = check_alignment(segs[i], &ok);
        if (rc) return rc;
        vec_ok[i] = ok;
    }
    std::vector<abx_hparams> derived;
    if (from_groups) {
        derived.resize(nsegs);
        for (int32_t i = 0; i < nsegs; ++i)
            if (segs[i]->n > 0) abx_hparams_for(segs[i], &derived[i]);
        hps = derived.data();
    }
    int rc = ABX_OK;
    DeviceInfo* dev = device_info(&rc);
    if (!dev) return rc;
    const int lanes = lanes_of(g_simd_level.load());
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    std::vector<int32_t> order;
    order.reserve(nsegs);
    for (int kind = 0; kind < kKinds; ++kind) {
        order.clear();
        for (int32_t i = 0; i < nsegs; ++i)
            if (segs[i]->n > 0 && kind_of(segs[i]) == kind) order.push_back(i);
        for (size_t b = 0; b < order.size(); b += kMaxSegs) {
            const int cnt = (int)(order.size() - b < (size_t)kMaxSegs ? order.size() - b : kMaxSegs);
            cudaError_t e;
            if (cnt == 1) {
                KArgs<1> a;
                std::memset(&a, 0, sizeof a);
                const int32_t i = order[b];
                fill_kseg(a.seg[0], segs[i], &hps[i], lanes, vec_ok[i], 0);
                a.nseg = 1;
                a.total_tiles = tiles_of(segs[i]->n);
                a.g_scale = g_scale;
                e = kLaunchOne[kind](a, grid_for(a.total_tiles, dev->blocks_one[kind], dev->sms, max_ctas), st);
            } else {
                static thread_local KArgs<kMaxSegs> a;   // ~9.8 KB: kept off the stack
                std::memset(&a, 0, sizeof a);
                int64_t tiles = 0;
                for (int j = 0; j < cnt; ++j) {
                    const int32_t i = order[b + j];
                    fill_kseg(a.seg[j], segs[i], &hps[i], lanes, vec_ok[i], tiles);
                    tiles += tiles_of(segs[i]->n);
                }
                a.nseg = cnt;
                a.total_tiles = tiles;
                a.g_scale = g_scale;
                e = kLaunchMany[kind](a, grid_for(tiles, dev->blocks_many[kind], dev->sms, max_ctas), st);
            }
            if (e != cudaSuccess) return set_error("kernel launch", e);
            g_launches.fetch_add(1, std::memory_order_relaxed);
        }
    }
    return ABX_OK;
}

// splitmix64-style mixing of (base seed, parameter index, step) (csrc:773-790).
uint64_t mix_round(uint64_t h, uint64_t v)
{
    h = (h ^ v) * 0xBF58476D1CE4E5B9ULL;
    h = (h ^ (h >> 31)) * 0x94D049BB133111EBULL;
    return h ^ (h >> 29);
}

uint32_t step_seed(uint64_t base, uint64_t index, int64_t step)
{
    uint64_t h = 0x9E3779B97F4A7C15ULL;
    h = mix_round(h, base);
    h = mix_round(h, index);
    h = mix_round(h, (uint64_t)step);
    return (uint32_t)h;
}

}  // namespace abx

// ---- C ABI ---------------------------------------------------------------------------------

ABX_API int abx_abi_version(void) { return ABX_ABI_VERSION; }
ABX_API int abx_hparams_size(void) { return (int)sizeof(abx_hparams); }
ABX_API int abx_group_size(void) { return (int)sizeof(abx_group); }
ABX_API int abx_segment_size(void) { return (int)sizeof(abx_segment); }

ABX_API int abx_set_simd_level(int level)
{
    if (level < 0) level = ABX_SIMD_AVX512;
    if (level > ABX_SIMD_NEON) return ABX_E_SIMD_LEVEL;
    abx::g_simd_level.store(level);
    return level;
}

ABX_API int abx_simd_level(void) { return abx::g_simd_level.load(); }
ABX_API int abx_detected_simd_level(void) { return ABX_SIMD_AVX512; }

ABX_API uint32_t abx_step_seed(uint64_t base_seed, uint64_t index, int64_t step)
{
    return abx::step_seed(base_seed, index, step);
}

// Per-step coefficients in double, narrowed to float (csrc:793-809).
ABX_API int abx_hparams_for(const abx_segment* s, abx_hparams* h)
{
    if (!s || !h || !s->group) return ABX_E_ARG;
    const abx_group* G = s->group;
    const double t = (double)s->step;
    const double bc1 = 1.0 - std::pow(G->beta1, t);
    const double bc2 = 1.0 - std::pow(G->beta2, t);
    h->beta1 = (float)G->beta1;
    h->beta2 = (float)G->beta2;
    h->one_minus_beta1 = (float)(1.0 - G->beta1);
    h->one_minus_beta2 = (float)(1.0 - G->beta2);
    h->decay = (float)(1.0 - G->lr * G->weight_decay);
    h->step_size = (float)(s->algorithm == ABX_ALGO_LION ? G->lr : G->lr / bc1);
    h->inv_sqrt_bc2 = (float)(1.0 / std::sqrt(bc2));
    h->eps = (float)G->eps;
    h->seed = abx::step_seed(G->seed, s->index, s->step);
    h->stochastic = G->stochastic;
    return ABX_OK;
}

ABX_API int abx_multi_step(void* stream, abx_segment* const* segs, int32_t nsegs, int32_t max_ctas)
{
    return abx::run(stream, segs, nullptr, nsegs, max_ctas, nullptr);
}

ABX_API int abx_multi_apply(void* stream, abx_segment* const* segs, const abx_hparams* hps, int32_t nsegs,
                            int32_t max_ctas)
{
    if (nsegs > 0 && (!segs || !hps)) return ABX_E_ARG;
    return abx::run(stream, segs, hps, nsegs, max_ctas, nullptr);
}

ABX_API int abx_multi_step_scaled(void* stream, abx_segment* const* segs, int32_t nsegs, int32_t max_ctas,
                                  const float* g_scale)
{
    return abx::run(stream, segs, nullptr, nsegs, max_ctas, g_scale);
}

ABX_API int abx_multi_apply_scaled(void* stream, abx_segment* const* segs, const abx_hparams* hps, int32_t nsegs,
                                   int32_t max_ctas, const float* g_scale)
{
    if (nsegs > 0 && (!segs || !hps)) return ABX_E_ARG;
    return abx::run(stream, segs, hps, nsegs, max_ctas, g_scale);
}

// Argument checks and codes of adambridge_fused_adamw (csrc:1518-1535).
ABX_API int abx_fused_adamw(float* p, const void* g, int g_dtype, void* m, void* v, int mv_dtype, void* out,
                            int out_dtype, int64_t n, uint64_t offset, const abx_hparams* hp, void* stream)
{
    if (n < 0 || !hp) return ABX_E_ARG;
    if (n == 0) return ABX_OK;
    if (!p || !g || !m || !v) return ABX_E_NULL_PTR;
    if (g_dtype != ABX_DT_F32 && g_dtype != ABX_DT_BF16) return ABX_E_G_DTYPE;
    if (mv_dtype != ABX_DT_F32 && mv_dtype != ABX_DT_BF16) return ABX_E_MV_DTYPE;
    if (out_dtype != ABX_DT_NONE && out_dtype != ABX_DT_F32 && out_dtype != ABX_DT_BF16) return ABX_E_OUT_DTYPE;
    if (out_dtype != ABX_DT_NONE && !out) return ABX_E_OUT_NULL;
    abx_segment s;
    std::memset(&s, 0, sizeof s);
    s.p = p;
    s.g = g;
    s.m = m;
    s.v = v;
    s.out = out_dtype == ABX_DT_NONE ? nullptr : out;
    s.n = n;
    s.offset = (int64_t)offset;
    s.g_dtype = g_dtype;
    s.mv_dtype = mv_dtype;
    s.out_dtype = out_dtype;
    s.algorithm = ABX_ALGO_ADAMW;
    s.p_dtype = ABX_DT_F32;
    abx_segment* ps = &s;
    return abx::run(stream, &ps, hp, 1, 0, nullptr);
}

ABX_API uint64_t abx_launch_count(void) { return abx::g_launches.load(); }

ABX_API const char* abx_last_error(void) { return abx::g_err; }
