// abx_kernels.cu -- libabx: fused AdamW / Lion optimizer updates on HBM-resident
// state for B200 (sm_100a), behind the C ABI declared in include/abx.h.
//
// Design (one pass over HBM, bandwidth-bound; no tensor cores):
//   * A launch covers up to kMaxSegs segments of one (algorithm, moment format,
//     master format, gradient format) combination.  Their descriptors travel by
//     value in the kernel parameters (__grid_constant__): no device-side table,
//     no host->device copy, no allocation.
//   * Each segment is cut into tiles of kTile = 2048 elements; the tiles of all
//     segments form one index space that a persistent grid walks with a grid
//     stride.  A CTA finds a tile's segment by a binary search over the
//     descriptors' first-tile indices.
//   * Inside a CTA, one producer warp streams whole tiles of every input array
//     (master, gradient, moments) into a ring of shared-memory stages with 1-D
//     TMA bulk copies (cp.async.bulk ... mbarrier::complete_tx), so the bytes in
//     flight per SM are set by the ring, not by registers or occupancy.  Eight
//     consumer warps compute from shared memory and store results straight to
//     HBM with vector stores.  Tiles that cannot be bulk-copied (the partial last
//     tile of a segment, unaligned buffers) are read directly from HBM.
//   * A consumer thread owns two groups of 4 consecutive elements per tile
//     (elements 4t..4t+3 and 1024+4t..), so every shared-memory read and every
//     global store of a warp covers one contiguous span without bank conflicts.
//     With FP8 moments one 128-element block is exactly one warp's group; the
//     block maxima for the new scales are reduced with xor-shuffles.
//   * Every mbarrier wait is bounded: a wait that gives up sets a status word in
//     mapped host memory (abx_status_word / abx_pipeline_status, readable by the
//     host without a device synchronization) and the CTA drains its copies and exits.
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

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;   // + one producer warp
constexpr int kGroup = 4;                              // elements per thread per half tile
constexpr int kHalf = kConsumerWarps * 32 * kGroup;    // 1024
constexpr int kTile = 2 * kHalf;                       // 2048 elements per tile
constexpr int kMaxSegs = 64;                           // segments per launch (parameter block ~10 KB)
constexpr int kMinCtasPerSm = 4;                       // residency the register budget is set for (<= 56 regs)
constexpr int kSmemTarget = 52 * 1024;                 // ring bytes per CTA (four CTAs per SM)
constexpr uint32_t kSpinLimit = 1u << 22;              // mbarrier polls before a wait gives up (default)
constexpr int kMaxReplicas = 7;                        // out replicas per segment (peers of an 8-GPU node)

// Bits of the status word a CTA sets (OR) when one of its pipeline waits gives up; never set in correct
// operation.  The word lives in mapped, pinned host memory, so the host reads it without synchronizing.
constexpr unsigned int kStatusConsumerWait = 1u;   // a consumer warp's wait for a staged tile
constexpr unsigned int kStatusProducerWait = 2u;   // the producer's wait for a free ring slot
constexpr unsigned int kStatusDrainWait = 4u;      // the producer's wait for its last copies before it exits

// Device copy of one segment with its per-step coefficients.
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
    int32_t out_dt;
    int32_t sr;
    int32_t vec_ok;           // 4-element vector access is aligned in every buffer (direct path)
    int32_t tma_ok;           // every streamed buffer is 16-byte aligned (bulk-copy path)
    int32_t nrep;             // replicas of out: each out element is also stored at out + rep_delta[j] bytes
    int32_t pad;
    int64_t rep_delta[kMaxReplicas];
};

template <int NSEG>
struct KArgs {
    int32_t nseg;
    int32_t stages;
    int64_t total_tiles;
    const float* g_scale;     // optional device scalar multiplying every gradient element
    unsigned int* status;     // the status word (mapped host memory)
    uint32_t spin_limit;      // mbarrier polls before a wait gives up
    int32_t pad0;
    int64_t skip_tile;        // failure-path test only (abx_test_pipeline_fault): the producer leaves this tile's
                              // stage untouched -- no copy, no arrival -- so its consumers' wait runs out; else -1
    KSeg seg[NSEG];
};

// Shared-memory layout of one pipeline stage for a kernel kind (every array a whole tile).
template <int ALGO, int MV, int PT, int GT>
struct Cfg {
    static constexpr int PB = PT == ABX_DT_F24 ? 2 : 4;
    static constexpr int LB = PT == ABX_DT_F24 ? 1 : 0;
    static constexpr int GB = GT == ABX_DT_BF16 ? 2 : 4;
    static constexpr int MB = MV == ABX_DT_F32 ? 4 : (MV == ABX_DT_BF16 ? 2 : 1);
    static constexpr int VB = ALGO == ABX_ALGO_LION ? 0 : MB;
    static constexpr int OFF_P = 0;
    static constexpr int OFF_L = OFF_P + kTile * PB;
    static constexpr int OFF_G = OFF_L + kTile * LB;
    static constexpr int OFF_M = OFF_G + kTile * GB;
    static constexpr int OFF_V = OFF_M + kTile * MB;
    static constexpr int ARR = OFF_V + kTile * VB;         // bytes of the element arrays
    static constexpr bool FP8 = MV == ABX_DT_FP8;
    // FP8: the tile's 16 block scales of m (and v), bulk-copied as the 16-byte-aligned window that holds
    // them (64 or 80 bytes) into a 128-byte slot; consumers index it from the window's start.
    static constexpr int OFF_SM = ARR;
    static constexpr int OFF_SV = ARR + 128;
    static constexpr int STAGE = ARR + (FP8 ? (VB > 0 ? 256 : 128) : 0);
};

// Per-stage description of the tile, written by the producer before it arrives on the stage's
// full barrier (so consumers see it after their wait): which segment, where, whether staged.
struct TileMeta {
    int32_t seg;
    int32_t staged;
    int64_t base;
};

// What consumers read per stage from shared memory: the tile's metadata and a copy of its segment's
// descriptor (so the per-tile field reads are shared-memory broadcasts, not dependent parameter loads).
struct __align__(16) StageHdr {
    TileMeta meta;
    KSeg seg;
};
constexpr int kHdrBytes = (int)sizeof(StageHdr);

// ---- PTX: mbarriers and 1-D TMA bulk copies -----------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Wait for the phase of `bar` with parity `parity`, at most `limit` polls; false (and `what` set in the
// status word) if it never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit, unsigned int* status,
                                          unsigned int what)
{
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicOr_system(status, what);
    return false;
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}

// ---- 4-element loads and stores -----------------------------------------------------
// Source: the staged tile in shared memory (s != nullptr: always 4 valid, aligned
// elements), else global memory -- one vector when the thread's 4 elements are valid
// and the segment is aligned, element by element otherwise.

__device__ __forceinline__ void ld4_f32(const float* g, const float* s, int cnt, bool vec, float (&x)[4])
{
    if (s != nullptr) {
        const float4 a = *reinterpret_cast<const float4*>(s);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    } else if (vec && cnt == 4) {
        const float4 a = *reinterpret_cast<const float4*>(g);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = k < cnt ? g[k] : 0.0f;
    }
}

// 4 bf16 values as two packed words (element 2j in the low half of w[j]).
__device__ __forceinline__ void ld4_b16(const uint16_t* g, const uint16_t* s, int cnt, bool vec, uint32_t (&w)[2])
{
    if (s != nullptr) {
        const uint2 a = *reinterpret_cast<const uint2*>(s);
        w[0] = a.x; w[1] = a.y;
    } else if (vec && cnt == 4) {
        const uint2 a = *reinterpret_cast<const uint2*>(g);
        w[0] = a.x; w[1] = a.y;
    } else {
        uint32_t h[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = k < cnt ? g[k] : 0U;
        w[0] = h[0] | (h[1] << 16);
        w[1] = h[2] | (h[3] << 16);
    }
}

__device__ __forceinline__ uint32_t ld4_b8(const uint8_t* g, const uint8_t* s, int cnt, bool vec)
{
    if (s != nullptr) return *reinterpret_cast<const uint32_t*>(s);
    if (vec && cnt == 4) return *reinterpret_cast<const uint32_t*>(g);
    uint32_t w = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) w |= (k < cnt ? (uint32_t)g[k] : 0U) << (8 * k);
    return w;
}

__device__ __forceinline__ void st4_f32(float* g, int cnt, bool vec, const float (&x)[4])
{
    if (vec && cnt == 4) {
        *reinterpret_cast<float4*>(g) = make_float4(x[0], x[1], x[2], x[3]);
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) if (k < cnt) g[k] = x[k];
    }
}

__device__ __forceinline__ void st4_b16(uint16_t* g, int cnt, bool vec, uint32_t w0, uint32_t w1)
{
    if (vec && cnt == 4) {
        *reinterpret_cast<uint2*>(g) = make_uint2(w0, w1);
    } else {
        const uint32_t h[4] = {w0 & 0xffffU, w0 >> 16, w1 & 0xffffU, w1 >> 16};
#pragma unroll
        for (int k = 0; k < 4; ++k) if (k < cnt) g[k] = (uint16_t)h[k];
    }
}

__device__ __forceinline__ void st4_b8(uint8_t* g, int cnt, bool vec, uint32_t w)
{
    if (vec && cnt == 4) {
        *reinterpret_cast<uint32_t*>(g) = w;
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) if (k < cnt) g[k] = (uint8_t)(w >> (8 * k));
    }
}

__device__ __forceinline__ void unpack_b16(const uint32_t (&w)[2], float (&x)[4])
{
    x[0] = u2f(w[0] << 16); x[1] = u2f(w[0] & 0xffff0000U);
    x[2] = u2f(w[1] << 16); x[3] = u2f(w[1] & 0xffff0000U);
}

// ---- typed element groups ------------------------------------------------------------

// Gradient with the optional clip / unscale factor (a bf16 gradient is rounded back to bf16,
// as torch's in-place multiply of a bf16 tensor leaves it).
template <int GT>
__device__ __forceinline__ void grad4(const KSeg& S, int64_t i0, int cnt, const uint8_t* s, const float* gs,
                                      float (&g)[4])
{
    if constexpr (GT == ABX_DT_BF16) {
        uint32_t w[2];
        ld4_b16(static_cast<const uint16_t*>(S.g) + i0, reinterpret_cast<const uint16_t*>(s), cnt, S.vec_ok, w);
        unpack_b16(w, g);
    } else {
        ld4_f32(static_cast<const float*>(S.g) + i0, reinterpret_cast<const float*>(s), cnt, S.vec_ok, g);
    }
    if (gs != nullptr) {
        // a bf16 gradient is scaled as torch scales a bf16 CUDA tensor in place by an fp32 scalar tensor:
        // by the scalar rounded to bf16, the product rounded back to bf16
        const float f = GT == ABX_DT_BF16 ? u2f(bf16_rne(f2u(*gs)) & 0xffff0000U) : *gs;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            g[k] = __fmul_rn(g[k], f);
            if constexpr (GT == ABX_DT_BF16) g[k] = u2f(bf16_rne(f2u(g[k])) & 0xffff0000U);
        }
    }
}

template <int PT>
__device__ __forceinline__ void master4(const KSeg& S, int64_t i0, int cnt, const uint8_t* sp, const uint8_t* sl,
                                        float (&p)[4])
{
    if constexpr (PT == ABX_DT_F24) {
        uint32_t w[2];
        ld4_b16(static_cast<const uint16_t*>(S.p) + i0, reinterpret_cast<const uint16_t*>(sp), cnt, S.vec_ok, w);
        const uint32_t lo = ld4_b8(S.p_lo + i0, sl, cnt, S.vec_ok);
        p[0] = u2f((w[0] << 16) | ((lo & 0xffU) << 8));
        p[1] = u2f((w[0] & 0xffff0000U) | (lo & 0xff00U));
        p[2] = u2f((w[1] << 16) | ((lo >> 8) & 0xff00U));
        p[3] = u2f((w[1] & 0xffff0000U) | ((lo >> 16) & 0xff00U));
    } else {
        ld4_f32(static_cast<const float*>(S.p) + i0, reinterpret_cast<const float*>(sp), cnt, S.vec_ok, p);
    }
}

// Round (fp24) and store the new master values; p[] becomes the values stored.
template <int PT, bool SR>
__device__ __forceinline__ void store_master4(const KSeg& S, int64_t i0, int cnt, float (&p)[4])
{
    if constexpr (PT == ABX_DT_F24) {
        uint32_t b[4], r[4] = {0U, 0U, 0U, 0U};
        if (SR) hash4(S.off32 + (uint32_t)i0, S.s_p, r);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            b[k] = f24_bits(f2u(p[k]), SR, r[k]);
            p[k] = u2f(b[k]);
        }
        // lo plane: byte 1 of each word, packed in element order
        const uint32_t lo = __byte_perm(__byte_perm(b[0], b[1], 0x0051), __byte_perm(b[2], b[3], 0x0051), 0x5410);
        st4_b16(static_cast<uint16_t*>(S.p) + i0, cnt, S.vec_ok, pack_hi16(b[0], b[1]), pack_hi16(b[2], b[3]));
        st4_b8(S.p_lo + i0, cnt, S.vec_ok, lo);
    } else {
        st4_f32(static_cast<float*>(S.p) + i0, cnt, S.vec_ok, p);
    }
}

// The new weights, into out and into each replica of out (peers' copies of the weights, written over
// NVLink with plain stores: the fused all-gather of a sharded update).
__device__ __forceinline__ void store_out4(const KSeg& S, int64_t i0, int cnt, const float (&p)[4])
{
    if (S.out_dt == ABX_DT_BF16) {
        const uint32_t w0 = pack_bf16_rne(p[0], p[1]), w1 = pack_bf16_rne(p[2], p[3]);
        uint16_t* o = static_cast<uint16_t*>(S.out) + i0;
        st4_b16(o, cnt, S.vec_ok, w0, w1);
        for (int j = 0; j < S.nrep; ++j)
            st4_b16(reinterpret_cast<uint16_t*>(reinterpret_cast<char*>(o) + S.rep_delta[j]), cnt, S.vec_ok, w0, w1);
    } else if (S.out_dt == ABX_DT_F32) {
        float* o = static_cast<float*>(S.out) + i0;
        st4_f32(o, cnt, S.vec_ok, p);
        for (int j = 0; j < S.nrep; ++j)
            st4_f32(reinterpret_cast<float*>(reinterpret_cast<char*>(o) + S.rep_delta[j]), cnt, S.vec_ok, p);
    }
}

template <int MV>
__device__ __forceinline__ void moment4(const void* base, int64_t i0, int cnt, bool vec, const uint8_t* s,
                                        float (&x)[4])
{
    if constexpr (MV == ABX_DT_BF16) {
        uint32_t w[2];
        ld4_b16(static_cast<const uint16_t*>(base) + i0, reinterpret_cast<const uint16_t*>(s), cnt, vec, w);
        unpack_b16(w, x);
    } else {
        ld4_f32(static_cast<const float*>(base) + i0, reinterpret_cast<const float*>(s), cnt, vec, x);
    }
}

// A bf16 moment: stochastic -- 16 random bits added below the kept half, then truncated -- or nearest-even.
template <int MV, bool SR>
__device__ __forceinline__ void store_moment4(void* base, int64_t i0, int cnt, bool vec, const float (&x)[4],
                                              uint32_t seed, uint32_t idx0)
{
    if constexpr (MV == ABX_DT_BF16) {
        uint32_t w0, w1;
        if constexpr (SR) {
            uint32_t b[4], r[4];
            hash4(idx0, seed, r);
#pragma unroll
            for (int k = 0; k < 4; ++k) b[k] = f2u(x[k]) + (r[k] & 0xffffU);
            w0 = pack_hi16(b[0], b[1]);
            w1 = pack_hi16(b[2], b[3]);
        } else {
            w0 = pack_bf16_rne(x[0], x[1]);
            w1 = pack_bf16_rne(x[2], x[3]);
        }
        st4_b16(static_cast<uint16_t*>(base) + i0, cnt, vec, w0, w1);
    } else {
        st4_f32(static_cast<float*>(base) + i0, cnt, vec, x);
    }
}

// ---- one tile ------------------------------------------------------------------------------

// FP32 / BF16 moments: each consumer thread updates its two groups of 4 elements.
template <int ALGO, int MV, int PT, int GT, bool SR>
__device__ __forceinline__ void tile_dense(const KSeg& S, int64_t base, const uint8_t* st, const float* gs)
{
    using C = Cfg<ALGO, MV, PT, GT>;
    const Coef c = S.c;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int e0 = h * kHalf + threadIdx.x * kGroup;
        const int64_t i0 = base + e0;
        const int64_t left = S.n - i0;
        if (left <= 0) continue;
        const int cnt = left < kGroup ? (int)left : kGroup;
        const uint32_t idx0 = S.off32 + (uint32_t)i0;
        float g[4], p[4], m[4];
        grad4<GT>(S, i0, cnt, st ? st + C::OFF_G + e0 * C::GB : nullptr, gs, g);
        master4<PT>(S, i0, cnt, st ? st + C::OFF_P + e0 * C::PB : nullptr, st ? st + C::OFF_L + e0 : nullptr, p);
        moment4<MV>(S.m, i0, cnt, S.vec_ok, st ? st + C::OFF_M + e0 * C::MB : nullptr, m);
        if constexpr (ALGO == ABX_ALGO_LION) {
#pragma unroll
            for (int k = 0; k < 4; ++k) p[k] = lion_elem(p[k], g[k], m[k], c);
            store_master4<PT, SR>(S, i0, cnt, p);
            store_moment4<MV, SR>(S.m, i0, cnt, S.vec_ok, m, S.s_m, idx0);
        } else {
            float v[4];
            moment4<MV>(S.v, i0, cnt, S.vec_ok, st ? st + C::OFF_V + e0 * C::MB : nullptr, v);
            if (i0 + kGroup <= S.fused_end) {
#pragma unroll
                for (int k = 0; k < 4; ++k) p[k] = adamw_elem<true>(p[k], g[k], m[k], v[k], c);
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) p[k] = adamw_elem_sel(p[k], g[k], m[k], v[k], c, i0 + k < S.fused_end);
            }
            store_master4<PT, SR>(S, i0, cnt, p);
            store_moment4<MV, SR>(S.m, i0, cnt, S.vec_ok, m, S.s_m, idx0);
            store_moment4<MV, SR>(S.v, i0, cnt, S.vec_ok, v, S.s_v, idx0);
        }
        store_out4(S, i0, cnt, p);
    }
}

__device__ __forceinline__ float warp_max(float x)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffU, x, o));
    return x;
}

// FP8 moments: in each half tile, warp w owns block w (128 elements, 4 per lane).  Called by whole
// warps; a warp whose block starts past the end of the segment skips it (the test is warp-uniform).
// Codes of 4 elements x[k] / s (zero for elements past the end, k >= cnt: the block padding), with the
// random bits of stream `seed`.  s is the block's scale (warp-uniform, so the branch is too).
template <bool E4M3, bool SR>
__device__ __forceinline__ uint32_t encode4(const float (&x)[4], float s, int cnt, uint32_t idx0, uint32_t seed)
{
    float q[4];
    if (__builtin_expect(fast_scale(s), 1)) {
        const float y = __frcp_rn(s);
#pragma unroll
        for (int k = 0; k < 4; ++k) q[k] = div_by_scale(x[k], s, y);
    } else {
        const float4 d = div4_ieee(make_float4(x[0], x[1], x[2], x[3]), s);
        q[0] = d.x; q[1] = d.y; q[2] = d.z; q[3] = d.w;
    }
    uint32_t r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) r[k] = SR ? hash32((idx0 + (uint32_t)k) ^ seed) : 0U;
    const uint32_t w = enc4_fp8<E4M3, SR>(q, r);
    return cnt >= 4 ? w : (cnt <= 0 ? 0U : w & (0xffffffffU >> (8 * (4 - cnt))));
}

template <int ALGO, int PT, int GT, bool SR>
__device__ __forceinline__ void tile_fp8(const KSeg& S, int64_t base, const uint8_t* st, const float* gs)
{
    using C = Cfg<ALGO, ABX_DT_FP8, PT, GT>;
    const Coef c = S.c;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int e0 = h * kHalf + threadIdx.x * kGroup;
        const int64_t i0 = base + e0;
        const int64_t b0 = i0 - lane * kGroup;      // start of this warp's block
        if (b0 >= S.n) continue;
        const int64_t blk = b0 >> 7;
        const int64_t left = S.n - i0;
        const int cnt = left <= 0 ? 0 : (left < kGroup ? (int)left : kGroup);
        const uint32_t idx0 = S.off32 + (uint32_t)i0;
        // the codes of the whole block exist (the buffer is padded to whole blocks): always 4 here
        const uint32_t mc = ld4_b8(static_cast<const uint8_t*>(S.m) + i0, st ? st + C::OFF_M + e0 : nullptr, 4, S.vec_ok);
        const float sm = S.m_scale[blk];
        float g[4], p[4], mt[4];
#pragma unroll
        dec4_fp8<true>(mc, mt);
#pragma unroll
        for (int k = 0; k < 4; ++k) mt[k] = __fmul_rn(mt[k], sm);
        grad4<GT>(S, i0, cnt, st ? st + C::OFF_G + e0 * C::GB : nullptr, gs, g);
        master4<PT>(S, i0, cnt, st ? st + C::OFF_P + e0 * C::PB : nullptr, st ? st + C::OFF_L + e0 : nullptr, p);
        if constexpr (ALGO == ABX_ALGO_LION) {
#pragma unroll
            for (int k = 0; k < 4; ++k) p[k] = lion_elem(p[k], g[k], mt[k], c);
            store_master4<PT, SR>(S, i0, cnt, p);
            store_out4(S, i0, cnt, p);
            float am = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) { const float a = fabsf(mt[k]); am = (k < cnt && a > am) ? a : am; }
            am = warp_max(am);
            const float scm = am > 0.0f ? __fdiv_rn(am, 448.0f) : 1.0f;
            st4_b8(static_cast<uint8_t*>(S.m) + i0, 4, S.vec_ok, encode4<true, SR>(mt, scm, cnt, idx0, S.s_m));
            if (lane == 0) S.m_scale[blk] = scm;
        } else {
            const uint32_t vc = ld4_b8(static_cast<const uint8_t*>(S.v) + i0, st ? st + C::OFF_V + e0 : nullptr, 4, S.vec_ok);
            const float su = S.v_scale[blk];
            float vt[4], ut[4];
            dec4_fp8<false>(vc, vt);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float u = __fmul_rn(vt[k], su);
                vt[k] = __fmul_rn(u, u);
            }
            if (i0 + kGroup <= S.fused_end) {
#pragma unroll
                for (int k = 0; k < 4; ++k) p[k] = adamw_elem_sq<true>(p[k], g[k], mt[k], vt[k], ut[k], c);
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    p[k] = i0 + k < S.fused_end ? adamw_elem_sq<true>(p[k], g[k], mt[k], vt[k], ut[k], c)
                                                : adamw_elem_sq<false>(p[k], g[k], mt[k], vt[k], ut[k], c);
            }
            store_master4<PT, SR>(S, i0, cnt, p);
            store_out4(S, i0, cnt, p);
            float am = 0.0f, au = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                ut[k] = vt[k] > 0.0f ? ut[k] : 0.0f;    // sqrt(max(v, 0)); NaN -> 0
                const float a = fabsf(mt[k]);
                am = (k < cnt && a > am) ? a : am;
                au = (k < cnt && ut[k] > au) ? ut[k] : au;
            }
            am = warp_max(am);
            au = warp_max(au);
            const float scm = am > 0.0f ? __fdiv_rn(am, 448.0f) : 1.0f;
            const float scu = au > 0.0f ? __fdiv_rn(au, 57344.0f) : 1.0f;
            st4_b8(static_cast<uint8_t*>(S.m) + i0, 4, S.vec_ok, encode4<true, SR>(mt, scm, cnt, idx0, S.s_m));
            st4_b8(static_cast<uint8_t*>(S.v) + i0, 4, S.vec_ok, encode4<false, SR>(ut, scu, cnt, idx0, S.s_v));
            if (lane == 0) { S.m_scale[blk] = scm; S.v_scale[blk] = scu; }
        }
    }
}

template <int ALGO, int MV, int PT, int GT, bool SR>
__device__ __forceinline__ void tile(const KSeg& S, int64_t base, const uint8_t* st, const float* gs)
{
    if constexpr (MV == ABX_DT_FP8) tile_fp8<ALGO, PT, GT, SR>(S, base, st, gs);
    else tile_dense<ALGO, MV, PT, GT, SR>(S, base, st, gs);
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

// Dynamic shared memory: S full + S empty barriers, S stage headers, then the 128-byte-aligned ring.
__host__ __device__ constexpr int ring_offset(int stages)
{
    return 128 * ((16 * ((16 * stages + 15) / 16) + stages * kHdrBytes + 127) / 128);
}

// A tile streams through shared memory when it is whole and every streamed buffer is 16-byte aligned.
__device__ __forceinline__ bool staged_tile(const KSeg& S, int64_t base) { return S.tma_ok && base + kTile <= S.n; }

// ---- fast path: a whole tile staged in shared memory ------------------------------------

// Fast-path stores.  In a staged tile every store address is aligned for its vector (the segment
// passed the bulk-copy alignment check, which includes the 4-element alignment of out, and peers'
// copies of out sit at the same offsets of identically aligned buffers).  They are st.global
// statements: the compiler then knows that they cannot write the shared-memory tile header, so it
// keeps the header's fields in registers instead of reloading them after every store.  The fence at
// the kernel's end is an asm statement too, so it stays after them.
__device__ __forceinline__ size_t gaddr(const void* p) { return __cvta_generic_to_global(p); }

__device__ __forceinline__ void stg_f32x4(void* p, float a, float b, float c, float d)
{
    asm volatile("st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(gaddr(p)), "f"(a), "f"(b), "f"(c), "f"(d));
}

__device__ __forceinline__ void stg_b32x2(void* p, uint32_t a, uint32_t b)
{
    asm volatile("st.global.v2.b32 [%0], {%1, %2};" ::"l"(gaddr(p)), "r"(a), "r"(b));
}

__device__ __forceinline__ void stg_b32(void* p, uint32_t a)
{
    asm volatile("st.global.b32 [%0], %1;" ::"l"(gaddr(p)), "r"(a));
}

template <int PT, bool SR>
__device__ __forceinline__ void fast_store_master4(const KSeg& S, int64_t i0, float (&p)[4])
{
    if constexpr (PT == ABX_DT_F24) {
        uint32_t b[4], r[4] = {0U, 0U, 0U, 0U};
        if (SR) hash4(S.off32 + (uint32_t)i0, S.s_p, r);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            b[k] = f24_bits(f2u(p[k]), SR, r[k]);
            p[k] = u2f(b[k]);
        }
        const uint32_t lo = __byte_perm(__byte_perm(b[0], b[1], 0x0051), __byte_perm(b[2], b[3], 0x0051), 0x5410);
        stg_b32x2(static_cast<uint16_t*>(S.p) + i0, pack_hi16(b[0], b[1]), pack_hi16(b[2], b[3]));
        stg_b32(S.p_lo + i0, lo);
    } else {
        stg_f32x4(static_cast<float*>(S.p) + i0, p[0], p[1], p[2], p[3]);
    }
}

__device__ __forceinline__ void fast_store_out4(const KSeg& S, int64_t i0, const float (&p)[4])
{
    if (S.out_dt == ABX_DT_BF16) {
        const uint32_t w0 = pack_bf16_rne(p[0], p[1]), w1 = pack_bf16_rne(p[2], p[3]);
        char* o = reinterpret_cast<char*>(static_cast<uint16_t*>(S.out) + i0);
        stg_b32x2(o, w0, w1);
        for (int j = 0; j < S.nrep; ++j) stg_b32x2(o + S.rep_delta[j], w0, w1);
    } else if (S.out_dt == ABX_DT_F32) {
        char* o = reinterpret_cast<char*>(static_cast<float*>(S.out) + i0);
        stg_f32x4(o, p[0], p[1], p[2], p[3]);
        for (int j = 0; j < S.nrep; ++j) stg_f32x4(o + S.rep_delta[j], p[0], p[1], p[2], p[3]);
    }
}

template <int MV, bool SR>
__device__ __forceinline__ void fast_store_moment4(void* base, int64_t i0, const float (&x)[4], uint32_t seed,
                                                   uint32_t idx0)
{
    if constexpr (MV == ABX_DT_BF16) {
        uint32_t w0, w1;
        if constexpr (SR) {
            uint32_t b[4], r[4];
            hash4(idx0, seed, r);
#pragma unroll
            for (int k = 0; k < 4; ++k) b[k] = f2u(x[k]) + (r[k] & 0xffffU);
            w0 = pack_hi16(b[0], b[1]);
            w1 = pack_hi16(b[2], b[3]);
        } else {
            w0 = pack_bf16_rne(x[0], x[1]);
            w1 = pack_bf16_rne(x[2], x[3]);
        }
        stg_b32x2(static_cast<uint16_t*>(base) + i0, w0, w1);
    } else {
        stg_f32x4(static_cast<float*>(base) + i0, x[0], x[1], x[2], x[3]);
    }
}
// Every element is valid and every buffer aligned, so loads come from shared memory and stores go
// straight to HBM as vectors, with no per-element masks or alignment branches.

__device__ __forceinline__ void lds_f32x4(const uint8_t* s, float (&x)[4])
{
    const float4 a = *reinterpret_cast<const float4*>(s);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
}

__device__ __forceinline__ void lds_b16x4(const uint8_t* s, float (&x)[4])
{
    const uint2 a = *reinterpret_cast<const uint2*>(s);
    const uint32_t w[2] = {a.x, a.y};
    unpack_b16(w, x);
}

template <int GT>
__device__ __forceinline__ void fast_grad4(const uint8_t* s, const float* gs, float (&g)[4])
{
    if constexpr (GT == ABX_DT_BF16) lds_b16x4(s, g);
    else lds_f32x4(s, g);
    if (gs != nullptr) {
        // a bf16 gradient is scaled as torch scales a bf16 CUDA tensor in place by an fp32 scalar tensor:
        // by the scalar rounded to bf16, the product rounded back to bf16
        const float f = GT == ABX_DT_BF16 ? u2f(bf16_rne(f2u(*gs)) & 0xffff0000U) : *gs;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            g[k] = __fmul_rn(g[k], f);
            if constexpr (GT == ABX_DT_BF16) g[k] = u2f(bf16_rne(f2u(g[k])) & 0xffff0000U);
        }
    }
}

template <int PT>
__device__ __forceinline__ void fast_master4(const uint8_t* sp, const uint8_t* sl, float (&p)[4])
{
    if constexpr (PT == ABX_DT_F24) {
        const uint2 a = *reinterpret_cast<const uint2*>(sp);
        const uint32_t lo = *reinterpret_cast<const uint32_t*>(sl);
        p[0] = u2f((a.x << 16) | ((lo & 0xffU) << 8));
        p[1] = u2f((a.x & 0xffff0000U) | (lo & 0xff00U));
        p[2] = u2f((a.y << 16) | ((lo >> 8) & 0xff00U));
        p[3] = u2f((a.y & 0xffff0000U) | ((lo >> 16) & 0xff00U));
    } else {
        lds_f32x4(sp, p);
    }
}

template <int MV>
__device__ __forceinline__ void fast_moment4(const uint8_t* s, float (&x)[4])
{
    if constexpr (MV == ABX_DT_BF16) lds_b16x4(s, x);
    else lds_f32x4(s, x);
}

template <int ALGO, int MV, int PT, int GT, bool SR>
__device__ __forceinline__ void fast_dense(const KSeg& S, int64_t base, const uint8_t* st, const float* gs)
{
    using C = Cfg<ALGO, MV, PT, GT>;
    const Coef c = S.c;
    const Coef2 c2 = coef2(c);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int e0 = h * kHalf + threadIdx.x * kGroup;
        const int64_t i0 = base + e0;
        const uint32_t idx0 = S.off32 + (uint32_t)i0;
        float g[4], p[4], m[4];
        fast_grad4<GT>(st + C::OFF_G + e0 * C::GB, gs, g);
        fast_master4<PT>(st + C::OFF_P + e0 * C::PB, st + C::OFF_L + e0, p);
        fast_moment4<MV>(st + C::OFF_M + e0 * C::MB, m);
        if constexpr (ALGO == ABX_ALGO_LION) {
            lion2(p[0], p[1], g[0], g[1], m[0], m[1], c2, c.step);
            lion2(p[2], p[3], g[2], g[3], m[2], m[3], c2, c.step);
            fast_store_master4<PT, SR>(S, i0, p);
            fast_store_moment4<MV, SR>(S.m, i0, m, S.s_m, idx0);
        } else {
            float v[4];
            fast_moment4<MV>(st + C::OFF_V + e0 * C::MB, v);
            if (i0 + kGroup <= S.fused_end) {
                float s0, s1, s2, s3;
                adamw2_fused(p[0], p[1], g[0], g[1], m[0], m[1], v[0], v[1], c2, s0, s1);
                adamw2_fused(p[2], p[3], g[2], g[3], m[2], m[3], v[2], v[3], c2, s2, s3);
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) p[k] = adamw_elem_sel(p[k], g[k], m[k], v[k], c, i0 + k < S.fused_end);
            }
            fast_store_master4<PT, SR>(S, i0, p);
            fast_store_moment4<MV, SR>(S.m, i0, m, S.s_m, idx0);
            fast_store_moment4<MV, SR>(S.v, i0, v, S.s_v, idx0);
        }
        fast_store_out4(S, i0, p);
    }
}

// Max over the warp of values >= 0 (never NaN): non-negative floats order like their bit patterns.
__device__ __forceinline__ float warp_max_nonneg(float x)
{
    return u2f(__reduce_max_sync(0xffffffffU, f2u(x)));
}

__device__ __forceinline__ float absmax4(const float (&x)[4])
{
    // fmaxf drops a NaN operand, as the reference's "a > am ? a : am" skips it
    return fmaxf(fmaxf(fmaxf(fmaxf(0.0f, fabsf(x[0])), fabsf(x[1])), fabsf(x[2])), fabsf(x[3]));
}

// Codes of a whole group of 4 (the fast path of encode4), for a block scale s and y = RN(1/s)
// (warp-uniform, so the branches are too).  In the common case -- s in Markstein's range -- the quotients are packed pairs.
// m: signed; a NaN m (from a NaN gradient; the block maximum skips it) is caught by a NaN sum of the
// group and encoded by the exact out-of-line path.  -0 keeps its sign (copysign after the division).
template <bool SR>
__device__ __forceinline__ uint32_t fast_encode_m4(const float (&x)[4], float s, float y, uint32_t idx0, uint32_t seed)
{
    uint32_t r[4] = {0U, 0U, 0U, 0U};
    if (SR) hash4(idx0, seed, r);
    float q[4];
    if (__builtin_expect(fast_scale(s), 1)) {
        const f2x Y = pk2(y, y), NS = pk2(-s, -s);
        up2(div2(pk2(x[0], x[1]), Y, NS), q[0], q[1]);
        up2(div2(pk2(x[2], x[3]), Y, NS), q[2], q[3]);
#pragma unroll
        for (int k = 0; k < 4; ++k) q[k] = copysignf(q[k], x[k]);
        const float sum = __fadd_rn(__fadd_rn(q[0], q[1]), __fadd_rn(q[2], q[3]));   // finite unless a q is NaN
        if (__builtin_expect(sum == sum, 1)) return enc4_plain<true, SR>(q, r);
    } else {
        const float4 d = div4_ieee(make_float4(x[0], x[1], x[2], x[3]), s);
        q[0] = d.x; q[1] = d.y; q[2] = d.z; q[3] = d.w;
    }
    return enc4_fp8_slow<true, SR>(q[0], q[1], q[2], q[3], r[0], r[1], r[2], r[3]);
}

// u = sqrt(max(v, 0)): never NaN and, with s in Markstein's range, finite, so the quotients need no NaN
// or sign handling; s outside that range (u infinite or tiny) takes the exact out-of-line path.
template <bool SR>
__device__ __forceinline__ uint32_t fast_encode_u4(const float (&x)[4], float s, float y, uint32_t idx0, uint32_t seed)
{
    uint32_t r[4] = {0U, 0U, 0U, 0U};
    if (SR) hash4(idx0, seed, r);
    float q[4];
    if (__builtin_expect(fast_scale(s), 1)) {
        const f2x Y = pk2(y, y), NS = pk2(-s, -s);
        up2(div2(pk2(x[0], x[1]), Y, NS), q[0], q[1]);
        up2(div2(pk2(x[2], x[3]), Y, NS), q[2], q[3]);
        return enc4_plain<false, SR>(q, r);
    }
    const float4 d = div4_ieee(make_float4(x[0], x[1], x[2], x[3]), s);
    return enc4_fp8_slow<false, SR>(d.x, d.y, d.z, d.w, r[0], r[1], r[2], r[3]);
}

// Lion with an FP8 moment: per half tile, warp w owns block w (4 elements per lane).
template <int PT, int GT, bool SR>
__device__ __forceinline__ void fast_fp8_lion(const KSeg& S, int64_t base, const uint8_t* st, const float* gs)
{
    using C = Cfg<ABX_ALGO_LION, ABX_DT_FP8, PT, GT>;
    const Coef c = S.c;
    const Coef2 c2 = coef2(c);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t blk0 = base >> 7;   // first block of the tile
    const float* swm = reinterpret_cast<const float*>(st + C::OFF_SM + (reinterpret_cast<uintptr_t>(S.m_scale + blk0) & 15));
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
        const int e0 = h * kHalf + threadIdx.x * kGroup;
        const int64_t i0 = base + e0;
        const uint32_t idx0 = S.off32 + (uint32_t)i0;
        const int bt = h * kConsumerWarps + warp;   // this warp's block within the tile
        float g[4], p[4], mt[4];
        const float sm = swm[bt];
        dec4_fp8<true>(*reinterpret_cast<const uint32_t*>(st + C::OFF_M + e0), mt);
        up2(mul2(pk2(mt[0], mt[1]), pk2(sm, sm)), mt[0], mt[1]);
        up2(mul2(pk2(mt[2], mt[3]), pk2(sm, sm)), mt[2], mt[3]);
        fast_grad4<GT>(st + C::OFF_G + e0 * C::GB, gs, g);
        fast_master4<PT>(st + C::OFF_P + e0 * C::PB, st + C::OFF_L + e0, p);
        lion2(p[0], p[1], g[0], g[1], mt[0], mt[1], c2, c.step);
        lion2(p[2], p[3], g[2], g[3], mt[2], mt[3], c2, c.step);
        fast_store_master4<PT, SR>(S, i0, p);
        fast_store_out4(S, i0, p);
        const float am = warp_max_nonneg(absmax4(mt));
        const float scm = am > 0.0f ? scale_of<true>(am) : 1.0f;
        stg_b32(static_cast<uint8_t*>(S.m) + i0, fast_encode_m4<SR>(mt, scm, __frcp_rn(scm), idx0, S.s_m));
        if (lane == 0) stg_b32(S.m_scale + blk0 + bt, f2u(scm));
    }
}

// AdamW with FP8 moments.  Warp w owns block w of each half tile (4 elements per lane).  Both halves are
// updated first, keeping their new m and u = sqrt(v); then the warp's four block scales (m and u of each
// half) are computed together, lane 4j+q computing scale q -- the scalar work of four blocks in one pass --
// and broadcast with shuffles; then the four groups of codes are encoded.
template <int PT, int GT, bool SR>
__device__ __forceinline__ void fast_fp8_adamw(const KSeg& S, int64_t base, const uint8_t* st, const float* gs)
{
    using C = Cfg<ABX_ALGO_ADAMW, ABX_DT_FP8, PT, GT>;
    const Coef c = S.c;
    const Coef2 c2 = coef2(c);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t blk0 = base >> 7;   // first block of the tile
    const float* swm = reinterpret_cast<const float*>(st + C::OFF_SM + (reinterpret_cast<uintptr_t>(S.m_scale + blk0) & 15));
    const float* swv = reinterpret_cast<const float*>(st + C::OFF_SV + (reinterpret_cast<uintptr_t>(S.v_scale + blk0) & 15));
    float mt[2][4], ut[2][4], mx[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int e0 = h * kHalf + threadIdx.x * kGroup;
        const int64_t i0 = base + e0;
        const int bt = h * kConsumerWarps + warp;   // this warp's block within the tile
        float g[4], p[4], vt[4];
        const float sm = swm[bt], su = swv[bt];
        dec4_fp8<true>(*reinterpret_cast<const uint32_t*>(st + C::OFF_M + e0), mt[h]);
        up2(mul2(pk2(mt[h][0], mt[h][1]), pk2(sm, sm)), mt[h][0], mt[h][1]);
        up2(mul2(pk2(mt[h][2], mt[h][3]), pk2(sm, sm)), mt[h][2], mt[h][3]);
        dec4_fp8<false>(*reinterpret_cast<const uint32_t*>(st + C::OFF_V + e0), vt);
        {
            const f2x SU = pk2(su, su);
            const f2x U01 = mul2(pk2(vt[0], vt[1]), SU), U23 = mul2(pk2(vt[2], vt[3]), SU);
            up2(mul2(U01, U01), vt[0], vt[1]);
            up2(mul2(U23, U23), vt[2], vt[3]);
        }
        fast_grad4<GT>(st + C::OFF_G + e0 * C::GB, gs, g);
        fast_master4<PT>(st + C::OFF_P + e0 * C::PB, st + C::OFF_L + e0, p);
        if (i0 + kGroup <= S.fused_end) {
            adamw2_fused(p[0], p[1], g[0], g[1], mt[h][0], mt[h][1], vt[0], vt[1], c2, ut[h][0], ut[h][1]);
            adamw2_fused(p[2], p[3], g[2], g[3], mt[h][2], mt[h][3], vt[2], vt[3], c2, ut[h][2], ut[h][3]);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                p[k] = i0 + k < S.fused_end ? adamw_elem_sq<true>(p[k], g[k], mt[h][k], vt[k], ut[h][k], c)
                                            : adamw_elem_sq<false>(p[k], g[k], mt[h][k], vt[k], ut[h][k], c);
        }
        fast_store_master4<PT, SR>(S, i0, p);
        fast_store_out4(S, i0, p);
        // u = sqrt(max(v, 0)) (csrc:1000): v >= 0 here, so only a NaN v differs, and fmaxf maps it to 0
#pragma unroll
        for (int k = 0; k < 4; ++k) ut[h][k] = fmaxf(ut[h][k], 0.0f);
        mx[2 * h] = warp_max_nonneg(absmax4(mt[h]));
        mx[2 * h + 1] = warp_max_nonneg(fmaxf(fmaxf(ut[h][0], ut[h][1]), fmaxf(ut[h][2], ut[h][3])));
    }
    // lane 4j+q: scale q of (m half 0, u half 0, m half 1, u half 1); E4M3 for m, E5M2 for u
    const int q = lane & 3;
    const float amax = q == 0 ? mx[0] : (q == 1 ? mx[1] : (q == 2 ? mx[2] : mx[3]));
    const bool e4 = (q & 1) == 0;
    const float sc = amax > 0.0f ? scale_fmt(amax, e4 ? 448.0f : 57344.0f, e4 ? 0x1.24924ap-9f : 0x1.24924ap-16f)
                                 : 1.0f;
    const float rc = __frcp_rn(sc);
    if (lane < 4) stg_b32(((q & 1) ? S.v_scale : S.m_scale) + blk0 + (q >> 1) * kConsumerWarps + warp, f2u(sc));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int64_t i0 = base + h * kHalf + threadIdx.x * kGroup;
        const uint32_t idx0 = S.off32 + (uint32_t)i0;
        const float scm = __shfl_sync(0xffffffffU, sc, 2 * h), ym = __shfl_sync(0xffffffffU, rc, 2 * h);
        const float scu = __shfl_sync(0xffffffffU, sc, 2 * h + 1), yu = __shfl_sync(0xffffffffU, rc, 2 * h + 1);
        stg_b32(static_cast<uint8_t*>(S.m) + i0, fast_encode_m4<SR>(mt[h], scm, ym, idx0, S.s_m));
        stg_b32(static_cast<uint8_t*>(S.v) + i0, fast_encode_u4<SR>(ut[h], scu, yu, idx0, S.s_v));
    }
}

template <int ALGO, int PT, int GT, bool SR>
__device__ __forceinline__ void fast_fp8(const KSeg& S, int64_t base, const uint8_t* st, const float* gs)
{
    if constexpr (ALGO == ABX_ALGO_LION) fast_fp8_lion<PT, GT, SR>(S, base, st, gs);
    else fast_fp8_adamw<PT, GT, SR>(S, base, st, gs);
}

template <int ALGO, int MV, int PT, int GT, bool SR>
__device__ __forceinline__ void fast_tile(const KSeg& S, int64_t base, const uint8_t* st, const float* gs)
{
    if constexpr (MV == ABX_DT_FP8) fast_fp8<ALGO, PT, GT, SR>(S, base, st, gs);
    else fast_dense<ALGO, MV, PT, GT, SR>(S, base, st, gs);
}

// The 16-byte-aligned window [floor16(p), ceil16(p + bytes)) around `bytes` valid bytes at p: the bulk
// copy reads only 16-byte chunks that hold valid bytes.
__device__ __forceinline__ uint32_t window_bytes(const void* p, uint32_t bytes)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    return (uint32_t)(((a + bytes + 15) & ~(uintptr_t)15) - (a & ~(uintptr_t)15));
}

__device__ __forceinline__ const void* window_start(const void* p)
{
    return reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(p) & ~(uintptr_t)15);
}

template <int ALGO, int MV, int PT, int GT, int NSEG>
__global__ void __launch_bounds__(kThreads, kMinCtasPerSm) update_kernel(const __grid_constant__ KArgs<NSEG> a)
{
    using C = Cfg<ALGO, MV, PT, GT>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = a.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + S;
    StageHdr* hdr = reinterpret_cast<StageHdr*>(smem + 16 * ((16 * S + 15) / 16));
    uint8_t* ring = smem + ring_offset(S);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---- producer: one lane describes each tile and streams staged ones into the ring ----
        if (lane != 0) return;
        int k = 0, s = 0;
        uint32_t ph = 0;   // parity of the current pass over the ring (s and ph track k % S and (k / S) & 1)
        for (int64_t t = blockIdx.x; t < a.total_tiles; t += gridDim.x, ++k) {
            if (!mbar_wait(&empty[s], ph ^ 1, a.spin_limit, a.status, kStatusProducerWait)) break;
            if (t == a.skip_tile) {   // failure-path test: nothing is copied into, or arrives on, this stage
                if (++s == S) { s = 0; ph ^= 1; }
                continue;
            }
            const int si = find_segment(a, t);
            const KSeg& Sg = a.seg[si];
            const int64_t base = (t - Sg.tile_begin) * kTile;
            const bool staged = staged_tile(Sg, base);
            if (k < S || hdr[s].meta.seg != si) hdr[s].seg = Sg;   // the slot may hold this segment already
            hdr[s].meta.seg = si;
            hdr[s].meta.staged = staged;
            hdr[s].meta.base = base;
            if (staged) {
                uint8_t* st = ring + s * C::STAGE;
                uint32_t bytes = C::ARR;
                uint32_t wm = 0, wv = 0;
                if constexpr (C::FP8) {
                    wm = window_bytes(Sg.m_scale + (base >> 7), 4 * (kTile / 128));
                    if constexpr (C::VB > 0) wv = window_bytes(Sg.v_scale + (base >> 7), 4 * (kTile / 128));
                    bytes += wm + wv;
                }
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_load(st + C::OFF_P, static_cast<const char*>(Sg.p) + base * C::PB, kTile * C::PB, &full[s]);
                if constexpr (C::LB > 0) bulk_load(st + C::OFF_L, Sg.p_lo + base, kTile, &full[s]);
                bulk_load(st + C::OFF_G, static_cast<const char*>(Sg.g) + base * C::GB, kTile * C::GB, &full[s]);
                bulk_load(st + C::OFF_M, static_cast<const char*>(Sg.m) + base * C::MB, kTile * C::MB, &full[s]);
                if constexpr (C::VB > 0)
                    bulk_load(st + C::OFF_V, static_cast<const char*>(Sg.v) + base * C::VB, kTile * C::VB, &full[s]);
                if constexpr (C::FP8) {
                    bulk_load(st + C::OFF_SM, window_start(Sg.m_scale + (base >> 7)), wm, &full[s]);
                    if constexpr (C::VB > 0) bulk_load(st + C::OFF_SV, window_start(Sg.v_scale + (base >> 7)), wv, &full[s]);
                }
            } else {
                mbar_arrive(&full[s]);   // consumers read this tile from global memory
            }
            if (++s == S) { s = 0; ph ^= 1; }
        }
        // never leave with bulk copies in flight into this CTA's shared memory (the stage of a skipped tile
        // had none, and its wait gives up like the others)
        for (int j = k - S < 0 ? 0 : k - S; j < k; ++j)
            mbar_wait(&full[j % S], (j / S) & 1, a.spin_limit, a.status, kStatusDrainWait);
        return;
    }

    // ---- consumers ----
    const float* gs = a.g_scale;
    int s = 0;
    uint32_t ph = 0;
    for (int64_t t = blockIdx.x; t < a.total_tiles; t += gridDim.x) {
        if (!mbar_wait(&full[s], ph, a.spin_limit, a.status, kStatusConsumerWait)) return;
        const TileMeta tm = hdr[s].meta;
        const KSeg& Sg = hdr[s].seg;
        if (tm.staged) {
            const uint8_t* st = ring + s * C::STAGE;
            if (Sg.sr) fast_tile<ALGO, MV, PT, GT, true>(Sg, tm.base, st, gs);
            else fast_tile<ALGO, MV, PT, GT, false>(Sg, tm.base, st, gs);
        } else {
            if (Sg.sr) tile<ALGO, MV, PT, GT, true>(Sg, tm.base, nullptr, gs);
            else tile<ALGO, MV, PT, GT, false>(Sg, tm.base, nullptr, gs);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == S) { s = 0; ph ^= 1; }
    }
    // Stores into peers' memory (replicated out) are performed system-wide before this CTA ends, so the
    // kernel's completion -- and any barrier the caller takes after it -- covers them.  (The fast path's
    // stores are asm statements; so is this fence, which keeps it after them.)
    asm volatile("fence.sc.sys;" ::: "memory");
}

// ---- host side ---------------------------------------------------------------------------

thread_local char g_err[512] = "";
std::atomic<int> g_simd_level{ABX_SIMD_AVX512};
std::atomic<uint64_t> g_launches{0};

// The pipeline status word: one unsigned int in pinned host memory mapped into every device's address
// space (portable), allocated at the first launch.  Kernels OR failure bits into it with system-scope
// atomics; the host reads it with no CUDA call.
std::once_flag g_status_once;
unsigned int* g_status = nullptr;          // host address
unsigned int* g_status_dev = nullptr;      // its alias in the devices' address space (portable mapping)
cudaError_t g_status_err = cudaSuccess;

// Failure-path test settings (abx_test_pipeline_fault), copied into the next launches' arguments.
std::atomic<int64_t> g_skip_tile{-1};
std::atomic<uint32_t> g_spin_limit{kSpinLimit};

int set_error(const char* what, cudaError_t e)
{
    snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
    return ABX_E_CUDA;
}

unsigned int* status_word(int* rc)
{
    std::call_once(g_status_once, [] {
        void* p = nullptr;
        g_status_err = cudaHostAlloc(&p, 64, cudaHostAllocMapped | cudaHostAllocPortable);
        void* d = nullptr;
        if (g_status_err == cudaSuccess) g_status_err = cudaHostGetDevicePointer(&d, p, 0);
        if (g_status_err == cudaSuccess) {
            *static_cast<volatile unsigned int*>(p) = 0;
            g_status_dev = static_cast<unsigned int*>(d);
            g_status = static_cast<unsigned int*>(p);
        }
    });
    if (!g_status) *rc = set_error("allocating the pipeline status word", g_status_err);
    return g_status;
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

// Kernel kinds: index = (((algo * 3 + mv) * 2 + f24) * 2 + bf16 grad), mv 0/1/2 = F32/BF16/FP8.
constexpr int kKinds = 24;
using LaunchOne = cudaError_t (*)(const KArgs<1>&, int, size_t, cudaStream_t);
using LaunchMany = cudaError_t (*)(const KArgs<kMaxSegs>&, int, size_t, cudaStream_t);

template <int A, int M, int P, int G, int N>
cudaError_t launch(const KArgs<N>& a, int grid, size_t smem, cudaStream_t st)
{
    update_kernel<A, M, P, G, N><<<grid, kThreads, smem, st>>>(a);
    return cudaGetLastError();
}

#define ABX_FOR_KINDS(X, N)                                                                                   \
    X(0, ABX_DT_F32, ABX_DT_F32, ABX_DT_F32, N), X(0, ABX_DT_F32, ABX_DT_F32, ABX_DT_BF16, N),                 \
    X(0, ABX_DT_F32, ABX_DT_F24, ABX_DT_F32, N), X(0, ABX_DT_F32, ABX_DT_F24, ABX_DT_BF16, N),                 \
    X(0, ABX_DT_BF16, ABX_DT_F32, ABX_DT_F32, N), X(0, ABX_DT_BF16, ABX_DT_F32, ABX_DT_BF16, N),               \
    X(0, ABX_DT_BF16, ABX_DT_F24, ABX_DT_F32, N), X(0, ABX_DT_BF16, ABX_DT_F24, ABX_DT_BF16, N),               \
    X(0, ABX_DT_FP8, ABX_DT_F32, ABX_DT_F32, N), X(0, ABX_DT_FP8, ABX_DT_F32, ABX_DT_BF16, N),                 \
    X(0, ABX_DT_FP8, ABX_DT_F24, ABX_DT_F32, N), X(0, ABX_DT_FP8, ABX_DT_F24, ABX_DT_BF16, N),                 \
    X(1, ABX_DT_F32, ABX_DT_F32, ABX_DT_F32, N), X(1, ABX_DT_F32, ABX_DT_F32, ABX_DT_BF16, N),                 \
    X(1, ABX_DT_F32, ABX_DT_F24, ABX_DT_F32, N), X(1, ABX_DT_F32, ABX_DT_F24, ABX_DT_BF16, N),                 \
    X(1, ABX_DT_BF16, ABX_DT_F32, ABX_DT_F32, N), X(1, ABX_DT_BF16, ABX_DT_F32, ABX_DT_BF16, N),               \
    X(1, ABX_DT_BF16, ABX_DT_F24, ABX_DT_F32, N), X(1, ABX_DT_BF16, ABX_DT_F24, ABX_DT_BF16, N),               \
    X(1, ABX_DT_FP8, ABX_DT_F32, ABX_DT_F32, N), X(1, ABX_DT_FP8, ABX_DT_F32, ABX_DT_BF16, N),                 \
    X(1, ABX_DT_FP8, ABX_DT_F24, ABX_DT_F32, N), X(1, ABX_DT_FP8, ABX_DT_F24, ABX_DT_BF16, N)

#define ABX_KERNEL_PTR(A, M, P, G, N) (const void*)update_kernel<A, M, P, G, N>
#define ABX_LAUNCH_PTR(A, M, P, G, N) launch<A, M, P, G, N>
#define ABX_STAGE(A, M, P, G, N) Cfg<A, M, P, G>::STAGE

const void* const kKernelsOne[kKinds] = {ABX_FOR_KINDS(ABX_KERNEL_PTR, 1)};
const void* const kKernelsMany[kKinds] = {ABX_FOR_KINDS(ABX_KERNEL_PTR, kMaxSegs)};
const LaunchOne kLaunchOne[kKinds] = {ABX_FOR_KINDS(ABX_LAUNCH_PTR, 1)};
const LaunchMany kLaunchMany[kKinds] = {ABX_FOR_KINDS(ABX_LAUNCH_PTR, kMaxSegs)};
const int kStageBytes[kKinds] = {ABX_FOR_KINDS(ABX_STAGE, 0)};

// Ring geometry of a kind: stages and dynamic shared memory (barriers first, then the 128-aligned ring).
int stages_of(int kind)
{
    const int s = kSmemTarget / kStageBytes[kind];
    return s < 2 ? 2 : (s > 8 ? 8 : s);
}

size_t smem_of(int kind)
{
    const int s = stages_of(kind);
    return (size_t)(ring_offset(s) + s * kStageBytes[kind]);
}

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
            const int smem = (int)smem_of(k);
            err = cudaFuncSetAttribute(kKernelsOne[k], cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (err == cudaSuccess)
                err = cudaFuncSetAttribute(kKernelsMany[k], cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (err == cudaSuccess)
                err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.blocks_one[k], kKernelsOne[k], kThreads, smem);
            if (err == cudaSuccess)
                err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.blocks_many[k], kKernelsMany[k], kThreads, smem);
        }
        d.err = err;
    });
    if (d.err != cudaSuccess) { *rc = set_error("querying the device", d.err); return nullptr; }
    return &d;
}

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

// Device accesses need natural alignment (the reference's host loads do not).  A segment whose buffers
// allow 4-element vectors takes vector accesses on the direct path; one whose streamed buffers are all
// 16-byte aligned has its whole tiles bulk-copied.
int check_alignment(const abx_segment* s, bool* vec_ok, bool* tma_ok)
{
    const bool lion = s->algorithm == ABX_ALGO_LION;
    const bool f24 = s->p_dtype == ABX_DT_F24;
    const uintptr_t pe = f24 ? 2 : 4, ge = s->g_dtype == ABX_DT_BF16 ? 2 : 4;
    const uintptr_t me = s->mv_dtype == ABX_DT_F32 ? 4 : (s->mv_dtype == ABX_DT_BF16 ? 2 : 1);
    const uintptr_t oe = s->out_dtype == ABX_DT_F32 ? 4 : 2;
    const void* out = s->out_dtype != ABX_DT_NONE ? s->out : nullptr;
    const void* v = lion ? nullptr : s->v;
    const uint8_t* lo = f24 ? s->p_lo : nullptr;
    const bool fp8 = s->mv_dtype == ABX_DT_FP8;
    if (!aligned(s->p, pe) || !aligned(s->g, ge) || !aligned(s->m, me) || !aligned(v, me) || !aligned(out, oe) ||
        (fp8 && (!aligned(s->m_scale, 4) || (!lion && !aligned(s->v_scale, 4))))) {
        snprintf(g_err, sizeof g_err, "segment buffer not aligned to its element size");
        return ABX_E_ALIGN;
    }
    *vec_ok = aligned(s->p, 4 * pe) && aligned(lo, 4) && aligned(s->g, 4 * ge) && aligned(s->m, 4 * me) &&
              aligned(v, 4 * me) && aligned(out, 4 * oe);
    *tma_ok = *vec_ok && aligned(s->p, 16) && aligned(lo, 16) && aligned(s->g, 16) && aligned(s->m, 16) &&
              aligned(v, 16);
    return ABX_OK;
}

uint32_t hash32_host(uint32_t x)
{
    x = (x ^ (x >> 16)) * 0x7feb352dU;
    x = (x ^ (x >> 15)) * 0x846ca68bU;
    return x ^ (x >> 16);
}

void fill_kseg(KSeg& k, const abx_segment* s, const abx_hparams* h, int lanes, bool vec_ok, bool tma_ok,
               int64_t tile_begin, const int64_t* rep, int32_t nrep)
{
    k.nrep = s->out_dtype != ABX_DT_NONE ? nrep : 0;
    for (int j = 0; j < k.nrep; ++j) k.rep_delta[j] = rep[j];
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
    k.out_dt = s->out_dtype;
    k.sr = h->stochastic != 0;
    k.vec_ok = vec_ok ? 1 : 0;
    k.tma_ok = tma_ok ? 1 : 0;
}

int kind_of(const abx_segment* s)
{
    const int mv = s->mv_dtype == ABX_DT_F32 ? 0 : (s->mv_dtype == ABX_DT_BF16 ? 1 : 2);
    return (((s->algorithm == ABX_ALGO_LION ? 1 : 0) * 3 + mv) * 2 + (s->p_dtype == ABX_DT_F24 ? 1 : 0)) * 2 +
           (s->g_dtype == ABX_DT_BF16 ? 1 : 0);
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
        const float* g_scale, const int64_t* rep = nullptr, int32_t nrep = 0)
{
    if (nsegs <= 0) return ABX_OK;
    if (nrep < 0 || nrep > kMaxReplicas || (nrep > 0 && !rep)) return ABX_E_ARG;
    for (int32_t j = 0; j < nrep; ++j)
        if (rep[j] % 16) {
            snprintf(g_err, sizeof g_err, "replica delta %lld is not a multiple of 16 bytes", (long long)rep[j]);
            return ABX_E_ALIGN;
        }
    if (!segs) return ABX_E_ARG;
    const bool from_groups = hps == nullptr;
    std::vector<char> vec_ok(nsegs), tma_ok(nsegs);
    for (int32_t i = 0; i < nsegs; ++i) {
        const int rc = check_segment(segs[i], from_groups);
        if (rc) return rc;
    }
    for (int32_t i = 0; i < nsegs; ++i) {
        if (segs[i]->n == 0) continue;
        bool vo = false, to = false;
        const int rc = check_alignment(segs[i], &vo, &to);
        if (rc) return rc;
        vec_ok[i] = vo;
        tma_ok[i] = to;
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
    if (!status_word(&rc)) return rc;
    unsigned int* status = g_status_dev;   // what the kernels write
    const uint32_t spin_limit = g_spin_limit.load();
    int64_t skip_tile = g_skip_tile.exchange(-1);   // a test's fault applies to the next launch only
    const int lanes = lanes_of(g_simd_level.load());
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    std::vector<int32_t> order;
    order.reserve(nsegs);
    for (int kind = 0; kind < kKinds; ++kind) {
        order.clear();
        for (int32_t i = 0; i < nsegs; ++i)
            if (segs[i]->n > 0 && kind_of(segs[i]) == kind) order.push_back(i);
        const size_t smem = smem_of(kind);
        for (size_t b = 0; b < order.size(); b += kMaxSegs) {
            const int cnt = (int)(order.size() - b < (size_t)kMaxSegs ? order.size() - b : kMaxSegs);
            cudaError_t e;
            if (cnt == 1) {
                KArgs<1> a;
                std::memset(&a, 0, sizeof a);
                const int32_t i = order[b];
                fill_kseg(a.seg[0], segs[i], &hps[i], lanes, vec_ok[i], tma_ok[i], 0, rep, nrep);
                a.nseg = 1;
                a.stages = stages_of(kind);
                a.total_tiles = tiles_of(segs[i]->n);
                a.g_scale = g_scale;
                a.status = status;
                a.spin_limit = spin_limit;
                a.skip_tile = skip_tile;
                skip_tile = -1;
                e = kLaunchOne[kind](a, grid_for(a.total_tiles, dev->blocks_one[kind], dev->sms, max_ctas), smem, st);
            } else {
                static thread_local KArgs<kMaxSegs> a;   // ~10 KB: kept off the stack
                std::memset(&a, 0, sizeof a);
                int64_t tiles = 0;
                for (int j = 0; j < cnt; ++j) {
                    const int32_t i = order[b + j];
                    fill_kseg(a.seg[j], segs[i], &hps[i], lanes, vec_ok[i], tma_ok[i], tiles, rep, nrep);
                    tiles += tiles_of(segs[i]->n);
                }
                a.nseg = cnt;
                a.stages = stages_of(kind);
                a.total_tiles = tiles;
                a.g_scale = g_scale;
                a.status = status;
                a.spin_limit = spin_limit;
                a.skip_tile = skip_tile;
                skip_tile = -1;
                e = kLaunchMany[kind](a, grid_for(tiles, dev->blocks_many[kind], dev->sms, max_ctas), smem, st);
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

ABX_API int abx_multi_step_replicated(void* stream, abx_segment* const* segs, int32_t nsegs, int32_t max_ctas,
                                      const float* g_scale, const int64_t* out_deltas, int32_t nreplicas)
{
    return abx::run(stream, segs, nullptr, nsegs, max_ctas, g_scale, out_deltas, nreplicas);
}

// The copy-engine form of the same all-gather: one asynchronous copy per replica, each on its own stream,
// so the copy engines move the bytes over NVLink while the SMs go on with the next update.
ABX_API int abx_replicate_async(void* const* streams, const void* src, int64_t bytes, const int64_t* deltas,
                                int32_t nreplicas)
{
    if (bytes < 0 || nreplicas < 0 || nreplicas > abx::kMaxReplicas) return ABX_E_ARG;
    if (bytes == 0 || nreplicas == 0) return ABX_OK;
    if (!src || !deltas || !streams) return ABX_E_NULL_PTR;
    for (int32_t j = 0; j < nreplicas; ++j)   // a replica may not overlap the source
        if (deltas[j] > -bytes && deltas[j] < bytes) return ABX_E_ARG;
    const char* s = static_cast<const char*>(src);
    for (int32_t j = 0; j < nreplicas; ++j) {
        const cudaError_t e = cudaMemcpyAsync(const_cast<char*>(s) + deltas[j], s, (size_t)bytes, cudaMemcpyDefault,
                                              static_cast<cudaStream_t>(streams[j]));
        if (e != cudaSuccess) return abx::set_error("replica copy", e);
    }
    return ABX_OK;
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

// The status word's bits (nonzero: an update kernel's pipeline wait gave up, so some update since the
// last call is incomplete), then cleared.  No device synchronization: it covers the kernels that have
// finished when it is called.
ABX_API int abx_pipeline_status(void)
{
    int rc = ABX_OK;
    unsigned int* w = abx::status_word(&rc);
    if (!w) return rc;
    return (int)__atomic_exchange_n(w, 0u, __ATOMIC_SEQ_CST);
}

// Host address of the status word (mapped pinned memory; NULL if it cannot be allocated): a caller may
// poll it directly, without any CUDA call.
ABX_API const volatile unsigned int* abx_status_word(void)
{
    int rc = ABX_OK;
    return abx::status_word(&rc);
}

// Failure-path testing only: the next launch's producer skips element tile `tile` of its tile space (no bulk
// copy is issued into that ring stage and nothing arrives on its barrier), and from now on every mbarrier
// wait gives up after `spin_limit` polls (0 restores the default).  The consumers waiting for the skipped
// tile give up, the status word is set, and the CTA's later tiles stay unupdated -- the effect of a pipeline
// fault, made without a fault.  tile < 0 cancels a pending skip.
ABX_API int abx_test_pipeline_fault(int64_t tile, uint32_t spin_limit)
{
    abx::g_spin_limit.store(spin_limit == 0 ? abx::kSpinLimit : spin_limit);
    abx::g_skip_tile.store(tile < 0 ? -1 : tile);
    return ABX_OK;
}
