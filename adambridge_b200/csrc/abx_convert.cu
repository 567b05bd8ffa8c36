// abx_convert.cu -- conversions between the optimizer-state formats, on the device.
//
// The optimizer state lives in HBM in one of the stored formats (fp32, bf16, the FP8
// block format, the fp24 master).  Changing a buffer's format -- set_precision,
// loading a checkpoint written in another precision or by torch.optim.AdamW, an fp24
// master from the weights, decoding a master for master_params() -- is one pass here:
// each value is decoded to fp32 in registers and re-encoded with round-to-nearest-even,
// with the roundings of the reference's own conversions, which are torch operations on
// the host (adambridge/precision.py: BF16Store.write :319-323 nearest-even copy_,
// FP8Store.write :383-398 with seed None, FP8Store.read :374-381, FP24Store.read/write
// :448-462 nearest-even, torch's float -> bfloat16 / float8 casts).
//
// One warp owns one 128-element block (4 consecutive values per lane), so an FP8
// destination's block maximum is a warp reduction; a grid-stride loop walks the blocks.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>

#include "../../include/abx.h"
#include "abx_device.cuh"

#define ABX_API extern "C" __attribute__((visibility("default")))

namespace abx {
int set_error(const char* what, cudaError_t e);   // abx_kernels.cu
extern std::atomic<uint64_t> g_launches;
}  // namespace abx

namespace {

using abx::f2u;
using abx::u2f;

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kBlock = ABX_FP8_BLOCK;   // values per warp per iteration (one FP8 block)

// Per-format description the kernel reads (the ABI struct, with the FP8 limits resolved on the host).
struct View {
    void* values;
    void* aux;
    int64_t block;
    int32_t dtype;
    int32_t v_role;    // FP8 second moment: E5M2 codes of sqrt(v)
};

struct ConvArgs {
    View src, dst;
    int64_t n;
    int64_t nblocks;   // 128-element blocks covering n
};

// ---- decoding ------------------------------------------------------------------------------

// FP8 code -> float, exact for every finite code and the infinities (E5M2 0x7c/0xfc).
__device__ __forceinline__ float fp8_value(uint32_t code, bool e5m2)
{
    const uint16_t c2 = (uint16_t)(code & 0xffU);
    uint32_t h2;
    if (e5m2)
        asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h2) : "h"(c2));
    else
        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(c2));
    float x;
    asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %1; cvt.f32.f16 %0, lo; }" : "=f"(x) : "r"(h2));
    return x;
}

// The NaN a NaN code decodes to on the host -- its sign, quiet, and for E5M2 the code's mantissa bits above the
// quiet bit -- or 0 for a code that is not NaN.  (GPU arithmetic would return the positive canonical NaN; the
// host keeps a NaN operand's sign and payload, so NaNs are carried around the arithmetic here.)
__device__ __forceinline__ uint32_t fp8_nan_bits(uint32_t c, bool e5m2)
{
    const uint32_t sign = (c & 0x80U) << 24;
    if (e5m2) return ((c & 0x7cU) == 0x7cU && (c & 3U)) ? (sign | 0x7fc00000U | ((c & 3U) << 21)) : 0U;
    return (c & 0x7fU) == 0x7fU ? (sign | 0x7fe00000U) : 0U;
}

// Value i of a state buffer as fp32 (FP8: code x block scale; a second moment is the square of that).
__device__ __forceinline__ float load_value(const View& s, int64_t i)
{
    switch (s.dtype) {
    case ABX_DT_F32:
        return static_cast<const float*>(s.values)[i];
    case ABX_DT_BF16:
        return u2f((uint32_t) static_cast<const uint16_t*>(s.values)[i] << 16);
    case ABX_DT_F24:
        return u2f(((uint32_t) static_cast<const uint16_t*>(s.values)[i] << 16) |
                   ((uint32_t) static_cast<const uint8_t*>(s.aux)[i] << 8));
    default: {
        const uint32_t c = static_cast<const uint8_t*>(s.values)[i];
        const uint32_t nan = fp8_nan_bits(c, s.v_role != 0);
        if (nan) return u2f(nan);
        const float sc = static_cast<const float*>(s.aux)[i / s.block];
        float x = __fmul_rn(fp8_value(c, s.v_role != 0), sc);
        if (x != x)   // a NaN scale propagates, quieted; 0 x inf is the host's default NaN, whose sign bit is set
            return sc != sc ? u2f(f2u(sc) | 0x00400000U) : u2f(0xffc00000U);
        return s.v_role ? __fmul_rn(x, x) : x;
    }
    }
}

// ---- encoding ------------------------------------------------------------------------------

// fp32 -> bf16 bits, nearest-even; every NaN becomes the quiet NaN 0x7fc0, as torch's cast does.
__device__ __forceinline__ uint32_t bf16_bits_of(float x)
{
    if (x != x) return 0x7fc0U;
    uint32_t d;
    asm("{ .reg .b16 h; cvt.rn.bf16.f32 h, %1; cvt.u32.u16 %0, h; }" : "=r"(d) : "f"(x));
    return d;
}

// A value already clamped to the format's finite range -> its FP8 code, nearest-even.  Zeros keep their sign.
__device__ __forceinline__ uint32_t fp8_code_of(float q, bool e5m2)
{
    uint16_t c2;
    if (e5m2)
        asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(c2) : "f"(0.0f), "f"(q));
    else
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(c2) : "f"(0.0f), "f"(q));
    return (uint32_t)c2 & 0xffU;
}

// Largest of four magnitudes over the warp, ignoring NaNs, and whether any value of the warp is NaN (torch's
// amax propagates NaN: the caller then treats the block maximum as NaN).
__device__ __forceinline__ float warp_absmax(const float (&a)[4], bool& any_nan)
{
    bool nan = false;
    uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        nan |= a[k] != a[k];
        const uint32_t b = f2u(a[k]) & 0x7fffffffU;   // |a|: non-negative floats order like their bits
        m = (a[k] == a[k] && b > m) ? b : m;
    }
    any_nan = __any_sync(0xffffffffU, nan);
    return u2f(__reduce_max_sync(0xffffffffU, m));
}

__device__ __forceinline__ uint32_t fp8_block_codes(float (&x)[4], bool v, float& scale)
{
    const float fmax = v ? 57344.0f : 448.0f;
    if (v) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (x[k] == x[k]) x[k] = __fsqrt_rn(x[k] < 0.0f ? 0.0f : x[k]);
    }
    bool any_nan;
    const float amax_finite = warp_absmax(x, any_nan);
    const float amax = any_nan ? __uint_as_float(0x7fc00000U) : amax_finite;
    // RN(amax / fmax): the constant reciprocal with Markstein's correction (abx_device.cuh: scale_of)
    scale = amax > 0.0f ? (v ? abx::scale_of<false>(amax) : abx::scale_of<true>(amax)) : 1.0f;
    if (__builtin_expect(!any_nan && abx::fast_scale(scale), 1)) {
        // Every value finite and the scale in Markstein's range: the correctly rounded quotients pairwise
        // (abx_device.cuh: div2, valid there for |x| >= 2^-100; smaller quotients encode to a zero code
        // whatever their last bits), the sign put back (a zero keeps its sign), then two values per
        // conversion.  cvt.satfinite saturates at the format's largest finite value, which is what the
        // reference's clamp to +-fmax before its nearest-even cast gives.
        const float y = __frcp_rn(scale);
        const abx::f2x Y = abx::pk2(y, y), NS = abx::pk2(-scale, -scale);
        float q[4];
        abx::up2(abx::div2(abx::pk2(x[0], x[1]), Y, NS), q[0], q[1]);
        abx::up2(abx::div2(abx::pk2(x[2], x[3]), Y, NS), q[2], q[3]);
        uint16_t c01, c23;
#pragma unroll
        for (int k = 0; k < 4; ++k) q[k] = copysignf(q[k], x[k]);
        if (v) {
            asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(c01) : "f"(q[1]), "f"(q[0]));
            asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(c23) : "f"(q[3]), "f"(q[2]));
        } else {
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(c01) : "f"(q[1]), "f"(q[0]));
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(c23) : "f"(q[3]), "f"(q[2]));
        }
        return (uint32_t)c01 | ((uint32_t)c23 << 16);
    }
    // A NaN in the block, or a scale outside Markstein's range (tiny or infinite): value by value, IEEE division.
    uint32_t w = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t code;
        if (x[k] != x[k]) {
            code = 0x7fU | ((f2u(x[k]) >> 24) & 0x80U);
        } else {
            float q = __fdiv_rn(x[k], scale);
            if (q != q) {
                code = 0xffU;   // inf / inf (an infinite value, so an infinite scale): the host's
                                // invalid-operation NaN has its sign bit set
            } else {
                q = q < -fmax ? -fmax : (q > fmax ? fmax : q);
                code = fp8_code_of(q, v);
            }
        }
        w |= code << (8 * k);
    }
    return w;
}

// One value into a non-FP8 destination.
__device__ __forceinline__ void store_value(const View& d, int64_t i, float x)
{
    switch (d.dtype) {
    case ABX_DT_F32:
        static_cast<float*>(d.values)[i] = x;
        break;
    case ABX_DT_BF16:
        static_cast<uint16_t*>(d.values)[i] = (uint16_t)bf16_bits_of(x);
        break;
    default: {   // ABX_DT_F24: nearest-even to the top 24 bits; NaN quieted and kept whole
        const uint32_t b = abx::f24_bits(f2u(x), false, 0U);
        static_cast<uint16_t*>(d.values)[i] = (uint16_t)(b >> 16);
        static_cast<uint8_t*>(d.aux)[i] = (uint8_t)(b >> 8);
    }
    }
}

// Any source (any FP8 block, any alignment), any destination: one value at a time.
__global__ void __launch_bounds__(kThreads) convert_kernel(const __grid_constant__ ConvArgs a)
{
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * kWarps;
    for (int64_t blk = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); blk < a.nblocks; blk += warps) {
        const int64_t i0 = blk * kBlock + lane * 4;
        float x[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = i0 + k < a.n ? load_value(a.src, i0 + k) : 0.0f;   // padding is 0
        const View& d = a.dst;
        if (d.dtype == ABX_DT_FP8) {
            float scale;
            const uint32_t w = fp8_block_codes(x, d.v_role != 0, scale);
            *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(d.values) + i0) = w;   // whole padded block
            if (lane == 0) static_cast<float*>(d.aux)[blk] = scale;
            continue;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (i0 + k < a.n) store_value(d, i0 + k, x[k]);
    }
}

// ---- vector path: one kernel per (source, destination) format pair -------------------------------
// Every buffer aligned for 4-value vectors and an FP8 source in 128-value blocks (so a warp's block is the
// source's block and its scale one load): each lane moves its 4 values with one load and one store per plane.

template <int DT>
__device__ __forceinline__ void load4(const View& s, int64_t i0, int64_t blk, float (&x)[4])
{
    if constexpr (DT == ABX_DT_F32) {
        const float4 q = *reinterpret_cast<const float4*>(static_cast<const float*>(s.values) + i0);
        x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
    } else if constexpr (DT == ABX_DT_BF16) {
        const uint2 q = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(s.values) + i0);
        x[0] = u2f(q.x << 16); x[1] = u2f(q.x & 0xffff0000U); x[2] = u2f(q.y << 16); x[3] = u2f(q.y & 0xffff0000U);
    } else if constexpr (DT == ABX_DT_F24) {
        const uint2 h = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(s.values) + i0);
        const uint32_t lo = *reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(s.aux) + i0);
        x[0] = u2f((h.x << 16) | ((lo & 0xffU) << 8));
        x[1] = u2f((h.x & 0xffff0000U) | (lo & 0xff00U));
        x[2] = u2f((h.y << 16) | ((lo >> 8) & 0xff00U));
        x[3] = u2f((h.y & 0xffff0000U) | ((lo >> 16) & 0xff00U));
    } else {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(s.values) + i0);
        const float sc = static_cast<const float*>(s.aux)[blk];
        const bool v = s.v_role != 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t c = (w >> (8 * k)) & 0xffU;
            const uint32_t nan = fp8_nan_bits(c, v);
            float y = __fmul_rn(fp8_value(c, v), sc);
            if (y != y) y = sc != sc ? u2f(f2u(sc) | 0x00400000U) : u2f(0xffc00000U);   // see load_value
            else if (v) y = __fmul_rn(y, y);
            x[k] = nan ? u2f(nan) : y;
        }
    }
}

template <int DT>
__device__ __forceinline__ void store4(const View& d, int64_t i0, const float (&x)[4])
{
    if constexpr (DT == ABX_DT_F32) {
        *reinterpret_cast<float4*>(static_cast<float*>(d.values) + i0) = make_float4(x[0], x[1], x[2], x[3]);
    } else if constexpr (DT == ABX_DT_BF16) {
        const uint32_t b0 = bf16_bits_of(x[0]), b1 = bf16_bits_of(x[1]), b2 = bf16_bits_of(x[2]), b3 = bf16_bits_of(x[3]);
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(d.values) + i0) = make_uint2(b0 | (b1 << 16), b2 | (b3 << 16));
    } else {   // ABX_DT_F24
        uint32_t b[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) b[k] = abx::f24_bits(f2u(x[k]), false, 0U);
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(d.values) + i0) =
            make_uint2((b[0] >> 16) | (b[1] & 0xffff0000U), (b[2] >> 16) | (b[3] & 0xffff0000U));
        *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(d.aux) + i0) =
            ((b[0] >> 8) & 0xffU) | (b[1] & 0xff00U) | ((b[2] << 8) & 0xff0000U) | ((b[3] << 16) & 0xff000000U);
    }
}

template <int SRC, int DST>
__global__ void __launch_bounds__(kThreads) convert_vec_kernel(const __grid_constant__ ConvArgs a)
{
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * kWarps;
    for (int64_t blk = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); blk < a.nblocks; blk += warps) {
        const int64_t i0 = blk * kBlock + lane * 4;
        const bool whole = i0 + 4 <= a.n;
        float x[4];
        if (whole) {
            load4<SRC>(a.src, i0, blk, x);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) x[k] = i0 + k < a.n ? load_value(a.src, i0 + k) : 0.0f;
        }
        if constexpr (DST == ABX_DT_FP8) {
            float scale;
            const uint32_t w = fp8_block_codes(x, a.dst.v_role != 0, scale);
            *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(a.dst.values) + i0) = w;
            if (lane == 0) static_cast<float*>(a.dst.aux)[blk] = scale;
        } else if (whole) {
            store4<DST>(a.dst, i0, x);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (i0 + k < a.n) store_value(a.dst, i0 + k, x[k]);
        }
    }
}

using VecKernel = void (*)(ConvArgs);
constexpr int kFormats = 4;   // ABX_DT_F32, _BF16, _FP8, _F24 are codes 1..4

#define ABX_VEC_ROW(S) convert_vec_kernel<S, ABX_DT_F32>, convert_vec_kernel<S, ABX_DT_BF16>, \
                       convert_vec_kernel<S, ABX_DT_FP8>, convert_vec_kernel<S, ABX_DT_F24>
const VecKernel kVecKernels[kFormats][kFormats] = {{ABX_VEC_ROW(ABX_DT_F32)}, {ABX_VEC_ROW(ABX_DT_BF16)},
                                                   {ABX_VEC_ROW(ABX_DT_FP8)}, {ABX_VEC_ROW(ABX_DT_F24)}};

// Whether a buffer's planes allow 4-value vector accesses (and, for an FP8 source, are in 128-value blocks).
bool vector_ready(const abx_state* s)
{
    const uintptr_t v = reinterpret_cast<uintptr_t>(s->values), x = reinterpret_cast<uintptr_t>(s->aux);
    switch (s->dtype) {
    case ABX_DT_F32: return v % 16 == 0;
    case ABX_DT_BF16: return v % 8 == 0;
    case ABX_DT_F24: return v % 8 == 0 && x % 4 == 0;
    default: return v % 4 == 0 && s->block == kBlock;
    }
}

bool valid_dtype(int32_t dt) { return dt == ABX_DT_F32 || dt == ABX_DT_BF16 || dt == ABX_DT_FP8 || dt == ABX_DT_F24; }

bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_state(const abx_state* s, bool dst)
{
    if (!s || !valid_dtype(s->dtype)) return ABX_E_MV_DTYPE;
    if (!s->values) return ABX_E_NULL_PTR;
    if ((s->dtype == ABX_DT_FP8 || s->dtype == ABX_DT_F24) && !s->aux) return ABX_E_SCALE_NULL;
    if (s->dtype == ABX_DT_FP8) {
        if (s->role != 0 && s->role != 1) return ABX_E_ARG;
        if (dst ? s->block != ABX_FP8_BLOCK : (s->block <= 0 || s->block > (int64_t(1) << 20))) return ABX_E_ARG;
        if (dst && !aligned_to(s->values, 4)) return ABX_E_ALIGN;   // whole blocks as 32-bit words
    }
    const uintptr_t es = s->dtype == ABX_DT_F32 ? 4 : (s->dtype == ABX_DT_FP8 ? 1 : 2);
    if (!aligned_to(s->values, es) || (s->dtype == ABX_DT_FP8 && !aligned_to(s->aux, 4))) return ABX_E_ALIGN;
    return ABX_OK;
}

}  // namespace

// Convert n values from one state buffer to another, on `stream` (see include/abx.h).
ABX_API int abx_convert(void* stream, const abx_state* src, const abx_state* dst, int64_t n)
{
    if (n < 0) return ABX_E_ARG;
    int rc = check_state(src, false);
    if (rc) return rc;
    rc = check_state(dst, true);
    if (rc) return rc;
    if (n == 0) return ABX_OK;
    ConvArgs a;
    std::memset(&a, 0, sizeof a);
    a.src = View{src->values, src->aux, src->dtype == ABX_DT_FP8 ? src->block : 1, src->dtype, src->role};
    a.dst = View{dst->values, dst->aux, dst->dtype == ABX_DT_FP8 ? dst->block : 1, dst->dtype, dst->role};
    a.n = n;
    a.nblocks = (n + kBlock - 1) / kBlock;
    int dev = 0, sms = 148;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return abx::set_error("abx_convert: querying the device", e);
    const int64_t want = (a.nblocks + kWarps - 1) / kWarps;
    const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (vector_ready(src) && vector_ready(dst))
        kVecKernels[src->dtype - 1][dst->dtype - 1]<<<grid, kThreads, 0, st>>>(a);
    else
        convert_kernel<<<grid, kThreads, 0, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return abx::set_error("abx_convert launch", e);
    abx::g_launches.fetch_add(1, std::memory_order_relaxed);
    return ABX_OK;
}
