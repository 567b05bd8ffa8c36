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

// Largest of four magnitudes over the warp, NaN if any value of the warp is NaN (torch's amax propagates NaN).
__device__ __forceinline__ float warp_absmax_nan(const float (&a)[4])
{
    bool nan = false;
    uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        nan |= a[k] != a[k];
        const uint32_t b = f2u(a[k]) & 0x7fffffffU;   // |a|: non-negative floats order like their bits
        m = (a[k] == a[k] && b > m) ? b : m;
    }
    m = __reduce_max_sync(0xffffffffU, m);
    return __any_sync(0xffffffffU, nan) ? __uint_as_float(0x7fc00000U) : u2f(m);
}

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
            // FP8Store.write: a second moment is kept as sqrt(max(v, 0)); the block's scale is absmax / fmax
            // (1 for an all-zero or NaN block); values are divided by it, clamped to +-fmax and cast.
            // A NaN passes through all of that on the host with its sign and becomes code 0x7f | sign (torch's
            // float8 casts); it is carried past the arithmetic here.
            const bool v = d.v_role != 0;
            const float fmax = v ? 57344.0f : 448.0f;
            if (v) {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (x[k] == x[k]) x[k] = __fsqrt_rn(x[k] < 0.0f ? 0.0f : x[k]);
            }
            const float amax = warp_absmax_nan(x);
            const float scale = amax > 0.0f ? __fdiv_rn(amax, fmax) : 1.0f;
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
            *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(d.values) + i0) = w;   // whole padded block
            if (lane == 0) static_cast<float*>(d.aux)[blk] = scale;
            continue;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t i = i0 + k;
            if (i >= a.n) break;
            switch (d.dtype) {
            case ABX_DT_F32:
                static_cast<float*>(d.values)[i] = x[k];
                break;
            case ABX_DT_BF16:
                static_cast<uint16_t*>(d.values)[i] = (uint16_t)bf16_bits_of(x[k]);
                break;
            default: {   // ABX_DT_F24: nearest-even to the top 24 bits; NaN quieted and kept whole
                const uint32_t b = abx::f24_bits(f2u(x[k]), false, 0U);
                static_cast<uint16_t*>(d.values)[i] = (uint16_t)(b >> 16);
                static_cast<uint8_t*>(d.aux)[i] = (uint8_t)(b >> 8);
            }
            }
        }
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
    convert_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return abx::set_error("abx_convert launch", e);
    abx::g_launches.fetch_add(1, std::memory_order_relaxed);
    return ABX_OK;
}
