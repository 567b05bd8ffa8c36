// abx_clip.cu -- gradient norms and the gradient-clipping coefficient on the device (libabx).
//
// torch.nn.utils.clip_grad_norm_(params, max_norm) reads every gradient for its norm and then
// reads and writes every gradient again to scale it.  Here the norm pass is one streaming read,
// and the scale is applied by the update kernel while it reads the gradient
// (abx_multi_step_scaled's g_scale): the clip costs one gradient read instead of three passes.
//
// Three launches, no atomics, deterministic for a given input:
//   1. norm_partials: fp32 sum of squares of every 16384-element tile of every tensor, each in
//      a fixed order (thread-strided, then a fixed reduction tree), into a workspace array;
//   2. norm_reduce:   one CTA per tensor sums its tiles' partials in a fixed order;
//   3. clip_final:    per-tensor norms (sqrt, rounded to the gradients' dtype), their L2 norm
//      and the coefficient, with the roundings of clip_grad_norm_ for that dtype
//      (total + 1e-6, reciprocal, * max_norm, clamp at 1 -- torch/nn/utils/clip_grad.py).
// The per-tile partials are the only scratch memory; the caller provides it.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/abx.h"

#define ABX_API extern "C" __attribute__((visibility("default")))

namespace abx {
int set_error(const char* what, cudaError_t e);   // abx_kernels.cu
extern std::atomic<uint64_t> g_launches;
extern thread_local char g_err[512];
}

namespace abx_clip {

constexpr int kThreads = 256;
constexpr int kVec = 8;                          // elements per thread per load
constexpr int kNormTile = 16384;                 // elements per partial sum
constexpr int kIters = kNormTile / (kThreads * kVec);
constexpr int kMaxTensors = 64;                  // tensors per launch (parameter block)

struct NTensor {
    const void* data;
    int64_t n;
    int64_t tile_begin;   // first partial of this tensor in the workspace
    int32_t bf16;
    int32_t vec;          // 16-byte vector loads allowed
};

struct PartialArgs {
    int32_t ntensor;
    int32_t pad;
    int64_t first_tile;   // tile index of this launch's first tile
    int64_t total_tiles;  // tiles in this launch
    float* partial;
    NTensor t[kMaxTensors];
};

struct ReduceArgs {
    int32_t ntensor;
    int32_t first;        // index of this launch's first tensor in `sq`
    const float* partial;
    float* sq;            // per-tensor sums of squares
    int64_t tile_begin[kMaxTensors];
    int64_t tiles[kMaxTensors];
};

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// Sum over the block in a fixed association (xor butterfly inside warps, then across the 8 warp
// sums): every thread gets the same bits.  `ws` holds kThreads / 32 floats.
__device__ __forceinline__ float block_sum(float x, float* ws)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = __fadd_rn(x, __shfl_xor_sync(0xffffffffU, x, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();                      // ws free (a previous call may still read it)
    if (lane == 0) ws[warp] = x;
    __syncthreads();
    x = lane < kThreads / 32 ? ws[lane] : 0.0f;
#pragma unroll
    for (int o = (kThreads / 32) / 2; o > 0; o >>= 1) x = __fadd_rn(x, __shfl_xor_sync(0xffffffffU, x, o));
    return x;
}

__device__ __forceinline__ float sq_acc8(const NTensor& T, int64_t i0, float acc)
{
    float x[8];
    const int64_t left = T.n - i0;
    if (T.bf16) {
        const uint16_t* p = static_cast<const uint16_t*>(T.data) + i0;
        if (T.vec && left >= 8) {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
            const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) { x[2 * j] = u2f(w[j] << 16); x[2 * j + 1] = u2f(w[j] & 0xffff0000U); }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = k < left ? u2f((uint32_t)__ldg(p + k) << 16) : 0.0f;
        }
    } else {
        const float* p = static_cast<const float*>(T.data) + i0;
        if (T.vec && left >= 8) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(p));
            const float4 b = __ldg(reinterpret_cast<const float4*>(p + 4));
            x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = k < left ? __ldg(p + k) : 0.0f;
        }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) acc = __fmaf_rn(x[k], x[k], acc);
    return acc;
}

__global__ void __launch_bounds__(kThreads) norm_partials(const __grid_constant__ PartialArgs a)
{
    __shared__ float ws[kThreads / 32];
    for (int64_t t = blockIdx.x; t < a.total_tiles; t += gridDim.x) {
        int lo = 0, hi = a.ntensor - 1;
        const int64_t gt = a.first_tile + t;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (a.t[mid].tile_begin <= gt) lo = mid; else hi = mid - 1;
        }
        const NTensor& T = a.t[lo];
        const int64_t base = (gt - T.tile_begin) * kNormTile;
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < kIters; ++j) {
            const int64_t i0 = base + ((int64_t)j * kThreads + threadIdx.x) * kVec;
            if (i0 < T.n && i0 < base + kNormTile) acc = sq_acc8(T, i0, acc);
        }
        const float s = block_sum(acc, ws);
        if (threadIdx.x == 0) a.partial[gt] = s;
    }
}

__global__ void __launch_bounds__(kThreads) norm_reduce(const __grid_constant__ ReduceArgs a)
{
    __shared__ float ws[kThreads / 32];
    const int i = blockIdx.x;
    const int64_t b = a.tile_begin[i], n = a.tiles[i];
    float acc = 0.0f;
    for (int64_t k = threadIdx.x; k < n; k += kThreads) acc = __fadd_rn(acc, a.partial[b + k]);
    const float s = block_sum(acc, ws);
    if (threadIdx.x == 0) a.sq[a.first + i] = s;
}

__device__ __forceinline__ float round_bf16(float x)
{
    const uint32_t b = __float_as_uint(x);
    const uint32_t r = (b & 0x7fffffffU) > 0x7f800000U ? (b | 0x00400000U) : b + 0x7fffU + ((b >> 16) & 1U);
    return __uint_as_float(r & 0xffff0000U);
}

// norms[i] = sqrt(sq[i]) in the gradients' dtype; out[0] = ||norms||, out[1] = clip coefficient.
__global__ void __launch_bounds__(kThreads) clip_final(const float* sq, int32_t n, int32_t bf16, float max_norm,
                                                       float* norms, float* out)
{
    __shared__ float ws[kThreads / 32];
    float acc = 0.0f;
    for (int i = threadIdx.x; i < n; i += kThreads) {
        float v = __fsqrt_rn(sq[i]);
        if (bf16) v = round_bf16(v);
        if (norms) norms[i] = v;
        acc = __fmaf_rn(v, v, acc);
    }
    const float s = block_sum(acc, ws);
    if (threadIdx.x == 0) {
        float total = __fsqrt_rn(s);
        float x = __fadd_rn(bf16 ? round_bf16(total) : total, 1e-6f);
        if (bf16) { total = round_bf16(total); x = round_bf16(x); }
        float r = __frcp_rn(x);
        if (bf16) r = round_bf16(r);
        float coef = __fmul_rn(r, max_norm);
        if (bf16) coef = round_bf16(coef);
        coef = coef > 1.0f ? 1.0f : coef;          // clamp(max=1): NaN stays NaN
        out[0] = total;
        out[1] = coef;
    }
}

int64_t tiles_of(int64_t n) { return (n + kNormTile - 1) / kNormTile; }

}  // namespace abx_clip

using namespace abx_clip;

ABX_API size_t abx_clip_workspace_bytes(const abx_tensor* grads, int32_t n)
{
    if (!grads || n <= 0) return 256;
    int64_t tiles = 0;
    for (int32_t i = 0; i < n; ++i) tiles += grads[i].n > 0 ? tiles_of(grads[i].n) : 0;
    return (size_t)((tiles * 4 + 255) / 256 * 256 + 256);
}

static int grid_of(int64_t tiles)
{
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t g = (int64_t)sms * 8;
    return (int)(tiles < g ? tiles : g);
}

ABX_API int abx_grad_sq_norms(void* stream, const abx_tensor* grads, int32_t n, float* sq, void* workspace,
                              size_t workspace_bytes)
{
    if (n < 0 || (n > 0 && (!grads || !sq))) return ABX_E_ARG;
    if (n == 0) return ABX_OK;
    for (int32_t i = 0; i < n; ++i) {
        if (grads[i].n < 0) return ABX_E_ARG;
        if (grads[i].n > 0 && !grads[i].data) return ABX_E_NULL_PTR;
        if (grads[i].dtype != ABX_DT_F32 && grads[i].dtype != ABX_DT_BF16) return ABX_E_G_DTYPE;
        const uintptr_t es = grads[i].dtype == ABX_DT_BF16 ? 2 : 4;
        if (reinterpret_cast<uintptr_t>(grads[i].data) % es) return ABX_E_ALIGN;
    }
    if (!workspace || workspace_bytes < abx_clip_workspace_bytes(grads, n)) return ABX_E_OOM;
    if (reinterpret_cast<uintptr_t>(workspace) % 16 || reinterpret_cast<uintptr_t>(sq) % 4) return ABX_E_ALIGN;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* partial = static_cast<float*>(workspace);
    std::vector<int64_t> begin(n), tiles(n);
    int64_t total = 0;
    for (int32_t i = 0; i < n; ++i) {
        begin[i] = total;
        tiles[i] = grads[i].n > 0 ? tiles_of(grads[i].n) : 0;
        total += tiles[i];
    }
    for (int32_t b = 0; b < n; b += kMaxTensors) {
        const int cnt = n - b < kMaxTensors ? n - b : kMaxTensors;
        PartialArgs pa;
        std::memset(&pa, 0, sizeof pa);
        ReduceArgs ra;
        std::memset(&ra, 0, sizeof ra);
        int64_t t0 = begin[b], tl = 0;
        for (int j = 0; j < cnt; ++j) {
            const abx_tensor& g = grads[b + j];
            pa.t[j] = NTensor{g.data, g.n, begin[b + j], g.dtype == ABX_DT_BF16, (reinterpret_cast<uintptr_t>(g.data) % 16) == 0};
            tl += tiles[b + j];
            ra.tile_begin[j] = begin[b + j];
            ra.tiles[j] = tiles[b + j];
        }
        pa.ntensor = cnt;
        pa.first_tile = t0;      // the launch's tiles are t0 .. t0 + tl of the workspace
        pa.total_tiles = tl;
        pa.partial = partial;
        if (tl > 0) {
            norm_partials<<<grid_of(tl), kThreads, 0, st>>>(pa);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return abx::set_error("norm_partials launch", e);
            abx::g_launches.fetch_add(1, std::memory_order_relaxed);
        }
        ra.ntensor = cnt;
        ra.first = b;
        ra.partial = partial;
        ra.sq = sq;
        norm_reduce<<<cnt, kThreads, 0, st>>>(ra);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return abx::set_error("norm_reduce launch", e);
        abx::g_launches.fetch_add(1, std::memory_order_relaxed);
    }
    return ABX_OK;
}

ABX_API int abx_clip_coef_from_sq(void* stream, const float* sq, int32_t n, int32_t dtype, float max_norm,
                                  float* norms, float* total_coef)
{
    if (n <= 0 || !sq || !total_coef) return ABX_E_ARG;
    if (dtype != ABX_DT_F32 && dtype != ABX_DT_BF16) return ABX_E_G_DTYPE;
    clip_final<<<1, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(sq, n, dtype == ABX_DT_BF16, max_norm, norms,
                                                                       total_coef);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return abx::set_error("clip_final launch", e);
    abx::g_launches.fetch_add(1, std::memory_order_relaxed);
    return ABX_OK;
}

ABX_API int abx_clip_coef(void* stream, const abx_tensor* grads, int32_t n, float max_norm, float* sq, float* norms,
                          float* total_coef, void* workspace, size_t workspace_bytes)
{
    if (n <= 0 || !grads) return ABX_E_ARG;
    const int32_t dtype = grads[0].dtype;
    for (int32_t i = 1; i < n; ++i)
        if (grads[i].dtype != dtype) return ABX_E_G_DTYPE;   // torch rounds the norms in one dtype
    int rc = abx_grad_sq_norms(stream, grads, n, sq, workspace, workspace_bytes);
    if (rc) return rc;
    return abx_clip_coef_from_sq(stream, sq, n, dtype, max_norm, norms, total_coef);
}

// ---- abx_clip_coef_noalloc: abx_clip_coef with its scratch in this library's own device memory ----
//
// The per-tile partial sums live in a file-scope __device__ array of kNoAllocTiles floats (2 MiB per
// device, enough for 524,288 tiles of 16384 elements: about 8.59e9 gradient elements), so a call
// needs no caller workspace and allocates nothing, on the device or the host.  The array's device
// address is looked up with the device current on the first call in a CUDA context (this is also when
// the module's device code is loaded there): make that first call before any stream capture.  The
// address is kept per device together with the context it belongs to, and looked up again when the
// calling thread's context is another one (after cudaDeviceReset, or under a context that is not the
// device's primary one), where the module is loaded again, at another address.
// Every partial that a call reads was written earlier in the same call, so nothing needs to start at
// zero.  All calls on one device share the array: calls whose work overlaps on the device (issued
// to two streams, or from two host threads without ordering) race on it.

constexpr int64_t kNoAllocTiles = int64_t(1) << 19;
constexpr int kNoAllocDevices = 64;

__device__ __align__(256) float g_noalloc_partials[kNoAllocTiles];

struct NoAllocSlot {
    unsigned long long ctx = 0;   // unique id of the context the address belongs to
    float* addr = nullptr;
};

static std::mutex g_noalloc_mu;
static NoAllocSlot g_noalloc[kNoAllocDevices];

// The unique id of the calling thread's current CUDA context (0: none current yet, or the driver does not
// report ids), through driver entry points the runtime resolves -- the library does not link libcuda.
static unsigned long long current_context_id()
{
    using GetCurrent = int (*)(void**);
    using GetId = int (*)(void*, unsigned long long*);
    static std::once_flag once;
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(f);
    });
    void* ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != 0 || !ctx || get_id(ctx, &id) != 0) return 0;
    return id;
}

static int noalloc_scratch(float** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return abx::set_error("abx_clip_coef_noalloc: cudaGetDevice", e);
    if (dev < 0 || dev >= kNoAllocDevices)
        return abx::set_error("abx_clip_coef_noalloc: device index out of range", cudaErrorInvalidDevice);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocSlot& slot = g_noalloc[dev];
    const unsigned long long ctx = current_context_id();
    if (!slot.addr || ctx == 0 || slot.ctx != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_partials);   // with the device current; loads the module
        if (e != cudaSuccess) return abx::set_error("abx_clip_coef_noalloc: cudaGetSymbolAddress", e);
        slot.addr = static_cast<float*>(p);
        slot.ctx = current_context_id();                     // current now, if it was not before
    }
    *out = slot.addr;
    return ABX_OK;
}

// The launches of abx_grad_sq_norms, with the tile offsets kept as a running count (no host buffers).
static int sq_norms_into(cudaStream_t st, const abx_tensor* grads, int32_t n, float* sq, float* partial)
{
    int64_t next = 0;
    for (int32_t b = 0; b < n; b += kMaxTensors) {
        const int cnt = n - b < kMaxTensors ? n - b : kMaxTensors;
        PartialArgs pa;
        std::memset(&pa, 0, sizeof pa);
        ReduceArgs ra;
        std::memset(&ra, 0, sizeof ra);
        const int64_t t0 = next;
        for (int j = 0; j < cnt; ++j) {
            const abx_tensor& g = grads[b + j];
            const int64_t tiles = g.n > 0 ? tiles_of(g.n) : 0;
            pa.t[j] = NTensor{g.data, g.n, next, g.dtype == ABX_DT_BF16, (reinterpret_cast<uintptr_t>(g.data) % 16) == 0};
            ra.tile_begin[j] = next;
            ra.tiles[j] = tiles;
            next += tiles;
        }
        pa.ntensor = cnt;
        pa.first_tile = t0;
        pa.total_tiles = next - t0;
        pa.partial = partial;
        if (pa.total_tiles > 0) {
            norm_partials<<<grid_of(pa.total_tiles), kThreads, 0, st>>>(pa);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return abx::set_error("norm_partials launch", e);
            abx::g_launches.fetch_add(1, std::memory_order_relaxed);
        }
        ra.ntensor = cnt;
        ra.first = b;
        ra.partial = partial;
        ra.sq = sq;
        norm_reduce<<<cnt, kThreads, 0, st>>>(ra);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return abx::set_error("norm_reduce launch", e);
        abx::g_launches.fetch_add(1, std::memory_order_relaxed);
    }
    return ABX_OK;
}

ABX_API int abx_clip_coef_noalloc(void* stream, const abx_tensor* grads, int32_t n, float max_norm, float* sq,
                                  float* norms, float* total_coef)
{
    if (n <= 0 || !grads || !sq || !total_coef) return ABX_E_ARG;
    const int32_t dtype = grads[0].dtype;
    int64_t tiles = 0;
    for (int32_t i = 0; i < n; ++i) {
        const abx_tensor& g = grads[i];
        if (g.n < 0) return ABX_E_ARG;
        if (g.n > 0 && !g.data) return ABX_E_NULL_PTR;
        if (g.dtype != ABX_DT_F32 && g.dtype != ABX_DT_BF16) return ABX_E_G_DTYPE;
        if (g.dtype != dtype) return ABX_E_G_DTYPE;           // torch rounds the norms in one dtype
        if (reinterpret_cast<uintptr_t>(g.data) % (g.dtype == ABX_DT_BF16 ? 2 : 4)) return ABX_E_ALIGN;
        const int64_t t = g.n > 0 ? tiles_of(g.n) : 0;
        if (t > kNoAllocTiles - tiles) {
            snprintf(abx::g_err, sizeof abx::g_err,
                     "abx_clip_coef_noalloc: the gradients need more than %lld norm tiles of %d elements "
                     "(the static scratch); use abx_clip_coef with a workspace",
                     (long long)kNoAllocTiles, kNormTile);
            return ABX_E_SCRATCH;
        }
        tiles += t;
    }
    if (reinterpret_cast<uintptr_t>(sq) % 4 || reinterpret_cast<uintptr_t>(total_coef) % 4) return ABX_E_ALIGN;
    float* partial = nullptr;
    int rc = noalloc_scratch(&partial);
    if (rc) return rc;
    rc = sq_norms_into(static_cast<cudaStream_t>(stream), grads, n, sq, partial);
    if (rc) return rc;
    return abx_clip_coef_from_sq(stream, sq, n, dtype, max_norm, norms, total_coef);
}
