/*
 * abx.h -- C ABI of libabx, the B200 (sm_100a) fused optimizer-update library.
 *
 * libabx replaces the host SIMD kernel library of adambridge
 * (adambridge/csrc/adambridge_kernels.c) with CUDA kernels that update
 * optimizer state resident in HBM.  The structs, dtype codes, algorithm codes
 * and error codes below keep the reference's layout and meaning, so a binding
 * written for the reference (adambridge/native.py:58-111) needs only its
 * function names, its first argument (a CUDA stream instead of a thread pool)
 * and its pointers (device instead of host memory) changed.
 *
 * Conventions shared by every entry point:
 *   - Every pointer inside a segment is a DEVICE pointer on the current CUDA
 *     device of the calling thread.  The caller owns all memory; the kernels
 *     update p, m, v, the scales and out in place.
 *   - `stream` is a cudaStream_t (NULL: the legacy default stream).  Work is
 *     enqueued asynchronously; argument errors are returned synchronously
 *     BEFORE anything is launched, and on such an error nothing is updated.
 *   - Results are bit-identical to the reference's native kernels built for
 *     the SIMD level selected with abx_set_simd_level (default AVX-512): the
 *     reference fuses multiply-adds in its vector loop and not in its scalar
 *     tail, and libabx reproduces exactly which elements take which path.
 *   - No entry point allocates device memory; no entry point synchronizes.
 */
#ifndef ABX_H
#define ABX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ABX_ABI_VERSION 1

/* Element formats; same codes as the reference (adambridge_kernels.c:73, native.py:47-51). */
enum {
    ABX_DT_NONE = 0,  /* no buffer (out only) */
    ABX_DT_F32  = 1,
    ABX_DT_BF16 = 2,
    ABX_DT_FP8  = 3,  /* moments: E4M3fn m, E5M2 sqrt(v), one fp32 scale per 128 elements */
    ABX_DT_F24  = 4   /* master: bf16 hi plane + uint8 lo plane (top 24 bits of fp32) */
};

/* Update rules; same codes as the reference (adambridge_kernels.c:75). */
enum { ABX_ALGO_ADAMW = 0, ABX_ALGO_LION = 1 };

/* Rounding patterns of the reference's SIMD levels (adambridge_kernels.c:74).
 * AVX-512 / AVX2 / NEON fuse the multiply-adds of their 16 / 8 / 4-lane loop and
 * run the last n % lanes elements of a segment unfused; SCALAR fuses none. */
enum { ABX_SIMD_SCALAR = 0, ABX_SIMD_AVX2 = 1, ABX_SIMD_AVX512 = 2, ABX_SIMD_NEON = 3 };

#define ABX_FP8_BLOCK 128

/* Error codes.  -1 .. -13 have the reference's meaning (check_segment,
 * adambridge_kernels.c:1537-1553, and adambridge_multi_step :1611-1626). */
#define ABX_OK                 0
#define ABX_E_ARG             -1   /* NULL segment array / negative n / NULL hparams */
#define ABX_E_NULL_PTR        -2   /* a required buffer is NULL */
#define ABX_E_G_DTYPE         -3
#define ABX_E_MV_DTYPE        -4
#define ABX_E_OUT_DTYPE       -5
#define ABX_E_OUT_NULL        -6
#define ABX_E_SCALE_NULL      -7   /* FP8 moments without scales */
#define ABX_E_GROUP_NULL      -8
#define ABX_E_TOO_MANY        -9
#define ABX_E_OOM            -10
#define ABX_E_OFFSET         -11   /* negative offset, or FP8 offset not a multiple of 128 */
#define ABX_E_ALGO           -12
#define ABX_E_P_DTYPE        -13
/* libabx-specific */
#define ABX_E_CUDA           -20   /* a CUDA runtime call failed; see abx_last_error() */
#define ABX_E_ALIGN          -21   /* a buffer is not aligned to its element size */
#define ABX_E_SIMD_LEVEL     -22   /* unknown SIMD level */
#define ABX_E_SCRATCH        -23   /* more gradient than abx_clip_coef_noalloc's static scratch covers */

/* Per-step coefficients (adambridge_hparams, adambridge_kernels.c:77-88). */
typedef struct abx_hparams {
    float beta1;
    float beta2;
    float one_minus_beta1;
    float one_minus_beta2;
    float decay;         /* 1 - lr * weight_decay */
    float step_size;     /* AdamW: lr / (1 - beta1^t); Lion: lr */
    float inv_sqrt_bc2;  /* 1 / sqrt(1 - beta2^t) */
    float eps;
    uint32_t seed;       /* stochastic-rounding stream of this (param, step) */
    int32_t stochastic;  /* nonzero: stochastic rounding of bf16/fp8 moments and the fp24 master */
} abx_hparams;

/* Hyperparameters of one parameter group (adambridge_group, adambridge_kernels.c:736-745). */
typedef struct abx_group {
    double lr;
    double beta1;
    double beta2;
    double eps;
    double weight_decay;
    uint64_t seed;       /* base seed for stochastic rounding */
    int32_t stochastic;
    int32_t reserved;
} abx_group;

/* One tensor (or a 128-aligned chunk of one) to update (adambridge_segment,
 * adambridge_kernels.c:747-769).  All pointers are device pointers. */
typedef struct abx_segment {
    void* p;                 /* master: fp32 values, or the fp24 hi plane (uint16) when p_dtype is ABX_DT_F24 */
    uint8_t* p_lo;           /* fp24 only: the lo plane */
    const void* g;           /* gradient, g_dtype */
    void* m;                 /* first moment, mv_dtype (FP8: E4M3 codes, padded to whole 128-blocks) */
    void* v;                 /* second moment (FP8: E5M2 codes of sqrt(v)); unused by Lion */
    float* m_scale;          /* FP8 only: one scale per 128 elements */
    float* v_scale;
    void* out;               /* optional copy of the stored master in out_dtype (the model's weights) */
    const abx_group* group;  /* host pointer; read by abx_multi_step only */
    int64_t n;
    int64_t step;            /* this update's step number (the caller increments it) */
    uint64_t index;          /* parameter index: selects the rounding stream */
    int64_t offset;          /* element offset of p[0] within its parameter (FP8: a multiple of 128) */
    int32_t g_dtype;
    int32_t mv_dtype;
    int32_t out_dtype;
    int32_t algorithm;
    int32_t p_dtype;         /* ABX_DT_F32 (or 0) or ABX_DT_F24 */
    int32_t reserved;
} abx_segment;

/* ---- version and layout probes (replace adambridge_kernels.c:1493-1514) ---- */
int abx_abi_version(void);
int abx_hparams_size(void);
int abx_group_size(void);
int abx_segment_size(void);

/* ---- rounding pattern (replaces adambridge_set_simd_level / _simd_level /
 *      _detected_simd_level, adambridge_kernels.c:1495-1510) ----
 * Selects which reference build the kernels reproduce bit for bit.  Any level
 * may be chosen (it is an emulation target, not a CPU feature); -1 restores the
 * default, AVX-512.  Returns the level now active, or ABX_E_SIMD_LEVEL. */
int abx_set_simd_level(int level);
int abx_simd_level(void);
int abx_detected_simd_level(void);   /* the default level: ABX_SIMD_AVX512 */

/* ---- host-side coefficient and seed computation (adambridge_kernels.c:773-809),
 *      exposed so bindings and tests can check them ---- */
uint32_t abx_step_seed(uint64_t base_seed, uint64_t index, int64_t step);
int abx_hparams_for(const abx_segment* seg, abx_hparams* out);

/* ---- updates ----
 * abx_multi_step (replaces adambridge_multi_step, adambridge_kernels.c:1611):
 *   validates every segment, derives each one's coefficients from its group and
 *   step in double precision, and enqueues the updates on `stream`.  Segments of
 *   any size, dtype mix and algorithm may be mixed; one kernel launch covers up
 *   to 64 segments of one dtype combination.  `max_ctas` caps the CTAs per launch
 *   (0: one wave of resident CTAs on every SM); it plays the role of the
 *   reference's `threads` argument, leaving SMs to concurrent work.
 * abx_multi_apply (replaces adambridge_multi_apply, :1630): the same with
 *   caller-supplied coefficients hps[i] for segs[i]; groups and steps are ignored.
 * abx_multi_step_scaled / abx_multi_apply_scaled: as above, and every gradient
 *   element is first multiplied by the device scalar *g_scale (gradient clipping
 *   or loss unscaling fused into the update), as an in-place torch multiply of
 *   the CUDA gradient by an fp32 scalar tensor leaves it: a bf16 gradient is
 *   multiplied by *g_scale rounded to bf16, and the product rounded to bf16.
 *   g_scale NULL means 1.  Not in the reference: its callers scale the
 *   gradient in place before calling it.
 */
int abx_multi_step(void* stream, abx_segment* const* segs, int32_t nsegs, int32_t max_ctas);
int abx_multi_apply(void* stream, abx_segment* const* segs, const abx_hparams* hps, int32_t nsegs,
                    int32_t max_ctas);
int abx_multi_step_scaled(void* stream, abx_segment* const* segs, int32_t nsegs, int32_t max_ctas,
                          const float* g_scale);
int abx_multi_apply_scaled(void* stream, abx_segment* const* segs, const abx_hparams* hps, int32_t nsegs,
                           int32_t max_ctas, const float* g_scale);

/* abx_multi_step_replicated: abx_multi_step_scaled, and every `out` element is also stored at
 * out + out_deltas[j] bytes for j < nreplicas (at most 7; each a multiple of 16).  With a weight
 * buffer mapped at the same offsets on every GPU of a node (peer / symmetric memory), the deltas
 * are the distances from this GPU's buffer to the peers': the sharded update then writes its new
 * weights into every peer's copy over NVLink -- an all-gather fused into the update, with plain
 * stores.  The caller orders the peers' later reads after the update (a barrier across ranks).
 * Not in the reference (no multi-GPU code). */
int abx_multi_step_replicated(void* stream, abx_segment* const* segs, int32_t nsegs, int32_t max_ctas,
                              const float* g_scale, const int64_t* out_deltas, int32_t nreplicas);

/* abx_replicate_async: the copy-engine form of that all-gather.  Copies `bytes` bytes at src to
 * src + deltas[j] (0 <= j < nreplicas <= 7) with one asynchronous copy on streams[j] each, so the
 * copy engines carry the weights to the peers while the SMs run the next update.  A replica may
 * not overlap the source (ABX_E_ARG).  The caller orders each stream after the update that wrote
 * src, and the peers' later reads after the copies.  Not in the reference. */
int abx_replicate_async(void* const* streams, const void* src, int64_t bytes, const int64_t* deltas,
                        int32_t nreplicas);

/* Single-tensor AdamW with fp32/bf16 moments and an fp32 master (replaces
 * adambridge_fused_adamw, adambridge_kernels.c:1518, same argument meaning and
 * error codes, plus the stream). */
int abx_fused_adamw(float* p, const void* g, int g_dtype, void* m, void* v, int mv_dtype, void* out,
                    int out_dtype, int64_t n, uint64_t offset, const abx_hparams* hp, void* stream);

/* ---- gradient norms and the clipping coefficient (not in the reference: its callers run
 *      torch.nn.utils.clip_grad_norm_, which reads the gradients once for the norm and then reads
 *      and writes them again to scale them) ----
 * abx_clip_coef computes on the device, without a host synchronization:
 *   sq[i]    = sum of squares of gradient i (fp32, fixed order: deterministic),
 *   norms[i] = sqrt(sq[i]) rounded to the gradients' dtype (may be NULL),
 *   total_coef[0] = the L2 norm of the norms, total_coef[1] = min(max_norm / (total + 1e-6), 1),
 * each rounded as clip_grad_norm_ rounds it for that dtype (all gradients share one dtype).
 * total_coef + 1 can be passed as abx_multi_step_scaled's g_scale: the update then applies the
 * clipping while it reads the gradient.  `workspace` is device scratch of at least
 * abx_clip_workspace_bytes(grads, n) bytes (16-byte aligned); too small: ABX_E_OOM.
 * abx_grad_sq_norms / abx_clip_coef_from_sq are the two halves, for callers that sum the squared
 * norms of sharded gradients across ranks in between. */
typedef struct abx_tensor {
    const void* data;    /* device pointer */
    int64_t n;
    int32_t dtype;       /* ABX_DT_F32 or ABX_DT_BF16 */
    int32_t reserved;
} abx_tensor;

size_t abx_clip_workspace_bytes(const abx_tensor* grads, int32_t n);
int abx_grad_sq_norms(void* stream, const abx_tensor* grads, int32_t n, float* sq, void* workspace,
                      size_t workspace_bytes);
int abx_clip_coef_from_sq(void* stream, const float* sq, int32_t n, int32_t dtype, float max_norm, float* norms,
                          float* total_coef);
int abx_clip_coef(void* stream, const abx_tensor* grads, int32_t n, float max_norm, float* sq, float* norms,
                  float* total_coef, void* workspace, size_t workspace_bytes);

/* abx_clip_coef without a caller workspace.  No counterpart in the reference (adambridge has no
 * device-side norm: its callers run torch.nn.utils.clip_grad_norm_).  For callers that cannot
 * allocate device memory: a C or FFI host that only holds the device pointers a framework gave it
 * and has no CUDA allocator of its own, or a training loop that reserved its device memory up
 * front and must not allocate per step (an allocation there can fail or fragment the pool).  The
 * per-tile partial sums live in a static device array inside this library (2 MiB on every device
 * that loads it, held until exit), so the call allocates nothing: no cudaMalloc, no caller buffer
 * beyond its outputs sq, norms (may be NULL) and total_coef, whose meaning is abx_clip_coef's.
 *   Limit: the gradients' 16384-element tiles, the sum of ceil(n_i / 16384), must number at most
 *   524,288 (about 8.59e9 elements); more is rejected before anything runs, with ABX_E_SCRATCH
 *   and a message in abx_last_error().
 *   Set-up: the first call on each device looks up the array's address (cudaGetSymbolAddress,
 *   with that device current); make that first call before any stream capture.  The address
 *   belongs to a CUDA context: a call under another context than the one it was looked up in
 *   (after cudaDeviceReset, or a non-primary context) looks it up again, as a first call does.
 *   Nothing needs to start at zero: every partial a call reads was written earlier in that call.
 *   All calls on one device share the array: calls whose work overlaps on the device (two
 *   streams, or two host threads without ordering between them) race on it. */
int abx_clip_coef_noalloc(void* stream, const abx_tensor* grads, int32_t n, float max_norm, float* sq, float* norms,
                          float* total_coef);

/* One optimizer-state buffer for abx_convert: n values stored in one of the state
 * formats.  No counterpart struct in the reference, whose stores are torch tensors
 * (adambridge/precision.py:286-480); the planes and their meaning are its formats. */
typedef struct abx_state {
    void* values;     /* ABX_DT_F32: float[n]; ABX_DT_BF16: bf16 bits uint16[n];
                         ABX_DT_FP8: codes uint8[nblocks * block] (padded to whole blocks);
                         ABX_DT_F24: the hi plane, bf16 bits uint16[n] */
    void* aux;        /* ABX_DT_FP8: float scale[nblocks]; ABX_DT_F24: the lo plane uint8[n]; else NULL */
    int32_t dtype;    /* ABX_DT_F32, ABX_DT_BF16, ABX_DT_FP8 or ABX_DT_F24 */
    int32_t role;     /* ABX_DT_FP8 only: 0 = first moment (E4M3 codes of m),
                         1 = second moment (E5M2 codes of sqrt(v)) */
    int64_t block;    /* ABX_DT_FP8 only: values per scale; a destination must use ABX_FP8_BLOCK,
                         a source any block in [1, 2^20] */
} abx_state;

/* Convert n values from src to dst (distinct buffers) on `stream`: each value is decoded
 * to fp32 and re-encoded in dst's format with round-to-nearest-even, as the reference's
 * own conversions round (adambridge/precision.py: BF16Store.write :319-323 and torch's
 * bfloat16 cast, FP8Store.read/write :374-398 without a seed -- a second moment kept as
 * sqrt(max(v, 0)), scale = block absmax / 448 or / 57344 (1 for an all-zero or NaN
 * block), values divided, clamped to the format's range and cast --, FP24Store.read/
 * write :448-462).  NaN becomes 0x7fc0 in bf16 and code 0x7f (with its sign) in FP8, as
 * torch's casts give them.  An FP8 destination's padding codes (up to the block end) are
 * written as 0.  No counterpart entry point in the reference (it converts with torch on
 * the host).  Errors before launch: ABX_E_ARG (n < 0, a bad role or block),
 * ABX_E_MV_DTYPE, ABX_E_NULL_PTR, ABX_E_SCALE_NULL (FP8 scales or the fp24 lo plane
 * missing), ABX_E_ALIGN; ABX_E_CUDA on a launch failure. */
int abx_convert(void* stream, const abx_state* src, const abx_state* dst, int64_t n);

/* Kernel launches this library has made in this process, all threads and devices. */
uint64_t abx_launch_count(void);

/* The update kernels stream tiles through shared memory behind mbarrier waits,
 * each bounded: a wait that gives up (never in correct operation) makes its CTA
 * drain its copies and exit, and ORs a bit into a status word held in pinned host
 * memory mapped into every device (1: a consumer's wait for a tile, 2: the
 * producer's wait for a free stage, 4: the producer's wait for its last copies).
 * No counterpart in the reference (its host kernels do not wait).
 * abx_pipeline_status returns the word and clears it (nonzero: some update since
 * the last call is incomplete), or ABX_E_CUDA if the word cannot be allocated.  It
 * does not synchronize: it covers the kernels that have finished by then. */
int abx_pipeline_status(void);

/* Host address of the status word, for callers that poll it without any CUDA
 * call (NULL if it cannot be allocated).  No counterpart in the reference. */
const volatile unsigned int* abx_status_word(void);

/* Failure-path testing only; no counterpart in the reference.  The next launch's
 * producer leaves tile `tile` of its tile space (2048-element tiles of all its
 * segments, in order) untouched -- no copy into its ring stage, no arrival on its
 * barrier -- and from now on every wait gives up after `spin_limit` polls (0: the
 * default, 2^22).  The consumers of that tile give up, the status word is set and
 * the rest of that CTA's tiles are left unupdated: the effect of a pipeline fault
 * without one.  tile < 0 cancels a pending skip.  Returns ABX_OK. */
int abx_test_pipeline_fault(int64_t tile, uint32_t spin_limit);

/* Message of the last ABX_E_CUDA / ABX_E_ALIGN / ABX_E_SCRATCH error on this thread (never NULL). */
const char* abx_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* ABX_H */
