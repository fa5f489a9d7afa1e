/* C ABI of the B200 (sm_100a) AudioVAE2 decoder hot path.
 *
 * This library replaces the decoder step of bevenky/fast-audiovae for
 * device="cuda". The reference drives that step from Python:
 *   - batch:     GPUDecoder.decode -> _run -> model.decode          (src/fast_audiovae/gpu.py:157-194)
 *   - streaming: GPUStream.decode_chunk -> _run, history committed on success
 *                                                                   (src/fast_audiovae/gpu.py:216-225)
 *   - the step:  MPSModel.decode(z, states) -> (audio, next_states)  (src/fast_audiovae/mps_decoder.py:309-325)
 * and its native libraries follow the conventions kept here: a versioned ABI,
 * int32 status codes, a thread-local last-error string, caller-owned buffers,
 * no hidden mutable stream state and immutable plans
 * (native/x86/native_kernels.h:16-106; experiments/intel-precision/native/precision.h:12-46).
 *
 * Conventions
 *   - Every function returns an fav_status (0 = FAV_OK) unless noted.
 *   - Device buffers are raw CUDA device pointers owned by the caller.
 *   - A plan belongs to the device that was current when it was created; every
 *     call that takes a plan must run with that device current
 *     (FAV_INVALID_ARGUMENT otherwise).
 *   - Work is enqueued on the caller's cudaStream_t (passed as void*); calls
 *     return without synchronising. Kernel-side failures (a bounded wait that
 *     expired) are reported through the caller's device status word.
 *   - Layouts: latents [streams][64][frames] fp32 (the reference's [1,64,L]
 *     per stream); audio [streams][1920*frames] fp32.
 *   - Causal history ("state") lives in a caller-allocated device pool of
 *     num_slots x FAV_SLOT_STRIDE_FLOATS fp32 (zero-initialised is not
 *     required). Each of a stream's 26 histories (H rows x C channels, the
 *     reference's inventory, mps_decoder.py:174-181) is a ring of 2H rows whose
 *     window starts at a head index; every slot ends in two head tables. A step
 *     reads the heads of the table its slot code names, writes new rows only
 *     into ring rows outside the current window and writes the advanced heads
 *     to the other table, so a failed step leaves the committed history
 *     untouched; the caller flips the stream's read table only after the step
 *     succeeded.
 */
#ifndef FAST_AUDIOVAE_CUDA_H
#define FAST_AUDIOVAE_CUDA_H
#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FAV_API __attribute__((visibility("default")))
#else
#define FAV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FAV_ABI_VERSION 1
/* Floats of causal history window per stream: the reference's 26 histories,
 * 647,424 bytes (mps_decoder.py:174-181, :280). */
#define FAV_SLOT_FLOATS 161856
/* Floats one stream slot occupies in a history pool: rings of twice the
 * window plus two head tables of 32 int32. */
#define FAV_SLOT_STRIDE_FLOATS (2 * FAV_SLOT_FLOATS + 64)
/* Number of coefficient arrays create_plan expects (order below). */
#define FAV_NUM_COEFFICIENTS 188

typedef enum fav_status {
  FAV_OK = 0,
  FAV_INVALID_ARGUMENT = 1,
  FAV_UNSUPPORTED = 2,
  FAV_OVERLAP = 3,
  FAV_SIZE_OVERFLOW = 4,
  FAV_DEVICE_ERROR = 5,
  FAV_TIMEOUT = 6
} fav_status;

typedef enum fav_precision {
  /* Stem 1x1 and transposed convs: split-bf16 operands (three bf16 MMAs,
   * hi*hi + hi*lo + lo*hi) with fp32 accumulation; residual 1x1s: f16
   * operands, fp32 accumulation; everything else fp32. */
  FAV_PRECISION_BF16 = 0,
  /* The reference's int8 recipe (experiments/intel-precision: precision.cpp
   * ip_create / ip_prepare / ip_run_rows, selection tools/rewrite.py:19-30):
   * every projection with min(rows, cols) >= 128 (transposed convs of stages
   * 0-4, one matrix per tap; residual 1x1s of stages 0-3) runs W8A8 on s8
   * tensor cores: per-row weight scales, per-time-step activation scales over
   * all input channels, round half to even, exact s32 dot, fp32 rescale. The
   * other layers run as FAV_PRECISION_BF16. */
  FAV_PRECISION_INT8 = 1
} fav_precision;

typedef struct fav_plan fav_plan;

/* ABI version (FAV_ABI_VERSION). Replaces ncc_abi_version / ip_abi
 * (native/x86/native_kernels.h:34; precision.h:27). */
FAV_API int32_t fav_abi_version(void);
/* Thread-local message of the last failing call on this thread
 * (native_kernels.h:39 ncc_status_string; precision.h:31 ip_last_error). */
FAV_API const char *fav_last_error(void);
FAV_API const char *fav_status_string(int32_t status);
/* 1 when the current CUDA device is a B200-class sm_100 part. */
FAV_API int32_t fav_device_supported(void);
/* Device address (cudaHostGetDevicePointer) of page-locked, mapped host
 * memory, so that a step's audio can be that host buffer: the kernels then
 * write the samples to the host as they finish and no device-to-host copy
 * follows. FAV_DEVICE_ERROR when `host` is not such memory. No counterpart in
 * the reference, whose GPU route copies its output tensor to the host
 * (gpu.py:177-185). */
FAV_API int32_t fav_host_device_pointer(void *host, void **device);

/* Immutable weight plan on the current device from FAV_NUM_COEFFICIENTS host
 * fp32 arrays, replacing MPSModel.from_onnx's coefficient load
 * (mps_decoder.py:190-286) and ip_create's weight preparation
 * (precision.cpp:343-380). Order (shapes as in the reference graph):
 *   0 stem.weight [64,1,7]   1 stem.bias [64]   2 pointwise.weight [2048,64,1]
 *   3 pointwise.bias [2048]
 *   stage i = 0..5, base 4 + 30*i, C_in = 2048>>i, C_out = C_in/2, s = (8,6,5,2,2,2)[i]:
 *     +0 scale [C_in] +1 offset [C_in] +2 snake.alpha [C_in] +3 snake.reciprocal [C_in]
 *     +4 transpose.weight [C_in,C_out,2s] +5 transpose.bias [C_out]
 *     residual j = 0..2 (dilation 1,3,9), +6+8j:
 *       pre.alpha, pre.reciprocal [C_out], depthwise.weight [C_out,1,7],
 *       depthwise.bias [C_out], post.alpha, post.reciprocal [C_out],
 *       pointwise.weight [C_out,C_out,1], pointwise.bias [C_out]
 *   184 final.snake.alpha [32] 185 final.snake.reciprocal [32]
 *   186 final.weight [1,32,7] 187 final.bias [1]
 * Coefficients must be finite. The plan is safe for concurrent use. */
FAV_API int32_t fav_plan_create(const float *const *coefficients, int32_t count, int32_t precision,
                                fav_plan **plan_out);
FAV_API void fav_plan_destroy(fav_plan *plan);
/* Device bytes held by the plan (packed weights and coefficients). */
FAV_API size_t fav_plan_bytes(const fav_plan *plan);

/* Bytes of a history pool with num_slots stream slots. */
FAV_API size_t fav_state_pool_bytes(int32_t num_slots);
/* Workspace bytes one fav_step with n_streams x frames needs. */
FAV_API size_t fav_step_workspace_bytes(int32_t n_streams, int32_t frames);
/* Workspace bytes one fav_step with this plan needs (fav_step_workspace_bytes
 * for either precision; kept so that callers need not know the plan's). */
FAV_API size_t fav_plan_workspace_bytes(const fav_plan *plan, int32_t n_streams, int32_t frames);
/* The plan's precision (fav_precision), -1 for NULL. */
FAV_API int32_t fav_plan_precision(const fav_plan *plan);

/* One decoder step for n_streams independent streams, each decoding `frames`
 * new latent frames (the reference's MPSModel.decode(z, states) for a batch of
 * streams; mps_decoder.py:309-325, gpu.py:157-185).
 *   slot_codes (device int32[n_streams]): (slot << 2) | (fresh << 1) | read_table.
 *     fresh=1 starts the stream from zero history (reference decode(z, {})).
 *     The advanced heads are written to head table (read_table ^ 1) of `slot`.
 *   latents [n_streams][64][frames], audio [n_streams][1920*frames] (device).
 *   workspace: >= fav_plan_workspace_bytes(plan, n_streams, frames) device bytes.
 *   status: device uint32 word, 0 on entry; nonzero after the step means a
 *     kernel gave up a bounded wait (FAV_TIMEOUT class failure). May be NULL.
 * Slots in one call must be distinct. */
FAV_API int32_t fav_step(const fav_plan *plan, float *state_pool, int32_t num_slots, const int32_t *slot_codes,
                         int32_t n_streams, int32_t frames, const float *latents, float *audio, void *workspace,
                         size_t workspace_bytes, uint32_t *status, void *cuda_stream);

/* Largest n_streams * frames one fav_step_static call accepts. */
#define FAV_STATIC_MAX_FRAMES 16

/* fav_step without a caller workspace and without any allocation. This entry
 * point has no counterpart in the reference. It serves callers that cannot
 * allocate device memory while they decode: a real-time audio callback (a
 * plugin's render thread, a telephony media loop) must not call cudaMalloc,
 * which can synchronise the device and block for an unbounded time, and some
 * hosts own all device memory and forbid allocation after start-up. The caller
 * still passes the plan, history pool, slot codes, latents and audio.
 * The step's scratch is a library-owned, file-scope device array sized for
 * n_streams * frames <= FAV_STATIC_MAX_FRAMES (22.5 MiB, held on every GPU
 * that loads the library until the process exits); larger calls are rejected
 * with FAV_SIZE_OVERFLOW. Either precision. The first call on a device looks up that array's
 * device address (cudaGetSymbolAddress) with the device current; make that
 * first call before any stream capture. Every call shares the one array and
 * it keeps the last call's contents (nothing in it needs to start at zero:
 * a step writes every scratch element before reading it), so calls that
 * overlap on the GPU (two streams, two threads) race: serialise them. */
FAV_API int32_t fav_step_static(const fav_plan *plan, float *state_pool, int32_t num_slots,
                                const int32_t *slot_codes, int32_t n_streams, int32_t frames,
                                const float *latents, float *audio, uint32_t *status, void *cuda_stream);

/* Workspace bytes fav_decode_batch needs for n_clips clips decoded in chunks
 * of chunk_frames frames (activations plus a temporary history pool). */
FAV_API size_t fav_batch_workspace_bytes(int32_t n_clips, int32_t chunk_frames);
/* fav_decode_batch workspace for this plan (see fav_plan_workspace_bytes). */
FAV_API size_t fav_plan_batch_workspace_bytes(const fav_plan *plan, int32_t n_clips, int32_t chunk_frames);
/* Batch decode of n_clips independent clips [n_clips][64][frames] from zero
 * history (reference GPUDecoder.decode, gpu.py:187-194). Long clips are
 * decoded in chunks of chunk_frames with carried history, which gives the same
 * bits as one call. */
FAV_API int32_t fav_decode_batch(const fav_plan *plan, const float *latents, int32_t n_clips, int32_t frames,
                                 int32_t chunk_frames, float *audio, void *workspace, size_t workspace_bytes,
                                 uint32_t *status, void *cuda_stream);

/* fav_step with per-layer timing (no reference counterpart; the reference
 * profiles ORT operators instead, benchmarks/profile_candidate.py:37-60):
 * CUDA events recorded on cuda_stream around each of the 26 layers;
 * layer_ms[26] receives their durations (0 = stem, 1+4i = stage i transposed
 * conv, 2+4i+j = stage i residual j, 25 = final conv). A stage 0-1 residual
 * unit's interval covers its depthwise pre-pass and its GEMM; stage 5's fused
 * kernel (three residual units and the final conv) counts as layer 22, and
 * layers 23-25 then read zero. Synchronises. */
FAV_API int32_t fav_step_profile(const fav_plan *plan, float *state_pool, int32_t num_slots,
                                 const int32_t *slot_codes, int32_t n_streams, int32_t frames,
                                 const float *latents, float *audio, void *workspace, size_t workspace_bytes,
                                 uint32_t *status, float *layer_ms, void *cuda_stream);

/* Diagnostic (no reference counterpart): run one step's layers 0..last_layer
 * (0 = stem, 1+4i = stage i transposed conv, 2+4i+j = stage i residual j,
 * last_layer <= 24) and return in *layer_out the device pointer, inside the
 * workspace, of that layer's fp32 output [n_streams * rows_per_stream][C]
 * (channels last). A NULL state_pool runs every stream from zero history. */
FAV_API int32_t fav_debug_step_layers(const fav_plan *plan, float *state_pool, int32_t num_slots,
                                      const int32_t *slot_codes, int32_t n_streams, int32_t frames,
                                      const float *latents, void *workspace, size_t workspace_bytes,
                                      uint32_t *status, int32_t last_layer, float **layer_out, void *cuda_stream);

/* Diagnostic (no reference counterpart): fav_step with every layer as its own
 * kernel (stage 5's residual units and the final conv unfused), for checking
 * the fused stage-5 kernel against the per-layer kernels. Same arguments and
 * contract as fav_step. */
FAV_API int32_t fav_debug_step_unfused(const fav_plan *plan, float *state_pool, int32_t num_slots,
                                       const int32_t *slot_codes, int32_t n_streams, int32_t frames,
                                       const float *latents, float *audio, void *workspace, size_t workspace_bytes,
                                       uint32_t *status, void *cuda_stream);

/* Diagnostic (no reference counterpart; the reference's transactional contract
 * is gpu.py:216-225): fav_step in which the GEMM-engine launch of `layer`
 * (0 = stem, 1+4i = stage i transposed conv, 2+4i+j = stage i residual unit j;
 * at most 21) gives up every mbarrier wait after `wait_limit` polls and whose
 * MMA issuer first waits for the device flag `gate` to become nonzero (a
 * residual unit of a stage that the step runs as one fused kernel names that
 * kernel). With a
 * gate that nothing sets, every role of that launch runs out of its waits: the
 * kernel drains the copies and MMAs it started, records a timeout code
 * (0x101-0x104, 0x107) in `status` (required here) and returns; the later
 * layers run on whatever the workspace holds. As with any failed step, the
 * history windows the slot codes name stay committed. FAV_PRECISION_BF16 plans
 * only. Same other arguments as fav_step. */
FAV_API int32_t fav_debug_step_gated(const fav_plan *plan, float *state_pool, int32_t num_slots,
                                     const int32_t *slot_codes, int32_t n_streams, int32_t frames,
                                     const float *latents, float *audio, void *workspace, size_t workspace_bytes,
                                     uint32_t *status, int32_t layer, uint32_t wait_limit, const uint32_t *gate,
                                     void *cuda_stream);

/* Engine self-test (diagnostic, no reference counterpart): C[M][N] = A[M][K] * B[N][K]^T
 * through the tcgen05 GEMM engine. a, c device fp32; b host fp32.
 * mode 0 = f16 operands, 1 = split-bf16, 2 = s8 (A and B hold integers in
 * [-127, 127]; C is the exact integer product). Synchronises. */
FAV_API int32_t fav_test_gemm(const float *a, int32_t m, int32_t k, const float *b, int32_t n, int32_t mode,
                              float *c, void *cuda_stream);

/* Diagnostic (no reference counterpart): out[i] = the fixed-order sine the
 * int8 path's Snake uses (Cody-Waite reduction, Taylor polynomials; the int8
 * oracle's oracle/exact.py sin_cw), for device arrays x and out of n floats.
 * Asynchronous on cuda_stream. */
FAV_API int32_t fav_test_sine(const float *x, int32_t n, float *out, void *cuda_stream);

#ifdef __cplusplus
}
#endif
#endif
