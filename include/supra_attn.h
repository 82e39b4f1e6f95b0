/*
 * libsupra_attn — C ABI of the B200 (sm_100a) fused attention operator of Supra2-Img.
 *
 * The operator surface mirrors the reference's JavaScript entry point
 *   attention(gpu, {q, k, v, Lq, Lk, H, D, ldq, ldk, ldv, qOff, kOff, vOff, oOff, scale, bias, out})
 * (app/gpu/ops.js:103-149) and the runtime it records into (app/gpu/device.js:41-269):
 *
 *   - q is [Lq, ldq] row-major fp32; head h of query row i is q[qOff + i*ldq + h*D + 0..D).
 *     k / v likewise with ldk / ldv and kOff / vOff, over Lk key rows.
 *   - The output row i is written at out[oOff + i*(H*D) + h*D + 0..D): row stride H*D.
 *   - scale multiplies the scores; the reference's default is 1/sqrt(D) (app/gpu/ops.js:109).
 *   - bias, when present, is an additive score bias laid out [H, Lq, Lk] (T5 relative
 *     positions, app/models/t5.js:55-65); it is added after scaling (app/gpu/kernels.js:34).
 *   - All offsets, strides and sizes are in ELEMENTS (floats), never bytes.
 *
 * Execution model ("record now, submit at flush", app/gpu/device.js:1-5,207-253):
 *   supra_attn_enqueue() validates a problem synchronously and records it; nothing runs yet.
 *   supra_attn_flush() groups every recorded problem by kernel configuration and issues one
 *   grouped launch per group on the context's stream; supra_attn_sync() waits and reports
 *   device-side failures (the reference surfaces asynchronous errors at read/sync,
 *   app/gpu/device.js:186,258,262-268). A recorded problem that reads memory written by an
 *   earlier recorded problem (or writes memory an earlier one touches) flushes the queue
 *   first, so results never depend on grouping.
 *
 * Every function returns a status code (SUPRA_ATTN_OK on success) and never throws or aborts.
 * supra_attn_last_error() returns the message of the most recent failure on a context.
 * A context is bound to one device and is not thread-safe (one context per host thread),
 * like the reference's single-threaded GPU object.
 */
#ifndef SUPRA_ATTN_H
#define SUPRA_ATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SUPRA_ATTN_API __attribute__((visibility("default")))
#else
#define SUPRA_ATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------- */
#define SUPRA_ATTN_OK 0
#define SUPRA_ATTN_EINVAL 1   /* bad argument: sizes, alignment, bounds, aliasing, unknown flag */
#define SUPRA_ATTN_ENOMEM 2   /* device or pinned host allocation failed                      */
#define SUPRA_ATTN_ECUDA 3    /* a CUDA runtime/driver call failed                            */
#define SUPRA_ATTN_ETIMEOUT 4 /* a device-side bounded wait ran out (reported at sync)        */
#define SUPRA_ATTN_EDEVICE 5  /* the device reported an error status (reported at sync)       */
#define SUPRA_ATTN_ESTATE 6   /* call not allowed in the context's current state              */

/* ---- numeric variants -------------------------------------------------------------------- */
#define SUPRA_ATTN_FP32 0 /* FFMA kernel, fp32 throughout: matches torch CPU fp32 to <=1e-5 */
/* tcgen05 tensor-core kernel with TF32 operands, fp32 accumulate. Covers head dim 64 with
 * whole-row, 16-byte aligned buffers (fused kernel, with or without a bias), and head dims above
 * 128 without a bias and with Lk >= 32 (Q K^T and P V on the tensor-core linear, the row softmax
 * between them); other requests run the FP32 kernels. */
#define SUPRA_ATTN_TF32 1
/* tcgen05 kernels with every operand split x = hi + lo (hi = TF32(x), lo = x - hi) and each
 * product formed as lo*hi + hi*lo + hi*hi ("3xTF32"): fp32-class accuracy on the tensor cores.
 * Same coverage as SUPRA_ATTN_TF32; other requests run the FP32 kernels. */
#define SUPRA_ATTN_TF32X3 2

/* ---- descriptor flags -------------------------------------------------------------------- */
#define SUPRA_ATTN_F_DEFAULT_SCALE 0x1u /* ignore .scale, use 1/sqrt(D) (ops.js:109 default) */
/* .bias is T5's relative-attention-bias TABLE, not an expanded bias: bias points at
 * bias_size >= buckets*H floats laid out [buckets, H] (encoder.block.0...relative_attention_bias
 * .weight, app/models/t5.js:44), and the kernels form the score bias themselves as
 *   bias[h, i, j] = table[relativeBucket(j - i)*H + h]   (app/models/t5.js:14-23,55-65)
 * with the bidirectional bucket of supra_attn_relative_bucket. .bias_param carries the bucket
 * parameters: buckets in bits 0-15, max_distance in bits 16-31. Not in the reference: its T5
 * builds the [H, L, L] bias on the host and uploads it per encode (app/models/t5.js:73); this
 * saves those 4*H*L*L bytes per prompt and the host loop. */
#define SUPRA_ATTN_F_T5_TABLE 0x2u

typedef struct supra_attn_ctx supra_attn_ctx;

/*
 * One attention problem: all H heads of one call of ops.attention (app/gpu/ops.js:109).
 * The *_size fields give the number of floats the caller owns at each pointer; every
 * element the problem reads or writes is checked against them at enqueue, so an
 * out-of-range offset is an EINVAL instead of a device fault. Pass 0 only for bias when
 * bias is NULL.
 */
typedef struct supra_attn_desc {
  const float* q;
  const float* k;
  const float* v;
  float* out;
  const float* bias; /* NULL, [H, Lq, Lk] additive score bias, or a T5 table (SUPRA_ATTN_F_T5_TABLE) */
  int64_t q_size, k_size, v_size, out_size, bias_size;
  int64_t ldq, ldk, ldv;
  int64_t q_off, k_off, v_off, o_off;
  int32_t Lq, Lk, H, D;
  float scale;
  int32_t variant; /* SUPRA_ATTN_FP32, SUPRA_ATTN_TF32 or SUPRA_ATTN_TF32X3 */
  uint32_t flags;  /* SUPRA_ATTN_F_* */
  uint32_t bias_param; /* with SUPRA_ATTN_F_T5_TABLE: buckets | max_distance << 16; else 0 */
} supra_attn_desc;

/* ---- context ----------------------------------------------------------------------------- */
/* Replaces GPU.create (app/gpu/device.js:92-118): binds a context to a CUDA device and
 * creates its stream, descriptor ring and device status word. Its first attention flush adds a
 * device table of TMA tensor maps (2 MiB, kept for the context's life; larger only if one flush
 * needs more than 16384 maps). */
SUPRA_ATTN_API int supra_attn_create(int device, supra_attn_ctx** out);
/* Flushes, synchronises and frees everything the context owns. NULL is a no-op. */
SUPRA_ATTN_API int supra_attn_destroy(supra_attn_ctx* ctx);
/* Runs subsequent launches and copies on a caller-owned cudaStream_t (NULL = the context's
 * own non-blocking stream; pass cudaStreamLegacy, (void*)1, for the legacy default stream).
 * Flushes and waits for pending work on the previous stream first. */
SUPRA_ATTN_API int supra_attn_set_stream(supra_attn_ctx* ctx, void* cuda_stream);
SUPRA_ATTN_API const char* supra_attn_last_error(const supra_attn_ctx* ctx);
/* Message for a status code. */
SUPRA_ATTN_API const char* supra_attn_status_string(int status);

/* ---- tensors (the Tensor/BufferPool surface, app/gpu/device.js:41-88,144-191) ------------ */
/* gpu.empty(shape): a pooled device buffer of n floats (size-bucketed like BufferPool.round). */
SUPRA_ATTN_API int supra_attn_tensor_alloc(supra_attn_ctx* ctx, int64_t n, float** dptr);
/* Tensor.release(): flushes recorded work, then returns the buffer to the pool. */
SUPRA_ATTN_API int supra_attn_tensor_free(supra_attn_ctx* ctx, float* dptr);
/* fromArray / write: flushes, then copies n floats host->device (stream-ordered). */
SUPRA_ATTN_API int supra_attn_upload(supra_attn_ctx* ctx, float* dst, const float* src, int64_t n);
/* read(): flushes, copies n floats device->host and waits for them. */
SUPRA_ATTN_API int supra_attn_download(supra_attn_ctx* ctx, float* dst, const float* src, int64_t n);
/* Page-locked host memory for fast upload/download (freed with supra_attn_host_free). */
SUPRA_ATTN_API int supra_attn_host_alloc(supra_attn_ctx* ctx, int64_t n, float** hptr);
SUPRA_ATTN_API int supra_attn_host_free(supra_attn_ctx* ctx, float* hptr);

/* ---- the operator (app/gpu/ops.js:103-149) ------------------------------------------------ */
/* Validates and records one problem. Synchronous EINVAL mirrors the reference's synchronous
 * throw (app/gpu/ops.js:122, app/gpu/device.js:208). */
SUPRA_ATTN_API int supra_attn_enqueue(supra_attn_ctx* ctx, const supra_attn_desc* desc);
/* Validates a descriptor exactly as supra_attn_enqueue does, without a context or a device
 * (pure host function). Writes the message of a failure into msg (cap bytes, may be NULL). */
SUPRA_ATTN_API int supra_attn_check_desc(const supra_attn_desc* desc, char* msg, int32_t cap);
/* Records n problems (an explicit varlen batch); all or none are recorded. */
SUPRA_ATTN_API int supra_attn_enqueue_batch(supra_attn_ctx* ctx, const supra_attn_desc* descs, int32_t n);
/* GPU.flush (app/gpu/device.js:243-253): one grouped launch per kernel configuration. */
SUPRA_ATTN_API int supra_attn_flush(supra_attn_ctx* ctx);
/* GPU.sync (app/gpu/device.js:255-259): flush, wait, and check the device status word.
 * *device_status (may be NULL) receives the raw device status (0 = clean). */
SUPRA_ATTN_API int supra_attn_sync(supra_attn_ctx* ctx, int32_t* device_status);
/* Number of problems recorded and not yet flushed. */
SUPRA_ATTN_API int supra_attn_pending(const supra_attn_ctx* ctx, int32_t* n);

/* ---- T5 relative-position bias (app/models/t5.js:14-23,55-65) ----------------------------- */
/* relativeBucket(rel, buckets, maxDistance) (app/models/t5.js:14-23), bidirectional, with the
 * same float32 rounding steps. Pure host function. Returns the bucket, or -1 on bad input. */
SUPRA_ATTN_API int32_t supra_attn_relative_bucket(int32_t rel, int32_t buckets, int32_t max_distance);
/* T5Encoder.positionBias(L) (app/models/t5.js:55-65) computed on the device:
 *   out[(h*L + i)*L + j] = table[relativeBucket(j - i)*H + h]
 * table is a DEVICE pointer to table_size >= buckets*H floats laid out [buckets, H]
 * (encoder.block.0...relative_attention_bias.weight, app/models/t5.js:44); out is a device
 * pointer to out_size >= H*L*L floats. Stream-ordered with the context's other work
 * (recorded attention is flushed first). */
SUPRA_ATTN_API int supra_attn_position_bias(supra_attn_ctx* ctx, const float* table, int64_t table_size,
                                            int32_t buckets, int32_t max_distance, int32_t H, int32_t L,
                                            float* out, int64_t out_size);

/* ---- linear: the projections beside the attention (ops.linear, app/gpu/ops.js:35-43) -------- */
/* One y = x W^T (+ bias) problem, recorded like an attention problem (same queue, same hazard
 * tracking, one grouped launch per flush). x: M rows of K floats, row stride ldx, first row at
 * x_off; w: [N, K] row-major with row stride ldw >= K (the reference's weight layout, x @ W^T);
 * bias: N floats or NULL; y: M rows of N floats, row stride ldy >= N, first row at y_off. All
 * counts in floats. SUPRA_ATTN_FP32: fp32 FFMA. SUPRA_ATTN_TF32 / SUPRA_ATTN_TF32X3 with K >= 32: on
 * the tensor cores, TF32 products or the split form (three TF32 products per product, held to the
 * FP32 tolerance); operands are read through tensor maps, in place for the TF32 products when
 * 16-byte aligned with row strides of a multiple of 4 floats, else (and always for the split
 * form) first copied as hi / lo parts, x normalised when asked, into a context-owned buffer.
 * Shallower products run the FFMA kernel.
 * Two optional fusions (the VAE mid-block attention, app/models/vae.js:77-94):
 *   - gn != NULL: x is GroupNorm-ed on the way in (ops.groupnorm, app/gpu/ops.js:82-92,
 *     app/gpu/kernels.js:117-162): x rows form images of gn->rows_per_image rows; per image and
 *     group of K / gn->groups channels the library computes (mean, 1/sqrt(var + eps)) in an extra
 *     launch, and the product uses (x - mean) * rstd * gamma[k] + beta[k] (then SiLU if
 *     gn->silu) in place of x. Needs x_off == 0 and ldx == K.
 *   - resid != NULL: y = resid + (x W^T + bias), resid rows of stride ldr at r_off (the residual
 *     add of app/models/vae.js:91). resid may be y itself (same rows: r_off == y_off and
 *     ldr == ldy), which is the reference's in-place `out: x, resid: true` (app/models/dit.js:
 *     175,187,193); otherwise it may not overlap y.
 *   - gate != NULL (needs resid): y = resid + gate[g_off + n] * (x W^T + bias), the gated
 *     residual of the DiT blocks (app/gpu/gemm.js:10,135, app/models/dit.js:175,193).
 *   - ln != NULL (not with gn): x is LayerNorm-ed on the way in, each row over its K channels
 *     (ops.layernorm, app/gpu/ops.js:71-79, app/gpu/kernels.js:87-114): the library computes
 *     (mean, 1/sqrt(var + eps)) per row in an extra launch, and the product uses
 *     (x - mean) * rstd, times (1 + mod[scale_off + k]) plus mod[shift_off + k] when ln->mod is
 *     set (adaLN modulation; app/models/dit.js:164,179,189). Needs x_off == 0 and ldx == K.
 *   With gn or ln on the FFMA kernel, a product whose x is read by two or more column tiles
 *   first writes the normalised x once into a context-owned buffer (one more launch), which the
 *   product then reads; products with one column tile normalise each staged x tile.
 *   - act: SUPRA_ATTN_ACT_NONE, _GELU (erf form), _GELU_TANH or _SILU, applied to x W^T + bias
 *     before the gate and the residual (ops.linear's act, app/gpu/gemm.js:9,28-36,130-135).
 * flags must be 0.
 * Cross-attention K/V preparation (app/models/dit.js:137-144) is two calls: ctx_proj, then ONE
 * product with the 14 blocks' kv weights stacked [14*1152, 576]; block b's cross attention then
 * reads K at column 1152*b and V at 1152*b + 576 of rows of stride 14*1152, without a copy. */
typedef struct supra_attn_groupnorm {
  const float* gamma; /* K floats */
  const float* beta;  /* K floats */
  int32_t groups;     /* K % groups == 0 */
  int32_t rows_per_image; /* M % rows_per_image == 0 */
  float eps;          /* the reference uses 1e-6 */
  int32_t silu;       /* nonzero: SiLU after the affine (ops.groupnorm's silu flag) */
} supra_attn_groupnorm;

enum { SUPRA_ATTN_ACT_NONE = 0, SUPRA_ATTN_ACT_GELU = 1, SUPRA_ATTN_ACT_GELU_TANH = 2, SUPRA_ATTN_ACT_SILU = 3 };

typedef struct supra_attn_layernorm {
  const float* mod;   /* NULL: plain LayerNorm; else the modulation vector (mod_size floats) */
  int64_t mod_size;
  int64_t shift_off;  /* LN(x) * (1 + mod[scale_off + k]) + mod[shift_off + k] */
  int64_t scale_off;
  float eps;          /* the reference uses 1e-6 */
  int32_t reserved;   /* 0 */
} supra_attn_layernorm;

typedef struct supra_attn_linear_desc {
  const float* x;
  const float* w;
  const float* bias;
  float* y;
  int64_t x_size, w_size, bias_size, y_size;
  int64_t ldx, ldw, ldy;
  int64_t x_off, y_off;
  int32_t M, N, K;
  int32_t variant;
  uint32_t flags;
  uint32_t act;                   /* SUPRA_ATTN_ACT_* */
  const supra_attn_groupnorm* gn; /* NULL, or GroupNorm x on the way in (copied at enqueue) */
  const float* resid;             /* NULL, or y = resid + ... (rows of stride ldr at r_off) */
  int64_t resid_size, ldr, r_off;
  const float* gate;              /* NULL, or the product is scaled by gate[g_off + n] */
  int64_t gate_size, g_off;
  const supra_attn_layernorm* ln; /* NULL, or LayerNorm x on the way in (copied at enqueue) */
} supra_attn_linear_desc;
SUPRA_ATTN_API int supra_attn_enqueue_linear(supra_attn_ctx* ctx, const supra_attn_linear_desc* desc);
/* Validates a linear descriptor as supra_attn_enqueue_linear does (pure host function). */
SUPRA_ATTN_API int supra_attn_check_linear_desc(const supra_attn_linear_desc* desc, char* msg, int32_t cap);

/* ---- profiling (the reference's Profiler, app/gpu/device.js:91-99,222-233,272-325) -------- */
/* When on, every grouped launch is bracketed by CUDA events on the launching stream and
 * aggregated by kernel name with its algorithmic FLOPs (4*Lq*Lk*D*H, app/gpu/ops.js:116) and
 * bytes (Q+K+V+O read/written once, plus the bias). */
SUPRA_ATTN_API int supra_attn_profile_enable(supra_attn_ctx* ctx, int32_t on);
typedef struct supra_attn_profile_entry {
  char name[48];
  int64_t launches;
  double ms;    /* summed device time */
  double flops; /* summed algorithmic FLOPs */
  double bytes; /* summed algorithmic bytes */
} supra_attn_profile_entry;
/* Synchronises, then copies up to cap entries (sorted by time) and sets *n. */
SUPRA_ATTN_API int supra_attn_profile_report(supra_attn_ctx* ctx, supra_attn_profile_entry* entries,
                              int32_t cap, int32_t* n);
SUPRA_ATTN_API int supra_attn_profile_reset(supra_attn_ctx* ctx);
/* Total kernels this context has launched since creation, all kinds: every flushed group is one
 * descriptor-staging kernel plus its attention kernel(s). */
SUPRA_ATTN_API int supra_attn_launch_count(const supra_attn_ctx* ctx, int64_t* n);

/* ---- attention without allocation ---------------------------------------------------------- */
/* No counterpart in the reference: this entry point exists for callers that cannot allocate
 * device memory when they need attention, such as a host whose allocator reserves the GPU's
 * memory up front and sub-allocates from it, or code on a latency-critical path that must not
 * call cudaMalloc/cudaFree (those can synchronise the device).
 *
 * Runs ONE problem (validated exactly as supra_attn_enqueue validates it, any head dim) on
 * `cuda_stream` through the score-materialising kernels (QK^T GEMM, row softmax, PV GEMM),
 * without a context and without any allocation: the score scratch is a 16 MiB array of static
 * device memory inside the library, used chunk by chunk, and the chunk's unit table sits in a
 * second static array of about 62 KB, written on the device by a small kernel from values passed
 * as kernel arguments (no host buffer is read after the call returns). Every GPU on which the
 * library's kernels are loaded holds both until the process exits. Limit: one row of scores
 * must fit the scratch, i.e. Lk <= 4,194,304; larger Lk is rejected with SUPRA_ATTN_EINVAL and a
 * message. The arithmetic is always FP32 FFMA, whatever desc->variant asks for: a TF32 or
 * TF32X3 request gets the FP32 result, which lies inside their tolerances.
 *
 * The caller passes inputs and outputs as for supra_attn_enqueue. The work is enqueued on
 * cuda_stream and the call returns without waiting for it. The first call on each device looks
 * up the arrays' device addresses (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture. All calls share the two arrays, which keep the last
 * call's contents: every call writes each score and unit entry it reads before reading it, so
 * nothing needs to start at zero. Calls that overlap on the GPU (different streams, or different
 * host threads on one device) race on the arrays; serialise them, e.g. on one stream.
 * msg (cap bytes, may be NULL) receives the message of a failure. */
SUPRA_ATTN_API int supra_attn_attention_noalloc(const supra_attn_desc* desc, void* cuda_stream, char* msg,
                                                int32_t cap);

#ifdef __cplusplus
}
#endif

#endif /* SUPRA_ATTN_H */
