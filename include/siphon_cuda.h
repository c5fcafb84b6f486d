/* libsiphon_cuda: the quantized-weight matrix path of Siphon on NVIDIA B200
 * (sm_100a), as a plain C ABI.
 *
 * Every entry point takes raw GGUF block bytes exactly as they sit in the
 * model file (block layouts of the reference's include/siphon/quant.h:31-100)
 * and plain device pointers. No torch or CUDA types cross the boundary: a
 * cudaStream_t travels as void* (NULL = the legacy default stream).
 *
 * Results are bit-identical with the reference's CPU code:
 *   - quantized activations byte-for-byte with si_quant_row_q8_K
 *     (src/kernels.c:561-595) and the AVX2 si_quant_row_q8_0 that x86 hosts
 *     dispatch to (src/kernels_avx2.c:594-645);
 *   - matvec outputs bit-for-bit with the scalar dot products
 *     si_dot_<fmt>_<pair> (src/kernels.c:189-523) applied row by row.
 *
 * Return values follow the reference's convention (include/siphon/common.h:
 * 25-34): 0 on success, a negative SICU_E* code on failure, with a message
 * for the calling thread from sicu_last_error(). Argument checks run on the
 * host before any CUDA call. All device memory handed in is owned by the
 * caller; the library allocates device memory only in sicu_init, sicu_upload
 * / sicu_malloc, the all-reduce groups, and the growable buffers of
 * sicu_gemv_host, sicu_row_to_f32, the prefill product, the batch matvec and
 * sicu_gemv_fused's F16 path.
 */
#ifndef SIPHON_CUDA_H
#define SIPHON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SICU_API __attribute__((visibility("default")))
#else
#define SICU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* error codes: the same values as the reference's SI_* (common.h:25-34) */
#define SICU_OK        0
#define SICU_ENOMEM   (-1)
#define SICU_EIO      (-2)   /* CUDA runtime / launch failure */
#define SICU_EFORMAT  (-3)
#define SICU_ENOTSUP  (-4)   /* type or device not supported */
#define SICU_EINVAL   (-5)   /* bad argument (size, alignment, null, state) */

/* ggml type ids (reference include/siphon/quant.h:103-119) */
#define SICU_T_F32   0
#define SICU_T_F16   1
#define SICU_T_Q4_0  2
#define SICU_T_Q5_0  6
#define SICU_T_Q8_0  8
#define SICU_T_Q2_K 10
#define SICU_T_Q3_K 11
#define SICU_T_Q4_K 12
#define SICU_T_Q5_K 13
#define SICU_T_Q6_K 14
#define SICU_T_Q8_K 15

/* ---- lifecycle ----------------------------------------------------------- */

/* Select and prepare a device (compute capability 10.0 required). Makes it
 * current for the calling thread. Replaces the reference's implicit CPU
 * backend singleton si_backend_cpu() (src/backend.c:133-142). */
SICU_API int sicu_init(int device);
/* Release library state on every initialised device. */
SICU_API int sicu_shutdown(void);
/* Copy the calling thread's last error message into buf (always
 * NUL-terminated). Returns the message length. Replaces si_errstr()
 * (include/siphon/common.h:37-38) with per-thread state. */
SICU_API int sicu_last_error(char *buf, size_t len);
/* Read and clear the device status word of the current device: bit 0 set
 * means a kernel's bounded wait on its own copies gave up (outputs of that
 * launch are invalid); SICU_STATUS_AR_TIMEOUT reports a failed all-reduce
 * group (below). Synchronises the device. */
SICU_API int sicu_status(int *flags);
#define SICU_STATUS_WAIT_TIMEOUT 1
#define SICU_STATUS_AR_TIMEOUT   2
#define SICU_STATUS_BAD_ROW      4   /* sicu_row_to_f32_dev: a row id out of range */

/* Programmatic dependent launch for the matvec kernels (default off). When
 * on, a matvec may start streaming its weight blocks while earlier work in
 * the same stream is still running (it still waits for that work before it
 * reads its activation or writes its output), which hides kernel ramp-up in
 * chains of matvecs. Only valid when no earlier work in the stream writes
 * the weight buffer. No counterpart in the reference, which has no kernel
 * launches. */
SICU_API int sicu_set_overlap(int on);

/* Tensor-core throughput probe for roofline denominators: one CTA on each of
 * `sms` SMs issues `rounds` x 64 dense MMAs (M = 128, N = 256; K = 16 for
 * SICU_TC_F16: f16 operands, f32 accumulation; K = 32 for SICU_TC_I8: int8
 * operands, s32 accumulation) with both operands in shared memory, on the
 * legacy default stream, and waits. *ms: device time; *tflops: 2 x
 * multiply-adds / time, in 10^12 per second. Run it alone on the GPU: it
 * holds every SM it is given. No counterpart in the reference, which has no
 * tensor-core code. */
#define SICU_TC_F16 0
#define SICU_TC_I8  1
SICU_API int sicu_tc_peak(int kind, int rounds, int sms, float *ms, double *tflops);

/* ---- memory ------------------------------------------------------------- */

SICU_API int sicu_malloc(void **dev, size_t bytes);
SICU_API int sicu_free(void *dev);
/* Make weight bytes device-resident once at load: allocate and copy. The
 * returned pointer is 256-byte aligned. Replaces the mmap'd host view of
 * si_tensor_from_gguf (src/backend.c:144-176). */
SICU_API int sicu_upload(const void *host, size_t bytes, void **dev);
SICU_API int sicu_memcpy_h2d(void *dev, const void *host, size_t bytes, void *stream);
SICU_API int sicu_memcpy_d2h(void *host, const void *dev, size_t bytes, void *stream);
SICU_API int sicu_stream_sync(void *stream);

/* ---- geometry ------------------------------------------------------------ */

/* Elements per block and bytes per block of a type.
 * Replaces si_quant_geometry (src/kernels.c:904-919). */
SICU_API int sicu_quant_geometry(uint32_t type, uint32_t *blck_size, uint32_t *type_size);
/* Activation format a weight type's dot product consumes.
 * Replaces si_quant_vec_dot_pair (src/kernels.c:946-960). */
SICU_API int sicu_vec_dot_pair(uint32_t wtype, uint32_t *pair_type);

/* ---- activation conversion ------------------------------------------------
 * m rows of n contiguous f32 (dx, 16-byte aligned) into m rows of the pair
 * format, each row quantized on its own. */

/* Replaces si_quant_row_q8_K (src/kernels.c:561-595). n % 256 == 0.
 * All-zero blocks get bsums = 0 (the reference leaves them unwritten). */
SICU_API int sicu_quantize_q8_K(const float *dx, void *dy, int64_t n, int64_t m, void *stream);
/* Replaces si_quant_row_q8_0 as dispatched on x86 (si_avx2_quant_row_q8_0,
 * src/kernels_avx2.c:594-645). n % 32 == 0. */
SICU_API int sicu_quantize_q8_0(const float *dx, void *dy, int64_t n, int64_t m, void *stream);
/* F16 pair: element-wise round-to-nearest-even (src/backend.c:19-27). */
SICU_API int sicu_convert_f16(const float *dx, void *dy, int64_t n, int64_t m, void *stream);
/* Dispatch on the weight type's pair format. Replaces conv_task_fn
 * (src/backend.c:17-47). */
SICU_API int sicu_quantize_pair(uint32_t wtype, const float *dx, void *dxq, int64_t n, int64_t m, void *stream);

/* ---- matrix-vector products ----------------------------------------------
 * dw: [n_out rows][row bytes] of wtype blocks, row-major, 16-byte aligned.
 * dy: [m][n_out] f32. Supported wtype: F16, Q4_0, Q5_0, Q8_0, Q2_K..Q6_K. */

/* y_i = dot(W, xq_i) for m pair-format activation rows (dxq: m rows, each
 * sicu pair-row bytes long). Replaces dot_task_fn (src/backend.c:61-71) with
 * si_vec_dot_for(wtype) (src/kernels.c:1058-1072), scalar semantics. */
SICU_API int sicu_gemv(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out,
              const void *dxq, float *dy, int64_t m, void *stream);
/* y = W x from f32 activations: the activation conversion happens inside
 * the matvec kernel (each CTA quantizes into shared memory), exactly once
 * per row as far as results go. Replaces the si_backend gemv vtable slot
 * cpu_gemv (src/backend.c:85-120; include/siphon/tensor.h:43-55). */
SICU_API int sicu_gemv_f32(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out,
                  const float *dx, float *dy, int64_t m, void *stream);
/* Several matvecs sharing one f32 activation: y_i = W_i x for i < n_mats
 * (1..64), every W_i of type wtype with row length n_in and n_out[i] rows;
 * dw, n_out and dy are host arrays of device pointers / sizes. One kernel
 * launch streams all the matrices back to back and quantizes x once, so the
 * launch ramp and drain are paid once. Replaces consecutive backend gemv
 * calls on one activation in the reference's forward pass (src/engine.c:
 * 317-319 for Wq/Wk/Wv, 375-376 for gate/up); results are identical to
 * n_mats separate sicu_gemv_f32 calls. */
SICU_API int sicu_gemv_multi(uint32_t wtype, int n_mats, const void *const *dw, const int64_t *n_out,
                             int64_t n_in, const float *dx, float *const *dy, void *stream);
/* Batch decode: dy_i[t] = W_i x_t for m (0..8) f32 activation rows x_t
 * (dx: [m][n_in], 16-byte aligned; dy[i]: [m][n_out[i]]) and n_mats (1..16)
 * matrices of one type and row length: one decode step of up to eight
 * sequences. Q4_K and Q6_K weights stream from memory once for all rows (a
 * tensor-core kernel: weight blocks decoded in registers to exact f16
 * products, exact integer lane sums, the reference's float chains); other
 * types, and m == 1, run the matvec per row. Every output is bit-identical to
 * sicu_gemv_f32 of that row, i.e. to the reference's scalar dot product per
 * token. The reference has no batched step: it runs one si_engine_forward per
 * token and sequence (src/engine.c:288-398), one backend gemv per matrix. A
 * per-device workspace (about 4.3 KB per 256 inputs) grows on the first call
 * with a larger n_in; make that call before any stream capture. */
SICU_API int sicu_gemv_batch(uint32_t wtype, int n_mats, const void *const *dw, const int64_t *n_out, int64_t n_in,
                             const float *dx, int64_t m, float *const *dy, void *stream);
/* Same, with host input and output buffers (one activation row): copies x
 * in, runs sicu_gemv_f32, copies y out and waits. This is the exact call
 * shape of the reference's backend gemv slot. When both buffers are
 * page-locked (cudaHostAlloc / cudaHostRegister) and the type is quantized,
 * the GPU reads x and writes y through their device views instead of two
 * copy-engine transfers, and the matvec starts streaming its weights while x
 * is being read; results are identical. */
SICU_API int sicu_gemv_host(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out,
                   const float *hx, float *hy, void *stream);

/* sicu_gemv_host for callers that must not allocate device memory: host
 * code running under an application-owned device allocator that has already
 * claimed the GPU's memory (so a library cudaMalloc would fail), hosts that
 * forbid device allocation on the hot path because cudaMalloc/cudaFree can
 * synchronise the device, and tools that load the library into a process
 * whose allocations they do not control. The activation copy, the output
 * before it returns to the host and a status word live in a fixed array
 * compiled into the library (1.25 MiB on every device that loads it, held
 * until the process exits); no call allocates anything. Limits: n_in <=
 * 65536 and n_out <= 262144 (larger shapes are rejected with SICU_EINVAL;
 * use sicu_gemv_host). The first call on a device resolves the array's device
 * address and reads the device's launch limits, so make that first call
 * before any stream capture. Every call uses the same array: calls whose GPU
 * work overlaps (other streams, other host threads on the same device) race
 * on it and must be serialised by the caller. sicu_init is not required.
 * The resolved address is kept for the life of the process and does not
 * survive a cudaDeviceReset of that device (do not reset a device this entry
 * point has used). Same results as sicu_gemv_host. No counterpart in the
 * reference. */
SICU_API int sicu_gemv_host_noalloc(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out,
                                    const float *hx, float *hy, void *stream);

/* ---- prefill ---------------------------------------------------------------
 * Y = X W^T for a block of m prompt tokens: dy[t * n_out + r] = (W x_t)[r]
 * for t < m (0 <= m <= 65535). dxq holds m consecutive rows of pair-format
 * blocks (Q8_K for the K formats: sicu_quantize_q8_K); the _f32 form takes m
 * f32 rows (16-byte aligned) and quantizes them first.
 * For m <= 8, Q4_K and Q6_K run the batch decode kernel of sicu_gemv_batch
 * (bit-identical with the per-token matvec). For larger m they run on the
 * tensor cores (tcgen05 MMAs, accumulators in tensor
 * memory, the token operand loaded by TMA): the integer sums per super-block are exact
 * and the d / dmin scaling is applied per super-block, so each output agrees
 * with the reference's per-row dot (src/kernels.c:349-410) within a relative
 * 1e-5 of the L1 norm of its products, but is not bit-identical. Q5_K, Q3_K
 * and Q2_K (src/kernels.c:412-478, 289-347, 249-287) run on the same tensor
 * cores for m > 32, from a prefill copy (below) that the call first writes
 * into the workspace when the caller has none. Q4_0, Q5_0 and Q8_0
 * (src/kernels.c:197-247) run on int8 MMAs for m > 32 and n_in >= 128, one
 * per 32-element block, with the reference's float operations per block in
 * order: bit-identical to the reference (a copy made in the workspace the
 * same way). F16 rows of whole 256-element chunks run on kind::f16 MMAs for
 * m > 32 (the f16 weights re-tiled, within the same tolerance of the
 * reference's double-accumulated dot, src/kernels.c:189-195). Other cases (at
 * most 32 tokens, short F16 rows) run the decode matvec once per token
 * (bit-identical to the reference).
 * The reference has no batched product: its prompt loop calls
 * si_engine_forward once per token (src/cmd_run.c:276), i.e. one backend gemv
 * per token and matrix. When a product has fewer 128-row x token tiles than
 * the GPU has SMs, each row's super-blocks are split into ranges computed by
 * separate CTAs and their partial products added in a fixed order (same bits
 * on every run). A per-device workspace grows on the first call with a larger
 * m, n_in or n_out; make that call before any stream capture. */
SICU_API int sicu_gemm_prefill(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out,
                               const void *dxq, int64_t m, float *dy, void *stream);
SICU_API int sicu_gemm_prefill_f32(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out,
                                   const float *dx, int64_t m, float *dy, void *stream);

/* ---- prefill copies of the weights -----------------------------------------
 * A second, re-tiled copy of a weight matrix (any format) for prompt products, made
 * once when the weights are loaded (the reference makes its tensor views at
 * load, si_tensor_from_gguf, src/backend.c:144-176); the raw GGUF bytes stay
 * on the device for decode. Per 128-row tile and super-block the copy holds
 * the exact f16 (scale x quant) operands in the shared-memory layout the
 * tensor cores read (128-byte swizzle), the mins operand and the row scales,
 * so the prefill kernel streams it with bulk copies and converts nothing.
 * Size per 128 rows and super-block: 4x16 KiB + 8.5 KiB for Q4_K, Q5_K and
 * Q2_K (about 3.6x, 3.3x and 6.9x the raw bytes), 4x16 KiB + 0.5 KiB for
 * Q3_K (4.7x), 8x16 KiB + 0.5 KiB for Q6_K (4.9x). Q5_K, Q3_K and Q2_K have
 * one exact f16 plane of scale x quant per K-step (|sc q| <= 1953, 128, 45).
 * Q4_0, Q5_0, Q8_0: per 128 rows and K-step of four 32-blocks 16 KiB of int8
 * quants + 2 KiB of block scales (n_in a multiple of 32, at least 128).
 * F16: per 128 rows and 256 elements 4x16 KiB of the re-tiled halves + 0.5 KiB.
 * sicu_prefill_pack_bytes: the copy's size (SICU_ENOTSUP for other types).
 * sicu_prefill_pack: writes the copy of device weights dw into dpack
 * (pack_bytes >= that size, 16-byte aligned), asynchronously on stream.
 * sicu_gemm_prefill_packed(_f32): sicu_gemm_prefill(_f32) with the copy
 * (dpack may be null: then the same as without). Blocks of more than 32
 * tokens run from the copy (128 rows x 128 or 256 tokens per CTA, both
 * operands in shared memory); smaller ones read dw as before. Results are
 * within the same tolerance as sicu_gemm_prefill, from the same exact integer
 * sums per super-block; the float additions of super-blocks may differ. */
SICU_API int sicu_prefill_pack_bytes(uint32_t wtype, int64_t n_in, int64_t n_out, size_t *bytes);
SICU_API int sicu_prefill_pack(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out, void *dpack,
                               size_t pack_bytes, void *stream);
SICU_API int sicu_gemm_prefill_packed(uint32_t wtype, const void *dw, const void *dpack, int64_t n_in,
                                      int64_t n_out, const void *dxq, int64_t m, float *dy, void *stream);
SICU_API int sicu_gemm_prefill_packed_f32(uint32_t wtype, const void *dw, const void *dpack, int64_t n_in,
                                          int64_t n_out, const float *dx, int64_t m, float *dy, void *stream);
/* dy_i = X W_i^T for n_mats (1..4) matrices of one type and row length that
 * read the same m-token activation (dx: [m][n_in] f32, 16-byte aligned;
 * dy[i]: [m][n_out[i]]), each with its prefill copy dpack[i]: the products
 * the reference's forward pass runs one after another on one activation
 * (src/engine.c:317-319 Wq/Wk/Wv, 375-376 W_gate/W_up), once per prompt
 * token. The activation is quantized once and one launch covers every
 * matrix's tiles, so products too small to fill the GPU alone share it.
 * Each result is within the sicu_gemm_prefill tolerance (the same exact
 * integer sums per super-block). dpack null (or any entry null), at most
 * 32 tokens, or Q4_0 / Q5_0 / Q8_0 weights: the products one after another as
 * sicu_gemm_prefill_packed_f32 (up to 8 tokens one batch launch for all
 * matrices). dw, dpack, n_out and dy are host arrays. */
SICU_API int sicu_gemm_prefill_multi_f32(uint32_t wtype, int n_mats, const void *const *dw,
                                         const void *const *dpack, const int64_t *n_out, int64_t n_in,
                                         const float *dx, int64_t m, float *const *dy, void *stream);

/* ---- tensor-parallel all-reduce fused into the matvec ------------------------
 * A row-split product (Wo, W_down split by input columns across a
 * tensor-parallel group) leaves a partial output vector on every rank that
 * must be summed before the next product reads it. The reference runs one
 * process on one CPU and has no such step: its forward pass applies Wo and
 * W_down to the whole activation (src/engine.c:368, 378). sicu_gemv_ar runs
 * the row-split matvec and the all-reduce as one kernel: each CTA sends the
 * partial outputs of the rows it computed to every rank with plain NVLink
 * peer stores (each element a 64-bit word carrying its delivery tag), then
 * waits (bounded) for the other ranks' parts of the same rows and writes
 * their sum, added in rank order in f32 (((p0 + p1) + p2) + ...), so every
 * rank ends with bit-identical outputs. No collective launch, fence or flag
 * is involved; the next matvec reads dy as a plain activation.
 *
 * A group has n_ranks (1..8) members, one process per GPU, and vectors of
 * len floats (a multiple of 256, <= 2^24). Setup, in every rank:
 *   sicu_ar_create(n, rank, len, &g, handle)  -> this rank's 64-byte handle
 *   exchange the handles (any host channel; all ranks get all n, rank order)
 *   sicu_ar_open(g, handles)                  -> maps the peers' buffers
 * Every rank issues the group's operations (sicu_gemv_ar, sicu_ar_allreduce)
 * on one stream, in the same order. The delivery counter lives on the device,
 * so a captured CUDA graph replays the sequence. A wait gives up after the
 * group's timeout (default 2 s, sicu_ar_set_timeout), sets
 * SICU_STATUS_AR_TIMEOUT and marks the group broken: every later operation
 * returns at once with the same bit and outputs the local partial; destroy
 * and create the group again. Teardown: every rank synchronises its streams
 * and meets the others (a host barrier) before sicu_ar_destroy. */
#define SICU_AR_HANDLE_BYTES 64
typedef struct sicu_ar sicu_ar;
SICU_API int sicu_ar_create(int n_ranks, int rank, int64_t len, sicu_ar **group, void *handle);
/* handles: n_ranks x SICU_AR_HANDLE_BYTES, rank order (this rank's own included) */
SICU_API int sicu_ar_open(sicu_ar *group, const void *handles);
SICU_API int sicu_ar_set_timeout(sicu_ar *group, uint64_t ns);
SICU_API int sicu_ar_destroy(sicu_ar *group);
/* ddst[i] = sum over ranks of their dsrc[i] (len floats, device; in place
 * allowed), same protocol, for partial sums the library did not produce. */
SICU_API int sicu_ar_allreduce(sicu_ar *group, const float *dsrc, float *ddst, void *stream);
/* dy = sum over the group's ranks of (W_rank x_rank): sicu_gemv_f32 of this
 * rank's column shard (n_out == the group's len) with the all-reduce fused
 * in. Quantized weight types only. */
SICU_API int sicu_gemv_ar(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_out,
                          const float *dx, float *dy, sicu_ar *group, void *stream);

/* ---- activation steps fused into the product ---------------------------------
 * Between two products the reference's forward pass runs a step on the f32
 * activation on the host: the residual add and RMS norm before Wq/Wk/Wv, before
 * W_gate/W_up and before the output head, and SwiGLU before W_down
 * (src/engine.c:313-315, 369-377, 379-389). sicu_gemv_fused takes the step's
 * inputs and runs it inside the matvec: each CTA applies it while quantizing
 * the activation, so the step needs no launch and no f32 round trip through
 * memory. Results are bit-identical to the reference's step followed by its
 * gemv, for finite inputs and results (non-finite values give NaN or inf as
 * there, but NaN payloads are not matched):
 *   SICU_PRO_RMS_NORM  h = x + residual (x alone when residual is NULL),
 *                      a_i = h_i * s * weight_i, s = 1 / sqrtf(mean(h^2) + eps),
 *                      mean(h^2) as the reference computes it (f32 squares
 *                      added in double in index order, the mean rounded to
 *                      f32); sum_out (optional) receives h, the new residual
 *                      stream (src/engine.c:12-18, 369; src/kernels.c:892-900)
 *   SICU_PRO_SWIGLU    a_i = silu(x_i) * up_i, silu(v) = v / (1 + e(0 - v)) with
 *                      the reference's exp polynomial
 *                      (src/engine.c:162-179; src/kernels.c:821-853)
 *   SICU_PRO_MUL       a_i = x_i * up_i: SwiGLU's product when x already holds
 *                      silu(gate), i.e. when the gate product ran with the
 *                      SICU_EPI_SILU epilogue. Computing silu once per element
 *                      in the gate product's epilogue costs little there, while
 *                      SICU_PRO_SWIGLU evaluates it in every CTA cluster that
 *                      quantizes x.
 * weight, residual, sum_out and up are device vectors of n_in floats, 16-byte
 * aligned; sum_out must not overlap x, residual, weight or an output. */
#define SICU_PRO_NONE     0
#define SICU_PRO_RMS_NORM 1
#define SICU_PRO_SWIGLU   2
#define SICU_PRO_MUL      3
typedef struct sicu_prologue {
    int32_t kind;            /* SICU_PRO_* */
    float eps;               /* RMS norm epsilon (the model's rms_eps) */
    const float *weight;     /* RMS norm weight */
    const float *residual;   /* added to x before the norm, or NULL */
    float *sum_out;          /* receives x + residual, or NULL */
    const float *up;         /* SwiGLU / MUL: the up projection's output */
} sicu_prologue;
/* Epilogues, per matrix: SICU_EPI_SILU writes silu(W_i a) instead of W_i a
 * (the gate half of SwiGLU, src/engine.c:162-179, with the reference's exp
 * polynomial), for a following SICU_PRO_MUL step. */
#define SICU_EPI_NONE 0
#define SICU_EPI_SILU 1
/* dy_i = W_i a for i < n_mats, a = the step pro (NULL: none) applied to dx,
 * each output through its epilogue epi[i] (epi NULL: none; a host array of
 * n_mats entries): sicu_gemv_multi with the steps fused in. group: NULL, or
 * an all-reduce group (n_mats == 1, n_out[0] == the group's len): the
 * sicu_gemv_ar form, the epilogue applied to the sum. Quantized weight types
 * run the steps inside the matvec; F16 weights run them as separate kernels,
 * the prologue into a per-device buffer (grown on first use, so make such a
 * call once before any stream capture). */
SICU_API int sicu_gemv_fused(uint32_t wtype, int n_mats, const void *const *dw, const int64_t *n_out,
                             int64_t n_in, const float *dx, const sicu_prologue *pro, const int32_t *epi,
                             float *const *dy, sicu_ar *group, void *stream);
/* sicu_gemv_fused with a bias per matrix: bias (NULL, or a host array of
 * n_mats device vectors of n_out[i] floats, NULL entries allowed) is added to
 * matrix i's outputs, y + b in f32, before its epilogue: the Q, K and V biases
 * of Qwen2-architecture models, which the reference adds after those products
 * (src/engine.c:320-334). */
SICU_API int sicu_gemv_fused_ex(uint32_t wtype, int n_mats, const void *const *dw, const int64_t *n_out,
                                int64_t n_in, const float *dx, const sicu_prologue *pro, const int32_t *epi,
                                const float *const *bias, float *const *dy, sicu_ar *group, void *stream);
/* The steps on their own, m rows of n floats (16-byte aligned rows, n a
 * multiple of 4): dy = rmsnorm(dx + dres) * dw with dsum = dx + dres (dres and
 * dsum per row, each NULL allowed), and dy = silu(dx) * dup. For prompts
 * (before sicu_gemm_prefill_f32) and other callers that need the f32 result.
 * The reference sends the last n % 8 elements of a SwiGLU row through libm's
 * expf instead of the polynomial; sicu_swiglu rejects such n (every K-quant
 * FFN width is a multiple of 256). */
SICU_API int sicu_rms_norm(const float *dx, const float *dres, float *dsum, const float *dw, int64_t n, int64_t m,
                           float eps, float *dy, void *stream);
SICU_API int sicu_swiglu(const float *dx, const float *dup, int64_t n, int64_t m, float *dy, void *stream);
/* dy_r += db for m rows of n floats, in place: the Q/K/V bias adds of
 * Qwen2-architecture models (src/engine.c:319-333, one f32 addition per
 * element) for a prompt's rows; a single token's adds ride in the QKV
 * product's epilogue (sicu_gemv_fused_ex). */
SICU_API int sicu_add_bias(float *dy, const float *db, int64_t n, int64_t m, void *stream);

/* ---- attention softmax ------------------------------------------------------
 * dy_r = softmax(dx_r) for m rows of n floats, as the reference's attention
 * computes it (src/engine.c:124-130 with si_softmax, src/kernels.c:855-890):
 * the row maximum, exp(x - max) through the exp polynomial in groups of 8 with
 * each group's sum in an 8-wide horizontal add's lane order added into a
 * double, the last n % 8 elements through libm's expf (restated as this image's
 * glibc computes it on hosts with FMA), then every element times
 * (float)(1 / sum). Bit-identical to the reference for finite inputs.
 * In place (dx == dy) allowed. A building block of the device attention. */
SICU_API int sicu_softmax(const float *dx, float *dy, int64_t n, int64_t m, void *stream);

/* ---- attention over the f16 KV cache ---------------------------------------
 * The reference's per-layer attention step (src/engine.c:90-147, 336-366) on
 * the device, on its cache layout (one layer's base pointers):
 *   K cache: f16 [n_head_kv][n_ctx][head_dim] (position-major)
 *   V cache: f16 [n_head_kv][head_dim][n_ctx] (transposed)
 * sicu_rope rotates n_heads heads of head_dim floats in place with the
 * position's cos / sin tables (n_rot / 2 entries, device; the engine computes
 * them with libm, src/engine.c:26-40): pairs (2j, 2j+1) as fma(x0, c, -(x1 s)),
 * fma(x0, s, x1 c) (neox = 0), or (j, j + head_dim/2) with plain products and
 * sums (neox != 0); channels from n_rot on unchanged.
 * sicu_kv_store writes one position's K and V (n_head_kv x head_dim floats
 * each) into the caches as f16 (round to nearest even).
 * sicu_attention computes, for every query head h (KV head h / (n_head /
 * n_head_kv)), the scores of positions 0..pos (f16 dot of the head's q as f16
 * with each cached K row, times kq_scale), their softmax (sicu_softmax), the
 * probabilities as f16, and out[h][c] = f16 dot of V row c with them. Every
 * f16 dot is the reference's scalar si_dot_f16 (src/kernels.c:189-195: exact
 * products added into a double in index order), so results are bit-identical
 * to the reference engine run with its scalar kernels (SI_SCALAR=1, the form
 * the library's parity tests use). pos + 1 <= 32768, head_dim <= 1024. */
SICU_API int sicu_rope(float *dx, int64_t n_heads, int64_t head_dim, int64_t n_rot, const float *dcos,
                       const float *dsin, int neox, void *stream);
SICU_API int sicu_kv_store(const float *dk, const float *dv, void *dk_cache, void *dv_cache, int64_t n_head_kv,
                           int64_t head_dim, int64_t n_ctx, int64_t pos, void *stream);
SICU_API int sicu_attention(const float *dq, const void *dk_cache, const void *dv_cache, int64_t n_head,
                            int64_t n_head_kv, int64_t head_dim, int64_t n_ctx, int64_t pos, float kq_scale,
                            float *dout, void *stream);
/* The three above in one launch, the engine's order for one layer and
 * position: RoPE on q (n_head heads) and k (n_head_kv heads) with the
 * position's tables, k and v stored into the caches at pos, then the
 * attention; dq and dk are left unrotated (the rotated values live only in
 * the launch). Same results as sicu_rope x2 + sicu_kv_store + sicu_attention.
 * With sicu_set_overlap(1) the matvec that follows may launch while it runs
 * (and stream its weights). pos + 1 <= 30000. */
SICU_API int sicu_attention_step(const float *dq, const float *dk, const float *dv, void *dk_cache, void *dv_cache,
                                 const float *dcos, const float *dsin, int64_t n_head, int64_t n_head_kv,
                                 int64_t head_dim, int64_t n_rot, int neox, int64_t n_ctx, int64_t pos,
                                 float kq_scale, float *dout, void *stream);

/* A prompt's attention: sicu_attention_step for the m consecutive positions
 * pos0 .. pos0 + m - 1 in one call, as the engine's token-serial prompt loop
 * (src/cmd_run.c:276) runs it one token at a time: dq [m][n_head * head_dim],
 * dk and dv [m][n_head_kv * head_dim], dcos and dsin [m][n_rot / 2] (the
 * tables of each token's position), dout [m][n_head * head_dim]. Every
 * token's k (rotated) and v are stored into the caches first, then every
 * (head, token) rotates its q and attends over positions 0 .. pos0 + t, which
 * then hold exactly what the engine's cache held at that token: outputs and
 * caches bit-identical to m sicu_attention_step calls. dq, dk, dv are left
 * unrotated. pos0 + m <= min(n_ctx, 30000). No counterpart as one call in
 * the reference. */
SICU_API int sicu_attention_prompt(const float *dq, const float *dk, const float *dv, void *dk_cache,
                                   void *dv_cache, const float *dcos, const float *dsin, int64_t n_head,
                                   int64_t n_head_kv, int64_t head_dim, int64_t n_rot, int neox, int64_t n_ctx,
                                   int64_t pos0, int64_t m, float kq_scale, float *dout, void *stream);

/* ---- dequantisation --------------------------------------------------------
 * Rows rows[0..nrows) (host array) of W into dout[nrows][n_in] f32, reference
 * semantics. Replaces cpu_row_to_f32 (src/backend.c:122-131) with
 * si_dequant_row (src/kernels.c:803-817). */
SICU_API int sicu_row_to_f32(uint32_t wtype, const void *dw, int64_t n_in, const int64_t *rows,
                    int64_t nrows, float *dout, void *stream);
/* The same with the row ids in device memory (e.g. the token the previous
 * decode step chose on the device, for the embedding lookup of
 * src/engine.c:295-300), so the call neither copies nor waits. W has n_rows
 * rows; an id outside [0, n_rows) yields a NaN row and sets
 * SICU_STATUS_BAD_ROW. */
SICU_API int sicu_row_to_f32_dev(uint32_t wtype, const void *dw, int64_t n_in, int64_t n_rows,
                                 const int64_t *drows, int64_t nrows, float *dout, void *stream);
/* dout[r] = the greedy choice of row r of m rows of n floats, as the
 * reference's si_sample_greedy picks it (src/sampler.c:6-12): the first
 * maximum among the non-NaN values, 0 when element 0 is NaN. */
SICU_API int sicu_argmax(const float *dx, int64_t n, int64_t m, int64_t *dout, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SIPHON_CUDA_H */
