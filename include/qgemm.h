/*
 * qgemm.h -- C ABI of libqgemm, the B200 (sm_100a) quantized-matmul library.
 *
 * This is the drop-in boundary for the quantized-matmul operators of
 * bytedeco/cuda-triton-scala.  The reference exposes them as Scala methods
 * taking device pointers (core/Ptr.scala:9-52, `address: Long`) and Ints
 * (src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala:17-247),
 * by kernel name (dsl/TritonKernelRunner.scala:68-73) and through a Java
 * bridge of raw Long addresses (driver/CUDARuntimeJavaBridge.scala:121-165).
 * Each entry point below names the reference interface it replaces.
 *
 * Conventions
 *  - Device buffers are passed as uint64_t device addresses (a Ptr.address);
 *    the caller owns every buffer.  Nothing here allocates per call.
 *  - Every compute call is asynchronous on the given stream and returns a
 *    status; errors never abort, exit or trap.  qgemm_last_error() gives a
 *    thread-local message for the last failing call on this thread.
 *  - Kernels that wait on barriers bound every wait; a wait that runs out sets
 *    a per-device error word that qgemm_stream_sync() reports as
 *    QGEMM_ERR_TIMEOUT.
 *  - Handles are thread-safe per distinct stream; a device handle may be
 *    shared across threads.
 *  - Kernels use programmatic dependent launch: one may start while the previous
 *    kernel on the stream finishes, and it waits for that kernel before it reads
 *    anything the kernel may have written.  The exception is the prepacked weights
 *    and scales of the W4A16 decode paths (_tiled, _frag), which are static model
 *    data and are read before that wait.  A caller's kernel that writes them and
 *    triggers programmatic launch early must be separated from the decode call
 *    (an event, or a launch without the programmatic attribute); this library's own
 *    kernels, memcpys and ordinary launches need nothing.
 */
#ifndef QGEMM_H
#define QGEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Every entry point is exported from libqgemm.so; everything else is hidden. */
#if defined(__GNUC__)
#define QGEMM_API __attribute__((visibility("default")))
#else
#define QGEMM_API
#endif

typedef int32_t qgemm_status;

enum {
  QGEMM_OK = 0,
  QGEMM_ERR_INVALID_ARG = -1,  /* bad size, null pointer, bad enum           */
  QGEMM_ERR_BAD_ALIGN = -2,    /* pointer or leading dimension misaligned    */
  QGEMM_ERR_CUDA = -3,         /* a CUDA runtime/driver call failed          */
  QGEMM_ERR_NCCL = -4,         /* an NCCL call failed or NCCL is unavailable */
  QGEMM_ERR_TIMEOUT = -5,      /* a bounded device-side wait ran out         */
  QGEMM_ERR_UNSUPPORTED = -6,  /* no kernel for this device / shape          */
  QGEMM_ERR_NO_DEVICE = -7,    /* no CUDA device, or ordinal out of range    */
  QGEMM_ERR_OOM = -8,          /* device allocation failed                   */
  QGEMM_ERR_BAD_HANDLE = -9    /* null or closed handle                      */
};

/* Output element types. */
enum { QGEMM_F32 = 0, QGEMM_BF16 = 1 };

/* Layouts of the int8 weight operand B of the W8A8 GEMM.
 * QGEMM_B_KN: [K, N] row-major, the reference layout (`wInt8(k*N+col)`,
 *             QuantizedGemmOps.scala:106).  Used as-is (MN-major operand).
 * QGEMM_B_NK: [N, K] row-major (K-major), e.g. from qgemm_prepack_w8_nk. */
enum { QGEMM_B_KN = 0, QGEMM_B_NK = 1 };

/* Kernel selection for the W8A8 GEMM. */
enum {
  QGEMM_ALGO_AUTO = 0,     /* tcgen05 when the shape allows it, else SIMT       */
  QGEMM_ALGO_TCGEN05 = 1,  /* tensor-core path only (UNSUPPORTED if it can't)   */
  QGEMM_ALGO_SIMT = 2      /* CUDA-core path (any shape), the independent check  */
};

typedef struct qgemm_device_s* qgemm_device_t;
typedef struct qgemm_stream_s* qgemm_stream_t;
typedef struct qgemm_comm_s* qgemm_comm_t;
typedef struct qgemm_window_s* qgemm_window_t;

/* ---- errors ----------------------------------------------------------------
 * Replaces the reference's swallowed exceptions (runtime/CUDARuntime.scala:216,
 * 256, 294) with statuses and a message. */
QGEMM_API const char* qgemm_last_error(void);
QGEMM_API const char* qgemm_status_string(qgemm_status s);
QGEMM_API int qgemm_version(void); /* major*10000 + minor*100 + patch */

/* ---- devices ---------------------------------------------------------------
 * Replaces runtime/DeviceRuntime.scala:13-45 (`init`) and CUDARuntime.init
 * (runtime/CUDARuntime.scala:120-183), which hard-codes device 0. */
QGEMM_API qgemm_status qgemm_device_count(int* count);
QGEMM_API qgemm_status qgemm_device_open(int ordinal, qgemm_device_t* out);
QGEMM_API qgemm_status qgemm_device_close(qgemm_device_t dev);
/* sm_count, compute capability, L2 bytes, and whether tcgen05 kernels run. */
QGEMM_API qgemm_status qgemm_device_info(qgemm_device_t dev, int* sm_count, int* cc_major,
                               int* cc_minor, size_t* l2_bytes, int* has_tcgen05);
/* Limit, in nanoseconds of the GPU's global timer, of every bounded device-side wait
 * in the tensor-core GEMM kernels (W8A8, bf16, fp32 entry points) launched on this
 * device from now on; default 2 s, accepted range 1 us .. 60 s.  A wait that runs out
 * ends its kernel early and qgemm_stream_sync() then reports QGEMM_ERR_TIMEOUT.  No
 * counterpart in the reference, whose launches never wait on the device. */
QGEMM_API qgemm_status qgemm_device_set_wait_limit(qgemm_device_t dev, uint64_t limit_ns);
QGEMM_API qgemm_status qgemm_device_get_wait_limit(qgemm_device_t dev, uint64_t* limit_ns);
/* Test hook for the timeout path (no counterpart in the reference): with enable != 0,
 * the final K part of every tile the W8A8 GEMM's last-wave split cuts waits for one
 * count-in more than the other parts make, so its bounded wait runs out after the
 * device's wait limit; the call then ends in QGEMM_ERR_TIMEOUT at qgemm_stream_sync()
 * (its output is undefined) and the stream stays usable.  Leave it off otherwise. */
QGEMM_API qgemm_status qgemm_debug_hold_split(qgemm_device_t dev, int enable);

/* ---- streams ---------------------------------------------------------------
 * Replaces driver/TritonDriverAPINative.scala:78-122 (NativeCUDAStream). */
QGEMM_API qgemm_status qgemm_stream_create(qgemm_device_t dev, qgemm_stream_t* out);
/* Adopt a caller-owned cudaStream_t (not destroyed by qgemm_stream_destroy). */
QGEMM_API qgemm_status qgemm_stream_wrap(qgemm_device_t dev, void* cuda_stream, qgemm_stream_t* out);
QGEMM_API qgemm_status qgemm_stream_destroy(qgemm_stream_t s);
/* Synchronise, then report (and clear) a device-side timeout on this device. */
QGEMM_API qgemm_status qgemm_stream_sync(qgemm_stream_t s);

/* ---- buffers ---------------------------------------------------------------
 * Replace DeviceRuntime.malloc/free/memcpyHtoD/memcpyDtoH
 * (runtime/DeviceRuntime.scala:13-45; runtime/CUDARuntime.scala:204-311). */
QGEMM_API qgemm_status qgemm_buffer_alloc(qgemm_device_t dev, size_t bytes, uint64_t* dev_addr);
QGEMM_API qgemm_status qgemm_buffer_free(qgemm_device_t dev, uint64_t dev_addr);
QGEMM_API qgemm_status qgemm_memcpy_h2d(qgemm_stream_t s, uint64_t dst, const void* src, size_t bytes);
QGEMM_API qgemm_status qgemm_memcpy_d2h(qgemm_stream_t s, void* dst, uint64_t src, size_t bytes);
QGEMM_API qgemm_status qgemm_memset(qgemm_stream_t s, uint64_t dst, int value, size_t bytes);
/* Page-locked host memory for fast copies (cudaMallocHost). */
QGEMM_API qgemm_status qgemm_host_alloc(size_t bytes, void** out);
QGEMM_API qgemm_status qgemm_host_free(void* p);

/* ---- reference operators (same names, argument order and meaning) -------- */

/* QuantizedGemmOps.w8a32Gemm (QuantizedGemmOps.scala:90-115):
 *   y[m,n] = float(sum_k x[m,k]*wInt8[k,n]) * scalesW[n] * scalesX[m]
 * wInt8 int8 [K,N], scalesW f32 [N], x int8 [M,K], scalesX f32 [M], y f32 [M,N].
 * Bit-exact with the reference arithmetic. */
QGEMM_API qgemm_status qgemm_w8a32_gemm(qgemm_stream_t s, uint64_t wInt8, uint64_t scalesW,
                              uint64_t x, uint64_t scalesX, uint64_t y,
                              int M, int N, int K);

/* QuantizedGemmOps.w4a16Gemm (QuantizedGemmOps.scala:218-247): wInt4 holds
 * K*N nibbles (element k*N+n in byte (k*N+n)/2, low nibble first), zero point
 * 8, per-column f32 scalesW [N], x f32 [M,K], y f32 [M,N].  Bit-exact (same
 * per-element fp32 summation order). */
QGEMM_API qgemm_status qgemm_w4a16_gemm(qgemm_stream_t s, uint64_t wInt4, uint64_t scalesW,
                              uint64_t x, uint64_t y, int M, int N, int K);

/* QuantizedGemmOps.w8a16Gemm (QuantizedGemmOps.scala:24-55). Bit-exact. */
QGEMM_API qgemm_status qgemm_w8a16_gemm(qgemm_stream_t s, uint64_t wInt8, uint64_t scalesW,
                              uint64_t x, uint64_t bias, uint64_t y,
                              int M, int N, int K, int hasBias);

/* QuantizedGemmOps.w8a16GemmRowWise (QuantizedGemmOps.scala:61-84). Bit-exact. */
QGEMM_API qgemm_status qgemm_w8a16_gemm_rowwise(qgemm_stream_t s, uint64_t wInt8, uint64_t scalesW,
                                      uint64_t x, uint64_t y, int M, int N, int K);

/* QuantizedGemmOps.dynamicQuantize (QuantizedGemmOps.scala:121-157). */
QGEMM_API qgemm_status qgemm_dynamic_quantize(qgemm_stream_t s, uint64_t weight, uint64_t scales,
                                    uint64_t qWeight, int K, int N, int qBits);

/* QuantizedGemmOps.weightOnlyQuantizePerChannel (QuantizedGemmOps.scala:163-192). */
QGEMM_API qgemm_status qgemm_weight_only_quantize_per_channel(qgemm_stream_t s, uint64_t weight,
                                                    uint64_t scales, uint64_t qWeight,
                                                    uint64_t zeros, int K, int N);

/* QuantizedGemmOps.dequantize (QuantizedGemmOps.scala:198-212). */
QGEMM_API qgemm_status qgemm_dequantize(qgemm_stream_t s, uint64_t qWeight, uint64_t scales,
                              uint64_t weight, int K, int N);

/* ---- B200 entry points behind the same facade ----------------------------- */

/* W8A8 GEMM with per-token x per-channel dequant: the w8a32Gemm arithmetic
 * (QuantizedGemmOps.scala:102-113) with a choice of B layout and output type.
 *   A    int8 [M,K] row-major (activations, the reference `x`)
 *   B    int8, b_layout QGEMM_B_KN ([K,N], the reference `wInt8`) or QGEMM_B_NK
 *   sA   f32 [M] (per token, `scalesX`);  sB f32 [N] (per channel, `scalesW`)
 *   out  [M, ldc] of out_dtype (QGEMM_F32 or QGEMM_BF16, RNE); ldc >= N
 *   acc_i32  optional int32 [M, N] (ld N) raw accumulators, 0 for none
 * The int8 GEMM names of TensorCoreOps and CutlassGemm (below) run on the same
 * kernel. */
QGEMM_API qgemm_status qgemm_w8a8_gemm(qgemm_stream_t s, uint64_t A, uint64_t B, int b_layout,
                             uint64_t sA, uint64_t sB, uint64_t out, int out_dtype,
                             int ldc, int M, int N, int K, uint64_t acc_i32, int algo);

/* TensorCoreOps.tensorCoreGemmInt8 (operators/intrinsic/TensorCoreOps.scala:294-340),
 * same parameters in the same order:
 *   d[m*ldd + n] = sum_k a[m*lda + k] * b[k*ldb + n]  (+ c[m*ldc + n] when hasC != 0)
 * a, b int8; c, d int32; sums wrap modulo 2^32 like Scala Int.  scalesA / scalesB are
 * accepted and not read (the reference body never reads them either).  The body's
 * -128 offset on signed bytes, its visiting only every 16th k and its one output per
 * 16 x 16 block are not reproduced: every output gets the whole sum.  Runs on the
 * tensor cores (sums plus c written from the accumulators) when lda and ldb are
 * multiples of 16 and a, b are 16-byte aligned, else on an exact CUDA-core kernel;
 * both give the same bits.  Requires lda >= K, ldb >= N, ldd >= N (ldc >= N with c),
 * 4-byte aligned c, d. */
QGEMM_API qgemm_status qgemm_tensor_core_gemm_int8(qgemm_stream_t s, uint64_t a, uint64_t b,
                                                   uint64_t scalesA, uint64_t scalesB,
                                                   uint64_t c, uint64_t d, int M, int N, int K,
                                                   int lda, int ldb, int ldc, int ldd, int hasC);

/* CutlassGemm.int8GemmKernel (cutlass/CutlassGemm.scala:987-1041), same parameters in
 * the same order:
 *   D[m*ldd + n] = (sum_k float(A[m*lda + k]) * float(B[k*ldb + n])) * scaleA * scaleB
 * A, B int32 arrays holding int8 values; D fp32.  Values in [-128, 127] run on the
 * tensor cores as an exact integer sum rounded once to fp32, then (x * scaleA) * scaleB:
 * bit-identical to the reference's fp32 loop while no partial sum leaves +-2^24 (always
 * for K <= 1040), the correctly rounded sum beyond that.  If any value lies outside
 * [-128, 127], the reference's own fp32 loop (k ascending, each product and sum rounded
 * on its own) computes the whole output on CUDA cores instead.  One accumulator per
 * output (the body shares one among 64 outputs).  Requires lda >= K, ldb >= N,
 * ldd >= N, M <= 65535, 4-byte aligned pointers.  Packed operands live in the stream
 * handle's scratch (made or grown by the call; make one call before graph capture). */
QGEMM_API qgemm_status qgemm_int8_gemm_kernel(qgemm_stream_t s, uint64_t D, uint64_t A,
                                              uint64_t B, int M, int N, int K, int lda, int ldb,
                                              int ldd, float scaleA, float scaleB);

/* qgemm_w8a8_gemm for callers that must not allocate device memory during the call
 * (no counterpart in the reference).  qgemm_w8a8_gemm may make scratch on the stream
 * handle the first time a shape's last tile round is split along K; this variant
 * takes that scratch from a 20 MiB static array inside the library instead, so a
 * serving loop with a fixed memory budget, or a host that accounts for every device
 * allocation, can call it at any time.  Same arguments, same results (bit for bit).
 * - Nothing is allocated.  The array's address is looked up once per device, on the
 *   first call there; make that first call during set-up.
 * - Its 4 KiB of counters must be zero when a GEMM starts; each call clears them
 *   on the stream before its kernel (and leaves them zero).
 * - One array per device: calls whose GEMMs could overlap (different streams, no
 *   ordering between them) race on it.  Issue them on one stream, or order them.
 * - A split larger than the array (more than 20 leftover pair tiles, i.e. GPUs with
 *   more than 160 SMs) is refused with QGEMM_ERR_UNSUPPORTED. */
QGEMM_API qgemm_status qgemm_w8a8_gemm_static_scratch(qgemm_stream_t s, uint64_t A, uint64_t B,
                                                      int b_layout, uint64_t sA, uint64_t sB,
                                                      uint64_t out, int out_dtype, int ldc, int M,
                                                      int N, int K, uint64_t acc_i32, int algo);

/* Group-wise W4A16 GEMV/GEMM for decode (the w4a16Gemm arithmetic,
 * QuantizedGemmOps.scala:229-245, with a zero point and per-group scales):
 *   x   bf16 [M,K];  wq uint32 [K, N/8]: nibble j of word (k, c) is q[k][8c+j]
 *       (the reference nibble order read as little-endian words)
 *   scales bf16 [K/group_size, N];  y bf16 [M,N] (RNE)
 *   y[m,n] = sum_k (q[k,n] - zero_point) * scales[k/G, n] * x[m,k]
 * Requires N % 8 == 0 and K % group_size == 0; 16-byte aligned wq, x, y. */
QGEMM_API qgemm_status qgemm_w4a16_grouped_gemm(qgemm_stream_t s, uint64_t x, uint64_t wq,
                                      uint64_t scales, int zero_point, int group_size,
                                      uint64_t y, int M, int N, int K);

/* The same group-wise W4A16 on weights repacked once by qgemm_prepack_w4_tiled
 * (64-column tiles, each tile's rows contiguous, so every CTA streams one block of
 * memory: the fast decode path).  Requires sm_100, K % 16 == 0, group_size a
 * multiple of 16 that divides 512 or is a multiple of 512, N % 8 == 0 and 16-byte
 * aligned x, wt and scales; otherwise QGEMM_ERR_UNSUPPORTED.  Deterministic. */
QGEMM_API qgemm_status qgemm_w4a16_grouped_gemm_tiled(qgemm_stream_t s, uint64_t x, uint64_t wt,
                                                      uint64_t scales, int zero_point,
                                                      int group_size, uint64_t y, int M, int N,
                                                      int K);

/* One-time int4 weight repack: uint32 [K, N/8] (reference nibble order) ->
 * tiled[t][k][32 bytes] = bytes [32*t, 32*t+32) of row k, for 64-column tiles t
 * (zero-padded past N).  qgemm_w4_tiled_bytes gives the buffer size. */
QGEMM_API qgemm_status qgemm_w4_tiled_bytes(int K, int N, size_t* bytes);
QGEMM_API qgemm_status qgemm_prepack_w4_tiled(qgemm_stream_t s, uint64_t wq, uint64_t dst, int K,
                                              int N);

/* The same group-wise W4A16 on weights repacked once by qgemm_prepack_w4_frag
 * (fragment order: each SM streams an equal, contiguous share of the columns; the
 * fast decode path).  M <= 4 reads 8-column groups; up to 16 rows with N % 16 == 0
 * and K <= 4096 read 16-column pairs; more rows, or K past 4096 (past 8192 at
 * M <= 4), with N % 16 == 0 run a K-split kernel over thread-block clusters in passes
 * of 32 rows, each weight read once a pass; other shapes run passes of 4 rows.
 * Requires sm_100, K % 16 == 0, K <= 16384 when N % 16 == 0 and K <= 8192
 * otherwise, group_size 32, 64 or a multiple of 128, N % 8 == 0 and 16-byte aligned
 * x, wf and scales; otherwise QGEMM_ERR_UNSUPPORTED.  Deterministic. */
QGEMM_API qgemm_status qgemm_w4a16_grouped_gemm_frag(qgemm_stream_t s, uint64_t x, uint64_t wf,
                                                     uint64_t scales, int zero_point,
                                                     int group_size, uint64_t y, int M, int N,
                                                     int K);

/* One-time int4 weight repack: uint32 [K, N/8] (reference nibble order) -> the
 * fragment order: unit (c, kb) = columns 8c..8c+7 x rows 128kb..128kb+127, 512 bytes,
 * units ordered c-major; inside a unit, lane 4g+t's four words (one per 32 rows)
 * hold column 8c+g at rows sb + 8t + {0, 4, 2, 6, 1, 5, 3, 7}
 * (sb = 128kb + 32*word), nibble i at bits 4i..4i+3, zero past K.
 * qgemm_w4_frag_bytes gives the buffer size (N/8 * ceil(K/128) * 512). */
QGEMM_API qgemm_status qgemm_w4_frag_bytes(int K, int N, size_t* bytes);
QGEMM_API qgemm_status qgemm_prepack_w4_frag(qgemm_stream_t s, uint64_t wq, uint64_t dst, int K,
                                             int N);

/* Group-wise W4A16 GEMM for prefill-sized M (the same arithmetic as
 * qgemm_w4a16_grouped_gemm on the same prepacked weights `wt`): the weights are
 * expanded slab by slab into the caller's workspace and multiplied on the tensor
 * cores with exact products and fp32 sums.  When group_size is a multiple of 64 and
 * `scales` is 16-byte aligned, the slab holds q - zero_point (exact in bf16) and the
 * scales are applied in fp32 to each group's partial sums (the algorithmic tensor
 * work); otherwise each (q - zero_point) * scale is stored as two bf16 values hi + lo
 * that sum to it exactly (twice the tensor work).  The two forms round differently.
 * Any M; meant for M in the hundreds and above, where the expansion is a few percent
 * of the call.  workspace: 16-byte aligned, at least 1024 * Kp bytes (one 256-column
 * slab; Kp = K rounded up to a multiple of 64); qgemm_w4a16_prefill_workspace_bytes
 * gives the size that holds all of N in one slab.  Requires sm_100, K % 8 == 0,
 * K % group_size == 0, N % 8 == 0 and 16-byte aligned x, wt, y.  Deterministic. */
QGEMM_API qgemm_status qgemm_w4a16_prefill_workspace_bytes(int K, int N, size_t* bytes);
QGEMM_API qgemm_status qgemm_w4a16_grouped_gemm_prefill(qgemm_stream_t s, uint64_t x, uint64_t wt,
                                                        uint64_t scales, int zero_point,
                                                        int group_size, uint64_t y, int M, int N,
                                                        int K, uint64_t workspace,
                                                        size_t workspace_bytes);
/* The same prefill GEMM on weights in the fragment order of qgemm_prepack_w4_frag,
 * so that one stored copy serves both prefill and the frag decode path.  The
 * workspace is as above; additionally requires K % 16 == 0 and group_size 32, 64 or
 * a multiple of 128. */
QGEMM_API qgemm_status qgemm_w4a16_grouped_gemm_prefill_frag(qgemm_stream_t s, uint64_t x,
                                                             uint64_t wf, uint64_t scales,
                                                             int zero_point, int group_size,
                                                             uint64_t y, int M, int N, int K,
                                                             uint64_t workspace,
                                                             size_t workspace_bytes);
/* Both prefill forms behind one call, with flags:
 *   QGEMM_PREFILL_FRAG      w is in the fragment order of qgemm_prepack_w4_frag (else
 *                           the 64-column tiles of qgemm_prepack_w4_tiled);
 *   QGEMM_PREFILL_ONE_TERM  each weight is expanded to one bf16 value, bf16((q - zp) *
 *                           scale) rounded to nearest even, instead of the exact pair:
 *                           the algorithmic tensor work and half the workspace
 *                           (512 * Kp bytes a 256-column slab); each product then
 *                           carries the weight's rounding (relative error <= 2^-9).
 * qgemm_w4a16_prefill_workspace_bytes_ex gives the full-N workspace for the flags.
 * Unknown flag bits are QGEMM_ERR_INVALID_ARG. */
#define QGEMM_PREFILL_FRAG 1
#define QGEMM_PREFILL_ONE_TERM 2
QGEMM_API qgemm_status qgemm_w4a16_prefill_workspace_bytes_ex(int K, int N, int flags,
                                                              size_t* bytes);
QGEMM_API qgemm_status qgemm_w4a16_grouped_gemm_prefill_ex(qgemm_stream_t s, uint64_t x,
                                                           uint64_t w, uint64_t scales,
                                                           int zero_point, int group_size,
                                                           uint64_t y, int M, int N, int K,
                                                           uint64_t workspace,
                                                           size_t workspace_bytes, int flags);

/* bf16 GEMM on the tcgen05 kernels (no counterpart among the reference's quantized
 * operators; it is the multiply of the W4A16 prefill path):
 *   out[M, ldc] (bf16, RNE) = A[M,K] * B[N,K]^T with fp32 sums; A, B bf16 K-major.
 * Requires sm_100, K % 8 == 0, ldc >= N, ldc % 8 == 0, 16-byte aligned A, B, out. */
QGEMM_API qgemm_status qgemm_gemm_bf16_nk(qgemm_stream_t s, uint64_t A, uint64_t B, uint64_t out,
                                          int ldc, int M, int N, int K);

/* Dynamic per-token int8 quantisation of activations: the arithmetic of
 * QuantizedGemmOps.dynamicQuantize (QuantizedGemmOps.scala:121-157) applied to each
 * row of x (a token) instead of each column of a weight.  x [M,K] fp32 or bf16
 * (in_dtype QGEMM_F32 / QGEMM_BF16), q int8 [M,K], sA f32 [M] = maxAbs / 127: the A
 * operand and per-token scales of qgemm_w8a8_gemm.  Bit-exact with the reference
 * arithmetic (NaN ignored by the max, Scala toInt truncation and saturation). */
QGEMM_API qgemm_status qgemm_quantize_per_token(qgemm_stream_t s, uint64_t x, int in_dtype,
                                                uint64_t q, uint64_t sA, int M, int K);

/* Epilogues of qgemm_gemm_f32. */
typedef enum {
  QGEMM_F32_MATMUL = 0,       /* C = A x B                          */
  QGEMM_F32_MATMUL_BIAS = 1,  /* C = A x B + bias[N]                */
  QGEMM_F32_SGEMM = 2         /* C = alpha * (A x B) + beta * C     */
} qgemm_f32_mode;

/* fp32 entry points of the same facade, all operands fp32 row-major:
 *   qgemm_matmul_f32           C[M,N] = A[M,K] x B[K,N]      MatrixOps.matmul
 *                              (operators/linalg/MatrixOps.scala:16-28)
 *   qgemm_matmul_add_bias_f32  C = A x B + bias[N]           MatrixOps.matmulAddBias (:31-44)
 *   qgemm_sgemm                C = alpha * (A x B) + beta * C BLASOps.sgemm (:230-243);
 *                              C is read whatever beta is, as in the reference
 *   qgemm_gemv_f32             y[M] = A[M,N] x x[N]          MatrixOps.gemv (:166-177)
 * The GEMMs (qgemm_gemm_f32 with algo QGEMM_ALGO_AUTO) run on the sm_100 tensor cores
 * as three tf32 products per fp32 product (hi/lo splits of both operands) with fp32
 * sums, or, for M <= 64 or N <= 64 (and on other GPUs), on CUDA cores as a split-K fp32
 * GEMM that reads B once.  Both meet |C - exact| <= 1e-5 * sum_k |A*B| terms, the
 * accuracy of the reference's sequential fp32 loop.  An infinite input sends the whole
 * call through a CUDA-core kernel in the reference's own order (bit-identical to the
 * loop).  Split operands (8 * (M + N) * roundup(K, 32) bytes) or partial sums live in
 * the stream handle's scratch, made or grown by the call (make one call before
 * capturing the stream into a graph).  Deterministic.  4-byte aligned pointers. */
QGEMM_API qgemm_status qgemm_gemm_f32(qgemm_stream_t s, uint64_t A, uint64_t B, uint64_t bias,
                                      uint64_t C, int M, int N, int K, float alpha, float beta,
                                      int mode, int algo);
QGEMM_API qgemm_status qgemm_matmul_f32(qgemm_stream_t s, uint64_t A, uint64_t B, uint64_t C,
                                        int M, int N, int K);
QGEMM_API qgemm_status qgemm_matmul_add_bias_f32(qgemm_stream_t s, uint64_t A, uint64_t B,
                                                 uint64_t bias, uint64_t C, int M, int N, int K);
QGEMM_API qgemm_status qgemm_sgemm(qgemm_stream_t s, uint64_t A, uint64_t B, uint64_t C, int M,
                                   int N, int K, float alpha, float beta);
QGEMM_API qgemm_status qgemm_gemv_f32(qgemm_stream_t s, uint64_t A, uint64_t x, uint64_t y, int M,
                                      int N);

/* One-time weight repack: int8 [K,N] (reference layout) -> [N,K] (K-major). */
QGEMM_API qgemm_status qgemm_prepack_w8_nk(qgemm_stream_t s, uint64_t src_kn, uint64_t dst_nk,
                                 int K, int N);

/* Launch by reference kernel name, the by-name path of
 * TritonKernelRunner.launchKernel (dsl/TritonKernelRunner.scala:68-73).
 * bufs are device addresses in the reference method's parameter order, ints
 * the Int parameters in order (Bool as 0/1).  Names: "w8a32Gemm", "w4a16Gemm",
 * "w8a16Gemm", "w8a16GemmRowWise", "dynamicQuantize",
 * "weightOnlyQuantizePerChannel", "dequantize", "matmul", "matmulAddBias", "gemv",
 * "tensorCoreGemmInt8" (sgemm and int8GemmKernel take Float parameters: use
 * qgemm_bridge_launch_kernel below).  Unknown name -> INVALID_ARG. */
QGEMM_API qgemm_status qgemm_launch_by_name(qgemm_stream_t s, const char* name,
                                  const uint64_t* bufs, int nbufs,
                                  const int* ints, int nints);

/* CUDARuntimeJavaBridge.launchKernel (driver/CUDARuntimeJavaBridge.scala:121-165), same
 * parameters in the same order after the stream: a kernel name, the grid and block
 * triples (accepted and not used: each kernel here picks its own launch shape),
 * bufferAddrs with the result buffer first and the method's other Ptr parameters after
 * it in declaration order, and scalarVals with scalarKeys naming the method's scalar
 * parameters ("M", "alpha", "hasBias", ...).  Without keys (scalarKeys null) the values
 * are the scalar parameters in declaration order.  Int and Bool parameters travel as
 * Float, as in the bridge: they must be integral (|v| <= 2^24; Bool 0 or 1).  A scalar
 * left out takes the method's default (qBits = 8) or is an error.  Names: every name of
 * qgemm_launch_by_name plus "sgemm" (alpha, beta) and "int8GemmKernel" (scaleA,
 * scaleB).  Returns bufferAddrs[0] once the launch is queued, -1 on any failure (the
 * message in qgemm_last_error()), like the bridge's -1L. */
QGEMM_API int64_t qgemm_bridge_launch_kernel(qgemm_stream_t s, const char* name, int gridX,
                                             int gridY, int gridZ, int blockX, int blockY,
                                             int blockZ, const uint64_t* bufferAddrs, int nbufs,
                                             const float* scalarVals,
                                             const char* const* scalarKeys, int nscalars);

/* ---- weight blobs ------------------------------------------------------------
 * A versioned file holding quantised weights already in a kernel layout, with
 * their scales, so that a model loads straight into device memory (no repack).
 * No counterpart in the reference, whose weights live in host arrays.  The int4
 * layout of the reference's w4a16Gemm (two nibbles per byte along the flattened
 * (k, n) index, low nibble first; QuantizedGemmOps.scala:234-238) is, for even N,
 * byte for byte the uint32 [K, N/8] layout of qgemm_w4a16_grouped_gemm, so
 * reference weights import with qgemm_prepack_w4_tiled and no other conversion.
 * Every read checks the magic, the version, the sizes against the shape and a
 * CRC-32 of each section; a mismatch is QGEMM_ERR_INVALID_ARG, another version
 * QGEMM_ERR_UNSUPPORTED. */
#define QGEMM_BLOB_VERSION 1
enum {
  QGEMM_BLOB_W4_TILED = 1,  /* qgemm_prepack_w4_tiled layout + bf16 scales [K/G, N]   */
  QGEMM_BLOB_W8_KN = 2,     /* int8 [K, N] (reference wInt8 layout) + f32 scales [N]  */
  QGEMM_BLOB_W8_NK = 3,     /* int8 [N, K] + f32 scales [N]                           */
  QGEMM_BLOB_W4_FRAG = 4    /* qgemm_prepack_w4_frag layout + bf16 scales [K/G, N]    */
};
typedef struct qgemm_blob_info {
  uint32_t version;      /* filled in by qgemm_blob_info_read                         */
  int32_t kind;
  int32_t K, N;
  int32_t group_size;    /* int4: rows per scale group; int8: 0                       */
  int32_t zero_point;    /* int4: 0..15; int8: 0                                      */
  uint64_t weight_bytes; /* filled in by qgemm_blob_info_read                         */
  uint64_t scale_bytes;  /* filled in by qgemm_blob_info_read                         */
} qgemm_blob_info;
/* Writes host buffers (sizes implied by kind and shape) to `path`. */
QGEMM_API qgemm_status qgemm_blob_save(const char* path, const qgemm_blob_info* info,
                                       const void* weights, const void* scales);
QGEMM_API qgemm_status qgemm_blob_info_read(const char* path, qgemm_blob_info* info);
/* Reads and verifies both sections into host buffers of at least the given sizes. */
QGEMM_API qgemm_status qgemm_blob_load(const char* path, void* weights, size_t weight_bytes,
                                       void* scales, size_t scale_bytes);
/* Verifies the whole file, then copies both sections to device buffers (returns
 * after the copies have finished). */
QGEMM_API qgemm_status qgemm_blob_load_device(qgemm_stream_t s, const char* path, uint64_t weights,
                                              size_t weight_bytes, uint64_t scales,
                                              size_t scale_bytes);

/* ---- column sharding and the output all-gather ----------------------------
 * The reference has only a host-array NCCL wrapper (nccl/NCCLCommunicator.scala:
 * 35-92, 151-163, 302-320) with no unique-id exchange.  Here rank r holds the
 * weight columns [n0, n1) of qgemm_shard_columns and the output all-gather is
 * a device-buffer ncclAllGather on the caller's stream. */
QGEMM_API qgemm_status qgemm_shard_columns(int N, int world, int rank, int align, int* n0, int* n1);
/* 128-byte ncclUniqueId, made on one rank and sent to the others by the caller. */
QGEMM_API qgemm_status qgemm_comm_unique_id(void* out_128_bytes);
QGEMM_API qgemm_status qgemm_comm_init(qgemm_device_t dev, const void* unique_id_128, int rank,
                             int world, qgemm_comm_t* out);
QGEMM_API qgemm_status qgemm_comm_destroy(qgemm_comm_t comm);
/* recv[r*count .. (r+1)*count) <- send of rank r; count in bf16 elements. */
QGEMM_API qgemm_status qgemm_comm_allgather_bf16(qgemm_comm_t comm, qgemm_stream_t s, uint64_t send,
                                       uint64_t recv, size_t count);
/* [world][M][ncols] bf16 gather buffer -> [M][world*ncols] row-major. */
QGEMM_API qgemm_status qgemm_unshard_columns_bf16(qgemm_stream_t s, uint64_t gathered, uint64_t out,
                                        int world, int M, int ncols);

/* The column-sharded W8A8 GEMM followed by its output all-gather, pipelined over
 * chunks of `chunk_rows` rows of M (the NCCL all-gather step of NCCLOps.ncclAllGather,
 * NCCLOps.scala:302-320, fed by the GEMM instead of host arrays): the GEMM of chunk i
 * runs on stream s while the in-place all-gather and unshard of chunk i-1 run on
 * stream cs, on every rank of `comm`.  This rank's B [K, N_local] (b_layout as in
 * qgemm_w8a8_gemm) and sB [N_local]; A [M, K] and sA [M] are the same on every rank.
 * out: bf16 [M, N_local * world], the whole output, on every rank.  work: at least
 * qgemm_w8a8_allgather_work_bytes(world, min(chunk_rows, M), N_local) bytes, 16-byte
 * aligned (two chunks of gather buffers).  s and cs must differ; when the call
 * returns, s is ordered after all of its work (cs too has finished it).  The events it
 * needs are made on the communicator's first call.  Every rank must make the same
 * calls in the same order, with the same M, N_local, K and chunk_rows: equal shards, so
 * N a multiple of align * world in qgemm_shard_columns.  NCCL requires equal counts and
 * a mismatch is not detected.  Argument errors are returned before the call queues its
 * first collective, on the rank that made them; a failure after that point aborts the
 * communicator (ncclCommAbort) and every later call on it returns
 * QGEMM_ERR_BAD_HANDLE, so that no rank goes on as if the step had completed. */
QGEMM_API size_t qgemm_w8a8_allgather_work_bytes(int world, int chunk_rows, int n_local);
QGEMM_API qgemm_status qgemm_w8a8_gemm_allgather_bf16(qgemm_comm_t comm, qgemm_stream_t s,
                                                      qgemm_stream_t cs, uint64_t A, uint64_t B,
                                                      int b_layout, uint64_t sA, uint64_t sB,
                                                      uint64_t out, int M, int N_local, int K,
                                                      int chunk_rows, uint64_t work,
                                                      size_t work_bytes);

/* A buffer registered by every rank of `comm` together (collective; every rank passes
 * its own buffer of the same size): `buf` must lie in one cudaMalloc allocation and be
 * 16-byte aligned.  Each rank maps the peers' buffers into its own address space (CUDA
 * IPC), so one process per GPU; one window per allocation at a time.  `s` carries the
 * exchange and is synchronised.  Release a window (a local call) after the work that
 * uses it has finished on every rank and before qgemm_comm_destroy.  Every rank returns
 * the same verdict: the buffers are checked on every rank and the results gathered
 * before any rank maps its peers' buffers, and the mapping results are gathered again
 * before any rank keeps the window. */
QGEMM_API qgemm_status qgemm_comm_window_register(qgemm_comm_t comm, qgemm_stream_t s,
                                                  uint64_t buf, size_t bytes,
                                                  qgemm_window_t* out);
QGEMM_API qgemm_status qgemm_comm_window_release(qgemm_window_t w);

/* The same sharded GEMM + all-gather into a registered window, [M, N_local * world]
 * bf16 on every rank.  The GEMM of each chunk of `chunk_rows` rows writes this rank's
 * columns of the window in place (ldc = N_local * world) on stream s; the copy engines
 * then write those columns into every peer's window over NVLink while the GEMM of the
 * next chunk runs, on a stream the communicator owns (or on as many as the environment
 * variable QGEMM_COPY_STREAMS says, 1 .. world-1, one peer's copies on each).  No gather buffer and no unshard pass: the copies
 * land in the final layout.  Two barriers on cs (one-element NCCL gathers) bracket
 * the copies: no rank writes into a peer's window before the peer has finished its
 * earlier work on s, and the call completes on s only when every peer's columns have
 * arrived.  Every rank must make the same calls in the same order, with the same M,
 * N_local, K and chunk_rows (equal shards); a mismatch is not detected (the window's
 * size bounds every copy).  Errors behave as in qgemm_w8a8_gemm_allgather_bf16. */
QGEMM_API qgemm_status qgemm_w8a8_gemm_allgather_window_bf16(qgemm_window_t w, qgemm_stream_t s,
                                                             qgemm_stream_t cs, uint64_t A,
                                                             uint64_t B, int b_layout,
                                                             uint64_t sA, uint64_t sB, int M,
                                                             int N_local, int K,
                                                             int chunk_rows);

/* The sharded GEMM and the all-gather as one kernel, into a registered window
 * ([M, N_local * world] bf16 on every rank): the GEMM's epilogue stores each output
 * chunk into this rank's columns of its own window and, with TMA stores over NVLink
 * from the same staging buffer (no multicast), into the same columns of every peer's
 * window.  A tile's transfer overlaps the next tile's MMAs, so the layer takes the
 * longer of the GEMM and this rank's egress instead of their sum; there is no gather
 * buffer, no copy stream and no unshard pass.  Two one-element NCCL gathers on s
 * bracket the GEMM: no rank writes into a peer's window before the peer has finished
 * its earlier work on s, and the call completes on s only when every rank's columns
 * have arrived.  Requires sm_100, world <= 8, K > 0 with K % 16 == 0, N_local % 8 == 0
 * (% 16 with B in [K,N]) and 16-byte aligned A and B; otherwise QGEMM_ERR_UNSUPPORTED,
 * before any collective (the same verdict on every rank when the shapes agree).  Every rank must make the same calls in the same order, with
 * the same M, N_local and K.  Errors after the first gather abort the communicator,
 * as in qgemm_w8a8_gemm_allgather_bf16. */
QGEMM_API qgemm_status qgemm_w8a8_gemm_allgather_fused_bf16(qgemm_window_t w, qgemm_stream_t s,
                                                            uint64_t A, uint64_t B,
                                                            int b_layout, uint64_t sA,
                                                            uint64_t sB, int M, int N_local,
                                                            int K);

#ifdef __cplusplus
}
#endif
#endif /* QGEMM_H */
