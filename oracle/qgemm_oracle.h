/*
 * qgemm_oracle.h -- CPU restatement of the reference's quantized-matmul operators
 * and of the fp32 matmul / sgemm / gemv of the same facade.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * libqgemm: only tests/, __graft_entry__.smoke() and the cpu_baseline /
 * reference legs of bench.py load it.  It is never linked into libqgemm and
 * never used as a fallback.
 *
 * Parity status: UNPINNED.  The reference (bytedeco/cuda-triton-scala) keeps
 * these operators as Scala bodies in
 *   src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala
 * that no test, fixture or golden vector exercises, and that cannot be run
 * here (no JVM; its thread builtins are constant stubs, so a JVM call computes
 * only element (0,0)).  Each function below restates one operator body
 * statement by statement, with the reference's arithmetic order, and is pinned
 * only by hand-computed known-answer cases and an independent pure-Python
 * restatement (tests/golden/make_golden.py).  The fp32 operators
 * (operators/linalg/MatrixOps.scala) are likewise untested in the reference; their
 * restatement is pinned by known answers and by float64 error bounds.
 *
 * Floating point: the library is compiled with -ffp-contract=off on x86-64
 * (SSE scalar float), which gives the same IEEE-754 binary32
 * round-to-nearest-even results as the JVM's float arithmetic.
 */
#ifndef QGEMM_ORACLE_H
#define QGEMM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* bf16 encoders.  RNE is the encoder the CUDA path uses; the truncating one is
 * the reference's BFloat16 conversion (core/Types.scala:515-519). */
uint16_t oracle_f32_to_bf16_rne(float f);
uint16_t oracle_f32_to_bf16_trunc(float f);
float    oracle_bf16_to_f32(uint16_t h);

/* Scala Float.toInt: truncation toward zero, NaN -> 0, saturating. */
int32_t  oracle_scala_f2i(float f);

/* QuantizedGemmOps.w8a32Gemm (QuantizedGemmOps.scala:90-115).
 * wInt8 [K,N] row-major, scalesW [N], x [M,K] int8 row-major, scalesX [M],
 * y [M,N] fp32.  acc (optional, may be NULL) receives the int32 sums. */
void oracle_w8a32_gemm(const int8_t* wInt8, const float* scalesW,
                       const int8_t* x, const float* scalesX, float* y,
                       int M, int N, int K, int32_t* acc);

/* Same arithmetic, loop-interchanged (m, k, n) and OpenMP-parallel over rows.
 * Integer sums are order-independent, so results are bit-identical to
 * oracle_w8a32_gemm.  out_bf16 (optional) receives RNE(y); y may be NULL
 * when only out_bf16 is wanted; acc (optional) receives the int32 sums.  Rows
 * [m0, m1) only (a bounded sample). */
void oracle_w8a8_gemm_rows(const int8_t* wInt8, const float* scalesW,
                           const int8_t* x, const float* scalesX,
                           float* y, uint16_t* out_bf16, int32_t* acc,
                           int M, int N, int K, int m0, int m1, int threads);

/* QuantizedGemmOps.w4a16Gemm (QuantizedGemmOps.scala:218-247).
 * wInt4: K*N nibbles, element i = k*N+n in byte i/2, low nibble when i is
 * even; zero point 8; scalesW [N]; x [M,K] fp32; y [M,N] fp32. */
void oracle_w4a16_gemm(const uint8_t* wInt4, const float* scalesW,
                       const float* x, float* y, int M, int N, int K);

/* Group-wise generalisation of w4a16Gemm used by the bf16 decode path:
 * wq uint32 [K, N/8] (the same bytes as the reference nibble order read as
 * little-endian words), scales bf16 [ceil(K/G), N], x bf16 [M,K].
 *   sum += ((float)(q - zp) * s[k/G][n]) * x[m][k]   (fp32, k ascending)
 * y_f32 (optional) gets sum, y_bf16 (optional) gets RNE(sum).
 * With G = K, zp = 8 and fp32 inputs this is exactly w4a16Gemm.
 * Columns [n0, n1) only; OpenMP over columns when threads > 1. */
void oracle_w4a16_grouped(const uint32_t* wq, const uint16_t* scales,
                          int zero_point, int group_size,
                          const uint16_t* x, float* y_f32, uint16_t* y_bf16,
                          int M, int N, int K, int n0, int n1, int threads);

/* QuantizedGemmOps.w8a16Gemm (QuantizedGemmOps.scala:24-55). */
void oracle_w8a16_gemm(const int8_t* wInt8, const float* scalesW,
                       const float* x, const float* bias, float* y,
                       int M, int N, int K, int hasBias);

/* QuantizedGemmOps.w8a16GemmRowWise (QuantizedGemmOps.scala:61-84). */
void oracle_w8a16_gemm_rowwise(const int8_t* wInt8, const float* scalesW,
                               const float* x, float* y, int M, int N, int K);

/* QuantizedGemmOps.dynamicQuantize (QuantizedGemmOps.scala:121-157). */
void oracle_dynamic_quantize(const float* weight, float* scales,
                             int8_t* qWeight, int K, int N, int qBits);

/* QuantizedGemmOps.weightOnlyQuantizePerChannel (QuantizedGemmOps.scala:163-192). */
void oracle_weight_only_quantize_per_channel(const float* weight, float* scales,
                                             int8_t* qWeight, int8_t* zeros,
                                             int K, int N);

/* QuantizedGemmOps.dequantize (QuantizedGemmOps.scala:198-212). */
void oracle_dequantize(const int8_t* qWeight, const float* scales,
                       float* weight, int K, int N);

/* MatrixOps.matmul / matmulAddBias / BLASOps.sgemm (MatrixOps.scala:16-44,
 * :230-243): mode 0 C = A x B, 1 C = A x B + bias, 2 C = alpha (A x B) + beta C.
 * threads <= 0: all (OpenMP over rows; each element's order is unchanged). */
void oracle_matmul_f32(const float* A, const float* B, const float* bias, float* C,
                       int M, int N, int K, float alpha, float beta, int mode,
                       int threads);

/* MatrixOps.gemv (MatrixOps.scala:166-177): y = A x, A [M,N]. */
void oracle_gemv_f32(const float* A, const float* x, float* y, int M, int N);

/* TensorCoreOps.tensorCoreGemmInt8 (operators/intrinsic/TensorCoreOps.scala:294-340),
 * its arithmetic for every output: d[m*ldd+n] = sum_k a[m*lda+k] * b[k*ldb+n]
 * (+ c[m*ldc+n] when hasC), int32 wrapping. */
void oracle_tensor_core_gemm_int8(const int8_t* a, const int8_t* b, const int32_t* c,
                                  int32_t* d, int M, int N, int K, int lda, int ldb,
                                  int ldc, int ldd, int hasC);

/* CutlassGemm.int8GemmKernel (cutlass/CutlassGemm.scala:987-1041), one fp32
 * accumulator per output: acc += float(A[m*lda+k]) * float(B[k*ldb+n]) in ascending
 * k, then D[m*ldd+n] = (acc * scaleA) * scaleB.  A, B int32 arrays.  OpenMP over rows
 * (threads <= 0: all); each element's order is unchanged. */
void oracle_int8_gemm_kernel(float* D, const int32_t* A, const int32_t* B, int M, int N, int K,
                             int lda, int ldb, int ldd, float scaleA, float scaleB,
                             int threads);

/* Threads the OpenMP build can use (1 without OpenMP). */
int oracle_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
