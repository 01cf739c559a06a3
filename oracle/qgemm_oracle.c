/*
 * qgemm_oracle.c -- CPU restatement of QuantizedGemmOps (test infrastructure).
 *
 * TEST INFRASTRUCTURE ONLY: the checker and the timed CPU baseline, never the
 * product path.  Parity status: UNPINNED (see qgemm_oracle.h for why).
 *
 * Every function cites the reference statements it restates, by
 * path:line within bytedeco/cuda-triton-scala.  Build:
 *   gcc -O2 -fPIC -shared -fopenmp -ffp-contract=off -fno-fast-math
 */
#include "qgemm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#if defined(__FLT_EVAL_METHOD__) && __FLT_EVAL_METHOD__ != 0
#error "the oracle needs binary32 evaluation (SSE), not x87 extended precision"
#endif

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t oracle_f32_to_bf16_rne(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) /* NaN: keep quiet */
    return (uint16_t)((u >> 16) | 0x0040u);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

/* core/Types.scala:515-519: floatToIntBits(value) >> 16, i.e. truncation. */
uint16_t oracle_f32_to_bf16_trunc(float f) { return (uint16_t)(f2u(f) >> 16); }

/* core/Types.scala:522-526. */
float oracle_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* JVM f2i (JLS 5.1.3): NaN -> 0, out of range saturates, else truncate. */
int32_t oracle_scala_f2i(float f) {
  if (f != f) return 0;
  if (f >= 2147483648.0f) return 2147483647;
  if (f <= -2147483648.0f) return (int32_t)0x80000000u;
  return (int32_t)f;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* QuantizedGemmOps.scala:102-113:
 *   var sum32 = 0
 *   for k: sum32 += wInt8(k*N+col).toInt * x(row*K+k).toInt
 *   y(row*N+col) = sum32.toFloat * scalesW(col) * scalesX(row)
 * Scala Int arithmetic wraps modulo 2^32, so the sum is accumulated in
 * uint32 and reinterpreted. */
void oracle_w8a32_gemm(const int8_t* wInt8, const float* scalesW,
                       const int8_t* x, const float* scalesX, float* y,
                       int M, int N, int K, int32_t* acc) {
  for (int row = 0; row < M; ++row) {
    for (int col = 0; col < N; ++col) {
      uint32_t sum32 = 0;
      for (int k = 0; k < K; ++k) {
        int32_t wVal = wInt8[(int64_t)k * N + col];
        int32_t xVal = x[(int64_t)row * K + k];
        sum32 += (uint32_t)(wVal * xVal);
      }
      int32_t s = (int32_t)sum32;
      if (acc) acc[(int64_t)row * N + col] = s;
      float finalVal = ((float)s * scalesW[col]) * scalesX[row];
      if (y) y[(int64_t)row * N + col] = finalVal;
    }
  }
}

void oracle_w8a8_gemm_rows(const int8_t* wInt8, const float* scalesW,
                           const int8_t* x, const float* scalesX,
                           float* y, uint16_t* out_bf16, int32_t* acc,
                           int M, int N, int K, int m0, int m1, int threads) {
  if (m0 < 0) m0 = 0;
  if (m1 > M) m1 = M;
  (void)threads;
#ifdef _OPENMP
  if (threads < 1) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
  for (int row = m0; row < m1; ++row) {
    /* One row of wrapping int32 partial sums; k outer so wInt8 streams
     * row-major.  Integer addition is associative, so this equals the
     * per-element k loop of oracle_w8a32_gemm bit for bit. */
    uint32_t* accrow = (uint32_t*)calloc((size_t)N, sizeof(uint32_t));
    if (!accrow) continue;
    const int8_t* xr = x + (int64_t)row * K;
    for (int k = 0; k < K; ++k) {
      uint32_t xv = (uint32_t)(int32_t)xr[k];
      const int8_t* wr = wInt8 + (int64_t)k * N;
      for (int col = 0; col < N; ++col) accrow[col] += xv * (uint32_t)(int32_t)wr[col];
    }
    for (int col = 0; col < N; ++col) {
      if (acc) acc[(int64_t)row * N + col] = (int32_t)accrow[col];
      float v = ((float)(int32_t)accrow[col] * scalesW[col]) * scalesX[row];
      if (y) y[(int64_t)row * N + col] = v;
      if (out_bf16) out_bf16[(int64_t)row * N + col] = oracle_f32_to_bf16_rne(v);
    }
    free(accrow);
  }
}

/* QuantizedGemmOps.scala:229-245:
 *   byteIdx = (k*N+col)/2 ; qIdx = (k*N+col)%2 ; packed = wInt4(byteIdx).toInt
 *   wVal = qIdx==0 ? (packed & 0x0F).toFloat - 8 : ((packed >> 4) & 0x0F).toFloat - 8
 *   sum += wVal * scale * xVal            (left to right)
 * Byte.toInt sign-extends; (packed >> 4) & 0x0F still yields the high nibble. */
void oracle_w4a16_gemm(const uint8_t* wInt4, const float* scalesW,
                       const float* x, float* y, int M, int N, int K) {
  for (int row = 0; row < M; ++row) {
    for (int col = 0; col < N; ++col) {
      float sum = 0.0f;
      for (int k = 0; k < K; ++k) {
        int64_t idx = (int64_t)k * N + col;
        int32_t packed = (int8_t)wInt4[idx / 2];
        float wVal = (idx % 2 == 0) ? (float)(packed & 0x0F) - 8.0f
                                    : (float)((packed >> 4) & 0x0F) - 8.0f;
        float scale = scalesW[col];
        float xVal = x[(int64_t)row * K + k];
        sum += (wVal * scale) * xVal;
      }
      y[(int64_t)row * N + col] = sum;
    }
  }
}

/* Group-wise form of the statements above: the nibble address rule of
 * QuantizedGemmOps.scala:234-238 (element k*N+n, low nibble first, i.e. nibble
 * (k*N+n)%8 of little-endian word (k*N+n)/8), the zero point generalised from
 * the constant 8, and the per-column scale indexed by group k/G. */
void oracle_w4a16_grouped(const uint32_t* wq, const uint16_t* scales,
                          int zero_point, int group_size,
                          const uint16_t* x, float* y_f32, uint16_t* y_bf16,
                          int M, int N, int K, int n0, int n1, int threads) {
  if (n0 < 0) n0 = 0;
  if (n1 > N) n1 = N;
  const float zp = (float)zero_point;
  (void)threads;
  for (int row = 0; row < M; ++row) {
#ifdef _OPENMP
    if (threads < 1) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
#endif
    for (int cb = n0; cb < n1; cb += 256) {
      int ce = cb + 256 < n1 ? cb + 256 : n1;
      float sum[256];
      for (int c = 0; c < ce - cb; ++c) sum[c] = 0.0f;
      for (int k = 0; k < K; ++k) {
        float xVal = oracle_bf16_to_f32(x[(int64_t)row * K + k]);
        const uint16_t* srow = scales + (int64_t)(k / group_size) * N;
        for (int col = cb; col < ce; ++col) {
          int64_t idx = (int64_t)k * N + col;
          uint32_t q = (wq[idx >> 3] >> (4 * (idx & 7))) & 0xFu;
          float wVal = (float)q - zp;
          float scale = oracle_bf16_to_f32(srow[col]);
          sum[col - cb] += (wVal * scale) * xVal;
        }
      }
      for (int col = cb; col < ce; ++col) {
        if (y_f32) y_f32[(int64_t)row * N + col] = sum[col - cb];
        if (y_bf16) y_bf16[(int64_t)row * N + col] = oracle_f32_to_bf16_rne(sum[col - cb]);
      }
    }
  }
}

/* QuantizedGemmOps.scala:37-53:
 *   for k: sum += wInt8(k*N+col).toFloat * scalesW(col) * x(row*K+k)
 *   if (hasBias) sum += bias(col) */
void oracle_w8a16_gemm(const int8_t* wInt8, const float* scalesW,
                       const float* x, const float* bias, float* y,
                       int M, int N, int K, int hasBias) {
  for (int row = 0; row < M; ++row) {
    for (int col = 0; col < N; ++col) {
      float sum = 0.0f;
      for (int k = 0; k < K; ++k) {
        float wVal = (float)wInt8[(int64_t)k * N + col];
        float scale = scalesW[col];
        float xVal = x[(int64_t)row * K + k];
        sum += (wVal * scale) * xVal;
      }
      if (hasBias) sum += bias[col];
      y[(int64_t)row * N + col] = sum;
    }
  }
}

/* QuantizedGemmOps.scala:72-82: as above with scalesW(k) (per-row of K). */
void oracle_w8a16_gemm_rowwise(const int8_t* wInt8, const float* scalesW,
                               const float* x, float* y, int M, int N, int K) {
  for (int row = 0; row < M; ++row) {
    for (int col = 0; col < N; ++col) {
      float sum = 0.0f;
      for (int k = 0; k < K; ++k) {
        float wVal = (float)wInt8[(int64_t)k * N + col];
        float scale = scalesW[k];
        float xVal = x[(int64_t)row * K + k];
        sum += (wVal * scale) * xVal;
      }
      y[(int64_t)row * N + col] = sum;
    }
  }
}

/* QuantizedGemmOps.scala:131-155.  Note the truncating .toInt (:147), the
 * stored scale maxAbs/qMax (:142) versus the applied qMax/maxAbs (:141), and
 * that NaN magnitudes never win the `v > maxAbs` test (:136). */
void oracle_dynamic_quantize(const float* weight, float* scales,
                             int8_t* qWeight, int K, int N, int qBits) {
  for (int col = 0; col < N; ++col) {
    float maxAbs = 0.0f;
    for (int k = 0; k < K; ++k) {
      float v = fabsf(weight[(int64_t)k * N + col]);
      if (v > maxAbs) maxAbs = v;
    }
    float qMax = (qBits == 8) ? 127.0f : 7.0f;
    float scale = (maxAbs > 1e-6f) ? qMax / maxAbs : 1.0f;
    scales[col] = maxAbs / qMax;
    for (int k = 0; k < K; ++k) {
      float fVal = weight[(int64_t)k * N + col];
      int32_t qVal = oracle_scala_f2i(fVal * scale);
      int32_t clamped;
      if (qBits == 8) clamped = qVal > 127 ? 127 : (qVal < -128 ? -128 : qVal);
      else            clamped = qVal > 7 ? 7 : (qVal < -8 ? -8 : qVal);
      qWeight[(int64_t)k * N + col] = (int8_t)clamped;
    }
  }
}

/* QuantizedGemmOps.scala:173-190. */
void oracle_weight_only_quantize_per_channel(const float* weight, float* scales,
                                             int8_t* qWeight, int8_t* zeros,
                                             int K, int N) {
  for (int col = 0; col < N; ++col) {
    float maxVal = 0.0f;
    for (int k = 0; k < K; ++k) {
      float v = fabsf(weight[(int64_t)k * N + col]);
      if (v > maxVal) maxVal = v;
    }
    float scale = (maxVal > 1e-6f) ? 127.0f / maxVal : 1.0f;
    scales[col] = maxVal / 127.0f;
    zeros[col] = 0;
    for (int k = 0; k < K; ++k) {
      float fVal = weight[(int64_t)k * N + col];
      int32_t qVal = oracle_scala_f2i(fVal * scale);
      int32_t clamped = qVal > 127 ? 127 : (qVal < -128 ? -128 : qVal);
      qWeight[(int64_t)k * N + col] = (int8_t)clamped;
    }
  }
}

/* QuantizedGemmOps.scala:207-211: weight(i) = qWeight(i).toFloat * scales(i % N). */
void oracle_dequantize(const int8_t* qWeight, const float* scales,
                       float* weight, int K, int N) {
  int64_t total = (int64_t)K * N;
  for (int64_t i = 0; i < total; ++i) {
    int col = (int)(i % N);
    weight[i] = (float)qWeight[i] * scales[col];
  }
}

/* ---- fp32 operators of the same facade (operators/linalg/MatrixOps.scala) ----
 *
 * MatrixOps.matmul :16-28, matmulAddBias :31-44, BLASOps.sgemm :230-243:
 *   var sum = 0.0f
 *   for (k <- 0 until K) sum += A(row*K + k) * B(k*N + col)
 *   matmul:        C(row*N + col) = sum
 *   matmulAddBias: C(row*N + col) = sum + bias(col)
 *   sgemm:         C(row*N + col) = alpha*sum + beta*C(row*N + col)
 * mode 0 / 1 / 2 selects the epilogue.  Each product and sum is rounded on its own
 * (JVM float semantics), k ascending per element; the loops run k outside the
 * columns so that B is read row by row, which keeps every element's order. */
void oracle_matmul_f32(const float* A, const float* B, const float* bias, float* C,
                       int M, int N, int K, float alpha, float beta, int mode,
                       int threads) {
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
  for (int row = 0; row < M; ++row) {
    float* sum = (float*)malloc(sizeof(float) * (N > 0 ? N : 1));
    for (int col = 0; col < N; ++col) sum[col] = 0.0f;
    for (int k = 0; k < K; ++k) {
      const float a = A[(int64_t)row * K + k];
      const float* b = B + (int64_t)k * N;
      for (int col = 0; col < N; ++col) sum[col] += a * b[col];
    }
    float* c = C + (int64_t)row * N;
    for (int col = 0; col < N; ++col) {
      if (mode == 1) c[col] = sum[col] + bias[col];
      else if (mode == 2) c[col] = alpha * sum[col] + beta * c[col];
      else c[col] = sum[col];
    }
    free(sum);
  }
  (void)threads;
}

/* MatrixOps.gemv :166-177:
 *   var sum = 0.0f
 *   for (j <- 0 until N) sum += A(i*N + j) * x(j)
 *   y(i) = sum */
void oracle_gemv_f32(const float* A, const float* x, float* y, int M, int N) {
  for (int i = 0; i < M; ++i) {
    float sum = 0.0f;
    for (int j = 0; j < N; ++j) sum += A[(int64_t)i * N + j] * x[j];
    y[i] = sum;
  }
}

/* ---- the int8 GEMM names of TensorCoreOps and CutlassGemm ----
 *
 * TensorCoreOps.tensorCoreGemmInt8 (operators/intrinsic/TensorCoreOps.scala:294-340):
 *   acc32 = sum over k of aVal * bVal   (Int, wraps modulo 2^32)
 *   d(mStart*ldd + nStart) = acc32 + (if (hasC) c(mStart*ldc + nStart) else 0)
 * restated as that arithmetic for every output (m, n) and every k, operands read
 * through their leading dimensions: d[m*ldd+n] = sum_k a[m*lda+k]*b[k*ldb+n] + c.
 * The body's own index arithmetic is not restated: it subtracts 128 from each
 * signed byte, visits every 16th k only and writes one element per 16 x 16 block,
 * which no caller can want.  scalesA / scalesB are parameters the body never reads;
 * they are not parameters here either. */
void oracle_tensor_core_gemm_int8(const int8_t* a, const int8_t* b, const int32_t* c,
                                  int32_t* d, int M, int N, int K, int lda, int ldb,
                                  int ldc, int ldd, int hasC) {
  for (int m = 0; m < M; ++m) {
    for (int n = 0; n < N; ++n) {
      uint32_t acc32 = 0;
      for (int k = 0; k < K; ++k)
        acc32 += (uint32_t)((int32_t)a[(int64_t)m * lda + k] * (int32_t)b[(int64_t)k * ldb + n]);
      if (hasC) acc32 += (uint32_t)c[(int64_t)m * ldc + n];
      d[(int64_t)m * ldd + n] = (int32_t)acc32;
    }
  }
}

/* CutlassGemm.int8GemmKernel (cutlass/CutlassGemm.scala:987-1041):
 *   var acc: Float = 0.0f
 *   for kk: acc = acc + tl.load(A, aRow*lda + kk).toFloat * tl.load(B, kk*ldb + bCol).toFloat
 *   tl.store(D, aRow*ldd + bCol, acc * scaleA * scaleB)
 * restated with one accumulator per output element, k ascending, each product and
 * sum rounded on its own (JVM float), then (acc * scaleA) * scaleB.  The body keeps
 * one accumulator for all 64 outputs of a thread, so every one of them would get the
 * same sum; that sharing is not restated. A and B are Int (32-bit) arrays. */
void oracle_int8_gemm_kernel(float* D, const int32_t* A, const int32_t* B, int M, int N, int K,
                             int lda, int ldb, int ldd, float scaleA, float scaleB,
                             int threads) {
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
  for (int m = 0; m < M; ++m) {
    float* acc = (float*)malloc(sizeof(float) * (N > 0 ? N : 1));
    for (int n = 0; n < N; ++n) acc[n] = 0.0f;
    for (int k = 0; k < K; ++k) {
      const float av = (float)A[(int64_t)m * lda + k];
      const int32_t* br = B + (int64_t)k * ldb;
      for (int n = 0; n < N; ++n) acc[n] = acc[n] + av * (float)br[n];
    }
    for (int n = 0; n < N; ++n) D[(int64_t)m * ldd + n] = acc[n] * scaleA * scaleB;
    free(acc);
  }
  (void)threads;
}
