// simt_kernels.cu -- CUDA-core kernels for the reference operators whose
// arithmetic order must be kept exactly, plus layout utilities.
//
//  * w8a8_simt: any-shape W8A8 (both B layouts); the integer sum is exact so the
//    result is bit-identical to the tensor-core path -- it is the independent
//    device-side check for shapes too large for the CPU oracle.
//  * w4a16_ref / w8a16_ref: one thread per output, fp32 sum in ascending k with
//    separately rounded products (__fmul_rn/__fadd_rn), i.e. exactly the
//    per-element loops of QuantizedGemmOps.scala:41-46, :75-80 and :232-243.
//  * quantize / dequantize: QuantizedGemmOps.scala:121-212.
//  * prepack [K,N] -> [N,K] and the [world][M][ncols] -> [M][N] unshard.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "internal.h"

namespace qg {

// ---- W8A8 (any shape) --------------------------------------------------------
namespace simt {
constexpr int TM = 64, TN = 64, TK = 32;

__global__ void __launch_bounds__(256)
    w8a8_simt_kernel(const int8_t* __restrict__ A, const int8_t* __restrict__ B, int b_kn,
                     const float* __restrict__ sA, const float* __restrict__ sB, void* out,
                     int out_dtype, int ldc, int M, int N, int K, int32_t* acc_out) {
  __shared__ int32_t As[TK][TM + 1];
  __shared__ int32_t Bs[TK][TN + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  int32_t acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < TM * TK; i += 256) {
      const int mm = i / TK, kk = i % TK;
      const int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? (int32_t)A[(size_t)m * K + k] : 0;
    }
    for (int i = threadIdx.x; i < TN * TK; i += 256) {
      int nn, kk;
      if (b_kn) { kk = i / TN; nn = i % TN; } else { nn = i / TK; kk = i % TK; }
      const int n = n0 + nn, k = k0 + kk;
      int32_t v = 0;
      if (n < N && k < K) v = b_kn ? (int32_t)B[(size_t)k * N + n] : (int32_t)B[(size_t)n * K + k];
      Bs[kk][nn] = v;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < TK; ++kk) {
      int32_t a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
    const float sa = sA[m];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= N) continue;
      if (acc_out) acc_out[(size_t)m * N + n] = acc[i][j];
      const float v = __fmul_rn(__fmul_rn(__int2float_rn(acc[i][j]), sB[n]), sa);
      if (out_dtype == QGEMM_BF16)
        reinterpret_cast<__nv_bfloat16*>(out)[(size_t)m * ldc + n] = __float2bfloat16_rn(v);
      else
        reinterpret_cast<float*>(out)[(size_t)m * ldc + n] = v;
    }
  }
}
}  // namespace simt

qgemm_status launch_w8a8_simt(qgemm_stream_s* s, const int8_t* A, const int8_t* B, int b_kn,
                              const float* sA, const float* sB, void* out, int out_dtype,
                              int ldc, int M, int N, int K, int32_t* acc) {
  dim3 grid((N + simt::TN - 1) / simt::TN, (M + simt::TM - 1) / simt::TM);
  if (grid.y > 65535) return fail(QGEMM_ERR_INVALID_ARG, "M too large for the SIMT path");
  simt::w8a8_simt_kernel<<<grid, 256, 0, s->stream>>>(A, B, b_kn, sA, sB, out, out_dtype, ldc,
                                                       M, N, K, acc);
  return cuda_fail(cudaGetLastError(), "w8a8_simt_kernel launch");
}

// ---- W4A16, reference layout and order (QuantizedGemmOps.scala:229-245) ----
__global__ void w4a16_ref_kernel(const uint8_t* __restrict__ w, const float* __restrict__ sw,
                                 const float* __restrict__ x, float* __restrict__ y, int M,
                                 int N, int K) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = blockIdx.y;
  if (row >= M || col >= N) return;
  const float scale = sw[col];
  float sum = 0.0f;
  for (int k = 0; k < K; ++k) {
    const size_t idx = (size_t)k * N + col;
    const int packed = (int)(int8_t)w[idx >> 1];
    const float wVal = (idx & 1) == 0 ? __fsub_rn((float)(packed & 0x0F), 8.0f)
                                      : __fsub_rn((float)((packed >> 4) & 0x0F), 8.0f);
    const float xVal = x[(size_t)row * K + k];
    sum = __fadd_rn(sum, __fmul_rn(__fmul_rn(wVal, scale), xVal));
  }
  y[(size_t)row * N + col] = sum;
}

qgemm_status launch_w4a16_ref(qgemm_stream_s* s, const uint8_t* w, const float* sw,
                              const float* x, float* y, int M, int N, int K) {
  if (M > 65535) return fail(QGEMM_ERR_INVALID_ARG, "M too large");
  dim3 grid((N + 127) / 128, M);
  w4a16_ref_kernel<<<grid, 128, 0, s->stream>>>(w, sw, x, y, M, N, K);
  return cuda_fail(cudaGetLastError(), "w4a16_ref_kernel launch");
}

// ---- W8A16 (QuantizedGemmOps.scala:37-53 and :72-82) ----
__global__ void w8a16_ref_kernel(const int8_t* __restrict__ w, const float* __restrict__ sw,
                                 const float* __restrict__ x, const float* __restrict__ bias,
                                 float* __restrict__ y, int M, int N, int K, int hasBias,
                                 int rowwise) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = blockIdx.y;
  if (row >= M || col >= N) return;
  float sum = 0.0f;
  for (int k = 0; k < K; ++k) {
    const float wVal = (float)w[(size_t)k * N + col];
    const float scale = rowwise ? sw[k] : sw[col];
    const float xVal = x[(size_t)row * K + k];
    sum = __fadd_rn(sum, __fmul_rn(__fmul_rn(wVal, scale), xVal));
  }
  if (!rowwise && hasBias) sum = __fadd_rn(sum, bias[col]);
  y[(size_t)row * N + col] = sum;
}

qgemm_status launch_w8a16_ref(qgemm_stream_s* s, const int8_t* w, const float* sw,
                              const float* x, const float* bias, float* y, int M, int N,
                              int K, int hasBias, int rowwise) {
  if (M > 65535) return fail(QGEMM_ERR_INVALID_ARG, "M too large");
  dim3 grid((N + 127) / 128, M);
  w8a16_ref_kernel<<<grid, 128, 0, s->stream>>>(w, sw, x, bias, y, M, N, K, hasBias, rowwise);
  return cuda_fail(cudaGetLastError(), "w8a16_ref_kernel launch");
}

// ---- quantize (QuantizedGemmOps.scala:131-155 and :173-190) ----
// One thread per column, as the reference's programId(0) = col.  Float.toInt is
// cvt.rzi.s32.f32 (truncates, saturates, NaN -> 0), i.e. __float2int_rz.
__global__ void quantize_kernel(const float* __restrict__ w, float* __restrict__ scales,
                                int8_t* __restrict__ q, int8_t* __restrict__ zeros, int K,
                                int N, int qBits) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= N) return;
  float maxAbs = 0.0f;
  for (int k = 0; k < K; ++k) {
    const float v = fabsf(w[(size_t)k * N + col]);
    if (v > maxAbs) maxAbs = v;
  }
  const float qMax = (qBits == 8) ? 127.0f : 7.0f;
  const float scale = (maxAbs > 1e-6f) ? __fdiv_rn(qMax, maxAbs) : 1.0f;
  scales[col] = __fdiv_rn(maxAbs, qMax);
  if (zeros) zeros[col] = 0;
  const int hi = (qBits == 8) ? 127 : 7, lo = (qBits == 8) ? -128 : -8;
  for (int k = 0; k < K; ++k) {
    const int qVal = __float2int_rz(__fmul_rn(w[(size_t)k * N + col], scale));
    const int c = qVal > hi ? hi : (qVal < lo ? lo : qVal);
    q[(size_t)k * N + col] = (int8_t)c;
  }
}

qgemm_status launch_quantize(qgemm_stream_s* s, const float* w, float* scales, int8_t* q,
                             int8_t* zeros, int K, int N, int qBits) {
  quantize_kernel<<<(N + 127) / 128, 128, 0, s->stream>>>(w, scales, q, zeros, K, N, qBits);
  return cuda_fail(cudaGetLastError(), "quantize_kernel launch");
}

// ---- dequantize (QuantizedGemmOps.scala:207-211) ----
__global__ void dequantize_kernel(const int8_t* __restrict__ q, const float* __restrict__ scales,
                                  float* __restrict__ w, size_t total, int N) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x)
    w[i] = __fmul_rn((float)q[i], scales[i % N]);
}

qgemm_status launch_dequantize(qgemm_stream_s* s, const int8_t* q, const float* scales,
                               float* w, int K, int N) {
  const size_t total = (size_t)K * N;
  const int grid = (int)((total + 255) / 256 < 65536 ? (total + 255) / 256 : 65536);
  dequantize_kernel<<<grid, 256, 0, s->stream>>>(q, scales, w, total, N);
  return cuda_fail(cudaGetLastError(), "dequantize_kernel launch");
}

// ---- prepack int8 [K,N] -> [N,K] ----
__global__ void transpose_i8_kernel(const int8_t* __restrict__ src, int8_t* __restrict__ dst,
                                    int K, int N) {
  __shared__ int8_t tile[64][65];
  const int n0 = blockIdx.x * 64, k0 = blockIdx.y * 64;
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int kk = i / 64, nn = i % 64;
    const int k = k0 + kk, n = n0 + nn;
    tile[kk][nn] = (k < K && n < N) ? src[(size_t)k * N + n] : 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int nn = i / 64, kk = i % 64;
    const int k = k0 + kk, n = n0 + nn;
    if (k < K && n < N) dst[(size_t)n * K + k] = tile[kk][nn];
  }
}

qgemm_status launch_prepack_w8_nk(qgemm_stream_s* s, const int8_t* src, int8_t* dst, int K,
                                  int N) {
  dim3 grid((N + 63) / 64, (K + 63) / 64);
  if (grid.y > 65535) return fail(QGEMM_ERR_INVALID_ARG, "K too large");
  transpose_i8_kernel<<<grid, 256, 0, s->stream>>>(src, dst, K, N);
  return cuda_fail(cudaGetLastError(), "transpose_i8_kernel launch");
}

// ---- [world][M][ncols] -> [M][world*ncols] (bf16) ----
__global__ void unshard_bf16_kernel(const uint16_t* __restrict__ g, uint16_t* __restrict__ out,
                                    int world, int M, int ncols) {
  const size_t total = (size_t)world * M * ncols;
  const int N = world * ncols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / ((size_t)M * ncols);
    const size_t rem = i - r * (size_t)M * ncols;
    const size_t m = rem / ncols, c = rem % ncols;
    out[m * N + r * ncols + c] = g[i];
  }
}

__global__ void unshard_bf16_vec_kernel(const uint4* __restrict__ g, uint4* __restrict__ out,
                                        int world, int M, int ncols8) {
  const size_t total = (size_t)world * M * ncols8;
  const size_t N8 = (size_t)world * ncols8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / ((size_t)M * ncols8);
    const size_t rem = i - r * (size_t)M * ncols8;
    const size_t m = rem / ncols8, c = rem % ncols8;
    out[m * N8 + r * ncols8 + c] = g[i];
  }
}

qgemm_status launch_unshard_bf16(qgemm_stream_s* s, const uint16_t* g, uint16_t* out,
                                 int world, int M, int ncols) {
  const int grid = s->dev->sm_count * 8;
  if (ncols % 8 == 0 && aligned((uint64_t)g, 16) && aligned((uint64_t)out, 16))
    unshard_bf16_vec_kernel<<<grid, 256, 0, s->stream>>>(reinterpret_cast<const uint4*>(g),
                                                         reinterpret_cast<uint4*>(out), world,
                                                         M, ncols / 8);
  else
    unshard_bf16_kernel<<<grid, 256, 0, s->stream>>>(g, out, world, M, ncols);
  return cuda_fail(cudaGetLastError(), "unshard_bf16 launch");
}

}  // namespace qg
