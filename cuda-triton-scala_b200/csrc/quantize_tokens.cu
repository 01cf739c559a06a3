// quantize_tokens.cu -- dynamic per-token int8 quantisation of activations, the step
// that produces the A operand and the per-token scales sA of the W8A8 GEMM.
//
// The arithmetic is that of QuantizedGemmOps.dynamicQuantize
// (src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala:121-157) applied to
// each row of x instead of each column of a weight:
//     maxAbs = max_k |x[m,k]|            (comparisons in order; NaN never wins)
//     mul    = maxAbs > 1e-6 ? 127 / maxAbs : 1
//     sA[m]  = maxAbs / 127
//     q[m,k] = clamp(trunc(x[m,k] * mul), -128, 127)   (Scala Float.toInt: NaN -> 0)
// with IEEE fp32 division and multiplication (no fused or approximate forms), so the
// result is bit-identical to the reference arithmetic.  x is fp32 or bf16 (widened).
//
// One CTA per row: a first pass over the row finds maxAbs (block reduction), a second
// pass (served from L2) writes the int8 row.  HBM-bound: one read of x, one write of q.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "internal.h"

namespace qg {
namespace qtok {

constexpr int THREADS = 256;

template <typename T>
__device__ __forceinline__ float load_f(const T* p, size_t i);
template <>
__device__ __forceinline__ float load_f<float>(const float* p, size_t i) { return __ldg(p + i); }
template <>
__device__ __forceinline__ float load_f<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) {
  return __bfloat162float(p[i]);
}

__device__ __forceinline__ int8_t quant(float v, float mul) {
  const int qv = __float2int_rz(__fmul_rn(v, mul));
  return (int8_t)(qv > 127 ? 127 : (qv < -128 ? -128 : qv));
}

template <typename T>
__global__ void __launch_bounds__(THREADS) quantize_rows_kernel(const T* __restrict__ x,
                                                                int8_t* __restrict__ q,
                                                                float* __restrict__ sA, int M,
                                                                int K) {
  const int m = blockIdx.x;
  if (m >= M) return;
  const T* row = x + (size_t)m * K;
  // pass 1: maxAbs.  Each thread keeps the larger of its values in the reference's
  // "if (v > maxAbs) maxAbs = v" form, so a NaN never replaces a number.
  float mx = 0.0f;
  for (int k = threadIdx.x; k < K; k += THREADS) {
    const float v = fabsf(load_f(row, k));
    if (v > mx) mx = v;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, mx, off);
    if (o > mx) mx = o;
  }
  __shared__ float wmax[THREADS / 32];
  __shared__ float bcast[2];
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = wmax[0];
    for (int w = 1; w < THREADS / 32; ++w)
      if (wmax[w] > v) v = wmax[w];
    const float mul = (v > 1e-6f) ? __fdiv_rn(127.0f, v) : 1.0f;
    bcast[0] = mul;
    sA[m] = __fdiv_rn(v, 127.0f);
  }
  __syncthreads();
  const float mul = bcast[0];
  // pass 2: quantise, four elements per store where the row allows it
  int8_t* qrow = q + (size_t)m * K;
  const bool vec = ((reinterpret_cast<uintptr_t>(qrow) & 3) == 0) && (K % 4 == 0);
  if (vec) {
    for (int k = 4 * threadIdx.x; k < K; k += 4 * THREADS) {
      char4 c;
      c.x = quant(load_f(row, k), mul);
      c.y = quant(load_f(row, k + 1), mul);
      c.z = quant(load_f(row, k + 2), mul);
      c.w = quant(load_f(row, k + 3), mul);
      *reinterpret_cast<char4*>(qrow + k) = c;
    }
  } else {
    for (int k = threadIdx.x; k < K; k += THREADS) qrow[k] = quant(load_f(row, k), mul);
  }
}

}  // namespace qtok

qgemm_status launch_quantize_tokens(qgemm_stream_s* s, const void* x, int in_dtype, int8_t* q,
                                    float* sA, int M, int K) {
  using namespace qtok;
  if (in_dtype == QGEMM_BF16)
    quantize_rows_kernel<__nv_bfloat16><<<M, THREADS, 0, s->stream>>>(
        static_cast<const __nv_bfloat16*>(x), q, sA, M, K);
  else
    quantize_rows_kernel<float><<<M, THREADS, 0, s->stream>>>(static_cast<const float*>(x), q,
                                                              sA, M, K);
  return cuda_fail(cudaGetLastError(), "quantize_rows launch");
}

}  // namespace qg
