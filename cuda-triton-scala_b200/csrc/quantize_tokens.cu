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
// Rows of up to 256 vectors of 16 bytes (bf16: K <= 2048, fp32: K <= 1024) with
// 16-byte aligned rows: one warp per row (quantize_rows_warp_kernel).  Each lane issues
// all its 16-byte loads at once (a whole 8 KB row in flight per warp), the maximum is a
// warp shuffle reduction (no block barrier), and the row is quantised from registers.
// Measured on B200 (same process, inputs larger than L2): 8192 x 2048 bf16 11.8 us
// against 13.0 us for a CTA per row; at K = 4096 the two are within 3 % and a warp
// would need 16 vectors a lane (registers for two CTAs an SM only), so longer rows of
// up to 256 x 4 vectors take one CTA per row, the same in registers with a block-wide
// maximum (quantize_rows_vec_kernel).  Other rows take two passes: maxAbs,
// then the int8 row, the second pass served from L2 (quantize_rows_kernel).
// HBM-bound: one read of x, one write of q.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "internal.h"
#include "ptx.cuh"

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

// Block-wide maxAbs of per-thread maxima, in the "if (v > m) m = v" form (NaN never
// replaces a number); thread 0 also writes sA[m].  Returns 127 / maxAbs (or 1).
__device__ __forceinline__ float block_mul(float mx, float* sA, int m) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, mx, off);
    if (o > mx) mx = o;
  }
  __shared__ float wmax[THREADS / 32];
  __shared__ float bcast;
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = wmax[0];
    for (int w = 1; w < THREADS / 32; ++w)
      if (wmax[w] > v) v = wmax[w];
    bcast = (v > 1e-6f) ? __fdiv_rn(127.0f, v) : 1.0f;
    sA[m] = __fdiv_rn(v, 127.0f);
  }
  __syncthreads();
  return bcast;
}

// 16-byte vectors of T: 8 bf16 or 4 fp32.
template <typename T> struct Vec;
template <> struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <> struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&v)[4]) {
    const float4 u = __ldcs(reinterpret_cast<const float4*>(p));
    v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
  }
};

// One row per CTA, NV vectors per thread held in registers; K % VEC == 0 and 16-byte
// aligned rows of x, (VEC)-byte aligned rows of q.
template <typename T, int NV>
__global__ void __launch_bounds__(THREADS) quantize_rows_vec_kernel(const T* __restrict__ x,
                                                                    int8_t* __restrict__ q,
                                                                    float* __restrict__ sA,
                                                                    int M, int K) {
  constexpr int VEC = Vec<T>::N;
  // The GEMM that consumes q and sA may begin its set-up; it reads them only after
  // griddepcontrol.wait, i.e. after this grid has finished.
  ptx::grid_launch_dependents();
  const int m = blockIdx.x;
  if (m >= M) return;
  const T* row = x + (size_t)m * K;
  const int nvec = K / VEC;
  float v[NV][VEC];
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int vi = threadIdx.x + j * THREADS;
    if (vi < nvec) {
      Vec<T>::load(row + (size_t)vi * VEC, v[j]);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const float a = fabsf(v[j][i]);
        if (a > mx) mx = a;
      }
    }
  }
  const float mul = block_mul(mx, sA, m);
  int8_t* qrow = q + (size_t)m * K;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int vi = threadIdx.x + j * THREADS;
    if (vi < nvec) {
      uint32_t packed[VEC / 4];
#pragma unroll
      for (int w = 0; w < VEC / 4; ++w) {
        uint32_t b = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          b |= (uint32_t)(uint8_t)quant(v[j][4 * w + i], mul) << (8 * i);
        packed[w] = b;
      }
      if constexpr (VEC == 8)
        *reinterpret_cast<uint2*>(qrow + (size_t)vi * VEC) = make_uint2(packed[0], packed[1]);
      else
        *reinterpret_cast<uint32_t*>(qrow + (size_t)vi * VEC) = packed[0];
    }
  }
}

// One row per warp, 8 warps per CTA; NVW vectors of 16 bytes per lane kept as loaded
// (raw bits) and widened twice, once for the maximum and once to quantise.
template <typename T, int NVW>
__global__ void __launch_bounds__(256, 3) quantize_rows_warp_kernel(const T* __restrict__ x,
                                                                 int8_t* __restrict__ q,
                                                                 float* __restrict__ sA, int M,
                                                                 int K) {
  constexpr int VEC = Vec<T>::N;
  // The GEMM that consumes q and sA may begin its set-up; it reads them only after
  // griddepcontrol.wait, i.e. after this grid has finished.
  ptx::grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int m = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (m >= M) return;
  const T* row = x + (size_t)m * K;
  const int nvec = K / VEC;
  uint4 raw[NVW];
#pragma unroll
  for (int j = 0; j < NVW; ++j) {
    const int vi = lane + 32 * j;
    raw[j] = vi < nvec ? __ldcs(reinterpret_cast<const uint4*>(row) + vi)
                       : make_uint4(0u, 0u, 0u, 0u);
  }
  auto widen = [](const uint4& u, float (&v)[VEC]) {
    if constexpr (VEC == 8) {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    } else {
      v[0] = __uint_as_float(u.x); v[1] = __uint_as_float(u.y);
      v[2] = __uint_as_float(u.z); v[3] = __uint_as_float(u.w);
    }
  };
  // maxAbs in the "if (v > m) m = v" form (NaN never replaces a number); lanes past the
  // row hold zeros, which never exceed a maximum that starts at zero
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < NVW; ++j) {
    float v[VEC];
    widen(raw[j], v);
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const float a = fabsf(v[i]);
      if (a > mx) mx = a;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, mx, off);
    if (o > mx) mx = o;
  }
  const float mul = (mx > 1e-6f) ? __fdiv_rn(127.0f, mx) : 1.0f;
  if (lane == 0) sA[m] = __fdiv_rn(mx, 127.0f);
  int8_t* qrow = q + (size_t)m * K;
#pragma unroll
  for (int j = 0; j < NVW; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) {
      float v[VEC];
      widen(raw[j], v);
      uint32_t packed[VEC / 4];
#pragma unroll
      for (int w = 0; w < VEC / 4; ++w) {
        uint32_t b = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          b |= (uint32_t)(uint8_t)quant(v[4 * w + i], mul) << (8 * i);
        packed[w] = b;
      }
      if constexpr (VEC == 8)
        *reinterpret_cast<uint2*>(qrow + (size_t)vi * VEC) = make_uint2(packed[0], packed[1]);
      else
        *reinterpret_cast<uint32_t*>(qrow + (size_t)vi * VEC) = packed[0];
    }
  }
}

}  // namespace qtok

qgemm_status launch_quantize_tokens(qgemm_stream_s* s, const void* x, int in_dtype, int8_t* q,
                                    float* sA, int M, int K) {
  using namespace qtok;
  const bool bf = in_dtype == QGEMM_BF16;
  const int VEC = bf ? 8 : 4;
  const int nv = (K / VEC + THREADS - 1) / THREADS;  // vectors per thread
  const bool vec = K > 0 && K % VEC == 0 && nv <= 4 && aligned((uint64_t)x, 16) &&
                   ((uint64_t)K * (bf ? 2 : 4)) % 16 == 0 && aligned((uint64_t)q, VEC) &&
                   K % VEC == 0;
  const int nvec = VEC > 0 ? K / VEC : 0;
  if (vec && nvec <= 8 * 32) {
    // a warp per row: 4 or 8 vectors per lane
    const unsigned grid = (unsigned)((M + 7) / 8);
    if (bf) {
      const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
      if (nvec <= 4 * 32) quantize_rows_warp_kernel<__nv_bfloat16, 4><<<grid, 256, 0, s->stream>>>(xb, q, sA, M, K);
      else quantize_rows_warp_kernel<__nv_bfloat16, 8><<<grid, 256, 0, s->stream>>>(xb, q, sA, M, K);
    } else {
      const float* xf = static_cast<const float*>(x);
      if (nvec <= 4 * 32) quantize_rows_warp_kernel<float, 4><<<grid, 256, 0, s->stream>>>(xf, q, sA, M, K);
      else quantize_rows_warp_kernel<float, 8><<<grid, 256, 0, s->stream>>>(xf, q, sA, M, K);
    }
    return cuda_fail(cudaGetLastError(), "quantize_rows_warp launch");
  }
  if (vec) {
    if (bf) {
      const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
      switch (nv) {
        case 1: quantize_rows_vec_kernel<__nv_bfloat16, 1><<<M, THREADS, 0, s->stream>>>(xb, q, sA, M, K); break;
        case 2: quantize_rows_vec_kernel<__nv_bfloat16, 2><<<M, THREADS, 0, s->stream>>>(xb, q, sA, M, K); break;
        default: quantize_rows_vec_kernel<__nv_bfloat16, 4><<<M, THREADS, 0, s->stream>>>(xb, q, sA, M, K); break;
      }
    } else {
      const float* xf = static_cast<const float*>(x);
      switch (nv) {
        case 1: quantize_rows_vec_kernel<float, 1><<<M, THREADS, 0, s->stream>>>(xf, q, sA, M, K); break;
        case 2: quantize_rows_vec_kernel<float, 2><<<M, THREADS, 0, s->stream>>>(xf, q, sA, M, K); break;
        default: quantize_rows_vec_kernel<float, 4><<<M, THREADS, 0, s->stream>>>(xf, q, sA, M, K); break;
      }
    }
    return cuda_fail(cudaGetLastError(), "quantize_rows_vec launch");
  }
  if (in_dtype == QGEMM_BF16)
    quantize_rows_kernel<__nv_bfloat16><<<M, THREADS, 0, s->stream>>>(
        static_cast<const __nv_bfloat16*>(x), q, sA, M, K);
  else
    quantize_rows_kernel<float><<<M, THREADS, 0, s->stream>>>(static_cast<const float*>(x), q,
                                                              sA, M, K);
  return cuda_fail(cudaGetLastError(), "quantize_rows launch");
}

}  // namespace qg
