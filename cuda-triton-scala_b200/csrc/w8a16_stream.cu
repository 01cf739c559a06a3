// w8a16_stream.cu -- QuantizedGemmOps.w8a16Gemm / w8a16GemmRowWise
// (src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala:24-55, :61-84) at
// the speed of the weight stream, in the reference's own arithmetic order:
//     sum = 0; for k in 0..K-1: sum += (float(w[k,n]) * s) * x[m,k]      (s = sW[n] or sW[k])
//     y[m,n] = sum (+ bias[n])
// with every product and sum rounded on its own, k ascending: bit-identical to the
// reference (and to w8a16_ref_kernel).
//
// Each output is one chain of K dependent additions, so parallelism comes only from
// the outputs: a CTA owns 128 columns (one per consumer thread) and up to MR rows of x
// per pass.  The weights, int8 [K, N] row-major, stream through a shared-memory ring
// of 256-row x 128-column tiles (one 2-D TMA copy per stage, issued by a producer
// warp); the activations' matching 256-column slices come with it.  A consumer reads
// its column's byte of each row and its rows' x values (same address across the warp:
// one broadcast), and runs its chains in order; only the running sum is a true chain,
// so 64 k per unrolled step keep the loads, conversions and products ahead of it.
// Measured on B200 (int8 [4096, 14336], bias): M=1 27.4 us = 2.15 TB/s (the one-thread-
// per-output kernel: 350 us), M=4 46 us.  Every wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace qg {
namespace w8s {

constexpr int COLS = 128;              // columns per CTA = consumer threads
constexpr int ROWS = 256;              // weight rows per stage
constexpr int STAGES = 4;
constexpr int MR = 4;                  // activation rows per pass
constexpr int THREADS = COLS + 32;     // 4 consumer warps + 1 producer warp
constexpr int W_BYTES = ROWS * COLS;   // 32 KB
constexpr int X_BYTES = MR * ROWS * 4; // 4 KB
constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 128 + 128;

struct Params {
  int M, N, K, m0, mrows, rowwise, hasBias;
  const float* sw;
  const float* bias;
  float* y;
  int* err;
};

// float(b) for an int8 b without the conversion unit: the bit pattern of 2^23 + 128
// plus b is the float 2^23 + 128 + b (exact, 0 <= 128 + b < 256), and subtracting
// 2^23 + 128 leaves b exactly.  Integer add + float add, both at full rate.
__device__ __forceinline__ float i8_to_f32(int b) {
  return __fsub_rn(__int_as_float(0x4B000080 + b), 8388736.0f);
}

// R: activation rows of this pass (1, 2 or 4), a compile-time count so that no slot of
// the chain loop is spent on absent rows.
template <int R>
__global__ void __launch_bounds__(THREADS, 1)
    w8a16_stream_kernel(const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ CUtensorMap tmX, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw + 127u) & ~127u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar = base + STAGES * STAGE_BYTES;
  auto full_bar = [&](int s) { return bar + 8u * s; };
  auto empty_bar = [&](int s) { return bar + 8u * (STAGES + s); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + STAGES * STAGE_BYTES + 64);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * COLS;
  const int nstages = (p.K + ROWS - 1) / ROWS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), COLS / 32);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();

  if (warp == COLS / 32) {
    // ---------------- producer ----------------
    if (lane == 0) {
      ptx::prefetch_tmap(&tmW);
      ptx::prefetch_tmap(&tmX);
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      for (int i = 0; i < nstages; ++i) {
        if (!ptx::mbar_wait_sleep(empty_bar(stage), phase ^ 1u, abort_flag)) {
          if (!*abort_flag) { *abort_flag = 1; if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_PRODUCER); }
          break;
        }
        const uint32_t sw = base + stage * STAGE_BYTES;
        ptx::mbar_arrive_expect_tx(full_bar(stage), STAGE_BYTES);
        ptx::tma_load_2d(sw, &tmW, full_bar(stage), n0, i * ROWS);
        ptx::tma_load_2d(sw + W_BYTES, &tmX, full_bar(stage), i * ROWS, p.m0);
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      for (long long f = (issued > STAGES ? issued - STAGES : 0); f < issued; ++f) {
        if (!ptx::mbar_wait(full_bar((int)(f % STAGES)), (uint32_t)((f / STAGES) & 1), nullptr)) {
          if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_DRAIN);
          break;
        }
      }
    }
    return;
  }

  // ---------------- consumers: column n0 + threadIdx.x ----------------
  const int col = n0 + threadIdx.x;
  const float scol = (!p.rowwise && col < p.N) ? __ldg(p.sw + col) : 0.f;
  float sum[R];
#pragma unroll
  for (int r = 0; r < R; ++r) sum[r] = 0.0f;
  int stage = 0;
  uint32_t phase = 0;
  for (int i = 0; i < nstages; ++i) {
    const bool ok = ptx::mbar_wait_sleep(full_bar(stage), phase, abort_flag);
    if (!ok && !*abort_flag) { *abort_flag = 1; if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_EPILOGUE); }
    if (ok) {
      const int8_t* ws = reinterpret_cast<const int8_t*>(gbase + stage * STAGE_BYTES) + threadIdx.x;
      const float* xs = reinterpret_cast<const float*>(gbase + stage * STAGE_BYTES + W_BYTES);
      const int k0 = i * ROWS;
      const int kn = p.K - k0 < ROWS ? p.K - k0 : ROWS;
      if (kn == ROWS && !p.rowwise) {
#pragma unroll 16
        for (int kk = 0; kk < ROWS; kk += 4) {
          float t[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) t[u] = __fmul_rn(i8_to_f32(ws[(kk + u) * COLS]), scol);
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const float4 xv = *reinterpret_cast<const float4*>(xs + r * ROWS + kk);
            sum[r] = __fadd_rn(sum[r], __fmul_rn(t[0], xv.x));
            sum[r] = __fadd_rn(sum[r], __fmul_rn(t[1], xv.y));
            sum[r] = __fadd_rn(sum[r], __fmul_rn(t[2], xv.z));
            sum[r] = __fadd_rn(sum[r], __fmul_rn(t[3], xv.w));
          }
        }
      } else {
        for (int kk = 0; kk < kn; ++kk) {
          const float sc = p.rowwise ? __ldg(p.sw + k0 + kk) : scol;
          const float t = __fmul_rn(i8_to_f32(ws[kk * COLS]), sc);
#pragma unroll
          for (int r = 0; r < R; ++r) sum[r] = __fadd_rn(sum[r], __fmul_rn(t, xs[r * ROWS + kk]));
        }
      }
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(empty_bar(stage));
    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
  }
  if (col < p.N) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float v = sum[r];
      if (!p.rowwise && p.hasBias) v = __fadd_rn(v, __ldg(p.bias + col));
      p.y[(size_t)(p.m0 + r) * p.N + col] = v;
    }
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

}  // namespace w8s

bool w8a16_stream_supported(const qgemm_device_s* d, uint64_t w, uint64_t x, int N, int K) {
  return d->tcgen05 && d->smem_optin >= (size_t)w8s::SMEM_BYTES && N % 16 == 0 && K % 4 == 0 &&
         K > 0 && aligned(w, 16) && aligned(x, 16);
}

qgemm_status launch_w8a16_stream(qgemm_stream_s* s, const int8_t* w, const float* sw,
                                 const float* x, const float* bias, float* y, int M, int N,
                                 int K, int hasBias, int rowwise) {
  using namespace w8s;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap tmW, tmX;
  {
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)K};
    cuuint64_t strides[1] = {(cuuint64_t)N};
    cuuint32_t box[2] = {COLS, ROWS};
    cuuint32_t es[2] = {1, 1};
    if (enc(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for wInt8 [%d,%d]", K, N);
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)K * 4};
    cuuint32_t box[2] = {ROWS, MR};
    cuuint32_t es[2] = {1, 1};
    if (enc(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for x [%d,%d]", M, K);
  }
  static bool attr_done[64] = {};
  const int ord = s->dev->ordinal;
  if (ord < 0 || ord >= 64 || !attr_done[ord]) {
    cudaError_t e = cudaFuncSetAttribute(w8a16_stream_kernel<1>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(w8a16_stream_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(w8a16_stream_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w8a16_stream)");
    if (ord >= 0 && ord < 64) attr_done[ord] = true;
  }
  Params p;
  p.M = M; p.N = N; p.K = K;
  p.rowwise = rowwise; p.hasBias = hasBias;
  p.sw = sw; p.bias = bias; p.y = y; p.err = s->dev->d_err;
  const int grid = (N + COLS - 1) / COLS;
  for (int m0 = 0; m0 < M;) {
    const int left = M - m0;
    const int r = left >= 4 ? 4 : left >= 2 ? 2 : 1;  // rows of this pass
    p.m0 = m0;
    p.mrows = r;
    if (r == 4) w8a16_stream_kernel<4><<<grid, THREADS, SMEM_BYTES, s->stream>>>(tmW, tmX, p);
    else if (r == 2) w8a16_stream_kernel<2><<<grid, THREADS, SMEM_BYTES, s->stream>>>(tmW, tmX, p);
    else w8a16_stream_kernel<1><<<grid, THREADS, SMEM_BYTES, s->stream>>>(tmW, tmX, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "w8a16_stream launch");
    m0 += r;
  }
  return QGEMM_OK;
}

}  // namespace qg
