// int8_names.cu -- the int8 GEMM names of the reference's intrinsic and CUTLASS-style
// operator objects, routed onto the tcgen05 W8A8 GEMM:
//
//  * TensorCoreOps.tensorCoreGemmInt8 (operators/intrinsic/TensorCoreOps.scala:294-340):
//      d[m*ldd+n] = sum_k a[m*lda+k] * b[k*ldb+n]  (+ c[m*ldc+n] when hasC)
//    int8 operands through leading dimensions, int32 sums (wrapping like Scala Int),
//    int32 output.  The tensor-core kernel writes the sums plus c straight from TMEM;
//    other shapes run an exact CUDA-core kernel.
//  * CutlassGemm.int8GemmKernel (cutlass/CutlassGemm.scala:987-1041):
//      D[m*ldd+n] = (sum_k float(A[m*lda+k]) * float(B[k*ldb+n])) * scaleA * scaleB
//    int8 values held in Int (32-bit) arrays.  A pass packs them to int8 (zero padded to
//    a multiple of 16 along K) and raises a device flag on any value outside
//    [-128, 127]; the tensor-core GEMM then computes the exact integer sum and its
//    epilogue (float(acc) * scaleA) * scaleB, the reference's rounding order.  When the
//    flag is up the epilogue stores nothing and a CUDA-core kernel runs the reference's
//    fp32 loop (k ascending, each product and sum rounded on its own) instead; without
//    the flag that kernel returns at once.  The integer sum equals the fp32 loop
//    whenever no partial sum leaves +-2^24 (always for K <= 1040 with int8 values);
//    beyond that it is the correctly rounded value of the same sum.
//
// Both bodies in the reference are unusable as written (a -128 offset on signed bytes,
// every 16th k, one output per block; one accumulator shared by 64 outputs), so only
// the arithmetic they name is kept.
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"

namespace qg {
namespace i8names {

// ---- exact int32 GEMM through leading dimensions (CUDA cores) ----
constexpr int TM = 64, TN = 64, TK = 32;

__global__ void __launch_bounds__(256)
    i8_gemm_ld_kernel(const int8_t* __restrict__ a, const int8_t* __restrict__ b,
                      const int32_t* __restrict__ c, int32_t* __restrict__ d, int M, int N,
                      int K, int lda, int ldb, int ldc, int ldd) {
  __shared__ int32_t As[TK][TM + 1];
  __shared__ int32_t Bs[TK][TN + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  uint32_t acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < TM * TK; i += 256) {
      const int mm = i / TK, kk = i % TK;
      const int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? (int32_t)a[(size_t)m * lda + k] : 0;
    }
    for (int i = threadIdx.x; i < TN * TK; i += 256) {
      const int kk = i / TN, nn = i % TN;
      const int n = n0 + nn, k = k0 + kk;
      Bs[kk][nn] = (n < N && k < K) ? (int32_t)b[(size_t)k * ldb + n] : 0;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < TK; ++kk) {
      uint32_t av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = (uint32_t)As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = (uint32_t)Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= N) continue;
      const uint32_t cv = c ? (uint32_t)c[(size_t)m * ldc + n] : 0u;
      d[(size_t)m * ldd + n] = (int32_t)(acc[i][j] + cv);
    }
  }
}

// ---- int8GemmKernel: pack, scale vectors, fp32-loop fallback ----

// dst[r * dst_pitch + k] = (int8) src[r * src_ld + k] for r < rows and k < cols, 0 for
// the padding (cols <= k < dst_pitch, rows <= r < dst_rows); *flag = 1 when a value is
// outside [-128, 127].  One thread per 4 output bytes, grid-stride over rows.
__global__ void pack_i32_to_i8_kernel(const int32_t* __restrict__ src, int8_t* __restrict__ dst,
                                      int rows, int dst_rows, int cols, int src_ld,
                                      int dst_pitch, int* flag) {
  const int quads = dst_pitch / 4;
  bool bad = false;
  for (int r = blockIdx.y; r < dst_rows; r += gridDim.y) {
    const int32_t* s = src + (size_t)r * src_ld;
    for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < quads; q += gridDim.x * blockDim.x) {
      uint32_t w = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = 4 * q + j;
        int32_t v = 0;
        if (r < rows && k < cols) {
          v = s[k];
          if (v < -128 || v > 127) bad = true;
        }
        w |= ((uint32_t)v & 0xFFu) << (8 * j);
      }
      *reinterpret_cast<uint32_t*>(dst + (size_t)r * dst_pitch + 4 * q) = w;
    }
  }
  if (bad) *flag = 1;
}

// sA[m] = scaleB (m < M), sB[n] = scaleA (n < N): the W8A8 epilogue
// (float(acc) * sB[n]) * sA[m] is then (acc * scaleA) * scaleB.
__global__ void fill_scales_kernel(float* sA, int M, float scaleB, float* sB, int N,
                                   float scaleA) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < M + N; i += gridDim.x * blockDim.x) {
    if (i < M) sA[i] = scaleB;
    else sB[i - M] = scaleA;
  }
}

// The reference's loop for every output: acc = acc + float(A) * float(B), k ascending,
// then (acc * scaleA) * scaleB.  Runs when *flag != 0 (or flag is null); otherwise
// returns at once.  One thread per output, columns across the warp.
__global__ void int8_gemm_fp32_loop_kernel(float* __restrict__ D, const int32_t* __restrict__ A,
                                           const int32_t* __restrict__ B, int M, int N, int K,
                                           int lda, int ldb, int ldd, float scaleA, float scaleB,
                                           const int* flag) {
  if (flag && *reinterpret_cast<const volatile int*>(flag) == 0) return;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N || m >= M) return;
  float acc = 0.0f;
  const int32_t* a = A + (size_t)m * lda;
  for (int k = 0; k < K; ++k)
    acc = __fadd_rn(acc, __fmul_rn(__int2float_rn(a[k]), __int2float_rn(B[(size_t)k * ldb + n])));
  D[(size_t)m * ldd + n] = __fmul_rn(__fmul_rn(acc, scaleA), scaleB);
}

}  // namespace i8names
}  // namespace qg

using namespace qg;

namespace {

qgemm_status check_ld(int M, int N, int K, int lda, int ldb, int ldd) {
  if (M < 0 || N < 0 || K < 0)
    return fail(QGEMM_ERR_INVALID_ARG, "negative size M=%d N=%d K=%d", M, N, K);
  if (lda < K || ldb < N || ldd < N)
    return fail(QGEMM_ERR_INVALID_ARG, "leading dimension too small (lda=%d K=%d, ldb=%d N=%d, "
                "ldd=%d N=%d)", lda, K, ldb, N, ldd, N);
  return QGEMM_OK;
}

}  // namespace

extern "C" {

qgemm_status qgemm_tensor_core_gemm_int8(qgemm_stream_t s, uint64_t a, uint64_t b,
                                         uint64_t scalesA, uint64_t scalesB, uint64_t c,
                                         uint64_t d, int M, int N, int K, int lda, int ldb,
                                         int ldc, int ldd, int hasC) {
  (void)scalesA;
  (void)scalesB;  // parameters of the reference method that its body never reads
  qgemm_status st = enter(s);
  if (st != QGEMM_OK) return st;
  if ((st = check_ld(M, N, K, lda, ldb, ldd)) != QGEMM_OK) return st;
  if (hasC && ldc < N) return fail(QGEMM_ERR_INVALID_ARG, "ldc %d < N %d", ldc, N);
  if (M == 0 || N == 0) return QGEMM_OK;
  if (!d) return fail(QGEMM_ERR_INVALID_ARG, "d is null");
  if (hasC && !c) return fail(QGEMM_ERR_INVALID_ARG, "hasC is set and c is null");
  if (K > 0 && (!a || !b)) return fail(QGEMM_ERR_INVALID_ARG, "a or b is null");
  if (!aligned(d, 4) || (hasC && !aligned(c, 4)))
    return fail(QGEMM_ERR_BAD_ALIGN, "c and d must be 4-byte aligned");
  const int32_t* cp = hasC ? reinterpret_cast<const int32_t*>(c) : nullptr;
  int32_t* dp = reinterpret_cast<int32_t*>(d);
  const bool tc = K > 0 && s->dev->tcgen05 && lda % 16 == 0 && ldb % 16 == 0 &&
                  aligned(a, 16) && aligned(b, 16);
  if (tc) {
    TcArgs t;
    t.kind = KIND_I8;
    t.A = reinterpret_cast<const void*>(a);
    t.a_pitch = (uint64_t)lda;
    t.a_extent = (uint64_t)K;
    t.B = reinterpret_cast<const void*>(b);
    t.b_kn = 1;
    t.b_kn_pitch = (uint64_t)ldb;
    t.M = M; t.N = N; t.K = K;
    t.acc = dp;
    t.acc_ld = ldd;
    t.acc_c = cp;
    t.acc_c_ld = ldc;
    t.no_out = 1;
    t.out_dtype = QGEMM_F32;
    t.ldc = N;
    return launch_tc_gemm(s, t);
  }
  dim3 grid((N + i8names::TN - 1) / i8names::TN, (M + i8names::TM - 1) / i8names::TM);
  if (grid.y > 65535) return fail(QGEMM_ERR_UNSUPPORTED, "M %d too large for the CUDA-core path", M);
  i8names::i8_gemm_ld_kernel<<<grid, 256, 0, s->stream>>>(
      reinterpret_cast<const int8_t*>(a), reinterpret_cast<const int8_t*>(b), cp, dp, M, N, K,
      lda, ldb, ldc, ldd);
  return cuda_fail(cudaGetLastError(), "i8_gemm_ld_kernel launch");
}

qgemm_status qgemm_int8_gemm_kernel(qgemm_stream_t s, uint64_t D, uint64_t A, uint64_t B, int M,
                                    int N, int K, int lda, int ldb, int ldd, float scaleA,
                                    float scaleB) {
  qgemm_status st = enter(s);
  if (st != QGEMM_OK) return st;
  if ((st = check_ld(M, N, K, lda, ldb, ldd)) != QGEMM_OK) return st;
  if (M == 0 || N == 0) return QGEMM_OK;
  if (!D) return fail(QGEMM_ERR_INVALID_ARG, "D is null");
  if (K > 0 && (!A || !B)) return fail(QGEMM_ERR_INVALID_ARG, "A or B is null");
  if (!aligned(D, 4) || !aligned(A, 4) || !aligned(B, 4))
    return fail(QGEMM_ERR_BAD_ALIGN, "D, A and B must be 4-byte aligned");
  if (M > 65535) return fail(QGEMM_ERR_UNSUPPORTED, "M %d > 65535", M);
  float* Dp = reinterpret_cast<float*>(D);
  const int32_t* Ap = reinterpret_cast<const int32_t*>(A);
  const int32_t* Bp = reinterpret_cast<const int32_t*>(B);
  const dim3 lgrid((N + 127) / 128, M);
  if (K == 0 || !s->dev->tcgen05) {
    i8names::int8_gemm_fp32_loop_kernel<<<lgrid, 128, 0, s->stream>>>(
        Dp, Ap, Bp, M, N, K, lda, ldb, ldd, scaleA, scaleB, nullptr);
    return cuda_fail(cudaGetLastError(), "int8_gemm_fp32_loop_kernel launch");
  }
  // Scratch after the GEMM's counter block: the range flag, sA [M], sB [N], A8 [M, Kp],
  // B8 [Kp, Np] (rows of A and of B, zero padded to multiples of 16 in both dimensions).
  const int Kp = (K + 15) / 16 * 16, Np = (N + 15) / 16 * 16;
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t o_flag = up(tc_gemm_scratch_bytes(s->dev, M, N, (Kp + 127) / 128));
  const size_t o_sa = o_flag + 256;
  const size_t o_sb = o_sa + up((size_t)M * 4);
  const size_t o_a8 = o_sb + up((size_t)N * 4);
  const size_t o_b8 = o_a8 + up((size_t)M * Kp);
  const size_t total = o_b8 + up((size_t)Kp * Np);
  void* ws = nullptr;
  if ((st = stream_workspace(s, total, &ws)) != QGEMM_OK) return st;
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  int* flag = reinterpret_cast<int*>(w8 + o_flag);
  float* sA = reinterpret_cast<float*>(w8 + o_sa);
  float* sB = reinterpret_cast<float*>(w8 + o_sb);
  int8_t* A8 = reinterpret_cast<int8_t*>(w8 + o_a8);
  int8_t* B8 = reinterpret_cast<int8_t*>(w8 + o_b8);
  cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), s->stream);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the range flag");
  const int gx_a = (Kp / 4 + 255) / 256, gx_b = (Np / 4 + 255) / 256;
  i8names::pack_i32_to_i8_kernel<<<dim3(gx_a, M < 65535 ? M : 65535), 256, 0, s->stream>>>(
      Ap, A8, M, M, K, lda, Kp, flag);
  i8names::pack_i32_to_i8_kernel<<<dim3(gx_b, Kp < 65535 ? Kp : 65535), 256, 0, s->stream>>>(
      Bp, B8, K, Kp, N, ldb, Np, flag);
  i8names::fill_scales_kernel<<<(M + N + 255) / 256 < 1024 ? (M + N + 255) / 256 : 1024, 256, 0,
                                s->stream>>>(sA, M, scaleB, sB, N, scaleA);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "int8GemmKernel packing");
  TcArgs t;
  t.kind = KIND_I8;
  t.A = A8;
  t.a_pitch = (uint64_t)Kp;
  t.B = B8;
  t.b_kn = 1;
  t.b_kn_pitch = (uint64_t)Np;
  t.M = M; t.N = N; t.K = Kp;
  t.sA = sA; t.sB = sB;
  t.out = Dp;
  t.out_dtype = QGEMM_F32;
  t.ldc = ldd;
  t.skip_flag = flag;
  if ((st = launch_tc_gemm(s, t)) != QGEMM_OK) return st;
  i8names::int8_gemm_fp32_loop_kernel<<<lgrid, 128, 0, s->stream>>>(
      Dp, Ap, Bp, M, N, K, lda, ldb, ldd, scaleA, scaleB, flag);
  return cuda_fail(cudaGetLastError(), "int8_gemm_fp32_loop_kernel launch");
}

}  // extern "C"
