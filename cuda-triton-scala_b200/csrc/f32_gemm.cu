// f32_gemm.cu -- the fp32 entry points of the same facade: MatrixOps.matmul,
// MatrixOps.matmulAddBias, BLASOps.sgemm and MatrixOps.gemv
// (src/main/scala/cuda/dsl/operators/linalg/MatrixOps.scala:16-28, :31-44, :230-243,
// :166-177).
//
// GEMM (A [M,K] x B [K,N], both row-major fp32) on the tcgen05 tensor cores with three
// tf32 products per fp32 product ("3xTF32"):
//     a = a_hi + a_lo,  a_hi = a rounded to tf32 (10 mantissa bits), a_lo = a - a_hi (exact)
//     a * b ~= a_lo * b_hi + a_hi * b_lo + a_hi * b_hi
// The dropped a_lo * b_lo term and the tf32 truncation of the lo parts are each below
// 2^-21 of |a * b|, so every product carries about the error of one fp32 rounding; the
// sums are fp32 (TMEM accumulators).  The result agrees with the reference's sequential
// fp32 loop to within fp32 summation error: |y - exact| <= 1e-5 * sum_k |a_k * b_k|.
//
// Two HBM passes split the operands before the GEMM:
//   split_rows_kernel    A [M,K]  -> [M, 2Kp]: hi at [m][k], lo at [m][Kp + k]
//   split_cols_kernel    B [K,N]  -> [N, 2Kp]: the transpose, so that both operands are
//                        K-major, through a 32 x 32 shared-memory tile
// (Kp = K rounded up to 32, one 128-byte k-block; the padding is zero).  The GEMM then
// walks K three times (segments lo*hi, hi*lo, hi*hi: the small terms first) over the
// same kernels as the W8A8 GEMM, with the fp32 epilogue of the entry point
// (alpha * acc + beta * C, or acc + bias[n]).
//
// Infinite inputs: a_hi * b_lo is inf * 0 = NaN when b is exact in tf32, and lo parts of
// opposite sign make inf - inf, where the reference's loop gives +-inf.  The split
// kernels therefore raise a device flag on any infinite value; the GEMM epilogue then
// stores nothing and exact_gemm_kernel (CUDA cores, the reference's loop order with
// each product and sum rounded on its own: bit-identical to it) writes the whole
// output.  Without the flag that kernel returns at once.  NaN inputs need no such
// path: they propagate through the three products as they do through the loop.
//
// Shapes that give the tensor cores few tiles (few rows, or small products) would pay
// the split passes for little; f32_prefer_tc estimates both paths' times and sends
// those to CUDA cores instead:
// rows_gemm_kernel<MT> gives each thread 4 columns of B and MT <= 16 rows of A (A's
// k-tile in shared memory, B read once per 16 rows, coalesced along N) over one K
// chunk, fp32 fma, and writes a partial tile; rows_reduce_kernel adds the chunks in chunk order (so the
// result is deterministic) and applies the epilogue; when the kernels saw an infinite
// input it computes every element in the reference's order instead.
//
// gemv (y = A x, A [M,N] row-major) is bound by the read of A: T threads per row
// (T = 32..256 so that short matrices still fill the GPU), float4 streaming loads,
// four independent partial sums per thread, a shuffle / shared-memory reduction.
// Matrices with fewer rows than 4 blocks per SM cut each row into chunks (one block
// each) whose partial sums a second kernel adds in chunk order.
#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"
#include "ptx.cuh"

namespace qg {
namespace f32 {

constexpr int KB = 32;  // fp32 values per 128-byte k-block

// a = hi + lo with hi exactly representable in tf32 (round half away from zero at the
// 10th mantissa bit) and lo = a - hi exact (Sterbenz: hi and a are within 2^-11 of each
// other).  Infinities and NaN pass whole through hi; a value that would round up to
// infinity is truncated instead.
__device__ __forceinline__ void split_tf32(float a, float& hi, float& lo) {
  const uint32_t u = __float_as_uint(a);
  if ((u & 0x7f800000u) == 0x7f800000u) {
    hi = a;
    lo = 0.f;
    return;
  }
  uint32_t h = (u + 0x1000u) & 0xffffe000u;
  if ((h & 0x7f800000u) == 0x7f800000u) h = u & 0xffffe000u;
  hi = __uint_as_float(h);
  lo = __fsub_rn(a, hi);
}

__device__ __forceinline__ bool is_inf(float v) {
  return (__float_as_uint(v) & 0x7fffffffu) == 0x7f800000u;
}

// x [R, K] (row pitch K) -> out [R, 2Kp].  Grid: x over 4-value groups of a row, y over
// rows (grid-stride in both).  *inf_flag = 1 when a value is infinite.
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ x,
                                                         float* __restrict__ out, int R, int K,
                                                         int Kp, int vec, int* inf_flag) {
  const int groups = Kp / 4;
  for (int r = blockIdx.y; r < R; r += gridDim.y) {
    const float* src = x + (size_t)r * K;
    float* dhi = out + (size_t)r * 2 * Kp;
    float* dlo = dhi + Kp;
    for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += gridDim.x * blockDim.x) {
      const int k = 4 * g;
      float v[4];
      if (vec && k < K) {  // K % 4 == 0: the group is whole
        const float4 t = __ldg(reinterpret_cast<const float4*>(src + k));
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = (k + i < K) ? __ldg(src + k + i) : 0.f;
      }
      float hi[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) split_tf32(v[i], hi[i], lo[i]);
      if (is_inf(v[0]) || is_inf(v[1]) || is_inf(v[2]) || is_inf(v[3])) *inf_flag = 1;
      *reinterpret_cast<float4*>(dhi + k) = make_float4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<float4*>(dlo + k) = make_float4(lo[0], lo[1], lo[2], lo[3]);
    }
  }
}

// B [K, N] (row pitch N) -> out [N, 2Kp], transposed through a 32 x 32 tile.  Block
// 32 x 8; grid x over 32-column blocks of B, y over 32-row blocks of Kp (grid-stride).
__global__ void __launch_bounds__(256) split_cols_kernel(const float* __restrict__ B,
                                                         float* __restrict__ out, int K, int N,
                                                         int Kp, int* inf_flag) {
  // The tf32 GEMM that follows may begin its set-up; it reads the split operands only
  // after griddepcontrol.wait, i.e. after this grid has finished.
  ptx::grid_launch_dependents();
  __shared__ float t[32][33];
  const int n0 = blockIdx.x * 32;
  for (int kb = blockIdx.y; kb < Kp / 32; kb += gridDim.y) {
    const int k0 = kb * 32;
#pragma unroll
    for (int i = threadIdx.y; i < 32; i += 8) {
      const int k = k0 + i, n = n0 + threadIdx.x;
      t[i][threadIdx.x] = (k < K && n < N) ? __ldg(B + (size_t)k * N + n) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = threadIdx.y; i < 32; i += 8) {
      const int n = n0 + i, k = k0 + threadIdx.x;
      if (n < N) {
        float hi, lo;
        const float v = t[threadIdx.x][i];
        split_tf32(v, hi, lo);
        if (is_inf(v)) *inf_flag = 1;
        float* row = out + (size_t)n * 2 * Kp;
        row[k] = hi;
        row[Kp + k] = lo;
      }
    }
    __syncthreads();
  }
}

// K = 0: every sum is 0, so C = 0 (+ bias[n]), or C = alpha * 0 + beta * C.
__global__ void empty_k_kernel(const float* __restrict__ bias, float* __restrict__ C, int M,
                               int N, float alpha, float beta, int mode) {
  const size_t total = (size_t)M * N;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    if (mode == F32_MATMUL_BIAS) v = __fadd_rn(v, bias[i % N]);
    if (mode == F32_SGEMM) v = __fadd_rn(__fmul_rn(alpha, v), __fmul_rn(beta, C[i]));
    C[i] = v;
  }
}

// The whole product on CUDA cores in the reference's order (k ascending per element,
// each product and sum rounded on its own) when *flag != 0; otherwise returns at once.
// 16 x 16 output tiles, 32-deep k tiles of A and B in shared memory; persistent grid.
__global__ void __launch_bounds__(256) exact_gemm_kernel(const float* __restrict__ A,
                                                         const float* __restrict__ B,
                                                         const float* __restrict__ bias,
                                                         float* __restrict__ C, int M, int N,
                                                         int K, float alpha, float beta, int mode,
                                                         const int* flag) {
  if (*reinterpret_cast<const volatile int*>(flag) == 0) return;
  __shared__ float As[16][33];
  __shared__ float Bs[32][17];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int tiles_n = (N + 15) / 16;
  const long long tiles = (long long)tiles_n * ((M + 15) / 16);
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int m0 = (int)(t / tiles_n) * 16, n0 = (int)(t % tiles_n) * 16;
    const int m = m0 + ty, n = n0 + tx;
    float sum = 0.f;
    for (int k0 = 0; k0 < K; k0 += 32) {
      for (int i = threadIdx.x; i < 512; i += 256) {
        const int r = i / 32, c = i % 32;
        As[r][c] = (m0 + r < M && k0 + c < K) ? A[(size_t)(m0 + r) * K + k0 + c] : 0.f;
        const int rb = i / 16, cb = i % 16;
        Bs[rb][cb] = (k0 + rb < K && n0 + cb < N) ? B[(size_t)(k0 + rb) * N + n0 + cb] : 0.f;
      }
      __syncthreads();
      const int kend = K - k0 < 32 ? K - k0 : 32;
      for (int kk = 0; kk < kend; ++kk) sum = __fadd_rn(sum, __fmul_rn(As[ty][kk], Bs[kk][tx]));
      __syncthreads();
    }
    if (m < M && n < N) {
      float* c = C + (size_t)m * N + n;
      if (mode == F32_MATMUL_BIAS) *c = __fadd_rn(sum, bias[n]);
      else if (mode == F32_SGEMM) *c = __fadd_rn(__fmul_rn(alpha, sum), __fmul_rn(beta, *c));
      else *c = sum;
    }
  }
}

// Partial products of rows [m0, m0 + MT) (blockIdx.z) x columns [1024 bx, +1024) over the
// K chunk [kc * by, +kc): part[by][m][n].  256 threads, each 4 adjacent columns x MT
// rows (4 * MT accumulators): per k one float4 of B from global memory (coalesced, B
// read once per row group) and MT / 4 broadcast float4 of A from shared memory for
// 4 * MT fma.  The B loads of the next 8 k are in flight while 8 k are computed.
// vec: N % 4 == 0 and B 16-byte aligned (float4 loads and stores).
template <int MT>
__global__ void __launch_bounds__(256, 2) rows_gemm_kernel(const float* __restrict__ A,
                                                           const float* __restrict__ B,
                                                           float* __restrict__ part, int M,
                                                           int N, int K, int kc, int vec,
                                                           int* inf_flag) {
  __shared__ __align__(16) float As[32][MT];
  const int n = blockIdx.x * 1024 + 4 * threadIdx.x;
  const int k_begin = blockIdx.y * kc;
  const int k_end = K - k_begin < kc ? K : k_begin + kc;
  const int m0 = blockIdx.z * MT;
  float acc[MT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[m][j] = 0.f;
  bool inf = false;
  auto load_b = [&](int k) -> float4 {
    const float* src = B + (size_t)k * N + n;
    if (vec && n + 3 < N) return __ldg(reinterpret_cast<const float4*>(src));
    float4 v;
    v.x = n < N ? __ldg(src) : 0.f;
    v.y = n + 1 < N ? __ldg(src + 1) : 0.f;
    v.z = n + 2 < N ? __ldg(src + 2) : 0.f;
    v.w = n + 3 < N ? __ldg(src + 3) : 0.f;
    return v;
  };
  for (int k0 = k_begin; k0 < k_end; k0 += 32) {
    const int kn = k_end - k0 < 32 ? k_end - k0 : 32;
    for (int i = threadIdx.x; i < 32 * MT; i += 256) {
      const int m = i / 32, kk = i % 32;
      const float v = (m0 + m < M && kk < kn) ? __ldg(A + (size_t)(m0 + m) * K + k0 + kk) : 0.f;
      inf |= is_inf(v);
      As[kk][m] = v;
    }
    __syncthreads();
    if (n < N) {
      for (int kb = 0; kb < kn; kb += 8) {
        float4 b[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) b[u] = (kb + u < kn) ? load_b(k0 + kb + u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          inf |= is_inf(b[u].x) | is_inf(b[u].y) | is_inf(b[u].z) | is_inf(b[u].w);
#pragma unroll
          for (int m = 0; m < MT; m += 4) {
            const float4 a = *reinterpret_cast<const float4*>(&As[kb + u][m]);
            const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              acc[m + i][0] = fmaf(av[i], b[u].x, acc[m + i][0]);
              acc[m + i][1] = fmaf(av[i], b[u].y, acc[m + i][1]);
              acc[m + i][2] = fmaf(av[i], b[u].z, acc[m + i][2]);
              acc[m + i][3] = fmaf(av[i], b[u].w, acc[m + i][3]);
            }
          }
        }
      }
    }
    __syncthreads();
  }
  if (inf) *inf_flag = 1;
  if (n < N) {
    float* dst = part + ((size_t)blockIdx.y * M + m0) * N + n;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m0 + m >= M) break;
      float* row = dst + (size_t)m * N;
      if (vec && n + 3 < N) {
        *reinterpret_cast<float4*>(row) = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (n + j < N) row[j] = acc[m][j];
      }
    }
  }
}

// C = epilogue(sum over chunks of part[c]).  With *flag set (an infinite input) each
// element is instead the reference's loop: k ascending, each product and sum rounded on
// its own (bit-identical to it).
__global__ void __launch_bounds__(256) rows_reduce_kernel(const float* __restrict__ part,
                                                          const float* __restrict__ A,
                                                          const float* __restrict__ B,
                                                          const float* __restrict__ bias,
                                                          float* __restrict__ C, int M, int N,
                                                          int K, int chunks, float alpha,
                                                          float beta, int mode, const int* flag) {
  const bool exact = *reinterpret_cast<const volatile int*>(flag) != 0;
  const size_t total = (size_t)M * N;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    float v;
    if (exact) {
      const size_t m = i / N, n = i % N;
      v = 0.f;
      for (int k = 0; k < K; ++k) v = __fadd_rn(v, __fmul_rn(A[m * K + k], B[(size_t)k * N + n]));
    } else {
      v = __ldcs(part + i);
      for (int c = 1; c < chunks; ++c) v = __fadd_rn(v, __ldcs(part + (size_t)c * total + i));
    }
    if (mode == F32_MATMUL_BIAS) v = __fadd_rn(v, bias[i % N]);
    else if (mode == F32_SGEMM) v = __fadd_rn(__fmul_rn(alpha, v), __fmul_rn(beta, C[i]));
    C[i] = v;
  }
}

// y[row] = sum_j A[row, j] * x[j]: groups of T threads per row, 256 / T rows per block.
template <int T>
__global__ void __launch_bounds__(256) gemv_kernel(const float* __restrict__ A,
                                                   const float* __restrict__ x,
                                                   float* __restrict__ y, int M, int N, int vec) {
  constexpr int R = 256 / T;
  const int g = threadIdx.x / T, t = threadIdx.x % T;
  __shared__ float red[8];
  for (int row0 = blockIdx.x * R; row0 < M; row0 += gridDim.x * R) {  // uniform per block
    const int row = row0 + g;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    if (row < M) {
      const float* a = A + (size_t)row * N;
      if (vec) {
        const float4* a4 = reinterpret_cast<const float4*>(a);
        const float4* x4 = reinterpret_cast<const float4*>(x);
        const int n4 = N / 4;
        int j = t;
        for (; j + 3 * T < n4; j += 4 * T) {
          float4 av[4], xv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) av[u] = __ldcs(a4 + j + u * T);
#pragma unroll
          for (int u = 0; u < 4; ++u) xv[u] = __ldg(x4 + j + u * T);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            s0 = fmaf(av[u].x, xv[u].x, s0);
            s1 = fmaf(av[u].y, xv[u].y, s1);
            s2 = fmaf(av[u].z, xv[u].z, s2);
            s3 = fmaf(av[u].w, xv[u].w, s3);
          }
        }
        for (; j < n4; j += T) {
          const float4 av = __ldcs(a4 + j), xv = __ldg(x4 + j);
          s0 = fmaf(av.x, xv.x, s0);
          s1 = fmaf(av.y, xv.y, s1);
          s2 = fmaf(av.z, xv.z, s2);
          s3 = fmaf(av.w, xv.w, s3);
        }
      } else {
        for (int j = t; j < N; j += T) s0 = fmaf(__ldcs(a + j), __ldg(x + j), s0);
      }
    }
    float s = (s0 + s1) + (s2 + s3);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if constexpr (T > 32) {
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
      __syncthreads();
      if (t == 0) {
        s = 0.f;
#pragma unroll
        for (int w = 0; w < T / 32; ++w) s += red[g * (T / 32) + w];
      }
      __syncthreads();
    }
    if (t == 0 && row < M) y[row] = s;
  }
}

// Short matrices (too few rows to fill the GPU): row blockIdx.y is cut into chunks of L
// values (a multiple of 1024), one block each; part[row * chunks + chunk].
__global__ void __launch_bounds__(256) gemv_split_kernel(const float* __restrict__ A,
                                                         const float* __restrict__ x,
                                                         float* __restrict__ part, int N, int L,
                                                         int vec) {
  const int row = blockIdx.y;
  const int j0 = blockIdx.x * L;
  const int j1 = N - j0 < L ? N : j0 + L;
  const float* a = A + (size_t)row * N;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (vec) {  // N % 4 == 0 and j0 % 4 == 0
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll 4
    for (int j = j0 / 4 + threadIdx.x; j < j1 / 4; j += 256) {
      const float4 av = __ldcs(a4 + j), xv = __ldg(x4 + j);
      s0 = fmaf(av.x, xv.x, s0);
      s1 = fmaf(av.y, xv.y, s1);
      s2 = fmaf(av.z, xv.z, s2);
      s3 = fmaf(av.w, xv.w, s3);
    }
  } else {
    for (int j = j0 + threadIdx.x; j < j1; j += 256) s0 = fmaf(__ldcs(a + j), __ldg(x + j), s0);
  }
  float s = (s0 + s1) + (s2 + s3);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w];
    part[(size_t)row * gridDim.x + blockIdx.x] = t;
  }
}

// y[row] = sum of the row's chunks: one block per row; thread t adds chunks t, t + 256,
// ... in order, then a fixed shuffle / shared-memory tree (deterministic).
__global__ void __launch_bounds__(256) gemv_reduce_kernel(const float* __restrict__ part,
                                                          float* __restrict__ y, int chunks) {
  const float* pr = part + (size_t)blockIdx.x * chunks;
  float s = 0.f;
  for (int c = threadIdx.x; c < chunks; c += 256) s += pr[c];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w];
    y[blockIdx.x] = t;
  }
}

}  // namespace f32

// Stream scratch layout of one fp32 GEMM: the tcgen05 GEMM's split scratch (its counter
// block first, kept in place for every other call on the stream), 1 KiB holding the
// infinity flag, then A split and B split (tensor cores) or the partial tiles (CUDA
// cores); 1 KiB aligned.
struct F32Layout {
  size_t sc, flag, a, b, total;
};

static F32Layout f32_layout_tc(const qgemm_device_s* d, int M, int N, int K) {
  const size_t Kp = ((size_t)K + f32::KB - 1) / f32::KB * f32::KB;
  F32Layout l;
  l.sc = (tc_gemm_scratch_bytes(d, M, N, 3 * (int)(Kp / f32::KB), true) + 1023) & ~(size_t)1023;
  l.flag = l.sc;
  l.a = l.flag + 1024;
  l.b = l.a + (((size_t)M * 2 * Kp * 4 + 1023) & ~(size_t)1023);
  l.total = l.b + (size_t)N * 2 * Kp * 4;
  return l;
}

// CUDA-core plan: rows per thread, K chunk, grid.
struct RowsPlan {
  int mt, kc, chunks;
  dim3 grid;
};

static RowsPlan rows_plan(const qgemm_device_s* d, int M, int N, int K) {
  RowsPlan r;
  r.mt = M <= 4 ? 4 : M <= 8 ? 8 : 16;
  const int gx = (N + 1023) / 1024, gz = (M + r.mt - 1) / r.mt;
  // Two resident blocks per SM (launch bounds); K chunks of at least 64 so that the
  // partial sums stay small next to the reads of B.
  const long long slots = (long long)d->sm_count * 2;
  const long long tiles = (long long)gx * gz;
  long long chunks = (slots + tiles - 1) / tiles;
  const long long max_chunks = (K + 63) / 64;
  if (chunks > max_chunks) chunks = max_chunks;
  if (chunks < 1) chunks = 1;
  r.kc = (int)(((K + chunks - 1) / chunks + 31) / 32 * 32);
  r.chunks = (K + r.kc - 1) / r.kc;
  r.grid = dim3(gx, r.chunks, gz);
  return r;
}

// Path choice for QGEMM_ALGO_AUTO from a time estimate of each path, with rates
// measured on B200 (CUDA events, fp32 inputs in HBM):
//   tensor cores: ~1.55 TFLOP/s of fp32 work per busy SM for the GEMM (4096^3: 598 of
//     663 us), SMs busy = min(2 x pair tiles x K parts, SMs) (pairs also for shapes
//     whose 1-CTA tiles cannot fill the GPU) or the 1-CTA tiles; plus
//     the split passes' 20 bytes per element of A and B at ~6 TB/s; plus ~40 us of
//     fixed cost (launches, tensor maps, pipeline fill; 256^3 takes 45 us);
//   CUDA cores: ~24 TFLOP/s when N fills 1024-column blocks (scaled down by N / 1024
//     below that) plus ~15 us of fixed cost.
static bool f32_prefer_tc(const qgemm_device_s* d, int M, int N, int K) {
  const double flops = 2.0 * M * (double)N * K;
  const int max_pairs = d->sm_count / 2;
  double busy, work;  // busy SMs; fp32 work of the whole tiles (edges included)
  const double tiles1 = (double)((M + 127) / 128) * (double)((N + 255) / 256);
  if ((M >= 256 && N >= 256) || tiles1 < d->sm_count) {  // tc_plan's pair choice
    const long long tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
    long long parts = 1;
    if (tiles < max_pairs) {  // tc_plan's full split
      const long long kb = 3LL * ((K + 31) / 32);
      parts = max_pairs / tiles;
      if (parts > 8) parts = 8;
      if (parts > kb / 8) parts = kb / 8;
      if (parts < 2) parts = 1;
    }
    busy = 2.0 * (double)tiles * (double)parts;
    work = 2.0 * (double)tiles * 256.0 * 256.0 * K;
  } else {
    busy = tiles1;
    work = 2.0 * tiles1 * 128.0 * 256.0 * K;
  }
  if (busy > d->sm_count) busy = d->sm_count;
  const double t_tc = work / (busy * 1.55e12) + 20.0 * (M + (double)N) * K / 6.0e12 + 40e-6;
  const double fill = N >= 1024 ? 1.0 : N / 1024.0;
  const double t_simt = flops / (24e12 * fill) + 15e-6;
  return t_tc < t_simt;
}

static qgemm_status launch_exact(qgemm_stream_s* s, const float* A, const float* B,
                                 const float* bias, float* C, int M, int N, int K, float alpha,
                                 float beta, int mode, const int* inf_flag) {
  f32::exact_gemm_kernel<<<s->dev->sm_count * 8, 256, 0, s->stream>>>(A, B, bias, C, M, N, K,
                                                                       alpha, beta, mode,
                                                                       inf_flag);
  return cuda_fail(cudaGetLastError(), "exact_gemm launch");
}

static qgemm_status launch_f32_rows(qgemm_stream_s* s, const float* A, const float* B,
                                    const float* bias, float* C, int M, int N, int K,
                                    float alpha, float beta, int mode) {
  using namespace f32;
  const RowsPlan r = rows_plan(s->dev, M, N, K);
  if (r.grid.z > 65535u || r.grid.y > 65535u)
    return fail(QGEMM_ERR_UNSUPPORTED, "CUDA-core fp32 GEMM: M=%d needs more than 65535 row groups", M);
  const size_t cnt = (tc_gemm_scratch_bytes(s->dev, 1, 1, 1) + 1023) & ~(size_t)1023;
  const size_t total = cnt + 1024 + (size_t)r.chunks * M * N * 4;
  void* ws = nullptr;
  const qgemm_status st = stream_workspace(s, total, &ws);
  if (st != QGEMM_OK) return st;
  int* inf_flag = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) + cnt);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + cnt + 1024);
  cudaError_t e = cudaMemsetAsync(inf_flag, 0, sizeof(int), s->stream);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the infinity flag");
  const int vec = (N % 4 == 0) && aligned((uint64_t)B, 16);
  switch (r.mt) {
    case 4: rows_gemm_kernel<4><<<r.grid, 256, 0, s->stream>>>(A, B, part, M, N, K, r.kc, vec, inf_flag); break;
    case 8: rows_gemm_kernel<8><<<r.grid, 256, 0, s->stream>>>(A, B, part, M, N, K, r.kc, vec, inf_flag); break;
    default: rows_gemm_kernel<16><<<r.grid, 256, 0, s->stream>>>(A, B, part, M, N, K, r.kc, vec, inf_flag); break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rows_gemm launch");
  const size_t elems = (size_t)M * N;
  const size_t cap = (size_t)s->dev->sm_count * 16;
  const int grid = (int)((elems + 255) / 256 < cap ? (elems + 255) / 256 : cap);
  rows_reduce_kernel<<<grid, 256, 0, s->stream>>>(part, A, B, bias, C, M, N, K, r.chunks, alpha,
                                                  beta, mode, inf_flag);
  return cuda_fail(cudaGetLastError(), "rows_reduce launch");
}

static qgemm_status launch_f32_tc(qgemm_stream_s* s, const float* A, const float* B,
                                  const float* bias, float* C, int M, int N, int K, float alpha,
                                  float beta, int mode) {
  using namespace f32;
  const int Kp = (K + KB - 1) / KB * KB;
  const F32Layout l = f32_layout_tc(s->dev, M, N, K);
  void* ws = nullptr;
  const qgemm_status st = stream_workspace(s, l.total, &ws);
  if (st != QGEMM_OK) return st;
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  int* inf_flag = reinterpret_cast<int*>(w8 + l.flag);
  float* As = reinterpret_cast<float*>(w8 + l.a);
  float* Bs = reinterpret_cast<float*>(w8 + l.b);

  cudaError_t e = cudaMemsetAsync(inf_flag, 0, sizeof(int), s->stream);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the infinity flag");
  const int vec = (K % 4 == 0) && aligned((uint64_t)A, 16);
  const int gx = (Kp / 4 + 255) / 256;
  const int gy = M < 65535 ? M : 65535;
  split_rows_kernel<<<dim3(gx, gy), 256, 0, s->stream>>>(A, As, M, K, Kp, vec, inf_flag);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "split_rows launch");
  const int cy = Kp / 32 < 65535 ? Kp / 32 : 65535;
  split_cols_kernel<<<dim3((N + 31) / 32, cy), dim3(32, 8), 0, s->stream>>>(B, Bs, K, N, Kp,
                                                                           inf_flag);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "split_cols launch");

  TcArgs a;
  a.kind = KIND_TF32;
  a.A = As;
  a.B = Bs;
  a.M = M;
  a.N = N;
  a.K = 4 * Kp;         // bytes of one segment
  a.nseg = 3;           // lo*hi, hi*lo, hi*hi
  a.a_seg = 0x1u;
  a.b_seg = 0x2u;
  a.a_pitch = 8 * (uint64_t)Kp;
  a.b_pitch = 8 * (uint64_t)Kp;
  a.out = C;
  a.out_dtype = QGEMM_F32;
  a.ldc = N;
  a.alpha = alpha;
  a.beta = beta;
  a.ep_alpha = mode == F32_SGEMM;
  a.ep_beta = mode == F32_SGEMM;
  a.bias = mode == F32_MATMUL_BIAS ? bias : nullptr;
  a.skip_flag = inf_flag;
  a.full_split = 1;
  a.scratch = ws;
  a.scratch_bytes = l.sc;
  const qgemm_status gs = launch_tc_gemm(s, a);
  if (gs != QGEMM_OK) return gs;
  return launch_exact(s, A, B, bias, C, M, N, K, alpha, beta, mode, inf_flag);
}

qgemm_status launch_f32_gemm(qgemm_stream_s* s, const float* A, const float* B,
                             const float* bias, float* C, int M, int N, int K, float alpha,
                             float beta, int mode, int algo) {
  using namespace f32;
  if (K == 0) {
    const size_t total = (size_t)M * N;
    const size_t cap = (size_t)s->dev->sm_count * 16;
    const int grid = (int)((total + 255) / 256 < cap ? (total + 255) / 256 : cap);
    empty_k_kernel<<<grid, 256, 0, s->stream>>>(bias, C, M, N, alpha, beta, mode);
    return cuda_fail(cudaGetLastError(), "empty_k launch");
  }
  bool tc = algo == QGEMM_ALGO_TCGEN05;
  if (algo == QGEMM_ALGO_AUTO)
    tc = s->dev->tcgen05 && (f32_prefer_tc(s->dev, M, N, K) || (M + 15) / 16 > 65535);
  if (tc && !s->dev->tcgen05) return fail(QGEMM_ERR_UNSUPPORTED, "device is not sm_100");
  return tc ? launch_f32_tc(s, A, B, bias, C, M, N, K, alpha, beta, mode)
            : launch_f32_rows(s, A, B, bias, C, M, N, K, alpha, beta, mode);
}

qgemm_status launch_f32_gemv(qgemm_stream_s* s, const float* A, const float* x, float* y, int M,
                             int N) {
  using namespace f32;
  // Threads per row: enough groups to fill the GPU (64 warps per SM), at least two
  // float4 per thread.
  const long long target_warps = (long long)s->dev->sm_count * 64;
  // Fewer rows than 8 blocks per SM: cut the rows into chunks of at least 1024 values.
  const long long target_blocks = (long long)s->dev->sm_count * 8;
  if ((long long)M < target_blocks / 2 && N >= 2048) {
    long long chunks = (target_blocks + M - 1) / M;
    if (chunks > N / 1024) chunks = N / 1024;
    const int L = (int)(((N + chunks - 1) / chunks + 1023) / 1024 * 1024);
    const int nch = (N + L - 1) / L;
    if (nch >= 2) {
      const size_t cnt = (tc_gemm_scratch_bytes(s->dev, 1, 1, 1) + 1023) & ~(size_t)1023;
      void* ws = nullptr;
      const qgemm_status st = stream_workspace(s, cnt + (size_t)M * nch * 4, &ws);
      if (st != QGEMM_OK) return st;
      float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + cnt);
      const int vec = (N % 4 == 0) && aligned((uint64_t)A, 16) && aligned((uint64_t)x, 16);
      gemv_split_kernel<<<dim3(nch, M), 256, 0, s->stream>>>(A, x, part, N, L, vec);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_fail(e, "gemv_split launch");
      gemv_reduce_kernel<<<M, 256, 0, s->stream>>>(part, y, nch);
      return cuda_fail(cudaGetLastError(), "gemv_reduce launch");
    }
  }
  int T = 32;
  while (T < 256 && (long long)M * (T / 32) < target_warps && (long long)T * 8 <= N) T *= 2;
  const int R = 256 / T;
  const long long blocks = ((long long)M + R - 1) / R;
  const long long cap = (long long)s->dev->sm_count * 32;
  const int grid = (int)(blocks < cap ? blocks : cap);
  const int vec = (N % 4 == 0) && aligned((uint64_t)A, 16) && aligned((uint64_t)x, 16);
  switch (T) {
    case 32: gemv_kernel<32><<<grid, 256, 0, s->stream>>>(A, x, y, M, N, vec); break;
    case 64: gemv_kernel<64><<<grid, 256, 0, s->stream>>>(A, x, y, M, N, vec); break;
    case 128: gemv_kernel<128><<<grid, 256, 0, s->stream>>>(A, x, y, M, N, vec); break;
    default: gemv_kernel<256><<<grid, 256, 0, s->stream>>>(A, x, y, M, N, vec); break;
  }
  return cuda_fail(cudaGetLastError(), "gemv launch");
}

}  // namespace qg
