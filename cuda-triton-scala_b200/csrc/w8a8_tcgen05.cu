// w8a8_tcgen05.cu -- W8A8 GEMM on the sm_100a tensor cores.
//
// Computes the arithmetic of QuantizedGemmOps.w8a32Gemm
// (src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala:102-113):
//     acc[m,n] = sum_k A[m,k] * B[k,n]            (int32, exact)
//     y[m,n]   = (float(acc) * sB[n]) * sA[m]      (fp32, two roundings, in order)
// with y stored as fp32 or as bf16 (round to nearest even).
//
// Design (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: A tile [128 x 128 B] and B tile [256 x 128 B] per stage,
//               128-byte swizzle, STAGES-deep ring of shared-memory buffers.
//   warp 1      allocates 512 TMEM columns; one thread issues tcgen05.mma kind::i8
//               (M=128, N=256, K=32) into one of two 256-column TMEM accumulators.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (one TMEM lane = one output
//               row per thread), dequant with the two scales, global stores.  The
//               two accumulators let the epilogue of tile i overlap the MMAs of i+1.
// B is read either in the reference layout [K,N] (MN-major UMMA operand) or as
// [N,K] (K-major).  Every barrier wait is bounded (ptx::mbar_wait); a wait that
// runs out records an error code in the device error word and the CTA drains
// its in-flight copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace qg {
namespace w8a8 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes of K per stage = one 128-byte swizzle row
constexpr int UMMA_K = 32;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;                   // 16 KB
constexpr int B_BYTES = BN * BK;                   // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;     // 48 KB
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 2 * BN;                  // two accumulators
constexpr int BAR_BYTES = 256;
// The whole opt-in shared memory of an SM (227 KB): STAGES * 48 KB of tiles plus
// barriers and 1 KB of alignment slack, and headroom so that every address a
// UMMA descriptor of the last stage can reach (under either reading of the
// MN-major leading/stride offsets) stays inside this CTA's allocation.
constexpr int SMEM_BYTES = 232448;
static_assert(STAGES * STAGE_BYTES + BAR_BYTES + 1024 <= SMEM_BYTES, "shared memory budget");
constexpr int GROUP_M = 16;                         // tile raster: 16 m-blocks per group

struct Params {
  int M, N, K, ldc;
  int out_dtype;   // QGEMM_F32 / QGEMM_BF16
  int b_kn;        // 1: B is [K,N] (MN-major operand); 0: B is [N,K]
  int num_m_blocks, num_n_blocks, num_k_blocks, num_tiles;
  const float* sA;
  const float* sB;
  void* out;
  int32_t* acc;
  int* err;
  int out_vec;     // out base 16-byte aligned and rows a multiple of 16 bytes
  int acc_vec;     // same for the int32 accumulator output
};

__device__ __forceinline__ void tile_coords(int tile, const Params& p, int& mb, int& nb) {
  const int group_size = GROUP_M * p.num_n_blocks;
  const int group = tile / group_size;
  const int first_m = group * GROUP_M;
  const int rows = min(p.num_m_blocks - first_m, GROUP_M);
  const int in_group = tile - group * group_size;
  mb = first_m + in_group % rows;
  nb = in_group / rows;
}

__device__ __forceinline__ void report(int* err, int code, volatile int* abort_flag) {
  *abort_flag = 1;
  if (err) atomicCAS(err, 0, code);
}

// Epilogue for 32 consecutive columns of one row.
__device__ __forceinline__ void store_chunk(const Params& p, int row, int n0, float sa,
                                            const uint32_t (&r)[32]) {
  if (row >= p.M || n0 >= p.N) return;
  const bool full = (n0 + 32 <= p.N);
  float sb[32];
  if (full && ((reinterpret_cast<uintptr_t>(p.sB + n0) & 15) == 0)) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p.sB + n0 + j));
      sb[j] = v.x; sb[j + 1] = v.y; sb[j + 2] = v.z; sb[j + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) sb[j] = (n0 + j < p.N) ? __ldg(p.sB + n0 + j) : 0.f;
  }
  if (p.acc) {
    int32_t* dst = p.acc + (size_t)row * p.N + n0;
    if (full && p.acc_vec) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<int4*>(dst + j) =
            make_int4((int)r[j], (int)r[j + 1], (int)r[j + 2], (int)r[j + 3]);
    } else {
      for (int j = 0; j < 32 && n0 + j < p.N; ++j) dst[j] = (int)r[j];
    }
  }
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j)
    v[j] = __fmul_rn(__fmul_rn(__int2float_rn((int)r[j]), sb[j]), sa);
  if (p.out_dtype == QGEMM_BF16) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldc + n0;
    if (full && p.out_vec) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 pk;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[j], v[j + 1]);
        __nv_bfloat162 h1 = __floats2bfloat162_rn(v[j + 2], v[j + 3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[j + 4], v[j + 5]);
        __nv_bfloat162 h3 = __floats2bfloat162_rn(v[j + 6], v[j + 7]);
        pk.x = *reinterpret_cast<uint32_t*>(&h0);
        pk.y = *reinterpret_cast<uint32_t*>(&h1);
        pk.z = *reinterpret_cast<uint32_t*>(&h2);
        pk.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(dst + j) = pk;
      }
    } else {
      for (int j = 0; j < 32 && n0 + j < p.N; ++j) dst[j] = __float2bfloat16_rn(v[j]);
    }
  } else {
    float* dst = reinterpret_cast<float*>(p.out) + (size_t)row * p.ldc + n0;
    if (full && p.out_vec) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
      for (int j = 0; j < 32 && n0 + j < p.N; ++j) dst[j] = v[j];
    }
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    w8a8_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment: required by the 128-byte swizzle pattern of TMA and UMMA.
  const uint32_t raw_base = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);

  const uint32_t bar_base = base + STAGES * STAGE_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * STAGES + 4);
  uint8_t* gbar = gbase + STAGES * STAGE_BYTES;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbar + 8 * (2 * STAGES + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbar + 8 * (2 * STAGES + 5) + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(tfull_bar(a), 1);
      ptx::mbar_init(tempty_bar(a), 128);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(const_cast<uint32_t*>(tmem_slot)), TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!ptx::mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) {
            if (!*abort_flag) report(p.err, DEVERR_TIMEOUT_PRODUCER, abort_flag);
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
          ptx::mbar_arrive_expect_tx(full_bar(stage), STAGE_BYTES);
          ptx::tma_load_2d(sa, &tmA, full_bar(stage), kb * BK, mb * BM);
          if (p.b_kn) {
            ptx::tma_load_2d(sb, &tmB, full_bar(stage), nb * BN, kb * BK);
            ptx::tma_load_2d(sb + B_BYTES / 2, &tmB, full_bar(stage), nb * BN + 128, kb * BK);
          } else {
            ptx::tma_load_2d(sb, &tmB, full_bar(stage), kb * BK, nb * BN);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: every copy this thread issued must land before the CTA exits.
      for (long long f = (issued > STAGES ? issued - STAGES : 0); f < issued; ++f) {
        const int s = (int)(f % STAGES);
        const uint32_t par = (uint32_t)((f / STAGES) & 1);
        if (!ptx::mbar_wait(full_bar(s), par, nullptr)) {
          report(p.err, DEVERR_TIMEOUT_DRAIN, abort_flag);
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_i8(BM, BN, false, p.b_kn != 0);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
        const int a = it & 1;
        const uint32_t aphase = (uint32_t)((it >> 1) & 1);
        if (!ptx::mbar_wait(tempty_bar(a), aphase ^ 1u, abort_flag)) {
          if (!*abort_flag) report(p.err, DEVERR_TIMEOUT_MMA, abort_flag);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(a * BN);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!ptx::mbar_wait(full_bar(stage), phase, abort_flag)) {
            if (!*abort_flag) report(p.err, DEVERR_TIMEOUT_MMA, abort_flag);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sa = base + stage * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            // A: K-major, 128-byte rows, 8-row core groups 1024 B apart; step K by
            // moving the start address 32 B inside the swizzle row.
            const uint64_t adesc = ptx::smem_desc_sw128(sa + kk * UMMA_K, 16, 1024);
            uint64_t bdesc;
            if (p.b_kn) {
              // B: MN-major; 128 N-bytes per row, 8 K-rows per 1024-B group (SBO),
              // second 128-column half 16 KB away (LBO); K step = 32 rows = 4 KB.
              bdesc = ptx::smem_desc_sw128(sb + kk * UMMA_K * 128, B_BYTES / 2, 1024);
            } else {
              bdesc = ptx::smem_desc_sw128(sb + kk * UMMA_K, 16, 1024);
            }
            ptx::umma_i8(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          ptx::umma_commit(empty_bar(stage));
          issued_any = true;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) ptx::umma_commit(tfull_bar(a));
      }
      if (!ok && issued_any) {
        // Wait for the MMAs already issued before TMEM is released.
        ptx::umma_commit(drain_bar);
        if (!ptx::mbar_wait(drain_bar, 0, nullptr)) report(p.err, DEVERR_TIMEOUT_DRAIN, abort_flag);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int a = it & 1;
      const uint32_t aphase = (uint32_t)((it >> 1) & 1);
      if (!ptx::mbar_wait(tfull_bar(a), aphase, abort_flag)) {
        if (!*abort_flag) report(p.err, DEVERR_TIMEOUT_EPILOGUE, abort_flag);
        break;
      }
      ptx::tc_fence_after();
      const int row = mb * BM + q * 32 + lane;
      const float sa = (row < p.M) ? __ldg(p.sA + row) : 0.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        const uint32_t taddr =
            tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN + c * 32);
        __syncwarp();
        ptx::tmem_ld_32x32b_x32(taddr, r);
        ptx::tmem_wait_ld();
        store_chunk(p, row, nb * BN + c * 32, sa, r);
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(tempty_bar(a));
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---- host side -------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static bool make_map_u8(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer,
                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace w8a8

bool w8a8_tcgen05_supported(const qgemm_device_s* d, uint64_t A, uint64_t B, int b_kn,
                            uint64_t out, int out_dtype, int ldc, int M, int N, int K,
                            const char** why) {
  auto no = [&](const char* w) { if (why) *why = w; return false; };
  if (!d->tcgen05) return no("device is not sm_100 (tcgen05 unavailable)");
  if (d->smem_optin < (size_t)w8a8::SMEM_BYTES) return no("not enough shared memory per block");
  if (M <= 0 || N <= 0 || K <= 0) return no("empty shape");
  if (K % 16 != 0) return no("K must be a multiple of 16 (TMA row stride)");
  if (b_kn && N % 16 != 0) return no("N must be a multiple of 16 for the [K,N] B layout");
  if (!aligned(A, 16) || !aligned(B, 16)) return no("A and B must be 16-byte aligned");
  (void)out; (void)out_dtype; (void)ldc;
  return true;
}

qgemm_status launch_w8a8_tcgen05(qgemm_stream_s* s, const void* A, const void* B, int b_kn,
                                 const float* sA, const float* sB, void* out, int out_dtype,
                                 int ldc, int M, int N, int K, int32_t* acc) {
  using namespace w8a8;
  CUtensorMap tmA, tmB;
  if (!make_map_u8(&tmA, A, (uint64_t)K, (uint64_t)M, (uint64_t)K, BK, BM))
    return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for A [%d,%d]", M, K);
  bool okb = b_kn ? make_map_u8(&tmB, B, (uint64_t)N, (uint64_t)K, (uint64_t)N, 128, BK)
                  : make_map_u8(&tmB, B, (uint64_t)K, (uint64_t)N, (uint64_t)K, BK, BN);
  if (!okb) return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for B");

  Params p;
  p.M = M; p.N = N; p.K = K; p.ldc = ldc;
  p.out_dtype = out_dtype;
  p.b_kn = b_kn;
  p.num_m_blocks = (M + BM - 1) / BM;
  p.num_n_blocks = (N + BN - 1) / BN;
  p.num_k_blocks = (K + BK - 1) / BK;
  p.num_tiles = p.num_m_blocks * p.num_n_blocks;
  p.sA = sA; p.sB = sB; p.out = out; p.acc = acc;
  p.err = s->dev->d_err;
  const int esize = out_dtype == QGEMM_BF16 ? 2 : 4;
  p.out_vec = aligned((uint64_t)out, 16) && ((uint64_t)ldc * esize) % 16 == 0;
  p.acc_vec = acc != nullptr && aligned((uint64_t)acc, 16) && N % 4 == 0;

  static bool attr_set[64] = {false};
  const int ord = s->dev->ordinal;
  if (ord >= 0 && ord < 64 && !attr_set[ord]) {
    cudaError_t e = cudaFuncSetAttribute(w8a8_tcgen05_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w8a8_tcgen05)");
    attr_set[ord] = true;
  }
  const int grid = p.num_tiles < s->dev->sm_count ? p.num_tiles : s->dev->sm_count;
  w8a8_tcgen05_kernel<<<grid, NUM_THREADS, SMEM_BYTES, s->stream>>>(tmA, tmB, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "w8a8_tcgen05_kernel launch");
  return QGEMM_OK;
}

}  // namespace qg
