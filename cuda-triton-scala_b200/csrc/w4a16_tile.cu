// w4a16_tile.cu -- W4A16 decode GEMV / skinny GEMM on prepacked weight tiles.
//
// Arithmetic (QuantizedGemmOps.scala:229-245 generalised to groups and a zero point):
//     y[m,n] = sum_g s[g,n] * sum_{k in g} (q[k,n] - zp) * x[m,k]
//
// Weight layout ("tiled", made once by qgemm_prepack_w4_tiled): the reference rows
// (nibble order of QuantizedGemmOps.scala:234-238, 8 columns per little-endian word)
// cut into 64-column tiles, each tile's K rows stored contiguously:
//     tiled[tile][k][0..31] = bytes [32*tile, 32*tile + 32) of reference row k
// so a CTA that owns a tile streams one contiguous block of memory.
//
// One CTA per (tile, k-split), two per SM.  Warp 8 is the producer: per stage a 1-D
// bulk copy of 512 weight rows (16 KB), a TMA tile of the stage's scales and two TMA
// tiles of the activations, into a shared-memory ring.  Warps 0-7 each take 64 rows
// of the stage: per 16-row chunk, prmt pairs two rows' nibbles and lop3 with the bf16
// bias 128 gives the exact value 128+q; mma.m16n8k16 (bf16 in, fp32 accumulate)
// multiplies 16 columns x 16 k of (128+q) by up to 8 activation rows, and one more
// MMA with an all-ones A gives sum_k x.  Once per group the fp32 partial is corrected,
// P - (128+zp) * sum_k x = sum_k (q - zp) x, and multiplied by the per-column scale.
// At the end the eight warps' partials are summed in shared memory and, when K is
// split over a cluster,
// across the cluster's CTAs through distributed shared memory (fixed order, so the
// result is deterministic).  No global workspace, no atomics.  The only waits are the
// bounded mbarrier waits of the ring.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace qg {
namespace w4x {

constexpr int TW = 64;                  // tile width in columns (32 bytes of a weight row)
constexpr int TWB = TW / 2;             // bytes of a tile row
constexpr int NCW = 8;                  // consumer warps
constexpr int THREADS = 32 * (NCW + 1);
constexpr int SR = 512;                 // weight rows per stage (64 per consumer warp)
constexpr int WR = SR / NCW;            // rows per consumer warp per stage
constexpr int W_BYTES = SR * TWB;       // 16 KB
constexpr int S_BYTES = 32 * TW * 2;    // up to 32 scale rows (group >= 16) x 64 columns
constexpr int MAX_KS = 8;

// MT = 1, 2: two CTAs per SM.  MT = 4 (32 activation rows): one CTA per SM, whose
// register file holds the 4x accumulators; the weights are streamed once for 32 rows
// instead of twice for two 16-row passes.  Measured on B200 (M = 32): 1.86x faster when
// the 16-row grid would leave SMs idle (N=4096, K=11008: 27.5 against 51.2 us), ~2 %
// slower when it already covers every SM (N=14336, K=4096: 38.7 against 37.8 us).
template <int MT>
struct Cfg {
  static constexpr int MR = 8 * MT;
  static constexpr int STAGES = MT == 2 ? 2 : 3;
  static constexpr int CTAS_PER_SM = MT == 4 ? 1 : 2;
  static constexpr int X_BYTES = SR * MR * 2;
  static constexpr int STAGE_BYTES = W_BYTES + S_BYTES + X_BYTES;
  static constexpr int RED_BYTES = NCW * MR * TW * 4;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES + RED_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 128 + 128;
  static_assert(STAGE_BYTES % 128 == 0, "stage alignment");
};

struct Params {
  int M, N, K, G, zp;
  int m0, mrows;      // activation rows of this pass
  int KS;             // k-split (cluster size)
  int kc;             // weight rows per CTA (a multiple of SR; the last CTA's share may
                      // run past K)
  int pdl;
  const uint8_t* wt;  // tiled weights
  __nv_bfloat16* y;
  int* err;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t mask, uint32_t bias) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(bias));
  return r;
}

__device__ __forceinline__ uint32_t bf162_sub(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a),
                             *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16_z(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                           uint32_t a3, uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

template <int MT>
__global__ void __launch_bounds__(THREADS, Cfg<MT>::CTAS_PER_SM)
    w4a16_tile_kernel(const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmX,
                      const Params p) {
  using C = Cfg<MT>;
  constexpr int MR = C::MR, STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw + 127u) & ~127u;
  uint8_t* gbase = smem_raw + (base - raw);
  float* red = reinterpret_cast<float*>(gbase + STAGES * C::STAGE_BYTES);  // [NCW][MR][TW]
  const uint32_t bar = base + C::BAR_OFF;
  auto full_bar = [&](int s) { return bar + 8u * s; };
  auto empty_bar = [&](int s) { return bar + 8u * (STAGES + s); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + C::BAR_OFF + 64);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = blockIdx.x;          // k-split index == rank in the cluster
  const int tile = blockIdx.y;
  const int kbeg = ks * p.kc;
  const int krows = (p.K - kbeg) < p.kc ? (p.K - kbeg) : p.kc;  // rows of K this CTA owns
  const int nstages = krows > 0 ? (krows + SR - 1) / SR : 0;
  const int gpr = SR / p.G > 0 ? SR / p.G : 1;  // scale rows per stage

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), NCW);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::grid_launch_dependents();
  }
  __syncthreads();

  // The last stage of a CTA may hold fewer than SR rows: only those are copied.  The
  // rest of the stage keeps older bytes, which dequantise to finite values and meet
  // activations that TMA zero-fills past K, so they add exactly zero.
  const uint32_t sx_bytes = (uint32_t)(gpr * TW * 2 + 2 * (SR / 2) * MR * 2);
  auto wbytes = [&](int i) {
    const int rows = krows - i * SR;
    return (uint32_t)((rows < SR ? rows : SR) * TWB);
  };

  if (warp == NCW) {
    // ---------------- producer ----------------
    if (lane == 0) {
      ptx::prefetch_tmap(&tmS);
      ptx::prefetch_tmap(&tmX);
      const uint8_t* wsrc = p.wt + ((size_t)tile * p.K + kbeg) * TWB;
      const int pre = nstages < STAGES ? nstages : STAGES;
      // Weights and scales do not depend on the previous kernel; activations do.
      for (int i = 0; i < pre; ++i) {
        const uint32_t sw = base + i * C::STAGE_BYTES;
        const int k0 = kbeg + i * SR;
        ptx::mbar_arrive_expect_tx(full_bar(i), wbytes(i) + sx_bytes);
        ptx::bulk_load(sw, wsrc + (size_t)i * W_BYTES, wbytes(i), full_bar(i));
        ptx::tma_load_2d(sw + W_BYTES, &tmS, full_bar(i), tile * TW, k0 / p.G);
      }
      if (p.pdl) ptx::grid_dependency_wait();
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      for (int i = 0; i < nstages; ++i) {
        const uint32_t sw = base + stage * C::STAGE_BYTES;
        const int k0 = kbeg + i * SR;
        if (i >= pre) {
          if (!ptx::mbar_wait_sleep(empty_bar(stage), phase ^ 1u, abort_flag)) {
            if (!*abort_flag) { *abort_flag = 1; if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_PRODUCER); }
            break;
          }
          ptx::mbar_arrive_expect_tx(full_bar(stage), wbytes(i) + sx_bytes);
          ptx::bulk_load(sw, wsrc + (size_t)i * W_BYTES, wbytes(i), full_bar(stage));
          ptx::tma_load_2d(sw + W_BYTES, &tmS, full_bar(stage), tile * TW, k0 / p.G);
        }
        const uint32_t sx = sw + W_BYTES + S_BYTES;
        ptx::tma_load_2d(sx, &tmX, full_bar(stage), k0, p.m0);
        ptx::tma_load_2d(sx + (SR / 2) * MR * 2, &tmX, full_bar(stage), k0 + SR / 2, p.m0);
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      if (issued < pre) issued = pre;
      for (long long f = (issued > STAGES ? issued - STAGES : 0); f < issued; ++f) {
        if (!ptx::mbar_wait(full_bar((int)(f % STAGES)), (uint32_t)((f / STAGES) & 1), nullptr)) {
          if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_DRAIN);
          break;
        }
      }
    }
  } else {
    // ---------------- consumers ----------------
    const int g = lane >> 2, t = lane & 3;
    const float zc = 128.0f + (float)p.zp;
    const uint32_t MASK = 0x000F000Fu, BIAS = 0x43004300u, ONES = 0x3F803F80u;
    const int cpg = p.G < WR ? p.G / 16 : WR / 16;  // chunks per scale application
    if (p.pdl) ptx::grid_dependency_wait();

    float acc[4][MT][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][mt][e] = 0.f;

    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < nstages; ++i) {
      const bool ok = ptx::mbar_wait_sleep(full_bar(stage), phase, abort_flag);
      if (!ok && !*abort_flag) { *abort_flag = 1; if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_EPILOGUE); }
      if (ok) {
        const uint8_t* sw = gbase + stage * C::STAGE_BYTES;
        const uint8_t* ss = sw + W_BYTES;
        // this warp's activations: rows [WR*warp, WR*warp + WR) of the stage live in
        // the first (warps 0-3) or second (warps 4-7) 256-row TMA tile
        const uint8_t* xs = sw + W_BYTES + S_BYTES + (warp >> 2) * (SR / 2) * MR * 2;
        const int xk0 = (warp & 3) * WR;
        float part[4][MT][4], sx[MT][4];
#pragma unroll
        for (int c = 0; c < WR / 16; ++c) {
          const int r0 = WR * warp + 16 * c;
          const uint8_t* wp = sw + (r0 + 2 * t) * TWB + 4 * g;
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(wp);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(wp + TWB);
          const uint32_t w8 = *reinterpret_cast<const uint32_t*>(wp + 8 * TWB);
          const uint32_t w9 = *reinterpret_cast<const uint32_t*>(wp + 9 * TWB);
          uint32_t bfr[MT][2];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint8_t* xr = xs + ((mt * 8 + g) * (SR / 2) + xk0 + 16 * c + 2 * t) * 2;
            bfr[mt][0] = *reinterpret_cast<const uint32_t*>(xr);       // k, k+1
            bfr[mt][1] = *reinterpret_cast<const uint32_t*>(xr + 16);  // k+8, k+9
          }
          const uint32_t lo01 = prmt(w0, w1, 0x5410), hi01 = prmt(w0, w1, 0x7632);
          const uint32_t lo89 = prmt(w8, w9, 0x5410), hi89 = prmt(w8, w9, 0x7632);
          const bool first = (c % cpg) == 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t a0 = and_or(lo01 >> (4 * q), MASK, BIAS);
            const uint32_t a1 = and_or(hi01 >> (4 * q), MASK, BIAS);
            const uint32_t a2 = and_or(lo89 >> (4 * q), MASK, BIAS);
            const uint32_t a3 = and_or(hi89 >> (4 * q), MASK, BIAS);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              if (first) mma_bf16_z(part[q][mt], a0, a1, a2, a3, bfr[mt][0], bfr[mt][1]);
              else       mma_bf16(part[q][mt], a0, a1, a2, a3, bfr[mt][0], bfr[mt][1]);
            }
          }
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            if (first) mma_bf16_z(sx[mt], ONES, ONES, ONES, ONES, bfr[mt][0], bfr[mt][1]);
            else       mma_bf16(sx[mt], ONES, ONES, ONES, ONES, bfr[mt][0], bfr[mt][1]);
          }
          if ((c % cpg) == cpg - 1) {
            // scale row of this group; this thread's 8 columns are 8g .. 8g+7
            const int sr = (WR * warp + 16 * c) / p.G;
            const uint4 sv = *reinterpret_cast<const uint4*>(ss + (sr * TW + 8 * g) * 2);
            const uint32_t s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              // column 8g+q (rows of MMA q) and 8g+q+4
              const float sa = (q & 1) ? bf16_hi(s4[q >> 1]) : bf16_lo(s4[q >> 1]);
              const float sb = (q & 1) ? bf16_hi(s4[2 + (q >> 1)]) : bf16_lo(s4[2 + (q >> 1)]);
#pragma unroll
              for (int mt = 0; mt < MT; ++mt) {
                acc[q][mt][0] = fmaf(sa, fmaf(-zc, sx[mt][0], part[q][mt][0]), acc[q][mt][0]);
                acc[q][mt][1] = fmaf(sa, fmaf(-zc, sx[mt][1], part[q][mt][1]), acc[q][mt][1]);
                acc[q][mt][2] = fmaf(sb, fmaf(-zc, sx[mt][2], part[q][mt][2]), acc[q][mt][2]);
                acc[q][mt][3] = fmaf(sb, fmaf(-zc, sx[mt][3], part[q][mt][3]), acc[q][mt][3]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(empty_bar(stage));
      if (++stage == STAGES) { stage = 0; phase ^= 1u; }
    }
    // partials of this warp -> red[warp][m][col]
    float* rw = red + warp * MR * TW;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int ca = 8 * g + q, cbb = ca + 4;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int m = mt * 8 + 2 * t;
        rw[m * TW + ca] = acc[q][mt][0];
        rw[(m + 1) * TW + ca] = acc[q][mt][1];
        rw[m * TW + cbb] = acc[q][mt][2];
        rw[(m + 1) * TW + cbb] = acc[q][mt][3];
      }
    }
  }
  __syncthreads();
  // sum the four warps (fixed order) into red[0]
  for (int idx = threadIdx.x; idx < MR * TW; idx += THREADS) {
    float s = red[idx];
#pragma unroll
    for (int w = 1; w < NCW; ++w) s += red[w * MR * TW + idx];
    red[idx] = s;
  }
  if (p.KS > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    // CTA r of the cluster finishes columns [r*TW/KS, (r+1)*TW/KS), summing ranks in order
    const int cw = TW / p.KS;
    for (int idx = threadIdx.x; idx < p.mrows * cw; idx += THREADS) {
      const int m = idx / cw, col = ks * cw + idx % cw;
      float s = 0.f;
      for (int r = 0; r < p.KS; ++r) s += cluster.map_shared_rank(red, r)[m * TW + col];
      const int n = tile * TW + col;
      if (n < p.N) p.y[(size_t)(p.m0 + m) * p.N + n] = __float2bfloat16_rn(s);
    }
    cluster.sync();  // peers' shared memory stays alive until everyone has read it
  } else {
    __syncthreads();
    for (int idx = threadIdx.x; idx < p.mrows * TW; idx += THREADS) {
      const int m = idx / TW, col = idx % TW;
      const int n = tile * TW + col;
      if (n < p.N) p.y[(size_t)(p.m0 + m) * p.N + n] = __float2bfloat16_rn(red[m * TW + col]);
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

static bool map_bf16_2d(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer,
                        uint64_t stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
             es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// k-split for a tile count: the smallest of 1, 2, 4, 8 that fills the SMs, as long as
// each CTA still gets whole 512-row stages.
static int choose_ks(int ntiles, int K, int sms) {
  int ks = 1;
  while (ks < MAX_KS && ntiles * ks < sms && (K % (SR * ks * 2)) == 0) ks *= 2;
  return ks;
}

}  // namespace w4x

bool w4a16_tile_supported(const qgemm_device_s* d, uint64_t x, uint64_t wt, uint64_t sc, int M,
                          int N, int K, int G, const char** why) {
  auto no = [&](const char* w) { if (why) *why = w; return false; };
  if (!d->tcgen05) return no("device is not sm_100");
  const int smem = M > 16 ? w4x::Cfg<4>::SMEM_BYTES  // the larger of the M > 16 configs
                 : M > 8 ? w4x::Cfg<2>::SMEM_BYTES : w4x::Cfg<1>::SMEM_BYTES;
  if (d->smem_optin < (size_t)smem) return no("not enough shared memory per block");
  if (K % 16 != 0) return no("K must be a multiple of 16");
  // every 512-row stage starts on a group boundary and every 16-row chunk lies in
  // one group
  if (G % 16 != 0 || !(w4x::SR % G == 0 || G % w4x::SR == 0))
    return no("group_size must be a multiple of 16 that divides 512 or a multiple of 512");
  if (N % 8 != 0) return no("N must be a multiple of 8");
  if (!aligned(x, 16) || !aligned(wt, 16) || !aligned(sc, 16))
    return no("x, weights and scales must be 16-byte aligned");
  return true;
}

size_t w4_tiled_bytes(int K, int N) {
  return (size_t)((N + w4x::TW - 1) / w4x::TW) * (size_t)K * w4x::TWB;
}

qgemm_status launch_w4a16_tile(qgemm_stream_s* s, const void* x, const uint8_t* wt,
                               const void* sc, int zp, int G, void* y, int M, int N, int K) {
  using namespace w4x;
  qgemm_device_s* d = s->dev;
  const int ntiles0 = (N + TW - 1) / TW;
  const int Kr0 = (K + SR - 1) / SR * SR;
  // MT = 4 for M > 16 when the 16-row grid has no more CTAs than SMs
  const bool wide = M > 16 && ntiles0 * choose_ks(ntiles0, Kr0, d->sm_count) <= d->sm_count;
  const int mti = wide ? 2 : M > 8 ? 1 : 0;  // MT = 4, 2, 1
  const int MR = 8 << mti;
  const int smem = mti == 2 ? Cfg<4>::SMEM_BYTES : mti == 1 ? Cfg<2>::SMEM_BYTES : Cfg<1>::SMEM_BYTES;
  const int ntiles = (N + TW - 1) / TW;
  Params p;
  p.M = M; p.N = N; p.K = K; p.G = G; p.zp = zp;
  const int Kr = (K + SR - 1) / SR * SR;  // K rounded up to whole stages
  p.KS = choose_ks(ntiles, Kr, d->sm_count);
  p.kc = Kr / p.KS;
  p.pdl = 1;
  p.wt = wt;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.err = d->d_err;

  CUtensorMap tmS, tmX;
  const int gpr = SR / G > 0 ? SR / G : 1;
  if (!map_bf16_2d(&tmS, sc, (uint64_t)N, (uint64_t)(K / G), (uint64_t)N * 2, TW, (uint32_t)gpr) ||
      !map_bf16_2d(&tmX, x, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, SR / 2, (uint32_t)MR))
    return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for the W4A16 operands");

  void (*kern)(const CUtensorMap, const CUtensorMap, const Params) =
      mti == 2 ? w4a16_tile_kernel<4> : mti == 1 ? w4a16_tile_kernel<2> : w4a16_tile_kernel<1>;
  static bool attr_done[64][3] = {};
  const int ord = d->ordinal;
  if (ord >= 0 && ord < 64 && !attr_done[ord][mti]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a16_tile)");
    attr_done[ord][mti] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.KS, ntiles, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = p.KS;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  for (int m0 = 0; m0 < M; m0 += MR) {
    p.m0 = m0;
    p.mrows = (M - m0) < MR ? (M - m0) : MR;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmS, tmX, p);
    if (e != cudaSuccess) return cuda_fail(e, "w4a16_tile_kernel launch");
  }
  return QGEMM_OK;
}

// ---- one-time weight repack: reference rows -> 64-column tiles -----------------
// dst[tile][k][j] = src_row_k[32*tile + j] (bytes), zero past the last column.
__global__ void prepack_w4_tiled_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                        int K, int N, int vec) {
  const size_t row_bytes = (size_t)N / 2;
  const int ntiles = (N + w4x::TW - 1) / w4x::TW;
  const size_t total16 = (size_t)ntiles * K * (w4x::TWB / 16);  // 16-byte pieces
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total16;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t piece = i % (w4x::TWB / 16), row = i / (w4x::TWB / 16);  // row = tile*K + k
    const size_t tile = row / K, k = row - tile * K;
    const size_t off = tile * w4x::TWB + piece * 16;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (vec && off + 16 <= row_bytes) {
      v = *reinterpret_cast<const uint4*>(src + k * row_bytes + off);
    } else {
      uint8_t b[16] = {};
      for (int j = 0; j < 16; ++j)
        if (off + j < row_bytes) b[j] = src[k * row_bytes + off + j];
      memcpy(&v, b, 16);
    }
    reinterpret_cast<uint4*>(dst)[i] = v;
  }
}

qgemm_status launch_prepack_w4_tiled(qgemm_stream_s* s, const uint32_t* src, uint8_t* dst, int K,
                                     int N) {
  const bool vec_ok = aligned((uint64_t)src, 16) && ((size_t)N / 2) % 16 == 0;
  const int grid = s->dev->sm_count * 8;
  prepack_w4_tiled_kernel<<<grid, 256, 0, s->stream>>>(reinterpret_cast<const uint8_t*>(src), dst,
                                                       K, N, vec_ok ? 1 : 0);
  return cuda_fail(cudaGetLastError(), "prepack_w4_tiled launch");
}

}  // namespace qg
