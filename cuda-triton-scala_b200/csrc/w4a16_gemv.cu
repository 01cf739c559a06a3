// w4a16_gemv.cu -- group-wise W4A16 decode GEMV / skinny GEMM (M <= 16 per pass).
//
// Arithmetic: the w4a16Gemm body (src/main/scala/cuda/dsl/operators/linalg/
// QuantizedGemmOps.scala:229-245) with a zero point and per-group scales:
//     y[m,n] = sum_g s[g,n] * sum_{k in g} (q[k,n] - zp) * x[m,k]
// Weights stay in the reference nibble order: uint32 word (k, c) holds columns
// 8c..8c+7 of row k, low nibble first (QuantizedGemmOps.scala:234-238).
//
// Kernel layout (fast path):
//  * A warp owns 128 output columns.  Thread (g = lane/4, t = lane%4) loads an
//    8-byte pair of words (16 columns) from each of the 4 rows k0+4t..k0+4t+3 of a
//    16-row chunk: coalesced 64-byte row segments.
//  * prmt pairs the nibbles of rows (0,1) and (2,3); lop3 with the bf16 bias
//    0x4300 (=128) turns a nibble into 128+q and one bf16x2 subtract yields the
//    exact (q - zp) pair.  Those registers are the A fragments of
//    mma.m16n8k16.bf16 (rows = 16 columns, k permuted identically in A and B);
//    x is the B fragment (n = up to 8 activation rows), fp32 accumulation.
//  * Per group the fp32 partial is scaled by s[g,n] in fp32 and accumulated.
//  * The K range is split across the warps of a CTA and across the CTAs of a
//    thread-block cluster; partial sums are reduced in shared memory and then
//    through distributed shared memory in a fixed order (deterministic).
// Any other shape goes to w4a16_grouped_simt (one thread per output, ascending-k
// fp32 sum with separately rounded products: the oracle's exact order).
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "internal.h"

namespace cg = cooperative_groups;

namespace qg {
namespace w4 {

constexpr int NW = 4;             // warps per CTA
constexpr int WARP_COLS = 128;    // output columns per warp (and per CTA)

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// (a & mask) | bias
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

// Dequantises the 16 columns x 2 rows held in (w_r0, w_r1) -- two words per
// row -- into 16 bf16x2 registers: out[c] = {q[r0][c] - zp, q[r1][c] - zp}.
__device__ __forceinline__ void dequant_pair(const uint2& w_r0, const uint2& w_r1,
                                             uint32_t zbias, uint32_t (&out)[16]) {
  const uint32_t MASK = 0x000F000Fu, BIAS = 0x43004300u;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const uint32_t a = j ? w_r0.y : w_r0.x;
    const uint32_t b = j ? w_r1.y : w_r1.x;
    const uint32_t lo = prmt(a, b, 0x5410);  // columns 8j+0..3 of both rows
    const uint32_t hi = prmt(a, b, 0x7632);  // columns 8j+4..7
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      out[8 * j + p] = bf162_sub(and_or(lo >> (4 * p), MASK, BIAS), zbias);
      out[8 * j + 4 + p] = bf162_sub(and_or(hi >> (4 * p), MASK, BIAS), zbias);
    }
  }
}

template <int MT, int KS>
__global__ void __launch_bounds__(NW * 32)
    w4a16_gemv_kernel(const __nv_bfloat16* __restrict__ x, const uint32_t* __restrict__ wq,
                      const __nv_bfloat16* __restrict__ scales, __nv_bfloat16* __restrict__ y,
                      int M, int N, int K, int G, int zp) {
  constexpr int MR = 8 * MT;  // activation rows per pass
  __shared__ float red[NW][MR][WARP_COLS];

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();  // k-split index (grid.x == KS)
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane >> 2, t = lane & 3;
  const int col_w = blockIdx.y * WARP_COLS;
  const int m_base = blockIdx.z * MR;
  const int NWORDS = N >> 3;
  const int word0 = (col_w >> 3) + 2 * g;  // this thread's first word in a row
  const bool cols_ok = word0 < NWORDS;     // N % 16 == 0: both words valid together

  // zero-point bias: 128 + zp as a bf16 pair
  const __nv_bfloat16 zb = __float2bfloat16_rn(128.0f + (float)zp);
  const uint32_t zbias = (uint32_t)__bfloat16_as_ushort(zb) * 0x00010001u;

  // Activation rows this thread feeds as MMA column g of each m-tile.
  const __nv_bfloat16* xrow[MT];
  bool xok[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int m = m_base + mt * 8 + g;
    xok[mt] = m < M;
    xrow[mt] = x + (size_t)(xok[mt] ? m : 0) * K;
  }

  float acc[8][MT][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][mt][e] = 0.f;

  const int NG = K / G;
  const int wi = crank * NW + warp;
  const int g_begin = (int)((long long)wi * NG / (KS * NW));
  const int g_end = (int)((long long)(wi + 1) * NG / (KS * NW));
  const int chunks = G >> 4;

  for (int gi = g_begin; gi < g_end; ++gi) {
    float part[8][MT][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) part[i][mt][e] = 0.f;

#pragma unroll 2
    for (int ch = 0; ch < chunks; ++ch) {
      const int k0 = gi * G + ch * 16 + 4 * t;
      uint2 w[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        w[r] = cols_ok ? __ldg(reinterpret_cast<const uint2*>(wq + (size_t)(k0 + r) * NWORDS + word0))
                       : make_uint2(0u, 0u);
      }
      uint32_t bfr[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint2 xv = xok[mt] ? __ldg(reinterpret_cast<const uint2*>(xrow[mt] + k0))
                                 : make_uint2(0u, 0u);
        bfr[mt][0] = xv.x;  // k0, k0+1
        bfr[mt][1] = xv.y;  // k0+2, k0+3
      }
      uint32_t d01[16], d23[16];
      dequant_pair(w[0], w[1], zbias, d01);
      dequant_pair(w[2], w[3], zbias, d23);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int ca = 8 * (i >> 2) + (i & 3), cb = ca + 4;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          mma_bf16(part[i][mt], d01[ca], d01[cb], d23[ca], d23[cb], bfr[mt][0], bfr[mt][1]);
      }
    }
    // Scale this group's partial sums: columns 16g + {ca, cb}.
    if (cols_ok) {
      const __nv_bfloat16* srow = scales + (size_t)gi * N + col_w + 16 * g;
      const uint4 s0 = __ldg(reinterpret_cast<const uint4*>(srow));
      const uint4 s1 = __ldg(reinterpret_cast<const uint4*>(srow + 8));
      const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      float sc[16];
#pragma unroll
      for (int c = 0; c < 16; ++c)
        sc[c] = __uint_as_float(((sw[c >> 1] >> (16 * (c & 1))) & 0xFFFFu) << 16);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int ca = 8 * (i >> 2) + (i & 3), cb = ca + 4;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          acc[i][mt][0] = fmaf(sc[ca], part[i][mt][0], acc[i][mt][0]);
          acc[i][mt][1] = fmaf(sc[ca], part[i][mt][1], acc[i][mt][1]);
          acc[i][mt][2] = fmaf(sc[cb], part[i][mt][2], acc[i][mt][2]);
          acc[i][mt][3] = fmaf(sc[cb], part[i][mt][3], acc[i][mt][3]);
        }
      }
    }
  }

  // Warp partials -> shared memory [warp][m][col].
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int ca = 16 * g + 8 * (i >> 2) + (i & 3), cb = ca + 4;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int m = mt * 8 + 2 * t;
      red[warp][m][ca] = acc[i][mt][0];
      red[warp][m + 1][ca] = acc[i][mt][1];
      red[warp][m][cb] = acc[i][mt][2];
      red[warp][m + 1][cb] = acc[i][mt][3];
    }
  }
  __syncthreads();
  // CTA sum over warps (fixed order) into red[0].
  for (int idx = threadIdx.x; idx < MR * WARP_COLS; idx += NW * 32) {
    const int m = idx / WARP_COLS, c = idx % WARP_COLS;
    float s = red[0][m][c];
#pragma unroll
    for (int w2 = 1; w2 < NW; ++w2) s += red[w2][m][c];
    red[0][m][c] = s;
  }
  cluster.sync();
  // Cluster sum over CTAs (rank order); CTA r finalises columns [r*CW, (r+1)*CW).
  constexpr int CW = WARP_COLS / KS;
  for (int idx = threadIdx.x; idx < MR * CW; idx += NW * 32) {
    const int m = idx / CW, c = crank * CW + idx % CW;
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < KS; ++r) {
      const float* peer = cluster.map_shared_rank(&red[0][0][0], r);
      s += peer[m * WARP_COLS + c];
    }
    const int mm = m_base + m, n = col_w + c;
    if (mm < M && n < N) y[(size_t)mm * N + n] = __float2bfloat16_rn(s);
  }
  cluster.sync();  // keep shared memory alive until every peer has read it
}

// Any shape: one thread per output, ascending k, products rounded separately --
// the same order as the oracle (and bit-identical to it).
__global__ void w4a16_grouped_simt_kernel(const __nv_bfloat16* __restrict__ x,
                                          const uint32_t* __restrict__ wq,
                                          const __nv_bfloat16* __restrict__ scales,
                                          __nv_bfloat16* __restrict__ y, int M, int N, int K,
                                          int G, int zp) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = blockIdx.y;
  if (row >= M || col >= N) return;
  const float zpf = (float)zp;
  float sum = 0.f;
  for (int k = 0; k < K; ++k) {
    const size_t idx = (size_t)k * N + col;
    const uint32_t q = (wq[idx >> 3] >> (4 * (idx & 7))) & 0xFu;
    const float wv = __fsub_rn((float)q, zpf);
    const float s = __bfloat162float(scales[(size_t)(k / G) * N + col]);
    const float xv = __bfloat162float(x[(size_t)row * K + k]);
    sum = __fadd_rn(sum, __fmul_rn(__fmul_rn(wv, s), xv));
  }
  y[(size_t)row * N + col] = __float2bfloat16_rn(sum);
}

template <int MT, int KS>
static cudaError_t launch_fast(cudaStream_t st, const __nv_bfloat16* x, const uint32_t* wq,
                               const __nv_bfloat16* sc, __nv_bfloat16* y, int M, int N, int K,
                               int G, int zp) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(KS, (N + WARP_COLS - 1) / WARP_COLS, (M + 8 * MT - 1) / (8 * MT));
  cfg.blockDim = dim3(NW * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = KS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, w4a16_gemv_kernel<MT, KS>, x, wq, sc, y, M, N, K, G, zp);
}

}  // namespace w4

qgemm_status launch_w4a16_grouped(qgemm_stream_s* s, const void* xv, const uint32_t* wq,
                                  const void* scv, int zp, int G, void* yv, int M, int N,
                                  int K) {
  using namespace w4;
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(xv);
  const __nv_bfloat16* sc = static_cast<const __nv_bfloat16*>(scv);
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(yv);
  const bool fast = s->dev->cc_major >= 9 && N % 16 == 0 && G % 16 == 0 && K % G == 0 &&
                    aligned((uint64_t)wq, 8) && aligned((uint64_t)x, 8) &&
                    aligned((uint64_t)sc, 16);
  cudaError_t e;
  if (fast) {
    const int NG = K / G;
    // k-split: 4 CTAs per cluster when there are enough groups to go around.
    const bool ks4 = NG >= 4 * NW;
    if (M <= 8)
      e = ks4 ? launch_fast<1, 4>(s->stream, x, wq, sc, y, M, N, K, G, zp)
              : launch_fast<1, 1>(s->stream, x, wq, sc, y, M, N, K, G, zp);
    else
      e = ks4 ? launch_fast<2, 4>(s->stream, x, wq, sc, y, M, N, K, G, zp)
              : launch_fast<2, 1>(s->stream, x, wq, sc, y, M, N, K, G, zp);
    if (e != cudaSuccess) return cuda_fail(e, "w4a16_gemv_kernel launch");
    return QGEMM_OK;
  }
  if (M > 65535) return fail(QGEMM_ERR_INVALID_ARG, "M too large");
  dim3 grid((N + 127) / 128, M);
  w4a16_grouped_simt_kernel<<<grid, 128, 0, s->stream>>>(x, wq, sc, y, M, N, K, G, zp);
  return cuda_fail(cudaGetLastError(), "w4a16_grouped_simt_kernel launch");
}

}  // namespace qg
