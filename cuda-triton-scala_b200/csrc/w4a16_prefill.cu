// w4a16_prefill.cu -- group-wise W4A16 GEMM for prefill-sized M.
//
// Arithmetic (QuantizedGemmOps.scala:229-245 generalised to groups and a zero point):
//     y[m,n] = sum_k x[m,k] * w[k,n],   w[k,n] = (q[k,n] - zp) * s[k/G, n]
//
// When M is large every weight is used by many rows, so the weights are expanded once
// per call instead of once per output tile: a slab of columns is dequantised into a
// bf16 buffer (K-major, the B operand layout of the tensor-core GEMM), then the bf16
// tcgen05 GEMM (the kernels of w8a8_tcgen05.cu in bf16 mode) multiplies the
// activations by it, and the next slab follows.
//
// Exactness: w = (q - zp) * s has up to 12 significant bits (a 4-bit integer times an
// 8-bit bf16 significand), more than bf16 holds.  Two expansions:
//   * exact (two terms, the default): each weight is written as two bf16 values,
//     hi = bf16(w) and lo = w - hi (exact: at most 4 bits remain), in two K-blocks of
//     the same slab row, and the GEMM reads the activations twice along K:
//         y = x * hi^T + x * lo^T,  with exact products and fp32 sums,
//     so the only roundings are those of the fp32 accumulation and of the bf16 output,
//     as on the decode path.  This doubles the tensor work.
//   * one term: the slab holds hi = bf16(w) alone (round to nearest even, relative
//     error at most 2^-9 per weight) and the GEMM runs once over K: the algorithmic
//     tensor work, half the workspace, and a relative output error of about 2^-9 / 2
//     on average against the exact sum.
//   * integer (the exact form when group_size % 64 == 0): the slab holds q - zp as bf16
//     (exact), and the group-scaled multiply (w4a16_prefill_gs.cu) applies s[g, n] in
//     fp32 to each group's tensor-core partial sums: exact products and fp32 sums with
//     one pass over K, and no rounding of the scaled weight.
// The expansion costs 2.5 (one term, integer) or 4.5 bytes of HBM traffic per weight
// against 4 * M multiply-adds.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "internal.h"

namespace qg {
namespace w4p {

constexpr int TW = 64;    // columns per tile of the tiled int4 layout
constexpr int TWB = 32;   // bytes of a tile row
constexpr int KR = 128;   // weight rows per CTA
constexpr int PAD = 8;    // bf16 padding per transposed row (keeps rows 16-byte aligned)

// MODE: 0 = q - zp (exact, no scale), 1 = bf16((q - zp) * s), 2 = hi + lo.
template <int MODE> struct SlabMode {
  static constexpr int TERMS = MODE == 2 ? 2 : 1;  // bf16 values per weight in the slab
};
__device__ __forceinline__ float slab_value(int mode, float q, float zp, float sc) {
  return mode == 0 ? q - zp : (q - zp) * sc;  // exact in fp32
}

// One CTA: one 64-column tile x 128 rows of the tiled weights -> rows n of the slab,
// dst[n - n0][k] = hi (or q - zp) and, with MODE = 2, dst[n - n0][Kp + k] = lo (bf16,
// row pitch TERMS * Kp, Kp = K rounded up to 64, zeros in between).  Thread t
// dequantises half a row (32 columns, one 16-byte load) into the transposed shared
// tiles; then each warp writes eight slab rows, 256 bytes of each term.
template <int MODE>
__global__ void __launch_bounds__(256) dequant_slab_kernel(
    const uint8_t* __restrict__ wt, const __nv_bfloat16* __restrict__ scales, int zp, int G,
    __nv_bfloat16* __restrict__ dst, int K, int Kp, int N, int n0, int ncols) {
  constexpr int TERMS = SlabMode<MODE>::TERMS;
  __shared__ __align__(16) __nv_bfloat16 tr[2][TW][KR + PAD];  // 34.8 KB
  const int tile = n0 / TW + blockIdx.x;
  const int k0 = blockIdx.y * KR;
  const int r = threadIdx.x & (KR - 1), half = threadIdx.x >> 7;
  const int k = k0 + r;
  if (k < K) {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(wt + ((size_t)tile * K + k) * TWB) + half);
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    const __nv_bfloat16* srow = scales + (size_t)(k / G) * N + tile * TW + 32 * half;
    const float fzp = (float)zp;
#pragma unroll
    for (int j = 0; j < 4; ++j) {       // word j holds columns 8j .. 8j+7 of this half
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = 32 * half + 8 * j + e;
        float v = 0.f;
        if (tile * TW + c < N) {
          const float q = (float)((wv[j] >> (4 * e)) & 0xFu);
          v = slab_value(MODE, q, fzp, MODE == 0 ? 1.f : __bfloat162float(srow[8 * j + e]));
        }
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        tr[0][c][r] = hi;
        if (TERMS == 2) tr[1][c][r] = __float2bfloat16_rn(v - __bfloat162float(hi));  // exact
      }
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = lane >> 4;                  // lanes 0-15 write hi, 16-31 write lo
  const int kk = 8 * (lane & 15);           // this lane's 8 elements (16 bytes)
#pragma unroll
  for (int i = 0; i < TW / 8; ++i) {
    const int c = warp * (TW / 8) + i;
    const int n = tile * TW + c - n0;       // slab row
    if (h >= TERMS || n >= ncols || k0 + kk >= Kp) continue;  // Kp % 64 == 0: whole pieces
    __nv_bfloat16* drow = dst + (size_t)n * TERMS * Kp + (size_t)h * Kp + k0 + kk;
    if (k0 + kk + 8 <= K) {
      *reinterpret_cast<uint4*>(drow) = *reinterpret_cast<const uint4*>(&tr[h][c][kk]);
    } else {  // the tail of K and the zero padding up to Kp
      for (int e = 0; e < 8; ++e)
        drow[e] = (k0 + kk + e < K) ? tr[h][c][kk + e] : __float2bfloat16_rn(0.f);
    }
  }
}

// The same expansion from the fragment order of w4a16_frag.cu (unit (c, kb) = columns
// 8c..8c+7 x rows 128kb..128kb+127, 512 bytes, c-major; lane 4g+t's word s holds
// column 8c+g at rows 128kb + 32s + 8t + {0, 4, 2, 6, 1, 5, 3, 7}, nibble i at bits
// 4i).  One CTA: 8 consecutive column groups (64 columns) x one 128-row block; thread
// 32u + lane loads that lane's 16 bytes of unit u and places its 32 weights in the
// transposed shared tiles; the write-out is the one above.
template <int MODE>
__global__ void __launch_bounds__(256) dequant_slab_frag_kernel(
    const uint4* __restrict__ wf, const __nv_bfloat16* __restrict__ scales, int zp, int G,
    __nv_bfloat16* __restrict__ dst, int K, int Kp, int N, int NKB, int n0, int ncols) {
  constexpr int TERMS = SlabMode<MODE>::TERMS;
  __shared__ __align__(16) __nv_bfloat16 tr[2][TW][KR + PAD];  // 34.8 KB
  const int col0 = n0 + blockIdx.x * TW;  // first column of this CTA (a multiple of 8)
  const int kb = blockIdx.y, k0 = kb * KR;
  const int u = threadIdx.x >> 5, ln = threadIdx.x & 31;
  const int g = ln >> 2, t = ln & 3;
  const int cg = col0 / 8 + u;            // column group
  const int c = 8 * u + g;                // column within the CTA
  const int n = col0 + c;
  const int srows = K / G;
  uint4 w = make_uint4(0u, 0u, 0u, 0u);
  if (n < N) w = __ldg(wf + ((size_t)cg * NKB + kb) * 32 + ln);
  const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
  const float fzp = (float)zp;
  const int off[8] = {0, 4, 2, 6, 1, 5, 3, 7};
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const int rb = 32 * s + 8 * t;        // this lane's 8 rows of step s: rb .. rb+7
    const int grow = (k0 + rb) / G;       // one scale group (G >= 32 and G | 32s)
    const float sc = MODE == 0 ? 1.f
                     : (n < N && k0 + rb < K && grow < srows)
                         ? __bfloat162float(scales[(size_t)grow * N + n]) : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = rb + off[i];
      float v = 0.f;
      if (n < N && k0 + r < K) v = slab_value(MODE, (float)((wv[s] >> (4 * i)) & 0xFu), fzp, sc);
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      tr[0][c][r] = hi;
      if (TERMS == 2) tr[1][c][r] = __float2bfloat16_rn(v - __bfloat162float(hi));  // exact
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = lane >> 4;                  // lanes 0-15 write hi, 16-31 write lo
  const int kk = 8 * (lane & 15);           // this lane's 8 elements (16 bytes)
#pragma unroll
  for (int i = 0; i < TW / 8; ++i) {
    const int cc = warp * (TW / 8) + i;
    const int nn = col0 + cc - n0;          // slab row
    if (h >= TERMS || nn >= ncols || k0 + kk >= Kp) continue;  // Kp % 64 == 0: whole pieces
    __nv_bfloat16* drow = dst + (size_t)nn * TERMS * Kp + (size_t)h * Kp + k0 + kk;
    if (k0 + kk + 8 <= K) {
      *reinterpret_cast<uint4*>(drow) = *reinterpret_cast<const uint4*>(&tr[h][cc][kk]);
    } else {  // the tail of K and the zero padding up to Kp
      for (int e = 0; e < 8; ++e)
        drow[e] = (k0 + kk + e < K) ? tr[h][cc][kk + e] : __float2bfloat16_rn(0.f);
    }
  }
}

}  // namespace w4p

static size_t padded_k(int K) { return ((size_t)K + 63) / 64 * 64; }

size_t w4a16_prefill_workspace_bytes(int K, int N, int terms) {
  const size_t ncols = ((size_t)N + 255) / 256 * 256;
  return ncols * padded_k(K) * 2 * (size_t)terms;  // bf16 terms per weight
}

qgemm_status launch_w4a16_prefill(qgemm_stream_s* s, const void* x, const uint8_t* wt,
                                  const void* scales, int zp, int G, void* y, int M, int N,
                                  int K, void* ws, size_t ws_bytes, bool frag, int terms) {
  using namespace w4p;
  if (terms != 1 && terms != 2) return fail(QGEMM_ERR_INVALID_ARG, "terms %d", terms);
  // The exact form: integer slab + group-scaled multiply where the group size and the
  // scales' alignment allow it, hi + lo otherwise.
  const bool gs = terms == 2 && w4a16_gs_supported(s->dev, G, (uint64_t)scales);
  const int mode = gs ? 0 : terms;
  const int slab_terms = mode == 2 ? 2 : 1;
  // slab width: as many columns as the workspace holds, a multiple of 256 (so that
  // every slab but the last fills whole 256-column GEMM tiles)
  const size_t Kp = padded_k(K);
  const size_t row_bytes = Kp * 2 * (size_t)slab_terms;
  size_t cols = ws_bytes / row_bytes;
  cols = cols / 256 * 256;
  if (cols == 0) {
    if ((size_t)N * row_bytes <= ws_bytes) cols = (size_t)N;
    else return fail(QGEMM_ERR_INVALID_ARG,
                     "workspace of %zu bytes is smaller than one 256-column slab (%zu bytes)",
                     ws_bytes, (size_t)256 * row_bytes);
  }
  __nv_bfloat16* slab = static_cast<__nv_bfloat16*>(ws);
  for (size_t n0 = 0; n0 < (size_t)N; n0 += cols) {
    const int ncols = (int)(((size_t)N - n0) < cols ? ((size_t)N - n0) : cols);
    dim3 grid2((ncols + TW - 1) / TW, (unsigned)((Kp + KR - 1) / KR));
    const uint4* wf = reinterpret_cast<const uint4*>(wt);
    const __nv_bfloat16* sc = static_cast<const __nv_bfloat16*>(scales);
    const int nkb = (K + KR - 1) / KR;
    // frag: Kp rounds K up to 64, the layout to 128: the grid's blocks are the layout's
    if (frag) {
      if (mode == 0)
        dequant_slab_frag_kernel<0><<<grid2, 256, 0, s->stream>>>(wf, sc, zp, G, slab, K,
                                                                    (int)Kp, N, nkb, (int)n0, ncols);
      else if (mode == 1)
        dequant_slab_frag_kernel<1><<<grid2, 256, 0, s->stream>>>(wf, sc, zp, G, slab, K,
                                                                    (int)Kp, N, nkb, (int)n0, ncols);
      else
        dequant_slab_frag_kernel<2><<<grid2, 256, 0, s->stream>>>(wf, sc, zp, G, slab, K,
                                                                    (int)Kp, N, nkb, (int)n0, ncols);
    } else {
      if (mode == 0)
        dequant_slab_kernel<0><<<grid2, 256, 0, s->stream>>>(wt, sc, zp, G, slab, K, (int)Kp, N,
                                                               (int)n0, ncols);
      else if (mode == 1)
        dequant_slab_kernel<1><<<grid2, 256, 0, s->stream>>>(wt, sc, zp, G, slab, K, (int)Kp, N,
                                                               (int)n0, ncols);
      else
        dequant_slab_kernel<2><<<grid2, 256, 0, s->stream>>>(wt, sc, zp, G, slab, K, (int)Kp, N,
                                                               (int)n0, ncols);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "dequant_slab launch");
    if (gs) {
      // y[:, n0 .. n0+ncols) = sum_g s[g, n] * (x * slab^T over group g)
      const qgemm_status st = launch_w4a16_gs_gemm(s, x, slab, row_bytes, sc + n0, (long long)N,
                                                   G, static_cast<__nv_bfloat16*>(y) + n0, N, M,
                                                   ncols, K);
      if (st != QGEMM_OK) return st;
      continue;
    }
    // y[:, n0 .. n0+ncols) = x * slab^T over one segment (hi) or two (hi, then lo)
    TcArgs a;
    a.kind = KIND_BF16;
    a.A = x; a.B = slab;
    a.M = M; a.N = ncols; a.K = 2 * K;
    a.nseg = slab_terms;
    a.b_seg = slab_terms == 2 ? 0x2u : 0u;
    a.b_pitch = row_bytes;
    a.out = static_cast<__nv_bfloat16*>(y) + n0; a.out_dtype = QGEMM_BF16; a.ldc = N;
    const qgemm_status st = launch_tc_gemm(s, a);
    if (st != QGEMM_OK) return st;
  }
  return QGEMM_OK;
}

}  // namespace qg
