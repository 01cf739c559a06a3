// w8a8_tcgen05.cu -- W8A8 GEMM on the sm_100a tensor cores.
//
// Computes the arithmetic of QuantizedGemmOps.w8a32Gemm
// (src/main/scala/cuda/dsl/operators/linalg/QuantizedGemmOps.scala:102-113):
//     acc[m,n] = sum_k A[m,k] * B[k,n]            (int32, exact)
//     y[m,n]   = (float(acc) * sB[n]) * sA[m]      (fp32, two roundings, in order)
// with y stored as fp32 or as bf16 (round to nearest even).
//
// Two persistent kernels, 6 warps per CTA, one CTA per SM:
//   w8a8_tcgen05_pair_kernel  (M >= 256 and N >= 256) CTA pairs of a 2-CTA cluster
//       share one 256 x 256 output tile through tcgen05.mma.cta_group::2 (M=256,
//       N=256, K=32): each CTA loads half of A (128 rows) and half of B (128
//       columns) per stage, so per-SM shared-memory traffic per MMA is half that of
//       a 1-CTA 128 x 256 tile.  6-stage ring of 32 KB stages.
//   w8a8_tcgen05_kernel       1-CTA 128 x 256 tiles, 4-stage ring of 48 KB stages,
//       for shapes with fewer than 256 rows or columns.
// Warp roles in both:
//   warp 0      TMA producer: 128-byte-swizzled tiles into the shared-memory ring.
//   warp 1      allocates 512 TMEM columns (two 256-column accumulators); one
//               thread issues tcgen05.mma kind::i8 (in a pair: the even CTA only).
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (one TMEM lane = one output
//               row per thread), dequant with the two scales, 128-byte-swizzled
//               staging in shared memory, TMA bulk tensor stores of the output.
//               The two accumulators let the epilogue of tile i overlap the MMAs
//               of tile i+1.
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
constexpr int UMMA_K = 32;  // bytes of K per MMA: 32 int8, 16 bf16 or 8 tf32 values
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;                   // 16 KB
constexpr int B_BYTES = BN * BK;                   // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;     // 48 KB
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 2 * BN;                  // two accumulators
constexpr int BAR_BYTES = 256;
// Output staging for TMA stores: two 16 KB buffers of 128 rows x 128 bytes (64 bf16 or
// 32 fp32 columns), 128-byte swizzled, placed right after the operand stages.
constexpr int STG_BYTES = 2 * 128 * 128;
// The whole opt-in shared memory of an SM (227 KB): STAGES * 48 KB of tiles plus
// barriers and 1 KB of alignment slack, and headroom so that every address a
// UMMA descriptor of the last stage can reach (under either reading of the
// MN-major leading/stride offsets) stays inside this CTA's allocation.
constexpr int SMEM_BYTES = 232448;
static_assert(STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES + 1024 <= SMEM_BYTES,
              "shared memory budget");
constexpr int GROUP_M = 16;                         // tile raster: 16 m-blocks per group

// The output windows of the other ranks of a column-sharded GEMM (the fused GEMM +
// all-gather): every output chunk the epilogue stores into this GPU's output is also
// stored, by the same TMA engine from the same staging buffer, into each peer's window
// over NVLink (plain TMA stores, no multicast).  npeer = 0 in every other use.
constexpr int MAX_PEERS = 7;
struct PeerMaps {
  CUtensorMap m[MAX_PEERS];
};

struct Params {
  int M, N, K, ldc;
  int npeer;       // peer output windows in PeerMaps (0: none)
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
  int tma_store;   // the output is written with TMA bulk tensor stores (needs out_vec)
  int fp_acc;      // 1: bf16 or tf32 operands (K counted in bytes), fp32 accumulators;
                   // no scales and no int32 output, the fp32 epilogue below instead
  // K is walked in segments of seg_kblocks k-blocks (one segment for an ordinary
  // product).  K-block r of segment s reads k-block r of A's row, or k-block
  // seg_kblocks + r when bit s of a_seg is set; likewise for B with b_seg.  The product
  // is the sum over the segments.
  int seg_kblocks;
  uint32_t a_seg, b_seg;
  // fp32 epilogue (fp_acc): v = acc; v = alpha * v (ep_alpha); v = v + bias[n] (bias);
  // v = v + beta * out[m, n] (ep_beta: out is read before it is written), each step
  // rounded on its own.
  float alpha, beta;
  const float* bias;
  int ep_alpha, ep_beta;
  // When set and *skip_flag != 0 at the epilogue, no output is stored (a later kernel
  // writes the whole output instead).
  const int* skip_flag;
  // Last-wave split of the CTA-pair kernel: the first split_w tiles are done whole,
  // one per pair per round; each of the remaining tiles is cut along K into split_s
  // parts that run on different pairs at once.  A part writes its partial sums (int32,
  // or fp32 with fp_acc) to `part`; the part that counts in last on `cnt` adds them all
  // in part order (a fixed order, so the fp32 sums are deterministic too) and runs the
  // epilogue.
  int split_w, split_s;
  int32_t* part;   // [(tail tile * 2 + rank) * split_s + part][128 x 256 words, part_index]
  int* cnt;        // [tail tile * 2 + rank], zero between launches
  // int32 accumulator output: row pitch acc_ld (elements); when acc_c is set, c[m, n]
  // (row pitch acc_c_ld) is added to each sum before it is stored (int32, wrapping).
  int acc_ld;
  const int32_t* acc_c;
  int acc_c_ld;
  int no_out;      // 1: the int32 accumulators are the only output (no scales, no out)
  // Every bounded wait of the kernel gives up after wait_ns of %globaltimer.
  unsigned long long wait_ns;
  // Test hook: the final K part of a split tile waits for one count-in more than the
  // other parts make, so that its bounded wait runs out (the timeout path).
  int hold_split;
  // Column-half tail of the CTA-pair kernel (halves = 1, split_s = 1): the first half_w
  // tiles are done whole, one per pair per round; each remaining tile is done as two
  // 256 x 128 items (columns [0,128) and [128,256) of the tile, M=256 N=128 MMAs, B
  // from the half-width map) on different pairs in the round after them.
  int halves, half_w;
};

// Work item i of pair `pair`: a whole tile, or one K part of a tail tile.  Returns
// false when the pair has no item i.
// half: -1 for a whole tile or a K part, else which column half of the tile.
__device__ __forceinline__ bool pair_item(const Params& p, int pair, int npairs, int i,
                                          int& tile, int& kb0, int& kb1, int& part, int& half) {
  const int T = p.num_m_blocks * p.num_n_blocks;
  half = -1;
  if (p.halves) {
    const int rounds = p.half_w / npairs;  // half_w is a multiple of npairs
    kb0 = 0;
    kb1 = p.num_k_blocks;
    part = -1;
    if (i < rounds) {
      tile = pair + i * npairs;
      return true;
    }
    if (i > rounds || pair >= 2 * (T - p.half_w)) return false;
    tile = p.half_w + pair / 2;
    half = pair & 1;
    return true;
  }
  const int rounds = p.split_w / npairs;  // split_w is a multiple of npairs when splitting
  if (p.split_s <= 1 || i < rounds) {
    tile = pair + i * npairs;
    if (tile >= (p.split_s <= 1 ? T : p.split_w)) return false;
    kb0 = 0;
    kb1 = p.num_k_blocks;
    part = -1;
    return true;
  }
  if (i > rounds || pair >= (T - p.split_w) * p.split_s) return false;
  tile = p.split_w + pair / p.split_s;
  part = pair % p.split_s;
  kb0 = (int)((long long)p.num_k_blocks * part / p.split_s);
  kb1 = (int)((long long)p.num_k_blocks * (part + 1) / p.split_s);
  return true;
}


// The k-blocks of A and of B that k-block kb of the K walk reads.
__device__ __forceinline__ void seg_blocks(const Params& p, int kb, int& akb, int& bkb) {
  const int s = kb / p.seg_kblocks;
  const int r = kb - s * p.seg_kblocks;
  akb = r + (int)((p.a_seg >> s) & 1u) * p.seg_kblocks;
  bkb = r + (int)((p.b_seg >> s) & 1u) * p.seg_kblocks;
}

// The fp32 epilogue steps after the accumulator (fp_acc): 32 columns n0.. of row `row`.
__device__ __forceinline__ void fp_epilogue(const Params& p, int row, int n0, float (&v)[32]) {
  if (p.ep_alpha) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(p.alpha, v[j]);
  }
  if (p.bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < p.N) v[j] = __fadd_rn(v[j], __ldg(p.bias + n0 + j));
  }
  if (p.ep_beta && row < p.M) {
    const float* c = reinterpret_cast<const float*>(p.out) + (size_t)row * p.ldc + n0;
    if (n0 + 32 <= p.N && p.out_vec) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 o = *reinterpret_cast<const float4*>(c + j);
        v[j] = __fadd_rn(v[j], __fmul_rn(p.beta, o.x));
        v[j + 1] = __fadd_rn(v[j + 1], __fmul_rn(p.beta, o.y));
        v[j + 2] = __fadd_rn(v[j + 2], __fmul_rn(p.beta, o.z));
        v[j + 3] = __fadd_rn(v[j + 3], __fmul_rn(p.beta, o.w));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) v[j] = __fadd_rn(v[j], __fmul_rn(p.beta, c[j]));
    }
  }
}

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

// As report(), and also raises the abort flag of the other CTA of the pair so that
// its waits give up at once instead of each running to its time limit.
__device__ __forceinline__ void report_pair(int* err, int code, volatile int* abort_flag,
                                            uint32_t rank) {
  report(err, code, abort_flag);
  const uint32_t peer = ptx::map_to_rank(ptx::smem_u32(const_cast<int*>(abort_flag)), rank ^ 1u);
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer), "r"(1) : "memory");
}

// The int32 accumulators of 32 consecutive columns of one row (row < M, n0 < N), plus
// the addend c when there is one.
__device__ __forceinline__ void store_acc(const Params& p, int row, int n0, bool full,
                                          const uint32_t (&r)[32]) {
  int32_t* dst = p.acc + (size_t)row * p.acc_ld + n0;
  const int32_t* c = p.acc_c ? p.acc_c + (size_t)row * p.acc_c_ld + n0 : nullptr;
  if (full && p.acc_vec) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      int4 v = make_int4((int)r[j], (int)r[j + 1], (int)r[j + 2], (int)r[j + 3]);
      if (c) {
        v.x = (int)((uint32_t)v.x + (uint32_t)__ldg(c + j));
        v.y = (int)((uint32_t)v.y + (uint32_t)__ldg(c + j + 1));
        v.z = (int)((uint32_t)v.z + (uint32_t)__ldg(c + j + 2));
        v.w = (int)((uint32_t)v.w + (uint32_t)__ldg(c + j + 3));
      }
      *reinterpret_cast<int4*>(dst + j) = v;
    }
  } else {
    for (int j = 0; j < 32 && n0 + j < p.N; ++j)
      dst[j] = (int)(r[j] + (c ? (uint32_t)__ldg(c + j) : 0u));
  }
}

// Epilogue for 32 consecutive columns of one row.
__device__ __forceinline__ void store_chunk(const Params& p, int row, int n0, float sa,
                                            const uint32_t (&r)[32]) {
  if (row >= p.M || n0 >= p.N) return;
  const bool full = (n0 + 32 <= p.N);
  if (p.acc) store_acc(p, row, n0, full, r);
  if (p.no_out) return;
  float sb[32];
  if (p.fp_acc) {
#pragma unroll
    for (int j = 0; j < 32; ++j) sb[j] = 1.f;
  } else if (full && ((reinterpret_cast<uintptr_t>(p.sB + n0) & 15) == 0)) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p.sB + n0 + j));
      sb[j] = v.x; sb[j + 1] = v.y; sb[j + 2] = v.z; sb[j + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) sb[j] = (n0 + j < p.N) ? __ldg(p.sB + n0 + j) : 0.f;
  }
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j)
    v[j] = p.fp_acc ? __uint_as_float(r[j])
                    : __fmul_rn(__fmul_rn(__int2float_rn((int)r[j]), sb[j]), sa);
  if (p.fp_acc) fp_epilogue(p, row, n0, v);
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


// Epilogue of one accumulator: this CTA's 128 rows (row0..row0+127) x ncols (256, or
// 128 for a column half) columns (n0..) held in TMEM columns [acc_col, acc_col+ncols).  Warp q reads TMEM lanes
// 32q..32q+31 (one output row per thread), dequantises, and writes 128-byte row pieces
// into the swizzled staging buffer; one elected thread then stores each 128-row x
// 128-byte block with a TMA bulk tensor store (clipped at the tensor edges).  `chunk_seq`
// counts staging buffers used so far (identical in all epilogue threads).
// Partial tiles of the last-wave split: 128 rows x 256 int32 columns of one CTA, stored
// so that the 32 rows a warp holds are contiguous: 16-byte piece v (columns 4v..4v+3)
// of 32-column chunk c of row rl sits at int4 index (c * 8 + v) * 128 + rl.
__device__ __forceinline__ size_t part_index(int c, int v, int rl) {
  return ((size_t)(c * 8 + v) * 128 + rl);
}

// With `parts` set, the accumulators are summed from `nparts` partial tiles,
// `part_stride` words apart, in part order: int32 sums, or fp32 sums when `fp` (the
// words are then fp32 accumulators).  from_r: the sum starts from r's values (the
// final part's own accumulator) instead of zero.
__device__ __forceinline__ uint32_t add_word(uint32_t a, int b, bool fp) {
  return fp ? __float_as_uint(__fadd_rn(__uint_as_float(a), __int_as_float(b))) : a + (uint32_t)b;
}

__device__ __forceinline__ void sum_parts(const int32_t* parts, int nparts, size_t part_stride,
                                          int rl, int col, bool fp, uint32_t (&r)[32],
                                          bool from_r = false) {
  if (!from_r) {
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] = 0u;  // also fp32 +0
  }
  for (int pp = 0; pp < nparts; ++pp) {
    const int4* src = reinterpret_cast<const int4*>(parts + pp * part_stride);
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      const int4 x = __ldcg(src + part_index(col / 32, v, rl));
      r[4 * v] = add_word(r[4 * v], x.x, fp);
      r[4 * v + 1] = add_word(r[4 * v + 1], x.y, fp);
      r[4 * v + 2] = add_word(r[4 * v + 2], x.z, fp);
      r[4 * v + 3] = add_word(r[4 * v + 3], x.w, fp);
    }
  }
}

__device__ __forceinline__ void epilogue_tile(const Params& p, const CUtensorMap* tmO,
                                              const PeerMaps* pm, uint32_t tmem_base, uint32_t acc_col, int q,
                                              int lane, int row0, int n0, uint32_t stg,
                                              bool elected, int& chunk_seq, bool ok,
                                              const int32_t* parts = nullptr, int nparts = 0,
                                              size_t part_stride = 0, bool add_tmem = false,
                                              int ncols = 256, const float* sb_smem = nullptr,
                                              const float* sa_pre = nullptr) {
  const int row = row0 + q * 32 + lane;
  const int rl = q * 32 + lane;  // row within the staging block
  // sb_smem / sa_pre: the item's column scales (from column n0 on) and this row's scale,
  // loaded by the caller before the accumulator was ready, off the epilogue's path
  const float sa = sa_pre ? *sa_pre
                          : (!p.fp_acc && !p.no_out && row < p.M) ? __ldg(p.sA + row) : 0.f;
  const bool skip = p.skip_flag != nullptr && *reinterpret_cast<const volatile int*>(p.skip_flag) != 0;
  if (!p.tma_store) {
#pragma unroll 1
    for (int c = 0; c < ncols / 32; ++c) {
      uint32_t r[32];
      __syncwarp();
      if (!ok) return;
      if (!parts || add_tmem) {
        ptx::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc_col + c * 32, r);
        ptx::tmem_wait_ld();
      }
      if (parts) sum_parts(parts, nparts, part_stride, rl, c * 32, p.fp_acc != 0, r, add_tmem);
      if (!skip) store_chunk(p, row, n0 + c * 32, sa, r);
    }
    return;
  }
  const bool bf16 = p.out_dtype == QGEMM_BF16;
  const int cwe = bf16 ? 64 : 32;  // columns per 128-byte staging row
#pragma unroll 1
  for (int ch = 0; ch < ncols / cwe; ++ch, ++chunk_seq) {
    const uint32_t buf = stg + (uint32_t)(chunk_seq & 1) * (128 * 128);
    // the store issued two chunks ago (same buffer) must have finished reading it
    if (elected) ptx::bulk_wait_group_read<1>();
    ptx::named_bar_sync(1, 128);
#pragma unroll 1
    for (int sub = 0; sub < cwe / 32; ++sub) {
      uint32_t r[32];
      const int nc = n0 + ch * cwe + sub * 32;
      __syncwarp();
      if (ok && (!parts || add_tmem)) {
        ptx::tmem_ld_32x32b_x32(
            tmem_base + ((uint32_t)(q * 32) << 16) + acc_col + (uint32_t)(ch * cwe + sub * 32), r);
        ptx::tmem_wait_ld();
      }
      if (ok && parts) {
        sum_parts(parts, nparts, part_stride, rl, ch * cwe + sub * 32, p.fp_acc != 0, r, add_tmem);
      } else if (!ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;  // a wait ran out: keep the barrier sequence
      }
      float sb[32];
      if (p.fp_acc) {
#pragma unroll
        for (int j = 0; j < 32; ++j) sb[j] = 1.f;
      } else if (sb_smem) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 v = *reinterpret_cast<const float4*>(sb_smem + ch * cwe + sub * 32 + j);
          sb[j] = v.x; sb[j + 1] = v.y; sb[j + 2] = v.z; sb[j + 3] = v.w;
        }
      } else if (nc + 32 <= p.N && ((reinterpret_cast<uintptr_t>(p.sB + nc) & 15) == 0)) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(p.sB + nc + j));
          sb[j] = v.x; sb[j + 1] = v.y; sb[j + 2] = v.z; sb[j + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) sb[j] = (nc + j < p.N) ? __ldg(p.sB + nc + j) : 0.f;
      }
      if (p.acc && row < p.M && nc < p.N) store_acc(p, row, nc, nc + 32 <= p.N, r);
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        v[j] = p.fp_acc ? __uint_as_float(r[j])
                        : __fmul_rn(__fmul_rn(__int2float_rn((int)r[j]), sb[j]), sa);
      if (p.fp_acc) fp_epilogue(p, row, nc, v);
      if (bf16) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // four 16-byte pieces = 32 bf16
          uint32_t w[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(v[8 * j + 2 * h], v[8 * j + 2 * h + 1]);
            w[h] = *reinterpret_cast<uint32_t*>(&b2);
          }
          const int piece = sub * 4 + j;
          ptx::st_shared_v4(buf + rl * 128 + ((piece ^ (rl & 7)) << 4), w[0], w[1], w[2], w[3]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // eight 16-byte pieces = 32 fp32
          ptx::st_shared_v4(buf + rl * 128 + ((j ^ (rl & 7)) << 4), __float_as_uint(v[4 * j]),
                            __float_as_uint(v[4 * j + 1]), __float_as_uint(v[4 * j + 2]),
                            __float_as_uint(v[4 * j + 3]));
        }
      }
    }
    ptx::fence_proxy_async_smem();  // generic-proxy writes -> visible to the TMA engine
    ptx::named_bar_sync(1, 128);
    if (elected && !skip && row0 < p.M && n0 + ch * cwe < p.N) {  // blocks past the edge: nothing to store
      ptx::tma_store_2d(tmO, buf, n0 + ch * cwe, row0);
      for (int i = 0; i < p.npeer; ++i) ptx::tma_store_2d(&pm->m[i], buf, n0 + ch * cwe, row0);
      ptx::bulk_commit_group();
    }
  }
}

// KIND selects the MMA kind at compile time: a run-time choice inside the issue loop
// cost a fifth of the tensor throughput.
template <int KIND>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    w8a8_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmBh,
                        const __grid_constant__ CUtensorMap tmO,
                        const __grid_constant__ PeerMaps pm, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment: required by the 128-byte swizzle pattern of TMA and UMMA.
  const uint32_t raw_base = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);

  const uint32_t stg_base = base + STAGES * STAGE_BYTES;  // output staging (1024-aligned)
  const uint32_t bar_base = stg_base + STG_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * STAGES + 4);
  uint8_t* gbar = gbase + STAGES * STAGE_BYTES + STG_BYTES;
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
    // The next kernel on the stream may start its own set-up on SMs this grid has
    // finished with; every global access below waits for the previous kernel.
    ptx::grid_launch_dependents();
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
      ptx::grid_dependency_wait();
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!ptx::mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, p.wait_ns)) {
            if (!*abort_flag) report(p.err, DEVERR_TIMEOUT_PRODUCER, abort_flag);
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
          int akb, bkb;
          seg_blocks(p, kb, akb, bkb);
          ptx::mbar_arrive_expect_tx(full_bar(stage), STAGE_BYTES);
          ptx::tma_load_2d(sa, &tmA, full_bar(stage), akb * BK, mb * BM);
          if (p.b_kn) {
            ptx::tma_load_2d(sb, &tmB, full_bar(stage), nb * BN, kb * BK);
            ptx::tma_load_2d(sb + B_BYTES / 2, &tmB, full_bar(stage), nb * BN + 128, kb * BK);
          } else {
            ptx::tma_load_2d(sb, &tmB, full_bar(stage), bkb * BK, nb * BN);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: every copy this thread issued must land before the CTA exits.
      for (long long f = (issued > STAGES ? issued - STAGES : 0); f < issued; ++f) {
        const int s = (int)(f % STAGES);
        const uint32_t par = (uint32_t)((f / STAGES) & 1);
        if (!ptx::mbar_wait(full_bar(s), par, nullptr, p.wait_ns)) {
          report(p.err, DEVERR_TIMEOUT_DRAIN, abort_flag);
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = KIND == KIND_BF16   ? ptx::idesc_bf16(BM, BN)
                             : KIND == KIND_TF32 ? ptx::idesc_tf32(BM, BN)
                                                 : ptx::idesc_i8(BM, BN, false, p.b_kn != 0);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
        const int a = it & 1;
        const uint32_t aphase = (uint32_t)((it >> 1) & 1);
        if (!ptx::mbar_wait(tempty_bar(a), aphase ^ 1u, abort_flag, p.wait_ns)) {
          if (!*abort_flag) report(p.err, DEVERR_TIMEOUT_MMA, abort_flag);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(a * BN);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!ptx::mbar_wait(full_bar(stage), phase, abort_flag, p.wait_ns)) {
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
            if constexpr (KIND == KIND_BF16)
              ptx::umma_bf16(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
            else if constexpr (KIND == KIND_TF32)
              ptx::umma_tf32(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
            else
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
        if (!ptx::mbar_wait(drain_bar, 0, nullptr, p.wait_ns)) report(p.err, DEVERR_TIMEOUT_DRAIN, abort_flag);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    ptx::grid_dependency_wait();  // scales and the output belong to the previous kernel until it ends
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const bool elected = (warp == 2 && lane == 0);
    int chunk_seq = 0;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int a = it & 1;
      const uint32_t aphase = (uint32_t)((it >> 1) & 1);
      bool ok = ptx::mbar_wait_sleep(tfull_bar(a), aphase, abort_flag, p.wait_ns);
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform: tcgen05.ld is .sync.aligned
      if (!ok && lane == 0 && !*abort_flag) report(p.err, DEVERR_TIMEOUT_EPILOGUE, abort_flag);
      ptx::tc_fence_after();
      epilogue_tile(p, &tmO, &pm, tmem_base, (uint32_t)(a * BN), q, lane, mb * BM, nb * BN, stg_base,
                    elected, chunk_seq, ok);
      ptx::tc_fence_before();
      ptx::mbar_arrive(tempty_bar(a));
    }
    // The CTA may exit once its last stores have read their staging buffers; the writes
    // themselves complete with the grid.  The peer windows of the fused all-gather are
    // waited for in full.
    if (elected) {
      if (p.npeer) ptx::bulk_wait_group_all();
      else ptx::bulk_wait_group_read<0>();
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


// ---------------------------------------------------------------------------------
// CTA-pair kernel: one 256 x 256 tile per cluster of two CTAs (tcgen05 cta_group::2).
// CTA r of the pair loads A rows [256*mb + 128*r, +128) and B columns
// [256*nb + 128*r, +128) into its own shared memory; both CTAs' copies complete on
// the even CTA's "full" barrier.  The even CTA's MMA thread issues M=256 N=256 K=32
// MMAs that read both CTAs' tiles and write rows 128*r.. of D into CTA r's TMEM, and
// its commits arrive on the "empty"/"tfull" barriers of both CTAs.  Each CTA's
// epilogue drains its own TMEM half and arrives on the even CTA's "tempty" barrier.
// Per SM and 128-deep k-block this moves 32 KB through shared memory for 512 cycles
// of MMA (the single-CTA 128 x 256 tile moves 48 KB), which is what lets the tensor
// pipe run near its rate without exceeding shared-memory bandwidth.
namespace pair {
constexpr int BM = 256;                        // rows per pair tile (128 per CTA)
constexpr int BN = 256;                        // columns per pair tile (128 of B per CTA)
constexpr int STAGES = 6;
constexpr int A_BYTES = 128 * BK;              // 16 KB
constexpr int B_BYTES = 128 * BK;              // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES; // 32 KB per CTA
constexpr int SB_BYTES = 256 * 4;              // the current item's column scales (fp32)
constexpr int SMEM_BYTES = 232448;
static_assert(STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES + SB_BYTES + 1024 <= SMEM_BYTES,
              "shared memory budget");
}  // namespace pair

template <int KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    w8a8_tcgen05_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmBh,
                             const __grid_constant__ CUtensorMap tmO,
                             const __grid_constant__ PeerMaps pm, const Params p) {
  constexpr int BM = pair::BM, BN = pair::BN, STAGES = pair::STAGES;
  constexpr int A_BYTES = pair::A_BYTES, B_BYTES = pair::B_BYTES, STAGE_BYTES = pair::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);

  const uint32_t stg_base = base + STAGES * STAGE_BYTES;  // output staging (1024-aligned)
  const uint32_t bar_base = stg_base + STG_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * STAGES + 4);
  uint8_t* gbar = gbase + STAGES * STAGE_BYTES + STG_BYTES;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbar + 8 * (2 * STAGES + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbar + 8 * (2 * STAGES + 5) + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = ptx::cluster_ctarank();   // 0: issues the MMAs
  const int pair_id = blockIdx.x / 2;
  const int npairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(tfull_bar(a), 1);
      ptx::mbar_init(tempty_bar(a), 2 * 128);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    // The next kernel on the stream may start its own set-up on SMs this grid has
    // finished with; every global access below waits for the previous kernel.
    ptx::grid_launch_dependents();
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmB);
    if (p.halves) ptx::prefetch_tmap(&tmBh);
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(ptx::smem_u32(const_cast<uint32_t*>(tmem_slot)), TMEM_COLS);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync_all();  // barriers of both CTAs initialised before any remote traffic
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      ptx::grid_dependency_wait();
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      int tile, kb0, kb1, part, half;
      for (int item = 0; ok && pair_item(p, pair_id, npairs, item, tile, kb0, kb1, part, half); ++item) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        // B per CTA: 128 columns of the tile, or 64 columns of one column half (the
        // half-width map: [K,N] boxes 64 columns x 128 k-rows with the 64-byte swizzle,
        // [N,K] boxes 128 k-bytes x 64 rows)
        const bool hf = half >= 0;
        const void* bmap = hf ? (const void*)&tmBh : (const void*)&tmB;
        const int bcol = nb * BN + (hf ? half * 128 + (int)rank * 64 : (int)rank * 128);
        const uint32_t tx = hf ? 2u * (A_BYTES + B_BYTES / 2) : 2u * STAGE_BYTES;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, p.wait_ns)) {
            if (!*abort_flag) report_pair(p.err, DEVERR_TIMEOUT_PRODUCER, abort_flag, rank);
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
          const uint32_t fb = ptx::map_to_rank(full_bar(stage), 0);
          int akb, bkb;
          seg_blocks(p, kb, akb, bkb);
          if (rank == 0) ptx::mbar_arrive_expect_tx(full_bar(stage), tx);
          ptx::tma_load_2d_pair(sa, &tmA, fb, akb * BK, mb * BM + (int)rank * 128);
          if (p.b_kn)
            ptx::tma_load_2d_pair(sb, bmap, fb, bcol, kb * BK);
          else
            ptx::tma_load_2d_pair(sb, bmap, fb, bkb * BK, bcol);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: the even CTA's full barriers count both CTAs' copies.
      if (rank == 0) {
        for (long long f = (issued > STAGES ? issued - STAGES : 0); f < issued; ++f) {
          if (!ptx::mbar_wait(full_bar((int)(f % STAGES)), (uint32_t)((f / STAGES) & 1), nullptr, p.wait_ns)) {
            report_pair(p.err, DEVERR_TIMEOUT_DRAIN, abort_flag, rank);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (lane == 0 && rank == 0) {
      const uint32_t idesc_w = KIND == KIND_BF16   ? ptx::idesc_bf16(BM, BN)
                               : KIND == KIND_TF32 ? ptx::idesc_tf32(BM, BN)
                                                   : ptx::idesc_i8(BM, BN, false, p.b_kn != 0);
      const uint32_t idesc_h = KIND == KIND_BF16   ? ptx::idesc_bf16(BM, BN / 2)
                               : KIND == KIND_TF32 ? ptx::idesc_tf32(BM, BN / 2)
                                                   : ptx::idesc_i8(BM, BN / 2, false, p.b_kn != 0);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      int tile, kb0, kb1, part, half;
      for (; ok && pair_item(p, pair_id, npairs, it, tile, kb0, kb1, part, half); ++it) {
        // B operand of this item.  [K,N] (MN-major): one 128-column swizzle row per CTA
        // (128-byte swizzle, k-row groups 1024 bytes apart), or for a column half one
        // 64-column row (64-byte swizzle, groups 512 bytes apart); the leading offset
        // is the B region's size, which no read reaches with a single MN atom.  [N,K]
        // (K-major): 128 or 64 rows of 128 k-bytes, the same descriptor.
        const bool hf = half >= 0;
        const uint32_t idesc = hf ? idesc_h : idesc_w;
        const uint32_t b_row = p.b_kn ? (hf ? 64u : 128u) : 1u;  // bytes per k of B
        const uint32_t b_lbo = p.b_kn ? (uint32_t)B_BYTES : 16u;
        const uint32_t b_sbo = p.b_kn ? 8u * b_row : 1024u;
        const uint32_t b_swz = (p.b_kn && hf) ? ptx::SWZ_64B : ptx::SWZ_128B;
        const int a = it & 1;
        const uint32_t aphase = (uint32_t)((it >> 1) & 1);
        if (!ptx::mbar_wait(tempty_bar(a), aphase ^ 1u, abort_flag, p.wait_ns)) {
          if (!*abort_flag) report_pair(p.err, DEVERR_TIMEOUT_MMA, abort_flag, rank);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(a * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait(full_bar(stage), phase, abort_flag, p.wait_ns)) {
            if (!*abort_flag) report_pair(p.err, DEVERR_TIMEOUT_MMA, abort_flag, rank);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sa = base + stage * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t adesc = ptx::smem_desc_sw128(sa + kk * UMMA_K, 16, 1024);
            const uint64_t bdesc = ptx::smem_desc(sb + kk * UMMA_K * b_row, b_lbo, b_sbo, b_swz);
            const uint32_t accum = (kb != kb0 || kk != 0) ? 1u : 0u;
            if constexpr (KIND == KIND_BF16)
              ptx::umma_bf16_pair(d_tmem, adesc, bdesc, idesc, accum);
            else if constexpr (KIND == KIND_TF32)
              ptx::umma_tf32_pair(d_tmem, adesc, bdesc, idesc, accum);
            else
              ptx::umma_i8_pair(d_tmem, adesc, bdesc, idesc, accum);
          }
          ptx::umma_commit_pair(empty_bar(stage), 0x3);
          issued_any = true;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) ptx::umma_commit_pair(tfull_bar(a), 0x3);
      }
      if (!ok && issued_any) {
        ptx::umma_commit_pair(drain_bar, 0x1);
        if (!ptx::mbar_wait(drain_bar, 0, nullptr, p.wait_ns)) report_pair(p.err, DEVERR_TIMEOUT_DRAIN, abort_flag, rank);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    ptx::grid_dependency_wait();  // scales and the output belong to the previous kernel until it ends
    const int q = warp & 3;
    const bool elected = (warp == 2 && lane == 0);
    int chunk_seq = 0;
    const uint32_t te_leader0 = ptx::map_to_rank(tempty_bar(0), 0);
    const uint32_t te_leader1 = ptx::map_to_rank(tempty_bar(1), 0);
    volatile int* last_flag = abort_flag + 1;
    const int rl = q * 32 + lane;  // row of this CTA's half-tile
    float* sb_smem = reinterpret_cast<float*>(gbar + BAR_BYTES);  // pair::SB_BYTES
    const bool scaled = !p.fp_acc && !p.no_out;
    int it = 0;
    int tile, kb0, kb1, part, half;
    for (; pair_item(p, pair_id, npairs, it, tile, kb0, kb1, part, half); ++it) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int a = it & 1;
      const uint32_t aphase = (uint32_t)((it >> 1) & 1);
      // This item's column scales into shared memory and this row's scale into a
      // register while the MMAs run: in the last item nothing else hides their latency.
      const int n0i = nb * BN + (half > 0 ? BN / 2 : 0);
      const int nci = half >= 0 ? BN / 2 : BN;
      ptx::named_bar_sync(1, 128);  // the previous item's epilogue is done with sb_smem
      if (scaled)
        for (int c = rl; c < nci; c += 128) sb_smem[c] = n0i + c < p.N ? __ldg(p.sB + n0i + c) : 0.f;
      const int row_i = mb * BM + (int)rank * 128 + rl;
      const float sa_i = (scaled && row_i < p.M) ? __ldg(p.sA + row_i) : 0.f;
      ptx::named_bar_sync(1, 128);
      const float* sbp = scaled ? sb_smem : nullptr;
      // a spinning wait: the last item's epilogue starts as soon as its accumulator is done
      bool ok = ptx::mbar_wait(tfull_bar(a), aphase, abort_flag, p.wait_ns);
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform: tcgen05.ld is .sync.aligned
      if (!ok && lane == 0 && !*abort_flag)
        report_pair(p.err, DEVERR_TIMEOUT_EPILOGUE, abort_flag, rank);
      ptx::tc_fence_after();
      if (part < 0) {
        epilogue_tile(p, &tmO, &pm, tmem_base, (uint32_t)(a * BN), q, lane,
                      mb * BM + (int)rank * 128, n0i, stg_base, elected, chunk_seq, ok, nullptr,
                      0, 0, false, nci, sbp, &sa_i);
        ptx::tc_fence_before();
        ptx::mbar_arrive_remote(a ? te_leader1 : te_leader0);
        continue;
      }
      // A K part of a tail tile.  Parts 0 .. split_s-2 park their partial sums (this
      // CTA's 128 rows) and count in.  The final part (the last K range) waits until the
      // others have counted in, adds their partials to its own accumulator in TMEM and
      // stores the tile; it neither writes nor re-reads a partial of its own.
      const size_t slot_ints = (size_t)128 * 256;
      const int tt = (tile - p.split_w) * 2 + (int)rank;
      if (part < p.split_s - 1) {
        int4* mine = reinterpret_cast<int4*>(p.part + ((size_t)tt * p.split_s + part) * slot_ints);
#pragma unroll 1
        for (int c = 0; c < 256 / 32; ++c) {
          uint32_t r[32];
          __syncwarp();
          if (ok) {
            ptx::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN + c * 32), r);
            ptx::tmem_wait_ld();
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = 0u;
          }
#pragma unroll
          for (int v = 0; v < 8; ++v)
            mine[part_index(c, v, rl)] =
                make_int4((int)r[4 * v], (int)r[4 * v + 1], (int)r[4 * v + 2], (int)r[4 * v + 3]);
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive_remote(a ? te_leader1 : te_leader0);  // TMEM is free again
        __threadfence();
        ptx::named_bar_sync(1, 128);
        if (elected) atomicAdd(p.cnt + tt, 1);
        continue;
      }
      if (elected) {
        // bounded wait for the other parts' count-ins.  They run on lower-numbered pairs
        // (pair = tail tile * split_s + part), which are dispatched before this one, and
        // wait on nothing: a resident final part never waits on a part that cannot run.
        bool got = false;
        const unsigned long long t0 = ptx::globaltimer();
        for (;;) {
          if (ptx::ld_acquire_gpu(p.cnt + tt) >= p.split_s - 1 + p.hold_split) { got = true; break; }
          if (*abort_flag || ptx::globaltimer() - t0 > p.wait_ns) break;
          __nanosleep(64);
        }
        if (!got && !*abort_flag) report_pair(p.err, DEVERR_TIMEOUT_EPILOGUE, abort_flag, rank);
        *last_flag = got ? 1 : 0;
      }
      ptx::named_bar_sync(1, 128);
      const bool ready = ok && *last_flag != 0;
      epilogue_tile(p, &tmO, &pm, tmem_base, (uint32_t)(a * BN), q, lane,
                    mb * BM + (int)rank * 128, nb * BN, stg_base, elected, chunk_seq, ready,
                    p.part + (size_t)tt * p.split_s * slot_ints, p.split_s - 1, slot_ints, true,
                    BN, sbp, &sa_i);
      ptx::tc_fence_before();
      ptx::mbar_arrive_remote(a ? te_leader1 : te_leader0);
      if (elected) p.cnt[tt] = 0;
      ptx::named_bar_sync(1, 128);  // the flag is rewritten only after everyone read it
    }
    // The CTA may exit once its last stores have read their staging buffers; the writes
    // themselves complete with the grid.  The peer windows of the fused all-gather are
    // waited for in full.
    if (elected) {
      if (p.npeer) ptx::bulk_wait_group_all();
      else ptx::bulk_wait_group_read<0>();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync_all();  // the pair's MMAs and remote arrivals are finished
  ptx::tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    ptx::tmem_dealloc_pair(tmem_base, TMEM_COLS);
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
                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
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

// Grid and last-wave split of one tcgen05 GEMM launch; a function of the shape and the
// device only, so callers can size the scratch before the launch.
struct TcPlan {
  bool use_pair;
  int grid;
  int num_tiles;
  int split_w, split_s;   // as in Params; split_s = 1: no split
  int halves, half_w;     // as in Params; halves = 0: whole tiles only
  size_t cnt_bytes;       // counter block at the start of the scratch
  size_t part_bytes;      // partial tiles after it (0: no split)
};

// full_split: a shape with fewer pair tiles than pairs has every tile cut along K (up
// to 8 parts of at least 8 k-blocks each) so that more pairs are busy.
static TcPlan tc_plan(const qgemm_device_s* d, int M, int N, int num_k_blocks, bool full_split) {
  using namespace w8a8;
  TcPlan t;
  // CTA pairs (256 x 256 tiles) whenever the problem has at least one full pair tile;
  // with full_split also for smaller shapes whose 1-CTA tiles cannot fill the GPU
  // (rows and columns past the edges are zero-filled by TMA and never stored).
  const long long tiles1 = (long long)((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  t.use_pair = d->sm_count >= 2 &&
               ((M >= 256 && N >= 256) || (full_split && tiles1 < d->sm_count));
  const int bm = t.use_pair ? pair::BM : BM, bn = t.use_pair ? pair::BN : BN;
  t.num_tiles = ((M + bm - 1) / bm) * ((N + bn - 1) / bn);
  t.split_w = t.num_tiles;
  t.split_s = 1;
  t.halves = 0;
  t.half_w = t.num_tiles;
  // The counter block has one fixed size on a device (counters for up to
  // 2 * max_pairs half-tiles; rest < max_pairs) and is counted in every plan, so that
  // callers which carve their own buffers out of the stream's scratch never place them
  // over it: the counters must sit at the same place in every call, as they are zero
  // between calls only because each call returns the ones it used to zero.
  const int max_pairs = d->sm_count / 2 > 0 ? d->sm_count / 2 : 1;
  t.cnt_bytes = ((size_t)max_pairs * 2 * sizeof(int) + 255) & ~(size_t)255;
  t.part_bytes = 0;
  if (!t.use_pair) {
    t.grid = t.num_tiles < d->sm_count ? t.num_tiles : d->sm_count;
    return t;
  }
  if (full_split && t.num_tiles < max_pairs) {
    // at most 8 parts of at least 8 k-blocks: the part that finishes last adds all the
    // partial tiles alone, so many short parts cost more than they save (512^3 with
    // 16 parts of 3 k-blocks: 89 us against 54 unsplit)
    int parts = max_pairs / t.num_tiles;
    if (parts > 8) parts = 8;
    if (parts > num_k_blocks / 8) parts = num_k_blocks / 8;
    if (parts >= 2) {
      // every tile is a tail tile: split_w = 0, one K part per pair
      t.split_w = 0;
      t.split_s = parts;
      t.grid = 2 * t.num_tiles * parts;
      t.part_bytes = (size_t)t.num_tiles * 2 * parts * 128 * 256 * sizeof(int32_t);
      return t;
    }
  }
  if (t.num_tiles < max_pairs && 2 * t.num_tiles <= max_pairs) {
    // fewer tiles than half the pairs: every tile as two column halves, one per pair
    t.halves = 1;
    t.half_w = 0;
    t.grid = 4 * t.num_tiles;
    return t;
  }
  const int pairs = t.num_tiles < max_pairs ? t.num_tiles : max_pairs;
  t.grid = 2 * pairs;
  // Last-wave split: when the final round would leave at least three quarters of the
  // pairs idle, cut each leftover tile along K into 4 parts (at least two k-blocks
  // each).  Measured (bf16 out, [K,N] B): four-way splits win (3840x4096x4096:
  // 1931 against 1874 TOPS unsplit); two-way splits lose even with the final part
  // adding the others' partials in TMEM (4096^3: 2295 against 2511; 4096x4096x2048:
  // 1494 against 1825).
  const int rounds = t.num_tiles / pairs, rest = t.num_tiles - rounds * pairs;
  int parts = (rest > 0 && rest * 4 <= pairs) ? 4 : 1;
  while (parts > 1 && num_k_blocks / parts < 2) --parts;
  if (parts < 4) parts = 1;
  if (rounds >= 1 && parts >= 2) {
    t.split_w = rounds * pairs;
    t.split_s = parts;
    t.part_bytes = (size_t)rest * 2 * parts * 128 * 256 * sizeof(int32_t);
  } else if (rounds >= 1 && rest > 0 && 2 * rest <= pairs) {
    // Column-half tail: the leftover tiles as 256 x 128 halves on twice as many pairs,
    // so the last round takes about half as long (4096^3: 34 leftover tiles on 74
    // pairs become 68 halves).  No scratch.
    t.halves = 1;
    t.half_w = rounds * pairs;
  }
  return t;
}

size_t tc_gemm_scratch_bytes(const qgemm_device_s* d, int M, int N, int num_k_blocks,
                             bool full_split) {
  const TcPlan t = tc_plan(d, M, N, num_k_blocks, full_split);
  return t.cnt_bytes + t.part_bytes;
}

// The tcgen05 GEMM behind the W8A8, bf16 and fp32 entry points (TcArgs in internal.h).
qgemm_status launch_tc_gemm(qgemm_stream_s* s, const TcArgs& a) {
  using namespace w8a8;
  if (a.kind < KIND_I8 || a.kind > KIND_TF32) return fail(QGEMM_ERR_INVALID_ARG, "MMA kind %d", a.kind);
  const int M = a.M, N = a.N, K = a.K;
  const uint64_t kblk = (uint64_t)((K + BK - 1) / BK);
  const int num_k_blocks = (int)kblk * a.nseg;
  const TcPlan t = tc_plan(s->dev, M, N, num_k_blocks, a.full_split != 0);
  const bool use_pair = t.use_pair;
  const int bm = use_pair ? pair::BM : BM, bn = use_pair ? pair::BN : BN;
  const uint64_t a_pitch = a.a_pitch ? a.a_pitch : (uint64_t)K;
  const uint64_t b_pitch = a.b_pitch ? a.b_pitch : (uint64_t)K;
  const uint64_t a_extent = a.a_extent ? a.a_extent : a_pitch;
  const uint64_t kn_pitch = a.b_kn_pitch ? a.b_kn_pitch : (uint64_t)N;
  CUtensorMap tmA, tmB;
  if (!make_map_u8(&tmA, a.A, a_extent, (uint64_t)M, a_pitch, BK, 128))
    return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for A [%d,%d]", M, K);
  // B boxes: [K,N] -> 128 columns x 128 k-rows; [N,K] -> 128 k-bytes x (bn per CTA) rows.
  const uint32_t nk_rows = use_pair ? 128 : BN;
  bool okb = a.b_kn ? make_map_u8(&tmB, a.B, (uint64_t)N, (uint64_t)K, kn_pitch, 128, BK)
                    : make_map_u8(&tmB, a.B, b_pitch, (uint64_t)N, b_pitch, BK, nk_rows);
  if (!okb) return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for B");
  // half-width B boxes for the column-half items of the pair kernel
  CUtensorMap tmBh;
  memset(&tmBh, 0, sizeof(tmBh));
  if (use_pair && t.halves) {
    okb = a.b_kn ? make_map_u8(&tmBh, a.B, (uint64_t)N, (uint64_t)K, kn_pitch, 64, BK,
                               CU_TENSOR_MAP_SWIZZLE_64B)
                 : make_map_u8(&tmBh, a.B, b_pitch, (uint64_t)N, b_pitch, BK, 64);
    if (!okb) return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for the B half map");
  }

  Params p;
  p.M = M; p.N = N; p.K = K; p.ldc = a.ldc;
  p.out_dtype = a.out_dtype;
  p.b_kn = a.b_kn;
  p.num_m_blocks = (M + bm - 1) / bm;
  p.num_n_blocks = (N + bn - 1) / bn;
  p.num_k_blocks = num_k_blocks;
  p.seg_kblocks = (int)kblk;
  p.a_seg = a.a_seg;
  p.b_seg = a.b_seg;
  p.num_tiles = t.num_tiles;
  p.sA = a.sA; p.sB = a.sB; p.out = a.out; p.acc = a.acc;
  p.acc_ld = a.acc_ld ? a.acc_ld : N;
  p.acc_c = a.acc_c;
  p.acc_c_ld = a.acc_c_ld;
  p.no_out = a.no_out;
  p.wait_ns = s->dev->wait_ns;
  p.hold_split = s->dev->hold_split ? 1 : 0;
  p.fp_acc = a.kind != KIND_I8;
  p.alpha = a.alpha; p.beta = a.beta; p.bias = a.bias;
  p.ep_alpha = a.ep_alpha; p.ep_beta = a.ep_beta;
  p.skip_flag = a.skip_flag;
  p.err = s->dev->d_err;
  const int esize = a.out_dtype == QGEMM_BF16 ? 2 : 4;
  p.out_vec = !a.no_out && aligned((uint64_t)a.out, 16) && ((uint64_t)a.ldc * esize) % 16 == 0;
  p.acc_vec = a.acc != nullptr && aligned((uint64_t)a.acc, 16) && p.acc_ld % 4 == 0 &&
              (a.acc_c == nullptr || (aligned((uint64_t)a.acc_c, 16) && a.acc_c_ld % 4 == 0));
  // Output tensor map for TMA stores: [M rows, N columns] with row pitch ldc, boxes of
  // 128 rows x 128 bytes, 128-byte swizzle (matching the staging buffer).
  CUtensorMap tmO;
  memset(&tmO, 0, sizeof(tmO));
  p.tma_store = 0;
  if (p.out_vec) {
    EncodeTiledFn enc = get_encode_fn();
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)a.ldc * esize};
    cuuint32_t box[2] = {(cuuint32_t)(128 / esize), 128};
    cuuint32_t estr[2] = {1, 1};
    if (enc && enc(&tmO, a.out_dtype == QGEMM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                   2, a.out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      p.tma_store = 1;
  }
  // peer output windows (fused sharded GEMM + all-gather): the same map on each peer's
  // address; TMA stores only
  PeerMaps pm;
  memset(&pm, 0, sizeof(pm));
  p.npeer = 0;
  if (a.npeer > 0) {
    if (a.npeer > MAX_PEERS)
      return fail(QGEMM_ERR_UNSUPPORTED, "%d peer windows (at most %d)", a.npeer, MAX_PEERS);
    if (!p.tma_store)
      return fail(QGEMM_ERR_UNSUPPORTED, "peer windows need the TMA-store epilogue: 16-byte "
                  "aligned output and rows a multiple of 16 bytes");
    EncodeTiledFn enc = get_encode_fn();
    for (int i = 0; i < a.npeer; ++i) {
      cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
      cuuint64_t strides[1] = {(cuuint64_t)a.ldc * esize};
      cuuint32_t box[2] = {(cuuint32_t)(128 / esize), 128};
      cuuint32_t estr[2] = {1, 1};
      if (!aligned((uint64_t)a.peer_out[i], 16) || !enc ||
          enc(&pm.m[i], a.out_dtype == QGEMM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
              2, const_cast<void*>(a.peer_out[i]), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for peer window %d", i);
    }
    p.npeer = a.npeer;
  }

  using Kern = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                        const PeerMaps, const Params);
  static const Kern kerns[2][3] = {
      {w8a8_tcgen05_kernel<KIND_I8>, w8a8_tcgen05_kernel<KIND_BF16>, w8a8_tcgen05_kernel<KIND_TF32>},
      {w8a8_tcgen05_pair_kernel<KIND_I8>, w8a8_tcgen05_pair_kernel<KIND_BF16>,
       w8a8_tcgen05_pair_kernel<KIND_TF32>}};
  const Kern kern = kerns[use_pair ? 1 : 0][a.kind];
  const int smem = use_pair ? pair::SMEM_BYTES : SMEM_BYTES;
  static bool attr_set[64][2][3] = {};
  const int ord = s->dev->ordinal;
  if (ord < 0 || ord >= 64 || !attr_set[ord][use_pair][a.kind]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w8a8_tcgen05)");
    if (ord >= 0 && ord < 64) attr_set[ord][use_pair][a.kind] = true;
  }
  p.split_w = t.num_tiles;
  p.split_s = 1;
  p.halves = t.halves;
  p.half_w = t.half_w;
  p.part = nullptr;
  p.cnt = nullptr;
  if (t.split_s > 1) {
    const size_t need = t.cnt_bytes + t.part_bytes;
    void* ws = nullptr;
    if (a.scratch) {
      if (a.scratch_bytes < need)
        return fail(QGEMM_ERR_UNSUPPORTED,
                    "this shape's last-wave split needs %zu bytes of scratch; the given "
                    "scratch holds %zu", need, a.scratch_bytes);
      ws = a.scratch;
    } else if (stream_workspace(s, need, &ws) != QGEMM_OK) {
      ws = nullptr;  // e.g. under graph capture: run the last round unsplit
    }
    if (ws) {
      p.split_w = t.split_w;
      p.split_s = t.split_s;
      p.cnt = static_cast<int*>(ws);
      p.part = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + t.cnt_bytes);
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(t.grid, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmBh, tmO, pm, p);
  if (e != cudaSuccess) return cuda_fail(e, "w8a8_tcgen05 launch");
  return QGEMM_OK;
}

static TcArgs w8a8_args(const void* A, const void* B, int b_kn, const float* sA, const float* sB,
                        void* out, int out_dtype, int ldc, int M, int N, int K, int32_t* acc) {
  TcArgs a;
  a.kind = KIND_I8;
  a.A = A; a.B = B; a.b_kn = b_kn;
  a.M = M; a.N = N; a.K = K;
  a.sA = sA; a.sB = sB; a.acc = acc;
  a.out = out; a.out_dtype = out_dtype; a.ldc = ldc;
  return a;
}

qgemm_status launch_w8a8_tcgen05(qgemm_stream_s* s, const void* A, const void* B, int b_kn,
                                 const float* sA, const float* sB, void* out, int out_dtype,
                                 int ldc, int M, int N, int K, int32_t* acc) {
  return launch_tc_gemm(s, w8a8_args(A, B, b_kn, sA, sB, out, out_dtype, ldc, M, N, K, acc));
}

qgemm_status launch_w8a8_tcgen05_peers(qgemm_stream_s* s, const void* A, const void* B, int b_kn,
                                       const float* sA, const float* sB, void* out, int ldc,
                                       int M, int N, int K, const uint64_t* peer_out,
                                       int npeer) {
  TcArgs a = w8a8_args(A, B, b_kn, sA, sB, out, QGEMM_BF16, ldc, M, N, K, nullptr);
  if (npeer < 0 || npeer > 7) return fail(QGEMM_ERR_INVALID_ARG, "npeer %d", npeer);
  for (int i = 0; i < npeer; ++i) a.peer_out[i] = reinterpret_cast<const void*>(peer_out[i]);
  a.npeer = npeer;
  return launch_tc_gemm(s, a);
}

// With a_repeat = 2, each row of B holds 2 blocks of ceil(2K / 128) * 128 bytes (zero past
// 2K bytes) and A is read twice along K: out = A * B_0^T + A * B_1^T.
qgemm_status launch_bf16_gemm_nk(qgemm_stream_s* s, const void* A, const void* B, void* out,
                                 int ldc, int M, int N, int K, int a_repeat) {
  if (a_repeat != 1 && a_repeat != 2) return fail(QGEMM_ERR_INVALID_ARG, "a_repeat %d", a_repeat);
  TcArgs a;
  a.kind = KIND_BF16;
  a.A = A; a.B = B;
  a.M = M; a.N = N; a.K = 2 * K;
  if (a_repeat == 2) {
    const uint64_t blk = (uint64_t)((a.K + w8a8::BK - 1) / w8a8::BK) * w8a8::BK;
    a.nseg = 2;
    a.b_seg = 0x2u;
    a.b_pitch = 2 * blk;
  }
  a.out = out; a.out_dtype = QGEMM_BF16; a.ldc = ldc;
  return launch_tc_gemm(s, a);
}

// ---- the W8A8 GEMM with a static scratch (qgemm_w8a8_gemm_static_scratch) ----------
// The last-wave split's counters and partial tiles live in this file-scope device
// array instead of scratch made on the stream handle, so the call never allocates.
// 4 KiB of counters (up to 512 CTA pairs) + 20 MiB of partial tiles: four int32
// 128 x 256 parts per half of up to 20 leftover pair tiles, the most a four-way split
// can leave on a GPU of up to 160 SMs.  Shared by every call on the device.
constexpr size_t STATIC_CNT_BYTES = 4096;
constexpr size_t STATIC_SCRATCH_BYTES = STATIC_CNT_BYTES + ((size_t)20 << 20);
static __device__ __align__(256) uint8_t g_static_scratch[STATIC_SCRATCH_BYTES];

static qgemm_status static_scratch(const qgemm_device_s* d, void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  if (d->ordinal < 0 || d->ordinal >= 64) return fail(QGEMM_ERR_UNSUPPORTED, "device ordinal >= 64");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[d->ordinal]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    addr[d->ordinal] = p;
  }
  *out = addr[d->ordinal];
  return QGEMM_OK;
}

qgemm_status launch_w8a8_tcgen05_static(qgemm_stream_s* s, const void* A, const void* B, int b_kn,
                                        const float* sA, const float* sB, void* out, int out_dtype,
                                        int ldc, int M, int N, int K, int32_t* acc) {
  void* ws = nullptr;
  const qgemm_status st = static_scratch(s->dev, &ws);
  if (st != QGEMM_OK) return st;
  // the counters must be zero when the kernel starts
  const cudaError_t e = cudaMemsetAsync(ws, 0, STATIC_CNT_BYTES, s->stream);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the static scratch counters");
  TcArgs a = w8a8_args(A, B, b_kn, sA, sB, out, out_dtype, ldc, M, N, K, acc);
  a.scratch = ws;
  a.scratch_bytes = STATIC_SCRATCH_BYTES;
  return launch_tc_gemm(s, a);
}

}  // namespace qg
