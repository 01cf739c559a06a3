// w4a16_frag.cu -- W4A16 decode GEMV / skinny GEMM on fragment-ordered weights.
//
// Arithmetic (QuantizedGemmOps.scala:229-245 generalised to groups and a zero point):
//     y[m,n] = sum_g s[g,n] * sum_{k in g} (q[k,n] - zp) * x[m,k]
//
// Weight layout ("frag", made once by qgemm_prepack_w4_frag).  The unit is one
// 8-column group c times one 128-row block kb: 512 bytes, 16 per lane of a warp.
//     frag[c][kb][lane][step] (uint32), lane = 4g + t, step s = 0..3 (32 rows each)
// Word (c, kb, lane, s) holds the eight nibbles of column 8c+g at rows sb + 8t +
// {0, 4, 2, 6, 1, 5, 3, 7} (sb = 128kb + 32s), nibble i at bits 4i..4i+3, zero past
// K.  `(word >> 4i) & 0x000F000F | 0x43004300` is then, exactly, the bf16 pair 128+q
// of A-fragment register i of mma.m16n8k16 whose 16 rows are (column g, k half h).
// The MMA sums over k, so the k order is free as long as A and B share it: lane t's
// MMA k positions {2t, 2t+1, 2t+8, 2t+9} of half h are rows 8t + 4h + {0, 1, 2, 3},
// which makes each lane's activations for a step one contiguous run of x (a single
// vector load).  The B operand carries the matching halves of x: column n = 4h + m is
// activation row m over k half h, so one MMA covers 8 columns x 32 k for up to 4
// activation rows and the useful outputs are D[g][n] (h=0, t<2) and D[g+8][n]
// (h=1, t>=2).  An all-ones MMA gives sum_k x per (h, m), which seeds the weight
// MMAs' accumulator with -(128+zp) * sum x, so D = sum_k (q - zp) x directly.
//
// Grid: one CTA per SM; CTA i owns a contiguous run of 8-column groups (the counts
// differ by at most one), so every SM streams the same bytes.  A column group's
// units are one contiguous block (all of K), which is one stage of a shared-memory
// ring of about 64 KB: warp 16 copies it with a single 1-D bulk copy, starting
// before the programmatic-launch wait (weights never depend on the previous kernel).
// Warps 0-15 take the 128-row blocks w, w+16, .. of every stage and keep those
// blocks' activation fragments in registers; the CTA's scales (as fp32) sit in
// shared memory.  Per column group a warp's partial sums go to shared memory and the
// sixteen warps' partials are added in a fixed order (deterministic).  Every wait is
// bounded.
//
// Measured on B200 (legacy tensor path, integer pipe): mma.m16n8k16 issues once per
// 8 cycles per sub-partition; lop3 and shifts take 2 cycles a warp instruction and
// overlap with the MMAs (28 of them and 4 MMAs: ~67 cycles), while mul.hi is slower
// than a shift.  The dequantisation (4 lop3 + 3 shifts per word) and the per-stage
// bookkeeping set the pace, so the loop keeps integer division out of the stage
// counters, and 16 consumer warps (4 per sub-partition) hide the latencies better
// than 8.  M = 1, N = 14336, K = 4096: 8.6 us against 11.5 us for the 64-column-tile
// kernel (w4a16_tile.cu), which leaves 76 SMs with twice the work of the others.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "internal.h"
#include "ptx.cuh"

namespace qg {
namespace w4f {

constexpr int KB = 128;          // rows per block
constexpr int UNIT_U4 = 32;      // uint4 per unit (512 bytes)
constexpr int NCW = 16;          // consumer warps
constexpr int THREADS = 32 * (NCW + 1);
constexpr int MAX_STAGES = 8;
constexpr size_t RING_BYTES = 64 * 1024;  // ring target per CTA
constexpr int MP = 4;            // activation rows per pass
constexpr int MAX_NKB = 64;      // K <= 8192: a stage is at most 32 KB, KBW at most 4

struct Params {
  int M, N, K, G, zp;
  int NKB;            // 128-row blocks (K rounded up)
  int stages;         // ring stages (one column group each)
  int cbase, crem;    // CTA i owns cbase + (i < crem) column groups
  const uint4* w;     // frag layout
  const __nv_bfloat16* x;
  const __nv_bfloat16* s;
  __nv_bfloat16* y;
  int* err;
};

__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t mask, uint32_t bias) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(bias));
  return r;
}

// d += A * B (no side effects: the compiler may schedule it freely)
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// d = A * B + (c0, c1, c0, c1)
__device__ __forceinline__ void mma_bf16_init(float (&d)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1, float c0, float c1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1));
}

// Shared memory: the ring [stages][NKB * 512 B], the CTA's scales as fp32
// [K/G][Cg*8], the warps' partial sums [NCW][MP][Cg*8] (fp32), the barriers.
struct Smem {
  size_t ring, sc, red, bar, total;
};
__host__ __device__ inline Smem smem_layout(int nkb, int stages, int srows, int cg) {
  Smem m;
  m.ring = 0;
  m.sc = m.ring + (size_t)stages * nkb * 512;
  m.red = m.sc + ((size_t)srows * cg * 8 * 4 + 15) / 16 * 16;
  m.bar = m.red + (size_t)NCW * MP * (cg * 8 + 4) * 4;
  m.total = m.bar + 8 * 2 * MAX_STAGES + 16;
  return m;
}
__host__ __device__ inline int ring_stages(int nkb, int cg) {
  int st = (int)(RING_BYTES / ((size_t)nkb * 512));
  st = st < 2 ? 2 : st > MAX_STAGES ? MAX_STAGES : st;
  return st < cg ? st : (cg > 2 ? cg : 2);
}

// KBW: 128-row blocks per consumer warp (ceil(NKB / NCW)); GS: 32-row steps per scale
// group (1, 2 or 4: group 32, 64 or a multiple of 128); FULL: NKB == KBW * NCW, every
// warp's blocks exist and the stage loop has no per-block branch (5-9 % faster at
// M <= 4 on wide N: a run-time branch keeps the compiler from scheduling across blocks).
template <int KBW, int GS, bool FULL>
__global__ void __launch_bounds__(THREADS, 1) w4a16_frag_kernel(const Params p) {
  constexpr int NQ = 4 / GS;  // scale groups per unit
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int cta = blockIdx.x;
  const int c0 = cta * p.cbase + (cta < p.crem ? cta : p.crem);
  const int Cg = p.cbase + (cta < p.crem ? 1 : 0);
  const int ncol = Cg * 8;
  const int srows = p.K / p.G;
  const int STAGES = p.stages;
  const Smem L = smem_layout(p.NKB, STAGES, srows, Cg);
  const uint4* ring = reinterpret_cast<const uint4*>(smem + L.ring);
  float* scf = reinterpret_cast<float*>(smem + L.sc);
  float* red = reinterpret_cast<float*>(smem + L.red);
  const uint32_t bar = ptx::smem_u32(smem + L.bar);
  auto full_bar = [&](int s) { return bar + 8u * s; };
  auto empty_bar = [&](int s) { return bar + 8u * (MAX_STAGES + s); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.bar + 8 * 2 * MAX_STAGES);
  const uint32_t stage_bytes = (uint32_t)p.NKB * 512u;

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

  if (warp == NCW) {
    // ---------------- producer: one bulk copy per column group ----------------
    if (lane == 0) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(p.w) + (size_t)c0 * stage_bytes;
      const uint32_t ring0 = ptx::smem_u32(smem + L.ring);
      int issued = 0, st = 0;
      uint32_t ph = 0;  // parity of the ring lap
      for (int c = 0; c < Cg; ++c) {
        if (c >= STAGES && !ptx::mbar_wait_sleep(empty_bar(st), ph ^ 1u, abort_flag)) {
          if (!*abort_flag) { *abort_flag = 1; if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_PRODUCER); }
          break;
        }
        ptx::mbar_arrive_expect_tx(full_bar(st), stage_bytes);
        ptx::bulk_load(ring0 + st * stage_bytes, src + (size_t)c * stage_bytes, stage_bytes,
                       full_bar(st));
        ++issued;
        if (++st == STAGES) { st = 0; ph ^= 1u; }
      }
      // the copies in flight land before the CTA may exit
      for (int c = (issued > STAGES ? issued - STAGES : 0); c < issued; ++c) {
        if (!ptx::mbar_wait(full_bar(c % STAGES), (uint32_t)((c / STAGES) & 1), nullptr)) {
          if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_DRAIN);
          break;
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int ctid = threadIdx.x;  // 0 .. 32*NCW-1
  // the CTA's scales, widened to fp32 (no dependence on the previous kernel)
  for (int i = ctid; i < srows * Cg; i += 32 * NCW) {
    const int r = i / Cg, c = i - r * Cg;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.s) + ((size_t)r * p.N + (size_t)(c0 + c) * 8) / 8);
    float4* d = reinterpret_cast<float4*>(scf + (size_t)r * ncol + c * 8);
    d[0] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                       __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
    d[1] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u),
                       __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u));
  }
  ptx::named_bar_sync(1, 32 * NCW);

  const float zc = 128.0f + (float)p.zp;
  const uint32_t MASK = 0x000F000Fu, BIAS = 0x43004300u, ONES = 0x3F803F80u;
  int kbj[KBW];
  bool vj[KBW];
  uint32_t bx[KBW][8];   // B fragments: register (e & 1) of 32-row step e/2
  float zs[KBW][NQ][2];  // -(128+zp) * sum_k x per scale group of this warp's blocks
  int srow[KBW][NQ];
#pragma unroll
  for (int j = 0; j < KBW; ++j) {
    kbj[j] = warp + j * NCW;
    vj[j] = kbj[j] < p.NKB;
  }
  // activations may be written by the previous kernel in the stream
  ptx::grid_dependency_wait();
  {
    const int m = g & 3, h = g >> 2;  // B column n = 4h + m: activation row m, k half h
#pragma unroll
    for (int j = 0; j < KBW; ++j)
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        // rows 8t + 4h .. +3 of the step: both B registers in one 8-byte load
        const int k = kbj[j] * KB + s * 32 + 8 * t + 4 * h;
        // K % 16 == 0: a lane's 8 rows of a step lie wholly inside or wholly past K
        uint2 v = make_uint2(0u, 0u);
        if (vj[j] && m < p.M && k < p.K)
          v = __ldg(reinterpret_cast<const uint2*>(p.x + (size_t)m * p.K + k));
        bx[j][2 * s] = v.x;
        bx[j][2 * s + 1] = v.y;
      }
  }
#pragma unroll
  for (int j = 0; j < KBW; ++j) {
    const int kb = vj[j] ? kbj[j] : 0;
    const uint32_t* b = bx[j];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = q * GS; s < q * GS + GS; ++s)
        mma_bf16(d, ONES, ONES, ONES, ONES, b[2 * s], b[2 * s + 1]);
      zs[j][q][0] = -zc * d[0];
      zs[j][q][1] = -zc * d[1];
      const int r = (kb * KB + q * GS * 32) / p.G;
      srow[j][q] = (r < srows ? r : 0) * ncol + g;
    }
  }

  const int rs4 = ncol + 4;  // partial-sum row stride: rows 2t apart on different banks
  float* redw = red + (size_t)warp * MP * rs4;
  int st = 0;
  uint32_t ph = 0;  // parity of the ring lap
  for (int c = 0; c < Cg; ++c) {
    const bool ok = ptx::mbar_wait_sleep(full_bar(st), ph, abort_flag);
    if (!ok) {
      if (!*abort_flag) { *abort_flag = 1; if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_EPILOGUE); }
      break;
    }
    const uint4* rs = ring + st * (p.NKB * UNIT_U4) + lane;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < KBW; ++j) {
      if (FULL || vj[j]) {
        const uint4 wv = rs[kbj[j] * UNIT_U4];
        const uint32_t* b = bx[j];
        const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
          float d[4];
#pragma unroll
          for (int s = q * GS; s < q * GS + GS; ++s) {
            const uint32_t w = wd[s];
            const uint32_t a0 = and_or(w, MASK, BIAS), a1 = and_or(w >> 4, MASK, BIAS);
            const uint32_t a2 = and_or(w >> 8, MASK, BIAS), a3 = and_or(w >> 12, MASK, BIAS);
            if (s == q * GS)
              mma_bf16_init(d, a0, a1, a2, a3, b[2 * s], b[2 * s + 1], zs[j][q][0], zs[j][q][1]);
            else
              mma_bf16(d, a0, a1, a2, a3, b[2 * s], b[2 * s + 1]);
          }
          const float sc = scf[srow[j][q] + c * 8];
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[e] = fmaf(sc, d[e], acc[e]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(empty_bar(st));
    if (++st == STAGES) { st = 0; ph ^= 1u; }
    // this lane's useful outputs: rows g (first k half, t < 2) or rows g+8 (second k
    // half, t >= 2); then first half + second half (lanes t, t+2)
    const float u0 = t >= 2 ? acc[2] : acc[0], u1 = t >= 2 ? acc[3] : acc[1];
    const float v0 = u0 + __shfl_down_sync(0xffffffffu, u0, 2);
    const float v1 = u1 + __shfl_down_sync(0xffffffffu, u1, 2);
    if (t < 2) {
      redw[(2 * t) * rs4 + c * 8 + g] = v0;
      redw[(2 * t + 1) * rs4 + c * 8 + g] = v1;
    }
  }
  ptx::named_bar_sync(1, 32 * NCW);
  if (*abort_flag) return;
  for (int idx = ctid; idx < p.M * ncol; idx += 32 * NCW) {
    const int m = idx / ncol, r = idx - m * ncol;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) s += red[((size_t)w * MP + m) * rs4 + r];
    p.y[(size_t)m * p.N + (size_t)c0 * 8 + r] = __float2bfloat16_rn(s);
  }
}

// ---- 5 to 16 activation rows: 16-column pairs --------------------------------------
// The same layout read as column pairs (groups 2p, 2p+1 are adjacent, so a pair's
// whole K is one contiguous block): the MMA rows are 16 columns, A of the first k
// half of a step is (lop3 w0, lop3 w1, lop3 w0>>8, lop3 w1>>8) and of the second
// (lop3 w0>>4, lop3 w1>>4, lop3 w0>>12, lop3 w1>>12), B is up to 8 activation rows
// per n tile, NB tiles.  Each dequantised word feeds 2 NB MMAs, so the weights are
// read once for 16 rows.  CTA i owns a contiguous run of pairs; warps take 128-row
// blocks as in the kernel above; the activation fragments (16 NB registers per block)
// stay in registers.  There is no producer warp (16 warps keep 128 registers a
// thread; a 17th would cap them at 96): thread 0 issues the first stages, and the
// warp that releases a stage last (an atomic count per stage) issues its refill.
__host__ __device__ inline Smem smem_layout16(int nkb, int stages, int srows, int ncol, int mr) {
  Smem m;
  m.ring = 0;
  m.sc = m.ring + (size_t)stages * nkb * 1024;
  m.red = m.sc + ((size_t)srows * ncol * 4 + 15) / 16 * 16;
  m.bar = m.red + (size_t)NCW * mr * (ncol + 4) * 4;
  m.total = m.bar + 8 * MAX_STAGES + 4 * 2 * MAX_STAGES + 16;
  return m;
}

template <int NB, int KBW, int GS>
__global__ void __launch_bounds__(32 * NCW, 1) w4a16_frag16_kernel(const Params p) {
  constexpr int NQ = 4 / GS;
  constexpr int MR = 8 * NB;  // activation rows of this pass (at most)
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int cta = blockIdx.x;
  const int c0p = cta * p.cbase + (cta < p.crem ? cta : p.crem);  // first pair
  const int Pg = p.cbase + (cta < p.crem ? 1 : 0);                  // pairs of this CTA
  const int ncol = Pg * 16;
  const int srows = p.K / p.G;
  const int STAGES = p.stages;
  const Smem L = smem_layout16(p.NKB, STAGES, srows, ncol, MR);
  const uint4* ring = reinterpret_cast<const uint4*>(smem + L.ring);
  float* scf = reinterpret_cast<float*>(smem + L.sc);
  float* red = reinterpret_cast<float*>(smem + L.red);
  const uint32_t bar = ptx::smem_u32(smem + L.bar);
  auto full_bar = [&](int s) { return bar + 8u * s; };
  int* released = reinterpret_cast<int*>(smem + L.bar + 8 * MAX_STAGES);  // per stage, never reset
  int* laps = released + MAX_STAGES;                                      // copies issued per stage
  volatile int* abort_flag = laps + MAX_STAGES;
  const uint32_t stage_bytes = (uint32_t)p.NKB * 1024u;
  const uint8_t* src = reinterpret_cast<const uint8_t*>(p.w) + (size_t)c0p * stage_bytes;
  const uint32_t ring0 = ptx::smem_u32(smem + L.ring);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      released[s] = 0;
      laps[s] = 0;
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::grid_launch_dependents();
    // the first stages, before the programmatic-launch wait
    for (int c = 0; c < STAGES && c < Pg; ++c) {
      ptx::mbar_arrive_expect_tx(full_bar(c), stage_bytes);
      ptx::bulk_load(ring0 + c * stage_bytes, src + (size_t)c * stage_bytes, stage_bytes,
                     full_bar(c));
      laps[c] = 1;
    }
  }
  __syncthreads();

  const int ctid = threadIdx.x;
  const int Cg = 2 * Pg, c0 = 2 * c0p;  // column groups of this CTA
  for (int i = ctid; i < srows * Cg; i += 32 * NCW) {
    const int r = i / Cg, c = i - r * Cg;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.s) + ((size_t)r * p.N + (size_t)(c0 + c) * 8) / 8);
    float4* d = reinterpret_cast<float4*>(scf + (size_t)r * ncol + c * 8);
    d[0] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                       __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
    d[1] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u),
                       __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u));
  }
  ptx::named_bar_sync(1, 32 * NCW);

  const float zc = 128.0f + (float)p.zp;
  const uint32_t MASK = 0x000F000Fu, BIAS = 0x43004300u, ONES = 0x3F803F80u;
  int kbj[KBW];
  bool vj[KBW];
  uint32_t bx[KBW][4][2][NB][2];  // [block][step][k half][n tile][register]
  float zs[KBW][NQ][NB][2];
  int srow[KBW][NQ];
#pragma unroll
  for (int j = 0; j < KBW; ++j) {
    kbj[j] = warp + j * NCW;
    vj[j] = kbj[j] < p.NKB;
  }
  ptx::grid_dependency_wait();
#pragma unroll
  for (int j = 0; j < KBW; ++j)
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        // rows 8t .. 8t+7 of the step: both k halves' B registers in one 16-byte load
        const int m = 8 * nb + g;
        const int k = kbj[j] * KB + s * 32 + 8 * t;
        // K % 16 == 0: a lane's 8 rows of a step lie wholly inside or wholly past K
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (vj[j] && m < p.M && k < p.K)
          v = __ldg(reinterpret_cast<const uint4*>(p.x + (size_t)m * p.K + k));
        bx[j][s][0][nb][0] = v.x;
        bx[j][s][0][nb][1] = v.y;
        bx[j][s][1][nb][0] = v.z;
        bx[j][s][1][nb][1] = v.w;
      }
#pragma unroll
  for (int j = 0; j < KBW; ++j) {
    const int kb = vj[j] ? kbj[j] : 0;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = q * GS; s < q * GS + GS; ++s)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            mma_bf16(d, ONES, ONES, ONES, ONES, bx[j][s][h][nb][0], bx[j][s][h][nb][1]);
        zs[j][q][nb][0] = -zc * d[0];
        zs[j][q][nb][1] = -zc * d[1];
      }
      const int r = (kb * KB + q * GS * 32) / p.G;
      srow[j][q] = (r < srows ? r : 0) * ncol + g;
    }
  }

  const int rs4 = ncol + 4;  // partial-sum row stride: rows 2t apart on different banks
  float* redw = red + (size_t)warp * MR * rs4;
  int st = 0;
  uint32_t ph = 0;
  for (int c = 0; c < Pg; ++c) {
    const bool ok = ptx::mbar_wait_sleep(full_bar(st), ph, abort_flag);
    if (!ok) {
      if (!*abort_flag) { *abort_flag = 1; if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_EPILOGUE); }
      break;
    }
    const uint4* rs = ring + st * (p.NKB * 2 * UNIT_U4) + lane;
    float acc[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nb][e] = 0.f;
#pragma unroll
    for (int j = 0; j < KBW; ++j) {
      if (vj[j]) {
        const uint4 v0 = rs[kbj[j] * UNIT_U4], v1 = rs[(p.NKB + kbj[j]) * UNIT_U4];
        const uint32_t w0s[4] = {v0.x, v0.y, v0.z, v0.w}, w1s[4] = {v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
          float d[NB][4];
#pragma unroll
          for (int s = q * GS; s < q * GS + GS; ++s) {
            const uint32_t w0 = w0s[s], w1 = w1s[s];
            const uint32_t l0 = and_or(w0, MASK, BIAS), l1 = and_or(w1, MASK, BIAS);
            const uint32_t l2 = and_or(w0 >> 8, MASK, BIAS), l3 = and_or(w1 >> 8, MASK, BIAS);
            const uint32_t h0 = and_or(w0 >> 4, MASK, BIAS), h1 = and_or(w1 >> 4, MASK, BIAS);
            const uint32_t h2 = and_or(w0 >> 12, MASK, BIAS), h3 = and_or(w1 >> 12, MASK, BIAS);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
              if (s == q * GS)
                mma_bf16_init(d[nb], l0, l1, l2, l3, bx[j][s][0][nb][0], bx[j][s][0][nb][1],
                              zs[j][q][nb][0], zs[j][q][nb][1]);
              else
                mma_bf16(d[nb], l0, l1, l2, l3, bx[j][s][0][nb][0], bx[j][s][0][nb][1]);
              mma_bf16(d[nb], h0, h1, h2, h3, bx[j][s][1][nb][0], bx[j][s][1][nb][1]);
            }
          }
          const float s0 = scf[srow[j][q] + c * 16], s1 = scf[srow[j][q] + c * 16 + 8];
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            acc[nb][0] = fmaf(s0, d[nb][0], acc[nb][0]);
            acc[nb][1] = fmaf(s0, d[nb][1], acc[nb][1]);
            acc[nb][2] = fmaf(s1, d[nb][2], acc[nb][2]);
            acc[nb][3] = fmaf(s1, d[nb][3], acc[nb][3]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      // this warp's reads of the stage are done; the last of the NCW releases refills it
      __threadfence_block();
      if (atomicAdd(&released[st], 1) % NCW == NCW - 1 && c + STAGES < Pg) {
        __threadfence_block();
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive_expect_tx(full_bar(st), stage_bytes);
        ptx::bulk_load(ring0 + st * stage_bytes, src + (size_t)(c + STAGES) * stage_bytes,
                       stage_bytes, full_bar(st));
        laps[st] += 1;
      }
    }
    if (++st == STAGES) { st = 0; ph ^= 1u; }
    // D rows g / g+8 are columns 16c+g / 16c+8+g; D columns 2t, 2t+1 are rows 8nb+2t(+1)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      float* r0 = redw + (size_t)(8 * nb + 2 * t) * rs4 + c * 16 + g;
      r0[0] = acc[nb][0];
      r0[rs4] = acc[nb][1];
      r0[8] = acc[nb][2];
      r0[rs4 + 8] = acc[nb][3];
    }
  }
  ptx::named_bar_sync(1, 32 * NCW);
  if (*abort_flag) {
    // copies still in flight land before the CTA exits
    if (ctid == 0)
      for (int s = 0; s < STAGES; ++s)
        if (laps[s] > 0 &&
            !ptx::mbar_wait(full_bar(s), (uint32_t)((laps[s] - 1) & 1), nullptr) && p.err)
          atomicCAS(p.err, 0, DEVERR_TIMEOUT_DRAIN);
    return;
  }
  for (int idx = ctid; idx < p.M * ncol; idx += 32 * NCW) {
    const int m = idx / ncol, r = idx - m * ncol;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) s += red[((size_t)w * MR + m) * rs4 + r];
    p.y[(size_t)m * p.N + (size_t)c0 * 8 + r] = __float2bfloat16_rn(s);
  }
}

// NB = 0: the 8-column kernel; NB = -1: the same with every block present (FULL)
template <int NB, int KBW, int GS>
static qgemm_status launch_one(qgemm_stream_s* s, const Params& p, int grid, size_t smem) {
  void (*kern)(const Params) =
      NB == 0    ? w4a16_frag_kernel<KBW, GS, false>
      : NB == -1 ? w4a16_frag_kernel<KBW, GS, true>
                 : w4a16_frag16_kernel<NB <= 0 ? 1 : NB, KBW, GS>;
  static bool attr_done[64] = {};
  const int ord = s->dev->ordinal;
  if (ord < 0 || ord >= 64 || !attr_done[ord]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)s->dev->smem_optin);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a16_frag)");
    if (ord >= 0 && ord < 64) attr_done[ord] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(NB <= 0 ? THREADS : 32 * NCW, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_fail(cudaLaunchKernelEx(&cfg, kern, p), "w4a16_frag_kernel launch");
}

// NB = 0 / -1: the 8-column kernel (at most 4 rows; -1: every block present); NB = 1, 2:
// column pairs, 8 NB rows
template <int NB, int KBW>
static qgemm_status launch_kbw(qgemm_stream_s* s, const Params& p, int gs, int grid,
                               size_t smem) {
  return gs == 1 ? launch_one<NB, KBW, 1>(s, p, grid, smem)
       : gs == 2 ? launch_one<NB, KBW, 2>(s, p, grid, smem)
                 : launch_one<NB, KBW, 4>(s, p, grid, smem);
}

template <int NB>
static qgemm_status launch_nb(qgemm_stream_s* s, const Params& p, int kbw, int gs, int grid,
                              size_t smem) {
  return kbw == 1 ? launch_kbw<NB, 1>(s, p, gs, grid, smem)
       : kbw == 2 ? launch_kbw<NB, 2>(s, p, gs, grid, smem)
                  : launch_kbw<NB, 4>(s, p, gs, grid, smem);
}

// 128-row blocks per consumer warp: 1, 2 or 4 (0: K too large)
static int kbw_for(int K) {
  const int nkb = (K + KB - 1) / KB;
  if (nkb > MAX_NKB) return 0;
  const int kbw = (nkb + NCW - 1) / NCW;
  return kbw <= 1 ? 1 : kbw <= 2 ? 2 : 4;
}

// the pair kernel's ring: as many stages of two column groups as the target allows
static int ring_stages16(int nkb, int pmax) { return ring_stages(2 * nkb, pmax); }

}  // namespace w4f

size_t w4_frag_bytes(int K, int N) {
  return (size_t)(N / 8) * (size_t)((K + w4f::KB - 1) / w4f::KB) * 512;
}

bool w4a16_frag_supported(const qgemm_device_s* d, uint64_t x, uint64_t wf, uint64_t sc, int M,
                          int N, int K, int G, const char** why) {
  auto no = [&](const char* w) { if (why) *why = w; return false; };
  if (!d->tcgen05) return no("device is not sm_100");
  if (K % 16 != 0) return no("K must be a multiple of 16");
  if (!(G == 32 || G == 64 || G % 128 == 0)) return no("group_size must be 32, 64 or a multiple of 128");
  if (N % 8 != 0) return no("N must be a multiple of 8");
  if (w4f::kbw_for(K) == 0 && !w4a16_frag_cluster_fits(N, K))
    return no("K must be at most 8192, or at most 16384 with N a multiple of 16");
  if (!aligned(x, 16) || !aligned(wf, 16) || !aligned(sc, 16))
    return no("x, weights and scales must be 16-byte aligned");
  (void)M;
  return true;
}

qgemm_status launch_w4a16_frag(qgemm_stream_s* s, const void* x, const void* wf, const void* sc,
                               int zp, int G, void* y, int M, int N, int K) {
  using namespace w4f;
  qgemm_device_s* d = s->dev;
  const int sms = d->sm_count;
  const int nkb = (K + KB - 1) / KB, srows = K / G;
  const int kbw = kbw_for(K);
  const int gs = G == 32 ? 1 : G == 64 ? 2 : 4;
  const __nv_bfloat16* x16 = static_cast<const __nv_bfloat16*>(x);
  __nv_bfloat16* y16 = static_cast<__nv_bfloat16*>(y);
  const __nv_bfloat16* s16 = static_cast<const __nv_bfloat16*>(sc);
  const uint4* w4 = static_cast<const uint4*>(wf);
  Params p;
  p.N = N; p.K = K; p.G = G; p.zp = zp;
  p.NKB = nkb;
  p.err = d->d_err;
  // The columns go out in chunks of at most (SMs x a width whose shared memory fits);
  // one chunk unless N is very wide.
  auto widest = [&](int want, auto smem_of) {
    while (want > 1 && smem_of(want) > d->smem_optin) --want;
    return want;
  };
  // 17 to 32 rows a pass, or K past the register-resident kernels' limit: the K-split
  // cluster kernel (w4a16_frag_cluster.cu) reads the weights once per 32 rows
  if (w4a16_frag_cluster_fits(N, K) && (M > 16 || kbw == 0 || (M > MP && kbw > 2)))
    return launch_w4a16_frag_cluster(s, x, wf, sc, zp, G, y, M, N, K);
  if (M > MP && N % 16 == 0 && kbw <= 2) {
    // more than 4 rows: 16-row passes on column pairs (weights read once per 16 rows)
    const int NP = N / 16;
    const int g0 = NP < sms ? NP : sms;
    const int wmax = widest((NP + g0 - 1) / g0, [&](int w) {
      return smem_layout16(nkb, ring_stages16(nkb, w), srows, 16 * w, 16).total;
    });
    for (int p0 = 0; p0 < NP; p0 += sms * wmax) {
      const int np = (NP - p0) < sms * wmax ? (NP - p0) : sms * wmax;
      const int grid = np < sms ? np : sms;
      Params q = p;
      q.cbase = np / grid;
      q.crem = np % grid;
      const int pmax = q.cbase + (q.crem > 0 ? 1 : 0);
      q.stages = ring_stages16(nkb, pmax);
      q.w = w4 + (size_t)p0 * 2 * nkb * UNIT_U4;
      q.s = s16 + (size_t)p0 * 16;
      for (int m0 = 0; m0 < M; m0 += 16) {
        q.M = (M - m0) < 16 ? (M - m0) : 16;
        q.x = x16 + (size_t)m0 * K;
        q.y = y16 + (size_t)m0 * N + (size_t)p0 * 16;
        const int nb = q.M > 8 ? 2 : 1;
        const size_t sm = smem_layout16(nkb, q.stages, srows, 16 * pmax, 8 * nb).total;
        qgemm_status st = nb == 2 ? launch_nb<2>(s, q, kbw, gs, grid, sm)
                                  : launch_nb<1>(s, q, kbw, gs, grid, sm);
        if (st != QGEMM_OK) return st;
      }
    }
    return QGEMM_OK;
  }
  const int NG = N / 8;
  const int g0 = NG < sms ? NG : sms;
  const int wmax = widest((NG + g0 - 1) / g0, [&](int w) {
    return smem_layout(nkb, ring_stages(nkb, w), srows, w).total;
  });
  for (int c0 = 0; c0 < NG; c0 += sms * wmax) {
    const int ng = (NG - c0) < sms * wmax ? (NG - c0) : sms * wmax;
    const int grid = ng < sms ? ng : sms;
    p.cbase = ng / grid;
    p.crem = ng % grid;
    const int cmax = p.cbase + (p.crem > 0 ? 1 : 0);
    p.stages = ring_stages(nkb, cmax);
    p.w = w4 + (size_t)c0 * nkb * UNIT_U4;
    p.s = s16 + (size_t)c0 * 8;
    const size_t sm = smem_layout(nkb, p.stages, srows, cmax).total;
    for (int m0 = 0; m0 < M; m0 += MP) {
      p.M = (M - m0) < MP ? (M - m0) : MP;
      p.x = x16 + (size_t)m0 * K;
      p.y = y16 + (size_t)m0 * N + (size_t)c0 * 8;
      qgemm_status st = nkb == kbw * NCW ? launch_nb<-1>(s, p, kbw, gs, grid, sm)
                                         : launch_nb<0>(s, p, kbw, gs, grid, sm);
      if (st != QGEMM_OK) return st;
    }
  }
  return QGEMM_OK;
}

// ---- one-time weight repack: reference words -> fragment-ordered units ----------
// dst word ((c * NKB + kb) * 32 + lane) * 4 + s; see the layout comment at the top.
__global__ void prepack_w4_frag_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst,
                                       int K, int N, int NKB) {
  const int NG = N / 8;
  const size_t total = (size_t)NG * NKB * 128;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int s = (int)(i & 3), lane = (int)((i >> 2) & 31);
    const size_t unit = i >> 7;
    const int kb = (int)(unit % NKB), c = (int)(unit / NKB);
    const int g = lane >> 2, t = lane & 3;
    const int sb = kb * w4f::KB + s * 32;
    const int r0 = sb + 8 * t;
    const int ks[8] = {r0 + 0, r0 + 4, r0 + 2, r0 + 6, r0 + 1, r0 + 5, r0 + 3, r0 + 7};
    uint32_t v = 0;
#pragma unroll
    for (int n = 0; n < 8; ++n)
      if (ks[n] < K) v |= ((src[(size_t)ks[n] * NG + c] >> (4 * g)) & 0xFu) << (4 * n);
    dst[i] = v;
  }
}

qgemm_status launch_prepack_w4_frag(qgemm_stream_s* s, const uint32_t* src, uint32_t* dst, int K,
                                    int N) {
  const int NKB = (K + w4f::KB - 1) / w4f::KB;
  const int grid = s->dev->sm_count * 8;
  prepack_w4_frag_kernel<<<grid, 256, 0, s->stream>>>(src, dst, K, N, NKB);
  return cuda_fail(cudaGetLastError(), "prepack_w4_frag launch");
}

}  // namespace qg
