// w4a16_frag_cluster.cu -- W4A16 skinny GEMM (up to 32 activation rows per pass) on
// fragment-ordered weights, with K split across the CTAs of a thread-block cluster.
//
// Arithmetic (QuantizedGemmOps.scala:229-245 generalised to groups and a zero point):
//     y[m,n] = sum_g s[g,n] * sum_{k in g} (q[k,n] - zp) * x[m,k]
//
// Weight layout: the fragment order of w4a16_frag.cu (unit (c, kb) = columns 8c..8c+7 x
// rows 128kb..128kb+127, 512 bytes at ((c * NKB) + kb) * 512; lane 4g+t's word s holds
// column 8c+g at rows 128kb + 32s + 8t + {0, 4, 2, 6, 1, 5, 3, 7}, nibble i at bits
// 4i).  As in w4a16_frag16_kernel, two column groups (2p, 2p+1) are the 16 A rows of
// mma.m16n8k16 and the activations are B, 8 rows per n tile, NB tiles.
//
// Decomposition:
//   * K is cut into S slices of whole 128-row blocks, one per CTA of a cluster of S
//     (S <= 8); the clusters split the columns in contiguous runs of column pairs.
//   * A CTA keeps its slice's activations (8 NB rows) in shared memory in fragment
//     order: the B registers of one (block, step, n tile) are one 16-byte load per lane
//     from 512 contiguous bytes, free of bank conflicts.
//   * Each of the 8 warps owns NP (1 to 4, a template parameter) of the CTA's 8 NP
//     column pairs over the whole slice and keeps their fp32 sums in registers, so no
//     partial sum crosses warps; every B fragment it loads feeds 2 NP MMAs per 8-row
//     tile.  Every warp has the same work (a warp with more pairs than the others would
//     set the pace, the loop being latency-bound at a few pairs a warp), and NP is known
//     to the compiler (the loop has no branches: 10.4 cycles per MMA per sub-partition
//     at NP = 3 against 13.3 with a run-time pair count, measured in isolation).  The
//     last cluster's pairs past N read zeros (TMA fills past the tensor) and are not
//     stored.  The weights are read from HBM once for all 32 rows.
//   * The slice streams one 128-row block of all the CTA's column groups per ring
//     stage: one 3-D TMA tile (512 bytes x 1 block x 2 * pairs).  There is no producer
//     warp (a ninth warp would put three warps on one sub-partition and cap registers at
//     168; the 32-row form needs ~200): thread 0 issues the first stages, and the warp
//     that releases a stage last (an atomic count per stage) issues its refill.
//   * Seeds: an all-ones MMA gives sum_k x per (block, scale group, row); it seeds each
//     group's MMA chain with -(128+zp) * sum x, so the chain sums (q - zp) x exactly as
//     in the other frag kernels, and the group's scale multiplies it in fp32.
//   * The S partial sums of an output meet through distributed shared memory: after a
//     cluster barrier, CTA r adds, in rank order, the partials of its 1/S share of the
//     cluster's columns from all S CTAs and writes bf16.  The order is fixed, so the
//     result does not depend on timing.
// The mma.sync tensor path issues one m16n8k16 per 8 cycles per sub-partition, so at
// 32 rows the MMAs (not HBM) set the pace: 2 * 32 * K * N / 4096 MMAs.
// Every mbarrier wait is bounded; the cluster barriers are reached by every thread on
// every path (a timed-out wait skips work, never a barrier).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <tuple>

#include "internal.h"
#include "ptx.cuh"

namespace qg {
namespace w4c {

constexpr int KB = 128;          // rows per block
constexpr int NCW = 8;           // warps
constexpr int THREADS = 32 * NCW;
constexpr int PMAX = 4;          // column pairs per warp, at most
constexpr int MAX_S = 8;         // K slices (cluster size), at most
constexpr int MAX_STAGES = 8;
constexpr int NBLK_MAX = 16;     // 128-row blocks per slice, at most
constexpr int MAX_NB = 4;        // 32 activation rows per pass

struct Params {
  int M, N, K, G, zp;
  int NKB, S;
  int nblk_max, npc_max, nsr_max;  // shared-memory layout sizes (the same in every CTA)
  int stages;
  int pair0, pair1;                // column pairs [pair0, pair1) of this launch
  int y_vec;                       // y rows are 8-byte aligned
  unsigned long long wait_ns;
  const __nv_bfloat16* x;
  const __nv_bfloat16* s;
  __nv_bfloat16* y;
  int* err;
};

__host__ __device__ inline size_t up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Shared memory: activations [nblk_max][4 steps][NB][32 lanes] uint4, the slice's
// scales (bf16) [nsr_max][npc_max * 16], seeds [nblk_max][NQ][32] fp32, the weight
// ring [stages][2 * npc_max units of 512 B]; after the main loop the partial sums
// [8 NB rows][npc_max * 16 + 4] fp32 reuse the space from offset 0; last the full
// barriers, the per-stage release counts and copy counts, and the abort flag.
struct Smem {
  size_t xs, sc, sx, ring, red, bar, total;
};
__host__ __device__ inline Smem smem_layout(int nb, int nq, int nblk_max, int npc_max,
                                            int nsr_max, int stages) {
  Smem m;
  m.xs = 0;
  m.sc = m.xs + (size_t)nblk_max * 4 * nb * 512;
  m.sx = m.sc + up((size_t)nsr_max * npc_max * 16 * 2, 16);
  m.ring = up(m.sx + (size_t)nblk_max * nq * 32 * 4, 128);
  const size_t main_end = m.ring + (size_t)stages * npc_max * 1024;
  m.red = 0;
  const size_t red_end = (size_t)8 * nb * (npc_max * 16 + 4) * 4;
  m.bar = up(main_end > red_end ? main_end : red_end, 16);
  m.total = m.bar + 8 * MAX_STAGES + 4 * 2 * MAX_STAGES + 16;
  return m;
}

__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t mask, uint32_t bias) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(bias));
  return r;
}

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

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t v) {
  return __uint_as_float((uint32_t)v << 16);
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int s) {
  return s == 0 ? v.x : s == 1 ? v.y : s == 2 ? v.z : v.w;
}

// NB: 8-row activation tiles (1, 2 or 4); NP: column pairs per warp; GS: 32-row steps
// per scale group (1, 2 or 4: group 32, 64 or a multiple of 128).
template <int NB, int NP, int GS>
__global__ void __launch_bounds__(THREADS, 1)
    w4a16_frag_cluster_kernel(const __grid_constant__ CUtensorMap tmW, const Params p) {
  constexpr int NQ = 4 / GS;  // scale groups per block
  constexpr int MR = 8 * NB;  // activation rows of this pass (at most)
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int S = p.S;
  const int rank = (int)ptx::cluster_ctarank();  // K slice
  constexpr int npc = NCW * NP;                  // column pairs of this CTA
  const int p0 = p.pair0 + blockIdx.x * npc;      // its first pair
  const int preal = (p.pair1 - p0) < npc ? (p.pair1 - p0) : npc;  // pairs inside the launch
  const int kb0 = (int)((long long)rank * p.NKB / S);
  const int kb1 = (int)((long long)(rank + 1) * p.NKB / S);
  const int nblk = kb1 - kb0;
  const int gr0 = kb0 * KB / p.G;     // first scale row of the slice
  const int ncs = p.npc_max * 16;     // scale row stride (bf16)
  const int rs = p.npc_max * 16 + 4;  // partial-sum row stride (fp32)
  const Smem L = smem_layout(NB, NQ, p.nblk_max, p.npc_max, p.nsr_max, p.stages);
  const uint4* xs = reinterpret_cast<const uint4*>(smem + L.xs);
  uint16_t* scs = reinterpret_cast<uint16_t*>(smem + L.sc);
  float* sx = reinterpret_cast<float*>(smem + L.sx);
  const uint4* ring = reinterpret_cast<const uint4*>(smem + L.ring);
  float* red = reinterpret_cast<float*>(smem + L.red);
  const uint32_t bar = ptx::smem_u32(smem + L.bar);
  auto full_bar = [&](int s) { return bar + 8u * s; };
  int* released = reinterpret_cast<int*>(smem + L.bar + 8 * MAX_STAGES);  // per stage, never reset
  int* laps = released + MAX_STAGES;                                      // copies issued per stage
  volatile int* abort_flag = laps + MAX_STAGES;
  const uint32_t stage_bytes = (uint32_t)p.npc_max * 1024u;  // 2 npc_max units of 512 B
  const int STAGES = p.stages;
  const uint32_t ring0 = ptx::smem_u32(smem + L.ring);
  const int gz = 2 * p0;              // first column group of the cluster's run

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      released[s] = 0;
      laps[s] = 0;
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::grid_launch_dependents();
    ptx::prefetch_tmap(&tmW);
  }
  __syncthreads();
  // the first stages, one per warp (lane 0 of warp j issues stage j: a TMA issue holds
  // its thread for some 150 ns, and the warps' fills below wait for the slowest warp);
  // weights never depend on the previous kernel, so this precedes the launch wait
  for (int j = warp; j < STAGES && j < nblk; j += NCW) {
    if (lane == 0) {
      ptx::mbar_arrive_expect_tx(full_bar(j), stage_bytes);
      ptx::tma_load_3d(ring0 + j * stage_bytes, &tmW, full_bar(j), 0, kb0 + j, gz);
      laps[j] = 1;
    }
  }

  float acc[NP][NB][4];
#pragma unroll
  for (int i = 0; i < NP; ++i)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][nb][e] = 0.f;
  const int pw0 = warp * NP;  // this warp's first pair within the CTA

  {
    // ---------------- consumers (all warps) ----------------
    const int ctid = threadIdx.x;  // 0 .. 32*NCW-1
    // the slice's scale rows for the cluster's columns, as bf16 (independent of the
    // previous kernel)
    {
      const int klast = (kb1 * KB < p.K ? kb1 * KB : p.K) - 1;
      const int nsr = klast / p.G - gr0 + 1;
      constexpr int c8 = npc * 2;  // 8-column pieces per row (zeros past the launch)
      const int c8real = preal * 2;
      const __nv_bfloat16* sbase = p.s + (size_t)p0 * 16;
      const uint32_t sc0 = ptx::smem_u32(scs);
      for (int i = ctid; i < nsr * c8; i += 32 * NCW) {
        const int r = i / c8, c = i - r * c8;
        const bool in = c < c8real;
        ptx::cp_async_16(sc0 + (uint32_t)((r * ncs + 8 * c) * 2),
                         in ? sbase + (size_t)(gr0 + r) * p.N + 8 * c : p.s, in ? 16u : 0u);
      }
    }
    // activations may be written by the previous kernel in the stream
    ptx::grid_dependency_wait();
    {
      // xs[((j*4 + s)*NB + nb)*32 + lane] = x[8nb + g][128(kb0+j) + 32s + 8t .. +7]
      const uint32_t xs0 = ptx::smem_u32(smem + L.xs);
      const int nx = nblk * 4 * NB * 32;
      for (int i = ctid; i < nx; i += 32 * NCW) {
        const int ln = i & 31, js = (i >> 5) / NB, nb = (i >> 5) - js * NB;
        const int m = 8 * nb + (ln >> 2);
        const int k = kb0 * KB + js * 32 + 8 * (ln & 3);
        // K % 16 == 0: a lane's 8 rows lie wholly inside or wholly past K (zeros then)
        const bool in = m < p.M && k < p.K;
        ptx::cp_async_16(xs0 + (uint32_t)i * 16u, in ? p.x + (size_t)m * p.K + k : p.x, in ? 16u : 0u);
      }
    }
    ptx::cp_async_wait_all();
    ptx::named_bar_sync(1, 32 * NCW);
    const float zc = 128.0f + (float)p.zp;
    const uint32_t MASK = 0x000F000Fu, BIAS = 0x43004300u, ONES = 0x3F803F80u;
    // seeds: sx[(j*NQ + q)*32 + m] = -(128+zp) * sum of x[m] over group q of block j
    for (int j = warp; j < nblk; j += NCW) {
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        float d[NB][4];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) d[nb][e] = 0.f;
#pragma unroll
        for (int s = q * GS; s < q * GS + GS; ++s)
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            const uint4 b = xs[((j * 4 + s) * NB + nb) * 32 + lane];
            mma_bf16(d[nb], ONES, ONES, ONES, ONES, b.x, b.y);
            mma_bf16(d[nb], ONES, ONES, ONES, ONES, b.z, b.w);
          }
        if (g == 0) {
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            sx[(j * NQ + q) * 32 + 8 * nb + 2 * t] = -zc * d[nb][0];
            sx[(j * NQ + q) * 32 + 8 * nb + 2 * t + 1] = -zc * d[nb][1];
          }
        }
      }
    }
    ptx::named_bar_sync(1, 32 * NCW);

    int st = 0;
    uint32_t ph = 0;
    for (int j = 0; j < nblk; ++j) {
      if (!ptx::mbar_wait_sleep(full_bar(st), ph, abort_flag, p.wait_ns)) {
        if (!*abort_flag) { *abort_flag = 1; if (p.err) atomicCAS(p.err, 0, DEVERR_TIMEOUT_EPILOGUE); }
        break;
      }
      // this warp's units of the stage: groups 2(pw0+i) and 2(pw0+i)+1, 16 bytes a lane
      const uint4* rw = ring + (size_t)st * (stage_bytes / 16) + lane;
      uint4 wa[NP], wb[NP];
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        wa[i] = rw[(2 * (pw0 + i)) * 32];
        wb[i] = rw[(2 * (pw0 + i) + 1) * 32];
      }
      __syncwarp();
      if (lane == 0) {
        // this warp's reads of the stage are done; the last of the NCW refills it
        __threadfence_block();
        if (atomicAdd(&released[st], 1) % NCW == NCW - 1 && j + STAGES < nblk) {
          __threadfence_block();
          ptx::fence_proxy_async_smem();
          ptx::mbar_arrive_expect_tx(full_bar(st), stage_bytes);
          ptx::tma_load_3d(ring0 + st * stage_bytes, &tmW, full_bar(st), 0, kb0 + j + STAGES, gz);
          laps[st] += 1;
        }
      }
      if (++st == STAGES) { st = 0; ph ^= 1u; }
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        float2 z[NB];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
          z[nb] = *reinterpret_cast<const float2*>(sx + (j * NQ + q) * 32 + 8 * nb + 2 * t);
        float d[NP][NB][4];
#pragma unroll
        for (int s = q * GS; s < q * GS + GS; ++s) {
          uint4 b[NB];
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) b[nb] = xs[((j * 4 + s) * NB + nb) * 32 + lane];
          // first k half of every pair, then the second: an MMA and the next one on the
          // same accumulator are NP * NB MMAs apart
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const uint32_t w0 = word_of(wa[i], s), w1 = word_of(wb[i], s);
            const uint32_t l0 = and_or(w0, MASK, BIAS), l1 = and_or(w1, MASK, BIAS);
            const uint32_t l2 = and_or(w0 >> 8, MASK, BIAS), l3 = and_or(w1 >> 8, MASK, BIAS);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
              if (s == q * GS)
                mma_bf16_init(d[i][nb], l0, l1, l2, l3, b[nb].x, b[nb].y, z[nb].x, z[nb].y);
              else
                mma_bf16(d[i][nb], l0, l1, l2, l3, b[nb].x, b[nb].y);
            }
          }
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const uint32_t w0 = word_of(wa[i], s), w1 = word_of(wb[i], s);
            const uint32_t h0 = and_or(w0 >> 4, MASK, BIAS), h1 = and_or(w1 >> 4, MASK, BIAS);
            const uint32_t h2 = and_or(w0 >> 12, MASK, BIAS), h3 = and_or(w1 >> 12, MASK, BIAS);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
              mma_bf16(d[i][nb], h0, h1, h2, h3, b[nb].z, b[nb].w);
          }
        }
        // a scale group wholly past K has no scale row (its sums are zero): skipped
        const int k0g = (kb0 + j) * KB + q * GS * 32;
        const int lr = k0g / p.G - gr0;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          if (k0g < p.K) {
            const uint16_t* sr = scs + (size_t)lr * ncs + 16 * (pw0 + i) + g;
            const float s0 = bf16_bits_to_f32(sr[0]), s1 = bf16_bits_to_f32(sr[8]);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
              acc[i][nb][0] = fmaf(s0, d[i][nb][0], acc[i][nb][0]);
              acc[i][nb][1] = fmaf(s0, d[i][nb][1], acc[i][nb][1]);
              acc[i][nb][2] = fmaf(s1, d[i][nb][2], acc[i][nb][2]);
              acc[i][nb][3] = fmaf(s1, d[i][nb][3], acc[i][nb][3]);
            }
          }
        }
      }
    }
  }
  // every warp is past its last read of the activations and the ring
  __syncthreads();
  const bool ok = *abort_flag == 0;
  if (!ok) {
    // copies still in flight land before their space takes the partial sums
    if (threadIdx.x == 0)
      for (int s = 0; s < STAGES; ++s)
        if (laps[s] > 0 &&
            !ptx::mbar_wait(full_bar(s), (uint32_t)((laps[s] - 1) & 1), nullptr, p.wait_ns) && p.err)
          atomicCAS(p.err, 0, DEVERR_TIMEOUT_DRAIN);
    __syncthreads();
  }
  if (ok) {
    // D rows g / g+8 are columns 16p+g / 16p+8+g; D columns 2t, 2t+1 are rows 8nb+2t(+1)
#pragma unroll
    for (int i = 0; i < NP; ++i) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        float* r0 = red + (size_t)(8 * nb + 2 * t) * rs + 16 * (pw0 + i) + g;
        r0[0] = acc[i][nb][0];
        r0[rs] = acc[i][nb][1];
        r0[8] = acc[i][nb][2];
        r0[rs + 8] = acc[i][nb][3];
      }
    }
  }
  ptx::cluster_sync_all();
  // CTA `rank` finishes pairs [rank*chunk, (rank+1)*chunk) of the cluster's run
  const int chunk = (npc + S - 1) / S;
  const int q0 = rank * chunk, q1 = (q0 + chunk < preal ? q0 + chunk : preal);
  if (ok && q1 > q0) {
    const int rows = p.M < MR ? p.M : MR;
    const int nc4 = (q1 - q0) * 4;  // float4 pieces per row
    const uint32_t red0 = ptx::smem_u32(red);
    for (int idx = threadIdx.x; idx < rows * nc4; idx += THREADS) {
      const int m = idx / nc4;
      const int c = 16 * q0 + 4 * (idx - m * nc4);  // column within the cluster's run
      const uint32_t a = red0 + (uint32_t)(((size_t)m * rs + c) * 4);
      // every rank's partial in flight at once, then added in rank order
      float4 u[MAX_S];
#pragma unroll
      for (int r = 0; r < MAX_S; ++r)
        if (r < S) u[r] = ptx::ld_cluster_f4(ptx::map_to_rank(a, (uint32_t)r));
      float4 v = u[0];
#pragma unroll
      for (int r = 1; r < MAX_S; ++r)
        if (r < S) { v.x += u[r].x; v.y += u[r].y; v.z += u[r].z; v.w += u[r].w; }
      __nv_bfloat16* yo = p.y + (size_t)m * p.N + (size_t)p0 * 16 + c;
      const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
      if (p.y_vec) {
        uint2 o;
        o.x = *reinterpret_cast<const uint32_t*>(&lo);
        o.y = *reinterpret_cast<const uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(yo) = o;
      } else {
        yo[0] = lo.x; yo[1] = lo.y; yo[2] = hi.x; yo[3] = hi.y;
      }
    }
  }
  // no CTA leaves while another may still read its partial sums
  ptx::cluster_sync_all();
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

// The fragment-ordered weights as a 3-D u32 tensor {128 words, NKB blocks, N/8 groups};
// one box is one block of `groups` consecutive column groups.
static bool map_weights(CUtensorMap* m, const void* wf, int NKB, int NG, int groups) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {128, (cuuint64_t)NKB, (cuuint64_t)NG};
  cuuint64_t strides[2] = {512, (cuuint64_t)NKB * 512};
  cuuint32_t box[3] = {128, 1, (cuuint32_t)groups};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(wf), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

using Kern = void (*)(const CUtensorMap, const Params);

template <int NB, int NP>
static Kern kernel_for_gs(int gs) {
  return gs == 1 ? w4a16_frag_cluster_kernel<NB, NP, 1>
       : gs == 2 ? w4a16_frag_cluster_kernel<NB, NP, 2>
                 : w4a16_frag_cluster_kernel<NB, NP, 4>;
}
template <int NB>
static Kern kernel_for_np(int np, int gs) {
  return np == 1 ? kernel_for_gs<NB, 1>(gs)
       : np == 2 ? kernel_for_gs<NB, 2>(gs)
       : np == 3 ? kernel_for_gs<NB, 3>(gs)
                 : kernel_for_gs<NB, 4>(gs);
}
static Kern kernel_for(int nb, int np, int gs) {
  return nb == 1 ? kernel_for_np<1>(np, gs) : nb == 2 ? kernel_for_np<2>(np, gs)
                                                      : kernel_for_np<4>(np, gs);
}

static std::mutex g_mu;
static std::map<std::tuple<int, int, int, int>, bool> g_attr;  // (device, nb, np, gs) -> set
static std::map<std::tuple<int, int>, int> g_clusters;          // (device, S) -> clusters

static qgemm_status set_attr(qgemm_device_s* d, int nb, int np, int gs) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_tuple(d->ordinal, nb, np, gs);
  if (g_attr.count(key)) return QGEMM_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel_for(nb, np, gs),
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)d->smem_optin);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a16_frag_cluster)");
  g_attr[key] = true;
  return QGEMM_OK;
}

// Clusters of S CTAs (one CTA per SM, the largest shared-memory request) that run at
// once: fewer than SMs / S, since a cluster must sit inside one GPU processing cluster
// (measured on B200: 148, 74, 45, 33, 26, 22, 15, 15 for S = 1 .. 8).
static int max_clusters(qgemm_device_s* d, int S) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_clusters.find(std::make_tuple(d->ordinal, S));
    if (it != g_clusters.end()) return it->second;
  }
  int n = 0;
  if (set_attr(d, MAX_NB, PMAX, 4) == QGEMM_OK) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, S, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = d->smem_optin;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = S;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kernel_for(MAX_NB, PMAX, 4), &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
  }
  if (n <= 0) n = d->sm_count / (S * 2);  // the query failed: a conservative guess
  if (n < 1) n = 1;
  std::lock_guard<std::mutex> lk(g_mu);
  g_clusters[std::make_tuple(d->ordinal, S)] = n;
  return n;
}

struct Plan {
  int np = 0, S = 0, X = 0, nblk_max = 0, nsr_max = 0, stages = 0;
  size_t smem = 0;
};

// Cycles per MMA per sub-partition of the main loop at NP pairs a warp (two warps a
// sub-partition, 32 rows, measured on B200 with the loop alone in shared memory).
static double loop_cycles_per_mma(int np) {
  return np == 1 ? 13.0 : np == 2 ? 10.9 : np == 3 ? 10.4 : 9.9;
}

// The pairs per warp NP and the slice count S for NPT column pairs: every cluster
// resident at once, the least modelled time (MMA issue on a sub-partition over the
// slice, plus the fixed cost of the prologue, and of the cross-CTA sum when S > 1).
static bool plan_for(qgemm_device_s* d, int NPT, int nkb, int G, int nb, Plan* out) {
  const int nq = G == 32 ? 4 : G == 64 ? 2 : 1;
  double best = 1e30;
  for (int np = 1; np <= PMAX; ++np) {
    const int npc = NCW * np;
    const int X = (NPT + npc - 1) / npc;
    for (int S = 1; S <= MAX_S && S <= nkb; ++S) {
      const int nblk = (nkb + S - 1) / S;
      if (nblk > NBLK_MAX) continue;
      if (X > max_clusters(d, S)) continue;
      Plan c;
      c.np = np; c.S = S; c.X = X; c.nblk_max = nblk;
      c.nsr_max = (nblk * KB + G - 1) / G + 1;
      const size_t fixed = smem_layout(nb, nq, nblk, npc, c.nsr_max, 0).total;
      const size_t per = (size_t)npc * 1024;
      if (fixed + 2 * per > d->smem_optin) continue;
      int stages = (int)((d->smem_optin - fixed) / per);
      stages = stages > MAX_STAGES ? MAX_STAGES : stages;
      stages = stages > nblk ? (nblk > 2 ? nblk : 2) : stages;
      c.stages = stages;
      c.smem = smem_layout(nb, nq, nblk, npc, c.nsr_max, stages).total;
      if (c.smem > d->smem_optin) continue;
      // two warps a sub-partition, NP pairs, 4 steps x 2 halves x NB MMAs a block
      const double mma = 2.0 * np * nblk * 8 * nb * loop_cycles_per_mma(np);
      const double cost = mma + 3000.0 + (S > 1 ? 1500.0 : 0.0);
      if (cost < best) { best = cost; *out = c; }
    }
  }
  return best < 1e29;
}

}  // namespace w4c

bool w4a16_frag_cluster_fits(int N, int K) {
  const int nkb = (K + w4c::KB - 1) / w4c::KB;
  return N % 16 == 0 && nkb <= w4c::NBLK_MAX * w4c::MAX_S;
}

qgemm_status launch_w4a16_frag_cluster(qgemm_stream_s* s, const void* x, const void* wf,
                                       const void* sc, int zp, int G, void* y, int M, int N,
                                       int K) {
  using namespace w4c;
  qgemm_device_s* d = s->dev;
  if (!w4a16_frag_cluster_fits(N, K))
    return fail(QGEMM_ERR_UNSUPPORTED, "cluster frag path: N %% 16 != 0 or K > %d", NBLK_MAX * MAX_S * KB);
  const int nkb = (K + KB - 1) / KB;
  const int NPT = N / 16;
  const int gs = G == 32 ? 1 : G == 64 ? 2 : 4;
  CUtensorMap tm;  // one box = one block of one CTA's 2 * 8 NP column groups
  Params p;
  p.N = N; p.K = K; p.G = G; p.zp = zp;
  p.NKB = nkb;
  p.wait_ns = d->wait_ns;
  p.err = d->d_err;
  p.s = static_cast<const __nv_bfloat16*>(sc);
  p.y_vec = aligned(reinterpret_cast<uint64_t>(y), 8) ? 1 : 0;
  for (int m0 = 0; m0 < M; m0 += 8 * MAX_NB) {
    const int rows = (M - m0) < 8 * MAX_NB ? (M - m0) : 8 * MAX_NB;
    const int nb = rows <= 8 ? 1 : rows <= 16 ? 2 : 4;
    p.M = rows;
    p.x = static_cast<const __nv_bfloat16*>(x) + (size_t)m0 * K;
    p.y = static_cast<__nv_bfloat16*>(y) + (size_t)m0 * N;
    // column chunks: one unless N is wider than every resident cluster can take
    int pc0 = 0;
    while (pc0 < NPT) {
      int nchunk = NPT - pc0;
      Plan pl;
      while (!plan_for(d, nchunk, nkb, G, nb, &pl)) {
        if (nchunk <= 1)
          return fail(QGEMM_ERR_UNSUPPORTED, "no cluster layout fits K=%d in shared memory", K);
        nchunk = (nchunk + 1) / 2;
      }
      const qgemm_status as = set_attr(d, nb, pl.np, gs);
      if (as != QGEMM_OK) return as;
      if (!map_weights(&tm, wf, nkb, N / 8, 2 * NCW * pl.np))
        return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for the frag weights");
      p.S = pl.S;
      p.nblk_max = pl.nblk_max;
      p.npc_max = NCW * pl.np;
      p.nsr_max = pl.nsr_max;
      p.stages = pl.stages;
      p.pair0 = pc0;
      p.pair1 = pc0 + nchunk;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(pl.X, pl.S, 1);
      cfg.blockDim = dim3(THREADS, 1, 1);
      cfg.dynamicSmemBytes = pl.smem;
      cfg.stream = s->stream;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = pl.S;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 2;
      cudaError_t e = cudaLaunchKernelEx(&cfg, kernel_for(nb, pl.np, gs), tm, p);
      if (e != cudaSuccess) return cuda_fail(e, "w4a16_frag_cluster_kernel launch");
      pc0 += nchunk;
    }
  }
  return QGEMM_OK;
}

}  // namespace qg
