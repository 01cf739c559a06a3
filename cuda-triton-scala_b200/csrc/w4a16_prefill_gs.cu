// w4a16_prefill_gs.cu -- the multiply of the W4A16 prefill GEMM with the group scales
// applied outside the tensor cores.
//
// Arithmetic (QuantizedGemmOps.scala:229-245 generalised to groups and a zero point):
//     y[m,n] = sum_g s[g,n] * P_g[m,n],   P_g[m,n] = sum_{k in group g} x[m,k] * (q[k,n] - zp)
//
// The slab holds q - zp as bf16 (integers in [-15, 15], exact), so every tensor-core
// product is exact and P_g is an fp32 sum, as in the two-term (hi + lo) expansion, but
// with one pass over K: the algorithmic tensor work.  The scales never meet a rounding
// to bf16: the epilogue warps multiply each group's partial sums by s[g,n] in fp32 and
// add them up in group order (deterministic).
//
// One persistent grid of CTA pairs (2-CTA clusters), 12 warps (3 warpgroups) per CTA:
//   warp 0      TMA producer: A (activations, bf16 [M,K]) and B (slab, bf16 [n,Kp]) in
//               128-byte-swizzled 64-element k-blocks, a ring of 4 stages of 32 KB.
//   warp 1      allocates 512 TMEM columns (two 256-column fp32 accumulators); the even
//               CTA's lane 0 issues tcgen05.mma.cta_group::2.kind::f16 (M=256, N=256,
//               K=16) for one scale group into one accumulator, commits it, and starts
//               the next group in the other accumulator.
//   warps 2, 3  idle (they complete the first warpgroup).
//   warps 4..11 epilogue: warp w reads TMEM lanes 32*(w%4).. (one output row per thread)
//               and one 128-column half of the tile, S += s[g, n] * P_g per group, with
//               the group's scales fetched two groups ahead (cp.async) and widened to fp32
//               in shared memory; after the last group, bf16 (RNE) through a swizzled
//               staging buffer and TMA bulk tensor stores.
// Registers: the CTA is launched with 168 a thread (12 warps x 32 x 168 = 64512); the
// first warpgroup gives its share down to 40 and the two epilogue warpgroups take 232
// (4 x 32 x 40 + 8 x 32 x 232 = 64512, the launch's total, so the increase never
// waits on registers that are not there), enough for 128 running sums and two
// 32-column TMEM loads in flight.  The host checks once that the kernel was built with
// exactly that launch count.
// Groups are whole k-blocks (group_size % 64 == 0).  Every barrier wait is bounded; a
// wait that runs out records an error code in the device error word and the CTA skips
// the rest of its work (keeping every barrier sequence), frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstring>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace qg {
namespace w4gs {

constexpr int BK = 128;                        // bytes of K per stage: 64 bf16
constexpr int KB_ELEMS = 64;
constexpr int UMMA_K = 32;                     // bytes of K per MMA: 16 bf16
constexpr int STAGES = 4;                      // 4 measured faster than 5 at 16384 x 22016 x 4096
constexpr int A_BYTES = 128 * BK;              // 16 KB: this CTA's 128 rows
constexpr int B_BYTES = 128 * BK;              // 16 KB: this CTA's 128 columns
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;
constexpr int EPI_WARP0 = 4;                   // first epilogue warp (second warpgroup)
constexpr int NUM_THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
constexpr int LAUNCH_REGS = 168, CTRL_REGS = 40, EPI_REGS = 232;
static_assert(4 * 32 * CTRL_REGS + EPI_WARPS * 32 * EPI_REGS == NUM_THREADS * LAUNCH_REGS,
              "the register split must add up to the launch's registers");
constexpr int STG_BYTES = 2 * 128 * 128;       // one 128-row x 64-column bf16 buffer per half
constexpr int SC_SLOTS = 3;                   // scale groups in flight per warp
constexpr int SC_WARP_BYTES = SC_SLOTS * 256 + 512;  // bf16 slots + one fp32 row of 128 scales
constexpr int SC_BYTES = EPI_WARPS * SC_WARP_BYTES;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + STG_BYTES + SC_BYTES + BAR_BYTES;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;                    // tile raster: 16 m-blocks per group

struct Params {
  int M, N, K;              // N: columns of this launch (the slab), K: bf16 elements
  int G;                    // group size, a multiple of 64
  int num_m_blocks, num_n_blocks, num_k_blocks, num_tiles, num_groups;
  const __nv_bfloat16* scales;  // s[g, 0] of this launch's first column
  long long ld_s;           // scale row pitch (elements)
  int* err;
  unsigned long long wait_ns;
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

__device__ __forceinline__ void report(int* err, int code, volatile int* abort_flag,
                                       uint32_t rank) {
  *abort_flag = 1;
  if (err) atomicCAS(err, 0, code);
  // the other CTA of the pair gives up its waits at once too
  const uint32_t peer = ptx::map_to_rank(ptx::smem_u32(const_cast<int*>(abort_flag)), rank ^ 1u);
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer), "r"(1) : "memory");
}

// 16 bytes global -> shared, zero-filled when !valid (no read then).
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// all but the last SC_SLOTS - 1 committed groups have landed
__device__ __forceinline__ void cp_async_wait_slots() {
  asm volatile("cp.async.wait_group %0;" ::"n"(SC_SLOTS - 1) : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    w4a16_gs_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmO, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;  // 128-byte swizzle: 1024-aligned
  uint8_t* gbase = smem_raw + (base - raw_base);
  const uint32_t stg_base = base + STAGES * STAGE_BYTES;
  const uint32_t sc_base = stg_base + STG_BYTES;
  uint8_t* gsc = gbase + STAGES * STAGE_BYTES + STG_BYTES;
  const uint32_t bar_base = sc_base + SC_BYTES;
  uint8_t* gbar = gsc + SC_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * STAGES + 4);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbar + 8 * (2 * STAGES + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbar + 8 * (2 * STAGES + 5) + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = ptx::cluster_ctarank();  // 0: issues the MMAs
  const int pair_id = blockIdx.x / 2;
  const int npairs = gridDim.x / 2;
  const int gkb = p.G / KB_ELEMS;  // k-blocks per scale group

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(tfull_bar(a), 1);
      ptx::mbar_init(tempty_bar(a), 2 * 32 * EPI_WARPS);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::grid_launch_dependents();
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(ptx::smem_u32(const_cast<uint32_t*>(tmem_slot)), TMEM_COLS);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync_all();  // barriers of both CTAs initialised before any remote traffic
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < EPI_WARP0) {
    // the first warpgroup: producer, MMA issuer, two idle warps
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(CTRL_REGS));
    if (warp == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      if (lane == 0) {
        ptx::grid_dependency_wait();  // the slab is written by the kernel before this one
        int stage = 0;
        uint32_t phase = 0;
        long long issued = 0;
        bool ok = true;
        for (int tile = pair_id; ok && tile < p.num_tiles; tile += npairs) {
          int mb, nb;
          tile_coords(tile, p, mb, nb);
          for (int kb = 0; kb < p.num_k_blocks; ++kb) {
            if (!ptx::mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, p.wait_ns)) {
              if (!*abort_flag) report(p.err, DEVERR_TIMEOUT_PRODUCER, abort_flag, rank);
              ok = false;
              break;
            }
            const uint32_t sa = base + stage * STAGE_BYTES;
            const uint32_t fb = ptx::map_to_rank(full_bar(stage), 0);
            if (rank == 0) ptx::mbar_arrive_expect_tx(full_bar(stage), 2 * STAGE_BYTES);
            ptx::tma_load_2d_pair(sa, &tmA, fb, kb * BK, mb * 256 + (int)rank * 128);
            ptx::tma_load_2d_pair(sa + A_BYTES, &tmB, fb, kb * BK, nb * 256 + (int)rank * 128);
            ++issued;
            if (++stage == STAGES) { stage = 0; phase ^= 1u; }
          }
        }
        if (rank == 0) {  // the copies in flight land before the CTA may exit
          for (long long f = (issued > STAGES ? issued - STAGES : 0); f < issued; ++f) {
            if (!ptx::mbar_wait(full_bar((int)(f % STAGES)), (uint32_t)((f / STAGES) & 1),
                                nullptr, p.wait_ns)) {
              report(p.err, DEVERR_TIMEOUT_DRAIN, abort_flag, rank);
              break;
            }
          }
        }
      }
    } else if (warp == 1) {
      // ---------------- MMA issuer (even CTA) ----------------
      if (lane == 0 && rank == 0) {
        const uint32_t idesc = ptx::idesc_bf16(256, 256);
        int stage = 0;
        uint32_t phase = 0;
        uint32_t pc = 0;  // accumulators used so far
        bool ok = true;
        bool issued_any = false;
        for (int tile = pair_id; ok && tile < p.num_tiles; tile += npairs) {
          for (int g = 0; ok && g < p.num_groups; ++g, ++pc) {
            const int a = (int)(pc & 1u);
            if (!ptx::mbar_wait(tempty_bar(a), ((pc >> 1) & 1u) ^ 1u, abort_flag, p.wait_ns)) {
              if (!*abort_flag) report(p.err, DEVERR_TIMEOUT_MMA, abort_flag, rank);
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            const uint32_t d_tmem = tmem_base + (uint32_t)(a * 256);
            const int kb0 = g * gkb;
            const int kb1 = min(kb0 + gkb, p.num_k_blocks);
            for (int kb = kb0; kb < kb1; ++kb) {
              if (!ptx::mbar_wait(full_bar(stage), phase, abort_flag, p.wait_ns)) {
                if (!*abort_flag) report(p.err, DEVERR_TIMEOUT_MMA, abort_flag, rank);
                ok = false;
                break;
              }
              ptx::tc_fence_after();
              const uint32_t sa = base + stage * STAGE_BYTES;
              const uint32_t sb = sa + A_BYTES;
#pragma unroll
              for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                const uint64_t adesc = ptx::smem_desc_sw128(sa + kk * UMMA_K, 16, 1024);
                const uint64_t bdesc = ptx::smem_desc_sw128(sb + kk * UMMA_K, 16, 1024);
                ptx::umma_bf16_pair(d_tmem, adesc, bdesc, idesc,
                                    (kb != kb0 || kk != 0) ? 1u : 0u);
              }
              ptx::umma_commit_pair(empty_bar(stage), 0x3);
              issued_any = true;
              if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            if (ok) ptx::umma_commit_pair(tfull_bar(a), 0x3);
          }
        }
        if (!ok && issued_any) {
          ptx::umma_commit_pair(drain_bar, 0x1);
          if (!ptx::mbar_wait(drain_bar, 0, nullptr, p.wait_ns))
            report(p.err, DEVERR_TIMEOUT_DRAIN, abort_flag, rank);
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(EPI_REGS));
    // ---------------- epilogue (warps 4..11, both CTAs) ----------------
    const int e = warp - EPI_WARP0;    // 0..7
    const int q = warp & 3;            // TMEM lane quadrant this warp may access
    const int ch = e >> 2;             // column half of the tile: 0 or 1
    const int rl = q * 32 + lane;      // row within this CTA's 128 rows
    const bool elected = (e == 0 || e == 4) && lane == 0;  // one thread per column half
    const int bar_id = 1 + ch;         // named barrier of the four warps of this half
    const uint32_t my_sc = sc_base + (uint32_t)e * SC_WARP_BYTES;  // bf16 slots, then fp32
    const uint32_t my_f32 = my_sc + SC_SLOTS * 256;
    const uint32_t stg = stg_base + (uint32_t)ch * (128 * 128);
    const uint32_t te0 = ptx::map_to_rank(tempty_bar(0), 0);
    const uint32_t te1 = ptx::map_to_rank(tempty_bar(1), 0);
    ptx::grid_dependency_wait();  // scales and the output belong to the previous kernel until it ends

    // the scales of the group `ahead` groups after (tile, g) in this pair's walk, for
    // this warp's 128 columns, into bf16 slot `slot`: lanes 0..15 copy 16 bytes each,
    // columns past N are zero-filled
    auto fetch_scales = [&](int tile, int g, int ahead, int slot) {
      g += ahead;
      while (g >= p.num_groups) { g -= p.num_groups; tile += npairs; }
      if (tile < p.num_tiles && lane < 16) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        const int col = nb * 256 + ch * 128 + lane * 8;
        const bool valid = col < p.N;
        const __nv_bfloat16* src = p.scales + (size_t)g * p.ld_s + (valid ? col : 0);
        cp_async_16(my_sc + (uint32_t)slot * 256 + lane * 16, src, valid);
      }
      cp_async_commit();
    };

    bool ok = true;
    uint32_t pc = 0;  // groups consumed so far (accumulator parity, scale slot)
    for (int i = 0; i < SC_SLOTS - 1; ++i) fetch_scales(pair_id, 0, i, i);
    for (int tile = pair_id; tile < p.num_tiles; tile += npairs) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      float S[128];
#pragma unroll
      for (int j = 0; j < 128; ++j) S[j] = 0.f;
      for (int g = 0; g < p.num_groups; ++g, ++pc) {
        // the scales SC_SLOTS - 1 groups ahead (far enough that their copy has landed
        // when that group comes up), then this group's
        fetch_scales(tile, g, SC_SLOTS - 1, (int)((pc + SC_SLOTS - 1) % SC_SLOTS));
        cp_async_wait_slots();
        __syncwarp();
        {  // widen this group's 128 scales to fp32: lane l takes 4 of them
          const uint2 v =
              *reinterpret_cast<const uint2*>(gsc + (my_sc - sc_base) + (pc % SC_SLOTS) * 256 + lane * 8);
          ptx::st_shared_v4(my_f32 + lane * 16, v.x << 16, v.x & 0xFFFF0000u, v.y << 16,
                            v.y & 0xFFFF0000u);
        }
        __syncwarp();
        const int a = (int)(pc & 1u);
        if (ok) {
          ok = ptx::mbar_wait(tfull_bar(a), (pc >> 1) & 1u, abort_flag, p.wait_ns);
          ok = __all_sync(0xffffffffu, ok);  // warp-uniform: tcgen05.ld is .sync.aligned
          if (!ok && lane == 0 && !*abort_flag)
            report(p.err, DEVERR_TIMEOUT_EPILOGUE, abort_flag, rank);
        }
        ptx::tc_fence_after();
        const float* sf = reinterpret_cast<const float*>(gsc + (my_f32 - sc_base));
#pragma unroll
        for (int c = 0; c < 2; ++c) {  // 64 columns a TMEM round trip: two loads, one wait
          uint32_t r[2][32];
          const uint32_t taddr =
              tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * 256 + ch * 128 + c * 64);
          if (ok) {
            ptx::tmem_ld_32x32b_x32(taddr, r[0]);
            ptx::tmem_ld_32x32b_x32(taddr + 32, r[1]);
            ptx::tmem_wait_ld();
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[0][j] = r[1][j] = 0u;
          }
          if (c == 1) {  // the accumulator is free for the group after next
            ptx::tc_fence_before();
            if (ok) ptx::mbar_arrive_remote(a ? te1 : te0);
          }
#pragma unroll
          for (int j = 0; j < 64; j += 4) {
            const float4 s4 = *reinterpret_cast<const float4*>(sf + c * 64 + j);
            const uint32_t* rr = r[j / 32];
            const int jj = j % 32;
            S[c * 64 + j] = fmaf(s4.x, __uint_as_float(rr[jj]), S[c * 64 + j]);
            S[c * 64 + j + 1] = fmaf(s4.y, __uint_as_float(rr[jj + 1]), S[c * 64 + j + 1]);
            S[c * 64 + j + 2] = fmaf(s4.z, __uint_as_float(rr[jj + 2]), S[c * 64 + j + 2]);
            S[c * 64 + j + 3] = fmaf(s4.w, __uint_as_float(rr[jj + 3]), S[c * 64 + j + 3]);
          }
        }
      }
      // the tile's 128 rows x this half's 128 columns, in two 64-column chunks
      const int row0 = mb * 256 + (int)rank * 128;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (elected) ptx::bulk_wait_group_read<0>();  // the buffer's last store has read it
        ptx::named_bar_sync(bar_id, 128);
#pragma unroll
        for (int pc8 = 0; pc8 < 8; ++pc8) {  // eight 16-byte pieces = 64 bf16
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(S[h * 64 + pc8 * 8 + 2 * i],
                                                      S[h * 64 + pc8 * 8 + 2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t*>(&b2);
          }
          ptx::st_shared_v4(stg + rl * 128 + ((pc8 ^ (rl & 7)) << 4), w[0], w[1], w[2], w[3]);
        }
        ptx::fence_proxy_async_smem();  // generic-proxy writes -> visible to the TMA engine
        ptx::named_bar_sync(bar_id, 128);
        const int col = nb * 256 + ch * 128 + h * 64;
        if (elected && ok && row0 < p.M && col < p.N) {
          ptx::tma_store_2d(&tmO, stg, col, row0);
          ptx::bulk_commit_group();
        }
      }
    }
    if (elected) ptx::bulk_wait_group_read<0>();  // the writes complete with the grid
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

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// 2-D map over bytes (rows of `inner` bytes, `pitch` apart), boxes of 128 bytes x 128
// rows, 128-byte swizzle; zeros past the edges.
static bool map_rows_u8(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t rows,
                        uint64_t pitch) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {BK, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace w4gs

// The kernel as built must be launched with exactly LAUNCH_REGS registers a thread:
// the warpgroups' register split adds up to that launch total, and an increase larger
// than the launch holds would wait forever.  Checked once per process.
static bool launch_regs_match() {
  static int state = 0;  // 1: match, -1: mismatch
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncAttributes fa;
    state = (cudaFuncGetAttributes(&fa, w4gs::w4a16_gs_pair_kernel) == cudaSuccess &&
             fa.numRegs == w4gs::LAUNCH_REGS)
                ? 1
                : -1;
  });
  return state == 1;
}

bool w4a16_gs_supported(const qgemm_device_s* d, int G, uint64_t scales) {
  return d->tcgen05 && d->sm_count >= 2 && d->smem_optin >= (size_t)w4gs::SMEM_BYTES &&
         G > 0 && G % w4gs::KB_ELEMS == 0 && aligned(scales, 16) && launch_regs_match();
}

qgemm_status launch_w4a16_gs_gemm(qgemm_stream_s* s, const void* x, const void* slab,
                                  size_t slab_pitch, const void* scales, long long ld_s, int G,
                                  void* y, int ldc, int M, int N, int K) {
  using namespace w4gs;
  if (!launch_regs_match())
    return fail(QGEMM_ERR_UNSUPPORTED, "w4a16_gs_pair_kernel was not built with %d registers",
                LAUNCH_REGS);
  CUtensorMap tmA, tmB, tmO;
  if (!map_rows_u8(&tmA, x, (uint64_t)K * 2, (uint64_t)M, (uint64_t)K * 2))
    return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for x [%d,%d]", M, K);
  if (!map_rows_u8(&tmB, slab, (uint64_t)slab_pitch, (uint64_t)N, (uint64_t)slab_pitch))
    return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for the slab");
  {
    EncodeTiledFn enc = encode_fn();
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)ldc * 2};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t estr[2] = {1, 1};
    if (!enc || enc(&tmO, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(QGEMM_ERR_CUDA, "cuTensorMapEncodeTiled failed for y");
  }
  Params p;
  p.M = M; p.N = N; p.K = K; p.G = G;
  p.num_m_blocks = (M + 255) / 256;
  p.num_n_blocks = (N + 255) / 256;
  p.num_k_blocks = (K + KB_ELEMS - 1) / KB_ELEMS;
  p.num_tiles = p.num_m_blocks * p.num_n_blocks;
  p.num_groups = (K + G - 1) / G;
  p.scales = static_cast<const __nv_bfloat16*>(scales);
  p.ld_s = ld_s;
  p.err = s->dev->d_err;
  p.wait_ns = s->dev->wait_ns;
  static bool attr_set[64] = {};
  const int ord = s->dev->ordinal;
  if (ord < 0 || ord >= 64 || !attr_set[ord]) {
    cudaError_t e = cudaFuncSetAttribute(w4a16_gs_pair_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w4a16_gs_pair)");
    if (ord >= 0 && ord < 64) attr_set[ord] = true;
  }
  const int max_pairs = s->dev->sm_count / 2;
  const int pairs = p.num_tiles < max_pairs ? p.num_tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = s->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, w4a16_gs_pair_kernel, tmA, tmB, tmO, p);
  if (e != cudaSuccess) return cuda_fail(e, "w4a16_gs_pair launch");
  return QGEMM_OK;
}

}  // namespace qg
