// internal.h -- handle structs, status helpers and launcher declarations shared
// by the libqgemm translation units.  Not part of the public ABI (include/qgemm.h).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>
#include <mutex>

#include "qgemm.h"

struct qgemm_device_s {
  int ordinal = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  size_t l2_bytes = 0;
  size_t smem_optin = 0;
  bool tcgen05 = false;       // sm_100 family: tcgen05 / TMEM / TMA kernels run
  int* d_err = nullptr;       // device error word written by bounded waits
  // Limit of every bounded wait in the tcgen05 GEMM kernels launched on this device
  // (qgemm_device_set_wait_limit), and the split hold-back test hook
  // (qgemm_debug_hold_split).
  unsigned long long wait_ns = 2000000000ull;
  int hold_split = 0;
  std::mutex mu;
  bool open = false;
};

struct qgemm_stream_s {
  qgemm_device_s* dev = nullptr;
  cudaStream_t stream = nullptr;
  bool owned = false;
  // Scratch of the tcgen05 GEMM's last-wave split (a counter block at offset 0 that
  // every kernel leaves zeroed, then partial tiles) and of the fp32 GEMM's split
  // operands; allocated by the first call that needs it on this handle, zeroed then,
  // and grown (outside graph capture) when a call needs more.
  void* ws = nullptr;
  size_t ws_bytes = 0;
};

namespace qg {

// Records a thread-local message and returns the status.
qgemm_status fail(qgemm_status s, const char* fmt, ...);
// Maps a CUDA error (after a launch or API call) to a status + message.
qgemm_status cuda_fail(cudaError_t e, const char* what);
// Checks the stream handle and makes its device current.
qgemm_status enter(qgemm_stream_t s);

inline bool aligned(uint64_t p, uint64_t a) { return (p % a) == 0; }

// The stream handle's scratch, at least `bytes` long and zero-filled when first
// made.  Allocating is refused while the stream is being captured into a graph.
qgemm_status stream_workspace(qgemm_stream_s* s, size_t bytes, void** out);

// Error codes a kernel writes into qgemm_device_s::d_err.
enum : int {
  DEVERR_NONE = 0,
  DEVERR_TIMEOUT_PRODUCER = 1,
  DEVERR_TIMEOUT_MMA = 2,
  DEVERR_TIMEOUT_EPILOGUE = 3,
  DEVERR_TIMEOUT_DRAIN = 4,
};

// ---- the tcgen05 GEMM (w8a8_tcgen05.cu) ----
// MMA kinds of the tcgen05 GEMM kernels.
enum : int { KIND_I8 = 0, KIND_BF16 = 1, KIND_TF32 = 2 };

// One tcgen05 GEMM launch: out[M, ldc] = sum over K segments of A_seg * B_seg^T.
struct TcArgs {
  int kind = KIND_I8;
  const void* A = nullptr;  // [M rows, a_pitch bytes], K-major
  const void* B = nullptr;  // [N rows, b_pitch bytes] K-major, or [K, N] int8 (b_kn)
  int b_kn = 0;             // B in [K,N] (MN-major operand): KIND_I8 with nseg = 1 only
  int M = 0, N = 0;
  int K = 0;                // bytes of K in one segment
  // nseg segments of ceil(K / 128) k-blocks each.  Segment s reads the first
  // ceil(K / 128) * 128 bytes of A's rows, or the next as many when bit s of a_seg is
  // set; likewise for B with b_seg.  Bytes past K inside a block must be zero (TMA
  // fills zeros past the row's end).
  int nseg = 1;
  uint32_t a_seg = 0, b_seg = 0;
  uint64_t a_pitch = 0, b_pitch = 0;  // row pitch in bytes, also the rows' extent (0: K)
  const float* sA = nullptr;          // KIND_I8: y = (float(acc) * sB[n]) * sA[m]
  const float* sB = nullptr;
  int32_t* acc = nullptr;             // KIND_I8: optional int32 accumulators [M, acc_ld]
  int acc_ld = 0;                     // row pitch of acc in elements (0: N)
  const int32_t* acc_c = nullptr;     // optional int32 addend of acc, [M, acc_c_ld]
  int acc_c_ld = 0;
  int no_out = 0;                     // 1: acc is the only output (out, sA, sB unused)
  uint64_t a_extent = 0;              // bytes of each A row that exist (0: a_pitch)
  uint64_t b_kn_pitch = 0;            // b_kn: row pitch of B [K, N] in bytes (0: N)
  void* out = nullptr;
  int out_dtype = QGEMM_F32;
  int ldc = 0;
  // The same output block in up to 7 peers' windows (same M, N, ldc): each output
  // chunk is also TMA-stored there (the fused sharded GEMM + all-gather).
  const void* peer_out[7] = {};
  int npeer = 0;
  // bf16 / tf32 kinds: v = acc; v = alpha * v (ep_alpha); v += bias[n] (bias);
  // v += beta * out[m, n] (ep_beta, fp32 out), each step rounded on its own.
  float alpha = 1.f, beta = 0.f;
  const float* bias = nullptr;
  int ep_alpha = 0, ep_beta = 0;
  // Device word read by the epilogue: non-zero -> store nothing.
  const int* skip_flag = nullptr;
  // Cut every tile along K when there are fewer pair tiles than CTA pairs.
  int full_split = 0;
  // Last-wave split scratch: counters (zero) at offset 0, partial tiles after them;
  // null: the stream handle's scratch.
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
};
qgemm_status launch_tc_gemm(qgemm_stream_s* s, const TcArgs& a);
// The W8A8 tcgen05 GEMM with bf16 output whose epilogue also TMA-stores every output
// chunk into npeer (<= 7) peers' copies of the output block (same ldc): the fused
// sharded GEMM + all-gather.
qgemm_status launch_w8a8_tcgen05_peers(qgemm_stream_s* s, const void* A, const void* B, int b_kn,
                                       const float* sA, const float* sB, void* out, int ldc,
                                       int M, int N, int K, const uint64_t* peer_out,
                                       int npeer);
// Scratch bytes a launch of this shape uses for its last-wave split: the counter block
// (always counted) and the partial tiles.
size_t tc_gemm_scratch_bytes(const qgemm_device_s* d, int M, int N, int num_k_blocks,
                             bool full_split = false);

// ---- launchers (each returns a status and never throws) ----
qgemm_status launch_w8a8_tcgen05(qgemm_stream_s* s, const void* A, const void* B, int b_kn,
                                 const float* sA, const float* sB, void* out, int out_dtype,
                                 int ldc, int M, int N, int K, int32_t* acc);
// As launch_w8a8_tcgen05, with the last-wave split's scratch in a static device array.
qgemm_status launch_w8a8_tcgen05_static(qgemm_stream_s* s, const void* A, const void* B, int b_kn,
                                        const float* sA, const float* sB, void* out, int out_dtype,
                                        int ldc, int M, int N, int K, int32_t* acc);
bool w8a8_tcgen05_supported(const qgemm_device_s* d, uint64_t A, uint64_t B, int b_kn,
                            uint64_t out, int out_dtype, int ldc, int M, int N, int K,
                            const char** why);
// bf16 GEMM on the same tcgen05 kernels: out[M, ldc] (bf16, RNE) = A[M,K] * B[N,K]^T,
// fp32 accumulation.  A and B bf16, K-major; K % 8 == 0; 16-byte aligned A and B.
// a_repeat = 2: B rows hold 2 blocks of K values, each padded with zeros to a
// multiple of 64, and out = A * B_0^T + A * B_1^T (two K segments of one launch).
qgemm_status launch_bf16_gemm_nk(qgemm_stream_s* s, const void* A, const void* B, void* out,
                                 int ldc, int M, int N, int K, int a_repeat = 1);
// fp32 entry points (f32_gemm.cu).  C [M,N] = A [M,K] x B [K,N], all fp32 row-major,
// through three tf32 tensor-core products per fp32 product; the split operands live in
// the stream's scratch after the GEMM's counter block.
enum : int { F32_MATMUL = QGEMM_F32_MATMUL, F32_MATMUL_BIAS = QGEMM_F32_MATMUL_BIAS,
              F32_SGEMM = QGEMM_F32_SGEMM };
// algo: QGEMM_ALGO_AUTO / _TCGEN05 (3xTF32 tensor cores) / _SIMT (CUDA-core split-K).
qgemm_status launch_f32_gemm(qgemm_stream_s* s, const float* A, const float* B,
                             const float* bias, float* C, int M, int N, int K, float alpha,
                             float beta, int mode, int algo);
qgemm_status launch_f32_gemv(qgemm_stream_s* s, const float* A, const float* x, float* y, int M,
                             int N);
qgemm_status launch_w8a8_simt(qgemm_stream_s* s, const int8_t* A, const int8_t* B, int b_kn,
                              const float* sA, const float* sB, void* out, int out_dtype,
                              int ldc, int M, int N, int K, int32_t* acc);
qgemm_status launch_w4a16_ref(qgemm_stream_s* s, const uint8_t* w, const float* sw,
                              const float* x, float* y, int M, int N, int K);
// Exact-order w8a16 on a TMA weight stream (w8a16_stream.cu); needs sm_100, N % 16 == 0,
// K % 4 == 0, 16-byte aligned wInt8 and x.
bool w8a16_stream_supported(const qgemm_device_s* d, uint64_t w, uint64_t x, int N, int K);
qgemm_status launch_w8a16_stream(qgemm_stream_s* s, const int8_t* w, const float* sw,
                                 const float* x, const float* bias, float* y, int M, int N,
                                 int K, int hasBias, int rowwise);
qgemm_status launch_w8a16_ref(qgemm_stream_s* s, const int8_t* w, const float* sw,
                              const float* x, const float* bias, float* y, int M, int N,
                              int K, int hasBias, int rowwise);
qgemm_status launch_quantize(qgemm_stream_s* s, const float* w, float* scales, int8_t* q,
                             int8_t* zeros, int K, int N, int qBits);
qgemm_status launch_quantize_tokens(qgemm_stream_s* s, const void* x, int in_dtype, int8_t* q,
                                    float* sA, int M, int K);
qgemm_status launch_dequantize(qgemm_stream_s* s, const int8_t* q, const float* scales,
                               float* w, int K, int N);
qgemm_status launch_prepack_w8_nk(qgemm_stream_s* s, const int8_t* src, int8_t* dst, int K,
                                  int N);
qgemm_status launch_unshard_bf16(qgemm_stream_s* s, const uint16_t* g, uint16_t* out,
                                 int world, int M, int ncols);
bool w4a16_tile_supported(const qgemm_device_s* d, uint64_t x, uint64_t wt, uint64_t sc, int M,
                          int N, int K, int G, const char** why);
qgemm_status launch_w4a16_tile(qgemm_stream_s* s, const void* x, const uint8_t* wt,
                               const void* sc, int zp, int G, void* y, int M, int N, int K);
size_t w4_tiled_bytes(int K, int N);
qgemm_status launch_prepack_w4_tiled(qgemm_stream_s* s, const uint32_t* src, uint8_t* dst, int K,
                                     int N);
bool w4a16_frag_supported(const qgemm_device_s* d, uint64_t x, uint64_t wf, uint64_t sc, int M,
                          int N, int K, int G, const char** why);
qgemm_status launch_w4a16_frag(qgemm_stream_s* s, const void* x, const void* wf, const void* sc,
                               int zp, int G, void* y, int M, int N, int K);
size_t w4_frag_bytes(int K, int N);
// The K-split cluster kernel on the same fragment-ordered weights (w4a16_frag_cluster.cu):
// up to 32 activation rows per pass, K up to 16384; needs N % 16 == 0.
bool w4a16_frag_cluster_fits(int N, int K);
qgemm_status launch_w4a16_frag_cluster(qgemm_stream_s* s, const void* x, const void* wf,
                                       const void* sc, int zp, int G, void* y, int M, int N,
                                       int K);
qgemm_status launch_prepack_w4_frag(qgemm_stream_s* s, const uint32_t* src, uint32_t* dst, int K,
                                    int N);
// terms: bf16 values per expanded weight (2: exact hi + lo, 1: bf16((q - zp) * s))
size_t w4a16_prefill_workspace_bytes(int K, int N, int terms);
// The group-scaled multiply of the prefill path (w4a16_prefill_gs.cu): y[M, ldc] (bf16) =
// sum_g s[g, n] * (x[:, group g] * slab[n, group g]^T), the slab holding q - zp as bf16
// [N rows, slab_pitch bytes], scales bf16 with row pitch ld_s (elements).  Needs
// w4a16_gs_supported (sm_100, G % 64 == 0, 16-byte aligned scales), K % 8 == 0,
// N % 8 == 0, ldc % 8 == 0 and 16-byte aligned x, slab, y.
bool w4a16_gs_supported(const qgemm_device_s* d, int G, uint64_t scales);
qgemm_status launch_w4a16_gs_gemm(qgemm_stream_s* s, const void* x, const void* slab,
                                  size_t slab_pitch, const void* scales, long long ld_s, int G,
                                  void* y, int ldc, int M, int N, int K);
// frag: wt is in the fragment order of qgemm_prepack_w4_frag instead of 64-column tiles
qgemm_status launch_w4a16_prefill(qgemm_stream_s* s, const void* x, const uint8_t* wt,
                                  const void* scales, int zp, int G, void* y, int M, int N,
                                  int K, void* ws, size_t ws_bytes, bool frag, int terms);
qgemm_status launch_w4a16_grouped(qgemm_stream_s* s, const void* x, const uint32_t* wq,
                                  const void* scales, int zp, int group, void* y, int M,
                                  int N, int K);

}  // namespace qg
