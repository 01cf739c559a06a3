// comm.cu -- NCCL communicator and the device-buffer output all-gather for the
// column-sharded W8A8 GEMM.
//
// Replaces nccl/NCCLCommunicator.scala (init :44-56, allGatherNative :151-163,
// NCCLOps.ncclAllGather :302-320), which passes host arrays to NCCL and calls
// ncclGetUniqueId on every rank.  Here one rank makes the unique id, the caller
// carries it to the others, and the gather runs on device buffers on the
// caller's stream.  NCCL is opened with dlopen("libnccl.so.2") on first use, so
// the library loads on machines without NCCL and shares the process's NCCL when
// one is already loaded.  Initialisation is non-blocking with a host-side
// deadline: a rank that never joins produces QGEMM_ERR_TIMEOUT, not a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "internal.h"

struct qgemm_comm_s {
  ncclComm_t comm = nullptr;
  qgemm_device_s* dev = nullptr;
  int rank = 0, world = 1;
  // events of the pipelined GEMM + all-gather, made on its first call
  cudaEvent_t ev_gemm[2] = {nullptr, nullptr}, ev_done[2] = {nullptr, nullptr};
  cudaEvent_t ev_end = nullptr, ev_start = nullptr, ev_open = nullptr;
  // the window copies' streams, one per peer at most, and an event on each
  std::vector<cudaStream_t> cp;
  std::vector<cudaEvent_t> ev_cp;
};

// A buffer that every rank of a communicator registered together: this rank's
// address, and every peer's buffer mapped into this process (CUDA IPC), so that
// copies on this GPU's copy engines can write into the peers' buffers over NVLink.
struct qgemm_window_s {
  qgemm_comm_s* comm = nullptr;
  uint64_t local = 0;
  size_t bytes = 0;
  std::vector<uint64_t> peer;  // peer[r]: rank r's buffer as mapped here (peer[rank] = local)
  std::vector<void*> opened;   // allocation bases cudaIpcOpenMemHandle returned
  void* sync = nullptr;        // bf16 [world]: the barrier gathers
};

namespace qg {
namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
#define QG_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
    QG_SYM(GetUniqueId, "ncclGetUniqueId");
    QG_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    QG_SYM(CommInitRank, "ncclCommInitRank");
    QG_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    QG_SYM(CommAbort, "ncclCommAbort");
    QG_SYM(CommDestroy, "ncclCommDestroy");
    QG_SYM(AllGather, "ncclAllGather");
    QG_SYM(GetErrorString, "ncclGetErrorString");
#undef QG_SYM
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllGather;
  });
  return api;
}

qgemm_status nccl_fail(ncclResult_t r, const char* what) {
  NcclApi& n = nccl();
  return fail(QGEMM_ERR_NCCL, "%s: %s (%d)", what,
              n.GetErrorString ? n.GetErrorString(r) : "nccl error", (int)r);
}

// Seconds a rank waits for its peers in qgemm_comm_init (QGEMM_COMM_TIMEOUT_S).
double init_timeout_s() {
  const char* e = getenv("QGEMM_COMM_TIMEOUT_S");
  if (e) {
    double v = atof(e);
    if (v > 0) return v;
  }
  return 120.0;
}

}  // namespace
}  // namespace qg

using namespace qg;

extern "C" {

qgemm_status qgemm_comm_unique_id(void* out) {
  if (!out) return fail(QGEMM_ERR_INVALID_ARG, "out is null");
  NcclApi& n = nccl();
  if (!n.ok) return fail(QGEMM_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  ncclResult_t r = n.GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  memcpy(out, &id, sizeof(id));
  return QGEMM_OK;
}

qgemm_status qgemm_comm_init(qgemm_device_t dev, const void* uid, int rank, int world,
                             qgemm_comm_t* out) {
  if (!out || !uid) return fail(QGEMM_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  if (!dev || !dev->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  if (world < 1 || rank < 0 || rank >= world)
    return fail(QGEMM_ERR_INVALID_ARG, "bad rank %d / world %d", rank, world);
  NcclApi& n = nccl();
  if (!n.ok) return fail(QGEMM_ERR_NCCL, "libnccl.so.2 could not be loaded");
  cudaError_t ce = cudaSetDevice(dev->ordinal);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaSetDevice");
  ncclUniqueId id;
  memcpy(&id, uid, sizeof(id));
  ncclComm_t comm = nullptr;
  if (n.CommInitRankConfig && n.CommGetAsyncError && n.CommAbort) {
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = n.CommInitRankConfig(&comm, world, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclCommInitRankConfig");
    const auto deadline = std::chrono::steady_clock::now() +
                          std::chrono::duration<double>(init_timeout_s());
    ncclResult_t st = ncclInProgress;
    while (true) {
      r = n.CommGetAsyncError(comm, &st);
      if (r != ncclSuccess) { n.CommAbort(comm); return nccl_fail(r, "ncclCommGetAsyncError"); }
      if (st != ncclInProgress) break;
      if (std::chrono::steady_clock::now() > deadline) {
        n.CommAbort(comm);
        return fail(QGEMM_ERR_TIMEOUT, "ncclCommInitRank: peers did not join within %.0f s",
                    init_timeout_s());
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    if (st != ncclSuccess) { n.CommAbort(comm); return nccl_fail(st, "ncclCommInitRank (async)"); }
  } else {
    ncclResult_t r = n.CommInitRank(&comm, world, id, rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
  }
  qgemm_comm_s* c = new (std::nothrow) qgemm_comm_s();
  if (!c) { n.CommDestroy(comm); return fail(QGEMM_ERR_OOM, "host allocation failed"); }
  c->comm = comm;
  c->dev = dev;
  c->rank = rank;
  c->world = world;
  *out = c;
  return QGEMM_OK;
}

qgemm_status qgemm_comm_destroy(qgemm_comm_t c) {
  if (!c) return fail(QGEMM_ERR_BAD_HANDLE, "null communicator");
  if (c->dev) cudaSetDevice(c->dev->ordinal);
  for (cudaEvent_t e : {c->ev_gemm[0], c->ev_gemm[1], c->ev_done[0], c->ev_done[1], c->ev_end,
                        c->ev_start, c->ev_open})
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : c->ev_cp) cudaEventDestroy(e);
  for (cudaStream_t x : c->cp) cudaStreamDestroy(x);
  NcclApi& n = nccl();
  ncclResult_t r = ncclSuccess;
  if (c->comm && n.CommDestroy) r = n.CommDestroy(c->comm);
  delete c;
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommDestroy");
  return QGEMM_OK;
}

qgemm_status qgemm_comm_allgather_bf16(qgemm_comm_t c, qgemm_stream_t s, uint64_t send,
                                       uint64_t recv, size_t count) {
  if (!c || !c->comm) return fail(QGEMM_ERR_BAD_HANDLE, "null communicator");
  qgemm_status st = enter(s);
  if (st != QGEMM_OK) return st;
  if (s->dev != c->dev) return fail(QGEMM_ERR_INVALID_ARG, "stream and communicator devices differ");
  if (count == 0) return QGEMM_OK;
  if (!send || !recv) return fail(QGEMM_ERR_INVALID_ARG, "null buffer");
  NcclApi& n = nccl();
  ncclResult_t r = n.AllGather(reinterpret_cast<const void*>(send), reinterpret_cast<void*>(recv),
                               count, ncclBfloat16, c->comm, s->stream);
  if (r == ncclInProgress && n.CommGetAsyncError) {
    // Non-blocking communicator: wait (bounded) until the call is enqueued.
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
    ncclResult_t as = ncclInProgress;
    while (as == ncclInProgress) {
      if (n.CommGetAsyncError(c->comm, &as) != ncclSuccess) break;
      if (std::chrono::steady_clock::now() > deadline)
        return fail(QGEMM_ERR_TIMEOUT, "ncclAllGather was not enqueued within 60 s");
    }
    r = as;
  }
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
  return QGEMM_OK;
}

// After a call has queued its first collective, its peers wait in that collective or
// the next one for this rank.  A failure after that point aborts the communicator
// (ncclCommAbort), so that NCCL tears down its side of the connections, and marks it
// dead: every later call on it returns QGEMM_ERR_BAD_HANDLE.
static qgemm_status abort_after(qgemm_comm_s* c, qgemm_status st) {
  NcclApi& n = nccl();
  if (c->comm && n.CommAbort) n.CommAbort(c->comm);
  c->comm = nullptr;
  return st;
}

// The argument checks of qgemm_w8a8_gemm for the chunks of a sharded call, made before
// its first collective so that a bad argument fails on the host before any peer waits.
static qgemm_status check_sharded_gemm(uint64_t A, uint64_t B, int b_layout, uint64_t sA,
                                       uint64_t sB, int K) {
  if (b_layout != QGEMM_B_KN && b_layout != QGEMM_B_NK)
    return fail(QGEMM_ERR_INVALID_ARG, "bad b_layout %d", b_layout);
  if (!A || !B || !sA || !sB) return fail(QGEMM_ERR_INVALID_ARG, "null operand");
  if (!aligned(sA, 4) || !aligned(sB, 4)) return fail(QGEMM_ERR_BAD_ALIGN, "sA / sB not 4-byte aligned");
  if (K < 0) return fail(QGEMM_ERR_INVALID_ARG, "K %d < 0", K);
  return QGEMM_OK;
}

// One rank's part of qgemm_comm_window_register, gathered over NCCL.
struct WindowRecord {
  cudaIpcMemHandle_t handle;  // of the allocation that holds the buffer
  uint64_t offset;            // buffer - allocation base
  uint64_t bytes;
  int32_t ok;                 // 0: this rank could not export its buffer
  int32_t pad[5];
};
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "cudaIpcMemHandle_t is 64 bytes");
static_assert(sizeof(WindowRecord) == 104, "WindowRecord layout");

// Streams that carry the window copies: QGEMM_COPY_STREAMS (1 .. world-1), by
// default 1.  Copies to different peers side by side on 3 streams measured slower at
// 4 ranks (layer 2.03 ms against 1.38 ms with one stream).
static int copy_streams(int world) {
  int n = 1;
  if (const char* e = getenv("QGEMM_COPY_STREAMS")) {
    const int v = atoi(e);
    if (v > 0) n = v;
  }
  return n < 1 ? 1 : n > world - 1 ? world - 1 : n;
}

static qgemm_status window_barrier(qgemm_window_s* w, qgemm_stream_s* s) {
  const int r = w->comm->rank;
  return qgemm_comm_allgather_bf16(w->comm, s, reinterpret_cast<uint64_t>(w->sync) + 2 * r,
                                   reinterpret_cast<uint64_t>(w->sync), 1);
}

qgemm_status qgemm_comm_window_register(qgemm_comm_t c, qgemm_stream_t s, uint64_t buf,
                                        size_t bytes, qgemm_window_t* out) {
  if (!out) return fail(QGEMM_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  if (!c || !c->comm) return fail(QGEMM_ERR_BAD_HANDLE, "null communicator");
  qgemm_status st = enter(s);
  if (st != QGEMM_OK) return st;
  if (s->dev != c->dev) return fail(QGEMM_ERR_INVALID_ARG, "stream and communicator devices differ");
  using GetRange = int (*)(uint64_t*, size_t*, uint64_t);  // cuMemGetAddressRange
  static GetRange get_range = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) !=
            cudaSuccess || q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<GetRange>(f);
  }();
  // Every rank takes part in the record gather even when its own export failed, so
  // that all ranks reach the same verdict instead of some of them waiting.
  WindowRecord mine;
  memset(&mine, 0, sizeof(mine));
  uint64_t base = 0;
  size_t range = 0;
  if (buf && bytes && aligned(buf, 16) && get_range && get_range(&base, &range, buf) == 0 &&
      buf + bytes <= base + range &&
      cudaIpcGetMemHandle(&mine.handle, reinterpret_cast<void*>(base)) == cudaSuccess) {
    mine.offset = buf - base;
    mine.bytes = bytes;
    mine.ok = 1;
  }
  cudaGetLastError();
  const int world = c->world;
  const size_t rec = sizeof(WindowRecord);
  void* d = nullptr;
  cudaError_t ce = cudaMalloc(&d, rec * world + 2 * world);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaMalloc");
  std::vector<WindowRecord> all(world);
  uint8_t* dm = static_cast<uint8_t*>(d);
  ce = cudaMemcpyAsync(dm + rec * c->rank, &mine, rec, cudaMemcpyHostToDevice, s->stream);
  if (ce != cudaSuccess) { cudaFree(d); return cuda_fail(ce, "cudaMemcpyAsync"); }
  // rec is a multiple of 2 bytes: the records travel as bf16 elements
  st = qgemm_comm_allgather_bf16(c, s, reinterpret_cast<uint64_t>(dm + rec * c->rank),
                                 reinterpret_cast<uint64_t>(dm), rec / 2);
  if (st != QGEMM_OK) { cudaFree(d); return st; }
  ce = cudaMemcpyAsync(all.data(), dm, rec * world, cudaMemcpyDeviceToHost, s->stream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(s->stream);
  if (ce != cudaSuccess) { cudaFree(d); return cuda_fail(ce, "gathering the window records"); }
  for (int r = 0; r < world; ++r)
    if (!all[r].ok || all[r].bytes != bytes) {
      cudaFree(d);
      return fail(QGEMM_ERR_INVALID_ARG,
                  "rank %d registered no exportable buffer of %zu bytes (a 16-byte aligned "
                  "cudaMalloc allocation, the same size on every rank)", r, bytes);
    }
  qgemm_window_s* w = new (std::nothrow) qgemm_window_s();
  if (!w) { cudaFree(d); return fail(QGEMM_ERR_OOM, "host allocation failed"); }
  w->comm = c;
  w->local = buf;
  w->bytes = bytes;
  w->sync = dm + rec * world;
  w->peer.assign(world, 0);
  cudaError_t open_err = cudaSuccess;
  for (int r = 0; r < world && open_err == cudaSuccess; ++r) {
    if (r == c->rank) { w->peer[r] = buf; continue; }
    void* p = nullptr;
    open_err = cudaIpcOpenMemHandle(&p, all[r].handle, cudaIpcMemLazyEnablePeerAccess);
    if (open_err != cudaSuccess) break;
    w->opened.push_back(p);
    w->peer[r] = reinterpret_cast<uint64_t>(p) + all[r].offset;
  }
  cudaGetLastError();
  // Opening a peer's buffer can fail on one rank only (no peer mapping to one GPU), so
  // every rank reports how its opens went and all of them reach the same verdict: a
  // window on every rank, or the same error on every rank.
  const uint16_t flag = open_err == cudaSuccess ? 0x3F80u : 0u;  // bf16 1.0 or 0
  std::vector<uint16_t> flags(world, 0);
  uint8_t* fl = static_cast<uint8_t*>(w->sync);
  ce = cudaMemcpyAsync(fl + 2 * c->rank, &flag, 2, cudaMemcpyHostToDevice, s->stream);
  if (ce != cudaSuccess) { qgemm_comm_window_release(w); return abort_after(c, cuda_fail(ce, "cudaMemcpyAsync")); }
  st = qgemm_comm_allgather_bf16(c, s, reinterpret_cast<uint64_t>(fl + 2 * c->rank),
                                 reinterpret_cast<uint64_t>(fl), 1);
  if (st != QGEMM_OK) { qgemm_comm_window_release(w); return abort_after(c, st); }
  ce = cudaMemcpyAsync(flags.data(), fl, 2 * world, cudaMemcpyDeviceToHost, s->stream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(s->stream);
  if (ce != cudaSuccess) {
    qgemm_comm_window_release(w);
    return abort_after(c, cuda_fail(ce, "gathering the window open results"));
  }
  for (int r = 0; r < world; ++r)
    if (flags[r] != 0x3F80u) {
      qgemm_comm_window_release(w);
      if (r == c->rank) return cuda_fail(open_err, "cudaIpcOpenMemHandle");
      return fail(QGEMM_ERR_CUDA, "rank %d could not map a peer's buffer (CUDA IPC); no rank "
                  "keeps the window", r);
    }
  *out = w;
  return QGEMM_OK;
}

qgemm_status qgemm_comm_window_release(qgemm_window_t w) {
  if (!w) return fail(QGEMM_ERR_BAD_HANDLE, "null window");
  cudaError_t first = cudaSuccess;
  if (w->comm && w->comm->dev) cudaSetDevice(w->comm->dev->ordinal);
  for (void* p : w->opened) {
    cudaError_t e = cudaIpcCloseMemHandle(p);
    if (first == cudaSuccess) first = e;
  }
  // the barrier bytes sit at the end of the record block allocated with them
  if (w->sync) {
    uint8_t* base = static_cast<uint8_t*>(w->sync) - sizeof(WindowRecord) * w->peer.size();
    cudaError_t e = cudaFree(base);
    if (first == cudaSuccess) first = e;
  }
  delete w;
  if (first != cudaSuccess) return cuda_fail(first, "releasing the window");
  return QGEMM_OK;
}

qgemm_status qgemm_w8a8_gemm_allgather_window_bf16(qgemm_window_t w, qgemm_stream_t s,
                                                   qgemm_stream_t cs, uint64_t A, uint64_t B,
                                                   int b_layout, uint64_t sA, uint64_t sB, int M,
                                                   int N_local, int K, int chunk_rows) {
  if (!w || !w->comm || !w->comm->comm) return fail(QGEMM_ERR_BAD_HANDLE, "null window");
  qgemm_comm_s* c = w->comm;
  qgemm_status st = enter(cs);
  if (st != QGEMM_OK) return st;
  st = enter(s);
  if (st != QGEMM_OK) return st;
  if (s->dev != c->dev || cs->dev != c->dev)
    return fail(QGEMM_ERR_INVALID_ARG, "streams and communicator are on different devices");
  if (s == cs || s->stream == cs->stream)
    return fail(QGEMM_ERR_INVALID_ARG, "the GEMM and the copies need two different streams");
  if (M < 0 || N_local < 0 || K < 0 || chunk_rows < 1)
    return fail(QGEMM_ERR_INVALID_ARG, "bad sizes M=%d N_local=%d K=%d chunk_rows=%d", M,
                N_local, K, chunk_rows);
  const int world = c->world, rank = c->rank;
  const size_t N = (size_t)N_local * world;
  if ((size_t)M * N * 2 > w->bytes)
    return fail(QGEMM_ERR_INVALID_ARG, "the window holds %zu bytes; [%d, %zu] bf16 needs %zu",
                w->bytes, M, N, (size_t)M * N * 2);
  if (M == 0 || N_local == 0) return QGEMM_OK;
  if ((st = check_sharded_gemm(A, B, b_layout, sA, sB, K)) != QGEMM_OK) return st;
  for (cudaEvent_t* e : {&c->ev_gemm[0], &c->ev_gemm[1], &c->ev_end, &c->ev_start, &c->ev_open})
    if (!*e) {
      cudaError_t ce = cudaEventCreateWithFlags(e, cudaEventDisableTiming);
      if (ce != cudaSuccess) return cuda_fail(ce, "cudaEventCreate");
    }
  const int ncp = copy_streams(world);
  while ((int)c->cp.size() < ncp) {
    cudaStream_t x = nullptr;
    cudaEvent_t e = nullptr;
    cudaError_t ce = cudaStreamCreateWithFlags(&x, cudaStreamNonBlocking);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamCreate");
    ce = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    if (ce != cudaSuccess) { cudaStreamDestroy(x); return cuda_fail(ce, "cudaEventCreate"); }
    c->cp.push_back(x);
    c->ev_cp.push_back(e);
  }
  // every rank is done with its earlier uses of the buffer before a peer writes into it
  cudaError_t ce = cudaEventRecord(c->ev_start, s->stream);
  if (ce == cudaSuccess) ce = cudaStreamWaitEvent(cs->stream, c->ev_start, 0);
  if (ce != cudaSuccess) return cuda_fail(ce, "ordering the copy stream after the caller's work");
  if ((st = window_barrier(w, cs)) != QGEMM_OK) return abort_after(c, st);
  // from here on every failure aborts the communicator (abort_after)
  ce = cudaEventRecord(c->ev_open, cs->stream);
  for (int k = 0; k < ncp && ce == cudaSuccess; ++k)
    ce = cudaStreamWaitEvent(c->cp[k], c->ev_open, 0);
  if (ce != cudaSuccess) return abort_after(c, cuda_fail(ce, "ordering the copies after the barrier"));
  const int R = chunk_rows < M ? chunk_rows : M;
  const size_t pitch = N * 2, width = (size_t)N_local * 2;
  for (int m0 = 0, i = 0; m0 < M; m0 += R, ++i) {
    const int rows = (M - m0) < R ? (M - m0) : R;
    const size_t off = (size_t)m0 * pitch + (size_t)rank * width;  // this rank's columns
    st = qgemm_w8a8_gemm(s, A + (uint64_t)m0 * K, B, b_layout, sA + (uint64_t)m0 * 4, sB,
                         w->local + off, QGEMM_BF16, (int)N, rows, N_local, K, 0,
                         QGEMM_ALGO_AUTO);
    if (st != QGEMM_OK) return abort_after(c, st);
    cudaEvent_t ev = c->ev_gemm[i & 1];
    if ((ce = cudaEventRecord(ev, s->stream)) != cudaSuccess)
      return abort_after(c, cuda_fail(ce, "cudaEventRecord"));
    for (int k = 0; k < ncp; ++k)
      if ((ce = cudaStreamWaitEvent(c->cp[k], ev, 0)) != cudaSuccess)
        return abort_after(c, cuda_fail(ce, "event between the GEMM and the copies"));
    for (int j = 1; j < world; ++j) {  // peers in rank order from this rank's right
      const int p = (rank + j) % world;
      ce = cudaMemcpy2DAsync(reinterpret_cast<void*>(w->peer[p] + off), pitch,
                             reinterpret_cast<const void*>(w->local + off), pitch, width, rows,
                             cudaMemcpyDeviceToDevice, c->cp[(j - 1) % ncp]);
      if (ce != cudaSuccess) return abort_after(c, cuda_fail(ce, "cudaMemcpy2DAsync to a peer"));
    }
  }
  for (int k = 0; k < ncp; ++k)
    if ((ce = cudaEventRecord(c->ev_cp[k], c->cp[k])) != cudaSuccess ||
        (ce = cudaStreamWaitEvent(cs->stream, c->ev_cp[k], 0)) != cudaSuccess)
      return abort_after(c, cuda_fail(ce, "joining the copy streams"));
  // every peer's columns have landed here once every rank has finished its copies
  if ((st = window_barrier(w, cs)) != QGEMM_OK) return abort_after(c, st);
  ce = cudaEventRecord(c->ev_end, cs->stream);
  if (ce == cudaSuccess) ce = cudaStreamWaitEvent(s->stream, c->ev_end, 0);
  if (ce != cudaSuccess) return abort_after(c, cuda_fail(ce, "joining the copy stream"));
  return QGEMM_OK;
}

// The GEMM and the all-gather as one kernel: the epilogue stores each output chunk into
// this rank's columns of its own window and, by TMA stores over NVLink from the same
// staging buffer, into the same columns of every peer's window.  The transfer of a
// tile overlaps the MMAs of the next (two TMEM accumulators), so the layer takes the
// longer of the GEMM and this rank's egress (N_local * M * 2 bytes to each of world-1
// peers) instead of their sum.
qgemm_status qgemm_w8a8_gemm_allgather_fused_bf16(qgemm_window_t w, qgemm_stream_t s, uint64_t A,
                                                  uint64_t B, int b_layout, uint64_t sA,
                                                  uint64_t sB, int M, int N_local, int K) {
  if (!w || !w->comm || !w->comm->comm) return fail(QGEMM_ERR_BAD_HANDLE, "null window");
  qgemm_comm_s* c = w->comm;
  qgemm_status st = enter(s);
  if (st != QGEMM_OK) return st;
  if (s->dev != c->dev)
    return fail(QGEMM_ERR_INVALID_ARG, "stream and communicator are on different devices");
  if (M < 0 || N_local < 0 || K < 0)
    return fail(QGEMM_ERR_INVALID_ARG, "bad sizes M=%d N_local=%d K=%d", M, N_local, K);
  const int world = c->world, rank = c->rank;
  if (world - 1 > 7)
    return fail(QGEMM_ERR_UNSUPPORTED, "the fused form stores to at most 7 peers (world %d)", world);
  const size_t N = (size_t)N_local * world;
  if ((size_t)M * N * 2 > w->bytes)
    return fail(QGEMM_ERR_INVALID_ARG, "the window holds %zu bytes; [%d, %zu] bf16 needs %zu",
                w->bytes, M, N, (size_t)M * N * 2);
  if (M == 0 || N_local == 0) return QGEMM_OK;
  if ((st = check_sharded_gemm(A, B, b_layout, sA, sB, K)) != QGEMM_OK) return st;
  // every check that depends on the shape, before the first collective: the same
  // verdict on every rank
  const size_t off = (size_t)rank * N_local * 2;  // this rank's columns, row 0
  const char* why = nullptr;
  if (K == 0 || N_local % 8 != 0 ||
      !w8a8_tcgen05_supported(c->dev, A, B, b_layout == QGEMM_B_KN, w->local + off, QGEMM_BF16,
                              (int)N, M, N_local, K, &why))
    return fail(QGEMM_ERR_UNSUPPORTED, "the fused form needs the tcgen05 GEMM with the TMA-store "
                "epilogue (K > 0, N_local %% 8 == 0)%s%s", why ? ": " : "", why ? why : "");
  uint64_t peers[7] = {};
  int np = 0;
  for (int j = 1; j < world; ++j) peers[np++] = w->peer[(rank + j) % world] + off;
  // every rank is done with its earlier uses of its window before a peer writes into it
  if ((st = window_barrier(w, s)) != QGEMM_OK) return abort_after(c, st);
  st = launch_w8a8_tcgen05_peers(s, reinterpret_cast<const void*>(A),
                                 reinterpret_cast<const void*>(B), b_layout == QGEMM_B_KN,
                                 reinterpret_cast<const float*>(sA),
                                 reinterpret_cast<const float*>(sB),
                                 reinterpret_cast<void*>(w->local + off), (int)N, M, N_local, K,
                                 peers, np);
  if (st != QGEMM_OK) return abort_after(c, st);
  // every peer's columns have landed here once every rank's GEMM has finished
  if ((st = window_barrier(w, s)) != QGEMM_OK) return abort_after(c, st);
  return QGEMM_OK;
}

size_t qgemm_w8a8_allgather_work_bytes(int world, int chunk_rows, int n_local) {
  if (world < 1 || chunk_rows < 1 || n_local < 1) return 0;
  return (size_t)2 * world * chunk_rows * n_local * 2;
}

qgemm_status qgemm_w8a8_gemm_allgather_bf16(qgemm_comm_t c, qgemm_stream_t s, qgemm_stream_t cs,
                                            uint64_t A, uint64_t B, int b_layout, uint64_t sA,
                                            uint64_t sB, uint64_t out, int M, int N_local, int K,
                                            int chunk_rows, uint64_t work, size_t work_bytes) {
  if (!c || !c->comm) return fail(QGEMM_ERR_BAD_HANDLE, "null communicator");
  qgemm_status st = enter(cs);
  if (st != QGEMM_OK) return st;
  st = enter(s);
  if (st != QGEMM_OK) return st;
  if (s->dev != c->dev || cs->dev != c->dev)
    return fail(QGEMM_ERR_INVALID_ARG, "streams and communicator are on different devices");
  if (s == cs || s->stream == cs->stream)
    return fail(QGEMM_ERR_INVALID_ARG, "the GEMM and the gather need two different streams");
  if (M < 0 || N_local < 0 || K < 0 || chunk_rows < 1)
    return fail(QGEMM_ERR_INVALID_ARG, "bad sizes M=%d N_local=%d K=%d chunk_rows=%d", M,
                N_local, K, chunk_rows);
  if (M == 0 || N_local == 0) return QGEMM_OK;
  const int world = c->world, rank = c->rank;
  const int R = chunk_rows < M ? chunk_rows : M;
  const size_t need = qgemm_w8a8_allgather_work_bytes(world, R, N_local);
  if (!work || work_bytes < need)
    return fail(QGEMM_ERR_INVALID_ARG, "work buffer of %zu bytes; %zu needed", work_bytes, need);
  if (!aligned(work, 16)) return fail(QGEMM_ERR_BAD_ALIGN, "work must be 16-byte aligned");
  if (!out) return fail(QGEMM_ERR_INVALID_ARG, "out is null");
  if ((st = check_sharded_gemm(A, B, b_layout, sA, sB, K)) != QGEMM_OK) return st;
  for (cudaEvent_t* e : {&c->ev_gemm[0], &c->ev_gemm[1], &c->ev_done[0], &c->ev_done[1], &c->ev_end})
    if (!*e) {
      cudaError_t ce = cudaEventCreateWithFlags(e, cudaEventDisableTiming);
      if (ce != cudaSuccess) return cuda_fail(ce, "cudaEventCreate");
    }
  const size_t slot_bytes = (size_t)world * R * N_local * 2;
  const int N = N_local * world;
  const int nchunks = (M + R - 1) / R;
  // Failures before the first gather is queued return on this rank alone (no peer waits
  // yet); after it they abort the communicator (abort_after).
  bool queued = false;
  auto bail = [&](qgemm_status e) { return queued ? abort_after(c, e) : e; };
  for (int i = 0; i < nchunks; ++i) {
    const int b = i & 1, m0 = i * R, rows = (M - m0) < R ? (M - m0) : R;
    const uint64_t buf = work + (uint64_t)b * slot_bytes;  // [world][rows][N_local]
    const size_t blk = (size_t)rows * N_local;             // bf16 elements per rank
    const uint64_t mine = buf + (uint64_t)rank * blk * 2;
    cudaError_t ce = cudaSuccess;
    if (i >= 2) ce = cudaStreamWaitEvent(s->stream, c->ev_done[b], 0);  // chunk i-2 let go of buf
    if (ce != cudaSuccess) return bail(cuda_fail(ce, "cudaStreamWaitEvent"));
    st = qgemm_w8a8_gemm(s, A + (uint64_t)m0 * K, B, b_layout, sA + (uint64_t)m0 * 4, sB, mine,
                         QGEMM_BF16, N_local, rows, N_local, K, 0, QGEMM_ALGO_AUTO);
    if (st != QGEMM_OK) return bail(st);
    if ((ce = cudaEventRecord(c->ev_gemm[b], s->stream)) != cudaSuccess ||
        (ce = cudaStreamWaitEvent(cs->stream, c->ev_gemm[b], 0)) != cudaSuccess)
      return bail(cuda_fail(ce, "event between the GEMM and the gather"));
    st = qgemm_comm_allgather_bf16(c, cs, mine, buf, blk);  // in place
    queued = true;
    if (st != QGEMM_OK) return bail(st);
    st = qgemm_unshard_columns_bf16(cs, buf, out + (uint64_t)m0 * N * 2, world, rows, N_local);
    if (st != QGEMM_OK) return bail(st);
    if ((ce = cudaEventRecord(c->ev_done[b], cs->stream)) != cudaSuccess)
      return bail(cuda_fail(ce, "cudaEventRecord"));
  }
  cudaError_t ce = cudaEventRecord(c->ev_end, cs->stream);
  if (ce == cudaSuccess) ce = cudaStreamWaitEvent(s->stream, c->ev_end, 0);
  if (ce != cudaSuccess) return bail(cuda_fail(ce, "joining the gather stream"));
  return QGEMM_OK;
}

}  // extern "C"
