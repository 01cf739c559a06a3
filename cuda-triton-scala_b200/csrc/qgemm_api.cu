// qgemm_api.cu -- the extern "C" boundary of libqgemm (include/qgemm.h):
// status and last-error handling, device / stream / buffer handles, argument
// checking and dispatch of the reference operator entry points.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "internal.h"

namespace qg {

static thread_local char g_last_error[512] = "";

qgemm_status fail(qgemm_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return s;
}

qgemm_status cuda_fail(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return QGEMM_OK;
  if (e == cudaErrorMemoryAllocation)
    return fail(QGEMM_ERR_OOM, "%s: %s", what, cudaGetErrorString(e));
  return fail(QGEMM_ERR_CUDA, "%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
}

qgemm_status enter(qgemm_stream_t s) {
  if (!s || !s->dev || !s->dev->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed stream");
  cudaError_t e = cudaSetDevice(s->dev->ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  return QGEMM_OK;
}

}  // namespace qg

using namespace qg;

#define QG_TRY(expr)                     \
  do {                                   \
    qgemm_status _st = (expr);           \
    if (_st != QGEMM_OK) return _st;     \
  } while (0)

static qgemm_status check_dims(int M, int N, int K) {
  if (M < 0 || N < 0 || K < 0) return fail(QGEMM_ERR_INVALID_ARG, "negative size M=%d N=%d K=%d", M, N, K);
  return QGEMM_OK;
}

static qgemm_status need(uint64_t p, const char* name) {
  if (p == 0) return fail(QGEMM_ERR_INVALID_ARG, "%s is null", name);
  return QGEMM_OK;
}

static qgemm_status need_align(uint64_t p, uint64_t a, const char* name) {
  if (!aligned(p, a)) return fail(QGEMM_ERR_BAD_ALIGN, "%s is not %llu-byte aligned", name, (unsigned long long)a);
  return QGEMM_OK;
}

namespace qg {
qgemm_status stream_workspace(qgemm_stream_s* s, size_t bytes, void** out) {
  if (s->ws && s->ws_bytes >= bytes) {
    *out = s->ws;
    return QGEMM_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(s->stream, &cs);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  if (cs != cudaStreamCaptureStatusNone)
    return fail(QGEMM_ERR_UNSUPPORTED,
                "this call needs the stream handle's scratch (%zu bytes), which is made by the "
                "first such call on the handle: make one call before capturing the stream",
                bytes);
  if (s->ws) {
    cudaStreamSynchronize(s->stream);
    cudaFree(s->ws);
    s->ws = nullptr;
    s->ws_bytes = 0;
  }
  void* p = nullptr;
  e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(QGEMM_ERR_OOM, "scratch allocation of %zu bytes failed", bytes);
  }
  e = cudaMemsetAsync(p, 0, bytes, s->stream);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "zeroing the scratch");
  }
  s->ws = p;
  s->ws_bytes = bytes;
  *out = p;
  return QGEMM_OK;
}
}  // namespace qg

extern "C" {

const char* qgemm_last_error(void) { return g_last_error; }

const char* qgemm_status_string(qgemm_status s) {
  switch (s) {
    case QGEMM_OK: return "QGEMM_OK";
    case QGEMM_ERR_INVALID_ARG: return "QGEMM_ERR_INVALID_ARG";
    case QGEMM_ERR_BAD_ALIGN: return "QGEMM_ERR_BAD_ALIGN";
    case QGEMM_ERR_CUDA: return "QGEMM_ERR_CUDA";
    case QGEMM_ERR_NCCL: return "QGEMM_ERR_NCCL";
    case QGEMM_ERR_TIMEOUT: return "QGEMM_ERR_TIMEOUT";
    case QGEMM_ERR_UNSUPPORTED: return "QGEMM_ERR_UNSUPPORTED";
    case QGEMM_ERR_NO_DEVICE: return "QGEMM_ERR_NO_DEVICE";
    case QGEMM_ERR_OOM: return "QGEMM_ERR_OOM";
    case QGEMM_ERR_BAD_HANDLE: return "QGEMM_ERR_BAD_HANDLE";
    default: return "QGEMM_ERR_UNKNOWN";
  }
}

int qgemm_version(void) { return 10000; }

// ---- devices ----

qgemm_status qgemm_device_count(int* count) {
  if (!count) return fail(QGEMM_ERR_INVALID_ARG, "count is null");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    *count = 0;
    cudaGetLastError();
    return QGEMM_OK;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  *count = n;
  return QGEMM_OK;
}

qgemm_status qgemm_device_open(int ordinal, qgemm_device_t* out) {
  if (!out) return fail(QGEMM_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  int n = 0;
  QG_TRY(qgemm_device_count(&n));
  if (ordinal < 0 || ordinal >= n)
    return fail(QGEMM_ERR_NO_DEVICE, "device %d not present (%d visible)", ordinal, n);
  cudaError_t e = cudaSetDevice(ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  qgemm_device_s* d = new (std::nothrow) qgemm_device_s();
  if (!d) return fail(QGEMM_ERR_OOM, "host allocation failed");
  d->ordinal = ordinal;
  d->sm_count = prop.multiProcessorCount;
  d->cc_major = prop.major;
  d->cc_minor = prop.minor;
  d->l2_bytes = prop.l2CacheSize;
  d->smem_optin = prop.sharedMemPerBlockOptin;
  // The library carries sm_100a code only: tcgen05/TMEM need compute capability 10.0.
  d->tcgen05 = (prop.major == 10 && prop.minor == 0);
  e = cudaMalloc(&d->d_err, 256);
  if (e == cudaSuccess) e = cudaMemset(d->d_err, 0, 256);
  if (e != cudaSuccess) {
    delete d;
    return cuda_fail(e, "device error word");
  }
  d->open = true;
  *out = d;
  return QGEMM_OK;
}

qgemm_status qgemm_device_close(qgemm_device_t d) {
  if (!d || !d->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  cudaSetDevice(d->ordinal);
  cudaFree(d->d_err);
  d->open = false;
  delete d;
  return QGEMM_OK;
}

qgemm_status qgemm_device_info(qgemm_device_t d, int* sm_count, int* cc_major, int* cc_minor,
                               size_t* l2_bytes, int* has_tcgen05) {
  if (!d || !d->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  if (sm_count) *sm_count = d->sm_count;
  if (cc_major) *cc_major = d->cc_major;
  if (cc_minor) *cc_minor = d->cc_minor;
  if (l2_bytes) *l2_bytes = d->l2_bytes;
  if (has_tcgen05) *has_tcgen05 = d->tcgen05 ? 1 : 0;
  return QGEMM_OK;
}

qgemm_status qgemm_device_set_wait_limit(qgemm_device_t d, uint64_t limit_ns) {
  if (!d || !d->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  if (limit_ns < 1000 || limit_ns > 60000000000ull)
    return fail(QGEMM_ERR_INVALID_ARG, "wait limit %llu ns outside [1 us, 60 s]",
                (unsigned long long)limit_ns);
  d->wait_ns = limit_ns;
  return QGEMM_OK;
}

qgemm_status qgemm_device_get_wait_limit(qgemm_device_t d, uint64_t* limit_ns) {
  if (!d || !d->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  if (!limit_ns) return fail(QGEMM_ERR_INVALID_ARG, "limit_ns is null");
  *limit_ns = d->wait_ns;
  return QGEMM_OK;
}

qgemm_status qgemm_debug_hold_split(qgemm_device_t d, int enable) {
  if (!d || !d->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  d->hold_split = enable ? 1 : 0;
  return QGEMM_OK;
}

// ---- streams ----

qgemm_status qgemm_stream_create(qgemm_device_t d, qgemm_stream_t* out) {
  if (!out) return fail(QGEMM_ERR_INVALID_ARG, "out is null");
  if (!d || !d->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  cudaError_t e = cudaSetDevice(d->ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  cudaStream_t st;
  e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate");
  qgemm_stream_s* s = new (std::nothrow) qgemm_stream_s();
  if (!s) {
    cudaStreamDestroy(st);
    return fail(QGEMM_ERR_OOM, "host allocation failed");
  }
  s->dev = d;
  s->stream = st;
  s->owned = true;
  *out = s;
  return QGEMM_OK;
}

qgemm_status qgemm_stream_wrap(qgemm_device_t d, void* cuda_stream, qgemm_stream_t* out) {
  if (!out) return fail(QGEMM_ERR_INVALID_ARG, "out is null");
  if (!d || !d->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  qgemm_stream_s* s = new (std::nothrow) qgemm_stream_s();
  if (!s) return fail(QGEMM_ERR_OOM, "host allocation failed");
  s->dev = d;
  s->stream = static_cast<cudaStream_t>(cuda_stream);
  s->owned = false;
  *out = s;
  return QGEMM_OK;
}

qgemm_status qgemm_stream_destroy(qgemm_stream_t s) {
  if (!s) return fail(QGEMM_ERR_BAD_HANDLE, "null stream");
  if (s->dev && s->dev->open) {
    cudaSetDevice(s->dev->ordinal);
    if (s->ws) {
      // kernels of this handle may still be using the scratch
      cudaStreamSynchronize(s->stream);
      cudaFree(s->ws);
    }
    if (s->owned) cudaStreamDestroy(s->stream);
  }
  delete s;
  return QGEMM_OK;
}


qgemm_status qgemm_stream_sync(qgemm_stream_t s) {
  QG_TRY(enter(s));
  cudaError_t e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int err = 0;
  e = cudaMemcpyAsync(&err, s->dev->d_err, sizeof(int), cudaMemcpyDeviceToHost, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (err != DEVERR_NONE) {
    const int zero = 0;
    cudaMemcpyAsync(s->dev->d_err, &zero, sizeof(int), cudaMemcpyHostToDevice, s->stream);
    // a kernel that gave up may have left split-tile counters raised
    if (s->ws) cudaMemsetAsync(s->ws, 0, s->ws_bytes, s->stream);
    cudaStreamSynchronize(s->stream);
    return fail(QGEMM_ERR_TIMEOUT, "a device-side wait ran out (code %d)", err);
  }
  return QGEMM_OK;
}

// ---- buffers ----

qgemm_status qgemm_buffer_alloc(qgemm_device_t d, size_t bytes, uint64_t* addr) {
  if (!addr) return fail(QGEMM_ERR_INVALID_ARG, "addr is null");
  if (!d || !d->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  *addr = 0;
  cudaError_t e = cudaSetDevice(d->ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  void* p = nullptr;
  e = cudaMalloc(&p, bytes ? bytes : 1);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  *addr = reinterpret_cast<uint64_t>(p);
  return QGEMM_OK;
}

qgemm_status qgemm_buffer_free(qgemm_device_t d, uint64_t addr) {
  if (!d || !d->open) return fail(QGEMM_ERR_BAD_HANDLE, "null or closed device");
  if (!addr) return QGEMM_OK;
  cudaSetDevice(d->ordinal);
  return cuda_fail(cudaFree(reinterpret_cast<void*>(addr)), "cudaFree");
}

qgemm_status qgemm_memcpy_h2d(qgemm_stream_t s, uint64_t dst, const void* src, size_t bytes) {
  QG_TRY(enter(s));
  if (!bytes) return QGEMM_OK;
  if (!dst || !src) return fail(QGEMM_ERR_INVALID_ARG, "null pointer");
  return cuda_fail(cudaMemcpyAsync(reinterpret_cast<void*>(dst), src, bytes,
                                   cudaMemcpyHostToDevice, s->stream),
                   "cudaMemcpyAsync H2D");
}

qgemm_status qgemm_memcpy_d2h(qgemm_stream_t s, void* dst, uint64_t src, size_t bytes) {
  QG_TRY(enter(s));
  if (!bytes) return QGEMM_OK;
  if (!dst || !src) return fail(QGEMM_ERR_INVALID_ARG, "null pointer");
  return cuda_fail(cudaMemcpyAsync(dst, reinterpret_cast<const void*>(src), bytes,
                                   cudaMemcpyDeviceToHost, s->stream),
                   "cudaMemcpyAsync D2H");
}

qgemm_status qgemm_memset(qgemm_stream_t s, uint64_t dst, int value, size_t bytes) {
  QG_TRY(enter(s));
  if (!bytes) return QGEMM_OK;
  if (!dst) return fail(QGEMM_ERR_INVALID_ARG, "null pointer");
  return cuda_fail(cudaMemsetAsync(reinterpret_cast<void*>(dst), value, bytes, s->stream),
                   "cudaMemsetAsync");
}

qgemm_status qgemm_host_alloc(size_t bytes, void** out) {
  if (!out) return fail(QGEMM_ERR_INVALID_ARG, "out is null");
  return cuda_fail(cudaMallocHost(out, bytes ? bytes : 1), "cudaMallocHost");
}

qgemm_status qgemm_host_free(void* p) {
  if (!p) return QGEMM_OK;
  return cuda_fail(cudaFreeHost(p), "cudaFreeHost");
}

// ---- W8A8 ----

qgemm_status qgemm_w8a8_gemm(qgemm_stream_t s, uint64_t A, uint64_t B, int b_layout,
                             uint64_t sA, uint64_t sB, uint64_t out, int out_dtype, int ldc,
                             int M, int N, int K, uint64_t acc_i32, int algo) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (b_layout != QGEMM_B_KN && b_layout != QGEMM_B_NK)
    return fail(QGEMM_ERR_INVALID_ARG, "bad b_layout %d", b_layout);
  if (out_dtype != QGEMM_F32 && out_dtype != QGEMM_BF16)
    return fail(QGEMM_ERR_INVALID_ARG, "bad out_dtype %d", out_dtype);
  if (algo < QGEMM_ALGO_AUTO || algo > QGEMM_ALGO_SIMT)
    return fail(QGEMM_ERR_INVALID_ARG, "bad algo %d", algo);
  if (M == 0 || N == 0) return QGEMM_OK;
  if (ldc < N) return fail(QGEMM_ERR_INVALID_ARG, "ldc %d < N %d", ldc, N);
  QG_TRY(need(A, "A")); QG_TRY(need(B, "B")); QG_TRY(need(sA, "sA"));
  QG_TRY(need(sB, "sB")); QG_TRY(need(out, "out"));
  QG_TRY(need_align(sA, 4, "sA")); QG_TRY(need_align(sB, 4, "sB"));
  QG_TRY(need_align(out, out_dtype == QGEMM_F32 ? 4 : 2, "out"));
  QG_TRY(need_align(acc_i32, 4, "acc_i32"));
  const int b_kn = b_layout == QGEMM_B_KN;
  const char* why = nullptr;
  const bool tc = K > 0 && w8a8_tcgen05_supported(s->dev, A, B, b_kn, out, out_dtype, ldc, M,
                                                  N, K, &why);
  if (algo == QGEMM_ALGO_TCGEN05 && !tc)
    return fail(QGEMM_ERR_UNSUPPORTED, "tcgen05 W8A8 path unavailable: %s",
                why ? why : "K == 0");
  if (algo != QGEMM_ALGO_SIMT && tc)
    return launch_w8a8_tcgen05(s, reinterpret_cast<const void*>(A),
                               reinterpret_cast<const void*>(B), b_kn,
                               reinterpret_cast<const float*>(sA),
                               reinterpret_cast<const float*>(sB), reinterpret_cast<void*>(out),
                               out_dtype, ldc, M, N, K, reinterpret_cast<int32_t*>(acc_i32));
  return launch_w8a8_simt(s, reinterpret_cast<const int8_t*>(A),
                          reinterpret_cast<const int8_t*>(B), b_kn,
                          reinterpret_cast<const float*>(sA), reinterpret_cast<const float*>(sB),
                          reinterpret_cast<void*>(out), out_dtype, ldc, M, N, K,
                          reinterpret_cast<int32_t*>(acc_i32));
}

qgemm_status qgemm_w8a8_gemm_static_scratch(qgemm_stream_t s, uint64_t A, uint64_t B,
                                            int b_layout, uint64_t sA, uint64_t sB, uint64_t out,
                                            int out_dtype, int ldc, int M, int N, int K,
                                            uint64_t acc_i32, int algo) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (b_layout != QGEMM_B_KN && b_layout != QGEMM_B_NK)
    return fail(QGEMM_ERR_INVALID_ARG, "bad b_layout %d", b_layout);
  if (out_dtype != QGEMM_F32 && out_dtype != QGEMM_BF16)
    return fail(QGEMM_ERR_INVALID_ARG, "bad out_dtype %d", out_dtype);
  if (algo < QGEMM_ALGO_AUTO || algo > QGEMM_ALGO_SIMT)
    return fail(QGEMM_ERR_INVALID_ARG, "bad algo %d", algo);
  if (M == 0 || N == 0) return QGEMM_OK;
  if (ldc < N) return fail(QGEMM_ERR_INVALID_ARG, "ldc %d < N %d", ldc, N);
  QG_TRY(need(A, "A")); QG_TRY(need(B, "B")); QG_TRY(need(sA, "sA"));
  QG_TRY(need(sB, "sB")); QG_TRY(need(out, "out"));
  QG_TRY(need_align(sA, 4, "sA")); QG_TRY(need_align(sB, 4, "sB"));
  QG_TRY(need_align(out, out_dtype == QGEMM_F32 ? 4 : 2, "out"));
  QG_TRY(need_align(acc_i32, 4, "acc_i32"));
  const int b_kn = b_layout == QGEMM_B_KN;
  const char* why = nullptr;
  const bool tc = K > 0 && w8a8_tcgen05_supported(s->dev, A, B, b_kn, out, out_dtype, ldc, M,
                                                  N, K, &why);
  if (algo == QGEMM_ALGO_TCGEN05 && !tc)
    return fail(QGEMM_ERR_UNSUPPORTED, "tcgen05 W8A8 path unavailable: %s",
                why ? why : "K == 0");
  if (algo != QGEMM_ALGO_SIMT && tc)
    return launch_w8a8_tcgen05_static(s, reinterpret_cast<const void*>(A),
                                      reinterpret_cast<const void*>(B), b_kn,
                                      reinterpret_cast<const float*>(sA),
                                      reinterpret_cast<const float*>(sB),
                                      reinterpret_cast<void*>(out), out_dtype, ldc, M, N, K,
                                      reinterpret_cast<int32_t*>(acc_i32));
  return launch_w8a8_simt(s, reinterpret_cast<const int8_t*>(A),
                          reinterpret_cast<const int8_t*>(B), b_kn,
                          reinterpret_cast<const float*>(sA), reinterpret_cast<const float*>(sB),
                          reinterpret_cast<void*>(out), out_dtype, ldc, M, N, K,
                          reinterpret_cast<int32_t*>(acc_i32));
}

qgemm_status qgemm_w8a32_gemm(qgemm_stream_t s, uint64_t wInt8, uint64_t scalesW, uint64_t x,
                              uint64_t scalesX, uint64_t y, int M, int N, int K) {
  return qgemm_w8a8_gemm(s, x, wInt8, QGEMM_B_KN, scalesX, scalesW, y, QGEMM_F32, N, M, N, K, 0,
                         QGEMM_ALGO_AUTO);
}

// ---- W4A16 ----

qgemm_status qgemm_w4a16_gemm(qgemm_stream_t s, uint64_t wInt4, uint64_t scalesW, uint64_t x,
                              uint64_t y, int M, int N, int K) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (M == 0 || N == 0) return QGEMM_OK;
  if (K > 0) { QG_TRY(need(wInt4, "wInt4")); QG_TRY(need(x, "x")); }
  QG_TRY(need(scalesW, "scalesW")); QG_TRY(need(y, "y"));
  QG_TRY(need_align(scalesW, 4, "scalesW")); QG_TRY(need_align(x, 4, "x"));
  QG_TRY(need_align(y, 4, "y"));
  return launch_w4a16_ref(s, reinterpret_cast<const uint8_t*>(wInt4),
                          reinterpret_cast<const float*>(scalesW),
                          reinterpret_cast<const float*>(x), reinterpret_cast<float*>(y), M, N, K);
}

qgemm_status qgemm_w4a16_grouped_gemm(qgemm_stream_t s, uint64_t x, uint64_t wq,
                                      uint64_t scales, int zero_point, int group_size,
                                      uint64_t y, int M, int N, int K) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (group_size <= 0) return fail(QGEMM_ERR_INVALID_ARG, "group_size %d <= 0", group_size);
  if (zero_point < 0 || zero_point > 15)
    return fail(QGEMM_ERR_INVALID_ARG, "zero_point %d outside [0,15]", zero_point);
  if (N % 8 != 0) return fail(QGEMM_ERR_INVALID_ARG, "N %d is not a multiple of 8", N);
  if (K % group_size != 0)
    return fail(QGEMM_ERR_INVALID_ARG, "K %d is not a multiple of group_size %d", K, group_size);
  if (M == 0 || N == 0) return QGEMM_OK;
  QG_TRY(need(y, "y"));
  if (K > 0) { QG_TRY(need(x, "x")); QG_TRY(need(wq, "wq")); QG_TRY(need(scales, "scales")); }
  QG_TRY(need_align(x, 2, "x")); QG_TRY(need_align(wq, 4, "wq"));
  QG_TRY(need_align(scales, 2, "scales")); QG_TRY(need_align(y, 2, "y"));
  return launch_w4a16_grouped(s, reinterpret_cast<const void*>(x),
                              reinterpret_cast<const uint32_t*>(wq),
                              reinterpret_cast<const void*>(scales), zero_point, group_size,
                              reinterpret_cast<void*>(y), M, N, K);
}

qgemm_status qgemm_w4_tiled_bytes(int K, int N, size_t* bytes) {
  if (!bytes) return fail(QGEMM_ERR_INVALID_ARG, "bytes is null");
  if (K < 0 || N < 0 || N % 8 != 0) return fail(QGEMM_ERR_INVALID_ARG, "bad K=%d N=%d", K, N);
  *bytes = w4_tiled_bytes(K, N);
  return QGEMM_OK;
}

qgemm_status qgemm_prepack_w4_tiled(qgemm_stream_t s, uint64_t wq, uint64_t dst, int K, int N) {
  QG_TRY(enter(s));
  if (K < 0 || N < 0 || N % 8 != 0) return fail(QGEMM_ERR_INVALID_ARG, "bad K=%d N=%d", K, N);
  if (K == 0 || N == 0) return QGEMM_OK;
  QG_TRY(need(wq, "wq")); QG_TRY(need(dst, "dst"));
  QG_TRY(need_align(wq, 4, "wq")); QG_TRY(need_align(dst, 16, "dst"));
  if (wq == dst) return fail(QGEMM_ERR_INVALID_ARG, "prepack cannot run in place");
  return launch_prepack_w4_tiled(s, reinterpret_cast<const uint32_t*>(wq),
                                 reinterpret_cast<uint8_t*>(dst), K, N);
}

qgemm_status qgemm_w4a16_grouped_gemm_tiled(qgemm_stream_t s, uint64_t x, uint64_t wt,
                                            uint64_t scales, int zero_point, int group_size,
                                            uint64_t y, int M, int N, int K) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (group_size <= 0) return fail(QGEMM_ERR_INVALID_ARG, "group_size %d <= 0", group_size);
  if (zero_point < 0 || zero_point > 15)
    return fail(QGEMM_ERR_INVALID_ARG, "zero_point %d outside [0,15]", zero_point);
  if (N % 8 != 0) return fail(QGEMM_ERR_INVALID_ARG, "N %d is not a multiple of 8", N);
  if (K % group_size != 0)
    return fail(QGEMM_ERR_INVALID_ARG, "K %d is not a multiple of group_size %d", K, group_size);
  if (M == 0 || N == 0) return QGEMM_OK;
  QG_TRY(need(y, "y"));
  if (K == 0) return fail(QGEMM_ERR_UNSUPPORTED, "K == 0 on the tiled path");
  QG_TRY(need(x, "x")); QG_TRY(need(wt, "wt")); QG_TRY(need(scales, "scales"));
  QG_TRY(need_align(y, 2, "y"));
  const char* why = nullptr;
  if (!w4a16_tile_supported(s->dev, x, wt, scales, M, N, K, group_size, &why))
    return fail(QGEMM_ERR_UNSUPPORTED, "tiled W4A16 path unavailable: %s", why);
  return launch_w4a16_tile(s, reinterpret_cast<const void*>(x), reinterpret_cast<const uint8_t*>(wt),
                          reinterpret_cast<const void*>(scales), zero_point, group_size,
                          reinterpret_cast<void*>(y), M, N, K);
}

qgemm_status qgemm_w4_frag_bytes(int K, int N, size_t* bytes) {
  if (!bytes) return fail(QGEMM_ERR_INVALID_ARG, "bytes is null");
  if (K < 0 || N < 0 || N % 8 != 0) return fail(QGEMM_ERR_INVALID_ARG, "bad K=%d N=%d", K, N);
  *bytes = w4_frag_bytes(K, N);
  return QGEMM_OK;
}

qgemm_status qgemm_prepack_w4_frag(qgemm_stream_t s, uint64_t wq, uint64_t dst, int K, int N) {
  QG_TRY(enter(s));
  if (K < 0 || N < 0 || N % 8 != 0) return fail(QGEMM_ERR_INVALID_ARG, "bad K=%d N=%d", K, N);
  if (K == 0 || N == 0) return QGEMM_OK;
  QG_TRY(need(wq, "wq")); QG_TRY(need(dst, "dst"));
  QG_TRY(need_align(wq, 4, "wq")); QG_TRY(need_align(dst, 16, "dst"));
  if (wq == dst) return fail(QGEMM_ERR_INVALID_ARG, "prepack cannot run in place");
  return launch_prepack_w4_frag(s, reinterpret_cast<const uint32_t*>(wq),
                                reinterpret_cast<uint32_t*>(dst), K, N);
}

qgemm_status qgemm_w4a16_grouped_gemm_frag(qgemm_stream_t s, uint64_t x, uint64_t wf,
                                           uint64_t scales, int zero_point, int group_size,
                                           uint64_t y, int M, int N, int K) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (group_size <= 0) return fail(QGEMM_ERR_INVALID_ARG, "group_size %d <= 0", group_size);
  if (zero_point < 0 || zero_point > 15)
    return fail(QGEMM_ERR_INVALID_ARG, "zero_point %d outside [0,15]", zero_point);
  if (N % 8 != 0) return fail(QGEMM_ERR_INVALID_ARG, "N %d is not a multiple of 8", N);
  if (K % group_size != 0)
    return fail(QGEMM_ERR_INVALID_ARG, "K %d is not a multiple of group_size %d", K, group_size);
  if (M == 0 || N == 0) return QGEMM_OK;
  QG_TRY(need(y, "y"));
  if (K == 0) return fail(QGEMM_ERR_UNSUPPORTED, "K == 0 on the frag path");
  QG_TRY(need(x, "x")); QG_TRY(need(wf, "wf")); QG_TRY(need(scales, "scales"));
  QG_TRY(need_align(y, 2, "y"));
  const char* why = nullptr;
  if (!w4a16_frag_supported(s->dev, x, wf, scales, M, N, K, group_size, &why))
    return fail(QGEMM_ERR_UNSUPPORTED, "frag W4A16 path unavailable: %s", why);
  return launch_w4a16_frag(s, reinterpret_cast<const void*>(x), reinterpret_cast<const void*>(wf),
                           reinterpret_cast<const void*>(scales), zero_point, group_size,
                           reinterpret_cast<void*>(y), M, N, K);
}

qgemm_status qgemm_w4a16_prefill_workspace_bytes(int K, int N, size_t* bytes) {
  if (!bytes) return fail(QGEMM_ERR_INVALID_ARG, "bytes is null");
  if (K < 0 || N < 0) return fail(QGEMM_ERR_INVALID_ARG, "negative size K=%d N=%d", K, N);
  *bytes = w4a16_prefill_workspace_bytes(K, N, 2);
  return QGEMM_OK;
}

qgemm_status qgemm_w4a16_prefill_workspace_bytes_ex(int K, int N, int flags, size_t* bytes) {
  if (!bytes) return fail(QGEMM_ERR_INVALID_ARG, "bytes is null");
  if (K < 0 || N < 0) return fail(QGEMM_ERR_INVALID_ARG, "negative size K=%d N=%d", K, N);
  if (flags & ~(QGEMM_PREFILL_FRAG | QGEMM_PREFILL_ONE_TERM))
    return fail(QGEMM_ERR_INVALID_ARG, "unknown prefill flags 0x%x", flags);
  *bytes = w4a16_prefill_workspace_bytes(K, N, (flags & QGEMM_PREFILL_ONE_TERM) ? 1 : 2);
  return QGEMM_OK;
}

static qgemm_status prefill_entry(qgemm_stream_t s, uint64_t x, uint64_t wt, uint64_t scales,
                                  int zero_point, int group_size, uint64_t y, int M, int N,
                                  int K, uint64_t workspace, size_t workspace_bytes, bool frag,
                                  int terms) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (group_size <= 0) return fail(QGEMM_ERR_INVALID_ARG, "group_size %d <= 0", group_size);
  if (zero_point < 0 || zero_point > 15)
    return fail(QGEMM_ERR_INVALID_ARG, "zero_point %d outside [0,15]", zero_point);
  if (N % 8 != 0) return fail(QGEMM_ERR_INVALID_ARG, "N %d is not a multiple of 8", N);
  if (K % group_size != 0)
    return fail(QGEMM_ERR_INVALID_ARG, "K %d is not a multiple of group_size %d", K, group_size);
  if (M == 0 || N == 0) return QGEMM_OK;
  if (K == 0) return fail(QGEMM_ERR_UNSUPPORTED, "K == 0 on the prefill path");
  if (K % 8 != 0) return fail(QGEMM_ERR_UNSUPPORTED, "K %d is not a multiple of 8", K);
  if (frag && (K % 16 != 0 || !(group_size == 32 || group_size == 64 || group_size % 128 == 0)))
    return fail(QGEMM_ERR_UNSUPPORTED,
                "fragment-ordered weights need K %% 16 == 0 and group_size 32, 64 or a "
                "multiple of 128 (K=%d, group_size=%d)", K, group_size);
  if (!s->dev->tcgen05) return fail(QGEMM_ERR_UNSUPPORTED, "device is not sm_100");
  QG_TRY(need(x, "x")); QG_TRY(need(wt, "wt")); QG_TRY(need(scales, "scales"));
  QG_TRY(need(y, "y")); QG_TRY(need(workspace, "workspace"));
  QG_TRY(need_align(x, 16, "x")); QG_TRY(need_align(wt, 16, "wt"));
  QG_TRY(need_align(scales, 2, "scales")); QG_TRY(need_align(y, 16, "y"));
  QG_TRY(need_align(workspace, 16, "workspace"));
  return launch_w4a16_prefill(s, reinterpret_cast<const void*>(x),
                              reinterpret_cast<const uint8_t*>(wt),
                              reinterpret_cast<const void*>(scales), zero_point, group_size,
                              reinterpret_cast<void*>(y), M, N, K,
                              reinterpret_cast<void*>(workspace), workspace_bytes, frag, terms);
}

qgemm_status qgemm_w4a16_grouped_gemm_prefill(qgemm_stream_t s, uint64_t x, uint64_t wt,
                                              uint64_t scales, int zero_point, int group_size,
                                              uint64_t y, int M, int N, int K, uint64_t workspace,
                                              size_t workspace_bytes) {
  return prefill_entry(s, x, wt, scales, zero_point, group_size, y, M, N, K, workspace,
                       workspace_bytes, false, 2);
}

qgemm_status qgemm_w4a16_grouped_gemm_prefill_frag(qgemm_stream_t s, uint64_t x, uint64_t wf,
                                                   uint64_t scales, int zero_point,
                                                   int group_size, uint64_t y, int M, int N,
                                                   int K, uint64_t workspace,
                                                   size_t workspace_bytes) {
  return prefill_entry(s, x, wf, scales, zero_point, group_size, y, M, N, K, workspace,
                       workspace_bytes, true, 2);
}

qgemm_status qgemm_w4a16_grouped_gemm_prefill_ex(qgemm_stream_t s, uint64_t x, uint64_t w,
                                                 uint64_t scales, int zero_point, int group_size,
                                                 uint64_t y, int M, int N, int K,
                                                 uint64_t workspace, size_t workspace_bytes,
                                                 int flags) {
  if (flags & ~(QGEMM_PREFILL_FRAG | QGEMM_PREFILL_ONE_TERM))
    return fail(QGEMM_ERR_INVALID_ARG, "unknown prefill flags 0x%x", flags);
  return prefill_entry(s, x, w, scales, zero_point, group_size, y, M, N, K, workspace,
                       workspace_bytes, (flags & QGEMM_PREFILL_FRAG) != 0,
                       (flags & QGEMM_PREFILL_ONE_TERM) ? 1 : 2);
}

qgemm_status qgemm_gemm_bf16_nk(qgemm_stream_t s, uint64_t A, uint64_t B, uint64_t out, int ldc,
                                int M, int N, int K) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (ldc < N) return fail(QGEMM_ERR_INVALID_ARG, "ldc %d < N %d", ldc, N);
  if (M == 0 || N == 0) return QGEMM_OK;
  if (K == 0 || K % 8 != 0) return fail(QGEMM_ERR_UNSUPPORTED, "K %d is not a positive multiple of 8", K);
  if (ldc % 8 != 0) return fail(QGEMM_ERR_UNSUPPORTED, "ldc %d is not a multiple of 8", ldc);
  if (!s->dev->tcgen05) return fail(QGEMM_ERR_UNSUPPORTED, "device is not sm_100");
  QG_TRY(need(A, "A")); QG_TRY(need(B, "B")); QG_TRY(need(out, "out"));
  QG_TRY(need_align(A, 16, "A")); QG_TRY(need_align(B, 16, "B")); QG_TRY(need_align(out, 16, "out"));
  return launch_bf16_gemm_nk(s, reinterpret_cast<const void*>(A), reinterpret_cast<const void*>(B),
                             reinterpret_cast<void*>(out), ldc, M, N, K);
}

qgemm_status qgemm_quantize_per_token(qgemm_stream_t s, uint64_t x, int in_dtype, uint64_t q,
                                      uint64_t sA, int M, int K) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, 0, K));
  if (in_dtype != QGEMM_F32 && in_dtype != QGEMM_BF16)
    return fail(QGEMM_ERR_INVALID_ARG, "in_dtype %d is neither QGEMM_F32 nor QGEMM_BF16", in_dtype);
  if (M == 0) return QGEMM_OK;
  QG_TRY(need(sA, "sA"));
  QG_TRY(need_align(sA, 4, "sA"));
  if (K > 0) {
    QG_TRY(need(x, "x")); QG_TRY(need(q, "q"));
    QG_TRY(need_align(x, in_dtype == QGEMM_BF16 ? 2 : 4, "x"));
  }
  return launch_quantize_tokens(s, reinterpret_cast<const void*>(x), in_dtype,
                                reinterpret_cast<int8_t*>(q), reinterpret_cast<float*>(sA), M, K);
}

// ---- W8A16 ----

qgemm_status qgemm_w8a16_gemm(qgemm_stream_t s, uint64_t wInt8, uint64_t scalesW, uint64_t x,
                              uint64_t bias, uint64_t y, int M, int N, int K, int hasBias) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (M == 0 || N == 0) return QGEMM_OK;
  if (K > 0) { QG_TRY(need(wInt8, "wInt8")); QG_TRY(need(x, "x")); }
  QG_TRY(need(scalesW, "scalesW")); QG_TRY(need(y, "y"));
  if (hasBias) QG_TRY(need(bias, "bias"));
  QG_TRY(need_align(scalesW, 4, "scalesW")); QG_TRY(need_align(x, 4, "x"));
  QG_TRY(need_align(y, 4, "y")); QG_TRY(need_align(bias, 4, "bias"));
  if (w8a16_stream_supported(s->dev, wInt8, x, N, K))
    return launch_w8a16_stream(s, reinterpret_cast<const int8_t*>(wInt8),
                               reinterpret_cast<const float*>(scalesW),
                               reinterpret_cast<const float*>(x),
                               reinterpret_cast<const float*>(bias), reinterpret_cast<float*>(y),
                               M, N, K, hasBias ? 1 : 0, 0);
  return launch_w8a16_ref(s, reinterpret_cast<const int8_t*>(wInt8),
                          reinterpret_cast<const float*>(scalesW),
                          reinterpret_cast<const float*>(x), reinterpret_cast<const float*>(bias),
                          reinterpret_cast<float*>(y), M, N, K, hasBias ? 1 : 0, 0);
}

qgemm_status qgemm_w8a16_gemm_rowwise(qgemm_stream_t s, uint64_t wInt8, uint64_t scalesW,
                                      uint64_t x, uint64_t y, int M, int N, int K) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (M == 0 || N == 0) return QGEMM_OK;
  if (K > 0) { QG_TRY(need(wInt8, "wInt8")); QG_TRY(need(x, "x")); QG_TRY(need(scalesW, "scalesW")); }
  QG_TRY(need(y, "y"));
  QG_TRY(need_align(scalesW, 4, "scalesW")); QG_TRY(need_align(x, 4, "x"));
  QG_TRY(need_align(y, 4, "y"));
  if (w8a16_stream_supported(s->dev, wInt8, x, N, K))
    return launch_w8a16_stream(s, reinterpret_cast<const int8_t*>(wInt8),
                               reinterpret_cast<const float*>(scalesW),
                               reinterpret_cast<const float*>(x), nullptr,
                               reinterpret_cast<float*>(y), M, N, K, 0, 1);
  return launch_w8a16_ref(s, reinterpret_cast<const int8_t*>(wInt8),
                          reinterpret_cast<const float*>(scalesW),
                          reinterpret_cast<const float*>(x), nullptr, reinterpret_cast<float*>(y),
                          M, N, K, 0, 1);
}

// ---- quantize / dequantize ----

qgemm_status qgemm_dynamic_quantize(qgemm_stream_t s, uint64_t weight, uint64_t scales,
                                    uint64_t qWeight, int K, int N, int qBits) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(1, N, K));
  if (N == 0) return QGEMM_OK;
  QG_TRY(need(scales, "scales"));
  if (K > 0) { QG_TRY(need(weight, "weight")); QG_TRY(need(qWeight, "qWeight")); }
  QG_TRY(need_align(weight, 4, "weight")); QG_TRY(need_align(scales, 4, "scales"));
  return launch_quantize(s, reinterpret_cast<const float*>(weight),
                         reinterpret_cast<float*>(scales), reinterpret_cast<int8_t*>(qWeight),
                         nullptr, K, N, qBits);
}

qgemm_status qgemm_weight_only_quantize_per_channel(qgemm_stream_t s, uint64_t weight,
                                                    uint64_t scales, uint64_t qWeight,
                                                    uint64_t zeros, int K, int N) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(1, N, K));
  if (N == 0) return QGEMM_OK;
  QG_TRY(need(scales, "scales")); QG_TRY(need(zeros, "zeros"));
  if (K > 0) { QG_TRY(need(weight, "weight")); QG_TRY(need(qWeight, "qWeight")); }
  QG_TRY(need_align(weight, 4, "weight")); QG_TRY(need_align(scales, 4, "scales"));
  return launch_quantize(s, reinterpret_cast<const float*>(weight),
                         reinterpret_cast<float*>(scales), reinterpret_cast<int8_t*>(qWeight),
                         reinterpret_cast<int8_t*>(zeros), K, N, 8);
}

qgemm_status qgemm_dequantize(qgemm_stream_t s, uint64_t qWeight, uint64_t scales,
                              uint64_t weight, int K, int N) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(1, N, K));
  if (N == 0 || K == 0) return QGEMM_OK;
  QG_TRY(need(qWeight, "qWeight")); QG_TRY(need(scales, "scales")); QG_TRY(need(weight, "weight"));
  QG_TRY(need_align(scales, 4, "scales")); QG_TRY(need_align(weight, 4, "weight"));
  return launch_dequantize(s, reinterpret_cast<const int8_t*>(qWeight),
                           reinterpret_cast<const float*>(scales),
                           reinterpret_cast<float*>(weight), K, N);
}

qgemm_status qgemm_prepack_w8_nk(qgemm_stream_t s, uint64_t src, uint64_t dst, int K, int N) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(1, N, K));
  if (N == 0 || K == 0) return QGEMM_OK;
  QG_TRY(need(src, "src")); QG_TRY(need(dst, "dst"));
  if (src == dst) return fail(QGEMM_ERR_INVALID_ARG, "prepack cannot run in place");
  return launch_prepack_w8_nk(s, reinterpret_cast<const int8_t*>(src),
                              reinterpret_cast<int8_t*>(dst), K, N);
}

// ---- fp32 entry points (MatrixOps / BLASOps) ----

qgemm_status qgemm_gemm_f32(qgemm_stream_t s, uint64_t A, uint64_t B, uint64_t bias, uint64_t C,
                            int M, int N, int K, float alpha, float beta, int mode, int algo) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, K));
  if (mode < QGEMM_F32_MATMUL || mode > QGEMM_F32_SGEMM)
    return fail(QGEMM_ERR_INVALID_ARG, "bad mode %d", mode);
  if (algo < QGEMM_ALGO_AUTO || algo > QGEMM_ALGO_SIMT)
    return fail(QGEMM_ERR_INVALID_ARG, "bad algo %d", algo);
  if (M == 0 || N == 0) return QGEMM_OK;
  if (algo == QGEMM_ALGO_TCGEN05 && !s->dev->tcgen05)
    return fail(QGEMM_ERR_UNSUPPORTED, "device is not sm_100");
  if (K > 0) { QG_TRY(need(A, "A")); QG_TRY(need(B, "B")); }
  QG_TRY(need(C, "C"));
  if (mode == F32_MATMUL_BIAS) QG_TRY(need(bias, "bias"));
  QG_TRY(need_align(A, 4, "A")); QG_TRY(need_align(B, 4, "B"));
  QG_TRY(need_align(C, 4, "C")); QG_TRY(need_align(bias, 4, "bias"));
  if (K > 0 && (M > (1 << 28) / ((K + 31) / 32) || N > (1 << 28) / ((K + 31) / 32)))
    return fail(QGEMM_ERR_UNSUPPORTED, "a split operand of M=%d N=%d K=%d would exceed 64 GiB", M, N, K);
  return launch_f32_gemm(s, reinterpret_cast<const float*>(A), reinterpret_cast<const float*>(B),
                         reinterpret_cast<const float*>(bias), reinterpret_cast<float*>(C), M, N,
                         K, alpha, beta, mode, algo);
}

qgemm_status qgemm_matmul_f32(qgemm_stream_t s, uint64_t A, uint64_t B, uint64_t C, int M, int N,
                              int K) {
  return qgemm_gemm_f32(s, A, B, 0, C, M, N, K, 1.f, 0.f, QGEMM_F32_MATMUL, QGEMM_ALGO_AUTO);
}

qgemm_status qgemm_matmul_add_bias_f32(qgemm_stream_t s, uint64_t A, uint64_t B, uint64_t bias,
                                       uint64_t C, int M, int N, int K) {
  return qgemm_gemm_f32(s, A, B, bias, C, M, N, K, 1.f, 0.f, QGEMM_F32_MATMUL_BIAS,
                        QGEMM_ALGO_AUTO);
}

qgemm_status qgemm_sgemm(qgemm_stream_t s, uint64_t A, uint64_t B, uint64_t C, int M, int N, int K,
                         float alpha, float beta) {
  return qgemm_gemm_f32(s, A, B, 0, C, M, N, K, alpha, beta, QGEMM_F32_SGEMM, QGEMM_ALGO_AUTO);
}

qgemm_status qgemm_gemv_f32(qgemm_stream_t s, uint64_t A, uint64_t x, uint64_t y, int M, int N) {
  QG_TRY(enter(s));
  QG_TRY(check_dims(M, N, 0));
  if (M == 0) return QGEMM_OK;
  if (N > 0) { QG_TRY(need(A, "A")); QG_TRY(need(x, "x")); }
  QG_TRY(need(y, "y"));
  QG_TRY(need_align(A, 4, "A")); QG_TRY(need_align(x, 4, "x")); QG_TRY(need_align(y, 4, "y"));
  return launch_f32_gemv(s, reinterpret_cast<const float*>(A), reinterpret_cast<const float*>(x),
                         reinterpret_cast<float*>(y), M, N);
}

// ---- by-name launch ----

qgemm_status qgemm_launch_by_name(qgemm_stream_t s, const char* name, const uint64_t* b,
                                  int nb, const int* v, int ni) {
  if (!name) return fail(QGEMM_ERR_INVALID_ARG, "name is null");
  auto want = [&](int bufs, int ints) -> qgemm_status {
    if (nb != bufs || (ni != ints) || (bufs && !b) || (ints && !v))
      return fail(QGEMM_ERR_INVALID_ARG, "%s takes %d buffers and %d ints (got %d, %d)", name,
                  bufs, ints, nb, ni);
    return QGEMM_OK;
  };
  if (!strcmp(name, "w8a32Gemm")) {
    QG_TRY(want(5, 3));
    return qgemm_w8a32_gemm(s, b[0], b[1], b[2], b[3], b[4], v[0], v[1], v[2]);
  }
  if (!strcmp(name, "w4a16Gemm")) {
    QG_TRY(want(4, 3));
    return qgemm_w4a16_gemm(s, b[0], b[1], b[2], b[3], v[0], v[1], v[2]);
  }
  if (!strcmp(name, "w8a16Gemm")) {
    QG_TRY(want(5, 4));
    return qgemm_w8a16_gemm(s, b[0], b[1], b[2], b[3], b[4], v[0], v[1], v[2], v[3]);
  }
  if (!strcmp(name, "w8a16GemmRowWise")) {
    QG_TRY(want(4, 3));
    return qgemm_w8a16_gemm_rowwise(s, b[0], b[1], b[2], b[3], v[0], v[1], v[2]);
  }
  if (!strcmp(name, "dynamicQuantize")) {
    // qBits has a default of 8 in the reference signature (QuantizedGemmOps.scala:127).
    if (ni == 2) {
      QG_TRY(want(3, 2));
      return qgemm_dynamic_quantize(s, b[0], b[1], b[2], v[0], v[1], 8);
    }
    QG_TRY(want(3, 3));
    return qgemm_dynamic_quantize(s, b[0], b[1], b[2], v[0], v[1], v[2]);
  }
  if (!strcmp(name, "weightOnlyQuantizePerChannel")) {
    QG_TRY(want(4, 2));
    return qgemm_weight_only_quantize_per_channel(s, b[0], b[1], b[2], b[3], v[0], v[1]);
  }
  if (!strcmp(name, "dequantize")) {
    QG_TRY(want(3, 2));
    return qgemm_dequantize(s, b[0], b[1], b[2], v[0], v[1]);
  }
  if (!strcmp(name, "matmul")) {
    QG_TRY(want(3, 3));
    return qgemm_matmul_f32(s, b[0], b[1], b[2], v[0], v[1], v[2]);
  }
  if (!strcmp(name, "matmulAddBias")) {
    QG_TRY(want(4, 3));
    return qgemm_matmul_add_bias_f32(s, b[0], b[1], b[2], b[3], v[0], v[1], v[2]);
  }
  if (!strcmp(name, "gemv")) {
    QG_TRY(want(3, 2));
    return qgemm_gemv_f32(s, b[0], b[1], b[2], v[0], v[1]);
  }
  if (!strcmp(name, "tensorCoreGemmInt8")) {
    QG_TRY(want(6, 8));
    return qgemm_tensor_core_gemm_int8(s, b[0], b[1], b[2], b[3], b[4], b[5], v[0], v[1], v[2],
                                       v[3], v[4], v[5], v[6], v[7]);
  }
  return fail(QGEMM_ERR_INVALID_ARG, "unknown kernel name '%s'", name);
}

// ---- the Java bridge's by-name form ----
//
// One row per reference method: its Ptr parameters in declaration order, which of them
// the bridge's bufferAddrs(0) names (the result buffer), and its scalar parameters in
// declaration order with their types (i: Int, b: Bool, f: Float).  Scalars left out of
// scalarKeys take the default in `defaults` (NaN: no default).

namespace {

struct BridgeOp {
  const char* name;
  const char* ptrs[8];
  int nptrs;
  int out;                 // index into ptrs of bufferAddrs(0)
  const char* scalars[16];
  const char* types;       // one letter per scalar
  float defaults[16];
};

constexpr float NO_DEFAULT = __builtin_nanf("");

const BridgeOp kBridgeOps[] = {
    {"w8a32Gemm", {"wInt8", "scalesW", "x", "scalesX", "y"}, 5, 4, {"M", "N", "K"}, "iii",
     {NO_DEFAULT, NO_DEFAULT, NO_DEFAULT}},
    {"w4a16Gemm", {"wInt4", "scalesW", "x", "y"}, 4, 3, {"M", "N", "K"}, "iii",
     {NO_DEFAULT, NO_DEFAULT, NO_DEFAULT}},
    {"w8a16Gemm", {"wInt8", "scalesW", "x", "bias", "y"}, 5, 4, {"M", "N", "K", "hasBias"},
     "iiib", {NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT}},
    {"w8a16GemmRowWise", {"wInt8", "scalesW", "x", "y"}, 4, 3, {"M", "N", "K"}, "iii",
     {NO_DEFAULT, NO_DEFAULT, NO_DEFAULT}},
    {"dynamicQuantize", {"weight", "scales", "qWeight"}, 3, 2, {"K", "N", "qBits"}, "iii",
     {NO_DEFAULT, NO_DEFAULT, 8.f}},
    {"weightOnlyQuantizePerChannel", {"weight", "scales", "qWeight", "zeros"}, 4, 2, {"K", "N"},
     "ii", {NO_DEFAULT, NO_DEFAULT}},
    {"dequantize", {"qWeight", "scales", "weight"}, 3, 2, {"K", "N"}, "ii",
     {NO_DEFAULT, NO_DEFAULT}},
    {"matmul", {"A", "B", "C"}, 3, 2, {"M", "N", "K"}, "iii", {NO_DEFAULT, NO_DEFAULT, NO_DEFAULT}},
    {"matmulAddBias", {"A", "B", "bias", "C"}, 4, 3, {"M", "N", "K"}, "iii",
     {NO_DEFAULT, NO_DEFAULT, NO_DEFAULT}},
    {"sgemm", {"A", "B", "C"}, 3, 2, {"M", "N", "K", "alpha", "beta"}, "iiiff",
     {NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT}},
    {"gemv", {"A", "x", "y"}, 3, 2, {"M", "N"}, "ii", {NO_DEFAULT, NO_DEFAULT}},
    {"tensorCoreGemmInt8", {"a", "b", "scalesA", "scalesB", "c", "d"}, 6, 5,
     {"M", "N", "K", "lda", "ldb", "ldc", "ldd", "hasC"}, "iiiiiiib",
     {NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT,
      NO_DEFAULT}},
    {"int8GemmKernel", {"D", "A", "B"}, 3, 0,
     {"M", "N", "K", "lda", "ldb", "ldd", "scaleA", "scaleB"}, "iiiiiiff",
     {NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT, NO_DEFAULT,
      NO_DEFAULT}},
};

// An Int passed as a Float must be integral and exactly representable (|v| <= 2^24).
bool float_to_int(float f, int* out) {
  if (!(f == f) || f < -16777216.f || f > 16777216.f) return false;
  const int v = (int)f;
  if ((float)v != f) return false;
  *out = v;
  return true;
}

}  // namespace

int64_t qgemm_bridge_launch_kernel(qgemm_stream_t s, const char* name, int gridX, int gridY,
                                   int gridZ, int blockX, int blockY, int blockZ,
                                   const uint64_t* bufferAddrs, int nbufs,
                                   const float* scalarVals, const char* const* scalarKeys,
                                   int nscalars) {
  (void)gridX; (void)gridY; (void)gridZ; (void)blockX; (void)blockY; (void)blockZ;
  if (!name) { fail(QGEMM_ERR_INVALID_ARG, "name is null"); return -1; }
  const BridgeOp* op = nullptr;
  for (const BridgeOp& o : kBridgeOps)
    if (!strcmp(o.name, name)) op = &o;
  if (!op) { fail(QGEMM_ERR_INVALID_ARG, "unknown kernel name '%s'", name); return -1; }
  if (nbufs != op->nptrs || !bufferAddrs) {
    fail(QGEMM_ERR_INVALID_ARG, "%s takes %d buffers (got %d)", name, op->nptrs, nbufs);
    return -1;
  }
  const int nsc = (int)strlen(op->types);
  if (nscalars < 0 || nscalars > nsc || (nscalars > 0 && !scalarVals)) {
    fail(QGEMM_ERR_INVALID_ARG, "%s takes up to %d scalars (got %d)", name, nsc, nscalars);
    return -1;
  }
  // Buffers: bufferAddrs(0) is the result buffer, the rest follow in declaration order.
  uint64_t b[8] = {};
  b[op->out] = bufferAddrs[0];
  for (int i = 0, j = 1; i < op->nptrs; ++i)
    if (i != op->out) b[i] = bufferAddrs[j++];
  // Scalars: by key when keys are given, else by position.
  float sv[16];
  bool set[16] = {};
  for (int i = 0; i < nscalars; ++i) {
    int slot = i;
    if (scalarKeys) {
      slot = -1;
      if (!scalarKeys[i]) { fail(QGEMM_ERR_INVALID_ARG, "scalar key %d is null", i); return -1; }
      for (int k = 0; k < nsc; ++k)
        if (!strcmp(scalarKeys[i], op->scalars[k])) slot = k;
      if (slot < 0) {
        fail(QGEMM_ERR_INVALID_ARG, "%s has no scalar '%s'", name, scalarKeys[i]);
        return -1;
      }
      if (set[slot]) {
        fail(QGEMM_ERR_INVALID_ARG, "scalar '%s' given twice", scalarKeys[i]);
        return -1;
      }
    }
    sv[slot] = scalarVals[i];
    set[slot] = true;
  }
  int iv[16] = {};
  float fv[16] = {};
  for (int k = 0; k < nsc; ++k) {
    if (!set[k]) {
      if (op->defaults[k] != op->defaults[k]) {
        fail(QGEMM_ERR_INVALID_ARG, "%s: scalar '%s' missing", name, op->scalars[k]);
        return -1;
      }
      sv[k] = op->defaults[k];
    }
    if (op->types[k] == 'f') {
      fv[k] = sv[k];
    } else if (!float_to_int(sv[k], &iv[k]) ||
               (op->types[k] == 'b' && iv[k] != 0 && iv[k] != 1)) {
      fail(QGEMM_ERR_INVALID_ARG, "%s: scalar '%s' = %g is not a%s", name, op->scalars[k],
           (double)sv[k], op->types[k] == 'b' ? " Bool (0 or 1)" : "n exact Int");
      return -1;
    }
  }
  qgemm_status st;
  if (!strcmp(name, "sgemm")) {
    st = qgemm_sgemm(s, b[0], b[1], b[2], iv[0], iv[1], iv[2], fv[3], fv[4]);
  } else if (!strcmp(name, "int8GemmKernel")) {
    st = qgemm_int8_gemm_kernel(s, b[0], b[1], b[2], iv[0], iv[1], iv[2], iv[3], iv[4], iv[5],
                                fv[6], fv[7]);
  } else {
    st = qgemm_launch_by_name(s, name, b, op->nptrs, iv, nsc);
  }
  return st == QGEMM_OK ? (int64_t)bufferAddrs[0] : -1;
}

// ---- sharding ----

qgemm_status qgemm_shard_columns(int N, int world, int rank, int align, int* n0, int* n1) {
  if (!n0 || !n1) return fail(QGEMM_ERR_INVALID_ARG, "null output");
  if (N < 0 || world < 1 || rank < 0 || rank >= world || align < 1)
    return fail(QGEMM_ERR_INVALID_ARG, "bad shard request N=%d world=%d rank=%d align=%d", N,
                world, rank, align);
  const long long units = ((long long)N + align - 1) / align;
  long long a = units * rank / world * align, c = units * (rank + 1) / world * align;
  *n0 = (int)(a < N ? a : N);
  *n1 = (int)(c < N ? c : N);
  return QGEMM_OK;
}

qgemm_status qgemm_unshard_columns_bf16(qgemm_stream_t s, uint64_t gathered, uint64_t out,
                                        int world, int M, int ncols) {
  QG_TRY(enter(s));
  if (world < 1 || M < 0 || ncols < 0)
    return fail(QGEMM_ERR_INVALID_ARG, "bad unshard request");
  if (M == 0 || ncols == 0) return QGEMM_OK;
  QG_TRY(need(gathered, "gathered")); QG_TRY(need(out, "out"));
  QG_TRY(need_align(gathered, 2, "gathered")); QG_TRY(need_align(out, 2, "out"));
  return launch_unshard_bf16(s, reinterpret_cast<const uint16_t*>(gathered),
                             reinterpret_cast<uint16_t*>(out), world, M, ncols);
}

}  // extern "C"
