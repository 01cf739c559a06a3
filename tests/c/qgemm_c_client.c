/*
 * qgemm_c_client.c -- a C client of libqgemm that uses nothing but include/qgemm.h,
 * the way a JNI, cgo or ctypes binding does.  Test code.
 *
 *   qgemm_c_client cpu   host-only entry points: version, status strings, handle and
 *                        argument errors, column sharding, a weight blob written, read
 *                        back and corrupted (no GPU needed)
 *   qgemm_c_client gpu   device 0: the reference w8a32Gemm at its own 64x512x512 case
 *                        and the W8A8 GEMM on the tensor cores (int32 accumulators and
 *                        fp32 outputs bit-exact against the loop below), the fp32
 *                        MatrixOps.matmul within 1e-5 of sum |a*b|, and the int8 GEMM
 *                        names (tensorCoreGemmInt8 direct, int8GemmKernel through the
 *                        Java bridge's by-name form) bit-exact against plain loops
 *
 * Exit status 0 when every check passes; each failure prints one line.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qgemm.h"

static int failures = 0;

#define CHECK(cond, ...)                      \
  do {                                        \
    if (!(cond)) {                            \
      ++failures;                             \
      fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
      fprintf(stderr, __VA_ARGS__);           \
      fprintf(stderr, "\n");                  \
    }                                         \
  } while (0)

#define CALL(expr)                                                                   \
  do {                                                                               \
    qgemm_status st_ = (expr);                                                       \
    if (st_ != QGEMM_OK) {                                                           \
      fprintf(stderr, "FAIL %s:%d: %s -> %s: %s\n", __FILE__, __LINE__, #expr,       \
              qgemm_status_string(st_), qgemm_last_error());                         \
      return 1;                                                                      \
    }                                                                                \
  } while (0)

/* A small linear congruential generator: the same numbers on every platform. */
static uint32_t lcg_state = 12345u;
static uint32_t lcg(void) {
  lcg_state = lcg_state * 1664525u + 1013904223u;
  return lcg_state >> 8;
}
static int8_t rand_i8(void) { return (int8_t)((int)(lcg() % 255u) - 127); }
static float rand_unit(float lo, float hi) { return lo + (hi - lo) * (float)(lcg() & 0xffff) / 65535.0f; }

static int cpu_checks(const char* tmpdir) {
  CHECK(qgemm_version() >= 10000, "version %d", qgemm_version());
  CHECK(strcmp(qgemm_status_string(QGEMM_OK), "QGEMM_OK") == 0, "status string");
  CHECK(qgemm_stream_sync(NULL) == QGEMM_ERR_BAD_HANDLE, "null stream handle");
  CHECK(qgemm_device_open(0, NULL) == QGEMM_ERR_INVALID_ARG, "null output pointer");
  CHECK(qgemm_w8a32_gemm(NULL, 1, 1, 1, 1, 1, 4, 4, 4) == QGEMM_ERR_BAD_HANDLE, "gemm on null stream");
  CHECK(qgemm_matmul_f32(NULL, 1, 1, 1, 4, 4, 4) == QGEMM_ERR_BAD_HANDLE, "matmul on null stream");
  CHECK(strlen(qgemm_last_error()) > 0, "last error message");

  /* column sharding covers N exactly, in 256-column units */
  int covered = 0, prev = 0;
  for (int r = 0; r < 8; ++r) {
    int n0 = -1, n1 = -1;
    CALL(qgemm_shard_columns(28672, 8, r, 256, &n0, &n1));
    CHECK(n0 == prev && n1 >= n0 && n0 % 256 == 0, "shard %d: [%d, %d)", r, n0, n1);
    covered += n1 - n0;
    prev = n1;
  }
  CHECK(covered == 28672, "shards cover %d columns", covered);

  /* weight blob: int8 [K, N] + f32 scales, written, read back, then corrupted */
  const int K = 64, N = 48;
  int8_t* w = (int8_t*)malloc((size_t)K * N);
  float* s = (float*)malloc(sizeof(float) * N);
  for (int i = 0; i < K * N; ++i) w[i] = rand_i8();
  for (int i = 0; i < N; ++i) s[i] = rand_unit(0.001f, 0.01f);
  char path[512];
  snprintf(path, sizeof path, "%s/c_client.qgemm", tmpdir);
  qgemm_blob_info info;
  memset(&info, 0, sizeof info);
  info.kind = QGEMM_BLOB_W8_KN;
  info.K = K;
  info.N = N;
  CALL(qgemm_blob_save(path, &info, w, s));
  qgemm_blob_info got;
  CALL(qgemm_blob_info_read(path, &got));
  CHECK(got.version == QGEMM_BLOB_VERSION && got.kind == QGEMM_BLOB_W8_KN && got.K == K &&
            got.N == N && got.weight_bytes == (uint64_t)K * N && got.scale_bytes == 4u * N,
        "blob header");
  int8_t* w2 = (int8_t*)malloc((size_t)K * N);
  float* s2 = (float*)malloc(sizeof(float) * N);
  CALL(qgemm_blob_load(path, w2, (size_t)K * N, s2, sizeof(float) * N));
  CHECK(memcmp(w, w2, (size_t)K * N) == 0 && memcmp(s, s2, sizeof(float) * N) == 0, "blob round trip");
  FILE* f = fopen(path, "r+b");
  CHECK(f != NULL, "reopen blob");
  if (f) {
    fseek(f, 64 + 5, SEEK_SET);  /* one byte inside the weight section */
    int c = fgetc(f);
    fseek(f, 64 + 5, SEEK_SET);
    fputc(c ^ 0x40, f);
    fclose(f);
    CHECK(qgemm_blob_load(path, w2, (size_t)K * N, s2, sizeof(float) * N) == QGEMM_ERR_INVALID_ARG,
          "a corrupted weight byte is caught by the CRC");
  }
  remove(path);
  free(w); free(s); free(w2); free(s2);
  return 0;
}

/* y[m,n] = (float(sum_k x[m,k] * w[k,n]) * sW[n]) * sX[m], the reference's order. */
static void w8a32_loop(const int8_t* w, const float* sW, const int8_t* x, const float* sX,
                       float* y, int32_t* acc, int M, int N, int K) {
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      int32_t a = 0;
      for (int k = 0; k < K; ++k) a += (int32_t)x[(size_t)m * K + k] * (int32_t)w[(size_t)k * N + n];
      acc[(size_t)m * N + n] = a;
      volatile float t = (float)a * sW[n];
      y[(size_t)m * N + n] = t * sX[m];
    }
}

static int gpu_checks(void) {
  int count = 0;
  CALL(qgemm_device_count(&count));
  CHECK(count >= 1, "no device");
  qgemm_device_t dev;
  CALL(qgemm_device_open(0, &dev));
  int sms = 0, ccM = 0, ccm = 0, tc = 0;
  size_t l2 = 0;
  CALL(qgemm_device_info(dev, &sms, &ccM, &ccm, &l2, &tc));
  qgemm_stream_t st;
  CALL(qgemm_stream_create(dev, &st));

  /* 1. the reference's own case: w8a32Gemm 64 x 512 x 512, then the W8A8 GEMM on the
   *    tensor cores at 256 x 512 x 1024 with int32 accumulators. */
  const int shapes[2][3] = {{64, 512, 512}, {256, 512, 1024}};
  for (int c = 0; c < 2; ++c) {
    const int M = shapes[c][0], N = shapes[c][1], K = shapes[c][2];
    int8_t* x = (int8_t*)malloc((size_t)M * K);
    int8_t* w = (int8_t*)malloc((size_t)K * N);
    float* sX = (float*)malloc(sizeof(float) * M);
    float* sW = (float*)malloc(sizeof(float) * N);
    for (int i = 0; i < M * K; ++i) x[i] = rand_i8();
    for (int i = 0; i < K * N; ++i) w[i] = rand_i8();
    for (int i = 0; i < M; ++i) sX[i] = rand_unit(0.001f, 0.01f);
    for (int i = 0; i < N; ++i) sW[i] = rand_unit(0.0005f, 0.005f);
    float* y = (float*)malloc(sizeof(float) * M * N);
    float* yref = (float*)malloc(sizeof(float) * M * N);
    int32_t* acc = (int32_t*)malloc(sizeof(int32_t) * M * N);
    int32_t* accref = (int32_t*)malloc(sizeof(int32_t) * M * N);
    w8a32_loop(w, sW, x, sX, yref, accref, M, N, K);
    uint64_t dx, dw, dsx, dsw, dy, dacc;
    CALL(qgemm_buffer_alloc(dev, (size_t)M * K, &dx));
    CALL(qgemm_buffer_alloc(dev, (size_t)K * N, &dw));
    CALL(qgemm_buffer_alloc(dev, sizeof(float) * M, &dsx));
    CALL(qgemm_buffer_alloc(dev, sizeof(float) * N, &dsw));
    CALL(qgemm_buffer_alloc(dev, sizeof(float) * M * N, &dy));
    CALL(qgemm_buffer_alloc(dev, sizeof(int32_t) * M * N, &dacc));
    CALL(qgemm_memcpy_h2d(st, dx, x, (size_t)M * K));
    CALL(qgemm_memcpy_h2d(st, dw, w, (size_t)K * N));
    CALL(qgemm_memcpy_h2d(st, dsx, sX, sizeof(float) * M));
    CALL(qgemm_memcpy_h2d(st, dsw, sW, sizeof(float) * N));
    if (c == 0) {
      CALL(qgemm_w8a32_gemm(st, dw, dsw, dx, dsx, dy, M, N, K));
    } else {
      CALL(qgemm_w8a8_gemm(st, dx, dw, QGEMM_B_KN, dsx, dsw, dy, QGEMM_F32, N, M, N, K, dacc,
                           tc ? QGEMM_ALGO_TCGEN05 : QGEMM_ALGO_SIMT));
      CALL(qgemm_memcpy_d2h(st, acc, dacc, sizeof(int32_t) * M * N));
    }
    CALL(qgemm_memcpy_d2h(st, y, dy, sizeof(float) * M * N));
    CALL(qgemm_stream_sync(st));
    if (c == 1) CHECK(memcmp(acc, accref, sizeof(int32_t) * M * N) == 0, "W8A8 int32 accumulators");
    CHECK(memcmp(y, yref, sizeof(float) * M * N) == 0, "%s fp32 outputs", c ? "W8A8" : "w8a32Gemm");
    CALL(qgemm_buffer_free(dev, dx)); CALL(qgemm_buffer_free(dev, dw));
    CALL(qgemm_buffer_free(dev, dsx)); CALL(qgemm_buffer_free(dev, dsw));
    CALL(qgemm_buffer_free(dev, dy)); CALL(qgemm_buffer_free(dev, dacc));
    free(x); free(w); free(sX); free(sW); free(y); free(yref); free(acc); free(accref);
  }

  /* 2. fp32 MatrixOps.matmul: forward error within 1e-5 of sum_k |a * b| (double loop). */
  {
    const int M = 96, N = 160, K = 200;
    float* A = (float*)malloc(sizeof(float) * M * K);
    float* B = (float*)malloc(sizeof(float) * K * N);
    float* C = (float*)malloc(sizeof(float) * M * N);
    for (int i = 0; i < M * K; ++i) A[i] = rand_unit(-2.f, 2.f);
    for (int i = 0; i < K * N; ++i) B[i] = rand_unit(-2.f, 2.f);
    uint64_t dA, dB, dC;
    CALL(qgemm_buffer_alloc(dev, sizeof(float) * M * K, &dA));
    CALL(qgemm_buffer_alloc(dev, sizeof(float) * K * N, &dB));
    CALL(qgemm_buffer_alloc(dev, sizeof(float) * M * N, &dC));
    CALL(qgemm_memcpy_h2d(st, dA, A, sizeof(float) * M * K));
    CALL(qgemm_memcpy_h2d(st, dB, B, sizeof(float) * K * N));
    CALL(qgemm_matmul_f32(st, dA, dB, dC, M, N, K));
    CALL(qgemm_memcpy_d2h(st, C, dC, sizeof(float) * M * N));
    CALL(qgemm_stream_sync(st));
    double worst = 0.0;
    for (int m = 0; m < M; ++m)
      for (int n = 0; n < N; ++n) {
        double exact = 0.0, scale = 0.0;
        for (int k = 0; k < K; ++k) {
          exact += (double)A[(size_t)m * K + k] * (double)B[(size_t)k * N + n];
          scale += fabs((double)A[(size_t)m * K + k] * (double)B[(size_t)k * N + n]);
        }
        const double r = fabs((double)C[(size_t)m * N + n] - exact) / scale;
        if (r > worst) worst = r;
      }
    CHECK(worst <= 1e-5, "matmul error %.3g of sum |a*b|", worst);
    CALL(qgemm_buffer_free(dev, dA)); CALL(qgemm_buffer_free(dev, dB)); CALL(qgemm_buffer_free(dev, dC));
    free(A); free(B); free(C);
  }

  /* 3. the int8 GEMM names: TensorCoreOps.tensorCoreGemmInt8 directly (d = a b + c through
   *    leading dimensions, int32) and CutlassGemm.int8GemmKernel through the Java bridge's
   *    by-name form (Float scalars named by keys, result buffer first), each against a
   *    plain loop. */
  {
    const int M = 256, N = 272, K = 160, lda = 176, ldb = 288, ldc = 280, ldd = 284;
    int8_t* a = (int8_t*)malloc((size_t)M * lda);
    int8_t* b = (int8_t*)malloc((size_t)K * ldb);
    int32_t* cc = (int32_t*)malloc(sizeof(int32_t) * M * ldc);
    int32_t* d = (int32_t*)malloc(sizeof(int32_t) * M * ldd);
    for (int i = 0; i < M * lda; ++i) a[i] = rand_i8();
    for (int i = 0; i < K * ldb; ++i) b[i] = rand_i8();
    for (int i = 0; i < M * ldc; ++i) cc[i] = (int32_t)(lcg() * 97u);
    uint64_t da, db, dc, dd;
    CALL(qgemm_buffer_alloc(dev, (size_t)M * lda, &da));
    CALL(qgemm_buffer_alloc(dev, (size_t)K * ldb, &db));
    CALL(qgemm_buffer_alloc(dev, sizeof(int32_t) * M * ldc, &dc));
    CALL(qgemm_buffer_alloc(dev, sizeof(int32_t) * M * ldd, &dd));
    CALL(qgemm_memcpy_h2d(st, da, a, (size_t)M * lda));
    CALL(qgemm_memcpy_h2d(st, db, b, (size_t)K * ldb));
    CALL(qgemm_memcpy_h2d(st, dc, cc, sizeof(int32_t) * M * ldc));
    CALL(qgemm_tensor_core_gemm_int8(st, da, db, 0, 0, dc, dd, M, N, K, lda, ldb, ldc, ldd, 1));
    CALL(qgemm_memcpy_d2h(st, d, dd, sizeof(int32_t) * M * ldd));
    CALL(qgemm_stream_sync(st));
    int bad = 0;
    for (int m = 0; m < M; ++m)
      for (int n = 0; n < N; ++n) {
        uint32_t sum = (uint32_t)cc[(size_t)m * ldc + n];
        for (int k = 0; k < K; ++k)
          sum += (uint32_t)((int32_t)a[(size_t)m * lda + k] * (int32_t)b[(size_t)k * ldb + n]);
        bad += d[(size_t)m * ldd + n] != (int32_t)sum;
      }
    CHECK(bad == 0, "tensorCoreGemmInt8: %d outputs differ", bad);

    /* int8GemmKernel: A [M, K], B [K, N] int32 holding int8 values, D [M, N] fp32 */
    int32_t* A = (int32_t*)malloc(sizeof(int32_t) * M * K);
    int32_t* B = (int32_t*)malloc(sizeof(int32_t) * K * N);
    float* D = (float*)malloc(sizeof(float) * M * N);
    for (int i = 0; i < M * K; ++i) A[i] = rand_i8();
    for (int i = 0; i < K * N; ++i) B[i] = rand_i8();
    uint64_t dA, dB, dD;
    CALL(qgemm_buffer_alloc(dev, sizeof(int32_t) * M * K, &dA));
    CALL(qgemm_buffer_alloc(dev, sizeof(int32_t) * K * N, &dB));
    CALL(qgemm_buffer_alloc(dev, sizeof(float) * M * N, &dD));
    CALL(qgemm_memcpy_h2d(st, dA, A, sizeof(int32_t) * M * K));
    CALL(qgemm_memcpy_h2d(st, dB, B, sizeof(int32_t) * K * N));
    const uint64_t addrs[3] = {dD, dA, dB};
    const float vals[8] = {(float)M, (float)N, (float)K, (float)K, (float)N, (float)N, 0.0625f,
                           3.0f};
    const char* keys[8] = {"M", "N", "K", "lda", "ldb", "ldd", "scaleA", "scaleB"};
    const int64_t r = qgemm_bridge_launch_kernel(st, "int8GemmKernel", (N + 63) / 64,
                                                 (M + 63) / 64, 1, 256, 1, 1, addrs, 3, vals,
                                                 keys, 8);
    CHECK(r == (int64_t)dD, "bridge returned %lld: %s", (long long)r, qgemm_last_error());
    CALL(qgemm_memcpy_d2h(st, D, dD, sizeof(float) * M * N));
    CALL(qgemm_stream_sync(st));
    bad = 0;
    for (int m = 0; m < M; ++m)
      for (int n = 0; n < N; ++n) {
        volatile float acc = 0.0f;
        for (int k = 0; k < K; ++k) {
          volatile float p = (float)A[(size_t)m * K + k] * (float)B[(size_t)k * N + n];
          acc = acc + p;
        }
        volatile float t = acc * 0.0625f;
        const float ref = t * 3.0f;
        bad += memcmp(&ref, &D[(size_t)m * N + n], sizeof(float)) != 0;
      }
    CHECK(bad == 0, "int8GemmKernel: %d outputs differ", bad);
    const char* bad_keys[1] = {"gamma"};
    CHECK(qgemm_bridge_launch_kernel(st, "int8GemmKernel", 1, 1, 1, 1, 1, 1, addrs, 3, vals,
                                     bad_keys, 1) == -1, "an unknown scalar key gives -1");
    CALL(qgemm_buffer_free(dev, da)); CALL(qgemm_buffer_free(dev, db));
    CALL(qgemm_buffer_free(dev, dc)); CALL(qgemm_buffer_free(dev, dd));
    CALL(qgemm_buffer_free(dev, dA)); CALL(qgemm_buffer_free(dev, dB));
    CALL(qgemm_buffer_free(dev, dD));
    free(a); free(b); free(cc); free(d); free(A); free(B); free(D);
  }

  /* 4. errors come back as statuses, and the handles stay usable */
  CHECK(qgemm_w8a8_gemm(st, 0, 0, QGEMM_B_KN, 0, 0, 0, QGEMM_BF16, 8, 8, 8, 16, 0, 0) ==
            QGEMM_ERR_INVALID_ARG, "null operands");
  CALL(qgemm_stream_sync(st));
  CALL(qgemm_stream_destroy(st));
  CALL(qgemm_device_close(dev));
  return 0;
}

int main(int argc, char** argv) {
  const char* mode = argc > 1 ? argv[1] : "cpu";
  const char* tmpdir = argc > 2 ? argv[2] : ".";
  int rc = strcmp(mode, "gpu") == 0 ? gpu_checks() : cpu_checks(tmpdir);
  if (rc != 0 || failures != 0) {
    fprintf(stderr, "qgemm_c_client %s: %d failure(s)\n", mode, failures + (rc != 0));
    return 1;
  }
  printf("qgemm_c_client %s: ok\n", mode);
  return 0;
}
