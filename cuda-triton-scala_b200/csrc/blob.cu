// blob.cu -- versioned on-disk container for quantised weights already in a kernel
// layout, so that a model's weights load straight into device memory without a
// repack.
//
// File layout (little-endian):
//   bytes 0..63    header
//     0   char[8]  magic "QGEMMBLB"
//     8   u32      format version (QGEMM_BLOB_VERSION)
//     12  i32      kind (QGEMM_BLOB_W4_TILED, QGEMM_BLOB_W8_KN, QGEMM_BLOB_W8_NK,
//                   QGEMM_BLOB_W4_FRAG)
//     16  i32      K
//     20  i32      N
//     24  i32      group_size (W4) or 0
//     28  i32      zero_point (W4) or 0
//     32  u64      weight section bytes
//     40  u64      scale section bytes
//     48  u32      CRC-32 of the weight section
//     52  u32      CRC-32 of the scale section
//     56  u32      CRC-32 of header bytes 0..55
//     60  u32      zero
//   then the weight section, then the scale section.
// Section sizes follow from the kind and the shape and are checked on every read:
//   W4_TILED  weights: qgemm_w4_tiled_bytes(K, N); scales: bf16 [K/group_size, N]
//   W8_KN     weights: int8 [K, N] (the reference wInt8 layout); scales: f32 [N]
//   W8_NK     weights: int8 [N, K]; scales: f32 [N]
//   W4_FRAG   weights: qgemm_w4_frag_bytes(K, N); scales: bf16 [K/group_size, N]
// CRC-32 is the common reflected polynomial 0xEDB88320 (initial and final value
// 0xFFFFFFFF).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "internal.h"

#define QG_TRY_BLOB(expr)              \
  do {                                 \
    qgemm_status _st = (expr);         \
    if (_st != QGEMM_OK) return _st;   \
  } while (0)

namespace qg {
namespace blob {

constexpr char MAGIC[8] = {'Q', 'G', 'E', 'M', 'M', 'B', 'L', 'B'};
constexpr size_t HEADER = 64;

struct CrcTable {
  uint32_t t[256];
  CrcTable() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int b = 0; b < 8; ++b) c = (c & 1u) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
      t[i] = c;
    }
  }
};

uint32_t crc32_update(uint32_t crc, const uint8_t* p, size_t n) {
  static const CrcTable table;  // built once, thread-safe
  for (size_t i = 0; i < n; ++i) crc = table.t[(crc ^ p[i]) & 0xFFu] ^ (crc >> 8);
  return crc;
}

uint32_t crc32(const void* p, size_t n) {
  return crc32_update(0xFFFFFFFFu, static_cast<const uint8_t*>(p), n) ^ 0xFFFFFFFFu;
}

template <typename T>
void put(uint8_t* h, size_t off, T v) { memcpy(h + off, &v, sizeof(T)); }
template <typename T>
T get(const uint8_t* h, size_t off) { T v; memcpy(&v, h + off, sizeof(T)); return v; }

// Expected section sizes for a shape; false (with a message) if the shape is invalid.
bool expected_sizes(const qgemm_blob_info& in, uint64_t* wb, uint64_t* sb, const char** why) {
  if (in.K <= 0 || in.N <= 0) { *why = "K and N must be positive"; return false; }
  switch (in.kind) {
    case QGEMM_BLOB_W4_TILED:
    case QGEMM_BLOB_W4_FRAG:
      if (in.N % 8 != 0) { *why = "N must be a multiple of 8 for int4 weights"; return false; }
      if (in.group_size <= 0 || in.K % in.group_size != 0) {
        *why = "group_size must be positive and divide K"; return false;
      }
      if (in.zero_point < 0 || in.zero_point > 15) { *why = "zero_point outside [0,15]"; return false; }
      *wb = in.kind == QGEMM_BLOB_W4_FRAG ? w4_frag_bytes(in.K, in.N) : w4_tiled_bytes(in.K, in.N);
      *sb = (uint64_t)(in.K / in.group_size) * (uint64_t)in.N * 2;
      return true;
    case QGEMM_BLOB_W8_KN:
    case QGEMM_BLOB_W8_NK:
      if (in.group_size != 0 || in.zero_point != 0) {
        *why = "int8 weights take group_size 0 and zero_point 0"; return false;
      }
      *wb = (uint64_t)in.K * (uint64_t)in.N;
      *sb = (uint64_t)in.N * 4;
      return true;
    default:
      *why = "unknown kind";
      return false;
  }
}

struct File {
  FILE* f = nullptr;
  ~File() { if (f) fclose(f); }
};

qgemm_status read_header(FILE* f, const char* path, qgemm_blob_info* info, uint32_t* wcrc,
                         uint32_t* scrc) {
  uint8_t h[HEADER];
  if (fread(h, 1, HEADER, f) != HEADER)
    return fail(QGEMM_ERR_INVALID_ARG, "%s: shorter than a blob header", path);
  if (memcmp(h, MAGIC, 8) != 0) return fail(QGEMM_ERR_INVALID_ARG, "%s: not a qgemm weight blob", path);
  if (get<uint32_t>(h, 56) != crc32(h, 56))
    return fail(QGEMM_ERR_INVALID_ARG, "%s: header checksum mismatch", path);
  const uint32_t version = get<uint32_t>(h, 8);
  if (version != QGEMM_BLOB_VERSION)
    return fail(QGEMM_ERR_UNSUPPORTED, "%s: blob format version %u, this library reads version %d",
                path, version, QGEMM_BLOB_VERSION);
  qgemm_blob_info in;
  memset(&in, 0, sizeof(in));
  in.version = version;
  in.kind = get<int32_t>(h, 12);
  in.K = get<int32_t>(h, 16);
  in.N = get<int32_t>(h, 20);
  in.group_size = get<int32_t>(h, 24);
  in.zero_point = get<int32_t>(h, 28);
  in.weight_bytes = get<uint64_t>(h, 32);
  in.scale_bytes = get<uint64_t>(h, 40);
  uint64_t wb = 0, sb = 0;
  const char* why = nullptr;
  if (!expected_sizes(in, &wb, &sb, &why)) return fail(QGEMM_ERR_INVALID_ARG, "%s: %s", path, why);
  if (wb != in.weight_bytes || sb != in.scale_bytes)
    return fail(QGEMM_ERR_INVALID_ARG, "%s: section sizes do not match the shape", path);
  *info = in;
  if (wcrc) *wcrc = get<uint32_t>(h, 48);
  if (scrc) *scrc = get<uint32_t>(h, 52);
  return QGEMM_OK;
}

// Reads `bytes` of a section into `dst` in pieces, checking its CRC.
qgemm_status read_section(FILE* f, const char* path, const char* what, void* dst, uint64_t bytes,
                          uint32_t crc_expected) {
  uint8_t* d = static_cast<uint8_t*>(dst);
  uint32_t crc = 0xFFFFFFFFu;
  uint64_t done = 0;
  while (done < bytes) {
    const size_t n = (size_t)((bytes - done) < (1u << 24) ? (bytes - done) : (1u << 24));
    if (fread(d + done, 1, n, f) != n)
      return fail(QGEMM_ERR_INVALID_ARG, "%s: %s section is truncated", path, what);
    crc = crc32_update(crc, d + done, n);
    done += n;
  }
  if ((crc ^ 0xFFFFFFFFu) != crc_expected)
    return fail(QGEMM_ERR_INVALID_ARG, "%s: %s section checksum mismatch", path, what);
  return QGEMM_OK;
}

}  // namespace blob
}  // namespace qg

using namespace qg;

extern "C" {

qgemm_status qgemm_blob_save(const char* path, const qgemm_blob_info* info, const void* weights,
                             const void* scales) {
  using namespace blob;
  if (!path || !info || !weights || !scales) return fail(QGEMM_ERR_INVALID_ARG, "null argument");
  qgemm_blob_info in = *info;
  uint64_t wb = 0, sb = 0;
  const char* why = nullptr;
  if (!expected_sizes(in, &wb, &sb, &why)) return fail(QGEMM_ERR_INVALID_ARG, "%s", why);
  uint8_t h[HEADER];
  memset(h, 0, sizeof(h));
  memcpy(h, MAGIC, 8);
  put<uint32_t>(h, 8, (uint32_t)QGEMM_BLOB_VERSION);
  put<int32_t>(h, 12, in.kind);
  put<int32_t>(h, 16, in.K);
  put<int32_t>(h, 20, in.N);
  put<int32_t>(h, 24, in.group_size);
  put<int32_t>(h, 28, in.zero_point);
  put<uint64_t>(h, 32, wb);
  put<uint64_t>(h, 40, sb);
  put<uint32_t>(h, 48, crc32(weights, (size_t)wb));
  put<uint32_t>(h, 52, crc32(scales, (size_t)sb));
  put<uint32_t>(h, 56, crc32(h, 56));
  File fh;
  fh.f = fopen(path, "wb");
  if (!fh.f) return fail(QGEMM_ERR_INVALID_ARG, "cannot open %s for writing", path);
  if (fwrite(h, 1, HEADER, fh.f) != HEADER || fwrite(weights, 1, (size_t)wb, fh.f) != wb ||
      fwrite(scales, 1, (size_t)sb, fh.f) != sb)
    return fail(QGEMM_ERR_INVALID_ARG, "short write to %s", path);
  if (fclose(fh.f) != 0) {
    fh.f = nullptr;
    return fail(QGEMM_ERR_INVALID_ARG, "closing %s failed", path);
  }
  fh.f = nullptr;
  return QGEMM_OK;
}

qgemm_status qgemm_blob_info_read(const char* path, qgemm_blob_info* info) {
  if (!path || !info) return fail(QGEMM_ERR_INVALID_ARG, "null argument");
  blob::File fh;
  fh.f = fopen(path, "rb");
  if (!fh.f) return fail(QGEMM_ERR_INVALID_ARG, "cannot open %s", path);
  return blob::read_header(fh.f, path, info, nullptr, nullptr);
}

qgemm_status qgemm_blob_load(const char* path, void* weights, size_t weight_bytes, void* scales,
                             size_t scale_bytes) {
  if (!path || !weights || !scales) return fail(QGEMM_ERR_INVALID_ARG, "null argument");
  blob::File fh;
  fh.f = fopen(path, "rb");
  if (!fh.f) return fail(QGEMM_ERR_INVALID_ARG, "cannot open %s", path);
  qgemm_blob_info in;
  uint32_t wcrc = 0, scrc = 0;
  QG_TRY_BLOB(blob::read_header(fh.f, path, &in, &wcrc, &scrc));
  if (weight_bytes < in.weight_bytes || scale_bytes < in.scale_bytes)
    return fail(QGEMM_ERR_INVALID_ARG, "%s: destination smaller than the sections (%llu, %llu bytes)",
                path, (unsigned long long)in.weight_bytes, (unsigned long long)in.scale_bytes);
  QG_TRY_BLOB(blob::read_section(fh.f, path, "weight", weights, in.weight_bytes, wcrc));
  return blob::read_section(fh.f, path, "scale", scales, in.scale_bytes, scrc);
}

qgemm_status qgemm_blob_load_device(qgemm_stream_t s, const char* path, uint64_t weights,
                                    size_t weight_bytes, uint64_t scales, size_t scale_bytes) {
  QG_TRY_BLOB(enter(s));
  if (!path || !weights || !scales) return fail(QGEMM_ERR_INVALID_ARG, "null argument");
  qgemm_blob_info in;
  QG_TRY_BLOB(qgemm_blob_info_read(path, &in));
  if (weight_bytes < in.weight_bytes || scale_bytes < in.scale_bytes)
    return fail(QGEMM_ERR_INVALID_ARG, "%s: device buffers smaller than the sections", path);
  // Host staging (the whole file is checked before anything is copied).
  std::vector<uint8_t> w((size_t)in.weight_bytes), sc((size_t)in.scale_bytes);
  QG_TRY_BLOB(qgemm_blob_load(path, w.data(), w.size(), sc.data(), sc.size()));
  cudaError_t e = cudaMemcpyAsync(reinterpret_cast<void*>(weights), w.data(), w.size(),
                                  cudaMemcpyHostToDevice, s->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(reinterpret_cast<void*>(scales), sc.data(), sc.size(),
                        cudaMemcpyHostToDevice, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);  // the staging is freed on return
  if (e != cudaSuccess) return cuda_fail(e, "copying the blob to the device");
  return QGEMM_OK;
}

}  // extern "C"
