// Library-wide C-ABI entry points: version, status text, last-error detail,
// and the per-device property cache used by every launcher.
#include <stdarg.h>
#include <string.h>

#include <mutex>

#include "host.cuh"

namespace {
thread_local char g_msg[512] = "";
constexpr int kMaxDevices = 64;
qfn::DeviceInfo g_dev[kMaxDevices];
bool g_dev_ok[kMaxDevices] = {};
std::mutex g_dev_mu;
}  // namespace

namespace qfn {

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}

int current_device(DeviceInfo** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(QFN_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_dev_ok[dev]) {
    DeviceInfo d{};
    d.device = dev;
    int v = 0;
    if ((e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
      return set_error(QFN_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    d.smem_optin = static_cast<size_t>(v);
    if (d.cc_major != 10)
      return set_error(QFN_ERR_DEVICE, "libqfn is built for sm_100a; device %d is sm_%d%d", dev, d.cc_major,
                       d.cc_minor);
    g_dev[dev] = d;
    g_dev_ok[dev] = true;
  }
  *out = &g_dev[dev];
  return QFN_OK;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QFN_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  g_msg[0] = '\0';
  return QFN_OK;
}

}  // namespace qfn

extern "C" {

int qfn_version(void) { return 100; }

const char* qfn_strerror(int status) {
  switch (status) {
    case QFN_OK: return "ok";
    case QFN_ERR_INVALID_ARG: return "invalid argument";
    case QFN_ERR_ALIGNMENT: return "misaligned pointer";
    case QFN_ERR_CUDA: return "CUDA runtime error";
    case QFN_ERR_UNSUPPORTED: return "unsupported shape";
    case QFN_ERR_WORKSPACE: return "workspace too small";
    case QFN_ERR_DEVICE: return "unsupported or missing device";
    default: return "unknown status";
  }
}

const char* qfn_last_error(void) { return g_msg; }

}  // extern "C"

// ---------------------------------------------------------------------------
// Tensor-map cache (driver entry point resolved once; no link-time libcuda use)
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::mutex g_tmap_mu;
EncodeTiledFn g_encode = nullptr;
}  // namespace

namespace qfn {

}  // namespace qfn

// ---------------------------------------------------------------------------
// Generic 2-D tensor-map cache
namespace {
struct Tmap2Entry {
  const void* base;
  int dtype, device, swizzle;
  uint64_t inner, rows, stride;
  uint32_t box_inner, box_rows;
  CUtensorMap map;
};
constexpr int kTmap2Slots = 64;
Tmap2Entry g_tmaps2[kTmap2Slots];
int g_tmap2_count = 0, g_tmap2_next = 0;
}  // namespace

namespace qfn {

int tensor_map_2d(const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t rows,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle,
                  int device, CUtensorMap* out) {
  std::lock_guard<std::mutex> lk(g_tmap_mu);
  for (int i = 0; i < g_tmap2_count; ++i) {
    const Tmap2Entry& t = g_tmaps2[i];
    if (t.base == base && t.dtype == static_cast<int>(dtype) && t.device == device &&
        t.swizzle == static_cast<int>(swizzle) && t.inner == inner && t.rows == rows && t.stride == row_stride_bytes &&
        t.box_inner == box_inner && t.box_rows == box_rows) {
      *out = t.map;
      return QFN_OK;
    }
  }
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || !fn) return set_error(QFN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(QFN_ERR_CUDA, "cuTensorMapEncodeTiled (2-D) failed (%d)", static_cast<int>(r));
  Tmap2Entry& t = g_tmaps2[g_tmap2_count < kTmap2Slots ? g_tmap2_count++ : (g_tmap2_next++ % kTmap2Slots)];
  t.base = base;
  t.dtype = static_cast<int>(dtype);
  t.device = device;
  t.swizzle = static_cast<int>(swizzle);
  t.inner = inner;
  t.rows = rows;
  t.stride = row_stride_bytes;
  t.box_inner = box_inner;
  t.box_rows = box_rows;
  t.map = m;
  *out = m;
  return QFN_OK;
}

}  // namespace qfn

namespace {
struct TmapNdEntry {
  const void* base;
  int dtype, device, rank, swizzle, promotion;
  uint64_t dims[5], strides[4];
  uint32_t box[5];
  CUtensorMap map;
};
constexpr int kTmapNdSlots = 32;
TmapNdEntry g_tmapsnd[kTmapNdSlots];
int g_tmapnd_count = 0, g_tmapnd_next = 0;
}  // namespace

namespace qfn {

int tensor_map_nd(const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                  const uint64_t* strides, const uint32_t* box, int device, CUtensorMap* out,
                  CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promotion) {
  if (rank < 1 || rank > 5) return set_error(QFN_ERR_INVALID_ARG, "tensor map rank %d", rank);
  std::lock_guard<std::mutex> lk(g_tmap_mu);
  for (int i = 0; i < g_tmapnd_count; ++i) {
    const TmapNdEntry& t = g_tmapsnd[i];
    if (t.base != base || t.dtype != static_cast<int>(dtype) || t.device != device || t.rank != rank ||
        t.swizzle != static_cast<int>(swizzle) || t.promotion != static_cast<int>(promotion))
      continue;
    bool same = true;
    for (int d = 0; d < rank; ++d) same = same && t.dims[d] == dims[d] && t.box[d] == box[d];
    for (int d = 0; d + 1 < rank; ++d) same = same && t.strides[d] == strides[d];
    if (same) {
      *out = t.map;
      return QFN_OK;
    }
  }
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || !fn) return set_error(QFN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  CUtensorMap m;
  cuuint64_t d64[5], s64[4];
  cuuint32_t b32[5], es[5];
  for (int d = 0; d < rank; ++d) {
    d64[d] = dims[d];
    b32[d] = box[d];
    es[d] = 1;
  }
  for (int d = 0; d + 1 < rank; ++d) s64[d] = strides[d];
  CUresult r = g_encode(&m, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d64, s64, b32, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promotion,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(QFN_ERR_CUDA, "cuTensorMapEncodeTiled (%d-D) failed (%d)", rank, static_cast<int>(r));
  TmapNdEntry& t = g_tmapsnd[g_tmapnd_count < kTmapNdSlots ? g_tmapnd_count++ : (g_tmapnd_next++ % kTmapNdSlots)];
  t.base = base;
  t.dtype = static_cast<int>(dtype);
  t.device = device;
  t.rank = rank;
  t.swizzle = static_cast<int>(swizzle);
  t.promotion = static_cast<int>(promotion);
  for (int d = 0; d < rank; ++d) {
    t.dims[d] = dims[d];
    t.box[d] = box[d];
  }
  for (int d = 0; d + 1 < rank; ++d) t.strides[d] = strides[d];
  t.map = m;
  *out = m;
  return QFN_OK;
}

}  // namespace qfn

