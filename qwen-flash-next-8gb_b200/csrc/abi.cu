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
