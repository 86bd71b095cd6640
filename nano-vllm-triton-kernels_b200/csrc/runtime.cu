// Host-side helpers of the C ABI: device checks, SM count cache, status strings.
#include <atomic>

#include "common.cuh"

namespace nvb200 {

namespace {
constexpr int kMaxDevices = 64;
std::atomic<int> g_sms[kMaxDevices];      // 0 = not queried yet
std::atomic<int> g_cc_ok[kMaxDevices];    // 0 = unknown, 1 = sm_100, 2 = other
}  // namespace

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int v = g_sms[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    g_sms[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return NVB200_ERR_NO_DEVICE;
  int ok = g_cc_ok[dev].load(std::memory_order_relaxed);
  if (ok == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    ok = (major == 10 && minor == 0) ? 1 : 2;
    g_cc_ok[dev].store(ok, std::memory_order_relaxed);
  }
  return ok == 1 ? NVB200_OK : NVB200_ERR_NO_DEVICE;
}

}  // namespace nvb200

extern "C" const char *nvb200_status_string(int code) {
  switch (code) {
    case NVB200_OK: return "ok";
    case NVB200_ERR_ARG: return "invalid argument (size, stride, pointer or dtype)";
    case NVB200_ERR_UNSUPPORTED: return "unsupported by this build";
    case NVB200_ERR_CUDA: return "CUDA launch or runtime error";
    case NVB200_ERR_NO_DEVICE: return "current device is not sm_100 (B200)";
    default: return "unknown status";
  }
}
