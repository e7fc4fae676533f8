// Host-side plumbing of the C ABI: status strings, the per-thread error text, the
// sm_100 device check and the cached SM count.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace w8host {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return W8_OK;
  set_error("CUDA error %d: %s", static_cast<int>(e), cudaGetErrorString(e));
  return W8_ERR_CUDA;
}

constexpr int kMaxDevices = 64;

// Per device: 0 = unknown, 1 = sm_100, -1 = anything else.
static int g_arch_ok[kMaxDevices] = {};
static int g_sms[kMaxDevices] = {};

int require_sm100(int* device) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device ordinal %d out of range", dev);
    return W8_ERR_UNSUPPORTED;
  }
  if (g_arch_ok[dev] == 0) {
    int major = 0, minor = 0, sms = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_status(e);
    e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e != cudaSuccess) return cuda_status(e);
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_status(e);
    g_sms[dev] = sms;
    g_arch_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
  }
  if (g_arch_ok[dev] != 1) {
    set_error("device %d is not an sm_100 (B200-class) GPU; these kernels are built for sm_100a only",
              dev);
    return W8_ERR_UNSUPPORTED;
  }
  *device = dev;
  return W8_OK;
}

int num_sms(int* out) {
  int dev = 0;
  const int st = require_sm100(&dev);
  if (st != W8_OK) return st;
  *out = g_sms[dev];
  return W8_OK;
}

int gemm_device_status(int clear, int* out);
int attention_device_status(int clear, int* out);
int peer_device_status(int clear, int* out);

}  // namespace w8host

extern "C" const char* w8_status_string(int status) {
  switch (status) {
    case W8_OK: return "ok";
    case W8_ERR_INVALID_ARG: return "invalid argument";
    case W8_ERR_ALIGNMENT: return "misaligned pointer or row pitch";
    case W8_ERR_UNSUPPORTED: return "unsupported device or shape";
    case W8_ERR_CUDA: return "CUDA error";
    case W8_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* w8_last_error(void) { return w8host::g_last_error; }

extern "C" int w8_abi_version(void) { return (1 << 16) | 1; }

extern "C" int w8_device_status(int clear) {
  int dev = 0;
  int st = w8host::require_sm100(&dev);
  if (st != W8_OK) return st;
  int v = W8_OK;
  st = w8host::gemm_device_status(clear, &v);
  if (st != W8_OK) return st;
  int va = W8_OK;
  st = w8host::attention_device_status(clear, &va);
  if (st != W8_OK) return st;
  int vp = W8_OK;
  st = w8host::peer_device_status(clear, &vp);
  if (st != W8_OK) return st;
  if (v != W8_OK) return v;
  return va != W8_OK ? va : vp;
}
