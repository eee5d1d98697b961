// Host-side error plumbing, device checks and small utility entry points.
#include <stdarg.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include "common.cuh"
#include "rgpt.h"

__device__ int g_rgpt_device_error = 0;

static thread_local char t_last_error[1024] = {0};

int rgpt_set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int rgpt_check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return rgpt_set_error(RGPT_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return RGPT_OK;
}

namespace {
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
int g_arch_ok[kMaxDevices] = {0};  // 0 unknown, 1 ok, -1 wrong arch
}  // namespace

int rgpt_check_device(int device) {
  if (device < 0 || device >= kMaxDevices) return rgpt_set_error(RGPT_ERR_INTERNAL, "device index %d", device);
  if (g_arch_ok[device] == 0) {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    g_sm_count[device] = sms;
    g_arch_ok[device] = (major == 10 && minor == 0) ? 1 : -1;
  }
  if (g_arch_ok[device] < 0)
    return rgpt_set_error(RGPT_ERR_UNSUPPORTED_ARCH, "librgpt_kernels is built for sm_100a (B200) only");
  return RGPT_OK;
}

int rgpt_num_sms(int device) {
  if (device < 0 || device >= kMaxDevices || g_sm_count[device] == 0) rgpt_check_device(device);
  return g_sm_count[device] > 0 ? g_sm_count[device] : 148;
}

int rgpt_pdl_enabled() {
  static const int enabled = [] {
    const char* v = getenv("RGPT_PDL");
    return (v != nullptr && v[0] == '0') ? 0 : 1;
  }();
  return enabled;
}

extern "C" int rgpt_last_error(char* buf, unsigned long long buflen) {
  if (buf == nullptr || buflen == 0) return RGPT_ERR_BAD_SHAPE;
  strncpy(buf, t_last_error, buflen - 1);
  buf[buflen - 1] = 0;
  return RGPT_OK;
}

extern "C" int rgpt_device_error(void) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return rgpt_set_error(RGPT_ERR_LAUNCH, "device sync: %s", cudaGetErrorString(e));
  int v = 0, zero = 0;
  cudaMemcpyFromSymbol(&v, g_rgpt_device_error, sizeof(int));
  cudaMemcpyToSymbol(g_rgpt_device_error, &zero, sizeof(int));
  if (v != 0) return rgpt_set_error(RGPT_ERR_DEVICE_TIMEOUT, "device error word = %d", v);
  return RGPT_OK;
}

extern "C" int rgpt_version(void) { return 100; }
