// Host-side helpers shared by the entry points: error reporting, the per-device
// status word, device properties.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "npl_common.cuh"

namespace {

thread_local char g_error[512] = "no error";

// Status word of the library's kernels on each device (see npl_device_status).
__device__ int g_device_status;

constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices];
int g_cc[kMaxDevices];
int* g_status_ptr[kMaxDevices];
std::mutex g_mu;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

bool init_device(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return false;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_status_ptr[dev]) return true;
  int sms = 0, major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return false;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return false;
  g_sms[dev] = sms;
  g_cc[dev] = major * 10 + minor;
  g_status_ptr[dev] = static_cast<int*>(p);
  return true;
}

}  // namespace

namespace npl {

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NPL_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return NPL_OK;
}

int num_sms() {
  int dev = current_device();
  if (!init_device(dev)) return 0;
  return g_sms[dev];
}

int* device_status_ptr() {
  int dev = current_device();
  if (!init_device(dev)) return nullptr;
  return g_status_ptr[dev];
}

// Every entry calls this first: the kernels are compiled for sm_100a only.
int check_device() {
  int dev = current_device();
  if (!init_device(dev)) return fail(NPL_ERR_LAUNCH, "cannot query CUDA device %d", dev);
  if (g_cc[dev] != 100)
    return fail(NPL_ERR_UNSUPPORTED, "device %d is sm_%d; libnpl_w8a8 is built for sm_100a", dev, g_cc[dev]);
  return NPL_OK;
}

}  // namespace npl

extern "C" const char* npl_last_error_string(void) { return g_error; }

extern "C" int npl_version(void) { return 1; }

extern "C" int npl_device_status(int* code, int reset) {
  int rc = npl::check_device();
  if (rc) return rc;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess)
    return npl::launch_status("npl_device_status");
  if (reset && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)) != cudaSuccess)
      return npl::launch_status("npl_device_status reset");
  }
  if (code) *code = v;
  return v ? npl::fail(NPL_ERR_TIMEOUT, "device wait expired (code %d)", v) : NPL_OK;
}
