// cf_api.cu — library-level entry points: version, error reporting, device
// checks and the device-side error word.
#include "cf_common.cuh"

#include <cstring>
#include <string>

namespace cf {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return CF_OK;
  return fail(CF_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

int require_sm100() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(CF_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return fail(CF_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                major, minor);
  return CF_OK;
}

}  // namespace cf

extern "C" {

const char* cf_version(void) { return "catfuse_b200 0.1.0 (sm_100a)"; }

size_t cf_get_last_error(char* buf, size_t buf_len) {
  const std::string& s = cf::g_last_error;
  if (buf && buf_len) {
    size_t n = s.size() < buf_len - 1 ? s.size() : buf_len - 1;
    memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
  return s.size();
}

int cf_device_supported(void) { return cf::require_sm100() == CF_OK ? 1 : 0; }

}  // extern "C"
