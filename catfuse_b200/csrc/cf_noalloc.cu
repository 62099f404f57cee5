// cf_noalloc.cu — a SparseFlow conv entry point that allocates nothing.
//
// cf_conv_bn_lif_egd needs a per-tile mask buffer between its prescan and the
// conv; every other entry point leaves that scratch to the caller.  Callers
// that cannot call cudaMalloc (a plugin host whose allocator owns all device
// memory and hands out only the tensors of a call, or code running under a
// memory budget that forbids allocation on the hot path) use
// cf_conv_bn_lif_egd_noalloc instead: the mask lives in a fixed array of
// device memory that this library defines at file scope, so the call needs
// only the inputs and outputs the caller already has.
#include "cf_common.cuh"

#include <atomic>

#include "catfuse_b200.h"

namespace {

// Largest number of M tiles (one 32-bit chunk mask each) the fixed mask array
// holds: 256 KB of device memory, which every GPU that loads this library
// keeps until the process exits.
constexpr int64_t kNoAllocMaxTiles = 65536;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint32_t g_noalloc_masks[kNoAllocMaxTiles];

// The array's device address on the current device.  In host code the symbol
// g_noalloc_masks is only a host-side stand-in, never a device address, so
// the address is looked up once per device (with that device current) and
// cached.
int noalloc_masks(uint32_t** out) {
  int dev = -1;
  if (int rc = cf::check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  static std::atomic<uint32_t*> cache[kNoAllocMaxDevices];
  if (dev >= 0 && dev < kNoAllocMaxDevices) {
    if (uint32_t* p = cache[dev].load(std::memory_order_acquire)) {
      *out = p;
      return CF_OK;
    }
  }
  void* p = nullptr;
  if (int rc = cf::check_cuda(cudaGetSymbolAddress(&p, g_noalloc_masks),
                              "cudaGetSymbolAddress(mask array)"))
    return rc;
  if (dev >= 0 && dev < kNoAllocMaxDevices)
    cache[dev].store(static_cast<uint32_t*>(p), std::memory_order_release);
  *out = static_cast<uint32_t*>(p);
  return CF_OK;
}

}  // namespace

extern "C" {

int cf_conv_bn_lif_egd_noalloc(const void* x, const void* wp, const float* scale,
                               const float* shift, const void* identity, int res_mode,
                               const float* v_in, float* v_out, void* out, int64_t T, int64_t B,
                               int64_t H, int64_t W, int64_t Cin_p, int64_t Cout, int64_t KH,
                               int64_t KW, int64_t stride, int64_t pad, float tau,
                               float v_threshold, float v_reset, int hard_reset,
                               int decay_input, float max_active_frac, void* stream) {
  if (!x || !wp || !out) return cf::fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (T <= 0 || B <= 0 || H <= 0 || W <= 0 || KH <= 0 || KW <= 0 || stride <= 0 || pad < 0)
    return cf::fail(CF_ERR_INVALID_ARG, "bad geometry");
  const int64_t Ho = (H + 2 * pad - KH) / stride + 1;
  const int64_t Wo = (W + 2 * pad - KW) / stride + 1;
  if (Ho <= 0 || Wo <= 0) return cf::fail(CF_ERR_INVALID_ARG, "empty output map");
  int32_t g[6];
  if (int rc = cf_conv_geometry_ex(T, B, Ho, Wo, Cout, Cin_p, stride, /*sparse*/ 1, g)) return rc;
  const int64_t n_mtiles = g[4];
  if (n_mtiles > kNoAllocMaxTiles)
    return cf::fail(CF_ERR_UNSUPPORTED,
                    "cf_conv_bn_lif_egd_noalloc: %lld M tiles exceed the fixed mask array "
                    "(at most %lld); use cf_prescan_conv_tiles + cf_conv_bn_lif_egd with a "
                    "caller-owned mask",
                    (long long)n_mtiles, (long long)kNoAllocMaxTiles);
  const int chunk = cf_conv_chunk(Cin_p, 0);
  if (chunk < 0) return chunk;
  if (int rc = cf::require_sm100()) return rc;
  uint32_t* masks = nullptr;
  if (int rc = noalloc_masks(&masks)) return rc;
  // The prescan clears the n_mtiles masks it uses before it ORs bits in, so
  // whatever a previous call left in the array never leaks into this one.
  if (int rc = cf_prescan_conv_tiles(x, masks, nullptr, T, B, H, W, Cin_p, Cout, KH, KW, stride,
                                     pad, chunk, stream))
    return rc;
  return cf_conv_bn_lif_egd(x, wp, scale, shift, identity, res_mode, v_in, v_out, out, masks, T,
                            B, H, W, Cin_p, Cout, KH, KW, stride, pad, tau, v_threshold, v_reset,
                            hard_reset, decay_input, max_active_frac, stream);
}

}  // extern "C"
