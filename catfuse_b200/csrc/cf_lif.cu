// cf_lif.cu — bandwidth-bound multi-step LIF family (lif_fwd, bn_lif,
// bn_add_lif, add_lif, StaticZero, avgpool_lif) on the reference layout
// [T][N].  One thread owns 4 consecutive neurons for all T steps: 128-bit
// loads of z, membrane v in registers across T, spikes written as fp32 /
// fp16 / u8 or bit-packed (a warp covers 128 neurons = 4 packed words).
#include "cf_common.cuh"

namespace cf {

namespace {

constexpr int kThreads = 256;

// Where z' (the LIF input at step t for neuron n) comes from.
enum ZMode : int {
  Z_PLAIN = 0,   // z' = z
  Z_AFFINE = 1,  // z' = z*scale[c] + shift[c]   (z may be absent: z = 0)
  Z_ADD2 = 2,    // z' = x1 + x2
};

struct LifArgs {
  const void* z;        // [T][N] (fmt zfmt) or nullptr (zero)
  const void* z2;       // second addend for Z_ADD2 (fp32)
  const float* scale;   // [C] or nullptr
  const float* shift;   // [C] or nullptr
  const void* ident;    // [T][N] identity (fmt ifmt) or nullptr
  const float* v0;      // [N] or nullptr
  void* spikes;         // [T][N]
  float* vT;            // [N] or nullptr
  int64_t T, N, C, HW;
  int zfmt, ifmt, sfmt;
  LifParams lp;
};

__device__ __forceinline__ float4 load4(const void* p, int fmt, int64_t i) {
  if (fmt == CF_FMT_F32) {
    return __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i));
  } else {  // F16
    const uint2 raw = __ldcs(reinterpret_cast<const uint2*>(static_cast<const __half*>(p) + i));
    const __half2 a = *reinterpret_cast<const __half2*>(&raw.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&raw.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
  }
}

__device__ __forceinline__ float load1(const void* p, int fmt, int64_t i) {
  if (fmt == CF_FMT_F32) return static_cast<const float*>(p)[i];
  return __half2float(static_cast<const __half*>(p)[i]);
}

// Store 4 spikes of neurons [i, i+4) at step t.  For CF_FMT_BITS the 8 lanes
// sharing a 32-bit word combine their nibbles with shuffles (all 32 lanes of
// the warp must call this; `valid` masks lanes past the end).
__device__ __forceinline__ void store4(void* out, int fmt, int64_t idx, float s0, float s1,
                                       float s2, float s3, bool valid) {
  if (fmt == CF_FMT_BITS) {
    uint32_t nib = (uint32_t)(s0 != 0.f) | ((uint32_t)(s1 != 0.f) << 1) |
                   ((uint32_t)(s2 != 0.f) << 2) | ((uint32_t)(s3 != 0.f) << 3);
    if (!valid) nib = 0;
    const int lane = threadIdx.x & 31;
    uint32_t w = nib << (4 * (lane & 7));
    w |= __shfl_xor_sync(0xffffffffu, w, 1);
    w |= __shfl_xor_sync(0xffffffffu, w, 2);
    w |= __shfl_xor_sync(0xffffffffu, w, 4);
    if (valid && (lane & 7) == 0) static_cast<uint32_t*>(out)[idx >> 5] = w;
    return;
  }
  if (!valid) return;
  if (fmt == CF_FMT_F32) {
    __stcs(reinterpret_cast<float4*>(static_cast<float*>(out) + idx), make_float4(s0, s1, s2, s3));
  } else if (fmt == CF_FMT_F16) {
    __half2 a = __floats2half2_rn(s0, s1), b = __floats2half2_rn(s2, s3);
    uint2 raw;
    raw.x = *reinterpret_cast<uint32_t*>(&a);
    raw.y = *reinterpret_cast<uint32_t*>(&b);
    __stcs(reinterpret_cast<uint2*>(static_cast<__half*>(out) + idx), raw);
  } else {  // U8
    uint32_t w = (uint32_t)s0 | ((uint32_t)s1 << 8) | ((uint32_t)s2 << 16) | ((uint32_t)s3 << 24);
    __stcs(reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(out) + idx), w);
  }
}

__device__ __forceinline__ void store1(void* out, int fmt, int64_t idx, float s) {
  if (fmt == CF_FMT_F32) static_cast<float*>(out)[idx] = s;
  else if (fmt == CF_FMT_F16) static_cast<__half*>(out)[idx] = __float2half_rn(s);
  else static_cast<uint8_t*>(out)[idx] = (uint8_t)s;
}

// Channel of neuron n in [B][C][HW]: 32-bit division when the sizes allow it
// (a 64-bit division by a runtime value costs several times more).
__device__ __forceinline__ int64_t channel_of(const LifArgs& a, int64_t n) {
  if (a.N <= 0xFFFFFFFFll)
    return (int64_t)(((uint32_t)n / (uint32_t)a.HW) % (uint32_t)a.C);
  return (n / a.HW) % a.C;
}

// For Z_AFFINE, sc / sh are the BN scale and shift of the 4 neurons' channel
// (HW % 4 == 0 on this path: they share one channel), looked up once per
// neuron group by the caller.
template <int MODE>
__device__ __forceinline__ float4 zprime4(const LifArgs& a, int64_t t, int64_t n, float sc,
                                          float sh) {
  const int64_t i = t * a.N + n;
  float4 z;
  if (MODE == Z_ADD2) {
    const float4 x1 = __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(a.z) + i));
    const float4 x2 = __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(a.z2) + i));
    z = make_float4(__fadd_rn(x1.x, x2.x), __fadd_rn(x1.y, x2.y), __fadd_rn(x1.z, x2.z),
                    __fadd_rn(x1.w, x2.w));
  } else {
    z = a.z ? load4(a.z, a.zfmt, i) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (MODE == Z_AFFINE) {
      if (a.z) {
        z.x = __fadd_rn(__fmul_rn(z.x, sc), sh);
        z.y = __fadd_rn(__fmul_rn(z.y, sc), sh);
        z.z = __fadd_rn(__fmul_rn(z.z, sc), sh);
        z.w = __fadd_rn(__fmul_rn(z.w, sc), sh);
      } else {
        z = make_float4(sh, sh, sh, sh);
      }
    }
  }
  if (a.ident) {
    const float4 d = load4(a.ident, a.ifmt, i);
    z.x = __fadd_rn(z.x, d.x);
    z.y = __fadd_rn(z.y, d.y);
    z.z = __fadd_rn(z.z, d.z);
    z.w = __fadd_rn(z.w, d.w);
  }
  return z;
}

template <int MODE>
__device__ __forceinline__ float zprime1(const LifArgs& a, int64_t t, int64_t n) {
  const int64_t i = t * a.N + n;
  float z;
  if (MODE == Z_ADD2) {
    z = __fadd_rn(static_cast<const float*>(a.z)[i], static_cast<const float*>(a.z2)[i]);
  } else {
    z = a.z ? load1(a.z, a.zfmt, i) : 0.f;
    if (MODE == Z_AFFINE) {
      const int64_t c = (n / a.HW) % a.C;
      const float sc = a.scale ? a.scale[c] : 1.f;
      const float sh = a.shift ? a.shift[c] : 0.f;
      z = a.z ? __fadd_rn(__fmul_rn(z, sc), sh) : sh;
    }
  }
  if (a.ident) z = __fadd_rn(z, load1(a.ident, a.ifmt, i));
  return z;
}

// Vector path: N % 4 == 0 (and HW % 4 == 0 for the affine mode).
template <int MODE>
__global__ void __launch_bounds__(kThreads) lif_vec_kernel(LifArgs a) {
  const int64_t ngroups = a.N >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // Every lane of a warp iterates the same number of times so that the
  // bit-packing shuffles in store4 see a full warp.
  const int64_t base0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31);
  for (int64_t wbase = base0; wbase < ngroups; wbase += stride) {
    const int64_t g = wbase + (threadIdx.x & 31);
    const bool valid = g < ngroups;
    const int64_t n = (valid ? g : 0) << 2;
    float sc = 1.f, sh = 0.f;
    if (MODE == Z_AFFINE && valid) {
      const int64_t c = channel_of(a, n);
      if (a.scale) sc = __ldg(a.scale + c);
      if (a.shift) sh = __ldg(a.shift + c);
    }
    float4 v = (a.v0 && valid) ? *reinterpret_cast<const float4*>(a.v0 + n)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 znext = valid ? zprime4<MODE>(a, 0, n, sc, sh) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t t = 0; t < a.T; ++t) {
      const float4 z = znext;
      if (t + 1 < a.T && valid) znext = zprime4<MODE>(a, t + 1, n, sc, sh);
      const float s0 = lif_step(v.x, z.x, a.lp);
      const float s1 = lif_step(v.y, z.y, a.lp);
      const float s2 = lif_step(v.z, z.z, a.lp);
      const float s3 = lif_step(v.w, z.w, a.lp);
      store4(a.spikes, a.sfmt, t * a.N + n, s0, s1, s2, s3, valid);
    }
    if (a.vT && valid) *reinterpret_cast<float4*>(a.vT + n) = v;
  }
}

// Store 8 spikes of neurons [i, i+8) at step t (fp32 / fp16 / u8 formats):
// one 16-byte store for fp16, where the 4-neuron path issues 8-byte ones.
__device__ __forceinline__ void store8(void* out, int fmt, int64_t idx, const float (&sp)[8]) {
  if (fmt == CF_FMT_F32) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + idx);
    __stcs(o, make_float4(sp[0], sp[1], sp[2], sp[3]));
    __stcs(o + 1, make_float4(sp[4], sp[5], sp[6], sp[7]));
  } else if (fmt == CF_FMT_F16) {
    // spikes are 0 or 1: select the fp16 bit patterns
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      w[k] = (sp[2 * k] != 0.f ? 0x3C00u : 0u) | (sp[2 * k + 1] != 0.f ? 0x3C000000u : 0u);
    __stcs(reinterpret_cast<uint4*>(static_cast<__half*>(out) + idx),
           make_uint4(w[0], w[1], w[2], w[3]));
  } else {  // U8
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      lo |= (uint32_t)sp[k] << (8 * k);
      hi |= (uint32_t)sp[4 + k] << (8 * k);
    }
    __stcs(reinterpret_cast<uint2*>(static_cast<uint8_t*>(out) + idx), make_uint2(lo, hi));
  }
}

// Vector path with 8 neurons per thread (N % 8 == 0, HW % 8 == 0 for the
// affine mode, spikes not bit-packed): two 16-byte z loads per step and
// 16-byte fp16 spike stores.
template <int MODE>
__global__ void __launch_bounds__(kThreads) lif_vec8_kernel(LifArgs a) {
  const int64_t ngroups = a.N >> 3;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < ngroups; g += stride) {
    const int64_t n = g << 3;
    float sc = 1.f, sh = 0.f;
    if (MODE == Z_AFFINE) {
      const int64_t c = channel_of(a, n);
      if (a.scale) sc = __ldg(a.scale + c);
      if (a.shift) sh = __ldg(a.shift + c);
    }
    float v[8];
    if (a.v0) {
      const float4 v0a = *reinterpret_cast<const float4*>(a.v0 + n);
      const float4 v0b = *reinterpret_cast<const float4*>(a.v0 + n + 4);
      v[0] = v0a.x; v[1] = v0a.y; v[2] = v0a.z; v[3] = v0a.w;
      v[4] = v0b.x; v[5] = v0b.y; v[6] = v0b.z; v[7] = v0b.w;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = 0.f;
    }
    float4 na = zprime4<MODE>(a, 0, n, sc, sh), nb = zprime4<MODE>(a, 0, n + 4, sc, sh);
    for (int64_t t = 0; t < a.T; ++t) {
      const float z[8] = {na.x, na.y, na.z, na.w, nb.x, nb.y, nb.z, nb.w};
      if (t + 1 < a.T) {
        na = zprime4<MODE>(a, t + 1, n, sc, sh);
        nb = zprime4<MODE>(a, t + 1, n + 4, sc, sh);
      }
      float sp[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) sp[k] = lif_step(v[k], z[k], a.lp);
      store8(a.spikes, a.sfmt, t * a.N + n, sp);
    }
    if (a.vT) {
      float4* o = reinterpret_cast<float4*>(a.vT + n);
      o[0] = make_float4(v[0], v[1], v[2], v[3]);
      o[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
}

// Scalar path for ragged sizes.
template <int MODE>
__global__ void __launch_bounds__(kThreads) lif_scalar_kernel(LifArgs a) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; n < a.N; n += stride) {
    float v = a.v0 ? a.v0[n] : 0.f;
    for (int64_t t = 0; t < a.T; ++t) {
      const float s = lif_step(v, zprime1<MODE>(a, t, n), a.lp);
      store1(a.spikes, a.sfmt, t * a.N + n, s);
    }
    if (a.vT) a.vT[n] = v;
  }
}

int grid_for(int64_t work_items) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t blocks = (work_items + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sms * 8;  // 8 resident blocks of 256 per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int launch_lif(LifArgs& a, int mode, cudaStream_t stream) {
  if (a.T < 0 || a.N < 0) return fail(CF_ERR_INVALID_ARG, "negative T or N");
  if (a.T == 0 || a.N == 0) return CF_OK;
  if (!a.spikes) return fail(CF_ERR_INVALID_ARG, "spikes must not be NULL");
  if (a.sfmt < CF_FMT_F32 || a.sfmt > CF_FMT_BITS)
    return fail(CF_ERR_INVALID_ARG, "bad spike format %d", a.sfmt);
  if (a.z && a.zfmt != CF_FMT_F32 && a.zfmt != CF_FMT_F16)
    return fail(CF_ERR_INVALID_ARG, "z must be fp32 or fp16");
  if (a.ident && a.ifmt != CF_FMT_F32 && a.ifmt != CF_FMT_F16)
    return fail(CF_ERR_INVALID_ARG, "identity must be fp32 or fp16");
  if (!(a.lp.tau > 0.f)) return fail(CF_ERR_INVALID_ARG, "tau must be > 0");
  if (int rc = require_sm100()) return rc;
  bool vec = (a.N % 4 == 0);
  if (mode == Z_AFFINE && (a.HW % 4 != 0)) vec = false;
  const void* ptrs[] = {a.z, a.z2, a.ident, a.v0, a.spikes, a.vT};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) vec = false;
  if (a.sfmt == CF_FMT_BITS) {
    if (a.N % 32 != 0) return fail(CF_ERR_UNSUPPORTED, "bit-packed spikes need N %% 32 == 0");
    if (!vec) return fail(CF_ERR_UNSUPPORTED, "bit-packed spikes need 16-byte aligned inputs");
  }
  const bool vec8 = vec && a.sfmt != CF_FMT_BITS && a.N % 8 == 0 &&
                    (mode != Z_AFFINE || a.HW % 8 == 0);
  if (vec8) {
    const int grid = grid_for(a.N / 8);
    switch (mode) {
      case Z_PLAIN: lif_vec8_kernel<Z_PLAIN><<<grid, kThreads, 0, stream>>>(a); break;
      case Z_AFFINE: lif_vec8_kernel<Z_AFFINE><<<grid, kThreads, 0, stream>>>(a); break;
      default: lif_vec8_kernel<Z_ADD2><<<grid, kThreads, 0, stream>>>(a); break;
    }
  } else if (vec) {
    const int grid = grid_for(a.N / 4);
    switch (mode) {
      case Z_PLAIN: lif_vec_kernel<Z_PLAIN><<<grid, kThreads, 0, stream>>>(a); break;
      case Z_AFFINE: lif_vec_kernel<Z_AFFINE><<<grid, kThreads, 0, stream>>>(a); break;
      default: lif_vec_kernel<Z_ADD2><<<grid, kThreads, 0, stream>>>(a); break;
    }
  } else {
    const int grid = grid_for(a.N);
    switch (mode) {
      case Z_PLAIN: lif_scalar_kernel<Z_PLAIN><<<grid, kThreads, 0, stream>>>(a); break;
      case Z_AFFINE: lif_scalar_kernel<Z_AFFINE><<<grid, kThreads, 0, stream>>>(a); break;
      default: lif_scalar_kernel<Z_ADD2><<<grid, kThreads, 0, stream>>>(a); break;
    }
  }
  return check_launch("lif kernel launch");
}

// ---- avgpool + LIF ---------------------------------------------------------
// One thread per pooled output neuron (b, c, ho, wo); k*k window mean of x in
// the reference's accumulation order (row-major window sum, then / (k*k)).
__global__ void __launch_bounds__(kThreads)
    avgpool_lif_kernel(const float* __restrict__ x, const float* __restrict__ v0, void* spikes,
                       int sfmt, float* __restrict__ vT, int64_t T, int64_t B, int64_t C,
                       int64_t H, int64_t W, int k, LifParams lp) {
  const int64_t Ho = H / k, Wo = W / k;
  const int64_t No = B * C * Ho * Wo;
  const int64_t Ni = B * C * H * W;
  const float inv = 1.0f / (float)(k * k);
  const bool pow2 = ((k * k) & (k * k - 1)) == 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < No; o += stride) {
    const int64_t wo = o % Wo;
    const int64_t ho = (o / Wo) % Ho;
    const int64_t bc = o / (Wo * Ho);
    const int64_t ibase = bc * H * W + (ho * k) * W + wo * k;
    float v = v0 ? v0[o] : 0.f;
    for (int64_t t = 0; t < T; ++t) {
      const float* xt = x + t * Ni + ibase;
      float s = 0.f;
      for (int i = 0; i < k; ++i)
        for (int j = 0; j < k; ++j) s = __fadd_rn(s, xt[i * W + j]);
      const float z = pow2 ? __fmul_rn(s, inv) : __fdiv_rn(s, (float)(k * k));
      store1(spikes, sfmt, t * No + o, lif_step(v, z, lp));
    }
    if (vT) vT[o] = v;
  }
}

}  // namespace

}  // namespace cf

using namespace cf;

extern "C" {

int cf_lif_fwd(const void* z, int z_fmt, const float* v0, void* spikes, int spike_fmt, float* vT,
               int64_t T, int64_t N, float tau, float v_threshold, float v_reset, int hard_reset,
               int decay_input, void* stream) {
  if (!z && T > 0 && N > 0) return fail(CF_ERR_INVALID_ARG, "z must not be NULL");
  LifArgs a{};
  a.z = z; a.zfmt = z_fmt; a.v0 = v0; a.spikes = spikes; a.sfmt = spike_fmt; a.vT = vT;
  a.T = T; a.N = N; a.C = 1; a.HW = 1;
  a.lp = make_lif(tau, v_threshold, v_reset, hard_reset, decay_input);
  return launch_lif(a, Z_PLAIN, static_cast<cudaStream_t>(stream));
}

int cf_bn_lif(const void* z, int z_fmt, const float* scale, const float* shift,
              const void* identity, int identity_fmt, const float* v0, void* spikes,
              int spike_fmt, float* vT, int64_t T, int64_t B, int64_t C, int64_t HW, float tau,
              float v_threshold, float v_reset, int hard_reset, int decay_input, void* stream) {
  if (C <= 0 || HW <= 0 || B < 0) return fail(CF_ERR_INVALID_ARG, "bad B/C/HW");
  LifArgs a{};
  a.z = z; a.zfmt = z_fmt; a.scale = scale; a.shift = shift;
  a.ident = identity; a.ifmt = identity_fmt;
  a.v0 = v0; a.spikes = spikes; a.sfmt = spike_fmt; a.vT = vT;
  a.T = T; a.N = B * C * HW; a.C = C; a.HW = HW;
  a.lp = make_lif(tau, v_threshold, v_reset, hard_reset, decay_input);
  return launch_lif(a, Z_AFFINE, static_cast<cudaStream_t>(stream));
}

int cf_add_lif(const float* x1, const float* x2, const float* v0, void* spikes, int spike_fmt,
               float* vT, int64_t T, int64_t N, float tau, float v_threshold, float v_reset,
               int hard_reset, int decay_input, void* stream) {
  if ((!x1 || !x2) && T > 0 && N > 0) return fail(CF_ERR_INVALID_ARG, "x1/x2 must not be NULL");
  LifArgs a{};
  a.z = x1; a.z2 = x2; a.zfmt = CF_FMT_F32; a.v0 = v0; a.spikes = spikes; a.sfmt = spike_fmt;
  a.vT = vT; a.T = T; a.N = N; a.C = 1; a.HW = 1;
  a.lp = make_lif(tau, v_threshold, v_reset, hard_reset, decay_input);
  return launch_lif(a, Z_ADD2, static_cast<cudaStream_t>(stream));
}

int cf_avgpool_lif(const float* x, const float* v0, void* spikes, int spike_fmt, float* vT,
                   int64_t T, int64_t B, int64_t C, int64_t H, int64_t W, int k, float tau,
                   float v_threshold, float v_reset, int hard_reset, int decay_input,
                   void* stream) {
  if (!x || !spikes) return fail(CF_ERR_INVALID_ARG, "x/spikes must not be NULL");
  if (k <= 0 || H % k || W % k) return fail(CF_ERR_UNSUPPORTED, "H, W must be multiples of k");
  if (spike_fmt == CF_FMT_BITS) return fail(CF_ERR_UNSUPPORTED, "avgpool_lif: no bit-packed out");
  if (!(tau > 0.f)) return fail(CF_ERR_INVALID_ARG, "tau must be > 0");
  if (T <= 0 || B * C * H * W == 0) return CF_OK;
  if (int rc = require_sm100()) return rc;
  const int64_t No = B * C * (H / k) * (W / k);
  const LifParams lp = make_lif(tau, v_threshold, v_reset, hard_reset, decay_input);
  avgpool_lif_kernel<<<grid_for(No), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, v0, spikes, spike_fmt, vT, T, B, C, H, W, k, lp);
  return check_launch("avgpool_lif launch");
}

}  // extern "C"
