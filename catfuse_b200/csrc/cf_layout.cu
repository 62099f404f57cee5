// cf_layout.cu — layout conversions between the reference layout
// [T][B][C][H][W] and the fused path's pixel-major/time-inner layout
// [B][H][W][T][C], weight packing, and the classifier head (global average
// pool + fc).  All transposes go through a 32x33 shared tile so that both the
// read and the write side are coalesced.
#include "cf_common.cuh"

namespace cf {
namespace {

constexpr int TB = 32;

__device__ __forceinline__ float ld_f(const void* p, int fmt, int64_t i) {
  return fmt == CF_FMT_F32 ? static_cast<const float*>(p)[i]
                           : __half2float(static_cast<const __half*>(p)[i]);
}

// x[T][B][C][H][W] -> y[B][H][W][T][Cp].  grid: (ceil(W/32), ceil(Cp/32), T*B*H)
__global__ void pack_kernel(const void* __restrict__ x, int fmt, __half* __restrict__ y, int T,
                            int B, int C, int H, int W, int Cp) {
  __shared__ float tile[TB][TB + 1];
  const int w0 = blockIdx.x * TB, c0 = blockIdx.y * TB;
  int z = blockIdx.z;
  const int h = z % H; z /= H;
  const int b = z % B;
  const int t = z / B;
  // read: threadIdx.x along w, threadIdx.y along c
  for (int cy = threadIdx.y; cy < TB; cy += blockDim.y) {
    const int c = c0 + cy, w = w0 + threadIdx.x;
    float v = 0.f;
    if (c < C && w < W) v = ld_f(x, fmt, ((((int64_t)t * B + b) * C + c) * H + h) * W + w);
    tile[cy][threadIdx.x] = v;
  }
  __syncthreads();
  // write: threadIdx.x along c
  for (int wy = threadIdx.y; wy < TB; wy += blockDim.y) {
    const int w = w0 + wy, c = c0 + threadIdx.x;
    if (w < W && c < Cp)
      y[((((int64_t)b * H + h) * W + w) * T + t) * Cp + c] = __float2half_rn(tile[threadIdx.x][wy]);
  }
}

// Few channels (C <= 8, Cp <= 32: image inputs): one thread per (t, b, h, w),
// w fastest so the C plane reads are coalesced; each thread writes its
// (b, h, w, t) row of Cp halves with 16-byte stores.
__global__ void pack_small_kernel(const void* __restrict__ x, int fmt, __half* __restrict__ y,
                                  int T, int B, int C, int H, int W, int Cp) {
  const int64_t plane = (int64_t)H * W;
  const int64_t n = (int64_t)T * B * plane;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tb = i / plane, hw = i - tb * plane;
    const int t = (int)(tb / B), b = (int)(tb - (int64_t)t * B);
    __align__(16) __half row[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) row[c] = __float2half_rn(0.f);
    for (int c = 0; c < C; ++c) row[c] = __float2half_rn(ld_f(x, fmt, (tb * C + c) * plane + hw));
    uint4* dst = reinterpret_cast<uint4*>(y + (((int64_t)b * plane + hw) * T + t) * Cp);
    for (int q = 0; q < Cp / 8; ++q) dst[q] = reinterpret_cast<const uint4*>(row)[q];
  }
}

// y[B][H][W][T][C] -> x[T][B][C][H][W].  grid: (ceil(W/32), ceil(C/32), T*B*H)
__global__ void unpack_kernel(const __half* __restrict__ y, void* __restrict__ x, int fmt, int T,
                              int B, int C, int H, int W) {
  __shared__ float tile[TB][TB + 1];
  const int w0 = blockIdx.x * TB, c0 = blockIdx.y * TB;
  int z = blockIdx.z;
  const int h = z % H; z /= H;
  const int b = z % B;
  const int t = z / B;
  for (int wy = threadIdx.y; wy < TB; wy += blockDim.y) {
    const int w = w0 + wy, c = c0 + threadIdx.x;
    float v = 0.f;
    if (w < W && c < C) v = __half2float(y[((((int64_t)b * H + h) * W + w) * T + t) * C + c]);
    tile[wy][threadIdx.x] = v;
  }
  __syncthreads();
  for (int cy = threadIdx.y; cy < TB; cy += blockDim.y) {
    const int c = c0 + cy, w = w0 + threadIdx.x;
    if (c < C && w < W) {
      const int64_t i = ((((int64_t)t * B + b) * C + c) * H + h) * W + w;
      if (fmt == CF_FMT_F32) static_cast<float*>(x)[i] = tile[threadIdx.x][cy];
      else static_cast<__half*>(x)[i] = __float2half_rn(tile[threadIdx.x][cy]);
    }
  }
}

// v[B][C][HW] <-> v[B][HW][C].  grid: (ceil(HW/32), ceil(C/32), B)
__global__ void v_layout_kernel(const float* __restrict__ src, float* __restrict__ dst, int C,
                                int HW, int to_nhwc) {
  __shared__ float tile[TB][TB + 1];
  const int p0 = blockIdx.x * TB, c0 = blockIdx.y * TB;
  const int64_t b = blockIdx.z;
  const int64_t off = b * (int64_t)C * HW;
  if (to_nhwc) {
    for (int cy = threadIdx.y; cy < TB; cy += blockDim.y) {
      const int c = c0 + cy, p = p0 + threadIdx.x;
      if (c < C && p < HW) tile[cy][threadIdx.x] = src[off + (int64_t)c * HW + p];
    }
    __syncthreads();
    for (int py = threadIdx.y; py < TB; py += blockDim.y) {
      const int p = p0 + py, c = c0 + threadIdx.x;
      if (p < HW && c < C) dst[off + (int64_t)p * C + c] = tile[threadIdx.x][py];
    }
  } else {
    for (int py = threadIdx.y; py < TB; py += blockDim.y) {
      const int p = p0 + py, c = c0 + threadIdx.x;
      if (p < HW && c < C) tile[py][threadIdx.x] = src[off + (int64_t)p * C + c];
    }
    __syncthreads();
    for (int cy = threadIdx.y; cy < TB; cy += blockDim.y) {
      const int c = c0 + cy, p = p0 + threadIdx.x;
      if (c < C && p < HW) dst[off + (int64_t)c * HW + p] = tile[threadIdx.x][cy];
    }
  }
}

__global__ void pack_weight_kernel(const float* __restrict__ w, __half* __restrict__ wp, int Cout,
                                   int Cin, int KH, int KW, int Cin_p) {
  const int64_t n = (int64_t)Cout * KH * KW * Cin_p;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int ci = (int)(i % Cin_p);
    int64_t r = i / Cin_p;
    const int kw = (int)(r % KW); r /= KW;
    const int kh = (int)(r % KH);
    const int co = (int)(r / KH);
    float v = 0.f;
    if (ci < Cin) v = w[(((int64_t)co * Cin + ci) * KH + kh) * KW + kw];
    wp[i] = __float2half_rn(v);
  }
}

// Split weights for the extended-precision conv: wp2[co][kh][kw][0][ci] =
// hi = fp16(w * prescale), wp2[co][kh][kw][1][ci] = lo = fp16(w * prescale - hi).
// prescale is a power of two, so w * prescale and the difference w*prescale - hi
// are exact in fp32; hi + lo carries 22 significant bits of the weight.
__global__ void pack_weight_split_kernel(const float* __restrict__ w, __half* __restrict__ wp,
                                         int Cout, int Cin, int KH, int KW, int Cin_p,
                                         float prescale) {
  const int64_t n = (int64_t)Cout * KH * KW * Cin_p;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int ci = (int)(i % Cin_p);
    const int64_t tap_row = i / Cin_p;  // (co, kh, kw)
    int64_t r = tap_row;
    const int kw = (int)(r % KW); r /= KW;
    const int kh = (int)(r % KH);
    const int co = (int)(r / KH);
    float v = 0.f;
    if (ci < Cin) v = __fmul_rn(w[(((int64_t)co * Cin + ci) * KH + kh) * KW + kw], prescale);
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
    wp[(tap_row * 2) * Cin_p + ci] = hi;
    wp[(tap_row * 2 + 1) * Cin_p + ci] = lo;
  }
}

// Integer weight planes: q = rint(w * prescale) (|q| < 2^28 for the
// prescale the caller picks), written as signed base-1024 digits
// q = q2 * 2^20 + q1 * 2^10 + q0 with q1, q0 in [-512, 512) and |q2| <= 257,
// each an exactly representable fp16 integer:
// wq[co][kh][kw][p][ci] = q_{2-p}, i.e. the most significant plane first.
__global__ void pack_weight_planes_kernel(const float* __restrict__ w, __half* __restrict__ wq,
                                          int Cout, int Cin, int KH, int KW, int Cin_p,
                                          float prescale) {
  const int64_t n = (int64_t)Cout * KH * KW * Cin_p;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int ci = (int)(i % Cin_p);
    const int64_t tap_row = i / Cin_p;  // (co, kh, kw)
    int64_t r = tap_row;
    const int kw = (int)(r % KW); r /= KW;
    const int kh = (int)(r % KH);
    const int co = (int)(r / KH);
    long long q = 0;
    if (ci < Cin) q = llrintf(__fmul_rn(w[(((int64_t)co * Cin + ci) * KH + kh) * KW + kw], prescale));
    const long long q2 = (q + (1ll << 19)) >> 20;  // floor division: round to nearest digit
    const long long rem = q - q2 * (1ll << 20);      // in [-2^19, 2^19)
    const long long q1 = (rem + 512) >> 10;
    const long long q0 = rem - q1 * 1024;            // in [-512, 512)
    __half* dst = wq + tap_row * 3 * Cin_p + ci;
    dst[0] = __float2half_rn((float)q2);
    dst[Cin_p] = __float2half_rn((float)q1);
    dst[2 * Cin_p] = __float2half_rn((float)q0);
  }
}

// `rows` (t, b) rows per CTA (1 for small heads, kFcRows when there are many
// classes): their means over H*W go to shared memory, then one warp per class
// reads the class's fc row once for all of them.
constexpr int kFcRows = 4;
__global__ void avgpool_fc_kernel(const __half* __restrict__ x, const float* __restrict__ fc_w,
                                  const float* __restrict__ fc_b, float* __restrict__ logits,
                                  int T, int B, int HW, int C, int K, int rows) {
  extern __shared__ float s_mean[];  // [rows][C]
  const int r0 = blockIdx.x * rows;
  const int nr = min(rows, T * B - r0);
  const float inv = 1.0f / (float)HW;
  for (int i = threadIdx.x; i < nr * C; i += blockDim.x) {
    const int rr = i / C, c = i - rr * C;
    const int row = r0 + rr;            // row = b * T + t
    const int b = row / T, t = row - b * T;
    float s = 0.f;
    const __half* p = x + (((int64_t)b * HW) * T + t) * C + c;
    for (int j = 0; j < HW; ++j) s += __half2float(p[(int64_t)j * T * C]);
    s_mean[rr * C + c] = s * inv;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int k = warp; k < K; k += blockDim.x >> 5) {
    float acc[kFcRows];
#pragma unroll
    for (int rr = 0; rr < kFcRows; ++rr) acc[rr] = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float wk = fc_w[(int64_t)k * C + c];
#pragma unroll
      for (int rr = 0; rr < kFcRows; ++rr)
        if (rr < nr) acc[rr] += s_mean[rr * C + c] * wk;
    }
#pragma unroll
    for (int rr = 0; rr < kFcRows; ++rr) {
      float a = acc[rr];
      for (int off = 16; off; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
      if (lane == 0 && rr < nr) {
        const int row = r0 + rr, b = row / T, t = row - b * T;
        logits[((int64_t)t * B + b) * K + k] = a + (fc_b ? fc_b[k] : 0.f);
      }
    }
  }
}

// Spikformer head: per sample b, the token mean m_t[c] = sum_n x[b][n][t][c] / N
// (x holds integer spike counts: the fp32 sum is exact), the pre-head LIF over
// t (one thread per channel, membrane in a register), the spikes kept in
// shared memory, then logits[t][b][k] = sum_c s_t[c] * fc_w[k][c] + fc_b[k]
// with one warp per (t, k).
__global__ void token_mean_lif_fc_kernel(const __half* __restrict__ x, const float* __restrict__ v_in,
                                         float* __restrict__ v_out, const float* __restrict__ fc_w,
                                         const float* __restrict__ fc_b, float* __restrict__ logits,
                                         int T, int B, int N, int C, int K, LifParams lp) {
  extern __shared__ float s_spk[];  // [T][C]
  const int b = blockIdx.x;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float v = v_in ? v_in[(int64_t)b * C + c] : 0.f;
    for (int t = 0; t < T; ++t) {
      const __half* p = x + (((int64_t)b * N) * T + t) * C + c;
      float sum = 0.f;
      for (int n = 0; n < N; ++n) sum = __fadd_rn(sum, __half2float(p[(int64_t)n * T * C]));
      const float m = __fdiv_rn(sum, (float)N);
      s_spk[t * C + c] = lif_step(v, m, lp);
    }
    if (v_out) v_out[(int64_t)b * C + c] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int tk = warp; tk < T * K; tk += nw) {
    const int t = tk / K, k = tk - t * K;
    float acc = 0.f;
    for (int c = lane; c < C; c += 32) acc = fmaf(s_spk[t * C + c], fc_w[(int64_t)k * C + c], acc);
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) logits[((int64_t)t * B + b) * K + k] = acc + (fc_b ? fc_b[k] : 0.f);
  }
}

// Max pool over x[B][H][W][T][C] fp16 (padding = -inf), one thread per
// output element group of 8 channels (16-byte vectors).
__global__ void maxpool_kernel(const __half* __restrict__ x, __half* __restrict__ y, int B, int H,
                               int W, int T, int C, int Ho, int Wo, int k, int s, int p) {
  const int cv = C / 8;
  const int64_t n = (int64_t)B * Ho * Wo * T * cv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c8 = (int)(i % cv);
    int64_t r = i / cv;
    const int t = (int)(r % T); r /= T;
    const int wo = (int)(r % Wo); r /= Wo;
    const int ho = (int)(r % Ho);
    const int b = (int)(r / Ho);
    __half2 m[4];
    const __half2 neg = __float2half2_rn(-65504.f);
    for (int j = 0; j < 4; ++j) m[j] = neg;
    for (int dh = 0; dh < k; ++dh) {
      const int ih = ho * s - p + dh;
      if (ih < 0 || ih >= H) continue;
      for (int dw = 0; dw < k; ++dw) {
        const int iw = wo * s - p + dw;
        if (iw < 0 || iw >= W) continue;
        const uint4 u = *reinterpret_cast<const uint4*>(
            x + ((((int64_t)b * H + ih) * W + iw) * T + t) * C + c8 * 8);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
        for (int j = 0; j < 4; ++j) m[j] = __hmax2(m[j], h[j]);
      }
    }
    *reinterpret_cast<uint4*>(y + ((((int64_t)b * Ho + ho) * Wo + wo) * T + t) * C + c8 * 8) =
        *reinterpret_cast<const uint4*>(m);
  }
}

// im2col packing for a convolution with few input channels (the network stem):
// y[b][ho][wo][t][q] = x[t][b][c][ho*s-p+kh][wo*s-p+kw] for q = (kh*k+kw)*C+c
// (zero outside the image and for q >= k*k*C).
// split = 1: y[..][q] = fp16(x) for q < k*k*C, and the rounding remainder
// fp16(x - fp16(x)) of the same element at q + k*k*C (the stem's real-valued
// input carried as hi + lo for the extended-precision conv).
__global__ void im2col_kernel(const void* __restrict__ x, int fmt, __half* __restrict__ y, int T,
                              int B, int C, int H, int W, int Ho, int Wo, int k, int s, int p,
                              int Kp, int split) {
  // One thread per output (pixel, t) row: gathers its k*k*C values and writes
  // the Kp-wide row with 16-byte stores.
  const int64_t n = (int64_t)B * Ho * Wo * T;
  const int KK = k * k * C;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i;
    const int t = (int)(r % T); r /= T;
    const int wo = (int)(r % Wo); r /= Wo;
    const int ho = (int)(r % Ho);
    const int b = (int)(r / Ho);
    uint4* dst = reinterpret_cast<uint4*>(y + i * Kp);
    // q = (kh*k + kw)*C + c walks with counters (no divisions per element)
    const int64_t plane = (int64_t)H * W;
    const int64_t base = ((int64_t)t * B + b) * C * plane;
    const int ih0 = ho * s - p, iw0 = wo * s - p;
    int c = 0, kw = 0, kh = 0;
    const int qend = split ? 2 * KK : KK;
    for (int q0 = 0; q0 < Kp; q0 += 8) {
      __align__(16) __half h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = q0 + j;
        float v = 0.f;
        if (q < qend) {
          const int ih = ih0 + kh, iw = iw0 + kw;
          if (ih >= 0 && ih < H && iw >= 0 && iw < W)
            v = ld_f(x, fmt, base + c * plane + (int64_t)ih * W + iw);
          if (q >= KK) v = __fsub_rn(v, __half2float(__float2half_rn(v)));  // lo part
          if (++c == C) {
            c = 0;
            if (++kw == k) {
              kw = 0;
              if (++kh == k) kh = 0;  // the lo pass restarts at tap (0, 0)
            }
          }
        }
        h[j] = __float2half_rn(v);
      }
      dst[q0 / 8] = *reinterpret_cast<const uint4*>(h);
    }
  }
}

}  // namespace
}  // namespace cf

using namespace cf;

extern "C" {

int cf_pack_tbchw(const void* x, int x_fmt, void* y, int64_t T, int64_t B, int64_t C, int64_t H,
                  int64_t W, int64_t Cp, void* stream) {
  if (!x || !y) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (x_fmt != CF_FMT_F32 && x_fmt != CF_FMT_F16) return fail(CF_ERR_INVALID_ARG, "bad x_fmt");
  if (T < 0 || B < 0 || C <= 0 || H <= 0 || W <= 0 || Cp < C || Cp % 16)
    return fail(CF_ERR_INVALID_ARG, "bad pack shape (Cp >= C, Cp %% 16 == 0)");
  if (T * B == 0) return CF_OK;
  if (T * B * H > 0x7FFFFFFF) return fail(CF_ERR_UNSUPPORTED, "T*B*H too large");
  if (int rc = require_sm100()) return rc;
  if (C <= 8 && Cp <= 32 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    const int64_t n = T * B * H * W;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    pack_small_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, x_fmt, static_cast<__half*>(y), (int)T, (int)B, (int)C, (int)H, (int)W, (int)Cp);
    return check_launch("pack launch");
  }
  dim3 grid((unsigned)((W + TB - 1) / TB), (unsigned)((Cp + TB - 1) / TB), (unsigned)(T * B * H));
  pack_kernel<<<grid, dim3(TB, 8), 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_fmt, static_cast<__half*>(y), (int)T, (int)B, (int)C, (int)H, (int)W, (int)Cp);
  return check_launch("pack launch");
}

int cf_unpack_bhwtc(const void* y, void* x, int x_fmt, int64_t T, int64_t B, int64_t C, int64_t H,
                    int64_t W, void* stream) {
  if (!x || !y) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (x_fmt != CF_FMT_F32 && x_fmt != CF_FMT_F16) return fail(CF_ERR_INVALID_ARG, "bad x_fmt");
  if (T < 0 || B < 0 || C <= 0 || H <= 0 || W <= 0) return fail(CF_ERR_INVALID_ARG, "bad shape");
  if (T * B == 0) return CF_OK;
  if (T * B * H > 0x7FFFFFFF) return fail(CF_ERR_UNSUPPORTED, "T*B*H too large");
  if (int rc = require_sm100()) return rc;
  dim3 grid((unsigned)((W + TB - 1) / TB), (unsigned)((C + TB - 1) / TB), (unsigned)(T * B * H));
  unpack_kernel<<<grid, dim3(TB, 8), 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(y), x, x_fmt, (int)T, (int)B, (int)C, (int)H, (int)W);
  return check_launch("unpack launch");
}

int cf_v_layout(const float* src, float* dst, int64_t B, int64_t C, int64_t H, int64_t W,
                int to_nhwc, void* stream) {
  if (!src || !dst || src == dst) return fail(CF_ERR_INVALID_ARG, "src/dst NULL or aliased");
  if (B < 0 || C <= 0 || H <= 0 || W <= 0) return fail(CF_ERR_INVALID_ARG, "bad shape");
  if (B == 0) return CF_OK;
  if (B > 65535) return fail(CF_ERR_UNSUPPORTED, "B too large");
  if (int rc = require_sm100()) return rc;
  const int64_t HW = H * W;
  dim3 grid((unsigned)((HW + TB - 1) / TB), (unsigned)((C + TB - 1) / TB), (unsigned)B);
  v_layout_kernel<<<grid, dim3(TB, 8), 0, static_cast<cudaStream_t>(stream)>>>(
      src, dst, (int)C, (int)HW, to_nhwc);
  return check_launch("v_layout launch");
}

int cf_pack_conv_weight(const float* w, void* wp, int64_t Cout, int64_t Cin, int64_t KH,
                        int64_t KW, int64_t Cin_p, void* stream) {
  if (!w || !wp) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (Cout <= 0 || Cin <= 0 || KH <= 0 || KW <= 0 || Cin_p < Cin || Cin_p % 16)
    return fail(CF_ERR_INVALID_ARG, "bad weight shape (Cin_p >= Cin, Cin_p %% 16 == 0)");
  if (int rc = require_sm100()) return rc;
  const int64_t n = Cout * KH * KW * Cin_p;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  pack_weight_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      w, static_cast<__half*>(wp), (int)Cout, (int)Cin, (int)KH, (int)KW, (int)Cin_p);
  return check_launch("pack_weight launch");
}

int cf_avgpool_fc(const void* x, const float* fc_w, const float* fc_b, float* logits, int64_t T,
                  int64_t B, int64_t H, int64_t W, int64_t C, int64_t K, void* stream) {
  if (!x || !fc_w || !logits) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (T <= 0 || B <= 0 || H <= 0 || W <= 0 || C <= 0 || K <= 0)
    return fail(CF_ERR_INVALID_ARG, "bad shape");
  if (C * 4 * kFcRows > 48 * 1024) return fail(CF_ERR_UNSUPPORTED, "C too large for the head kernel");
  if (int rc = require_sm100()) return rc;
  const int rows = K >= 64 ? kFcRows : 1;
  avgpool_fc_kernel<<<(unsigned)((T * B + rows - 1) / rows), 256, (size_t)C * 4 * rows,
                      static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), fc_w, fc_b, logits, (int)T, (int)B, (int)(H * W), (int)C,
      (int)K, rows);
  return check_launch("avgpool_fc launch");
}

static int im2col_impl(const void* x, int x_fmt, void* y, int64_t T, int64_t B, int64_t C,
                       int64_t H, int64_t W, int64_t k, int64_t stride, int64_t pad, int64_t Kp,
                       int split, void* stream) {
  if (!x || !y) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (x_fmt != CF_FMT_F32 && x_fmt != CF_FMT_F16) return fail(CF_ERR_INVALID_ARG, "bad x_fmt");
  const int64_t need = (split ? 2 : 1) * k * k * C;
  if (T <= 0 || B <= 0 || C <= 0 || H <= 0 || W <= 0 || k <= 0 || stride <= 0 || pad < 0 ||
      Kp < need || Kp % 16)
    return fail(CF_ERR_INVALID_ARG, "bad im2col shape (Kp >= %sk*k*C, Kp %% 16 == 0)",
                split ? "2*" : "");
  const int64_t Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
  if (Ho <= 0 || Wo <= 0) return fail(CF_ERR_INVALID_ARG, "empty output map");
  if (int rc = require_sm100()) return rc;
  if ((reinterpret_cast<uintptr_t>(y) & 15) != 0)
    return fail(CF_ERR_UNSUPPORTED, "y must be 16-byte aligned");
  const int64_t n = B * Ho * Wo * T;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  im2col_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_fmt, static_cast<__half*>(y), (int)T, (int)B, (int)C, (int)H, (int)W, (int)Ho,
      (int)Wo, (int)k, (int)stride, (int)pad, (int)Kp, split);
  return check_launch("im2col launch");
}

int cf_token_mean_lif_fc(const void* x, const float* v_in, float* v_out, const float* fc_w,
                         const float* fc_b, float* logits, int64_t T, int64_t B, int64_t N,
                         int64_t C, int64_t K, float tau, float v_threshold, float v_reset,
                         int hard_reset, int decay_input, void* stream) {
  if (!x || !fc_w || !logits) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (T <= 0 || B <= 0 || N <= 0 || C <= 0 || K <= 0) return fail(CF_ERR_INVALID_ARG, "bad shape");
  if (!(tau > 0.f)) return fail(CF_ERR_INVALID_ARG, "tau must be > 0");
  if (T * C * 4 > 48 * 1024) return fail(CF_ERR_UNSUPPORTED, "T * C too large for the head kernel");
  if (int rc = require_sm100()) return rc;
  token_mean_lif_fc_kernel<<<(unsigned)B, 256, (size_t)(T * C) * 4,
                             static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), v_in, v_out, fc_w, fc_b, logits, (int)T, (int)B, (int)N,
      (int)C, (int)K, make_lif(tau, v_threshold, v_reset, hard_reset, decay_input));
  return check_launch("token_mean_lif_fc launch");
}

int cf_pack_im2col(const void* x, int x_fmt, void* y, int64_t T, int64_t B, int64_t C, int64_t H,
                   int64_t W, int64_t k, int64_t stride, int64_t pad, int64_t Kp, void* stream) {
  return im2col_impl(x, x_fmt, y, T, B, C, H, W, k, stride, pad, Kp, 0, stream);
}

int cf_pack_im2col_split(const void* x, int x_fmt, void* y, int64_t T, int64_t B, int64_t C,
                         int64_t H, int64_t W, int64_t k, int64_t stride, int64_t pad, int64_t Kp,
                         void* stream) {
  return im2col_impl(x, x_fmt, y, T, B, C, H, W, k, stride, pad, Kp, 1, stream);
}

int cf_pack_conv_weight_planes(const float* w, void* wq, int64_t Cout, int64_t Cin, int64_t KH,
                               int64_t KW, int64_t Cin_p, float prescale, void* stream) {
  if (!w || !wq) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (Cout <= 0 || Cin <= 0 || KH <= 0 || KW <= 0 || Cin_p < Cin || Cin_p % 16)
    return fail(CF_ERR_INVALID_ARG, "bad weight shape (Cin_p >= Cin, Cin_p %% 16 == 0)");
  int e = 0;
  if (!(prescale > 0.f) || frexpf(prescale, &e) != 0.5f)
    return fail(CF_ERR_INVALID_ARG, "prescale must be a positive power of two");
  if (int rc = require_sm100()) return rc;
  const int64_t n = Cout * KH * KW * Cin_p;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  pack_weight_planes_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      w, static_cast<__half*>(wq), (int)Cout, (int)Cin, (int)KH, (int)KW, (int)Cin_p, prescale);
  return check_launch("pack_weight_planes launch");
}

int cf_pack_conv_weight_split(const float* w, void* wp2, int64_t Cout, int64_t Cin, int64_t KH,
                              int64_t KW, int64_t Cin_p, float prescale, void* stream) {
  if (!w || !wp2) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (Cout <= 0 || Cin <= 0 || KH <= 0 || KW <= 0 || Cin_p < Cin || Cin_p % 16)
    return fail(CF_ERR_INVALID_ARG, "bad weight shape (Cin_p >= Cin, Cin_p %% 16 == 0)");
  int e = 0;
  if (!(prescale > 0.f) || frexpf(prescale, &e) != 0.5f)
    return fail(CF_ERR_INVALID_ARG, "prescale must be a positive power of two");
  if (int rc = require_sm100()) return rc;
  const int64_t n = Cout * KH * KW * Cin_p;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  pack_weight_split_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      w, static_cast<__half*>(wp2), (int)Cout, (int)Cin, (int)KH, (int)KW, (int)Cin_p, prescale);
  return check_launch("pack_weight_split launch");
}

int cf_maxpool_bhwtc(const void* x, void* y, int64_t B, int64_t H, int64_t W, int64_t T,
                     int64_t C, int64_t k, int64_t stride, int64_t pad, void* stream) {
  if (!x || !y) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (B <= 0 || H <= 0 || W <= 0 || T <= 0 || C <= 0 || k <= 0 || stride <= 0 || pad < 0 ||
      pad > k / 2)
    return fail(CF_ERR_INVALID_ARG, "bad maxpool shape");
  if (C % 8) return fail(CF_ERR_UNSUPPORTED, "C must be a multiple of 8");
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) != 0)
    return fail(CF_ERR_UNSUPPORTED, "x and y must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  const int64_t Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
  const int64_t n = B * Ho * Wo * T * (C / 8);
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  maxpool_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), static_cast<__half*>(y), (int)B, (int)H, (int)W, (int)T,
      (int)C, (int)Ho, (int)Wo, (int)k, (int)stride, (int)pad);
  return check_launch("maxpool launch");
}

}  // extern "C"
