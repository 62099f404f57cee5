// cf_prescan.cu — SparseFlow prescan kernels.
//
// cf_prescan: the reference geometry.  For output tile (n, gh, gw) of size
// BH x BW, bit g of ag_mask is set iff some |x| > threshold lies in channel
// group g inside the receptive field of the tile's valid output pixels —
// the semantics of the reference's max-pool cascade (abs-amax per channel
// group -> max_pool(k, s, p) -> max_pool(tile, ceil) -> > threshold).  One
// CTA per tile; the CTA's warps stride over the receptive field, coalesced
// along W, and combine their per-thread group masks with warp ballots and a
// shared-memory OR.
//
// cf_prescan_conv_tiles: the fused conv kernel's own M-tile geometry over the
// [B][H][W][T][Cin_p] fp16 activations, one 16-byte vector per thread step.
#include "cf_common.cuh"

namespace cf {

int conv_geometry_for(int64_t T, int64_t B, int64_t Ho, int64_t Wo, int64_t Cout, int64_t Cin_p,
                      int64_t stride, bool sparse, int* TP, int* Wb, int* Hb, int* Bb,
                      int* n_wt, int* n_ht, int* n_mtiles, int* BK);

namespace {

constexpr int kPrescanThreads = 256;

__device__ __forceinline__ float load_any(const void* p, int fmt, int64_t i) {
  if (fmt == CF_FMT_F32) return static_cast<const float*>(p)[i];
  if (fmt == CF_FMT_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return (float)static_cast<const uint8_t*>(p)[i];
}

// Does input row `i` feed some output row in [o0, o1] (inclusive) of a
// (k, s, p) convolution?
__device__ __forceinline__ bool feeds(int i, int o0, int o1, int k, int s, int p) {
  // outputs o with 0 <= i + p - o*s < k
  const int num_hi = i + p;          // o*s <= i + p
  const int num_lo = i + p - k + 1;  // o*s >= i + p - k + 1
  int omax = num_hi >= 0 ? num_hi / s : -1;
  int omin = num_lo <= 0 ? 0 : (num_lo + s - 1) / s;
  if (omin < o0) omin = o0;
  if (omax > o1) omax = o1;
  return omin <= omax;
}

__global__ void __launch_bounds__(kPrescanThreads)
    prescan_ref_kernel(const void* __restrict__ x, int fmt, int32_t* __restrict__ ag_mask,
                       int32_t* __restrict__ tile_class, int C, int H, int W, int H_out,
                       int W_out, int k, int s, int p, int BH, int BW, int GS, int G, int GH,
                       int GW, float thr) {
  __shared__ uint32_t s_mask;
  const int tile = blockIdx.x;
  const int gw = tile % GW;
  const int gh = (tile / GW) % GH;
  const int n = tile / (GW * GH);
  const int o_h0 = gh * BH, o_h1 = min(H_out, o_h0 + BH) - 1;
  const int o_w0 = gw * BW, o_w1 = min(W_out, o_w0 + BW) - 1;
  const int r0 = max(0, o_h0 * s - p), r1 = min(H, o_h1 * s - p + k);
  const int c0 = max(0, o_w0 * s - p), c1 = min(W, o_w1 * s - p + k);
  const int rh = max(0, r1 - r0), rw = max(0, c1 - c0);
  if (threadIdx.x == 0) s_mask = 0;
  __syncthreads();
  uint32_t m = 0;
  const int64_t plane = (int64_t)H * W;
  const int64_t base = (int64_t)n * C * plane;
  // Thread -> fixed receptive-field position (row, col), channels strided by
  // the number of threads that share a position: divisions and the "does it
  // feed an output of the tile" test run once per position, not per element.
  const int P = rh * rw;
  if (P > 0) {
    // P <= blockDim: nrep threads share each position (channels strided by
    // nrep); otherwise each thread walks positions tid, tid + blockDim, ...
    const bool rep = (int)blockDim.x >= P;
    const int nrep = rep ? (int)blockDim.x / P : 1;
    const int pos_step = rep ? P : (int)blockDim.x;
    const int tid = threadIdx.x;
    if (tid < (rep ? nrep * P : (int)blockDim.x)) {
      const int c_first = rep ? tid / P : 0;
      for (int pos = rep ? tid % P : tid; pos < P; pos += pos_step) {
        const int row = pos / rw, col = pos - (pos / rw) * rw;
        const int ih = r0 + row, iw = c0 + col;
        if (feeds(ih, o_h0, o_h1, k, s, p) && feeds(iw, o_w0, o_w1, k, s, p)) {
          const int64_t off = base + (int64_t)ih * W + iw;
          // four channels' loads in flight together, then the group bits
          for (int c = c_first; c < C; c += 4 * nrep) {
            float v4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int cu = c + u * nrep;
              v4[u] = cu < C ? load_any(x, fmt, off + cu * plane) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (c + u * nrep < C && fabsf(v4[u]) > thr) m |= 1u << ((c + u * nrep) / GS);
          }
        }
      }
    }
  }
  // warp-level OR, then one shared atomic per warp
  for (int off = 16; off; off >>= 1) m |= __shfl_xor_sync(0xffffffffu, m, off);
  if ((threadIdx.x & 31) == 0 && m) atomicOr(&s_mask, m);
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t all = (G >= 32) ? 0xFFFFFFFFu : ((1u << G) - 1u);
    const uint32_t mk = s_mask;
    ag_mask[tile] = (int32_t)mk;
    tile_class[tile] = (mk == 0) ? 0 : (mk == all ? 2 : 1);
  }
}

// Count nonzero elements (any format), grid-stride, one atomic per block.
__global__ void __launch_bounds__(kPrescanThreads)
    count_nonzero_kernel(const void* __restrict__ x, int fmt, int64_t n, int64_t* nnz) {
  __shared__ unsigned long long s_cnt;
  if (threadIdx.x == 0) s_cnt = 0;
  __syncthreads();
  unsigned long long c = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t head = 0;
  if (fmt == CF_FMT_F16 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    // 8 halves per 16-byte load; the scalar loop below takes the tail
    const int64_t nv = n / 8;
    const uint4* xv = static_cast<const uint4*>(x);
    for (int64_t i = first; i < nv; i += stride) {
      const uint4 u = __ldg(xv + i);
      const uint32_t w4[4] = {u.x & 0x7FFF7FFFu, u.y & 0x7FFF7FFFu, u.z & 0x7FFF7FFFu,
                              u.w & 0x7FFF7FFFu};
#pragma unroll
      for (int j = 0; j < 4; ++j) c += ((w4[j] & 0xFFFFu) != 0) + ((w4[j] >> 16) != 0);
    }
    head = nv * 8;
  }
  for (int64_t i = head + first; i < n; i += stride)
    c += (load_any(x, fmt, i) != 0.f) ? 1ull : 0ull;
  for (int off = 16; off; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(&s_cnt, c);
  __syncthreads();
  if (threadIdx.x == 0 && s_cnt) atomicAdd(reinterpret_cast<unsigned long long*>(nnz), s_cnt);
}

// Conv-tile prescan over x[B][H][W][T][Cin_p] fp16.
__global__ void __launch_bounds__(kPrescanThreads)
    prescan_conv_kernel(const __half* __restrict__ x, uint32_t* __restrict__ mask,
                        int64_t* nnz, int T, int B, int H, int W, int Cin_p, int KH, int KW,
                        int s, int p, int Wb, int Hb, int Bb, int n_wt, int n_ht, int chunk) {
  __shared__ uint32_t s_mask;
  __shared__ unsigned long long s_cnt;
  const int mt = blockIdx.x;
  const int wt = mt % n_wt;
  const int ht = (mt / n_wt) % n_ht;
  const int bt = mt / (n_wt * n_ht);
  const int Ho = (H + 2 * p - KH) / s + 1;
  const int Wo = (W + 2 * p - KW) / s + 1;
  const int oh0 = ht * Hb, oh1 = min(Ho, oh0 + Hb) - 1;
  const int ow0 = wt * Wb, ow1 = min(Wo, ow0 + Wb) - 1;
  // receptive field (rows/cols read by the conv for this tile)
  const int rf_r0 = max(0, oh0 * s - p), rf_r1 = min(H, oh1 * s - p + KH);
  const int rf_c0 = max(0, ow0 * s - p), rf_c1 = min(W, ow1 * s - p + KW);
  // own region (each input element is counted by exactly one tile)
  const int own_r0 = min(H, ht * Hb * s), own_r1 = (ht == n_ht - 1) ? H : min(H, (ht + 1) * Hb * s);
  const int own_c0 = min(W, wt * Wb * s), own_c1 = (wt == n_wt - 1) ? W : min(W, (wt + 1) * Wb * s);
  const bool count = nnz != nullptr;
  const int r0 = count ? min(rf_r0, own_r0) : rf_r0;
  const int r1 = count ? max(rf_r1, own_r1) : rf_r1;
  const int c0 = count ? min(rf_c0, own_c0) : rf_c0;
  const int c1 = count ? max(rf_c1, own_c1) : rf_c1;
  const int b0 = bt * Bb, b1 = min(B, b0 + Bb);
  if (threadIdx.x == 0) {
    s_mask = 0;
    s_cnt = 0;
  }
  __syncthreads();
  const int vec_per_pix = T * Cin_p / 8;  // 16-byte vectors per pixel
  const int rh = max(0, r1 - r0), rw = max(0, c1 - c0), nb = max(0, b1 - b0);
  const int npix = nb * rh * rw;
  uint32_t m = 0;
  unsigned long long cnt = 0;
  // Thread -> fixed vector slot v of a pixel (its channel chunk bit is then
  // fixed too); pixels advance by a cursor (col, row, b), no divisions in the
  // loop.  With more vectors per pixel than threads, each thread takes
  // v = tid, tid + blockDim, ... of every pixel.
  const int tid = threadIdx.x;
  const bool rep = vec_per_pix <= (int)blockDim.x;
  const int ppp = rep ? (int)blockDim.x / vec_per_pix : 1;  // pixels per pass
  if (npix > 0 && (!rep || tid < ppp * vec_per_pix)) {
    const int v0 = rep ? tid % vec_per_pix : tid;
    int pix = rep ? tid / vec_per_pix : 0;
    int col = pix % rw, row = (pix / rw) % rh, bb = pix / (rw * rh);
    const int vstep = rep ? vec_per_pix : (int)blockDim.x;
    constexpr int U = 4;  // pixels whose loads are in flight together
    while (pix < npix) {
      const uint4* px[U];
      bool ok[U], in_rf[U], own[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        ok[u] = pix < npix;
        const int ih = r0 + row, iw = c0 + col;
        px[u] = reinterpret_cast<const uint4*>(
            x + (((int64_t)(b0 + bb) * H + ih) * W + iw) * (int64_t)T * Cin_p);
        in_rf[u] = ih >= rf_r0 && ih < rf_r1 && iw >= rf_c0 && iw < rf_c1;
        own[u] = count && ih >= own_r0 && ih < own_r1 && iw >= own_c0 && iw < own_c1;
        // advance the cursor by ppp pixels
        pix += ppp;
        col += ppp;
        while (col >= rw) {
          col -= rw;
          if (++row == rh) {
            row = 0;
            ++bb;
          }
        }
      }
      for (int v = v0; v < vec_per_pix; v += vstep) {
        uint4 q[U];
#pragma unroll
        for (int u = 0; u < U; ++u) q[u] = ok[u] ? __ldg(px[u] + v) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t cbit = 1u << (((v * 8) % Cin_p) / chunk);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const uint32_t w4[4] = {q[u].x & 0x7FFF7FFFu, q[u].y & 0x7FFF7FFFu,
                                  q[u].z & 0x7FFF7FFFu, q[u].w & 0x7FFF7FFFu};
          if ((w4[0] | w4[1] | w4[2] | w4[3]) == 0) continue;
          if (in_rf[u]) m |= cbit;
          if (own[u]) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              cnt += ((w4[j] & 0xFFFFu) != 0) + ((w4[j] >> 16) != 0);
          }
        }
      }
    }
  }
  for (int off = 16; off; off >>= 1) {
    m |= __shfl_xor_sync(0xffffffffu, m, off);
    cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
  }
  if ((threadIdx.x & 31) == 0) {
    if (m) atomicOr(&s_mask, m);
    if (cnt) atomicAdd(&s_cnt, cnt);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mask[mt] = s_mask;
    if (count && s_cnt) atomicAdd(reinterpret_cast<unsigned long long*>(nnz), s_cnt);
  }
}

}  // namespace
}  // namespace cf

using namespace cf;

extern "C" {

int cf_prescan(const void* x, int x_fmt, int32_t* ag_mask, int32_t* tile_class, int64_t* nnz_out,
               int64_t N, int64_t C, int64_t H, int64_t W, int64_t H_out, int64_t W_out,
               int64_t k, int64_t stride, int64_t pad, int64_t BH, int64_t BW, int64_t GS,
               float threshold, void* stream) {
  if (!x || !ag_mask || !tile_class) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (x_fmt != CF_FMT_F32 && x_fmt != CF_FMT_F16 && x_fmt != CF_FMT_U8)
    return fail(CF_ERR_INVALID_ARG, "x_fmt must be F32, F16 or U8");
  if (N < 0 || C <= 0 || H <= 0 || W <= 0 || H_out <= 0 || W_out <= 0 || k <= 0 || stride <= 0 ||
      pad < 0 || BH <= 0 || BW <= 0 || GS <= 0)
    return fail(CF_ERR_INVALID_ARG, "bad prescan geometry");
  if (pad > k / 2) return fail(CF_ERR_INVALID_ARG, "pad must be <= k/2 (max-pool semantics)");
  const int64_t G = (C + GS - 1) / GS;
  if (G > 32) return fail(CF_ERR_UNSUPPORTED, "at most 32 channel groups");
  const int64_t GH = (H_out + BH - 1) / BH, GW = (W_out + BW - 1) / BW;
  const int64_t tiles = N * GH * GW;
  if (tiles == 0) return CF_OK;
  if (tiles > 0x7FFFFFFF) return fail(CF_ERR_UNSUPPORTED, "too many tiles");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  prescan_ref_kernel<<<(unsigned)tiles, kPrescanThreads, 0, s>>>(
      x, x_fmt, ag_mask, tile_class, (int)C, (int)H, (int)W, (int)H_out, (int)W_out, (int)k,
      (int)stride, (int)pad, (int)BH, (int)BW, (int)GS, (int)G, (int)GH, (int)GW, threshold);
  if (int rc = check_launch("prescan launch")) return rc;
  if (nnz_out) {
    const int64_t n = N * C * H * W;
    int64_t blocks = (n + kPrescanThreads - 1) / kPrescanThreads;
    if (blocks > 148 * 8) blocks = 148 * 8;
    count_nonzero_kernel<<<(unsigned)blocks, kPrescanThreads, 0, s>>>(x, x_fmt, n, nnz_out);
    if (int rc = check_launch("count_nonzero launch")) return rc;
  }
  return CF_OK;
}

int cf_prescan_conv_tiles(const void* x, uint32_t* mask, int64_t* nnz_out, int64_t T, int64_t B,
                          int64_t H, int64_t W, int64_t Cin_p, int64_t Cout, int64_t KH,
                          int64_t KW, int64_t stride, int64_t pad, int64_t chunk, void* stream) {
  if (!x || !mask) return fail(CF_ERR_INVALID_ARG, "NULL pointer");
  if (T <= 0 || B <= 0 || H <= 0 || W <= 0 || KH <= 0 || KW <= 0 || stride <= 0 || pad < 0)
    return fail(CF_ERR_INVALID_ARG, "bad geometry");
  if (Cin_p % 16) return fail(CF_ERR_UNSUPPORTED, "Cin_p must be a multiple of 16");
  if (chunk < 16 || chunk % 8 || Cin_p % chunk || Cin_p / chunk > 32)
    return fail(CF_ERR_INVALID_ARG, "chunk must divide Cin_p into at most 32 chunks");
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return fail(CF_ERR_UNSUPPORTED, "x must be 16-byte aligned");
  const int64_t Ho = (H + 2 * pad - KH) / stride + 1;
  const int64_t Wo = (W + 2 * pad - KW) / stride + 1;
  if (Ho <= 0 || Wo <= 0) return fail(CF_ERR_INVALID_ARG, "empty output map");
  int TP, Wb, Hb, Bb, n_wt, n_ht, n_mt, BK;
  if (int rc = conv_geometry_for(T, B, Ho, Wo, Cout, Cin_p, stride, true, &TP, &Wb, &Hb, &Bb,
                                 &n_wt, &n_ht, &n_mt, &BK))
    return rc;
  if (int rc = require_sm100()) return rc;
  prescan_conv_kernel<<<n_mt, kPrescanThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), mask, nnz_out, (int)T, (int)B, (int)H, (int)W, (int)Cin_p,
      (int)KH, (int)KW, (int)stride, (int)pad, Wb, Hb, Bb, n_wt, n_ht, (int)chunk);
  return check_launch("prescan_conv launch");
}

}  // extern "C"
