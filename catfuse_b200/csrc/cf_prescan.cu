// cf_prescan.cu — SparseFlow prescan kernels.
//
// cf_prescan: the reference geometry.  For output tile (n, gh, gw) of size
// BH x BW, bit g of ag_mask is set iff some |x| > threshold lies in channel
// group g inside the receptive field of the tile's valid output pixels --
// the semantics of the reference's max-pool cascade (abs-amax per channel
// group -> max_pool(k, s, p) -> max_pool(tile, ceil) -> > threshold).  Every
// input element is read once (see prescan_ref_kernel).
//
// cf_prescan_conv_tiles: the fused conv kernel's own M-tile geometry over the
// [B][H][W][T][Cin_p] fp16 activations, one pass (every element read once).
#include "cf_common.cuh"

#include <atomic>

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

// Reference-geometry prescan, one pass over x[N][C][H][W]: CTA (n, channel
// block) streams the block's H*W planes (thread = pixel, coalesced along the
// plane, eight channels' loads in flight), ORs each pixel's group bits
// together over its channels, then ORs them into the shared masks of every
// tile whose valid output pixels' receptive fields contain the pixel (row and
// column -> tile-range tables), and flushes the sample's masks with
// atomicOr into the zeroed ag_mask.  The tile classes follow in
// prescan_classify_kernel once every channel block has been merged.
constexpr int kMaxTilesPerSample = 8192;
constexpr int kRefChannelsPerCta = 32;

__global__ void __launch_bounds__(kPrescanThreads)
    prescan_ref_kernel(const void* __restrict__ x, int fmt, int32_t* __restrict__ ag_mask,
                       int64_t* nnz, int C, int H, int W, int H_out, int W_out, int k, int s,
                       int p, int BH, int BW, int GS, int GH, int GW, float thr, int sep) {
  extern __shared__ uint32_t s_tiles[];           // GH * GW masks of this sample
  uint16_t* s_row = reinterpret_cast<uint16_t*>(s_tiles + GH * GW);  // (first tile, count)
  uint16_t* s_col = s_row + 2 * H;
  // Separable mode (small planes): every pixel's group bits land in s_pix,
  // then the tile masks are OR-reduced from it along rows (s_cor[ih][tc]) and
  // then along columns, instead of every pixel OR-ing into the shared masks of
  // all its tiles (which piles same-address atomics onto a few words).
  uint32_t* s_pix = reinterpret_cast<uint32_t*>(s_col + 2 * W);  // H * W
  uint32_t* s_cor = s_pix + H * W;                                // H * GW
  __shared__ unsigned long long s_cnt;
  const int n_cb = (C + kRefChannelsPerCta - 1) / kRefChannelsPerCta;
  const int n = blockIdx.x / n_cb;
  const int cb = blockIdx.x - n * n_cb;
  const int c0 = cb * kRefChannelsPerCta, c1 = min(C, c0 + kRefChannelsPerCta);
  for (int i = threadIdx.x; i < GH * GW; i += blockDim.x) s_tiles[i] = 0;
  if (sep)
    for (int i = threadIdx.x; i < H * W; i += blockDim.x) s_pix[i] = 0;
  if (threadIdx.x == 0) s_cnt = 0;
  // input row ih feeds output rows o with o*s in [ih + p - k + 1, ih + p],
  // o < H_out; tile rows o / BH of that range
  for (int i = threadIdx.x; i < H + W; i += blockDim.x) {
    const bool is_row = i < H;
    const int pos = is_row ? i : i - H;
    const int n_out = is_row ? H_out : W_out, tb = is_row ? BH : BW;
    int olo = pos + p - k + 1, ohi = pos + p;
    olo = olo <= 0 ? 0 : (olo + s - 1) / s;
    ohi = ohi < 0 ? -1 : min(n_out - 1, ohi / s);
    uint16_t first = 0, cntt = 0;
    if (olo <= ohi) {
      first = (uint16_t)(olo / tb);
      cntt = (uint16_t)(ohi / tb - olo / tb + 1);
    }
    uint16_t* dst = is_row ? s_row + 2 * pos : s_col + 2 * pos;
    dst[0] = first;
    dst[1] = cntt;
  }
  __syncthreads();
  const int64_t plane = (int64_t)H * W;
  const int64_t base = ((int64_t)n * C + c0) * plane;
  const bool count = nnz != nullptr;
  unsigned long long cnt = 0;
  // Thread -> group of 8 consecutive pixels of the plane (one 16-byte fp16
  // load, two fp32 loads or one 8-byte u8 load per channel when the plane
  // allows it), four channels' loads in flight.
  const int HW = H * W;
  const int esz = fmt == CF_FMT_F32 ? 4 : (fmt == CF_FMT_F16 ? 2 : 1);
  const bool vec = (HW % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(x) + (uintptr_t)(base * esz)) % 16 == 0);
  const int ngrp = vec ? HW / 8 : HW;
  const __half2 thr2 = __half2half2(__float2half_rd(thr));  // |h| > thr  <=>  |h| > rd_half(thr)
  // Small planes: csplit subsets of the threads share the pixel groups, each
  // taking every csplit-th channel (their partial bits meet in the atomicOr).
  const int csplit = ngrp >= (int)blockDim.x ? 1 : max(1, min(4, (int)blockDim.x / ngrp));
  const int tpc = ngrp >= (int)blockDim.x ? (int)blockDim.x : ngrp;  // threads per subset
  const int sub = (int)threadIdx.x / tpc;
  for (int grp = (int)threadIdx.x - sub * tpc; sub < csplit && grp < ngrp; grp += tpc) {
    const int px0 = vec ? grp * 8 : grp;
    const int npx = vec ? 8 : 1;
    uint32_t bits[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    // nonzero-pixel mask of the current channel group, folded into bits[]
    // when the group changes (group bits are per GS channels)
    int g_cur = (c0 + sub) / GS;
    uint32_t nzpix = 0;
    auto fold = [&]() {
      if (!nzpix) return;
      const uint32_t gbit = 1u << g_cur;
#pragma unroll
      for (int j = 0; j < 8; ++j) bits[j] |= ((nzpix >> j) & 1u) ? gbit : 0u;
      nzpix = 0;
    };
    for (int c = c0 + sub; c < c1; c += 4 * csplit) {
      uint32_t nzf[4];  // bit j: pixel px0 + j of channel c + u * csplit has |x| > thr
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        nzf[u] = 0u;
        const int ch = c + u * csplit;
        if (ch >= c1) continue;
        const int64_t e0 = base + (int64_t)(ch - c0) * plane + px0;
        if (vec && fmt == CF_FMT_F16) {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(x) + e0));
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const unsigned gt = __hgt2_mask(__habs2(*reinterpret_cast<const __half2*>(&w[k])), thr2);
            nzf[u] |= ((gt & 1u) | ((gt >> 15) & 2u)) << (2 * k);
            if (count) cnt += ((w[k] & 0x7FFFu) != 0) + ((w[k] & 0x7FFF0000u) != 0);
          }
        } else if (vec) {
          float f[8];
          if (fmt == CF_FMT_F32) {
            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(x) + e0);
            const float4 a = __ldg(src), b = __ldg(src + 1);
            f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
            f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
          } else {
            const uint2 q = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(x) + e0));
            const uint8_t* b8 = reinterpret_cast<const uint8_t*>(&q);
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] = (float)b8[j];
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            nzf[u] |= (fabsf(f[j]) > thr ? 1u : 0u) << j;
            if (count) cnt += f[j] != 0.f ? 1ull : 0ull;
          }
        } else {
          const float f = load_any(x, fmt, e0);
          nzf[u] = fabsf(f) > thr ? 1u : 0u;
          if (count) cnt += f != 0.f ? 1ull : 0ull;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int ch = c + u * csplit;
        if (ch >= c1) continue;
        const int g = ch / GS;
        if (g != g_cur) {
          fold();
          g_cur = g;
        }
        nzpix |= nzf[u];
      }
    }
    fold();
    if (sep) {
      for (int j = 0; j < npx; ++j)
        if (bits[j]) atomicOr(&s_pix[px0 + j], bits[j]);
      continue;
    }
    for (int j = 0; j < npx; ++j) {
      if (!bits[j]) continue;
      const int pix = px0 + j;
      const int ih = pix / W, iw = pix - (pix / W) * W;
      const int tr0 = s_row[2 * ih], nr = s_row[2 * ih + 1];
      const int tc0 = s_col[2 * iw], nc = s_col[2 * iw + 1];
      for (int a = 0; a < nr; ++a)
        for (int b = 0; b < nc; ++b) atomicOr(&s_tiles[(tr0 + a) * GW + tc0 + b], bits[j]);
    }
  }
  if (count) {
    for (int off = 16; off; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
    if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(&s_cnt, cnt);
  }
  __syncthreads();
  int32_t* dst = ag_mask + (int64_t)n * GH * GW;
  if (sep) {
    // rows: s_cor[ih][tc] = OR of the pixels of row ih that feed tile column tc
    for (int i = threadIdx.x; i < H * GW; i += blockDim.x) {
      const int ih = i / GW, tc = i - (i / GW) * GW;
      const int o_lo = tc * BW, o_hi = min(W_out - 1, o_lo + BW - 1);
      const int lo = max(0, o_lo * s - p), hi = min(W - 1, o_hi * s - p + k - 1);
      uint32_t acc = 0;
      for (int iw = lo; iw <= hi; ++iw) {
        const int f = s_col[2 * iw], c = s_col[2 * iw + 1];
        if (tc >= f && tc < f + c) acc |= s_pix[ih * W + iw];
      }
      s_cor[i] = acc;
    }
    __syncthreads();
    // columns: tile (th, tc) = OR of s_cor over the input rows feeding tile row th
    for (int i = threadIdx.x; i < GH * GW; i += blockDim.x) {
      const int th = i / GW, tc = i - (i / GW) * GW;
      const int o_lo = th * BH, o_hi = min(H_out - 1, o_lo + BH - 1);
      const int lo = max(0, o_lo * s - p), hi = min(H - 1, o_hi * s - p + k - 1);
      uint32_t acc = 0;
      for (int ih = lo; ih <= hi; ++ih) {
        const int f = s_row[2 * ih], c = s_row[2 * ih + 1];
        if (th >= f && th < f + c) acc |= s_cor[ih * GW + tc];
      }
      if (acc) atomicOr(reinterpret_cast<unsigned int*>(dst + i), acc);
    }
  } else {
    for (int i = threadIdx.x; i < GH * GW; i += blockDim.x)
      if (s_tiles[i]) atomicOr(reinterpret_cast<unsigned int*>(dst + i), s_tiles[i]);
  }
  if (threadIdx.x == 0 && count && s_cnt)
    atomicAdd(reinterpret_cast<unsigned long long*>(nnz), s_cnt);
}

__global__ void prescan_classify_kernel(const int32_t* __restrict__ ag_mask,
                                        int32_t* __restrict__ tile_class, int64_t tiles, int G) {
  const uint32_t all = (G >= 32) ? 0xFFFFFFFFu : ((1u << G) - 1u);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < tiles;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t mk = (uint32_t)ag_mask[i];
    tile_class[i] = (mk == 0) ? 0 : (mk == all ? 2 : 1);
  }
}

// Conv-tile prescan over x[B][H][W][T][Cin_p] fp16, one pass over the input.
// CTA (b, band) streams R consecutive input rows of image b -- one contiguous
// range of R * W * vpp 16-byte vectors -- and ORs every nonzero vector's
// channel-chunk bit into the masks of the tiles whose receptive field holds
// its pixel (input row / column -> tile-range tables), kept for the band's
// tile rows in shared memory and flushed with atomicOr into the zeroed masks.
// When 32 divides the vectors per pixel, a warp-wide load covers one pixel:
// the lanes' bits are OR-reduced and the pixel's tiles updated once.
constexpr int kMaxMapSide = 1024;  // H, W limits of the row / column tables
constexpr int kMaxVpp = 1024;      // vector slots per pixel with a precomputed chunk bit
constexpr int kMaxBandTiles = 2048;
constexpr int kMaxBandPix = 5120;  // pixels of a band with separate chunk bits (R * W)

__global__ void __launch_bounds__(kPrescanThreads)
    prescan_conv_kernel(const __half* __restrict__ x, uint32_t* __restrict__ mask,
                        int64_t* nnz, int T, int B, int H, int W, int Cin_p, int KH, int KW,
                        int s, int p, int Wb, int Hb, int Bb, int n_wt, int n_ht, int chunk,
                        int R, int lvpp) {
  __shared__ uint32_t s_m[kMaxBandTiles];          // masks of the band's tile rows
  __shared__ uint16_t s_row[2 * kMaxMapSide], s_col[2 * kMaxMapSide];  // (first tile, count)
  __shared__ uint32_t s_cbit[kMaxVpp];
  // Separable mode: each band pixel's chunk bits (s_pix) are collected first
  // and every tile mask is then OR-reduced from them by one thread, instead
  // of each pixel OR-ing into the shared masks of all its tiles (same-address
  // atomics from many warps).
  __shared__ uint32_t s_pix[kMaxBandPix];
  __shared__ unsigned long long s_cnt;
  const int n_band = (H + R - 1) / R;
  const int b = blockIdx.x / n_band;
  const int band = blockIdx.x - b * n_band;
  const int r0 = band * R, r1 = min(H, r0 + R);
  const int Ho = (H + 2 * p - KH) / s + 1;
  const int Wo = (W + 2 * p - KW) / s + 1;
  const int vpp = T * Cin_p / 8;  // 16-byte vectors per pixel
  // row / column tables: input index i feeds output indices o with
  // o * s in [i + p - k + 1, i + p], o < n_out -> tiles o / tile
  for (int i = threadIdx.x; i < H + W; i += blockDim.x) {
    const bool is_row = i < H;
    const int pos = is_row ? i : i - H;
    const int n_out = is_row ? Ho : Wo, tb = is_row ? Hb : Wb, k = is_row ? KH : KW;
    int olo = pos + p - k + 1, ohi = pos + p;
    olo = olo <= 0 ? 0 : (olo + s - 1) / s;
    ohi = ohi < 0 ? -1 : min(n_out - 1, ohi / s);
    uint16_t first = 0, cntt = 0;
    if (olo <= ohi) {
      first = (uint16_t)(olo / tb);
      cntt = (uint16_t)(ohi / tb - olo / tb + 1);
    }
    uint16_t* dst = is_row ? s_row + 2 * pos : s_col + 2 * pos;
    dst[0] = first;
    dst[1] = cntt;
  }
  for (int v = threadIdx.x; v < vpp && v < kMaxVpp; v += blockDim.x)
    s_cbit[v] = 1u << (((v * 8) % Cin_p) / chunk);
  if (threadIdx.x == 0) s_cnt = 0;
  __syncthreads();
  // tile rows this band touches
  int th_lo = 1 << 30, th_hi = -1;
  for (int r = r0; r < r1; ++r) {
    if (s_row[2 * r + 1]) {
      th_lo = min(th_lo, (int)s_row[2 * r]);
      th_hi = max(th_hi, (int)s_row[2 * r] + (int)s_row[2 * r + 1] - 1);
    }
  }
  const int n_th = th_hi >= th_lo ? th_hi - th_lo + 1 : 0;
  const bool sep = (r1 - r0) * W <= kMaxBandPix;
  if (sep) {
    for (int i = threadIdx.x; i < (r1 - r0) * W; i += blockDim.x) s_pix[i] = 0;
  } else {
    for (int i = threadIdx.x; i < n_th * n_wt; i += blockDim.x) s_m[i] = 0;
  }
  __syncthreads();
  const bool count = nnz != nullptr;
  unsigned long long cnt = 0;
  const int row_vecs = W * vpp;
  const int nvec = (r1 - r0) * row_vecs;  // < 2^31 (checked on the host)
  const uint4* base = reinterpret_cast<const uint4*>(x) + ((int64_t)b * H + r0) * row_vecs;
  const bool warp_uniform = (vpp % 32) == 0 && vpp <= kMaxVpp;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  // OR `bits` into the masks of every tile pixel (ih, col) feeds
  auto scatter = [&](int ih, int col, uint32_t bits) {
    if (sep) {
      atomicOr(&s_pix[(ih - r0) * W + col], bits);
      return;
    }
    const int tr0 = s_row[2 * ih], nr = s_row[2 * ih + 1];
    const int tc0 = s_col[2 * col], nc = s_col[2 * col + 1];
    for (int a = 0; a < nr; ++a)
      for (int c = 0; c < nc; ++c) atomicOr(&s_m[(tr0 + a - th_lo) * n_wt + tc0 + c], bits);
  };
  if (warp_uniform) {
    // a warp takes two pixels at a time: each lane loads vpp/32 vectors of
    // each (eight loads in flight), ORs their chunk bits, the warp OR-reduces
    // once per pixel and lane 0 updates the pixel's tiles
    const int npix = (r1 - r0) * W, nj = vpp / 32;
    for (int pa = 2 * warp; pa < npix; pa += 2 * nwarps) {
      const int pb = pa + 1;
      const bool hb = pb < npix;
      const uint4* xa = base + (int64_t)pa * vpp + lane;
      const uint4* xb = base + (int64_t)pb * vpp + lane;
      uint32_t ba = 0, bb2 = 0;
      for (int j0 = 0; j0 < nj; j0 += 4) {
        uint4 q[8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const bool ok = j0 + u < nj;
          q[u] = ok ? __ldg(xa + 32 * (j0 + u)) : make_uint4(0u, 0u, 0u, 0u);
          q[4 + u] = (ok && hb) ? __ldg(xb + 32 * (j0 + u)) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint32_t w4[4] = {q[u].x & 0x7FFF7FFFu, q[u].y & 0x7FFF7FFFu,
                                  q[u].z & 0x7FFF7FFFu, q[u].w & 0x7FFF7FFFu};
          if ((w4[0] | w4[1] | w4[2] | w4[3]) == 0) continue;
          const uint32_t cb = s_cbit[lane + 32 * (j0 + (u & 3))];
          if (u < 4) ba |= cb;
          else bb2 |= cb;
          if (count) {
#pragma unroll
            for (int k = 0; k < 4; ++k) cnt += ((w4[k] & 0xFFFFu) != 0) + ((w4[k] >> 16) != 0);
          }
        }
      }
      ba = __reduce_or_sync(0xffffffffu, ba);
      bb2 = __reduce_or_sync(0xffffffffu, bb2);
      if (lane == 0) {
        if (ba) {
          const int rr = pa / W;
          scatter(r0 + rr, pa - rr * W, ba);
        }
        if (hb && bb2) {
          const int rr = pb / W;
          scatter(r0 + rr, pb - rr * W, bb2);
        }
      }
    }
  } else {
    const int step = blockDim.x;
    for (int i0 = threadIdx.x; i0 < nvec; i0 += 8 * step) {
      uint4 q[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * step;
        q[u] = i < nvec ? __ldg(base + i) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * step;
        const uint32_t w4[4] = {q[u].x & 0x7FFF7FFFu, q[u].y & 0x7FFF7FFFu,
                                q[u].z & 0x7FFF7FFFu, q[u].w & 0x7FFF7FFFu};
        if (i >= nvec || (w4[0] | w4[1] | w4[2] | w4[3]) == 0) continue;
        if (count) {
#pragma unroll
          for (int k = 0; k < 4; ++k) cnt += ((w4[k] & 0xFFFFu) != 0) + ((w4[k] >> 16) != 0);
        }
        const int v = lvpp >= 0 ? (i & (vpp - 1)) : i % vpp;
        const uint32_t bits = v < kMaxVpp ? s_cbit[v] : 1u << (((v * 8) % Cin_p) / chunk);
        const int rr = i / row_vecs;
        const int rem = i - rr * row_vecs;
        const int col = lvpp >= 0 ? (rem >> lvpp) : rem / vpp;
        scatter(r0 + rr, col, bits);
      }
    }
  }
  if (count) {
    for (int off = 16; off; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
    if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(&s_cnt, cnt);
  }
  __syncthreads();
  const int bt = b / Bb;
  for (int i = threadIdx.x; i < n_th * n_wt; i += blockDim.x) {
    uint32_t mk;
    if (sep) {
      // tile (th, tw): OR of the band pixels whose tables name it
      const int th = th_lo + i / n_wt, tw = i - (i / n_wt) * n_wt;
      const int oh_lo = th * Hb, oh_hi = min(Ho - 1, oh_lo + Hb - 1);
      const int ow_lo = tw * Wb, ow_hi = min(Wo - 1, ow_lo + Wb - 1);
      const int ih_lo = max(r0, oh_lo * s - p), ih_hi = min(r1 - 1, oh_hi * s - p + KH - 1);
      const int iw_lo = max(0, ow_lo * s - p), iw_hi = min(W - 1, ow_hi * s - p + KW - 1);
      mk = 0;
      for (int ih = ih_lo; ih <= ih_hi; ++ih) {
        const int f = s_row[2 * ih], c = s_row[2 * ih + 1];
        if (th < f || th >= f + c) continue;
        for (int iw = iw_lo; iw <= iw_hi; ++iw) {
          const int fc = s_col[2 * iw], cc = s_col[2 * iw + 1];
          if (tw >= fc && tw < fc + cc) mk |= s_pix[(ih - r0) * W + iw];
        }
      }
    } else {
      mk = s_m[i];
    }
    if (!mk) continue;
    const int th = th_lo + i / n_wt, tw = i - (i / n_wt) * n_wt;
    atomicOr(mask + ((int64_t)bt * n_ht + th) * n_wt + tw, mk);
  }
  if (threadIdx.x == 0 && count && s_cnt)
    atomicAdd(reinterpret_cast<unsigned long long*>(nnz), s_cnt);
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
  if (GH * GW > kMaxTilesPerSample) return fail(CF_ERR_UNSUPPORTED, "too many tiles per sample");
  if (H > 65535 || W > 65535) return fail(CF_ERR_UNSUPPORTED, "map too large");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int rc = check_cuda(cudaMemsetAsync(ag_mask, 0, (size_t)tiles * sizeof(int32_t), s),
                          "zero the masks"))
    return rc;
  const int n_cb = (int)((C + kRefChannelsPerCta - 1) / kRefChannelsPerCta);
  size_t smem = (size_t)GH * GW * 4 + (size_t)(H + W) * 4;
  // separable tile reduction when the plane's pixel bits and the row partials
  // fit 32 KB next to the masks (keeps several CTAs per SM)
  const size_t sep_bytes = (size_t)(H * W + H * GW) * 4;
  const int sep = sep_bytes <= 32 * 1024 ? 1 : 0;
  if (sep) smem += sep_bytes;
  if (smem > 200 * 1024) return fail(CF_ERR_UNSUPPORTED, "prescan tables exceed shared memory");
  static std::atomic<bool> attr_done[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev >= 0 && dev < 64 && !attr_done[dev].load()) {
    // the attribute is a ceiling: raise it once to the largest size allowed above
    if (int rc = check_cuda(cudaFuncSetAttribute(prescan_ref_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 200 * 1024),
                            "cudaFuncSetAttribute(prescan)"))
      return rc;
    attr_done[dev].store(true);
  }
  prescan_ref_kernel<<<(unsigned)(N * n_cb), kPrescanThreads, smem, s>>>(
      x, x_fmt, ag_mask, nnz_out, (int)C, (int)H, (int)W, (int)H_out, (int)W_out, (int)k,
      (int)stride, (int)pad, (int)BH, (int)BW, (int)GS, (int)GH, (int)GW, threshold, sep);
  if (int rc = check_launch("prescan launch")) return rc;
  int64_t blocks = (tiles + 255) / 256;
  if (blocks > 148 * 4) blocks = 148 * 4;
  prescan_classify_kernel<<<(unsigned)blocks, 256, 0, s>>>(ag_mask, tile_class, tiles, (int)G);
  if (int rc = check_launch("prescan classify launch")) return rc;
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
  if (H > kMaxMapSide || W > kMaxMapSide) return fail(CF_ERR_UNSUPPORTED, "map too large for the prescan");
  if ((int64_t)W * T * Cin_p / 8 > (1 << 24)) return fail(CF_ERR_UNSUPPORTED, "rows too long for the prescan");
  const int64_t vpp = T * Cin_p / 8;
  int lvpp = -1;  // log2 of the vectors per pixel when a power of two
  for (int l = 0; l < 31; ++l)
    if ((int64_t)1 << l == vpp) lvpp = l;
  // rows per CTA: ~8K vectors each, but at least two CTAs per SM when possible
  int64_t R = (8192 + W * vpp - 1) / (W * vpp);
  if (R > H) R = H;
  if (R < 1) R = 1;
  while (R > 1 && B * ((H + R - 1) / R) < 2 * 148) R = (R + 1) / 2;
  // the band's tile rows must fit the shared mask array
  while (R > 1 && ((R * stride) / Hb + 3) * (int64_t)n_wt > kMaxBandTiles) R = (R + 1) / 2;
  if ((R * stride / Hb + 3) * (int64_t)n_wt > kMaxBandTiles)
    return fail(CF_ERR_UNSUPPORTED, "too many tile columns for the prescan");
  if (int rc = require_sm100()) return rc;
  if (int rc = check_cuda(cudaMemsetAsync(mask, 0, (size_t)n_mt * sizeof(uint32_t),
                                          static_cast<cudaStream_t>(stream)),
                          "zero the tile masks"))
    return rc;
  const int64_t n_band = (H + R - 1) / R;
  prescan_conv_kernel<<<(unsigned)(B * n_band), kPrescanThreads, 0,
                        static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), mask, nnz_out, (int)T, (int)B, (int)H, (int)W, (int)Cin_p,
      (int)KH, (int)KW, (int)stride, (int)pad, Wb, Hb, Bb, n_wt, n_ht, (int)chunk, (int)R, lvpp);
  return check_launch("prescan_conv launch");
}

}  // extern "C"
