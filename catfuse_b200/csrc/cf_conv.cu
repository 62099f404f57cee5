// cf_conv.cu — fused Conv -> BN -> (residual) -> multi-step LIF on the
// 5th-generation tensor cores (tcgen05, sm_100a).
//
// GEMM view.  Activations live as x[B][H][W][T][Cin_p] (fp16).  One M tile is
// 128 GEMM rows = (128/TP) output pixels x TP time steps, time innermost, so
// all time steps of a pixel sit in TP adjacent TMEM lanes of one warp.  The
// pixel block is a (Wb x Hb x Bb) box of the output map.  N = output
// channels (BN per tile), K = KH*KW taps x Cin_p channels, walked as
// (tap, channel chunk of BK).  For every (tap, chunk) one 5-D TMA load brings
// the shifted input box (zero-filled at the padding, element stride = conv
// stride) and one 2-D TMA load brings the weight slice; BK/16 tcgen05.mma
// (M=128, N=BN, K=16) accumulate into TMEM.
//
// Epilogue.  Four warps read the accumulator from TMEM (tcgen05.ld 32x32b),
// transpose each 32x32 block through shared memory so that a lane owns one
// pixel x (32/TP) channels x all TP steps, apply the BN affine (and a
// pre-LIF residual), run the LIF recurrence over time in registers, and write
// spikes (fp16, optionally combined with a SEW identity) and the final
// membrane.  Neither z nor the per-step v ever reaches global memory.
//
// Warp roles (192 threads, one persistent CTA per SM):
//   warp 0     TMA producer          warp 1     MMA issuer + TMEM owner
//   warps 2-5  epilogue (TMEM lane quarter = warp % 4)
// The accumulator is double-buffered in TMEM so the epilogue of tile i
// overlaps the main loop of tile i+1.
//
// Sparse mode (SparseFlow).  With a per-M-tile mask of active input channel
// chunks, the producer and the MMA issuer walk only the active chunks; a
// zero-mask tile issues no MMA and its epilogue uses acc = 0 (StaticZero per
// tile).  Skipped chunks contribute exact zeros, so sparse and dense results
// are bit-identical.
#include "cf_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>

namespace cf {

// Device error word written by bounded waits that expire.  Nonzero = the site
// code of the first expiry.  Read and cleared by cf_check_device_error.
__device__ int32_t g_dev_error = 0;

namespace {

constexpr int kConvThreads = 192;
constexpr int kEpiRowStride = 36;  // floats per transpose row (bank-conflict free)
constexpr int kEpiBytes = 4 * 32 * kEpiRowStride * 4;
constexpr int kSmemBudget = 220 * 1024;
constexpr int kMaxTP = 8;  // time steps per launch; longer T runs in blocks of 8

struct ConvArgs {
  const float* scale;
  const float* shift;
  const __half* identity;
  const float* v_in;
  float* v_out;
  __half* out;
  const uint32_t* tile_mask;
  int T;        // total time steps (layout stride)
  int t0;       // first step of this launch
  int tcount;   // steps in this launch (<= TP)
  int B, Ho, Wo, Cout, Cin_p;
  int KH, KW, stride, pad;
  int Wb, Hb, Bb;
  int n_wt, n_ht, n_mtiles, n_ntiles, n_tiles;
  int n_kc;         // channel chunks per tap
  uint32_t kc_all;  // mask with n_kc low bits set
  int res_mode;
  int stages;
  LifParams lp;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, int32_t site,
                                              volatile int* abort_flag) {
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort_flag) return false;
  }
  atomicCAS(&g_dev_error, 0, site);
  *abort_flag = 1;
  return false;
}

__device__ __forceinline__ uint32_t tile_kmask(const ConvArgs& a, int mt) {
  return a.tile_mask ? (__ldg(a.tile_mask + mt) & a.kc_all) : a.kc_all;
}

template <int BN, int BK, int TP>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_bn_lif_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB, const ConvArgs a) {
  constexpr int A_BYTES = 128 * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr int ROWB = BK * 2;  // bytes per operand row = swizzle width
  constexpr int CW = 32 / TP;   // channels per lane after the transpose
  constexpr int PPW = 32 / TP;  // pixels per warp
  constexpr uint32_t TMEM_COLS = (2 * BN < 32) ? 32 : 2 * BN;
  constexpr uint32_t IDESC = make_idesc_f16(128, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int S = a.stages;
  uint8_t* sA = smem;
  uint8_t* sB = sA + (size_t)S * A_BYTES;
  float* sEpi = reinterpret_cast<float*>(sB + (size_t)S * B_BYTES);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sEpi) + kEpiBytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull_bar = empty_bar + S;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* done_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 4);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < a.n_tiles && ok; tile += gridDim.x) {
        const int mt = tile / a.n_ntiles;
        const int nt = tile - mt * a.n_ntiles;
        const int wt = mt % a.n_wt;
        const int ht = (mt / a.n_wt) % a.n_ht;
        const int bt = mt / (a.n_wt * a.n_ht);
        const int wi0 = wt * a.Wb * a.stride - a.pad;
        const int hi0 = ht * a.Hb * a.stride - a.pad;
        const int b0 = bt * a.Bb;
        const uint32_t km = tile_kmask(a, mt);
        if (km == 0) continue;
        for (int kh = 0; kh < a.KH && ok; ++kh) {
          for (int kw = 0; kw < a.KW && ok; ++kw) {
            const int tap = kh * a.KW + kw;
            for (int kc = 0; kc < a.n_kc; ++kc) {
              if (!((km >> kc) & 1u)) continue;
              if (!wait_or_abort(&empty_bar[stage], phase ^ 1u, ERR_SITE_PRODUCER_EMPTY,
                                 abort_flag)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&full_bar[stage], A_BYTES + B_BYTES);
              tma_load_5d(sA + (size_t)stage * A_BYTES, &tmA, &full_bar[stage], kc * BK, a.t0,
                          wi0 + kw, hi0 + kh, b0);
              tma_load_2d(sB + (size_t)stage * B_BYTES, &tmB, &full_bar[stage],
                          tap * a.Cin_p + kc * BK, nt * BN);
              ++issued;
              if (++stage == S) {
                stage = 0;
                phase ^= 1u;
              }
            }
          }
        }
      }
      // Drain: wait (bounded) until the last loads issued have landed so no
      // bulk copy is still writing this CTA's shared memory when it exits.
      const uint32_t outstanding = issued < (uint32_t)S ? issued : (uint32_t)S;
      for (uint32_t i = 0; i < outstanding; ++i) {
        if (stage == 0) {
          stage = S - 1;
          phase ^= 1u;
        } else {
          --stage;
        }
        for (uint32_t p = 0; p < kMaxPolls; ++p)
          if (mbar_try_wait(&full_bar[stage], phase)) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < a.n_tiles && ok; tile += gridDim.x) {
        const int mt = tile / a.n_ntiles;
        const uint32_t km = tile_kmask(a, mt);
        const int count = a.KH * a.KW * __popc(km);
        if (!wait_or_abort(&tempty_bar[acc], acc_phase ^ 1u, ERR_SITE_MMA_TEMPTY, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (count == 0) {
          mbar_arrive(&tfull_bar[acc]);
        } else {
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
          for (int i = 0; i < count; ++i) {
            if (!wait_or_abort(&full_bar[stage], phase, ERR_SITE_MMA_FULL, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(sA + (size_t)stage * A_BYTES);
            const uint32_t b_base = smem_u32(sB + (size_t)stage * B_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              umma_f16(d_tmem, make_smem_desc(a_base + kk * 32, ROWB),
                       make_smem_desc(b_base + kk * 32, ROWB), IDESC, (i | kk) != 0 ? 1u : 0u);
            }
            umma_commit(&empty_bar[stage]);
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(&tfull_bar[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // All MMAs of this thread must retire before TMEM is released.
      umma_commit(done_bar);
      for (uint32_t p = 0; p < kMaxPolls; ++p)
        if (mbar_try_wait(done_bar, 0)) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter of this warp
    float* epi = sEpi + q * 32 * kEpiRowStride;
    const int pp = lane / TP;       // pixel of this lane within the warp's rows
    const int cs = lane - pp * TP;  // channel sub-block of this lane
    const int pix_in_tile = q * PPW + pp;
    const int wb = pix_in_tile % a.Wb;
    const int hb = (pix_in_tile / a.Wb) % a.Hb;
    const int bb = pix_in_tile / (a.Wb * a.Hb);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x) {
      const int mt = tile / a.n_ntiles;
      const int nt = tile - mt * a.n_ntiles;
      const int wt = mt % a.n_wt;
      const int ht = (mt / a.n_wt) % a.n_ht;
      const int bt = mt / (a.n_wt * a.n_ht);
      const bool has_acc = tile_kmask(a, mt) != 0;
      if (!wait_or_abort(&tfull_bar[acc], acc_phase, ERR_SITE_EPI_TFULL, abort_flag)) break;
      tc_fence_after();

      const int wo = wt * a.Wb + wb;
      const int ho = ht * a.Hb + hb;
      const int b = bt * a.Bb + bb;
      const bool pix_ok = (wo < a.Wo) && (ho < a.Ho) && (b < a.B);
      const int64_t pix = ((int64_t)b * a.Ho + ho) * a.Wo + wo;

#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        float r[32];
        if (has_acc) {
          tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + ch * 32), r);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0.f;
        }
        if (ch == BN / 32 - 1) {
          // Accumulator fully read: hand the TMEM buffer back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[acc]);
        }
        // Transpose the 32(rows) x 32(cols) block through shared memory.
        float4* row4 = reinterpret_cast<float4*>(epi + lane * kEpiRowStride);
#pragma unroll
        for (int j = 0; j < 8; ++j) row4[j] = make_float4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
        __syncwarp();

        const int col0 = nt * BN + ch * 32 + cs * CW;
        float sc[CW], sh[CW], v[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          sc[j] = a.scale ? __ldg(a.scale + col0 + j) : 1.f;
          sh[j] = a.shift ? __ldg(a.shift + col0 + j) : 0.f;
        }
        if (a.v_in && pix_ok) {
          const float4* vp = reinterpret_cast<const float4*>(a.v_in + pix * a.Cout + col0);
#pragma unroll
          for (int j = 0; j < CW / 4; ++j) {
            const float4 t4 = vp[j];
            v[4 * j] = t4.x; v[4 * j + 1] = t4.y; v[4 * j + 2] = t4.z; v[4 * j + 3] = t4.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < CW; ++j) v[j] = 0.f;
        }

#pragma unroll
        for (int t = 0; t < TP; ++t) {
          if (t < a.tcount) {
            float z[CW];
            const float4* src =
                reinterpret_cast<const float4*>(epi + (pp * TP + t) * kEpiRowStride + cs * CW);
#pragma unroll
            for (int j = 0; j < CW / 4; ++j) {
              const float4 t4 = src[j];
              z[4 * j] = t4.x; z[4 * j + 1] = t4.y; z[4 * j + 2] = t4.z; z[4 * j + 3] = t4.w;
            }
            const int64_t row = (pix * a.T + a.t0 + t) * a.Cout + col0;
            float idv[CW];
            if (a.res_mode != CF_RES_NONE && a.res_mode != CF_RES_Z_ONLY && pix_ok) {
              const __half2* ip = reinterpret_cast<const __half2*>(a.identity + row);
#pragma unroll
              for (int j = 0; j < CW / 2; ++j) {
                const float2 f = __half22float2(ip[j]);
                idv[2 * j] = f.x; idv[2 * j + 1] = f.y;
              }
            } else {
#pragma unroll
              for (int j = 0; j < CW; ++j) idv[j] = 0.f;
            }
            __half2 o[CW / 2];
#pragma unroll
            for (int j = 0; j < CW; j += 2) {
              float zz0 = __fadd_rn(__fmul_rn(z[j], sc[j]), sh[j]);
              float zz1 = __fadd_rn(__fmul_rn(z[j + 1], sc[j + 1]), sh[j + 1]);
              if (a.res_mode == CF_RES_ADD_PRE) {
                zz0 = __fadd_rn(zz0, idv[j]);
                zz1 = __fadd_rn(zz1, idv[j + 1]);
              }
              if (a.res_mode == CF_RES_Z_ONLY) {
                o[j / 2] = __floats2half2_rn(zz0, zz1);
                continue;
              }
              float s0 = lif_step(v[j], zz0, a.lp);
              float s1 = lif_step(v[j + 1], zz1, a.lp);
              if (a.res_mode == CF_RES_ADD_POST) {
                s0 += idv[j]; s1 += idv[j + 1];
              } else if (a.res_mode == CF_RES_AND_POST) {
                s0 *= idv[j]; s1 *= idv[j + 1];
              } else if (a.res_mode == CF_RES_IAND_POST) {
                s0 = idv[j] * (1.f - s0); s1 = idv[j + 1] * (1.f - s1);
              }
              o[j / 2] = __floats2half2_rn(s0, s1);
            }
            if (pix_ok) {
              if constexpr (CW >= 8) {
                uint4* dst = reinterpret_cast<uint4*>(a.out + row);
#pragma unroll
                for (int j = 0; j < CW / 8; ++j) dst[j] = reinterpret_cast<const uint4*>(o)[j];
              } else if constexpr (CW == 4) {
                *reinterpret_cast<uint2*>(a.out + row) = *reinterpret_cast<const uint2*>(o);
              } else {
                *reinterpret_cast<uint32_t*>(a.out + row) = *reinterpret_cast<const uint32_t*>(o);
              }
            }
          }
        }
        if (a.v_out && pix_ok && a.res_mode != CF_RES_Z_ONLY) {
          float4* vp = reinterpret_cast<float4*>(a.v_out + pix * a.Cout + col0);
#pragma unroll
          for (int j = 0; j < CW / 4; ++j)
            vp[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        __syncwarp();  // transpose buffer is reused by the next chunk
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// --------------------------------------------------------------------------
// host side
// --------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

CUtensorMapSwizzle swizzle_for(int row_bytes) {
  return row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : (row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

int next_pow2(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

struct Geometry {
  int TP, Wb, Hb, Bb, n_wt, n_ht, n_bt, n_mtiles, BN, BK, n_kc;
};

// Choose the pixel box (Wb x Hb x Bb = 128/TP, powers of two) that wastes the
// fewest padded output pixels; ties go to the wider box (longer contiguous
// rows for the output stores).
void choose_box(int P, int B, int Ho, int Wo, int stride, Geometry& g) {
  long best = -1;
  for (int wb = 1; wb <= P; wb <<= 1) {
    if (wb * stride > 256) break;
    for (int hb = 1; wb * hb <= P; hb <<= 1) {
      if (hb * stride > 256) break;
      const int bb = P / (wb * hb);
      if (bb > 256) continue;
      const long nwt = (Wo + wb - 1) / wb, nht = (Ho + hb - 1) / hb, nbt = (B + bb - 1) / bb;
      const long cost = nwt * nht * nbt;
      if (best < 0 || cost < best || (cost == best && wb > g.Wb)) {
        best = cost;
        g.Wb = wb; g.Hb = hb; g.Bb = bb;
        g.n_wt = (int)nwt; g.n_ht = (int)nht; g.n_bt = (int)nbt;
      }
    }
  }
  g.n_mtiles = g.n_wt * g.n_ht * g.n_bt;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int choose_bn(int Cout, int n_mtiles) {
  int bn = 128;
  while (bn > 32 && (Cout % bn != 0)) bn >>= 1;
  if (Cout % bn != 0) return 0;
  // Prefer more, smaller tiles while the grid would not fill the SMs.
  const int sms = 148;
  while (bn > 64 && (long)n_mtiles * (Cout / bn) < sms) bn >>= 1;
  return bn;
}

int choose_bk(int Cin_p, bool sparse) {
  if (sparse && Cin_p > 128 && Cin_p % 32 == 0) return 32;
  if (Cin_p % 64 == 0) return 64;
  if (Cin_p % 32 == 0) return 32;
  return 16;
}

int make_geometry(int64_t T, int64_t B, int64_t Ho, int64_t Wo, int64_t Cout, int64_t Cin_p,
                  int64_t stride, bool sparse, Geometry& g) {
  const int tc = (int)(T < kMaxTP ? T : kMaxTP);
  g.TP = next_pow2(tc);
  choose_box(128 / g.TP, (int)B, (int)Ho, (int)Wo, (int)stride, g);
  g.BN = choose_bn((int)Cout, g.n_mtiles);
  g.BK = choose_bk((int)Cin_p, sparse);
  g.n_kc = (int)(Cin_p / g.BK);
  return g.BN ? CF_OK : fail(CF_ERR_UNSUPPORTED, "Cout=%lld must be a multiple of 32", (long long)Cout);
}

template <int BN, int BK, int TP>
int launch_inst(const CUtensorMap& tmA, const CUtensorMap& tmB, ConvArgs args, int grid,
                cudaStream_t stream) {
  constexpr int A_BYTES = 128 * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  const int fixed = 1024 + kEpiBytes + 256;
  int stages = (kSmemBudget - fixed) / (A_BYTES + B_BYTES);
  if (stages > 8) stages = 8;
  if (stages < 2) return fail(CF_ERR_UNSUPPORTED, "conv tile does not fit shared memory");
  args.stages = stages;
  int smem = fixed + stages * (A_BYTES + B_BYTES);
  // Keep every TMEM-using CTA above half the SM's shared memory so that two
  // of them can never be co-resident and contend for TMEM columns.
  if (smem < 120 * 1024) smem = 120 * 1024;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(conv_bn_lif_kernel<BN, BK, TP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(conv)");
    attr_set = true;
  }
  conv_bn_lif_kernel<BN, BK, TP><<<grid, kConvThreads, smem, stream>>>(tmA, tmB, args);
  return check_launch("conv_bn_lif launch");
}

template <int BN, int BK>
int dispatch_tp(int TP, const CUtensorMap& A, const CUtensorMap& W, const ConvArgs& args, int grid,
                cudaStream_t s) {
  switch (TP) {
    case 1: return launch_inst<BN, BK, 1>(A, W, args, grid, s);
    case 2: return launch_inst<BN, BK, 2>(A, W, args, grid, s);
    case 4: return launch_inst<BN, BK, 4>(A, W, args, grid, s);
    default: return launch_inst<BN, BK, 8>(A, W, args, grid, s);
  }
}

template <int BN>
int dispatch_bk(int BK, int TP, const CUtensorMap& A, const CUtensorMap& W, const ConvArgs& args,
                int grid, cudaStream_t s) {
  switch (BK) {
    case 16: return dispatch_tp<BN, 16>(TP, A, W, args, grid, s);
    case 32: return dispatch_tp<BN, 32>(TP, A, W, args, grid, s);
    default: return dispatch_tp<BN, 64>(TP, A, W, args, grid, s);
  }
}

int dispatch(const Geometry& g, const CUtensorMap& A, const CUtensorMap& W, const ConvArgs& args,
             int grid, cudaStream_t s) {
  switch (g.BN) {
    case 32: return dispatch_bk<32>(g.BK, g.TP, A, W, args, grid, s);
    case 64: return dispatch_bk<64>(g.BK, g.TP, A, W, args, grid, s);
    case 128: return dispatch_bk<128>(g.BK, g.TP, A, W, args, grid, s);
    default: return dispatch_bk<256>(g.BK, g.TP, A, W, args, grid, s);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

// Shared with cf_prescan.cu: the geometry the conv kernel will use.
int conv_geometry_for(int64_t T, int64_t B, int64_t Ho, int64_t Wo, int64_t Cout, int64_t Cin_p,
                      int64_t stride, bool sparse, int* TP, int* Wb, int* Hb, int* Bb,
                      int* n_wt, int* n_ht, int* n_mtiles, int* BK) {
  Geometry g{};
  int rc = make_geometry(T, B, Ho, Wo, Cout, Cin_p, stride, sparse, g);
  if (rc) return rc;
  *TP = g.TP; *Wb = g.Wb; *Hb = g.Hb; *Bb = g.Bb;
  *n_wt = g.n_wt; *n_ht = g.n_ht; *n_mtiles = g.n_mtiles; *BK = g.BK;
  return CF_OK;
}

int conv_bn_lif_impl(const void* x, const void* wp, const float* scale, const float* shift,
                     const void* identity, int res_mode, const float* v_in, float* v_out,
                     void* out, const uint32_t* tile_mask, int64_t T, int64_t B, int64_t H,
                     int64_t W, int64_t Cin_p, int64_t Cout, int64_t KH, int64_t KW,
                     int64_t stride, int64_t pad, float tau, float v_th, float v_reset,
                     int hard_reset, int decay_input, cudaStream_t stream) {
  if (!x || !wp || !out) return fail(CF_ERR_INVALID_ARG, "x, wp and out must not be NULL");
  if (T <= 0 || B <= 0 || H <= 0 || W <= 0 || Cin_p <= 0 || Cout <= 0 || KH <= 0 || KW <= 0 ||
      stride <= 0 || pad < 0)
    return fail(CF_ERR_INVALID_ARG, "non-positive size");
  if (Cin_p % 16) return fail(CF_ERR_UNSUPPORTED, "Cin_p must be a multiple of 16");
  if (Cout % 32) return fail(CF_ERR_UNSUPPORTED, "Cout must be a multiple of 32");
  if (stride > 8) return fail(CF_ERR_UNSUPPORTED, "stride must be <= 8");
  if (res_mode < CF_RES_NONE || res_mode > CF_RES_Z_ONLY)
    return fail(CF_ERR_INVALID_ARG, "bad residual mode %d", res_mode);
  if (res_mode != CF_RES_NONE && res_mode != CF_RES_Z_ONLY && !identity)
    return fail(CF_ERR_INVALID_ARG, "residual mode needs an identity tensor");
  if (!(tau > 0.f)) return fail(CF_ERR_INVALID_ARG, "tau must be > 0");
  if (T > kMaxTP && !v_out && res_mode != CF_RES_Z_ONLY)
    return fail(CF_ERR_INVALID_ARG,
                "T > %d runs in time blocks and needs v_out to carry the membrane", kMaxTP);
  const void* ptrs16[] = {x, wp, identity, v_in, v_out, out};
  for (const void* p : ptrs16)
    if (p && !al16(p)) return fail(CF_ERR_UNSUPPORTED, "tensor pointers must be 16-byte aligned");
  const int64_t Ho = (H + 2 * pad - KH) / stride + 1;
  const int64_t Wo = (W + 2 * pad - KW) / stride + 1;
  if (Ho <= 0 || Wo <= 0) return fail(CF_ERR_INVALID_ARG, "empty output map");
  if (B * Ho * Wo * T * Cout >= (int64_t)1 << 40) return fail(CF_ERR_UNSUPPORTED, "tensor too large");
  if (int rc = require_sm100()) return rc;

  Geometry g{};
  if (int rc = make_geometry(T, B, Ho, Wo, Cout, Cin_p, stride, tile_mask != nullptr, g)) return rc;
  if (tile_mask && g.n_kc > 32)
    return fail(CF_ERR_UNSUPPORTED, "sparse mode supports at most 32 channel chunks");

  auto encode = get_encode_fn();
  if (!encode) return fail(CF_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");

  // A: x[B][H][W][T][Cin_p] fp16, 5-D, box (BK, TP, Wb*s, Hb*s, Bb) with
  // element stride s along W and H (the TMA then loads Wb x Hb elements).
  CUtensorMap tmA, tmB;
  {
    cuuint64_t dims[5] = {(cuuint64_t)Cin_p, (cuuint64_t)T, (cuuint64_t)W, (cuuint64_t)H,
                          (cuuint64_t)B};
    cuuint64_t strides[4] = {(cuuint64_t)(Cin_p * 2), (cuuint64_t)(T * Cin_p * 2),
                             (cuuint64_t)(W * T * Cin_p * 2), (cuuint64_t)(H * W * T * Cin_p * 2)};
    cuuint32_t box[5] = {(cuuint32_t)g.BK, (cuuint32_t)g.TP, (cuuint32_t)(g.Wb * stride),
                         (cuuint32_t)(g.Hb * stride), (cuuint32_t)g.Bb};
    cuuint32_t estr[5] = {1, 1, (cuuint32_t)stride, (cuuint32_t)stride, 1};
    CUresult r = encode(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(x), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(g.BK * 2),
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CF_ERR_CUDA, "tensor map (activations) failed: %d", (int)r);
  }
  {
    const int64_t K = KH * KW * Cin_p;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)Cout};
    cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
    cuuint32_t box[2] = {(cuuint32_t)g.BK, (cuuint32_t)g.BN};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(wp), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(g.BK * 2),
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CF_ERR_CUDA, "tensor map (weights) failed: %d", (int)r);
  }

  ConvArgs args{};
  args.scale = scale;
  args.shift = shift;
  args.identity = static_cast<const __half*>(identity);
  args.out = static_cast<__half*>(out);
  args.tile_mask = tile_mask;
  args.T = (int)T;
  args.B = (int)B; args.Ho = (int)Ho; args.Wo = (int)Wo;
  args.Cout = (int)Cout; args.Cin_p = (int)Cin_p;
  args.KH = (int)KH; args.KW = (int)KW; args.stride = (int)stride; args.pad = (int)pad;
  args.Wb = g.Wb; args.Hb = g.Hb; args.Bb = g.Bb;
  args.n_wt = g.n_wt; args.n_ht = g.n_ht; args.n_mtiles = g.n_mtiles;
  args.n_ntiles = (int)(Cout / g.BN);
  args.n_tiles = args.n_mtiles * args.n_ntiles;
  args.n_kc = g.n_kc;
  args.kc_all = g.n_kc >= 32 ? 0xFFFFFFFFu : ((1u << g.n_kc) - 1u);
  args.res_mode = res_mode;
  args.lp = make_lif(tau, v_th, v_reset, hard_reset, decay_input);
  const int grid = args.n_tiles < sm_count() ? args.n_tiles : sm_count();

  for (int64_t t0 = 0; t0 < T; t0 += kMaxTP) {
    args.t0 = (int)t0;
    args.tcount = (int)((T - t0) < kMaxTP ? (T - t0) : kMaxTP);
    args.v_in = (t0 == 0) ? v_in : v_out;
    args.v_out = v_out;
    if (int rc = dispatch(g, tmA, tmB, args, grid, stream)) return rc;
  }
  return CF_OK;
}

}  // namespace cf

using namespace cf;

extern "C" {

int cf_check_device_error(void* stream, int32_t* code) {
  int32_t v = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaMemcpyFromSymbolAsync(&v, g_dev_error, sizeof(v), 0,
                                                cudaMemcpyDeviceToHost, s),
                      "read device error word");
  if (rc) return rc;
  rc = check_cuda(cudaStreamSynchronize(s), "synchronize for device error word");
  if (rc) return rc;
  if (code) *code = v;
  if (v != 0) {
    const int32_t zero = 0;
    cudaMemcpyToSymbolAsync(g_dev_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
    return fail(CF_ERR_DEVICE_TIMEOUT, "a bounded device-side wait expired (site %d)", v);
  }
  return CF_OK;
}

int cf_conv_geometry(int64_t T, int64_t B, int64_t Ho, int64_t Wo, int64_t Cout, int32_t* out6) {
  if (!out6 || T <= 0 || B <= 0 || Ho <= 0 || Wo <= 0 || Cout <= 0)
    return fail(CF_ERR_INVALID_ARG, "bad geometry query");
  Geometry g{};
  if (int rc = make_geometry(T, B, Ho, Wo, Cout, 64, 1, false, g)) return rc;
  out6[0] = g.TP; out6[1] = g.Wb; out6[2] = g.Hb; out6[3] = g.Bb;
  out6[4] = g.n_mtiles; out6[5] = g.BN;
  return CF_OK;
}

int cf_conv_chunk(int64_t Cin_p, int sparse) {
  if (Cin_p <= 0 || Cin_p % 16) return fail(CF_ERR_INVALID_ARG, "Cin_p must be a positive multiple of 16");
  return choose_bk((int)Cin_p, sparse != 0);
}

int cf_conv_bn_lif(const void* x, const void* wp, const float* scale, const float* shift,
                   const void* identity, int res_mode, const float* v_in, float* v_out, void* out,
                   const uint32_t* tile_mask, int64_t T, int64_t B, int64_t H, int64_t W,
                   int64_t Cin_p, int64_t Cout, int64_t KH, int64_t KW, int64_t stride,
                   int64_t pad, float tau, float v_threshold, float v_reset, int hard_reset,
                   int decay_input, void* stream) {
  return conv_bn_lif_impl(x, wp, scale, shift, identity, res_mode, v_in, v_out, out, tile_mask, T,
                          B, H, W, Cin_p, Cout, KH, KW, stride, pad, tau, v_threshold, v_reset,
                          hard_reset, decay_input, static_cast<cudaStream_t>(stream));
}

int cf_linear_bn_lif(const void* x, const void* w, const float* scale, const float* shift,
                     const void* identity, int res_mode, const float* v_in, float* v_out,
                     void* out, int64_t T, int64_t B, int64_t L, int64_t Cin_p, int64_t Cout,
                     float tau, float v_threshold, float v_reset, int hard_reset, int decay_input,
                     void* stream) {
  // Tokens are pixels of an L x 1 map: a 1x1 convolution.
  return conv_bn_lif_impl(x, w, scale, shift, identity, res_mode, v_in, v_out, out, nullptr, T, B,
                          L, 1, Cin_p, Cout, 1, 1, 1, 0, tau, v_threshold, v_reset, hard_reset,
                          decay_input, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
