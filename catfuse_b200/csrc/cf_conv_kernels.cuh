// cf_conv_kernels.cuh — the fused Conv -> BN -> (residual) -> multi-step LIF
// kernels on the 5th-generation tensor cores (tcgen05, sm_100a) and their
// launch templates.  Included by cf_conv.cu (host side: geometry, tensor maps,
// C ABI) and by cf_conv_tp{1,2,4,8}.cu, which each instantiate the kernels of
// one time-block width so the library builds in parallel.
//
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
// Warp roles (416 threads, one persistent CTA per SM):
//   warps 0-3   TMA producers (a TMA instruction occupies its issuing thread
//               for hundreds of cycles, so four threads issue in parallel)
//   warp 4      MMA issuer + TMEM owner
//   warps 5-12  epilogue (TMEM lane quarter = warp % 4, two warps per quarter)
// The accumulator is double-buffered in TMEM so the epilogue of tile i
// overlaps the main loop of tile i+1.
//
// Sparse mode (SparseFlow).  With a per-M-tile mask of active input channel
// chunks, the producer and the MMA issuer walk only the active chunks; a
// zero-mask tile issues no MMA and its epilogue uses acc = 0 (StaticZero per
// tile).  Skipped chunks contribute exact zeros, so sparse and dense results
// are bit-identical.
#pragma once

#include "cf_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <atomic>

namespace cf {
namespace convk {


constexpr int kProdWarps = 4;  // a TMA instruction holds its issuing thread for ~400 cycles
constexpr int kMmaWarp = kProdWarps;
constexpr int kEpiWarp0 = kProdWarps + 1;
constexpr int kEpiWarps = 8;   // two warps per TMEM lane quarter
constexpr int kConvThreads = 32 * (kProdWarps + 1 + kEpiWarps);
constexpr int kEpiRowStride = 36;  // floats per transpose row (bank-conflict free)
constexpr int kEpiBytes = kEpiWarps * 32 * kEpiRowStride * 4;
// Channel-major kernel: two epilogue warps per TMEM lane quarter (a third
// one measured no faster and lowers the register cap below what the
// residual epilogues need).
constexpr int kTEpiWarps = 8;
constexpr int kTSmemBudget = 227 * 1024;  // the whole opt-in shared memory of a CTA
constexpr int kTThreads = 32 * (kProdWarps + 1 + kTEpiWarps);
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
  // dual output (channel-major kernel): channels [co_split, Cout) go to out2 /
  // v_in2 / v_out2 (a second conv sharing the input and the LIF parameters);
  // co_split = Cout for single-output launches
  __half* out2;
  const float* v_in2;
  float* v_out2;
  int co_split;
  int T;        // total time steps (layout stride)
  int t0;       // first step of this launch
  int tcount;   // steps in this launch (<= TP)
  int B, Ho, Wo, Cout, Cin_p;
  int Cin_w;        // weight channels per tap: wparts * Cin_p
  int wparts;       // weight parts per tap: 1 (fp16), 2 (hi, lo) or 3 (integer digit planes)
  int n_kx;         // activation channel chunks per tap (n_kc / wparts)
  int nplanes;      // channel-major: separate accumulators (1, or 3 for integer weight planes)
  int nbuf;         // channel-major: accumulator buffers in TMEM (2 = double-buffered, or 1)
  int KH, KW, stride, pad;
  int Wb, Hb, Bb;
  int n_wt, n_ht, n_mtiles, n_ntiles, n_tiles;
  int BN, BK;       // N tile (output channels), K chunk (input channels)
  int n_kc;         // channel chunks per tap
  uint32_t kc_all;  // mask with n_kc low bits set
  uint32_t idesc;   // tcgen05 instruction descriptor (M=128, N=BN)
  uint32_t tmem_cols;
  int stages;
  uint32_t max_polls;  // bounded-wait limit (mbarrier polls before a wait gives up)
  int32_t* err;     // device error word (site code of the first expired wait)
  int drop_load;    // test hook: CTA 0's producers skip the first load (the wait for it expires)
  int egd;          // 1: decide on the device whether the tile masks are used (egd_count_active)
  uint32_t egd_max_active;  // most active (tile, chunk) pairs for which the masks run
  int nprod;        // producer threads in use (<= stages)
  int wres;         // 1: the whole weight slab of the (single) N tile stays in shared memory
  int halo;         // 1: one TMA box per tile carries the whole receptive field (all taps)
  int Wh;           // halo box width (Wb + KW - 1)
  int a_bytes;      // bytes of one activation stage
  int backoff;      // ns of sleep between polls for the non-critical waiters
  int tmode;        // 1: channel-major kernel (conv_t_kernel)
  int khbox;        // channel-major: one activation box covers all kh taps of a kw column
  int kwgroup;      // channel-major: one stage carries the KW taps of a kernel row
  int NR;           // channel-major kernel: pixel x time rows per tile (MMA N)
  int MT;           // channel-major kernel: output channels per tile (MMA M), 128 or 64
  int lwb, lhb;     // log2 of Wb and Hb
  LifParams lp;
};

#ifndef CF_SPIN_POLL
#define CF_SPIN_POLL 0
#endif
constexpr bool kSpinPoll = CF_SPIN_POLL;

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, int32_t site,
                                              volatile int* abort_flag, const ConvArgs& a,
                                              int backoff_ns = 0) {
  for (uint32_t i = 0; i < a.max_polls; ++i) {
    if (kSpinPoll ? mbar_test_wait(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort_flag) return false;
    if (backoff_ns) __nanosleep(backoff_ns);
  }
  atomicCAS(a.err, 0, site);
  *abort_flag = 1;
  return false;
}

// Warp-converged variant of wait_or_abort: all 32 lanes poll together (one
// warp-wide try_wait) and a vote keeps the result uniform.  Role loops run on
// whole warps with one lane issuing; a lone polling lane whose 31 siblings
// sit in a warp-sync or block barrier ran its loop several times slower.
__device__ __forceinline__ bool warp_wait_or_abort(uint64_t* bar, uint32_t parity, int32_t site,
                                                   volatile int* abort_flag, const ConvArgs& a,
                                                   int backoff_ns = 0) {
  for (uint32_t i = 0; i < a.max_polls; ++i) {
    const bool done = kSpinPoll ? mbar_test_wait(bar, parity) : mbar_try_wait(bar, parity);
    if (__any_sync(0xffffffffu, done)) return true;
    if ((i & 255u) == 255u && __any_sync(0xffffffffu, *abort_flag != 0)) return false;
    if (backoff_ns) __nanosleep(backoff_ns);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicCAS(a.err, 0, site);
    *abort_flag = 1;
  }
  __syncwarp();
  return false;
}

// Chunk mask of a tile: bit kc = weight chunk kc has work.  Multi-part
// weights walk wparts * n_kx chunks (part 0, then part 1, ...) over the same
// activation chunks, so an activation chunk mask is repeated for every part.
// Sparse launches have at most 32 chunks; dense ones may have more (chunk_on).
__device__ __forceinline__ uint32_t tile_kmask(const ConvArgs& a, int mt, bool use_mask) {
  if (!a.tile_mask || !use_mask) return a.kc_all;
  const uint32_t m = __ldg(a.tile_mask + mt);
  uint32_t r = m;
  for (int p = 1; p < a.wparts; ++p) r |= m << (p * a.n_kx);
  return r & a.kc_all;
}

// Execution-grounded dispatch on the device (egd launches): every CTA sums
// the popcounts of all tile masks (active (tile, chunk) pairs) before the
// pipeline starts and runs the masks only if at most egd_max_active pairs are
// active; otherwise every tile runs every chunk (dense).  Both choices give
// the same result bit for bit (skipped chunks add exact zeros); only the
// speed differs.  `s_active` is the CTA's shared counter, zeroed by the caller.
__device__ __forceinline__ void egd_count_active(const ConvArgs& a, unsigned int* s_active) {
  const uint32_t kx_all = a.n_kx >= 32 ? 0xFFFFFFFFu : ((1u << a.n_kx) - 1u);
  unsigned int c = 0;
  for (int i = threadIdx.x; i < a.n_mtiles; i += blockDim.x)
    c += __popc(__ldg(a.tile_mask + i) & kx_all);
  for (int off = 16; off; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(s_active, c);
}

__device__ __forceinline__ bool chunk_on(uint32_t km, int kc) {
  return kc >= 32 || ((km >> kc) & 1u);
}

// Activation channel chunk read by weight chunk kc (every weight part
// multiplies the same activations).
__device__ __forceinline__ int xchunk(const ConvArgs& a, int kc) {
  return kc >= 2 * a.n_kx ? kc - 2 * a.n_kx : (kc >= a.n_kx ? kc - a.n_kx : kc);
}

// LIF step for the common configuration (decay_input, hard reset to 0, tau a
// power of two).  With v_reset = 0, v - v_reset is v exactly and
// (z - v) * (1/tau) is exact, so the fused multiply-add rounds exactly once,
// like the separately rounded SpikingJelly form.
__device__ __forceinline__ float lif_step_fast(float& v, float z, const LifParams& p) {
  const float h = fmaf(__fsub_rn(z, v), p.rtau, v);
  const bool s = h >= p.v_th;
  v = s ? 0.0f : h;
  return s ? 1.0f : 0.0f;
}

template <bool FAST>
__device__ __forceinline__ float lif_any(float& v, float z, const LifParams& p) {
  if constexpr (FAST) return lif_step_fast(v, z, p);
  else return lif_step(v, z, p);
}

// Epilogue of one 32-row x 32-column accumulator block held (row-major,
// stride kEpiRowStride) in this warp's transpose buffer.  Lane (pp, cs) owns
// pixel pp of the warp and channels [cs*CW, cs*CW+CW) for all TP steps.
template <int TP, int RES, bool FAST>
__device__ __forceinline__ void epi_block(const ConvArgs& a, const float* epi, int pp, int cs,
                                          bool pix_ok, int64_t pix, int col0) {
  constexpr int CW = 32 / TP;
  float sc[CW], sh[CW], v[CW];
#pragma unroll
  for (int j = 0; j < CW; j += 4) {
    const float4 s4 = a.scale ? __ldg(reinterpret_cast<const float4*>(a.scale + col0 + j))
                              : make_float4(1.f, 1.f, 1.f, 1.f);
    const float4 h4 = a.shift ? __ldg(reinterpret_cast<const float4*>(a.shift + col0 + j))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
    sc[j] = s4.x; sc[j + 1] = s4.y; sc[j + 2] = s4.z; sc[j + 3] = s4.w;
    sh[j] = h4.x; sh[j + 1] = h4.y; sh[j + 2] = h4.z; sh[j + 3] = h4.w;
  }
  if (RES != CF_RES_Z_ONLY && a.v_in && pix_ok) {
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
  constexpr bool kIdent = (RES != CF_RES_NONE && RES != CF_RES_Z_ONLY);
  float idv[kIdent ? TP : 1][CW];
  if constexpr (kIdent) {
    // All steps' identity loads are independent: issue them before the recurrence.
#pragma unroll
    for (int t = 0; t < TP; ++t) {
      if (t < a.tcount && pix_ok) {
        const int64_t row = (pix * a.T + a.t0 + t) * a.Cout + col0;
        const __half2* ip = reinterpret_cast<const __half2*>(a.identity + row);
#pragma unroll
        for (int j = 0; j < CW / 2; ++j) {
          const float2 f = __half22float2(ip[j]);
          idv[t][2 * j] = f.x; idv[t][2 * j + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < CW; ++j) idv[t][j] = 0.f;
      }
    }
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
      __half2 o[CW / 2];
#pragma unroll
      for (int j = 0; j < CW; j += 2) {
        float zz0 = fmaf(z[j], sc[j], sh[j]);
        float zz1 = fmaf(z[j + 1], sc[j + 1], sh[j + 1]);
        if constexpr (RES == CF_RES_ADD_PRE) {
          zz0 = __fadd_rn(zz0, idv[t][j]);
          zz1 = __fadd_rn(zz1, idv[t][j + 1]);
        }
        if constexpr (RES == CF_RES_Z_ONLY) {
          o[j / 2] = __floats2half2_rn(zz0, zz1);
        } else {
          float s0 = lif_any<FAST>(v[j], zz0, a.lp);
          float s1 = lif_any<FAST>(v[j + 1], zz1, a.lp);
          if constexpr (RES == CF_RES_ADD_POST) {
            s0 += idv[t][j]; s1 += idv[t][j + 1];
          } else if constexpr (RES == CF_RES_AND_POST) {
            s0 *= idv[t][j]; s1 *= idv[t][j + 1];
          } else if constexpr (RES == CF_RES_IAND_POST) {
            s0 = idv[t][j] * (1.f - s0); s1 = idv[t][j + 1] * (1.f - s1);
          }
          o[j / 2] = __floats2half2_rn(s0, s1);
        }
      }
      if (pix_ok) {
        const int64_t row = (pix * a.T + a.t0 + t) * a.Cout + col0;
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
  if (RES != CF_RES_Z_ONLY && a.v_out && pix_ok) {
    float4* vp = reinterpret_cast<float4*>(a.v_out + pix * a.Cout + col0);
#pragma unroll
    for (int j = 0; j < CW / 4; ++j)
      vp[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

// Issue the KS = BK/16 MMAs of one (tap, channel chunk) back to back.  The
// descriptors advance 32 bytes (2 in the >>4 address field) per K step; the
// base-offset bits (address bits 7-9) are unchanged by that step.  Keeping
// this straight-line, with the commit outside, lets the issuing thread sustain
// one MMA per tensor-core slot; a runtime-bounded loop here issued at less
// than half that rate.
template <int KS>
__device__ __forceinline__ void issue_kchunk(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t first_accum) {
#pragma unroll
  for (int kk = 0; kk < KS; ++kk)
    umma_f16(d_tmem, adesc + 2ull * kk, bdesc + 2ull * kk, idesc, kk == 0 ? first_accum : 1u);
}

template <int TP, int RES, bool FAST>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_bn_lif_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB, const ConvArgs a) {
  constexpr int PPW = 32 / TP;  // pixels per warp
  const int BN = a.BN, BK = a.BK;
  const int A_BYTES = a.a_bytes;
  const int B_BYTES = BN * BK * 2;
  const uint32_t ROWB = (uint32_t)BK * 2;  // bytes per operand row = swizzle width

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int S = a.stages;
  // Weight-resident mode: sB holds all KH*KW*n_kc weight blocks for good and
  // the stages carry only activation tiles.
  const int n_wblk = a.wres ? a.KH * a.KW * a.n_kc : S;
  const int STAGE_B = a.wres ? 0 : B_BYTES;
  uint8_t* sA = smem;
  uint8_t* sB = sA + (size_t)S * A_BYTES;
  float* sEpi = reinterpret_cast<float*>(sB + (size_t)n_wblk * B_BYTES);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sEpi) + kEpiBytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull_bar = empty_bar + S;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* done_bar = tempty_bar + 2;
  uint64_t* w_bar = done_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(w_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // EGD counter: the word after the abort flag (a static __shared__ variable
  // would come out of the 227 KB the dynamic allocation already claims)
  unsigned int* s_active = reinterpret_cast<unsigned int*>(const_cast<int*>(abort_flag) + 1);
  // The tile masks (egd) and the activations come from earlier launches:
  // read nothing of them before the dependency has resolved.
  if (a.egd) griddep_wait();
  if (a.egd) {
    if (threadIdx.x == 0) *s_active = 0;
    __syncthreads();
    egd_count_active(a, s_active);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], kEpiWarps);
    }
    mbar_init(done_bar, 1);
    mbar_init(w_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp < kProdWarps && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Barrier set-up and the TMEM allocation above overlap the previous launch;
  // everything below reads or writes tensors earlier launches produce or use.
  if (!a.egd) griddep_wait();
  griddep_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const bool use_mask = !a.egd || *s_active <= a.egd_max_active;

  if (warp < kProdWarps) {
    // ------------------------------------------------------------ producers
    // Producer p issues the loads of global k-iterations i with i % kProdWarps
    // == p (stage i % S, phase (i / S) & 1); the MMA warp consumes in order.
    if (warp < a.nprod) {
      const int p = warp;
      if (a.wres && p == 0 && lane == 0) {
        // Load the weight slab once: block (tap, kc) at sB + (tap*n_kc + kc)*B_BYTES.
        mbar_arrive_expect_tx(w_bar, (uint32_t)(n_wblk * B_BYTES));
        for (int tap = 0; tap < a.KH * a.KW; ++tap)
          for (int kc = 0; kc < a.n_kc; ++kc)
            tma_load_2d(sB + (size_t)(tap * a.n_kc + kc) * B_BYTES, &tmB, w_bar,
                        tap * a.Cin_w + kc * BK, 0);
      }
      // Schedule counters advance incrementally: runtime-divisor divisions on
      // this single-warp critical path cost more than the loads they issue.
      int owner = 0;            // producer of the next k-iteration (it % nprod)
      int stage = 0;            // its stage (it % S)
      uint32_t phase = 0;       // and phase ((it / S) & 1)
      uint32_t used = 0;        // stages this producer loaded into (bit s)
      uint32_t used_phase = 0;  // phase of its latest load per stage (bit s)
      bool drop_next = a.drop_load && blockIdx.x == 0;  // test hook, see ConvArgs
      const int KHs = a.halo ? 1 : a.KH;  // halo: all taps in one box
      const int KWs = a.halo ? 1 : a.KW;
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
        const uint32_t km = tile_kmask(a, mt, use_mask);
        if (km == 0) continue;
        int tap = 0;
        for (int kh = 0; kh < KHs && ok; ++kh) {
          for (int kw = 0; kw < KWs && ok; ++kw, ++tap) {
            for (int kc = 0; kc < a.n_kc; ++kc) {
              if (!chunk_on(km, kc)) continue;
              const bool mine = owner == p;
              const int my_stage = stage;
              const uint32_t my_phase = phase;
              if (++owner == a.nprod) owner = 0;
              if (++stage == S) {
                stage = 0;
                phase ^= 1u;
              }
              if (!mine) continue;
              if (!warp_wait_or_abort(&empty_bar[my_stage], my_phase ^ 1u,
                                      ERR_SITE_PRODUCER_EMPTY, abort_flag, a,
                                      a.backoff)) {
                ok = false;
                break;
              }
              const bool dropped = drop_next;
              drop_next = false;
              if (lane == 0 && !dropped) {
                mbar_arrive_expect_tx(&full_bar[my_stage], A_BYTES + STAGE_B);
                tma_load_5d(sA + (size_t)my_stage * A_BYTES, &tmA, &full_bar[my_stage],
                            xchunk(a, kc) * BK, a.t0, wi0 + kw, hi0 + kh, b0);
                if (!a.wres)
                  tma_load_2d(sB + (size_t)my_stage * B_BYTES, &tmB, &full_bar[my_stage],
                              tap * a.Cin_w + kc * BK, nt * BN);
              }
              __syncwarp();
              if (!dropped) {
                used |= 1u << my_stage;
                used_phase = (used_phase & ~(1u << my_stage)) | (my_phase << my_stage);
              }
            }
          }
        }
      }
      // On a normal exit every load was consumed by the MMA warp, which
      // finishes before the final barrier.  After an abort, wait (bounded)
      // for this producer's loads so no bulk copy still writes this CTA's
      // shared memory when it exits.
      if (!ok) {
        for (int st = 0; st < S; ++st) {
          if (!((used >> st) & 1u)) continue;
          for (uint32_t q = 0; q < (1u << 16); ++q)
            if (mbar_try_wait(&full_bar[st], (used_phase >> st) & 1u)) break;
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // Lane 0 issues.  tcgen05.mma queues only a few instructions ahead, so
    // everything this thread does between two stages is a bubble in the
    // tensor pipe unless it is shorter than the queued work: descriptors
    // advance by adds, the schedule by compares, and the wait is one
    // try_wait on the common path.
    if (lane == 0) {
      const uint32_t a_step = (uint32_t)A_BYTES >> 4;  // descriptor units (16 B)
      const uint32_t b_step = (uint32_t)B_BYTES >> 4;
      const uint64_t a_desc0 = make_smem_desc(smem_u32(sA), ROWB);
      const uint64_t b_desc0 = make_smem_desc(smem_u32(sB), ROWB);
      // halo: tap (kh, kw) reads the box from row (kh*Wh + kw)*TP
      const uint32_t row_kw = ((uint32_t)TP * ROWB) >> 4;
      const uint32_t row_kh = ((uint32_t)(a.Wh * TP) * ROWB) >> 4;
      const int ksteps = BK / 16;
      const int n_tg = a.halo ? 1 : a.KH * a.KW;
      int stage = 0;
      uint32_t phase = 0;
      uint64_t a_desc = a_desc0;  // descriptor of stage `stage`
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool w_ready = false;
      for (int tile = blockIdx.x; tile < a.n_tiles && ok; tile += gridDim.x) {
        const int mt = tile / a.n_ntiles;
        const uint32_t km = tile_kmask(a, mt, use_mask);
        if (!wait_or_abort(&tempty_bar[acc], acc_phase ^ 1u, ERR_SITE_MMA_TEMPTY, abort_flag, a)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (km == 0) {
          mbar_arrive(&tfull_bar[acc]);
        } else {
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
          if (a.wres && !w_ready) {
            if (!wait_or_abort(w_bar, 0, ERR_SITE_MMA_FULL, abort_flag, a)) {
              ok = false;
              break;
            }
            w_ready = true;
          }
          uint32_t accum = 0u;
          uint64_t b_desc_w = b_desc0;  // weight-resident: block (tg, kc) in order
          for (int tg = 0; tg < n_tg && ok; ++tg) {
            for (int kc = 0; kc < a.n_kc; ++kc) {
              if (a.wres) {
                if (kc) b_desc_w += b_step;
              }
              if (!chunk_on(km, kc)) continue;
              if (!mbar_try_wait(&full_bar[stage], phase) &&
                  !wait_or_abort(&full_bar[stage], phase, ERR_SITE_MMA_FULL, abort_flag, a)) {
                ok = false;
                break;
              }
              // No tcgen05 fence here: the mbarrier completion already orders
              // the TMA writes before the MMA reads.
              {
                if (a.halo) {
                  // All KH*KW taps from this stage's box; weights resident,
                  // block (tap, kc) at tap*n_kc + kc.
                  uint64_t bd = b_desc0 + (uint64_t)((uint32_t)kc * b_step);
                  const uint64_t bstride = (uint64_t)((uint32_t)a.n_kc * b_step);
                  uint64_t ad_row = a_desc;
                  for (int kh = 0; kh < a.KH; ++kh, ad_row += row_kh) {
                    uint64_t ad = ad_row;
                    for (int kw = 0; kw < a.KW; ++kw, ad += row_kw, bd += bstride) {
                      if (ksteps == 4) issue_kchunk<4>(d_tmem, ad, bd, a.idesc, accum);
                      else if (ksteps == 2) issue_kchunk<2>(d_tmem, ad, bd, a.idesc, accum);
                      else issue_kchunk<1>(d_tmem, ad, bd, a.idesc, accum);
                      accum = 1u;
                    }
                  }
                } else {
                  const uint64_t bd =
                      a.wres ? b_desc_w : b_desc0 + (uint64_t)((uint32_t)stage * b_step);
                  if (ksteps == 4) issue_kchunk<4>(d_tmem, a_desc, bd, a.idesc, accum);
                  else if (ksteps == 2) issue_kchunk<2>(d_tmem, a_desc, bd, a.idesc, accum);
                  else issue_kchunk<1>(d_tmem, a_desc, bd, a.idesc, accum);
                  accum = 1u;
                }
              }
              umma_commit(&empty_bar[stage]);
              if (++stage == S) {
                stage = 0;
                phase ^= 1u;
                a_desc = a_desc0;
              } else {
                a_desc += a_step;
              }
            }
            if (a.wres) b_desc_w += b_step;
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
    const int e = warp - kEpiWarp0;  // 0..kEpiWarps-1
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int half = e / 4;          // which 32-column blocks this warp takes
    float* epi = sEpi + e * 32 * kEpiRowStride;
    const int pp = lane / TP;       // pixel of this lane within the warp's rows
    const int cs = lane - pp * TP;  // channel sub-block of this lane
    const int pix_in_tile = q * PPW + pp;
    const int wb = pix_in_tile % a.Wb;
    const int hb = (pix_in_tile / a.Wb) % a.Hb;
    const int bb = pix_in_tile / (a.Wb * a.Hb);
    const int nblk = BN / 32;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x) {
      const int mt = tile / a.n_ntiles;
      const int nt = tile - mt * a.n_ntiles;
      const int wt = mt % a.n_wt;
      const int ht = (mt / a.n_wt) % a.n_ht;
      const int bt = mt / (a.n_wt * a.n_ht);
      const bool has_acc = tile_kmask(a, mt, use_mask) != 0;
      // The whole warp waits for the accumulator (backed off, converged).
      if (!warp_wait_or_abort(&tfull_bar[acc], acc_phase, ERR_SITE_EPI_TFULL, abort_flag,
                              a, a.backoff))
        break;
      tc_fence_after();

      const int wo = wt * a.Wb + wb;
      const int ho = ht * a.Hb + hb;
      const int b = bt * a.Bb + bb;
      const bool pix_ok = (wo < a.Wo) && (ho < a.Ho) && (b < a.B);
      const int64_t pix = ((int64_t)b * a.Ho + ho) * a.Wo + wo;
      // This warp's column blocks are half, half+2, ...; after reading the
      // last of them it releases the accumulator (one arrival per warp).
      int last = -1;
      for (int ch = half; ch < nblk; ch += 2) last = ch;
      if (last < 0) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      }
      for (int ch = half; ch < nblk; ch += 2) {
        float r[32];
        if (has_acc) {
          tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + ch * 32), r);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0.f;
        }
        if (ch == last) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[acc]);
        }
        float4* row4 = reinterpret_cast<float4*>(epi + lane * kEpiRowStride);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          row4[j] = make_float4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
        __syncwarp();
        epi_block<TP, RES, FAST>(a, epi, pp, cs, pix_ok, pix, nt * BN + ch * 32 + cs * (32 / TP));
        __syncwarp();  // transpose buffer is reused by the next block
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, a.tmem_cols);
  }
}


// --------------------------------------------------------------------------
// Channel-major variant (Cout % 128 == 0).  The GEMM roles swap: D[co][row] =
// sum_k W[co][k] X[row][k] with M = 128 output channels (operand A = weight
// tile) and N = NR (256 or 128) pixel x time rows (operand B = activation
// tile).  An M=128, N=256 MMA carries 128 tensor-core cycles of work per
// instruction, twice the N=128 case, so the issuing thread's per-stage
// bookkeeping (barrier wait, commit) hides behind the queued MMAs instead of
// stalling the pipe.  The accumulator lane is the output channel: each
// epilogue thread owns one channel and runs the LIF recurrence of 32/TP
// pixels over TP steps straight from its tcgen05.ld registers, with the BN
// affine as two per-thread scalars and no shared-memory transpose.
// Warp roles and the producer/MMA pipeline are those of conv_bn_lif_kernel.
// --------------------------------------------------------------------------
// Epilogue staging of one warp.  M=128 tiles: 32 rows (pixel-time columns of
// the chunk) x 32 channels, row stride 80 B.  M=64 tiles: two sets (one per
// half-warp) of 32 rows x 16 channels, row stride 48 B, the second set 32 B
// further on so the two half-warps' 2-byte writes hit disjoint banks.
template <int MT>
__device__ __forceinline__ int stage_row_off(int r) {
  if constexpr (MT == 128) return r * 80;
  else return (r >> 5) * (32 * 48 + 32) + (r & 31) * 48;
}
constexpr int kStageBytes = 3200;  // >= max(32 * 80, 2 * (32 * 48 + 32)), 16-B multiple
// Channel-major kernel: 1 KB alignment slack, epilogue staging, up to 2*8+5
// barriers and two words.
constexpr int kTFixedBytes = 1024 + kTEpiWarps * kStageBytes + 256;

// Epilogue of one chunk of the channel-major accumulator.  This lane owns
// channel co (local index cl) and the 32 pixel-time columns cb .. cb+31 with
// cb = col0 (M=128) or col0 + 32 * (lane / 16) (M=64): r[pp*TP + t] = z of
// pixel cb/TP + pp, step t.  The LIF runs in these registers; the fp16
// results go through the staging rows (row = column - col0) so that each lane
// then writes whole (pixel, step) rows of the chunk's channels with 16-byte
// stores.  Post-LIF SEW combines are applied to those rows; the add-before-LIF
// identity comes in the same way in reverse.
template <int TP, int RES, bool FAST, bool FULLT, int MT>
__device__ __forceinline__ void epi_chunk_t(const ConvArgs& a, const float (&r)[32], int co,
                                            int co_base, float sc, float sh, int wt, int ht,
                                            int bt, int col0, uint8_t* stage, int lane) {
  constexpr int PP = 32 / TP;               // pixels per lane
  constexpr int CPR = MT == 128 ? 32 : 16;  // channels per staged row
  constexpr int NQ = CPR / 8;               // 16-byte pieces per row
  constexpr int RL = MT == 128 ? 1 : 2;     // staged rows written out per lane
  constexpr bool kIdent = (RES == CF_RES_ADD_PRE);
  constexpr bool kPost = (RES == CF_RES_ADD_POST || RES == CF_RES_AND_POST ||
                          RES == CF_RES_IAND_POST);
  constexpr bool kLif = (RES != CF_RES_Z_ONLY);
  constexpr bool full_t = FULLT;  // all TP steps valid: straight-line recurrences
  // Dual-output launches: output channels from co_split on belong to a second
  // conv (its own out / v buffers, Cout - co_split channels wide).
  const bool second = co_base >= a.co_split;
  __half* const outp = second ? a.out2 : a.out;
  const float* const vinp = second ? a.v_in2 : a.v_in;
  float* const voutp = second ? a.v_out2 : a.v_out;
  const int cstride = second ? a.Cout - a.co_split : a.co_split;
  const int cbase = second ? co_base - a.co_split : co_base;
  const int cown = second ? co - a.co_split : co;
  const int h = MT == 128 ? 0 : (lane >> 4);
  const int cl = MT == 128 ? lane : (lane & 15);
  const int p0 = (col0 + 32 * h) / TP;

  // Output rows of this lane in the transposed phase: staged row i*32 + lane
  // = column col0 + i*32 + lane.
  int64_t row_off[RL];
  bool rok[RL];
#pragma unroll
  for (int i = 0; i < RL; ++i) {
    const int c = col0 + i * 32 + lane;
    const int p = c / TP, t = c - (c / TP) * TP;
    const int wo = (wt << a.lwb) + (p & ((1 << a.lwb) - 1));
    const int ho = (ht << a.lhb) + ((p >> a.lwb) & ((1 << a.lhb) - 1));
    const int b = bt * a.Bb + (p >> (a.lwb + a.lhb));
    rok[i] = wo < a.Wo && ho < a.Ho && b < a.B && t < a.tcount;
    const int64_t pix = ((int64_t)b * a.Ho + ho) * a.Wo + wo;
    row_off[i] = (pix * a.T + a.t0 + t) * cstride + cbase;
  }

  // Post-LIF combines: fetch this lane's identity rows now so their latency
  // overlaps the recurrence below.
  uint4 idr[kPost ? RL : 1][kPost ? NQ : 1];
  if constexpr (kPost) {
#pragma unroll
    for (int i = 0; i < RL; ++i) {
      const uint4* src = reinterpret_cast<const uint4*>(a.identity + row_off[i]);
#pragma unroll
      for (int k = 0; k < NQ; ++k) idr[i][k] = rok[i] ? src[k] : make_uint4(0u, 0u, 0u, 0u);
    }
  }

  float idv[kIdent ? 32 : 1];
  if constexpr (kIdent) {
#pragma unroll
    for (int i = 0; i < RL; ++i) {
      uint4 q4[NQ];
#pragma unroll
      for (int k = 0; k < NQ; ++k) q4[k] = make_uint4(0u, 0u, 0u, 0u);
      if (rok[i]) {
        const uint4* src = reinterpret_cast<const uint4*>(a.identity + row_off[i]);
#pragma unroll
        for (int k = 0; k < NQ; ++k) q4[k] = src[k];
      }
      uint4* srow = reinterpret_cast<uint4*>(stage + stage_row_off<MT>(i * 32 + lane));
#pragma unroll
      for (int k = 0; k < NQ; ++k) srow[k] = q4[k];
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 32; ++j)
      idv[j] = __half2float(
          *reinterpret_cast<const __half*>(stage + stage_row_off<MT>(h * 32 + j) + cl * 2));
    __syncwarp();
  }

  // Membranes of this lane's channel for its pixels, all issued before any store.
  int64_t pix[PP];
  bool ok[PP];
  float v[PP];
  if ((1 << a.lwb) >= PP) {
    // The lane's pixels are consecutive in one output row.
    const int wo0 = (wt << a.lwb) + (p0 & ((1 << a.lwb) - 1));
    const int ho = (ht << a.lhb) + ((p0 >> a.lwb) & ((1 << a.lhb) - 1));
    const int b = bt * a.Bb + (p0 >> (a.lwb + a.lhb));
    const bool row_ok = ho < a.Ho && b < a.B;
    const int64_t pix0 = ((int64_t)b * a.Ho + ho) * a.Wo + wo0;
#pragma unroll
    for (int pp = 0; pp < PP; ++pp) {
      ok[pp] = row_ok && wo0 + pp < a.Wo;
      pix[pp] = pix0 + pp;
    }
  } else {
#pragma unroll
    for (int pp = 0; pp < PP; ++pp) {
      const int p = p0 + pp;
      const int wo = (wt << a.lwb) + (p & ((1 << a.lwb) - 1));
      const int ho = (ht << a.lhb) + ((p >> a.lwb) & ((1 << a.lhb) - 1));
      const int b = bt * a.Bb + (p >> (a.lwb + a.lhb));
      ok[pp] = wo < a.Wo && ho < a.Ho && b < a.B;
      pix[pp] = ((int64_t)b * a.Ho + ho) * a.Wo + wo;
    }
  }
  if constexpr (kLif) {
#pragma unroll
    for (int pp = 0; pp < PP; ++pp) v[pp] = (vinp && ok[pp]) ? vinp[pix[pp] * cstride + cown] : 0.f;
  }

  uint8_t* hbase = stage + cl * 2;
#pragma unroll
  for (int pp = 0; pp < PP; ++pp) {
    float vv = kLif ? v[pp] : 0.f;
#pragma unroll
    for (int t = 0; t < TP; ++t) {
      const int j = pp * TP + t;
      if (full_t || t < a.tcount) {
        float z = fmaf(r[j], sc, sh);
        float o;
        if constexpr (RES == CF_RES_ADD_PRE) z = __fadd_rn(z, idv[j]);
        __half oh;
        if constexpr (!kLif) {
          o = z;
          oh = __float2half_rn(o);
        } else {
          // a spike is 0 or 1: select its fp16 bits instead of converting
          o = lif_any<FAST>(vv, z, a.lp);
          oh = __ushort_as_half(o != 0.f ? (unsigned short)0x3C00u : (unsigned short)0u);
        }
        *reinterpret_cast<__half*>(hbase + stage_row_off<MT>(h * 32 + j)) = oh;
      }
    }
    if (kLif) v[pp] = vv;
  }
  if constexpr (kLif) {
    if (voutp) {
#pragma unroll
      for (int pp = 0; pp < PP; ++pp)
        if (ok[pp]) voutp[pix[pp] * cstride + cown] = v[pp];
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < RL; ++i) {
    if (!rok[i]) continue;
    const uint4* srow = reinterpret_cast<const uint4*>(stage + stage_row_off<MT>(i * 32 + lane));
    uint4 o4[NQ];
#pragma unroll
    for (int k = 0; k < NQ; ++k) o4[k] = srow[k];
    if constexpr (kPost) {
      // spikes {0,1} combined with identity spikes {0,1,2}: exact in fp16
#pragma unroll
      for (int k = 0; k < NQ; ++k) {
        const uint4 i4 = idr[i][k];
        __half2* s2 = reinterpret_cast<__half2*>(&o4[k]);
        const __half2* d2 = reinterpret_cast<const __half2*>(&i4);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          if constexpr (RES == CF_RES_ADD_POST) s2[m] = __hadd2(s2[m], d2[m]);
          else if constexpr (RES == CF_RES_AND_POST) s2[m] = __hmul2(s2[m], d2[m]);
          else s2[m] = __hmul2(d2[m], __hsub2(__float2half2_rn(1.f), s2[m]));
        }
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(outp + row_off[i]);
#pragma unroll
    for (int k = 0; k < NQ; ++k) dst[k] = o4[k];
  }
  __syncwarp();  // the staging rows are reused by the next chunk
}

// Integer weight planes (PL = 3): the weight is quantised to a 30-bit integer
// q = q2 * 2^20 + q1 * 2^10 + q0 with signed digits |q_i| <= 512, each digit
// plane an fp16 operand holding exact integers.  With integer activations
// (spike counts) every product and every partial sum is an integer below
// 2^24, so each plane's fp32 TMEM accumulation is exact whatever the tensor
// core's internal rounding; the planes sit in separate accumulators and the
// epilogue joins them in fp64 (exact) before one rounding to fp32.
template <int PL>
__device__ __forceinline__ void load_acc(uint32_t taddr, uint32_t plane_cols, bool m128,
                                         float (&r)[32]) {
  if constexpr (PL == 1) {
    if (m128) tmem_ld32(taddr, r);
    else tmem_ld16x2_32(taddr, r);
  } else {
    // plane p (accumulator columns p * plane_cols on) holds sum x * q_{2-p}
    float t[32];
    double d[32];
    if (m128) tmem_ld32(taddr, t);
    else tmem_ld16x2_32(taddr, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) d[j] = (double)t[j] * 1048576.0;
    if (m128) tmem_ld32(taddr + plane_cols, t);
    else tmem_ld16x2_32(taddr + plane_cols, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) d[j] = fma((double)t[j], 1024.0, d[j]);
    if (m128) tmem_ld32(taddr + 2 * plane_cols, t);
    else tmem_ld16x2_32(taddr + 2 * plane_cols, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] = (float)(d[j] + (double)t[j]);
  }
}

template <int TP, int RES, bool FAST, int PL>
__global__ void __launch_bounds__(kTThreads, 1)
    conv_t_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                  const ConvArgs a) {
  const int BK = a.BK;
  const int NR = a.NR;
  const int XA = a.a_bytes;          // activation box of one stage
  const int MT = a.MT;               // output channels per tile (MMA M): 128 or 64
  const int W_BYTES = MT * BK * 2;   // one weight tile
  const uint32_t ROWB = (uint32_t)BK * 2;
  const int S = a.stages;
  const int n_ct = a.n_ntiles;       // output-channel tiles
  // A stage carries one activation box and the nsub weight tiles it serves.
  // Steps walk (gh, gw, kc).  In the kh-box mode (stride 1, tile inside one
  // image) one activation box of Hb+KH-1 rows covers all kh taps of a kw
  // column: tap (kh, kw) reads it from row kh*Wb*TP on, the step loop has
  // gh = 0 only and the stage holds KH weight tiles.  One barrier wait and one
  // commit then cover KH*BK/16 MMAs.
  // kw-group mode (a.kwgroup, no kh-box): a stage carries the KW taps of one
  // kernel row, each with its own activation box (XA bytes apart) and weight
  // tile, and the step loop has gw = 0 only.
  const int n_gh = a.khbox ? 1 : a.KH;
  const int n_gw = a.kwgroup ? 1 : a.KW;
  const int nsub = a.khbox ? a.KH : (a.kwgroup ? a.KW : 1);
  const int XSB = a.kwgroup ? nsub * XA : XA;  // activation bytes of one stage
  const int WSB = nsub * W_BYTES;    // weight bytes of one stage

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sX = smem;
  uint8_t* sW = sX + (size_t)S * XSB;
  uint8_t* sStage = sW + (size_t)S * WSB;  // epilogue staging, kStageBytes per warp
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sStage + kTEpiWarps * kStageBytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull_bar = empty_bar + S;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* done_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // EGD counter: the word after the abort flag (a static __shared__ variable
  // would come out of the 227 KB the dynamic allocation already claims)
  unsigned int* s_active = reinterpret_cast<unsigned int*>(const_cast<int*>(abort_flag) + 1);
  // The tile masks (egd) and the activations come from earlier launches:
  // read nothing of them before the dependency has resolved.
  if (a.egd) griddep_wait();
  if (a.egd) {
    if (threadIdx.x == 0) *s_active = 0;
    __syncthreads();
    egd_count_active(a, s_active);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], kTEpiWarps);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp < kProdWarps && lane == 0) {
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmW);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Barrier set-up and the TMEM allocation above overlap the previous launch;
  // everything below reads or writes tensors earlier launches produce or use.
  if (!a.egd) griddep_wait();
  griddep_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const bool use_mask = !a.egd || *s_active <= a.egd_max_active;

  if (warp < kProdWarps) {
    // ------------------------------------------------------------ producers
    // Producer p issues the steps i with i % nprod == p (stage i % S, phase
    // (i / S) & 1): one activation box and nsub weight tiles on full[stage].
    if (warp < a.nprod) {
      const int p = warp;
      int owner = 0, stage = 0;
      uint32_t phase = 0;
      uint32_t used = 0, used_phase = 0;
      bool ok = true;
      bool drop_next = a.drop_load && blockIdx.x == 0;  // test hook, see ConvArgs
      for (int tile = blockIdx.x; tile < a.n_tiles && ok; tile += gridDim.x) {
        const int pt = tile / n_ct;
        const int ct = tile - pt * n_ct;
        const int wt = pt % a.n_wt;
        const int ht = (pt / a.n_wt) % a.n_ht;
        const int bt = pt / (a.n_wt * a.n_ht);
        const int wi0 = wt * a.Wb * a.stride - a.pad;
        const int hi0 = ht * a.Hb * a.stride - a.pad;
        const int b0 = bt * a.Bb;
        const uint32_t km = tile_kmask(a, pt, use_mask);
        if (km == 0) continue;
        for (int gh = 0; gh < n_gh && ok; ++gh) {
          for (int gw = 0; gw < n_gw && ok; ++gw) {
            for (int kc = 0; kc < a.n_kc; ++kc) {
              if (!chunk_on(km, kc)) continue;
              const bool mine = owner == p;
              const int my_stage = stage;
              const uint32_t my_phase = phase;
              if (++owner == a.nprod) owner = 0;
              if (++stage == S) {
                stage = 0;
                phase ^= 1u;
              }
              if (!mine) continue;
              if (!warp_wait_or_abort(&empty_bar[my_stage], my_phase ^ 1u,
                                      ERR_SITE_PRODUCER_EMPTY, abort_flag, a,
                                      a.backoff)) {
                ok = false;
                break;
              }
              const bool dropped = drop_next;
              drop_next = false;
              if (lane == 0 && !dropped) {
                mbar_arrive_expect_tx(&full_bar[my_stage], XSB + WSB);
                const int xc = xchunk(a, kc) * BK;
                if (a.kwgroup) {
                  for (int j = 0; j < nsub; ++j)
                    tma_load_5d(sX + (size_t)my_stage * XSB + (size_t)j * XA, &tmX,
                                &full_bar[my_stage], xc, a.t0, wi0 + j, hi0 + gh, b0);
                } else {
                  tma_load_5d(sX + (size_t)my_stage * XSB, &tmX, &full_bar[my_stage], xc,
                              a.t0, wi0 + gw, hi0 + gh, b0);
                }
                // sub-step j meets tap (gh + j, gw) in kh-box mode, (gh, j) in
                // kw-group mode, (gh, gw) otherwise
                const int tap_step = a.khbox ? a.KW : 1;
                int tap = gh * a.KW + gw;
                for (int j = 0; j < nsub; ++j, tap += tap_step)
                  tma_load_2d(sW + (size_t)my_stage * WSB + (size_t)j * W_BYTES, &tmW,
                              &full_bar[my_stage], tap * a.Cin_w + kc * BK, ct * MT);
              }
              __syncwarp();
              if (!dropped) {
                used |= 1u << my_stage;
                used_phase = (used_phase & ~(1u << my_stage)) | (my_phase << my_stage);
              }
            }
          }
        }
      }
      if (!ok) {
        for (int st = 0; st < S; ++st) {
          if (!((used >> st) & 1u)) continue;
          for (uint32_t q = 0; q < (1u << 16); ++q)
            if (mbar_try_wait(&full_bar[st], (used_phase >> st) & 1u)) break;
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t xa_step = (uint32_t)XSB >> 4;
      const uint32_t ws_step = (uint32_t)WSB >> 4;
      const uint32_t w_step = (uint32_t)W_BYTES >> 4;
      // B operand advance per sub-step: kh-box row shift, or the next box
      const uint32_t sub_step = a.kwgroup ? ((uint32_t)XA >> 4)
                                          : (((uint32_t)(a.Wb * TP) * ROWB) >> 4);
      const uint64_t x_desc0 = make_smem_desc(smem_u32(sX), ROWB);
      const uint64_t w_desc0 = make_smem_desc(smem_u32(sW), ROWB);
      const int ksteps = BK / 16;
      int stage = 0;
      uint32_t phase = 0;
      uint64_t xd = x_desc0, wd = w_desc0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < a.n_tiles && ok; tile += gridDim.x) {
        const int pt = tile / n_ct;
        const uint32_t km = tile_kmask(a, pt, use_mask);
        if (!wait_or_abort(&tempty_bar[acc], acc_phase ^ 1u, ERR_SITE_MMA_TEMPTY, abort_flag, a)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (km == 0) {
          mbar_arrive(&tfull_bar[acc]);
        } else {
          const uint32_t d_base = tmem_base + (uint32_t)(acc * PL * NR);
          uint32_t started = 0u;  // planes whose accumulator holds a first product
          const int n_g = n_gh * n_gw;
          for (int g = 0; g < n_g && ok; ++g) {
            int plane = 0, pk = 0;  // weight plane of chunk kc (kc / n_kx), and kc % n_kx
            for (int kc = 0; kc < a.n_kc; ++kc) {
              const int cur_plane = plane;
              if (PL > 1 && ++pk == a.n_kx) {
                pk = 0;
                ++plane;
              }
              if (!chunk_on(km, kc)) continue;
              if (!mbar_try_wait(&full_bar[stage], phase) &&
                  !wait_or_abort(&full_bar[stage], phase, ERR_SITE_MMA_FULL, abort_flag, a)) {
                ok = false;
                break;
              }
              {
                const uint32_t d_tmem = d_base + (uint32_t)(PL > 1 ? cur_plane * NR : 0);
                uint32_t accum = (started >> cur_plane) & 1u;
                uint64_t bd = xd, ad = wd;
                for (int j = 0; j < nsub; ++j, bd += sub_step, ad += w_step) {
                  if (ksteps == 4) issue_kchunk<4>(d_tmem, ad, bd, a.idesc, accum);
                  else if (ksteps == 2) issue_kchunk<2>(d_tmem, ad, bd, a.idesc, accum);
                  else issue_kchunk<1>(d_tmem, ad, bd, a.idesc, accum);
                  accum = 1u;
                }
                started |= 1u << cur_plane;
              }
              umma_commit(&empty_bar[stage]);
              if (++stage == S) {
                stage = 0;
                phase ^= 1u;
                xd = x_desc0;
                wd = w_desc0;
              } else {
                xd += xa_step;
                wd += ws_step;
              }
            }
          }
          if (!ok) break;
          umma_commit(&tfull_bar[acc]);
        }
        if (++acc == a.nbuf) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      umma_commit(done_bar);
      for (uint32_t p = 0; p < kMaxPolls; ++p)
        if (mbar_try_wait(done_bar, 0)) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp e reads TMEM lane quarter q = warp % 4 and the column chunks k,
    // k+E, ... with k = e / 4, E = warps per quarter.  M=128: the quarter's 32
    // lanes are channels q*32 + lane, a chunk is 32 columns.  M=64: lanes 0-15
    // of the quarter hold channels q*16 + 0..15, a chunk is 64 columns and each
    // half-warp takes 32 of them (tcgen05.ld 16x32bx2).
    constexpr int E = kTEpiWarps / 4;
    const int e = warp - kEpiWarp0;
    const int q = warp & 3;
    const int k = e >> 2;
    const int CW = MT == 128 ? 32 : 64;  // columns per chunk
    const int n_chunk = NR / CW;
    int last_chunk = k;
    while (last_chunk + E < n_chunk) last_chunk += E;
    uint8_t* stage = sStage + e * kStageBytes;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x) {
      const int pt = tile / n_ct;
      const int ct = tile - pt * n_ct;
      const int wt = pt % a.n_wt;
      const int ht = (pt / a.n_wt) % a.n_ht;
      const int bt = pt / (a.n_wt * a.n_ht);
      const bool has_acc = tile_kmask(a, pt, use_mask) != 0;
      const int co_base = ct * MT + q * (MT / 4);
      const int co = co_base + (MT == 128 ? lane : (lane & 15));
      const float sc = a.scale ? __ldg(a.scale + co) : 1.f;
      const float sh = a.shift ? __ldg(a.shift + co) : 0.f;
      if (!warp_wait_or_abort(&tfull_bar[acc], acc_phase, ERR_SITE_EPI_TFULL, abort_flag,
                              a, a.backoff))
        break;
      tc_fence_after();
      for (int ch = k; ch < n_chunk; ch += E) {
        const int col = ch * CW;
        float r[32];
        const uint32_t taddr =
            tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * PL * NR + col);
        if (!has_acc) {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0.f;
        } else {
          load_acc<PL>(taddr, (uint32_t)NR, MT == 128, r);
        }
        if (ch == last_chunk) {
          // Last read of this warp: hand the accumulator back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[acc]);
        }
        if (MT == 128) {
          if (a.tcount == TP)
            epi_chunk_t<TP, RES, FAST, true, 128>(a, r, co, co_base, sc, sh, wt, ht, bt, col,
                                                  stage, lane);
          else
            epi_chunk_t<TP, RES, FAST, false, 128>(a, r, co, co_base, sc, sh, wt, ht, bt, col,
                                                   stage, lane);
        } else {
          if (a.tcount == TP)
            epi_chunk_t<TP, RES, FAST, true, 64>(a, r, co, co_base, sc, sh, wt, ht, bt, col,
                                                 stage, lane);
          else
            epi_chunk_t<TP, RES, FAST, false, 64>(a, r, co, co_base, sc, sh, wt, ht, bt, col,
                                                  stage, lane);
        }
      }
      if (++acc == a.nbuf) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, a.tmem_cols);
  }
}

// --------------------------------------------------------------------------
// launch templates (instantiated per TP in cf_conv_tp*.cu)
// --------------------------------------------------------------------------
constexpr int kMaxDevices = 64;

inline int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

// Raise a kernel's dynamic shared-memory limit to 227 KB once per device
// (the attribute is per device; `done` holds one flag per device ordinal).
inline int allow_big_smem(const void* fn, std::atomic<bool>* done, const char* what) {
  const int dev = current_device();
  if (dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire)) return CF_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) return check_cuda(e, what);
  if (dev >= 0 && dev < kMaxDevices) done[dev].store(true, std::memory_order_release);
  return CF_OK;
}

// Launch with programmatic stream serialisation: the kernel's CTAs may start
// while the previous launch in the stream drains (each kernel waits in
// griddep_wait before touching tensors; inside a captured graph this becomes
// a programmatic dependency edge).
template <typename K>
int launch_pdl(K kernel, int grid, int threads, int smem, cudaStream_t stream,
               const CUtensorMap& t0, const CUtensorMap& t1, const ConvArgs& args,
               const char* what) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, t0, t1, args), what);
}

template <int TP, int RES, bool FAST>
int launch_inst(const CUtensorMap& tmA, const CUtensorMap& tmB, ConvArgs args, int grid,
                cudaStream_t stream) {
  const int A_BYTES = args.a_bytes;
  const int B_BYTES = args.BN * args.BK * 2;
  const int fixed = 1024 + kEpiBytes + 256;
  const int wslab = args.wres ? args.KH * args.KW * args.n_kc * B_BYTES : 0;
  const int per_stage = A_BYTES + (args.wres ? 0 : B_BYTES);
  int stages = (kSmemBudget - fixed - wslab) / per_stage;
  if (stages > 8) stages = 8;
  if (stages < 2) return fail(CF_ERR_UNSUPPORTED, "conv tile does not fit shared memory");
  args.stages = stages;
  // A producer may run at most `stages` iterations ahead of the consumer
  // safely only if there are no more producers than stages.
  args.nprod = stages < kProdWarps ? stages : kProdWarps;
  int smem = fixed + wslab + stages * per_stage;
  // Keep every TMEM-using CTA above half the SM's shared memory so that two
  // of them can never be co-resident and contend for TMEM columns.
  if (smem < 120 * 1024) smem = 120 * 1024;
  static std::atomic<bool> attr_done[kMaxDevices];
  if (int rc = allow_big_smem(reinterpret_cast<const void*>(conv_bn_lif_kernel<TP, RES, FAST>),
                              attr_done, "cudaFuncSetAttribute(conv)"))
    return rc;
  return launch_pdl(conv_bn_lif_kernel<TP, RES, FAST>, grid, kConvThreads, smem, stream, tmA,
                    tmB, args, "conv_bn_lif launch");
}

template <int TP, int RES, bool FAST, int PL>
int launch_t(const CUtensorMap& tmX, const CUtensorMap& tmW, ConvArgs args, int grid,
             cudaStream_t stream) {
  const int nsub = args.khbox ? args.KH : (args.kwgroup ? args.KW : 1);
  const int stage_bytes = (args.kwgroup ? nsub : 1) * args.a_bytes +
                          nsub * args.MT * args.BK * 2;
  const int fixed = kTFixedBytes;
  int stages = (kTSmemBudget - fixed) / stage_bytes;
  if (stages > 8) stages = 8;
  if (stages < 2) return fail(CF_ERR_UNSUPPORTED, "conv tile does not fit shared memory");
  args.stages = stages;
  // Round-robin producers may run at most one ring ahead only if there are
  // no more of them than stages.
  args.nprod = stages < kProdWarps ? stages : kProdWarps;
  int smem = fixed + stages * stage_bytes;
  if (smem < 120 * 1024) smem = 120 * 1024;  // one TMEM-owning CTA per SM
  static std::atomic<bool> attr_done[kMaxDevices];
  if (int rc = allow_big_smem(reinterpret_cast<const void*>(conv_t_kernel<TP, RES, FAST, PL>),
                              attr_done, "cudaFuncSetAttribute(conv_t)"))
    return rc;
  return launch_pdl(conv_t_kernel<TP, RES, FAST, PL>, grid, kTThreads, smem, stream, tmX, tmW,
                    args, "conv_t launch");
}

template <int TP, int RES, bool FAST>
int launch_any(const CUtensorMap& A, const CUtensorMap& W, const ConvArgs& args, int grid,
               cudaStream_t s) {
  if (args.nplanes == 3) return launch_t<TP, RES, FAST, 3>(A, W, args, grid, s);
  return args.tmode ? launch_t<TP, RES, FAST, 1>(A, W, args, grid, s)
                    : launch_inst<TP, RES, FAST>(A, W, args, grid, s);
}

template <int TP, int RES>
int dispatch_fast(bool fast, const CUtensorMap& A, const CUtensorMap& W, const ConvArgs& args,
                  int grid, cudaStream_t s) {
  return fast ? launch_any<TP, RES, true>(A, W, args, grid, s)
              : launch_any<TP, RES, false>(A, W, args, grid, s);
}

template <int TP>
int dispatch_res(int res, bool fast, const CUtensorMap& A, const CUtensorMap& W,
                 const ConvArgs& args, int grid, cudaStream_t s) {
  switch (res) {
    case CF_RES_NONE: return dispatch_fast<TP, CF_RES_NONE>(fast, A, W, args, grid, s);
    case CF_RES_ADD_POST: return dispatch_fast<TP, CF_RES_ADD_POST>(fast, A, W, args, grid, s);
    case CF_RES_AND_POST: return dispatch_fast<TP, CF_RES_AND_POST>(fast, A, W, args, grid, s);
    case CF_RES_IAND_POST: return dispatch_fast<TP, CF_RES_IAND_POST>(fast, A, W, args, grid, s);
    case CF_RES_ADD_PRE: return dispatch_fast<TP, CF_RES_ADD_PRE>(fast, A, W, args, grid, s);
    default: return launch_any<TP, CF_RES_Z_ONLY, true>(A, W, args, grid, s);
  }
}

#ifndef CF_CONV_INSTANTIATE
extern template int dispatch_res<1>(int, bool, const CUtensorMap&, const CUtensorMap&,
                                    const ConvArgs&, int, cudaStream_t);
extern template int dispatch_res<2>(int, bool, const CUtensorMap&, const CUtensorMap&,
                                    const ConvArgs&, int, cudaStream_t);
extern template int dispatch_res<4>(int, bool, const CUtensorMap&, const CUtensorMap&,
                                    const ConvArgs&, int, cudaStream_t);
extern template int dispatch_res<8>(int, bool, const CUtensorMap&, const CUtensorMap&,
                                    const ConvArgs&, int, cudaStream_t);
#endif

}  // namespace convk
}  // namespace cf
