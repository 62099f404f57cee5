// cf_conv.cu — fused Conv -> BN -> (residual) -> multi-step LIF on the
// 5th-generation tensor cores (tcgen05, sm_100a).
// Host side: tile geometry, tensor maps, argument checks and the C ABI.  The
// kernels themselves are in cf_conv_kernels.cuh.
#include "cf_conv_kernels.cuh"

#include <cstdlib>
#include <mutex>

namespace cf {

// Device error word written by bounded waits that expire.  Nonzero = the site
// code of the first expiry.  Read and cleared by cf_check_device_error.
__device__ int32_t g_dev_error = 0;

namespace {
using namespace convk;

// Device address of g_dev_error for the current device (cached per device).
int32_t* dev_error_ptr() {
  static std::atomic<int32_t*> cache[kMaxDevices];
  const int dev = current_device();
  if (dev >= 0 && dev < kMaxDevices) {
    if (int32_t* p = cache[dev].load(std::memory_order_acquire)) return p;
  }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_dev_error) != cudaSuccess) return nullptr;
  if (dev >= 0 && dev < kMaxDevices) cache[dev].store(static_cast<int32_t*>(p), std::memory_order_release);
  return static_cast<int32_t*>(p);
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

CUtensorMapL2promotion l2promo() { return CU_TENSOR_MAP_L2_PROMOTION_L2_256B; }

// Process-wide bounded-wait settings (cf_set_wait_limit / cf_test_arm_stalled_load).
std::atomic<uint32_t> g_wait_limit{0};
std::atomic<int> g_stall_armed{0};

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
  int tmode;  // 1: channel-major kernel (conv_t_kernel), M = 128 channels, N = NR rows
  int NR;
};

// The channel-major kernel serves every layer whose output channels come in
// whole 128-channel tiles (M = 128) or 64-channel tiles (M = 64, half the
// per-MAC rate of M = 128 but still 128 tensor cycles per N = 256 MMA, and
// 80 instead of 192 B/clk of operand reads compared with N = 64 tiles of the
// pixel-major kernel).
// Narrow-input 64-channel layers (the stem's im2col with K <= 32) have too
// little MMA work per tile to hide the channel-major epilogue and stay on the
// pixel-major kernel.
bool use_tmode(int64_t Cout, int64_t Cin_p) {
  return Cout % 128 == 0 || (Cout % 64 == 0 && Cin_p >= 64);
}

// Choose the pixel box (Wb x Hb x Bb = P, powers of two) that wastes the
// fewest padded output pixels; ties go to boxes inside one image, then to the
// wider box (longer contiguous rows for the output stores).
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
      // ties: fewer images per tile (boxes stay inside one image), then wider
      if (best < 0 || cost < best ||
          (cost == best && (bb < g.Bb || (bb == g.Bb && wb > g.Wb)))) {
        best = cost;
        g.Wb = wb; g.Hb = hb; g.Bb = bb;
        g.n_wt = (int)nwt; g.n_ht = (int)nht; g.n_bt = (int)nbt;
      }
    }
  }
  g.n_mtiles = g.n_wt * g.n_ht * g.n_bt;
}


// SM count of the current device (cached per device ordinal).
int sm_count() {
  static std::atomic<int> cache[kMaxDevices];
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}


int choose_bn(int Cout, int n_mtiles) {
  int bn = 128;
  while (bn > 32 && (Cout % bn != 0)) bn >>= 1;
  if (Cout % bn != 0) return 0;
  const int sms = 148;
  // N=256 halves the MMA instructions and the activation re-reads per output,
  // worth it while the grid still covers most SMs.
  if (Cout % 256 == 0 && (long)n_mtiles * (Cout / 256) >= (sms * 3) / 4) bn = 256;
  return bn;
}

int choose_bk(int Cin_p, bool sparse) {
  if (sparse && Cin_p > 128 && Cin_p % 32 == 0) return 32;
  if (Cin_p % 64 == 0) return 64;
  if (Cin_p % 32 == 0) return 32;
  return 16;
}

// nplanes = 3: integer weight planes in three accumulators, which fit TMEM
// (512 columns) only as single-buffered N = 128 tiles of the channel-major kernel.
int make_geometry(int64_t T, int64_t B, int64_t Ho, int64_t Wo, int64_t Cout, int64_t Cin_p,
                  int64_t stride, bool sparse, Geometry& g, int nplanes = 1) {
  const int tc = (int)(T < kMaxTP ? T : kMaxTP);
  g.TP = next_pow2(tc);
  g.BK = choose_bk((int)Cin_p, sparse);
  g.n_kc = (int)(Cin_p / g.BK);
  if (use_tmode(Cout, Cin_p)) {
    // N = 256 rows per tile unless that leaves a quarter of the SMs idle.
    g.tmode = 1;
    g.BN = Cout % 128 == 0 ? 128 : 64;
    g.NR = 256;
    choose_box(g.NR / g.TP, (int)B, (int)Ho, (int)Wo, (int)stride, g);
    if (nplanes > 1 || (long)g.n_mtiles * (Cout / g.BN) < (148 * 3) / 4) {
      g.NR = 128;
      choose_box(g.NR / g.TP, (int)B, (int)Ho, (int)Wo, (int)stride, g);
    }
    return CF_OK;
  }
  if (nplanes > 1)
    return fail(CF_ERR_UNSUPPORTED,
                "integer weight planes need the channel-major kernel (Cout %% 128 == 0, or "
                "Cout %% 64 == 0 with Cin_p >= 64)");
  g.tmode = 0;
  g.NR = 128;
  choose_box(128 / g.TP, (int)B, (int)Ho, (int)Wo, (int)stride, g);
  g.BN = choose_bn((int)Cout, g.n_mtiles);
  return g.BN ? CF_OK : fail(CF_ERR_UNSUPPORTED, "Cout=%lld must be a multiple of 32", (long long)Cout);
}

int dispatch(const Geometry& g, int res, bool fast, const CUtensorMap& A, const CUtensorMap& W,
             const ConvArgs& args, int grid, cudaStream_t s) {
  switch (g.TP) {
    case 1: return dispatch_res<1>(res, fast, A, W, args, grid, s);
    case 2: return dispatch_res<2>(res, fast, A, W, args, grid, s);
    case 4: return dispatch_res<4>(res, fast, A, W, args, grid, s);
    default: return dispatch_res<8>(res, fast, A, W, args, grid, s);
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
                     int hard_reset, int decay_input, int wparts, cudaStream_t stream,
                     float egd_max_active_frac = -1.f, int64_t co_split = -1,
                     void* out2 = nullptr, const float* v_in2 = nullptr, float* v_out2 = nullptr) {
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
  const int nplanes = wparts == 3 ? 3 : 1;
  if (nplanes > 1 && tile_mask)
    return fail(CF_ERR_UNSUPPORTED, "integer weight planes run dense only (no tile mask)");
  // Device-EGD launches use the dense channel chunk (their masks come from a
  // prescan with that chunk); the tile boxes do not depend on the chunk.
  const bool egd_launch = tile_mask && egd_max_active_frac >= 0.f;
  if (int rc = make_geometry(T, B, Ho, Wo, Cout, Cin_p, stride, tile_mask != nullptr && !egd_launch,
                             g, nplanes))
    return rc;
  // Dense launches whose kh-box stage does not fit twice at BK = 64 take
  // BK = 32 when that fits it at least three times: the stage then carries
  // KH * 2 MMAs per barrier round trip and the activation rows serve every kh
  // tap, 73 instead of 96 operand bytes per MMA cycle, i.e. about 30 % more
  // MMA work buffered in the same shared memory (config-0 layer: -5 % time).
  // Masked launches keep the mask's chunk.
  if (!tile_mask && g.tmode && stride == 1 && KH > 1 && g.Bb == 1 && g.BK == 64 &&
      (g.Wb * g.TP) % 16 == 0) {
    auto khstage = [&](int64_t bk) {
      return (int64_t)(g.Hb + KH - 1) * g.Wb * g.TP * bk * 2 + KH * (int64_t)g.BN * bk * 2;
    };
    if ((kTSmemBudget - kTFixedBytes) / khstage(64) < 2 &&
        (kTSmemBudget - kTFixedBytes) / khstage(32) >= 3) {
      g.BK = 32;
      g.n_kc = (int)(Cin_p / 32);
    }
  }
  const int n_kx = g.n_kc;  // activation chunks per tap
  g.n_kc *= wparts;          // weight chunks: part 0 chunks, then part 1, ...
  if (tile_mask && g.n_kc > 32)
    return fail(CF_ERR_UNSUPPORTED, "sparse mode supports at most 32 channel chunks");
  const int64_t Cin_w = wparts * Cin_p;

  auto encode = get_encode_fn();
  if (!encode) return fail(CF_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");

  // A: x[B][H][W][T][Cin_p] fp16, 5-D, box (BK, TP, Wb*s, Hb*s, Bb) with
  // element stride s along W and H (the TMA then loads Wb x Hb elements).
  // Weight residency: a single N tile whose whole weight slab fits stays in
  // shared memory for the CTA's lifetime.  Halo mode (stride 1, tile = one
  // full output row): one activation box per tile covers all taps.
  const int64_t wslab = KH * KW * g.n_kc * (int64_t)g.BN * g.BK * 2;
  const int wres = (!g.tmode && Cout == g.BN && wslab <= 80 * 1024) ? 1 : 0;
  const int Wh = g.Wb + (int)KW - 1;
  const int halo_bytes = ((g.TP * Wh * (int)KH * g.BK * 2) + 1023) / 1024 * 1024;
  const int fixed_bytes = 1024 + kEpiBytes + 256;
  // The kh shift (Wb*TP rows) must keep the operand on a 1 KB swizzle boundary.
  // Two stages of (activation box + KH weight tiles) must fit beside the epilogue staging.
  const int64_t khbox_stage = (int64_t)(g.Hb + KH - 1) * g.Wb * g.TP * g.BK * 2 +
                              KH * (int64_t)g.BN * g.BK * 2;
  const int khbox = (g.tmode && stride == 1 && KH > 1 && g.Bb == 1 &&
                     g.Hb + KH - 1 <= 256 && (g.Wb * g.TP * g.BK * 2) % 1024 == 0 &&
                     2 * khbox_stage + kTFixedBytes <= kTSmemBudget) ? 1 : 0;
  const int halo = (!g.tmode && wres && stride == 1 && g.Hb == 1 && g.Bb == 1 &&
                    g.Wb * g.TP == 128 && g.TP >= 4 && g.BK == 64 && Wh <= 256 && KH <= 256 &&
                    fixed_bytes + wslab + 2 * halo_bytes <= kSmemBudget) ? 1 : 0;
  CUtensorMap tmA, tmB;
  {
    cuuint64_t dims[5] = {(cuuint64_t)Cin_p, (cuuint64_t)T, (cuuint64_t)W, (cuuint64_t)H,
                          (cuuint64_t)B};
    cuuint64_t strides[4] = {(cuuint64_t)(Cin_p * 2), (cuuint64_t)(T * Cin_p * 2),
                             (cuuint64_t)(W * T * Cin_p * 2), (cuuint64_t)(H * W * T * Cin_p * 2)};
    cuuint32_t box[5] = {(cuuint32_t)g.BK, (cuuint32_t)g.TP, (cuuint32_t)(g.Wb * stride),
                         (cuuint32_t)(g.Hb * stride), (cuuint32_t)g.Bb};
    if (halo) {
      box[2] = (cuuint32_t)Wh;
      box[3] = (cuuint32_t)KH;
    }
    if (khbox) box[3] = (cuuint32_t)(g.Hb + KH - 1);
    cuuint32_t estr[5] = {1, 1, (cuuint32_t)stride, (cuuint32_t)stride, 1};
    CUresult r = encode(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(x), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(g.BK * 2),
                        l2promo(), CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CF_ERR_CUDA, "tensor map (activations) failed: %d", (int)r);
  }
  {
    const int64_t K = KH * KW * Cin_w;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)Cout};
    cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
    cuuint32_t box[2] = {(cuuint32_t)g.BK, (cuuint32_t)g.BN};  // channel-major: BN = 128 = M
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(wp), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(g.BK * 2),
                        l2promo(), CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CF_ERR_CUDA, "tensor map (weights) failed: %d", (int)r);
  }

  ConvArgs args{};
  args.scale = scale;
  args.shift = shift;
  args.identity = static_cast<const __half*>(identity);
  args.out = static_cast<__half*>(out);
  args.co_split = co_split >= 0 ? (int)co_split : (int)Cout;
  args.out2 = static_cast<__half*>(out2);
  args.v_in2 = v_in2;
  args.v_out2 = v_out2;
  if (co_split >= 0) {
    if (!g.tmode || co_split % g.BN || co_split <= 0 || co_split >= Cout || !out2 ||
        res_mode != CF_RES_NONE || tile_mask || wparts != 1)
      return fail(CF_ERR_UNSUPPORTED,
                  "dual output needs the channel-major kernel, a split on an output-channel "
                  "tile (multiple of %d), no residual, no mask and fp16 weights", g.BN);
    const void* p2[] = {out2, v_in2, v_out2};
    for (const void* p : p2)
      if (p && !al16(p)) return fail(CF_ERR_UNSUPPORTED, "tensor pointers must be 16-byte aligned");
  }
  args.tile_mask = tile_mask;
  args.T = (int)T;
  args.B = (int)B; args.Ho = (int)Ho; args.Wo = (int)Wo;
  args.Cout = (int)Cout; args.Cin_p = (int)Cin_p;
  args.Cin_w = (int)Cin_w;
  args.n_kx = n_kx;
  args.wparts = wparts;
  args.nplanes = nplanes;
  args.KH = (int)KH; args.KW = (int)KW; args.stride = (int)stride; args.pad = (int)pad;
  args.Wb = g.Wb; args.Hb = g.Hb; args.Bb = g.Bb;
  args.n_wt = g.n_wt; args.n_ht = g.n_ht; args.n_mtiles = g.n_mtiles;
  args.n_ntiles = (int)(Cout / g.BN);
  args.n_tiles = args.n_mtiles * args.n_ntiles;
  args.n_kc = g.n_kc;
  args.kc_all = g.n_kc >= 32 ? 0xFFFFFFFFu : ((1u << g.n_kc) - 1u);
  args.BN = g.BN;
  args.BK = g.BK;
  args.tmode = g.tmode;
  args.NR = g.NR;
  args.lwb = __builtin_ctz((unsigned)g.Wb);
  args.lhb = __builtin_ctz((unsigned)g.Hb);
  if (g.tmode) {
    args.MT = g.BN;
    args.idesc = make_idesc_f16(g.BN, g.NR);
    args.nbuf = nplanes > 1 ? 1 : 2;  // 3 planes x 128 columns leave no room for a second buffer
    const uint32_t cols = (uint32_t)(args.nbuf * nplanes * g.NR);
    args.tmem_cols = cols <= 256 ? (cols <= 128 ? 128u : 256u) : 512u;  // a power of two
  } else {
    args.nbuf = 2;
    args.idesc = make_idesc_f16(128, g.BN);
    args.tmem_cols = (uint32_t)(2 * g.BN < 32 ? 32 : 2 * g.BN);
  }
  args.lp = make_lif(tau, v_th, v_reset, hard_reset, decay_input);
  const bool fast = args.lp.decay_input && args.lp.hard_reset && args.lp.tau_pow2 &&
                    args.lp.v_reset == 0.0f;
  const uint32_t lim = g_wait_limit.load(std::memory_order_relaxed);
  args.max_polls = lim ? lim : kMaxPolls;
  args.err = dev_error_ptr();
  if (!args.err) return fail(CF_ERR_CUDA, "device error word is not addressable");
  args.drop_load = g_stall_armed.exchange(0) ? 1 : 0;
  args.egd = (tile_mask && egd_max_active_frac >= 0.f) ? 1 : 0;
  if (args.egd) {
    const double pairs = (double)g.n_mtiles * n_kx;
    const double lim = egd_max_active_frac >= 1.f ? pairs : floor(egd_max_active_frac * pairs);
    args.egd_max_active = (uint32_t)(lim > 4294967295.0 ? 4294967295.0 : lim);
  }
  args.stages = 0;
  args.wres = wres;
  args.halo = halo;
  args.Wh = Wh;
  args.backoff = 256;
  args.khbox = khbox;
  // Without a kh-box, group a kernel row's KW taps into one stage when two
  // such stages fit: one barrier round trip per KW*BK/16 MMAs.
  {
    const int64_t xa = (int64_t)g.NR * g.BK * 2;
    const int64_t kwg_stage = KW * (xa + (int64_t)g.BN * g.BK * 2);
    args.kwgroup = (g.tmode && !khbox && KW > 1 &&
                    2 * kwg_stage + kTFixedBytes <= kTSmemBudget) ? 1 : 0;
  }
  if (g.tmode)
    args.a_bytes = khbox ? (g.Hb + (int)KH - 1) * g.Wb * g.TP * g.BK * 2  // 1 KB multiple
                         : g.NR * g.BK * 2;
  else
    args.a_bytes = halo ? halo_bytes : 128 * g.BK * 2;
  const int grid = args.n_tiles < sm_count() ? args.n_tiles : sm_count();

  for (int64_t t0 = 0; t0 < T; t0 += kMaxTP) {
    args.t0 = (int)t0;
    args.tcount = (int)((T - t0) < kMaxTP ? (T - t0) : kMaxTP);
    args.v_in = (t0 == 0) ? v_in : v_out;
    args.v_out = v_out;
    args.v_in2 = (t0 == 0) ? v_in2 : v_out2;
    if (int rc = dispatch(g, res_mode, fast, tmA, tmB, args, grid, stream)) return rc;
    args.drop_load = 0;
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

int cf_set_wait_limit(uint32_t max_polls) {
  g_wait_limit.store(max_polls, std::memory_order_relaxed);
  return CF_OK;
}

int cf_test_arm_stalled_load(int armed) {
  g_stall_armed.store(armed ? 1 : 0);
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

int cf_conv_geometry_ex(int64_t T, int64_t B, int64_t Ho, int64_t Wo, int64_t Cout,
                        int64_t Cin_p, int64_t stride, int flags, int32_t* out6) {
  const bool sparse = (flags & 1) != 0;
  const int nplanes = (flags & 2) ? 3 : 1;
  if (!out6 || T <= 0 || B <= 0 || Ho <= 0 || Wo <= 0 || Cout <= 0 || Cin_p <= 0 ||
      Cin_p % 16 || stride <= 0)
    return fail(CF_ERR_INVALID_ARG, "bad geometry query");
  Geometry g{};
  if (int rc = make_geometry(T, B, Ho, Wo, Cout, Cin_p, stride, sparse, g, nplanes)) return rc;
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
                          hard_reset, decay_input, 1, static_cast<cudaStream_t>(stream));
}

int cf_conv_bn_lif_split(const void* x, const void* wp2, const float* scale, const float* shift,
                         const void* identity, int res_mode, const float* v_in, float* v_out,
                         void* out, const uint32_t* tile_mask, int64_t T, int64_t B, int64_t H,
                         int64_t W, int64_t Cin_p, int64_t Cout, int64_t KH, int64_t KW,
                         int64_t stride, int64_t pad, float tau, float v_threshold, float v_reset,
                         int hard_reset, int decay_input, void* stream) {
  return conv_bn_lif_impl(x, wp2, scale, shift, identity, res_mode, v_in, v_out, out, tile_mask, T,
                          B, H, W, Cin_p, Cout, KH, KW, stride, pad, tau, v_threshold, v_reset,
                          hard_reset, decay_input, 2, static_cast<cudaStream_t>(stream));
}

int cf_conv_bn_lif_egd(const void* x, const void* wp, const float* scale, const float* shift,
                       const void* identity, int res_mode, const float* v_in, float* v_out,
                       void* out, const uint32_t* tile_mask, int64_t T, int64_t B, int64_t H,
                       int64_t W, int64_t Cin_p, int64_t Cout, int64_t KH, int64_t KW,
                       int64_t stride, int64_t pad, float tau, float v_threshold, float v_reset,
                       int hard_reset, int decay_input, float max_active_frac, void* stream) {
  if (!tile_mask) return fail(CF_ERR_INVALID_ARG, "the device dispatch needs the tile masks");
  if (!(max_active_frac >= 0.f)) return fail(CF_ERR_INVALID_ARG, "max_active_frac must be >= 0");
  return conv_bn_lif_impl(x, wp, scale, shift, identity, res_mode, v_in, v_out, out, tile_mask, T,
                          B, H, W, Cin_p, Cout, KH, KW, stride, pad, tau, v_threshold, v_reset,
                          hard_reset, decay_input, 1, static_cast<cudaStream_t>(stream),
                          max_active_frac);
}

int cf_conv_bn_lif_dual(const void* x, const void* wp, const float* scale, const float* shift,
                        const float* v_in, float* v_out, void* out, const float* v_in2,
                        float* v_out2, void* out2, int64_t Cout1, int64_t T, int64_t B, int64_t H,
                        int64_t W, int64_t Cin_p, int64_t Cout, int64_t KH, int64_t KW,
                        int64_t stride, int64_t pad, float tau, float v_threshold, float v_reset,
                        int hard_reset, int decay_input, void* stream) {
  if (Cout1 <= 0 || Cout1 >= Cout) return fail(CF_ERR_INVALID_ARG, "need 0 < Cout1 < Cout");
  if (T > 8 && !v_out2) return fail(CF_ERR_INVALID_ARG, "T > 8 needs v_out2 to carry the membrane");
  return conv_bn_lif_impl(x, wp, scale, shift, nullptr, CF_RES_NONE, v_in, v_out, out, nullptr, T,
                          B, H, W, Cin_p, Cout, KH, KW, stride, pad, tau, v_threshold, v_reset,
                          hard_reset, decay_input, 1, static_cast<cudaStream_t>(stream), -1.f,
                          Cout1, out2, v_in2, v_out2);
}

int cf_conv_bn_lif_planes(const void* x, const void* wq, const float* scale, const float* shift,
                          const void* identity, int res_mode, const float* v_in, float* v_out,
                          void* out, int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin_p,
                          int64_t Cout, int64_t KH, int64_t KW, int64_t stride, int64_t pad,
                          float tau, float v_threshold, float v_reset, int hard_reset,
                          int decay_input, void* stream) {
  return conv_bn_lif_impl(x, wq, scale, shift, identity, res_mode, v_in, v_out, out, nullptr, T,
                          B, H, W, Cin_p, Cout, KH, KW, stride, pad, tau, v_threshold, v_reset,
                          hard_reset, decay_input, 3, static_cast<cudaStream_t>(stream));
}

int cf_linear_bn_lif(const void* x, const void* w, const float* scale, const float* shift,
                     const void* identity, int res_mode, const float* v_in, float* v_out,
                     void* out, int64_t T, int64_t B, int64_t L, int64_t Cin_p, int64_t Cout,
                     float tau, float v_threshold, float v_reset, int hard_reset, int decay_input,
                     void* stream) {
  // Tokens are pixels of an L x 1 map: a 1x1 convolution.
  return conv_bn_lif_impl(x, w, scale, shift, identity, res_mode, v_in, v_out, out, nullptr, T, B,
                          L, 1, Cin_p, Cout, 1, 1, 1, 0, tau, v_threshold, v_reset, hard_reset,
                          decay_input, 1, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
