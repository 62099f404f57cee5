/*
 * catfuse_b200.h — C ABI of the B200-native (sm_100a) multi-step SNN inference
 * kernels.  Every entry point:
 *   - takes raw device pointers, sizes and scalars (no framework types);
 *   - is stream-ordered on the `stream` argument (a cudaStream_t, passed as
 *     void* so this header needs no CUDA include; NULL = legacy default stream);
 *   - never allocates device memory and never synchronises the host;
 *   - returns CF_OK (0) or a negative CF_ERR_* code; the message of the last
 *     failure on the calling thread is available through cf_get_last_error().
 * The device is the current CUDA device of the calling thread.
 *
 * Tensor layouts used by the fused conv path ("pixel-major, time-inner"):
 *   activations  [B][H][W][T][C]   fp16 (spike counts {0,1,2,...} are exact)
 *   membrane v   [B][H][W][C]      fp32
 *   conv weights [Cout][KH][KW][Cin_p] fp16, Cin_p = Cin rounded up to 16
 * The LIF-family kernels use the reference's own layout [T][B][C][H][W]
 * (flattened as [T][N] with N = B*C*H*W).
 *
 * LIF semantics (SpikingJelly LIFNode, multi-step, as reproduced by CATFuse):
 *   decay_input: h = v + (z - (v - v_reset)) / tau
 *   otherwise  : h = v - (v - v_reset) / tau + z
 *   spike s = (h >= v_threshold)
 *   hard reset : v = s ? v_reset : h        soft reset: v = h - s * v_threshold
 */
#ifndef CATFUSE_B200_H
#define CATFUSE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CF_API __attribute__((visibility("default")))
#else
#define CF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define CF_OK               0
#define CF_ERR_INVALID_ARG (-1)   /* null pointer, bad size, bad enum      */
#define CF_ERR_UNSUPPORTED (-2)   /* shape/alignment this build can't run  */
#define CF_ERR_CUDA        (-3)   /* a CUDA runtime/driver call failed     */
#define CF_ERR_NO_DEVICE   (-4)   /* no sm_100 device is current           */
#define CF_ERR_DEVICE_TIMEOUT (-5)/* a bounded device-side wait expired    */

/* ---- element formats ---------------------------------------------------- */
#define CF_FMT_F32  0   /* float32                                       */
#define CF_FMT_F16  1   /* float16                                       */
#define CF_FMT_U8   2   /* uint8 (spikes / spike counts)                  */
#define CF_FMT_BITS 3   /* bit-packed spikes: bit (i%32) of word i/32     */

/* ---- residual modes of the fused conv epilogue -------------------------- */
#define CF_RES_NONE      0  /* out = s                                      */
#define CF_RES_ADD_POST  1  /* SEW 'ADD' : out = identity + s               */
#define CF_RES_AND_POST  2  /* SEW 'AND' : out = identity * s               */
#define CF_RES_IAND_POST 3  /* SEW 'IAND': out = identity * (1 - s)         */
#define CF_RES_ADD_PRE   4  /* Spiking-ResNet: z += identity before the LIF */
#define CF_RES_Z_ONLY    5  /* no LIF: out = BN(conv(x)) (a Conv+BN branch)  */

/* ---- library / error ---------------------------------------------------- */
CF_API const char* cf_version(void);
/* Copies the last error message of this thread into buf (always
 * NUL-terminated) and returns its full length. */
CF_API size_t cf_get_last_error(char* buf, size_t buf_len);
/* 1 if the current device is sm_100 (B200-class), 0 otherwise. */
CF_API int cf_device_supported(void);
/* Reads and clears the device-side error word that bounded waits inside the
 * kernels set on expiry (synchronises `stream`). Returns CF_OK, or
 * CF_ERR_DEVICE_TIMEOUT with *code = the recorded site. */
CF_API int cf_check_device_error(void* stream, int32_t* code);

/* ---- bandwidth-bound LIF family (reference layout [T][N]) --------------- */

/* Multi-step LIF over z[T][N].  Replaces `lif_sequential`
 * (catfuse/sparseflow/lif_seq_kernel.py:51-90) and `lif_fwd_kernel`
 * (catfuse/kernels/lif_fwd.py:39-72).  z_fmt: CF_FMT_F32 or CF_FMT_F16.
 * v0 may be NULL (v0 = 0).  vT may be NULL (final v not stored).
 * spike_fmt: F32 / F16 / U8 / BITS (BITS requires N % 32 == 0). */
CF_API int cf_lif_fwd(const void* z, int z_fmt, const float* v0,
               void* spikes, int spike_fmt, float* vT,
               int64_t T, int64_t N,
               float tau, float v_threshold, float v_reset,
               int hard_reset, int decay_input, void* stream);

/* Per-channel affine + LIF over z[T][B][C][HW]:  z' = z*scale[c] + shift[c]
 * (+ identity when identity != NULL).  z == NULL means z == 0 (StaticZero:
 * z' = shift).  Replaces `_bn_lif_state_carry_kernel`
 * (catfuse/kernels/partial_fusion_conv_bn_lif_impl.py:110-154),
 * `_bn_add_lif_state_carry_kernel`
 * (catfuse/kernels/partial_fusion_conv_bn_add_lif_impl.py:76-123) and
 * `static_zero_forward` (catfuse/implementations/base.py:250-308).
 * scale may be NULL (=1).  identity_fmt: F32 or F16. */
CF_API int cf_bn_lif(const void* z, int z_fmt, const float* scale, const float* shift,
              const void* identity, int identity_fmt,
              const float* v0, void* spikes, int spike_fmt, float* vT,
              int64_t T, int64_t B, int64_t C, int64_t HW,
              float tau, float v_threshold, float v_reset,
              int hard_reset, int decay_input, void* stream);

/* z = x1 + x2, then LIF.  Replaces `add_lif_block_kernel`
 * (catfuse/kernels/add_lif.py:63-110). x1/x2 fp32 [T][N]. */
CF_API int cf_add_lif(const float* x1, const float* x2, const float* v0,
               void* spikes, int spike_fmt, float* vT, int64_t T, int64_t N,
               float tau, float v_threshold, float v_reset,
               int hard_reset, int decay_input, void* stream);

/* k x k / stride k average pool over x[T][B][C][H][W] (fp32), then LIF on the
 * pooled map [T][B][C][H/k][W/k].  Replaces `avgpool_lif_block_kernel`
 * (catfuse/kernels/avgpool_lif.py:61-145).  H and W must be multiples of k. */
CF_API int cf_avgpool_lif(const float* x, const float* v0, void* spikes, int spike_fmt,
                   float* vT, int64_t T, int64_t B, int64_t C, int64_t H,
                   int64_t W, int k, float tau, float v_threshold,
                   float v_reset, int hard_reset, int decay_input,
                   void* stream);

/* ---- layout conversion ---------------------------------------------------- */

/* x[T][B][C][H][W] (fp32 or fp16) -> y[B][H][W][T][Cp] fp16, channels
 * C..Cp-1 zero-filled.  Cp >= C, Cp % 16 == 0. */
CF_API int cf_pack_tbchw(const void* x, int x_fmt, void* y, int64_t T, int64_t B,
                  int64_t C, int64_t H, int64_t W, int64_t Cp, void* stream);
/* im2col for a k x k convolution with few input channels (the stem):
 * x[T][B][C][H][W] (fp32/fp16) -> y[B][Ho][Wo][T][Kp] fp16 with
 * y[..][q] = x[t][b][c][ho*stride-pad+kh][wo*stride-pad+kw], q = (kh*k+kw)*C+c,
 * zero outside the image and for q >= k*k*C.  The convolution then runs as a
 * 1x1 convolution with Cin_p = Kp (one K chunk per tile instead of k*k). */
CF_API int cf_pack_im2col(const void* x, int x_fmt, void* y, int64_t T, int64_t B, int64_t C,
                          int64_t H, int64_t W, int64_t k, int64_t stride, int64_t pad,
                          int64_t Kp, void* stream);
/* y[B][H][W][T][C] fp16 -> x[T][B][C][H][W] (fp32 or fp16). */
CF_API int cf_unpack_bhwtc(const void* y, void* x, int x_fmt, int64_t T, int64_t B,
                    int64_t C, int64_t H, int64_t W, void* stream);
/* v[B][C][H][W] <-> v[B][H][W][C], fp32.  to_nhwc = 1: NCHW -> NHWC. */
CF_API int cf_v_layout(const float* src, float* dst, int64_t B, int64_t C,
                int64_t H, int64_t W, int to_nhwc, void* stream);
/* w[Cout][Cin][KH][KW] fp32 -> wp[Cout][KH][KW][Cin_p] fp16 (zero-padded).
 * Replaces SparseFlow's `_ensure_w_cl`
 * (catfuse/implementations/sparse_flow.py:92-99). */
CF_API int cf_pack_conv_weight(const float* w, void* wp, int64_t Cout, int64_t Cin,
                        int64_t KH, int64_t KW, int64_t Cin_p, void* stream);

/* ---- fused Conv -> BN -> LIF on tcgen05 ----------------------------------- */

/* Tile geometry of cf_conv_bn_lif for a shape; lets the caller size the
 * per-tile mask buffer.  out[0..5] = {Tp, Wb, Hb, Bb, n_mtiles, BN}.
 * cf_conv_geometry assumes Cin_p = 64, stride 1 and dense chunks; the tile
 * choice depends on Cin_p, so callers that know it use cf_conv_geometry_ex
 * (same output, the arguments cf_conv_bn_lif / cf_prescan_conv_tiles get).
 * flags: bit 0 = sparse (tile-mask launch), bit 1 = integer weight planes
 * (cf_conv_bn_lif_planes). */
CF_API int cf_conv_geometry(int64_t T, int64_t B, int64_t Ho, int64_t Wo,
                     int64_t Cout, int32_t* out6);
CF_API int cf_conv_geometry_ex(int64_t T, int64_t B, int64_t Ho, int64_t Wo, int64_t Cout,
                               int64_t Cin_p, int64_t stride, int flags, int32_t* out6);

/* Implicit-GEMM convolution on the 5th-generation tensor cores (fp16
 * operands, fp32 accumulation in TMEM) with the BN affine, the optional
 * residual and the multi-step LIF in the epilogue, looping over all time
 * steps inside the kernel (z and v never reach HBM).
 *   x        [B][H][W][T][Cin_p] fp16
 *   wp       [Cout][KH][KW][Cin_p] fp16 (cf_pack_conv_weight)
 *   scale/shift [Cout] fp32: z' = acc*scale + shift (scale NULL = 1)
 *   identity [B][Ho][Wo][T][Cout] fp16 or NULL (see CF_RES_*)
 *   v_in / v_out [B][Ho][Wo][Cout] fp32, either may be NULL (v_in NULL: v0=0);
 *            v_in == v_out is allowed (in-place StateCarry)
 *   out      [B][Ho][Wo][T][Cout] fp16
 *   tile_mask per-M-tile bit mask of active input channel chunks
 *            (cf_prescan_conv_tiles) or NULL (dense: DenseKeep).  A tile whose
 *            mask is 0 runs no MMA at all (StaticZero for that tile).
 * Replaces DenseKeep.forward (catfuse/implementations/dense_keep.py:97-155),
 * SparseFlow.forward + `sparse_streamfuse_conv3x3_bn_lif`
 * (catfuse/implementations/sparse_flow.py:186-270,
 *  catfuse/sparseflow/streamfuse_kernel.py:32-187) and the per-step
 * `fused_bm_conv3x3_bn_lif_8x8/8x16`
 * (catfuse/sparseflow/fused_conv_bn_lif_kernel.py:63-335).
 * Requirements: Cin_p % 16 == 0, Cout % 32 == 0, 1 <= T. */
CF_API int cf_conv_bn_lif(const void* x, const void* wp, const float* scale,
                   const float* shift, const void* identity, int res_mode,
                   const float* v_in, float* v_out, void* out,
                   const uint32_t* tile_mask,
                   int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin_p,
                   int64_t Cout, int64_t KH, int64_t KW, int64_t stride,
                   int64_t pad, float tau, float v_threshold, float v_reset,
                   int hard_reset, int decay_input, void* stream);

/* Spikformer spiking self-attention core + attention LIF: per head,
 * y_t = (q_t k_t^T * scale) v_t, then the multi-step LIF over t.  q, k, v, out
 * [B][N][T][C] fp16 spikes (the layout of cf_linear_bn_lif; any nonzero value
 * is a spike), C = heads * head_dim, head_dim in {8,16,24,32}, N <= 64;
 * v_in / v_out [B][N][C] fp32 (may be NULL; may alias).  Computed exactly as
 * scale * (Q (K^T V)) in integers, one fp32 rounding per element.  Replaces
 * the two matmuls and attn_lif of SSA.forward
 * (models/spikformer_github.py:147-153). */
CF_API int cf_ssa_lif(const void* q, const void* k, const void* v, void* out,
                      const float* v_in, float* v_out, int64_t T, int64_t B, int64_t N,
                      int64_t C, int64_t heads, float scale, float tau, float v_threshold,
                      float v_reset, int hard_reset, int decay_input, void* stream);

/* Linear -> (BN1d) -> LIF over tokens: x [B][L][T][Cin_p] fp16,
 * w [Cout][Cin_p] fp16, out [B][L][T][Cout] fp16.  A 1x1 convolution on the
 * same tensor-core kernel.  Replaces FusedLinearLIF
 * (catfuse/patterns.py:493-596) and `linear_lif_block_kernel`
 * (catfuse/kernels/linear_lif.py:51-102). */
CF_API int cf_linear_bn_lif(const void* x, const void* w, const float* scale,
                     const float* shift, const void* identity, int res_mode,
                     const float* v_in, float* v_out, void* out,
                     int64_t T, int64_t B, int64_t L, int64_t Cin_p,
                     int64_t Cout, float tau, float v_threshold,
                     float v_reset, int hard_reset, int decay_input,
                     void* stream);

/* ---- SparseFlow prescan ---------------------------------------------------- */

/* Receptive-field prescan with the reference's geometry over x[N][C][H][W]
 * (N = T*B): bit g of ag_mask[n][gh][gw] is 1 iff some |x| > threshold in
 * channels [g*GS, (g+1)*GS) of the receptive field of the tile's valid output
 * pixels; tile_class = 0 (mask 0), 2 (all groups), else 1; nnz_out (int64,
 * may be NULL) receives the number of nonzero elements of x (atomically
 * accumulated: the caller zeroes it).  Replaces
 * `fast_spike_prescan_2d_v2` (catfuse/sparseflow/fast_prescan_v2.py:92-137)
 * and `build_rf_prescan_metadata` (catfuse/sparseflow/prescan.py:153-189).
 * x_fmt: F32 / F16 / U8.  NUM_GROUPS = ceil(C/GS) must be <= 32. */
CF_API int cf_prescan(const void* x, int x_fmt, int32_t* ag_mask, int32_t* tile_class,
               int64_t* nnz_out, int64_t N, int64_t C, int64_t H, int64_t W,
               int64_t H_out, int64_t W_out, int64_t k, int64_t stride,
               int64_t pad, int64_t BH, int64_t BW, int64_t GS,
               float threshold, void* stream);

/* Prescan in the fused conv kernel's own tile geometry over
 * x[B][H][W][T][Cin_p] fp16: mask[m] bit c = 1 iff a nonzero exists in input
 * channel chunk c (chunk = `chunk` channels) of M-tile m's receptive field,
 * over the tile's time steps.  nnz_out as for cf_prescan (may be NULL). */
CF_API int cf_prescan_conv_tiles(const void* x, uint32_t* mask, int64_t* nnz_out,
                          int64_t T, int64_t B, int64_t H, int64_t W,
                          int64_t Cin_p, int64_t Cout, int64_t KH, int64_t KW,
                          int64_t stride, int64_t pad, int64_t chunk,
                          void* stream);
/* Channel chunk the conv kernel uses for a given Cin_p in sparse mode. */
CF_API int cf_conv_chunk(int64_t Cin_p, int sparse);

/* Max pool (k, stride, pad; padding never wins) over x[B][H][W][T][C] fp16
 * -> y[B][Ho][Wo][T][C].  The ResNet stem max-pool on spikes.  C % 8 == 0. */
CF_API int cf_maxpool_bhwtc(const void* x, void* y, int64_t B, int64_t H, int64_t W,
                            int64_t T, int64_t C, int64_t k, int64_t stride, int64_t pad,
                            void* stream);

/* cf_conv_bn_lif with SparseFlow / DenseKeep chosen on the device: the
 * kernel counts the active (tile, chunk) pairs of `tile_mask`
 * (cf_prescan_conv_tiles) before its pipeline starts and runs the masks only
 * if at most max_active_frac of all pairs are active, otherwise every chunk of
 * every tile (an all-zero input leaves every mask empty: StaticZero).  The
 * masks use the dense channel chunk: cf_prescan_conv_tiles with
 * chunk = cf_conv_chunk(Cin_p, 0).  No host
 * synchronisation, so it can sit inside a CUDA graph.  The result is the same
 * bit for bit either way; only the speed differs.  Replaces the runtime EGD of
 * STFusionConvBNLIF.forward (catfuse/sparseflow/ops/st_fusion_conv_bn_lif.py:
 * 510-524: sparsity = 1 - nnz/numel read on the host, > 0.7 -> SparseFlow),
 * with the measured work (active pairs) in place of the element count. */
CF_API int cf_conv_bn_lif_egd(const void* x, const void* wp, const float* scale,
                              const float* shift, const void* identity, int res_mode,
                              const float* v_in, float* v_out, void* out,
                              const uint32_t* tile_mask,
                              int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin_p,
                              int64_t Cout, int64_t KH, int64_t KW, int64_t stride,
                              int64_t pad, float tau, float v_threshold, float v_reset,
                              int hard_reset, int decay_input, float max_active_frac,
                              void* stream);

/* cf_conv_bn_lif_egd with its prescan, for callers that cannot allocate
 * device memory (a host framework whose allocator owns the device and passes
 * in only a call's tensors, or a hot path under a no-allocation rule): it
 * runs cf_prescan_conv_tiles (dense chunk) into a mask array that this
 * library holds in device memory, then cf_conv_bn_lif_egd on those masks.
 * No counterpart in the reference (its SparseFlow allocates the prescan's
 * outputs with torch on every call).
 *   - Limit: at most 65536 M tiles (cf_conv_geometry_ex with flags = 1, out[4]);
 *     larger shapes return CF_ERR_UNSUPPORTED.  The array takes 256 KB on
 *     every GPU that loads the library, until the process exits.
 *   - It calls no cudaMalloc / cudaFree.  Its first call on a device looks up
 *     the array's device address (cudaGetSymbolAddress) with that device
 *     current; make that first call before any stream capture.
 *   - Every call shares the one array: calls whose kernels overlap on the GPU
 *     (different streams without ordering) race on it.  Calls ordered on one
 *     stream are safe; the prescan clears the masks it uses on each call.
 * Arguments as cf_conv_bn_lif_egd without tile_mask; the result is bit for
 * bit that of cf_prescan_conv_tiles + cf_conv_bn_lif_egd. */
CF_API int cf_conv_bn_lif_egd_noalloc(const void* x, const void* wp, const float* scale,
                                      const float* shift, const void* identity, int res_mode,
                                      const float* v_in, float* v_out, void* out,
                                      int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin_p,
                                      int64_t Cout, int64_t KH, int64_t KW, int64_t stride,
                                      int64_t pad, float tau, float v_threshold, float v_reset,
                                      int hard_reset, int decay_input, float max_active_frac,
                                      void* stream);

/* Two convolutions over the same input in one launch: output channels
 * [0, Cout1) are written to out / v_in / v_out ([B][Ho][Wo][T][Cout1],
 * [B][Ho][Wo][Cout1]) and [Cout1, Cout) to out2 / v_in2 / v_out2 (Cout - Cout1
 * channels wide); wp / scale / shift hold both convs' rows.  A SEW block's
 * 1x1 stride-s downsample conv (+BN+LIF) rides along its 3x3 stride-s first
 * conv this way: its weights sit at the centre tap of a 3x3 slab (the centre
 * tap of a pad-1 3x3 conv reads exactly the pixel a pad-0 1x1 conv reads), so
 * the input is read once for both (catfuse/patterns.py:676-715: conv1 and
 * downsample of the same block).  Channel-major shapes only, Cout1 a multiple
 * of the output-channel tile, no residual, no mask, fp16 weights. */
CF_API int cf_conv_bn_lif_dual(const void* x, const void* wp, const float* scale,
                               const float* shift, const float* v_in, float* v_out, void* out,
                               const float* v_in2, float* v_out2, void* out2, int64_t Cout1,
                               int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin_p,
                               int64_t Cout, int64_t KH, int64_t KW, int64_t stride,
                               int64_t pad, float tau, float v_threshold, float v_reset,
                               int hard_reset, int decay_input, void* stream);

/* Extended-precision variant of cf_conv_bn_lif: the weight is carried as two
 * fp16 parts, wp2[Cout][KH][KW][2][Cin_p] = {hi, lo} (cf_pack_conv_weight_split),
 * and every (tap, channel chunk) issues the hi and the lo MMAs into the same
 * fp32 TMEM accumulator, so the conv sums x * (hi + lo) with 22 significant
 * weight bits (fp32-faithful for spike inputs, which fp16 holds exactly; a
 * real-valued stem input is split the same way by cf_pack_im2col_split).
 * Twice the MMA work of cf_conv_bn_lif; same arguments otherwise, with `scale`
 * already divided by the prescale the weights were packed with.  Serves the
 * fp32 reference path of DenseKeep (catfuse/implementations/dense_keep.py:97-155,
 * cuDNN fp32 conv) where fp16 weight rounding is not acceptable. */
CF_API int cf_conv_bn_lif_split(const void* x, const void* wp2, const float* scale,
                                const float* shift, const void* identity, int res_mode,
                                const float* v_in, float* v_out, void* out,
                                const uint32_t* tile_mask,
                                int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin_p,
                                int64_t Cout, int64_t KH, int64_t KW, int64_t stride,
                                int64_t pad, float tau, float v_threshold, float v_reset,
                                int hard_reset, int decay_input, void* stream);
/* w[Cout][Cin][KH][KW] fp32 -> wp2[Cout][KH][KW][2][Cin_p] fp16 with
 * hi = fp16(w * prescale) and lo = fp16(w * prescale - hi); prescale is a
 * power of two (chosen so that the largest |w * prescale| is near 2^14 and lo
 * stays out of the fp16 subnormal range). */
CF_API int cf_pack_conv_weight_split(const float* w, void* wp2, int64_t Cout, int64_t Cin,
                                     int64_t KH, int64_t KW, int64_t Cin_p, float prescale,
                                     void* stream);
/* cf_pack_im2col for the extended-precision stem: y[..][q] = fp16(v) for
 * q < k*k*C and fp16(v - fp16(v)) of the same element at q + k*k*C
 * (Kp >= 2*k*k*C).  With the weight row [w, w] this gives x*w with both
 * operands carried as hi + lo. */
CF_API int cf_pack_im2col_split(const void* x, int x_fmt, void* y, int64_t T, int64_t B,
                                int64_t C, int64_t H, int64_t W, int64_t k, int64_t stride,
                                int64_t pad, int64_t Kp, void* stream);

/* Exact-accumulation variant for integer activations (spike counts): the
 * weight is quantised to q = rint(w * prescale), |q| < 2^28, and carried as
 * three planes of signed base-1024 digits wq[Cout][KH][KW][3][Cin_p] fp16
 * (cf_pack_conv_weight_planes; most significant plane first).  Each plane is
 * accumulated in its own TMEM accumulator; with |x| <= 2^24 / (512*KH*KW*Cin_p)
 * (e.g. |x| <= 7 at KH*KW*Cin_p = 4608) every partial sum is an integer below
 * 2^24, so the accumulation is exact, and the epilogue joins the planes in
 * fp64 and rounds once: conv = round_fp32(sum x * q), i.e. the convolution with
 * the 29-bit quantised weight, correctly rounded.  `scale` is the BN scale
 * divided by prescale.  Three MMAs per chunk, single-buffered N = 128 tiles;
 * channel-major shapes only (Cout % 128 == 0, or Cout % 64 == 0 with
 * Cin_p >= 64); dense only (no tile mask).  This is the fp32 reference path
 * of DenseKeep (catfuse/implementations/dense_keep.py:97-155) made exact. */
CF_API int cf_conv_bn_lif_planes(const void* x, const void* wq, const float* scale,
                                 const float* shift, const void* identity, int res_mode,
                                 const float* v_in, float* v_out, void* out,
                                 int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin_p,
                                 int64_t Cout, int64_t KH, int64_t KW, int64_t stride,
                                 int64_t pad, float tau, float v_threshold, float v_reset,
                                 int hard_reset, int decay_input, void* stream);
/* w[Cout][Cin][KH][KW] fp32 -> wq[Cout][KH][KW][3][Cin_p] fp16 digit planes of
 * q = rint(w * prescale) (see cf_conv_bn_lif_planes); prescale a power of two
 * with max |w| * prescale < 2^28. */
CF_API int cf_pack_conv_weight_planes(const float* w, void* wq, int64_t Cout, int64_t Cin,
                                      int64_t KH, int64_t KW, int64_t Cin_p, float prescale,
                                      void* stream);

/* ---- bounded device-side waits ------------------------------------------- */

/* Every mbarrier wait inside the fused conv kernel gives up after a bounded
 * number of polls, records a site code in the device error word
 * (cf_check_device_error) and ends the kernel early.  This sets that bound for
 * later launches in this process (0 = the default, 2^24 polls, i.e. seconds).
 * The reference has no counterpart (Triton kernels there have no waits). */
CF_API int cf_set_wait_limit(uint32_t max_polls);
/* Test hook for that expiry path: when armed, the next cf_conv_bn_lif launch
 * has CTA 0's producers skip their first load, so the consumer's wait for it
 * runs out; the kernel ends early and cf_check_device_error reports
 * CF_ERR_DEVICE_TIMEOUT.  One-shot (disarmed by that launch); 0 disarms. */
CF_API int cf_test_arm_stalled_load(int armed);

/* ---- network head ---------------------------------------------------------- */

/* Global average pool over x[B][H][W][T][C] fp16 then fc: logits[T][B][K] =
 * mean_hw(x) @ fc_w[K][C]^T + fc_b (fc_b may be NULL).  The SEW/Spiking
 * ResNet classifier (avgpool -> flatten(2) -> fc). */
CF_API int cf_avgpool_fc(const void* x, const float* fc_w, const float* fc_b,
                  float* logits, int64_t T, int64_t B, int64_t H, int64_t W,
                  int64_t C, int64_t K, void* stream);

/* Spikformer head: token mean over x[B][N][T][C] fp16 (spike counts), the
 * pre-head LIF over t (v_in / v_out [B][C] fp32, either may be NULL), then
 * logits[T][B][K] = s_t @ fc_w[K][C]^T + fc_b (fc_b may be NULL).  Replaces
 * forward_features' y.mean(dim=2) -> pre_head_lif -> head
 * (models/spikformer_github.py:311-329), the avgpool_lif pattern of the
 * reference (catfuse/kernels/avgpool_lif.py:61-145) over the token axis. */
CF_API int cf_token_mean_lif_fc(const void* x, const float* v_in, float* v_out,
                                const float* fc_w, const float* fc_b, float* logits,
                                int64_t T, int64_t B, int64_t N, int64_t C, int64_t K,
                                float tau, float v_threshold, float v_reset, int hard_reset,
                                int decay_input, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CATFUSE_B200_H */
