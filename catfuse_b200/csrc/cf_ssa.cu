// cf_ssa.cu — Spikformer spiking self-attention (SSA) core fused with its
// attention LIF: y_t = (q_t k_t^T * scale) v_t per head, then a multi-step LIF
// over t.  Replaces the matmul/matmul/attn_lif sequence of SSA.forward
// (models/spikformer_github.py:147-153 in the reference).
//
// q, k, v are spike tensors {0,1} (outputs of Linear->BN->LIF), so the
// attention is integer arithmetic: with bit rows q_i, k_j, v_j over the head
// dimension,  sum_j (q_i . k_j) v_jd  =  sum_e q_ie M_ed  with  M = K^T V,
// M_ed = popcount(kcol_e & vcol_d) over the tokens.  Both sides are exact
// integers (<= N * head_dim), so y = O * scale is one correctly rounded fp32
// product per element.  (The reference rounds every attention entry to fp32
// and sums the rounded terms; the two differ by a few ulp of y.)
//
// Layout: q, k, v, out [B][N][T][C] fp16 (token-major, time, channels: the
// layout of cf_linear_bn_lif), C = heads * head_dim; v_in / v_out [B][N][C]
// fp32 (StateCarry of the attention LIF).  One CTA per (batch, head), one
// thread per (token, 8 channels of the head), loop over t with the membranes
// in registers; the inputs of four steps load together.  Any nonzero input
// value counts as a spike.
#include "cf_common.cuh"

namespace cf {
namespace {

constexpr int kSsaMaxN = 64;   // tokens per head: bit columns are one uint64
constexpr int kSsaMaxD = 32;   // head dim: bit rows are one uint32

__device__ __forceinline__ uint32_t spike_bits8(uint4 q) {
  // 8 fp16 values -> 8 bits (value != 0)
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (w[i] & 0x7FFFu) m |= 1u << (2 * i);
    if (w[i] & 0x7FFF0000u) m |= 1u << (2 * i + 1);
  }
  return m;
}

constexpr int kSsaThreads = 256;
constexpr int kSsaTC = kSsaThreads / kSsaMaxN;  // time steps whose inputs load together

__global__ void __launch_bounds__(kSsaThreads) ssa_lif_kernel(
    const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
    __half* __restrict__ out, const float* v_in, float* v_out, int T, int B, int N, int C,
    int heads, float scale, LifParams lp) {
  const int d = C / heads;
  const int G = d / 8;  // 8-channel groups per head
  const int b = blockIdx.x / heads, h = blockIdx.x - (blockIdx.x / heads) * heads;
  __shared__ uint32_t s_q[kSsaTC][kSsaMaxN];
  __shared__ uint32_t s_kc[kSsaTC][kSsaMaxD][2];  // token bit columns (two 32-token halves)
  __shared__ uint32_t s_vc[kSsaTC][kSsaMaxD][2];
  __shared__ __align__(16) int s_m[kSsaTC][kSsaMaxD][kSsaMaxD];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int i = tid / G, g = tid - (tid / G) * G;  // output token, channel group
  const bool owner = i < N;
  const int64_t col = (int64_t)h * d + g * 8;

  float vm[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) vm[c] = 0.f;
  if (owner && v_in) {
    const float4* src = reinterpret_cast<const float4*>(v_in + ((int64_t)b * N + i) * C + col);
    const float4 a0 = src[0], a1 = src[1];
    vm[0] = a0.x; vm[1] = a0.y; vm[2] = a0.z; vm[3] = a0.w;
    vm[4] = a1.x; vm[5] = a1.y; vm[6] = a1.z; vm[7] = a1.w;
  }

  for (int t0 = 0; t0 < T; t0 += kSsaTC) {
    // 1. bit rows of q, k, v: thread (tt, n) loads token n of step t0 + tt;
    //    each warp holds 32 tokens of one step and ballots the bit columns.
    {
      const int tt = tid / kSsaMaxN, n = tid - tt * kSsaMaxN;
      const int t = t0 + tt;
      uint32_t qr = 0, kr = 0, vr = 0;
      if (n < N && t < T) {
        // all (up to 12) 16-byte loads first, then the bit extraction
        const int64_t off = (((int64_t)b * N + n) * T + t) * C + (int64_t)h * d;
        uint4 rq[kSsaMaxD / 8], rk[kSsaMaxD / 8], rv[kSsaMaxD / 8];
#pragma unroll
        for (int gg = 0; gg < kSsaMaxD / 8; ++gg) {
          if (gg < G) {
            rq[gg] = reinterpret_cast<const uint4*>(q + off)[gg];
            rk[gg] = reinterpret_cast<const uint4*>(k + off)[gg];
            rv[gg] = reinterpret_cast<const uint4*>(v + off)[gg];
          }
        }
#pragma unroll
        for (int gg = 0; gg < kSsaMaxD / 8; ++gg) {
          if (gg < G) {
            qr |= spike_bits8(rq[gg]) << (8 * gg);
            kr |= spike_bits8(rk[gg]) << (8 * gg);
            vr |= spike_bits8(rv[gg]) << (8 * gg);
          }
        }
      }
      s_q[tt][n] = qr;
      for (int e = 0; e < d; ++e) {
        const uint32_t kb = __ballot_sync(0xffffffffu, (kr >> e) & 1u);
        const uint32_t vb = __ballot_sync(0xffffffffu, (vr >> e) & 1u);
        if (lane == 0) {
          s_kc[tt][e][n >> 5] = kb;
          s_vc[tt][e][n >> 5] = vb;
        }
      }
    }
    __syncthreads();
    // 2. M_t = K_t^T V_t (integers) for the loaded steps
    for (int x = tid; x < kSsaTC * d * d; x += kSsaThreads) {
      const int tt = x / (d * d), r = x - tt * d * d;
      const int e = r / d, dd = r - (r / d) * d;
      s_m[tt][e][dd] = __popc(s_kc[tt][e][0] & s_vc[tt][dd][0]) +
                       __popc(s_kc[tt][e][1] & s_vc[tt][dd][1]);
    }
    __syncthreads();
    // 3. per step: O = Q M, y = O * scale, LIF (membranes in registers),
    //    16-byte spike stores
    if (owner) {
      for (int tt = 0; tt < kSsaTC && t0 + tt < T; ++tt) {
        const uint32_t qi = s_q[tt][i];
        int acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int e = 0; e < d; ++e) {
          if ((qi >> e) & 1u) {
            const int4 m0 = *reinterpret_cast<const int4*>(&s_m[tt][e][g * 8]);
            const int4 m1 = *reinterpret_cast<const int4*>(&s_m[tt][e][g * 8 + 4]);
            acc[0] += m0.x; acc[1] += m0.y; acc[2] += m0.z; acc[3] += m0.w;
            acc[4] += m1.x; acc[5] += m1.y; acc[6] += m1.z; acc[7] += m1.w;
          }
        }
        __align__(16) __half o[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float y = __fmul_rn((float)acc[c], scale);
          o[c] = __float2half_rn(lif_step(vm[c], y, lp));
        }
        *reinterpret_cast<uint4*>(out + (((int64_t)b * N + i) * T + t0 + tt) * C + col) =
            *reinterpret_cast<const uint4*>(o);
      }
    }
    __syncthreads();  // the bit rows and M are rebuilt for the next steps
  }
  if (owner && v_out) {
    float4* dst = reinterpret_cast<float4*>(v_out + ((int64_t)b * N + i) * C + col);
    dst[0] = make_float4(vm[0], vm[1], vm[2], vm[3]);
    dst[1] = make_float4(vm[4], vm[5], vm[6], vm[7]);
  }
}

}  // namespace
}  // namespace cf

using namespace cf;

extern "C" int cf_ssa_lif(const void* q, const void* k, const void* v, void* out,
                          const float* v_in, float* v_out, int64_t T, int64_t B, int64_t N,
                          int64_t C, int64_t heads, float scale, float tau, float v_threshold,
                          float v_reset, int hard_reset, int decay_input, void* stream) {
  if (!q || !k || !v || !out) return fail(CF_ERR_INVALID_ARG, "q, k, v and out must not be NULL");
  if (T <= 0 || B <= 0 || N <= 0 || C <= 0 || heads <= 0 || C % heads)
    return fail(CF_ERR_INVALID_ARG, "bad SSA shape (C must be a multiple of heads)");
  const int64_t d = C / heads;
  if (N > kSsaMaxN || d > kSsaMaxD || d % 8)
    return fail(CF_ERR_UNSUPPORTED, "SSA supports N <= %d tokens and head_dim in {8,16,24,32}",
                kSsaMaxN);
  if (!(tau > 0.f)) return fail(CF_ERR_INVALID_ARG, "tau must be > 0");
  const void* ptrs[] = {q, k, v, out, v_in, v_out};
  for (const void* p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) & 15))
      return fail(CF_ERR_UNSUPPORTED, "tensor pointers must be 16-byte aligned");
  if (B * heads > 0x7FFFFFFF) return fail(CF_ERR_UNSUPPORTED, "B * heads too large");
  if (int rc = require_sm100()) return rc;
  ssa_lif_kernel<<<(unsigned)(B * heads), kSsaThreads, 0,
                   static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(q), static_cast<const __half*>(k),
      static_cast<const __half*>(v), static_cast<__half*>(out), v_in, v_out, (int)T, (int)B,
      (int)N, (int)C, (int)heads, scale, make_lif(tau, v_threshold, v_reset, hard_reset, decay_input));
  return check_launch("ssa launch");
}
