// cf_common.cuh — shared helpers for the sm_100a kernels: error plumbing,
// LIF arithmetic, and thin inline-PTX wrappers for mbarriers, TMA and tcgen05.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>
#include <cstdarg>

#include "../../include/catfuse_b200.h"

namespace cf {

// ---------------------------------------------------------------------------
// host-side error plumbing
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
int check_launch(const char* what);
int require_sm100();

// Site codes for g_dev_error.
enum : int32_t {
  ERR_SITE_PRODUCER_EMPTY = 1,
  ERR_SITE_MMA_FULL = 2,
  ERR_SITE_MMA_TEMPTY = 3,
  ERR_SITE_EPI_TFULL = 4,
};

// Upper bound on mbarrier polls before a wait gives up (each try_wait already
// suspends for a hardware-defined interval, so this is seconds of waiting).
constexpr uint32_t kMaxPolls = 1u << 24;

// ---------------------------------------------------------------------------
// LIF arithmetic (SpikingJelly multi-step LIFNode semantics).  Explicit
// round-to-nearest intrinsics keep every operation separately rounded, exactly
// as the fp32 CPU formulation evaluates it (no FMA contraction).
// ---------------------------------------------------------------------------
struct LifParams {
  float tau, rtau, v_th, v_reset;
  int hard_reset, decay_input, tau_pow2;
};

__host__ inline LifParams make_lif(float tau, float v_th, float v_reset,
                                   int hard_reset, int decay_input) {
  LifParams p;
  p.tau = tau;
  p.rtau = 1.0f / tau;
  p.v_th = v_th;
  p.v_reset = hard_reset ? v_reset : 0.0f;
  p.hard_reset = hard_reset;
  p.decay_input = decay_input;
  // x / tau == x * (1/tau) exactly (both correctly rounded from the same real
  // value) when tau is a power of two; then the multiply is used.
  int e;
  float m = frexpf(tau, &e);
  p.tau_pow2 = (m == 0.5f) ? 1 : 0;
  return p;
}

__device__ __forceinline__ float lif_div(float x, const LifParams& p) {
  return p.tau_pow2 ? __fmul_rn(x, p.rtau) : __fdiv_rn(x, p.tau);
}

// One LIF step: charge, fire, reset.  Returns the spike (0/1) and updates v.
__device__ __forceinline__ float lif_step(float& v, float z, const LifParams& p) {
  float h;
  if (p.decay_input) {
    // h = v + (z - (v - v_reset)) / tau
    h = __fadd_rn(v, lif_div(__fsub_rn(z, __fsub_rn(v, p.v_reset)), p));
  } else {
    // h = v - (v - v_reset) / tau + z
    h = __fadd_rn(__fsub_rn(v, lif_div(__fsub_rn(v, p.v_reset), p)), z);
  }
  const bool s = h >= p.v_th;
  if (p.hard_reset) {
    v = s ? p.v_reset : h;
  } else {
    v = s ? __fsub_rn(h, p.v_th) : h;
  }
  return s ? 1.0f : 0.0f;
}

// ---------------------------------------------------------------------------
// PTX wrappers (sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Non-blocking probe of an mbarrier phase (no thread suspension).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Suspend-time hint of mbarrier.try_wait, in ns: a thread whose phase is not
// complete sleeps at most this long before it polls again.  Without a hint the
// conv pipeline's producer -> MMA -> producer barrier round trip measured
// ~1.8k cycles on B200; with 200 ns the same pipeline runs 15 % faster and the
// 256->256 28x28 conv layer 7 % faster.
constexpr int kTryWaitHintNs = 200;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
        , "n"(kTryWaitHintNs)
      : "memory");
  return ok != 0;
}

// 2-D / 5-D tiled TMA loads into shared memory, completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* dst, const void* tmap, uint64_t* bar, int c0,
                                            int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch.  griddep_wait blocks until the grid this
// launch depends on has completed and its memory is visible (a no-op when the
// kernel was launched without the programmatic-serialisation attribute);
// griddep_launch_dependents lets the next launch in the stream start its
// CTAs (they run their own set-up, then block in their griddep_wait).
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- tcgen05 -------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16 or bf16 in, fp32 acc).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05 ops of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Load 32 consecutive fp32 columns of this warp's 32 TMEM lanes (lane i of
// the warp receives row i of its lane quarter).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
  uint32_t* u = reinterpret_cast<uint32_t*>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
        "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]),
        "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]),
        "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]),
        "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Load 32 consecutive fp32 columns of 16 TMEM lanes into a full warp: thread
// t receives lane t % 16 of the warp's lane quarter, columns starting at
// taddr's column + (t / 16) * 32 (the accumulator layout of an M=64 MMA puts
// its rows in lanes 0-15 of each quarter).
__device__ __forceinline__ void tmem_ld16x2_32(uint32_t taddr, float (&r)[32]) {
  uint32_t* u = reinterpret_cast<uint32_t*>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32], 32;"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
        "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]),
        "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]),
        "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]),
        "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile whose rows are
// `row_bytes` long (32/64/128) and swizzled with the matching TMA swizzle.
// Eight rows form one swizzle atom; consecutive atoms are 8*row_bytes apart.
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t row_bytes) {
  uint64_t layout = (row_bytes == 128) ? 2ull : (row_bytes == 64 ? 4ull : 6ull);
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);           // start address
  d |= (uint64_t)1 << 16;                             // leading byte offset (unused)
  d |= (uint64_t)(((8u * row_bytes) >> 4) & 0x3FFFu) << 32;  // stride byte offset
  d |= (uint64_t)1 << 46;                             // descriptor version (sm100)
  d |= layout << 61;                                  // swizzle mode
  return d;
}

// Global nanosecond timer (tuning traces).
__device__ __forceinline__ long long globaltimer_ns() {
  long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Instruction descriptor: kind::f16, A/B fp16, K-major both, fp32 accum.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N) {
  return (1u << 4)                          // D format: f32
         | (0u << 7) | (0u << 10)           // A, B format: f16
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

}  // namespace cf
