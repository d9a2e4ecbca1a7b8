// Shared device helpers for the Cortex B200 kernels (sm_100a only).
//
// * status word: every kernel that detects bad input or gives up on a bounded
//   wait records a code in a per-device global word that the host reads back
//   through ck_get_last_status(); no kernel traps or asserts.
// * PTX wrappers for mbarriers, TMA tile loads, and the tcgen05 family
//   (TMEM alloc/dealloc, MMA, commit, TMEM loads, fences).
// * bf16 helpers that reproduce torch's eager rounding points.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cortex_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "cortex-b200 kernels are written for sm_100a only"
#endif

namespace ck {

// Per-device status word (first error wins). Defined in status.cu.
extern __device__ int g_status;
extern __device__ int g_status_info[4];

__device__ __forceinline__ void set_status(int code, int a = 0, int b = 0) {
  if (atomicCAS(&g_status, 0, code) == 0) {
    g_status_info[0] = a;
    g_status_info[1] = b;
    g_status_info[2] = blockIdx.x;
    g_status_info[3] = threadIdx.x;
  }
}

// ── programmatic dependent launch ────────────────────────────────────────────
// Every kernel is launched with programmatic stream serialisation (launch_pdl
// in kernels.h), so it may start while its stream predecessor is still
// running. grid_dep_wait() blocks until the predecessor grid has completed and
// its writes are visible; each kernel calls it before its first global-memory
// read or write (setup that only touches shared memory, TMEM or kernel
// parameters may come first). grid_dep_launch() lets the successor grid be
// scheduled; kernels call it only after any blocking resource acquisition of
// their own (TMEM allocation), so a successor that occupies an SM early can
// never hold a resource a running CTA of this grid still has to acquire. Both
// are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ── bf16 helpers ─────────────────────────────────────────────────────────────

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }
// Round an fp32 value through bf16 and back (torch eager bf16 op output).
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Exact-erf GELU (nn.GELU(approximate='none')).
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

// Erf GELU for epilogues, 0.5 x (1 + erf(x / sqrt 2)), with erf evaluated by
// Abramowitz & Stegun, Handbook of Mathematical Functions (1964), eq. 7.1.28:
//   erf(y) = 1 - (1 + a1 y + a2 y^2 + ... + a6 y^6)^-16 + e(y),  |e| <= 3e-7, y >= 0.
// One reciprocal and a degree-6 polynomial instead of a library erf: the GEMM
// epilogue that applies it stays under the tensor-core time of its tile. The
// result is rounded to bf16 right after, so the 3e-7 bound is far below the
// output resolution for x >= kGeluTail. Below it GELU is tiny and torch's own
// value is 0.5 x (1 + erf) with erf rounded to fp32; callers recompute those
// elements with gelu_erf (see gelu32), which also matches torch there.
constexpr float kGeluTail = -3.0f;

__device__ __forceinline__ float gelu_as(float x) {
  const float y = fminf(fabsf(x) * 0.70710678118654752440f, 1.0e4f);
  float q = fmaf(4.30638e-5f, y, 2.765672e-4f);
  q = fmaf(q, y, 1.520143e-4f);
  q = fmaf(q, y, 9.2705272e-3f);
  q = fmaf(q, y, 4.22820123e-2f);
  q = fmaf(q, y, 7.05230784e-2f);
  q = fmaf(q, y, 1.0f);
  float r = __fdividef(1.0f, q);  // q >= 1
  r = r * r;                      // r^2
  r = r * r;                      // r^4
  r = r * r;                      // r^8
  r = r * r;                      // r^16 = 1 - erf(y)
  const float h = 0.5f * x * r;  // 0.5 x (1 - erf(|x| / sqrt 2))
  return x >= 0.f ? x - h : h;
}

// Paired fp32 arithmetic (sm_100: one instruction for two lanes of a .b64 pair).
__device__ __forceinline__ unsigned long long f2pk(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2up(unsigned long long r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b,
                                                    unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long fadd2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long fmul2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// bf16x2 add, round to nearest even. For bf16 a and b this equals the fp32 sum
// rounded to bf16 (torch's bf16 add): fp32 holds 24 >= 2 * 8 + 2 significand
// bits, so rounding first to fp32 and then to bf16 gives the single rounding.
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// bf16 pair conversions: one cvt for two values (round to nearest even).
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float bf16_lo(uint32_t r) { return __uint_as_float(r << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t r) { return __uint_as_float(r & 0xffff0000u); }
// Round two fp32 values through bf16 (torch's bf16 op output), one conversion.
__device__ __forceinline__ void rbf2(float& a, float& b) {
  const uint32_t r = cvt_bf16x2(a, b);
  a = bf16_lo(r);
  b = bf16_hi(r);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Four int8 values (one 32-bit word, little-endian) to four bf16 values, exact,
// with integer logic and one bf16x2 subtraction per pair, never the conversion
// unit (I2F and F2F issue at a fraction of the FMA rate; with one I2F per
// element and one F2F per pair they made the int8 weight tiles the slowest
// stage of the GEMM pipeline). For a byte v (two's complement), the bf16 with
// exponent 2^7 and mantissa v & 0x7F is 128 + (v & 127), which is 128 + v for
// v >= 0 and 256 + v for v < 0; subtracting the bf16 whose mantissa is the
// sign bit, 128 or 256, leaves v, exactly (every integer of magnitude <= 256
// is a bf16). One byte permute first orders the word (b0, b2, b1, b3), so the
// even / odd 16-bit lanes hold (b0, b1) and (b2, b3), the output pairs.
__device__ __forceinline__ uint32_t sub_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t r = prmt(w, 0u, 0x3120u);  // bytes (b0, b2, b1, b3)
  const uint32_t r8 = r >> 8;               // (b2, ., b3, .) in the low bytes of the halves
  lo = sub_bf16x2((r & 0x007F007Fu) | 0x43004300u, (r & 0x00800080u) | 0x43004300u);
  hi = sub_bf16x2((r8 & 0x007F007Fu) | 0x43004300u, (r8 & 0x00800080u) | 0x43004300u);
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU of 32 values, each >= kGeluTail: the same A&S 7.1.28 evaluation as
// gelu_as, arranged for the issue rate of the epilogue warps. The polynomial
// runs on |x| with its coefficients pre-scaled by 2^(-k/2) (erf's argument is
// x / sqrt 2) and by 2^(1/16), so the 16th power of the reciprocal is
// t = (1 - erf(|x|/sqrt 2)) / 2 directly; then GELU(x) = x Phi(x) =
// x / 2 + |x| (1/2 - t) for either sign of x, with no select. The 16 value
// pairs go through each step together (paired fp32 instructions), so every
// step has 16 independent operations to hide the latency of the previous one.
template <bool KEEP_TAIL = false>
__device__ __forceinline__ void gelu32_pairs(float* v) {
  unsigned long long y[16], q[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) y[i] = f2pk(fabsf(v[2 * i]), fabsf(v[2 * i + 1]));
#pragma unroll
  for (int i = 0; i < 16; ++i)
    q[i] = ffma2(f2pk(5.6212996639622074e-06f, 5.6212996639622074e-06f), y[i],
                 f2pk(5.1055209008659824e-05f, 5.1055209008659824e-05f));
#pragma unroll
  for (int i = 0; i < 16; ++i) q[i] = ffma2(q[i], y[i], f2pk(3.96861370110139e-05f, 3.96861370110139e-05f));
#pragma unroll
  for (int i = 0; i < 16; ++i)
    q[i] = ffma2(q[i], y[i], f2pk(3.422739238900824e-03f, 3.422739238900824e-03f));
#pragma unroll
  for (int i = 0; i < 16; ++i)
    q[i] = ffma2(q[i], y[i], f2pk(2.2076998456581714e-02f, 2.2076998456581714e-02f));
#pragma unroll
  for (int i = 0; i < 16; ++i)
    q[i] = ffma2(q[i], y[i], f2pk(5.207516303663057e-02f, 5.207516303663057e-02f));
#pragma unroll
  for (int i = 0; i < 16; ++i) q[i] = ffma2(q[i], y[i], f2pk(1.0442737824274138f, 1.0442737824274138f));
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float qa, qb;
    f2up(q[i], qa, qb);
    q[i] = f2pk(rcp_approx(qa), rcp_approx(qb));
  }
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int i = 0; i < 16; ++i) q[i] = fmul2(q[i], q[i]);
  const unsigned long long half = f2pk(0.5f, 0.5f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const unsigned long long h = ffma2(q[i], f2pk(-1.f, -1.f), half);  // erf(|x|/sqrt 2) / 2
    float r0, r1;
    f2up(ffma2(y[i], h, fmul2(f2pk(v[2 * i], v[2 * i + 1]), half)), r0, r1);
    // KEEP_TAIL: values below kGeluTail stay as they are, for gelu_tail
    v[2 * i] = (KEEP_TAIL && v[2 * i] < kGeluTail) ? v[2 * i] : r0;
    v[2 * i + 1] = (KEEP_TAIL && v[2 * i + 1] < kGeluTail) ? v[2 * i + 1] : r1;
  }
}

// Kept out of line so that the compiler cannot if-convert the rare tail path
// into every element of an unrolled epilogue loop.
static __device__ __noinline__ float gelu_tail(float x) { return gelu_erf(x); }

// GELU of 32 values in place: the polynomial form for all, then -- only when a
// lane of the warp holds a tail value, which is rare after a LayerNorm -- the
// library-erf form for the tail elements. All 32 lanes of the warp must call it.
__device__ __forceinline__ void gelu32(float* v) {
  float lo = v[0];
#pragma unroll
  for (int i = 1; i < 32; ++i) lo = fminf(lo, v[i]);
  if (__any_sync(0xffffffffu, lo < kGeluTail)) {
    // the polynomial form on the paired pipe for every value but the tail
    // ones, which keep x (GELU itself is never below -0.2) and then take the
    // library-erf form
    gelu32_pairs<true>(v);
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (v[i] < kGeluTail) v[i] = gelu_tail(v[i]);
  } else {
    gelu32_pairs(v);
  }
}

// ── shared-memory address helpers ────────────────────────────────────────────

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte shared-memory load / store by shared-window address (smem_u32).
// The kernels align their dynamic shared memory by integer arithmetic, after
// which the compiler no longer knows a pointer is shared; these keep the
// accesses on the shared-memory path instead of generic loads and stores.
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// ── mbarrier ─────────────────────────────────────────────────────────────────

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
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

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a barrier phase (never suspends the thread).
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

// test_wait with acquire at cluster scope: the phase may have been completed by
// arrivals of other CTAs of the cluster, whose writes become visible here.
__device__ __forceinline__ bool mbar_test_wait_cl(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait. Polls the barrier phase (test_wait: the thread is never parked,
// so a phase completed by a tcgen05.commit is seen at once) until it completes,
// the shared abort flag is raised by another thread, or ~kWaitCycles SM cycles
// pass. On a timeout it records CK_ERR_TIMEOUT with a site code, raises the
// abort flag and returns false; callers then leave their loops and the kernel
// exits cleanly.
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int site) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t n = 1;; ++n) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((n & 63u) == 0) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (clock64() - t0 > kWaitCycles) {
        set_status(CK_ERR_TIMEOUT, site, (int)parity);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// try_wait with a suspend-time hint (ns): while the phase is incomplete the
// thread is parked by the hardware, issuing nothing, until the phase completes
// or the hint expires.
__device__ __forceinline__ bool mbar_try_wait_ns(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait for roles that wait long and whose wake-up latency is not on
// the critical path (the epilogue waiting out a tile's main loop, the TMA
// producer waiting for a free stage, the operand transform warps waiting for
// their next stage): the thread is parked between checks, so that the warps
// sharing its scheduler -- the ones doing the work -- get its issue slots.
// Same timeout and abort behaviour as mbar_wait.
__device__ __forceinline__ bool mbar_wait_park(uint64_t* bar, uint32_t parity,
                                               volatile int* abort_flag, int site) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait_ns(bar, parity, 20000u)) return true;
    if (abort_flag != nullptr && *abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      set_status(CK_ERR_TIMEOUT, site, (int)parity);
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
  }
}

// ── thread-block clusters (distributed shared memory) ─────────────────────────

__device__ __forceinline__ uint32_t cl_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of `local` (an address in this CTA's smem) in CTA `rank`
__device__ __forceinline__ uint32_t cl_map(const void* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  return remote;
}

__device__ __forceinline__ void cl_store_f2(uint32_t remote, float2 v) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(remote), "f"(v.x), "f"(v.y)
               : "memory");
}

__device__ __forceinline__ void cl_store_v4(uint32_t remote, uint4 v) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster, releasing this thread's
// earlier (distributed) shared-memory writes at cluster scope.
__device__ __forceinline__ void cl_mbar_arrive(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar)
               : "memory");
}

// All threads of all CTAs of the cluster (every thread must call it).
__device__ __forceinline__ void cl_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// mbar_wait for a barrier that other CTAs of the cluster arrive on.
__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity,
                                             volatile int* abort_flag, int site) {
  const long long t0 = clock64();
  for (uint32_t n = 0;; ++n) {
    if (mbar_test_wait_cl(bar, parity)) return true;
    if ((n & 63u) == 63u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (clock64() - t0 > kWaitCycles) {
        set_status(CK_ERR_TIMEOUT, site, (int)parity);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ── TMA ──────────────────────────────────────────────────────────────────────

// A tile load of one CTA of a 2-SM MMA pair: the data land in this CTA's shared
// memory and the byte count completes on the barrier at shared::cluster
// address bar_cluster (the even CTA's, from cl_map).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Tiled TMA store shared -> global (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0,
                                             int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N bulk groups of this thread are still in flight.
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor core operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ── tcgen05 ──────────────────────────────────────────────────────────────────

// Allocate `ncols` TMEM columns (power of two >= 32); whole warp executes.
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

// The same for a pair of CTAs (cta_group::2): both CTAs of the cluster pair
// call them from the same warp, with the same shared-memory slot.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 inputs, fp32 accum).
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 2-SM MMA (cta_group::2), issued by the even CTA of the pair: M rows split over
// the two CTAs (A and D), B's N rows split likewise, operands at the same
// shared-memory offsets in both CTAs.
__device__ __forceinline__ void tc_mma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once the pair MMAs issued so far complete, on the mbarrier at this
// shared-memory offset in every CTA of cta_mask.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Load 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 32-bit words per thread to / from TMEM columns taddr..taddr+15 of the
// warp's lane quarter (32x32b shape), and the wait for this thread's stores.
__device__ __forceinline__ void tmem_st16w(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld16w(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tc_wait_store() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile.
//   K-major: rows of 128 B (64 bf16 along K), 8-row groups 1024 B apart (SBO).
//   MN-major: rows of 128 B (64 bf16 along M/N) per K index, 8-K groups 1024 B
//   apart (SBO), 64-wide M/N blocks `lbo_bytes` apart (LBO).
// Bits: [0,14) addr>>4, [16,30) LBO>>4, [32,46) SBO>>4, [46,48) version=1,
// [61,64) layout 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: bf16 A/B, fp32 D, dense.
//   [4,6) D fmt (1 = f32), [7,10) A fmt (1 = bf16), [10,13) B fmt (1 = bf16),
//   [15] A major (0 = K), [16] B major (0 = K, 1 = MN), [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t M, uint32_t N, uint32_t b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}

// Byte offset of element (row, col16) -- a 16-byte chunk -- inside a 128B-swizzled
// tile whose rows are 128 B and whose base is 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128_off(uint32_t row, uint32_t chunk16) {
  return row * 128u + ((chunk16 ^ (row & 7u)) << 4);
}

}  // namespace ck
