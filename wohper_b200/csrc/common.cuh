// common.cuh -- device helpers shared by every wohper_b200 kernel (sm_100a).
//
// * bounded mbarrier waits (every spin has a %globaltimer deadline; on expiry
//   the kernel records WH_DEV_TIMEOUT in the context status word and returns,
//   it never traps),
// * TMA (cp.async.bulk.tensor, no multicast) and 1-D bulk copies into shared
//   memory,
// * exact decoders for the reference's FP8 E4M3 / UE8M0 / FP4 tables,
// * the reference's FP8 activation quant-dequant rounding, bit for bit.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#define WH_DEV_NONFINITE 1u  // an output was NaN/Inf (DeepSeekV4KernelError::NonFiniteOutput)
#define WH_DEV_TIMEOUT 2u    // a bounded wait expired
#define WH_DEV_BADARG 4u     // a device-side argument check failed (index out of range)

#ifndef WH_WAIT_NS
#define WH_WAIT_NS 2000000000ull  // 2 s: far above any legitimate wait in these kernels
#endif

namespace wh {

__host__ __device__ __forceinline__ uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}
__host__ __device__ __forceinline__ float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void flag(uint32_t* status, uint32_t bits) {
  if (status) atomicOr(status, bits);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Round a dynamic shared-memory pointer up to a 1024-byte boundary of the
// SHARED address space (what TMA's 128-byte swizzle requires).  The extern
// array is declared with 16-byte alignment only, so the compiler cannot fold
// this computation away; a CTA's dynamic shared memory is not 1024-aligned in
// general when several CTAs share an SM.
__device__ __forceinline__ uint8_t* align_smem_1024(uint8_t* p) {
  const uint32_t a = smem_u32(p);
  return p + ((1024u - (a & 1023u)) & 1023u);
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
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
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Non-blocking test of a phase (try_wait may suspend the thread for a while,
// which a producer polling several rings must not do).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and flags WH_DEV_TIMEOUT) if the phase did not
// complete before the deadline.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t* status) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t start = globaltimer();
  while (!mbar_try_wait(bar, phase)) {
    if (globaltimer() - start > WH_WAIT_NS) {
      flag(status, WH_DEV_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Producer drain before it leaves the kernel: a bounded wait that gives up at
// once when a wait of this launch sequence has already timed out, so a failed
// kernel returns after one timeout instead of one per ring stage.  A copy that
// has landed (the normal case: its consumer waited for it) returns without
// reading the status word; that read goes to L2 and, once per ring stage,
// would hold the CTA -- and the next kernel's dependency wait -- by
// microseconds.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t phase, uint32_t* status) {
  if (mbar_try_wait(bar, phase)) return true;
  if (status && (*(volatile uint32_t*)status & WH_DEV_TIMEOUT)) return false;
  return mbar_wait(bar, phase, status);
}

// ---------------------------------------------------------------------------
// system-scope flags between ranks (bounded waits, never a trap)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Wait until *p >= epoch; false (and WH_DEV_TIMEOUT) after the deadline or when
// another wait of this launch sequence already timed out.
__device__ __forceinline__ bool wait_epoch(const uint64_t* p, uint64_t epoch, uint32_t* status) {
  if (ld_acquire_sys(p) >= epoch) return true;
  const uint64_t start = globaltimer();
  for (uint32_t it = 0; ld_acquire_sys(p) < epoch; ++it) {
    if ((status && (*(volatile uint32_t*)status & WH_DEV_TIMEOUT)) ||
        globaltimer() - start > WH_WAIT_NS || it > (1u << 26)) {
      flag(status, WH_DEV_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// every thread of the CTA calls this after its last global store; returns
// true in the (one) CTA that arrived last, after which all its threads may
// read what the other CTAs stored
__device__ __forceinline__ bool last_cta_arrival(uint32_t* done) {
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(done, 1u);
    last = prev == gridDim.x - 1;
    if (last) {
      __threadfence_system();
      *done = 0;
    }
  }
  __syncthreads();
  return last;
}

// Named barrier `id` over `nthreads` threads (a multiple of 32) that also ANDs
// a predicate across them; warps that already left the kernel are not counted.
__device__ __forceinline__ int bar_and(int id, int nthreads, int pred) {
  int r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.s32 p, %1, 0; bar.red.and.pred q, %2, %3, p;"
      " selp.s32 %0, 1, 0, q; }"
      : "=r"(r)
      : "r"(pred), "r"(id), "r"(nthreads)
      : "memory");
  return r;
}

// ---------------------------------------------------------------------------
// TMA / bulk copies (plain loads only: no cluster-multicast form anywhere here)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tiled load; c0 = innermost coordinate (bytes for u8 maps; multiple of 16).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// 1-D bulk copy: src, dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue early / wait for the previous kernel's memory to be visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Packed / mixed-precision FP32 arithmetic (sm_100)
// ---------------------------------------------------------------------------
// Two independent IEEE fmas: (a.x*b.x+c.x, a.y*b.y+c.y), each rounded once
// (fma.rn.f32x2 through the toolkit's sm_100 intrinsic).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
// fp32 fma whose multiplicands are f16 (exactly widened): round(a*b + c) once.
__device__ __forceinline__ float fma_f16lo(uint32_t a2, uint32_t b2, float c) {
  float d;
  asm("{ .reg .b16 al, ah, bl, bh; mov.b32 {al, ah}, %1; mov.b32 {bl, bh}, %2;"
      " fma.rn.f32.f16 %0, al, bl, %3; }"
      : "=f"(d)
      : "r"(a2), "r"(b2), "f"(c));
  return d;
}
__device__ __forceinline__ float fma_f16hi(uint32_t a2, uint32_t b2, float c) {
  float d;
  asm("{ .reg .b16 al, ah, bl, bh; mov.b32 {al, ah}, %1; mov.b32 {bl, bh}, %2;"
      " fma.rn.f32.f16 %0, ah, bh, %3; }"
      : "=f"(d)
      : "r"(a2), "r"(b2), "f"(c));
  return d;
}

// ---------------------------------------------------------------------------
// Decoders
// ---------------------------------------------------------------------------
// Two E4M3 bytes (low 16 bits of v) -> f16x2 via the hardware converter.  Exact
// for every byte except 0x7F/0xFF, which the hardware maps to NaN and the
// reference maps to +-480; callers detect a non-finite row and recompute it
// with decode_fp8_exact().
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t v) {
  uint32_t h;
  asm("{ .reg .b16 t; cvt.u16.u32 t, %1; cvt.rn.f16x2.e4m3x2 %0, t; }" : "=r"(h) : "r"(v));
  return h;
}
__device__ __forceinline__ float2 h2_to_f2(uint32_t h) {
  __half2 v = *reinterpret_cast<__half2*>(&h);
  return __half22float2(v);
}
// decode_fp8_e4m3(byte, 1.0) of the reference, exactly (0x7F -> 480, 0x80 -> +0).
__host__ __device__ __forceinline__ float decode_fp8_exact(uint32_t b) {
  // e at bits 23..26, m at 20..22 of a float whose value is decode * 2^-120;
  // the multiply by 2^120 is exact (this library is built without FTZ).
  if ((b & 0x7Fu) == 0) return 0.0f;
  const float v = u2f((b & 0x7Fu) << 20) * 1.329227995784916e36f;
  return (b & 0x80u) ? -v : v;
}
// UE8M0 scale byte -> float: 0 -> 0, else 2^(b-127) (b=255 -> +inf), exactly
// decode_ue8m0_scale of the reference: the byte placed in the f32 exponent
// field gives all three cases (0 -> +0.0, 1 -> 2^-126, 255 -> +inf).
__host__ __device__ __forceinline__ float decode_ue8m0(uint32_t b) { return u2f((b & 0xffu) << 23); }

// One packed FP4 byte (low nibble = even column) -> f16x2 of the reference's
// FP4_E2M1_BASE_LUT values (nibble 1 = 0.125, not OCP's 0.5).  The hardware
// e2m1 converter gives OCP values; the only difference is +-0.5 -> +-0.125,
// i.e. f16 0x3800 -> 0x3000: bit 11 is cleared whenever bit 10 is clear (the
// only OCP magnitudes with bit 11 set are 0.5, 1.0, 1.5, and 1.0/1.5 have
// bit 10 set).
__device__ __forceinline__ uint32_t fp4x2_to_f16x2_ref(uint32_t byte_in_low8) {
  uint32_t h;
  asm("{ .reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(h) : "r"(byte_in_low8));
  // clear bit 11 of each half where bit 10 is 0
  uint32_t keep = (h << 1) | ~0x08000800u;
  return h & keep;
}

// ---------------------------------------------------------------------------
// FP8 activation quant-dequant (src/compute.rs:2504-2545), exact.
//   amax = max(max|v|, 1e-4); scale = exp2(ceil(log2(amax/448))) in f32 with
//   libm log2f; q = nearest E4M3 grid point of clamp(v/scale, +-448), ties to
//   the lower (more negative) entry; v = q*scale.
// ceil(log2f(q)) equals the exact ceil(log2 q) except in a narrow band just
// above each power of two where log2f rounds to the integer itself; the band's
// upper mantissa limit per exponent is measured once on the host from the
// platform log2f (the same libm the reference engine calls) and passed in.
// ---------------------------------------------------------------------------
struct ActQuantTable {
  // For biased exponent E of q = amax/448: ceil(log2f(q)) == E-127 iff the
  // mantissa m satisfies m < thr[E] (m == 0 is always inside).
  uint32_t thr[256];
};

__device__ __forceinline__ int ceil_log2f_thr(float q, const uint32_t* thr) {
  uint32_t u = __float_as_uint(q);
  uint32_t E = (u >> 23) & 0xFF;
  uint32_t m = u & 0x7FFFFF;
  int k = int(E) - 127;
  if (m == 0 || m < thr[E]) return k;
  return k + 1;
}
__device__ __forceinline__ int ceil_log2f_ref(float q, const ActQuantTable* t) {
  return ceil_log2f_thr(q, t->thr);
}

// scale = 2^k as float for k in the normal range (k >= -126 always holds here:
// amax >= 1e-4).
__device__ __forceinline__ float exp2i(int k) {
  if (k > 127) return __int_as_float(0x7f800000);
  return __uint_as_float(uint32_t(k + 127) << 23);
}

// The block scale 2^k of an act-quant block with the given amax, and 2^-k.
// v / 2^k equals v * 2^-k bit for bit: both round the same real quotient
// once, and 2^-k is a normal float for every k reachable (the 1e-4 amax floor
// gives k >= -22, a finite amax k <= 120).  amax = inf gives k = 128, scale
// inf and 2^-k = 0: v * 0 is the +-0 (NaN for +-inf) that v / inf is.
struct AqScale {
  float scale, inv;
};
__device__ __forceinline__ AqScale aq_block_scale(float amax, const uint32_t* thr) {
  amax = fmaxf(amax, 1.0e-4f);
  const int k = ceil_log2f_thr(__fdiv_rn(amax, 448.0f), thr);
  return {exp2i(k), k > 126 ? 0.0f : exp2i(-k)};
}
__host__ __device__ __forceinline__ float e4m3_nearest_ties_lower(float t);
// Quant-dequant of one value: nearest E4M3 of clamp(v / scale, +-448) times scale.
__device__ __forceinline__ float aq_value(float v, AqScale s) {
  float t = __fmul_rn(v, s.inv);
  t = t < -448.0f ? -448.0f : t;
  t = t > 448.0f ? 448.0f : t;
  return __fmul_rn(e4m3_nearest_ties_lower(t), s.scale);
}

// Nearest E4M3 grid value of t (|t| <= 448 or NaN) with ties to the lower
// entry, as nearest_in_sorted_lut over the reference's sorted LUT.  Returns
// +0.0 for results that are zero.
__host__ __device__ __forceinline__ float e4m3_nearest_ties_lower(float t) {
  if (t != t) return -480.0f;  // NaN: partition_point == 0 -> lut[0]
  const bool neg = t < 0.0f;
  const float a = fabsf(t);
  float r;
  if (a < 0.015625f) {  // E4M3 subnormal range: grid 2^-9
    const float q = a * 512.0f;  // exact
    float n = floorf(q);
    const float f = q - n;  // exact
    if (f > 0.5f || (f == 0.5f && neg)) n += 1.0f;
    r = n * 0.001953125f;
  } else {
    const uint32_t u = f2u(a);
    const uint32_t rem = u & 0xFFFFFu;
    uint32_t base = u & ~0xFFFFFu;
    if (rem > 0x80000u || (rem == 0x80000u && neg)) base += 0x100000u;
    r = u2f(base);
  }
  if (r == 0.0f) return 0.0f;
  return neg ? -r : r;
}

}  // namespace wh
