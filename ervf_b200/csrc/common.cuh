// common.cuh -- shared device helpers of the ERVF B200 kernels.
//
// Numeric contract (kennydd001/ervf src/moe_lab/lightningstream_nemotron/
// fused_nvfp4.py:31-122 and :295-406): one output row is the sum of 256
// "virtual thread" chains.  Chain t walks uchar4 index v = t, t+256, ... and
// takes, per uchar4, s = RN(e4m3[scale[4v>>3]] * g) and for each of its eight
// codes (lo,hi nibble of bytes 0..3) acc = fmaf(RN(e2m1[nib] * s), x[k], acc).
// The 256 chain values are then reduced by a fixed binary tree: a butterfly
// over each group of 32 consecutive chains (shfl_down 16,8,4,2,1) and the
// combine ((S0+S4)+(S2+S6))+((S1+S5)+(S3+S7)) of the 8 group sums.
//
// Every kernel in this library reproduces that sum bit for bit with its own
// thread mapping: the chains are formed in registers, written to shared memory
// and reduced there by the same tree.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <stdint.h>

namespace ervf {

// ------------------------------------------------------------------ status

enum : int {
  kOk = 0,
  kErrNull = -1,
  kErrShape = -2,
  kErrAlign = -3,
  kErrLaunch = -4,
  kErrTimeout = -5,
  kErrArg = -6,
  kErrDevice = -7,
};

// Device-side error word: set by a kernel whose bounded wait ran out.  One
// copy per translation unit; each unit that waits exports a host reader
// (read_*_device_error in kernels.h), and ervf_device_status() reads them all.
static __device__ int g_device_error;

// Host reader of this unit's error word (each unit wraps it in a named
// function declared in kernels.h).
static inline int read_unit_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return kErrLaunch;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return kErrLaunch;
  }
  return v;
}

// ------------------------------------------------------------- decoding

// E4M3 (bias 7, subnormal 2^-6*m/8, NaN only at 0x7F/0xFF) as the device LUT
// of the reference holds it: NaN bytes decode to +0.0
// (nvfp4.py:58-69, fused_nvfp4.py:760-762).  Exact in binary32.
__host__ __device__ __forceinline__ float e4m3_lut_value(uint32_t b) {
  const uint32_t e = (b >> 3) & 0xFu, m = b & 7u;
  if (e == 0xFu && m == 7u) return 0.0f;
  float v;
  if (e == 0u) {
    v = (float)m * 0.001953125f;  // m * 2^-9, exact
  } else {
    const uint32_t bits = ((e + 120u) << 23) | (m << 20);
#ifdef __CUDA_ARCH__
    v = __uint_as_float(bits);
#else
    union { uint32_t u; float f; } cvt;
    cvt.u = bits;
    v = cvt.f;
#endif
  }
  return (b & 0x80u) ? -v : v;
}

// E2M1 (sign bit 3; magnitudes 0,0.5,1,1.5,2,3,4,6), nvfp4.py:49-55.
__host__ __device__ __forceinline__ float e2m1_value(uint32_t c) {
  const uint32_t m = c & 7u;
  float v = (m < 4u) ? 0.5f * (float)m : (m == 4u ? 2.0f : (m == 5u ? 3.0f : (m == 6u ? 4.0f : 6.0f)));
  return (c & 8u) ? -v : v;
}

// The eight E2M1 codes of one 32-bit word to four f16x2 (byte i -> h[i];
// low nibble -> low half) with the sm_100a hardware converter
// (cvt.rn.f16x2.e2m1x2, exact: every E2M1 value is an f16).
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t q, uint32_t (&h)[4]) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(q));
}

// f16x2 -> two binary32 (exact widening).
__device__ __forceinline__ float2 f16x2_to_f32x2(uint32_t h) {
  float2 r;
  asm("{\n .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %2;\n cvt.f32.f16 %0, lo;\n cvt.f32.f16 %1, hi;\n}"
      : "=f"(r.x), "=f"(r.y)
      : "r"(h));
  return r;
}

// The eight E2M1 codes of a 32-bit word (code i = nibble i, low first) as
// exact binary32 values f[0..7]: hardware e2m1x2 -> f16x2, then f16 -> f32.
// The halves are widened with __low2float / __high2float, which the compiler
// folds into the half-select of the conversion (an explicit unpack of the
// f16x2 word costs one more integer instruction per two weights).
__device__ __forceinline__ void e2m1x8_to_f32(uint32_t q, float (&f)[8]) {
  uint32_t h[4];
  e2m1x8_to_f16x2(q, h);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 v = *reinterpret_cast<const __half2*>(&h[i]);
    f[2 * i] = __low2float(v);
    f[2 * i + 1] = __high2float(v);
  }
}

// ------------------------------------------------- packed fp32 arithmetic

__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// ---------------------------------------------------- the 256-leaf tree

// Shared-memory layout of one row's 256 chain values: 8 groups of 32 floats,
// each group padded to 36 floats so that the 8 readers of one row (one per
// group) hit 8 different 16-byte bank groups.
constexpr int kGroupPitch = 36;
constexpr int kRowPitch = 8 * kGroupPitch;  // floats per row of partials

__device__ __forceinline__ int part_index(int chain) {
  return (chain >> 5) * kGroupPitch + (chain & 31);
}

// T(a_0..a_31): level `off` = 16,8,4,2,1 adds a_{l+off} into a_l for l < off;
// returns a_0.  Pairs of independent adds go through the packed adder.
__device__ __forceinline__ float group_tree(const float* __restrict__ g32) {
  const float4* p = reinterpret_cast<const float4*>(g32);
  float y[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v = p[i];
    y[4 * i + 0] = v.x; y[4 * i + 1] = v.y; y[4 * i + 2] = v.z; y[4 * i + 3] = v.w;
  }
#pragma unroll
  for (int off = 16; off >= 2; off >>= 1) {
#pragma unroll
    for (int l = 0; l < off; l += 2) {
      const float2 r = add2(make_float2(y[l], y[l + 1]), make_float2(y[l + off], y[l + off + 1]));
      y[l] = r.x; y[l + 1] = r.y;
    }
  }
  return y[0] + y[1];
}

// Combine of the 8 group sums held by 8 consecutive lanes (lane&7 == group):
// pairs (w, w+4), then (w, w+2), then (w, w+1) -- the reference's
// ((S0+S4)+(S2+S6))+((S1+S5)+(S3+S7)).  Valid in lane&7 == 0.
__device__ __forceinline__ float combine8(float s) {
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  return s;
}

__device__ __forceinline__ float epilogue(float v, int relu2, float out_scale) {
  if (relu2) {
    const float r = fmaxf(v, 0.0f);
    return r * r;
  }
  return v * out_scale;
}

// ------------------------------------------------------ mbarrier / bulk

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread may sleep in hardware (up to
// `ns` nanoseconds, woken when the phase completes) instead of spinning, so
// a waiting warp does not take issue slots from the warps that compute.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(ns) : "memory");
  return ok != 0;
}

// Non-blocking probe: has the phase with this parity completed?
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

__device__ __forceinline__ void nanosleep_ns(uint32_t ns) { asm volatile("nanosleep.u32 %0;" ::"r"(ns)); }

// Bounded wait: gives up after ~`budget` cycles, records kErrTimeout in the
// device error word and returns false.  A wait that completes returns true.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          long long budget = 4000000000LL) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_sleep(bar, parity, 500)) {
    if (clock64() - t0 > budget) {
      atomicExch(&g_device_error, kErrTimeout);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared (no multicast); completes `bytes` of
// transaction count on `bar`.  dst, src 16-B aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ int named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
  return 0;
}

// Named barrier that also ORs a predicate over the participating threads, so
// that a timeout seen by any thread becomes one uniform decision.
__device__ __forceinline__ bool named_bar_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(nthreads) : "memory");
  return r != 0;
}

}  // namespace ervf
