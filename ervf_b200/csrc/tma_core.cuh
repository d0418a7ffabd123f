// tma_core.cuh -- the consumer side of the TMA-staged NVFP4 GEMV schedule,
// shared by nvfp4_gemv.cu (per-launch GEMVs) and moe_token.cu (the one-launch
// decode token): the exact ERVF chain over one 16-byte code unit, the
// swizzled activation layout, the per-thread segment walk of an item and the
// PTX helpers of the producer / consumer / publisher hand-offs.  Numeric
// contract: kennydd001/ervf fused_nvfp4.py:31-122 and :295-406.
#pragma once

#include "common.cuh"

namespace ervf {

constexpr int kCW = 8;          // consumer warps
constexpr int kCT = kCW * 32;   // consumer threads
constexpr int kBarC = 1;        // named barrier of the consumer threads

// One 16-byte code unit (4 chains x 8 codes) of one row, continuing the four
// chain accumulators: acc[0] = (chain 0, chain 1), acc[1] = (chain 2, chain 3).
// Chains 0,1 use the block scale s0 = s_2u, chains 2,3 use s1 = s_2u+1.  The
// activation comes pre-paired: xp[m] = (x[m], x[8 + m]) and xp[8 + m] =
// (x[16 + m], x[24 + m]) for code m of the chain pair, x[8j + m] being the
// activation of chain j's m-th code.  Per code: w = RN(e2m1 * s) (FMUL) and
// acc = fmaf(w, x, acc) (FFMA), in each chain's order.  Scalar FMUL / FFMA
// issue to either FMA sub-pipe, so they run beside the f16 -> f32 widenings
// (measured on B200: 27.7 vs 25.9 weights per clock per SM for the packed
// f32x2 forms in an isolated core loop).
__device__ __forceinline__ void unit_fma(const uint4 q, const float s0, const float s1,
                                         const float2 (&xp)[16], float2 (&acc)[2]) {
  uint32_t h0[4], h1[4], h2[4], h3[4];
  e2m1x8_to_f16x2(q.x, h0);
  e2m1x8_to_f16x2(q.y, h1);
  e2m1x8_to_f16x2(q.z, h2);
  e2m1x8_to_f16x2(q.w, h3);
  float a0 = acc[0].x, a1 = acc[0].y, a2 = acc[1].x, a3 = acc[1].y;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 v0 = *reinterpret_cast<const __half2*>(&h0[i]);
    const __half2 v1 = *reinterpret_cast<const __half2*>(&h1[i]);
    const __half2 v2 = *reinterpret_cast<const __half2*>(&h2[i]);
    const __half2 v3 = *reinterpret_cast<const __half2*>(&h3[i]);
    a0 = fmaf(__low2float(v0) * s0, xp[2 * i].x, a0);
    a1 = fmaf(__low2float(v1) * s0, xp[2 * i].y, a1);
    a2 = fmaf(__low2float(v2) * s1, xp[8 + 2 * i].x, a2);
    a3 = fmaf(__low2float(v3) * s1, xp[8 + 2 * i].y, a3);
    a0 = fmaf(__high2float(v0) * s0, xp[2 * i + 1].x, a0);
    a1 = fmaf(__high2float(v1) * s0, xp[2 * i + 1].y, a1);
    a2 = fmaf(__high2float(v2) * s1, xp[9 + 2 * i].x, a2);
    a3 = fmaf(__high2float(v3) * s1, xp[9 + 2 * i].y, a3);
  }
  acc[0] = make_float2(a0, a1);
  acc[1] = make_float2(a2, a3);
}

// SiLU of the gate row, v / (1 + e^-v) in binary32 (CUDA expf).
__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// Shared copy of the activation: unit t (32 columns) holds 8 float4 slots;
// slot k = (x[c], x[c + 8], x[c + 1], x[c + 9]) with c = 16 (k >> 2) + 2 (k & 3)
// (column offsets inside the unit), stored at t * 8 + (k ^ (t & 7)) so that
// the eight readers of one slot index hit different bank groups.  One slot
// is two of the pairs unit_fma consumes.
__device__ __forceinline__ float4 x_slot(const float* x, int t, int k) {
  const int c = 32 * t + 16 * (k >> 2) + 2 * (k & 3);
  const float2 a = *reinterpret_cast<const float2*>(x + c);
  const float2 b = *reinterpret_cast<const float2*>(x + c + 8);
  return make_float4(a.x, b.x, a.y, b.y);
}

__device__ __forceinline__ float4 x_slot_cg(const float* x, int t, int k) {
  const int c = 32 * t + 16 * (k >> 2) + 2 * (k & 3);
  const float2 a = __ldcg(reinterpret_cast<const float2*>(x + c));
  const float2 b = __ldcg(reinterpret_cast<const float2*>(x + c + 8));
  return make_float4(a.x, b.x, a.y, b.y);
}

// The activation pairs of unit u from the shared copy.
__device__ __forceinline__ void load_unit_x(const float4* xs, int u, float2 (&xp)[16]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float4 v = xs[u * 8 + (k ^ (u & 7))];
    xp[2 * k] = make_float2(v.x, v.y);
    xp[2 * k + 1] = make_float2(v.z, v.w);
  }
}

// The two segments of one consumer thread for one item (see the schedule
// above).  FULL: every row of the item exists, so the H rows of a segment run
// unconditionally and interleave.
// H rows of one segment, unit fixed: code / scale byte offsets (into the
// stage, relative to smem) advance by rstep / sstep per row; block scales come
// from the job's table of RN(e4m3 * g).
template <int H, bool FULL>
__device__ __forceinline__ void seg_rows(const uint8_t* smem, uint32_t coff, uint32_t soff,
                                         uint32_t rstep, uint32_t sstep, const float* lut,
                                         const float2 (&x)[16], float2 (&acc)[H][2], int row0,
                                         int rowstep, int nrows) {
#pragma unroll
  for (int h = 0; h < H; ++h) {
    if (FULL || row0 + h * rowstep < nrows) {
      const uint4 q = *reinterpret_cast<const uint4*>(smem + coff + h * rstep);
      const uint32_t s2 = *reinterpret_cast<const uint16_t*>(smem + soff + h * sstep);
      unit_fma(q, lut[s2 & 0xFFu], lut[s2 >> 8], x, acc[h]);
    }
  }
}

template <int H, bool FULL>
__device__ __forceinline__ void seg_store(float* part, uint32_t poff, uint32_t pstep,
                                          const float2 (&acc)[H][2], int row0, int rowstep,
                                          int nrows) {
#pragma unroll
  for (int h = 0; h < H; ++h)
    if (FULL || row0 + h * rowstep < nrows)
      *reinterpret_cast<float4*>(part + poff + h * pstep) =
          make_float4(acc[h][0].x, acc[h][0].y, acc[h][1].x, acc[h][1].y);
}

// The two segments of one consumer thread for one item (see the schedule
// above).  FULL: every row of the item exists, so the H rows of a segment run
// unconditionally and interleave.  stage_off: the stage's byte offset in smem.
template <int H, bool FULL>
__device__ __forceinline__ void segments(const uint8_t* smem, uint32_t stage_off, int scale_off,
                                         int cb, int sb, int team, int T, int par1, int par2,
                                         bool cont, int u1, int u2, int grp, int nrows,
                                         const float* lut, const float4* xs, float2 (&x)[16],
                                         bool& x_stale, float* part) {
  float2 acc[H][2];
#pragma unroll
  for (int h = 0; h < H; ++h) acc[h][0] = acc[h][1] = make_float2(0.0f, 0.0f);
  const int rowstep = 2 * T;
  const uint32_t rstep = (uint32_t)(rowstep * cb), sstep = (uint32_t)(rowstep * sb);
  const uint32_t pstep = (uint32_t)(rowstep * kRowPitch);
  const int row1 = team + T * par1, row2 = team + T * par2;
  if (cont || x_stale) load_unit_x(xs, u1, x);
  x_stale = false;
  seg_rows<H, FULL>(smem, stage_off + row1 * cb + 16 * u1, stage_off + scale_off + row1 * sb + 2 * u1,
                    rstep, sstep, lut, x, acc, row1, rowstep, nrows);
  if (!cont) {
    seg_store<H, FULL>(part, row1 * kRowPitch + part_index(4 * grp), pstep, acc, row1, rowstep, nrows);
#pragma unroll
    for (int h = 0; h < H; ++h) acc[h][0] = acc[h][1] = make_float2(0.0f, 0.0f);
  } else {
    load_unit_x(xs, u2, x);
  }
  seg_rows<H, FULL>(smem, stage_off + row2 * cb + 16 * u2, stage_off + scale_off + row2 * sb + 2 * u2,
                    rstep, sstep, lut, x, acc, row2, rowstep, nrows);
  seg_store<H, FULL>(part, row2 * kRowPitch + part_index(4 * grp), pstep, acc, row2, rowstep, nrows);
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void st_release_cta(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_cta(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}

}  // namespace ervf
