// route.cuh -- the router of one problem on one warp: the FP32 router row
// (f32_row, with the legacy 256-chain tree row_tree) and the sigmoid top-k,
// shared by the batched router launch (aux.cu), the fused router GEMV +
// top-k (bf16_gemv.cu) and the token kernel's router items (moe_token.cu).
// route_topk_f32 (kennydd001/ervf
// src/moe_lab/lightningstream_nemotron/fused_nvfp4.py:433-465):
// sc = 1/(1+expf(-logit)), selection on sc + bias with the strictly greater
// value winning (lowest index on ties), weights sc / (wsum + 1e-20) * scaling
// with wsum added in route order; bad_pick drops the best candidate of the
// last slot.  Scores are held in registers (lane l owns experts l, l+32, ...);
// logits are read through L2 (another CTA may have just written them).
// n <= 32 * NPL, top_k <= 64.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace ervf {

// The router projection rows (gemv_f32, gpu_kernels.py:51-74), shared by the
// dense-GEMV kernels (bf16_gemv.cu) and the router items of the one-launch
// token kernel (moe_token.cu).
// Reduce the 8 chain values of this lane (chains 8c+j) of one row to the
// row sum, valid in lane 0.
__device__ __forceinline__ float row_tree(float (&a)[8]) {
  // chain offset 16 -> lane xor 2; offset 8 -> lane xor 1
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] += __shfl_xor_sync(0xffffffffu, a[j], 2);
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] += __shfl_xor_sync(0xffffffffu, a[j], 1);
  // offsets 4, 2, 1 inside the lane
  const float2 l4a = add2(make_float2(a[0], a[1]), make_float2(a[4], a[5]));
  const float2 l4b = add2(make_float2(a[2], a[3]), make_float2(a[6], a[7]));
  const float2 l2 = add2(l4a, l4b);
  float s = l2.x + l2.y;
  // legacy combine: group sum + 0.0, then (w,w+4),(w,w+2),(w,w+1) = lanes xor 16, 8, 4
  s = s + 0.0f;
  s += __shfl_xor_sync(0xffffffffu, s, 16);
  s += __shfl_xor_sync(0xffffffffu, s, 8);
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  return s;
}

// gemv_f32 (gpu_kernels.py:51-74): the same 256-chain walk, warp butterfly
// and legacy combine as gemv_bf16 with fp32 weights.  One warp per row; lane
// c owns chains 8c..8c+7 (two 128-bit loads per round).  Row sum in lane 0.
// XS: x is in shared memory (plain loads); else global, read through L2.
template <bool XS = false>
__device__ __forceinline__ float f32_row(const float* __restrict__ wr, const float* __restrict__ x,
                                         int cols, int lane) {
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  const int nfull = cols >> 8;
  // x from shared memory leaves the weight loads as the only long ones: more
  // of them in flight per round
  constexpr int kUnroll = XS ? 5 : 4;
#pragma unroll kUnroll
  for (int i = 0; i < nfull; ++i) {
    const int k = 256 * i + 8 * lane;
    const float4 w0 = __ldcs(reinterpret_cast<const float4*>(wr + k));
    const float4 w1 = __ldcs(reinterpret_cast<const float4*>(wr + k + 4));
    const float4 x0 = XS ? *reinterpret_cast<const float4*>(x + k) : __ldcg(reinterpret_cast<const float4*>(x + k));
    const float4 x1 =
        XS ? *reinterpret_cast<const float4*>(x + k + 4) : __ldcg(reinterpret_cast<const float4*>(x + k + 4));
    const float2 a01 = fma2(make_float2(w0.x, w0.y), make_float2(x0.x, x0.y), make_float2(acc[0], acc[1]));
    const float2 a23 = fma2(make_float2(w0.z, w0.w), make_float2(x0.z, x0.w), make_float2(acc[2], acc[3]));
    const float2 a45 = fma2(make_float2(w1.x, w1.y), make_float2(x1.x, x1.y), make_float2(acc[4], acc[5]));
    const float2 a67 = fma2(make_float2(w1.z, w1.w), make_float2(x1.z, x1.w), make_float2(acc[6], acc[7]));
    acc[0] = a01.x; acc[1] = a01.y; acc[2] = a23.x; acc[3] = a23.y;
    acc[4] = a45.x; acc[5] = a45.y; acc[6] = a67.x; acc[7] = a67.y;
  }
  {
    const int k = 256 * nfull + 8 * lane;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (k + j < cols) acc[j] = fmaf(wr[k + j], XS ? x[k + j] : __ldcg(x + k + j), acc[j]);
  }
  return row_tree(acc);
}


template <int NPL>
__device__ __forceinline__ void route_topk_warp(const float* lg, const float* bs, int* io, float* wo,
                                                int n, int top_k, float scaling, int bad_pick) {
  const int lane = threadIdx.x & 31;
  float sc[NPL], ch[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int e = lane + 32 * i;
    if (e < n) {
      const float s = 1.0f / (1.0f + expf(-__ldcg(&lg[e])));
      sc[i] = s;
      ch[i] = s + (bs ? bs[e] : 0.0f);
    } else {
      sc[i] = 0.0f;
      ch[i] = -3.0e38f;
    }
  }
  auto argmax = [&]() -> int {
    float bv = -3.0e38f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (ch[i] > bv) { bv = ch[i]; bi = lane + 32 * i; }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    return bi == 0x7fffffff ? 0 : bi;
  };
  auto drop = [&](int e) {
    if ((e & 31) == lane) {
#pragma unroll
      for (int i = 0; i < NPL; ++i)
        if (i == (e >> 5)) ch[i] = -3.0e38f;
    }
  };
  auto score_of = [&](int e) -> float {
    float v = 0.0f;
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (i == (e >> 5)) v = sc[i];
    return __shfl_sync(0xffffffffu, v, e & 31);
  };
  // Selection s is kept by lane s % 32 (top_k <= 64: two per lane at most),
  // so the final normalisation runs on all lanes in parallel.
  int my_id[2] = {0, 0};
  float my_v[2] = {0.0f, 0.0f};
  float wsum = 0.0f;
  for (int s = 0; s < top_k; ++s) {
    int bi = argmax();
    if (bad_pick && s == top_k - 1) {
      drop(bi);
      bi = argmax();
    }
    drop(bi);
    const float v = score_of(bi);
    if ((s & 31) == lane) {
      my_id[s >> 5] = bi;
      my_v[s >> 5] = v;
    }
    wsum += v;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int s = lane + 32 * h;
    if (s < top_k) {
      io[s] = my_id[h];
      wo[s] = my_v[h] / (wsum + 1e-20f) * scaling;
    }
  }
}

}  // namespace ervf
