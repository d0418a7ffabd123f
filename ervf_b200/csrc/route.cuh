// route.cuh -- the sigmoid top-k router of one problem on one warp, shared by
// the batched router launch (aux.cu) and the fused router GEMV + top-k
// (bf16_gemv.cu).  route_topk_f32 (kennydd001/ervf
// src/moe_lab/lightningstream_nemotron/fused_nvfp4.py:433-465):
// sc = 1/(1+expf(-logit)), selection on sc + bias with the strictly greater
// value winning (lowest index on ties), weights sc / (wsum + 1e-20) * scaling
// with wsum added in route order; bad_pick drops the best candidate of the
// last slot.  Scores are held in registers (lane l owns experts l, l+32, ...);
// logits are read through L2 (another CTA may have just written them).
// n <= 32 * NPL, top_k <= 64.
#pragma once

#include <cuda_runtime.h>

namespace ervf {

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
