// bf16_gemv.cu -- BF16 dense GEMV for the hybrid's non-expert projections,
// bit-exact to the reference's gemv_bf16 (kennydd001/ervf
// src/moe_lab/lightningstream_nemotron/gpu_kernels.py:21-49) for every column
// of a batch of up to 8 activation vectors.
//
// Reference arithmetic: thread t of a 256-thread block walks k = t, t+256, ...
// with acc = fmaf(bf16_to_f32(W[row,k]), x[k], acc); the 256 chains are
// reduced by the warp butterfly and the 8 warp sums by a second butterfly
// that also adds zero lanes (the "legacy" combine).
//
// B200 mapping: one warp per row.  Lane c owns chains 8c..8c+7, so one
// 128-bit load per lane and round covers elements 256*i + 8c .. +7 and a warp
// streams 512 contiguous bytes per round.  The group butterfly's first two
// levels (chain offsets 16 and 8) are lane shuffles (xor 2, xor 1), the last
// three are in registers; the group sums are combined across lanes 0,4,..,28.
#include "common.cuh"
#include "kernels.h"

namespace ervf {

namespace {

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

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

template <int B>
__global__ void __launch_bounds__(256) bf16_gemv_kernel(const uint16_t* __restrict__ W,
                                                        const float* __restrict__ x,
                                                        float* __restrict__ out, int rows,
                                                        int cols) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= rows) return;
  const uint16_t* wr = W + (size_t)row * cols;
  float acc[B][8];
#pragma unroll
  for (int b = 0; b < B; ++b)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[b][j] = 0.0f;

  const int nfull = cols >> 8;  // complete rounds of 256 elements
#pragma unroll 4
  for (int i = 0; i < nfull; ++i) {
    const int k = 256 * i + 8 * lane;
    const uint4 q = __ldcs(reinterpret_cast<const uint4*>(wr + k));
    float w[8] = {bf16lo(q.x), bf16hi(q.x), bf16lo(q.y), bf16hi(q.y),
                  bf16lo(q.z), bf16hi(q.z), bf16lo(q.w), bf16hi(q.w)};
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float4 x0 = __ldg(reinterpret_cast<const float4*>(x + (size_t)b * cols + k));
      const float4 x1 = __ldg(reinterpret_cast<const float4*>(x + (size_t)b * cols + k + 4));
      float2 a01 = fma2(make_float2(w[0], w[1]), make_float2(x0.x, x0.y), make_float2(acc[b][0], acc[b][1]));
      float2 a23 = fma2(make_float2(w[2], w[3]), make_float2(x0.z, x0.w), make_float2(acc[b][2], acc[b][3]));
      float2 a45 = fma2(make_float2(w[4], w[5]), make_float2(x1.x, x1.y), make_float2(acc[b][4], acc[b][5]));
      float2 a67 = fma2(make_float2(w[6], w[7]), make_float2(x1.z, x1.w), make_float2(acc[b][6], acc[b][7]));
      acc[b][0] = a01.x; acc[b][1] = a01.y; acc[b][2] = a23.x; acc[b][3] = a23.y;
      acc[b][4] = a45.x; acc[b][5] = a45.y; acc[b][6] = a67.x; acc[b][7] = a67.y;
    }
  }
  // last partial round: elements 256*nfull + 8*lane + j < cols
  {
    const int k = 256 * nfull + 8 * lane;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (k + j < cols) {
        const float wf = __uint_as_float(((uint32_t)wr[k + j]) << 16);
#pragma unroll
        for (int b = 0; b < B; ++b) acc[b][j] = fmaf(wf, x[(size_t)b * cols + k + j], acc[b][j]);
      }
    }
  }
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float s = row_tree(acc[b]);
    if (lane == 0) out[(size_t)b * rows + row] = s;
  }
}

}  // namespace

int launch_bf16_gemv(const uint16_t* W, const float* x, float* out, int rows, int cols, int batch,
                     cudaStream_t stream) {
  const int grid = (rows + 7) / 8;
  switch (batch) {
#define ERVF_BF16_CASE(B) \
  case B: bf16_gemv_kernel<B><<<grid, 256, 0, stream>>>(W, x, out, rows, cols); break;
    ERVF_BF16_CASE(1)
    ERVF_BF16_CASE(2)
    ERVF_BF16_CASE(3)
    ERVF_BF16_CASE(4)
    ERVF_BF16_CASE(5)
    ERVF_BF16_CASE(6)
    ERVF_BF16_CASE(7)
    ERVF_BF16_CASE(8)
#undef ERVF_BF16_CASE
    default: return kErrArg;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace ervf
