// bf16_gemv.cu -- dense GEMVs: BF16 for the hybrid's non-expert projections,
// bit-exact to the reference's gemv_bf16 (kennydd001/ervf
// src/moe_lab/lightningstream_nemotron/gpu_kernels.py:21-49) for every column
// of a batch of up to 8 activation vectors; FP32 for the MoE router
// (gemv_f32, gpu_kernels.py:51-74), alone or fused with the top-k router.
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
#include "route.cuh"

namespace ervf {

namespace {

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

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

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__global__ void __launch_bounds__(256) f32_gemv_kernel(const float* __restrict__ W,
                                                       const float* __restrict__ x,
                                                       float* __restrict__ out, int rows, int cols) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= rows) return;
  const float s = f32_row(W + (size_t)row * cols, x, cols, lane);
  if (lane == 0) out[row] = s;
}

// Router of one MoE layer in one launch: rlog = gemv_f32(gate_w, x) (one
// warp per expert, kRouterWarps experts per CTA so that the 1.4 MB of router
// weights spread over many SMs: the up launch that follows cannot start
// streaming its experts before the ids exist), then the last CTA to finish
// (counter, left zero) runs route_topk_f32 on rlog with one warp.  x may
// come from the previous kernel on the stream (PDL-safe: it waits before
// reading x).
constexpr int kRouterWarps = 2;

template <int NPL>
__global__ void __launch_bounds__(32 * kRouterWarps) route_gemv_topk_kernel(
    const float* __restrict__ W, const float* __restrict__ x, float* rlog,
    const float* __restrict__ gate_b, int* __restrict__ ids, float* __restrict__ w, int n,
    int cols, int top_k, float scaling, int bad_pick, unsigned* counter) {
  __shared__ int last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRouterWarps + warp;
  pdl_wait();
  pdl_launch();
  if (row < n) {
    const float s = f32_row(W + (size_t)row * cols, x, cols, lane);
    if (lane == 0) {
      rlog[row] = s;
      __threadfence();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (warp == 0) route_topk_warp<NPL>(rlog, gate_b, ids, w, n, top_k, scaling, bad_pick);
  if (threadIdx.x == 0) *counter = 0u;
}

}  // namespace

int launch_f32_gemv(const float* W, const float* x, float* out, int rows, int cols,
                    cudaStream_t stream) {
  f32_gemv_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(W, x, out, rows, cols);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_route_gemv_topk(const float* W, const float* x, float* rlog, const float* gate_b, int* ids,
                           float* w, int n, int cols, int top_k, float scaling, int bad_pick,
                           unsigned* counter, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((n + kRouterWarps - 1) / kRouterWarps);
  cfg.blockDim = dim3(32 * kRouterWarps);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e;
  if (n <= 128) {
    e = cudaLaunchKernelEx(&cfg, route_gemv_topk_kernel<4>, W, x, rlog, gate_b, ids, w, n, cols, top_k,
                           scaling, bad_pick, counter);
  } else {
    e = cudaLaunchKernelEx(&cfg, route_gemv_topk_kernel<8>, W, x, rlog, gate_b, ids, w, n, cols, top_k,
                           scaling, bad_pick, counter);
  }
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return kErrLaunch;
  }
  return kOk;
}

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
