// ep_p2p.cu -- expert-parallel exchange of the routed slot outputs over
// NVLink peer memory, fused with the route-order sum.
//
// Every rank owns one exchange region (allocated and shared once at set-up
// through CUDA IPC; capi.cu), laid out as
//
//   [0, 512)        u64 flag[kEpMaxRanks]  flag[src] = last epoch rank src published
//   [512, 520)      u64 seq                epochs this rank has published
//   [520, 524)      u32 done               CTAs of a batched exchange finished
//   [1024, ...)     f32 slots[kEpBufs][top_k][hidden]
//
// Per layer each rank's down launch writes the outputs of the slots it owns
// into slots[buf] of its OWN region (plain local stores).  The exchange
// kernel then (1) publishes epoch e = seq + 1 into flag[rank] of every
// rank's region (st.release.sys after a system-scope fence), (2) waits --
// bounded -- until every rank's flag in its own region reached e, and (3)
// reads slot s from the region of the rank owning expert ids[s] (peer loads
// over NVLink) and writes out[r] = x[r] + acc, acc = fmaf(y_s[r], w[s], acc)
// over s in route order from 0.0: the arithmetic of ep_route_sum_kernel and
// of the single-GPU routed-sum epilogue, so the result is bit-identical to
// one GPU (route-order contract of kennydd001/ervf runtime.py:588-596).
//
// Reuse of slots[buf]: a rank writes slots[b] for epoch e only after its
// exchange of epoch e-1 saw every rank's flag e-1, which each rank publishes
// after its exchange of epoch e-2 has finished reading; so two consecutive
// exchanges must use different buffers (the caller alternates; with an odd
// layer count the last layer takes the third buffer).
//
// The epoch lives in device memory (seq), so a captured CUDA graph replays
// with fresh epochs.  No NCCL call, no multicast: flags are single stores,
// data moves by peer loads.
#include "common.cuh"
#include "kernels.h"

namespace ervf {
namespace {

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Threads (float4 columns) per CTA of the batched exchange.
constexpr int kEpBatchThreads = 128;

// Backstop on the number of polls, independent of the timer.
constexpr uint32_t kEpSpinCap = 1u << 26;

__global__ void __launch_bounds__(kEpThreads, 1) ep_exchange_sum_kernel(EpExchange a) {
  __shared__ uint64_t s_epoch;
  __shared__ const float4* s_src[kMaxJobs];
  __shared__ float s_w[kMaxJobs];
  const int tid = threadIdx.x;
  // The down launch before this one wrote this rank's slots; x comes from the
  // layer before.  Both are complete after the wait.
  dep_wait();
  dep_launch();
  uint64_t* flags = reinterpret_cast<uint64_t*>(a.peers[a.rank]);
  uint64_t* seq = flags + kEpMaxRanks;
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile uint64_t*>(seq) + 1;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
  }
  __syncthreads();
  const uint64_t e = s_epoch;
  if (tid < a.nranks) st_release_sys(reinterpret_cast<uint64_t*>(a.peers[tid]) + a.rank, e);

  int ok = 1;
  if (tid < a.nranks) {
    const uint64_t* f = flags + tid;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      if ((int64_t)(ld_acquire_sys(f) - e) >= 0) break;
      if (it >= kEpSpinCap || ((it & 15u) == 15u && globaltimer_ns() - t0 > a.timeout_ns)) {
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
  }
  int good_ids = 1;
  if (tid < a.top_k) {
    const int id = a.ids[tid];
    int o = id % a.nranks;
    if (id < 0) {
      good_ids = 0;
      o = a.rank;
    }
    s_src[tid] = reinterpret_cast<const float4*>(
        reinterpret_cast<const uint8_t*>(a.peers[o]) + kEpSlotsOffset +
        ((size_t)a.buf * a.top_k + tid) * a.hidden * sizeof(float));
    s_w[tid] = a.route_w[tid];
  }
  ok = __syncthreads_and(ok);
  good_ids = __syncthreads_and(good_ids);
  if (ok && good_ids) {
    const int n4 = a.hidden >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    float4* o4 = reinterpret_cast<float4*>(a.out);
    for (int i = tid; i < n4; i += blockDim.x) {
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      // slots in groups of eight: all loads of a group in flight at once,
      // then the fmaf chain in route order
#pragma unroll
      for (int g = 0; g < kMaxJobs; g += 8) {
        if (g >= a.top_k) break;
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (g + j < a.top_k) v[j] = __ldcg(s_src[g + j] + i);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (g + j < a.top_k) {
            const float w = s_w[g + j];
            acc.x = fmaf(v[j].x, w, acc.x);
            acc.y = fmaf(v[j].y, w, acc.y);
            acc.z = fmaf(v[j].z, w, acc.z);
            acc.w = fmaf(v[j].w, w, acc.w);
          }
        }
      }
      if (x4) {
        const float4 xv = __ldcg(x4 + i);
        acc = make_float4(xv.x + acc.x, xv.y + acc.y, xv.z + acc.z, xv.w + acc.w);
      }
      o4[i] = acc;
    }
  } else if (tid == 0) {
    atomicExch(&g_device_error, ok ? kErrArg : kErrTimeout);
  }
  // Only this kernel touches seq, one launch after another on the stream.
  if (tid == 0) *reinterpret_cast<volatile uint64_t*>(seq) = e;
}

// Batched exchange (expert-major block of a decode batch): grid (column
// slices, tokens).  CTA (0, 0) publishes this rank's flag; every CTA waits for
// all flags, then sums its token's pairs in route order; the last CTA to
// finish advances seq (u32 counter at byte 520 of the region).
__global__ void __launch_bounds__(kEpBatchThreads) ep_batch_exchange_kernel(EpBatchExchange a) {
  __shared__ uint64_t s_epoch;
  __shared__ const float4* s_src[kMaxJobs];
  __shared__ float s_w[kMaxJobs];
  const int tid = threadIdx.x, t = blockIdx.y;
  const bool lead = blockIdx.x == 0 && blockIdx.y == 0;
  uint64_t* flags = reinterpret_cast<uint64_t*>(a.peers[a.rank]);
  uint64_t* seq = flags + kEpMaxRanks;
  unsigned* done = reinterpret_cast<unsigned*>(seq + 1);
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile uint64_t*>(seq) + 1;
    if (lead) asm volatile("fence.acq_rel.sys;" ::: "memory");
  }
  __syncthreads();
  const uint64_t e = s_epoch;
  if (lead && tid < a.nranks) st_release_sys(reinterpret_cast<uint64_t*>(a.peers[tid]) + a.rank, e);

  int ok = 1;
  if (tid < a.nranks) {
    const uint64_t* f = flags + tid;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      if ((int64_t)(ld_acquire_sys(f) - e) >= 0) break;
      if (it >= kEpSpinCap || ((it & 15u) == 15u && globaltimer_ns() - t0 > a.timeout_ns)) {
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
  }
  int good_ids = 1;
  if (tid < a.top_k) {
    const int p = t * a.top_k + tid;
    const int id = a.ids[p];
    int o = id % a.nranks;
    if (id < 0) {
      good_ids = 0;
      o = a.rank;
    }
    s_src[tid] = reinterpret_cast<const float4*>(
        reinterpret_cast<const uint8_t*>(a.peers[o]) + kEpSlotsOffset +
        ((size_t)a.buf * a.tokens * a.top_k + a.pos[p]) * a.hidden * sizeof(float));
    s_w[tid] = a.route_w[p];
  }
  ok = __syncthreads_and(ok);
  good_ids = __syncthreads_and(good_ids);
  const int n4 = a.hidden >> 2;
  const int i = blockIdx.x * blockDim.x + tid;
  if (ok && good_ids) {
    if (i < n4) {
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int g = 0; g < kMaxJobs; g += 8) {
        if (g >= a.top_k) break;
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (g + j < a.top_k) v[j] = __ldcg(s_src[g + j] + i);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (g + j < a.top_k) {
            const float w = s_w[g + j];
            acc.x = fmaf(v[j].x, w, acc.x);
            acc.y = fmaf(v[j].y, w, acc.y);
            acc.z = fmaf(v[j].z, w, acc.z);
            acc.w = fmaf(v[j].w, w, acc.w);
          }
        }
      }
      if (a.x) {
        const float4 xv = __ldcg(reinterpret_cast<const float4*>(a.x + (size_t)t * a.hidden) + i);
        acc = make_float4(xv.x + acc.x, xv.y + acc.y, xv.z + acc.z, xv.w + acc.w);
      }
      reinterpret_cast<float4*>(a.out + (size_t)t * a.hidden)[i] = acc;
    }
  } else if (tid == 0) {
    atomicExch(&g_device_error, ok ? kErrArg : kErrTimeout);
  }
  // every CTA read seq before it counts itself done; the next exchange on
  // this region is stream-ordered after this grid
  if (tid == 0) {
    const unsigned total = gridDim.x * gridDim.y;
    if (atomicAdd(done, 1u) == total - 1) {
      *done = 0u;
      *reinterpret_cast<volatile uint64_t*>(seq) = e;
    }
  }
}

}  // namespace

int launch_ep_batch_exchange_sum(const EpBatchExchange& a, cudaStream_t stream) {
  const int n4 = a.hidden / 4;
  const dim3 grid((n4 + kEpBatchThreads - 1) / kEpBatchThreads, a.tokens);
  ep_batch_exchange_kernel<<<grid, kEpBatchThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_ep_exchange_sum(const EpExchange& a, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kEpThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, ep_exchange_sum_kernel, a) != cudaSuccess) {
    (void)cudaGetLastError();
    return kErrLaunch;
  }
  return kOk;
}

int read_ep_device_error(bool clear) { return read_unit_error(clear); }

}  // namespace ervf
