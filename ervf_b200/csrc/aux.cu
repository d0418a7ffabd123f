// aux.cu -- the small kernels around the expert GEMV: route-order weighted
// accumulate, the device router, the device LRU slot table, the expert fetch
// into cache slots, and the order-exact masked down projection over the
// panel-major record.  Each one reproduces the arithmetic of the reference
// kernel it replaces (kennydd001/ervf
// src/moe_lab/lightningstream_nemotron/fused_nvfp4.py, lines cited per kernel).
#include "common.cuh"
#include "kernels.h"
#include "aux.h"
#include "route.cuh"

namespace ervf {

namespace {

// dst[i] = fmaf(src[i], w, dst[i])        (fused_nvfp4.py:125-133, :736-744)
__global__ void weighted_accumulate_kernel(float* __restrict__ dst, const float* __restrict__ src,
                                           float weight, const float* __restrict__ w_ptr, int n) {
  const float w = w_ptr ? *w_ptr : weight;
  const int i4 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i4 + 3 < n && ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0) {
    float4 d = *reinterpret_cast<float4*>(dst + i4);
    const float4 s = *reinterpret_cast<const float4*>(src + i4);
    d.x = fmaf(s.x, w, d.x);
    d.y = fmaf(s.y, w, d.y);
    d.z = fmaf(s.z, w, d.z);
    d.w = fmaf(s.w, w, d.w);
    *reinterpret_cast<float4*>(dst + i4) = d;
  } else {
    for (int i = i4; i < n && i < i4 + 4; ++i) dst[i] = fmaf(src[i], w, dst[i]);
  }
}

// ---------------------------------------------------------------- router
//
// route_topk_f32 (fused_nvfp4.py:433-465): sc = 1/(1+expf(-logit)),
// choice = sc + bias; top_k serial selections of the strictly greatest choice
// (lowest index on ties, nothing selected above -3e38 -> expert 0); weights
// sc[id] / (wsum + 1e-20f) * scaling with wsum summed in route order.
// One warp: each selection is a warp argmax with (value desc, index asc).
__global__ void route_topk_kernel(const float* __restrict__ rlog, const float* __restrict__ gate_b,
                                  int* __restrict__ ids, float* __restrict__ w, int n, int top_k,
                                  float scaling, int bad_pick) {
  __shared__ float sc[1024], ch[1024];
  __shared__ int sel[64];
  const int lane = threadIdx.x;
  for (int i = lane; i < n; i += 32) {
    const float s = 1.0f / (1.0f + expf(-rlog[i]));
    sc[i] = s;
    ch[i] = s + gate_b[i];
  }
  __syncwarp();
  auto argmax = [&]() -> int {
    float bv = -3.0e38f;
    int bi = 0;
    for (int e = lane; e < n; e += 32)
      if (ch[e] > bv) { bv = ch[e]; bi = e; }
    if (bv == -3.0e38f) bi = 0x7fffffff;  // nothing valid in this lane
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    return bi == 0x7fffffff ? 0 : bi;
  };
  for (int s = 0; s < top_k; ++s) {
    int bi = argmax();
    if (bad_pick && s == top_k - 1) {
      __syncwarp();
      if (lane == 0) ch[bi] = -3.0e38f;
      __syncwarp();
      bi = argmax();
    }
    __syncwarp();
    if (lane == 0) {
      sel[s] = bi;
      ch[bi] = -3.0e38f;
    }
    __syncwarp();
  }
  if (lane == 0) {
    float wsum = 0.0f;
    for (int s = 0; s < top_k; ++s) {
      ids[s] = sel[s];
      w[s] = sc[sel[s]];
      wsum += sc[sel[s]];
    }
    for (int s = 0; s < top_k; ++s) w[s] = w[s] / (wsum + 1e-20f) * scaling;
  }
}

// The same router for `layers` independent problems, one warp each, with the
// scores held in registers (lane l owns experts l, l+32, ...).  Identical
// selections and weights as route_topk_kernel: the arithmetic per expert and
// the route-order weight sum are the same operations in the same order.
template <int NPL>
__global__ void route_topk_warp_kernel(const float* __restrict__ rlog, const float* __restrict__ gate_b,
                                       int* __restrict__ ids, float* __restrict__ w, int layers, int n,
                                       int top_k, float scaling, int bad_pick, int bias_stride) {
  const int layer = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (layer >= layers) return;
  route_topk_warp<NPL>(rlog + (size_t)layer * n, gate_b ? gate_b + (size_t)layer * bias_stride : nullptr,
                       ids + (size_t)layer * top_k, w + (size_t)layer * top_k, n, top_k, scaling,
                       bad_pick);
}

// ------------------------------------------------------------- device LRU
//
// cache_assign (fused_nvfp4.py:470-511): one thread walks the route slots in
// order; hits refresh last_used, misses append while filling and then evict
// the minimum last_used slot (lowest slot on ties).  This is a restatement of
// the reference's serial state machine step for step, by contract: the
// runtime reads the same slot / victim / stats state, so the order of every
// update is part of the interface.  It is a compat path (the resident bank
// needs no LRU) and is not on the timed decode path.
__global__ void cache_assign_kernel(int* __restrict__ slot_of, int* __restrict__ expert_of,
                                    int* __restrict__ last_used, int* __restrict__ state2,
                                    const int* __restrict__ ids, int* __restrict__ slots,
                                    int* __restrict__ need, int* __restrict__ stats2, int cap,
                                    int top_k) {
  if (threadIdx.x != 0) return;
  int tick = state2[0], filled = state2[1];
  for (int s = 0; s < top_k; ++s) {
    const int e = ids[s];
    const int sl = slot_of[e];
    if (sl >= 0) {
      last_used[sl] = ++tick;
      slots[s] = sl;
      need[s] = 0;
      stats2[0] += 1;
      continue;
    }
    stats2[1] += 1;
    int v;
    if (filled < cap) {
      v = filled++;
    } else {
      v = 0;
      int mnv = last_used[0];
      for (int c = 1; c < cap; ++c)
        if (last_used[c] < mnv) { mnv = last_used[c]; v = c; }
      slot_of[expert_of[v]] = -1;
    }
    slot_of[e] = v;
    expert_of[v] = e;
    last_used[v] = ++tick;
    slots[s] = v;
    need[s] = 1;
  }
  state2[0] = tick;
  state2[1] = filled;
}

// cache_fetch (fused_nvfp4.py:516-543): copy the code and scale records of
// every missed route slot from the bank (device or mapped host memory) into
// its cache slot.  blockIdx.y = route slot; 16-byte vectors when aligned.
__global__ void cache_fetch_kernel(const uint8_t* __restrict__ bank_c, const uint8_t* __restrict__ bank_s,
                                   uint8_t* __restrict__ cache_c, uint8_t* __restrict__ cache_s,
                                   const int* __restrict__ ids, const int* __restrict__ slots,
                                   const int* __restrict__ need, size_t code_bytes,
                                   size_t scale_bytes) {
  const int s = blockIdx.y;
  if (!need[s]) return;
  const uint8_t* cs = bank_c + (size_t)ids[s] * code_bytes;
  const uint8_t* ss = bank_s + (size_t)ids[s] * scale_bytes;
  uint8_t* cd = cache_c + (size_t)slots[s] * code_bytes;
  uint8_t* sd = cache_s + (size_t)slots[s] * scale_bytes;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t t0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool vec = (((uintptr_t)cs | (uintptr_t)ss | (uintptr_t)cd | (uintptr_t)sd |
                     code_bytes | scale_bytes) & 15u) == 0;
  if (vec) {
    const size_t nc = code_bytes >> 4, ns = scale_bytes >> 4;
    for (size_t v = t0; v < nc + ns; v += stride) {
      if (v < nc) reinterpret_cast<uint4*>(cd)[v] = reinterpret_cast<const uint4*>(cs)[v];
      else reinterpret_cast<uint4*>(sd)[v - nc] = reinterpret_cast<const uint4*>(ss)[v - nc];
    }
  } else {
    for (size_t v = t0; v < code_bytes + scale_bytes; v += stride) {
      if (v < code_bytes) cd[v] = cs[v];
      else sd[v - code_bytes] = ss[v - code_bytes];
    }
  }
}

// ------------------------------------------------------ masked down path
//
// panel_scan (fused_nvfp4.py:157-187): per 16-column panel, the bit mask of
// nonzero activations and the ascending list of active panels.  One block.
__global__ void panel_scan_kernel(const float* __restrict__ act, int inter,
                                  unsigned* __restrict__ masks, int* __restrict__ plist,
                                  int* __restrict__ pcount, int* __restrict__ nz,
                                  int* __restrict__ nzc) {
  extern __shared__ unsigned smask[];
  const int npanel = inter >> 4;
  for (int p = threadIdx.x; p < npanel; p += blockDim.x) {
    unsigned m = 0;
    for (int c = 0; c < 16; ++c)
      if (act[16 * p + c] != 0.0f) m |= 1u << c;
    smask[p] = m;
    masks[p] = m;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int n = 0, m = 0;
    for (int p = 0; p < npanel; ++p) {
      const unsigned mk = smask[p];
      if (mk) {
        plist[n++] = p;
        for (int c = 0; c < 16; ++c)
          if (mk & (1u << c)) nz[m++] = (p << 4) + c;
      }
    }
    *pcount = n;
    *nzc = m;
  }
}

// gemv_down_masked_partial + reduce_partials (fused_nvfp4.py:225-271,
// :408-419) in one launch.  Block = 32 rows x nchunks chunks; chunk c of row
// r accumulates active panels pi = c, c+nchunks, ... with columns ascending,
// then the row's partials are summed in chunk order from 0.0.  The inner loop
// restates the reference's panel walk (panel stride, mask-bit order, fmaf per
// set bit) by contract: that order is the masked down path's numeric result.
// A compat path for the runtime's panel-major records, not on the timed
// decode path.
__global__ void down_masked_kernel(const uint8_t* __restrict__ bank, const float* __restrict__ act,
                                   const unsigned* __restrict__ masks, const int* __restrict__ plist,
                                   const int* __restrict__ pcount, float global_scale,
                                   const int* __restrict__ id_ptr, const float* __restrict__ globals,
                                   size_t panel_bytes, float* __restrict__ out, int rows, int inter,
                                   int nchunks) {
  __shared__ float lut[256];
  __shared__ float parts[32 * 33];
  float g = global_scale;
  const uint8_t* rec = bank;
  if (id_ptr) {
    const int e = *id_ptr;
    g = globals[e * 2 + 0];
    rec = bank + (size_t)e * panel_bytes;
  }
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = e4m3_lut_value((uint32_t)i) * g;
  __syncthreads();
  const int lr = threadIdx.x & 31, chunk = threadIdx.x >> 5;
  const int row = blockIdx.x * 32 + lr;
  const int rowhalf = rows >> 1;
  const size_t stride = (size_t)rows + 16u * (size_t)rowhalf;
  const int pc = *pcount;
  float acc = 0.0f;
  if (row < rows && chunk < nchunks) {
    const int hb = row >> 1, hi = row & 1;
    for (int pi = chunk; pi < pc; pi += nchunks) {
      const int p = plist[pi];
      const uint8_t* pb = rec + (size_t)p * stride;
      const float s = lut[pb[row]];
      unsigned m = masks[p];
      while (m) {
        const int c = __ffs(m) - 1;
        m &= m - 1;
        const uint32_t byte = pb[rows + (size_t)c * rowhalf + hb];
        const float w = e2m1_value(hi ? (byte >> 4) : (byte & 15u)) * s;
        acc = fmaf(w, act[(p << 4) + c], acc);
      }
    }
  }
  if (chunk < nchunks) parts[chunk * 33 + lr] = acc;
  __syncthreads();
  if (chunk == 0 && row < rows) {
    float a = 0.0f;
    for (int c = 0; c < nchunks; ++c) a += parts[c * 33 + lr];
    out[row] = a;
  }
}

// Row-major NVFP4 down record -> panel-major record (runtime.py:34-52), one
// thread per (panel, output byte).  Used by the residency path.
__global__ void panel_major_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                   uint8_t* __restrict__ block, int rows, int inter) {
  const int npanel = inter >> 4, rowhalf = rows >> 1;
  const size_t stride = (size_t)rows + 16u * (size_t)rowhalf;
  const size_t total = (size_t)npanel * stride;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int p = (int)(i / stride);
    const int o = (int)(i - (size_t)p * stride);
    uint8_t v;
    if (o < rows) {
      v = scales[(size_t)o * npanel + p];
    } else {
      const int c = (o - rows) / rowhalf, h = (o - rows) % rowhalf;
      const int j = 16 * p + c;
      const uint8_t b0 = codes[(size_t)(2 * h) * (inter >> 1) + (j >> 1)];
      const uint8_t b1 = codes[(size_t)(2 * h + 1) * (inter >> 1) + (j >> 1)];
      const uint8_t n0 = (j & 1) ? (b0 >> 4) : (b0 & 15);
      const uint8_t n1 = (j & 1) ? (b1 >> 4) : (b1 & 15);
      v = (uint8_t)(n0 | (n1 << 4));
    }
    block[i] = v;
  }
}

// Expert-parallel route-order sum: slot s's down output sits in the gathered
// buffer of the rank that owns expert ids[s] (ids[s] % nranks);
// out[r] = x[r] + chain_s fmaf(y_s[r], w[s], .) from 0.0 -- the same
// arithmetic as the single-GPU routed-sum epilogue.
__global__ void ep_route_sum_kernel(const float* __restrict__ gathered, const int* __restrict__ ids,
                                    const float* __restrict__ w, int top_k, const float* __restrict__ x,
                                    float* __restrict__ out, int hidden, int nranks) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= hidden) return;
  float acc = 0.0f;
  for (int s = 0; s < top_k; ++s) {
    const int owner = ids[s] % nranks;
    acc = fmaf(gathered[((size_t)owner * top_k + s) * hidden + r], w[s], acc);
  }
  out[r] = x ? x[r] + acc : acc;
}

inline int launched() { return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch; }

}  // namespace

int launch_ep_route_sum(const float* gathered, const int* ids, const float* w, int top_k,
                        const float* x, float* out, int hidden, int nranks, cudaStream_t stream) {
  ep_route_sum_kernel<<<(hidden + 255) / 256, 256, 0, stream>>>(gathered, ids, w, top_k, x, out,
                                                                 hidden, nranks);
  return launched();
}

int launch_weighted_accumulate(float* dst, const float* src, float weight, const float* w_ptr,
                               int n, cudaStream_t stream) {
  const int threads = 256;
  const int blocks = ((n + 3) / 4 + threads - 1) / threads;
  weighted_accumulate_kernel<<<blocks, threads, 0, stream>>>(dst, src, weight, w_ptr, n);
  return launched();
}

int launch_route_topk(const float* rlog, const float* gate_b, int* ids, float* w, int n, int top_k,
                      float scaling, int bad_pick, cudaStream_t stream) {
  return launch_route_topk_batched(rlog, gate_b, ids, w, 1, n, top_k, scaling, bad_pick, 0, stream);
}

// Softmax top-k routing (config 2, Qwen shape), one warp per layer: the k
// largest logits in descending order, ties to the lowest index (the order of
// the reference router's strict `>` scan), then w_i = e_i / sum with
// e_i = expf(logit_i - logit_max) over the selected experts and sum added in
// selection order from 0 -- the renormalised softmax of the selected experts
// (the full softmax denominator cancels).  n <= 32 * NPL, top_k <= 32.
template <int NPL>
__global__ void route_topk_softmax_kernel(const float* __restrict__ rlog, int* __restrict__ ids,
                                          float* __restrict__ w, int layers, int n, int top_k) {
  const int lane = threadIdx.x & 31;
  const int layer = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (layer >= layers) return;
  const float* lg = rlog + (size_t)layer * n;
  float v[NPL];
  bool taken[NPL];
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < n ? lg[e] : 0.0f;
    taken[j] = e >= n;
  }
  float top = 0.0f, mine = 0.0f, sum = 0.0f;
  int my_id = 0;
  for (int s = 0; s < top_k; ++s) {
    float bv = 0.0f;
    int bi = -1;
#pragma unroll
    for (int j = 0; j < NPL; ++j)
      if (!taken[j] && (bi < 0 || v[j] > bv)) {
        bv = v[j];
        bi = lane + 32 * j;
      }
    // warp arg-max: larger value wins, equal values go to the lower index
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if (s == 0) top = bv;
    const float e = expf(bv - top);
    sum += e;
    if (lane == s) {
      my_id = bi;
      mine = e;
    }
#pragma unroll
    for (int j = 0; j < NPL; ++j)
      if (bi == lane + 32 * j) taken[j] = true;
  }
  if (lane < top_k) {
    ids[(size_t)layer * top_k + lane] = my_id;
    w[(size_t)layer * top_k + lane] = mine / sum;
  }
}

int launch_route_topk_softmax(const float* rlog, int* ids, float* w, int layers, int n, int top_k,
                              cudaStream_t stream) {
  const int warps = 4;
  const int grid = (layers + warps - 1) / warps;
  if (n <= 128) {
    route_topk_softmax_kernel<4><<<grid, 32 * warps, 0, stream>>>(rlog, ids, w, layers, n, top_k);
  } else if (n <= 256) {
    route_topk_softmax_kernel<8><<<grid, 32 * warps, 0, stream>>>(rlog, ids, w, layers, n, top_k);
  } else {
    route_topk_softmax_kernel<32><<<grid, 32 * warps, 0, stream>>>(rlog, ids, w, layers, n, top_k);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

// Expert-major lists of a decode batch (one CTA): the P = T * k route pairs
// (token t, slot s) at p = t*k + s, sorted by expert and, inside an expert,
// by p (deterministic).  pos[p] = sorted position, tok_sorted[q] = token of
// the pair at sorted position q; chunks of <= 16 pairs of one expert:
// chunk_expert / chunk_off / chunk_n, n_chunks.  An id outside [0, E) is
// recorded in the device error word and counted as expert 0.  With expert
// parallelism every rank sorts all pairs (so pos is the same on every rank)
// but makes chunks only of the experts it owns (e % ep_ranks == ep_rank).
__global__ void moe_batch_lists_kernel(const int* __restrict__ ids, int P, int k, int E,
                                       int* chunk_expert, int* chunk_off, int* chunk_n,
                                       int* n_chunks, int* tok_sorted, int* pos, int ep_ranks,
                                       int ep_rank) {
  __shared__ int cnt[kMaxBatchExperts];
  __shared__ int off[kMaxBatchExperts];
  __shared__ int choff[kMaxBatchExperts];
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int q = tid; q < P; q += blockDim.x) {
    int e = ids[q];
    if (e < 0 || e >= E) {
      atomicExch(&g_device_error, kErrArg);
      e = 0;
    }
    atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int o = 0, c = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = o;
      choff[e] = c;
      o += cnt[e];
      if (e % ep_ranks == ep_rank) c += (cnt[e] + 15) / 16;
    }
    *n_chunks = c;
  }
  __syncthreads();
  for (int q = tid; q < P; q += blockDim.x) {
    int e = ids[q];
    if (e < 0 || e >= E) e = 0;
    int rank = 0;
    for (int r = 0; r < q; ++r) {
      int f = ids[r];
      if (f < 0 || f >= E) f = 0;
      rank += f == e;
    }
    const int sp = off[e] + rank;
    pos[q] = sp;
    tok_sorted[sp] = q / k;
  }
  for (int e = tid; e < E; e += blockDim.x) {
    if (e % ep_ranks != ep_rank) continue;
    const int nc = (cnt[e] + 15) / 16;
    for (int c = 0; c < nc; ++c) {
      chunk_expert[choff[e] + c] = e;
      chunk_off[choff[e] + c] = off[e] + 16 * c;
      chunk_n[choff[e] + c] = min(16, cnt[e] - 16 * c);
    }
  }
}

// out[t][r] = x[t][r] + acc, acc = fmaf(contrib[pos[t*k+s]][r], w[t*k+s], acc)
// over the route slots s = 0..k-1 in order from 0.0 (route-order contract).
__global__ void moe_batch_routesum_kernel(const float* __restrict__ contrib, const int* __restrict__ pos,
                                          const float* __restrict__ w, const float* __restrict__ x,
                                          float* __restrict__ out, int hidden, int k) {
  const int t = blockIdx.y;
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= hidden) return;
  float acc = 0.0f;
  for (int s = 0; s < k; ++s)
    acc = fmaf(__ldcg(&contrib[(size_t)pos[t * k + s] * hidden + r]), w[t * k + s], acc);
  out[(size_t)t * hidden + r] = (x ? x[(size_t)t * hidden + r] : 0.0f) + acc;
}

int launch_moe_batch_lists(const int* ids, int P, int k, int E, int* chunk_expert, int* chunk_off,
                           int* chunk_n, int* n_chunks, int* tok_sorted, int* pos, int ep_ranks,
                           int ep_rank, cudaStream_t stream) {
  moe_batch_lists_kernel<<<1, 512, 0, stream>>>(ids, P, k, E, chunk_expert, chunk_off, chunk_n, n_chunks,
                                               tok_sorted, pos, ep_ranks, ep_rank);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_moe_batch_routesum(const float* contrib, const int* pos, const float* w, const float* x,
                              float* out, int T, int hidden, int k, cudaStream_t stream) {
  moe_batch_routesum_kernel<<<dim3((hidden + 255) / 256, T), 256, 0, stream>>>(contrib, pos, w, x, out,
                                                                               hidden, k);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_route_topk_batched(const float* rlog, const float* gate_b, int* ids, float* w, int layers,
                              int n, int top_k, float scaling, int bad_pick, int bias_stride,
                              cudaStream_t stream) {
  const int warps = 4;
  const int grid = (layers + warps - 1) / warps;
  if (n <= 128) {
    route_topk_warp_kernel<4><<<grid, 32 * warps, 0, stream>>>(rlog, gate_b, ids, w, layers, n, top_k,
                                                               scaling, bad_pick, bias_stride);
  } else if (n <= 256) {
    route_topk_warp_kernel<8><<<grid, 32 * warps, 0, stream>>>(rlog, gate_b, ids, w, layers, n, top_k,
                                                               scaling, bad_pick, bias_stride);
  } else {
    for (int l = 0; l < layers; ++l) {
      route_topk_kernel<<<1, 32, 0, stream>>>(rlog + (size_t)l * n,
                                              gate_b + (size_t)l * bias_stride, ids + (size_t)l * top_k,
                                              w + (size_t)l * top_k, n, top_k, scaling, bad_pick);
    }
  }
  return launched();
}

int launch_cache_assign(int* slot_of, int* expert_of, int* last_used, int* state2, const int* ids,
                        int* slots, int* need, int* stats2, int cap, int top_k, cudaStream_t stream) {
  cache_assign_kernel<<<1, 32, 0, stream>>>(slot_of, expert_of, last_used, state2, ids, slots, need,
                                            stats2, cap, top_k);
  return launched();
}

int launch_cache_fetch(const uint8_t* bank_c, const uint8_t* bank_s, uint8_t* cache_c, uint8_t* cache_s,
                       const int* ids, const int* slots, const int* need, size_t code_bytes,
                       size_t scale_bytes, int top_k, cudaStream_t stream) {
  const dim3 grid(64, top_k);
  cache_fetch_kernel<<<grid, 256, 0, stream>>>(bank_c, bank_s, cache_c, cache_s, ids, slots, need,
                                               code_bytes, scale_bytes);
  return launched();
}

int launch_down_masked(const uint8_t* bank, const float* act, unsigned* masks, int* plist,
                       int* pcount, int* nz, int* nzc, float global_scale, const int* id_ptr,
                       const float* globals, size_t panel_bytes, float* out, int rows, int inter,
                       int nchunks, cudaStream_t stream) {
  const int npanel = inter >> 4;
  panel_scan_kernel<<<1, 256, npanel * sizeof(unsigned), stream>>>(act, inter, masks, plist, pcount,
                                                                   nz, nzc);
  if (launched() != kOk) return kErrLaunch;
  down_masked_kernel<<<(rows + 31) / 32, 32 * nchunks, 0, stream>>>(
      bank, act, masks, plist, pcount, global_scale, id_ptr, globals, panel_bytes, out, rows, inter,
      nchunks);
  return launched();
}

// sum[c] = sum over b < n of acts[b][c], nodes in order: the union panel
// mask of the batched masked down (down_union, sweepspec.py:337-343) is the
// nonzero pattern of this sum.
__global__ void node_sum_kernel(const float* __restrict__ acts, int n, int inter, float* __restrict__ sum) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= inter) return;
  float a = 0.0f;
  for (int b = 0; b < n; ++b) a += acts[(size_t)b * inter + c];
  sum[c] = a;
}

int launch_down_union(const uint8_t* bank, const float* acts, int n, float* act_sum, unsigned* masks,
                      int* plist, int* pcount, int* nz, int* nzc, float global_scale, float* out, int rows,
                      int inter, int nchunks, cudaStream_t stream) {
  const int npanel = inter >> 4;
  node_sum_kernel<<<(inter + 255) / 256, 256, 0, stream>>>(acts, n, inter, act_sum);
  if (launched() != kOk) return kErrLaunch;
  panel_scan_kernel<<<1, 256, npanel * sizeof(unsigned), stream>>>(act_sum, inter, masks, plist, pcount,
                                                                   nz, nzc);
  if (launched() != kOk) return kErrLaunch;
  // every node walks the union panel list and masks: a column where the
  // node is zero adds fmaf(w, 0, acc) = acc, and the panel -> chunk
  // assignment (by position in the list) is the reference's
  for (int b = 0; b < n; ++b) {
    down_masked_kernel<<<(rows + 31) / 32, 32 * nchunks, 0, stream>>>(
        bank, acts + (size_t)b * inter, masks, plist, pcount, global_scale, nullptr, nullptr, 0,
        out + (size_t)b * rows, rows, inter, nchunks);
    if (launched() != kOk) return kErrLaunch;
  }
  return kOk;
}

int launch_panel_major(const uint8_t* codes, const uint8_t* scales, uint8_t* block, int rows,
                       int inter, cudaStream_t stream) {
  const size_t total = (size_t)(inter >> 4) * ((size_t)rows + 16u * (size_t)(rows >> 1));
  int blocks = (int)((total + 255) / 256);
  if (blocks > 8192) blocks = 8192;
  panel_major_kernel<<<blocks, 256, 0, stream>>>(codes, scales, block, rows, inter);
  return launched();
}

int read_aux_device_error(bool clear) { return read_unit_error(clear); }

// ------------------------------------------------------ SweepMoE plumbing
//
// Row gather / scatter by a device index list and the batched route-order
// slot sum of the expert-major block (sweepspec.py:244-375).

namespace {

// dst[b][:] = src[idx[b]][:] (cols floats each), b < n
__global__ void gather_rows_kernel(const float* __restrict__ src, const int* __restrict__ idx, int cols,
                                   float* __restrict__ dst) {
  const int b = blockIdx.y;
  const size_t row = (size_t)__ldg(&idx[b]);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x)
    dst[(size_t)b * cols + i] = src[row * cols + i];
}

// dst[idx[b]][:] = src[b][:]
__global__ void scatter_rows_kernel(const float* __restrict__ src, const int* __restrict__ idx, int cols,
                                    float* __restrict__ dst) {
  const int b = blockIdx.y;
  const size_t row = (size_t)__ldg(&idx[b]);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x)
    dst[row * cols + i] = src[(size_t)b * cols + i];
}

// out[b][r] = fmaf(w[b][s], contrib[b][s][r], out[b][r]) for s = 0..top_k-1
// in route-slot order, starting from out's value (reduce_slots,
// sweepspec.py:219-240: the per-node order of the token-major path).
__global__ void reduce_slots_kernel(const float* __restrict__ contrib, const float* __restrict__ w,
                                    float* __restrict__ out, int rows, int top_k) {
  const int b = blockIdx.y;
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float a = out[(size_t)b * rows + r];
  for (int s = 0; s < top_k; ++s)
    a = fmaf(__ldg(&w[b * top_k + s]), contrib[((size_t)b * top_k + s) * rows + r], a);
  out[(size_t)b * rows + r] = a;
}

}  // namespace

int launch_gather_rows(const float* src, const int* idx, int n, int cols, float* dst, cudaStream_t stream) {
  gather_rows_kernel<<<dim3((cols + 1023) / 1024, n), 256, 0, stream>>>(src, idx, cols, dst);
  return launched();
}

int launch_scatter_rows(const float* src, const int* idx, int n, int cols, float* dst, cudaStream_t stream) {
  scatter_rows_kernel<<<dim3((cols + 1023) / 1024, n), 256, 0, stream>>>(src, idx, cols, dst);
  return launched();
}

int launch_reduce_slots(const float* contrib, const float* w, float* out, int rows, int top_k, int B,
                        cudaStream_t stream) {
  reduce_slots_kernel<<<dim3((rows + 255) / 256, B), 256, 0, stream>>>(contrib, w, out, rows, top_k);
  return launched();
}

}  // namespace ervf
