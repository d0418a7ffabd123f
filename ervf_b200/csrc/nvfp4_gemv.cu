// nvfp4_gemv.cu -- NVFP4 decode-GEMV kernels (batch 1), bit-exact to the
// reference ERVF reduction (kennydd001/ervf fused_nvfp4.py:295-406; numeric
// contract fused_nvfp4.py:31-122).
//
// Two families:
//
//  * nvfp4_gemv_tma  -- the B200 schedule.  A producer warp streams tiles of
//    RT rows (codes, block scales and, for the routed-sum launch, the
//    activation) into a ring of shared-memory stages with 1-D bulk copies
//    (cp.async.bulk, no multicast) completing on mbarriers.  Each consumer
//    thread owns one "chain group" c (four consecutive reference chains
//    4c..4c+3, i.e. one 16-byte code unit per round) and keeps the activation
//    of its columns in registers for the whole launch.  Codes are decoded two
//    at a time with the sm_100a e2m1x2 converter and the fp32 products and
//    fused multiply-adds run on the packed f32x2 pipe, pairing chains j and
//    j+2 of the same unit (same row, same column offset).  Chain values go to
//    shared memory and are reduced by the reference tree.
//
//  * nvfp4_gemv_sched<W> -- the reference's ERVF widths 4/8/16/32 as
//    schedules: W lanes per row, lane L owns chains L + W*i.  Same chains,
//    same tree, any alignment >= 4 bytes; also the fallback where the TMA
//    schedule's preconditions (cols % 32 == 0, cols <= 4096, 16-B aligned
//    bases) do not hold.
#include "common.cuh"
#include "kernels.h"

namespace ervf {

// -------------------------------------------------------------- helpers

__device__ __forceinline__ void resolve(const MatRef& m, const uint8_t*& c, const uint8_t*& s,
                                        float& g) {
  c = m.codes;
  s = m.scales;
  g = m.g;
  if (m.slot_ptr) {
    const size_t slot = (size_t)(*m.slot_ptr);
    c += slot * m.code_stride;
    s += slot * m.scale_stride;
  }
  if (m.id_ptr) g = m.globals[(*m.id_ptr) * 2 + m.gsel];
}

// Canonicalised group sum for the legacy tree: its second butterfly adds the
// zero lanes, i.e. S + 0.0 (fused_nvfp4.py:107-112).
__device__ __forceinline__ float legacy_fix(float s, int legacy) { return legacy ? s + 0.0f : s; }

// Eight fmaf of one uchar4, in the order lo,hi of .x,.y,.z,.w
// (fused_nvfp4.py:336-344); s is RN(e4m3 * g).
__device__ __forceinline__ float uchar4_chain(uint32_t q, float s, const float* __restrict__ xk,
                                              float acc) {
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t byte = (q >> (8 * b)) & 0xFFu;
    acc = fmaf(e2m1_value(byte & 15u) * s, xk[2 * b], acc);
    acc = fmaf(e2m1_value(byte >> 4) * s, xk[2 * b + 1], acc);
  }
  return acc;
}

// ======================================================================
// Width schedules (and general fallback)
// ======================================================================

template <int W>
__global__ void __launch_bounds__(256) nvfp4_gemv_sched(GemvBatch p, int tiles_per_job) {
  constexpr int RP = 256 / W;          // rows per pass
  constexpr int ITEMS = (RP * 8 + 255) / 256;  // tree items per thread
  extern __shared__ __align__(16) float sm[];
  float* sx = sm;                      // [cols]
  float* lut = sx + p.cols;            // [256]  RN(e4m3 * g)
  float* part = lut + 256;             // [RP][kRowPitch]

  const int tid = threadIdx.x;
  const int cols = p.cols;
  const int n_bytes = cols >> 1, n_vec = n_bytes >> 2, n_sc = cols >> 4;
  const int T = blockIdx.x;
  int job0, njob, r0;
  if (p.mode == 0) {
    job0 = T / tiles_per_job;
    njob = 1;
    r0 = (T % tiles_per_job) * RP;
  } else {
    job0 = 0;
    njob = p.njobs;
    r0 = T * RP;
  }
  if (p.mode == 0 && !job_active(p, job0)) return;  // expert owned by another rank
  const int nrows = min(RP, p.rows - r0);
  float racc[ITEMS];
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) racc[i] = 0.0f;

  const int lrow = tid / W, L = tid % W;
  for (int jj = 0; jj < njob; ++jj) {
    const int j = job0 + jj;
    const GemvJob& J = p.job[j];
    const uint8_t *codes, *scales;
    float g;
    resolve(J.mat, codes, scales, g);
    __syncthreads();  // previous job's readers of sx / lut / part are done
    for (int i = tid; i < cols; i += 256) sx[i] = J.x[i];
    lut[tid] = e4m3_lut_value((uint32_t)tid) * g;
    __syncthreads();

    if (lrow < nrows) {
      const size_t row = (size_t)(r0 + lrow);
      const uint32_t* crow = reinterpret_cast<const uint32_t*>(codes + row * n_bytes);
      const uint8_t* srow = scales + row * n_sc;
      float* prow = part + lrow * kRowPitch;
#pragma unroll 1
      for (int vi = 0; vi < 256 / W; ++vi) {
        const int t = L + W * vi;
        float acc = 0.0f;
        for (int v = t; v < n_vec; v += 256) {
          const float s = lut[srow[v >> 1]];
          acc = uchar4_chain(crow[v], s, sx + (v << 3), acc);
        }
        prow[part_index(t)] = acc;
      }
    }
    __syncthreads();

#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int item = tid + 256 * i;
      const int tr = item >> 3, tw = item & 7;
      float y = 0.0f;
      if (tr < nrows) y = group_tree(part + tr * kRowPitch + tw * kGroupPitch);
      y = combine8(legacy_fix(y, p.legacy_tree));
      if (tw == 0 && tr < nrows) {
        const int r = r0 + tr;
        if (p.mode == 0) {
          J.out[r] = epilogue(y, p.relu2, p.out_scale);
        } else {
          if (jj == 0) racc[i] = p.base ? p.base[r] : 0.0f;
          racc[i] = fmaf(y, p.route_w[j], racc[i]);
          if (jj == njob - 1) p.rs_out[r] = p.resid ? p.resid[r] + racc[i] : racc[i];
        }
      }
    }
  }
}

// ======================================================================
// TMA-staged B200 schedule
// ======================================================================
//
// CTA = 4 consumer warps + 1 producer warp, three CTAs per SM.  A work item
// is a block of kRt rows of one job; the items of a launch (job-major) are
// dealt to the CTAs round-robin.
//
// Producer warp: bulk-copies an item's codes and scale bytes into a free
// stage and, when the job's activation differs per item (mode 1), copies the
// activation into the stage in a rotated layout (float4 i of unit u at slot
// (i + u) & 7) so that the consumers of eight consecutive units read eight
// different bank groups.
//
// Consumer thread (row_off, c): chain group c = reference chains 4c..4c+3,
// i.e. one 16-byte code unit per round, for rows row_off, row_off + p_rows,
// ... of the item, activation of its columns in registers.  Codes are decoded
// with the hardware e2m1x2 converter; each weight is w = RN(e2m1 * s) (FMUL)
// and acc = fmaf(w, x, acc) (FFMA), in the reference's order.  Chain values
// go to shared memory; after a consumer barrier two warps run the 256-leaf
// tree of the item's rows.
//
// mode 1 (routed sum): a tree thread writes its row's job output y_s to
// contrib[s][row], publishes it with a release fence and a per-row atomic
// count, and the thread that completes a row's count adds the row up in
// ROUTE order, acc = fmaf(y_s, w_s, acc) for s = 0..njobs-1, writes x + acc
// and resets the count.  Rows therefore spread over all CTAs, and the sum is
// the same as one thread walking the slots in order.

constexpr int kRt = 8;  // rows per item

struct TmaCfg {
  int stages;
  int stage_bytes;  // bytes per stage (128-aligned)
  int scale_off;    // scale bytes inside a stage
  int x_off;        // mode 1: rotated activation inside a stage
  int part_off;     // chain buffers [2][kRt][kRowPitch] floats
  int stage_base;
  int n_u, gw, p_rows;
  int tiles_per_job;  // row blocks per job
  int ntiles;         // njobs * tiles_per_job
  int stage_x;        // 1: the activation travels with each item (mode 1)
};

__device__ __forceinline__ void item_of(const TmaCfg& c, int T, int& job, int& rb) {
  job = T / c.tiles_per_job;
  rb = T - job * c.tiles_per_job;
}

// One 16-byte code unit (4 chains x 8 codes) of one row.  Chains 0,1 use the
// block scale s0 = s_2u, chains 2,3 use s1 = s_2u+1; xr[8j + m] is the
// activation of chain j's m-th code.
__device__ __forceinline__ void unit_fma(const uint4 q, const float s0, const float s1,
                                         const float (&xr)[32], float (&acc)[4]) {
  float f0[8], f1[8], f2[8], f3[8];
  e2m1x8_to_f32(q.x, f0);
  e2m1x8_to_f32(q.y, f1);
  e2m1x8_to_f32(q.z, f2);
  e2m1x8_to_f32(q.w, f3);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    acc[0] = fmaf(f0[m] * s0, xr[m], acc[0]);
    acc[1] = fmaf(f1[m] * s0, xr[8 + m], acc[1]);
    acc[2] = fmaf(f2[m] * s1, xr[16 + m], acc[2]);
    acc[3] = fmaf(f3[m] * s1, xr[24 + m], acc[3]);
  }
}

__device__ __forceinline__ void unpack_x(const float4 (&v4)[8], float (&xr)[32]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    xr[4 * i] = v4[i].x; xr[4 * i + 1] = v4[i].y; xr[4 * i + 2] = v4[i].z; xr[4 * i + 3] = v4[i].w;
  }
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <int ROUNDS>
__global__ void __launch_bounds__(160, 3) nvfp4_gemv_tma(GemvBatch p, TmaCfg c) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int NC = 128;  // consumer threads
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = c.stages;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  const uint8_t** jc = reinterpret_cast<const uint8_t**>(smem + 128);
  const uint8_t** js = jc + kMaxJobs;
  float* jg = reinterpret_cast<float*>(js + kMaxJobs);
  float* luts = reinterpret_cast<float*>(smem + 448);  // [njobs][256]
  float* part = reinterpret_cast<float*>(smem + c.part_off);
  uint8_t* stages = smem + c.stage_base;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], c.stage_x ? 2 : 1);
      mbar_init(&empty[i], NC / 32);
    }
    fence_mbar_init();
  }
  for (int i = tid; i < 2 * kRt * kRowPitch; i += blockDim.x) part[i] = 0.0f;
  // Slot / id tables and globals: readable now if they were produced before
  // the predecessor kernel, otherwise only after the dependency wait.
  if (!p.ids_ready) grid_dep_wait();
  if (tid < p.njobs) {
    const uint8_t *cc, *ss;
    float g;
    resolve(p.job[tid].mat, cc, ss, g);
    jc[tid] = cc;
    js[tid] = ss;
    jg[tid] = g;
  }
  __syncthreads();
  for (int i = tid; i < p.njobs * 256; i += blockDim.x)
    luts[i] = e4m3_lut_value((uint32_t)(i & 255)) * jg[i >> 8];
  __syncthreads();

  const int cols = p.cols;
  const int cb = cols >> 1, sb = cols >> 4;

  // ------------------------------------------------------------ producer
  if (warp == NC / 32) {
    int it = 0;
    bool waited = false;
    for (int T = blockIdx.x; T < c.ntiles; T += gridDim.x) {
      int job, rb;
      item_of(c, T, job, rb);
      if (!job_active(p, job)) continue;
      const int st = it % S;
      if (!mbar_wait(&empty[st], ((it / S) & 1) ^ 1)) break;
      ++it;
      const int r0 = rb * kRt;
      const int nrows = min(kRt, p.rows - r0);
      uint8_t* dst = stages + (size_t)st * c.stage_bytes;
      if (lane == 0) {
        const uint32_t code_bytes = (uint32_t)(nrows * cb);
        const uint32_t scale_bytes = (uint32_t)(nrows * sb);
        const uint32_t s16 = scale_bytes & ~15u;
        const uint8_t* ssrc = js[job] + (size_t)r0 * sb;
        for (uint32_t i = s16; i < scale_bytes; ++i) dst[c.scale_off + i] = ssrc[i];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_expect_tx(&full[st], code_bytes + s16);
        bulk_g2s(dst, jc[job] + (size_t)r0 * cb, code_bytes, &full[st]);
        if (s16) bulk_g2s(dst + c.scale_off, ssrc, s16, &full[st]);
      }
      if (c.stage_x) {
        if (!waited) { grid_dep_wait(); waited = true; }
        const float4* src = reinterpret_cast<const float4*>(p.job[job].x);
        float4* xs = reinterpret_cast<float4*>(dst + c.x_off);
        for (int f = lane; f < (cols >> 2); f += 32) {
          const int u = f >> 3, i = f & 7;
          xs[u * 8 + ((i + u) & 7)] = src[f];
        }
        __threadfence_block();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[st]);
      }
    }
    if (lane == 0)  // leave no bulk copy in flight: wait (bounded) for the last stages
      for (int k = (it > S ? it - S : 0); k < it; ++k) mbar_wait(&full[k % S], (k / S) & 1);
    if (!waited) grid_dep_wait();
    grid_dep_launch();
    return;
  }

  // ----------------------------------------------------------- consumers
  grid_dep_wait();  // activations / residual are written by the predecessor
  grid_dep_launch();
  const int row_off = tid / c.gw, cg = tid % c.gw;
  const bool active = row_off < c.p_rows;
  float xr[ROUNDS][32];
#pragma unroll
  for (int i = 0; i < ROUNDS; ++i)
#pragma unroll
    for (int m = 0; m < 32; ++m) xr[i][m] = 0.0f;
  const float* cur_x = nullptr;
  // The tree runs on warps 1 and 3: with 64 chain groups per row these hold
  // groups 32..63, which have no second round when 64 < cols/32 <= 128, so
  // the tree lands on the warps with the least decode work.
  const bool tree_warp = (warp & 1) == 1;
  const int tt = ((warp >> 1) << 5) | lane;  // 0..63 over warps 1 and 3
  const int tr = tt >> 3, tw = tt & 7;

  int it = 0;
  for (int T = blockIdx.x; T < c.ntiles; T += gridDim.x) {
    int job, rb;
    item_of(c, T, job, rb);
    if (!job_active(p, job)) continue;
    const int cur = it++;
    const int st = cur % S, pb = cur & 1;
    const int r0 = rb * kRt;
    const int nrows = min(kRt, p.rows - r0);
    const GemvJob& J = p.job[job];
    if (!c.stage_x && J.x != cur_x) {
      if (active) {
#pragma unroll
        for (int i = 0; i < ROUNDS; ++i) {
          const int u = cg + 64 * i;
          if (u < c.n_u) {
            const float4* src = reinterpret_cast<const float4*>(J.x + 32 * u);
            float4 v4[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) v4[m] = src[m];
            unpack_x(v4, xr[i]);
          }
        }
      }
      cur_x = J.x;
    }
    const bool to = !mbar_wait(&full[st], (cur / S) & 1);
    const uint8_t* stage = stages + (size_t)st * c.stage_bytes;
    if (active && !to) {
      if (c.stage_x) {
        const float4* xs = reinterpret_cast<const float4*>(stage + c.x_off);
#pragma unroll
        for (int i = 0; i < ROUNDS; ++i) {
          const int u = cg + 64 * i;
          if (u < c.n_u) {
            float4 v4[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) v4[m] = xs[u * 8 + ((m + u) & 7)];
            unpack_x(v4, xr[i]);
          }
        }
      }
      const float* lut = luts + job * 256;
      float* pbuf = part + pb * kRt * kRowPitch;
#pragma unroll 2
      for (int rr = row_off; rr < nrows; rr += c.p_rows) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < ROUNDS; ++i) {
          const int u = cg + 64 * i;
          if (i == 0 || u < c.n_u) {
            const uint4 q = *reinterpret_cast<const uint4*>(stage + rr * cb + 16 * u);
            const uint32_t sv = *reinterpret_cast<const uint16_t*>(stage + c.scale_off + rr * sb + 2 * u);
            unit_fma(q, lut[sv & 0xFFu], lut[sv >> 8], xr[i], acc);
          }
        }
        *reinterpret_cast<float4*>(pbuf + rr * kRowPitch + part_index(4 * cg)) =
            make_float4(acc[0], acc[1], acc[2], acc[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (named_bar_or(1, NC, to)) break;

    if (tree_warp) {
      const float* pbuf = part + pb * kRt * kRowPitch;
      float y = 0.0f;
      if (tr < nrows) y = group_tree(pbuf + tr * kRowPitch + tw * kGroupPitch);
      y = combine8(legacy_fix(y, p.legacy_tree));
      if (tw == 0 && tr < nrows) {
        const int r = r0 + tr;
        if (p.mode == 0) {
          J.out[r] = epilogue(y, p.relu2, p.out_scale);
        } else {
          p.contrib[(size_t)job * p.rows + r] = y;
          __threadfence();
          if (atomicAdd(&p.row_count[r], 1) == p.njobs - 1) {
            __threadfence();
            float acc = p.base ? p.base[r] : 0.0f;
            for (int s = 0; s < p.njobs; ++s)
              acc = fmaf(__ldcg(&p.contrib[(size_t)s * p.rows + r]), p.route_w[s], acc);
            p.rs_out[r] = p.resid ? p.resid[r] + acc : acc;
            p.row_count[r] = 0;
          }
        }
      }
    }
  }
}

// ======================================================================
// host side
// ======================================================================

namespace {

struct DevInfo {
  int sms = 0, smem_optin = 0, smem_sm = 0;
};

DevInfo& dev_info() {
  static DevInfo info[64];
  int d = 0;
  cudaGetDevice(&d);
  DevInfo& i = info[d & 63];
  if (i.sms == 0) {
    cudaDeviceGetAttribute(&i.sms, cudaDevAttrMultiProcessorCount, d);
    cudaDeviceGetAttribute(&i.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d);
    cudaDeviceGetAttribute(&i.smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, d);
  }
  return i;
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

template <typename K>
int set_smem(K kernel, int bytes) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return kErrLaunch;
  return kOk;
}

bool tma_ok(const GemvBatch& b) {
  if (b.cols % 32 != 0 || b.cols > 4096) return false;
  if (b.mode == 1 && (!b.contrib || !b.row_count)) return false;
  for (int j = 0; j < b.njobs; ++j) {
    const MatRef& m = b.job[j].mat;
    if (!al16(m.codes) || !al16(m.scales) || !al16(b.job[j].x)) return false;
    if (m.slot_ptr && ((m.code_stride & 15u) || (m.scale_stride & 15u))) return false;
  }
  return true;
}

template <typename K>
int launch_ex(K kernel, dim3 grid, dim3 block, int smem, cudaStream_t stream, bool pdl,
              const GemvBatch& b, const TmaCfg& c) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, b, c) == cudaSuccess ? kOk : kErrLaunch;
}

constexpr int kCtasPerSm = 3;

int launch_tma(const GemvBatch& b, cudaStream_t stream) {
  const DevInfo& di = dev_info();
  TmaCfg c{};
  c.n_u = b.cols / 32;
  c.gw = c.n_u < 64 ? c.n_u : 64;
  const int rounds = (c.n_u + 63) / 64;
  const int NC = 128;
  c.p_rows = NC / c.gw;
  const int cb = b.cols / 2, sb = b.cols / 16;
  c.stage_x = b.mode == 1 ? 1 : 0;
  c.part_off = align_up(448 + b.njobs * 1024, 16);
  c.stage_base = align_up(c.part_off + 2 * kRt * kRowPitch * 4, 128);
  c.scale_off = kRt * cb;
  c.x_off = c.scale_off + align_up(kRt * sb, 16);
  c.stage_bytes = align_up(c.x_off + (c.stage_x ? b.cols * 4 : 0), 128);
  const int budget = (di.smem_sm - kCtasPerSm * 1024) / kCtasPerSm;
  c.stages = (budget - c.stage_base) / c.stage_bytes;
  if (c.stages > 6) c.stages = 6;
  if (c.stages < 2) {
    c.stages = 2;
    if (c.stage_base + 2 * c.stage_bytes > di.smem_optin) return kErrShape;
  }
  const int smem = c.stage_base + c.stages * c.stage_bytes;
  c.tiles_per_job = (b.rows + kRt - 1) / kRt;
  c.ntiles = c.tiles_per_job * b.njobs;
  int grid = di.sms * kCtasPerSm;
  if (grid > c.ntiles) grid = c.ntiles;
  const dim3 block(NC + 32);
  const bool pdl = b.pdl != 0;
  if (rounds == 1) {
    if (set_smem(nvfp4_gemv_tma<1>, smem)) return kErrLaunch;
    return launch_ex(nvfp4_gemv_tma<1>, dim3(grid), block, smem, stream, pdl, b, c);
  }
  if (set_smem(nvfp4_gemv_tma<2>, smem)) return kErrLaunch;
  return launch_ex(nvfp4_gemv_tma<2>, dim3(grid), block, smem, stream, pdl, b, c);
}

template <int W>
int launch_sched_w(const GemvBatch& b, cudaStream_t stream) {
  constexpr int RP = 256 / W;
  const int smem = (b.cols + 256 + RP * kRowPitch) * 4;
  if (smem > dev_info().smem_optin) return kErrShape;
  if (set_smem(nvfp4_gemv_sched<W>, smem)) return kErrLaunch;
  const int tiles = (b.rows + RP - 1) / RP;
  const int grid = b.mode == 0 ? tiles * b.njobs : tiles;
  nvfp4_gemv_sched<W><<<grid, 256, smem, stream>>>(b, tiles);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

int device_sm_count() { return dev_info().sms; }
int device_smem_optin() { return dev_info().smem_optin; }

int read_device_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return kErrLaunch;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return kErrLaunch;
  }
  return v;
}

int launch_nvfp4_batch(const GemvBatch& b, int width, cudaStream_t stream) {
  switch (width) {
    case 0:
      if (tma_ok(b)) return launch_tma(b, stream);
      return launch_sched_w<32>(b, stream);
    case 4: return launch_sched_w<4>(b, stream);
    case 8: return launch_sched_w<8>(b, stream);
    case 16: return launch_sched_w<16>(b, stream);
    case 32: return launch_sched_w<32>(b, stream);
    default: return kErrArg;
  }
}

}  // namespace ervf
