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

struct TmaCfg {
  int rt;           // rows per sub-tile
  int stages;
  int stage_bytes;  // bytes per stage (128-aligned)
  int scale_off;    // offset of scales inside a stage
  int x_off;        // offset of the activation inside a stage (stage_x)
  int stage_x;      // 1: the activation travels with each sub-tile (mode 1)
  int n_u, gw, p_rows;
  int tiles_per_job, ntiles, nsub;
};

__device__ __forceinline__ void tile_coords(const GemvBatch& p, const TmaCfg& c, int T, int sub,
                                            int& job, int& r0, int& nrows) {
  if (p.mode == 0) {
    job = T / c.tiles_per_job;
    r0 = (T % c.tiles_per_job) * c.rt;
  } else {
    job = sub;
    r0 = T * c.rt;
  }
  nrows = min(c.rt, p.rows - r0);
}

// One 16-byte code unit (4 chains x 8 codes) of one row.  Pair A = chains
// (0,2), pair B = chains (1,3); both pairs use the scale pair (s_2u, s_2u+1).
__device__ __forceinline__ void unit_fma(const uint4 q, const float2 s, const float2 (&xa)[8],
                                         const float2 (&xb)[8], float2& accA, float2& accB) {
  uint32_t h0[4], h1[4], h2[4], h3[4];
  e2m1x8_to_f16x2(q.x, h0);
  e2m1x8_to_f16x2(q.y, h1);
  e2m1x8_to_f16x2(q.z, h2);
  e2m1x8_to_f16x2(q.w, h3);
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const float2 e0 = f16x2_to_f32x2(h0[b]);
    const float2 e2 = f16x2_to_f32x2(h2[b]);
    const float2 e1 = f16x2_to_f32x2(h1[b]);
    const float2 e3 = f16x2_to_f32x2(h3[b]);
    accA = fma2(mul2(make_float2(e0.x, e2.x), s), xa[2 * b], accA);
    accB = fma2(mul2(make_float2(e1.x, e3.x), s), xb[2 * b], accB);
    accA = fma2(mul2(make_float2(e0.y, e2.y), s), xa[2 * b + 1], accA);
    accB = fma2(mul2(make_float2(e1.y, e3.y), s), xb[2 * b + 1], accB);
  }
}

// Activation columns of unit u as the chain pairs use them:
// xa[m] = (x[32u+m], x[32u+16+m]), xb[m] = (x[32u+8+m], x[32u+24+m]).
__device__ __forceinline__ void load_x_unit(const float* __restrict__ x, int u, float2 (&xa)[8],
                                            float2 (&xb)[8]) {
  const float4* p = reinterpret_cast<const float4*>(x + 32 * u);
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 f = p[i];
    v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    xa[m] = make_float2(v[m], v[16 + m]);
    xb[m] = make_float2(v[8 + m], v[24 + m]);
  }
}

template <int ROUNDS>
__global__ void __launch_bounds__(288, 1) nvfp4_gemv_tma(GemvBatch p, TmaCfg c) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int NC = blockDim.x - 32;  // consumer threads
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = c.stages;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  float* luts = reinterpret_cast<float*>(smem + 128);
  float* part = luts + p.njobs * 256;                    // [2][rt][kRowPitch]
  uint8_t* stages = reinterpret_cast<uint8_t*>(part + 2 * c.rt * kRowPitch);

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NC / 32);
    }
    fence_mbar_init();
  }
  for (int i = tid; i < p.njobs * 256; i += blockDim.x) {
    const uint8_t *cc, *ss;
    float g;
    resolve(p.job[i >> 8].mat, cc, ss, g);
    luts[i] = e4m3_lut_value((uint32_t)(i & 255)) * g;
  }
  for (int i = tid; i < 2 * c.rt * kRowPitch; i += blockDim.x) part[i] = 0.0f;
  __syncthreads();

  const int cols = p.cols;
  const int cb = cols >> 1, sb = cols >> 4;

  // ------------------------------------------------------------ producer
  if (warp == NC / 32) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int T = blockIdx.x; ok && T < c.ntiles; T += gridDim.x) {
        for (int sub = 0; sub < c.nsub; ++sub) {
          int job, r0, nrows;
          tile_coords(p, c, T, sub, job, r0, nrows);
          if (!job_active(p, job)) continue;
          const int st = it % S;
          if (!mbar_wait(&empty[st], ((it / S) & 1) ^ 1)) { ok = false; break; }
          ++it;
          const uint8_t *cc, *ss;
          float g;
          resolve(p.job[job].mat, cc, ss, g);
          uint8_t* dst = stages + (size_t)st * c.stage_bytes;
          const uint32_t code_bytes = (uint32_t)(nrows * cb);
          const uint32_t scale_bytes = (uint32_t)(nrows * sb);
          const uint32_t s16 = scale_bytes & ~15u;
          const uint8_t* ssrc = ss + (size_t)r0 * sb;
          for (uint32_t i = s16; i < scale_bytes; ++i) dst[c.scale_off + i] = ssrc[i];
          const uint32_t xbytes = c.stage_x ? (uint32_t)(cols * 4) : 0u;
          mbar_arrive_expect_tx(&full[st], code_bytes + s16 + xbytes);
          bulk_g2s(dst, cc + (size_t)r0 * cb, code_bytes, &full[st]);
          if (s16) bulk_g2s(dst + c.scale_off, ssrc, s16, &full[st]);
          if (xbytes) bulk_g2s(dst + c.x_off, p.job[job].x, xbytes, &full[st]);
        }
      }
      // Leave no bulk copy in flight: wait (bounded) for the last issued stages.
      for (int k = (it > S ? it - S : 0); k < it; ++k) mbar_wait(&full[k % S], (k / S) & 1);
    }
    return;
  }

  // ----------------------------------------------------------- consumers
  const int row_off = tid / c.gw, cg = tid % c.gw;
  const bool active = row_off < c.p_rows;
  float2 xa[ROUNDS][8], xb[ROUNDS][8];
#pragma unroll
  for (int i = 0; i < ROUNDS; ++i)
#pragma unroll
    for (int m = 0; m < 8; ++m) { xa[i][m] = make_float2(0.f, 0.f); xb[i][m] = xa[i][m]; }
  const float* cur_x = nullptr;
  float racc = 0.0f;
  const int tr = tid >> 3, tw = tid & 7;
  const bool tree_warp = warp < (8 * c.rt + 31) / 32;

  int it = 0;
  bool dead = false;
  for (int T = blockIdx.x; !dead && T < c.ntiles; T += gridDim.x) {
    for (int sub = 0; sub < c.nsub; ++sub) {
      int job, r0, nrows;
      tile_coords(p, c, T, sub, job, r0, nrows);
      if (!job_active(p, job)) continue;
      const int cur = it++;
      const int st = cur % S, pb = cur & 1;
      const GemvJob& J = p.job[job];
      if (!c.stage_x && active && J.x != cur_x) {
#pragma unroll
        for (int i = 0; i < ROUNDS; ++i) {
          const int u = cg + 64 * i;
          if (u < c.n_u) load_x_unit(J.x, u, xa[i], xb[i]);
        }
        cur_x = J.x;
      }
      const bool to = !mbar_wait(&full[st], (cur / S) & 1);
      const uint8_t* stage = stages + (size_t)st * c.stage_bytes;
      if (active && !to) {
        if (c.stage_x) {
          const float* xs = reinterpret_cast<const float*>(stage + c.x_off);
#pragma unroll
          for (int i = 0; i < ROUNDS; ++i) {
            const int u = cg + 64 * i;
            if (u < c.n_u) load_x_unit(xs, u, xa[i], xb[i]);
          }
        }
        const float* lut = luts + job * 256;
        float* pbuf = part + pb * c.rt * kRowPitch;
#pragma unroll 2
        for (int rr = row_off; rr < nrows; rr += c.p_rows) {
          float2 accA = make_float2(0.f, 0.f), accB = make_float2(0.f, 0.f);
#pragma unroll
          for (int i = 0; i < ROUNDS; ++i) {
            const int u = cg + 64 * i;
            if (i == 0 || u < c.n_u) {
              const uint4 q = *reinterpret_cast<const uint4*>(stage + rr * cb + 16 * u);
              const uint32_t sv = *reinterpret_cast<const uint16_t*>(stage + c.scale_off + rr * sb + 2 * u);
              const float2 s = make_float2(lut[sv & 0xFFu], lut[sv >> 8]);
              unit_fma(q, s, xa[i], xb[i], accA, accB);
            }
          }
          *reinterpret_cast<float4*>(pbuf + rr * kRowPitch + part_index(4 * cg)) =
              make_float4(accA.x, accB.x, accA.y, accB.y);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (named_bar_or(1, NC, to)) { dead = true; break; }

      if (tree_warp) {
        const float* pbuf = part + pb * c.rt * kRowPitch;
        float y = 0.0f;
        if (tr < nrows) y = group_tree(pbuf + tr * kRowPitch + tw * kGroupPitch);
        y = combine8(legacy_fix(y, p.legacy_tree));
        if (tw == 0 && tr < nrows) {
          const int r = r0 + tr;
          if (p.mode == 0) {
            J.out[r] = epilogue(y, p.relu2, p.out_scale);
          } else {
            if (sub == 0) racc = p.base ? p.base[r] : 0.0f;
            racc = fmaf(y, p.route_w[sub], racc);
            if (sub == c.nsub - 1) p.rs_out[r] = p.resid ? p.resid[r] + racc : racc;
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
  int sms = 0, smem_optin = 0;
};

DevInfo& dev_info() {
  static DevInfo info[64];
  int d = 0;
  cudaGetDevice(&d);
  DevInfo& i = info[d & 63];
  if (i.sms == 0) {
    cudaDeviceGetAttribute(&i.sms, cudaDevAttrMultiProcessorCount, d);
    cudaDeviceGetAttribute(&i.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d);
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
  for (int j = 0; j < b.njobs; ++j) {
    const MatRef& m = b.job[j].mat;
    if (!al16(m.codes) || !al16(m.scales) || !al16(b.job[j].x)) return false;
    if (m.slot_ptr && ((m.code_stride & 15u) || (m.scale_stride & 15u))) return false;
  }
  return true;
}

int launch_tma(const GemvBatch& b, cudaStream_t stream) {
  const DevInfo& di = dev_info();
  TmaCfg c{};
  c.n_u = b.cols / 32;
  c.gw = c.n_u < 64 ? c.n_u : 64;
  const int rounds = (c.n_u + 63) / 64;
  const int NC = 256;
  c.p_rows = NC / c.gw;
  c.stage_x = b.mode == 1 ? 1 : 0;
  c.rt = 16;
  const int fixed = 128 + b.njobs * 1024 + 2 * c.rt * kRowPitch * 4;
  c.scale_off = c.rt * (b.cols / 2);
  c.x_off = c.scale_off + align_up(c.rt * (b.cols / 16), 16);
  c.stage_bytes = align_up(c.x_off + (c.stage_x ? b.cols * 4 : 0), 128);
  c.stages = (di.smem_optin - fixed) / c.stage_bytes;
  if (c.stages > 4) c.stages = 4;
  if (c.stages < 2) return kErrShape;
  const int tiles = (b.rows + c.rt - 1) / c.rt;
  if (b.mode == 0) {
    c.tiles_per_job = tiles;
    c.ntiles = tiles * b.njobs;
    c.nsub = 1;
  } else {
    c.tiles_per_job = tiles;
    c.ntiles = tiles;
    c.nsub = b.njobs;
  }
  const int smem = fixed + c.stages * c.stage_bytes;
  int grid = c.ntiles < di.sms ? c.ntiles : di.sms;
  const dim3 block(NC + 32);
  cudaError_t e;
  if (rounds == 1) {
    if (set_smem(nvfp4_gemv_tma<1>, smem)) return kErrLaunch;
    nvfp4_gemv_tma<1><<<grid, block, smem, stream>>>(b, c);
  } else {
    if (set_smem(nvfp4_gemv_tma<2>, smem)) return kErrLaunch;
    nvfp4_gemv_tma<2><<<grid, block, smem, stream>>>(b, c);
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? kOk : kErrLaunch;
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
