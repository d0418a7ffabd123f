// nvfp4_gemv.cu -- NVFP4 decode-GEMV kernels (batch 1), bit-exact to the
// reference ERVF reduction (kennydd001/ervf fused_nvfp4.py:295-406; numeric
// contract fused_nvfp4.py:31-122).
//
// Two families:
//
//  * nvfp4_gemv_tma  -- the B200 schedule.  A producer warp streams items of
//    up to 32 rows (codes and block scales) into a ring of shared-memory
//    stages with 1-D bulk copies (cp.async.bulk, no multicast) completing on
//    mbarriers.  Each of 256 consumer threads owns one "chain group" g (four
//    consecutive reference chains 4g..4g+3, i.e. the 16-byte code unit g) for
//    a slot of rows and keeps that unit's activation in registers; second-
//    round units (cols > 2048) are spread evenly over all threads.  Codes and
//    scales are decoded with the sm_100a e2m1x2 / e4m3x2 converters.  Chain
//    values go to shared memory and are reduced by the reference tree.
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
// CTA = 8 consumer warps + 1 producer warp, two CTAs per SM.  Each CTA owns a
// contiguous, balanced range of row blocks over the launch's active jobs and
// walks it in items of up to kRt rows.
//
// Producer warp (lane 0): per item, one bulk copy of the item's code rows and
// one of its scale rows (cp.async.bulk, no multicast) into a ring of stages
// completing on mbarriers; the consumers release a stage through a second
// mbarrier.  Weight streaming starts before the dependency wait of a
// programmatic launch (the weights do not depend on the predecessor).
//
// Consumers: a row of n_u code units (16 bytes = 4 chains x 8 codes each) has
// 64 chain groups; group c (the reference's chains 4c..4c+3) covers unit c
// and, when cols > 2048, unit 64 + c (its second round, which continues the
// same four chains).  The consumer threads form T = 256 / n_u teams of n_u
// threads; team k owns rows k + T*j, j < 2H, of every item (kRt = T * 2H),
// interleaved so that a partial item splits evenly, and every team thread
// runs exactly two "segments" of H rows (even j, or odd j) x one unit:
//   thread m <  n2          : group m,    even rows: unit m, then unit 64+m
//   thread n2 <= m < 2*n2   : group m-n2, odd rows:  unit c, then unit 64+c
//   thread m >= 2*n2        : group m-n2, even rows, then odd rows, unit c
// with n2 = n_u - 64 groups that have a second unit.  Every thread therefore
// does 2H unit-rows per item (an even split of the row's n_u units).  The
// segment's activation (32 values) is read into registers from a swizzled
// shared copy of x (kept across items when both segments use one unit);
// codes and block scales are decoded with the sm_100a
// e2m1x2 / e4m3x2 converters, w = RN(e2m1 * s) (FMUL) and acc = fmaf(w, x,
// acc) (FFMA) in the reference's order.  Chain values go to the item's chain
// buffer; after a consumer barrier thread (row tr, segment tw) reduces chains
// 32tw..32tw+31 of its row with the reference's shuffle tree (offsets 16..1)
// and eight lanes combine ((S0+S4)+(S2+S6))+((S1+S5)+(S3+S7)).
//
// mode 1 (routed sum): the tree lane of a row writes the job's row value y_s
// to contrib[s][row], publishes it (acq_rel atomic on a per-row count), and
// the lane that completes a row's count adds the row up in ROUTE order,
// acc = fmaf(y_s, w_s, acc) for s = 0..njobs-1 from base or 0, writes
// resid + acc and resets the count -- the same sum as one thread walking the
// slots in order, with the rows spread over every SM.

constexpr int kCW = 8;          // consumer warps
constexpr int kCT = kCW * 32;   // consumer threads
constexpr int kBarC = 1;        // named barrier of the consumer threads

struct TmaCfg {
  int stages;       // ring depth
  int stage_bytes;  // bytes per stage (128-aligned)
  int scale_off;    // scale rows inside a stage
  int part_off;     // chain buffer [kRt][kRowPitch] floats
  int xs_off;       // activation [n_u][8] float4, swizzled
  int stage_base;
  int n_u;          // code units per row (cols / 32)
  int n2;           // chain groups with a second unit (n_u - 64, or 0)
  int teams;        // T
  int blk;          // rows per row block (4 or 8: 16-byte aligned scale rows)
  int kb;           // row blocks per item (kRt / blk)
  int bpj;          // row blocks per job
};

// One 16-byte code unit (4 chains x 8 codes) of one row, continuing the four
// chain accumulators acc[0..3].  Chains 0,1 use the block scale s0 = s_2u,
// chains 2,3 use s1 = s_2u+1; x[8j + m] is the activation of chain j's m-th
// code.
__device__ __forceinline__ void unit_fma(const uint4 q, const float s0, const float s1,
                                         const float (&x)[32], float* acc) {
  float f0[8], f1[8], f2[8], f3[8];
  e2m1x8_to_f32(q.x, f0);
  e2m1x8_to_f32(q.y, f1);
  e2m1x8_to_f32(q.z, f2);
  e2m1x8_to_f32(q.w, f3);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    acc[0] = fmaf(f0[m] * s0, x[m], acc[0]);
    acc[1] = fmaf(f1[m] * s0, x[8 + m], acc[1]);
    acc[2] = fmaf(f2[m] * s1, x[16 + m], acc[2]);
    acc[3] = fmaf(f3[m] * s1, x[24 + m], acc[3]);
  }
}

// Block scales s_2u, s_2u+1 of a unit: RN(e4m3 * g) from two scale bytes.
__device__ __forceinline__ float2 unit_scales(uint32_t sv, float g) {
  const float2 e = e4m3x2_to_f32x2(sv);
  return make_float2(e.x * g, e.y * g);
}

// Row `row` of a stage, unit u: continue acc[0..3].
__device__ __forceinline__ void stage_unit(const uint8_t* stage, int scale_off, int cb, int sb,
                                           int row, int u, float g, const float (&x)[32],
                                           float* acc) {
  const uint4 qv = *reinterpret_cast<const uint4*>(stage + row * cb + 16 * u);
  const uint32_t sv = *reinterpret_cast<const uint16_t*>(stage + scale_off + row * sb + 2 * u);
  const float2 s = unit_scales(sv, g);
  unit_fma(qv, s.x, s.y, x, acc);
}

// Activation of unit u from the swizzled shared copy (float4 i at u*8 + (i ^ (u & 7))).
__device__ __forceinline__ void load_unit_x(const float4* xs, int u, float (&x)[32]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v = xs[u * 8 + (i ^ (u & 7))];
    x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
  }
}

// The two segments of one consumer thread for one item (see the schedule
// above).  FULL: every row of the item exists, so the H rows of a segment run
// unconditionally and interleave.
template <int H, bool FULL>
__device__ __forceinline__ void segments(const uint8_t* stage, int scale_off, int cb, int sb,
                                         int team, int T, int par1, int par2, bool cont, int u1,
                                         int u2, int grp, int nrows, float gs, const float4* xs,
                                         float (&x)[32], bool& x_stale, float* part) {
  float acc[H][4];
#pragma unroll
  for (int h = 0; h < H; ++h) acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.0f;
  if (cont || x_stale) load_unit_x(xs, u1, x);
  x_stale = false;
#pragma unroll
  for (int h = 0; h < H; ++h) {
    const int row = team + T * (2 * h + par1);
    if (FULL || row < nrows) stage_unit(stage, scale_off, cb, sb, row, u1, gs, x, acc[h]);
  }
  if (!cont) {
#pragma unroll
    for (int h = 0; h < H; ++h) {
      const int row = team + T * (2 * h + par1);
      if (FULL || row < nrows)
        *reinterpret_cast<float4*>(part + row * kRowPitch + part_index(4 * grp)) =
            make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
      acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.0f;
    }
  } else {
    load_unit_x(xs, u2, x);
  }
#pragma unroll
  for (int h = 0; h < H; ++h) {
    const int row = team + T * (2 * h + par2);
    if (FULL || row < nrows) stage_unit(stage, scale_off, cb, sb, row, u2, gs, x, acc[h]);
  }
#pragma unroll
  for (int h = 0; h < H; ++h) {
    const int row = team + T * (2 * h + par2);
    if (FULL || row < nrows)
      *reinterpret_cast<float4*>(part + row * kRowPitch + part_index(4 * grp)) =
          make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
  }
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// The CTA's items: row blocks [blk, blk_end) of the flattened (active job,
// block) space, cut at job ends and at kb blocks.
struct ItemSeq {
  int blk, blk_end;
};

__device__ __forceinline__ void cta_blocks(int total, ItemSeq& q) {
  const int G = gridDim.x, b = blockIdx.x;
  const int per = total / G, rem = total % G;
  q.blk = b * per + min(b, rem);
  q.blk_end = q.blk + per + (b < rem ? 1 : 0);
}

__device__ __forceinline__ bool next_item(ItemSeq& q, const TmaCfg& c, const int* jlist, int rows,
                                          int& job, int& r0, int& nrows) {
  if (q.blk >= q.blk_end) return false;
  const int ji = q.blk / c.bpj, jb = q.blk - ji * c.bpj;
  const int n = min(c.kb, min(c.bpj - jb, q.blk_end - q.blk));
  job = jlist[ji];
  r0 = jb * c.blk;
  nrows = min(n * c.blk, rows - r0);
  q.blk += n;
  return true;
}

template <int H>
__global__ void __launch_bounds__(kCT + 32, 2) nvfp4_gemv_tma(GemvBatch p, TmaCfg c) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int S = c.stages;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [S], S <= 8
  uint64_t* empty = full + 8;                         // [S]
  const uint8_t** jc = reinterpret_cast<const uint8_t**>(smem + 128);
  const uint8_t** js = jc + kMaxJobs;
  float* jg = reinterpret_cast<float*>(smem + 384);
  int* jlist = reinterpret_cast<int*>(smem + 448);
  int* nact = jlist + kMaxJobs;
  float* part = reinterpret_cast<float*>(smem + c.part_off);
  float4* xs = reinterpret_cast<float4*>(smem + c.xs_off);
  uint8_t* stages = smem + c.stage_base;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    fence_mbar_init();
  }
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
  if (tid == 0) {
    int n = 0;
    for (int j = 0; j < p.njobs; ++j)
      if (job_active(p, j)) jlist[n++] = j;
    *nact = n;
  }
  __syncthreads();

  const int cb = p.cols >> 1, sb = p.cols >> 4;
  ItemSeq q;
  cta_blocks(*nact * c.bpj, q);

  // ------------------------------------------------------------ producer
  if (tid >= kCT) {
    if (tid == kCT) {
      int it = 0, job, r0, nrows;
      while (next_item(q, c, jlist, p.rows, job, r0, nrows)) {
        const int st = it % S;
        if (!mbar_wait(&empty[st], ((it / S) & 1) ^ 1)) break;
        ++it;
        uint8_t* dst = stages + (size_t)st * c.stage_bytes;
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
      // Leave no bulk copy in flight: wait (bounded) for the last stages.
      for (int k = (it > S ? it - S : 0); k < it; ++k) mbar_wait(&full[k % S], (k / S) & 1);
    }
    grid_dep_wait();
    grid_dep_launch();
    return;
  }

  // ----------------------------------------------------------- consumers
  grid_dep_wait();  // activations / base / residual come from the predecessor
  grid_dep_launch();
  const int krt = c.teams * 2 * H;
  for (int i = tid; i < krt * kRowPitch; i += kCT) part[i] = 0.0f;

  // this thread's two segments (see the schedule above)
  const int nu = c.n_u, n2 = c.n2;
  const int team = tid / nu, m = tid - team * nu;
  const bool active = team < c.teams;
  const bool cont = m < 2 * n2;                // segment 2 continues segment 1
  const int grp = m < n2 ? m : m - n2;         // chain group
  const int u1 = grp, u2 = cont ? grp + 64 : grp;
  // team rows team + T*j, j < 2H; segment rows j = 2h + parity
  const int T = c.teams;
  const int par1 = (m >= n2 && m < 2 * n2) ? 1 : 0;
  const int par2 = cont ? par1 : 1;
  const int tr = tid >> 3, tw = tid & 7;
  const float* cur_x = nullptr;
  // segment activation; a thread whose two segments share one unit keeps it
  // in registers until the job's activation changes
  float x[32];
  bool x_stale = true;
  named_bar_sync(kBarC, kCT);

  int it = 0, job, r0, nrows;
  while (next_item(q, c, jlist, p.rows, job, r0, nrows)) {
    const int st = it % S;
    const uint32_t ph = (it / S) & 1;
    ++it;
    const GemvJob& J = p.job[job];
    if (J.x != cur_x) {  // the previous item ended with a consumer barrier
      const float4* src = reinterpret_cast<const float4*>(J.x);
      for (int f = tid; f < nu * 8; f += kCT) {
        const int t = f >> 3, i = f & 7;
        xs[t * 8 + (i ^ (t & 7))] = __ldg(src + f);
      }
      named_bar_sync(kBarC, kCT);
      cur_x = J.x;
      x_stale = true;
    }
    const float gs = jg[job];
    const bool to = !mbar_wait(&full[st], ph);
    const uint8_t* stage = stages + (size_t)st * c.stage_bytes;

    if (active) {
      if (nrows == krt) {
        segments<H, true>(stage, c.scale_off, cb, sb, team, T, par1, par2, cont, u1, u2, grp, nrows,
                          gs, xs, x, x_stale, part);
      } else {
        segments<H, false>(stage, c.scale_off, cb, sb, team, T, par1, par2, cont, u1, u2, grp, nrows,
                           gs, xs, x, x_stale, part);
      }
    }
    // every read of the stage is done; a timeout anywhere stops all consumers
    const bool stop = named_bar_or(kBarC, kCT, to);
    if (tid == 0) mbar_arrive(&empty[st]);
    if (stop) break;

    // tree: thread (row tr, segment tw)
    float y = 0.0f;
    if (tr < nrows) y = group_tree(part + tr * kRowPitch + tw * kGroupPitch);
    y = combine8(legacy_fix(y, p.legacy_tree));
    named_bar_sync(kBarC, kCT);  // the chain buffer is rewritten by the next item
    if (tw == 0 && tr < nrows) {
      const int r = r0 + tr;
      if (p.mode == 0) {
        J.out[r] = epilogue(y, p.relu2, p.out_scale);
      } else {
        p.contrib[(size_t)job * p.rows + r] = y;
        unsigned old_cnt;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old_cnt) : "l"(&p.row_count[r]) : "memory");
        if ((int)old_cnt == p.njobs - 1) {
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

constexpr int kCtasPerSm = 2;

template <int H>
int launch_h(const GemvBatch& b, const TmaCfg& c, int smem, cudaStream_t stream) {
  const int total = c.bpj * b.njobs;  // upper bound (inactive jobs drop out on the device)
  int grid = dev_info().sms * kCtasPerSm;
  if (grid > total) grid = total;
  if (set_smem(nvfp4_gemv_tma<H>, smem)) return kErrLaunch;
  return launch_ex(nvfp4_gemv_tma<H>, dim3(grid), dim3(kCT + 32), smem, stream, b.pdl != 0, b, c);
}

int launch_tma(const GemvBatch& b, cudaStream_t stream) {
  const DevInfo& di = dev_info();
  TmaCfg c{};
  c.n_u = b.cols / 32;
  c.n2 = c.n_u > 64 ? c.n_u - 64 : 0;
  c.teams = kCT / c.n_u;
  if (c.teams > 16) c.teams = 16;
  // Scale rows of a block start 16-byte aligned: blk * cols / 16 % 16 == 0.
  c.blk = (b.cols % 64 == 0) ? 4 : 8;
  const int cb = b.cols / 2, sb = b.cols / 16;
  const int budget = (di.smem_sm - kCtasPerSm * 1024) / kCtasPerSm;
  // Largest H (rows per segment) whose chain buffer, activation and two
  // stages fit two CTAs per SM, with kRt = teams * 2H <= 32 rows.
  int h = 0;
  for (int cand = 4; cand >= 1; --cand) {
    const int krt = c.teams * 2 * cand;
    if (krt > 32 || krt % c.blk != 0) continue;
    const int part_off = 576;  // after barriers, job tables and the active-job list
    const int xs_off = align_up(part_off + krt * kRowPitch * 4, 16);
    const int base = align_up(xs_off + c.n_u * 128, 128);
    const int stage = align_up(krt * cb + align_up(krt * sb, 16), 128);
    if (base + 2 * stage <= budget) {
      h = cand;
      c.part_off = part_off;
      c.xs_off = xs_off;
      c.stage_base = base;
      c.scale_off = krt * cb;
      c.stage_bytes = stage;
      c.kb = krt / c.blk;
      break;
    }
  }
  if (h == 0) return kErrShape;
  c.stages = (budget - c.stage_base) / c.stage_bytes;
  if (c.stages > 4) c.stages = 4;
  const int smem = c.stage_base + c.stages * c.stage_bytes;
  c.bpj = (b.rows + c.blk - 1) / c.blk;
  switch (h) {
    case 4: return launch_h<4>(b, c, smem, stream);
    case 3: return launch_h<3>(b, c, smem, stream);
    case 2: return launch_h<2>(b, c, smem, stream);
    default: return launch_h<1>(b, c, smem, stream);
  }
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
