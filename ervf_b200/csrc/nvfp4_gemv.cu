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
//    round units (cols > 2048) are spread evenly over all threads.  Codes are
//    decoded with the sm_100a e2m1x2 converter, block scales through a
//    per-job shared table of RN(e4m3 * g).  Chain
//    values go to shared memory and are reduced by the reference tree.
//
//  * nvfp4_gemv_sched<W> -- the reference's ERVF widths 4/8/16/32 as
//    schedules: W lanes per row, lane L owns chains L + W*i.  Same chains,
//    same tree, any alignment >= 4 bytes; also the fallback where the TMA
//    schedule's preconditions (cols % 32 == 0, cols <= 4096, 16-B aligned
//    bases) do not hold.
#include <stdlib.h>

#include "common.cuh"
#include "kernels.h"
#include "tma_core.cuh"

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
// e2m1x2 converter and block scales read from the job's shared table of
// RN(e4m3 * g) (the reference's LUT product), w = RN(e2m1 * s) (FMUL) and acc = fmaf(w, x,
// acc) (FFMA) in the reference's order.  Chain values go to the item's chain
// buffer; after a consumer barrier thread (row tr, segment tw) reduces chains
// 32tw..32tw+31 of its row with the reference's shuffle tree (offsets 16..1)
// and eight lanes combine ((S0+S4)+(S2+S6))+((S1+S5)+(S3+S7)).
//
// mode 1 (routed sum): the tree lane of a row writes the job's row value y_s
// to contrib[s][row].  Rows are counted in groups of 32: after the item's
// values are stored, the producer warp (idle once its copies are issued)
// adds the item's row count to each group it touches with one acq_rel atomic
// per group; the atomic that completes a group (njobs x its rows) makes its
// warp add the group's 32 rows up in ROUTE order, acc = fmaf(y_s, w_s, acc)
// for s = 0..njobs-1 from base or 0, and write resid + acc -- the same sum as
// one thread walking the slots in order, with the rows spread over every SM
// and no consumer thread ever waiting on an atomic.
//
// L2 prefetch: a launch may name the expert records the NEXT launch will read
// (codes and scales of pf_n experts); each CTA issues cp.async.bulk.prefetch.L2
// (this GPU's memory, no multicast) for a slice of them once its own ring is
// filled, so that their HBM stream runs under this launch's compute.  A hint:
// results do not depend on it.
//
// mode 1 with a cluster (2 <= njobs <= 8): the grid is cut into thread-block
// clusters of njobs CTAs; cluster i owns one range of rows, and its CTA of
// rank s computes job s on those rows, keeping each row value in shared
// memory.  After a cluster barrier every CTA sums a slice of the range in
// route order, reading the njobs values of a row from the cluster's shared
// memories (distributed shared memory), then a second barrier keeps the
// memories alive until all reads are done.  Same arithmetic, no atomics and
// no contrib round trip through L2.

struct TmaCfg {
  int stages;       // ring depth
  int stage_bytes;  // bytes per stage (128-aligned)
  int scale_off;    // scale rows inside a stage
  int part_off;     // chain buffer [kRt][kRowPitch] floats
  int xs_off;       // activation [n_u][8] float4, swizzled
  int lut_off;      // block-scale table of the current job: 256 floats RN(e4m3 * g)
  int stage_base;
  int n_u;          // code units per row (cols / 32)
  int n2;           // chain groups with a second unit (n_u - 64, or 0)
  int teams;        // T
  int blk;          // rows per row block (4 or 8: 16-byte aligned scale rows)
  int kb;           // row blocks per item (kRt / blk)
  int bpj;          // row blocks per job
  int cluster;      // mode 1: CTAs per cluster (= njobs), 0 = group-counter route sum
  int ysm_off;      // cluster mode: row values of this CTA's range, kYsmRows floats
};

// Shared-memory header of nvfp4_gemv_tma (the chain buffer starts at 576):
//   0   full[8]    mbarriers, a stage holds data
//   64  empty[8]   mbarriers, a stage was read by the consumers
//   128 jc[16]     code base of each job
//   256 js[16]     scale base of each job
//   384 jg[16]     global scale of each job
//   448 jlist[16]  active jobs (expert-parallel filter)
//   512 nact       number of active jobs
//   516 done       items whose row values are stored (mode-1 publishing)
constexpr int kPartOff = 576;

constexpr int kYsmRows = 512;  // rows per cluster range (cluster mode)
#ifndef ERVF_BULK_PIECE
#define ERVF_BULK_PIECE 4096
#endif
constexpr uint32_t kBulkPiece = ERVF_BULK_PIECE;  // bytes per bulk copy of an item's code rows

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// fp32 at the same shared-memory offset in the CTA of cluster rank `rank`.
__device__ __forceinline__ float ld_dsmem(const float* p, uint32_t rank) {
  uint32_t ra;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(p)), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
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


// This CTA's slice of the L2 prefetch: the records are cut into 32 KB chunks,
// numbered across records, and CTA b issues chunks b, b + grid, ...  Ids are
// clamped into [0, pf_experts) so that a stale id cannot leave the bank.
__device__ __forceinline__ void l2_prefetch_slice(const GemvBatch& p) {
  constexpr uint32_t kChunk = 32768;
  const long long G = gridDim.x, b = blockIdx.x;
  long long idx = 0;
  for (int j = 0; j < p.pf_n; ++j) {
    int id = p.pf_ids[j];
    id = id < 0 ? 0 : (id >= p.pf_experts ? p.pf_experts - 1 : id);
    for (int r = 0; r < 2; ++r) {
      const uint8_t* base = r ? p.pf_scales + (size_t)id * p.pf_scale_stride
                              : p.pf_codes + (size_t)id * p.pf_code_stride;
      const size_t bytes = r ? p.pf_scale_bytes : p.pf_code_bytes;
      const long long n = (long long)((bytes + kChunk - 1) / kChunk);
      for (long long c = ((b - idx) % G + G) % G; c < n; c += G) {
        const size_t off = (size_t)c * kChunk;
        const uint32_t sz = (uint32_t)(bytes - off < kChunk ? bytes - off : kChunk);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off), "r"(sz) : "memory");
      }
      idx += n;
    }
  }
}

// Mode-1 publishing, run by the whole producer warp over the CTA's items in
// order: wait (bounded) until the consumers have stored item i's row values,
// add its rows to the 32-row groups it touches, and sum every group whose
// count this completed.  Returns false when the wait ran out.
__device__ __forceinline__ bool publish_items(const GemvBatch& p, const TmaCfg& c, ItemSeq q,
                                              const int* jlist, const int* done, int lane) {
  int it = 0, job, r0, nrows;
  while (next_item(q, c, jlist, p.rows, job, r0, nrows)) {
    bool ok = true;
    if (lane == 0) {
      const long long t0 = clock64();
      while (ld_acquire_cta(done) <= it) {
        if (clock64() - t0 > 4000000000LL) {
          atomicExch(&g_device_error, kErrTimeout);
          ok = false;
          break;
        }
        nanosleep_ns(32);
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) return false;
    ++it;
    const int g0 = r0 >> 5, g1 = (r0 + nrows - 1) >> 5;
    int last = -1;
    if (lane <= g1 - g0) {
      const int g = g0 + lane;
      const int lo = max(r0, g << 5), hi = min(r0 + nrows, (g << 5) + 32);
      const int target = p.njobs * (min(p.rows, (g << 5) + 32) - (g << 5));
      const unsigned old = atom_add_acq_rel_gpu(p.grp_count + g, (unsigned)(hi - lo));
      if ((int)old + (hi - lo) == target) last = g;
    }
    unsigned m = __ballot_sync(0xffffffffu, last >= 0);
    while (m) {
      const int src = __ffs(m) - 1;
      m &= m - 1;
      const int g = __shfl_sync(0xffffffffu, last, src);
      const int r = (g << 5) + lane;
      if (r < p.rows) {
        float acc = p.base ? p.base[r] : 0.0f;
        for (int s2 = 0; s2 < p.njobs; ++s2)
          acc = fmaf(__ldcg(&p.contrib[(size_t)s2 * p.rows + r]), p.route_w[s2], acc);
        p.rs_out[r] = p.resid ? p.resid[r] + acc : acc;
      }
      if (lane == src) p.grp_count[g] = 0u;  // every add of this group is in
    }
  }
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
  int* done = nact + 1;
  float* part = reinterpret_cast<float*>(smem + c.part_off);
  float4* xs = reinterpret_cast<float4*>(smem + c.xs_off);
  float* lut = reinterpret_cast<float*>(smem + c.lut_off);  // [256] of the current job
  uint8_t* stages = smem + c.stage_base;
  const bool publish = p.mode == 1 && !c.cluster;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    *done = 0;
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
  int row_lo = 0, row_hi = 0;  // cluster mode: the cluster's rows
  if (c.cluster) {
    const int k = c.cluster, nc = gridDim.x / k, ci = blockIdx.x / k, rank = blockIdx.x % k;
    const int per = c.bpj / nc, rem = c.bpj % nc;
    const int b0 = ci * per + min(ci, rem), b1 = b0 + per + (ci < rem ? 1 : 0);
    q.blk = rank * c.bpj + b0;
    q.blk_end = rank * c.bpj + b1;
    row_lo = b0 * c.blk;
    row_hi = min(b1 * c.blk, p.rows);
  } else {
    cta_blocks(*nact * c.bpj, q);
  }
  float* ysm = reinterpret_cast<float*>(smem + c.ysm_off);

  // ------------------------------------------------------------ producer
  if (tid >= kCT) {
    const int lane = tid - kCT;
    if (lane == 0) {
      ItemSeq qp = q;
      int it = 0, job, r0, nrows;
      bool prefetched = p.pf_n == 0;
      while (next_item(qp, c, jlist, p.rows, job, r0, nrows)) {
        if (it == S && !prefetched) {  // the ring is full: queue the next launch's records
          l2_prefetch_slice(p);
          prefetched = true;
        }
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
        // The code rows go as several bulk copies in flight at once: one
        // copy streams at ~10 GB/s on B200 however large it is, so a whole
        // item in one copy leaves HBM idle (measured: ~4 us for 36 KB)
        const uint8_t* csrc = jc[job] + (size_t)r0 * cb;
        for (uint32_t off = 0; off < code_bytes; off += kBulkPiece) {
          const uint32_t n = code_bytes - off < kBulkPiece ? code_bytes - off : kBulkPiece;
          bulk_g2s(dst + off, csrc + off, n, &full[st]);
        }
        if (s16) bulk_g2s(dst + c.scale_off, ssrc, s16, &full[st]);
      }
      if (!prefetched) l2_prefetch_slice(p);
      // Leave no bulk copy in flight: wait (bounded) for the last stages.
      for (int k = (it > S ? it - S : 0); k < it; ++k) mbar_wait(&full[k % S], (k / S) & 1);
    }
    __syncwarp();
    grid_dep_wait();  // base / residual / route weights come from the predecessor
    grid_dep_launch();
    if (publish) publish_items(p, c, q, jlist, done, lane);
    if (c.cluster) {  // every thread of the cluster takes both barriers
      cluster_sync_all();
      cluster_sync_all();
    }
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
  int cur_job = -1;
  // segment activation; a thread whose two segments share one unit keeps it
  // in registers until the job's activation changes
  float2 x[16];
  bool x_stale = true;
  named_bar_sync(kBarC, kCT);

  int it = 0, job, r0, nrows;
  while (next_item(q, c, jlist, p.rows, job, r0, nrows)) {
    const int st = it % S;
    const uint32_t ph = (it / S) & 1;
    ++it;
    const GemvJob& J = p.job[job];
    if (J.x != cur_x || job != cur_job) {  // the previous item ended with a consumer barrier
      if (J.x != cur_x) {
        for (int f = tid; f < nu * 8; f += kCT) {
          const int t = f >> 3, k = f & 7;
          xs[t * 8 + (k ^ (t & 7))] = x_slot(J.x, t, k);
        }
        cur_x = J.x;
        x_stale = true;
      }
      if (job != cur_job) {
        lut[tid] = e4m3_lut_value((uint32_t)tid) * jg[job];
        cur_job = job;
      }
      named_bar_sync(kBarC, kCT);
    }
    const bool to = !mbar_wait(&full[st], ph);
    const uint32_t stage_off = (uint32_t)(c.stage_base + st * c.stage_bytes);

    if (active) {
      if (nrows == krt) {
        segments<H, true>(smem, stage_off, c.scale_off, cb, sb, team, T, par1, par2, cont, u1, u2, grp,
                          nrows, lut, xs, x, x_stale, part);
      } else {
        segments<H, false>(smem, stage_off, c.scale_off, cb, sb, team, T, par1, par2, cont, u1, u2,
                           grp, nrows, lut, xs, x, x_stale, part);
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
    // SwiGLU: rows 2i (gate) and 2i+1 (up) sit 8 lanes apart in one warp
    const float y_up = __shfl_down_sync(0xffffffffu, y, 8);
    if (publish && tw == 0 && tr < nrows) p.contrib[(size_t)job * p.rows + r0 + tr] = y;
    named_bar_sync(kBarC, kCT);  // the chain buffer is rewritten by the next item
    if (publish) {
      if (tid == 0) st_release_cta(done, it);  // the item's row values are stored
    } else if (p.swiglu) {
      if (tw == 0 && (tr & 1) == 0 && tr + 1 < nrows)
        J.out[(r0 + tr) >> 1] = silu(y) * y_up;
    } else if (tw == 0 && tr < nrows) {
      const int r = r0 + tr;
      if (p.mode == 0) {
        J.out[r] = epilogue(y, p.relu2, p.out_scale);
      } else {
        ysm[r - row_lo] = y;  // cluster mode
      }
    }
  }
  if (c.cluster) {
    // route-order sum of this CTA's slice of the cluster's rows from the
    // njobs CTAs' row values (rank s holds job s)
    cluster_sync_all();
    const int k = c.cluster, rank = blockIdx.x % k, n = row_hi - row_lo;
    const int lo = n * rank / k, hi = n * (rank + 1) / k;
    for (int i = lo + tid; i < hi; i += kCT) {
      const int r = row_lo + i;
      float acc = p.base ? p.base[r] : 0.0f;
      for (int s2 = 0; s2 < k; ++s2) acc = fmaf(ld_dsmem(ysm + i, (uint32_t)s2), p.route_w[s2], acc);
      p.rs_out[r] = p.resid ? p.resid[r] + acc : acc;
    }
    cluster_sync_all();  // peers have read this CTA's row values
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

// Dynamic shared memory of a kernel, with the shared-memory carve-out at its
// maximum: the driver otherwise may pick the smallest carve-out that fits
// one CTA, and two ~113 KB CTAs of the TMA schedule then no longer share an SM.
template <typename K>
int set_smem(K kernel, int bytes) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return kErrLaunch;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return kErrLaunch;
  return kOk;
}

// Smallest row block whose bulk copies start 16-byte aligned: code rows need
// r0 * cols / 2 % 16 == 0 and scale rows r0 * cols / 16 % 16 == 0, i.e.
// r0 * cols % 256 == 0 (cols % 32 == 0): blk = 256 / gcd(cols, 256).
int row_block(int cols) {
  int g = 256;
  while (cols % g != 0) g >>= 1;
  return 256 / g;
}

bool tma_ok(const GemvBatch& b) {
  if (b.cols % 32 != 0 || b.cols > 4096) return false;
  if (b.mode == 1 && (!b.contrib || !b.grp_count)) return false;
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

int max_h() {
  static const int h = [] {
    const char* e = getenv("ERVF_TMA_MAX_H");
    const int v = e ? atoi(e) : 4;
    return v < 1 ? 1 : (v > 4 ? 4 : v);
  }();
  return h;
}

// Cluster launch of the mode-1 (routed-sum) kernel: clusters of njobs CTAs,
// as many as fit the SMs at two CTAs per SM; 0 when the cluster form does not
// apply (then the atomic route sum runs).
template <int H>
int cluster_grid(const TmaCfg& c, int k, int smem) {
  int nc = dev_info().sms * kCtasPerSm / k;
  if (nc > c.bpj) nc = c.bpj;
  if (nc < 1) return 0;
  if ((c.bpj + nc - 1) / nc * c.blk > kYsmRows) return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(nc * k);
  cfg.blockDim = dim3(kCT + 32);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = k;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int active = 0;
  if (cudaOccupancyMaxActiveClusters(&active, nvfp4_gemv_tma<H>, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  if (active < 1) return 0;
  if (nc > active) nc = active;
  return nc * k;
}

template <int H>
int launch_h(const GemvBatch& b, TmaCfg c, int smem, cudaStream_t stream) {
  const int total = c.bpj * b.njobs;  // upper bound (inactive jobs drop out on the device)
  int grid = dev_info().sms * kCtasPerSm;
  if (grid > total) grid = total;
  if (set_smem(nvfp4_gemv_tma<H>, smem)) return kErrLaunch;
  if (c.cluster) {
    const int cg = cluster_grid<H>(c, c.cluster, smem);
    if (cg > 0) {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(cg);
      cfg.blockDim = dim3(kCT + 32);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = c.cluster;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = b.pdl ? 2 : 1;
      return cudaLaunchKernelEx(&cfg, nvfp4_gemv_tma<H>, b, c) == cudaSuccess ? kOk : kErrLaunch;
    }
    c.cluster = 0;  // atomic route sum
  }
  return launch_ex(nvfp4_gemv_tma<H>, dim3(grid), dim3(kCT + 32), smem, stream, b.pdl != 0, b, c);
}

int launch_tma(const GemvBatch& b, cudaStream_t stream) {
  const DevInfo& di = dev_info();
  TmaCfg c{};
  c.n_u = b.cols / 32;
  c.n2 = c.n_u > 64 ? c.n_u - 64 : 0;
  c.teams = kCT / c.n_u;
  if (c.teams > 16) c.teams = 16;
  c.blk = row_block(b.cols);
  if (b.swiglu && c.blk < 2) c.blk = 2;  // gate / up row pairs stay in one item
  const int cb = b.cols / 2, sb = b.cols / 16;
  const int budget = (di.smem_sm - kCtasPerSm * 1024) / kCtasPerSm;
  // Routed sum through a cluster of njobs CTAs (every job active: no expert
  // filter in mode 1) for launches that are not PDL-chained: alone it is
  // faster than the atomic route sum (13.1 vs 14.6 us for six 2688 x 1856
  // experts on B200), but a cluster can only start once njobs CTA slots are
  // free in one GPC, which cancels the overlap with the previous kernel that
  // PDL buys (29.0 vs 25.0 us per decode layer).
  const bool want_cluster = b.mode == 1 && !b.pdl && b.njobs >= 2 && b.njobs <= 8 && b.ep_ranks <= 1;
  // Largest H (rows per segment) whose chain buffer, activation and two
  // stages fit two CTAs per SM, with kRt = teams * 2H <= 32 rows (capped by
  // ERVF_TMA_MAX_H, a tuning knob read once per process; same results).
  int h = 0;
  for (int cand = max_h(); cand >= 1; --cand) {
    const int krt = c.teams * 2 * cand;
    if (krt > 32 || krt % c.blk != 0) continue;
    const int part_off = kPartOff;  // after barriers, job tables and the active-job list
    const int xs_off = align_up(part_off + krt * kRowPitch * 4, 16);
    const int lut_off = xs_off + c.n_u * 128;
    const int ysm_off = lut_off + 1024;
    const int base = align_up(ysm_off + (want_cluster ? kYsmRows * 4 : 0), 128);
    const int stage = align_up(krt * cb + align_up(krt * sb, 16), 128);
    if (base + 2 * stage <= budget) {
      h = cand;
      c.part_off = part_off;
      c.xs_off = xs_off;
      c.lut_off = lut_off;
      c.ysm_off = ysm_off;
      c.cluster = want_cluster ? b.njobs : 0;
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

bool nvfp4_tma_ok(const GemvBatch& b) { return tma_ok(b); }

int device_sm_count() { return dev_info().sms; }
int device_smem_optin() { return dev_info().smem_optin; }

int read_gemv_device_error(bool clear) { return read_unit_error(clear); }

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
