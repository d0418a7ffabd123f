// moe_token.cu -- one decode token through every routed MoE layer in ONE
// launch (single GPU), bit-exact to the per-layer path (ervf_moe_layer: the
// reference's per-layer up GEMV + relu^2, masked down GEMV and route-order
// sum, kennydd001/ervf runtime.py:705-746 over fused_nvfp4.py:295-406).
//
// Work is a single ordered list of items, claimed one at a time from a global
// counter by each CTA's producer warp:
//   item 0                      PREP: x -> the layer-0 activation buffers
//   per layer l, in order:      UP   items: slot-major, krt_u rows of up_e(x_l)
//                               DOWN items: slot-major, krt_d rows of down_e(act)
// An UP item needs x_l complete (every row group of layer l-1's route sum
// written); a DOWN item needs its slot's act complete (all UP items of that
// slot).  Dependencies point only at items with a SMALLER index, and every
// CTA runs its claimed items in claim order, so the unfinished item with the
// smallest index always has its inputs ready and its CTA running it: the
// token completes whatever the number of co-resident CTAs (no grid-wide
// residency assumption).  Every wait is bounded and ends with kErrTimeout.
//
// CTA = 8 consumer warps (the exact ERVF chain schedule of tma_core.cuh) +
// one producer warp + one publisher warp, two CTAs per SM.
//   producer  claims an item when a stage frees, writes the item header and
//             the item's block-scale table RN(e4m3 * g) into the stage, bulk
//             copies the weight rows (cp.async.bulk, no multicast) at once,
//             then waits for the item's activation and bulk copies it (kept
//             in global memory in the swizzled unit layout the consumers
//             read, so no permutation pass) -- weights stream while the
//             activation is still being produced elsewhere.
//   consumers reduce the item's rows (chains -> shared chain buffer -> tree)
//             and hand the row values to the publisher through shared memory.
//   publisher stores them -- UP rows as relu^2 into the slot's swizzled act
//             buffer, DOWN rows into contrib[slot][row], one row per lane --
//             and after a warp barrier lane 0's release (cumulative over
//             the lanes' stores) makes the item visible: UP adds its rows to
//             the slot's act counter (release); DOWN adds its rows to the 32-row groups it
//             touches (acq_rel); the add that completes a group makes the
//             warp sum the group in ROUTE order, acc = fmaf(y_s, w_s, acc)
//             from 0, x_{l+1} = x_l + acc (the per-layer path's arithmetic),
//             writes x_{l+1} (linear and swizzled, or `out` after the last
//             layer) and adds the group's rows to the x counter of layer l+1.
// With the router on the device (ROUTE instantiation) each layer starts with
// router items: one consumer warp per expert row computes the reference's
// gemv_f32 row, the item that completes the layer runs route_topk_f32 and
// releases the layer's ids; expert items of that layer wait for them.
// With expert parallelism (EP instantiation, ervf_moe_token_ep) each rank's
// list holds only the UP / DOWN items of the slots whose expert it owns, plus
// one SUM item per down row block per layer: DOWN rows go to every rank's
// contrib[l][slot] as raw peer stores, and each rank's SUM items wait for the
// words themselves (kUnwritten), add them in route order and write x_{l+1};
// an entry handshake per token orders one token's writes after every rank's
// previous token (see TokArgs and the PREP publisher).
// The last CTA to leave zeroes every counter, so the scratch is ready for
// the next token (also after a timeout, once all CTAs have left).
#include <stdlib.h>

#include "common.cuh"
#include "kernels.h"
#include "route.cuh"
#include "tma_core.cuh"

namespace ervf {

namespace {

constexpr int kTokWarps = kCW + 2;  // consumers, producer, publisher
constexpr int kTokThreads = kTokWarps * 32;
constexpr int kProd = kCT;       // first thread of the producer warp
constexpr int kPub = kCT + 32;   // first thread of the publisher warp
constexpr int kTokMaxStages = 4;  // ring depth is chosen per launch (2..4)
constexpr int kPubRing = 16;     // item descriptors between consumers and publisher
constexpr int kLutOff = 64;      // stage: header [0, 64), block-scale table [64, 1088)
constexpr int kXOff = kLutOff + 1024;
constexpr int kPubFullOff = 384;  // [kPubRing] mbarriers: ring slot filled (pubq at 128 .. 384)
constexpr int kYRingOff = 512;    // [kPubRing][32] row values handed to the publisher
constexpr int kTabOff = kYRingOff + kPubRing * 32 * 4;  // per-token routing table, then the chain buffer
static_assert(128 + 16 * kPubRing <= kPubFullOff && kPubFullOff + 8 * kPubRing <= kYRingOff,
              "publisher ring layout");
constexpr unsigned kFull = 0xffffffffu;

enum : int { kItemPrep = 0, kItemUp = 1, kItemDown = 2, kItemEnd = 3, kItemRoute = 4, kItemSum = 5 };
constexpr int kTokMaxRanks = 8;  // expert-parallel ranks of one token launch
constexpr int kRouteRows = kCW;  // router rows per item: one per consumer warp
constexpr int kTokMaxRouteExperts = 256;  // experts a layer's router items can route

// One projection: up (rows = inter, cols = hidden) or down (rows = hidden,
// cols = inter).
struct TokPhase {
  int rows, cols, n_u, n2, teams, krt, cb, sb, scale_off, n_items;
};

struct TokArgs {
  // [5][L]: up codes, up scales, dn codes, dn scales, globals; with the
  // router two more rows: router weights f32 [E][hidden], router bias f32 [E]
  // (0 = none)
  const unsigned long long* layer_ptrs;
  size_t up_cs, up_ss, dn_cs, dn_ss;     // per-expert record strides
  const int* ids;                        // [L][K] (written by the router items when route)
  const float* route_w;                  // [L][K]
  int route;                             // router items compute ids / route_w per layer
  float scaling;
  int bad_pick;
  int n_route;                           // router items per layer
  float* rlog;                           // [L][E] router logits (route)
  const float* x_in;                     // [hidden]
  float* out;                            // [hidden]
  int L, K, E, hidden, inter;
  int B;                                 // down row blocks per slot (the block counters' stride)
  TokPhase up, dn;
  int per_layer, total;
  int stages, stage_bytes, codes_off, stage_base, part_off;
  int prefetch;  // queue the next claimed item's weight rows into L2
  unsigned* ctr;                         // claim, exited, xrows[L], actrows[L][K], grp[L][G]
  int n_ctr;
  float* xlin;     // [L][hidden]  x_l (x_0 = the input)
  float* xsw;      // [L][hidden]  x_l in the swizzled unit layout
  float* actsw;    // [2][K][inter] relu^2(up) per slot, swizzled
  float* contrib;  // [2][K][hidden] down rows per slot ([L][K][hidden] with EP)
  // Expert parallelism (EP instantiation): this rank owns the experts e with
  // e % ep_n == ep_rank.  peer[q] is rank q's scratch as mapped on this GPU
  // (peer[ep_rank] = this rank's own); every rank's scratch has the same
  // layout, so a peer's contrib and entry flags sit at this rank's offsets.
  int ep_n, ep_rank;
  unsigned long long peer[kTokMaxRanks];
  size_t contrib_off;              // byte offset of contrib in every rank's scratch
  size_t hello_off;                // byte offset of the token-entry flags [kTokMaxRanks] (never reset)
  unsigned* hello;                 // this rank's entry flags; its epoch word 32 words later
  unsigned long long timeout_ns;   // limit of the waits on other ranks
};

// Counter words.  The claim counter (hit by every claim), the exit counter
// and every counter that producers poll sit on their own 128-byte line, so
// that polling does not slow the atomics on a neighbour.
constexpr int kCtrLine = 32;
__device__ __forceinline__ unsigned* ctr_claim(const TokArgs& a) { return a.ctr; }
__device__ __forceinline__ unsigned* ctr_exited(const TokArgs& a) { return a.ctr + kCtrLine; }
// EP: set by the first wait on another rank that runs out (same line)
__device__ __forceinline__ unsigned* ctr_abort(const TokArgs& a) { return a.ctr + kCtrLine + 1; }
__device__ __forceinline__ unsigned* ctr_xrows(const TokArgs& a, int l) {
  return a.ctr + kCtrLine * (2 + l);
}
__device__ __forceinline__ unsigned* ctr_act(const TokArgs& a, int l, int s) {
  return a.ctr + kCtrLine * (2 + a.L + l * a.K + s);
}
__device__ __forceinline__ unsigned* ctr_route_ready(const TokArgs& a, int l) {
  return a.ctr + kCtrLine * (2 + a.L + a.L * a.K + l);
}
// router rows done per layer, then per (layer, down row block) the slots
// 0..K-2 whose rows of the block are stored: atomics and one poller each
__host__ __device__ __forceinline__ size_t token_rows_base(int L, int K) {
  return (size_t)kCtrLine * (2 + 2 * L + (size_t)L * K);
}
__host__ __device__ __forceinline__ size_t token_blk_base(int L, int K) {
  return token_rows_base(L, K) + (size_t)(L + kCtrLine - 1) / kCtrLine * kCtrLine;
}
__device__ __forceinline__ unsigned* ctr_route_rows(const TokArgs& a, int l) {
  return a.ctr + token_rows_base(a.L, a.K) + l;
}
__device__ __forceinline__ unsigned* ctr_blk(const TokArgs& a, int l, int b) {
  return a.ctr + token_blk_base(a.L, a.K) + (size_t)l * a.B + b;
}

// Counter words for B down row blocks per slot (B <= hidden / 2: a down item
// has at least two rows).
__host__ __device__ __forceinline__ size_t token_ctr_words(int L, int K, int B) {
  return token_blk_base(L, K) + (size_t)L * B;
}

// Shared routing table of the token, loaded once per CTA: record bases of
// every layer (up codes, up scales, down codes, down scales), the clamped
// expert id of every (layer, slot) and its (down, up) global scales -- the
// producer then forms an item's addresses without a global-memory round trip.
__host__ __device__ __forceinline__ int token_tab_bytes(int L, int K) { return 36 * L + 12 * L * K; }
// With EP the table is followed by this rank's slot lists: owned slots
// [L][K], item offsets of the layers [L + 1], owned-slot counts [L], total.
__host__ __device__ __forceinline__ int token_tab_bytes_ep(int L, int K) {
  return token_tab_bytes(L, K) + 4 * (L * K + 2 * L + 2);
}

// Float index of column j in the swizzled unit layout that x_slot / the
// consumers use: unit t = j / 32 holds 8 float4 slots, slot k =
// (x[c], x[c+8], x[c+1], x[c+9]) with c = 32t + 16(k>>2) + 2(k&3), stored at
// float4 t*8 + (k ^ (t & 7)).
__device__ __forceinline__ int sw_index(int j) {
  const int t = j >> 5, o = j & 31;
  const int k = 4 * (o >> 4) + ((o >> 1) & 3);
  return ((t << 3) + (k ^ (t & 7))) * 4 + 2 * (o & 1) + ((o >> 3) & 1);
}

__device__ __forceinline__ void decode_item(const TokArgs& a, int idx, int& kind, int& l, int& slot,
                                            int& r0, int& nrows) {
  if (idx == 0) {
    kind = kItemPrep;
    l = slot = r0 = nrows = 0;
    return;
  }
  const int i = idx - 1;
  l = i / a.per_layer;
  int j = i - l * a.per_layer;
  if (j < a.n_route) {  // router rows kRouteRows * j .. (before the layer's up items)
    kind = kItemRoute;
    slot = 0;
    r0 = kRouteRows * j;
    nrows = min(kRouteRows, a.E - r0);
    return;
  }
  j -= a.n_route;
  const int nu = a.K * a.up.n_items;
  const TokPhase* ph;
  if (j < nu) {
    kind = kItemUp;
    ph = &a.up;
  } else {
    kind = kItemDown;
    j -= nu;
    ph = &a.dn;
  }
  slot = j / ph->n_items;
  r0 = (j - slot * ph->n_items) * ph->krt;
  nrows = min(ph->krt, ph->rows - r0);
}

// EP: this rank's items.  Per layer l (item offset loff[l]): the UP items
// of the slots it owns (own[l][0 .. nown[l]), in route order), their DOWN
// items, then one SUM item per down row block (the route-order sum of that
// block from every rank's slot rows).  `hint` is the layer of the caller's
// previous decode (claims only grow).
__device__ __forceinline__ void decode_item_ep(const TokArgs& a, const int* own, const int* loff,
                                               const int* nown, int idx, int& hint, int& kind,
                                               int& l, int& slot, int& r0, int& nrows) {
  if (idx == 0) {
    kind = kItemPrep;
    l = slot = r0 = nrows = 0;
    return;
  }
  const int i = idx - 1;
  int ll = hint;
  while (ll > 0 && i < loff[ll]) --ll;
  while (ll + 1 < a.L && i >= loff[ll + 1]) ++ll;
  hint = ll;
  l = ll;
  int j = i - loff[ll];
  const int nu = nown[ll] * a.up.n_items, nd = nown[ll] * a.dn.n_items;
  if (j < nu) {
    kind = kItemUp;
    slot = own[ll * a.K + j / a.up.n_items];
    r0 = (j % a.up.n_items) * a.up.krt;
    nrows = min(a.up.krt, a.up.rows - r0);
  } else if (j < nu + nd) {
    j -= nu;
    kind = kItemDown;
    slot = own[ll * a.K + j / a.dn.n_items];
    r0 = (j % a.dn.n_items) * a.dn.krt;
    nrows = min(a.dn.krt, a.dn.rows - r0);
  } else {
    kind = kItemSum;
    slot = 0;
    r0 = (j - nu - nd) * a.dn.krt;
    nrows = min(a.dn.krt, a.hidden - r0);
  }
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Relaxed system-scope accesses of the slot rows other GPUs write.
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// EP: a contrib word not yet written for this token holds this pattern (a
// NaN that no arithmetic result has: GPU arithmetic returns the canonical NaN
// 0x7FFFFFFF); a row value with these bits is stored as 0x7FFFFFFF, which
// gives the same (canonical NaN) route sum.
constexpr unsigned kUnwritten = 0xFFFFFFFFu;

__device__ __forceinline__ unsigned long long globaltimer_tok() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait until *p >= target for a counter that other GPUs add to
// (acquire at system scope): false after timeout_ns (or 2^28 polls), and at
// once when another wait of the launch has run out (*abort, zeroed with the
// counters when the launch ends), so that a rank that never arrives costs
// one timeout, not one per wait.
__device__ __forceinline__ bool wait_count_sys(const unsigned* p, unsigned target,
                                               unsigned long long timeout_ns, unsigned* abort) {
  if (ld_acquire_sys(p) >= target) return true;
  const unsigned long long t0 = globaltimer_tok();
  for (unsigned it = 0;; ++it) {
    if (ld_acquire_sys(p) >= target) return true;
    if ((it & 15u) == 15u) {
      if (*reinterpret_cast<volatile unsigned*>(abort)) return false;
      if (it >= (1u << 28) || globaltimer_tok() - t0 > timeout_ns) {
        atomicExch(&g_device_error, kErrTimeout);
        atomicExch(abort, 1u);
        return false;
      }
    }
    nanosleep_ns(64);
  }
}

// Orders this thread's generic-proxy view of global memory with its
// async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// L2 prefetch of `bytes` (a multiple of 16, may be 0) at a 16-byte aligned
// global address; a hint, no data moves into this SM.
__device__ __forceinline__ void l2_prefetch(const void* p, uint32_t bytes) {
  if (bytes) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Bounded wait until *p >= target (acquire); false after ~2 s.
__device__ __forceinline__ bool wait_count(const unsigned* p, unsigned target) {
  if (ld_acquire_gpu(p) >= target) return true;
  const long long t0 = clock64();
  while (ld_acquire_gpu(p) < target) {
    if (clock64() - t0 > 4000000000LL) {
      atomicExch(&g_device_error, kErrTimeout);
      return false;
    }
    nanosleep_ns(128);
  }
  return true;
}

// Bounded wait until the shared counter *p > v (acquire at CTA scope).
__device__ __forceinline__ bool wait_smem_gt(const int* p, int v) {
  if (ld_acquire_cta(p) > v) return true;
  const long long t0 = clock64();
  while (ld_acquire_cta(p) <= v) {
    if (clock64() - t0 > 4000000000LL) {
      atomicExch(&g_device_error, kErrTimeout);
      return false;
    }
    nanosleep_ns(32);
  }
  return true;
}

// Router logit of one expert row (one warp; lane 0 holds it; x in shared
// memory).  Kept out of line so that the router's registers do not weigh on
// the expert paths.
__device__ __noinline__ float router_row(const float* gw, const float* x, int cols, int lane) {
  return f32_row<true>(gw, x, cols, lane);
}

// route_topk_f32 of one layer on the calling (full) warp.
__device__ __noinline__ void router_topk(const float* lg, const float* gb, int* io, float* wo, int n,
                                         int top_k, float scaling, int bad_pick) {
  if (n <= 128)
    route_topk_warp<4>(lg, gb, io, wo, n, top_k, scaling, bad_pick);
  else
    route_topk_warp<8>(lg, gb, io, wo, n, top_k, scaling, bad_pick);
}

// Per-thread place in the consumer schedule of one projection (see the TMA
// schedule in nvfp4_gemv.cu: teams of n_u threads, two segments per thread).
struct SegPlace {
  int team, par1, par2, u1, u2, grp;
  bool active, cont;
};

__device__ __forceinline__ SegPlace seg_place(const TokPhase& ph, int tid) {
  SegPlace s;
  const int nu = ph.n_u, n2 = ph.n2;
  s.team = tid / nu;
  const int m = tid - s.team * nu;
  s.active = s.team < ph.teams;
  s.cont = m < 2 * n2;
  s.grp = m < n2 ? m : m - n2;
  s.u1 = s.grp;
  s.u2 = s.cont ? s.grp + 64 : s.grp;
  s.par1 = (m >= n2 && m < 2 * n2) ? 1 : 0;
  s.par2 = s.cont ? s.par1 : 1;
  return s;
}

// ROUTE: the launch has router items (ervf_moe_token_router); the plain
// instantiation carries no router code at all.
// EP: expert-parallel rank of a token (given routes only; see TokArgs).
template <int H, bool ROUTE, bool EP>
__global__ void __launch_bounds__(kTokThreads, 2) moe_token_kernel(const __grid_constant__ TokArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_last;
  const int tid = threadIdx.x;
  const int S = a.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [kTokMaxStages]
  uint64_t* empty = full + kTokMaxStages;              // [kTokMaxStages]
  int* pub_done = reinterpret_cast<int*>(smem + 64);    // items published
  // consumers -> publisher: one mbarrier per ring slot, so that the idle
  // publisher waits suspended instead of taking issue slots from the
  // consumer warps
  uint64_t* pub_full = reinterpret_cast<uint64_t*>(smem + kPubFullOff);  // [kPubRing]
  int* pubq = reinterpret_cast<int*>(smem + 128);      // [kPubRing][4] kind, layer, slot, r0 | nrows << 16
  float* yring = reinterpret_cast<float*>(smem + kYRingOff);
  float* part = reinterpret_cast<float*>(smem + a.part_off);
  // routing table: 8-byte entries first, so that every entry is aligned
  unsigned long long* tab_base = reinterpret_cast<unsigned long long*>(smem + kTabOff);  // [4][L]
  float2* tab_g = reinterpret_cast<float2*>(smem + kTabOff + 32 * a.L);                 // [L][K]
  int* tab_id = reinterpret_cast<int*>(smem + kTabOff + 32 * a.L + 8 * a.L * a.K);       // [L][K]
  int* tab_ok = tab_id + a.L * a.K;  // [L]: the layer's (id, g) entries are filled
  // EP: this rank's slot lists (token_tab_bytes_ep)
  int* ep_own = tab_ok + a.L;           // [L][K]
  int* ep_loff = ep_own + a.L * a.K;    // [L + 1]
  int* ep_nown = ep_loff + a.L + 1;     // [L]
  int* ep_total = ep_nown + a.L;        // [1]
  uint8_t* stages = smem + a.stage_base;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kPubRing; ++i) mbar_init(&pub_full[i], 1);
    *pub_done = 0;
    fence_mbar_init();
  }
  grid_dep_wait();  // ids, route weights and x come from the predecessor
  for (int i = tid; i < 4 * a.L; i += kTokThreads) tab_base[i] = a.layer_ptrs[i];
  for (int i = tid; i < a.L; i += kTokThreads) tab_ok[i] = a.route ? 0 : 1;
  for (int i = tid; i < (a.route ? 0 : a.L * a.K); i += kTokThreads) {
    int e = a.ids[i];
    e = e < 0 ? 0 : (e >= a.E ? a.E - 1 : e);  // a stale id cannot leave the bank
    const float* gl = reinterpret_cast<const float*>(a.layer_ptrs[4 * a.L + i / a.K]);
    tab_id[i] = e;
    tab_g[i] = make_float2(gl[2 * e], gl[2 * e + 1]);
  }
  if (EP) {
    __syncthreads();
    if (tid == 0) {
      int off = 0;
      for (int l = 0; l < a.L; ++l) {
        int n = 0;
        for (int s2 = 0; s2 < a.K; ++s2)
          if (tab_id[l * a.K + s2] % a.ep_n == a.ep_rank) ep_own[l * a.K + n++] = s2;
        ep_nown[l] = n;
        ep_loff[l] = off;
        off += n * (a.up.n_items + a.dn.n_items) + a.B;
      }
      ep_loff[a.L] = off;
      *ep_total = 1 + off;
    }
  }
  __syncthreads();

  if (tid >= kProd && tid < kPub) {
    // ------------------------------------------------------------ producer
    const int lane = tid - kProd;
    int it = 0;
    bool ok = true;
    // the next item is claimed while the current one streams, so the claim's
    // round trip is off the path from a free stage to its copies
    int next = 0;
    if (lane == 0) next = (int)atomicAdd(ctr_claim(a), 1u);
    const int total = EP ? *ep_total : a.total;
    int hint = 0;  // EP: layer of the last decode
    for (;;) {
      if (EP) {
        // a SUM item takes no stage: the producer warp runs it here.  Once
        // every rank's slot rows of the block are in (count K, released by
        // the owners' publishers at system scope), the route-order sum of
        // the block: acc = fmaf(y_s, w_s, acc) over s = 0..K-1 from 0 and
        // x_{l+1} = x_l + acc, the arithmetic of the one-GPU path.
        const int idx0 = __shfl_sync(kFull, next, 0);
        if (idx0 < total) {
          int kind0, l0, s0, q0, n0;
          decode_item_ep(a, ep_own, ep_loff, ep_nown, idx0, hint, kind0, l0, s0, q0, n0);
          if (kind0 == kItemSum) {
            if (lane == 0) {
              next = (int)atomicAdd(ctr_claim(a), 1u);
              // (a wait that runs out records kErrTimeout; the sum goes on)
              // x_l of the block's rows is this rank's own (its SUM items of
              // layer l - 1): with no slot of layer l here, nothing else
              // orders them before this sum
              wait_count_sys(ctr_xrows(a, l0), (unsigned)a.hidden, a.timeout_ns, ctr_abort(a));
            }
            __syncwarp();
            const int r = q0 + lane;
            if (lane < n0) {
              // every slot's word of this row, written by its owner (peer
              // stores, no fence): wait until none is unwritten, sum in
              // route order, then mark the words unwritten for the next
              // token (peers write them again only after every rank has
              // entered that token)
              unsigned* cw = reinterpret_cast<unsigned*>(a.contrib) + (size_t)l0 * a.K * a.hidden + r;
              const unsigned long long t0 = globaltimer_tok();
              unsigned polls = 0;
              for (int s2 = 0; s2 < a.K;) {
                if (ld_relaxed_sys(cw + (size_t)s2 * a.hidden) != kUnwritten) {
                  ++s2;
                  continue;
                }
                if ((++polls & 15u) == 0u) {
                  if (*reinterpret_cast<volatile unsigned*>(ctr_abort(a))) break;
                  if (polls >= (1u << 28) || globaltimer_tok() - t0 > a.timeout_ns) {
                    atomicExch(&g_device_error, kErrTimeout);
                    atomicExch(ctr_abort(a), 1u);
                    break;
                  }
                }
                nanosleep_ns(32);
              }
              float acc = 0.0f;
              for (int s2 = 0; s2 < a.K; ++s2)
                acc = fmaf(__uint_as_float(ld_relaxed_sys(cw + (size_t)s2 * a.hidden)),
                           a.route_w[l0 * a.K + s2], acc);
              for (int s2 = 0; s2 < a.K; ++s2) cw[(size_t)s2 * a.hidden] = kUnwritten;
              const float xv = __ldcg(a.xlin + (size_t)l0 * a.hidden + r) + acc;
              if (l0 + 1 < a.L) {
                a.xlin[(size_t)(l0 + 1) * a.hidden + r] = xv;
                a.xsw[(size_t)(l0 + 1) * a.hidden + sw_index(r)] = xv;
              } else {
                a.out[r] = xv;
              }
            }
            __syncwarp();
            if (lane == 0 && l0 + 1 < a.L) red_release_gpu(ctr_xrows(a, l0 + 1), (unsigned)n0);
            continue;
          }
        }
      }
      const int st = it % S;
      uint8_t* sp = stages + (size_t)st * a.stage_bytes;
      if (lane == 0) ok = mbar_wait(&empty[st], ((it / S) & 1) ^ 1);
      ok = __shfl_sync(kFull, ok, 0);
      if (!ok) break;
      const int idx = __shfl_sync(kFull, next, 0);
      if (idx >= total) break;
      int kind, l, slot, r0, nrows;
      if (EP)
        decode_item_ep(a, ep_own, ep_loff, ep_nown, idx, hint, kind, l, slot, r0, nrows);
      else
        decode_item(a, idx, kind, l, slot, r0, nrows);
      int* hdr = reinterpret_cast<int*>(sp);
      if (ROUTE && kind == kItemRoute) {
        // router rows: no weights to stage (the consumer warps read them
        // directly); the stage completes with a copy of x_l (linear), made
        // once x_l is complete (and after a timeout, in bounds)
        bool okx = true;
        if (lane == 0) {
          reinterpret_cast<int4*>(hdr)[0] = make_int4(kind, l, slot, r0);
          hdr[4] = nrows;
          // the item's router rows do not depend on x: queue them into L2
          // now, so that the warps read them from L2 once x_l is complete
          const uint8_t* gw = reinterpret_cast<const uint8_t*>(a.layer_ptrs[5 * a.L + l]) +
                              (size_t)r0 * a.hidden * 4;
          const uint32_t gbytes = (uint32_t)nrows * (uint32_t)a.hidden * 4u;
          for (uint32_t off = 0; off < gbytes; off += 32768u)
            l2_prefetch(gw + off, gbytes - off < 32768u ? gbytes - off : 32768u);
          okx = wait_count(ctr_xrows(a, l), (unsigned)a.hidden);
          fence_proxy_async_global();
          mbar_arrive_expect_tx(&full[st], (uint32_t)a.hidden * 4u);
          bulk_g2s(sp + kXOff, a.xlin + (size_t)l * a.hidden, (uint32_t)a.hidden * 4u, &full[st]);
          next = (int)atomicAdd(ctr_claim(a), 1u);
        }
        ok = __shfl_sync(kFull, okx, 0);
        ++it;
        if (!ok) break;
        continue;
      }
      if (kind == kItemPrep) {
        if (lane == 0) {
          hdr[0] = kind;
          mbar_arrive(&full[st]);
          next = (int)atomicAdd(ctr_claim(a), 1u);
        }
        ++it;
        continue;
      }
      if (ROUTE && !tab_ok[l]) {
        // routed on the device: this layer's ids exist once its router
        // items are published
        bool okr = true;
        if (lane == 0) okr = wait_count(ctr_route_ready(a, l), 1u);
        __syncwarp();
        if (lane < a.K) {
          int e = __ldcg(a.ids + l * a.K + lane);
          e = e < 0 ? 0 : (e >= a.E ? a.E - 1 : e);
          const float* gl = reinterpret_cast<const float*>(a.layer_ptrs[4 * a.L + l]);
          tab_id[l * a.K + lane] = e;
          tab_g[l * a.K + lane] = make_float2(gl[2 * e], gl[2 * e + 1]);
        }
        __syncwarp();
        if (lane == 0) tab_ok[l] = 1;
        __syncwarp();
        ok = __shfl_sync(kFull, okr, 0);
        if (!ok) break;
      }
      const bool up = kind == kItemUp;
      const TokPhase& ph = up ? a.up : a.dn;
      const int e = tab_id[l * a.K + slot];
      const uint8_t* cbase = reinterpret_cast<const uint8_t*>(tab_base[(up ? 0 : 2) * a.L + l]) +
                             (size_t)e * (up ? a.up_cs : a.dn_cs);
      const uint8_t* sbase = reinterpret_cast<const uint8_t*>(tab_base[(up ? 1 : 3) * a.L + l]) +
                             (size_t)e * (up ? a.up_ss : a.dn_ss);
      const float2 g2 = tab_g[l * a.K + slot];
      const float g = up ? g2.y : g2.x;
      float4* lut4 = reinterpret_cast<float4*>(sp + kLutOff);
      for (int q4 = lane; q4 < 64; q4 += 32) {
        const uint32_t v = 4u * (uint32_t)q4;
        lut4[q4] = make_float4(e4m3_lut_value(v) * g, e4m3_lut_value(v + 1) * g,
                               e4m3_lut_value(v + 2) * g, e4m3_lut_value(v + 3) * g);
      }
      if (lane == 0) {
        reinterpret_cast<int4*>(hdr)[0] = make_int4(kind, l, slot, r0);
        hdr[4] = nrows;
      }
      __syncwarp();
      if (lane == 0) {
        uint8_t* codes = sp + a.codes_off;
        const uint32_t code_bytes = (uint32_t)(nrows * ph.cb);
        const uint32_t scale_bytes = (uint32_t)(nrows * ph.sb);
        const uint32_t s16 = scale_bytes & ~15u;
        const uint8_t* csrc = cbase + (size_t)r0 * ph.cb;
        const uint8_t* ssrc = sbase + (size_t)r0 * ph.sb;
        for (uint32_t i = s16; i < scale_bytes; ++i) codes[ph.scale_off + i] = ssrc[i];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const uint32_t x_bytes = (uint32_t)ph.cols * 4u;
        mbar_arrive_expect_tx(&full[st], code_bytes + s16 + x_bytes);
        for (uint32_t off = 0; off < code_bytes; off += 4096u) {
          const uint32_t n = code_bytes - off < 4096u ? code_bytes - off : 4096u;
          bulk_g2s(codes + off, csrc + off, n, &full[st]);
        }
        if (s16) bulk_g2s(codes + ph.scale_off, ssrc, s16, &full[st]);
        next = (int)atomicAdd(ctr_claim(a), 1u);
        if (a.prefetch && next < total) {
          // its weight rows stream from HBM into L2 while this item waits
          int k2, l2, s2, q0, n2;
          if (EP)
            decode_item_ep(a, ep_own, ep_loff, ep_nown, next, hint, k2, l2, s2, q0, n2);
          else
            decode_item(a, next, k2, l2, s2, q0, n2);
          if ((k2 == kItemUp || k2 == kItemDown) && (!ROUTE || tab_ok[l2])) {
            const bool up2 = k2 == kItemUp;
            const TokPhase& p2 = up2 ? a.up : a.dn;
            const int e2 = tab_id[l2 * a.K + s2];
            const uint8_t* c2 = reinterpret_cast<const uint8_t*>(tab_base[(up2 ? 0 : 2) * a.L + l2]) +
                                (size_t)e2 * (up2 ? a.up_cs : a.dn_cs) + (size_t)q0 * p2.cb;
            const uint8_t* sc2 = reinterpret_cast<const uint8_t*>(tab_base[(up2 ? 1 : 3) * a.L + l2]) +
                                 (size_t)e2 * (up2 ? a.up_ss : a.dn_ss) + (size_t)q0 * p2.sb;
            l2_prefetch(c2, (uint32_t)(n2 * p2.cb));
            l2_prefetch(sc2, (uint32_t)(n2 * p2.sb) & ~15u);
          }
        }
        // the item's activation: x_l (UP) or the slot's act (DOWN)
        ok = up ? wait_count(ctr_xrows(a, l), (unsigned)a.hidden)
                : wait_count(ctr_act(a, l, slot), (unsigned)a.inter);
        fence_proxy_async_global();
        // copied even after a timeout (in bounds), so that the stage completes
        const float* xsrc = up ? a.xsw + (size_t)l * a.hidden
                               : a.actsw + ((size_t)(l & 1) * a.K + slot) * a.inter;
        bulk_g2s(sp + kXOff, xsrc, x_bytes, &full[st]);
      }
      ok = __shfl_sync(kFull, ok, 0);
      ++it;
      if (!ok) break;
    }
    // end marker for the consumers, then leave no bulk copy in flight
    if (lane == 0) {
      const int st = it % S;
      if (mbar_wait(&empty[st], ((it / S) & 1) ^ 1)) {
        *reinterpret_cast<int*>(stages + (size_t)st * a.stage_bytes) = kItemEnd;
        mbar_arrive(&full[st]);
      }
      ++it;
      for (int k = (it > S ? it - S : 0); k < it; ++k) mbar_wait(&full[k % S], (k / S) & 1);
    }
  } else if (tid >= kPub) {
    // ----------------------------------------------------------- publisher
    const int lane = tid - kPub;
    for (int k = 0;; ++k) {
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&pub_full[k % kPubRing], (k / kPubRing) & 1);
      ok = __shfl_sync(kFull, ok, 0);
      __syncwarp();
      if (!ok) break;
      const int4 q = reinterpret_cast<const int4*>(pubq)[k % kPubRing];
      const int kind = q.x, l = q.y, slot = q.z, rr = q.w;
      const int r0 = rr & 0xFFFF, nrows = rr >> 16;
      const float* yv = yring + (k % kPubRing) * 32;
      if (kind == kItemEnd) break;
      // Every lane stores its own row value; after the warp barrier lane 0's
      // release (red / atom .release.gpu, cumulative over the stores ordered
      // before it) publishes them.  All lanes work at once: the warp's path
      // through shared memory and L2 stays a few round trips long even while
      // the consumers keep the shared-memory pipe busy.  Readers acquire,
      // then bulk copy (after a proxy fence) or load with __ldcg.
      const float y = lane < nrows ? yv[lane] : 0.0f;
      if (kind == kItemPrep) {
        if (EP) {
          // Every rank enters the token before any slot row moves: a rank's
          // counters are zeroed when its previous token ends, and no peer may
          // add to them before.  Token t (this rank's epoch word, counted by
          // its last CTA) writes t + 1 into entry[ep_rank] of every rank's
          // entry flags (never reset; each entry has one writer, so a later
          // token of one rank cannot stand in for another rank's entry),
          // then lane q waits for entry[q] >= t + 1 here.
          const unsigned epoch = *reinterpret_cast<volatile unsigned*>(a.hello + kCtrLine);
          if (lane < a.ep_n) {
            st_release_sys(reinterpret_cast<unsigned*>(a.peer[lane] + a.hello_off) + a.ep_rank, epoch + 1u);
            wait_count_sys(a.hello + lane, epoch + 1u, a.timeout_ns, ctr_abort(a));
          }
          __syncwarp();
        }
        if (lane == 0) red_release_gpu(ctr_xrows(a, 0), (unsigned)a.hidden);  // stores fenced by the consumers
      } else if (ROUTE && kind == kItemRoute) {
        // router logits.  The layer's last router item (claimed after the
        // others) waits for their rows, routes the layer (the reference's
        // route_topk_f32 on one warp) and releases the layer's ids; the
        // others release their rows
        float* lg = a.rlog + (size_t)l * a.E;
        if (lane < nrows) lg[r0 + lane] = y;
        __syncwarp();
        const bool last = r0 + nrows == a.E;
        if (!last) {
          if (lane == 0) red_release_gpu(ctr_route_rows(a, l), (unsigned)nrows);
        } else {
          // (a wait that runs out records kErrTimeout; the routing goes on)
          if (lane == 0 && r0 > 0) wait_count(ctr_route_rows(a, l), (unsigned)r0);
          __syncwarp();
          const float* gb = reinterpret_cast<const float*>(a.layer_ptrs[6 * a.L + l]);
          int* io = const_cast<int*>(a.ids) + l * a.K;
          float* wo = const_cast<float*>(a.route_w) + l * a.K;
          router_topk(lg, gb, io, wo, a.E, a.K, a.scaling, a.bad_pick);
          __syncwarp();
          if (lane == 0) red_release_gpu(ctr_route_ready(a, l), 1u);
        }
      } else if (kind == kItemUp) {
        if (lane < nrows) {
          const float v = fmaxf(y, 0.0f);
          a.actsw[((size_t)(l & 1) * a.K + slot) * a.inter + sw_index(r0 + lane)] = v * v;
        }
        __syncwarp();
        if (lane == 0) red_release_gpu(ctr_act(a, l, slot), (unsigned)nrows);
      } else if (EP) {
        // a down block of an owned slot: its rows into every rank's
        // contrib[l][slot] (peer stores over NVLink).  No fence and no
        // counter: each word arrives whole, and the SUM items wait for the
        // words themselves (see kUnwritten)
        if (lane < nrows) {
          const size_t at = ((size_t)l * a.K + slot) * a.hidden + r0 + lane;
          unsigned u = __float_as_uint(y);
          if (u == kUnwritten) u = 0x7FFFFFFFu;
          for (int q2 = 0; q2 < a.ep_n; ++q2)
            st_relaxed_sys(reinterpret_cast<unsigned*>(a.peer[q2] + a.contrib_off) + at, u);
        }
      } else if (slot + 1 < a.K) {
        // a down block of slots 0..K-2: its rows, then the block's count
        if (lane < nrows) a.contrib[((size_t)(l & 1) * a.K + slot) * a.hidden + r0 + lane] = y;
        __syncwarp();
        if (lane == 0) red_release_gpu(ctr_blk(a, l, r0 / a.dn.krt), 1u);
      } else {
        // the block of the last slot: once the other slots' rows of the block
        // are in (their items were claimed earlier, so the wait is usually
        // over), the route sum of its rows in ROUTE order, acc = fmaf(y_s,
        // w_s, acc) from 0, and x_{l+1} = x_l + acc
        // (a wait that runs out records kErrTimeout; the sum then goes on)
        if (lane == 0 && a.K > 1) wait_count(ctr_blk(a, l, r0 / a.dn.krt), (unsigned)(a.K - 1));
        __syncwarp();
        const int r = r0 + lane;
        if (lane < nrows) {
          const float* cb = a.contrib + (size_t)(l & 1) * a.K * a.hidden;
          float acc = 0.0f;
          for (int s2 = 0; s2 + 1 < a.K; ++s2)
            acc = fmaf(__ldcg(cb + (size_t)s2 * a.hidden + r),
                       ROUTE ? __ldcg(a.route_w + l * a.K + s2) : a.route_w[l * a.K + s2], acc);
          acc = fmaf(y, ROUTE ? __ldcg(a.route_w + l * a.K + a.K - 1) : a.route_w[l * a.K + a.K - 1], acc);
          const float xv = __ldcg(a.xlin + (size_t)l * a.hidden + r) + acc;
          if (l + 1 < a.L) {
            a.xlin[(size_t)(l + 1) * a.hidden + r] = xv;
            a.xsw[(size_t)(l + 1) * a.hidden + sw_index(r)] = xv;
          } else {
            a.out[r] = xv;
          }
        }
        __syncwarp();
        if (lane == 0 && l + 1 < a.L) red_release_gpu(ctr_xrows(a, l + 1), (unsigned)nrows);
      }
      __syncwarp();
      if (lane == 0) st_release_cta(pub_done, k + 1);
    }
  } else {
    // ----------------------------------------------------------- consumers
    const SegPlace pu = seg_place(a.up, tid), pd = seg_place(a.dn, tid);
    const int tr = tid >> 3, tw = tid & 7;
    float2 x[16];
    int last_key = -1;
    bool ring_fail = false;  // tid 0: the publisher stopped taking items
    int it = 0;
    for (;; ++it) {
      const int st = it % S;
      const bool to = !mbar_wait(&full[st], (it / S) & 1) || ring_fail;
      const uint8_t* sp = stages + (size_t)st * a.stage_bytes;
      const int* hdr = reinterpret_cast<const int*>(sp);
      const int kind = to ? kItemEnd : hdr[0];
      int l = 0, slot = 0, r0 = 0, nrows = 0;
      float route_v = 0.0f;  // kItemRoute: this warp's router logit (lane 0)
      if (ROUTE && kind == kItemRoute) {
        l = hdr[1];
        r0 = hdr[3];
        nrows = hdr[4];
        const int w = tid >> 5;
        if (w < nrows) {
          const float* gw = reinterpret_cast<const float*>(a.layer_ptrs[5 * a.L + l]) +
                            (size_t)(r0 + w) * a.hidden;
          route_v = router_row(gw, reinterpret_cast<const float*>(sp + kXOff), a.hidden, tid & 31);
        }
      } else if (kind == kItemPrep) {
        const int nu = a.hidden >> 5;
        float4* xs0 = reinterpret_cast<float4*>(a.xsw);
        for (int f = tid; f < nu * 8; f += kCT) {
          const int t = f >> 3, k = f & 7;
          xs0[t * 8 + (k ^ (t & 7))] = x_slot(a.x_in, t, k);
        }
        for (int i = tid; i < a.hidden; i += kCT) a.xlin[i] = a.x_in[i];
        fence_proxy_async_global();
        __threadfence();
      } else if (kind == kItemUp || kind == kItemDown) {
        l = hdr[1];
        slot = hdr[2];
        r0 = hdr[3];
        nrows = hdr[4];
        const bool up = kind == kItemUp;
        const TokPhase& ph = up ? a.up : a.dn;
        const SegPlace& sp2 = up ? pu : pd;
        const int key = (kind << 24) | (l << 8) | slot;
        bool x_stale = key != last_key;
        last_key = key;
        // a row of fewer than 64 units leaves chains 4 n_u..255 unwritten:
        // zero them (the other projection's item may have left values there)
        const int nch = 4 * ph.n_u;
        if (nch < 256) {
          const int w = 256 - nch;
          for (int i = tid; i < nrows * w; i += kCT) {
            const int rr = i / w;
            part[rr * kRowPitch + part_index(nch + (i - rr * w))] = 0.0f;
          }
        }
        if (sp2.active) {
          const uint32_t stage_off = (uint32_t)(a.stage_base + st * a.stage_bytes + a.codes_off);
          const float* lut = reinterpret_cast<const float*>(sp + kLutOff);
          const float4* xs = reinterpret_cast<const float4*>(sp + kXOff);
          if (nrows == ph.krt) {
            segments<H, true>(smem, stage_off, ph.scale_off, ph.cb, ph.sb, sp2.team, ph.teams, sp2.par1,
                              sp2.par2, sp2.cont, sp2.u1, sp2.u2, sp2.grp, nrows, lut, xs, x, x_stale,
                              part);
          } else {
            segments<H, false>(smem, stage_off, ph.scale_off, ph.cb, ph.sb, sp2.team, ph.teams, sp2.par1,
                               sp2.par2, sp2.cont, sp2.u1, sp2.u2, sp2.grp, nrows, lut, xs, x, x_stale,
                               part);
          }
        }
      }
      // tid 0: this item's publisher ring slot must be free (the publisher
      // has taken item it - kPubRing); a wait that runs out stops everyone
      if (tid == 0 && !to && kind != kItemEnd && !wait_smem_gt(pub_done, it - kPubRing)) ring_fail = true;
      // every read of the stage is done; a timeout anywhere stops all consumers
      const bool stop = named_bar_or(kBarC, kCT, to || ring_fail);
      if (tid == 0 && !stop && kind != kItemEnd) mbar_arrive(&empty[st]);
      if (stop || kind == kItemEnd) break;
      if (ROUTE && kind == kItemRoute) {
        if ((tid & 31) == 0 && (tid >> 5) < nrows) yring[(it % kPubRing) * 32 + (tid >> 5)] = route_v;
      } else if (kind != kItemPrep) {
        float y = 0.0f;
        if (tr < nrows) y = group_tree(part + tr * kRowPitch + tw * kGroupPitch);
        y = combine8(y);
        if (tw == 0 && tr < nrows) yring[(it % kPubRing) * 32 + tr] = y;
      }
      named_bar_sync(kBarC, kCT);  // the chain buffer is rewritten by the next item
      if (tid == 0) {  // hand the item to the publisher
        reinterpret_cast<int4*>(pubq)[it % kPubRing] = make_int4(kind, l, slot, r0 | (nrows << 16));
        mbar_arrive(&pub_full[it % kPubRing]);
      }
    }
    // end marker for the publisher
    if (tid == 0 && !ring_fail && wait_smem_gt(pub_done, it - kPubRing)) {
      pubq[(it % kPubRing) * 4] = kItemEnd;
      mbar_arrive(&pub_full[it % kPubRing]);
    }
  }

  // the last CTA to leave resets the counters for the next token
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(ctr_exited(a), 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    for (int i = tid; i < a.n_ctr; i += kTokThreads) a.ctr[i] = 0u;
    if (EP && tid == 0) atomicAdd(a.hello + kCtrLine, 1u);  // this rank's next token
  }
}

// ---------------------------------------------------------------- host

int row_block_tok(int cols) {
  int g = 256;
  while (cols % g != 0) g >>= 1;
  return 256 / g;
}

inline int align_up_tok(int v, int a) { return (v + a - 1) / a * a; }

int env_int(const char* name, int dflt, int lo, int hi) {
  const char* e = getenv(name);
  int v = e ? atoi(e) : dflt;
  return v < lo ? lo : (v > hi ? hi : v);
}

TokPhase make_phase(int rows, int cols) {
  TokPhase p{};
  p.rows = rows;
  p.cols = cols;
  p.n_u = cols / 32;
  p.n2 = p.n_u > 64 ? p.n_u - 64 : 0;
  p.teams = kCT / p.n_u;
  if (p.teams > 16) p.teams = 16;
  p.cb = cols / 2;
  p.sb = cols / 16;
  return p;
}

template <typename K>
int set_smem_tok(K kernel, int bytes) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return kErrLaunch;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return kErrLaunch;
  return kOk;
}

template <int H, bool ROUTE, bool EP = false>
int launch_token_h(const TokArgs& a, int smem, bool pdl, cudaStream_t stream) {
  if (set_smem_tok(moe_token_kernel<H, ROUTE, EP>, smem)) return kErrLaunch;
  int dev = 0, sms = 0, occ = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, moe_token_kernel<H, ROUTE, EP>, kTokThreads, smem) !=
      cudaSuccess)
    return kErrLaunch;
  if (occ < 1) return kErrShape;
  if (occ > 2) occ = 2;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(sms * occ);
  cfg.blockDim = dim3(kTokThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, moe_token_kernel<H, ROUTE, EP>, a) == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

size_t moe_token_scratch_bytes(int n_layers, int hidden, int inter, int top_k) {
  const size_t n_ctr = token_ctr_words(n_layers, top_k, hidden / 2);
  const size_t ctr = (n_ctr * 4 + 255) / 256 * 256;
  return ctr + 4 * ((size_t)2 * n_layers * hidden + (size_t)2 * top_k * inter + (size_t)2 * top_k * hidden +
                    (size_t)n_layers * kTokMaxRouteExperts);
}

// EP scratch (the same on every rank): counters, the token-entry flags and
// the epoch word (256 bytes, never reset), x_l linear and swizzled [L][hidden], act
// [2][K][inter], contrib [L][K][hidden].
size_t moe_token_ep_contrib_offset(int n_layers, int hidden, int inter, int top_k) {
  const size_t n_ctr = token_ctr_words(n_layers, top_k, hidden / 2);
  const size_t ctr = (n_ctr * 4 + 255) / 256 * 256;
  return ctr + 256 + 4 * ((size_t)2 * n_layers * hidden + (size_t)2 * top_k * inter);
}

size_t moe_token_ep_scratch_bytes(int n_layers, int hidden, int inter, int top_k) {
  return moe_token_ep_contrib_offset(n_layers, hidden, inter, top_k) +
         4 * (size_t)n_layers * top_k * hidden;
}

// Counters, entry flags and epoch zero; every contrib word unwritten.
int prepare_moe_token_ep(void* scratch, int n_layers, int hidden, int inter, int top_k,
                         cudaStream_t stream) {
  const size_t off = moe_token_ep_contrib_offset(n_layers, hidden, inter, top_k);
  const size_t n = moe_token_ep_scratch_bytes(n_layers, hidden, inter, top_k) - off;
  if (cudaMemsetAsync(scratch, 0, off, stream) != cudaSuccess ||
      cudaMemsetAsync(reinterpret_cast<uint8_t*>(scratch) + off, 0xFF, n, stream) != cudaSuccess)
    return kErrLaunch;
  return kOk;
}

int launch_moe_token(const MoeTokenArgs& in, cudaStream_t stream) {
  TokArgs a{};
  a.layer_ptrs = in.layer_ptrs;
  a.up_cs = in.up_code_stride;
  a.up_ss = in.up_scale_stride;
  a.dn_cs = in.dn_code_stride;
  a.dn_ss = in.dn_scale_stride;
  a.ids = in.ids;
  a.route_w = in.route_w;
  a.route = in.route ? 1 : 0;
  a.scaling = in.scaling;
  a.bad_pick = in.bad_pick;
  if (a.route && in.n_experts > kTokMaxRouteExperts) return kErrShape;
  a.x_in = in.x;
  a.out = in.out;
  a.L = in.n_layers;
  a.K = in.top_k;
  a.E = in.n_experts;
  a.hidden = in.hidden;
  a.inter = in.inter;
  a.up = make_phase(in.inter, in.hidden);
  a.dn = make_phase(in.hidden, in.inter);
  const bool ep = in.ep_ranks > 1;
  if (ep && (a.route || in.ep_ranks > kTokMaxRanks || in.ep_rank < 0 || in.ep_rank >= in.ep_ranks ||
             !in.peers))
    return kErrArg;
  const int blk_u = row_block_tok(in.hidden), blk_d = row_block_tok(in.inter);

  int dev = 0, smem_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  const int budget = (smem_sm - 2 * 1024) / 2;  // two CTAs per SM
  const int x_bytes = 4 * (in.hidden > in.inter ? in.hidden : in.inter);
  // Largest rows-per-segment H whose ring of at least min_stages stages fits
  // two CTAs per SM; the ring then takes every stage that fits (at most 4).
  // ERVF_TOKEN_H / ERVF_TOKEN_STAGES (read once per process) cap H and raise
  // the minimum depth for tuning; results are the same for every choice.
  static const int max_h = env_int("ERVF_TOKEN_H", 4, 1, 4);
  static const int min_stages = env_int("ERVF_TOKEN_STAGES", 2, 2, kTokMaxStages);
  static const int prefetch = env_int("ERVF_TOKEN_PREFETCH", 1, 0, 1);
  a.prefetch = prefetch;
  int h = 0, smem = 0;
  for (int cand = max_h; cand >= 1; --cand) {
    const int ku = a.up.teams * 2 * cand, kd = a.dn.teams * 2 * cand;
    if (ku > 32 || kd > 32 || ku % blk_u || kd % blk_d) continue;
    const int codes_off = align_up_tok(kXOff + x_bytes, 128);
    const int wu = ku * a.up.cb + align_up_tok(ku * a.up.sb, 16);
    const int wd = kd * a.dn.cb + align_up_tok(kd * a.dn.sb, 16);
    const int stage = align_up_tok(codes_off + (wu > wd ? wu : wd), 128);
    const int kmax = ku > kd ? ku : kd;
    const int tab = ep ? token_tab_bytes_ep(in.n_layers, in.top_k) : token_tab_bytes(in.n_layers, in.top_k);
    const int part_off = align_up_tok(kTabOff + tab, 128);
    const int base = align_up_tok(part_off + kmax * kRowPitch * 4, 128);
    int stages = (budget - base) / stage;
    if (stages > kTokMaxStages) stages = kTokMaxStages;
    if (stages >= min_stages) {
      h = cand;
      a.up.krt = ku;
      a.dn.krt = kd;
      a.codes_off = codes_off;
      a.stage_bytes = stage;
      a.stage_base = base;
      a.part_off = part_off;
      a.stages = stages;
      smem = base + stages * stage;
      break;
    }
  }
  if (h == 0) return kErrShape;
  a.up.scale_off = a.up.krt * a.up.cb;
  a.dn.scale_off = a.dn.krt * a.dn.cb;
  a.up.n_items = (a.up.rows + a.up.krt - 1) / a.up.krt;
  a.dn.n_items = (a.dn.rows + a.dn.krt - 1) / a.dn.krt;
  a.n_route = a.route ? (a.E + kRouteRows - 1) / kRouteRows : 0;
  a.per_layer = a.n_route + a.K * (a.up.n_items + a.dn.n_items);
  a.total = 1 + a.L * a.per_layer;

  uint8_t* s = reinterpret_cast<uint8_t*>(in.scratch);
  // counters of this launch's row blocks; the area is laid out for the
  // most blocks any H gives, so that the vectors after it do not move
  a.B = a.dn.n_items;
  a.n_ctr = (int)token_ctr_words(a.L, a.K, a.B);
  a.ctr = reinterpret_cast<unsigned*>(s);
  s += (token_ctr_words(a.L, a.K, a.hidden / 2) * 4 + 255) / 256 * 256;
  if (ep) {
    const uint8_t* base = reinterpret_cast<const uint8_t*>(in.scratch);
    a.ep_n = in.ep_ranks;
    a.ep_rank = in.ep_rank;
    for (int q = 0; q < in.ep_ranks; ++q) a.peer[q] = in.peers[q];
    a.hello = reinterpret_cast<unsigned*>(s);
    a.hello_off = (size_t)(s - base);
    a.timeout_ns = in.timeout_ns;
    s += 256;
    a.xlin = reinterpret_cast<float*>(s);
    s += (size_t)4 * a.L * a.hidden;
    a.xsw = reinterpret_cast<float*>(s);
    s += (size_t)4 * a.L * a.hidden;
    a.actsw = reinterpret_cast<float*>(s);
    s += (size_t)4 * 2 * a.K * a.inter;
    a.contrib = reinterpret_cast<float*>(s);
    a.contrib_off = (size_t)(s - base);
    a.rlog = nullptr;
    switch (h) {
      case 4: return launch_token_h<4, false, true>(a, smem, in.pdl, stream);
      case 3: return launch_token_h<3, false, true>(a, smem, in.pdl, stream);
      case 2: return launch_token_h<2, false, true>(a, smem, in.pdl, stream);
      default: return launch_token_h<1, false, true>(a, smem, in.pdl, stream);
    }
  }
  a.xlin = reinterpret_cast<float*>(s);
  s += (size_t)4 * a.L * a.hidden;
  a.xsw = reinterpret_cast<float*>(s);
  s += (size_t)4 * a.L * a.hidden;
  a.actsw = reinterpret_cast<float*>(s);
  s += (size_t)4 * 2 * a.K * a.inter;
  a.contrib = reinterpret_cast<float*>(s);
  s += (size_t)4 * 2 * a.K * a.hidden;
  a.rlog = reinterpret_cast<float*>(s);

  if (a.route) {
    switch (h) {
      case 4: return launch_token_h<4, true>(a, smem, in.pdl, stream);
      case 3: return launch_token_h<3, true>(a, smem, in.pdl, stream);
      case 2: return launch_token_h<2, true>(a, smem, in.pdl, stream);
      default: return launch_token_h<1, true>(a, smem, in.pdl, stream);
    }
  }
  switch (h) {
    case 4: return launch_token_h<4, false>(a, smem, in.pdl, stream);
    case 3: return launch_token_h<3, false>(a, smem, in.pdl, stream);
    case 2: return launch_token_h<2, false>(a, smem, in.pdl, stream);
    default: return launch_token_h<1, false>(a, smem, in.pdl, stream);
  }
}

int read_token_device_error(bool clear) { return read_unit_error(clear); }

}  // namespace ervf
