// nvfp4_mma.cu -- batched NVFP4 GEMM on the sm_100a tensor cores, warp
// specialised:
//
//   out[n][r] = g * sum_k (e2m1[r][k] * e4m3[r][k/16]) * X[n][k],  n < N <= 16
//
// the decode-batch variant of the expert / head GEMV (the reference's batched
// path is the SIMT gemm_nvfp4_rows_b, sweepspec.py:28-240), and the
// expert-major grouped form of the batched MoE block (sweepspec.py:244-375).
// A tolerance path (rel-L2 <= 1e-3 against a float64 dequantise-then-matmul),
// not the batch-1 chain order: the weights are exact in f16 (e2m1 has two
// significant bits, E4M3 four: a 6-bit product in 2^-10 .. 2688), X is
// rounded to f16, the global scale g is applied to the fp32 accumulator.
//
// One CTA per SM, 17 warps, persistent over work units: 128 weight rows x one
// K range (grouped mode: unit = (expert chunk, 128-row tile, K range)).  The
// K range walks k-blocks of 256 columns through a ring of shared-memory
// stages and tensor-memory A stages:
//
//   warp 0, one lane   producer.  Per unit: one 1-D bulk copy of the tile's
//                      block-scale rows (contiguous: 128 rows x cols/16
//                      bytes).  Per k-block: one 2-D TMA load of the code
//                      tile [128 rows][128 B] (128-byte swizzle; columns or
//                      rows past the matrix read as zero) and one 1-D bulk
//                      copy of the activation tile (16 x 256 f16 in the MMA's
//                      K-major core-matrix layout, 8 KB, prepared once per
//                      call by pack_panel_kernel) into ring stage s.  This
//                      GPU's own memory only; no multicast anywhere.
//   warps 1..4, lane 0 MMA.  Issuer c issues MMAs c, c+4, c+8, c+12 of the
//                      16 tcgen05.mma.cta_group::1.kind::f16 of a k-block
//                      (M128 N16 K16, A from tensor memory, B from the
//                      stage) into its own fp32 accumulator chain c of
//                      buffer d; each issuer's tcgen05.commit counts once on
//                      the barriers that free the smem stage and the A stage,
//                      and, after the unit's last k-block, fill buffer d.
//   warps 5..12        decoders.  Warp w owns tensor-memory lanes 32 (w % 4)
//                      .. +31 (= tile rows) and half (w - 5) / 4 of the
//                      k-block's 256 columns: codes from the swizzled tile,
//                      e2m1 pairs -> f16x2 (hardware converter) times the
//                      f16x2 block scale, tcgen05.st into A stage a.
//   warps 13..16       epilogue.  tcgen05.ld of the four chains of buffer d
//                      (warp w: lanes 32 (w % 4) ..), added in a fixed order,
//                      times g, then the mode's store, and frees d.  With a
//                      K split, each split stores its fp32 partial; the last
//                      split of a unit (counter) adds them in split order --
//                      deterministic, the same bits whatever the arrival
//                      order or the grid.
//
// Every wait is bounded (%clock64); a wait that runs out records
// kErrTimeout, marks the CTA dead, and every role drains: no copy or MMA is
// left in flight when tensor memory is released.
#include <cuda.h>  // CUtensorMap and the encode function's types (driver entry point)

#include "common.cuh"
#include "kernels.h"

namespace ervf {

namespace {

// MMA issue: one tcgen05.mma takes its issuing thread ~95 cycles whatever the
// shape (measured on B200 for M128 / M64 x N16..N128), while issuers in
// different warps overlap (4 issuers: ~30 cycles per MMA in aggregate).  So
// kMmaIssuers warps issue a k-block's MMAs, each its own accumulator chain.
constexpr int kMmaIssuers = 4;
#ifndef ERVF_MMA_DEC_WARPS
#define ERVF_MMA_DEC_WARPS 8
#endif
// Decoders: kDecWarps warps, kDecWarps / 4 per tensor-memory lane quadrant,
// each of a quadrant's warps on kDecCols of the k-block's 256 columns.
constexpr int kDecWarps = ERVF_MMA_DEC_WARPS;
constexpr int kDecGroups = kDecWarps / 4;
constexpr int kDecCols = 256 / kDecGroups;  // columns per decoder thread and k-block
constexpr int kDecSc = kDecCols / 16;       // their block-scale bytes
constexpr int kDecSt = kDecCols / 64;       // their tcgen05.st of 32 columns
static_assert(kDecWarps % 4 == 0 && kDecSt >= 1 && kDecSc % 4 == 0, "decoder split");
constexpr int kMmaWarps = 1 + kMmaIssuers + kDecWarps + 4;
constexpr int kMmaThreads = kMmaWarps * 32;
constexpr int kM = 128;               // rows per unit (UMMA M)
constexpr int kN = 16;                // batch columns (UMMA N)
constexpr int kKB = 256;              // columns per k-block
#ifndef ERVF_MMA_STAGES
#define ERVF_MMA_STAGES 4
#endif
constexpr int kStages = ERVF_MMA_STAGES;  // smem ring depth
constexpr int kAStages = 3;           // tensor-memory A stages
constexpr int kCodeTile = kM * kKB / 2;       // 16 KB
constexpr int kBTile = kN * kKB * 2;          // 8 KB
constexpr int kStageBytes = kCodeTile + kBTile;
constexpr int kScaleBuf = kM * 256;           // scale rows of a tile, cols <= 4096
constexpr int kTmemCols = 512;
// Accumulators: kDAcc independent chains per buffer (the 16 MMAs of a
// k-block go round-robin over them, so that consecutive MMAs do not wait on
// each other's result), two buffers: columns (d * kDAcc + c) * 16 .. + 15.
constexpr int kDAcc = 4;
static_assert(kMmaIssuers == kDAcc, "one accumulator chain per MMA issuer");
constexpr int kDCol = 0;
constexpr int kACol = 2 * kDAcc * kN;          // A stages: 128 + 128 a
constexpr int kAStageCols = kKB / 2;          // 128 (two f16 per 32-bit column)
static_assert(kACol + kAStages * kAStageCols <= kTmemCols, "tensor-memory columns");
constexpr int kDecodeWarp0 = 1 + kMmaIssuers, kEpiWarp0 = kDecodeWarp0 + kDecWarps;

// shared memory: [0, 1024) barriers and slots, then the ring (1024-aligned
// stages: the 128-byte swizzle repeats every 1024 bytes), then two scale buffers
constexpr int kRingOff = 1024;
constexpr int kScaleOff = kRingOff + kStages * kStageBytes;
constexpr int kSmem = kScaleOff + 2 * kScaleBuf;

enum MmaMode { kSingle = 0, kUp = 1, kDown = 2 };

struct MmaArgs {
  // weights: rows [row0_of(unit) ..) of the code tensor map (codes viewed as
  // [R][cols/2] bytes) and of `scales` ([R][cols/16] bytes, row-major)
  const uint8_t* scales;
  int rows, cols, R;  // rows of one matrix (expert), its cols, rows of the whole map
  int mode;
  float g;            // kSingle: the global scale
  const float* globals;  // grouped: [E][2], column gsel
  int gsel;
  // activations: pre-packed f16 panels, one per chunk (kSingle: one), nkb
  // k-block tiles of 8 KB each
  const uint8_t* panel;
  // grouped units: chunk c = expert chunk_expert[c] with pairs chunk_off[c] ..
  // + chunk_n[c]; kSingle: one chunk of n columns
  const int* chunk_expert;
  const int* chunk_off;
  const int* chunk_n;
  const int* n_chunks;
  int max_chunks, n;
  int tiles, splits, nkb;
  // outputs.  kSingle: out[j * rows + r].  kDown: out[(chunk_off + j) * rows
  // + r].  kUp: relu^2 (or SwiGLU of row pairs 2i / 2i+1) as f16 into the
  // down launch's panels, panel_out[c] at K index r (or i)
  float* out;
  uint8_t* panel_out;
  int out_kb;      // k-blocks of a panel_out chunk
  int out_rows;    // kUp: K extent written into panel_out (rows, or rows / 2 with SwiGLU)
  int relu2, swiglu;
  // K split: part[split][col][rows] fp32 for (chunk, tile) unit counter
  // ucnt[(chunk * tiles + tile)] (zero before, left zero)
  float* part;
  unsigned* ucnt;
  int part_cols;
};

// 16 consecutive 32-bit tensor-memory columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// kind::f16 instruction descriptor: D f32, A / B f16, both K-major, N, M.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Four E4M3 scale bytes (NaN bytes 0x7F / 0xFF -> +0, the reference's table)
// as f16x2 broadcasts bc[i] = (s_i, s_i).
__device__ __forceinline__ void scales4(uint32_t q, uint32_t (&bc)[4]) {
  const uint32_t nan = __vcmpeq4(q & 0x7F7F7F7Fu, 0x7F7F7F7Fu);
  q &= ~nan;
  uint32_t lo, hi;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"((uint16_t)(q & 0xFFFFu)));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"((uint16_t)(q >> 16)));
  bc[0] = __byte_perm(lo, 0, 0x1010);
  bc[1] = __byte_perm(lo, 0, 0x3232);
  bc[2] = __byte_perm(hi, 0, 0x1010);
  bc[3] = __byte_perm(hi, 0, 0x3232);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
        "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that also gives up when another role of the CTA died.
__device__ __forceinline__ bool wait_or_dead(uint64_t* bar, uint32_t parity, volatile int* dead) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*dead) return false;
    if (clock64() - t0 > 2000000000LL) {
      atomicExch(&g_device_error, kErrTimeout);
      *dead = 1;
      return false;
    }
  }
  return true;
}

// The CTA's units: a balanced contiguous range of the valid units (chunks
// known on the device).  Unit u -> (chunk, tile, split), split fastest.
struct Unit {
  int chunk, tile, split, kb0, kb1;
};

__device__ __forceinline__ void unit_range(const MmaArgs& a, int& u0, int& u1) {
  const int chunks = a.mode == kSingle ? 1 : min(__ldg(a.n_chunks), a.max_chunks);
  const long long total = (long long)chunks * a.tiles * a.splits;
  const long long G = gridDim.x, b = blockIdx.x;
  u0 = (int)(total * b / G);
  u1 = (int)(total * (b + 1) / G);
}

__device__ __forceinline__ Unit unit_of(const MmaArgs& a, int u) {
  Unit r;
  r.split = u % a.splits;
  const int ct = u / a.splits;
  r.tile = ct % a.tiles;
  r.chunk = ct / a.tiles;
  r.kb0 = (int)((long long)r.split * a.nkb / a.splits);
  r.kb1 = (int)((long long)(r.split + 1) * a.nkb / a.splits);
  return r;
}

__device__ __forceinline__ int unit_expert(const MmaArgs& a, const Unit& un) {
  return a.mode == kSingle ? 0 : __ldg(&a.chunk_expert[un.chunk]);
}

__device__ __forceinline__ int unit_n(const MmaArgs& a, const Unit& un) {
  return a.mode == kSingle ? a.n : __ldg(&a.chunk_n[un.chunk]);
}

__device__ __forceinline__ int unit_off(const MmaArgs& a, const Unit& un) {
  return a.mode == kSingle ? 0 : __ldg(&a.chunk_off[un.chunk]);
}

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// f16 value v of (chunk c, column j, K index k) into the down launch's panel
__device__ __forceinline__ void panel_put(uint8_t* panel, int kbs, int c, int j, int k, __half v) {
  uint8_t* t = panel + ((size_t)c * kbs + (k >> 8)) * kBTile;
  const int kk = k & 255;
  *reinterpret_cast<__half*>(t + (j >> 3) * 4096 + (kk >> 3) * 128 + (j & 7) * 16 + (kk & 7) * 2) = v;
}

__global__ void __launch_bounds__(kMmaThreads, 1)
    nvfp4_mma_kernel(const __grid_constant__ CUtensorMap codes_map, MmaArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);    // [kStages]
  uint64_t* empty = full + kStages;                      // [kStages]
  uint64_t* afull = empty + kStages;                     // [kAStages]
  uint64_t* aempty = afull + kAStages;                   // [kAStages]
  uint64_t* dfull = aempty + kAStages;                   // [2]
  uint64_t* dempty = dfull + 2;                          // [2]
  uint64_t* sfull = dempty + 2;                          // [2] scale buffers
  uint64_t* sempty = sfull + 2;                          // [2]
  uint64_t* mma_done = sempty + 2;                       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 512);
  volatile int* dead = reinterpret_cast<volatile int*>(smem + 516);
  int* s_last = reinterpret_cast<int*>(smem + 520);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kMmaIssuers);
    }
    for (int i = 0; i < kAStages; ++i) {
      mbar_init(&afull[i], kDecWarps);
      mbar_init(&aempty[i], kMmaIssuers);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull[i], kMmaIssuers);
      mbar_init(&dempty[i], 4);
      mbar_init(&sfull[i], 1);
      mbar_init(&sempty[i], kDecWarps);
    }
    mbar_init(mma_done, kMmaIssuers);
    *dead = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  int u0, u1;
  unit_range(a, u0, u1);
  const int sb = a.cols >> 4;
  uint8_t* ring = smem + kRingOff;
  uint8_t* sbuf = smem + kScaleOff;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      uint32_t gk = 0;
      int nu = 0;
      for (int u = u0; u < u1 && !*dead; ++u, ++nu) {
        const Unit un = unit_of(a, u);
        const int e = unit_expert(a, un);
        const int row0 = e * a.rows + un.tile * kM;  // row of the tile in the code map
        // block scales of the tile's rows (all K: contiguous), one buffer per unit parity
        const int sbi = nu & 1;
        if (!wait_or_dead(&sempty[sbi], ((nu >> 1) & 1) ^ 1, dead)) break;
        {
          const int nrow = min(kM, a.rows - un.tile * kM);
          const uint32_t bytes = (uint32_t)(nrow * sb), b16 = bytes & ~15u;
          const uint8_t* src = a.scales + (size_t)row0 * sb;
          uint8_t* dst = sbuf + sbi * kScaleBuf;
          for (uint32_t i = b16; i < bytes; ++i) dst[i] = src[i];
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive_expect_tx(&sfull[sbi], b16);
          if (b16) bulk_g2s(dst, src, b16, &sfull[sbi]);
        }
        const uint8_t* pan = a.panel + (size_t)(a.mode == kSingle ? 0 : un.chunk) * a.nkb * kBTile;
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++gk) {
          const int s = (int)(gk % kStages);
          if (!wait_or_dead(&empty[s], ((gk / kStages) & 1) ^ 1, dead)) break;
          uint8_t* st = ring + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kCodeTile + kBTile);
          tma_load_2d(st, &codes_map, kb * (kKB / 2), row0, &full[s]);
          bulk_g2s(st + kCodeTile, pan + (size_t)kb * kBTile, kBTile, &full[s]);
        }
      }
      // leave no copy in flight: wait (bounded) for the last stages
      for (uint32_t k = gk > (uint32_t)kStages ? gk - kStages : 0; k < gk; ++k)
        mbar_wait(&full[k % kStages], (k / kStages) & 1, 2000000000LL);
    }
  } else if (warp <= kMmaIssuers) {
    // ----------------------------------------------------------- MMA issue
    // issuer c = warp - 1: MMAs c, c + 4, ... of every k-block, accumulator
    // chain c; every stage / buffer barrier counts one commit per issuer
    const int c = warp - 1;
    if (lane == 0) {
      uint32_t gk = 0;
      int nu = 0;
      for (int u = u0; u < u1 && !*dead; ++u, ++nu) {
        const Unit un = unit_of(a, u);
        const int d = nu & 1;
        if (!wait_or_dead(&dempty[d], ((nu >> 1) & 1) ^ 1, dead)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        bool ok = true;
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++gk) {
          const int s = (int)(gk % kStages), as = (int)(gk % kAStages);
          // the stage's activation tile has landed (the decoders saw the same
          // phase) and the decoded A stage is in tensor memory
          if (!wait_or_dead(&full[s], (gk / kStages) & 1, dead) ||
              !wait_or_dead(&afull[as], (gk / kAStages) & 1, dead)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t b0 = smem_u32(ring + s * kStageBytes + kCodeTile);
#pragma unroll
          for (int jj = 0; jj < kKB / 16 / kMmaIssuers; ++jj) {
            const int j = c + kMmaIssuers * jj;
            const uint64_t db = umma_desc(b0 + 256 * j, 128, 4096);
            const uint32_t acc = (kb > un.kb0 || jj > 0) ? 1u : 0u;
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
                ::"r"(tmem + kDCol + (d * kDAcc + c) * kN),
                  "r"(tmem + kACol + as * kAStageCols + 8 * j), "l"(db),
                  "r"(kIdesc), "r"(acc) : "memory");
          }
          umma_commit(&empty[s]);
          umma_commit(&aempty[as]);
        }
        if (!ok) break;
        umma_commit(&dfull[d]);
      }
      // every MMA issued by this thread is complete before tensor memory is freed
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, 2000000000LL);
    }
  } else if (warp < kEpiWarp0) {
    // ---------------------------------------------------------- decoders
    const int q = warp & 3, h = (warp - kDecodeWarp0) >> 2;
    const int r = 32 * q + lane;  // tile row = tensor-memory lane
    uint32_t gk = 0;
    int nu = 0;
    for (int u = u0; u < u1 && !*dead; ++u, ++nu) {
      const Unit un = unit_of(a, u);
      const int sbi = nu & 1;
      if (!__all_sync(0xffffffffu, wait_or_dead(&sfull[sbi], (nu >> 1) & 1, dead))) break;
      const uint8_t* srow = sbuf + sbi * kScaleBuf + r * sb;
      bool ok = true;
      for (int kb = un.kb0; kb < un.kb1; ++kb, ++gk) {
        const int s = (int)(gk % kStages), as = (int)(gk % kAStages);
        bool w_ok = wait_or_dead(&full[s], (gk / kStages) & 1, dead);
        w_ok = w_ok && wait_or_dead(&aempty[as], ((gk / kAStages) & 1) ^ 1, dead);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        const uint8_t* tile = ring + s * kStageBytes + r * 128;
        // this group's kDecSc scale bytes (blocks kDecSc h .. of the
        // k-block).  Bytes past the row belong to the next row or to stale
        // data: finite after the NaN mask, and their columns' codes are zero
        // (TMA zero fill).
        const int sc = kb * 16 + kDecSc * h;
        uint32_t sq[kDecSc / 4];
        if ((sb & 3) == 0) {
#pragma unroll
          for (int j = 0; j < kDecSc / 4; ++j) sq[j] = *reinterpret_cast<const uint32_t*>(srow + sc + 4 * j);
        } else {
          const uint16_t* p2 = reinterpret_cast<const uint16_t*>(srow + sc);
#pragma unroll
          for (int j = 0; j < kDecSc / 4; ++j) sq[j] = (uint32_t)p2[2 * j] | ((uint32_t)p2[2 * j + 1] << 16);
        }
        uint32_t bc[kDecSc];
#pragma unroll
        for (int j = 0; j < kDecSc / 4; ++j) {
          uint32_t t[4];
          scales4(sq[j], t);
          bc[4 * j] = t[0]; bc[4 * j + 1] = t[1]; bc[4 * j + 2] = t[2]; bc[4 * j + 3] = t[3];
        }
        const uint32_t acol =
            tmem + ((uint32_t)(32 * q) << 16) + kACol + as * kAStageCols + (kDecCols / 2) * h;
#pragma unroll
        for (int half2 = 0; half2 < kDecSt; ++half2) {
          uint32_t w[32];
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int c = (kDecCols / 32) * h + 2 * half2 + cc;  // 16-byte chunk of the row (32 columns)
            const uint4 qv = *reinterpret_cast<const uint4*>(tile + ((c ^ (r & 7)) << 4));
            const uint32_t words[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              uint32_t f[4];
              e2m1x8_to_f16x2(words[wi], f);
              const uint32_t sv = bc[(2 * half2 + cc) * 2 + (wi >> 1)];
#pragma unroll
              for (int i = 0; i < 4; ++i) w[16 * cc + 4 * wi + i] = hmul2(f[i], sv);
            }
          }
          tmem_st32(acol + 32 * half2, w);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[as]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[sbi]);  // this warp is done with the unit's scales
      if (!ok) break;
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int r = 32 * q + lane;
    int nu = 0;
    for (int u = u0; u < u1 && !*dead; ++u, ++nu) {
      const Unit un = unit_of(a, u);
      const int d = nu & 1;
      // one decision for the four epilogue warps (they share named barriers)
      const bool w_ok = wait_or_dead(&dfull[d], (nu >> 1) & 1, dead);
      if (named_bar_or(2, 128, !w_ok)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // the kDAcc chains of buffer d, added ((c0 + c1) + (c2 + c3))
      float y[16];
      {
        uint32_t v[kDAcc][16];
#pragma unroll
        for (int c = 0; c < kDAcc; ++c)
          tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + kDCol + (d * kDAcc + c) * kN, v[c]);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 16; ++j)
          y[j] = (__uint_as_float(v[0][j]) + __uint_as_float(v[1][j])) +
                 (__uint_as_float(v[2][j]) + __uint_as_float(v[3][j]));
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[d]);  // the accumulator may be rewritten
      const int n = unit_n(a, un), off = unit_off(a, un);
      const int row = un.tile * kM + r;
      const bool row_ok = row < a.rows;
      const float g = a.mode == kSingle ? a.g : __ldg(&a.globals[unit_expert(a, un) * 2 + a.gsel]);
      if (a.splits > 1) {
        // partial of this split; the last split of the unit adds them in split order
        const int ct = un.chunk * a.tiles + un.tile;
        if (row_ok) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < n) a.part[((size_t)un.split * a.part_cols + off + j) * a.rows + row] = y[j];
        }
        named_bar_sync(2, 128);
        if (warp == kEpiWarp0 && lane == 0) {
          __threadfence();
          *s_last = atomicAdd(&a.ucnt[ct], 1u) == (unsigned)(a.splits - 1);
        }
        named_bar_sync(2, 128);
        const int last = *s_last;
        named_bar_sync(2, 128);  // s_last is rewritten by the next unit
        if (!last) continue;
        __threadfence();
        if (row_ok) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (j >= n) continue;
            const float* pp = a.part + ((size_t)off + j) * a.rows + row;
            float t = __ldcg(pp);
            for (int sp = 1; sp < a.splits; ++sp) t += __ldcg(pp + (size_t)sp * a.part_cols * a.rows);
            y[j] = t;
          }
        }
        if (warp == kEpiWarp0 && lane == 0) a.ucnt[ct] = 0u;
      }
      if (a.mode == kUp) {
        if (un.tile == a.tiles - 1) {
          // K indices of the down panels past the last tile's rows: zero, so
          // that the down launch multiplies its zero-filled codes by zeros
          const int kend = a.swiglu ? a.tiles * (kM / 2) : a.tiles * kM;
          for (int k = kend + r; k < a.out_kb * kKB; k += kM)
#pragma unroll
            for (int j = 0; j < 16; ++j) panel_put(a.panel_out, a.out_kb, un.chunk, j, k, __float2half_rn(0.0f));
        }
        if (a.swiglu) {
          // rows 2i (gate) and 2i + 1 (up) are adjacent lanes
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float gate = y[j] * g;
            const float upv = __shfl_down_sync(0xffffffffu, y[j] * g, 1);
            if ((lane & 1) == 0 && row < a.out_rows * 2) {
              const float act = (j < n && row_ok) ? silu(gate) * upv : 0.0f;
              panel_put(a.panel_out, a.out_kb, un.chunk, j, row >> 1, __float2half_rn(act));
            }
          }
        } else if (row < a.out_kb * kKB) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float act = 0.0f;
            if (j < n && row_ok) {
              const float t = fmaxf(y[j] * g, 0.0f);
              act = a.relu2 ? t * t : y[j] * g;
            }
            panel_put(a.panel_out, a.out_kb, un.chunk, j, row, __float2half_rn(act));
          }
        }
      } else if (row_ok) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < n) a.out[((size_t)off + j) * a.rows + row] = y[j] * g;
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Activation panels: panel[c][kb] = the f16 tile of columns kb*256 .. +255 of
// chunk c's (up to 16) activation rows, in the MMA's K-major core-matrix
// layout (core matrix (token group g, 8-column group kc) at g*4096 +
// kc*128, token rows 16 bytes apart); rows past the chunk and columns past
// `cols` are zero.  Source row of column j: src[idx[off + j]] (idx NULL:
// off + j).  Grid (nkb, max_chunks).
__global__ void __launch_bounds__(256) pack_panel_kernel(const float* __restrict__ src, int cols,
                                                         const int* __restrict__ idx,
                                                         const int* chunk_off, const int* chunk_n,
                                                         const int* n_chunks, int n_single,
                                                         uint8_t* __restrict__ panel, int nkb) {
  const int kb = blockIdx.x, c = blockIdx.y;
  if (n_chunks && c >= __ldg(n_chunks)) return;
  const int n = chunk_n ? __ldg(&chunk_n[c]) : n_single;
  const int off = chunk_off ? __ldg(&chunk_off[c]) : 0;
  uint8_t* t = panel + ((size_t)c * nkb + kb) * kBTile;
  // thread: token j = tid >> 4, 16 consecutive columns 16 * (tid & 15)
  const int j = threadIdx.x >> 4, k0 = 16 * (threadIdx.x & 15);
  uint32_t hw[8];
  const int col0 = kb * kKB + k0;
  if (j < n && col0 < cols) {
    const size_t row = idx ? (size_t)__ldg(&idx[off + j]) : (size_t)(off + j);
    const float* p = src + row * cols + col0;
    float v[16];
    if (col0 + 16 <= cols) {  // cols % 32 == 0: 64-byte aligned
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 f = __ldcg(reinterpret_cast<const float4*>(p) + i);
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = col0 + i < cols ? __ldcg(p + i) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __half2 hv = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      hw[i] = *reinterpret_cast<const uint32_t*>(&hv);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) hw[i] = 0u;
  }
  // two 16-byte rows of two core matrices (8 columns each)
  uint8_t* base = t + (j >> 3) * 4096 + (j & 7) * 16;
  *reinterpret_cast<uint4*>(base + (k0 >> 3) * 128) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  *reinterpret_cast<uint4*>(base + ((k0 >> 3) + 1) * 128) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
}

// ------------------------------------------------------------------- host

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Codes viewed as [R rows][cols/2 bytes]: box 128 rows x 128 bytes, 128-byte
// swizzle, zero fill past the edges.
int code_map(CUtensorMap& m, const uint8_t* codes, int R, int cols) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return kErrLaunch;
  const cuuint64_t dims[2] = {(cuuint64_t)(cols / 2), (cuuint64_t)R};
  const cuuint64_t strides[1] = {(cuuint64_t)(cols / 2)};
  const cuuint32_t box[2] = {kKB / 2, kM};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(codes), dims, strides,
                         box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrArg;
}

int launch_mma(const CUtensorMap& map, const MmaArgs& a, int units, cudaStream_t stream) {
  if (cudaFuncSetAttribute(nvfp4_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
      cudaSuccess)
    return kErrLaunch;
  int grid = device_sm_count();
  if (grid > units) grid = units;
  if (grid < 1) grid = 1;
  nvfp4_mma_kernel<<<grid, kMmaThreads, kSmem, stream>>>(map, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

size_t mma_panel_bytes(int chunks, int cols) {
  return (size_t)chunks * ((cols + kKB - 1) / kKB) * kBTile;
}

int launch_pack_panel(const float* src, int cols, const int* idx, const int* chunk_off, const int* chunk_n,
                      const int* n_chunks, int max_chunks, int n_single, uint8_t* panel,
                      cudaStream_t stream) {
  const int nkb = (cols + kKB - 1) / kKB;
  pack_panel_kernel<<<dim3(nkb, max_chunks), 256, 0, stream>>>(src, cols, idx, chunk_off, chunk_n, n_chunks,
                                                              n_single, panel, nkb);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_nvfp4_mma_single(const uint8_t* codes, const uint8_t* scales, float g, const uint8_t* panel,
                            float* out, int rows, int cols, int n, float* part, unsigned* ucnt,
                            int max_splits, cudaStream_t stream) {
  CUtensorMap map;
  if (int e = code_map(map, codes, rows, cols)) return e;
  MmaArgs a{};
  a.scales = scales;
  a.rows = rows;
  a.cols = cols;
  a.R = rows;
  a.mode = kSingle;
  a.g = g;
  a.panel = panel;
  a.n = n;
  a.max_chunks = 1;
  a.tiles = (rows + kM - 1) / kM;
  a.nkb = (cols + kKB - 1) / kKB;
  // split K when the row tiles alone leave SMs idle (deterministic partials)
  int splits = 1;
  const int sms = device_sm_count();
  if (part && ucnt) {
    while (splits < max_splits && a.tiles * splits * 2 <= sms && splits * 2 <= a.nkb) splits *= 2;
  }
  a.splits = splits;
  a.part = part;
  a.ucnt = ucnt;
  a.part_cols = n;
  a.out = out;
  return launch_mma(map, a, a.tiles * splits, stream);
}

int launch_nvfp4_mma_grouped(const MmaGrouped& gp, cudaStream_t stream) {
  CUtensorMap map;
  if (int e = code_map(map, gp.codes, gp.n_experts * gp.rows, gp.cols)) return e;
  MmaArgs a{};
  a.scales = gp.scales;
  a.rows = gp.rows;
  a.cols = gp.cols;
  a.R = gp.n_experts * gp.rows;
  a.mode = gp.down ? kDown : kUp;
  a.globals = gp.globals;
  a.gsel = gp.gsel;
  a.panel = gp.panel;
  a.chunk_expert = gp.chunk_expert;
  a.chunk_off = gp.chunk_off;
  a.chunk_n = gp.chunk_n;
  a.n_chunks = gp.n_chunks;
  a.max_chunks = gp.max_chunks;
  a.tiles = (gp.rows + kM - 1) / kM;
  a.nkb = (gp.cols + kKB - 1) / kKB;
  a.splits = gp.ksplit > 1 ? gp.ksplit : 1;
  if (a.splits > a.nkb) a.splits = a.nkb;  // every split holds at least one k-block
  a.part = gp.part;
  a.ucnt = gp.ucnt;
  a.part_cols = gp.max_pairs;
  a.out = gp.out;
  a.panel_out = gp.panel_out;
  a.relu2 = gp.relu2;
  a.swiglu = gp.swiglu;
  a.out_rows = gp.swiglu ? gp.rows / 2 : gp.rows;
  a.out_kb = (a.out_rows + kKB - 1) / kKB;
  if (a.splits > 1 && (!a.part || !a.ucnt)) return kErrArg;
  const int units = gp.max_chunks * a.tiles * a.splits;
  return launch_mma(map, a, units, stream);
}

int read_mma_device_error(bool clear) { return read_unit_error(clear); }

}  // namespace ervf
