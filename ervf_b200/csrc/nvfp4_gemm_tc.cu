// nvfp4_gemm_tc.cu -- batched NVFP4 GEMM on the sm_100a tensor cores
// (tcgen05.mma, accumulator in tensor memory):
//
//   out[n][r] = g * sum_k (e2m1[r][k] * e4m3[r][k/16]) * X[n][k],  n < N <= 16
//
// for decode batches of up to 16 tokens on one NVFP4 matrix (the batched
// variant of the expert / head GEMV; the reference's batched path is the
// SIMT gemm_nvfp4_rows_b, sweepspec.py:28-240).  Held to a tolerance (rel-L2
// <= 1e-3 against an FP32 dequantise-then-matmul), not to the bit-exact
// chain order of the batch-1 kernels.
//
// Exactness of the operands: e2m1 (2 significant bits) times an E4M3 scale
// (4 bits, 2^-9 .. 448) is a 6-bit product in 2^-10 .. 2688, exact in f16;
// X is rounded to f16 (exact for bf16 activations inside f16's range).  The
// global scale g is applied to the fp32 accumulator in the epilogue.
//
// CTA = 8 warps, up to four CTAs per SM; work unit = 128 weight rows x one
// K-split.  Per k-block of 64 columns, thread (warp w, lane l) owns weight row
// 32*(w % 4) + l -- its TMEM lane -- and code unit w / 4 of the k-block: the
// unit arrives by cp.async in an 8-deep per-thread ring (the thread that
// copies a unit decodes it), its scale bytes in a register ring of the same
// depth.  The decode (hardware e2m1x2 / e4m3x2 converters, one f16x2 multiply
// per two weights) writes the row's 32 f16 straight into tensor memory with
// tcgen05.st (row = lane, two f16 per 32-bit column in K order): the A operand
// never touches shared memory.  X (rounded to f16) goes to a shared B tile in
// the canonical K-major core-matrix layout.  One thread issues four
// tcgen05.mma.kind::f16 (A from tensor memory, M=128, N=16, K=16, f32
// accumulate) per k-block and commits them to the stage's mbarrier; two A / B
// stages let the decode of k-block i+1 overlap the MMAs of k-block i.  The
// epilogue reads the accumulator with tcgen05.ld (warp w: TMEM lanes
// 32w..32w+31 = rows), scales by g and stores (or, with a K-split, adds
// atomically into the zeroed output).
#include "common.cuh"
#include "kernels.h"

namespace ervf {

namespace {

constexpr int kTcThreads = 256;
constexpr int kTcM = 128;            // rows per work unit (UMMA M)
constexpr int kTcN = 16;             // batch columns (UMMA N)
constexpr int kTcKB = 64;            // columns per k-block (4 MMAs of K = 16)
constexpr int kTcBSBO = kTcKB / 8 * 128;                // B: bytes between 8-row core groups
constexpr int kTcBStage = kTcN * kTcKB * 2;             // 2 KB
constexpr int kTcRawDepth = 8;                          // k-blocks of codes in flight
constexpr int kTcRawStage = kTcM * (kTcKB / 2);         // 4 KB of code bytes
constexpr int kTcSmem = 1024 + 2 * kTcBStage + kTcRawDepth * kTcRawStage;
// BF16 weights (dense projections): 64 B of one row per thread and k-block
constexpr int kTcRawDepthBf = 4;
constexpr int kTcRawStageBf = kTcM * kTcKB * 2;         // 16 KB
constexpr int kTcSmemBf = 1024 + 2 * kTcBStage + kTcRawDepthBf * kTcRawStageBf;

enum TcMode { kTcNvfp4 = 0, kTcBf16 = 1, kTcGrouped = 2 };
constexpr int kTcTmemCols = 128;     // D: columns 0..15; A stages: 32..63, 64..95
constexpr int kTcACol = 32;
constexpr int kTcAStageCols = kTcKB / 2;  // two f16 per 32-bit column

struct TcArgs {
  const uint8_t* codes;   // [rows][cols/2]; kTcBf16: bf16 weights [rows][cols]
  const uint8_t* scales;  // [rows][cols/16]
  float g;
  const float* x;         // [n][cols]
  float* out;             // [n][rows]
  int rows, cols, n;
  int splits;             // K-splits per row tile (atomic accumulation when > 1)
  int units;              // row tiles * splits
  // kTcGrouped (expert-major batched MoE): unit = (chunk, row tile); chunk c
  // is expert chunk_expert[c] with the n = chunk_n[c] <= 16 route pairs
  // chunk_off[c] .. +n of the expert-sorted pair list.  B column j gathers X
  // row b_idx[chunk_off + j] (b_idx NULL: row chunk_off + j); output row of
  // pair p is out[p * rows + r].  Weights: codes + e*code_stride, global scale
  // globals[e*2 + gsel]; relu2 squares the positive part.
  const int* chunk_expert;
  const int* chunk_off;
  const int* chunk_n;
  const int* n_chunks;
  const int* b_idx;
  size_t code_stride, scale_stride;
  const float* globals;
  int gsel, relu2, tiles;
  // kTcGrouped K-split: unit = ((chunk, tile), split); each split writes its
  // fp32 accumulator to part[split][pair][row]; the last of a unit's splits
  // (counter ucnt[chunk * tiles + tile], left zero) adds them in split order,
  // scales and stores -- deterministic, the same bits whatever the arrival
  // order or the grid.
  int ksplit, max_pairs;
  float* part;
  unsigned* ucnt;
};

// UMMA shared-memory descriptor, K-major, no swizzle (sm100 version 1).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// kind::f16 instruction descriptor: D f32, A / B f16 (or bf16), K-major, N, M.
constexpr uint32_t kTcIdesc = (1u << 4) | ((uint32_t)(kTcN >> 3) << 17) | ((uint32_t)(kTcM >> 4) << 24);
constexpr uint32_t kTcIdescBf = kTcIdesc | (1u << 7) | (1u << 10);

__device__ __forceinline__ uint32_t f32x2_to_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Two E4M3 scale bytes as f16x2 broadcasts of the first (low) byte and of the
// second; NaN bytes (0x7F, 0xFF) read as +0 (the reference's table).
__device__ __forceinline__ void scales_f16(uint32_t sv, uint32_t& s0, uint32_t& s1) {
  const uint32_t b0 = sv & 0xFFu, b1 = (sv >> 8) & 0xFFu;
  const uint32_t c0 = (b0 & 0x7Fu) == 0x7Fu ? 0u : b0;
  const uint32_t c1 = (b1 & 0x7Fu) == 0x7Fu ? 0u : b1;
  const uint16_t pair0 = (uint16_t)(c0 | (c0 << 8)), pair1 = (uint16_t)(c1 | (c1 << 8));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(s0) : "h"(pair0));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(s1) : "h"(pair1));
}

// 32 weights of one code unit as 16 f16x2 words in column order.
__device__ __forceinline__ void decode_unit(uint4 q, uint32_t sv, uint32_t (&w)[16]) {
  uint32_t s0, s1;
  scales_f16(sv, s0, s1);
  const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t h[4];
    e2m1x8_to_f16x2(words[j], h);
    const uint32_t s = j < 2 ? s0 : s1;
#pragma unroll
    for (int i = 0; i < 4; ++i) w[4 * j + i] = hmul2(h[i], s);
  }
}

__device__ __forceinline__ uint32_t f32x2_to_f16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// 16-byte asynchronous global -> shared copy; src_bytes = 0 writes zeros.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait(bar, parity, 2000000000LL);
}

template <int MODE>
__global__ void __launch_bounds__(kTcThreads) nvfp4_gemm_tc_kernel(TcArgs a) {
  constexpr int kDepth = MODE == kTcBf16 ? kTcRawDepthBf : kTcRawDepth;
  constexpr int kRawStage = MODE == kTcBf16 ? kTcRawStageBf : kTcRawStage;
  constexpr int kUnitBytes = MODE == kTcBf16 ? 64 : 16;  // per thread and k-block
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* mb = reinterpret_cast<uint64_t*>(smem);  // [0,1]: stage done, [2]: accumulator done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 64);
  uint8_t* bst0 = smem + 1024;                       // two B stages
  uint8_t* raw0 = bst0 + 2 * kTcBStage;              // [depth][128 rows][2 x unit bytes]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cb = a.cols >> 1, sb = a.cols >> 4, n_u = a.cols >> 5;
  const int nkb = (a.cols + kTcKB - 1) / kTcKB;

  if (tid == 0) {
    mbar_init(&mb[0], 1);
    mbar_init(&mb[1], 1);
    mbar_init(&mb[2], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(kTcTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // decode role: row rr = TMEM lane of this warp's quarter, code unit
  // 2*kb + half (the k-block's columns 32*half .. 32*half + 31)
  const int rr = 32 * (warp & 3) + lane, half = warp >> 2;
  const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
  // B role (threads < 128): batch row bn, 8-column chunk bc of the k-block
  const int bn = tid >> 3, bc = tid & 7;
  __shared__ int s_last;
  bool dead = false;
  uint32_t gkb = 0;   // k-blocks issued by this CTA (stage ring position)
  uint32_t nacc = 0;  // accumulator commits waited for

  for (int unit = blockIdx.x; unit < a.units; unit += gridDim.x) {
    int tile, split, un, uoff = 0;
    const uint8_t* ucodes = a.codes;
    const uint8_t* uscales = a.scales;
    float ug = a.g;
    int us = 0;  // grouped: the unit without its split
    if constexpr (MODE == kTcGrouped) {
      us = unit / a.ksplit;
      split = unit - us * a.ksplit;
      const int chunk = us / a.tiles;
      if (chunk >= __ldg(a.n_chunks)) continue;  // uniform over the CTA
      tile = us - chunk * a.tiles;
      const int e = __ldg(&a.chunk_expert[chunk]);
      un = __ldg(&a.chunk_n[chunk]);
      uoff = __ldg(&a.chunk_off[chunk]);
      ucodes = a.codes + (size_t)e * a.code_stride;
      uscales = a.scales + (size_t)e * a.scale_stride;
      ug = __ldg(&a.globals[e * 2 + a.gsel]);
    } else {
      tile = unit / a.splits;
      split = unit - tile * a.splits;
      un = a.n;
    }
    const int nsplit = MODE == kTcGrouped ? a.ksplit : a.splits;
    const int kb0 = (int)((long long)split * nkb / nsplit);
    const int kb1 = (int)((long long)(split + 1) * nkb / nsplit);
    const int row = tile * kTcM + rr;
    const bool row_ok = row < a.rows;
    const uint8_t* crow = ucodes + (size_t)row * cb;
    const uint8_t* srow = uscales + (size_t)row * sb;

    // This thread's code unit of k-block kb goes, by cp.async, to raw ring
    // slot kb % depth (the thread that copies a unit decodes it: no barrier);
    // its two scale bytes go to a register ring of the same depth.
    uint8_t* my_raw = raw0 + rr * (2 * kUnitBytes) + kUnitBytes * half;
    const uint8_t* wrow = a.codes + (size_t)row * a.cols * 2;  // kTcBf16
    auto copy_unit = [&](int kb) {
      const int u = 2 * kb + half;
      const bool ok = row_ok && u < n_u;
      uint8_t* dst = my_raw + (kb % kDepth) * kRawStage;
      if constexpr (MODE == kTcBf16) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          cp_async16(dst + 16 * i, ok ? wrow + 64 * u + 16 * i : a.codes, ok ? 16u : 0u);
      } else {
        cp_async16(dst, ok ? crow + 16 * u : a.codes, ok ? 16u : 0u);
      }
    };
    auto scale_of = [&](int kb) -> uint32_t {
      if constexpr (MODE == kTcBf16) return 0u;
      const int u = 2 * kb + half;
      return (row_ok && u < n_u) ? (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(srow + 2 * u)) : 0u;
    };
    uint32_t svr[kDepth];
#pragma unroll
    for (int d = 0; d < kDepth - 1; ++d) {
      if (kb0 + d < kb1) {
        copy_unit(kb0 + d);
        svr[d] = scale_of(kb0 + d);
      }
      cp_async_commit();
    }
    // B role, per unit: this thread's activation row (gathered once per unit
    // in the grouped mode) and its 16-byte slot of the B tile
    const int xn = MODE == kTcBf16 ? (bn & 7) : bn;  // kTcBf16: rows n and n + 8 share X[n]
    const bool x_row = tid < 128 && xn < un;
    const float* xrow = a.x;
    if (x_row) {
      size_t src = (size_t)xn;
      if constexpr (MODE == kTcGrouped)
        src = a.b_idx ? (size_t)__ldg(&a.b_idx[uoff + xn]) : (size_t)(uoff + xn);
      xrow = a.x + src * a.cols + bc * 8;
    }
    const uint32_t b_slot = (uint32_t)((bn >> 3) * kTcBSBO + bc * 128 + (bn & 7) * 16);
    auto load_x = [&](int kb, float4 (&v)[2]) {
      if (x_row && kb * kTcKB + bc * 8 < a.cols) {
        // activations may come from the previous launch: read through L2
        const float* p = xrow + kb * kTcKB;
        v[0] = __ldcg(reinterpret_cast<const float4*>(p));
        v[1] = __ldcg(reinterpret_cast<const float4*>(p + 4));
      } else {
        v[0] = v[1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    };
    float4 xv[2];
    load_x(kb0, xv);

    for (int kb = kb0; kb < kb1; ++kb, ++gkb) {
      const int s = (int)(gkb & 1u);
      // the MMAs that last read this stage (two k-blocks ago) are complete
      if (gkb >= 2 && !dead) dead = !tc_wait(&mb[s], ((gkb >> 1) - 1) & 1u);
      const int slot = (kb - kb0) % kDepth;
      {
        const int ahead = kb + kDepth - 1;
        if (ahead < kb1) {
          copy_unit(ahead);
          const int idx = (ahead - kb0) % kDepth;
#pragma unroll
          for (int d = 0; d < kDepth; ++d)  // static slots keep the ring in registers
            if (d == idx) svr[d] = scale_of(ahead);
        }
        cp_async_commit();
      }
      cp_async_wait<kDepth - 1>();  // this k-block's unit has landed
      const uint8_t* mine = my_raw + (kb % kDepth) * kRawStage;
      uint32_t w[16];
      if constexpr (MODE == kTcBf16) {
        // bf16 pairs are already the 32-bit column layout (K order, low first)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 v = *reinterpret_cast<const uint4*>(mine + 16 * i);
          w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
      } else {
        uint32_t sv = 0;
#pragma unroll
        for (int d = 0; d < kDepth; ++d)
          if (d == slot) sv = svr[d];
        decode_unit(*reinterpret_cast<const uint4*>(mine), sv, w);
      }
      // A: this row's 32 columns of the k-block into tensor memory
      tmem_st16(lane_base + kTcACol + s * kTcAStageCols + 16 * half, w);
      // B: X rows as f16 (loaded one k-block ahead), zero beyond batch / cols;
      // kTcBf16: rows 0..7 the bf16 rounding of X, rows 8..15 its remainder
      if (tid < 128) {
        uint8_t* sbuf = bst0 + s * kTcBStage;
        uint4 v;
        if constexpr (MODE == kTcBf16) {
          const float e[8] = {xv[0].x, xv[0].y, xv[0].z, xv[0].w, xv[1].x, xv[1].y, xv[1].z, xv[1].w};
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            hw[i] = f32x2_to_bf16x2(e[2 * i], e[2 * i + 1]);
            lw[i] = f32x2_to_bf16x2(e[2 * i] - bf16_lo(hw[i]), e[2 * i + 1] - bf16_hi(hw[i]));
          }
          v = bn < 8 ? make_uint4(hw[0], hw[1], hw[2], hw[3]) : make_uint4(lw[0], lw[1], lw[2], lw[3]);
        } else {
          v = make_uint4(f32x2_to_f16x2(xv[0].x, xv[0].y), f32x2_to_f16x2(xv[0].z, xv[0].w),
                         f32x2_to_f16x2(xv[1].x, xv[1].y), f32x2_to_f16x2(xv[1].z, xv[1].w));
        }
        *reinterpret_cast<uint4*>(sbuf + b_slot) = v;
      }
      if (kb + 1 < kb1) load_x(kb + 1, xv);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncthreads();
      if (tid == 0 && !dead) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t b0 = smem_u32(bst0 + s * kTcBStage);
#pragma unroll
        for (int j = 0; j < kTcKB / 16; ++j) {
          const uint64_t db = umma_desc(b0 + 256 * j, 128, kTcBSBO);
          const uint32_t accum = (kb > kb0 || j > 0) ? 1u : 0u;
          asm volatile(
              "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
              " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
              ::"r"(tmem), "r"(tmem + kTcACol + s * kTcAStageCols + 8 * j), "l"(db),
                "r"(MODE == kTcBf16 ? kTcIdescBf : kTcIdesc), "r"(accum) : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&mb[s])) : "memory");
        if (kb + 1 == kb1)
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                       ::"r"(smem_u32(&mb[2])) : "memory");
      }
    }
    // epilogue: accumulator -> out
    if (!dead) dead = !tc_wait(&mb[2], nacc & 1u);
    ++nacc;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp < 4) {
      uint32_t v[16];
      const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
            "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
            "=r"(v[14]), "=r"(v[15])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      const int orow = tile * kTcM + warp * 32 + lane;
      if (!dead && orow < a.rows) {
#pragma unroll
        for (int j = 0; j < kTcN; ++j) {
          if (MODE == kTcGrouped && a.ksplit > 1) {
            if (j < un)
              a.part[((size_t)split * a.max_pairs + uoff + j) * a.rows + orow] = __uint_as_float(v[j]);
            continue;
          }
          if (j < un) {
            float y = MODE == kTcBf16 ? (j < 8 ? __uint_as_float(v[j]) + __uint_as_float(v[j + 8]) : 0.0f)
                                      : __uint_as_float(v[j]) * ug;
            if (MODE == kTcGrouped && a.relu2) {
              const float r = fmaxf(y, 0.0f);
              y = r * r;
            }
            float* o = a.out + (size_t)(uoff + j) * a.rows + orow;
            if (a.splits > 1) {
              atomicAdd(o, y);
            } else {
              *o = y;
            }
          }
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();  // the accumulator is read before the next unit's MMAs
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if constexpr (MODE == kTcGrouped) {
      if (a.ksplit > 1) {
        // the last split of this unit adds the partial accumulators in split
        // order, applies the global scale (and relu^2) and stores
        if (tid == 0) {
          __threadfence();
          s_last = atomicAdd(&a.ucnt[us], 1u) == (unsigned)(a.ksplit - 1);
        }
        __syncthreads();
        if (s_last) {
          __threadfence();
          const int orow = tile * kTcM + tid;
          if (tid < kTcM && !dead && orow < a.rows) {
            for (int j = 0; j < un; ++j) {
              const float* pp = a.part + (size_t)(uoff + j) * a.rows + orow;
              float t = __ldcg(pp);
              for (int sp = 1; sp < a.ksplit; ++sp) t += __ldcg(pp + (size_t)sp * a.max_pairs * a.rows);
              float y = t * ug;
              if (a.relu2) {
                const float r = fmaxf(y, 0.0f);
                y = r * r;
              }
              a.out[(size_t)(uoff + j) * a.rows + orow] = y;
            }
          }
          if (tid == 0) a.ucnt[us] = 0u;
        }
        __syncthreads();  // s_last is rewritten for the next unit
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
}

}  // namespace

namespace {

template <int MODE>
int launch_tc(const uint8_t* w, const uint8_t* scales, float g, const float* x, float* out, int rows,
              int cols, int n, cudaStream_t stream) {
  constexpr int smem = MODE == kTcBf16 ? kTcSmemBf : kTcSmem;
  auto kern = nvfp4_gemm_tc_kernel<MODE>;
  const int sms = device_sm_count();
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return kErrLaunch;
  // CTAs per SM from the shared-memory footprint and the 512 tensor-memory
  // columns of an SM
  int smem_sm = 0;
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, 0);
  int per_sm = smem_sm / (smem + 1024);
  if (per_sm > 512 / kTcTmemCols) per_sm = 512 / kTcTmemCols;
  if (per_sm < 1) return kErrShape;
  TcArgs a{};
  a.codes = w;
  a.scales = scales;
  a.g = g;
  a.x = x;
  a.out = out;
  a.rows = rows;
  a.cols = cols;
  a.n = n;
  const int tiles = (rows + kTcM - 1) / kTcM;
  const int nkb = (cols + kTcKB - 1) / kTcKB;
  const int slots = sms * per_sm;
  int splits = (slots + tiles - 1) / tiles;
  if (splits > nkb) splits = nkb;
  if (splits < 1) splits = 1;
  a.splits = splits;
  a.units = tiles * splits;
  if (splits > 1 && cudaMemsetAsync(out, 0, (size_t)n * rows * sizeof(float), stream) != cudaSuccess)
    return kErrLaunch;
  const int grid = a.units < slots ? a.units : slots;
  kern<<<grid, kTcThreads, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

int launch_nvfp4_gemm_tc(const uint8_t* codes, const uint8_t* scales, float g, const float* x,
                         float* out, int rows, int cols, int n, cudaStream_t stream) {
  if (n < 1 || n > kTcN) return kErrShape;
  return launch_tc<kTcNvfp4>(codes, scales, g, x, out, rows, cols, n, stream);
}

int launch_grouped_tc(const GroupedTc& g, cudaStream_t stream) {
  constexpr int smem = kTcSmem;
  auto kern = nvfp4_gemm_tc_kernel<kTcGrouped>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return kErrLaunch;
  int smem_sm = 0;
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, 0);
  int per_sm = smem_sm / (smem + 1024);
  if (per_sm > 512 / kTcTmemCols) per_sm = 512 / kTcTmemCols;
  if (per_sm < 1) return kErrShape;
  TcArgs a{};
  a.codes = g.codes;
  a.scales = g.scales;
  a.x = g.x;
  a.out = g.out;
  a.rows = g.rows;
  a.cols = g.cols;
  a.n = 16;
  a.splits = 1;
  a.tiles = (g.rows + kTcM - 1) / kTcM;
  a.ksplit = g.ksplit > 1 ? g.ksplit : 1;
  a.max_pairs = g.max_chunks;
  a.part = g.part;
  a.ucnt = g.ucnt;
  if (a.ksplit > 1 && (!a.part || !a.ucnt)) return kErrArg;
  a.units = g.max_chunks * a.tiles * a.ksplit;
  a.chunk_expert = g.chunk_expert;
  a.chunk_off = g.chunk_off;
  a.chunk_n = g.chunk_n;
  a.n_chunks = g.n_chunks;
  a.b_idx = g.b_idx;
  a.code_stride = g.code_stride;
  a.scale_stride = g.scale_stride;
  a.globals = g.globals;
  a.gsel = g.gsel;
  a.relu2 = g.relu2;
  const int slots = device_sm_count() * per_sm;
  const int grid = a.units < slots ? a.units : slots;
  kern<<<grid, kTcThreads, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_bf16_gemm_tc(const uint16_t* W, const float* x, float* out, int rows, int cols, int n,
                        cudaStream_t stream) {
  if (n < 1 || n > 8) return kErrShape;
  return launch_tc<kTcBf16>(reinterpret_cast<const uint8_t*>(W), nullptr, 1.0f, x, out, rows, cols, n,
                            stream);
}

int read_tc_device_error(bool clear) { return read_unit_error(clear); }

}  // namespace ervf
