// bf16_gemm_tc.cu -- batched BF16 GEMM on the sm_100a tensor cores for the
// dense projections (tcgen05.mma, A from shared memory, accumulators in
// tensor memory):
//
//   out[n][r] = sum_k W[r][k] * X[n][k],  n < N <= 8,  W bf16, X fp32
//
// The reference has no batched BF16 kernel (its gemv_bf16, gpu_kernels.py:
// 21-49, runs one activation row at a time; ervf_bf16_gemv keeps that chain
// order).  Here X is split into its bf16 rounding (MMA columns 0..7) and the
// bf16 rounding of the remainder (columns 8..15); the epilogue adds the two
// fp32 accumulators, which holds the result to rel-L2 <= 1e-3 (~1e-5
// measured) against an fp32 matmul.
//
// Warp-specialised, one CTA per SM, persistent over (128-row tile, K range)
// units; per k-block of 64 columns a ring stage holds the 128 x 64 bf16
// weight tile (16 KB, 2-D TMA load with 128-byte swizzle -- the weights go
// from global memory to the MMA without touching a register) and the
// 16 x 64 bf16 activation tile (2 KB, K-major core matrices):
//   warp 0, lane 0     producer: TMA of the weight tile into ring stage s.
//                      This GPU's own memory only; no multicast anywhere.
//   warps 1..4, lane 0 MMA.  Issuer j issues the k-block's MMA j
//                      (tcgen05.mma.cta_group::1.kind::f16, bf16 A / B,
//                      M128 N16 K16, f32 accumulate) into its own chain j of
//                      accumulator buffer d and commits it to the barriers
//                      that free stage s and, after the unit's last k-block,
//                      fill buffer d.  An MMA takes its issuing thread ~95
//                      cycles whatever N is; issuers in different warps
//                      overlap.
//   warps 5..8         activation tile of stage s: X rows split into their
//                      bf16 high and low halves, written in the MMA's
//                      K-major core-matrix layout.
//   warps 9..12        epilogue: tcgen05.ld of the four chains of buffer d
//                      (warp w: tensor-memory lanes 32 (w % 4) ..), added in a
//                      fixed order, high + low, then the store, and frees d.
// Small matrices split K over several units per row tile so that every SM
// works; the splits then add into the zeroed output with fp32 atomics, so the
// last bits depend on their arrival order (within the tolerance above).
// Every wait is bounded (%clock64); a wait that runs out records
// kErrTimeout, marks the CTA dead, and every role drains: no copy or MMA is
// left in flight when tensor memory is released.
#include <cuda.h>  // CUtensorMap and the encode function's types (driver entry point)

#include "common.cuh"
#include "kernels.h"

namespace ervf {

namespace {

constexpr int kTcM = 128;            // rows per work unit (UMMA M)
constexpr int kTcN = 16;             // MMA columns: X high halves 0..7, low halves 8..15
constexpr int kTcKB = 64;            // columns per k-block (4 MMAs of K = 16; 128 bytes of a row)
constexpr int kTcIssuers = kTcKB / 16;
constexpr int kTcBuilders = 4;       // warps that write the activation tiles
constexpr int kTcWarps = 1 + kTcIssuers + kTcBuilders + 4;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcIssuer0 = 1, kTcBuilder0 = kTcIssuer0 + kTcIssuers, kTcEpi0 = kTcBuilder0 + kTcBuilders;
constexpr int kTcATile = kTcM * kTcKB * 2;   // 16 KB, 1024-aligned (the swizzle repeats every 1024 B)
constexpr int kTcBTile = kTcN * kTcKB * 2;   // 2 KB
constexpr int kTcBSBO = kTcKB / 8 * 128;     // B: bytes between 8-row core-matrix groups
constexpr int kTcStageBytes = (kTcATile + kTcBTile + 1023) / 1024 * 1024;  // 1024-aligned stages
constexpr int kTcStages = 8;
constexpr int kTcRingOff = 1024;
constexpr int kTcSmem = kTcRingOff + kTcStages * kTcStageBytes;
constexpr int kTcTmemCols = 128;     // accumulators: buffer d, chain c at columns (4 d + c) * 16
static_assert(2 * kTcIssuers * kTcN <= kTcTmemCols, "tensor-memory columns");
static_assert(kTcBuilders * 32 == kTcN * kTcKB / 8, "one builder thread per 8-column row chunk");

struct TcArgs {
  const float* x;         // [n][cols]
  float* out;             // [n][rows]
  int rows, cols, n;
  int nkb;                // k-blocks of a row
  int tiles, splits;      // row tiles, K ranges per tile (atomic accumulation when > 1)
  int units;              // tiles * splits
};

// UMMA shared-memory descriptor (sm100 version 1): K-major, start address,
// leading / stride byte offsets, layout (0: no swizzle, 2: 128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)layout << 61);
}

// kind::f16 instruction descriptor: D f32, A / B bf16, K-major, N, M.
constexpr uint32_t kTcIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTcN >> 3) << 17) |
                              ((uint32_t)(kTcM >> 4) << 24);

__device__ __forceinline__ uint32_t f32x2_to_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// Bounded wait that also gives up when another role of the CTA died.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* dead) {
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

// Unit u of the grid -> (row tile, k-block range), split fastest.
__device__ __forceinline__ void unit_k(const TcArgs& a, int u, int& tile, int& kb0, int& kb1) {
  tile = u / a.splits;
  const int split = u - tile * a.splits;
  kb0 = (int)((long long)split * a.nkb / a.splits);
  kb1 = (int)((long long)(split + 1) * a.nkb / a.splits);
}

__global__ void __launch_bounds__(kTcThreads, 1)
    bf16_gemm_tc_kernel(const __grid_constant__ CUtensorMap w_map, TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [kTcStages]
  uint64_t* empty = full + kTcStages;                  // [kTcStages]
  uint64_t* dfull = empty + kTcStages;                 // [2]
  uint64_t* dempty = dfull + 2;                        // [2]
  uint64_t* mma_done = dempty + 2;                     // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 512);
  volatile int* dead = reinterpret_cast<volatile int*>(smem + 516);
  uint8_t* ring = smem + kTcRingOff;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(&full[i], 1 + kTcBuilders);  // the weight tile's bytes + the activation tile's writers
      mbar_init(&empty[i], kTcIssuers);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull[i], kTcIssuers);
      mbar_init(&dempty[i], 4);
    }
    mbar_init(mma_done, kTcIssuers);
    *dead = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(kTcTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const long long G = gridDim.x, b = blockIdx.x;
  const int u0 = (int)((long long)a.units * b / G), u1 = (int)((long long)a.units * (b + 1) / G);

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      uint32_t gk = 0;
      for (int u = u0; u < u1 && !*dead; ++u) {
        int tile, kb0, kb1;
        unit_k(a, u, tile, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++gk) {
          const int s = (int)(gk % kTcStages);
          if (!tc_wait(&empty[s], ((gk / kTcStages) & 1) ^ 1, dead)) break;
          mbar_arrive_expect_tx(&full[s], kTcATile);
          tma_load_2d(ring + s * kTcStageBytes, &w_map, kb * kTcKB, tile * kTcM, &full[s]);
        }
      }
      // leave no tensor copy in flight
      for (uint32_t k = gk > (uint32_t)kTcStages ? gk - kTcStages : 0; k < gk; ++k)
        tc_wait(&full[k % kTcStages], (k / kTcStages) & 1, dead);
    }
  } else if (warp < kTcBuilder0) {
    // ---------------------------------------------------------- MMA issuers
    const int j = warp - kTcIssuer0;  // the k-block's MMA j, accumulator chain j
    if (lane == 0) {
      uint32_t gk = 0;
      int nu = 0;
      for (int u = u0; u < u1 && !*dead; ++u, ++nu) {
        int tile, kb0, kb1;
        unit_k(a, u, tile, kb0, kb1);
        const int d = nu & 1;
        if (!tc_wait(&dempty[d], ((nu >> 1) & 1) ^ 1, dead)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++gk) {
          const int s = (int)(gk % kTcStages);
          if (!tc_wait(&full[s], (gk / kTcStages) & 1, dead)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t st = smem_u32(ring + s * kTcStageBytes);
          // A: the 128 x 64 weight tile, 128-byte swizzle, K-major (8-row
          // groups 1024 bytes apart); MMA j starts 32 bytes into each row
          const uint64_t da = umma_desc(st + 32 * j, 16, 1024, 2);
          const uint64_t db = umma_desc(st + kTcATile + 256 * j, 128, kTcBSBO, 0);
          const uint32_t acc = kb > kb0 ? 1u : 0u;
          asm volatile(
              "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
              " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
              ::"r"(tmem + (uint32_t)((d * kTcIssuers + j) * kTcN)), "l"(da), "l"(db), "r"(kTcIdesc),
                "r"(acc) : "memory");
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&dfull[d]);
      }
      // every MMA issued by this thread is complete before tensor memory is freed
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, 2000000000LL);
    }
  } else if (warp < kTcEpi0) {
    // ---------------------------------------------------------- activation tiles
    // thread: MMA column bn (X row bn & 7, high half below 8, low half from
    // 8), 8-column chunk bc of the k-block
    const int t = tid - kTcBuilder0 * 32, bn = t >> 3, bc = t & 7;
    const int xn = bn & 7;
    const bool x_row = xn < a.n;
    const float* xrow = a.x + (size_t)(x_row ? xn : 0) * a.cols + bc * 8;
    const uint32_t b_slot = (uint32_t)(kTcATile + (bn >> 3) * kTcBSBO + bc * 128 + (bn & 7) * 16);
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
    uint32_t gk = 0;
    for (int u = u0; u < u1 && !*dead; ++u) {
      int tile, kb0, kb1;
      unit_k(a, u, tile, kb0, kb1);
      float4 xv[2];
      load_x(kb0, xv);
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb, ++gk) {
        const int s = (int)(gk % kTcStages);
        const bool w_ok = tc_wait(&empty[s], ((gk / kTcStages) & 1) ^ 1, dead);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        const float e[8] = {xv[0].x, xv[0].y, xv[0].z, xv[0].w, xv[1].x, xv[1].y, xv[1].z, xv[1].w};
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          hw[i] = f32x2_to_bf16x2(e[2 * i], e[2 * i + 1]);
          lw[i] = f32x2_to_bf16x2(e[2 * i] - bf16_lo(hw[i]), e[2 * i + 1] - bf16_hi(hw[i]));
        }
        *reinterpret_cast<uint4*>(ring + s * kTcStageBytes + b_slot) =
            bn < 8 ? make_uint4(hw[0], hw[1], hw[2], hw[3]) : make_uint4(lw[0], lw[1], lw[2], lw[3]);
        if (kb + 1 < kb1) load_x(kb + 1, xv);  // the next k-block's activations in flight
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // seen by the MMA
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
      }
      if (!ok) break;
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int q = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    int nu = 0;
    for (int u = u0; u < u1 && !*dead; ++u, ++nu) {
      int tile, kb0, kb1;
      unit_k(a, u, tile, kb0, kb1);
      const int d = nu & 1;
      const bool w_ok = tc_wait(&dfull[d], (nu >> 1) & 1, dead);
      if (!__all_sync(0xffffffffu, w_ok)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t v[kTcIssuers][16];
#pragma unroll
      for (int c = 0; c < kTcIssuers; ++c) tmem_ld16(lane_base + (uint32_t)((d * kTcIssuers + c) * kTcN), v[c]);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[d]);  // the accumulators are read: buffer d is free
      const int orow = tile * kTcM + 32 * q + lane;
      if (orow < a.rows) {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          if (jj < a.n) {
            const auto f = [&](int c, int k) { return __uint_as_float(v[c][k]); };
            const float hi = (f(0, jj) + f(1, jj)) + (f(2, jj) + f(3, jj));
            const float lo = (f(0, jj + 8) + f(1, jj + 8)) + (f(2, jj + 8) + f(3, jj + 8));
            float* o = a.out + (size_t)jj * a.rows + orow;
            if (a.splits > 1) {
              atomicAdd(o, hi + lo);
            } else {
              *o = hi + lo;
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
}

// ------------------------------------------------------------------- host

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn tc_encode_fn() {
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

}  // namespace

int launch_bf16_gemm_tc(const uint16_t* W, const float* x, float* out, int rows, int cols, int n,
                        cudaStream_t stream) {
  if (n < 1 || n > 8) return kErrShape;
  // W as [rows][cols] bf16: box 128 rows x 64 columns (128 bytes), 128-byte
  // swizzle, zero fill past the edges (cols % 32 == 0: 16-byte row pitch)
  EncodeTiledFn enc = tc_encode_fn();
  if (!enc) return kErrLaunch;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {kTcKB, kTcM};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(W), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return kErrArg;
  if (cudaFuncSetAttribute(bf16_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem) !=
      cudaSuccess)
    return kErrLaunch;
  TcArgs a{};
  a.x = x;
  a.out = out;
  a.rows = rows;
  a.cols = cols;
  a.n = n;
  a.nkb = (cols + kTcKB - 1) / kTcKB;
  a.tiles = (rows + kTcM - 1) / kTcM;
  // split K when the row tiles alone leave SMs idle
  const int sms = device_sm_count();
  int splits = (sms + a.tiles - 1) / a.tiles;
  if (splits > a.nkb) splits = a.nkb;
  if (splits < 1) splits = 1;
  a.splits = splits;
  a.units = a.tiles * splits;
  if (splits > 1 && cudaMemsetAsync(out, 0, (size_t)n * rows * sizeof(float), stream) != cudaSuccess)
    return kErrLaunch;
  const int grid = a.units < sms ? a.units : sms;
  bf16_gemm_tc_kernel<<<grid, kTcThreads, kTcSmem, stream>>>(map, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int read_tc_device_error(bool clear) { return read_unit_error(clear); }

}  // namespace ervf
