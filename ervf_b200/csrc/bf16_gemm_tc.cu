// bf16_gemm_tc.cu -- batched BF16 GEMM on the sm_100a tensor cores for the
// dense projections (tcgen05.mma, accumulator in tensor memory):
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
// CTA = 8 warps, up to four CTAs per SM; work unit = 128 weight rows x one
// K range.  Per k-block of 64 columns, thread (warp w, lane l) owns weight row
// 32*(w % 4) + l -- its tensor-memory lane -- and half w / 4 of the k-block
// (32 bf16 = 64 bytes): it copies them by cp.async into a 4-deep per-thread
// ring (the thread that copies a unit also moves it on, so no barrier) and
// stores them with tcgen05.st (row = lane; a bf16 pair is one 32-bit column,
// K order): the A operand never touches the MMA's shared-memory path.  The X
// halves go to a shared B tile in the canonical K-major core-matrix layout.
// Four threads (lane 0 of warps 0..3) each issue one of the k-block's four
// tcgen05.mma.kind::f16 (bf16 inputs, A from tensor memory, M=128, N=16,
// K=16, f32 accumulate) into their own accumulator chain and commit it to the
// stage's mbarrier -- an MMA takes its issuing thread ~95 cycles, and issuers
// in different warps overlap; two A / B stages overlap the next k-block's
// copies with this one's MMAs.  The epilogue reads the four chains with
// tcgen05.ld and adds them in a fixed order.
// Small matrices split K over several units per row tile so that every SM
// works; the splits then add into the zeroed output with fp32 atomics, so the
// last bits depend on their arrival order (within the tolerance above).
#include "common.cuh"
#include "kernels.h"

namespace ervf {

namespace {

constexpr int kTcThreads = 256;
constexpr int kTcM = 128;            // rows per work unit (UMMA M)
constexpr int kTcN = 16;             // MMA columns: X high halves 0..7, low halves 8..15
constexpr int kTcKB = 64;            // columns per k-block (4 MMAs of K = 16)
constexpr int kTcBSBO = kTcKB / 8 * 128;                // B: bytes between 8-row core groups
constexpr int kTcBStage = kTcN * kTcKB * 2;             // 2 KB
constexpr int kTcDepth = 4;                             // k-blocks of weights in flight
constexpr int kTcRawStage = kTcM * kTcKB * 2;           // 16 KB of weight bytes
constexpr int kTcSmem = 1024 + 2 * kTcBStage + kTcDepth * kTcRawStage;
constexpr int kTcUnitBytes = 64;                        // per thread and k-block
constexpr int kTcIssuers = 4;        // MMA-issuing threads = accumulator chains
constexpr int kTcTmemCols = 128;     // D: chains at columns 16 c (0..63); A stages: 64..95, 96..127
constexpr int kTcACol = kTcIssuers * kTcN;
constexpr int kTcAStageCols = kTcKB / 2;  // two bf16 per 32-bit column

struct TcArgs {
  const uint16_t* w;      // [rows][cols] bf16
  const float* x;         // [n][cols]
  float* out;             // [n][rows]
  int rows, cols, n;
  int splits;             // K ranges per row tile (atomic accumulation when > 1)
  int units;              // row tiles * splits
};

// UMMA shared-memory descriptor, K-major, no swizzle (sm100 version 1).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
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

__global__ void __launch_bounds__(kTcThreads) bf16_gemm_tc_kernel(TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* mb = reinterpret_cast<uint64_t*>(smem);  // [0,1]: stage done, [2]: accumulator done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 64);
  uint8_t* bst0 = smem + 1024;                       // two B stages
  uint8_t* raw0 = bst0 + 2 * kTcBStage;              // [depth][128 rows][2 x unit bytes]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_u = a.cols >> 5;                       // 32-column units per row
  const int nkb = (a.cols + kTcKB - 1) / kTcKB;

  if (tid == 0) {
    mbar_init(&mb[0], kTcIssuers);
    mbar_init(&mb[1], kTcIssuers);
    mbar_init(&mb[2], kTcIssuers);
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

  // A role: row rr = tensor-memory lane of this warp's quarter, unit
  // 2*kb + half (the k-block's columns 32*half .. 32*half + 31)
  const int rr = 32 * (warp & 3) + lane, half = warp >> 2;
  const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
  // B role (threads < 128): MMA column bn (X row bn & 7, high half below 8,
  // low half from 8), 8-column chunk bc of the k-block
  const int bn = tid >> 3, bc = tid & 7;
  bool dead = false;
  uint32_t gkb = 0;   // k-blocks issued by this CTA (stage ring position)
  uint32_t nacc = 0;  // accumulator commits waited for

  for (int unit = blockIdx.x; unit < a.units; unit += gridDim.x) {
    const int tile = unit / a.splits, split = unit - tile * a.splits;
    const int kb0 = (int)((long long)split * nkb / a.splits);
    const int kb1 = (int)((long long)(split + 1) * nkb / a.splits);
    const int row = tile * kTcM + rr;
    const bool row_ok = row < a.rows;
    const uint8_t* wrow = reinterpret_cast<const uint8_t*>(a.w) + (size_t)row * a.cols * 2;
    uint8_t* my_raw = raw0 + rr * (2 * kTcUnitBytes) + kTcUnitBytes * half;
    auto copy_unit = [&](int kb) {
      const int u = 2 * kb + half;
      const bool ok = row_ok && u < n_u;
      uint8_t* dst = my_raw + (kb % kTcDepth) * kTcRawStage;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        cp_async16(dst + 16 * i, ok ? wrow + 64 * u + 16 * i : reinterpret_cast<const uint8_t*>(a.w),
                   ok ? 16u : 0u);
    };
#pragma unroll
    for (int d = 0; d < kTcDepth - 1; ++d) {
      if (kb0 + d < kb1) copy_unit(kb0 + d);
      cp_async_commit();
    }
    const int xn = bn & 7;
    const bool x_row = tid < 128 && xn < a.n;
    const float* xrow = x_row ? a.x + (size_t)xn * a.cols + bc * 8 : a.x;
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
      if (kb + kTcDepth - 1 < kb1) copy_unit(kb + kTcDepth - 1);
      cp_async_commit();
      cp_async_wait<kTcDepth - 1>();  // this k-block's unit has landed
      const uint8_t* mine = my_raw + (kb % kTcDepth) * kTcRawStage;
      // bf16 pairs are already the 32-bit column layout (K order, low first)
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(mine + 16 * i);
        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
      }
      tmem_st16(lane_base + kTcACol + s * kTcAStageCols + 16 * half, w);
      // B: rows 0..7 the bf16 rounding of X, rows 8..15 its remainder (X
      // loaded one k-block ahead), zero beyond the batch / columns
      if (tid < 128) {
        const float e[8] = {xv[0].x, xv[0].y, xv[0].z, xv[0].w, xv[1].x, xv[1].y, xv[1].z, xv[1].w};
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          hw[i] = f32x2_to_bf16x2(e[2 * i], e[2 * i + 1]);
          lw[i] = f32x2_to_bf16x2(e[2 * i] - bf16_lo(hw[i]), e[2 * i + 1] - bf16_hi(hw[i]));
        }
        *reinterpret_cast<uint4*>(bst0 + s * kTcBStage + b_slot) =
            bn < 8 ? make_uint4(hw[0], hw[1], hw[2], hw[3]) : make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      if (kb + 1 < kb1) load_x(kb + 1, xv);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncthreads();
      if (lane == 0 && warp < kTcIssuers && !dead) {
        // issuer j: the k-block's MMA j (columns 16 j .. 16 j + 15) into chain j
        const int j = warp;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t b0 = smem_u32(bst0 + s * kTcBStage);
        const uint64_t db = umma_desc(b0 + 256 * j, 128, kTcBSBO);
        const uint32_t accum = kb > kb0 ? 1u : 0u;
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
            ::"r"(tmem + kTcN * j), "r"(tmem + kTcACol + s * kTcAStageCols + 8 * j), "l"(db), "r"(kTcIdesc),
              "r"(accum) : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&mb[s])) : "memory");
        if (kb + 1 == kb1)
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                       ::"r"(smem_u32(&mb[2])) : "memory");
      }
    }
    // epilogue: the four chains (high and low halves) -> out
    if (!dead) dead = !tc_wait(&mb[2], nacc & 1u);
    ++nacc;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp < 4) {
      uint32_t v[kTcIssuers][16];
      const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll
      for (int c = 0; c < kTcIssuers; ++c)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(v[c][0]), "=r"(v[c][1]), "=r"(v[c][2]), "=r"(v[c][3]), "=r"(v[c][4]), "=r"(v[c][5]),
              "=r"(v[c][6]), "=r"(v[c][7]), "=r"(v[c][8]), "=r"(v[c][9]), "=r"(v[c][10]), "=r"(v[c][11]),
              "=r"(v[c][12]), "=r"(v[c][13]), "=r"(v[c][14]), "=r"(v[c][15])
            : "r"(taddr + kTcN * c));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      const int orow = tile * kTcM + warp * 32 + lane;
      if (!dead && orow < a.rows) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j < a.n) {
            const auto f = [&](int c, int k) { return __uint_as_float(v[c][k]); };
            const float hi = (f(0, j) + f(1, j)) + (f(2, j) + f(3, j));
            const float lo = (f(0, j + 8) + f(1, j + 8)) + (f(2, j + 8) + f(3, j + 8));
            const float y = hi + lo;
            float* o = a.out + (size_t)j * a.rows + orow;
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
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
}

}  // namespace

int launch_bf16_gemm_tc(const uint16_t* W, const float* x, float* out, int rows, int cols, int n,
                        cudaStream_t stream) {
  if (n < 1 || n > 8) return kErrShape;
  if (cudaFuncSetAttribute(bf16_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem) !=
      cudaSuccess)
    return kErrLaunch;
  // CTAs per SM from the shared-memory footprint and the 512 tensor-memory
  // columns of an SM (the calling thread's current device)
  int dev = 0, smem_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  int per_sm = smem_sm / (kTcSmem + 1024);
  if (per_sm > 512 / kTcTmemCols) per_sm = 512 / kTcTmemCols;
  if (per_sm < 1) return kErrShape;
  TcArgs a{};
  a.w = W;
  a.x = x;
  a.out = out;
  a.rows = rows;
  a.cols = cols;
  a.n = n;
  const int tiles = (rows + kTcM - 1) / kTcM;
  const int nkb = (cols + kTcKB - 1) / kTcKB;
  const int slots = device_sm_count() * per_sm;
  int splits = (slots + tiles - 1) / tiles;
  if (splits > nkb) splits = nkb;
  if (splits < 1) splits = 1;
  a.splits = splits;
  a.units = tiles * splits;
  if (splits > 1 && cudaMemsetAsync(out, 0, (size_t)n * rows * sizeof(float), stream) != cudaSuccess)
    return kErrLaunch;
  const int grid = a.units < slots ? a.units : slots;
  bf16_gemm_tc_kernel<<<grid, kTcThreads, kTcSmem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int read_tc_device_error(bool clear) { return read_unit_error(clear); }

}  // namespace ervf
