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
// CTA = 8 warps, several CTAs per SM; work unit = 128 weight rows x one
// K-split.  Per k-block of 128 columns every thread decodes two 16-byte code
// units of one row (hardware e2m1x2 / e4m3x2 converters, one f16x2 multiply
// per two weights) into a shared-memory A tile in the canonical K-major
// (no-swizzle) core-matrix layout, and one 8x16-byte chunk of X into the B
// tile; one thread then issues eight tcgen05.mma (M=128, N=16, K=16, f16 in,
// f32 accumulate) and commits them to the stage's mbarrier.  Two stages: the
// decode of k-block i+1 overlaps the MMAs of k-block i.  Code units travel by
// cp.async into a 4-deep per-thread ring (the thread that copies a unit
// decodes it), scales and X one k-block ahead in registers.
// The epilogue reads the accumulator with tcgen05.ld (warp w: TMEM lanes
// 32w..32w+31 = rows), scales by g and stores (or, with a K-split, adds
// atomically into the zeroed output).
#include "common.cuh"
#include "kernels.h"

namespace ervf {

namespace {

constexpr int kTcThreads = 256;
constexpr int kTcM = 128;            // rows per work unit (UMMA M)
constexpr int kTcN = 16;             // batch columns (UMMA N)
constexpr int kTcKB = 128;           // columns per k-block
constexpr int kTcSBO = kTcKB / 8 * 128;                 // bytes between 8-row core groups
constexpr int kTcAStage = kTcM * kTcKB * 2;             // 32 KB
constexpr int kTcBStage = kTcN * kTcKB * 2;             // 4 KB
constexpr int kTcStage = kTcAStage + kTcBStage;
constexpr int kTcRawDepth = 4;                          // k-blocks of codes in flight
constexpr int kTcRawStage = kTcM * (kTcKB / 2);         // 8 KB of code bytes
constexpr int kTcSmem = 1024 + 2 * kTcStage + kTcRawDepth * kTcRawStage;
constexpr int kTcTmemCols = 32;

struct TcArgs {
  const uint8_t* codes;   // [rows][cols/2]
  const uint8_t* scales;  // [rows][cols/16]
  float g;
  const float* x;         // [n][cols]
  float* out;             // [n][rows]
  int rows, cols, n;
  int splits;             // K-splits per row tile (atomic accumulation when > 1)
  int units;              // row tiles * splits
};

// UMMA shared-memory descriptor, K-major, no swizzle (sm100 version 1).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// kind::f16 instruction descriptor: D f32, A f16, B f16, K-major, N, M.
constexpr uint32_t kTcIdesc = (1u << 4) | ((uint32_t)(kTcN >> 3) << 17) | ((uint32_t)(kTcM >> 4) << 24);

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Two E4M3 scale bytes as an f16x2 of the first (low) byte broadcast, and of
// the second; NaN bytes (0x7F, 0xFF) read as +0 (the reference's table).
__device__ __forceinline__ void scales_f16(uint32_t sv, uint32_t& s0, uint32_t& s1) {
  const uint32_t b0 = sv & 0xFFu, b1 = (sv >> 8) & 0xFFu;
  const uint32_t c0 = (b0 & 0x7Fu) == 0x7Fu ? 0u : b0;
  const uint32_t c1 = (b1 & 0x7Fu) == 0x7Fu ? 0u : b1;
  const uint16_t pair0 = (uint16_t)(c0 | (c0 << 8)), pair1 = (uint16_t)(c1 | (c1 << 8));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(s0) : "h"(pair0));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(s1) : "h"(pair1));
}

// 32 weights of one code unit as four chunks of eight f16 (column order).
__device__ __forceinline__ void decode_unit(uint4 q, uint32_t sv, uint4 (&w)[4]) {
  uint32_t s0, s1;
  scales_f16(sv, s0, s1);
  const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t h[4];
    e2m1x8_to_f16x2(words[j], h);
    const uint32_t s = j < 2 ? s0 : s1;
    w[j] = make_uint4(hmul2(h[0], s), hmul2(h[1], s), hmul2(h[2], s), hmul2(h[3], s));
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

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait(bar, parity, 2000000000LL);
}

__global__ void __launch_bounds__(kTcThreads) nvfp4_gemm_tc_kernel(TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* mb = reinterpret_cast<uint64_t*>(smem);  // [0,1]: stage done, [2]: accumulator done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 64);
  uint8_t* stage0 = smem + 1024;
  uint8_t* raw0 = stage0 + 2 * kTcStage;  // [depth][128 rows][64 code bytes]
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

  // decode role: row rr of the tile, code units 4*kb + 2*half + {0,1}
  const int rr = tid >> 1, half = tid & 1;
  // B role: batch row bn, 8-column chunk bc of the k-block
  const int bn = tid >> 4, bc = tid & 15;
  bool dead = false;
  uint32_t gkb = 0;   // k-blocks issued by this CTA (stage ring position)
  uint32_t nacc = 0;  // accumulator commits waited for

  for (int unit = blockIdx.x; unit < a.units; unit += gridDim.x) {
    const int tile = unit / a.splits, split = unit - tile * a.splits;
    const int kb0 = (int)((long long)split * nkb / a.splits);
    const int kb1 = (int)((long long)(split + 1) * nkb / a.splits);
    const int row = tile * kTcM + rr;
    const bool row_ok = row < a.rows;
    const uint8_t* crow = a.codes + (size_t)row * cb;
    const uint8_t* srow = a.scales + (size_t)row * sb;

    // This thread's two code units of k-block kb go, by cp.async, to raw
    // ring slot kb % depth (the same thread decodes them: no barrier needed);
    // their scale bytes are read with plain loads one k-block ahead.
    uint8_t* my_raw = raw0 + rr * (kTcKB / 2) + 32 * half;
    auto copy_units = [&](int kb) {
      uint8_t* dst = my_raw + (kb % kTcRawDepth) * kTcRawStage;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int u = 4 * kb + 2 * half + i;
        const bool ok = row_ok && u < n_u;
        cp_async16(dst + 16 * i, ok ? crow + 16 * u : a.codes, ok ? 16u : 0u);
      }
    };
    auto load_scales = [&](int kb, uint32_t (&sv)[2]) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int u = 4 * kb + 2 * half + i;
        sv[i] = (row_ok && u < n_u) ? (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(srow + 2 * u)) : 0u;
      }
    };
#pragma unroll
    for (int d = 0; d < kTcRawDepth - 1; ++d) {
      if (kb0 + d < kb1) copy_units(kb0 + d);
      cp_async_commit();
    }
    uint32_t sv[2];
    load_scales(kb0, sv);
    auto load_x = [&](int kb, float4 (&v)[2]) {
      const int k = kb * kTcKB + bc * 8;
      if (bn < a.n && k < a.cols) {
        v[0] = __ldg(reinterpret_cast<const float4*>(a.x + (size_t)bn * a.cols + k));
        v[1] = __ldg(reinterpret_cast<const float4*>(a.x + (size_t)bn * a.cols + k + 4));
      } else {
        v[0] = v[1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    };
    float4 xv[2];
    load_x(kb0, xv);

    for (int kb = kb0; kb < kb1; ++kb, ++gkb) {
      const int s = (int)(gkb & 1u);
      uint8_t* sa = stage0 + s * kTcStage;
      uint8_t* sbuf = sa + kTcAStage;
      // the MMAs that last read this stage (two k-blocks ago) are complete
      if (gkb >= 2 && !dead) dead = !tc_wait(&mb[s], ((gkb >> 1) - 1) & 1u);
      // A: decode into the core-matrix layout
      if (kb + kTcRawDepth - 1 < kb1) copy_units(kb + kTcRawDepth - 1);
      cp_async_commit();
      cp_async_wait<kTcRawDepth - 1>();  // this k-block's units have landed
      const uint8_t* mine = my_raw + (kb % kTcRawDepth) * kTcRawStage;
      const uint4 q0 = *reinterpret_cast<const uint4*>(mine);
      const uint4 q1 = *reinterpret_cast<const uint4*>(mine + 16);
      uint4 w[2][4];
      decode_unit(q0, sv[0], w[0]);
      decode_unit(q1, sv[1], w[1]);
      if (kb + 1 < kb1) load_scales(kb + 1, sv);
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = (2 * half + i) * 4 + j;  // 8-column chunk inside the k-block
          *reinterpret_cast<uint4*>(sa + (rr >> 3) * kTcSBO + c * 128 + (rr & 7) * 16) = w[i][j];
        }
      // B: X rows as f16 (loaded one k-block ahead), zero beyond the batch
      // and beyond cols
      *reinterpret_cast<uint4*>(sbuf + (bn >> 3) * kTcSBO + bc * 128 + (bn & 7) * 16) =
          make_uint4(f32x2_to_f16x2(xv[0].x, xv[0].y), f32x2_to_f16x2(xv[0].z, xv[0].w),
                     f32x2_to_f16x2(xv[1].x, xv[1].y), f32x2_to_f16x2(xv[1].z, xv[1].w));
      if (kb + 1 < kb1) load_x(kb + 1, xv);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      if (tid == 0 && !dead) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sbuf);
#pragma unroll
        for (int j = 0; j < kTcKB / 16; ++j) {
          const uint64_t da = umma_desc(a0 + 256 * j, 128, kTcSBO);
          const uint64_t db = umma_desc(b0 + 256 * j, 128, kTcSBO);
          const uint32_t accum = (kb > kb0 || j > 0) ? 1u : 0u;
          asm volatile(
              "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
              " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
              ::"r"(tmem), "l"(da), "l"(db), "r"(kTcIdesc), "r"(accum) : "memory");
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
          if (j < a.n) {
            const float y = __uint_as_float(v[j]) * a.g;
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
  // wait (bounded) for the last stage commits, then free the tensor memory
  if (gkb >= 1 && !dead) tc_wait(&mb[(gkb - 1) & 1u], ((gkb - 1) >> 1) & 1u);
  if (gkb >= 2 && !dead) tc_wait(&mb[gkb & 1u], ((gkb - 2) >> 1) & 1u);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
}

}  // namespace

int launch_nvfp4_gemm_tc(const uint8_t* codes, const uint8_t* scales, float g, const float* x,
                         float* out, int rows, int cols, int n, cudaStream_t stream) {
  if (n < 1 || n > kTcN) return kErrShape;
  const int sms = device_sm_count();
  if (cudaFuncSetAttribute(nvfp4_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kTcSmem) != cudaSuccess)
    return kErrLaunch;
  // CTAs per SM from the shared-memory footprint (each CTA also holds 32 of
  // the SM's 512 tensor-memory columns)
  int smem_sm = 0;
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, 0);
  int per_sm = smem_sm / (kTcSmem + 1024);
  if (per_sm > 3) per_sm = 3;
  if (per_sm < 1) return kErrShape;
  TcArgs a{};
  a.codes = codes;
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
  nvfp4_gemm_tc_kernel<<<grid, kTcThreads, kTcSmem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace ervf
