// kernels.h -- host-side launch interfaces shared by the .cu files and capi.cu.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ervf {

constexpr int kMaxJobs = 16;

// Where one NVFP4 matrix lives.  Direct: codes/scales/g as given.  Indirect
// (the reference's *_ind kernels, fused_nvfp4.py:548-646): codes/scales are
// cache bases offset by (*slot_ptr) * stride, and g = globals[(*id_ptr)*2+gsel]
// is read on the device.
struct MatRef {
  const uint8_t* codes;
  const uint8_t* scales;
  float g;
  const int* slot_ptr;
  const int* id_ptr;
  const float* globals;
  int gsel;
  size_t code_stride;
  size_t scale_stride;
};

struct GemvJob {
  MatRef mat;
  const float* x;
  float* out;
};

// One launch over `njobs` matrices of identical shape [rows x cols].
//   mode 0: every job writes out[r] = epilogue(row sum)           (grouped GEMV)
//   mode 1: row block r gets, in ROUTE order s = 0..njobs-1,
//           acc = fmaf(y_s[r], route_w[s], acc) from acc = base[r] (or 0),
//           then rs_out[r] = resid[r] + acc (or acc)               (down + routed sum)
struct GemvBatch {
  int rows, cols, njobs, mode;
  int relu2;
  int swiglu;  // mode 0, TMA schedule: rows 2i / 2i+1 are gate / up, out[i] = silu(gate) * up
  float out_scale;
  int legacy_tree;  // 1: the 256-thread kernel's combine (S + 0.0 per group sum)
  GemvJob job[kMaxJobs];
  const float* route_w;
  const float* base;
  const float* resid;
  float* rs_out;
  // Expert parallelism (mode 0 only): job j runs only on the rank that owns
  // expert ep_ids[j], i.e. ep_ids[j] % ep_ranks == ep_rank (read on device).
  const int* ep_ids;
  int ep_ranks, ep_rank;
  // Launch with programmatic stream serialisation (PDL): the kernel may start
  // while its predecessor drains; it waits (griddepcontrol.wait) before it
  // reads activations.  ids_ready: the slot / id tables and globals were
  // written by a kernel that finished before the predecessor started, so
  // weight streaming may begin before the wait.
  int pdl;
  int ids_ready;
  // mode 1 scratch on the TMA schedule: contrib[njobs][rows] fp32 and
  // grp_count[ceil(rows / 32)] u32 (all zero before the first call; every
  // call that completes leaves them zero; after ERVF_ERR_TIMEOUT the caller
  // zeroes them again).  Each job's row values land in contrib; the producer
  // warp that completes a 32-row group's count adds those rows up in route
  // order.  NULL: the width schedules are used.
  float* contrib;
  unsigned* grp_count;
  // L2 prefetch hint for the next launch: records of pf_n experts pf_ids[i]
  // (clamped to [0, pf_experts)), codes at pf_codes + id * pf_code_stride
  // (pf_code_bytes each) and scales at pf_scales + id * pf_scale_stride.  All
  // addresses, strides and sizes multiples of 16 bytes; pf_n = 0: none.
  const uint8_t* pf_codes;
  const uint8_t* pf_scales;
  size_t pf_code_stride, pf_scale_stride, pf_code_bytes, pf_scale_bytes;
  const int* pf_ids;
  int pf_n, pf_experts;
};

// Scratch of the routed-sum launch: the group counters first (one u32 per
// row reserved, rounded up to 16 bytes: the same place for every top_k, so a
// buffer stays ready when reused with another top_k), then contrib.
inline size_t routesum_counter_bytes(int rows) { return ((size_t)rows * sizeof(int) + 15) / 16 * 16; }
inline size_t routesum_scratch_bytes(int rows, int njobs) {
  return routesum_counter_bytes(rows) + (size_t)njobs * rows * sizeof(float);
}

__host__ __device__ inline bool job_active(const GemvBatch& b, int job) {
#ifdef __CUDA_ARCH__
  return b.ep_ranks <= 1 || (b.ep_ids[job] % b.ep_ranks) == b.ep_rank;
#else
  (void)b;
  (void)job;
  return true;
#endif
}

// width 0: the TMA-staged B200 schedule (falls back to width 32 where its
// preconditions do not hold); 4/8/16/32: W lanes per row, lane L owning the
// chains L + W*i.  Every schedule returns the same bits.
int launch_nvfp4_batch(const GemvBatch& b, int width, cudaStream_t stream);

// True when the batch meets the B200 schedule's preconditions (cols % 32,
// cols <= 4096, 16-byte aligned bases and strides, routed-sum scratch).
bool nvfp4_tma_ok(const GemvBatch& b);


// Warp-specialised NVFP4 GEMM on the tensor cores (nvfp4_mma.cu).  The
// activations come as f16 panels in the MMA's layout: panel[c][kb] = 8 KB
// tile of up to 16 activation rows x 256 columns (launch_pack_panel builds
// them from fp32 rows).
size_t mma_panel_bytes(int chunks, int cols);
int launch_pack_panel(const float* src, int cols, const int* idx, const int* chunk_off, const int* chunk_n,
                      const int* n_chunks, int max_chunks, int n_single, uint8_t* panel,
                      cudaStream_t stream);
// out[j][r] = g * (W @ X[j])[r], j < n <= 16.  part / ucnt (may be NULL): K
// split partials f32[max_splits][n][rows] and counters u32[ceil(rows/128)]
// (zero before, left zero) -- used when the row tiles leave SMs idle.
int launch_nvfp4_mma_single(const uint8_t* codes, const uint8_t* scales, float g, const uint8_t* panel,
                            float* out, int rows, int cols, int n, float* part, unsigned* ucnt,
                            int max_splits, cudaStream_t stream);
// Grouped (expert-major) form: unit = (chunk, 128-row tile, K split) over a
// bank of n_experts contiguous [rows x cols] records (code stride rows*cols/2,
// scale stride rows*cols/16).  up (down = 0): relu^2 (or SwiGLU of row pairs)
// of g_up * W x as f16 into panel_out, the down launch's panels; down: fp32
// out[(chunk_off + j) * rows + r] = g_down * (W act)[r].
struct MmaGrouped {
  const uint8_t* codes;
  const uint8_t* scales;
  int n_experts, rows, cols;
  const float* globals;
  int gsel;
  const uint8_t* panel;
  const int* chunk_expert;
  const int* chunk_off;
  const int* chunk_n;
  const int* n_chunks;
  int max_chunks, max_pairs;
  int down, relu2, swiglu;
  float* out;
  uint8_t* panel_out;
  int ksplit;
  float* part;      // [ksplit][max_pairs][rows]
  unsigned* ucnt;   // [max_chunks * ceil(rows / 128)], zero before, left zero
};
int launch_nvfp4_mma_grouped(const MmaGrouped& g, cudaStream_t stream);

// Batched BF16 GEMM on the tensor cores: out[n][r] = (W @ X[n])[r] for
// n < N <= 8 (X split into bf16 high / low halves), fp32 accumulate.
int launch_bf16_gemm_tc(const uint16_t* W, const float* x, float* out, int rows, int cols, int n,
                        cudaStream_t stream);

// BF16 GEMV (gpu_kernels.py:21-49 semantics), out[b*rows + r].
int launch_bf16_gemv(const uint16_t* W, const float* x, float* out, int rows, int cols,
                     int batch, cudaStream_t stream);

// FP32 GEMV (gemv_f32 semantics) and the fused router GEMV + sigmoid top-k
// (counter: zero before, left zero).  n <= 256 experts.
int launch_f32_gemv(const float* W, const float* x, float* out, int rows, int cols,
                    cudaStream_t stream);
int launch_route_gemv_topk(const float* W, const float* x, float* rlog, const float* gate_b, int* ids,
                           float* w, int n, int cols, int top_k, float scaling, int bad_pick,
                           unsigned* counter, bool pdl, cudaStream_t stream);

int launch_weighted_accumulate(float* dst, const float* src, float weight, const float* w_ptr,
                               int n, cudaStream_t stream);

int device_sm_count();
int device_smem_optin();

// Device error words (one per translation unit: bounded waits that ran out,
// ids out of range).  Each reader returns the unit's word and, with clear,
// resets it.
int read_gemv_device_error(bool clear);
int read_aux_device_error(bool clear);
int read_tc_device_error(bool clear);
int read_ep_device_error(bool clear);
int read_mma_device_error(bool clear);
int read_token_device_error(bool clear);

// One decode token through every routed MoE layer in one launch
// (moe_token.cu).  layer_ptrs: device array [5][n_layers] (+2 rows with the
// router) of up code, up scale, down code, down scale and globals (f32
// [E][2]) bases per layer.
struct MoeTokenArgs {
  const unsigned long long* layer_ptrs;
  size_t up_code_stride, up_scale_stride, dn_code_stride, dn_scale_stride;
  const int* ids;        // [n_layers][top_k]
  const float* route_w;  // [n_layers][top_k]
  const float* x;        // [hidden]
  float* out;            // [hidden]
  int n_layers, top_k, n_experts, hidden, inter;
  void* scratch;         // moe_token_scratch_bytes, counters zero
  bool pdl;
  // router on the device: layer_ptrs has two more rows (router weights
  // f32 [E][hidden], router bias f32 [E] or 0); ids / route_w are outputs
  bool route;
  float scaling;
  int bad_pick;
  // expert parallelism (ep_ranks > 1, given routes only): scratch is this
  // rank's moe_token_ep_scratch_bytes region, peers[q] (host array) every
  // rank's region as mapped on this GPU, timeout_ns the limit of the waits
  // on other ranks
  int ep_ranks, ep_rank;
  const unsigned long long* peers;
  unsigned long long timeout_ns;
};

size_t moe_token_scratch_bytes(int n_layers, int hidden, int inter, int top_k);
size_t moe_token_ep_scratch_bytes(int n_layers, int hidden, int inter, int top_k);
int prepare_moe_token_ep(void* scratch, int n_layers, int hidden, int inter, int top_k,
                         cudaStream_t stream);
int launch_moe_token(const MoeTokenArgs& a, cudaStream_t stream);

// Expert-parallel exchange over NVLink peer memory (ep_p2p.cu).  Region
// layout of every rank: u64 flag[kEpMaxRanks] at 0, u64 seq at 512, f32
// slots[kEpBufs][top_k][hidden] at kEpSlotsOffset.
constexpr int kEpMaxRanks = 64;
constexpr int kEpBufs = 3;
constexpr size_t kEpSlotsOffset = 1024;
constexpr int kEpThreads = 1024;

inline size_t ep_region_bytes(int hidden, int slots) {
  return kEpSlotsOffset + (size_t)kEpBufs * slots * hidden * sizeof(float);
}

struct EpExchange {
  const uint64_t* peers;  // [nranks] device: every rank's region as mapped here
  int nranks, rank, buf, top_k, hidden;
  const int* ids;         // [top_k]
  const float* route_w;   // [top_k]
  const float* x;         // [hidden] or NULL
  float* out;             // [hidden]
  uint64_t timeout_ns;
};

int launch_ep_exchange_sum(const EpExchange& a, bool pdl, cudaStream_t stream);

// Batched form: pair p = t * top_k + s of token t; its output is slot
// pos[p] of the region of rank ids[p] % nranks.
struct EpBatchExchange {
  const uint64_t* peers;
  int nranks, rank, buf, tokens, top_k, hidden;
  const int* ids;        // [tokens * top_k]
  const int* pos;        // [tokens * top_k], the same on every rank
  const float* route_w;  // [tokens * top_k]
  const float* x;        // [tokens][hidden] or NULL
  float* out;            // [tokens][hidden]
  uint64_t timeout_ns;
};

int launch_ep_batch_exchange_sum(const EpBatchExchange& a, cudaStream_t stream);

}  // namespace ervf
