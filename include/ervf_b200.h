/*
 * ervf_b200.h -- C ABI of the B200 (sm_100a) NVFP4 expert-GEMV path.
 *
 * Every entry point is extern "C", takes plain device pointers, sizes and a
 * cudaStream_t passed as void*, launches asynchronously on that stream,
 * allocates nothing and returns an int status (ERVF_OK or a negative
 * ERVF_ERR_*).  Each one replaces a kernel / wrapper of kennydd001/ervf,
 * cited as file:line of src/moe_lab/lightningstream_nemotron/.
 *
 * Numeric contract: the NVFP4 GEMV entry points return, bit for bit, what the
 * reference's gemv_nvfp4_ervf kernel returns on the same bytes
 * (fused_nvfp4.py:295-406), for every `width`; legacy_tree=1 returns what
 * gemv_nvfp4_rows returns (fused_nvfp4.py:31-122).
 *
 * Shapes the reference silently assumed are checked here: cols % 16 == 0,
 * codes 4-byte aligned, pointers non-null.
 */
#ifndef ERVF_B200_H
#define ERVF_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ERVF_API __attribute__((visibility("default")))
#else
#define ERVF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ERVF_OK 0
#define ERVF_ERR_NULL -1     /* a required pointer is NULL */
#define ERVF_ERR_SHAPE -2    /* rows/cols/k outside what the kernels support */
#define ERVF_ERR_ALIGN -3    /* a pointer or stride is misaligned */
#define ERVF_ERR_LAUNCH -4   /* the CUDA launch failed */
#define ERVF_ERR_TIMEOUT -5  /* a bounded device wait ran out (ervf_device_status) */
#define ERVF_ERR_ARG -6      /* an argument value is invalid (width, batch, ...) */
#define ERVF_ERR_DEVICE -7    /* a set-up CUDA call failed (allocation, IPC mapping) */
#define ERVF_ERR_SCRATCH_LIMIT -8 /* larger than the library's fixed scratch array */

/* Launch flags of the grouped MoE entry points.
 * ERVF_LAUNCH_PDL: launch with programmatic stream serialisation, so the
 *   kernel's prologue and weight streaming overlap the previous kernel on the
 *   stream; it waits for that kernel before reading activations.
 * ERVF_LAUNCH_IDS_READY: the route ids / globals were written by a kernel that
 *   completed before the previous kernel on the stream started (e.g. one
 *   routing launch for all layers at the start of a decode step), so they may
 *   be read -- and the routed experts' weights streamed -- before the wait. */
#define ERVF_LAUNCH_PDL 1
#define ERVF_LAUNCH_IDS_READY 2
/* ervf_moe_up_grouped only: SwiGLU experts (Qwen shape).  The up record has
 * 2*inter rows, gate and up interleaved (row 2i = gate i, row 2i+1 = up i),
 * and act[s*inter + i] = silu(gate_i) * up_i, silu(v) = v / (1 + expf(-v)).
 * B200 schedule (width 0) only.  The reference has no SwiGLU NVFP4 kernel. */
#define ERVF_UP_SWIGLU 4

/* Library version, e.g. 100 for 0.1.0. */
ERVF_API int ervf_version(void);

/* Reads and clears the device-side error word of the current device
 * (ERVF_OK or ERVF_ERR_TIMEOUT).  Synchronous. */
ERVF_API int ervf_device_status(void);

/* out[r] = op(sum_k dequant(W)[r,k] * x[k]) for one NVFP4 matrix.
 * codes u8[rows][cols/2] (low nibble first), scales E4M3 u8[rows][cols/16],
 * x f32[cols], out f32[rows].  op = relu(v)^2 if apply_relu2 else v*out_scale.
 * width: 0 = B200 schedule, or 4/8/16/32 = the ERVF subwarp widths.
 * Replaces gemv_nvfp4_ervf / gemv_nvfp4_rows and FusedNVFP4.gemv_into
 * (fused_nvfp4.py:295-406, :31-122, :944-968). */
ERVF_API int ervf_nvfp4_gemv(const uint8_t* codes, const uint8_t* scales, const float* x, float* out,
                    float global_scale, int rows, int cols, int apply_relu2, float out_scale,
                    int width, int legacy_tree, void* stream);

/* Indirect form: codes = codes_base + slot_ptr[0]*code_stride, scales likewise,
 * global scale = globals[id_ptr[0]*2 + gsel], all read on the device.
 * Replaces gemv_nvfp4_ervf_ind / FusedNVFP4.gemv_ervf_indirect
 * (fused_nvfp4.py:548-646, :817-830). */
ERVF_API int ervf_nvfp4_gemv_ind(const uint8_t* codes_base, const uint8_t* scales_base,
                        const int32_t* slot_ptr, const int32_t* id_ptr, const float* globals,
                        int gsel, const float* x, float* out, int rows, int cols, int apply_relu2,
                        float out_scale, size_t code_stride, size_t scale_stride, int width,
                        void* stream);

/* njobs (<= 16) same-shape NVFP4 GEMVs in one launch; the pointer arrays
 * live in HOST memory.  Equal, per job, to ervf_nvfp4_gemv.  Replaces the
 * per-expert gemv_into loop of the MoE layer (runtime.py:571-578). */
ERVF_API int ervf_nvfp4_gemv_grouped(int njobs, const uint8_t* const* codes, const uint8_t* const* scales,
                            const float* global_scales, const float* const* xs, float* const* outs,
                            int rows, int cols, int apply_relu2, float out_scale, int width,
                            void* stream);

/* dst[i] = fmaf(src[i], weight, dst[i]).  Replaces weighted_accumulate /
 * FusedNVFP4.accumulate_into (fused_nvfp4.py:125-133, :980-984). */
ERVF_API int ervf_weighted_accumulate(float* dst, const float* src, float weight, int n, void* stream);

/* Same with the weight read from device memory.  Replaces
 * weighted_accumulate_ind (fused_nvfp4.py:736-744, :855-859). */
ERVF_API int ervf_weighted_accumulate_ind(float* dst, const float* src, const float* w_ptr, int n,
                                 void* stream);

/* Routed up projections of one token, one launch: for s in [0, top_k),
 * e = ids[s] (device), act[s*inter + r] = relu(up_e(x)[r])^2 with
 * up_e = (up_codes + e*up_code_stride, up_scales + e*up_scale_stride,
 * globals[e*2 + 1]).  Equal, per slot, to FusedNVFP4.gemv_into(...,
 * apply_relu2=True) (fused_nvfp4.py:970-978, first half). */
ERVF_API int ervf_moe_up_grouped(const uint8_t* up_codes, const uint8_t* up_scales, size_t up_code_stride,
                        size_t up_scale_stride, const int32_t* ids, const float* globals, int top_k,
                        const float* x, float* act, int inter, int hidden, int width, int flags,
                        void* stream);

/* Routed down projections plus the route-order sum, one launch: for every
 * output row r, acc = base ? base[r] : 0; for s = 0..top_k-1 in ROUTE order
 * acc = fmaf(down_{ids[s]}(act[s])[r], route_w[s], acc); out[r] = resid ?
 * resid[r] + acc : acc.  Equal to top_k down gemv_into calls followed by
 * accumulate_into in route order (fused_nvfp4.py:970-984; route-order
 * contract runtime.py:588-596).
 * scratch: caller-owned device buffer of ervf_routesum_scratch_bytes(hidden,
 * top_k) bytes, 16-byte aligned, zero-filled once before its first use; each
 * call that completes leaves it ready for the next (calls that share it must
 * not overlap on the GPU).  After ervf_device_status reports
 * ERVF_ERR_TIMEOUT, zero it again before reusing it.  With scratch the rows
 * spread over all SMs; scratch = NULL runs a slower schedule that needs none.
 * Without ERVF_LAUNCH_PDL and with 2 <= top_k <= 8 the sum runs through a
 * thread-block cluster (distributed shared memory) and leaves the scratch
 * untouched; otherwise every launch uses it.  Same bits either way. */
ERVF_API int ervf_moe_down_routesum(const uint8_t* dn_codes, const uint8_t* dn_scales,
                           size_t dn_code_stride, size_t dn_scale_stride, const int32_t* ids,
                           const float* globals, const float* route_w, int top_k, const float* act,
                           const float* base, const float* resid, float* out, int hidden, int inter,
                           void* scratch, size_t scratch_bytes, int width, int flags, void* stream);

/* Bytes of scratch ervf_moe_down_routesum uses for (hidden, top_k). */
ERVF_API size_t ervf_routesum_scratch_bytes(int hidden, int top_k);

/* One routed-MoE layer of one token, two launches: act[s] =
 * relu(up_{ids[s]}(x))^2, then out[r] = x[r] + acc with acc =
 * fmaf(down_{ids[s]}(act[s])[r], route_w[s], acc) over s = 0..top_k-1 in route
 * order from 0.0 -- bit-identical to ervf_moe_up_grouped followed by
 * ervf_moe_down_routesum(resid = x), i.e. to the reference's per-expert
 * gemv_into + accumulate_into sequence (fused_nvfp4.py:970-984, route order
 * runtime.py:571-596).  Adds an L2 prefetch: the up launch queues this
 * layer's routed down records into L2, and the down launch queues the next
 * layer's routed up records (next_up_codes / next_up_scales / next_ids, same
 * strides as this layer's up bank; all three NULL for none), so that expert
 * weights stream from HBM under the previous launch's compute.  The hint
 * never changes results; prefetch ids are clamped to [0, n_experts).
 * scratch: as for ervf_moe_down_routesum (zeroed once, left ready).  All
 * pointers and record strides 16-byte aligned; hidden, inter multiples of 32,
 * <= 4096; top_k <= 16.  B200 schedule only. */
ERVF_API int ervf_moe_layer(const uint8_t* up_codes, const uint8_t* up_scales, size_t up_code_stride,
                            size_t up_scale_stride, const uint8_t* dn_codes, const uint8_t* dn_scales,
                            size_t dn_code_stride, size_t dn_scale_stride, const int32_t* ids,
                            const float* globals, const float* route_w, int top_k, const float* x,
                            float* act, float* out, int hidden, int inter, int n_experts,
                            void* scratch, size_t scratch_bytes, const uint8_t* next_up_codes,
                            const uint8_t* next_up_scales, const int32_t* next_ids, int flags,
                            void* stream);

/* One decode token through EVERY routed MoE layer, one launch (single GPU):
 * for l = 0..n_layers-1, x_{l+1} = ervf_moe_layer(layer l, x_l) bit for bit
 * (same chains, tree, relu^2 and route-order sum; x_0 = x), out = x_L.  The
 * CTAs claim row items of every layer's up and down projections in order
 * from a device counter and wait (bounded) only on the activations an item
 * needs, so expert weights stream while the previous projection finishes and
 * no launch boundary separates the layers.  The reference runs the same
 * layers as per-expert launches (runtime.py:705-746 over
 * fused_nvfp4.py:970-984).
 * layer_ptrs: device array of 5 * n_layers addresses: [0, L) up code bases,
 * [L, 2L) up scale bases, [2L, 3L) down code bases, [3L, 4L) down scale
 * bases, [4L, 5L) globals f32[n_experts][2] (down, up) of each layer; expert
 * e of layer l sits at base + e * stride.  ids int32[L][top_k] and route_w
 * f32[L][top_k] on the device (ids clamped into [0, n_experts)).  out may be
 * x.  scratch: ervf_moe_token_scratch_bytes bytes, 256-byte aligned, zeroed
 * once before first use; every launch leaves its counters zero again, also
 * after a timeout (the last CTA to leave resets them).  Launches sharing a
 * scratch must not overlap.  flags: ERVF_LAUNCH_PDL or 0.  Bases and strides
 * 16-byte aligned; hidden, inter multiples of 32, <= 4096; top_k <= 16. */
ERVF_API int ervf_moe_token(const uint64_t* layer_ptrs, int n_layers, size_t up_code_stride,
                            size_t up_scale_stride, size_t dn_code_stride, size_t dn_scale_stride,
                            const int32_t* ids, const float* route_w, int top_k, int n_experts,
                            const float* x, float* out, int hidden, int inter, void* scratch,
                            size_t scratch_bytes, int flags, void* stream);

/* ervf_moe_token with the router on the device: before each layer's experts,
 * router items compute rlog = gemv_f32(gate_w[l], x_l) (the reference's
 * mv_f32, gpu_kernels.py:51-74, one warp per expert) and the item that
 * completes the layer routes it with route_topk_f32 (fused_nvfp4.py:433-465;
 * sigmoid + bias, ties to the lowest index, scaling, bad_pick) into
 * ids[l] / route_w[l]; the layer's expert items wait for those ids before
 * streaming their weights.  Bit-identical to ervf_route_gemv_topk followed
 * by ervf_moe_layer, layer after layer (the reference's per-layer mv_f32 +
 * route_topk + experts, runtime.py:705-746).  layer_ptrs: 7 * n_layers
 * addresses: the five rows of ervf_moe_token, then [5L, 6L) router weights
 * f32[n_experts][hidden] and [6L, 7L) router bias f32[n_experts] (0 = no
 * bias) of each layer.  ids int32[L][top_k], route_w f32[L][top_k]: outputs.
 * n_experts <= 256, top_k <= min(16, n_experts), bad_pick 0 or 1; scratch
 * and the other arguments as for ervf_moe_token. */
ERVF_API int ervf_moe_token_router(const uint64_t* layer_ptrs, int n_layers, size_t up_code_stride,
                                   size_t up_scale_stride, size_t dn_code_stride,
                                   size_t dn_scale_stride, int32_t* ids, float* route_w, int top_k,
                                   int n_experts, float scaling, int bad_pick, const float* x,
                                   float* out, int hidden, int inter, void* scratch,
                                   size_t scratch_bytes, int flags, void* stream);

/* Bytes of scratch ervf_moe_token uses (counters and per-layer activations). */
ERVF_API size_t ervf_moe_token_scratch_bytes(int n_layers, int hidden, int inter, int top_k);

/* ervf_moe_token on one rank of ep_ranks (2..8) GPUs, experts sharded by id:
 * this rank runs the up / down rows of the route slots whose expert it owns
 * (ids[l][s] % ep_ranks == ep_rank; the bank holds at least those records,
 * indexed by the global id), stores each down row into every rank's scratch
 * over NVLink (peer stores, then a system-scope release of the block's count
 * on every rank; no NCCL call, no multicast) and sums every row block of
 * every layer itself, in route order, once all ranks' slot rows are in: every
 * rank ends with the same out, bit-identical to ervf_moe_token on one GPU.
 * The slot rows cross NVLink as plain peer stores (no fence, no counter):
 * the summing rank waits for the words themselves, which hold 0xFFFFFFFF
 * until written (a NaN pattern no arithmetic produces), and marks them
 * unwritten again after its sum; one entry handshake per token keeps a fast
 * rank from writing the next token's rows before every rank has entered it.
 * peer_scratch: host array [ep_ranks] of every rank's scratch as mapped on
 * this GPU (entry ep_rank = this rank's own; the others through CUDA IPC,
 * ervf_ep_region_alloc / _open), each ervf_moe_token_ep_scratch_bytes long
 * and 256-byte aligned; ervf_moe_token_ep_prepare must have run on every
 * rank's scratch (and completed) before any rank's first token.  Every rank
 * launches the same tokens with the same ids and route_w, in the same order;
 * a wait on another rank gives up after timeout_ms (ERVF_ERR_TIMEOUT in
 * ervf_device_status; prepare every rank's scratch again before the next
 * token).  The reference is single-GPU; this is its routed block
 * (runtime.py:705-746) expert-parallel, route-order contract
 * runtime.py:588-596. */
ERVF_API size_t ervf_moe_token_ep_scratch_bytes(int n_layers, int hidden, int inter, int top_k);
ERVF_API int ervf_moe_token_ep_prepare(void* scratch, size_t scratch_bytes, int n_layers, int hidden,
                                       int inter, int top_k, void* stream);
ERVF_API int ervf_moe_token_ep(const uint64_t* layer_ptrs, int n_layers, size_t up_code_stride,
                               size_t up_scale_stride, size_t dn_code_stride,
                               size_t dn_scale_stride, const int32_t* ids, const float* route_w,
                               int top_k, int n_experts, const float* x, float* out, int hidden,
                               int inter, const uint64_t* peer_scratch, int ep_ranks, int ep_rank,
                               size_t scratch_bytes, int timeout_ms, int flags, void* stream);

/* ervf_moe_down_routesum without a scratch argument.  No counterpart in the
 * reference.  The scratch is a fixed device array inside the library, so the
 * call allocates nothing: hidden <= 8192 and top_k <= 8, else
 * ERVF_ERR_SCRATCH_LIMIT before anything runs.  The first call on a device
 * looks up the array's address with that device current; make it before any
 * stream capture begins.  Each call clears the array's group counters with
 * cudaMemsetAsync on `stream` before its launch.  `flags` as for
 * ervf_moe_down_routesum: with ERVF_LAUNCH_PDL (or top_k == 1) the route sum
 * runs through the array; without it, 2..8 slots take the cluster route sum,
 * which needs no scratch.  All calls on a device share the one array: calls
 * that overlap on the GPU race.  Results are bit-identical to
 * ervf_moe_down_routesum. */
ERVF_API int ervf_moe_down_routesum_static(const uint8_t* dn_codes, const uint8_t* dn_scales,
                                           size_t dn_code_stride, size_t dn_scale_stride,
                                           const int32_t* ids, const float* globals,
                                           const float* route_w, int top_k, const float* act,
                                           const float* base, const float* resid, float* out,
                                           int hidden, int inter, int width, int flags,
                                           void* stream);

/* Expert parallelism, per rank and layer: for the route slots whose expert
 * this rank owns (ids[s] % ep_ranks == ep_rank, read on the device), act[s] =
 * relu(up(x))^2 and contrib[s*hidden + r] = down(act[s])[r] (unweighted); the
 * other slots are left untouched.  Two launches.  The reference is single-GPU
 * only; this is the per-rank half of its routed block (fused_nvfp4.py:970-978)
 * with the route-order sum deferred to ervf_ep_route_sum. */
ERVF_API int ervf_ep_expert_slots(const uint8_t* up_codes, const uint8_t* up_scales,
                                  size_t up_code_stride, size_t up_scale_stride,
                                  const uint8_t* dn_codes, const uint8_t* dn_scales,
                                  size_t dn_code_stride, size_t dn_scale_stride, const int32_t* ids,
                                  const float* globals, int top_k, const float* x, float* act,
                                  float* contrib, int hidden, int inter, int ep_ranks, int ep_rank,
                                  int width, void* stream);

/* After an all-gather of every rank's contrib buffer into
 * gathered[ep_ranks][top_k][hidden]: out[r] = x[r] + acc with acc =
 * fmaf(gathered[ids[s] % ep_ranks][s][r], route_w[s], acc) for s = 0..top_k-1
 * from 0.0 (x may be NULL: out = acc).  Bit-identical to the single-GPU
 * ervf_moe_down_routesum (route-order contract runtime.py:588-596). */
ERVF_API int ervf_ep_route_sum(const float* gathered, const int32_t* ids, const float* route_w,
                               int top_k, const float* x, float* out, int hidden, int ep_ranks,
                               void* stream);

/* ervf_ep_expert_slots with launch flags (ERVF_LAUNCH_PDL, ERVF_LAUNCH_IDS_READY,
 * as for ervf_moe_up_grouped; the down launch always follows the up launch
 * with the ids already complete). */
ERVF_API int ervf_ep_expert_slots_ex(const uint8_t* up_codes, const uint8_t* up_scales,
                                     size_t up_code_stride, size_t up_scale_stride,
                                     const uint8_t* dn_codes, const uint8_t* dn_scales,
                                     size_t dn_code_stride, size_t dn_scale_stride,
                                     const int32_t* ids, const float* globals, int top_k,
                                     const float* x, float* act, float* contrib, int hidden,
                                     int inter, int ep_ranks, int ep_rank, int width, int flags,
                                     void* stream);

/* Expert-parallel exchange over NVLink peer memory (no counterpart in the
 * reference, which is single-GPU; it replaces the all-gather +
 * ervf_ep_route_sum pair).  Each rank owns one exchange region:
 *   [0, 512)  u64 flag[64]   flag[src] = last epoch rank src published
 *   [512]     u64 seq        epochs this rank has published
 *   [ERVF_EP_SLOTS_OFFSET]   f32 slots[ERVF_EP_BUFS][top_k][hidden]
 * Set-up (once, not per token; these calls allocate / map and synchronise):
 *   ervf_ep_region_alloc  cudaMalloc + zero + 64-byte CUDA IPC handle;
 *   exchange the handles between the ranks (e.g. an all-gather);
 *   ervf_ep_region_open   map a peer's region (peer access enabled);
 *   a device table u64 peers[nranks] of every rank's region as mapped on
 *   this rank (its own region at [rank]).
 * Every rank must have finished ervf_ep_region_alloc before any rank runs an
 * exchange.  Tear-down: ervf_ep_region_close on peers' regions, a barrier
 * between the ranks, then ervf_ep_region_free on the own region. */
#define ERVF_EP_SLOTS_OFFSET 1024
#define ERVF_EP_BUFS 3
#define ERVF_EP_MAX_RANKS 64
ERVF_API size_t ervf_ep_region_bytes(int hidden, int slots);  /* slots = top_k, or tokens*top_k */
ERVF_API int ervf_ep_region_alloc(size_t bytes, void** region, void* ipc_handle);
ERVF_API int ervf_ep_region_open(const void* ipc_handle, void** region);
ERVF_API int ervf_ep_region_close(void* region);
ERVF_API int ervf_ep_region_free(void* region);

/* One layer's exchange + route-order sum, one CTA: the slots this rank owns
 * must already be in slots[buf] of its own region (ervf_ep_expert_slots_ex
 * with contrib = region + ERVF_EP_SLOTS_OFFSET + buf*top_k*hidden*4).  The
 * kernel publishes epoch seq+1 into every rank's flag[rank]
 * (st.release.sys), waits until all ranks published it (bounded by
 * timeout_ms; on time-out out is left unwritten and ervf_device_status
 * reports ERVF_ERR_TIMEOUT), reads slot s from the region of rank
 * ids[s] % nranks over NVLink and writes out[r] = x[r] + acc, acc =
 * fmaf(slot_s[r], route_w[s], acc) in route order from 0.0 (x may be NULL):
 * bit-identical to ervf_moe_down_routesum on one GPU.  Two consecutive
 * exchanges must use different bufs.  hidden % 4 == 0, x/out 16-byte
 * aligned; flags: ERVF_LAUNCH_PDL or 0. */
ERVF_API int ervf_ep_exchange_route_sum(const uint64_t* peers, int nranks, int rank, int buf,
                                        const int32_t* ids, const float* route_w, int top_k,
                                        const float* x, float* out, int hidden, int timeout_ms,
                                        int flags, void* stream);

/* The runtime's masked down path over one panel-major down record
 * (runtime.py:34-52): panel_scan + gemv_down_masked_partial +
 * reduce_partials, same order (fused_nvfp4.py:157-187, :225-271, :408-419,
 * :902-942).  state buffers: masks u32[inter/16], plist i32[inter/16],
 * pcount i32[1], nz i32[inter], nzc i32[1].  bank is a device or mapped host
 * pointer. */
ERVF_API int ervf_down_masked(float* out, const uint8_t* bank, const float* act, uint32_t* masks,
                     int32_t* plist, int32_t* pcount, int32_t* nz, int32_t* nzc,
                     float global_scale, int hidden, int inter, int nchunks, void* stream);

/* Indirect form: bank = down_base + ids_s[0]*panel_bytes, global scale =
 * globals[ids_s[0]*2 + 0].  Replaces down_masked_into_indirect
 * (fused_nvfp4.py:832-853). */
ERVF_API int ervf_down_masked_ind(float* out, const uint8_t* down_base, const int32_t* id_ptr,
                         size_t panel_bytes, const float* globals, const float* act,
                         uint32_t* masks, int32_t* plist, int32_t* pcount, int32_t* nz,
                         int32_t* nzc, int hidden, int inter, int nchunks, void* stream);

/* Row-major NVFP4 down record -> panel-major record (runtime.py:34-52). */
ERVF_API int ervf_panel_major(const uint8_t* codes, const uint8_t* scales, uint8_t* block, int rows,
                     int inter, void* stream);

/* BF16 GEMV, batch 1..8: out[b*rows + r] = sum_k bf16(W[r,k]) * x[b*cols + k],
 * bit-exact per column to gemv_bf16 (gpu_kernels.py:21-49) and
 * GPUKernels.mv_bf16 (gpu_kernels.py:1549-1551).  cols % 8 == 0, W and x
 * 16-byte aligned. */
ERVF_API int ervf_bf16_gemv(const uint16_t* W, const float* x, float* out, int rows, int cols, int batch,
                   void* stream);

/* FP32 GEMV out[r] = sum_k W[r][k] * x[k], bit-exact to the reference's
 * gemv_f32 at its default 256-thread block (gpu_kernels.py:51-74) and
 * GPUKernels.mv_f32 (gpu_kernels.py:1553-1555): the router projection.
 * cols % 4 == 0; W and x 16-byte aligned. */
ERVF_API int ervf_f32_gemv(const float* W, const float* x, float* out, int rows, int cols,
                           void* stream);

/* The MoE router of one layer in one launch: rlog = gemv_f32(gate_w, x)
 * (gate_w f32[n][hidden]) followed by route_topk_f32 on rlog -- the
 * reference's mv_f32 + route_topk pair (runtime.py:710-713,
 * gpu_kernels.py:51-74, fused_nvfp4.py:433-465), same rlog, ids and w bit for
 * bit.  The last CTA to finish its experts routes; counter is one int32, zero
 * before the first call and left zero.  flags: ERVF_LAUNCH_PDL (x may be the
 * output of the previous kernel on the stream).  n <= 256, top_k <= 64,
 * hidden % 4 == 0. */
ERVF_API int ervf_route_gemv_topk(const float* gate_w, const float* x, float* rlog,
                                  const float* gate_b, int32_t* ids, float* w, int n, int hidden,
                                  int top_k, float scaling, int bad_pick, int32_t* counter,
                                  int flags, void* stream);

/* Device router head: replaces route_topk_f32 / FusedNVFP4.route_topk
 * (fused_nvfp4.py:433-465, :797-801).  n <= 1024, top_k <= 64. */
ERVF_API int ervf_route_topk(const float* rlog, const float* gate_b, int32_t* ids, float* w, int n,
                    int top_k, float scaling, int bad_pick, void* stream);

/* The device router for `layers` independent problems in one launch (one
 * warp each): rlog f32[layers][n], gate_b f32[layers][bias_stride] (NULL for
 * no bias when n <= 256), ids i32[layers][top_k], w f32[layers][top_k].
 * Same selections and weights as ervf_route_topk per layer. */
ERVF_API int ervf_route_topk_batched(const float* rlog, const float* gate_b, int32_t* ids, float* w,
                                     int layers, int n, int top_k, float scaling, int bad_pick,
                                     int bias_stride, void* stream);

/* SweepMoE (sweepspec.py:244-375) building blocks.
 *
 * ervf_nvfp4_gemm_rows_b: out[b*rows + r] = op(W x[nodes[b]])[r] for b < n
 * <= 16, each column bit-identical to the reference's gemm_nvfp4_rows_b
 * (sweepspec.py:28-141), i.e. to gemv_nvfp4_rows on that activation row (the
 * legacy 256-chain tree); op = relu(v)^2 when apply_relu2.  x is [*][cols]
 * with rows picked by the device list nodes[n]; xbuf: caller scratch of
 * n*cols floats, 16-byte aligned (the gathered rows). */
ERVF_API int ervf_nvfp4_gemm_rows_b(const uint8_t* codes, const uint8_t* scales, const float* x,
                                   const int32_t* nodes, float* out, float global_scale, int rows,
                                   int cols, int n, int apply_relu2, float* xbuf, void* stream);

/* ervf_down_union: contrib[dst[b]*hidden + r] = the masked panel-major down
 * projection of acts[b*inter ..] (the record at `bank`, runtime.py:34-52
 * layout), b < n <= 64, walking the UNION panel list and masks of the n nodes
 * -- bit-identical to the reference's down_union (act_sum = sum of the
 * nodes' rows, panel_scan of it, gemm_down_masked_b, reduce_partials_scatter;
 * sweepspec.py:143-216, :331-360).  The union matters: panels go to chunks
 * by their position in the active list, so a node's bits depend on the other
 * nodes' zero pattern.  act_sum: inter floats; masks .. nzc: the masked-down
 * state of ervf_down_masked; tmp: n*hidden floats. */
ERVF_API int ervf_down_union(const uint8_t* bank, const float* acts, int n, const int32_t* dst,
                            float* contrib, float global_scale, int hidden, int inter, int nchunks,
                            float* act_sum, uint32_t* masks, int32_t* plist, int32_t* pcount,
                            int32_t* nz, int32_t* nzc, float* tmp, void* stream);

/* ervf_reduce_slots: out[b*rows + r] = fmaf(weights[b*top_k + s],
 * contrib[(b*top_k + s)*rows + r], .) over s = 0..top_k-1 in route-slot
 * order, starting from out's value (reduce_slots, sweepspec.py:219-240). */
ERVF_API int ervf_reduce_slots(const float* contrib, const float* weights, float* out, int rows,
                              int top_k, int B, void* stream);

/* Batched NVFP4 GEMM on the tensor cores for decode batches:
 * out[b*rows + r] = global_scale * sum_k W[r][k] * x[b*cols + k] for b < n <= 16,
 * W the NVFP4 matrix (codes + E4M3 block scales as in ervf_nvfp4_gemv).
 * Weights decoded exactly to f16, x rounded to f16, fp32 accumulate in tensor
 * memory: held to rel-L2 <= 1e-3 against a float64 dequantise-then-matmul,
 * not to the batch-1 chain order.  Deterministic: a K split (used when the
 * row tiles alone leave SMs idle) adds its partials in split order, so the
 * bits do not change from run to run.  cols % 32 == 0, cols <= 4096; codes,
 * scales and x 16-byte aligned.  scratch: ervf_nvfp4_gemm_tc_scratch_bytes
 * (rows, cols, n) bytes, 16-byte aligned, zero-filled once (its split
 * counters are left zero by every call that completes).  Replaces the batched
 * SIMT gemm_nvfp4_rows_b (sweepspec.py:28-240) for one matrix. */
ERVF_API int ervf_nvfp4_gemm_tc(const uint8_t* codes, const uint8_t* scales, float global_scale,
                                const float* x, float* out, int rows, int cols, int n,
                                void* scratch, size_t scratch_bytes, void* stream);

/* Bytes of scratch ervf_nvfp4_gemm_tc uses for (rows, cols, n). */
ERVF_API size_t ervf_nvfp4_gemm_tc_scratch_bytes(int rows, int cols, int n);

/* Batched BF16 GEMM on the tensor cores for the dense projections:
 * out[b*rows + r] = sum_k W[r][k] * x[b*cols + k] for b < batch <= 8, fp32
 * accumulate; x is split into bf16 high and low halves (16 MMA columns), so
 * the result is held to rel-L2 <= 1e-3, not to gemv_bf16's chain order (the
 * reference has no batched BF16 kernel; ervf_bf16_gemv keeps that order).
 * When a matrix has fewer 128-row tiles than the GPU has CTA slots, K is split
 * over several CTAs whose fp32 partial sums are added atomically into out: the
 * last bits then vary with the arrival order from call to call (always within
 * the tolerance).  cols % 32 == 0; W and x 16-byte aligned. */
ERVF_API int ervf_bf16_gemm_tc(const uint16_t* W, const float* x, float* out, int rows, int cols,
                               int batch, void* stream);

/* Expert-major batched routed-MoE block of a decode batch on the tensor cores
 * (the reference's SweepMoE block, sweepspec.py:244-375): tokens x[t] (f32
 * [tokens][hidden]) routed to ids[t*top_k + s] with weights route_w[...]:
 * every expert is read once for all the tokens routed to it (chunks of <= 16
 * tokens as the MMA's N columns), act = relu(up(x))^2, contrib = down(act),
 * then out[t] = x[t] + acc, acc = fmaf(contrib[t,s], w[t,s], acc) over s in
 * route order.  Five launches (lists, activation panels, up, down, route
 * sum); up and down run on the warp-specialised tensor-core kernel, the up
 * epilogue writing act as f16 straight into the down launch's activation
 * panels.  Tolerance path (rel-L2 <= 1e-3; weights exact in f16, x and act
 * rounded to f16).  Bank as in ervf_moe_up_grouped / ervf_moe_down_routesum,
 * records contiguous (code stride = rows * cols / 2, scale stride = rows *
 * cols / 16, 16-byte aligned); hidden, inter multiples of 32, <= 4096;
 * tokens*top_k <= 4096, n_experts <= 1024; scratch:
 * ervf_moe_batched_scratch_bytes(...) bytes, 16-byte aligned. */
ERVF_API int ervf_moe_batched(const uint8_t* up_codes, const uint8_t* up_scales,
                              size_t up_code_stride, size_t up_scale_stride,
                              const uint8_t* dn_codes, const uint8_t* dn_scales,
                              size_t dn_code_stride, size_t dn_scale_stride, const float* globals,
                              const int32_t* ids, const float* route_w, int tokens, int top_k,
                              int n_experts, const float* x, float* out, int hidden, int inter,
                              void* scratch, size_t scratch_bytes, void* stream);

/* ervf_moe_batched with a K-split of the tensor-core launches (ksplit 1 or
 * 2): each (expert chunk, 128-row tile) is computed as ksplit CTAs over
 * consecutive halves of the columns, and the last one adds the fp32 partial
 * accumulators in split order before the global scale -- more CTAs for a
 * small batch or a small expert shard.  Deterministic; the result depends on
 * ksplit (association of the partial sums), not on the grid, the arrival
 * order or the rank.  flags: ERVF_UP_SWIGLU for SwiGLU experts (up records of
 * 2*inter rows, gate / up interleaved; act = silu(gate) * up with CUDA expf,
 * the Qwen3-shaped block).  No counterpart in the reference. */
ERVF_API int ervf_moe_batched_ex(const uint8_t* up_codes, const uint8_t* up_scales,
                                 size_t up_code_stride, size_t up_scale_stride,
                                 const uint8_t* dn_codes, const uint8_t* dn_scales,
                                 size_t dn_code_stride, size_t dn_scale_stride, const float* globals,
                                 const int32_t* ids, const float* route_w, int tokens, int top_k,
                                 int n_experts, const float* x, float* out, int hidden, int inter,
                                 int ksplit, int flags, void* scratch, size_t scratch_bytes,
                                 void* stream);

/* Bytes of scratch ervf_moe_batched uses. */
ERVF_API size_t ervf_moe_batched_scratch_bytes(int tokens, int top_k, int hidden, int inter);

/* Expert-parallel form of ervf_moe_batched (no counterpart in the reference,
 * which is single-GPU): the lists sort every pair on every rank (so the
 * sorted position pos[p] of pair p is the same everywhere) but this rank runs
 * up and down only for the experts it owns (e % ep_ranks == ep_rank), writing
 * slots[pos[p]] (f32 [tokens*top_k][hidden]; normally slots[buf] of the
 * rank's exchange region, see ervf_ep_region_alloc).  Scratch as for
 * ervf_moe_batched. */
ERVF_API int ervf_moe_batched_ep_slots(const uint8_t* up_codes, const uint8_t* up_scales,
                                       size_t up_code_stride, size_t up_scale_stride,
                                       const uint8_t* dn_codes, const uint8_t* dn_scales,
                                       size_t dn_code_stride, size_t dn_scale_stride,
                                       const float* globals, const int32_t* ids, int tokens,
                                       int top_k, int n_experts, const float* x, float* slots,
                                       int hidden, int inter, int ep_ranks, int ep_rank,
                                       void* scratch, size_t scratch_bytes, void* stream);
/* ervf_moe_batched_ep_slots with the K-split of ervf_moe_batched_ex. */
ERVF_API int ervf_moe_batched_ep_slots_ex(const uint8_t* up_codes, const uint8_t* up_scales,
                                          size_t up_code_stride, size_t up_scale_stride,
                                          const uint8_t* dn_codes, const uint8_t* dn_scales,
                                          size_t dn_code_stride, size_t dn_scale_stride,
                                          const float* globals, const int32_t* ids, int tokens,
                                          int top_k, int n_experts, const float* x, float* slots,
                                          int hidden, int inter, int ep_ranks, int ep_rank,
                                          int ksplit, void* scratch, size_t scratch_bytes,
                                          void* stream);

/* The batched exchange + route-order sum over NVLink peer memory, after
 * ervf_moe_batched_ep_slots on every rank with the same scratch: publishes
 * and waits for the epoch as ervf_ep_exchange_route_sum does, then out[t] =
 * x[t] + acc, acc = fmaf(slot(p)[r], route_w[p], acc) over p = t*top_k + s,
 * s in route order, slot(p) read from slots[buf][pos[p]] of the region of
 * rank ids[p] % nranks -- identical to ervf_moe_batched on one GPU.  The
 * region must hold tokens*top_k slots (ervf_ep_region_bytes(hidden,
 * tokens*top_k)); two consecutive exchanges use different bufs. */
ERVF_API int ervf_ep_batch_exchange_route_sum(const uint64_t* peers, int nranks, int rank, int buf,
                                              const int32_t* ids, const float* route_w, int tokens,
                                              int top_k, const float* x, float* out, int hidden,
                                              int inter, const void* scratch, size_t scratch_bytes,
                                              int timeout_ms, void* stream);

/* Softmax top-k routing of `layers` logit rows f32[layers][n] (config 2,
 * Qwen shape; the reference's router is sigmoid only): per layer the top_k
 * largest logits in descending order (ties to the lowest index), ids[l][s]
 * and w[l][s] = e_s / sum, e_s = expf(logit_s - logit_max), sum added in
 * selection order -- the renormalised softmax of the selected experts.
 * n <= 1024, top_k <= 32.  No counterpart in the reference. */
ERVF_API int ervf_route_topk_softmax(const float* rlog, int32_t* ids, float* w, int layers, int n,
                                     int top_k, void* stream);

/* Device LRU slot assignment: replaces cache_assign / FusedNVFP4.cache_assign
 * (fused_nvfp4.py:470-511, :803-808). */
ERVF_API int ervf_cache_assign(int32_t* slot_of, int32_t* expert_of, int32_t* last_used, int32_t* state2,
                      const int32_t* ids, int32_t* slots, int32_t* need, int32_t* stats2, int cap,
                      int top_k, void* stream);

/* Copies the records of missed route slots from the bank (device or mapped
 * host) into cache slots: replaces cache_fetch / FusedNVFP4.cache_fetch
 * (fused_nvfp4.py:516-543, :810-815). */
ERVF_API int ervf_cache_fetch(const uint8_t* bank_c, const uint8_t* bank_s, uint8_t* cache_c,
                     uint8_t* cache_s, const int32_t* ids, const int32_t* slots,
                     const int32_t* need, size_t code_bytes, size_t scale_bytes, int top_k,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ERVF_B200_H */
