// aux.h -- launchers of the kernels in aux.cu.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ervf {

int launch_route_topk(const float* rlog, const float* gate_b, int* ids, float* w, int n, int top_k,
                      float scaling, int bad_pick, cudaStream_t stream);
int launch_route_topk_softmax(const float* rlog, int* ids, float* w, int layers, int n, int top_k,
                              cudaStream_t stream);
constexpr int kMaxBatchExperts = 1024;
int launch_moe_batch_lists(const int* ids, int P, int k, int E, int* chunk_expert, int* chunk_off,
                           int* chunk_n, int* n_chunks, int* tok_sorted, int* pos, int ep_ranks,
                           int ep_rank, cudaStream_t stream);
int launch_moe_batch_routesum(const float* contrib, const int* pos, const float* w, const float* x,
                              float* out, int T, int hidden, int k, cudaStream_t stream);
int launch_route_topk_batched(const float* rlog, const float* gate_b, int* ids, float* w, int layers,
                              int n, int top_k, float scaling, int bad_pick, int bias_stride,
                              cudaStream_t stream);
int launch_cache_assign(int* slot_of, int* expert_of, int* last_used, int* state2, const int* ids,
                        int* slots, int* need, int* stats2, int cap, int top_k, cudaStream_t stream);
int launch_cache_fetch(const uint8_t* bank_c, const uint8_t* bank_s, uint8_t* cache_c, uint8_t* cache_s,
                       const int* ids, const int* slots, const int* need, size_t code_bytes,
                       size_t scale_bytes, int top_k, cudaStream_t stream);
int launch_down_masked(const uint8_t* bank, const float* act, unsigned* masks, int* plist,
                       int* pcount, int* nz, int* nzc, float global_scale, const int* id_ptr,
                       const float* globals, size_t panel_bytes, float* out, int rows, int inter,
                       int nchunks, cudaStream_t stream);
int launch_ep_route_sum(const float* gathered, const int* ids, const float* w, int top_k,
                        const float* x, float* out, int hidden, int nranks, cudaStream_t stream);
int launch_down_union(const uint8_t* bank, const float* acts, int n, float* act_sum, unsigned* masks,
                      int* plist, int* pcount, int* nz, int* nzc, float global_scale, float* out, int rows,
                      int inter, int nchunks, cudaStream_t stream);
int launch_gather_rows(const float* src, const int* idx, int n, int cols, float* dst, cudaStream_t stream);
int launch_scatter_rows(const float* src, const int* idx, int n, int cols, float* dst, cudaStream_t stream);
int launch_reduce_slots(const float* contrib, const float* w, float* out, int rows, int top_k, int B,
                        cudaStream_t stream);
int launch_panel_major(const uint8_t* codes, const uint8_t* scales, uint8_t* block, int rows,
                       int inter, cudaStream_t stream);

}  // namespace ervf
