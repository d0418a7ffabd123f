// ref_launch.cu -- host launchers for the REFERENCE's own CUDA kernels.
//
// TEST INFRASTRUCTURE.  oracle/build_ref.py extracts the kernel source
// strings of kennydd001/ervf (they live inside Python files and the
// reference compiles them at run time with NVRTC) into oracle/_ref/, and
// compiles them together with this file into oracle/_ref/libervf_ref.so for
// sm_100a.  The launchers below reproduce the reference wrappers' launch
// geometry and arguments:
//   gemv_nvfp4_rows      fused_nvfp4.py:962-968   grid rows, block 256, smem cols*4
//   gemv_nvfp4_ervf      fused_nvfp4.py:954-960   grid ceil(rows/(256/W)), block 256
//   ERVF width template  nervf01_geometry_audit.py:470-480
//   gemv_nvfp4_ervf_ind  fused_nvfp4.py:817-830
//   weighted_accumulate(_ind) fused_nvfp4.py:980-984, :855-859
//   masked down          fused_nvfp4.py:902-942 (gatherless: the bank is read in place)
//   route_topk_f32       fused_nvfp4.py:797-801
//   cache_assign         fused_nvfp4.py:803-808
//   gemv_bf16            gpu_kernels.py:1549-1551
//   gemv_f32             gpu_kernels.py:1553-1555
//   panel_scan           fused_nvfp4.py:157-187 (as down_union calls it, sweepspec.py:339-343)
//   SweepMoE kernels     sweepspec.py:317-375 (gemm_nvfp4_rows_b grid rows, block 256, smem
//                        n*cols*4; gemm_down_masked_b grid (ceil(hidden/128), nchunks), block
//                        128; reduce_partials_scatter / reduce_slots grid ceil(rows/256), 256)
// Only tests/ and bench.py's reference leg load this library.
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#define REF_API extern "C" __attribute__((visibility("default")))

static inline int ref_status() { return cudaGetLastError() == cudaSuccess ? 0 : -4; }

#if defined(REF_FUSED)
#include "ref_fused.cu"

REF_API int ref_gemv_rows(const unsigned char* codes, const unsigned char* scales, const float* e2m1,
                          const float* e4m3, const float* x, float* out, float g, int rows, int cols,
                          int relu2, float out_scale, void* stream) {
  gemv_nvfp4_rows<<<rows, 256, cols * 4, (cudaStream_t)stream>>>(codes, scales, e2m1, e4m3, x, out, g,
                                                                 rows, cols, relu2, out_scale);
  return ref_status();
}

REF_API int ref_gemv_ervf16(const unsigned char* codes, const unsigned char* scales, const float* e2m1,
                            const float* e4m3, const float* x, float* out, float g, int rows, int cols,
                            int relu2, float out_scale, void* stream) {
  gemv_nvfp4_ervf<<<(rows + 15) / 16, 256, cols * 4, (cudaStream_t)stream>>>(
      codes, scales, e2m1, e4m3, x, out, g, rows, cols, relu2, out_scale);
  return ref_status();
}

REF_API int ref_gemv_ervf_ind(const unsigned char* codes_base, const unsigned char* scales_base,
                              const int* slot_ptr, const int* id_ptr, const float* globals, int gsel,
                              const float* e2m1, const float* e4m3, const float* x, float* out,
                              int rows, int cols, int relu2, size_t code_stride, size_t scale_stride,
                              void* stream) {
  gemv_nvfp4_ervf_ind<<<(rows + 15) / 16, 256, cols * 4, (cudaStream_t)stream>>>(
      codes_base, scales_base, slot_ptr, id_ptr, globals, gsel, e2m1, e4m3, x, out, rows, cols, relu2,
      1.0f, code_stride, scale_stride);
  return ref_status();
}

REF_API int ref_weighted_accumulate(float* dst, const float* src, float w, const float* w_ptr, int n,
                                    void* stream) {
  const int blocks = (n + 255) / 256;
  if (w_ptr)
    weighted_accumulate_ind<<<blocks, 256, 0, (cudaStream_t)stream>>>(dst, src, w_ptr, n);
  else
    weighted_accumulate<<<blocks, 256, 0, (cudaStream_t)stream>>>(dst, src, w, n);
  return ref_status();
}

REF_API int ref_down_masked(float* out, const unsigned char* bank, const float* act,
                            unsigned int* masks, int* plist, int* pcount, int* nz, int* nzc,
                            float* partials, const float* e2m1, const float* e4m3, float g,
                            int hidden, int inter, int nchunks, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  panel_scan<<<1, 256, 0, s>>>(act, inter, masks, plist, pcount, nz, nzc);
  dim3 grid((hidden + 127) / 128, nchunks);
  gemv_down_masked_partial<<<grid, 128, 0, s>>>(bank, act, plist, masks, pcount, e2m1, e4m3, partials,
                                                g, hidden, inter);
  reduce_partials<<<(hidden + 255) / 256, 256, 0, s>>>(partials, out, hidden, nchunks);
  return ref_status();
}

REF_API int ref_panel_scan(const float* act, int inter, unsigned int* masks, int* plist, int* pcount,
                           int* nz, int* nzc, void* stream) {
  panel_scan<<<1, 256, 0, (cudaStream_t)stream>>>(act, inter, masks, plist, pcount, nz, nzc);
  return ref_status();
}

REF_API int ref_route_topk(const float* rlog, const float* gate_b, int* ids, float* w, int n, int top_k,
                           float scaling, int bad_pick, void* stream) {
  route_topk_f32<<<1, 128, 0, (cudaStream_t)stream>>>(rlog, gate_b, ids, w, n, top_k, scaling,
                                                      bad_pick);
  return ref_status();
}

REF_API int ref_cache_assign(int* slot_of, int* expert_of, int* last_used, int* state2, const int* ids,
                             int* slots, int* need, int* stats2, int cap, int top_k, void* stream) {
  cache_assign<<<1, 32, 0, (cudaStream_t)stream>>>(slot_of, expert_of, last_used, state2, ids, slots,
                                                   need, stats2, cap, top_k);
  return ref_status();
}

#elif defined(REF_ERVF_W)
#define gemv_nvfp4_ervf REF_KERNEL_NAME
#include REF_ERVF_FILE

REF_API int REF_LAUNCH_NAME(const unsigned char* codes, const unsigned char* scales, const float* e2m1,
                            const float* e4m3, const float* x, float* out, float g, int rows, int cols,
                            int relu2, float out_scale, void* stream) {
  const int rpb = 256 / REF_ERVF_W;
  REF_KERNEL_NAME<<<(rows + rpb - 1) / rpb, 256, cols * 4, (cudaStream_t)stream>>>(
      codes, scales, e2m1, e4m3, x, out, g, rows, cols, relu2, out_scale);
  return ref_status();
}

#elif defined(REF_SWEEP)
#include "ref_sweep.cu"

REF_API int ref_gemm_rows_b(const unsigned char* codes, const unsigned char* scales, const float* e2m1,
                            const float* e4m3, const float* x, const int* nodes, float* out, float g,
                            int rows, int cols, int B, int relu2, void* stream) {
  const int shared = B * cols * 4;
  if (cudaFuncSetAttribute(gemm_nvfp4_rows_b, cudaFuncAttributeMaxDynamicSharedMemorySize, shared) !=
      cudaSuccess)
    return -4;
  gemm_nvfp4_rows_b<<<rows, 256, shared, (cudaStream_t)stream>>>(codes, scales, e2m1, e4m3, x, nodes, out,
                                                                 g, rows, cols, B, relu2);
  return ref_status();
}

REF_API int ref_down_masked_b(const unsigned char* bank, const float* act, const int* plist,
                              const unsigned int* masks, const int* pcount, const float* e2m1,
                              const float* e4m3, float* partials, float g, int hidden, int inter, int B,
                              int nchunks, void* stream) {
  dim3 grid((hidden + 127) / 128, nchunks);
  gemm_down_masked_b<<<grid, 128, 0, (cudaStream_t)stream>>>(bank, act, plist, masks, pcount, e2m1, e4m3,
                                                             partials, g, hidden, inter, B);
  return ref_status();
}

REF_API int ref_reduce_partials_scatter(const float* partials, const int* dst, float* contrib, int rows,
                                        int nchunks, int B, void* stream) {
  reduce_partials_scatter<<<(rows + 255) / 256, 256, 0, (cudaStream_t)stream>>>(partials, dst, contrib,
                                                                               rows, nchunks, B);
  return ref_status();
}

REF_API int ref_reduce_slots(const float* contrib, const float* weights, float* out, int rows, int top_k,
                             int B, void* stream) {
  reduce_slots<<<(rows + 255) / 256, 256, 0, (cudaStream_t)stream>>>(contrib, weights, out, rows, top_k,
                                                                     B);
  return ref_status();
}

#elif defined(REF_GPU_KERNELS)
#include "ref_gpu_kernels.cu"

REF_API int ref_gemv_bf16(const unsigned short* W, const float* x, float* out, int rows, int cols,
                          void* stream) {
  gemv_bf16<<<rows, 256, cols * 4, (cudaStream_t)stream>>>(W, x, out, rows, cols);
  return ref_status();
}

REF_API int ref_gemv_f32(const float* W, const float* x, float* out, int rows, int cols,
                         void* stream) {
  gemv_f32<<<rows, 256, cols * 4, (cudaStream_t)stream>>>(W, x, out, rows, cols);
  return ref_status();
}
#endif
