// capi.cu -- the extern "C" boundary (include/ervf_b200.h): argument checks,
// then one or two launches on the caller's stream.  No allocation, no host
// synchronisation (except ervf_device_status, which is documented as such).
#include "../../include/ervf_b200.h"

#include <atomic>
#include <cstring>

#include "aux.h"
#include "common.cuh"
#include "kernels.h"

using namespace ervf;

namespace {

inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool al(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
inline bool width_ok(int w) { return w == 0 || w == 4 || w == 8 || w == 16 || w == 32; }

// Shape limits of the NVFP4 schedules: cols % 16 == 0 and the width-32
// fallback's shared-memory footprint (activation + LUT + 8 rows of chains).
int check_nvfp4_shape(int rows, int cols, int width) {
  if (rows <= 0 || cols <= 0 || (cols & 15)) return kErrShape;
  if (!width_ok(width)) return kErrArg;
  const int rp = width ? 256 / width : 8;
  const long long smem = (long long)(cols + 256 + rp * kRowPitch) * 4;
  if (smem > device_smem_optin()) return kErrShape;
  return kOk;
}

MatRef direct(const uint8_t* c, const uint8_t* s, float g) {
  MatRef m{};
  m.codes = c;
  m.scales = s;
  m.g = g;
  return m;
}

}  // namespace

extern "C" {

int ervf_version(void) { return 100; }

int ervf_device_status(void) {
  // read and clear every unit's word; report the first error found
  const int v[6] = {read_gemv_device_error(true), read_aux_device_error(true),
                    read_tc_device_error(true), read_ep_device_error(true),
                    read_mma_device_error(true), read_token_device_error(true)};
  for (int e : v)
    if (e) return e;
  return kOk;
}

int ervf_nvfp4_gemv(const uint8_t* codes, const uint8_t* scales, const float* x, float* out,
                    float global_scale, int rows, int cols, int apply_relu2, float out_scale,
                    int width, int legacy_tree, void* stream) {
  if (!codes || !scales || !x || !out) return kErrNull;
  if (int e = check_nvfp4_shape(rows, cols, width)) return e;
  if (!al(codes, 4) || !al(x, 4) || !al(out, 4)) return kErrAlign;
  GemvBatch b{};
  b.rows = rows;
  b.cols = cols;
  b.njobs = 1;
  b.mode = 0;
  b.relu2 = apply_relu2 ? 1 : 0;
  b.out_scale = out_scale;
  b.legacy_tree = legacy_tree ? 1 : 0;
  b.job[0].mat = direct(codes, scales, global_scale);
  b.job[0].x = x;
  b.job[0].out = out;
  return launch_nvfp4_batch(b, width, S(stream));
}

int ervf_nvfp4_gemv_ind(const uint8_t* codes_base, const uint8_t* scales_base,
                        const int32_t* slot_ptr, const int32_t* id_ptr, const float* globals,
                        int gsel, const float* x, float* out, int rows, int cols, int apply_relu2,
                        float out_scale, size_t code_stride, size_t scale_stride, int width,
                        void* stream) {
  if (!codes_base || !scales_base || !slot_ptr || !id_ptr || !globals || !x || !out) return kErrNull;
  if (int e = check_nvfp4_shape(rows, cols, width)) return e;
  if (gsel < 0 || gsel > 1) return kErrArg;
  if (!al(codes_base, 4) || (code_stride & 3) || !al(x, 4) || !al(out, 4)) return kErrAlign;
  GemvBatch b{};
  b.rows = rows;
  b.cols = cols;
  b.njobs = 1;
  b.relu2 = apply_relu2 ? 1 : 0;
  b.out_scale = out_scale;
  MatRef m{};
  m.codes = codes_base;
  m.scales = scales_base;
  m.slot_ptr = slot_ptr;
  m.id_ptr = id_ptr;
  m.globals = globals;
  m.gsel = gsel;
  m.code_stride = code_stride;
  m.scale_stride = scale_stride;
  b.job[0].mat = m;
  b.job[0].x = x;
  b.job[0].out = out;
  return launch_nvfp4_batch(b, width, S(stream));
}

int ervf_nvfp4_gemv_grouped(int njobs, const uint8_t* const* codes, const uint8_t* const* scales,
                            const float* global_scales, const float* const* xs, float* const* outs,
                            int rows, int cols, int apply_relu2, float out_scale, int width,
                            void* stream) {
  if (!codes || !scales || !global_scales || !xs || !outs) return kErrNull;
  if (njobs <= 0 || njobs > kMaxJobs) return kErrShape;
  if (int e = check_nvfp4_shape(rows, cols, width)) return e;
  GemvBatch b{};
  b.rows = rows;
  b.cols = cols;
  b.njobs = njobs;
  b.relu2 = apply_relu2 ? 1 : 0;
  b.out_scale = out_scale;
  for (int j = 0; j < njobs; ++j) {
    if (!codes[j] || !scales[j] || !xs[j] || !outs[j]) return kErrNull;
    if (!al(codes[j], 4) || !al(xs[j], 4) || !al(outs[j], 4)) return kErrAlign;
    b.job[j].mat = direct(codes[j], scales[j], global_scales[j]);
    b.job[j].x = xs[j];
    b.job[j].out = outs[j];
  }
  return launch_nvfp4_batch(b, width, S(stream));
}

int ervf_weighted_accumulate(float* dst, const float* src, float weight, int n, void* stream) {
  if (!dst || !src) return kErrNull;
  if (n < 0) return kErrShape;
  if (n == 0) return kOk;
  return launch_weighted_accumulate(dst, src, weight, nullptr, n, S(stream));
}

int ervf_weighted_accumulate_ind(float* dst, const float* src, const float* w_ptr, int n,
                                 void* stream) {
  if (!dst || !src || !w_ptr) return kErrNull;
  if (n < 0) return kErrShape;
  if (n == 0) return kOk;
  return launch_weighted_accumulate(dst, src, 0.0f, w_ptr, n, S(stream));
}

int ervf_moe_up_grouped(const uint8_t* up_codes, const uint8_t* up_scales, size_t up_code_stride,
                        size_t up_scale_stride, const int32_t* ids, const float* globals, int top_k,
                        const float* x, float* act, int inter, int hidden, int width, int flags,
                        void* stream) {
  if (!up_codes || !up_scales || !ids || !globals || !x || !act) return kErrNull;
  if (top_k <= 0 || top_k > kMaxJobs) return kErrShape;
  const bool swiglu = (flags & ERVF_UP_SWIGLU) != 0;
  const int rows = swiglu ? 2 * inter : inter;
  if (int e = check_nvfp4_shape(rows, hidden, width)) return e;
  if (!al(up_codes, 4) || (up_code_stride & 3) || !al(x, 4) || !al(act, 4)) return kErrAlign;
  GemvBatch b{};
  b.rows = rows;
  b.cols = hidden;
  b.njobs = top_k;
  b.relu2 = swiglu ? 0 : 1;
  b.swiglu = swiglu ? 1 : 0;
  b.out_scale = 1.0f;
  b.pdl = (flags & ERVF_LAUNCH_PDL) ? 1 : 0;
  b.ids_ready = (flags & ERVF_LAUNCH_IDS_READY) ? 1 : 0;
  for (int s = 0; s < top_k; ++s) {
    MatRef m{};
    m.codes = up_codes;
    m.scales = up_scales;
    m.slot_ptr = ids + s;
    m.id_ptr = ids + s;
    m.globals = globals;
    m.gsel = 1;
    m.code_stride = up_code_stride;
    m.scale_stride = up_scale_stride;
    b.job[s].mat = m;
    b.job[s].x = x;
    b.job[s].out = act + (size_t)s * inter;
  }
  if (swiglu && (width != 0 || !nvfp4_tma_ok(b))) return kErrArg;  // B200 schedule only
  return launch_nvfp4_batch(b, width, S(stream));
}

int ervf_moe_down_routesum(const uint8_t* dn_codes, const uint8_t* dn_scales,
                           size_t dn_code_stride, size_t dn_scale_stride, const int32_t* ids,
                           const float* globals, const float* route_w, int top_k, const float* act,
                           const float* base, const float* resid, float* out, int hidden, int inter,
                           void* scratch, size_t scratch_bytes, int width, int flags, void* stream) {
  if (!dn_codes || !dn_scales || !ids || !globals || !route_w || !act || !out) return kErrNull;
  if (scratch && (scratch_bytes < routesum_scratch_bytes(hidden, top_k) || !al(scratch, 16)))
    return kErrArg;
  if (top_k <= 0 || top_k > kMaxJobs) return kErrShape;
  if (int e = check_nvfp4_shape(hidden, inter, width)) return e;
  if (!al(dn_codes, 4) || (dn_code_stride & 3) || !al(act, 4) || !al(out, 4)) return kErrAlign;
  GemvBatch b{};
  b.rows = hidden;
  b.cols = inter;
  b.njobs = top_k;
  b.mode = 1;
  b.out_scale = 1.0f;
  b.route_w = route_w;
  b.base = base;
  b.resid = resid;
  b.rs_out = out;
  if (scratch) {
    b.grp_count = reinterpret_cast<unsigned*>(scratch);
    b.contrib = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scratch) + routesum_counter_bytes(hidden));
  }
  b.pdl = (flags & ERVF_LAUNCH_PDL) ? 1 : 0;
  b.ids_ready = (flags & ERVF_LAUNCH_IDS_READY) ? 1 : 0;
  for (int s = 0; s < top_k; ++s) {
    MatRef m{};
    m.codes = dn_codes;
    m.scales = dn_scales;
    m.slot_ptr = ids + s;
    m.id_ptr = ids + s;
    m.globals = globals;
    m.gsel = 0;
    m.code_stride = dn_code_stride;
    m.scale_stride = dn_scale_stride;
    b.job[s].mat = m;
    b.job[s].x = act + (size_t)s * inter;
    b.job[s].out = nullptr;
  }
  return launch_nvfp4_batch(b, width, S(stream));
}

int ervf_moe_layer(const uint8_t* up_codes, const uint8_t* up_scales, size_t up_code_stride,
                   size_t up_scale_stride, const uint8_t* dn_codes, const uint8_t* dn_scales,
                   size_t dn_code_stride, size_t dn_scale_stride, const int32_t* ids,
                   const float* globals, const float* route_w, int top_k, const float* x, float* act,
                   float* out, int hidden, int inter, int n_experts, void* scratch,
                   size_t scratch_bytes, const uint8_t* next_up_codes, const uint8_t* next_up_scales,
                   const int32_t* next_ids, int flags, void* stream) {
  if (!up_codes || !up_scales || !dn_codes || !dn_scales || !ids || !globals || !route_w || !x ||
      !act || !out || !scratch)
    return kErrNull;
  if (flags & ~(ERVF_LAUNCH_PDL | ERVF_LAUNCH_IDS_READY)) return kErrArg;
  if (top_k <= 0 || top_k > kMaxJobs || n_experts <= 0) return kErrShape;
  if (hidden <= 0 || inter <= 0 || hidden % 32 || inter % 32 || hidden > 4096 || inter > 4096)
    return kErrShape;
  if (scratch_bytes < routesum_scratch_bytes(hidden, top_k)) return kErrArg;
  if ((next_up_codes != nullptr) != (next_ids != nullptr) ||
      (next_up_codes != nullptr) != (next_up_scales != nullptr))
    return kErrArg;
  const uintptr_t ptr_bits = reinterpret_cast<uintptr_t>(up_codes) | reinterpret_cast<uintptr_t>(up_scales) |
                             reinterpret_cast<uintptr_t>(dn_codes) | reinterpret_cast<uintptr_t>(dn_scales) |
                             reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(act) |
                             reinterpret_cast<uintptr_t>(scratch) |
                             reinterpret_cast<uintptr_t>(next_up_codes) |
                             reinterpret_cast<uintptr_t>(next_up_scales);
  if ((ptr_bits & 15u) || ((up_code_stride | up_scale_stride | dn_code_stride | dn_scale_stride) & 15u) ||
      !al(out, 4))
    return kErrAlign;
  const size_t up_cb = (size_t)inter * hidden / 2, up_sb = (size_t)inter * hidden / 16;
  const size_t dn_cb = up_cb, dn_sb = up_sb;
  if (up_code_stride < up_cb || up_scale_stride < up_sb || dn_code_stride < dn_cb ||
      dn_scale_stride < dn_sb)
    return kErrArg;
  const bool pdl = (flags & ERVF_LAUNCH_PDL) != 0;
  GemvBatch u{};
  u.rows = inter;
  u.cols = hidden;
  u.njobs = top_k;
  u.relu2 = 1;
  u.out_scale = 1.0f;
  u.pdl = pdl ? 1 : 0;
  u.ids_ready = (flags & ERVF_LAUNCH_IDS_READY) ? 1 : 0;
  GemvBatch d{};
  d.rows = hidden;
  d.cols = inter;
  d.njobs = top_k;
  d.mode = 1;
  d.out_scale = 1.0f;
  d.route_w = route_w;
  d.resid = x;
  d.rs_out = out;
  d.grp_count = reinterpret_cast<unsigned*>(scratch);
  d.contrib = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scratch) + routesum_counter_bytes(hidden));
  d.pdl = pdl ? 1 : 0;
  d.ids_ready = pdl ? 1 : 0;  // the up launch read the ids after its wait
  for (int s = 0; s < top_k; ++s) {
    MatRef m{};
    m.codes = up_codes;
    m.scales = up_scales;
    m.slot_ptr = ids + s;
    m.id_ptr = ids + s;
    m.globals = globals;
    m.gsel = 1;
    m.code_stride = up_code_stride;
    m.scale_stride = up_scale_stride;
    u.job[s].mat = m;
    u.job[s].x = x;
    u.job[s].out = act + (size_t)s * inter;
    m.codes = dn_codes;
    m.scales = dn_scales;
    m.gsel = 0;
    m.code_stride = dn_code_stride;
    m.scale_stride = dn_scale_stride;
    d.job[s].mat = m;
    d.job[s].x = act + (size_t)s * inter;
    d.job[s].out = nullptr;
  }
  // the up launch queues this layer's down records in L2, the down launch
  // the next layer's up records (when given)
  u.pf_codes = dn_codes;
  u.pf_scales = dn_scales;
  u.pf_code_stride = dn_code_stride;
  u.pf_scale_stride = dn_scale_stride;
  u.pf_code_bytes = dn_cb;
  u.pf_scale_bytes = dn_sb;
  u.pf_ids = ids;
  u.pf_n = top_k;
  u.pf_experts = n_experts;
  if (next_ids) {
    d.pf_codes = next_up_codes;
    d.pf_scales = next_up_scales;
    d.pf_code_stride = up_code_stride;
    d.pf_scale_stride = up_scale_stride;
    d.pf_code_bytes = up_cb;
    d.pf_scale_bytes = up_sb;
    d.pf_ids = next_ids;
    d.pf_n = top_k;
    d.pf_experts = n_experts;
  }
  if (!nvfp4_tma_ok(u) || !nvfp4_tma_ok(d)) return kErrShape;
  if (int e = launch_nvfp4_batch(u, 0, S(stream))) return e;
  return launch_nvfp4_batch(d, 0, S(stream));
}

int ervf_moe_token(const uint64_t* layer_ptrs, int n_layers, size_t up_code_stride,
                   size_t up_scale_stride, size_t dn_code_stride, size_t dn_scale_stride,
                   const int32_t* ids, const float* route_w, int top_k, int n_experts, const float* x,
                   float* out, int hidden, int inter, void* scratch, size_t scratch_bytes, int flags,
                   void* stream) {
  if (!layer_ptrs || !ids || !route_w || !x || !out || !scratch) return kErrNull;
  if (flags & ~ERVF_LAUNCH_PDL) return kErrArg;
  if (n_layers <= 0 || top_k <= 0 || top_k > kMaxJobs || n_experts <= 0) return kErrShape;
  if (hidden <= 0 || inter <= 0 || hidden % 32 || inter % 32 || hidden > 4096 || inter > 4096)
    return kErrShape;
  if (scratch_bytes < moe_token_scratch_bytes(n_layers, hidden, inter, top_k)) return kErrArg;
  if (!al(scratch, 256) || !al(x, 16) || !al(out, 4) || !al(layer_ptrs, 8) ||
      ((up_code_stride | up_scale_stride | dn_code_stride | dn_scale_stride) & 15u))
    return kErrAlign;
  const size_t cb = (size_t)inter * hidden / 2, sb = (size_t)inter * hidden / 16;
  if (up_code_stride < cb || up_scale_stride < sb || dn_code_stride < cb || dn_scale_stride < sb)
    return kErrArg;
  MoeTokenArgs a{};
  a.layer_ptrs = reinterpret_cast<const unsigned long long*>(layer_ptrs);
  a.up_code_stride = up_code_stride;
  a.up_scale_stride = up_scale_stride;
  a.dn_code_stride = dn_code_stride;
  a.dn_scale_stride = dn_scale_stride;
  a.ids = ids;
  a.route_w = route_w;
  a.x = x;
  a.out = out;
  a.n_layers = n_layers;
  a.top_k = top_k;
  a.n_experts = n_experts;
  a.hidden = hidden;
  a.inter = inter;
  a.scratch = scratch;
  a.pdl = (flags & ERVF_LAUNCH_PDL) != 0;
  return launch_moe_token(a, S(stream));
}

int ervf_moe_token_router(const uint64_t* layer_ptrs, int n_layers, size_t up_code_stride,
                          size_t up_scale_stride, size_t dn_code_stride, size_t dn_scale_stride,
                          int32_t* ids, float* route_w, int top_k, int n_experts, float scaling,
                          int bad_pick, const float* x, float* out, int hidden, int inter, void* scratch,
                          size_t scratch_bytes, int flags, void* stream) {
  if (!layer_ptrs || !ids || !route_w || !x || !out || !scratch) return kErrNull;
  if (flags & ~ERVF_LAUNCH_PDL) return kErrArg;
  if (n_layers <= 0 || top_k <= 0 || top_k > kMaxJobs || n_experts <= 0 || n_experts > 256 ||
      top_k > n_experts)
    return kErrShape;
  if (bad_pick != 0 && bad_pick != 1) return kErrArg;
  if (hidden <= 0 || inter <= 0 || hidden % 32 || inter % 32 || hidden > 4096 || inter > 4096)
    return kErrShape;
  if (scratch_bytes < moe_token_scratch_bytes(n_layers, hidden, inter, top_k)) return kErrArg;
  if (!al(scratch, 256) || !al(x, 16) || !al(out, 4) || !al(layer_ptrs, 8) || !al(ids, 4) ||
      !al(route_w, 4) || ((up_code_stride | up_scale_stride | dn_code_stride | dn_scale_stride) & 15u))
    return kErrAlign;
  const size_t cb = (size_t)inter * hidden / 2, sb = (size_t)inter * hidden / 16;
  if (up_code_stride < cb || up_scale_stride < sb || dn_code_stride < cb || dn_scale_stride < sb)
    return kErrArg;
  MoeTokenArgs a{};
  a.layer_ptrs = reinterpret_cast<const unsigned long long*>(layer_ptrs);
  a.up_code_stride = up_code_stride;
  a.up_scale_stride = up_scale_stride;
  a.dn_code_stride = dn_code_stride;
  a.dn_scale_stride = dn_scale_stride;
  a.ids = ids;
  a.route_w = route_w;
  a.x = x;
  a.out = out;
  a.n_layers = n_layers;
  a.top_k = top_k;
  a.n_experts = n_experts;
  a.hidden = hidden;
  a.inter = inter;
  a.scratch = scratch;
  a.pdl = (flags & ERVF_LAUNCH_PDL) != 0;
  a.route = true;
  a.scaling = scaling;
  a.bad_pick = bad_pick;
  return launch_moe_token(a, S(stream));
}

size_t ervf_moe_token_scratch_bytes(int n_layers, int hidden, int inter, int top_k) {
  if (n_layers <= 0 || hidden <= 0 || inter <= 0 || top_k <= 0) return 0;
  return moe_token_scratch_bytes(n_layers, hidden, inter, top_k);
}

size_t ervf_moe_token_ep_scratch_bytes(int n_layers, int hidden, int inter, int top_k) {
  if (n_layers <= 0 || hidden <= 0 || inter <= 0 || top_k <= 0) return 0;
  return moe_token_ep_scratch_bytes(n_layers, hidden, inter, top_k);
}

int ervf_moe_token_ep_prepare(void* scratch, size_t scratch_bytes, int n_layers, int hidden, int inter,
                              int top_k, void* stream) {
  if (!scratch) return kErrNull;
  if (n_layers <= 0 || hidden <= 0 || inter <= 0 || top_k <= 0) return kErrShape;
  if (scratch_bytes < moe_token_ep_scratch_bytes(n_layers, hidden, inter, top_k)) return kErrArg;
  if (!al(scratch, 256)) return kErrAlign;
  return prepare_moe_token_ep(scratch, n_layers, hidden, inter, top_k, S(stream));
}

int ervf_moe_token_ep(const uint64_t* layer_ptrs, int n_layers, size_t up_code_stride,
                      size_t up_scale_stride, size_t dn_code_stride, size_t dn_scale_stride,
                      const int32_t* ids, const float* route_w, int top_k, int n_experts,
                      const float* x, float* out, int hidden, int inter, const uint64_t* peer_scratch,
                      int ep_ranks, int ep_rank, size_t scratch_bytes, int timeout_ms, int flags,
                      void* stream) {
  if (!layer_ptrs || !ids || !route_w || !x || !out || !peer_scratch) return kErrNull;
  if (flags & ~ERVF_LAUNCH_PDL) return kErrArg;
  if (ep_ranks < 2 || ep_ranks > 8 || ep_rank < 0 || ep_rank >= ep_ranks || timeout_ms <= 0)
    return kErrArg;
  if (n_layers <= 0 || top_k <= 0 || top_k > kMaxJobs || n_experts <= 0) return kErrShape;
  if (hidden <= 0 || inter <= 0 || hidden % 32 || inter % 32 || hidden > 4096 || inter > 4096)
    return kErrShape;
  if (scratch_bytes < moe_token_ep_scratch_bytes(n_layers, hidden, inter, top_k)) return kErrArg;
  for (int q = 0; q < ep_ranks; ++q) {
    if (!peer_scratch[q]) return kErrNull;
    if (peer_scratch[q] & 255u) return kErrAlign;
  }
  if (!al(x, 16) || !al(out, 4) || !al(layer_ptrs, 8) ||
      ((up_code_stride | up_scale_stride | dn_code_stride | dn_scale_stride) & 15u))
    return kErrAlign;
  const size_t cb = (size_t)inter * hidden / 2, sb = (size_t)inter * hidden / 16;
  if (up_code_stride < cb || up_scale_stride < sb || dn_code_stride < cb || dn_scale_stride < sb)
    return kErrArg;
  MoeTokenArgs a{};
  a.layer_ptrs = reinterpret_cast<const unsigned long long*>(layer_ptrs);
  a.up_code_stride = up_code_stride;
  a.up_scale_stride = up_scale_stride;
  a.dn_code_stride = dn_code_stride;
  a.dn_scale_stride = dn_scale_stride;
  a.ids = ids;
  a.route_w = route_w;
  a.x = x;
  a.out = out;
  a.n_layers = n_layers;
  a.top_k = top_k;
  a.n_experts = n_experts;
  a.hidden = hidden;
  a.inter = inter;
  a.scratch = reinterpret_cast<void*>(peer_scratch[ep_rank]);
  a.pdl = (flags & ERVF_LAUNCH_PDL) != 0;
  a.ep_ranks = ep_ranks;
  a.ep_rank = ep_rank;
  a.peers = reinterpret_cast<const unsigned long long*>(peer_scratch);
  a.timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
  return launch_moe_token(a, S(stream));
}

size_t ervf_routesum_scratch_bytes(int hidden, int top_k) {
  if (hidden <= 0 || top_k <= 0) return 0;
  return routesum_scratch_bytes(hidden, top_k);
}

int ervf_ep_expert_slots(const uint8_t* up_codes, const uint8_t* up_scales, size_t up_code_stride,
                         size_t up_scale_stride, const uint8_t* dn_codes, const uint8_t* dn_scales,
                         size_t dn_code_stride, size_t dn_scale_stride, const int32_t* ids,
                         const float* globals, int top_k, const float* x, float* act,
                         float* contrib, int hidden, int inter, int ep_ranks, int ep_rank,
                         int width, void* stream) {
  return ervf_ep_expert_slots_ex(up_codes, up_scales, up_code_stride, up_scale_stride, dn_codes,
                                 dn_scales, dn_code_stride, dn_scale_stride, ids, globals, top_k, x,
                                 act, contrib, hidden, inter, ep_ranks, ep_rank, width, 0, stream);
}

int ervf_ep_expert_slots_ex(const uint8_t* up_codes, const uint8_t* up_scales,
                            size_t up_code_stride, size_t up_scale_stride,
                            const uint8_t* dn_codes, const uint8_t* dn_scales,
                            size_t dn_code_stride, size_t dn_scale_stride, const int32_t* ids,
                            const float* globals, int top_k, const float* x, float* act,
                            float* contrib, int hidden, int inter, int ep_ranks, int ep_rank,
                            int width, int flags, void* stream) {
  if (!up_codes || !up_scales || !dn_codes || !dn_scales || !ids || !globals || !x || !act || !contrib)
    return kErrNull;
  if (top_k <= 0 || top_k > kMaxJobs || ep_ranks < 1 || ep_rank < 0 || ep_rank >= ep_ranks)
    return kErrShape;
  if (int e = check_nvfp4_shape(inter, hidden, width)) return e;
  if (int e = check_nvfp4_shape(hidden, inter, width)) return e;
  if (!al(up_codes, 4) || !al(dn_codes, 4) || (up_code_stride & 3) || (dn_code_stride & 3) ||
      !al(x, 4) || !al(act, 4) || !al(contrib, 4))
    return kErrAlign;
  if (flags & ~(ERVF_LAUNCH_PDL | ERVF_LAUNCH_IDS_READY)) return kErrArg;
  GemvBatch b{};
  b.njobs = top_k;
  b.out_scale = 1.0f;
  b.pdl = (flags & ERVF_LAUNCH_PDL) ? 1 : 0;
  b.ids_ready = (flags & ERVF_LAUNCH_IDS_READY) ? 1 : 0;
  b.ep_ids = ids;
  b.ep_ranks = ep_ranks;
  b.ep_rank = ep_rank;
  b.rows = inter;
  b.cols = hidden;
  b.relu2 = 1;
  for (int s = 0; s < top_k; ++s) {
    MatRef m{};
    m.codes = up_codes;
    m.scales = up_scales;
    m.slot_ptr = ids + s;
    m.id_ptr = ids + s;
    m.globals = globals;
    m.gsel = 1;
    m.code_stride = up_code_stride;
    m.scale_stride = up_scale_stride;
    b.job[s].mat = m;
    b.job[s].x = x;
    b.job[s].out = act + (size_t)s * inter;
  }
  if (int e = launch_nvfp4_batch(b, width, S(stream))) return e;
  b.rows = hidden;
  b.cols = inter;
  b.relu2 = 0;
  if (b.pdl) b.ids_ready = 1;  // ids were complete before the up launch began
  for (int s = 0; s < top_k; ++s) {
    MatRef& m = b.job[s].mat;
    m.codes = dn_codes;
    m.scales = dn_scales;
    m.gsel = 0;
    m.code_stride = dn_code_stride;
    m.scale_stride = dn_scale_stride;
    b.job[s].x = act + (size_t)s * inter;
    b.job[s].out = contrib + (size_t)s * hidden;
  }
  return launch_nvfp4_batch(b, width, S(stream));
}

int ervf_ep_route_sum(const float* gathered, const int32_t* ids, const float* route_w, int top_k,
                      const float* x, float* out, int hidden, int ep_ranks, void* stream) {
  if (!gathered || !ids || !route_w || !out) return kErrNull;
  if (top_k <= 0 || hidden <= 0 || ep_ranks < 1) return kErrShape;
  return launch_ep_route_sum(gathered, ids, route_w, top_k, x, out, hidden, ep_ranks, S(stream));
}

int ervf_down_masked(float* out, const uint8_t* bank, const float* act, uint32_t* masks,
                     int32_t* plist, int32_t* pcount, int32_t* nz, int32_t* nzc,
                     float global_scale, int hidden, int inter, int nchunks, void* stream) {
  if (!out || !bank || !act || !masks || !plist || !pcount || !nz || !nzc) return kErrNull;
  if (hidden <= 0 || (hidden & 1) || inter <= 0 || (inter & 15) || inter > 65536) return kErrShape;
  if (nchunks <= 0 || nchunks > 32) return kErrArg;
  return launch_down_masked(bank, act, masks, plist, pcount, nz, nzc, global_scale, nullptr,
                            nullptr, 0, out, hidden, inter, nchunks, S(stream));
}

int ervf_down_masked_ind(float* out, const uint8_t* down_base, const int32_t* id_ptr,
                         size_t panel_bytes, const float* globals, const float* act,
                         uint32_t* masks, int32_t* plist, int32_t* pcount, int32_t* nz,
                         int32_t* nzc, int hidden, int inter, int nchunks, void* stream) {
  if (!out || !down_base || !id_ptr || !globals || !act || !masks || !plist || !pcount || !nz || !nzc)
    return kErrNull;
  if (hidden <= 0 || (hidden & 1) || inter <= 0 || (inter & 15) || inter > 65536) return kErrShape;
  if (nchunks <= 0 || nchunks > 32) return kErrArg;
  return launch_down_masked(down_base, act, masks, plist, pcount, nz, nzc, 0.0f, id_ptr, globals,
                            panel_bytes, out, hidden, inter, nchunks, S(stream));
}

int ervf_panel_major(const uint8_t* codes, const uint8_t* scales, uint8_t* block, int rows,
                     int inter, void* stream) {
  if (!codes || !scales || !block) return kErrNull;
  if (rows <= 0 || (rows & 1) || inter <= 0 || (inter & 15)) return kErrShape;
  return launch_panel_major(codes, scales, block, rows, inter, S(stream));
}

int ervf_bf16_gemv(const uint16_t* W, const float* x, float* out, int rows, int cols, int batch,
                   void* stream) {
  if (!W || !x || !out) return kErrNull;
  if (rows <= 0 || cols <= 0 || (cols & 7)) return kErrShape;
  if (batch < 1 || batch > 8) return kErrArg;
  if (!al(W, 16) || !al(x, 16) || !al(out, 4)) return kErrAlign;
  return launch_bf16_gemv(W, x, out, rows, cols, batch, S(stream));
}

int ervf_nvfp4_gemm_rows_b(const uint8_t* codes, const uint8_t* scales, const float* x,
                           const int32_t* nodes, float* out, float global_scale, int rows, int cols,
                           int n, int apply_relu2, float* xbuf, void* stream) {
  if (!codes || !scales || !x || !nodes || !out || !xbuf) return kErrNull;
  if (n < 1 || n > kMaxJobs) return kErrShape;
  if (int e = check_nvfp4_shape(rows, cols, 0)) return e;
  if (!al(codes, 4) || !al(x, 4) || !al(out, 4) || !al(xbuf, 16)) return kErrAlign;
  if (int e = launch_gather_rows(x, nodes, n, cols, xbuf, S(stream))) return e;
  GemvBatch b{};
  b.rows = rows;
  b.cols = cols;
  b.njobs = n;
  b.relu2 = apply_relu2 ? 1 : 0;
  b.out_scale = 1.0f;
  b.legacy_tree = 1;  // the reference's batched kernel keeps gemv_nvfp4_rows' tree per column
  for (int j = 0; j < n; ++j) {
    b.job[j].mat = direct(codes, scales, global_scale);
    b.job[j].x = xbuf + (size_t)j * cols;
    b.job[j].out = out + (size_t)j * rows;
  }
  return launch_nvfp4_batch(b, 0, S(stream));
}

int ervf_down_union(const uint8_t* bank, const float* acts, int n, const int32_t* dst, float* contrib,
                    float global_scale, int hidden, int inter, int nchunks, float* act_sum,
                    uint32_t* masks, int32_t* plist, int32_t* pcount, int32_t* nz, int32_t* nzc,
                    float* tmp, void* stream) {
  if (!bank || !acts || !dst || !contrib || !act_sum || !masks || !plist || !pcount || !nz || !nzc || !tmp)
    return kErrNull;
  if (n < 1 || n > 64 || hidden <= 0 || (hidden & 1) || inter <= 0 || (inter & 15) || inter > 65536)
    return kErrShape;
  if (nchunks <= 0 || nchunks > 32) return kErrArg;
  if (int e = launch_down_union(bank, acts, n, act_sum, masks, plist, pcount, nz, nzc, global_scale, tmp,
                                hidden, inter, nchunks, S(stream)))
    return e;
  return launch_scatter_rows(tmp, dst, n, hidden, contrib, S(stream));
}

int ervf_reduce_slots(const float* contrib, const float* weights, float* out, int rows, int top_k, int B,
                      void* stream) {
  if (!contrib || !weights || !out) return kErrNull;
  if (rows <= 0 || top_k <= 0 || B <= 0 || B > 65535) return kErrShape;
  return launch_reduce_slots(contrib, weights, out, rows, top_k, B, S(stream));
}

int ervf_route_topk(const float* rlog, const float* gate_b, int32_t* ids, float* w, int n,
                    int top_k, float scaling, int bad_pick, void* stream) {
  if (!rlog || !gate_b || !ids || !w) return kErrNull;
  if (n <= 0 || n > 1024 || top_k <= 0 || top_k > 64 || top_k > n) return kErrShape;
  return launch_route_topk(rlog, gate_b, ids, w, n, top_k, scaling, bad_pick, S(stream));
}

int ervf_route_topk_batched(const float* rlog, const float* gate_b, int32_t* ids, float* w,
                            int layers, int n, int top_k, float scaling, int bad_pick,
                            int bias_stride, void* stream) {
  if (!rlog || !ids || !w) return kErrNull;
  if (layers <= 0 || n <= 0 || n > 1024 || top_k <= 0 || top_k > 64 || top_k > n || bias_stride < 0)
    return kErrShape;
  if (n > 256 && !gate_b) return kErrNull;
  return launch_route_topk_batched(rlog, gate_b, ids, w, layers, n, top_k, scaling, bad_pick,
                                   bias_stride, S(stream));
}

int ervf_route_topk_softmax(const float* rlog, int32_t* ids, float* w, int layers, int n,
                            int top_k, void* stream) {
  if (!rlog || !ids || !w) return kErrNull;
  if (layers <= 0 || n <= 0 || n > 1024 || top_k <= 0 || top_k > 32 || top_k > n) return kErrShape;
  return launch_route_topk_softmax(rlog, ids, w, layers, n, top_k, S(stream));
}

namespace {
constexpr int kTcMaxSplits = 4;
struct TcScratch {
  uint8_t* panel;
  float* part;
  unsigned* ucnt;
  size_t bytes;
};
TcScratch tc_scratch(void* base, int rows, int cols, int n) {
  TcScratch t{};
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  const size_t pan = mma_panel_bytes(1, cols);
  const size_t part = (size_t)kTcMaxSplits * n * rows * sizeof(float);
  const size_t cnt = ((size_t)(rows + 127) / 128 * sizeof(unsigned) + 15) / 16 * 16;
  t.panel = p;
  t.part = reinterpret_cast<float*>(p + pan);
  t.ucnt = reinterpret_cast<unsigned*>(p + pan + part);
  t.bytes = pan + part + cnt;
  return t;
}
}  // namespace

size_t ervf_nvfp4_gemm_tc_scratch_bytes(int rows, int cols, int n) {
  if (rows <= 0 || cols <= 0 || n <= 0) return 0;
  return tc_scratch(nullptr, rows, cols, n).bytes;
}

int ervf_nvfp4_gemm_tc(const uint8_t* codes, const uint8_t* scales, float global_scale,
                       const float* x, float* out, int rows, int cols, int n, void* scratch,
                       size_t scratch_bytes, void* stream) {
  if (!codes || !scales || !x || !out || !scratch) return kErrNull;
  if (rows <= 0 || cols <= 0 || cols % 32 || cols > 4096 || n < 1 || n > 16) return kErrShape;
  if (!al(codes, 16) || !al(scales, 16) || !al(x, 16) || !al(out, 4) || !al(scratch, 16)) return kErrAlign;
  const TcScratch t = tc_scratch(scratch, rows, cols, n);
  if (scratch_bytes < t.bytes) return kErrArg;
  if (int e = launch_pack_panel(x, cols, nullptr, nullptr, nullptr, nullptr, 1, n, t.panel, S(stream)))
    return e;
  return launch_nvfp4_mma_single(codes, scales, global_scale, t.panel, out, rows, cols, n, t.part, t.ucnt,
                                 kTcMaxSplits, S(stream));
}

int ervf_bf16_gemm_tc(const uint16_t* W, const float* x, float* out, int rows, int cols, int batch,
                      void* stream) {
  if (!W || !x || !out) return kErrNull;
  if (rows <= 0 || cols <= 0 || cols % 32 || batch < 1 || batch > 8) return kErrShape;
  if (!al(W, 16) || !al(x, 16) || !al(out, 4)) return kErrAlign;
  return launch_bf16_gemm_tc(W, x, out, rows, cols, batch, S(stream));
}

namespace {
struct BatchScratch {
  int *chunk_expert, *chunk_off, *chunk_n, *n_chunks, *tok_sorted, *pos;
  uint8_t *up_panel, *dn_panel;  // f16 activation panels of the up / down launches
  float* contrib;
  float* part;     // K-split partial accumulators [2][pairs][max(hidden, inter)]
  unsigned* ucnt;  // K-split unit counters [pairs][ceil(max(hidden, inter) / 128)]
  size_t ucnt_bytes;
  size_t bytes;
};
constexpr int kMaxKsplit = 2;
BatchScratch batch_scratch(void* base, int pairs, int hidden, int inter) {
  BatchScratch b{};
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  const size_t ints = ((size_t)5 * pairs + 4 + 3) / 4 * 4;
  int* ip = reinterpret_cast<int*>(p);
  b.chunk_expert = ip;
  b.chunk_off = ip + pairs;
  b.chunk_n = ip + 2 * (size_t)pairs;
  b.tok_sorted = ip + 3 * (size_t)pairs;
  b.pos = ip + 4 * (size_t)pairs;
  b.n_chunks = ip + 5 * (size_t)pairs;
  size_t o = ints * 4;
  b.up_panel = p + o;
  o += mma_panel_bytes(pairs, hidden);
  b.dn_panel = p + o;
  o += mma_panel_bytes(pairs, inter);
  b.contrib = reinterpret_cast<float*>(p + o);
  o += (size_t)pairs * hidden * 4;
  // rows of the tensor-core launches: hidden (down), inter or 2*inter (up, SwiGLU)
  const size_t rmax = (size_t)(hidden > 2 * inter ? hidden : 2 * inter);
  b.part = reinterpret_cast<float*>(p + o);
  o += (size_t)kMaxKsplit * pairs * rmax * 4;
  b.ucnt = reinterpret_cast<unsigned*>(p + o);
  b.ucnt_bytes = (size_t)pairs * ((rmax + 127) / 128) * 4;
  b.bytes = o + b.ucnt_bytes;
  return b;
}

// Lists, activation panels, up and down of the batched block: contrib[pos[p]]
// = the down output of pair p for the pairs whose expert this rank owns (all
// with ep_ranks 1).  SwiGLU: the up records hold 2*inter rows (gate / up
// interleaved).
int batch_slots(const uint8_t* up_codes, const uint8_t* up_scales, const uint8_t* dn_codes,
                const uint8_t* dn_scales, const float* globals, const int32_t* ids, int pairs,
                int top_k, int n_experts, const float* x, int hidden, int inter, bool swiglu,
                const BatchScratch& b, float* contrib, int ep_ranks, int ep_rank, int ksplit,
                cudaStream_t st) {
  if (ksplit > 1 && cudaMemsetAsync(b.ucnt, 0, b.ucnt_bytes, st) != cudaSuccess) return kErrLaunch;
  if (int e = launch_moe_batch_lists(ids, pairs, top_k, n_experts, b.chunk_expert, b.chunk_off, b.chunk_n,
                                     b.n_chunks, b.tok_sorted, b.pos, ep_ranks, ep_rank, st))
    return e;
  if (int e = launch_pack_panel(x, hidden, b.tok_sorted, b.chunk_off, b.chunk_n, b.n_chunks, pairs, 0,
                                b.up_panel, st))
    return e;
  MmaGrouped g{};
  g.chunk_expert = b.chunk_expert;
  g.chunk_off = b.chunk_off;
  g.chunk_n = b.chunk_n;
  g.n_chunks = b.n_chunks;
  g.max_chunks = pairs;
  g.max_pairs = pairs;
  g.n_experts = n_experts;
  g.globals = globals;
  g.ksplit = ksplit;
  g.part = b.part;
  g.ucnt = b.ucnt;
  // up: relu(g_up * W_up x)^2 (or SwiGLU) as f16 into the down panels
  g.codes = up_codes;
  g.scales = up_scales;
  g.rows = swiglu ? 2 * inter : inter;
  g.cols = hidden;
  g.gsel = 1;
  g.panel = b.up_panel;
  g.down = 0;
  g.relu2 = swiglu ? 0 : 1;
  g.swiglu = swiglu ? 1 : 0;
  g.panel_out = b.dn_panel;
  if (int e = launch_nvfp4_mma_grouped(g, st)) return e;
  // down: contrib[q] = g_down * W_down act[q]
  g.codes = dn_codes;
  g.scales = dn_scales;
  g.rows = hidden;
  g.cols = inter;
  g.gsel = 0;
  g.panel = b.dn_panel;
  g.down = 1;
  g.relu2 = 0;
  g.swiglu = 0;
  g.panel_out = nullptr;
  g.out = contrib;
  return launch_nvfp4_mma_grouped(g, st);
}

int check_batched(const uint8_t* up_codes, const uint8_t* up_scales, size_t up_code_stride,
                  size_t up_scale_stride, const uint8_t* dn_codes, const uint8_t* dn_scales,
                  size_t dn_code_stride, size_t dn_scale_stride, const float* x, int tokens,
                  int top_k, int n_experts, int hidden, int inter, int up_rows, const void* scratch,
                  size_t scratch_bytes) {
  const int pairs = tokens * top_k;
  if (tokens <= 0 || top_k <= 0 || top_k > kMaxJobs || pairs > 4096 || n_experts <= 0 ||
      n_experts > kMaxBatchExperts)
    return kErrShape;
  if (hidden <= 0 || inter <= 0 || hidden % 32 || inter % 32 || hidden > 4096 || inter > 4096)
    return kErrShape;
  if (scratch_bytes < batch_scratch(nullptr, pairs, hidden, inter).bytes) return kErrArg;
  if (n_experts * (size_t)up_rows > 0x7FFFFFFF || n_experts * (size_t)hidden > 0x7FFFFFFF) return kErrShape;
  if (!al(up_codes, 16) || !al(dn_codes, 16) || !al(up_scales, 16) || !al(dn_scales, 16) || !al(x, 16) ||
      !al(scratch, 16))
    return kErrAlign;
  // the tensor-core path reads each bank as one [n_experts * rows][cols] matrix
  const size_t urows = (size_t)(up_rows), drows = (size_t)hidden;
  if (up_code_stride != urows * hidden / 2 || up_scale_stride != urows * hidden / 16 ||
      dn_code_stride != drows * inter / 2 || dn_scale_stride != drows * inter / 16)
    return kErrArg;
  if ((up_scale_stride | dn_scale_stride) & 15u) return kErrAlign;
  return kOk;
}
}  // namespace

size_t ervf_moe_batched_scratch_bytes(int tokens, int top_k, int hidden, int inter) {
  if (tokens <= 0 || top_k <= 0 || hidden <= 0 || inter <= 0) return 0;
  return batch_scratch(nullptr, tokens * top_k, hidden, inter).bytes;
}

int ervf_moe_batched(const uint8_t* up_codes, const uint8_t* up_scales, size_t up_code_stride,
                     size_t up_scale_stride, const uint8_t* dn_codes, const uint8_t* dn_scales,
                     size_t dn_code_stride, size_t dn_scale_stride, const float* globals,
                     const int32_t* ids, const float* route_w, int tokens, int top_k, int n_experts,
                     const float* x, float* out, int hidden, int inter, void* scratch,
                     size_t scratch_bytes, void* stream) {
  return ervf_moe_batched_ex(up_codes, up_scales, up_code_stride, up_scale_stride, dn_codes,
                             dn_scales, dn_code_stride, dn_scale_stride, globals, ids, route_w,
                             tokens, top_k, n_experts, x, out, hidden, inter, 1, 0, scratch,
                             scratch_bytes, stream);
}

int ervf_moe_batched_ex(const uint8_t* up_codes, const uint8_t* up_scales, size_t up_code_stride,
                        size_t up_scale_stride, const uint8_t* dn_codes, const uint8_t* dn_scales,
                        size_t dn_code_stride, size_t dn_scale_stride, const float* globals,
                        const int32_t* ids, const float* route_w, int tokens, int top_k,
                        int n_experts, const float* x, float* out, int hidden, int inter,
                        int ksplit, int flags, void* scratch, size_t scratch_bytes, void* stream) {
  if (ksplit < 1 || ksplit > kMaxKsplit || (flags & ~ERVF_UP_SWIGLU)) return kErrArg;
  if (!up_codes || !up_scales || !dn_codes || !dn_scales || !globals || !ids || !route_w || !x ||
      !out || !scratch)
    return kErrNull;
  const bool swiglu = (flags & ERVF_UP_SWIGLU) != 0;
  if (int e = check_batched(up_codes, up_scales, up_code_stride, up_scale_stride, dn_codes, dn_scales,
                            dn_code_stride, dn_scale_stride, x, tokens, top_k, n_experts, hidden,
                            inter, swiglu ? 2 * inter : inter, scratch, scratch_bytes))
    return e;
  const int pairs = tokens * top_k;
  const BatchScratch b = batch_scratch(scratch, pairs, hidden, inter);
  cudaStream_t st = S(stream);
  if (int e = batch_slots(up_codes, up_scales, dn_codes, dn_scales, globals, ids, pairs, top_k, n_experts, x,
                          hidden, inter, swiglu, b, b.contrib, 1, 0, ksplit, st))
    return e;
  return launch_moe_batch_routesum(b.contrib, b.pos, route_w, x, out, tokens, hidden, top_k, st);
}

int ervf_moe_batched_ep_slots(const uint8_t* up_codes, const uint8_t* up_scales,
                              size_t up_code_stride, size_t up_scale_stride,
                              const uint8_t* dn_codes, const uint8_t* dn_scales,
                              size_t dn_code_stride, size_t dn_scale_stride, const float* globals,
                              const int32_t* ids, int tokens, int top_k, int n_experts,
                              const float* x, float* slots, int hidden, int inter, int ep_ranks,
                              int ep_rank, void* scratch, size_t scratch_bytes, void* stream) {
  return ervf_moe_batched_ep_slots_ex(up_codes, up_scales, up_code_stride, up_scale_stride,
                                      dn_codes, dn_scales, dn_code_stride, dn_scale_stride, globals,
                                      ids, tokens, top_k, n_experts, x, slots, hidden, inter,
                                      ep_ranks, ep_rank, 1, scratch, scratch_bytes, stream);
}

int ervf_moe_batched_ep_slots_ex(const uint8_t* up_codes, const uint8_t* up_scales,
                                 size_t up_code_stride, size_t up_scale_stride,
                                 const uint8_t* dn_codes, const uint8_t* dn_scales,
                                 size_t dn_code_stride, size_t dn_scale_stride,
                                 const float* globals, const int32_t* ids, int tokens, int top_k,
                                 int n_experts, const float* x, float* slots, int hidden,
                                 int inter, int ep_ranks, int ep_rank, int ksplit, void* scratch,
                                 size_t scratch_bytes, void* stream) {
  if (ksplit < 1 || ksplit > kMaxKsplit) return kErrArg;
  if (!up_codes || !up_scales || !dn_codes || !dn_scales || !globals || !ids || !x || !slots ||
      !scratch)
    return kErrNull;
  if (ep_ranks < 1 || ep_ranks > kEpMaxRanks || ep_rank < 0 || ep_rank >= ep_ranks) return kErrShape;
  if (int e = check_batched(up_codes, up_scales, up_code_stride, up_scale_stride, dn_codes, dn_scales,
                            dn_code_stride, dn_scale_stride, x, tokens, top_k, n_experts, hidden,
                            inter, inter, scratch, scratch_bytes))
    return e;
  if (!al(slots, 16)) return kErrAlign;
  const BatchScratch b = batch_scratch(scratch, tokens * top_k, hidden, inter);
  return batch_slots(up_codes, up_scales, dn_codes, dn_scales, globals, ids, tokens * top_k, top_k,
                     n_experts, x, hidden, inter, false, b, slots, ep_ranks, ep_rank, ksplit, S(stream));
}

int ervf_ep_batch_exchange_route_sum(const uint64_t* peers, int nranks, int rank, int buf,
                                     const int32_t* ids, const float* route_w, int tokens,
                                     int top_k, const float* x, float* out, int hidden, int inter,
                                     const void* scratch, size_t scratch_bytes, int timeout_ms,
                                     void* stream) {
  if (!peers || !ids || !route_w || !out || !scratch) return kErrNull;
  const int pairs = tokens * top_k;
  if (nranks < 1 || nranks > kEpMaxRanks || rank < 0 || rank >= nranks) return kErrShape;
  if (tokens <= 0 || top_k <= 0 || top_k > kMaxJobs || pairs > 4096 || hidden <= 0 || hidden % 4 ||
      inter <= 0)
    return kErrShape;
  if (buf < 0 || buf >= kEpBufs || timeout_ms <= 0 || timeout_ms > 600000) return kErrArg;
  const BatchScratch b = batch_scratch(const_cast<void*>(scratch), pairs, hidden, inter);
  if (scratch_bytes < b.bytes) return kErrArg;
  if (!al(peers, 8) || !al(out, 16) || (x && !al(x, 16))) return kErrAlign;
  EpBatchExchange a{};
  a.peers = peers;
  a.nranks = nranks;
  a.rank = rank;
  a.buf = buf;
  a.tokens = tokens;
  a.top_k = top_k;
  a.hidden = hidden;
  a.ids = ids;
  a.pos = b.pos;
  a.route_w = route_w;
  a.x = x;
  a.out = out;
  a.timeout_ns = (uint64_t)timeout_ms * 1000000ull;
  return launch_ep_batch_exchange_sum(a, S(stream));
}

size_t ervf_ep_region_bytes(int hidden, int slots) {
  if (hidden <= 0 || slots <= 0 || slots > 4096) return 0;
  return ep_region_bytes(hidden, slots);
}

int ervf_ep_region_alloc(size_t bytes, void** region, void* ipc_handle) {
  if (!region || !ipc_handle) return kErrNull;
  if (bytes <= kEpSlotsOffset) return kErrShape;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    return kErrDevice;
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    (void)cudaGetLastError();
    cudaFree(p);
    return kErrDevice;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *region = p;
  return kOk;
}

int ervf_ep_region_open(const void* ipc_handle, void** region) {
  if (!ipc_handle || !region) return kErrNull;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    (void)cudaGetLastError();
    return kErrDevice;
  }
  *region = p;
  return kOk;
}

int ervf_ep_region_close(void* region) {
  if (!region) return kErrNull;
  if (cudaIpcCloseMemHandle(region) != cudaSuccess) {
    (void)cudaGetLastError();
    return kErrDevice;
  }
  return kOk;
}

int ervf_ep_region_free(void* region) {
  if (!region) return kErrNull;
  if (cudaFree(region) != cudaSuccess) {
    (void)cudaGetLastError();
    return kErrDevice;
  }
  return kOk;
}

int ervf_ep_exchange_route_sum(const uint64_t* peers, int nranks, int rank, int buf,
                               const int32_t* ids, const float* route_w, int top_k, const float* x,
                               float* out, int hidden, int timeout_ms, int flags, void* stream) {
  if (!peers || !ids || !route_w || !out) return kErrNull;
  if (nranks < 1 || nranks > kEpMaxRanks || rank < 0 || rank >= nranks) return kErrShape;
  if (top_k <= 0 || top_k > kMaxJobs || hidden <= 0 || hidden % 4) return kErrShape;
  if (buf < 0 || buf >= kEpBufs || timeout_ms <= 0 || timeout_ms > 600000) return kErrArg;
  if (flags & ~ERVF_LAUNCH_PDL) return kErrArg;
  if (!al(peers, 8) || !al(out, 16) || (x && !al(x, 16))) return kErrAlign;
  EpExchange a{};
  a.peers = peers;
  a.nranks = nranks;
  a.rank = rank;
  a.buf = buf;
  a.top_k = top_k;
  a.hidden = hidden;
  a.ids = ids;
  a.route_w = route_w;
  a.x = x;
  a.out = out;
  a.timeout_ns = (uint64_t)timeout_ms * 1000000ull;
  return launch_ep_exchange_sum(a, (flags & ERVF_LAUNCH_PDL) != 0, S(stream));
}

int ervf_f32_gemv(const float* W, const float* x, float* out, int rows, int cols, void* stream) {
  if (!W || !x || !out) return kErrNull;
  if (rows <= 0 || cols <= 0 || cols % 4) return kErrShape;
  if (!al(W, 16) || !al(x, 16) || !al(out, 4)) return kErrAlign;
  return launch_f32_gemv(W, x, out, rows, cols, S(stream));
}

int ervf_route_gemv_topk(const float* gate_w, const float* x, float* rlog, const float* gate_b,
                         int32_t* ids, float* w, int n, int hidden, int top_k, float scaling,
                         int bad_pick, int32_t* counter, int flags, void* stream) {
  if (!gate_w || !x || !rlog || !ids || !w || !counter) return kErrNull;
  if (n <= 0 || n > 256 || hidden <= 0 || hidden % 4 || top_k <= 0 || top_k > 64 || top_k > n)
    return kErrShape;
  if (flags & ~ERVF_LAUNCH_PDL) return kErrArg;
  if (!al(gate_w, 16) || !al(x, 16) || !al(rlog, 4) || !al(counter, 4)) return kErrAlign;
  return launch_route_gemv_topk(gate_w, x, rlog, gate_b, ids, w, n, hidden, top_k, scaling, bad_pick,
                                reinterpret_cast<unsigned*>(counter), (flags & ERVF_LAUNCH_PDL) != 0,
                                S(stream));
}

int ervf_cache_assign(int32_t* slot_of, int32_t* expert_of, int32_t* last_used, int32_t* state2,
                      const int32_t* ids, int32_t* slots, int32_t* need, int32_t* stats2, int cap,
                      int top_k, void* stream) {
  if (!slot_of || !expert_of || !last_used || !state2 || !ids || !slots || !need || !stats2)
    return kErrNull;
  if (cap <= 0 || top_k <= 0) return kErrShape;
  return launch_cache_assign(slot_of, expert_of, last_used, state2, ids, slots, need, stats2, cap,
                             top_k, S(stream));
}

int ervf_cache_fetch(const uint8_t* bank_c, const uint8_t* bank_s, uint8_t* cache_c,
                     uint8_t* cache_s, const int32_t* ids, const int32_t* slots,
                     const int32_t* need, size_t code_bytes, size_t scale_bytes, int top_k,
                     void* stream) {
  if (!bank_c || !bank_s || !cache_c || !cache_s || !ids || !slots || !need) return kErrNull;
  if (top_k <= 0 || top_k > 65535) return kErrShape;
  return launch_cache_fetch(bank_c, bank_s, cache_c, cache_s, ids, slots, need, code_bytes,
                            scale_bytes, top_k, S(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free routed sum (no counterpart in the reference).
//
// The scratch of the spread-rows routed sum (contrib[top_k][hidden] floats +
// the 32-row group counters) lives in this file-scope device array instead
// of a caller buffer.  Limits: hidden <= kStaticRows, top_k <= kStaticJobs
// (294,912 bytes).  Its device address is looked up once per device, with
// that device current, on the first call.  Every call clears the group
// counters on the stream (cudaMemsetAsync; no allocation) before the launch.
// All calls on one device share the array: calls that overlap on the GPU race.

namespace {

constexpr int kStaticRows = 8192;
constexpr int kStaticJobs = 8;
constexpr size_t kStaticScratchBytes =
    (size_t)kStaticRows * sizeof(int) + (size_t)kStaticJobs * kStaticRows * sizeof(float);

static __device__ __align__(256) unsigned char g_routesum_static[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_static_addr[kMaxDevices];

// Device address of g_routesum_static on the current device (cached).
void* static_scratch() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return nullptr;
  void* p = g_static_addr[d].load(std::memory_order_acquire);
  if (!p) {
    if (cudaGetSymbolAddress(&p, g_routesum_static) != cudaSuccess) return nullptr;
    g_static_addr[d].store(p, std::memory_order_release);
  }
  return p;
}

}  // namespace

extern "C" {

int ervf_moe_down_routesum_static(const uint8_t* dn_codes, const uint8_t* dn_scales,
                                  size_t dn_code_stride, size_t dn_scale_stride,
                                  const int32_t* ids, const float* globals, const float* route_w,
                                  int top_k, const float* act, const float* base,
                                  const float* resid, float* out, int hidden, int inter,
                                  int width, int flags, void* stream) {
  if (hidden > kStaticRows || top_k > kStaticJobs) return ERVF_ERR_SCRATCH_LIMIT;
  if (!dn_codes || !dn_scales || !ids || !globals || !route_w || !act || !out) return kErrNull;
  if (top_k <= 0 || hidden <= 0) return kErrShape;
  void* scratch = static_scratch();
  if (!scratch) return kErrLaunch;
  // the group counters sit at the start of the array for every top_k
  if (cudaMemsetAsync(scratch, 0, (size_t)(hidden + 31) / 32 * sizeof(unsigned), S(stream)) != cudaSuccess)
    return kErrLaunch;
  // The memset is an ordinary stream dependency of the launch that follows;
  // ERVF_LAUNCH_PDL keeps the spread-rows route sum (group counters in the
  // array), without it a launch of 2..8 slots takes the cluster route sum.
  return ervf_moe_down_routesum(dn_codes, dn_scales, dn_code_stride, dn_scale_stride, ids, globals,
                                route_w, top_k, act, base, resid, out, hidden, inter, scratch,
                                kStaticScratchBytes, width, flags, stream);
}

}  // extern "C"
