/*
 * ervf_oracle.c -- CPU restatement of the reference's NVFP4 / BF16 decode-GEMV
 * arithmetic, used ONLY as the checker of the CUDA product.
 *
 * TEST INFRASTRUCTURE.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference arm may load this library.  The product path
 * (ervf_b200/) never calls it.
 *
 * Every function follows a named piece of kennydd001/ervf:
 *   - LUTs:            src/moe_lab/lightningstream_nemotron/nvfp4.py:49-76 (tables),
 *                      fused_nvfp4.py:760-762 (E4M3 NaN bytes -> 0.0 on device)
 *   - chain + tree:    fused_nvfp4.py:31-122 (gemv_nvfp4_rows, numeric contract),
 *                      fused_nvfp4.py:295-406 (gemv_nvfp4_ervf, fixed 8-sum combine),
 *                      scripts/nervf_nemotron/nervf01_geometry_audit.py:110-243
 *   - accumulate:      fused_nvfp4.py:125-133, :736-744
 *   - masked down:     fused_nvfp4.py:157-187 (panel_scan), :225-271
 *                      (gemv_down_masked_partial), :408-419 (reduce_partials);
 *                      panel-major layout runtime.py:34-52
 *   - BF16 GEMV:       gpu_kernels.py:21-49 (gemv_bf16)
 *   - FP32 GEMV:       gpu_kernels.py:51-74 (gemv_f32, the router projection)
 *   - device router:   fused_nvfp4.py:433-465 (route_topk_f32)
 *   - device LRU:      fused_nvfp4.py:470-511 (cache_assign)
 *
 * Build with -O2 -ffp-contract=off and without -ffast-math: every product and
 * sum below must be one IEEE binary32 operation, exactly as in the CUDA source
 * it restates (fmaf is the correctly rounded fused multiply-add of C99).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>

#define ORACLE_API __attribute__((visibility("default")))

/* Tree selectors.  ERVF rebuilds the warp tree and combines the 8 warp sums
 * as ((S0+S4)+(S2+S6))+((S1+S5)+(S3+S7)) (fused_nvfp4.py:397-403).  LEGACY is
 * the 256-thread kernel, whose second butterfly also adds the zero lanes
 * 8..31 (fused_nvfp4.py:108-112): S + 0.0 turns -0.0 into +0.0, the only
 * place the two trees can differ. */
enum { ORACLE_TREE_ERVF = 0, ORACLE_TREE_LEGACY = 1 };

/* ------------------------------------------------------------------ LUTs */

static float e2m1_value(int code)
{
    /* nvfp4.py:49-55: sign bit 3, magnitudes {0,0.5,1,1.5,2,3,4,6} */
    static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    float m = mag[code & 7];
    return (code & 8) ? -m : m;
}

static float e4m3_value(int byte, int nan_to_zero)
{
    /* nvfp4.py:58-69: bias 7, subnormal 2^-6 * m/8, NaN only at 0x7F/0xFF */
    int sign = (byte >> 7) & 1;
    int e = (byte >> 3) & 0xF;
    int m = byte & 7;
    float v;
    if (e == 0xF && m == 7) {
        return nan_to_zero ? 0.0f : NAN;
    } else if (e == 0) {
        v = ldexpf((float)m / 8.0f, -6);
    } else {
        v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    }
    return sign ? -v : v;
}

ORACLE_API void oracle_luts(float *e2m1, float *e4m3_device, float *e4m3_raw)
{
    for (int c = 0; c < 16; ++c) e2m1[c] = e2m1_value(c);
    for (int b = 0; b < 256; ++b) {
        e4m3_device[b] = e4m3_value(b, 1);
        e4m3_raw[b] = e4m3_value(b, 0);
    }
}

/* ------------------------------------------------------------------ tree */

/* T(a_0..a_31): shfl_down offsets 16,8,4,2,1; level `off` replaces y_l by
 * y_l + y_{l+off} for l < off and returns y_0. */
static float warp_tree(const float *a)
{
    float y[32];
    memcpy(y, a, sizeof(y));
    for (int off = 16; off > 0; off >>= 1)
        for (int l = 0; l < off; ++l) y[l] = y[l] + y[l + off];
    return y[0];
}

static float tree256(const float *a, int tree)
{
    float S[8];
    for (int w = 0; w < 8; ++w) S[w] = warp_tree(a + 32 * w);
    if (tree == ORACLE_TREE_LEGACY) {
        float v[32];
        for (int l = 0; l < 32; ++l) v[l] = (l < 8) ? S[l] : 0.0f;
        return warp_tree(v);
    }
    const float t0 = S[0] + S[4], t1 = S[1] + S[5];
    const float t2 = S[2] + S[6], t3 = S[3] + S[7];
    const float u0 = t0 + t2, u1 = t1 + t3;
    return u0 + u1;
}

static float epilogue(float v, int relu2, float out_scale)
{
    if (relu2) {
        const float r = fmaxf(v, 0.0f);
        return r * r;
    }
    return v * out_scale;
}

/* ---------------------------------------------------------- NVFP4 GEMV */

/* One output row of the numeric contract (fused_nvfp4.py:63-94).  Virtual
 * thread t walks uchar4 index v = t, t+256, ...; per uchar4 the block scale is
 * s = RN(e4m3[scale[b>>3]] * g) and each weight w = RN(e2m1[nib] * s) feeds
 * fmaf(w, x[k], acc) in the order lo,hi of .x,.y,.z,.w.  Tail bytes use 2
 * fmaf per byte. */
static float nvfp4_row(const uint8_t *crow, const uint8_t *srow, const float *x,
                       float g, int cols, int tree, const float *e2m1,
                       const float *e4m3)
{
    const int n_bytes = cols >> 1;
    const int n_vec = n_bytes >> 2;
    float a[256];
    for (int t = 0; t < 256; ++t) {
        float acc = 0.0f;
        for (int v = t; v < n_vec; v += 256) {
            const int b = v << 2;
            const float s = e4m3[srow[b >> 3]] * g;
            const int k = b << 1;
            for (int i = 0; i < 4; ++i) {
                const uint8_t q = crow[b + i];
                acc = fmaf(e2m1[q & 0x0F] * s, x[k + 2 * i], acc);
                acc = fmaf(e2m1[q >> 4] * s, x[k + 2 * i + 1], acc);
            }
        }
        for (int b = (n_vec << 2) + t; b < n_bytes; b += 256) {
            const uint8_t q = crow[b];
            const float s = e4m3[srow[b >> 3]] * g;
            const int k = b << 1;
            acc = fmaf(e2m1[q & 0x0F] * s, x[k], acc);
            acc = fmaf(e2m1[q >> 4] * s, x[k + 1], acc);
        }
        a[t] = acc;
    }
    return tree256(a, tree);
}

ORACLE_API void oracle_nvfp4_gemv(const uint8_t *codes, const uint8_t *scales,
                                  const float *x, float *out, float global_scale,
                                  int rows, int cols, int apply_relu2,
                                  float out_scale, int tree)
{
    float e2m1[16], e4m3[256], raw[256];
    oracle_luts(e2m1, e4m3, raw);
    const size_t n_bytes = (size_t)(cols >> 1), n_scales = (size_t)(cols >> 4);
    for (int r = 0; r < rows; ++r) {
        const float v = nvfp4_row(codes + (size_t)r * n_bytes, scales + (size_t)r * n_scales,
                                  x, global_scale, cols, tree, e2m1, e4m3);
        out[r] = epilogue(v, apply_relu2, out_scale);
    }
}

/* fused_nvfp4.py:125-133 */
ORACLE_API void oracle_weighted_accumulate(float *dst, const float *src, float weight, int n)
{
    for (int i = 0; i < n; ++i) dst[i] = fmaf(src[i], weight, dst[i]);
}

/* FusedNVFP4.expert (fused_nvfp4.py:970-978): up GEMV with relu^2 into act,
 * then the down GEMV into out. */
ORACLE_API void oracle_expert(const uint8_t *up_c, const uint8_t *up_s, float up_g,
                              const uint8_t *dn_c, const uint8_t *dn_s, float dn_g,
                              const float *x, float *act, float *out, int hidden,
                              int inter)
{
    oracle_nvfp4_gemv(up_c, up_s, x, act, up_g, inter, hidden, 1, 1.0f, ORACLE_TREE_ERVF);
    oracle_nvfp4_gemv(dn_c, dn_s, act, out, dn_g, hidden, inter, 0, 1.0f, ORACLE_TREE_ERVF);
}

/* ------------------------------------------------------ masked down path */

/* The panel-major down record (runtime.py:34-52): panel p covers input columns
 * 16p..16p+15; per panel first `rows` scale bytes (one per output row), then
 * the 16 columns, each rows/2 bytes (row 2h in the low nibble of byte h). */
ORACLE_API void oracle_panel_major(const uint8_t *codes, const uint8_t *scales,
                                   uint8_t *block, int rows, int inter)
{
    const int npanel = inter >> 4, rowhalf = rows >> 1;
    const size_t stride = (size_t)rows + 16u * (size_t)rowhalf;
    for (int p = 0; p < npanel; ++p) {
        uint8_t *pb = block + (size_t)p * stride;
        for (int r = 0; r < rows; ++r) pb[r] = scales[(size_t)r * npanel + p];
        for (int c = 0; c < 16; ++c) {
            const int j = 16 * p + c;
            uint8_t *col = pb + rows + (size_t)c * rowhalf;
            for (int h = 0; h < rowhalf; ++h) {
                const uint8_t b0 = codes[(size_t)(2 * h) * (inter >> 1) + (j >> 1)];
                const uint8_t b1 = codes[(size_t)(2 * h + 1) * (inter >> 1) + (j >> 1)];
                const uint8_t n0 = (j & 1) ? (b0 >> 4) : (b0 & 15);
                const uint8_t n1 = (j & 1) ? (b1 >> 4) : (b1 & 15);
                col[h] = (uint8_t)(n0 | (n1 << 4));
            }
        }
    }
}

/* panel_scan + gemv_down_masked_partial + reduce_partials: chunk c walks the
 * ACTIVE panel list at pi = c, c+nchunks, ...; inside a panel the set mask bits
 * ascend; partials are summed sequentially from 0.0. */
ORACLE_API void oracle_down_masked(const uint8_t *bank, const float *act, float *out,
                                   float global_scale, int rows, int inter, int nchunks)
{
    float e2m1[16], e4m3[256], raw[256];
    oracle_luts(e2m1, e4m3, raw);
    const int npanel = inter >> 4, rowhalf = rows >> 1;
    const size_t stride = (size_t)rows + 16u * (size_t)rowhalf;
    unsigned masks[4096];
    int plist[4096];
    int pcount = 0;
    for (int p = 0; p < npanel; ++p) {
        unsigned m = 0;
        for (int c = 0; c < 16; ++c)
            if (act[16 * p + c] != 0.0f) m |= 1u << c;
        masks[p] = m;
        if (m) plist[pcount++] = p;
    }
    for (int r = 0; r < rows; ++r) {
        float total = 0.0f;
        for (int ch = 0; ch < nchunks; ++ch) {
            float acc = 0.0f;
            for (int pi = ch; pi < pcount; pi += nchunks) {
                const int p = plist[pi];
                const uint8_t *pb = bank + (size_t)p * stride;
                const float s = e4m3[pb[r]] * global_scale;
                for (int c = 0; c < 16; ++c) {
                    if (!(masks[p] & (1u << c))) continue;
                    const uint8_t byte = pb[rows + (size_t)c * rowhalf + (r >> 1)];
                    const float w = e2m1[(r & 1) ? (byte >> 4) : (byte & 15)] * s;
                    acc = fmaf(w, act[16 * p + c], acc);
                }
            }
            total += acc;
        }
        out[r] = total;
    }
}

/* ------------------------------------------------------------- BF16 GEMV */

/* gemv_bf16 (gpu_kernels.py:21-49): thread t walks k = t, t+256, ... with one
 * fmaf per element; legacy tree (the 8 warp sums go through a full butterfly
 * with zero lanes). `batch` columns of x are independent problems. */
ORACLE_API void oracle_bf16_gemv(const uint16_t *W, const float *x, float *out,
                                 int rows, int cols, int batch)
{
    float a[256];
    for (int b = 0; b < batch; ++b) {
        const float *xb = x + (size_t)b * cols;
        for (int r = 0; r < rows; ++r) {
            const uint16_t *wr = W + (size_t)r * cols;
            for (int t = 0; t < 256; ++t) {
                float acc = 0.0f;
                for (int k = t; k < cols; k += 256) {
                    uint32_t u = ((uint32_t)wr[k]) << 16;
                    float wf;
                    memcpy(&wf, &u, 4);
                    acc = fmaf(wf, xb[k], acc);
                }
                a[t] = acc;
            }
            out[(size_t)b * rows + r] = tree256(a, ORACLE_TREE_LEGACY);
        }
    }
}

/* gemv_f32 (gpu_kernels.py:51-74), 256-thread block: thread t walks
 * k = t, t+256, ... with fmaf, then the same legacy tree as gemv_bf16. */
ORACLE_API void oracle_f32_gemv(const float *W, const float *x, float *out, int rows, int cols)
{
    float a[256];
    for (int r = 0; r < rows; ++r) {
        const float *wr = W + (size_t)r * cols;
        for (int t = 0; t < 256; ++t) {
            float acc = 0.0f;
            for (int k = t; k < cols; k += 256) acc = fmaf(wr[k], x[k], acc);
            a[t] = acc;
        }
        out[r] = tree256(a, ORACLE_TREE_LEGACY);
    }
}

/* ----------------------------------------------------------- routing */

/* route_topk_f32 (fused_nvfp4.py:433-465): sigmoid scores, selection on
 * score + bias, serial top-k where the strictly greater value wins (lowest
 * index on ties), weights renormalised in route order. */
ORACLE_API void oracle_route_topk(const float *rlog, const float *gate_b, int *ids,
                                  float *w, int n, int top_k, float scaling,
                                  int bad_pick)
{
    float sc[1024], ch[1024];
    for (int i = 0; i < n; ++i) {
        const float s = 1.0f / (1.0f + expf(-rlog[i]));
        sc[i] = s;
        ch[i] = s + gate_b[i];
    }
    float wsum = 0.0f;
    for (int s = 0; s < top_k; ++s) {
        int bi = 0;
        float bv = -3.0e38f;
        for (int e = 0; e < n; ++e)
            if (ch[e] > bv) { bv = ch[e]; bi = e; }
        if (bad_pick && s == top_k - 1) {
            ch[bi] = -3.0e38f; bi = 0; bv = -3.0e38f;
            for (int e = 0; e < n; ++e)
                if (ch[e] > bv) { bv = ch[e]; bi = e; }
        }
        ids[s] = bi;
        w[s] = sc[bi];
        ch[bi] = -3.0e38f;
        wsum += sc[bi];
    }
    for (int s = 0; s < top_k; ++s) w[s] = w[s] / (wsum + 1e-20f) * scaling;
}

/* cache_assign (fused_nvfp4.py:470-511): route-order LRU with append while
 * filling, then min-last-used eviction, lowest slot on ties. */
ORACLE_API void oracle_cache_assign(int *slot_of, int *expert_of, int *last_used,
                                    int *state2, const int *ids, int *slots, int *need,
                                    int *stats2, int cap, int top_k)
{
    int tick = state2[0], filled = state2[1];
    for (int s = 0; s < top_k; ++s) {
        const int e = ids[s];
        const int sl = slot_of[e];
        if (sl >= 0) {
            last_used[sl] = ++tick;
            slots[s] = sl;
            need[s] = 0;
            stats2[0] += 1;
            continue;
        }
        stats2[1] += 1;
        int v;
        if (filled < cap) {
            v = filled++;
        } else {
            v = 0;
            int mnv = last_used[0];
            for (int c = 1; c < cap; ++c)
                if (last_used[c] < mnv) { mnv = last_used[c]; v = c; }
            slot_of[expert_of[v]] = -1;
        }
        slot_of[e] = v;
        expert_of[v] = e;
        last_used[v] = ++tick;
        slots[s] = v;
        need[s] = 1;
    }
    state2[0] = tick;
    state2[1] = filled;
}
