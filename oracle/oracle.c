/*
 * Frizzle Gemma 3 forward-pass oracle: TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement, in plain C and f32, of the arithmetic Frizzle's WGSL
 * kernels perform for the Gemma 3 1B forward pass and its steering hook.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
 * it, as the checker of the CUDA path; nothing in the product links it.
 *
 * Each function names the reference file and lines it restates (paths inside
 * the plainsight-systems/frizzle project).  Summation orders follow the
 * shaders: every fused multiply-add the shaders write as fma() is fmaf() here,
 * and every other product and sum is a separate rounding, so this file is
 * built with -ffp-contract=off.  WGSL built-ins (exp2, exp, inverseSqrt, cos,
 * sin) are called through libm: the shaders leave their last bits to the
 * implementation, so agreement is to within those functions' error bounds.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------ f16 / bits */

static inline uint32_t bits_of_f32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float f32_of_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* unpack2x16float of one half, exact, subnormals kept (q4_0.wgsl:14). */
EXPORT float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff;
    if (e == 0) {
        float v = ldexpf((float)m, -24);
        return sign ? -v : v;
    }
    if (e == 31) return f32_of_bits(sign | 0x7f800000u | (m << 13));
    return f32_of_bits(sign | ((e + 112) << 23) | (m << 13));
}

/* pack2x16float of one value: round to nearest, ties to even. */
EXPORT uint16_t oracle_f32_to_f16(float f) {
    uint32_t x = bits_of_f32(f);
    uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (ax >= 0x47800000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return (uint16_t)sign;
        uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e, q = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((((ax >> 23) - 112)) << 10) | ((ax & 0x7fffffu) >> 13);
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

/* The KV cache's pack: saturate to +-65,504, then round once
 * (formats/f16/f16_pack.wgsl:16-19). */
EXPORT uint16_t oracle_f16_pack(float v) {
    if (v > 65504.0f) v = 65504.0f;
    if (v < -65504.0f) v = -65504.0f;
    return oracle_f32_to_f16(v);
}

/* ------------------------------------------------------------ Q4_0 */

/* Block of 18 bytes as the file stores it: fp16 d, then 16 code bytes; weight
 * j = ((qs[j] & 0xF) - 8) * d, weight j + 16 = ((qs[j] >> 4) - 8) * d
 * (formats/q4_0/q4_0.h:21-23, formats/q4_0/q4_0.wgsl:12-24). */
EXPORT void oracle_q4_0_unpack(const uint8_t *block, float out[32]) {
    uint16_t dh = (uint16_t)(block[0] | (block[1] << 8));
    float d = oracle_f16_to_f32(dh);
    for (int j = 0; j < 16; j++) {
        out[j] = ((float)(block[2 + j] & 0xF) - 8.0f) * d;
        out[j + 16] = ((float)(block[2 + j] >> 4) - 8.0f) * d;
    }
}

EXPORT void oracle_q4_0_dequant(const uint8_t *blocks, int64_t nblocks, float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblocks; b++) oracle_q4_0_unpack(blocks + 18 * b, out + 32 * b);
}

/* ------------------------------------------------------------ Q8_0 and Q4_1 */

/* Q8_0 block of 34 bytes as the file stores it: fp16 d, then 32 signed code
 * bytes; weight j = qs[j] * d, exact in f32 (formats/q8_0/q8_0.h:19-21,
 * formats/q8_0/q8_0.wgsl:11-23). */
EXPORT void oracle_q8_0_unpack(const uint8_t *block, float out[32]) {
    float d = oracle_f16_to_f32((uint16_t)(block[0] | (block[1] << 8)));
    for (int j = 0; j < 32; j++) out[j] = (float)(int8_t)block[2 + j] * d;
}

/* Q4_1 block of 20 bytes: fp16 d, fp16 m, then 16 code bytes; weight j =
 * (qs[j] & 0xF) * d + m, weight j + 16 = (qs[j] >> 4) * d + m
 * (formats/q4_1/q4_1.h:20-23, formats/q4_1/q4_1.wgsl:12-26).  The product of
 * a 4-bit code and an 11-bit significand is exact in f32, so the shader's
 * `code * d + m` rounds once whether or not it is fused. */
EXPORT void oracle_q4_1_unpack(const uint8_t *block, float out[32]) {
    float d = oracle_f16_to_f32((uint16_t)(block[0] | (block[1] << 8)));
    float m = oracle_f16_to_f32((uint16_t)(block[2] | (block[3] << 8)));
    for (int j = 0; j < 16; j++) {
        out[j] = (float)(block[4 + j] & 0xF) * d + m;
        out[j + 16] = (float)(block[4 + j] >> 4) * d + m;
    }
}

typedef void (*unpack_fn)(const uint8_t *, float *);

/* Formats by their GGUF type number (gguf::TensorType): 2 Q4_0, 3 Q4_1, 8 Q8_0. */
static int format_of(int type, unpack_fn *unpack) {
    switch (type) {
    case 2: *unpack = oracle_q4_0_unpack; return 18;
    case 3: *unpack = oracle_q4_1_unpack; return 20;
    case 8: *unpack = oracle_q8_0_unpack; return 34;
    default: *unpack = 0; return 0;
    }
}

/* Every block of a run of `nblocks` blocks of GGUF type `type`, unpacked;
 * returns 0, or -1 for a type this oracle does not restate. */
EXPORT int oracle_blocks_dequant(int type, const uint8_t *blocks, int64_t nblocks, float *out) {
    unpack_fn unpack;
    int bytes = format_of(type, &unpack);
    if (!bytes) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblocks; b++) unpack(blocks + (int64_t)bytes * b, out + 32 * b);
    return 0;
}

/* ------------------------------------------------------------ matmul */

/* y[t][o] = sum_k W[o][k] x[t][k] over K/32 groups split into 32 ranges,
 * range r being groups r*G/32 .. (r+1)*G/32; each range summed from zero by
 * fma over k in order, the 32 range sums then added in order to a total from
 * zero (matmul.wgsl:154-185 decode_ranges/slot_total, :320-405 tile_range/
 * prefill_tile, :548-571 combine; matmul.h:88-97).  Every form of the
 * reference produces these bits. */
static void matmul_rows_fmt(unpack_fn unpack, int block_bytes, const uint8_t *W, int K, const float *X, int M,
                            int row_stride_x, int o, float *y_out /* M values, stride given */, int y_stride) {
    int G = K / 32;
    float w[32];
    float totals[64];
    float parts[64];
    /* process tokens in groups of 64 to bound stack use */
    for (int t0 = 0; t0 < M; t0 += 64) {
        int tn = M - t0 < 64 ? M - t0 : 64;
        for (int t = 0; t < tn; t++) totals[t] = 0.0f;
        for (int r = 0; r < 32; r++) {
            int lo = r * G / 32, hi = (r + 1) * G / 32;
            for (int t = 0; t < tn; t++) parts[t] = 0.0f;
            for (int g = lo; g < hi; g++) {
                unpack(W + ((int64_t)o * G + g) * block_bytes, w);
                for (int t = 0; t < tn; t++) {
                    const float *x = X + (int64_t)(t0 + t) * row_stride_x + g * 32;
                    float a = parts[t];
                    for (int k = 0; k < 32; k++) a = fmaf(w[k], x[k], a);
                    parts[t] = a;
                }
            }
            for (int t = 0; t < tn; t++) totals[t] = totals[t] + parts[t];
        }
        for (int t = 0; t < tn; t++) y_out[(int64_t)(t0 + t) * y_stride] = totals[t];
    }
}

static void matmul_rows(const uint8_t *W, int K, const float *X, int M, int row_stride_x,
                        int o, float *y_out, int y_stride) {
    matmul_rows_fmt(oracle_q4_0_unpack, 18, W, K, X, M, row_stride_x, o, y_out, y_stride);
}

/* The same product over blocks of GGUF type `type` (the reference's matmul
 * is one shader over every format's unpack: matmul.wgsl:84-245 with
 * formats/format.h); returns -1 for a type this oracle does not restate. */
EXPORT int oracle_matmul_fmt(int type, const uint8_t *W, int N, int K, const float *X, int M, float *Y) {
    unpack_fn unpack;
    int bytes = format_of(type, &unpack);
    if (!bytes) return -1;
#pragma omp parallel for schedule(dynamic, 16)
    for (int o = 0; o < N; o++) matmul_rows_fmt(unpack, bytes, W, K, X, M, K, o, Y + o, N);
    return 0;
}

EXPORT void oracle_matmul(const uint8_t *W, int N, int K, const float *X, int M, float *Y) {
#pragma omp parallel for schedule(dynamic, 16)
    for (int o = 0; o < N; o++) matmul_rows(W, K, X, M, K, o, Y + o, N);
}

/* e^x for x <= 0 (matmul.wgsl:122-138): Cody-Waite reduction with ln 2 in
 * two parts, Taylor series to r^6 in Horner form, every multiply-add an fma. */
EXPORT float oracle_exp_nonpositive(float x) {
    float xc = fmaxf(x, -100.0f);
    float k = floorf(fmaf(xc, 1.4426950408889634f, 0.5f));
    float r = fmaf(k, -0.693145751953125f, xc);
    r = fmaf(k, -1.4286068203094172e-06f, r);
    float p = (float)(1.0 / 720.0);
    p = fmaf(p, r, (float)(1.0 / 120.0));
    p = fmaf(p, r, (float)(1.0 / 24.0));
    p = fmaf(p, r, (float)(1.0 / 6.0));
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return ldexpf(p, (int)k);
}

/* GELU, tanh form (matmul.wgsl:140-152). */
EXPORT float oracle_gelu(float g) {
    float z = 0.7978845608028654f * fmaf(0.044715f * g * g, g, g);
    float e = oracle_exp_nonpositive(-2.0f * fabsf(z));
    float s = z > 0.0f ? 1.0f : (z < 0.0f ? -1.0f : 0.0f);
    float t = s * ((1.0f - e) * (1.0f / (1.0f + e)));
    float half_g = 0.5f * g;
    return fmaf(half_g, t, half_g);
}

/* act[t][n] = gelu(gate . x_t) * (up . x_t) (matmul.wgsl:247-270, 487-501). */
EXPORT void oracle_gated(const uint8_t *Wg, const uint8_t *Wu, int F, int K, const float *X, int M, float *act) {
#pragma omp parallel for schedule(dynamic, 16)
    for (int o = 0; o < F; o++) {
        float g[64], u[64];
        for (int t0 = 0; t0 < M; t0 += 64) {
            int tn = M - t0 < 64 ? M - t0 : 64;
            matmul_rows(Wg, K, X + (int64_t)t0 * K, tn, K, o, g, 1);
            matmul_rows(Wu, K, X + (int64_t)t0 * K, tn, K, o, u, 1);
            for (int t = 0; t < tn; t++) act[(int64_t)(t0 + t) * F + o] = oracle_gelu(g[t]) * u[t];
        }
    }
}

/* ------------------------------------------------------------ norms */

/* The workgroup's fixed-order sum (norm.wgsl:75-85): invocation i of 256 sums
 * the squares of its vec4s i, i + 256, ... in order, each vec4's squares
 * x*x + y*y + z*z + w*w left to right; the 256 partials are then halved
 * level by level. */
static float norm_sum_squares(const float *x, int width) {
    float part[256];
    int vec4s = width / 4;
    for (int i = 0; i < 256; i++) {
        float s = 0.0f;
        for (int v = i; v < vec4s; v += 256) {
            const float *q = x + 4 * v;
            float d = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
            s = s + d;
        }
        part[i] = s;
    }
    for (int stride = 128; stride > 0; stride /= 2)
        for (int i = 0; i < stride; i++) part[i] = part[i] + part[i + stride];
    return part[0];
}

static float inverse_sqrt(float v) { return 1.0f / sqrtf(v); }

/* One row of the norm launch (norm.wgsl:97-198): optionally y through its
 * post-norm ((y*r_y)*post_gain)*post_scale is added into x and x written
 * back; then normed = (x*r)*gain.  `added` receives y as added. */
EXPORT void oracle_norm_row(float *x, const float *y, const float *post_gain, const float *gain,
                            int width, float eps, float *normed, float *added) {
    float n = (float)width;
    if (y) {
        float yy[8192];
        memcpy(yy, y, sizeof(float) * width);
        if (post_gain) {
            float r = inverse_sqrt(norm_sum_squares(yy, width) / n + eps);
            for (int i = 0; i < width; i++) yy[i] = ((yy[i] * r) * post_gain[i]) * 1.0f;
        }
        if (added) memcpy(added, yy, sizeof(float) * width);
        for (int i = 0; i < width; i++) x[i] = x[i] + yy[i];
    }
    float r = inverse_sqrt(norm_sum_squares(x, width) / n + eps);
    for (int i = 0; i < width; i++) normed[i] = (x[i] * r) * gain[i];
}

/* ------------------------------------------------------------ rope */

/* Each pair's theta_k / 2 pi, in f64 then rounded once (rope.cpp:95-107). */
EXPORT void oracle_rope_turns(float base, int d, float *turns) {
    for (int k = 0; k < d / 2; k++) {
        double theta = pow((double)base, -2.0 * (double)k / (double)d);
        turns[k] = (float)(theta / (2.0 * 3.14159265358979323846));
    }
}

/* QK-norm of one head (rope.wgsl:40-56, rope_cache.wgsl:44-60): lane l of
 * d/8 holds elements 4l..4l+3 and d/2+4l..; its partial dot(a,a) + dot(b,b)
 * is reduced by halving; then (x*r)*gain. */
static void qk_norm_head(float *h, const float *gain, int d, float eps) {
    int lanes = d / 8;
    float part[64];
    for (int l = 0; l < lanes; l++) {
        const float *a = h + 4 * l, *b = h + d / 2 + 4 * l;
        float da = a[0] * a[0] + a[1] * a[1] + a[2] * a[2] + a[3] * a[3];
        float db = b[0] * b[0] + b[1] * b[1] + b[2] * b[2] + b[3] * b[3];
        part[l] = da + db;
    }
    for (int stride = lanes / 2; stride > 0; stride /= 2)
        for (int l = 0; l < stride; l++) part[l] = part[l] + part[l + stride];
    float r = inverse_sqrt(part[0] / (float)d + eps);
    for (int i = 0; i < d; i++) h[i] = (h[i] * r) * gain[i];
}

/* Pairs (k, k + d/2) turned by angle 2 pi (t - round t), t = f32(p) * turn_k
 * (rope.wgsl:122-138). */
static void rotate_head(float *h, const float *turns, int d, uint32_t p) {
    const float tau = (float)6.283185307179586;
    for (int k = 0; k < d / 2; k++) {
        float t = (float)p * turns[k];
        float angle = tau * (t - rintf(t));
        float c = cosf(angle), s = sinf(angle);
        float a = h[k], b = h[k + d / 2];
        h[k] = a * c - b * s;
        h[k + d / 2] = a * s + b * c;
    }
}

/* ------------------------------------------------------------ attention */

static float dot4(const float *a, const float *b) {
    return a[0] * b[0] + a[1] * b[1] + a[2] * b[2] + a[3] * b[3];
}

/* One query of one head at position p over the cached keys and values of its
 * window, in the reference's order (attention.wgsl:166-400, combine :403-438,
 * fold_factors :135-151): 64-key chunks fixed by position, each from an empty
 * state, tiles of B = 2048/d keys inside a chunk from its start (or the tile
 * holding the earliest live key), an online softmax in log2 units, and chunk
 * states folded in chunk order.  One row a tile (M = 1024/d query vectors
 * = the group), which is Gemma 3 1B's shape. */
static void attend_query(const float *q_in, const uint16_t *kc, const uint16_t *vc, uint32_t slots,
                         int kv_heads, int kvh, int d, uint32_t window, float scale_log2e, uint32_t p,
                         float *out, float *scores_out, uint32_t scores_first, float *stats_out) {
    float q[512], vrow[512], o_chunk[512], o_run[512], kk[512];
    float pt[64], e[64];
    int B = 2048 / d;
    for (int i = 0; i < d; i++) { q[i] = q_in[i] * scale_log2e; o_run[i] = 0.0f; }
    uint32_t earliest = p + 1 > window ? p + 1 - window : 0;
    int run_live = 0;
    float run_m = 0.0f, run_l = 0.0f;
    for (uint32_t c = earliest / 64; c <= p / 64; c++) {
        int chunk_live = 0;
        float chunk_m = 0.0f, chunk_l = 0.0f;
        for (int i = 0; i < d; i++) o_chunk[i] = 0.0f;
        uint32_t k_begin = c * 64 > earliest / B * B ? c * 64 : earliest / B * B;
        uint32_t k_end = (c + 1) * 64 < p + 1 ? (c + 1) * 64 : p + 1;
        for (uint32_t j0 = k_begin; j0 < k_end; j0 += B) {
            int live[64];
            for (int b = 0; b < B; b++) {
                uint32_t j = j0 + b;
                live[b] = j < k_end && j <= p && j + window > p;
                pt[b] = 0.0f;
                if (live[b]) {
                    const uint16_t *kr = kc + ((size_t)(j % slots) * kv_heads + kvh) * d;
                    for (int i = 0; i < d; i++) kk[i] = oracle_f16_to_f32(kr[i]);
                    float s = 0.0f;
                    for (int w = 0; w < d / 4; w++) s += dot4(q + 4 * w, kk + 4 * w);
                    pt[b] = s;
                    if (scores_out) scores_out[j - scores_first] = s;
                }
            }
            float top_tile = 0.0f;
            int seen = 0;
            for (int b = 0; b < B; b++)
                if (live[b]) { top_tile = seen ? fmaxf(top_tile, pt[b]) : pt[b]; seen = 1; }
            float a = 1.0f;
            if (seen) {
                float old = chunk_live ? chunk_m : top_tile;
                chunk_live = 1;
                float top = fmaxf(old, top_tile);
                a = old == top ? 1.0f : exp2f(old - top);
                float sum = 0.0f;
                for (int b = 0; b < B; b++) {
                    e[b] = live[b] ? exp2f(pt[b] - top) : 0.0f;
                    sum += e[b];
                }
                chunk_l = chunk_l * a + sum;
                chunk_m = top;
            } else {
                for (int b = 0; b < B; b++) e[b] = 0.0f;
            }
            for (int i = 0; i < d; i++) o_chunk[i] = o_chunk[i] * a;
            for (int b = 0; b < B; b++) {
                uint32_t j = j0 + b;
                if (j < k_end) {
                    const uint16_t *vr = vc + ((size_t)(j % slots) * kv_heads + kvh) * d;
                    for (int i = 0; i < d; i++) vrow[i] = oracle_f16_to_f32(vr[i]);
                } else {
                    for (int i = 0; i < d; i++) vrow[i] = 0.0f;
                }
                for (int i = 0; i < d; i++) o_chunk[i] = o_chunk[i] + e[b] * vrow[i];
            }
        }
        /* fold (attention.wgsl:135-159) */
        float fa, fb, fm;
        if (!chunk_live) { fa = 1.0f; fb = 0.0f; fm = run_m; }
        else if (!run_live) { fa = 0.0f; fb = 1.0f; fm = chunk_m; }
        else if (run_m == chunk_m) { fa = 1.0f; fb = 1.0f; fm = run_m; }
        else if (run_m > chunk_m) { fa = 1.0f; fb = exp2f(chunk_m - run_m); fm = run_m; }
        else { fa = exp2f(run_m - chunk_m); fb = 1.0f; fm = chunk_m; }
        run_l = run_l * fa + chunk_l * fb;
        for (int i = 0; i < d; i++) o_run[i] = o_run[i] * fa + o_chunk[i] * fb;
        run_m = fm;
        run_live = run_live || chunk_live;
    }
    for (int i = 0; i < d; i++) out[i] = run_live ? o_run[i] / run_l : 0.0f;
    if (stats_out) { stats_out[0] = run_m; stats_out[1] = run_l; }
}

/* Attention over a KV cache for `rows` consecutive query rows at positions
 * position + r, every query head (the attention launch with its combine,
 * attention.wgsl:166-438): q [rows][heads][d], caches [slots][kv_heads][d]
 * f16 words, out [rows][heads][d]. */
EXPORT void oracle_attention(const float *q, const uint16_t *kc, const uint16_t *vc, uint32_t slots, int heads,
                             int kv_heads, int d, uint32_t window, float scale_log2e, uint32_t position, int rows,
                             float *out) {
    int G = heads / kv_heads;
#pragma omp parallel for collapse(2)
    for (int r = 0; r < rows; r++)
        for (int h = 0; h < heads; h++)
            attend_query(q + ((size_t)r * heads + h) * d, kc, vc, slots, kv_heads, h / G, d, window, scale_log2e,
                         position + (uint32_t)r, out + ((size_t)r * heads + h) * d, NULL, 0, NULL);
}

/* ------------------------------------------------------------ edits */

/* The edit launch over a step's rows (edit.wgsl:55-76): for each of the
 * layer's edits whose placed range holds the row's position, Set stores the
 * value, Zero stores 0, Scale multiplies once, and Scale by exactly 1 keeps
 * the neuron's bits. */
EXPORT void oracle_edit_apply(const uint32_t *table, uint32_t layer, uint32_t position, int rows,
                              int width, float *activation) {
    if (!table) return;
    uint32_t first = table[2 * layer], count = table[2 * layer + 1];
    for (int r = 0; r < rows; r++) {
        uint32_t pos = position + (uint32_t)r;
        for (uint32_t i = 0; i < count; i++) {
            const uint32_t *e = table + first + 5 * i;
            if (pos < e[3] || pos >= e[4]) continue;
            float *a = activation + (int64_t)r * width + e[0];
            float v = f32_of_bits(e[2]);
            float edited = v;
            if (e[1] == 1u) edited = v == 1.0f ? *a : *a * v;
            *a = edited;
        }
    }
}

/* ------------------------------------------------------------ selection and draw */

/* Order-preserving key of a logit's bits: -0 as +0, every NaN above +inf
 * (topk.wgsl:32-44). */
EXPORT uint32_t oracle_topk_key(uint32_t b) {
    if (b == 0x80000000u) b = 0;
    if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x007FFFFFu) != 0) return 0xFFFFFFFFu;
    if (b & 0x80000000u) return ~b;
    return b | 0x80000000u;
}

static uint32_t topk_bits(uint32_t key) {
    if (key == 0xFFFFFFFFu) return 0x7FC00000u;
    if (key & 0x80000000u) return key & 0x7FFFFFFFu;
    return ~key;
}

/* The top 64 of `count` logits, larger first, ties to the lower token, as
 * (logit bits, token) pairs (topk.wgsl:32-169: the three bitonic passes keep
 * exactly this set in this order). */
EXPORT void oracle_topk64(const float *logits, int64_t count, uint32_t *pairs) {
    uint32_t keys[64], ids[64];
    int n = 0;
    for (int64_t i = 0; i < count; i++) {
        uint32_t k = oracle_topk_key(bits_of_f32(logits[i]));
        if (n == 64 && !(k > keys[63])) continue;  /* ties keep the earlier (lower) id */
        int at = n < 64 ? n++ : 63;
        while (at > 0 && k > keys[at - 1]) { keys[at] = keys[at - 1]; ids[at] = ids[at - 1]; at--; }
        keys[at] = k;
        ids[at] = (uint32_t)i;
    }
    for (int i = 0; i < 64; i++) {
        pairs[2 * i] = i < n ? topk_bits(keys[i]) : 0;
        pairs[2 * i + 1] = i < n ? ids[i] : 0xFFFFFFFFu;
    }
}

/* Philox4x32-10 (draw.wgsl:48-60). */
EXPORT void oracle_philox(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* The draw (draw.wgsl:78-170): top-k, top-p, min-p and temperature over the
 * 64 candidates, and an inverse transform of one uniform from
 * Philox4x32-10(key = seed, counter = (position + tokens, 0, 0, 0)).
 * record = {token, failed, bits of u, 0}. */
EXPORT void oracle_draw(const uint32_t *cand, uint32_t top_k, float temperature, float top_p, float min_p,
                        float log_min_p, const uint32_t seed[2], uint32_t counter, uint32_t record[4]) {
    uint32_t k = top_k < 64 ? top_k : 64;
    int use_top_p = top_p < 1.0f;
    float weight[64], tempered[64], running[64];
    uint32_t above[64];
    uint32_t first_bits = cand[0];
    int failed = (first_bits & 0x7F800000u) == 0x7F800000u;
    for (uint32_t t = 0; t < k; t++) {
        uint32_t mine_bits = cand[2 * t];
        weight[t] = 0.0f;
        tempered[t] = 0.0f;
        above[t] = 0;
        if (!failed && mine_bits != 0xFF800000u) {
            float first = f32_of_bits(first_bits), mine = f32_of_bits(mine_bits);
            if (use_top_p) weight[t] = expf(mine - first);
            if (temperature > 0.0f) tempered[t] = expf((mine - first) / temperature);
            above[t] = (min_p == 0.0f || mine >= first + log_min_p) ? 1u : 0u;
        }
    }
    uint32_t ctr[4] = {counter, 0, 0, 0}, rnd[4];
    oracle_philox(ctr, seed, rnd);
    float u = (float)(rnd[0] >> 9) * (1.0f / 8388608.0f) + (1.0f / 16777216.0f);
    if (use_top_p) {
        float sum = 0.0f;
        for (uint32_t i = 0; i < k; i++) sum = sum + weight[i];
        if (!failed)
            for (uint32_t i = 0; i < k; i++) weight[i] = weight[i] / sum;
    }
    uint32_t kept = k;
    float cumulative = 0.0f, tsum = 0.0f;
    for (uint32_t i = 0; i < k; i++) {
        tsum = tsum + tempered[i];
        running[i] = tsum;
        if (use_top_p) {
            cumulative = cumulative + weight[i];
            if (cumulative >= top_p) { kept = i + 1; break; }
        }
    }
    uint32_t survivors = 1;
    while (survivors < kept && above[survivors] == 1u) survivors++;
    uint32_t chosen = 0;
    if (temperature > 0.0f) {
        float goal = u * running[survivors - 1];
        chosen = survivors - 1;
        for (uint32_t i = 0; i < survivors; i++)
            if (running[i] > goal) { chosen = i; break; }
    }
    record[0] = failed ? 0u : cand[2 * chosen + 1];
    record[1] = failed ? 1u : 0u;
    record[2] = bits_of_f32(u);
    record[3] = 0;
}

/* ------------------------------------------------------------ the model */

typedef struct {
    int layers, hidden, ffn, heads, kv_heads, head_dim, vocab, window, pattern;
    float rope_global, rope_local, eps;
    int context;
} oracle_shape;

typedef struct {
    const float *attn_norm, *q_norm, *k_norm, *post_attn_norm, *ffn_norm, *post_ffw_norm;
    const uint8_t *q, *k, *v, *o, *gate, *up, *down;  /* Q4_0 blocks as the file stores them */
} oracle_layer;

typedef struct {
    oracle_shape s;
    const uint8_t *token_embd;  /* tied head; GGUF type embd_type (Q4_0 unless set) */
    int embd_type;
    int *down_type;             /* each layer's ffn_down GGUF type (Q4_0 unless set) */
    const float *output_norm;
    oracle_layer *layer;
    uint32_t *slots;            /* ring slots per layer */
    uint16_t **kc, **vc;        /* f16 caches [slots][kv_heads][d] per layer */
    float *turns_global, *turns_local;
    float scale_log2e;
    float *hidden;              /* carried across nothing: per step scratch */
} oracle_ctx;

EXPORT oracle_ctx *oracle_ctx_new(const oracle_shape *s, const uint8_t *token_embd, const float *output_norm,
                                  const void *const *layer_ptrs /* 13 per layer in role order */,
                                  uint32_t context, uint32_t rollback) {
    oracle_ctx *c = calloc(1, sizeof(*c));
    c->s = *s;
    c->token_embd = token_embd;
    c->embd_type = 2;
    c->down_type = calloc(s->layers, sizeof(int));
    for (int l = 0; l < s->layers; l++) c->down_type[l] = 2;
    c->output_norm = output_norm;
    c->layer = calloc(s->layers, sizeof(oracle_layer));
    c->slots = calloc(s->layers, sizeof(uint32_t));
    c->kc = calloc(s->layers, sizeof(uint16_t *));
    c->vc = calloc(s->layers, sizeof(uint16_t *));
    for (int l = 0; l < s->layers; l++) {
        const void *const *p = layer_ptrs + 13 * l;
        oracle_layer *L = &c->layer[l];
        L->attn_norm = p[0]; L->q = p[1]; L->k = p[2]; L->v = p[3]; L->q_norm = p[4]; L->k_norm = p[5];
        L->o = p[6]; L->post_attn_norm = p[7]; L->ffn_norm = p[8]; L->gate = p[9]; L->up = p[10];
        L->down = p[11]; L->post_ffw_norm = p[12];
        int global = l % s->pattern == s->pattern - 1;
        uint32_t window = global ? (uint32_t)s->context : (uint32_t)s->window;
        uint64_t ring = (uint64_t)window + 512 + rollback;  /* residency/plan.cpp:335-336, :296-298 */
        c->slots[l] = (uint32_t)(context < ring ? context : ring);
        size_t n = (size_t)c->slots[l] * s->kv_heads * s->head_dim;
        c->kc[l] = calloc(n, 2);
        c->vc[l] = calloc(n, 2);
    }
    c->turns_global = calloc(s->head_dim / 2, sizeof(float));
    c->turns_local = calloc(s->head_dim / 2, sizeof(float));
    oracle_rope_turns(s->rope_global, s->head_dim, c->turns_global);
    oracle_rope_turns(s->rope_local, s->head_dim, c->turns_local);
    float scale = 1.0f / sqrtf((float)s->head_dim);               /* describe.cpp:359 */
    c->scale_log2e = (float)((double)scale * 1.4426950408889634);  /* attention.cpp:45 */
    return c;
}

EXPORT void oracle_ctx_free(oracle_ctx *c) {
    if (!c) return;
    for (int l = 0; l < c->s.layers; l++) { free(c->kc[l]); free(c->vc[l]); }
    free(c->kc); free(c->vc); free(c->slots); free(c->layer); free(c->down_type);
    free(c->turns_global); free(c->turns_local);
    free(c);
}

/* The pinned file's mix (docs/architecture/logical-overview.md:63-64): the
 * tied embedding's and each layer's ffn_down GGUF types (2 Q4_0, 3 Q4_1,
 * 8 Q8_0); the reference reads every format through the one matmul and
 * gather over the format's unpack (formats/format.h).  Returns -1 for a
 * type not restated. */
EXPORT int oracle_ctx_set_types(oracle_ctx *c, int embd_type, const int *down_types) {
    unpack_fn u;
    if (!format_of(embd_type, &u)) return -1;
    for (int l = 0; l < c->s.layers; l++)
        if (!format_of(down_types[l], &u)) return -1;
    c->embd_type = embd_type;
    for (int l = 0; l < c->s.layers; l++) c->down_type[l] = down_types[l];
    return 0;
}

EXPORT uint32_t oracle_ctx_slots(const oracle_ctx *c, int layer) { return c->slots[layer]; }
EXPORT const uint16_t *oracle_ctx_keys(const oracle_ctx *c, int layer) { return c->kc[layer]; }
EXPORT const uint16_t *oracle_ctx_values(const oracle_ctx *c, int layer) { return c->vc[layer]; }

/* The capture store's layout in 32-bit words (capture/capture.cpp:31-73):
 * region 1 every layer's neurons (ffn words each, in layer order); region 2,
 * for each layer, its residual, attention addition, feed-forward addition
 * (hidden each), query (heads x d), weights (heads x keys, keys = min(window,
 * trained context)), stats (2 x heads) and readout (128 words).  slots[0..7]
 * get layer `layer`'s first words in that order (neurons first); returns
 * the store's size. */
static uint32_t layer_window(const oracle_shape *s, int l) {
    return s->window == 0 || l % s->pattern == s->pattern - 1 ? (uint32_t)s->context : (uint32_t)s->window;
}

EXPORT int64_t oracle_capture_slots(const oracle_shape *s, int layer, int64_t *slots, uint32_t *keys_out) {
    int64_t at = (int64_t)s->layers * s->ffn;
    for (int l = 0; l < s->layers; l++) {
        uint32_t w = layer_window(s, l);
        int64_t keys = w < (uint32_t)s->context ? w : (uint32_t)s->context;
        int64_t first[8];
        first[0] = (int64_t)l * s->ffn;
        first[1] = at;
        first[2] = first[1] + s->hidden;
        first[3] = first[2] + s->hidden;
        first[4] = first[3] + s->hidden;
        first[5] = first[4] + (int64_t)s->heads * s->head_dim;
        first[6] = first[5] + (int64_t)s->heads * keys;
        first[7] = first[6] + 2 * s->heads;
        at = first[7] + 128;
        if (l == layer) {
            if (slots) memcpy(slots, first, sizeof(first));
            if (keys_out) *keys_out = (uint32_t)keys;
        }
    }
    return at;
}

EXPORT int64_t oracle_capture_floats(const oracle_shape *s) { return oracle_capture_slots(s, -1, NULL, NULL); }

/* One step (graph/graph.cpp:298-476, arch/gemma3/gemma3.cpp:100-111): embed,
 * 26 x (attention block, gated feed-forward block), and, when `logits_out`
 * is given, the final norm and tied head over the last row. */
EXPORT void oracle_step(oracle_ctx *c, uint32_t position, int tokens, const uint32_t *ids,
                        const uint32_t *edit_table, float *logits_out, float *capture) {
    const oracle_shape *s = &c->s;
    int H = s->hidden, F = s->ffn, d = s->head_dim, QW = s->heads * d, KW = s->kv_heads * d;
    int T = tokens;
    float *hidden = malloc(sizeof(float) * T * H), *normed = malloc(sizeof(float) * T * H);
    float *output = malloc(sizeof(float) * T * H), *q = malloc(sizeof(float) * T * QW);
    float *k = malloc(sizeof(float) * T * KW), *v = malloc(sizeof(float) * T * KW);
    float *att = malloc(sizeof(float) * T * QW), *act = malloc(sizeof(float) * (size_t)T * F);
    float *cap = capture;
    /* slot first words, per layer: neurons, residual, attention addition,
     * feed-forward addition, query, weights, stats, readout */
    int64_t (*slot)[8] = cap ? malloc(sizeof(int64_t[8]) * s->layers) : NULL;
    uint32_t *keys = cap ? malloc(sizeof(uint32_t) * s->layers) : NULL;
    for (int l = 0; cap && l < s->layers; l++) oracle_capture_slots(s, l, slot[l], &keys[l]);
    /* embed (gather.wgsl:25-48), scale sqrt(width) in f32 (gemma3.cpp:105) */
    float scale = sqrtf((float)H);
    unpack_fn embd_unpack;
    const int embd_bytes = format_of(c->embd_type, &embd_unpack);
    for (int t = 0; t < T; t++) {
        float w[32];
        for (int g = 0; g < H / 32; g++) {
            embd_unpack(c->token_embd + ((int64_t)ids[t] * (H / 32) + g) * embd_bytes, w);
            for (int i = 0; i < 32; i++) hidden[(int64_t)t * H + g * 32 + i] = w[i] * scale;
        }
    }
    for (int l = 0; l < s->layers; l++) {
        oracle_layer *L = &c->layer[l];
        int global = l % s->pattern == s->pattern - 1;
        uint32_t window = global ? (uint32_t)s->context : (uint32_t)s->window;
        const float *turns = global ? c->turns_global : c->turns_local;
        int lc = cap != NULL;
        /* attention.norm: with the last layer's post-ffw norm add, except layer 0 */
#pragma omp parallel for
        for (int t = 0; t < T; t++)
            oracle_norm_row(hidden + (int64_t)t * H, l ? output + (int64_t)t * H : NULL,
                            l ? c->layer[l - 1].post_ffw_norm : NULL, L->attn_norm, H, s->eps,
                            normed + (int64_t)t * H,
                            (l && lc && t == T - 1) ? cap + slot[l - 1][3] : NULL);
        if (lc) memcpy(cap + slot[l][1], hidden + (int64_t)(T - 1) * H, sizeof(float) * H);
        oracle_matmul(L->q, QW, H, normed, T, q);
        oracle_matmul(L->k, KW, H, normed, T, k);
        oracle_matmul(L->v, KW, H, normed, T, v);
        /* rope + KV append (rope_cache.wgsl:16-91) */
        for (int t = 0; t < T; t++) {
            uint32_t p = position + (uint32_t)t;
            for (int h = 0; h < s->heads; h++) {
                float *qh = q + (int64_t)t * QW + h * d;
                qk_norm_head(qh, L->q_norm, d, s->eps);
                rotate_head(qh, turns, d, p);
            }
            for (int h = 0; h < s->kv_heads; h++) {
                float *kh = k + (int64_t)t * KW + h * d, *vh = v + (int64_t)t * KW + h * d;
                qk_norm_head(kh, L->k_norm, d, s->eps);
                rotate_head(kh, turns, d, p);
                uint16_t *kd = c->kc[l] + ((size_t)(p % c->slots[l]) * s->kv_heads + h) * d;
                uint16_t *vd = c->vc[l] + ((size_t)(p % c->slots[l]) * s->kv_heads + h) * d;
                for (int i = 0; i < d; i++) { kd[i] = oracle_f16_pack(kh[i]); vd[i] = oracle_f16_pack(vh[i]); }
            }
        }
        if (lc) memcpy(cap + slot[l][4], q + (int64_t)(T - 1) * QW, sizeof(float) * QW);
        int G = s->heads / s->kv_heads;
        /* The captured row's scores and the fold's statistics
         * (attention.wgsl:290-295, :394-395), then its weights
         * (weights.wgsl): exp2(s - m) / l for the keys read, 0 past them. */
        uint32_t p_last = position + (uint32_t)T - 1;
        uint32_t count = lc ? (p_last + 1 < keys[l] ? p_last + 1 : keys[l]) : 0;
        uint32_t earliest = p_last + 1 - count;
#pragma omp parallel for collapse(2)
        for (int t = 0; t < T; t++)
            for (int h = 0; h < s->heads; h++) {
                int cap_row = lc && t == T - 1;
                float *w = cap_row ? cap + slot[l][5] + (int64_t)h * keys[l] : NULL;
                float *st = cap_row ? cap + slot[l][6] + 2 * h : NULL;
                attend_query(q + (int64_t)t * QW + h * d, c->kc[l], c->vc[l], c->slots[l], s->kv_heads, h / G, d,
                             window, c->scale_log2e, position + (uint32_t)t, att + (int64_t)t * QW + h * d, w,
                             earliest, st);
                if (cap_row)
                    for (uint32_t i = 0; i < keys[l]; i++) w[i] = i < count ? exp2f(w[i] - st[0]) / st[1] : 0.0f;
            }
        oracle_matmul(L->o, H, QW, att, T, output);
        /* ffn.norm: add the attention block's output through its post-norm */
#pragma omp parallel for
        for (int t = 0; t < T; t++)
            oracle_norm_row(hidden + (int64_t)t * H, output + (int64_t)t * H, L->post_attn_norm, L->ffn_norm, H,
                            s->eps, normed + (int64_t)t * H, (lc && t == T - 1) ? cap + slot[l][2] : NULL);
        oracle_gated(L->gate, L->up, F, H, normed, T, act);
        oracle_edit_apply(edit_table, (uint32_t)l, position, T, F, act);
        if (lc) memcpy(cap + slot[l][0], act + (int64_t)(T - 1) * F, sizeof(float) * F);
        oracle_matmul_fmt(c->down_type[l], L->down, H, F, act, T, output);
    }
    if (logits_out) {
        float *x = hidden + (int64_t)(T - 1) * H;
        float fin[8192];
        oracle_norm_row(x, output + (int64_t)(T - 1) * H, c->layer[s->layers - 1].post_ffw_norm, c->output_norm, H,
                        s->eps, fin, cap ? cap + slot[s->layers - 1][3] : NULL);
        oracle_matmul_fmt(c->embd_type, c->token_embd, s->vocab, H, fin, 1, logits_out);
    }
    if (cap) {
        const int L = s->layers;
        /* No logits: no final norm, so neither the last block's addition nor
         * the last readout exists; both slots are zero. */
        if (!logits_out) {
            memset(cap + slot[L - 1][3], 0, sizeof(float) * H);
            memset(cap + slot[L - 1][7], 0, sizeof(float) * 128);
        } else {
            oracle_topk64(logits_out, s->vocab, (uint32_t *)(cap + slot[L - 1][7]));
        }
        /* Readouts of the layers before the last (capture.h:26-33): the
         * residual each leaves, which is the next layer's captured residual,
         * through the final norm and the tied head, its top 64. */
        float *lrow = malloc(sizeof(float) * (size_t)s->vocab);
        for (int l = 0; l + 1 < L; l++) {
            float xr[8192], fin[8192];
            memcpy(xr, cap + slot[l + 1][1], sizeof(float) * H);
            oracle_norm_row(xr, NULL, NULL, c->output_norm, H, s->eps, fin, NULL);
            oracle_matmul_fmt(c->embd_type, c->token_embd, s->vocab, H, fin, 1, lrow);
            oracle_topk64(lrow, s->vocab, (uint32_t *)(cap + slot[l][7]));
        }
        free(lrow);
        free(slot);
        free(keys);
    }
    free(hidden); free(normed); free(output); free(q); free(k); free(v); free(att); free(act);
}

EXPORT int oracle_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Sets the host threads the restatement runs on (a launcher such as torchrun
 * may have set OMP_NUM_THREADS=1 for the process). */
EXPORT void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
