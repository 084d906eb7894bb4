/*
 * k2_oracle.c -- CPU restatement of the Krea2 W4A4 DiT block hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links or calls this file;
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it,
 * and only as the checker.
 *
 * Every function states the reference code it restates (paths are relative to
 * the ComfyUI-K2-Precompile project).  Where this project's W4A4 contract
 * differs from the reference (group-128 fp16 scales, normalised H128
 * rotation, RNE quant), the contract is the one both this file and the CUDA
 * kernels follow; the
 * reference's rounding points (bf16 after every modulation step, fp32 fmaf
 * chains) are kept.
 *
 * Parity status: the rotation/quantisation helpers of the reference live in the
 * un-vendored comfy-kitchen sources, so the INT4 contract here is pinned by this
 * restatement and by golden fixtures of the reference's own Triton kernels
 * (norm/modulation, QK-norm+RoPE, SiLU product, attention) run under the Triton
 * interpreter; see tests/golden/make_golden.py.
 *
 * Build: gcc -O3 -ffp-contract=off -fno-fast-math -shared -fPIC
 * (oracle/Makefile).  fp contraction must stay off: every fused multiply-add
 * below is an explicit fmaf(), every other operation rounds to fp32.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- numerics */

static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float k2o_bf16_to_f32(uint16_t h) { return bits_f((uint32_t)h << 16); }

/* fp32 -> bf16 rounding mode.  0 (default): round to nearest even, like
 * __float2bfloat16_rn on the GPU -- the contract.  1: truncation, which is what
 * the Triton CPU interpreter does for .to(tl.bfloat16); used only to compare
 * bit for bit with the reference's Triton kernels run under that interpreter
 * (tests/golden). */
static int g_bf16_truncate = 0;
void k2o_set_bf16_truncate(int on) { g_bf16_truncate = on; }

/* fp32 -> bf16 (NaN kept quiet) */
uint16_t k2o_f32_to_bf16(float f) {
    uint32_t u = f_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    if (!g_bf16_truncate) u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float bf(uint16_t h) { return k2o_bf16_to_f32(h); }
static inline float bfr(float f) { return k2o_bf16_to_f32(k2o_f32_to_bf16(f)); }

/* IEEE binary16 conversions (round-to-nearest-even), like __float2half_rn */
uint16_t k2o_f32_to_f16(float f) {
    _Float16 h = (_Float16)f;
    uint16_t u; memcpy(&u, &h, 2); return u;
}
float k2o_f16_to_f32(uint16_t u) {
    _Float16 h; memcpy(&h, &u, 2); return (float)h;
}

/* correctly rounded 1/sqrt(x) (the CUDA side calls __frsqrt_rn) */
float k2o_rsqrt_rn(float x) { return (float)(1.0L / sqrtl((long double)x)); }

/*
 * exp(x) in fp32 from basic correctly-rounded operations only, so that the CUDA
 * kernels (same sequence, __fmaf_rn/__fmul_rn) produce identical bits.
 * Method: Cody-Waite range reduction x = n*ln2 + r with a two-part ln2 (the
 * split used by fdlibm's e_expf.c), Taylor polynomial of degree 7 in Horner
 * form (|r| <= ln2/2 -> truncation error < 0.2 ulp), scaling by 2^n through
 * the exponent field.  Max error vs a correctly rounded exp: ~2 ulp.
 */
float k2o_exp(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    float n = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(n, -0.693145751953125f, x);
    r = fmaf(n, -1.428606765330187045037746429443359375e-06f, r);
    float p = 1.98412698412698412526e-4f;
    p = fmaf(p, r, 1.38888888888888894189e-3f);
    p = fmaf(p, r, 8.33333333333333321769e-3f);
    p = fmaf(p, r, 4.16666666666666643537e-2f);
    p = fmaf(p, r, 1.66666666666666657415e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int e = (int)n;
    if (e > 127) { p = p * 1.7014118346046923e38f; e -= 127; }      /* 2^127 */
    if (e < -126) { p = p * 1.1754943508222875e-38f; e += 126; }    /* 2^-126 */
    return p * bits_f((uint32_t)(e + 127) << 23);
}

/* SiLU and sigmoid as kernels/joint_projection.cu:95 and :136 write them
 * (x / (1 + exp(-x)), 1 / (1 + exp(-x))), with k2o_exp for exp. */
float k2o_silu(float x) { return x / (1.0f + k2o_exp(-x)); }
float k2o_sigmoid(float x) { return 1.0f / (1.0f + k2o_exp(-x)); }

/* ------------------------------------------------ rotation + INT4 packing */

/* fp32(1/sqrt(128)): the normalisation of the Sylvester H128 block. */
#define K2_HSCALE 0.0883883461356163024902343750f

/* In-place unnormalised Walsh-Hadamard transform of 128 fp32 values: seven
 * butterfly stages (a, b) -> (a + b, a - b) between elements h apart, each
 * sum rounded to fp32, in the order h = 2, 4, 8, 1, 16, 32, 64.  The
 * 1/sqrt(128) normalisation of the orthonormal 128x128 block-Hadamard is not
 * applied here: k2o_quant_group128 folds it into the scale and the
 * per-element multiplier.  The reference rotates with comfy-kitchen's
 * ConvRot stages (kernels/norm_quant.cu:40-60, helpers not vendored); the
 * stage order and rounding here are this project's own contract (any order
 * is the same transform in exact arithmetic). */
static const int k2o_hadamard_order[7] = {2, 4, 8, 1, 16, 32, 64};
void k2o_hadamard128(float* v) {
    for (int st = 0; st < 7; ++st) {
        const int h = k2o_hadamard_order[st];
        for (int i = 0; i < 128; i += 2 * h)
            for (int j = i; j < i + h; ++j) {
                float a = v[j], b = v[j + h];
                v[j] = a + b;
                v[j + h] = a - b;
            }
    }
}

/* Quantise one group of 128 raw Hadamard outputs u (k2o_hadamard128) to
 * INT4 codes of the normalised rotation u * K2_HSCALE:
 *   scale = fp16(min(fp32(max|u| * K2_QSCALE), 65504))
 *           K2_QSCALE = fp32(1/(7*sqrt(128))): absmax of the normalised
 *           group over the INT4 maximum 7, as one multiply
 *   c     = fp32(K2_HSCALE * fp32(1 / scale))   (0 for a zero scale)
 *   code  = clamp(rne(u * c), -8, 7)      (u * c exact: one rounding)
 * two codes per byte, low nibble = even column.  Multiplying by the
 * reciprocal of the scale is the reference's quantisation step
 * (kernels/norm_quant.cu:62-66: inverse = 1.f/row_scale, then
 * quantize_int4_pack4_word(..., inverse, ...)), here with one fp16 scale per
 * group of 128.  The rounding is written as fma(u, c, 1.5*2^23): its sum
 * lies on the integer grid, so it is rne(u*c) + 1.5*2^23 exactly; codes of
 * NaN inputs are unspecified (the scale ignores them). */
#define K2_ROUND_MAGIC 12582912.0f
#define K2_QSCALE 0.012626906856894493103027343750f
void k2o_quant_group128(const float* u, uint8_t* q, uint16_t* s) {
    float amax = 0.0f;
    for (int j = 0; j < 128; ++j) amax = fmaxf(amax, fabsf(u[j]));
    float sf = amax * K2_QSCALE;
    if (sf > 65504.0f) sf = 65504.0f;
    uint16_t sh = k2o_f32_to_f16(sf);
    float sd = k2o_f16_to_f32(sh);
    *s = sh;
    float c = sd > 0.0f ? K2_HSCALE * (1.0f / sd) : 0.0f;
    for (int j = 0; j < 128; j += 2) {
        int code[2];
        for (int t = 0; t < 2; ++t) {
            float r = fmaf(u[j + t], c, K2_ROUND_MAGIC);
            r = fminf(fmaxf(r, K2_ROUND_MAGIC - 8.0f), K2_ROUND_MAGIC + 7.0f);
            code[t] = (int)(r - K2_ROUND_MAGIC);
        }
        q[j / 2] = (uint8_t)((code[0] & 0xf) | ((code[1] & 0xf) << 4));
    }
}

/* ------------------------------------------------------------- norm_quant */

/* Reduction order of kernels/norm_quant.cu:20-31 (ATen's vectorised RMSNorm):
 * 128 lanes, lane t accumulates fmaf(v, v, sum) over columns t*4 + j + 512*i
 * (j inner), a shfl_down tree (16, 8, 4, 2, 1) inside each warp of 32 lanes,
 * then (w2 + w0) + (w3 + w1). */
static float row_sumsq(const uint16_t* x, int K) {
    float warp[4];
    for (int w = 0; w < 4; ++w) {
        float lane[32];
        for (int l = 0; l < 32; ++l) {
            int t = 32 * w + l;
            float sum = 0.0f;
            for (int col = t * 4; col < K; col += 512)
                for (int j = 0; j < 4; ++j) {
                    float v = col + j < K ? bf(x[col + j]) : 0.0f;
                    sum = fmaf(v, v, sum);
                }
            lane[l] = sum;
        }
        for (int off = 16; off; off >>= 1)
            for (int l = 0; l < off; ++l) lane[l] = lane[l] + lane[l + off];
        warp[w] = lane[0];
    }
    return (warp[2] + warp[0]) + (warp[3] + warp[1]);
}

/* Batch row of the modulation vectors, kernels/norm_quant.cu:32. */
static int mod_row(int row, int length, int cut, int batch) {
    int b = row / length;
    if (cut >= 0 && row % length >= cut) b += batch;
    return b;
}

/*
 * Fused RMSNorm -> adaLN modulation -> H128 rotation -> group-128 INT4 pack.
 * Restates kernels/norm_quant.cu:11-67 (norm_mod_quant), with the group-128
 * rotation and fp16 scales of k2o_hadamard128 / k2o_quant_group128:
 *   inv = rsqrt_rn(sum/K + eps)                          (:30-31)
 *   y   = bf16((x*inv)*(w+1))                            (:34)
 *   f   = bf16(scale+1); y = bf16(y*f); v = bf16(y+shift) (:35-37)
 * x bf16 [rows,K]; w fp32 [K] (the "w+1" form, native_schedule.py:252-253);
 * scale/shift bf16 [nbatch,K]; q u8 [rows,K/2]; s fp16 [rows,K/128].
 */
int k2o_norm_quant(const uint16_t* x, const float* w, const uint16_t* scale,
                   const uint16_t* shift, uint8_t* q, uint16_t* s, int rows, int K,
                   int length, int cut, int batch, float eps) {
    if (rows <= 0 || K <= 0 || K % 128 || length <= 0) return 1;
    for (int row = 0; row < rows; ++row) {
        const uint16_t* xr = x + (int64_t)row * K;
        float* v = (float*)malloc(sizeof(float) * (size_t)K);
        float sum = row_sumsq(xr, K);
        float inv = k2o_rsqrt_rn(sum / (float)K + eps);
        int b = mod_row(row, length, cut, batch);
        for (int col = 0; col < K; ++col) {
            float t = bf(xr[col]) * inv;
            float w1 = w[col] + 1.0f;
            float y = bfr(t * w1);
            float f = bfr(bf(scale[(int64_t)b * K + col]) + 1.0f);
            y = bfr(y * f);
            v[col] = bfr(y + bf(shift[(int64_t)b * K + col]));
        }
        for (int g = 0; g < K / 128; ++g) {
            k2o_hadamard128(v + g * 128);
            k2o_quant_group128(v + g * 128, q + (int64_t)row * (K / 2) + g * 64,
                               s + (int64_t)row * (K / 128) + g);
        }
        free(v);
    }
    return 0;
}

/* The RMSNorm + modulation half of k2o_norm_quant alone (bf16 out): the
 * semantics of kernels/native_dispatch.cu:44-62 (norm_mod) and the Triton
 * twin forward_kernels.py:13-45 (_norm_mod), with the reduction order above. */
int k2o_norm_mod(const uint16_t* x, const float* w, const uint16_t* scale, const uint16_t* shift,
                 uint16_t* out, int rows, int K, int length, int cut, int batch, float eps) {
    if (rows <= 0 || K <= 0 || length <= 0) return 1;
    for (int row = 0; row < rows; ++row) {
        const uint16_t* xr = x + (int64_t)row * K;
        float sum = row_sumsq(xr, K);
        float inv = k2o_rsqrt_rn(sum / (float)K + eps);
        int b = mod_row(row, length, cut, batch);
        for (int col = 0; col < K; ++col) {
            float t = bf(xr[col]) * inv;
            float w1 = w[col] + 1.0f;
            float y = bfr(t * w1);
            float f = bfr(bf(scale[(int64_t)b * K + col]) + 1.0f);
            y = bfr(y * f);
            out[(int64_t)row * K + col] = k2o_f32_to_bf16(y + bf(shift[(int64_t)b * K + col]));
        }
    }
    return 0;
}

/* Rotation + quantisation of an already-formed bf16 activation (the input
 * quantisation that native_runtime.cpp:268-271 `quantize` performs before the
 * out-projection), with the group-128 rotation and scales above. */
int k2o_rotate_quant(const uint16_t* x, uint8_t* q, uint16_t* s, int rows, int K) {
    if (rows <= 0 || K <= 0 || K % 128) return 1;
    for (int row = 0; row < rows; ++row) {
        float v[128];
        for (int g = 0; g < K / 128; ++g) {
            for (int j = 0; j < 128; ++j) v[j] = bf(x[(int64_t)row * K + g * 128 + j]);
            k2o_hadamard128(v);
            k2o_quant_group128(v, q + (int64_t)row * (K / 2) + g * 64,
                               s + (int64_t)row * (K / 128) + g);
        }
    }
    return 0;
}

/* ------------------------------------------------------------- W4A4 GEMM */

static void unpack_row(const uint8_t* p, int8_t* out, int K) {
    for (int i = 0; i < K / 2; ++i) {
        int lo = p[i] & 0xf, hi = p[i] >> 4;
        out[2 * i] = (int8_t)(lo >= 8 ? lo - 16 : lo);
        out[2 * i + 1] = (int8_t)(hi >= 8 ? hi - 16 : hi);
    }
}

/* Unpacks packed INT4 rows [n, K/2] (+ fp16 scales [n, K/128]) into int8
 * codes [n, K] and fp32 scales [n, K/128]. */
int k2o_unpack_weight(const uint8_t* W, const uint16_t* sW, int n, int K, int8_t* wu, float* swf) {
    if (K % 128) return 1;
    int G = K / 128;
    for (int c = 0; c < n; ++c) {
        unpack_row(W + (int64_t)c * (K / 2), wu + (int64_t)c * K, K);
        for (int g = 0; g < G; ++g) swf[(int64_t)c * G + g] = k2o_f16_to_f32(sW[(int64_t)c * G + g]);
    }
    return 0;
}

/*
 * Group-scaled W4A4 GEMM, fp32 result p[r,c] for the selected rows and the
 * output columns [c0, c1).
 * Accumulation: int32 per (row, 128-wide K group) as the s4 mma of
 * kernels/joint_projection.cu:51-56 produces; dequant of the contract
 * (group-128 scales on both operands; the reference's per-row/per-channel
 * version is T(float(acc)*xs*ws), kernels/joint_projection.cu:57-59):
 *     p = 0;  for g:  u = fp32(float(acc_g) * sA[r,g]);  p = fmaf(u, sW[c,g], p)
 * A u8 [M,K/2] + fp16 [M,K/128]; W given unpacked (k2o_unpack_weight).
 * rows == NULL selects rows 0..nrows-1.  out fp32 [nrows, ldo] (column c at
 * out[i*ldo + c]); acc_out (optional) int32 [nrows, N, K/128].
 */
int k2o_gemm_w4a4_cols(const uint8_t* A, const uint16_t* sA, const int8_t* wu, const float* swf, int M, int N,
                       int K, const int* rows, int nrows, int c0, int c1, float* out, int ldo, int32_t* acc_out) {
    if (K % 128 || M <= 0 || N <= 0 || c0 < 0 || c1 > N) return 1;
    int G = K / 128;
    int8_t* au = (int8_t*)malloc((size_t)K);
    float* saf = (float*)malloc(sizeof(float) * (size_t)G);
    for (int i = 0; i < nrows; ++i) {
        int r = rows ? rows[i] : i;
        unpack_row(A + (int64_t)r * (K / 2), au, K);
        for (int g = 0; g < G; ++g) saf[g] = k2o_f16_to_f32(sA[(int64_t)r * G + g]);
        for (int c = c0; c < c1; ++c) {
            const int8_t* wr = wu + (int64_t)c * K;
            float p = 0.0f;
            for (int g = 0; g < G; ++g) {
                int32_t acc = 0;
                for (int k = 0; k < 128; ++k) acc += (int32_t)au[g * 128 + k] * (int32_t)wr[g * 128 + k];
                if (acc_out) acc_out[((int64_t)i * N + c) * G + g] = acc;
                float u = (float)acc * saf[g];
                p = fmaf(u, swf[(int64_t)c * G + g], p);
            }
            out[(int64_t)i * ldo + c] = p;
        }
    }
    free(au);
    free(saf);
    return 0;
}

/* One group step of the dequant above, for callers that form the group's
 * int32 accumulators elsewhere (oracle.py sums the integer codes of a group
 * with an fp32 BLAS matmul: every product and partial sum is an integer of
 * magnitude <= 128*8*8 < 2^24, so the fp32 sum is the exact accumulator in
 * any order):
 *     p[i,c] = fmaf(fp32(acc[i,c] * sa[i]), sw[c], p[i,c])
 * acc, p fp32 [rows, N]; sa fp32 [rows] (this group's activation scales);
 * sw fp32 [N] (this group's weight scales). */
static void dequant_group_rows(const float* acc, const float* sa, const float* sw, float* p, int rows, int N) {
    for (int i = 0; i < rows; ++i) {
        const float* a = acc + (int64_t)i * N;
        float* o = p + (int64_t)i * N;
        const float s = sa[i];
        for (int c = 0; c < N; ++c) {
            float u = a[c] * s;
            o[c] = fmaf(u, sw[c], o[c]);
        }
    }
}
/* The same loop compiled for CPUs with an FMA unit: fmaf() becomes the
 * (correctly rounded) fused instruction and the loop vectorises; chosen at run
 * time, so the library still loads on x86-64-v2 hosts. */
__attribute__((target("avx2,fma"))) static void dequant_group_rows_fma(const float* acc, const float* sa,
                                                                        const float* sw, float* p, int rows,
                                                                        int N) {
    for (int i = 0; i < rows; ++i) {
        const float* a = acc + (int64_t)i * N;
        float* o = p + (int64_t)i * N;
        const float s = sa[i];
        for (int c = 0; c < N; ++c) {
            float u = a[c] * s;
            o[c] = fmaf(u, sw[c], o[c]);
        }
    }
}
int k2o_dequant_group(const float* acc, const float* sa, const float* sw, float* p, int rows, int N) {
    if (rows < 0 || N <= 0) return 1;
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma"))
        dequant_group_rows_fma(acc, sa, sw, p, rows, N);
    else
        dequant_group_rows(acc, sa, sw, p, rows, N);
    return 0;
}

/* ------------------------------------------------------------- epilogues */

/* Per-head RMSNorm over 128 channels with the reduction order of
 * kernels/joint_projection.cu:141-146 (lane l holds channels 4l..4l+3, fmaf in
 * j order, shfl_down tree, lane 0's total), then adjacent-pair RoPE
 * (:147-152):  a = bf16((v*inv)*(w+1)), o0 = bf16(fmaf(f0,a,f1*b)),
 * o1 = bf16(fmaf(f2,a,f3*b)).  v = bf16(p) is the rounded projection (:134).
 * p fp32 [nrows, ld] (cols [0, heads*128) used); normw fp32 [128];
 * freqs fp32 [L,64,2,2]; token = row_index % L; out bf16 [nrows, heads*128]. */
int k2o_qk_norm_rope(const float* p, int nrows, int ld, int heads, const float* normw, float eps,
                     const float* freqs, int L, const int* rows, uint16_t* out) {
    for (int i = 0; i < nrows; ++i) {
        int r = rows ? rows[i] : i;
        int token = r % L;
        for (int h = 0; h < heads; ++h) {
            float v[128];
            for (int j = 0; j < 128; ++j) v[j] = bfr(p[(int64_t)i * ld + h * 128 + j]);
            float lane[32];
            for (int l = 0; l < 32; ++l) {
                float s = 0.0f;
                for (int j = 0; j < 4; ++j) s = fmaf(v[4 * l + j], v[4 * l + j], s);
                lane[l] = s;
            }
            for (int off = 16; off; off >>= 1)
                for (int l = 0; l < off; ++l) lane[l] = lane[l] + lane[l + off];
            float inv = k2o_rsqrt_rn(lane[0] / 128.0f + eps);
            for (int pr = 0; pr < 64; ++pr) {
                int c = 2 * pr;
                float a = bfr((v[c] * inv) * (normw[c] + 1.0f));
                float b = bfr((v[c + 1] * inv) * (normw[c + 1] + 1.0f));
                const float* f = freqs + ((int64_t)token * 64 + pr) * 4;
                uint16_t* o = out + (int64_t)i * heads * 128 + h * 128 + c;
                o[0] = k2o_f32_to_bf16(fmaf(f[0], a, f[1] * b));
                o[1] = k2o_f32_to_bf16(fmaf(f[2], a, f[3] * b));
            }
        }
    }
    return 0;
}

/* Gated residual of kernels/int4_epilogue.cu:24-37 / joint_projection.cu:178-179:
 * out = bf16(resid + bf16(bf16(p) * gate[b,c])), b = row / length.
 * p fp32 [nrows,N]; gate bf16 [nbatch,N]; resid/out bf16 [nrows,N]. */
int k2o_gated_residual(const float* p, int nrows, int N, const uint16_t* gate,
                       const uint16_t* resid, int length, const int* rows, uint16_t* out) {
    for (int i = 0; i < nrows; ++i) {
        int r = rows ? rows[i] : i;
        int b = r / length;
        for (int c = 0; c < N; ++c) {
            float pv = bfr(p[(int64_t)i * N + c]);
            float g = bfr(pv * bf(gate[(int64_t)b * N + c]));
            out[(int64_t)i * N + c] = k2o_f32_to_bf16(bf(resid[(int64_t)i * N + c]) + g);
        }
    }
    return 0;
}

/* SwiGLU of kernels/joint_projection.cu:94-96 (g = bf16(pg), u = bf16(pu),
 * a = bf16(silu(g)), h = bf16(a*u)) followed by the contract's fused input
 * quantisation of the down projection (H128 rotation + group-128 INT4).
 * pg/pu fp32 [nrows,F]; hq u8 [nrows,F/2]; hs fp16 [nrows,F/128];
 * h (optional) bf16 [nrows,F]. */
int k2o_swiglu_quant(const float* pg, const float* pu, int nrows, int F, uint8_t* hq,
                     uint16_t* hs, uint16_t* h) {
    if (F % 128) return 1;
    for (int i = 0; i < nrows; ++i) {
        float v[128];
        for (int g = 0; g < F / 128; ++g) {
            for (int j = 0; j < 128; ++j) {
                int64_t idx = (int64_t)i * F + g * 128 + j;
                float gv = bfr(pg[idx]);
                float uv = bfr(pu[idx]);
                float a = bfr(k2o_silu(gv));
                v[j] = bfr(a * uv);
                if (h) h[idx] = k2o_f32_to_bf16(v[j]);
            }
            k2o_hadamard128(v);
            k2o_quant_group128(v, hq + (int64_t)i * (F / 2) + g * 64, hs + (int64_t)i * (F / 128) + g);
        }
    }
    return 0;
}

/* Attention gate of kernels/joint_projection.cu:136: bf16(sigmoid(bf16(p))). */
int k2o_sigmoid_gate(const float* p, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = k2o_f32_to_bf16(k2o_sigmoid(bfr(p[i])));
    return 0;
}

/* Vectorised helpers for the Python side. */
void k2o_exp_vec(const float* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = k2o_exp(x[i]);
}
void k2o_bf16_round_vec(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = k2o_f32_to_bf16(x[i]);
}

/* ------------------------------------------- reference contract (parity) */

/* The reference runtime's INT4 / int8 activation quantisation (its own data
 * contract, native_runtime.cpp:262-271, 432-447), as the library's
 * reference-named exports compute it (csrc/ref_contract.cuh):
 *   optional RMSNorm + modulation with the rounding points of k2o_norm_mod
 *   (kernels/norm_quant.cu:20-38), bf16 values v;
 *   ConvRot in groups of G = 16, 64 or 256 (0: none): radix-4 stages at
 *   strides 1, 4, 16, 64 (kernels/norm_quant.cu:48-60 names the stages; the
 *   stage arithmetic lives in comfy-kitchen, not in the reference, and is this
 *   project's restatement): (a, b, c, d) -> bf16(((a+b)+(c+d))*0.5),
 *   bf16(((a-b)+(c-d))*0.5), bf16(((a+b)-(c+d))*0.5), bf16(((a-b)-(c-d))*0.5);
 *   scale = max(min(amax, bf16 max)/qmax, 1e-10) per row (qmax 7 or 127),
 *   inverse = 1/scale, code = clamp(rne(v*inverse), -8|-127, 7|127)
 *   (kernels/norm_quant.cu:61-66);
 *   bits 4: two codes per byte, even column low; bits 8: int8 codes.
 * x bf16 [rows, K]; w/scale/shift as k2o_norm_mod (w == NULL: no norm). */
int k2o_ref_quant(const uint16_t* x, const float* w, const uint16_t* scale, const uint16_t* shift, uint8_t* q,
                  float* s, int rows, int K, int length, int cut, int batch, float eps, int group, int bits) {
    if (rows <= 0 || K <= 0 || K % 8 || (group != 0 && group != 16 && group != 64 && group != 256) ||
        (group && K % group) || (bits != 4 && bits != 8))
        return 1;
    uint16_t* v = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)K);
    const float qmax = bits == 4 ? 7.0f : 127.0f;
    for (int r = 0; r < rows; ++r) {
        const uint16_t* xr = x + (int64_t)r * K;
        if (w) {
            /* one row through the norm/mod restatement, with the row's latent */
            int b = r / length;
            if (cut >= 0 && r % length >= cut) b += batch;
            k2o_norm_mod(xr, w, scale ? scale + (int64_t)b * K : NULL, shift ? shift + (int64_t)b * K : NULL, v, 1,
                         K, 1, -1, 1, eps);
        } else {
            memcpy(v, xr, sizeof(uint16_t) * (size_t)K);
        }
        for (int st = 1; group && st < group; st *= 4) {
            for (int t = 0; t < K / 4; ++t) {
                const int base = (t / st) * 4 * st + (t % st);
                const float a = bf(v[base]), bb = bf(v[base + st]), c = bf(v[base + 2 * st]), d = bf(v[base + 3 * st]);
                const float s01 = a + bb, d01 = a - bb, s23 = c + d, d23 = c - d;
                v[base] = k2o_f32_to_bf16((s01 + s23) * 0.5f);
                v[base + st] = k2o_f32_to_bf16((d01 + d23) * 0.5f);
                v[base + 2 * st] = k2o_f32_to_bf16((s01 - s23) * 0.5f);
                v[base + 3 * st] = k2o_f32_to_bf16((d01 - d23) * 0.5f);
            }
        }
        float amax = 0.0f;
        for (int c = 0; c < K; ++c) amax = fmaxf(amax, fabsf(bf(v[c])));
        if (amax > 3.3895313892515355e38f) amax = 3.3895313892515355e38f;
        float sc = amax / qmax;
        if (sc < 1e-10f) sc = 1e-10f;
        s[r] = sc;
        const float inverse = 1.0f / sc;
        if (bits == 4) {
            uint8_t* qr = q + (int64_t)r * (K / 2);
            for (int i = 0; i < K / 2; ++i) {
                float c0 = rintf(bf(v[2 * i]) * inverse), c1 = rintf(bf(v[2 * i + 1]) * inverse);
                c0 = fminf(fmaxf(c0, -8.0f), 7.0f);
                c1 = fminf(fmaxf(c1, -8.0f), 7.0f);
                qr[i] = (uint8_t)(((int)c0 & 0xF) | (((int)c1 & 0xF) << 4));
            }
        } else {
            int8_t* qr = (int8_t*)q + (int64_t)r * K;
            for (int i = 0; i < K; ++i) {
                float c = rintf(bf(v[i]) * inverse);
                qr[i] = (int8_t)(int)fminf(fmaxf(c, -127.0f), 127.0f);
            }
        }
    }
    free(v);
    return 0;
}
