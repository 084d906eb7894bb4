// abi_reference.cuh -- exports under the reference's kernel-library names,
// with the reference's data contract.
//
// native_runtime.cpp resolves these with dlopen(RTLD_NOW|RTLD_LOCAL) + dlsym:
// configure() loads k2_quant4, k2_quant8, k2_gemm4, k2_dequant8, k2_fp8,
// k2_norm, k2_elementwise and k2_rope (native_runtime.cpp:514-519), the
// epilogue / QK libraries k2_int4_gated_residual and k2_int4_qk_norm_rope
// (:520-521), configure_joint() k2_int4_swiglu, k2_int4_qkv and
// k2_int4_residual_norm (:524-528), configure_norm_quant()
// k2_norm_mod_quant4 (:529).  Every one of them is exported here with the
// reference's argument order and with the buffers the reference runtime
// allocates for it (native_runtime.cpp:262-311, 399-447):
//   * INT4 activations: packed [m, k/2] (even column in the low nibble) with
//     ONE fp32 scale per row [m, 1], rotated by ConvRot in groups of 16, 64
//     or 256 (ref_contract.cuh);
//   * INT4 weights: packed [n, k/2] as a ConvRot W4A4 checkpoint stores them,
//     with one fp32 scale per output channel [n]; nothing is prepared ahead:
//     the GEMM unpacks the rows it streams (GM_REF4);
//   * projections: T(fp32(fp32(acc * xs[r]) * ws[c])), acc over all of k
//     (kernels/joint_projection.cu:57-59), then the epilogues of
//     kernels/joint_projection.cu and kernels/int4_epilogue.cu;
//   * dtype: 0 = bf16 for the k2_int4_* family (kernels/joint_projection.cu:208),
//     2 = bf16 for the others (native_runtime.cpp:83).  fp16 (and fp32)
//     tensors are rejected: this build computes bf16 activations only.
// Return codes: 0, or cudaErrorInvalidValue for unsupported shapes/dtypes.
// The reference's void exports cannot return a status: they launch nothing
// on unsupported input and leave the status for k2b_shim_status() (the
// reference's callers check cudaGetLastError() after them,
// native_runtime.cpp:265,284).
// The group-128 BASELINE contract of this library is served by the k2b_*
// entry points only; no reference-named export writes group-128 scales.

namespace {
thread_local int g_shim_status = 0;
void shim_status(int rc) {
  if (rc) g_shim_status = rc;
}
bool ref_group_ok(int group, int64_t k) {
  return (group == 0 || group == 16 || group == 64 || group == 256) && (group == 0 || k % group == 0);
}
// Reference-contract quantisation launch: per-row scale, optional norm +
// modulation (x bf16 [rows, K]).
// INT4 rows of K % 512 == 0 with a ConvRot group take the fast kernel
// (ref_quant4_fast_kernel; bytes: e4m3 code bytes [rows, K] instead of
// packed nibbles), the rest the one-CTA-per-row kernel.
template <bool NORM, int BITS>
int ref_quant_launch(const void* x, const void* w, const void* scale, const void* shift, void* q, void* s,
                     int64_t rows, int64_t K, int length, int cut, int batch, float eps, int group,
                     cudaStream_t st, bool bytes = false) {
  if (rows <= 0 || K <= 0 || K % 8 || K > 32768 || rows > INT32_MAX || !ref_group_ok(group, K) || !x || !q || !s)
    return (int)cudaErrorInvalidValue;
  if (NORM && (!w || length <= 0 || batch <= 0 || (scale == nullptr) != (shift == nullptr)))
    return (int)cudaErrorInvalidValue;
  const bool fast = BITS == 4 && K % 512 == 0 && group != 0 && aligned16(x) && aligned16(q) &&
                    (!NORM || (aligned16(w) && (!scale || (aligned16(scale) && aligned16(shift)))));
  if (bytes && !fast) return (int)cudaErrorInvalidValue;
  if (fast) {
    const size_t smem = (size_t)K * 2;
    auto kern = bytes ? k2b::ref_quant4_fast_kernel<NORM, true> : k2b::ref_quant4_fast_kernel<NORM, false>;
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return (int)e;
    }
    kern<<<(unsigned)rows, k2b::kRefFastThreads, smem, st>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const float*>(w), static_cast<const __nv_bfloat16*>(scale),
        static_cast<const __nv_bfloat16*>(shift), static_cast<uint8_t*>(q), static_cast<float*>(s), (int)K, length,
        cut, batch, eps, group);
    return (int)cudaGetLastError();
  }
  const size_t smem = (size_t)K * 2;
  auto kern = k2b::ref_quant_kernel<NORM, BITS>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
  }
  kern<<<(unsigned)rows, k2b::kRefThreads, smem, st>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const float*>(w), static_cast<const __nv_bfloat16*>(scale),
      static_cast<const __nv_bfloat16*>(shift), static_cast<uint8_t*>(q), static_cast<float*>(s), (int)K, length,
      cut, batch, eps, group);
  return (int)cudaGetLastError();
}
// Reference-contract INT4 GEMM over the segments `d` (GM_REF4).
int ref_gemm(const void* a, const void* xs, int m, int k, SegDesc* d, int nseg, const float* freqs,
             const void* gate, const void* resid, const float* bias, cudaStream_t st) {
  if (m <= 0 || k <= 0 || k % 128) return (int)cudaErrorInvalidValue;
  RefScales r;
  r.xs = static_cast<const float*>(xs);
  r.bias = bias;
  return gemm_launch(a, nullptr, m, k, d, nseg, m, freqs, gate, resid, st, nullptr, 0, 0, 0, GM_REF4, &r);
}
}  // namespace

// Last non-zero status of a void shim on this host thread (0 if none).
K2B_EXPORT int k2b_shim_status(int reset) {
  const int rc = g_shim_status;
  if (reset) g_shim_status = 0;
  return rc;
}

// kernels/norm_quant.cu:89-96: RMSNorm + modulation + ConvRot (group 16, 64,
// 256) + per-row INT4; q int8 [rows, K/2], scales fp32 [rows, 1].
K2B_EXPORT int k2_norm_mod_quant4(const void* x, const void* norm, const void* scale, const void* shift, void* q,
                                  void* scales, int rows, int K, int length, int cut, int batch, float eps, int group,
                                  int dtype, void* stream) {
  if (dtype != 2 || group == 0 || !scale || !shift) return (int)cudaErrorInvalidValue;
  return ref_quant_launch<true, 4>(x, norm, scale, shift, q, scales, rows, K, length, cut, batch, eps, group,
                                   (cudaStream_t)stream);
}

// kernels/native_dispatch.cu:23-25 (comfy-kitchen's ConvRot INT4 quantiser):
// q int8 [m, k/2], s fp32 [m, 1].
K2B_EXPORT void k2_quant4(const void* x, void* q, void* s, int64_t m, int64_t k, int group, int dtype, void* stream) {
  shim_status(dtype != 2 || group == 0
                  ? (int)cudaErrorInvalidValue
                  : ref_quant_launch<false, 4>(x, nullptr, nullptr, nullptr, q, s, m, k, 1, -1, 1, 0.0f, group,
                                               (cudaStream_t)stream));
}

// k2_quant4 / k2_norm_mod_quant4 with the codes as e4m3 bytes [rows, K] (the
// byte-operand GEMMs' container) instead of packed nibbles; K % 512 == 0.
K2B_EXPORT int k2b_ref_quant4_e4m3(const void* x, void* q8, void* s, long long m, long long k, int group,
                                   void* stream) {
  if (group == 0) return (int)cudaErrorInvalidValue;
  return ref_quant_launch<false, 4>(x, nullptr, nullptr, nullptr, q8, s, m, k, 1, -1, 1, 0.0f, group,
                                    (cudaStream_t)stream, true);
}
K2B_EXPORT int k2b_ref_norm_quant4_e4m3(const void* x, const void* norm, const void* scale, const void* shift,
                                        void* q8, void* scales, int rows, int K, int length, int cut, int batch,
                                        float eps, int group, void* stream) {
  if (group == 0 || !scale || !shift) return (int)cudaErrorInvalidValue;
  return ref_quant_launch<true, 4>(x, norm, scale, shift, q8, scales, rows, K, length, cut, batch, eps, group,
                                   (cudaStream_t)stream, true);
}

// kernels/native_dispatch.cu:30-33: rowwise int8 (after ConvRot when group
// != 0); q int8 [m, k], s fp32 [m, 1].
K2B_EXPORT void k2_quant8(const void* x, void* q, void* s, int64_t m, int64_t k, int group, int dtype, void* stream) {
  shim_status(dtype != 2 ? (int)cudaErrorInvalidValue
                         : ref_quant_launch<false, 8>(x, nullptr, nullptr, nullptr, q, s, m, k, 1, -1, 1, 0.0f, group,
                                                      (cudaStream_t)stream));
}

// kernels/native_dispatch.cu:26-29: INT4 projection T(acc * xs * ws [+ bias])
// of packed a [m, k/2] (xs fp32 [m]) and packed w [n, k/2] (ws fp32 [n]);
// bias fp32 [n] or null; out bf16 [m, n].
K2B_EXPORT void k2_gemm4(const void* a, const void* w, const void* xs, const void* ws, const void* bias, void* out,
                         int64_t m, int64_t n, int64_t k, int dtype, void* stream) {
  if (dtype != 2 || m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) {
    shim_status((int)cudaErrorInvalidValue);
    return;
  }
  SegDesc d = {SEG_BF16, (int)n, w, ws, out, (int)n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  shim_status(ref_gemm(a, xs, (int)m, (int)k, &d, 1, nullptr, nullptr, nullptr, static_cast<const float*>(bias),
                       (cudaStream_t)stream));
}

// kernels/native_dispatch.cu:34-36: int32 a [m, n] (an INT8 GEMM's
// accumulators, native_runtime.cpp:300-305) -> bf16 T(a * xs * ws + bias),
// ws per channel (ns = n) or one value (ns = 1), bias bf16 [n] or null.
K2B_EXPORT void k2_dequant8(const void* a, const void* xs, const void* ws, const void* bias, void* out, int64_t m,
                            int64_t n, int64_t ns, int dtype, void* stream) {
  if (dtype != 2 || m <= 0 || n <= 0 || n > INT32_MAX || (ns != 1 && ns != n) || !a || !xs || !ws || !out) {
    shim_status((int)cudaErrorInvalidValue);
    return;
  }
  const int64_t total = m * n;
  const int64_t blocks = (total + 255) / 256;
  ref_dequant8_kernel<<<(unsigned)(blocks < 148 * 32 ? blocks : 148 * 32), 256, 0, (cudaStream_t)stream>>>(
      static_cast<const int32_t*>(a), static_cast<const float*>(xs), static_cast<const float*>(ws),
      static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(out), m, (int)n, (int)ns);
  shim_status((int)cudaGetLastError());
}

// kernels/native_dispatch.cu:37-40: fp8 quantise (y = fp8(x / s)) or
// dequantise (y = T(x * s)) with one fp32 scale s[0]; element codes 0 fp32,
// 1 fp16, 2 bf16, 5 e4m3, 6 e5m2 (native_runtime.cpp:273-283, 307-310).
K2B_EXPORT void k2_fp8(const void* x, void* y, const void* s, int64_t n, int src, int dst, bool quant, void* stream) {
  const bool ok = n >= 0 && x && y && s &&
                  (quant ? (src >= 0 && src <= 2 && (dst == 5 || dst == 6))
                         : ((src == 5 || src == 6) && dst >= 0 && dst <= 2));
  if (!ok) {
    shim_status((int)cudaErrorInvalidValue);
    return;
  }
  if (n == 0) return;
  const int64_t blocks = (n + 255) / 256;
  ref_fp8_kernel<<<(unsigned)(blocks < 148 * 32 ? blocks : 148 * 32), 256, 0, (cudaStream_t)stream>>>(
      x, y, static_cast<const float*>(s), n, src, dst, quant ? 1 : 0);
  shim_status((int)cudaGetLastError());
}

// kernels/joint_projection.cu:222-225 (batch 1: freq [m, 64, 2, 2]): Q and K
// per-head RMSNorm + RoPE, V plain, the optional gate sigmoided.
K2B_EXPORT int k2_int4_qkv(const void* a, const void* wq, const void* wk, const void* wv, const void* wg,
                           const void* xs, const void* sq, const void* sk, const void* sv, const void* sg,
                           const void* nq, const void* nk, const void* freq, void* qo, void* ko, void* vo, void* go,
                           int m, int qwidth, int kvwidth, int k, int dtype, float eq, float ek, void* stream) {
  if (dtype != 0 || qwidth <= 0 || kvwidth <= 0 || qwidth % 128 || kvwidth % 128 || !freq)
    return (int)cudaErrorInvalidValue;
  SegDesc d[4] = {
      {SEG_QKNORM, qwidth, wq, sq, qo, qwidth, static_cast<const float*>(nq), eq, nullptr, nullptr, nullptr},
      {SEG_QKNORM, kvwidth, wk, sk, ko, kvwidth, static_cast<const float*>(nk), ek, nullptr, nullptr, nullptr},
      {SEG_BF16, kvwidth, wv, sv, vo, kvwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
      {SEG_SIGMOID, qwidth, wg, sg, go, qwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
  };
  return ref_gemm(a, xs, m, k, d, (wg && go) ? 4 : 3, static_cast<const float*>(freq), nullptr, nullptr, nullptr,
                  (cudaStream_t)stream);
}

// kernels/joint_projection.cu:204-205: h = T(T(silu(T(p_g))) * T(p_u)).
K2B_EXPORT int k2_int4_swiglu(const void* a, const void* wg, const void* wu, const void* xs, const void* sg,
                              const void* su, void* out, int m, int n, int k, int dtype, void* stream) {
  if (dtype != 0 || n <= 0 || n % 128) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_SWIGLU_BF16, n, wg, sg, out, n, nullptr, 0.0f, nullptr, wu, su};
  return ref_gemm(a, xs, m, k, &d, 1, nullptr, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

// kernels/int4_epilogue.cu:77-78: out = T(resid + T(T(p) * gate[c])); config
// selects a CUTLASS tile there, one tile here (gate bf16 [n], batch 1).
K2B_EXPORT int k2_int4_gated_residual(void* a, void* w, void* xs, void* ws, void* gate, void* residual, void* output,
                                      int m, int n, int k, int dtype, int config, void* stream) {
  if (dtype != 0 || (config != 0 && config != 1)) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_RESIDUAL, n, w, ws, output, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  return ref_gemm(a, xs, m, k, &d, 1, nullptr, gate, residual, nullptr, (cudaStream_t)stream);
}

// kernels/qk_norm_rope.cu:135: per-head RMSNorm + RoPE of T(p), n % 128 == 0.
K2B_EXPORT int k2_int4_qk_norm_rope(void* a, void* w, void* xs, void* ws, void* norm, void* freqs, void* output, int m,
                                    int n, int k, int dtype, float eps, void* stream) {
  if (dtype != 0 || n % 128 || !freqs) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_QKNORM, n, w, ws, output, n, static_cast<const float*>(norm), eps, nullptr, nullptr, nullptr};
  return ref_gemm(a, xs, m, k, &d, 1, static_cast<const float*>(freqs), nullptr, nullptr, nullptr,
                  (cudaStream_t)stream);
}

// kernels/native_dispatch.cu:79-83 (dtype 2 = bf16; scale == null: plain RMSNorm)
K2B_EXPORT void k2_norm(const void* x, const void* w, const void* scale, const void* shift, void* y, int rows, int d,
                        int length, int cut, int batch, float eps, int dtype, void* stream) {
  shim_status(dtype != 2 ? (int)cudaErrorInvalidValue
                         : k2b_norm_mod(x, w, scale, shift, y, rows, d, length, cut, batch, eps, stream));
}

// kernels/native_dispatch.cu:84-89 (dtype 2)
K2B_EXPORT void k2_elementwise(const void* a, const void* b, const void* r, void* y, int64_t n, int mode, int width,
                               int dtype, void* stream) {
  shim_status(dtype != 2 ? (int)cudaErrorInvalidValue : k2b_elementwise(a, b, r, y, (long long)n, mode, width, stream));
}

// kernels/native_dispatch.cu:90-95 (dtype 2)
K2B_EXPORT void k2_rope(const void* q, const void* k, const void* f, void* qo, void* ko, int batch, int length, int qh,
                        int kh, int dim, int fb, int dtype, void* stream) {
  shim_status(dtype != 2 ? (int)cudaErrorInvalidValue
                         : k2b_rope(q, k, f, qo, ko, batch, length, qh, kh, dim, fb, stream));
}

// kernels/joint_projection.cu:212-214: output = gated residual projection,
// normalized = bf16 RMSNorm + modulation of it (batch 1, scale/shift [n]).
// The reference's counters scratch (its grid-wide row hand-off) is not
// touched: the two stages run as two launches.
K2B_EXPORT int k2_int4_residual_norm(void* a, void* w, void* xs, void* ws, void* gate, void* residual, void* norm,
                                     void* scale, void* shift, void* output, void* normalized, void* counters, int m,
                                     int n, int k, int dtype, float eps, void* stream) {
  (void)counters;
  if (dtype != 0) return (int)cudaErrorInvalidValue;
  const int rc = k2_int4_gated_residual(a, w, xs, ws, gate, residual, output, m, n, k, dtype, 0, stream);
  if (rc) return rc;
  return k2b_norm_mod(output, norm, scale, shift, normalized, m, n, m, -1, 1, eps, stream);
}
