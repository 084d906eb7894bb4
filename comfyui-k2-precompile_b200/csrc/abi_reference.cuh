// abi_reference.cuh -- exports under the reference's kernel-library names.
//
// native_runtime.cpp resolves these with dlopen(RTLD_NOW|RTLD_LOCAL) + dlsym
// (native_runtime.cpp:34-48, 514-527).  Argument order and meaning follow the
// reference exports; the data they point at follows the B200 contract:
//   * activations: packed INT4 [m, k/2] + fp16 group-128 scales [m, k/128]
//     (the reference passes one fp32 scale per row);
//   * weights: prepared s8 [n, k] + fp32 scales [k/128, n] produced by
//     k2b_prepare_weight (the reference passes packed INT4 + fp32 [n]);
//   * dtype: 0 = bf16 for the k2_int4_* family, 2 = bf16 for
//     k2_norm_mod_quant4 (the reference's two enums, native_runtime.cpp:83
//     and kernels/joint_projection.cu:208); fp16 activations are rejected.
// Return codes: 0, or cudaErrorInvalidValue for unsupported shapes/dtypes.
// The reference's void exports (k2_norm, k2_quant4, k2_elementwise, k2_rope)
// cannot return a status: they launch nothing on unsupported input and leave
// the status for k2b_shim_status() (the reference's callers check
// cudaGetLastError() after them, native_runtime.cpp:265,284).

namespace {
thread_local int g_shim_status = 0;
void shim_status(int rc) {
  if (rc) g_shim_status = rc;
}
}  // namespace

// Last non-zero status of a void shim on this host thread (0 if none).
K2B_EXPORT int k2b_shim_status(int reset) {
  const int rc = g_shim_status;
  if (reset) g_shim_status = 0;
  return rc;
}

// kernels/norm_quant.cu:89-91
K2B_EXPORT int k2_norm_mod_quant4(const void* x, const void* norm, const void* scale, const void* shift, void* q,
                                  void* scales, int rows, int K, int length, int cut, int batch, float eps, int group,
                                  int dtype, void* stream) {
  if (group != 128 || dtype != 2) return (int)cudaErrorInvalidValue;
  return k2b_norm_quant(x, norm, scale, shift, q, scales, rows, K, length, cut, batch, eps, stream);
}

// kernels/joint_projection.cu:222-225 (batch 1: freqs [m, 64, 2, 2])
K2B_EXPORT int k2_int4_qkv(const void* a, const void* wq, const void* wk, const void* wv, const void* wg,
                           const void* xs, const void* sq, const void* sk, const void* sv, const void* sg,
                           const void* nq, const void* nk, const void* freq, void* qo, void* ko, void* vo, void* go,
                           int m, int qwidth, int kvwidth, int k, int dtype, float eq, float ek, void* stream) {
  if (dtype != 0) return (int)cudaErrorInvalidValue;
  return k2b_qkv(a, xs, wq, sq, wk, sk, wv, sv, wg, sg, nq, nk, freq, qo, ko, vo, go, m, m, qwidth, kvwidth, k, eq, ek,
                 stream);
}

// kernels/joint_projection.cu:204-205 (bf16 h = bf16(bf16(silu(g)) * u))
K2B_EXPORT int k2_int4_swiglu(const void* a, const void* wg, const void* wu, const void* xs, const void* sg,
                              const void* su, void* out, int m, int n, int k, int dtype, void* stream) {
  if (dtype != 0) return (int)cudaErrorInvalidValue;
  return k2b_swiglu_bf16(a, xs, wg, sg, wu, su, out, m, n, k, stream);
}

// kernels/int4_epilogue.cu:77-78 (config selects a CUTLASS tile there; one tile here)
K2B_EXPORT int k2_int4_gated_residual(void* a, void* w, void* xs, void* ws, void* gate, void* residual, void* output,
                                      int m, int n, int k, int dtype, int config, void* stream) {
  if (dtype != 0 || (config != 0 && config != 1)) return (int)cudaErrorInvalidValue;
  return k2b_gated_residual(a, xs, w, ws, gate, residual, output, m, m, n, k, stream);
}

// kernels/qk_norm_rope.cu:135 (batch 1: freqs [m, 64, 2, 2])
K2B_EXPORT int k2_int4_qk_norm_rope(void* a, void* w, void* xs, void* ws, void* norm, void* freqs, void* output, int m,
                                    int n, int k, int dtype, float eps, void* stream) {
  if (dtype != 0 || n % 128) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_QKNORM, n, w, ws, output, n, static_cast<const float*>(norm), eps, nullptr, nullptr, nullptr};
  return gemm_launch(a, xs, m, k, &d, 1, m, static_cast<const float*>(freqs), nullptr, nullptr, (cudaStream_t)stream);
}

// kernels/native_dispatch.cu:79-83 (dtype 2 = bf16; scale == null: plain RMSNorm)
K2B_EXPORT void k2_norm(const void* x, const void* w, const void* scale, const void* shift, void* y, int rows, int d,
                        int length, int cut, int batch, float eps, int dtype, void* stream) {
  shim_status(dtype != 2 ? (int)cudaErrorInvalidValue
                         : k2b_norm_mod(x, w, scale, shift, y, rows, d, length, cut, batch, eps, stream));
}

// kernels/native_dispatch.cu:23-25 (group 128, dtype 2; scales fp16 [m, k/128])
K2B_EXPORT void k2_quant4(const void* x, void* q, void* s, int64_t m, int64_t k, int group, int dtype, void* stream) {
  shim_status(group != 128 || dtype != 2 || m > INT32_MAX || k > INT32_MAX
                  ? (int)cudaErrorInvalidValue
                  : k2b_rotate_quant(x, q, s, (int)m, (int)k, stream));
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
// The reference's counters scratch (grid-wide row-sum hand-off) is not used:
// the two stages run as two launches.
K2B_EXPORT int k2_int4_residual_norm(void* a, void* w, void* xs, void* ws, void* gate, void* residual, void* norm,
                                     void* scale, void* shift, void* output, void* normalized, void* counters, int m,
                                     int n, int k, int dtype, float eps, void* stream) {
  (void)counters;
  if (dtype != 0) return (int)cudaErrorInvalidValue;
  const int rc = k2b_gated_residual(a, xs, w, ws, gate, residual, output, m, m, n, k, stream);
  if (rc) return rc;
  return k2b_norm_mod(output, norm, scale, shift, normalized, m, n, m, -1, 1, eps, stream);
}
