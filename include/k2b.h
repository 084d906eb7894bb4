/*
 * k2b.h -- C ABI of libk2b, the B200 (sm_100a) kernel library for the Krea2
 * W4A4 DiT block hot path.
 *
 * Conventions (all entry points):
 *   - plain device pointers, sizes, and a cudaStream_t passed as void*; every
 *     launch goes on that stream (the reference launches on the caller's
 *     current stream, native_runtime.cpp:195);
 *   - nothing is allocated: the caller owns every output and workspace
 *     (native_runtime.cpp:373,413-414,441);
 *   - return 0 on success, otherwise a cudaError_t value; 1
 *     (cudaErrorInvalidValue) for unsupported shapes, dtypes or misaligned
 *     pointers, as kernels/norm_quant.cu:92 does;
 *   - kernels never trap; a device-side wait that runs out of time records a
 *     bit readable through k2b_device_error().
 *
 * Data contract (BASELINE contract; the reference's per-row fp32 scales are
 * replaced by group-128 fp16 scales):
 *   - activations: bf16 row-major [rows, K];
 *   - packed INT4: uint8 [rows, K/2], two codes per byte, low nibble = even
 *     column, plus fp16 scales [rows, K/128]; codes are clamp(rne(v/s),-8,7) of
 *     the Sylvester H128-rotated values, s = fp16(absmax/7);
 *   - prepared weights (k2b_prepare_weight): the codes as e4m3 bytes [n, K]
 *     and fp32 scales [K/128, n]; GEMM dequant: p = sum_g fmaf(fp32(acc_g *
 *     sA[r,g]), sW[c,g], .) in increasing g, acc_g the exact group sum;
 *   - RMSNorm weights are fp32 in the "w+1" form (native_schedule.py:252-253).
 */
#ifndef K2B_H
#define K2B_H

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Library identification string. */
const char* k2b_version(void);

/* Reads (and with reset != 0 clears) the device-side error word: bit 0..5 =
 * a bounded wait in the TMA / MMA / unpack / epilogue / softmax / load role
 * gave up; bit 6 = the self-test below.  Synchronises `stream`.  Returns the
 * word, or -cudaError. */
int k2b_device_error(int reset, void* stream);

/* Self-test of the bounded-wait failure path that every kernel's waits share
 * (no reference counterpart).  One CTA waits on an mbarrier that, with
 * mode = 1, nothing completes: the wait gives up after limit_ns (at most one
 * second) and sets bit 6 of the error word, and a second warp of the CTA
 * leaves its own endless wait through the CTA's abort flag.  mode = 0 is the
 * control (the barrier completes).  `result` is a device int[3]: warp 0's
 * wait succeeded, warp 1 left through the abort flag, warp 1's wait in us.
 * The context stays usable afterwards. */
int k2b_selftest_wait(int mode, long long limit_ns, void* result, void* stream);

/* ----------------------------------------------------------- norm_quant --
 * Fused RMSNorm -> adaLN modulation -> H128 rotation -> group-128 INT4.
 * Replaces k2_norm_mod_quant4 (kernels/norm_quant.cu:89-91) behind the op
 * k2_native::norm_quant (native_runtime.cpp:432-447).
 *   y = bf16((x*inv)*(w+1)), y = bf16(y*bf16(scale+1)), v = bf16(y+shift),
 *   inv = rsqrt_rn(sum(x^2)/K + eps) in the reference's reduction order;
 * the modulation row is b = row/length (+batch when cut >= 0 and
 * row%length >= cut), kernels/norm_quant.cu:32.
 * x bf16 [rows,K]; w fp32 [K]; scale/shift bf16 [nb,K]; q u8 [rows,K/2];
 * s fp16 [rows,K/128].  K a multiple of 512, at most 16384. */
int k2b_norm_quant(const void* x, const void* w, const void* scale, const void* shift, void* q, void* s,
                   int rows, int K, int length, int cut, int batch, float eps, void* stream);

/* k2b_norm_quant of rows [base_row, base_row+rows) of a latent stream (x, q,
 * s point at the first of them): the modulation row follows the row's index
 * in the whole stream, so a row shard of a tensor-parallel group quantises
 * exactly as the unsharded call. */
int k2b_norm_quant_rows(const void* x, const void* w, const void* scale, const void* shift, void* q, void* s,
                        int base_row, int rows, int K, int length, int cut, int batch, float eps, void* stream);

/* H128 rotation + group-128 INT4 of a bf16 activation: the input quantisation
 * `quantize()` performs before an INT4 projection (native_runtime.cpp:268-271;
 * comfy-kitchen quantize_int4_rowwise_convrot64 via k2_quant4,
 * kernels/native_dispatch.cu:23-25).  Same K constraint as k2b_norm_quant. */
int k2b_rotate_quant(const void* x, void* q, void* s, int rows, int K, void* stream);

/* bf16 RMSNorm (+ adaLN modulation when scale/shift are given) with the
 * rounding points and reduction order of k2b_norm_quant, output bf16
 * [rows,K].  Replaces k2_norm / norm_mod (kernels/native_dispatch.cu:44-62,
 * 79-83) behind k2_native::norm_mod and residual_norm (native_runtime.cpp:
 * 262-266, 513).  scale and shift are both given or both null. */
int k2b_norm_mod(const void* x, const void* w, const void* scale, const void* shift, void* y, int rows, int K,
                 int length, int cut, int batch, float eps, void* stream);

/* bf16 elementwise of kernels/native_dispatch.cu:63-70 / k2_elementwise:
 * mode 0 y = bf16(silu(a)) [* b], mode 1 y = bf16(sigmoid(a)) [* b]
 * (b may be null), mode 2 y = bf16(r + bf16(b * a[i % width])). */
int k2b_elementwise(const void* a, const void* b, const void* r, void* y, long long n, int mode, int width,
                    void* stream);

/* Adjacent-pair RoPE of kernels/native_dispatch.cu:71-77 / k2_rope on bf16
 * [batch, heads, length, dim] q and k; f fp32 [fb, length, dim/2, 2, 2],
 * fb = 1 or batch. */
int k2b_rope(const void* q, const void* k, const void* f, void* qo, void* ko, int batch, int length, int qh, int kh,
             int dim, int fb, void* stream);

/* ---------------------------------------------------- weight preparation --
 * Registration-time conversion of a packed INT4 weight [n, k/2] + fp16 group
 * scales [n, k/128] into the resident layout the GEMM streams with TMA:
 * e4m3 bytes [.., k] (each code exactly, column order) at row
 * dst(r) = (r/block_rows)*dst_block_stride + dst_offset + r%block_rows, and
 * fp32 scales [k/128, scale_ld] at column dst(r).  Replaces the per-call
 * weight leases of native_runtime.cpp:84-260 (weights stay resident). */
int k2b_prepare_weight(const void* w_packed, const void* w_scale, void* w_prepared, void* scale_t, int n, int k,
                       int block_rows, int dst_block_stride, int dst_offset, int scale_ld, void* stream);

/* -------------------------------------------------------------- W4A4 GEMM --
 * a u8 [m,k/2] + sa fp16 [m,k/128]; w/wscale prepared; n % 128 == 0. */
/* fp32 result p (exact group accumulation; k2b's test hook for the int32
 * accumulators). */
int k2b_gemm_f32(const void* a, const void* sa, const void* w, const void* wscale, void* out, int m, int n, int k,
                 void* stream);
/* bf16(p): the plain projection of k2_gemm4 (kernels/native_dispatch.cu:26-29). */
int k2b_gemm_bf16(const void* a, const void* sa, const void* w, const void* wscale, void* out, int m, int n, int k,
                  void* stream);

/* Fused Q/K/V(/gate) projection: replaces k2_int4_qkv
 * (kernels/joint_projection.cu:222-231) and the split QKGemm + k2_gemm4 group
 * (native_runtime.cpp:333-358, kernels/qk_norm_rope.cu:135).
 * Q, K: per-head RMSNorm (nq/nk fp32 [128], eq/ek) + adjacent-pair RoPE with
 * freqs fp32 [length,64,2,2] (token = row % length); V: bf16(p);
 * gate (optional, wg/go non-null): bf16(sigmoid(bf16(p))).
 * Outputs token-major bf16: qo [m,qwidth], ko/vo [m,kvwidth], go [m,qwidth].
 * qwidth, kvwidth multiples of 128. */
int k2b_qkv(const void* a, const void* sa, const void* wq, const void* swq, const void* wk, const void* swk,
            const void* wv, const void* swv, const void* wg, const void* swg, const void* nq, const void* nk,
            const void* freqs, void* qo, void* ko, void* vo, void* go, int m, int length, int qwidth, int kvwidth,
            int k, float eq, float ek, void* stream);

/* Projection with gated residual: out = bf16(resid + bf16(bf16(p)*gate[b,c])),
 * b = row/length; gate bf16 [batch, n], resid/out bf16 [m, n].  Replaces
 * k2_int4_gated_residual (kernels/int4_epilogue.cu:77-85) and the
 * output half of k2_int4_residual_norm (kernels/joint_projection.cu:178-179). */
int k2b_gated_residual(const void* a, const void* sa, const void* w, const void* wscale, const void* gate,
                       const void* residual, void* out, int m, int length, int n, int k, void* stream);

/* The gated residual applied to an already reduced fp32 projection p
 * [rows, n] (the tail of a tensor-parallel out/down projection after its
 * reduce-scatter): out = bf16(resid + bf16(bf16(p)*gate[(base_row+row)/length])),
 * the rounding of k2b_gated_residual.  n % 8 == 0. */
int k2b_gated_add(const void* p, const void* gate, const void* resid, void* out, int base_row, int rows, int n,
                  int length, void* stream);

/* fp32 a@W of one tensor-parallel rank written straight into the owners'
 * receive buffers over NVLink peer memory (the GEMM half of a fused
 * reduce-scatter): row r goes to peers[r/chunk] (fp32 [tp, chunk, n], this
 * GPU's buffer or a peer's CUDA-IPC mapping, tp <= 4) in slot `rank` at row
 * r%chunk, so the transfer overlaps the math tile by tile.  The owner sums
 * its slots with k2b_reduce_gated_add after a barrier that follows this
 * launch on every rank.  Replaces the NCCL reduce-scatter of the fp32
 * partials after the out- and down-projections. */
int k2b_gemm_f32_scatter(const void* a, const void* sa, const void* w, const void* wscale, void* const* peers, int tp,
                         int rank, int chunk, int m, int n, int k, void* stream);

/* k2b_gated_add of p = ((s_0 + s_1) + ...) + s_{nslots-1}, the fp32 sum of
 * nslots partial slots slot_stride floats apart (the receive buffer of
 * k2b_gemm_f32_scatter, base at this rank's first row). */
int k2b_reduce_gated_add(const void* slots, int nslots, long long slot_stride, const void* gate, const void* resid,
                         void* out, int base_row, int rows, int n, int length, void* stream);

/* Peer buffers for the scatter: cudaMalloc + IPC handle (64 bytes), open /
 * close a peer's handle in another process, free. */
int k2b_ipc_alloc(long long bytes, void** ptr, void* handle);
int k2b_ipc_open(const void* handle, void** ptr);
int k2b_ipc_close(void* ptr);
int k2b_ipc_free(void* ptr);

/* Gate/up projection + SwiGLU + INT4 requant of the down-projection input:
 * h = bf16(bf16(silu(bf16(pg)))*bf16(pu)), then H128 rotation + group-128
 * INT4 -> hq u8 [m, width/2], hs fp16 [m, width/128].  Replaces
 * k2_int4_swiglu (kernels/joint_projection.cu:204-211) plus the separate
 * quantize() before the down projection (native_runtime.cpp:327).
 * width % 128 == 0. */
int k2b_swiglu_quant(const void* a, const void* sa, const void* wg, const void* sg, const void* wu, const void* su,
                     void* hq, void* hs, int m, int width, int k, void* stream);
/* As above with bf16 h [m, width] out (k2_int4_swiglu's output). */
int k2b_swiglu_bf16(const void* a, const void* sa, const void* wg, const void* sg, const void* wu, const void* su,
                    void* h, int m, int width, int k, void* stream);

/* ------------------------------------------------------------- attention --
 * GQA flash attention, non-causal, head_dim 128, (heads/kvheads) even.
 * Replaces k2_fullgraph::kohaku_fa (KohakuKernelRouter/attention.py:189-193,
 * fwd_kernel :63-110).  q [B,heads,lq,128], k/v [B,kvheads,lk,128] given by
 * element strides (batch, head, token; last dim contiguous; all multiples of
 * 8); out bf16 [B, lq, heads*128]; gate (optional) bf16 with out's layout,
 * gate_kind 1 = sigmoid applied here, 2 = already sigmoided. */
int k2b_attention(const void* q, const void* k, const void* v, const void* gate, void* out, int batch, int heads,
                  int kvheads, int lq, int lk, int dim, long long q_sb, long long q_sh, long long q_st,
                  long long k_sb, long long k_sh, long long k_st, long long v_sb, long long v_sh, long long v_st,
                  int gate_kind, void* stream);
/* Attention with the out-projection's input quantisation fused into the
 * store: oq u8 [B*lq, heads*64], os fp16 [B*lq, heads] (one group per head). */
int k2b_attention_quant(const void* q, const void* k, const void* v, void* oq, void* os, int batch, int heads,
                        int kvheads, int lq, int lk, int dim, long long q_sb, long long q_sh, long long q_st,
                        long long k_sb, long long k_sh, long long k_st, long long v_sb, long long v_sh,
                        long long v_st, void* stream);

/* ------------------------------------------------ e4m3 byte containers --
 * Forms of the ops above whose INT4 codes travel as e4m3 bytes [rows, K], one
 * byte per code in column order (e4m3 represents -8..7 exactly), instead of
 * packed nibbles [rows, K/2]; scales are unchanged.  The native block loop
 * keeps its intermediate activations in this container so that every GEMM
 * loads A with TMA straight into the tensor-core layout.  No reference
 * counterpart (the reference's kernels take packed INT4 only).
 * k2b_norm_quant_e4m3: k2b_norm_quant with q8 u8 [rows, K];
 * k2b_attention_quant_e4m3: k2b_attention_quant with oq8 u8 [B*lq, heads*128];
 * k2b_gemm_f32_e4m3 / k2b_qkv_e4m3 / k2b_gated_residual_e4m3: their packed
 *   twins with a8 u8 [m, k];
 * k2b_swiglu_quant_e4m3: a8 u8 [m, k] in, h8 u8 [m, width] + hs out;
 * k2b_gemm_bf16_e4m3 / k2b_swiglu_bf16_e4m3 / k2b_gemm_f32_scatter_e4m3:
 *   likewise; k2b_swiglu_quant_a8: a8 u8 [m, k] in, packed hq [m, width/2]
 *   + hs out (k2b_swiglu_quant's output).
 * k2b_expand_e4m3: packed codes [rows, K/2] -> e4m3 bytes [rows, K]
 *   (nbytes = rows*K/2, a multiple of 16).  The byte-A GEMM takes about 40%
 *   less time than the packed-A form, which unpacks A inside the CTA (gate/up
 *   at 33792 x 16384 x 6144: 12.0 against 19.8 ms), so a caller holding
 *   packed codes expands them first (a pass over 1.5 bytes per code). */
int k2b_norm_quant_e4m3(const void* x, const void* w, const void* scale, const void* shift, void* q8, void* s,
                        int rows, int K, int length, int cut, int batch, float eps, void* stream);
int k2b_attention_quant_e4m3(const void* q, const void* k, const void* v, void* oq8, void* os, int batch, int heads,
                             int kvheads, int lq, int lk, int dim, long long q_sb, long long q_sh, long long q_st,
                             long long k_sb, long long k_sh, long long k_st, long long v_sb, long long v_sh,
                             long long v_st, void* stream);
int k2b_gemm_f32_e4m3(const void* a8, const void* sa, const void* w, const void* wscale, void* out, int m, int n,
                      int k, void* stream);
int k2b_qkv_e4m3(const void* a8, const void* sa, const void* wq, const void* swq, const void* wk, const void* swk,
                 const void* wv, const void* swv, const void* wg, const void* swg, const void* nq, const void* nk,
                 const void* freqs, void* qo, void* ko, void* vo, void* go, int m, int length, int qwidth,
                 int kvwidth, int k, float eq, float ek, void* stream);
int k2b_gated_residual_e4m3(const void* a8, const void* sa, const void* w, const void* wscale, const void* gate,
                            const void* residual, void* out, int m, int length, int n, int k, void* stream);
int k2b_swiglu_quant_e4m3(const void* a8, const void* sa, const void* wg, const void* sg, const void* wu,
                          const void* su, void* h8, void* hs, int m, int width, int k, void* stream);
int k2b_gemm_bf16_e4m3(const void* a8, const void* sa, const void* w, const void* wscale, void* out, int m, int n,
                       int k, void* stream);
int k2b_swiglu_bf16_e4m3(const void* a8, const void* sa, const void* wg, const void* sg, const void* wu,
                         const void* su, void* h, int m, int width, int k, void* stream);
int k2b_gemm_f32_scatter_e4m3(const void* a8, const void* sa, const void* w, const void* wscale, void* const* peers,
                              int tp, int rank, int chunk, int m, int n, int k, void* stream);
int k2b_swiglu_quant_a8(const void* a8, const void* sa, const void* wg, const void* sg, const void* wu,
                        const void* su, void* hq, void* hs, int m, int width, int k, void* stream);
int k2b_expand_e4m3(const void* a, void* a8, long long nbytes, void* stream);

/* ------------------------------------ INT8 / FP8 weights, reference contract --
 * Projections of INT8 / FP8 checkpoint weights (the reference's formats 2 and
 * 3/4: at::_int_mm + k2_dequant8, at::_scaled_mm; native_runtime.cpp:271-283,
 * 298-311) on the tcgen05 pair GEMM, the whole of k in one accumulator and the
 * dequant fused: out bf16 = bf16(fp32(fp32(acc*xs[r*xs_stride])*ws[c*ws_stride])
 * + bias[c]); strides 0 = one scale; bias fp32 [n] or null; k, n % 128 == 0.
 * k2b_gemm8: int8 a8 [m,k] / w8 [n,k].  k2b_gemm_f8: fp8 with afmt / bfmt
 * 0 = e4m3, 1 = e5m2.
 * k2b_ref_qkv / k2b_ref_gated_residual: k2_int4_qkv / k2_int4_gated_residual
 * (reference contract) over `batch` latents of `length` tokens (RoPE token =
 * row % length, gate row = row / length, gate bf16 [batch, n]). */
int k2b_gemm8(const void* a8, const void* xs, int xs_stride, const void* w8, const void* ws, int ws_stride,
              const void* bias, void* out, int m, int n, int k, void* stream);
int k2b_gemm_f8(const void* a8, const void* xs, int xs_stride, const void* w8, const void* ws, int ws_stride,
                const void* bias, void* out, int m, int n, int k, int afmt, int bfmt, void* stream);
int k2b_ref_qkv(const void* a, const void* xs, const void* wq, const void* sq, const void* wk, const void* sk,
                const void* wv, const void* sv, const void* wg, const void* sg, const void* nq, const void* nk,
                const void* freq, void* qo, void* ko, void* vo, void* go, int m, int length, int qwidth, int kvwidth,
                int k, float eq, float ek, void* stream);
int k2b_ref_gated_residual(const void* a, const void* xs, const void* w, const void* ws, const void* gate,
                           const void* residual, void* out, int m, int length, int n, int k, void* stream);
/* The same with A and W as e4m3 code bytes (A [m, k] from k2b_expand_e4m3,
 * W [n, k] expanded once from the packed checkpoint rows): identical results
 * (exact integer sums in the fp32 accumulator) without the in-CTA unpacking
 * of the packed forms.  k2b_ref_swiglu8: k2_int4_swiglu's arguments with a8,
 * wg8, wu8.  The plain projection of this form is k2b_gemm_f8 with e4m3
 * operands and per-row / per-channel scales. */
/* k2_quant4 / k2_norm_mod_quant4 (reference contract, ConvRot group 16, 64 or
 * 256) with the codes written as e4m3 bytes q8 [rows, K] for the forms below;
 * K % 512 == 0. */
int k2b_ref_quant4_e4m3(const void* x, void* q8, void* s, long long m, long long k, int group, void* stream);
int k2b_ref_norm_quant4_e4m3(const void* x, const void* norm, const void* scale, const void* shift, void* q8,
                             void* scales, int rows, int K, int length, int cut, int batch, float eps, int group,
                             void* stream);
int k2b_ref_qkv8(const void* a8, const void* xs, const void* wq, const void* sq, const void* wk, const void* sk,
                 const void* wv, const void* sv, const void* wg, const void* sg, const void* nq, const void* nk,
                 const void* freq, void* qo, void* ko, void* vo, void* go, int m, int length, int qwidth,
                 int kvwidth, int k, float eq, float ek, void* stream);
int k2b_ref_swiglu8(const void* a8, const void* wg, const void* wu, const void* xs, const void* sg, const void* su,
                    void* out, int m, int n, int k, void* stream);
int k2b_ref_gated_residual8(const void* a8, const void* xs, const void* w, const void* ws, const void* gate,
                            const void* residual, void* out, int m, int length, int n, int k, void* stream);

/* ------------------------------------------------------ LoRA bypass deltas --
 * One LoRA bypass factor pair fused into a projection's epilogue (the
 * reference composes value + T(T(x down^T) up^T) * s after the projection,
 * graph_ops.py:246-249; native_schedule.py:169-182 collects the factors):
 * out = E(T(T(p) + T(T(t up^T) * s))), t bf16 [m, lr] = T(x down^T), up bf16
 * [n, lr], lr % 8 == 0 and <= 1024; E = T, or the gated residual
 * T(residual + T(p' * gate[row / length])) when gate and residual are given.
 * contract 0: group-128 W4A4 (a packed, s fp16 [m, k/128], prepared w / ws);
 * contract 2: the same with a as e4m3 bytes [m, k];
 * contract 1: the reference's INT4 (a packed, s fp32 [m], w packed [n, k/2],
 * ws fp32 [n], bias fp32 [n] or null).  k2b_lora_swiglu: SwiGLU with a pair
 * per half (either may be null), bf16 h [m, width]. */
int k2b_lora_gemm(int contract, const void* a, const void* s, const void* w, const void* ws, const void* bias,
                  const void* gate, const void* residual, int length, const void* lt, const void* lup, int lr,
                  float ls, void* out, int m, int n, int k, void* stream);
int k2b_lora_swiglu(int contract, const void* a, const void* s, const void* wg, const void* sg, const void* wu,
                    const void* su, const void* lt_g, const void* lup_g, int lr_g, float ls_g, const void* lt_u,
                    const void* lup_u, int lr_u, float ls_u, void* h, int m, int width, int k, void* stream);

/* ------------------------------------------------------------ block loop --
 * Native loop over transformer blocks (replaces the compiled entry that
 * NativeGraph::run drives, native_runtime.cpp:543-571, over graph_model.py's
 * quant chain :108-114, :266-295).  block_ptrs holds k2b_block_slots()
 * pointers per block in this order:
 *   0 prenorm w (fp32 [hidden])   1 postnorm w   2 q-norm w (fp32 [128])
 *   3 k-norm w   4/5 Wq, Sq   6/7 Wk, Sk   8/9 Wv, Sv   10/11 Wo, So
 *   12/13 Wgate, Sgate   14/15 Wup, Sup   16/17 Wdown, Sdown
 *   18 modulation bf16 [6, batch, hidden] = (ps, ph, pg, ss, sh, sg)
 * (W = prepared int8, S = prepared fp32 scales).  x bf16 [batch*length,
 * hidden] is updated in place; freqs fp32 [length,64,2,2];
 * workspace >= k2b_block_workspace_bytes(). hidden == heads*128.
 * events (nullable): nblocks*8 cudaEvent_t; events[8b+i] is recorded on the
 * stream before launch i of block b (0 norm_quant, 1 qkv, 2 attention,
 * 3 out-proj, 4 norm_quant, 5 gate/up, 6 down) and events[8b+7] after it. */
int k2b_block_slots(void);
long long k2b_block_workspace_bytes(int rows, int hidden, int heads, int kvheads, int mlp);
int k2b_forward_blocks(const void* const* block_ptrs, int nblocks, void* x, const void* freqs, void* workspace,
                       long long workspace_bytes, int batch, int length, int hidden, int heads, int kvheads, int mlp,
                       float eps, float qk_eps, void* const* events, void* stream);

/* Block loop that allocates nothing, for callers that cannot call cudaMalloc
 * (an embedding host that owns the device allocator, a plugin handed only its
 * input/output buffers).  No counterpart in the reference: it is
 * k2b_forward_blocks with the workspace taken from a file-scope device array
 * of k2b_static_workspace_bytes() (64 MiB; ~1120 token rows at the Krea2
 * widths); larger batch*length is rejected with cudaErrorInvalidValue.  The
 * array's device address is looked up (cudaGetSymbolAddress) in the calling
 * thread's current CUDA context on every call made outside stream capture, so
 * it follows a cudaDeviceReset or a caller-owned context; during capture the
 * address cached for that context is used, so the first call in each context
 * must come before any stream capture.  Calls that overlap on the GPU race on
 * the shared array.  Nothing in it needs to start at zero. */
long long k2b_static_workspace_bytes(void);
int k2b_forward_blocks_static(const void* const* block_ptrs, int nblocks, void* x, const void* freqs, int batch,
                              int length, int hidden, int heads, int kvheads, int mlp, float eps, float qk_eps,
                              void* stream);

/* ------------------------------- reference-named exports (reference contract) --
 * The symbols the reference's runtime dlsym's (configure(): k2_quant4,
 * k2_quant8, k2_gemm4, k2_dequant8, k2_fp8, k2_norm, k2_elementwise, k2_rope;
 * the epilogue/QK libraries: k2_int4_gated_residual, k2_int4_qk_norm_rope;
 * configure_joint(): k2_int4_swiglu, k2_int4_qkv, k2_int4_residual_norm;
 * configure_norm_quant(): k2_norm_mod_quant4; native_runtime.cpp:514-529),
 * with the reference's argument order AND its data contract, i.e. the
 * buffers native_runtime.cpp allocates for them (:262-311, 399-447):
 *   - INT4 activations packed [m, k/2] + ONE fp32 scale per row [m, 1],
 *     ConvRot-rotated in groups of 16, 64 or 256;
 *   - INT4 weights packed [n, k/2] as stored by a ConvRot W4A4 checkpoint,
 *     one fp32 scale per channel [n] (nothing prepared ahead);
 *   - projections T(fp32(fp32(acc*xs[r])*ws[c])), acc over all of k;
 *   - dtype 0 = bf16 for k2_int4_*, 2 = bf16 for the others; fp16 rejected.
 * The group-128 BASELINE contract is served by the k2b_* entry points only. */
int k2_norm_mod_quant4(const void* x, const void* norm, const void* scale, const void* shift, void* q, void* scales,
                       int rows, int K, int length, int cut, int batch, float eps, int group, int dtype,
                       void* stream); /* kernels/norm_quant.cu:89-91 */
int k2_int4_qkv(const void* a, const void* wq, const void* wk, const void* wv, const void* wg, const void* xs,
                const void* sq, const void* sk, const void* sv, const void* sg, const void* nq, const void* nk,
                const void* freq, void* qo, void* ko, void* vo, void* go, int m, int qwidth, int kvwidth, int k,
                int dtype, float eq, float ek, void* stream); /* kernels/joint_projection.cu:222-225 */
int k2_int4_swiglu(const void* a, const void* wg, const void* wu, const void* xs, const void* sg, const void* su,
                   void* out, int m, int n, int k, int dtype, void* stream); /* kernels/joint_projection.cu:204-205 */
int k2_int4_gated_residual(void* a, void* w, void* xs, void* ws, void* gate, void* residual, void* output, int m,
                           int n, int k, int dtype, int config, void* stream); /* kernels/int4_epilogue.cu:77-78 */
int k2_int4_qk_norm_rope(void* a, void* w, void* xs, void* ws, void* norm, void* freqs, void* output, int m, int n,
                         int k, int dtype, float eps, void* stream); /* kernels/qk_norm_rope.cu:135 */
int k2_int4_residual_norm(void* a, void* w, void* xs, void* ws, void* gate, void* residual, void* norm, void* scale,
                          void* shift, void* output, void* normalized, void* counters, int m, int n, int k, int dtype,
                          float eps, void* stream); /* kernels/joint_projection.cu:212-214 */
/* The reference's void exports (kernels/native_dispatch.cu:23-40, 79-95):
 * unsupported input launches nothing and sets the status k2b_shim_status()
 * returns.  k2_quant4 / k2_quant8: q [m, k/2] INT4 / [m, k] int8, s fp32
 * [m, 1] (group 16/64/256, k2_quant8 also 0 = no rotation); k2_gemm4: bias
 * fp32 [n] or null, out bf16 [m, n]; k2_dequant8: int32 a [m, n] -> bf16,
 * ws [ns] with ns = n or 1, bias bf16 [n] or null; k2_fp8: y = fp8(x / s[0])
 * (quant) or T(x * s[0]), codes 0 fp32 / 1 fp16 / 2 bf16 / 5 e4m3 / 6 e5m2. */
void k2_norm(const void* x, const void* w, const void* scale, const void* shift, void* y, int rows, int d, int length,
             int cut, int batch, float eps, int dtype, void* stream); /* kernels/native_dispatch.cu:79-83 */
void k2_quant4(const void* x, void* q, void* s, int64_t m, int64_t k, int group, int dtype,
               void* stream); /* kernels/native_dispatch.cu:23-25 */
void k2_quant8(const void* x, void* q, void* s, int64_t m, int64_t k, int group, int dtype,
               void* stream); /* kernels/native_dispatch.cu:30-33 */
void k2_gemm4(const void* a, const void* w, const void* xs, const void* ws, const void* bias, void* out, int64_t m,
              int64_t n, int64_t k, int dtype, void* stream); /* kernels/native_dispatch.cu:26-29 */
void k2_dequant8(const void* a, const void* xs, const void* ws, const void* bias, void* out, int64_t m, int64_t n,
                 int64_t ns, int dtype, void* stream); /* kernels/native_dispatch.cu:34-36 */
void k2_fp8(const void* x, void* y, const void* s, int64_t n, int src, int dst, bool quant,
            void* stream); /* kernels/native_dispatch.cu:37-40 */
void k2_elementwise(const void* a, const void* b, const void* r, void* y, int64_t n, int mode, int width, int dtype,
                    void* stream); /* kernels/native_dispatch.cu:84-89 */
void k2_rope(const void* q, const void* k, const void* f, void* qo, void* ko, int batch, int length, int qh, int kh,
             int dim, int fb, int dtype, void* stream); /* kernels/native_dispatch.cu:90-95 */
/* Last non-zero status of a void shim on this host thread; reset clears it.
 * No counterpart in the reference (its void exports rely on
 * cudaGetLastError()). */
int k2b_shim_status(int reset);

#ifdef __cplusplus
}
#endif
#endif /* K2B_H */
