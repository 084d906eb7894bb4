// k2b_lib.cu -- the single translation unit of libk2b: kernels + C-ABI.
//
// Every exported entry point takes plain device pointers, sizes and a
// cudaStream_t (as void*), launches on that stream, allocates nothing, and
// returns 0 or a cudaError_t code (cudaErrorInvalidValue for shapes/pointers
// the kernels do not support).  Declarations: include/k2b.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/k2b.h"
#include "attention.cuh"
#include "gemm_w4a4.cuh"
#include "k2b_common.cuh"
#include "elementwise.cuh"
#include "norm_quant.cuh"
#include "ref_contract.cuh"

#define K2B_EXPORT extern "C" __attribute__((visibility("default")))

namespace k2b {

// ------------------------------------------------------------- utilities
static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D row-major tensor map: `cols` elements per row (innermost), `rows` rows.
static int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, size_t esize, const void* base, uint64_t cols,
                       uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows,
                       CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return (int)cudaErrorInitializationError;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  (void)esize;
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

// 4-D map (d, token, head, batch) over a strided bf16 [B, H, L, D] view.
static int make_map_4d_bf16(CUtensorMap* map, const void* base, uint64_t D, uint64_t L, uint64_t H, uint64_t B,
                            uint64_t s_tok, uint64_t s_head, uint64_t s_batch, uint32_t box_d, uint32_t box_tok) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return (int)cudaErrorInitializationError;
  cuuint64_t dims[4] = {D, L, H, B};
  cuuint64_t strides[3] = {s_tok * 2, s_head * 2, s_batch * 2};
  cuuint32_t box[4] = {box_d, box_tok, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

static int launch_status() { return (int)cudaGetLastError(); }

// ----------------------------------------------------------- norm_quant
template <bool NORM, bool MOD, bool QUANT, bool BYTES = false>
static int norm_quant_launch(const void* x, const void* w, const void* scale, const void* shift, void* q, void* s,
                             int rows, int K, int length, int cut, int batch, float eps, cudaStream_t st,
                             int base_row = 0) {
  if (rows <= 0 || K <= 0 || K % 512 || K > 16384 || (MOD && (length <= 0 || batch <= 0)) || base_row < 0)
    return (int)cudaErrorInvalidValue;
  if (!aligned16(x) || !aligned16(q) || (QUANT && !s) || (NORM && !aligned16(w)) ||
      (MOD && (!aligned16(scale) || !aligned16(shift))))
    return (int)cudaErrorInvalidValue;
  // One wave of resident CTAs looping over row tiles; the residency is
  // queried once per device (the same value may be stored twice by racing
  // first calls, which is harmless).
  static int resident[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
  int& per_sm = resident[dev];
  if (per_sm == 0) {
    int n = 0, sms = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, norm_quant_kernel<NORM, MOD, QUANT, BYTES>, kNqThreads, 0);
    if (e != cudaSuccess) return (int)e;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return (int)e;
    per_sm = (n > 0 ? n : 1) * sms;
  }
  const int tiles = (rows + kNqRows - 1) / kNqRows;
  const int grid = tiles < per_sm ? tiles : per_sm;
  norm_quant_kernel<NORM, MOD, QUANT, BYTES><<<grid, kNqThreads, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const float*>(w), static_cast<const __nv_bfloat16*>(scale),
      static_cast<const __nv_bfloat16*>(shift), static_cast<uint8_t*>(q), static_cast<__half*>(s), rows, K, length,
      cut, batch, eps, base_row);
  return launch_status();
}

// --------------------------------------------------- weight preparation
// Packed INT4 [n, k/2] + fp16 group scales [n, k/128] -> e4m3 bytes [.., k]
// (the codes in column order, the encoding the in-kernel A unpacker uses) at
// row dst(r) = (r / block_rows) * dst_block_stride + dst_offset + r % block_rows,
// and fp32 scales transposed to [k/128, scale_ld] at column dst(r).
__global__ void prepare_weight_kernel(const uint8_t* __restrict__ wp, const __half* __restrict__ ws,
                                      uint8_t* __restrict__ out, float* __restrict__ st, int n, int k, int block_rows,
                                      int dst_block_stride, int dst_offset, int scale_ld) {
  const int chunks = k / 32;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)n * chunks) return;
  const int r = (int)(idx / chunks), c = (int)(idx % chunks);
  const int64_t dr = (int64_t)(r / block_rows) * dst_block_stride + dst_offset + (r % block_rows);
  const uint4 v = *reinterpret_cast<const uint4*>(wp + (int64_t)r * (k / 2) + 16 * c);
  uint4 lo, hi;
  unpack_chunk(v, lo, hi);
  *reinterpret_cast<uint4*>(out + dr * k + 32 * c) = lo;
  *reinterpret_cast<uint4*>(out + dr * k + 32 * c + 16) = hi;
  if ((c & 3) == 0) st[(int64_t)(c >> 2) * scale_ld + dr] = __half2float(ws[(int64_t)r * (k / 128) + (c >> 2)]);
}

// ---------------------------------------------------------------- GEMM
struct SegDesc {
  int kind;
  int n;                  // columns (= weight rows) of this segment
  const void* w;          // prepared s8 [n, K]
  const void* wscale;     // fp32 [K/128, n]
  void* out;
  int ld;
  const float* normw;
  float eps;
  void* out_scale;
  const void* w2;         // SwiGLU: up projection, prepared s8 [n, K]
  const void* wscale2;    // SwiGLU: fp32 [K/128, n]
  // optional LoRA bypass factors (GemmSegment::lt ...): lt bf16 [M, lr],
  // lup bf16 [n, lr], strength ls; lt2 / lup2 / lr2 / ls2 for SwiGLU's up half
  const void* lt = nullptr;
  const void* lup = nullptr;
  int lr = 0;
  float ls = 0.0f;
  const void* lt2 = nullptr;
  const void* lup2 = nullptr;
  int lr2 = 0;
  float ls2 = 0.0f;
};

// Reference-contract arguments of gemm_launch (GM_REF* modes): activation
// scales xs[r * xs_stride] and weight scales wscale[c * ws_stride] (fp32),
// optional fp32 bias [n] (SEG_BF16), fp8 formats a | b << 3.
struct RefScales {
  const float* xs = nullptr;
  int xs_stride = 1, ws_stride = 1;
  const float* bias = nullptr;
  uint32_t f8fmt = 0;
};

// mode (GemmMode): GM_PACKED `a` packed INT4 [M, K/2]; GM_BYTES e4m3 bytes
// [M, K] (the block loop's activation containers); GM_REF4 packed INT4 A and
// W with per-row / per-channel fp32 scales; GM_REF8 int8 A and W bytes;
// GM_REFF8 fp8 A and W bytes.
static int gemm_launch(const void* a, const void* sa, int M, int K, const SegDesc* segs, int nseg, int length,
                       const float* freqs, const void* gate, const void* resid, cudaStream_t st,
                       void* const* peers = nullptr, int tp = 0, int rank = 0, int chunk = 0, int mode = GM_PACKED,
                       const RefScales* ref = nullptr) {
  const bool refm = mode >= GM_REF4;
  const bool bytea = mode == GM_BYTES || mode == GM_REF8 || mode == GM_REFF8;
  if (M <= 0 || K <= 0 || K % 128 || nseg < 1 || nseg > 4 || length <= 0) return (int)cudaErrorInvalidValue;
  if (!aligned16(a) || (refm ? (!ref || !ref->xs) : !sa)) return (int)cudaErrorInvalidValue;
  CUtensorMap amap;
  WeightMaps wm;
  memset(&wm, 0, sizeof(wm));
  GemmParams p;
  memset(&p, 0, sizeof(p));
  int tiles = 0;
  for (int i = 0; i < nseg; ++i) {
    const SegDesc& d = segs[i];
    const bool pairw = d.kind == SEG_SWIGLU || d.kind == SEG_SWIGLU_BF16 || d.kind == SEG_SWIGLU_E4M3;
    if (pairw && nseg != 1) return (int)cudaErrorInvalidValue;
    // SwiGLU pairs 128 gate + 128 up columns per tile; other segments take
    // any multiple of 128 columns (a last tile may be half used)
    const int tile_n = pairw ? GEMM_BN / 2 : GEMM_BN;
    if (d.n <= 0 || d.n % 128 || !aligned16(d.w) || (refm ? !d.wscale : !aligned16(d.wscale)) || !d.out)
      return (int)cudaErrorInvalidValue;
    // each CTA of a pair loads 128 weight rows per K group: prepared / byte
    // weights in the UMMA layout, or (GM_REF4) the packed rows as stored
    auto wmap = [&](CUtensorMap* m, const void* w) {
      return mode == GM_REF4 ? make_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, (uint64_t)K / 2, (uint64_t)d.n,
                                           (uint64_t)K / 2, 64, GEMM_BN / 2, CU_TENSOR_MAP_SWIZZLE_NONE)
                             : make_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, (uint64_t)K, (uint64_t)d.n,
                                           (uint64_t)K, 128, GEMM_BN / 2, CU_TENSOR_MAP_SWIZZLE_128B);
    };
    int rc = wmap(&wm.m[i], d.w);
    if (rc) return rc;
    if (pairw) {
      if (!aligned16(d.w2) || (refm ? !d.wscale2 : !aligned16(d.wscale2))) return (int)cudaErrorInvalidValue;
      rc = wmap(&wm.m[1], d.w2);
      if (rc) return rc;
    }
    GemmSegment& g = p.seg[i];
    g.tiles = (d.n + tile_n - 1) / tile_n;
    g.kind = d.kind;
    g.n = d.n;
    g.ld = d.ld;
    g.out = d.out;
    g.wscale = static_cast<const float*>(d.wscale);
    g.wscale2 = static_cast<const float*>(d.wscale2);
    g.normw = d.normw;
    g.eps = d.eps;
    g.out_scale = static_cast<__half*>(d.out_scale);
    auto lora_ok = [](const void* t, const void* up, int r) {
      return (t == nullptr && up == nullptr) ||
             (t && up && aligned16(t) && aligned16(up) && r > 0 && r % 8 == 0 && r <= 1024);
    };
    if (!lora_ok(d.lt, d.lup, d.lr) || !lora_ok(d.lt2, d.lup2, d.lr2) || (d.lt2 && !pairw) ||
        ((d.lt || d.lt2) && (d.kind == SEG_F32 || d.kind == SEG_F32_SCATTER)))
      return (int)cudaErrorInvalidValue;
    g.lt = static_cast<const __nv_bfloat16*>(d.lt);
    g.lup = static_cast<const __nv_bfloat16*>(d.lup);
    g.lr = d.lr;
    g.ls = d.ls;
    g.lt2 = static_cast<const __nv_bfloat16*>(d.lt2);
    g.lup2 = static_cast<const __nv_bfloat16*>(d.lup2);
    g.lr2 = d.lr2;
    g.ls2 = d.ls2;
    if (d.kind == SEG_QKNORM && (!d.normw || !freqs || !aligned16(freqs))) return (int)cudaErrorInvalidValue;
    if (d.kind == SEG_RESIDUAL && (!gate || !resid || !aligned16(gate) || !aligned16(resid) || d.ld % 8))
      return (int)cudaErrorInvalidValue;
    if ((d.kind == SEG_SWIGLU || d.kind == SEG_SWIGLU_E4M3) && (!d.out_scale || d.ld % 16 || !aligned16(d.out)))
      return (int)cudaErrorInvalidValue;
    if ((d.kind == SEG_BF16 || d.kind == SEG_SIGMOID || d.kind == SEG_QKNORM || d.kind == SEG_SWIGLU_BF16) &&
        (d.ld % 8 || !aligned16(d.out)))
      return (int)cudaErrorInvalidValue;
    if ((d.kind == SEG_F32 || d.kind == SEG_F32_SCATTER) && (d.ld % 4 || !aligned16(d.out)))
      return (int)cudaErrorInvalidValue;
    tiles += g.tiles;
  }
  int rc = bytea ? make_map_2d(&amap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, 128,
                               GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B)
                 : make_map_2d(&amap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a, (uint64_t)K / 2, (uint64_t)M, (uint64_t)K / 2,
                               64, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  p.nseg = nseg;
  p.M = M;
  p.K = K;
  p.G = K / 128;
  p.length = length;
  p.sa = static_cast<const __half*>(sa);
  p.freqs = freqs;
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.resid = static_cast<const __nv_bfloat16*>(resid);
  if (refm) {
    p.xs = ref->xs;
    p.xs_stride = ref->xs_stride;
    p.ws_stride = ref->ws_stride;
    p.bias = ref->bias;
    p.f8fmt = ref->f8fmt;
  }
  if (segs[0].kind == SEG_F32_SCATTER) {
    // rows 0..M-1 go to ranks row / chunk, all of which must exist
    if (nseg != 1 || !peers || tp < 1 || tp > 4 || rank < 0 || rank >= tp || chunk <= 0 ||
        (long long)chunk * tp < M)
      return (int)cudaErrorInvalidValue;
    for (int i = 0; i < tp; ++i) {
      if (!aligned16(peers[i])) return (int)cudaErrorInvalidValue;
      p.peer[i] = static_cast<float*>(peers[i]);
    }
    p.scatter_chunk = chunk;
    p.scatter_rank = rank;
  }
  const bool pairw = segs[0].kind == SEG_SWIGLU || segs[0].kind == SEG_SWIGLU_BF16 || segs[0].kind == SEG_SWIGLU_E4M3;
  typedef void (*GemmKernel)(CUtensorMap, WeightMaps, GemmParams);
  static const GemmKernel kernels[5][2] = {
      {gemm_w4a4_kernel<false, GM_PACKED>, gemm_w4a4_kernel<true, GM_PACKED>},
      {gemm_w4a4_kernel<false, GM_BYTES>, gemm_w4a4_kernel<true, GM_BYTES>},
      {gemm_w4a4_kernel<false, GM_REF4>, gemm_w4a4_kernel<true, GM_REF4>},
      {gemm_w4a4_kernel<false, GM_REF8>, nullptr},
      {gemm_w4a4_kernel<false, GM_REFF8>, gemm_w4a4_kernel<true, GM_REFF8>}};
  // LoRA variants: the group-128 (packed or e4m3 byte A) and the reference INT4 contracts
  static const GemmKernel lora_kernels[5][2] = {
      {gemm_w4a4_kernel<false, GM_PACKED, true>, gemm_w4a4_kernel<true, GM_PACKED, true>},
      {gemm_w4a4_kernel<false, GM_BYTES, true>, gemm_w4a4_kernel<true, GM_BYTES, true>},
      {gemm_w4a4_kernel<false, GM_REF4, true>, gemm_w4a4_kernel<true, GM_REF4, true>},
      {nullptr, nullptr},
      {nullptr, nullptr}};
  bool lora = false;
  for (int i = 0; i < nseg; ++i) lora = lora || segs[i].lt || segs[i].lt2;
  if (mode < 0 || mode > GM_REFF8) return (int)cudaErrorInvalidValue;
  GemmKernel kern = (lora ? lora_kernels : kernels)[mode][pairw ? 1 : 0];
  if (!kern) return (int)cudaErrorInvalidValue;
  const int variant = 10 * (lora ? 1 : 0) + 2 * mode + (pairw ? 1 : 0);
  static bool attr_set[64][20] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
  if (!attr_set[dev][variant]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    // setmaxnreg splits exactly the registers the CTA is launched with: any
    // other allocation could leave a warpgroup waiting for registers.
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return (int)e;
    if (fa.numRegs != GEMM_LAUNCH_REGS) return (int)cudaErrorInvalidConfiguration;
    attr_set[dev][variant] = true;
  }
  // CTA pairs along M (cluster 2 x 1 x 1): 256 rows per pair.
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(2 * ((M + 2 * GEMM_BM - 1) / (2 * GEMM_BM)), tiles, 1);
  cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = GEMM_SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, amap, wm, p);
  if (e != cudaSuccess) return (int)e;
  return launch_status();
}

// ----------------------------------------------------------- attention
static int attention_launch(const void* q, const void* k, const void* v, const void* gate, void* out, void* oq,
                            void* os, int batch, int heads, int kvheads, int lq, int lk, int dim, long long q_sb,
                            long long q_sh, long long q_st, long long k_sb, long long k_sh, long long k_st,
                            long long v_sb, long long v_sh, long long v_st, int gate_kind, cudaStream_t st,
                            bool oq_bytes = false) {
  if (batch <= 0 || heads <= 0 || kvheads <= 0 || heads % kvheads || lq <= 0 || lk <= 0 || dim != FA_D)
    return (int)cudaErrorInvalidValue;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (!out && !oq) || (oq && !os)) return (int)cudaErrorInvalidValue;
  if (out && !aligned16(out)) return (int)cudaErrorInvalidValue;
  if (oq && !aligned16(oq)) return (int)cudaErrorInvalidValue;
  if (gate && (!aligned16(gate) || (gate_kind != 1 && gate_kind != 2))) return (int)cudaErrorInvalidValue;
  // TMA strides must be multiples of 16 bytes (8 bf16 elements)
  const long long strides[9] = {q_sb, q_sh, q_st, k_sb, k_sh, k_st, v_sb, v_sh, v_st};
  for (long long s : strides)
    if (s <= 0 || s % 8) return (int)cudaErrorInvalidValue;
  AttnMaps maps;
  int rc = make_map_4d_bf16(&maps.q, q, FA_D, lq, heads, batch, q_st, q_sh, q_sb, 64, FA_BM);
  if (!rc) rc = make_map_4d_bf16(&maps.k, k, FA_D, lk, kvheads, batch, k_st, k_sh, k_sb, 64, FA_BN);
  if (!rc) rc = make_map_4d_bf16(&maps.v, v, FA_D, lk, kvheads, batch, v_st, v_sh, v_sb, 64, FA_BN);
  if (rc) return rc;
  AttnParams p;
  p.batch = batch;
  p.heads = heads;
  p.kvheads = kvheads;
  p.lq = lq;
  p.lk = lk;
  p.c = (float)(1.4426950408889634 / 11.313708498984761);  // log2(e)/sqrt(128)
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.gate_kind = gate ? gate_kind : 0;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.oq = static_cast<uint8_t*>(oq);
  p.os = static_cast<__half*>(os);
  p.oq_bytes = oq_bytes ? 1 : 0;
  // an odd GQA group cannot pair two heads on one KV head: pair two Q tiles
  p.qpair = (heads / kvheads) % 2 ? 1 : 0;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    attr_set[dev] = true;
  }
  dim3 grid(p.qpair ? (lq + 2 * FA_BM - 1) / (2 * FA_BM) : (lq + FA_BM - 1) / FA_BM, p.qpair ? heads : heads / 2,
            batch);
  attention_kernel<<<grid, FA_THREADS, FA_SMEM_BYTES, st>>>(maps, p);
  return launch_status();
}

// ------------------------------------------------ bounded-wait self-test
// Exercises the failure path every kernel's waits share (mbar_wait), on a
// barrier of its own.  One CTA of two warps:
//   mode 0: lane 0 of warp 1 completes the barrier warp 0 waits on;
//   mode 1: nothing completes it, so warp 0 gives up after `limit_ns`
//           (raising the CTA's abort flag and ERR_WAIT_SELFTEST), while warp 1
//           waits with a 64x longer limit on a second barrier that nothing
//           completes, and leaves when it sees the abort flag.
// result[0] = warp 0's wait succeeded, result[1] = warp 1 left through the
// abort flag (its wait failed before its own limit), result[2] = warp 1's
// time in its wait in microseconds.
__global__ void selftest_wait_kernel(int mode, unsigned long long limit_ns, int* result) {
  __shared__ __align__(8) uint64_t bar[2];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    const bool ok = mbar_wait(&bar[0], 0, &abort_flag, ERR_WAIT_SELFTEST, limit_ns);
    if (lane == 0) result[0] = ok ? 1 : 0;
  } else if (mode == 0) {
    if (lane == 0) {
      mbar_arrive(&bar[0]);
      result[1] = 0;
      result[2] = 0;
    }
  } else {
    const unsigned long long t0 = global_timer();
    const bool ok = mbar_wait(&bar[1], 0, &abort_flag, ERR_WAIT_SELFTEST, 64 * limit_ns);
    const unsigned long long dt = global_timer() - t0;
    if (lane == 0) {
      result[1] = (!ok && dt < 64 * limit_ns) ? 1 : 0;
      result[2] = (int)(dt / 1000);
    }
  }
}

}  // namespace k2b

using namespace k2b;

// =====================================================================
//                                C-ABI
// =====================================================================

K2B_EXPORT const char* k2b_version(void) { return "k2b 0.1 sm_100a"; }

// Bounded-wait self-test (see selftest_wait_kernel); `result` is a device
// int[3].  limit_ns is capped at one second.
K2B_EXPORT int k2b_selftest_wait(int mode, long long limit_ns, void* result, void* stream) {
  if ((mode != 0 && mode != 1) || limit_ns <= 0 || limit_ns > 1000000000ll || !result)
    return (int)cudaErrorInvalidValue;
  selftest_wait_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(mode, (unsigned long long)limit_ns,
                                                          static_cast<int*>(result));
  return launch_status();
}

K2B_EXPORT int k2b_device_error(int reset, void* stream) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_error, sizeof(int), 0, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e != cudaSuccess) return -(int)e;
  e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return -(int)e;
  if (reset) {
    int z = 0;
    e = cudaMemcpyToSymbolAsync(g_error, &z, sizeof(int), 0, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return -(int)e;
  }
  return v;
}

K2B_EXPORT int k2b_norm_quant(const void* x, const void* w, const void* scale, const void* shift, void* q, void* s,
                              int rows, int K, int length, int cut, int batch, float eps, void* stream) {
  return norm_quant_launch<true, true, true>(x, w, scale, shift, q, s, rows, K, length, cut, batch, eps,
                                             (cudaStream_t)stream);
}

// norm_quant of rows [base_row, base_row + rows) of a latent stream (x, q, s
// point at the first of them): the modulation row of each row follows its
// index in the whole stream, so a row shard quantises exactly as the
// unsharded call would.
K2B_EXPORT int k2b_norm_quant_rows(const void* x, const void* w, const void* scale, const void* shift, void* q,
                                   void* s, int base_row, int rows, int K, int length, int cut, int batch, float eps,
                                   void* stream) {
  return norm_quant_launch<true, true, true>(x, w, scale, shift, q, s, rows, K, length, cut, batch, eps,
                                             (cudaStream_t)stream, base_row);
}

K2B_EXPORT int k2b_rotate_quant(const void* x, void* q, void* s, int rows, int K, void* stream) {
  return norm_quant_launch<false, false, true>(x, nullptr, nullptr, nullptr, q, s, rows, K, 1, -1, 1, 0.0f,
                                               (cudaStream_t)stream);
}

K2B_EXPORT int k2b_norm_mod(const void* x, const void* w, const void* scale, const void* shift, void* y, int rows,
                            int K, int length, int cut, int batch, float eps, void* stream) {
  if ((scale == nullptr) != (shift == nullptr)) return (int)cudaErrorInvalidValue;
  if (scale)
    return norm_quant_launch<true, true, false>(x, w, scale, shift, y, nullptr, rows, K, length, cut, batch, eps,
                                                (cudaStream_t)stream);
  return norm_quant_launch<true, false, false>(x, w, nullptr, nullptr, y, nullptr, rows, K, 1, -1, 1, eps,
                                               (cudaStream_t)stream);
}

static int gated_add_launch(const void* p, int nslots, long long slot_stride, const void* gate, const void* resid,
                            void* out, int base_row, int rows, int n, int length, cudaStream_t st) {
  if (rows < 0 || n <= 0 || n % 8 || length <= 0 || base_row < 0 || nslots < 1 || nslots > 8 || slot_stride % 4 ||
      !aligned16(p) || !aligned16(gate) || !aligned16(resid) || !aligned16(out))
    return (int)cudaErrorInvalidValue;
  if (rows == 0) return 0;
  const long long work = (long long)rows * (n / 8);
  const long long blocks = (work + 255) / 256;
  const int grid = (int)(blocks < 148 * 16 ? blocks : 148 * 16);
  gated_add_kernel<<<grid, 256, 0, st>>>(static_cast<const float*>(p), nslots, (int64_t)slot_stride,
                                         static_cast<const __nv_bfloat16*>(gate),
                                         static_cast<const __nv_bfloat16*>(resid), static_cast<__nv_bfloat16*>(out),
                                         base_row, rows, n, length);
  return launch_status();
}

K2B_EXPORT int k2b_gated_add(const void* p, const void* gate, const void* resid, void* out, int base_row, int rows,
                             int n, int length, void* stream) {
  return gated_add_launch(p, 1, 0, gate, resid, out, base_row, rows, n, length, (cudaStream_t)stream);
}

K2B_EXPORT int k2b_reduce_gated_add(const void* slots, int nslots, long long slot_stride, const void* gate,
                                    const void* resid, void* out, int base_row, int rows, int n, int length,
                                    void* stream) {
  return gated_add_launch(slots, nslots, slot_stride, gate, resid, out, base_row, rows, n, length,
                          (cudaStream_t)stream);
}

// --------------------------------------------- peer buffers (CUDA IPC)
// A device buffer another process on this node can map: the tensor-parallel
// receive slots of k2b_gemm_f32_scatter.  handle: 64 bytes (cudaIpcMemHandle_t).
K2B_EXPORT int k2b_ipc_alloc(long long bytes, void** ptr, void* handle) {
  if (bytes <= 0 || !ptr || !handle) return (int)cudaErrorInvalidValue;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return (int)e;
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return (int)e;
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return 0;
}
K2B_EXPORT int k2b_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return (int)cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return (int)cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}
K2B_EXPORT int k2b_ipc_close(void* ptr) { return (int)cudaIpcCloseMemHandle(ptr); }
K2B_EXPORT int k2b_ipc_free(void* ptr) { return (int)cudaFree(ptr); }

K2B_EXPORT int k2b_elementwise(const void* a, const void* b, const void* r, void* y, long long n, int mode, int width,
                               void* stream) {
  if (n < 0 || !a || !y || mode < 0 || mode > 2 || (mode == 2 && (!b || !r || width <= 0)))
    return (int)cudaErrorInvalidValue;
  if (n == 0) return 0;
  const long long blocks = (n + 255) / 256;
  const int grid = (int)(blocks < 148 * 32 ? blocks : 148 * 32);
  elementwise_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), static_cast<const __nv_bfloat16*>(r),
      static_cast<__nv_bfloat16*>(y), (int64_t)n, mode, width);
  return launch_status();
}

// Packed INT4 codes [rows, K/2] -> e4m3 bytes [rows, K] (nbytes = packed
// bytes, a multiple of 16; both buffers 16-byte aligned).
K2B_EXPORT int k2b_expand_e4m3(const void* a, void* a8, long long nbytes, void* stream) {
  if (nbytes < 0 || nbytes % 16 || !aligned16(a) || !aligned16(a8)) return (int)cudaErrorInvalidValue;
  if (nbytes == 0) return 0;
  const long long n16 = nbytes / 16;
  const long long blocks = (n16 + 255) / 256;
  const int grid = (int)(blocks < 148 * 16 ? blocks : 148 * 16);
  expand_e4m3_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(static_cast<const uint4*>(a), static_cast<uint4*>(a8),
                                                              (int64_t)n16);
  return launch_status();
}

K2B_EXPORT int k2b_rope(const void* q, const void* k, const void* f, void* qo, void* ko, int batch, int length, int qh,
                        int kh, int dim, int fb, void* stream) {
  if (batch <= 0 || length <= 0 || qh < 0 || kh < 0 || qh + kh == 0 || dim <= 0 || dim % 2 || (fb != 1 && fb != batch))
    return (int)cudaErrorInvalidValue;
  if (!f || !aligned16(f) || (qh && (!q || !qo)) || (kh && (!k || !ko))) return (int)cudaErrorInvalidValue;
  const long long rows = (long long)batch * length * (qh + kh);
  const int grid = (int)(rows < 148 * 64 ? rows : 148 * 64);
  rope_kernel<<<grid, 64, 0, (cudaStream_t)stream>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), static_cast<const float*>(f),
      static_cast<__nv_bfloat16*>(qo), static_cast<__nv_bfloat16*>(ko), batch, length, qh, kh, dim, fb);
  return launch_status();
}

K2B_EXPORT int k2b_prepare_weight(const void* w_packed, const void* w_scale, void* w_prepared, void* scale_t, int n,
                                  int k, int block_rows, int dst_block_stride, int dst_offset, int scale_ld,
                                  void* stream) {
  if (n <= 0 || k <= 0 || k % 128 || block_rows <= 0 || dst_block_stride < block_rows || dst_offset < 0 ||
      scale_ld <= 0 || !aligned16(w_packed) || !aligned16(w_prepared))
    return (int)cudaErrorInvalidValue;
  const int64_t total = (int64_t)n * (k / 32);
  const int threads = 256;
  prepare_weight_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, (cudaStream_t)stream>>>(
      static_cast<const uint8_t*>(w_packed), static_cast<const __half*>(w_scale), static_cast<uint8_t*>(w_prepared),
      static_cast<float*>(scale_t), n, k, block_rows, dst_block_stride, dst_offset, scale_ld);
  return launch_status();
}

K2B_EXPORT int k2b_gemm_f32(const void* a, const void* sa, const void* w, const void* wscale, void* out, int m, int n,
                            int k, void* stream) {
  SegDesc d = {SEG_F32, n, w, wscale, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  return gemm_launch(a, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

// fp32 a@W of a tensor-parallel rank, stored straight into the owners' receive
// buffers: row r goes to peers[r / chunk] (fp32 [tp, chunk, n], local or an
// NVLink peer's mapping) in slot `rank`, row r % chunk.  The owner sums its tp
// slots (k2b_reduce_gated_add) after a barrier that follows this launch on
// every rank.
K2B_EXPORT int k2b_gemm_f32_scatter(const void* a, const void* sa, const void* w, const void* wscale,
                                    void* const* peers, int tp, int rank, int chunk, int m, int n, int k,
                                    void* stream) {
  if (!peers) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_F32_SCATTER, n, w, wscale, peers[0], n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  return gemm_launch(a, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, peers, tp, rank, chunk);
}

K2B_EXPORT int k2b_gemm_bf16(const void* a, const void* sa, const void* w, const void* wscale, void* out, int m, int n,
                             int k, void* stream) {
  SegDesc d = {SEG_BF16, n, w, wscale, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  return gemm_launch(a, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

K2B_EXPORT int k2b_qkv(const void* a, const void* sa, const void* wq, const void* swq, const void* wk,
                       const void* swk, const void* wv, const void* swv, const void* wg, const void* swg,
                       const void* nq, const void* nk, const void* freqs, void* qo, void* ko, void* vo, void* go,
                       int m, int length, int qwidth, int kvwidth, int k, float eq, float ek, void* stream) {
  if (qwidth <= 0 || kvwidth <= 0 || qwidth % 128 || kvwidth % 128) return (int)cudaErrorInvalidValue;
  SegDesc d[4] = {
      {SEG_QKNORM, qwidth, wq, swq, qo, qwidth, static_cast<const float*>(nq), eq, nullptr, nullptr, nullptr},
      {SEG_QKNORM, kvwidth, wk, swk, ko, kvwidth, static_cast<const float*>(nk), ek, nullptr, nullptr, nullptr},
      {SEG_BF16, kvwidth, wv, swv, vo, kvwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
      {SEG_SIGMOID, qwidth, wg, swg, go, qwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
  };
  const int nseg = (wg && go) ? 4 : 3;
  return gemm_launch(a, sa, m, k, d, nseg, length, static_cast<const float*>(freqs), nullptr, nullptr,
                     (cudaStream_t)stream);
}

K2B_EXPORT int k2b_gated_residual(const void* a, const void* sa, const void* w, const void* wscale, const void* gate,
                                  const void* residual, void* out, int m, int length, int n, int k, void* stream) {
  SegDesc d = {SEG_RESIDUAL, n, w, wscale, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  return gemm_launch(a, sa, m, k, &d, 1, length, nullptr, gate, residual, (cudaStream_t)stream);
}

K2B_EXPORT int k2b_swiglu_quant(const void* a, const void* sa, const void* wg, const void* sg, const void* wu,
                                const void* su, void* hq, void* hs, int m, int width, int k, void* stream) {
  if (width <= 0 || width % 128) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_SWIGLU, width, wg, sg, hq, width / 2, nullptr, 0.0f, hs, wu, su};
  return gemm_launch(a, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

K2B_EXPORT int k2b_swiglu_bf16(const void* a, const void* sa, const void* wg, const void* sg, const void* wu,
                               const void* su, void* h, int m, int width, int k, void* stream) {
  if (width <= 0 || width % 128) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_SWIGLU_BF16, width, wg, sg, h, width, nullptr, 0.0f, nullptr, wu, su};
  return gemm_launch(a, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream);
}

K2B_EXPORT int k2b_attention(const void* q, const void* k, const void* v, const void* gate, void* out, int batch,
                             int heads, int kvheads, int lq, int lk, int dim, long long q_sb, long long q_sh,
                             long long q_st, long long k_sb, long long k_sh, long long k_st, long long v_sb,
                             long long v_sh, long long v_st, int gate_kind, void* stream) {
  return attention_launch(q, k, v, gate, out, nullptr, nullptr, batch, heads, kvheads, lq, lk, dim, q_sb, q_sh, q_st,
                          k_sb, k_sh, k_st, v_sb, v_sh, v_st, gate_kind, (cudaStream_t)stream);
}

K2B_EXPORT int k2b_attention_quant(const void* q, const void* k, const void* v, void* oq, void* os, int batch,
                                   int heads, int kvheads, int lq, int lk, int dim, long long q_sb, long long q_sh,
                                   long long q_st, long long k_sb, long long k_sh, long long k_st, long long v_sb,
                                   long long v_sh, long long v_st, void* stream) {
  return attention_launch(q, k, v, nullptr, nullptr, oq, os, batch, heads, kvheads, lq, lk, dim, q_sb, q_sh, q_st,
                          k_sb, k_sh, k_st, v_sb, v_sh, v_st, 0, (cudaStream_t)stream);
}

// ---------------------------------------------- e4m3 byte containers
// The block loop keeps the INT4 codes between its kernels as e4m3 bytes
// [rows, K] (same codes, one byte each) so that its GEMMs load A with TMA
// straight into the tensor-core layout; these are the producers and
// consumers of that container, with the arguments of their packed twins.
K2B_EXPORT int k2b_norm_quant_e4m3(const void* x, const void* w, const void* scale, const void* shift, void* q8,
                                   void* s, int rows, int K, int length, int cut, int batch, float eps, void* stream) {
  return norm_quant_launch<true, true, true, true>(x, w, scale, shift, q8, s, rows, K, length, cut, batch, eps,
                                                   (cudaStream_t)stream);
}

K2B_EXPORT int k2b_attention_quant_e4m3(const void* q, const void* k, const void* v, void* oq8, void* os, int batch,
                                        int heads, int kvheads, int lq, int lk, int dim, long long q_sb,
                                        long long q_sh, long long q_st, long long k_sb, long long k_sh,
                                        long long k_st, long long v_sb, long long v_sh, long long v_st,
                                        void* stream) {
  return attention_launch(q, k, v, nullptr, nullptr, oq8, os, batch, heads, kvheads, lq, lk, dim, q_sb, q_sh, q_st,
                          k_sb, k_sh, k_st, v_sb, v_sh, v_st, 0, (cudaStream_t)stream, true);
}

K2B_EXPORT int k2b_gemm_f32_e4m3(const void* a8, const void* sa, const void* w, const void* wscale, void* out, int m,
                                 int n, int k, void* stream) {
  SegDesc d = {SEG_F32, n, w, wscale, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  return gemm_launch(a8, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0, GM_BYTES);
}

K2B_EXPORT int k2b_qkv_e4m3(const void* a8, const void* sa, const void* wq, const void* swq, const void* wk,
                            const void* swk, const void* wv, const void* swv, const void* wg, const void* swg,
                            const void* nq, const void* nk, const void* freqs, void* qo, void* ko, void* vo, void* go,
                            int m, int length, int qwidth, int kvwidth, int k, float eq, float ek, void* stream) {
  if (qwidth <= 0 || kvwidth <= 0 || qwidth % 128 || kvwidth % 128) return (int)cudaErrorInvalidValue;
  SegDesc d[4] = {
      {SEG_QKNORM, qwidth, wq, swq, qo, qwidth, static_cast<const float*>(nq), eq, nullptr, nullptr, nullptr},
      {SEG_QKNORM, kvwidth, wk, swk, ko, kvwidth, static_cast<const float*>(nk), ek, nullptr, nullptr, nullptr},
      {SEG_BF16, kvwidth, wv, swv, vo, kvwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
      {SEG_SIGMOID, qwidth, wg, swg, go, qwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
  };
  const int nseg = (wg && go) ? 4 : 3;
  return gemm_launch(a8, sa, m, k, d, nseg, length, static_cast<const float*>(freqs), nullptr, nullptr,
                     (cudaStream_t)stream, nullptr, 0, 0, 0, GM_BYTES);
}

K2B_EXPORT int k2b_gated_residual_e4m3(const void* a8, const void* sa, const void* w, const void* wscale,
                                       const void* gate, const void* residual, void* out, int m, int length, int n,
                                       int k, void* stream) {
  SegDesc d = {SEG_RESIDUAL, n, w, wscale, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  return gemm_launch(a8, sa, m, k, &d, 1, length, nullptr, gate, residual, (cudaStream_t)stream, nullptr, 0, 0, 0,
                     GM_BYTES);
}

K2B_EXPORT int k2b_swiglu_quant_e4m3(const void* a8, const void* sa, const void* wg, const void* sg, const void* wu,
                                     const void* su, void* h8, void* hs, int m, int width, int k, void* stream) {
  if (width <= 0 || width % 128) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_SWIGLU_E4M3, width, wg, sg, h8, width, nullptr, 0.0f, hs, wu, su};
  return gemm_launch(a8, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0, GM_BYTES);
}

K2B_EXPORT int k2b_gemm_bf16_e4m3(const void* a8, const void* sa, const void* w, const void* wscale, void* out, int m,
                                  int n, int k, void* stream) {
  SegDesc d = {SEG_BF16, n, w, wscale, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  return gemm_launch(a8, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0, GM_BYTES);
}

K2B_EXPORT int k2b_swiglu_quant_a8(const void* a8, const void* sa, const void* wg, const void* sg, const void* wu,
                                   const void* su, void* hq, void* hs, int m, int width, int k, void* stream) {
  if (width <= 0 || width % 128) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_SWIGLU, width, wg, sg, hq, width / 2, nullptr, 0.0f, hs, wu, su};
  return gemm_launch(a8, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0, GM_BYTES);
}

K2B_EXPORT int k2b_swiglu_bf16_e4m3(const void* a8, const void* sa, const void* wg, const void* sg, const void* wu,
                                    const void* su, void* h, int m, int width, int k, void* stream) {
  if (width <= 0 || width % 128) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_SWIGLU_BF16, width, wg, sg, h, width, nullptr, 0.0f, nullptr, wu, su};
  return gemm_launch(a8, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0, GM_BYTES);
}

K2B_EXPORT int k2b_gemm_f32_scatter_e4m3(const void* a8, const void* sa, const void* w, const void* wscale,
                                         void* const* peers, int tp, int rank, int chunk, int m, int n, int k,
                                         void* stream) {
  SegDesc d = {SEG_F32_SCATTER, n, w, wscale, peers ? peers[0] : nullptr, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  return gemm_launch(a8, sa, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, peers, tp, rank, chunk,
                     GM_BYTES);
}

// ------------------------------------------------ INT8 / FP8 weight formats
// Projections of checkpoints stored as INT8 or FP8 weights (the reference's
// formats 2 and 3/4, native_runtime.cpp:271-283, 298-311), on the same pair
// GEMM with the whole of K in one accumulator and the dequant in the
// epilogue: out = bf16(fp32(fp32(acc * xs[r * xs_stride]) * ws[c * ws_stride])
// + bias[c]).  The reference runs at::_int_mm + k2_dequant8 (INT8) and
// at::_scaled_mm (FP8) there.
//   k2b_gemm8:  a8 int8 [m, k] (k2_quant8's rows), w8 int8 [n, k], int32
//               accumulator;
//   k2b_gemm_f8: a8 / w8 fp8 [m, k] / [n, k], fmt 0 e4m3 / 1 e5m2 each, fp32
//               accumulator.
// ws_stride / xs_stride 0: one scale for the whole operand.  bias fp32 [n] or
// null.  k % 128 == 0, n % 128 == 0.
K2B_EXPORT int k2b_gemm8(const void* a8, const void* xs, int xs_stride, const void* w8, const void* ws, int ws_stride,
                         const void* bias, void* out, int m, int n, int k, void* stream) {
  if ((xs_stride != 0 && xs_stride != 1) || (ws_stride != 0 && ws_stride != 1)) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_BF16, n, w8, ws, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  RefScales r;
  r.xs = static_cast<const float*>(xs);
  r.xs_stride = xs_stride;
  r.ws_stride = ws_stride;
  r.bias = static_cast<const float*>(bias);
  return gemm_launch(a8, nullptr, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0,
                     GM_REF8, &r);
}

K2B_EXPORT int k2b_gemm_f8(const void* a8, const void* xs, int xs_stride, const void* w8, const void* ws,
                           int ws_stride, const void* bias, void* out, int m, int n, int k, int afmt, int bfmt,
                           void* stream) {
  if ((xs_stride != 0 && xs_stride != 1) || (ws_stride != 0 && ws_stride != 1) || (afmt != 0 && afmt != 1) ||
      (bfmt != 0 && bfmt != 1))
    return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_BF16, n, w8, ws, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  RefScales r;
  r.xs = static_cast<const float*>(xs);
  r.xs_stride = xs_stride;
  r.ws_stride = ws_stride;
  r.bias = static_cast<const float*>(bias);
  r.f8fmt = (uint32_t)afmt | ((uint32_t)bfmt << 3);
  return gemm_launch(a8, nullptr, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0,
                     GM_REFF8, &r);
}

// Reference-contract INT4 joint QKV / SwiGLU / gated residual for a stream of
// `batch` latents of `length` tokens (the reference-named exports take one
// latent): RoPE token = row % length, gate row = row / length.
K2B_EXPORT int k2b_ref_qkv(const void* a, const void* xs, const void* wq, const void* sq, const void* wk,
                           const void* sk, const void* wv, const void* sv, const void* wg, const void* sg,
                           const void* nq, const void* nk, const void* freq, void* qo, void* ko, void* vo, void* go,
                           int m, int length, int qwidth, int kvwidth, int k, float eq, float ek, void* stream) {
  if (qwidth <= 0 || kvwidth <= 0 || qwidth % 128 || kvwidth % 128 || length <= 0 || !freq)
    return (int)cudaErrorInvalidValue;
  SegDesc d[4] = {
      {SEG_QKNORM, qwidth, wq, sq, qo, qwidth, static_cast<const float*>(nq), eq, nullptr, nullptr, nullptr},
      {SEG_QKNORM, kvwidth, wk, sk, ko, kvwidth, static_cast<const float*>(nk), ek, nullptr, nullptr, nullptr},
      {SEG_BF16, kvwidth, wv, sv, vo, kvwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
      {SEG_SIGMOID, qwidth, wg, sg, go, qwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
  };
  RefScales r;
  r.xs = static_cast<const float*>(xs);
  return gemm_launch(a, nullptr, m, k, d, (wg && go) ? 4 : 3, length, static_cast<const float*>(freq), nullptr,
                     nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0, GM_REF4, &r);
}

// The same reference-contract INT4 projections with A and W as e4m3 code
// bytes ([m, k] from k2b_expand_e4m3, [n, k] expanded once from the packed
// checkpoint rows): the INT4 codes are exact e4m3 values and every partial
// sum an integer below 2^24, so the fp32 accumulator and the result are those
// of the packed form (GM_REF4), without its in-CTA unpacking (gate/up at
// 33792 x 16384 x 6144: the packed joint SwiGLU takes 19.2 ms).
//   k2b_ref_qkv8 / k2b_ref_gated_residual8: as k2b_ref_qkv /
//   k2b_ref_gated_residual; k2b_ref_swiglu8: as k2_int4_swiglu (bf16 h).
K2B_EXPORT int k2b_ref_qkv8(const void* a8, const void* xs, const void* wq, const void* sq, const void* wk,
                            const void* sk, const void* wv, const void* sv, const void* wg, const void* sg,
                            const void* nq, const void* nk, const void* freq, void* qo, void* ko, void* vo, void* go,
                            int m, int length, int qwidth, int kvwidth, int k, float eq, float ek, void* stream) {
  if (qwidth <= 0 || kvwidth <= 0 || qwidth % 128 || kvwidth % 128 || length <= 0 || !freq)
    return (int)cudaErrorInvalidValue;
  SegDesc d[4] = {
      {SEG_QKNORM, qwidth, wq, sq, qo, qwidth, static_cast<const float*>(nq), eq, nullptr, nullptr, nullptr},
      {SEG_QKNORM, kvwidth, wk, sk, ko, kvwidth, static_cast<const float*>(nk), ek, nullptr, nullptr, nullptr},
      {SEG_BF16, kvwidth, wv, sv, vo, kvwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
      {SEG_SIGMOID, qwidth, wg, sg, go, qwidth, nullptr, 0.0f, nullptr, nullptr, nullptr},
  };
  RefScales r;
  r.xs = static_cast<const float*>(xs);
  return gemm_launch(a8, nullptr, m, k, d, (wg && go) ? 4 : 3, length, static_cast<const float*>(freq), nullptr,
                     nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0, GM_REFF8, &r);
}

K2B_EXPORT int k2b_ref_swiglu8(const void* a8, const void* wg, const void* wu, const void* xs, const void* sg,
                               const void* su, void* out, int m, int n, int k, void* stream) {
  if (n <= 0 || n % 128) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_SWIGLU_BF16, n, wg, sg, out, n, nullptr, 0.0f, nullptr, wu, su};
  RefScales r;
  r.xs = static_cast<const float*>(xs);
  return gemm_launch(a8, nullptr, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0,
                     GM_REFF8, &r);
}

K2B_EXPORT int k2b_ref_gated_residual8(const void* a8, const void* xs, const void* w, const void* ws,
                                       const void* gate, const void* residual, void* out, int m, int length, int n,
                                       int k, void* stream) {
  SegDesc d = {SEG_RESIDUAL, n, w, ws, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  RefScales r;
  r.xs = static_cast<const float*>(xs);
  return gemm_launch(a8, nullptr, m, k, &d, 1, length, nullptr, gate, residual, (cudaStream_t)stream, nullptr, 0, 0,
                     0, GM_REFF8, &r);
}

K2B_EXPORT int k2b_ref_gated_residual(const void* a, const void* xs, const void* w, const void* ws, const void* gate,
                                      const void* residual, void* out, int m, int length, int n, int k,
                                      void* stream) {
  SegDesc d = {SEG_RESIDUAL, n, w, ws, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  RefScales r;
  r.xs = static_cast<const float*>(xs);
  return gemm_launch(a, nullptr, m, k, &d, 1, length, nullptr, gate, residual, (cudaStream_t)stream, nullptr, 0, 0,
                     0, GM_REF4, &r);
}

// ------------------------------------------------------ LoRA bypass deltas
// A projection with one LoRA bypass factor pair fused into its epilogue
// (graph_ops.py:246-249 composes value + T(T(x down^T) up^T) * s after the
// projection):  out = E(T(T(p) + T(T(t up^T) * s))), t = T(x down^T) bf16
// [m, lr] (the caller's rank-lr product of the bf16 input), up bf16 [n, lr],
// lr % 8 == 0; E = T (gate and residual null) or the gated residual
// T(residual + T(p' * gate[row / length])).
//   contract 0: group-128 W4A4 (a packed [m, k/2], s fp16 [m, k/128], w / ws
//               prepared); 2: the same with a as e4m3 bytes [m, k];
//               contract 1: the reference's INT4 (a packed, s fp32 [m], w
//               packed [n, k/2], ws fp32 [n]; bias fp32 [n] or null).
K2B_EXPORT int k2b_lora_gemm(int contract, const void* a, const void* s, const void* w, const void* ws,
                             const void* bias, const void* gate, const void* residual, int length, const void* lt,
                             const void* lup, int lr, float ls, void* out, int m, int n, int k, void* stream) {
  if (contract < 0 || contract > 2 || !lt || !lup || (gate == nullptr) != (residual == nullptr) ||
      (bias && (contract != 1 || gate)) || length <= 0)
    return (int)cudaErrorInvalidValue;
  SegDesc d = {gate ? SEG_RESIDUAL : SEG_BF16, n, w, ws, out, n, nullptr, 0.0f, nullptr, nullptr, nullptr};
  d.lt = lt;
  d.lup = lup;
  d.lr = lr;
  d.ls = ls;
  if (contract != 1)
    return gemm_launch(a, s, m, k, &d, 1, length, nullptr, gate, residual, (cudaStream_t)stream, nullptr, 0, 0, 0,
                       contract == 2 ? GM_BYTES : GM_PACKED);
  RefScales r;
  r.xs = static_cast<const float*>(s);
  r.bias = static_cast<const float*>(bias);
  return gemm_launch(a, nullptr, m, k, &d, 1, length, nullptr, gate, residual, (cudaStream_t)stream, nullptr, 0, 0,
                     0, GM_REF4, &r);
}

// SwiGLU with a LoRA pair on each half: h = T(T(silu(g')) * u'), g' / u' the
// LoRA-corrected T(p) of the gate / up projections (either pair may be null),
// bf16 h [m, width]; contract as k2b_lora_gemm.
K2B_EXPORT int k2b_lora_swiglu(int contract, const void* a, const void* s, const void* wg, const void* sg,
                               const void* wu, const void* su, const void* lt_g, const void* lup_g, int lr_g,
                               float ls_g, const void* lt_u, const void* lup_u, int lr_u, float ls_u, void* h,
                               int m, int width, int k, void* stream) {
  if (contract < 0 || contract > 2 || width <= 0 || width % 128) return (int)cudaErrorInvalidValue;
  SegDesc d = {SEG_SWIGLU_BF16, width, wg, sg, h, width, nullptr, 0.0f, nullptr, wu, su};
  d.lt = lt_g;
  d.lup = lup_g;
  d.lr = lr_g;
  d.ls = ls_g;
  d.lt2 = lt_u;
  d.lup2 = lup_u;
  d.lr2 = lr_u;
  d.ls2 = ls_u;
  if (contract != 1)
    return gemm_launch(a, s, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0,
                       contract == 2 ? GM_BYTES : GM_PACKED);
  RefScales r;
  r.xs = static_cast<const float*>(s);
  return gemm_launch(a, nullptr, m, k, &d, 1, m, nullptr, nullptr, nullptr, (cudaStream_t)stream, nullptr, 0, 0, 0,
                     GM_REF4, &r);
}

#include "abi_reference.cuh"
#include "block_loop.cuh"
