// ref_contract.cuh -- the quantisers and element kernels of the reference's
// own data contract, behind the reference's symbol names (abi_reference.cuh).
//
// The reference runtime (native_runtime.cpp:262-311, 432-447) hands its kernel
// library one fp32 scale per activation row ([m, 1]) and per weight channel,
// INT4 activations rotated by ConvRot in groups of 16, 64 or 256
// (kernels/norm_quant.cu:40-66; the real checkpoint uses 256), int8 rowwise
// activations for INT8 weights and fp8 tensors with one scale for FP8
// weights.  The group-128 kernels of this library (norm_quant.cuh) keep
// BASELINE's contract; these keep the reference's, so a buffer the reference
// sized can never be overrun.
//
// Rotation (restated; comfy-kitchen, whose helpers the reference links, is not
// part of the reference's sources): a normalised block Walsh-Hadamard
// transform of G = 4^s columns in radix-4 stages at strides 1, 4, 16, 64,
// each stage rounding its outputs to T, as the reference's typed stages do
// (kernels/norm_quant.cu:48-60).  One stage maps (a, b, c, d) to
//   T(((a+b) + (c+d)) * 0.5), T(((a-b) + (c-d)) * 0.5),
//   T(((a+b) - (c+d)) * 0.5), T(((a-b) - (c-d)) * 0.5)
// (fp32 sums; the Sylvester order of H4 / 2, an orthonormal stage).
// Quantisation (kernels/norm_quant.cu:61-66): amax over the rotated row
// (NaN ignored, infinity clamped to T's largest finite value), scale =
// max(amax / 7, 1e-10) in fp32, inverse = 1 / scale (correctly rounded),
// code = clamp(rne(v * inverse), -8, 7); two codes per byte, the even column
// in the low nibble.
#pragma once
#include "k2b_common.cuh"

namespace k2b {

constexpr int kRefThreads = 256;
constexpr float kBf16MaxFinite = 3.3895313892515355e38f;

// One radix-4 rotation stage over the row held in shared memory (bf16), for
// every group of G columns, at stride st.
__device__ __forceinline__ void ref_rot_stage(__nv_bfloat16* v, int K, int st) {
  const int quads = K >> 2;
  for (int t = threadIdx.x; t < quads; t += blockDim.x) {
    // t-th quadruple: blocks of 4*st columns, st quadruples per block
    const int base = (t / st) * 4 * st + (t % st);
    const float a = __bfloat162float(v[base]), b = __bfloat162float(v[base + st]);
    const float c = __bfloat162float(v[base + 2 * st]), d = __bfloat162float(v[base + 3 * st]);
    const float s01 = __fadd_rn(a, b), d01 = __fsub_rn(a, b), s23 = __fadd_rn(c, d), d23 = __fsub_rn(c, d);
    v[base] = __float2bfloat16_rn(__fmul_rn(__fadd_rn(s01, s23), 0.5f));
    v[base + st] = __float2bfloat16_rn(__fmul_rn(__fadd_rn(d01, d23), 0.5f));
    v[base + 2 * st] = __float2bfloat16_rn(__fmul_rn(__fsub_rn(s01, s23), 0.5f));
    v[base + 3 * st] = __float2bfloat16_rn(__fmul_rn(__fsub_rn(d01, d23), 0.5f));
  }
}

// Block max of non-negative values (NaN ignored by fmaxf).
__device__ __forceinline__ float ref_block_max(float m, float* red) {
#pragma unroll
  for (int d = 16; d; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int d = 16; d; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    if (lane == 0) red[32] = m;
  }
  __syncthreads();
  return red[32];
}

// Reference-contract norm + modulation (NORM) + ConvRot + per-row INT4 (BITS
// = 4) or int8 (BITS = 8, codes clamped to [-127, 127], scale = amax / 127)
// of bf16 rows; one CTA per row.  group = 0: no rotation.
//   q: packed INT4 [rows, K/2] or int8 [rows, K];  s: fp32 [rows].
template <bool NORM, int BITS>
__global__ void __launch_bounds__(kRefThreads) ref_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                              const float* __restrict__ w,
                                                              const __nv_bfloat16* __restrict__ scale,
                                                              const __nv_bfloat16* __restrict__ shift,
                                                              uint8_t* __restrict__ q, float* __restrict__ s,
                                                              int K, int length, int cut, int batch, float eps,
                                                              int group) {
  extern __shared__ __align__(16) uint8_t ref_smem[];
  __nv_bfloat16* v = reinterpret_cast<__nv_bfloat16*>(ref_smem);
  __shared__ float red[33];
  const int row = blockIdx.x, tid = threadIdx.x;
  const __nv_bfloat16* xr = x + (int64_t)row * K;
  if (NORM) {
    // sum of squares in the reference's order (kernels/norm_quant.cu:20-31):
    // 128 lanes, lane l runs fmaf over columns 512i + 4l .. +3, then the warp
    // shfl_down tree and (s2 + s0) + (s3 + s1)
    float sum = 0.0f;
    if (tid < 128) {
      for (int col = tid * 4; col < K; col += 512) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float xv = col + j < K ? __bfloat162float(xr[col + j]) : 0.0f;
          sum = __fmaf_rn(xv, xv, sum);
        }
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) sum = __fadd_rn(sum, __shfl_down_sync(0xffffffffu, sum, off));
      if ((tid & 31) == 0) red[tid >> 5] = sum;
    }
    __syncthreads();
    if (tid == 0) {
      const float total = __fadd_rn(__fadd_rn(red[2], red[0]), __fadd_rn(red[3], red[1]));
      red[32] = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)K), eps));
    }
    __syncthreads();
    const float inv = red[32];
    int b = row / length;
    if (cut >= 0 && row % length >= cut) b += batch;
    for (int col = tid; col < K; col += kRefThreads) {
      float y = bf16_round(__fmul_rn(__fmul_rn(__bfloat162float(xr[col]), inv), __fadd_rn(w[col], 1.0f)));
      if (scale) {
        const float f = bf16_round(__fadd_rn(__bfloat162float(scale[(int64_t)b * K + col]), 1.0f));
        y = bf16_round(__fmul_rn(y, f));
        y = bf16_round(__fadd_rn(y, __bfloat162float(shift[(int64_t)b * K + col])));
      }
      v[col] = __float2bfloat16_rn(y);
    }
  } else {
    for (int col = tid; col < K; col += kRefThreads) v[col] = xr[col];
  }
  __syncthreads();
  for (int st = 1; st < group; st *= 4) {
    ref_rot_stage(v, K, st);
    __syncthreads();
  }
  float m = 0.0f;
  for (int col = tid; col < K; col += kRefThreads) m = fmaxf(m, fabsf(__bfloat162float(v[col])));
  m = ref_block_max(m, red);
  const float qmax = BITS == 4 ? 7.0f : 127.0f;
  const float sc = fmaxf(__fdiv_rn(fminf(m, kBf16MaxFinite), qmax), 1e-10f);
  if (tid == 0) s[row] = sc;
  const float inverse = __fdiv_rn(1.0f, sc);
  if (BITS == 4) {
    uint8_t* qr = q + (int64_t)row * (K / 2);
    for (int i = tid; i < K / 2; i += kRefThreads) {
      const float c0 = fminf(fmaxf(rintf(__fmul_rn(__bfloat162float(v[2 * i]), inverse)), -8.0f), 7.0f);
      const float c1 = fminf(fmaxf(rintf(__fmul_rn(__bfloat162float(v[2 * i + 1]), inverse)), -8.0f), 7.0f);
      qr[i] = (uint8_t)(((int)c0 & 0xF) | (((int)c1 & 0xF) << 4));
    }
  } else {
    int8_t* qr = reinterpret_cast<int8_t*>(q) + (int64_t)row * K;
    for (int i = tid; i < K; i += kRefThreads)
      qr[i] = (int8_t)(int)fminf(fmaxf(rintf(__fmul_rn(__bfloat162float(v[i]), inverse)), -127.0f), 127.0f);
  }
}

// The INT4 quantiser above for rows of K % 512 == 0 and a ConvRot group of
// 16, 64 or 256 (the reference checkpoints' case), with the same arithmetic
// and rounding points, laid out for throughput: one CTA of 4 warps per row.
// * NORM: thread t (= reference lane t of the 128) runs its fmaf chain over
//   columns 512 i + 4 t .. +3, then the reference's shfl_down tree and
//   (s2 + s0) + (s3 + s1) (kernels/norm_quant.cu:20-31);
// * warp w takes the 512-column slabs w, w + 4, ...: lane l loads columns
//   16 l .. +15 (two 16-byte loads), normalises / modulates them, and runs the
//   stride-1 and stride-4 radix-4 stages in registers; for groups of 64 and
//   256 a 1 KB shared transpose gives half-warp h of the slab's 256-column
//   block h, lane r holding columns r + 16 j, j = 0..15, where the stride-16
//   and stride-64 stages are in registers too;
// * the rotated row (bf16, K*2 bytes of shared memory) and a block max give
//   the row scale; thread t then quantises 16 consecutive columns at a time
//   and stores them with one 8-byte (packed) or 16-byte (BYTES: e4m3 code
//   bytes [rows, K], the byte-operand GEMMs' container) store.
constexpr int kRefFastThreads = 128;

__device__ __forceinline__ void ref_quad(float& a, float& b, float& c, float& d) {
  const float s01 = __fadd_rn(a, b), d01 = __fsub_rn(a, b), s23 = __fadd_rn(c, d), d23 = __fsub_rn(c, d);
  a = bf16_round(__fmul_rn(__fadd_rn(s01, s23), 0.5f));
  b = bf16_round(__fmul_rn(__fadd_rn(d01, d23), 0.5f));
  c = bf16_round(__fmul_rn(__fsub_rn(s01, s23), 0.5f));
  d = bf16_round(__fmul_rn(__fsub_rn(d01, d23), 0.5f));
}

template <bool NORM, bool BYTES>
__global__ void __launch_bounds__(kRefFastThreads) ref_quant4_fast_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ w, const __nv_bfloat16* __restrict__ scale,
    const __nv_bfloat16* __restrict__ shift, uint8_t* __restrict__ q, float* __restrict__ s, int K, int length,
    int cut, int batch, float eps, int group) {
  extern __shared__ __align__(16) uint8_t ref_fast_smem[];
  __nv_bfloat16* v = reinterpret_cast<__nv_bfloat16*>(ref_fast_smem);  // rotated row [K]
  __shared__ __align__(16) __nv_bfloat16 tr[4][512];
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* xr = x + (int64_t)row * K;
  float inv = 0.0f;
  int bb = 0;
  if (NORM) {
    float sum = 0.0f;
    for (int col = 4 * tid; col < K; col += 512) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(xr + col));
      const float2 p0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      const float2 p1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
      sum = __fmaf_rn(p0.x, p0.x, sum);
      sum = __fmaf_rn(p0.y, p0.y, sum);
      sum = __fmaf_rn(p1.x, p1.x, sum);
      sum = __fmaf_rn(p1.y, p1.y, sum);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) sum = __fadd_rn(sum, __shfl_down_sync(0xffffffffu, sum, off));
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    const float total = __fadd_rn(__fadd_rn(red[2], red[0]), __fadd_rn(red[3], red[1]));
    inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)K), eps));
    bb = row / length;
    if (cut >= 0 && row % length >= cut) bb += batch;
  }
  float amax = 0.0f;
  const int h = lane >> 4, r = lane & 15;
  for (int slab = warp; slab < (K >> 9); slab += 4) {
    const int col = 512 * slab + 16 * lane;
    float e[16];
    {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(xr + col));
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(xr + col + 8));
      const uint32_t ws[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[k]));
        e[2 * k] = f.x;
        e[2 * k + 1] = f.y;
      }
    }
    if (NORM) {
#pragma unroll
      for (int k = 0; k < 16; k += 4) {
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w + col + k));
        const float wk[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) e[k + j] = bf16_round(__fmul_rn(__fmul_rn(e[k + j], inv), __fadd_rn(wk[j], 1.0f)));
      }
      if (scale) {
        const __nv_bfloat16* sc = scale + (int64_t)bb * K + col;
        const __nv_bfloat16* sh = shift + (int64_t)bb * K + col;
#pragma unroll
        for (int k = 0; k < 16; k += 8) {
          const uint4 su = __ldg(reinterpret_cast<const uint4*>(sc + k));
          const uint4 hu = __ldg(reinterpret_cast<const uint4*>(sh + k));
          const uint32_t sw[4] = {su.x, su.y, su.z, su.w}, hw[4] = {hu.x, hu.y, hu.z, hu.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 sf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sw[j]));
            const float2 hf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hw[j]));
            float& y0 = e[k + 2 * j];
            float& y1 = e[k + 2 * j + 1];
            y0 = bf16_round(__fadd_rn(bf16_round(__fmul_rn(y0, bf16_round(__fadd_rn(sf.x, 1.0f)))), hf.x));
            y1 = bf16_round(__fadd_rn(bf16_round(__fmul_rn(y1, bf16_round(__fadd_rn(sf.y, 1.0f)))), hf.y));
          }
        }
      }
    }
    // stride 1 and stride 4 (16 consecutive columns per lane)
#pragma unroll
    for (int k = 0; k < 16; k += 4) ref_quad(e[k], e[k + 1], e[k + 2], e[k + 3]);
#pragma unroll
    for (int k = 0; k < 4; ++k) ref_quad(e[k], e[k + 4], e[k + 8], e[k + 12]);
    if (group == 16) {
      uint32_t pk[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const __nv_bfloat162 t2 = __floats2bfloat162_rn(e[2 * k], e[2 * k + 1]);
        pk[k] = *reinterpret_cast<const uint32_t*>(&t2);
        amax = fmax3(amax, fabsf(e[2 * k]), fabsf(e[2 * k + 1]));
      }
      *reinterpret_cast<uint4*>(v + col) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      *reinterpret_cast<uint4*>(v + col + 8) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      continue;
    }
    // to the strided layout: half-warp h holds the slab's 256-column block h,
    // lane r the columns r + 16 j
    {
      uint32_t pk[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const __nv_bfloat162 t2 = __floats2bfloat162_rn(e[2 * k], e[2 * k + 1]);
        pk[k] = *reinterpret_cast<const uint32_t*>(&t2);
      }
      __syncwarp();
      *reinterpret_cast<uint4*>(&tr[warp][16 * lane]) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      *reinterpret_cast<uint4*>(&tr[warp][16 * lane + 8]) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 16; ++j) e[j] = __bfloat162float(tr[warp][256 * h + r + 16 * j]);
    }
#pragma unroll
    for (int k = 0; k < 16; k += 4) ref_quad(e[k], e[k + 1], e[k + 2], e[k + 3]);  // stride 16
    if (group == 256) {
#pragma unroll
      for (int k = 0; k < 4; ++k) ref_quad(e[k], e[k + 4], e[k + 8], e[k + 12]);  // stride 64
    }
    __nv_bfloat16* vb = v + 512 * slab + 256 * h + r;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      vb[16 * j] = __float2bfloat16_rn(e[j]);
      amax = fmaxf(amax, fabsf(e[j]));
    }
  }
  // row scale: block max (NaN ignored by fmaxf, infinity clamped)
#pragma unroll
  for (int d = 16; d; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
  if (NORM) __syncthreads();  // red[] reuse after the sum of squares
  if (lane == 0) red[4 + warp] = amax;
  __syncthreads();
  const float m = fmaxf(fmaxf(red[4], red[5]), fmaxf(red[6], red[7]));
  const float sc = fmaxf(__fdiv_rn(fminf(m, kBf16MaxFinite), 7.0f), 1e-10f);
  if (tid == 0) s[row] = sc;
  const float inverse = __fdiv_rn(1.0f, sc);
  for (int c = 16 * tid; c < K; c += 16 * kRefFastThreads) {
    const uint4 a = *reinterpret_cast<const uint4*>(v + c);
    const uint4 b = *reinterpret_cast<const uint4*>(v + c + 8);
    const uint32_t ws[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float cd[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[k]));
      // + 0: a code of -0 (rint of a small negative value) becomes +0, the
      // e4m3 container's zero byte
      cd[2 * k] = __fadd_rn(fminf(fmaxf(rintf(__fmul_rn(f.x, inverse)), -8.0f), 7.0f), 0.0f);
      cd[2 * k + 1] = __fadd_rn(fminf(fmaxf(rintf(__fmul_rn(f.y, inverse)), -8.0f), 7.0f), 0.0f);
    }
    if (BYTES) {
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint16_t lo, hi;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(cd[4 * k + 1]), "f"(cd[4 * k]));
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(cd[4 * k + 3]), "f"(cd[4 * k + 2]));
        o[k] = (uint32_t)lo | ((uint32_t)hi << 16);
      }
      *reinterpret_cast<uint4*>(q + (int64_t)row * K + c) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
      uint32_t o[2] = {0u, 0u};
#pragma unroll
      for (int k = 0; k < 16; ++k) o[k >> 3] |= ((uint32_t)(int)cd[k] & 0xFu) << (4 * (k & 7));
      *reinterpret_cast<uint2*>(q + (int64_t)row * (K / 2) + c / 2) = make_uint2(o[0], o[1]);
    }
  }
}

// k2_dequant8 of the reference contract: out = bf16(fp32(fp32(float(a) *
// xs[r]) * ws[c or 0]) + bias[c]) for int32 a [m, n]; ns = 1 (one weight
// scale) or n (per channel); bias bf16 [n] or null.
__global__ void ref_dequant8_kernel(const int32_t* __restrict__ a, const float* __restrict__ xs,
                                    const float* __restrict__ ws, const __nv_bfloat16* __restrict__ bias,
                                    __nv_bfloat16* __restrict__ out, int64_t m, int n, int ns) {
  const int64_t total = m * n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n;
    const int c = (int)(i - r * n);
    float p = __fmul_rn(__fmul_rn(__int2float_rn(a[i]), xs[r]), ws[ns == 1 ? 0 : c]);
    if (bias) p = __fadd_rn(p, __bfloat162float(bias[c]));
    out[i] = __float2bfloat16_rn(p);
  }
}

// k2_fp8 of the reference contract, one scale s[0]:
//   quant:   y = fp8(x / s) (round to nearest, saturating to the largest finite);
//   dequant: y = T(fp8 * s).
// Element types: 0 fp32, 1 fp16, 2 bf16, 5 e4m3, 6 e5m2.
__device__ __forceinline__ float ref_load(const void* p, int64_t i, int t) {
  if (t == 0) return static_cast<const float*>(p)[i];
  if (t == 1) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ void ref_store(void* p, int64_t i, int t, float v) {
  if (t == 0) static_cast<float*>(p)[i] = v;
  else if (t == 1) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}
__device__ __forceinline__ uint8_t ref_to_fp8(float v, int f) {
  uint16_t r;  // the pair form: the second source lands in the low byte
  if (f == 5)
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(v), "f"(0.0f));
  else
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %2, %1;" : "=h"(r) : "f"(v), "f"(0.0f));
  return (uint8_t)(r & 0xFF);
}
__device__ __forceinline__ float ref_from_fp8(uint8_t b, int f) {
  uint32_t h2;
  const uint16_t in = b;
  if (f == 5)
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(in));
  else
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h2) : "h"(in));
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFF)));
}
__global__ void ref_fp8_kernel(const void* __restrict__ x, void* __restrict__ y, const float* __restrict__ s,
                               int64_t n, int src, int dst, int quant) {
  const float sc = s[0];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if (quant) {
      static_cast<uint8_t*>(y)[i] = ref_to_fp8(__fdiv_rn(ref_load(x, i, src), sc), dst);
    } else {
      ref_store(y, i, dst, __fmul_rn(ref_from_fp8(static_cast<const uint8_t*>(x)[i], src), sc));
    }
  }
}

}  // namespace k2b
