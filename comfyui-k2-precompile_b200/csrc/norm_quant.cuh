// norm_quant.cuh -- fused RMSNorm -> adaLN modulation -> H128 rotation ->
// group-128 INT4 pack, and its rotation-only twin (rotate_quant).
//
// Replaces kernels/norm_quant.cu:11-67 (norm_mod_quant) of the reference.
// Layout: one CTA of 128 threads per row.  Thread t loads columns
// 512*i + 4t .. +3 for every 512-column slab i (8-byte loads, 1 KB per warp
// instruction), which is exactly the lane partition of the reference's
// sum-of-squares (kernels/norm_quant.cu:20-31), so the fp32 reduction order
// is reproduced without any reshuffle.  In slab i, warp w holds the 128-column
// quantisation group 4i + w (4 consecutive columns per lane): the Hadamard
// stages h = 1, 2 run in registers and h = 4..64 as lane-xor shuffles.
#pragma once
#include "k2b_common.cuh"

namespace k2b {

template <int SLABS, bool NORM>
__global__ void __launch_bounds__(128) norm_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                         const float* __restrict__ w,
                                                         const __nv_bfloat16* __restrict__ scale,
                                                         const __nv_bfloat16* __restrict__ shift,
                                                         uint8_t* __restrict__ q, __half* __restrict__ s,
                                                         int length, int cut, int batch, float eps) {
  constexpr int K = SLABS * 512;
  constexpr int G = K / 128;
  const int row = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const __nv_bfloat16* xr = x + (int64_t)row * K;

  uint2 raw[SLABS];
#pragma unroll
  for (int i = 0; i < SLABS; ++i) raw[i] = __ldg(reinterpret_cast<const uint2*>(xr + 512 * i + 4 * t));

  float inv = 1.0f;
  int b = 0;
  if constexpr (NORM) {
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < SLABS; ++i) {
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float2 f = __bfloat1622float2(h2[j]);
        sum = __fmaf_rn(f.x, f.x, sum);
        sum = __fmaf_rn(f.y, f.y, sum);
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) sum = __fadd_rn(sum, __shfl_down_sync(0xffffffffu, sum, off));
    __shared__ float warp_sums[4];
    if (lane == 0) warp_sums[warp] = sum;
    __syncthreads();
    const float total = __fadd_rn(__fadd_rn(warp_sums[2], warp_sums[0]), __fadd_rn(warp_sums[3], warp_sums[1]));
    inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)K), eps));
    b = row / length;
    if (cut >= 0 && row % length >= cut) b += batch;
  }

  uint8_t* qr = q + (int64_t)row * (K / 2);
  __half* sr = s + (int64_t)row * G;
#pragma unroll
  for (int i = 0; i < SLABS; ++i) {
    const int col = 512 * i + 4 * t;
    float v[4];
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
    {
      float2 a = __bfloat1622float2(h2[0]), c = __bfloat1622float2(h2[1]);
      v[0] = a.x; v[1] = a.y; v[2] = c.x; v[3] = c.y;
    }
    if constexpr (NORM) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w + col));
      const uint2 sc = __ldg(reinterpret_cast<const uint2*>(scale + (int64_t)b * K + col));
      const uint2 sh = __ldg(reinterpret_cast<const uint2*>(shift + (int64_t)b * K + col));
      const __nv_bfloat162* sc2 = reinterpret_cast<const __nv_bfloat162*>(&sc);
      const __nv_bfloat162* sh2 = reinterpret_cast<const __nv_bfloat162*>(&sh);
      const float ww[4] = {wv.x, wv.y, wv.z, wv.w};
      float scf[4], shf[4];
      {
        float2 a = __bfloat1622float2(sc2[0]), c = __bfloat1622float2(sc2[1]);
        scf[0] = a.x; scf[1] = a.y; scf[2] = c.x; scf[3] = c.y;
        a = __bfloat1622float2(sh2[0]); c = __bfloat1622float2(sh2[1]);
        shf[0] = a.x; shf[1] = a.y; shf[2] = c.x; shf[3] = c.y;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float y = bf16_round(__fmul_rn(__fmul_rn(v[j], inv), __fadd_rn(ww[j], 1.0f)));
        const float f = bf16_round(__fadd_rn(scf[j], 1.0f));
        y = bf16_round(__fmul_rn(y, f));
        v[j] = bf16_round(__fadd_rn(y, shf[j]));
      }
    }
    // Sylvester H128, stages h = 1, 2 in registers ...
    {
      const float a0 = __fadd_rn(v[0], v[1]), a1 = __fsub_rn(v[0], v[1]);
      const float a2 = __fadd_rn(v[2], v[3]), a3 = __fsub_rn(v[2], v[3]);
      v[0] = __fadd_rn(a0, a2); v[2] = __fsub_rn(a0, a2);
      v[1] = __fadd_rn(a1, a3); v[3] = __fsub_rn(a1, a3);
    }
    // ... h = 4 .. 64 across lanes (partner = lane ^ h/4).
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const bool upper = (lane & m) != 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float o = __shfl_xor_sync(0xffffffffu, v[j], m);
        v[j] = upper ? __fsub_rn(o, v[j]) : __fadd_rn(v[j], o);
      }
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = __fmul_rn(v[j], kHadamardScale);
      amax = fmaxf(amax, fabsf(v[j]));
    }
#pragma unroll
    for (int m = 16; m; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    const __half hs = group_scale(amax);
    const float sd = __half2float(hs);
    const int gidx = 4 * i + warp;
    if (lane == 0) sr[gidx] = hs;
    uint32_t packed = 0;
    if (sd > 0.0f) {
      const float rcp = __frcp_rn(sd);
#pragma unroll
      for (int j = 0; j < 4; ++j) packed |= (uint32_t)(quant_code(v[j], sd, rcp) & 0xF) << (4 * j);
    }
    reinterpret_cast<uint16_t*>(qr + gidx * 64)[lane] = (uint16_t)packed;
  }
}

}  // namespace k2b
