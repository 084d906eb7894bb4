// elementwise.cuh -- the reference's small bf16 kernels that sit beside the
// hot path: the activation / gated-residual elementwise op and the
// standalone RoPE (kernels/native_dispatch.cu:63-77, k2_elementwise and
// k2_rope).  HBM-bound and simple; they are here so the reference's
// composed (non-fused) routes resolve to B200 code as well.
#pragma once
#include "k2b_common.cuh"

namespace k2b {

// Packed INT4 codes (two per byte, even column in the low nibble, two's
// complement) -> one e4m3 byte per code, the GEMMs' byte-A container.  n16
// chunks of 16 packed bytes (32 codes); each thread turns one chunk into 32
// contiguous output bytes, so loads and stores are coalesced.
__global__ void expand_e4m3_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, int64_t n16) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    uint4 lo, hi;
    unpack_chunk(__ldg(in + i), lo, hi);
    out[2 * i] = lo;
    out[2 * i + 1] = hi;
  }
}

// mode 0: z = bf16(silu(a)), mode 1: z = bf16(sigmoid(a)); y = b ? bf16(z*b) : z.
// mode 2: y = bf16(r + bf16(b * a[i % width]))  (gated residual, gate row a).
__global__ void elementwise_kernel(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,
                                   const __nv_bfloat16* __restrict__ r, __nv_bfloat16* __restrict__ y, int64_t n,
                                   int mode, int width) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (mode == 2) {
      const float z = bf16_round(__fmul_rn(__bfloat162float(b[i]), __bfloat162float(a[i % width])));
      y[i] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(r[i]), z));
      continue;
    }
    const float v = __bfloat162float(a[i]);
    const float z = bf16_round(mode == 0 ? silu_contract(v) : sigmoid_contract(v));
    y[i] = __float2bfloat16_rn(b ? __fmul_rn(z, __bfloat162float(b[i])) : z);
  }
}

// Adjacent-pair RoPE on [batch, heads, length, dim] (contiguous) q and k:
// o0 = bf16(fma(f0, a, f1*b)), o1 = bf16(fma(f2, a, f3*b)) with the 2x2
// rotation of (token, pair) from f fp32 [fb, length, dim/2, 2, 2]
// (fb = 1: shared by every batch row).
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                            const float* __restrict__ f, __nv_bfloat16* __restrict__ qo, __nv_bfloat16* __restrict__ ko,
                            int batch, int length, int qh, int kh, int dim, int fb) {
  const int64_t rows = (int64_t)batch * length * (qh + kh);
  const int half = dim / 2;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int h = (int)(row % (qh + kh));
    const int token = (int)((row / (qh + kh)) % length);
    const int bi = (int)(row / ((int64_t)(qh + kh) * length));
    const bool isq = h < qh;
    const __nv_bfloat16* src = isq ? q : k;
    __nv_bfloat16* dst = isq ? qo : ko;
    const int heads = isq ? qh : kh, head = isq ? h : h - qh;
    const int64_t base = (((int64_t)bi * heads + head) * length + token) * dim;
    const float* rot0 = f + ((int64_t)(fb == 1 ? 0 : bi) * length + token) * half * 4;
    for (int p = threadIdx.x; p < half; p += blockDim.x) {
      const float a = __bfloat162float(src[base + 2 * p]), v = __bfloat162float(src[base + 2 * p + 1]);
      const float4 rot = *reinterpret_cast<const float4*>(rot0 + 4 * p);
      dst[base + 2 * p] = __float2bfloat16_rn(__fmaf_rn(rot.x, a, __fmul_rn(rot.y, v)));
      dst[base + 2 * p + 1] = __float2bfloat16_rn(__fmaf_rn(rot.z, a, __fmul_rn(rot.w, v)));
    }
  }
}

// Gated residual of a reduced fp32 projection (the tensor-parallel tail of
// the out- and down-projections, the same rounding as the GEMM's
// SEG_RESIDUAL epilogue): out = bf16(r + bf16(bf16(p) * gate[latent])),
// latent = (base_row + row) / length, with p = ((s_0 + s_1) + s_2) + ... the
// fp32 sum of `nslots` partial slots slot_stride floats apart (1: p itself).
// 8 columns per thread, n % 8 == 0.
__global__ void gated_add_kernel(const float* __restrict__ p, int nslots, int64_t slot_stride,
                                 const __nv_bfloat16* __restrict__ gate, const __nv_bfloat16* __restrict__ r,
                                 __nv_bfloat16* __restrict__ out, int base_row, int rows, int n, int length) {
  const int per_row = n / 8;
  const int64_t total = (int64_t)rows * per_row;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int row = (int)(i / per_row), c = (int)(i % per_row) * 8;
    const int64_t off = (int64_t)row * n + c;
    float4 p0 = __ldg(reinterpret_cast<const float4*>(p + off));
    float4 p1 = __ldg(reinterpret_cast<const float4*>(p + off + 4));
    for (int sl = 1; sl < nslots; ++sl) {
      const float4 q0 = __ldg(reinterpret_cast<const float4*>(p + sl * slot_stride + off));
      const float4 q1 = __ldg(reinterpret_cast<const float4*>(p + sl * slot_stride + off + 4));
      p0 = make_float4(__fadd_rn(p0.x, q0.x), __fadd_rn(p0.y, q0.y), __fadd_rn(p0.z, q0.z), __fadd_rn(p0.w, q0.w));
      p1 = make_float4(__fadd_rn(p1.x, q1.x), __fadd_rn(p1.y, q1.y), __fadd_rn(p1.z, q1.z), __fadd_rn(p1.w, q1.w));
    }
    const uint4 g4 = __ldg(reinterpret_cast<const uint4*>(gate + (int64_t)((base_row + row) / length) * n + c));
    const uint4 r4 = __ldg(reinterpret_cast<const uint4*>(r + off));
    const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g4);
    const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&r4);
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 gf = __bfloat1622float2(g2[j]), rf = __bfloat1622float2(r2[j]);
      const float x0 = bf16_round(__fmul_rn(bf16_round(pv[2 * j]), gf.x));
      const float x1 = bf16_round(__fmul_rn(bf16_round(pv[2 * j + 1]), gf.y));
      w[j] = pack_bf16x2(__fadd_rn(rf.x, x0), __fadd_rn(rf.y, x1));
    }
    *reinterpret_cast<uint4*>(out + off) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace k2b
