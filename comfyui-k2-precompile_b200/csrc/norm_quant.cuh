// norm_quant.cuh -- fused RMSNorm -> adaLN modulation -> H128 rotation ->
// group-128 INT4 pack, and its rotation-only twin (rotate_quant).
//
// Replaces kernels/norm_quant.cu:11-67 (norm_mod_quant) of the reference.
//
// HBM traffic per row of K bf16: 2K bytes read, K/2 code bytes + K/64 scale
// bytes written.  Organisation:
//
// * A CTA (4 warps) owns a tile of kNqRows rows and loops over tiles
//   (persistent grid, one wave of resident CTAs).
// * Stage A (NORM only), one warp per row: lane l loads columns 512i + 16l
//   .. +15 of every 512-column slab i.  Those are the columns of the
//   reference's sum-of-squares lanes 4l..4l+3 (kernels/norm_quant.cu:20-26:
//   lane r owns 512i + 4r .. +3), so each lane runs those four fmaf chains in
//   the reference's order, and the reference's shfl_down tree (offsets 16, 8,
//   4, 2, 1, then (w2 + w0) + (w3 + w1)) is replayed as width-8 shuffles
//   plus in-lane adds: the fp32 sum is the reference's bit for bit.
// * Stage B, column-stationary: warp w takes slabs w, w+4, ...; lane l keeps
//   the modulation constants of its 16 columns in registers for every row of
//   the tile, re-reads x (an L2 hit; two row buffers alternate), modulates,
//   and runs the Hadamard:
//     layout A (lane owns 16 consecutive columns, pairs (e, e+1)): stages
//       h = 2, 4, 8 on packed f32x2;
//     a shared-memory transpose to layout B (lane v of a group owns
//       e = 2v + b0 + 16m, m = 0..7, pairs (e, e+1)): stage h = 1 (inside
//       each pair) and h = 16, 32, 64 on packed f32x2.
//   The 8 lanes of a group then reduce max|u| with 3 xor-shuffles, quantise
//   (one fma per element), and stage the 64 code bytes in shared memory so
//   every warp writes its 256 code bytes with one 8-byte store per lane.
#pragma once
#include "k2b_common.cuh"

namespace k2b {

constexpr int kNqThreads = 128;  // 4 warps
constexpr int kNqRows = 8;       // rows per tile

__device__ __forceinline__ float2 bf2_unpack(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __nv_bfloat162 bf2_from(uint32_t w) { return *reinterpret_cast<__nv_bfloat162*>(&w); }
// (a + b, a - b) for packed pairs; fma(b, -1, a) is a - b rounded once.
__device__ __forceinline__ void bfly2(float2& a, float2& b) {
  const float2 s = __fadd2_rn(a, b);
  b = __ffma2_rn(b, make_float2(-1.0f, -1.0f), a);
  a = s;
}
// Per-warp transpose buffer: group g (128 fp32) at 144*g floats, logical
// 16-byte chunk c at chunk c + c/8.  The layout-A stores (lane u of a group
// writes chunks 4u..4u+3, 8 lanes per wavefront) land on chunks
// 4u + u/2 + k: eight distinct bank quads; the layout-B 8-byte loads (lane v
// reads pair v of chunk row m, 16 lanes per wavefront) cover 16 consecutive
// banks per group and groups g, g+1 sit 16 banks apart.  Every address is a
// per-lane base plus a compile-time offset.
constexpr int kNqGroupFloats = 144;
__device__ __forceinline__ constexpr int nq_pad_chunk(int c) { return c + (c >> 3); }

// NORM: RMS-normalise (y = bf16(x*inv*(w+1))); MOD: then apply the adaLN
// scale/shift; QUANT: then rotate + INT4 (else store the bf16 row to q).
//   <1,1,1> norm_quant   <0,0,1> rotate_quant   <1,1,0> norm_mod   <1,0,0> norm
// BYTES (with QUANT): the codes are stored as e4m3 bytes [rows, K], the
// container the block loop hands to its GEMMs, instead of packed nibbles.
template <bool NORM, bool MOD, bool QUANT, bool BYTES = false>
__global__ void __launch_bounds__(kNqThreads, 4) norm_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                                const float* __restrict__ w,
                                                                const __nv_bfloat16* __restrict__ scale,
                                                                const __nv_bfloat16* __restrict__ shift,
                                                                uint8_t* __restrict__ q, __half* __restrict__ s,
                                                                int rows, int K, int length, int cut, int batch,
                                                                float eps, int base_row) {
  __shared__ float s_inv[kNqRows];
  __shared__ int s_lat[kNqRows];  // modulation row (latent) of each tile row
  __shared__ __align__(16) float s_tr[4][4 * kNqGroupFloats];
  // code staging per warp: packed nibbles (64 bytes per group, groups
  // 16 bytes apart in pairs) or, BYTES, e4m3 bytes (128 per group at 144 g)
  __shared__ __align__(16) uint8_t s_codes[4][BYTES ? 4 * 144 : 320];
  __shared__ float s_rcp[1024];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 3, v = lane & 7;  // group within the slab, lane within the group
  const int slabs = K >> 9;
  const int tiles = (rows + kNqRows - 1) / kNqRows;
  float* tr = s_tr[warp] + g * kNqGroupFloats;
  float* tra = tr + 4 * nq_pad_chunk(4 * v);                   // layout-A store base
  const float* trb = tr + 4 * (v >> 1) + 2 * (v & 1);          // layout-B load base
  uint8_t* cb = s_codes[warp];
  const int cpos = 64 * g + 16 * (g >> 1);  // this group's 64 code bytes in cb
  quant_table_init(s_rcp, threadIdx.x, kNqThreads);
  __syncthreads();

  for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int row0 = tile * kNqRows;
    const int nrows = min(kNqRows, rows - row0);

    if constexpr (NORM) {
      // ---- stage A: inverse RMS of each row, reference reduction order
      for (int r = warp; r < nrows; r += 4) {
        const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)(row0 + r) * K) + 2 * lane;
        float2 s01 = make_float2(0.0f, 0.0f), s23 = make_float2(0.0f, 0.0f);
        // 12 loads in flight per lane (unroll 4: 229 us, 6: 226 us at 33792 x 6144)
#pragma unroll 6
        for (int i = 0; i < slabs; ++i) {
          const uint4 a = __ldg(xr + 64 * i), b = __ldg(xr + 64 * i + 1);
          // chains: lane 4l+c <- words 2c, 2c+1 of (a, b), low half first.
          // fma.rn.f32.bf16 widens its bf16 operands exactly, so each step is
          // fmaf(x, x, sum) of the reference.
          const uint32_t ws[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float& acc = c == 0 ? s01.x : c == 1 ? s01.y : c == 2 ? s23.x : s23.y;
            asm("{.reg .b16 l0, h0, l1, h1;\n\t"
                "mov.b32 {l0, h0}, %1;\n\t"
                "mov.b32 {l1, h1}, %2;\n\t"
                "fma.rn.f32.bf16 %0, l0, l0, %0;\n\t"
                "fma.rn.f32.bf16 %0, h0, h0, %0;\n\t"
                "fma.rn.f32.bf16 %0, l1, l1, %0;\n\t"
                "fma.rn.f32.bf16 %0, h1, h1, %0;}"
                : "+f"(acc)
                : "r"(ws[2 * c]), "r"(ws[2 * c + 1]));
          }
        }
        float c0 = s01.x, c1 = s01.y, c2 = s23.x, c3 = s23.y;
        // reference offsets 16, 8, 4 = lanes +4, +2, +1 within 8-lane segments
#pragma unroll
        for (int d = 4; d; d >>= 1) {
          c0 = __fadd_rn(c0, __shfl_down_sync(0xffffffffu, c0, d, 8));
          c1 = __fadd_rn(c1, __shfl_down_sync(0xffffffffu, c1, d, 8));
          c2 = __fadd_rn(c2, __shfl_down_sync(0xffffffffu, c2, d, 8));
          c3 = __fadd_rn(c3, __shfl_down_sync(0xffffffffu, c3, d, 8));
        }
        c0 = __fadd_rn(c0, c2);  // offset 2
        c1 = __fadd_rn(c1, c3);
        c0 = __fadd_rn(c0, c1);  // offset 1
        const float w0 = __shfl_sync(0xffffffffu, c0, 0), w1 = __shfl_sync(0xffffffffu, c0, 8);
        const float w2 = __shfl_sync(0xffffffffu, c0, 16), w3 = __shfl_sync(0xffffffffu, c0, 24);
        const float total = __fadd_rn(__fadd_rn(w2, w0), __fadd_rn(w3, w1));
        if (lane == 0) {
          s_inv[r] = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)K), eps));
          if constexpr (MOD) {
            const int row = base_row + row0 + r;  // row index within the latent stream
            int bb = row / length;
            if (cut >= 0 && row % length >= cut) bb += batch;
            s_lat[r] = bb;
          }
        }
      }
      __syncthreads();
    }

    // ---- stage B: modulation + rotation + quantisation, column-stationary
    for (int i = warp; i < slabs; i += 4) {
      const int col = 512 * i + 16 * lane;
      float2 w1[8];
      uint32_t fm[8], sh[8];
      int bcur = -1;
      if constexpr (NORM) {  // (w + 1) of this lane's 16 columns
        const float4* wp = reinterpret_cast<const float4*>(w + col);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 t = __ldg(wp + k);
          w1[2 * k] = __fadd2_rn(make_float2(t.x, t.y), make_float2(1.0f, 1.0f));
          w1[2 * k + 1] = __fadd2_rn(make_float2(t.z, t.w), make_float2(1.0f, 1.0f));
        }
      }
      const int kv = K >> 3;  // uint4 per row
      const uint4* xc = reinterpret_cast<const uint4*>(x + (int64_t)row0 * K + col);
      // one row: x words (xa, xb) -> codes at qp, scale at sp
      auto row_body = [&](const uint4 xa, const uint4 xb, int r, uint8_t* qp, __half* sp) {
        uint32_t vw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        if constexpr (MOD) {
          const int bb = s_lat[r];
          if (bb != bcur) {  // warp-uniform: every lane works on the same row
            bcur = bb;
            const uint4* cp = reinterpret_cast<const uint4*>(scale + (int64_t)bb * K + col);
            const uint4* hp = reinterpret_cast<const uint4*>(shift + (int64_t)bb * K + col);
            const uint4 s0 = __ldg(cp), s1 = __ldg(cp + 1), h0 = __ldg(hp), h1 = __ldg(hp + 1);
            const uint32_t sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
            const uint32_t hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
            const __nv_bfloat162 one = __floats2bfloat162_rn(1.0f, 1.0f);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              fm[k] = bf2_bits(__hadd2_rn(bf2_from(sv[k]), one));  // bf16(scale + 1)
              sh[k] = hv[k];
            }
          }
        }
        if constexpr (NORM) {
          const float inv = s_inv[r];
          const float2 inv2 = make_float2(inv, inv);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            // y = bf16((x*inv)*(w+1)); y = bf16(y*f); v = bf16(y + shift).  The last
            // two are bf16x2 ops: a bf16-by-bf16 product or sum rounded once to
            // bf16 equals its fp32 result rounded to bf16 (fp32 carries more than
            // 2*8+2 bits), which is the reference's fp32-then-bf16 rounding.  The
            // .rn forms keep the compiler from contracting them into one fma.
            const float2 t = __fmul2_rn(__fmul2_rn(bf2_unpack(vw[k]), inv2), w1[k]);
            if constexpr (MOD) {
              const __nv_bfloat162 y = __hmul2_rn(__float22bfloat162_rn(t), bf2_from(fm[k]));
              vw[k] = bf2_bits(__hadd2_rn(y, bf2_from(sh[k])));
            } else {
              vw[k] = bf2_bits(__float22bfloat162_rn(t));
            }
          }
        }
        if constexpr (!QUANT) {  // bf16 row out (q holds the bf16 output)
          uint4* yo = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(q) + (int64_t)(row0 + r) * K + col);
          yo[0] = make_uint4(vw[0], vw[1], vw[2], vw[3]);
          yo[1] = make_uint4(vw[4], vw[5], vw[6], vw[7]);
        } else {
          // layout A: p[k] = (x[2k], x[2k+1]) of this lane's 16 columns
          float2 p[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) p[k] = bf2_unpack(vw[k]);
#pragma unroll
          for (int lk = 0; lk < 3; ++lk) {  // h = 2, 4, 8
#pragma unroll
            for (int k = 0; k < 8; ++k)
              if (!(k & (1 << lk))) bfly2(p[k], p[k | (1 << lk)]);
          }
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 4; ++k)
            *reinterpret_cast<float4*>(tra + 4 * k) =
                make_float4(p[2 * k].x, p[2 * k].y, p[2 * k + 1].x, p[2 * k + 1].y);
          __syncwarp();
          // layout B: o[m] = (x[e], x[e+1]), e = 2v + 16m
          float2 o[8];
#pragma unroll
          for (int m = 0; m < 8; ++m)
            o[m] = *reinterpret_cast<const float2*>(trb + 4 * (4 * m + (m >> 1)));
#pragma unroll
          for (int m = 0; m < 8; ++m) {  // h = 1
            const float a = o[m].x, b = o[m].y;
            o[m] = make_float2(__fadd_rn(a, b), __fsub_rn(a, b));
          }
#pragma unroll
          for (int lm = 0; lm < 3; ++lm) {  // h = 16, 32, 64
#pragma unroll
            for (int m = 0; m < 8; ++m)
              if (!(m & (1 << lm))) bfly2(o[m], o[m | (1 << lm)]);
          }
          float amax = 0.0f;
#pragma unroll
          for (int m = 0; m < 8; ++m) amax = fmax3(amax, fabsf(o[m].x), fabsf(o[m].y));
#pragma unroll
          for (int d = 1; d < 8; d <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
          const QuantGroup qg = quant_scale(amax);
          const float c = quant_c_table(qg.sd, s_rcp);
          const bool clamp = __any_sync(0xffffffffu, qg.clamp);
          const float2 c2 = make_float2(c, c), mg = make_float2(kRoundMagic8, kRoundMagic8);
          if constexpr (BYTES) {
            // code = r - (1.5*2^23 + 8) exactly, then two codes per e4m3x2
            // conversion (-8..7 are exact e4m3 values; the second source is
            // the low byte), staged in column order; this lane's 16 columns
            // then leave as one 16-byte store
            uint8_t* cb8 = cb + 144 * g;
#pragma unroll
            for (int m = 0; m < 8; ++m) {
              float2 r2 = __ffma2_rn(o[m], c2, mg);
              if (clamp) {
                r2.x = fminf(fmaxf(r2.x, kRoundMagic), kRoundMagic + 15.0f);
                r2.y = fminf(fmaxf(r2.y, kRoundMagic), kRoundMagic + 15.0f);
              }
              const float2 cf = __fadd2_rn(r2, make_float2(-kRoundMagic8, -kRoundMagic8));
              uint16_t e;
              asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(e) : "f"(cf.y), "f"(cf.x));
              *reinterpret_cast<uint16_t*>(cb8 + 2 * v + 16 * m) = e;
            }
            __syncwarp();
            *reinterpret_cast<uint4*>(qp) = *reinterpret_cast<const uint4*>(cb8 + 16 * v);
          } else {
#pragma unroll
            for (int m = 0; m < 8; ++m) {
              float2 r2 = __ffma2_rn(o[m], c2, mg);
              if (clamp) {
                r2.x = fminf(fmaxf(r2.x, kRoundMagic), kRoundMagic + 15.0f);
                r2.y = fminf(fmaxf(r2.y, kRoundMagic), kRoundMagic + 15.0f);
              }
              // low byte = offset-8 nibbles (even element low); bits 4..21 of
              // each word are zero, so the shifted add carries nothing into it
              cb[cpos + v + 8 * m] = (uint8_t)((__float_as_uint(r2.y) << 4) + __float_as_uint(r2.x));
            }
            __syncwarp();
            uint2 packed = *reinterpret_cast<const uint2*>(cb + cpos + 8 * v);
            packed.x ^= 0x88888888u;  // offset-8 -> two's-complement nibbles
            packed.y ^= 0x88888888u;
            *reinterpret_cast<uint2*>(qp) = packed;
          }
          if (v == 0) *sp = qg.scale;
        }
      };
      // Two x buffers alternate (row r in A, r+1 in B); each is refilled as
      // soon as its row is consumed, a row ahead, with no register copies.
      uint4 a0 = __ldg(xc), a1 = __ldg(xc + 1), b0 = a0, b1 = a1;
      if (nrows > 1) {
        b0 = __ldg(xc + kv);
        b1 = __ldg(xc + kv + 1);
      }
      // code bytes per row: K/2 packed, or K e4m3 bytes
      const int qrow = BYTES ? K : (K >> 1);
      uint8_t* qp = BYTES ? q + (int64_t)row0 * K + col : q + (int64_t)row0 * (K >> 1) + 256 * i + 8 * lane;
      __half* sp = s + (int64_t)row0 * (K >> 7) + 4 * i + g;
      const uint4* xn = xc + 2 * kv;
      for (int r = 0; r < nrows; r += 2, qp += 2 * qrow, sp += 2 * (K >> 7), xn += 2 * kv) {
        row_body(a0, a1, r, qp, sp);
        if (r + 2 < nrows) {
          a0 = __ldg(xn);
          a1 = __ldg(xn + 1);
        }
        if (r + 1 < nrows) {
          row_body(b0, b1, r + 1, qp + qrow, sp + (K >> 7));
          if (r + 3 < nrows) {
            b0 = __ldg(xn + kv);
            b1 = __ldg(xn + kv + 1);
          }
        }
      }
    }
    __syncthreads();  // s_inv is rewritten by the next tile's stage A
  }
}

}  // namespace k2b
