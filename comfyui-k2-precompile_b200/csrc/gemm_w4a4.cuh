// gemm_w4a4.cuh -- group-scaled W4A4 GEMM on tcgen05 kind::i8 with fused
// epilogues (dequant, per-head QK RMSNorm + RoPE, sigmoid gate, gated
// residual, SwiGLU + INT4 requant of the down-projection input).
//
// Replaces the reference's SM89 mma.sync s4 kernels: qkv_kernel / swiglu_kernel
// / residual_norm_kernel (kernels/joint_projection.cu:68-202), the CUTLASS EVT
// ResidualGemm (kernels/int4_epilogue.cu:18-66) and QKGemm + NormRopeStore
// (kernels/qk_norm_rope.cu:19-133).
//
// Tile: 128 rows (M) x 256 columns (N) per CTA, K consumed one 128-wide
// quantisation group per pipeline stage.  Roles (384 threads):
//   warp 0      TMA producer: packed A group tile (128 x 64 B), prepared W
//               group tile (256 x 128 B, 128B-swizzled), W group scales (1 KB)
//   warp 1      TMEM allocator + single-thread MMA issuer (4 x K=32 MMAs per group)
//   warps 2-3   A unpackers: s4 -> s8 (x16) into the 128B-swizzled UMMA layout
//   warps 4-11  epilogue: TMEM lane quadrant = warp % 4, column half = (warp-4)/4
// TMEM: 2 x 256 int32 columns, one per group in flight (ping-pong), so the MMA
// of group g+1 overlaps the dequant of group g.  The fp32 group sum lives in
// the epilogue registers (128 per thread).
//
// Dequant contract (oracle: k2o_gemm_w4a4):
//   p = 0;  for g:  u = fp32(acc_g * sA[r,g]);  p = fmaf(u, sW[c,g], p)
// The s8 operands carry 16x the INT4 codes (the nibble is kept in the high
// half of each byte), so the TMEM accumulator is 256*acc_g (|.| <= 2^21).
// It is turned into fp32 with the exponent-bias trick (bits + 0x4B400000 ->
// 12582912 + x exactly) and the bias is removed inside the first fma:
//   u = fma(12582912 + x, sA/256, -12582912*sA/256) = fp32(acc_g * sA)
// (both sA/256 and 12582912*sA/256 are exact for an fp16-valued sA).
#pragma once
#include "k2b_common.cuh"

namespace k2b {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BN = 256;
constexpr int GEMM_STAGES = 3;   // prepared W + unpacked A
constexpr int GEMM_PSTAGES = 4;  // packed A and W scales
constexpr int GEMM_THREADS = 384;

constexpr int GEMM_W_BYTES = GEMM_BN * 128;       // 32 KB
constexpr int GEMM_UA_BYTES = GEMM_BM * 128;      // 16 KB
constexpr int GEMM_PA_BYTES = GEMM_BM * 64;       // 8 KB
constexpr int GEMM_SC_BYTES = GEMM_BN * 4;        // 1 KB
constexpr int GEMM_OFF_W = 0;
constexpr int GEMM_OFF_UA = GEMM_OFF_W + GEMM_STAGES * GEMM_W_BYTES;
constexpr int GEMM_OFF_PA = GEMM_OFF_UA + GEMM_STAGES * GEMM_UA_BYTES;
constexpr int GEMM_OFF_SC = GEMM_OFF_PA + GEMM_PSTAGES * GEMM_PA_BYTES;
constexpr int GEMM_OFF_BAR = GEMM_OFF_SC + GEMM_PSTAGES * GEMM_SC_BYTES;
constexpr int GEMM_NBARS = 3 * GEMM_STAGES + 4 * GEMM_PSTAGES + 4;
constexpr int GEMM_SMEM_BYTES = GEMM_OFF_BAR + GEMM_NBARS * 8 + 16 + 1024;  // + alignment slack
// The SwiGLU exchange buffer reuses the W stages after the main loop.
constexpr int GEMM_XCH_STRIDE = 272;  // bytes per row: 128 bf16 + 16 B pad

enum SegKind : int {
  SEG_BF16 = 0,       // bf16(p)
  SEG_QKNORM = 1,     // per-head RMSNorm + RoPE of bf16(p)
  SEG_SIGMOID = 2,    // bf16(sigmoid(bf16(p)))
  SEG_RESIDUAL = 3,   // bf16(resid + bf16(bf16(p) * gate))
  SEG_SWIGLU = 4,     // SwiGLU of (gate, up) column pairs + H128 + INT4 requant
  SEG_F32 = 5,        // p itself (tests: exact accumulators)
  SEG_SWIGLU_BF16 = 6 // SwiGLU of (gate, up) column pairs, bf16 h
};

struct GemmSegment {
  int tiles;             // N tiles of this segment (256 columns; SwiGLU: 128 output columns)
  int kind;              // SegKind
  int n;                 // columns of the segment's prepared weight(s)
  int ld;                // leading dimension (elements) of the output
  void* out;             // output base (bf16 / fp32 / packed u8)
  const float* wscale;   // prepared W scales, fp32 [G, n]
  const float* wscale2;  // SwiGLU: up-projection scales, fp32 [G, n]
  const float* normw;    // SEG_QKNORM: fp32 [128] ("w+1" form)
  float eps;             // SEG_QKNORM
  __half* out_scale;     // SEG_SWIGLU: fp16 [M, n/128]
};

struct GemmParams {
  GemmSegment seg[4];
  int nseg;
  int M, K, G;
  int length;                      // rows per latent (RoPE token, gate batch)
  const __half* sa;                // activation scales fp16 [M, G]
  const float* freqs;              // fp32 [length, 64, 2, 2]
  const __nv_bfloat16* gate;       // SEG_RESIDUAL: bf16 [batch, n]
  const __nv_bfloat16* resid;      // SEG_RESIDUAL: bf16 [M, n]
};

struct WeightMaps {
  CUtensorMap m[4];
};

__device__ __forceinline__ void unpack_chunk(uint4 v, uint4& lo, uint4& hi) {
  lo.x = (v.x << 4) & 0xF0F0F0F0u; hi.x = v.x & 0xF0F0F0F0u;
  lo.y = (v.y << 4) & 0xF0F0F0F0u; hi.y = v.y & 0xF0F0F0F0u;
  lo.z = (v.z << 4) & 0xF0F0F0F0u; hi.z = v.z & 0xF0F0F0F0u;
  lo.w = (v.w << 4) & 0xF0F0F0F0u; hi.w = v.w & 0xF0F0F0F0u;
}

__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_w4a4_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ WeightMaps wmaps,
                     const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + GEMM_OFF_BAR);
  uint64_t* full_w = bars;                          // [STAGES] TMA W landed
  uint64_t* full_ua = full_w + GEMM_STAGES;         // [STAGES] A unpacked
  uint64_t* empty_s = full_ua + GEMM_STAGES;        // [STAGES] MMAs done with W/A stage
  uint64_t* full_pa = empty_s + GEMM_STAGES;        // [PSTAGES] TMA packed A landed
  uint64_t* empty_pa = full_pa + GEMM_PSTAGES;      // [PSTAGES] unpackers done
  uint64_t* full_sc = empty_pa + GEMM_PSTAGES;      // [PSTAGES] W scales landed
  uint64_t* empty_sc = full_sc + GEMM_PSTAGES;      // [PSTAGES] epilogue done with scales
  uint64_t* tmem_full = empty_sc + GEMM_PSTAGES;    // [2]
  uint64_t* tmem_empty = tmem_full + 2;             // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + GEMM_NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * GEMM_BM;
  // Segment of this N tile.
  int seg = 0, tile = blockIdx.y;
  while (seg + 1 < p.nseg && tile >= p.seg[seg].tiles) {
    tile -= p.seg[seg].tiles;
    ++seg;
  }
  const GemmSegment& S = p.seg[seg];
  // SwiGLU tiles pair 128 gate rows (map 0) with the same 128 up rows (map 1).
  const bool pairw = (S.kind == SEG_SWIGLU || S.kind == SEG_SWIGLU_BF16);
  const int n0 = tile * (pairw ? GEMM_BN / 2 : GEMM_BN);
  const int G = p.G;

  if (threadIdx.x == 0) {
    for (int i = 0; i < GEMM_STAGES; ++i) {
      mbar_init(&full_w[i], 1);
      mbar_init(&full_ua[i], 2);
      mbar_init(&empty_s[i], 1);
    }
    for (int i = 0; i < GEMM_PSTAGES; ++i) {
      mbar_init(&full_pa[i], 1);
      mbar_init(&empty_pa[i], 2);
      mbar_init(&full_sc[i], 1);
      mbar_init(&empty_sc[i], 8);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 8);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int issued_w = 0, issued_pa = 0, issued_sc = 0, issued_mma = 0;
  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      const CUtensorMap* wmap = &wmaps.m[pairw ? 0 : seg];
      for (int g = 0; g < G; ++g) {
        const int s = g % GEMM_STAGES, ps = g % GEMM_PSTAGES;
        const uint32_t ph = (g / GEMM_STAGES) & 1, pph = (g / GEMM_PSTAGES) & 1;
        if (g >= GEMM_STAGES && !mbar_wait(&empty_s[s], ph ^ 1, abort_flag, ERR_WAIT_PRODUCER)) break;
        mbar_arrive_expect_tx(&full_w[s], GEMM_W_BYTES);
        if (pairw) {
          tma_load_2d(smem + GEMM_OFF_W + s * GEMM_W_BYTES, &wmaps.m[0], &full_w[s], g * 128, n0);
          tma_load_2d(smem + GEMM_OFF_W + s * GEMM_W_BYTES + GEMM_W_BYTES / 2, &wmaps.m[1], &full_w[s], g * 128, n0);
        } else {
          tma_load_2d(smem + GEMM_OFF_W + s * GEMM_W_BYTES, wmap, &full_w[s], g * 128, n0);
        }
        issued_w = g + 1;
        if (g >= GEMM_PSTAGES && !mbar_wait(&empty_pa[ps], pph ^ 1, abort_flag, ERR_WAIT_PRODUCER)) break;
        mbar_arrive_expect_tx(&full_pa[ps], GEMM_PA_BYTES);
        tma_load_2d(smem + GEMM_OFF_PA + ps * GEMM_PA_BYTES, &amap, &full_pa[ps], g * 64, m0);
        issued_pa = g + 1;
        if (g >= GEMM_PSTAGES && !mbar_wait(&empty_sc[ps], pph ^ 1, abort_flag, ERR_WAIT_PRODUCER)) break;
        mbar_arrive_expect_tx(&full_sc[ps], GEMM_SC_BYTES);
        if (pairw) {
          bulk_load(smem + GEMM_OFF_SC + ps * GEMM_SC_BYTES, S.wscale + (int64_t)g * S.n + n0, GEMM_SC_BYTES / 2,
                    &full_sc[ps]);
          bulk_load(smem + GEMM_OFF_SC + ps * GEMM_SC_BYTES + GEMM_SC_BYTES / 2, S.wscale2 + (int64_t)g * S.n + n0,
                    GEMM_SC_BYTES / 2, &full_sc[ps]);
        } else {
          bulk_load(smem + GEMM_OFF_SC + ps * GEMM_SC_BYTES, S.wscale + (int64_t)g * S.n + n0, GEMM_SC_BYTES,
                    &full_sc[ps]);
        }
        issued_sc = g + 1;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(2, 1, 1, 0, 0, GEMM_BM, GEMM_BN);
      for (int g = 0; g < G; ++g) {
        const int s = g % GEMM_STAGES, b = g & 1;
        const uint32_t ph = (g / GEMM_STAGES) & 1, bph = (g >> 1) & 1;
        if (!mbar_wait(&full_w[s], ph, abort_flag, ERR_WAIT_MMA)) break;
        if (!mbar_wait(&full_ua[s], ph, abort_flag, ERR_WAIT_MMA)) break;
        if (g >= 2 && !mbar_wait(&tmem_empty[b], bph ^ 1, abort_flag, ERR_WAIT_MMA)) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + GEMM_OFF_UA + s * GEMM_UA_BYTES);
        const uint32_t w_base = smem_u32(smem + GEMM_OFF_W + s * GEMM_W_BYTES);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t ad = umma_desc_sw128(a_base + 32 * k, 16, 1024);
          const uint64_t bd = umma_desc_sw128(w_base + 32 * k, 16, 1024);
          mma_i8_ss(tmem + b * GEMM_BN, ad, bd, idesc, k > 0 ? 1u : 0u);
        }
        mma_commit(&empty_s[s]);
        mma_commit(&tmem_full[b]);
        issued_mma = g + 1;
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------- A unpackers
    const int t = threadIdx.x - 64;  // 0..63
    for (int g = 0; g < G; ++g) {
      const int s = g % GEMM_STAGES, ps = g % GEMM_PSTAGES;
      const uint32_t ph = (g / GEMM_STAGES) & 1, pph = (g / GEMM_PSTAGES) & 1;
      if (!mbar_wait(&full_pa[ps], pph, abort_flag, ERR_WAIT_UNPACK)) break;
      if (g >= GEMM_STAGES && !mbar_wait(&empty_s[s], ph ^ 1, abort_flag, ERR_WAIT_UNPACK)) break;
      const uint4* src = reinterpret_cast<const uint4*>(smem + GEMM_OFF_PA + ps * GEMM_PA_BYTES);
      uint8_t* dst = smem + GEMM_OFF_UA + s * GEMM_UA_BYTES;
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int i = t + 64 * it;  // 16-byte chunk: row i/4, K columns 32*(i%4) .. +31
        const int r = i >> 2, c = i & 3;
        uint4 lo, hi;
        unpack_chunk(src[i], lo, hi);
        *reinterpret_cast<uint4*>(dst + r * 128 + (((2 * c) ^ (r & 7)) << 4)) = lo;
        *reinterpret_cast<uint4*>(dst + r * 128 + (((2 * c + 1) ^ (r & 7)) << 4)) = hi;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty_pa[ps]);
        mbar_arrive(&full_ua[s]);
      }
    }
  } else {
    // ------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;
    const int rloc = 32 * q + lane;
    const int row = m0 + rloc;
    const bool row_ok = row < p.M;
    const __half* sa_row = p.sa + (int64_t)(row_ok ? row : 0) * G;
    float acc[128];
#pragma unroll
    for (int i = 0; i < 128; ++i) acc[i] = 0.0f;
    bool ok = true;
    for (int g = 0; g < G && ok; ++g) {
      const int b = g & 1, ps = g % GEMM_PSTAGES;
      const uint32_t bph = (g >> 1) & 1, pph = (g / GEMM_PSTAGES) & 1;
      const float sa = row_ok ? __fmul_rn(__half2float(sa_row[g]), 0.00390625f) : 0.0f;
      const float sbias = __fmul_rn(sa, -12582912.0f);
      if (!mbar_wait(&full_sc[ps], pph, abort_flag, ERR_WAIT_EPILOGUE)) { ok = false; break; }
      if (!mbar_wait(&tmem_full[b], bph, abort_flag, ERR_WAIT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
      const float* scs = reinterpret_cast<const float*>(smem + GEMM_OFF_SC + ps * GEMM_SC_BYTES) + half * 128;
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + b * GEMM_BN + half * 128;
      uint32_t buf[2][16];
      tmem_ld16(taddr, buf[0]);
      tmem_wait_ld_regs(buf[0]);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c + 1 < 8) tmem_ld16(taddr + 16 * (c + 1), buf[(c + 1) & 1]);
        if (c + 1 == 8) {
          // every column of this buffer is in registers: hand it back to the MMA
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tmem_empty[b]);
        }
        const uint32_t* v = buf[c & 1];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float4 sw4 = *reinterpret_cast<const float4*>(scs + 16 * c + (i & ~3));
          const float swa = (i & 2) ? sw4.z : sw4.x, swb = (i & 2) ? sw4.w : sw4.y;
          const float2 fb = make_float2(__int_as_float((int)(v[i] + 0x4B400000u)),
                                        __int_as_float((int)(v[i + 1] + 0x4B400000u)));
          const float2 u = ffma2(fb, make_float2(sa, sa), make_float2(sbias, sbias));
          const float2 r = ffma2(u, make_float2(swa, swb), make_float2(acc[16 * c + i], acc[16 * c + i + 1]));
          acc[16 * c + i] = r.x;
          acc[16 * c + i + 1] = r.y;
        }
        if (c + 1 < 8) tmem_wait_ld_regs(buf[(c + 1) & 1]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_sc[ps]);
    }

    // ---------------------------------------------------- final epilogue
    // CTA-uniform decision: every epilogue warp reaches this barrier, then all
    // of them see the same abort flag (the SwiGLU path has a second barrier).
    asm volatile("bar.sync 2, 256;" ::: "memory");
    ok = ok && (*abort_flag == 0);
    if (ok) {
      const int col0 = n0 + half * 128;  // first column (within the segment) of this thread
      if (S.kind == SEG_F32) {
        if (row_ok) {
          float* o = reinterpret_cast<float*>(S.out) + (int64_t)row * S.ld + col0;
#pragma unroll
          for (int i = 0; i < 128; i += 4)
            *reinterpret_cast<float4*>(o + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
        }
      } else if (S.kind == SEG_BF16 || S.kind == SEG_SIGMOID) {
        if (row_ok) {
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(S.out) + (int64_t)row * S.ld + col0;
#pragma unroll
          for (int i = 0; i < 128; i += 8) {
            float t[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              t[j] = acc[i + j];
              if (S.kind == SEG_SIGMOID) t[j] = sigmoid_contract(bf16_round(t[j]));
            }
            uint4 w4 = make_uint4(pack_bf16x2(t[0], t[1]), pack_bf16x2(t[2], t[3]), pack_bf16x2(t[4], t[5]),
                                  pack_bf16x2(t[6], t[7]));
            *reinterpret_cast<uint4*>(o + i) = w4;
          }
        }
      } else if (S.kind == SEG_QKNORM) {
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 128; ++i) acc[i] = bf16_round(acc[i]);
          // reduction order of kernels/joint_projection.cu:141-146
          float part[32];
#pragma unroll
          for (int l = 0; l < 32; ++l) {
            float s2 = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) s2 = __fmaf_rn(acc[4 * l + j], acc[4 * l + j], s2);
            part[l] = s2;
          }
#pragma unroll
          for (int off = 16; off; off >>= 1)
#pragma unroll
            for (int l = 0; l < off; ++l) part[l] = __fadd_rn(part[l], part[l + off]);
          const float inv = __frsqrt_rn(__fadd_rn(__fmul_rn(part[0], 0.0078125f), S.eps));
          const int token = row % p.length;
          const float* f = p.freqs + (int64_t)token * 256;
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(S.out) + (int64_t)row * S.ld + col0;
#pragma unroll
          for (int i = 0; i < 128; i += 8) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const int c = i + j;
              const float a = bf16_round(__fmul_rn(__fmul_rn(acc[c], inv), __fadd_rn(S.normw[c], 1.0f)));
              const float bb = bf16_round(__fmul_rn(__fmul_rn(acc[c + 1], inv), __fadd_rn(S.normw[c + 1], 1.0f)));
              const float4 fr = __ldg(reinterpret_cast<const float4*>(f + 2 * c));
              const float o0 = __fmaf_rn(fr.x, a, __fmul_rn(fr.y, bb));
              const float o1 = __fmaf_rn(fr.z, a, __fmul_rn(fr.w, bb));
              w[j / 2] = pack_bf16x2(o0, o1);
            }
            *reinterpret_cast<uint4*>(o + i) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      } else if (S.kind == SEG_RESIDUAL) {
        if (row_ok) {
          const int bidx = row / p.length;
          const __nv_bfloat16* gt = p.gate + (int64_t)bidx * S.n + col0;
          const __nv_bfloat16* rs = p.resid + (int64_t)row * S.ld + col0;
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(S.out) + (int64_t)row * S.ld + col0;
#pragma unroll
          for (int i = 0; i < 128; i += 8) {
            const uint4 g4 = __ldg(reinterpret_cast<const uint4*>(gt + i));
            const uint4 r4 = __ldg(reinterpret_cast<const uint4*>(rs + i));
            const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g4);
            const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&r4);
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 gf = __bfloat1622float2(g2[j]), rf = __bfloat1622float2(r2[j]);
              const float p0 = bf16_round(acc[i + 2 * j]), p1 = bf16_round(acc[i + 2 * j + 1]);
              const float x0 = bf16_round(__fmul_rn(p0, gf.x)), x1 = bf16_round(__fmul_rn(p1, gf.y));
              w[j] = pack_bf16x2(__fadd_rn(rf.x, x0), __fadd_rn(rf.y, x1));
            }
            *reinterpret_cast<uint4*>(o + i) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      } else if (pairw) {
        // Column half 0 holds the gate projection and half 1 the up projection
        // of the same 128 output columns; half 1 hands bf16(up) over in smem.
        uint8_t* xch = smem + GEMM_OFF_W;  // W stages are idle once every MMA has completed
        if (half == 1) {
          uint8_t* dst = xch + rloc * GEMM_XCH_STRIDE;
#pragma unroll
          for (int i = 0; i < 128; i += 8) {
            uint4 w4 = make_uint4(pack_bf16x2(acc[i], acc[i + 1]), pack_bf16x2(acc[i + 2], acc[i + 3]),
                                  pack_bf16x2(acc[i + 4], acc[i + 5]), pack_bf16x2(acc[i + 6], acc[i + 7]));
            *reinterpret_cast<uint4*>(dst + 2 * i) = w4;
          }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (half == 0 && row_ok) {
          const uint8_t* src = xch + rloc * GEMM_XCH_STRIDE;
#pragma unroll
          for (int i = 0; i < 128; i += 8) {
            const uint4 u4 = *reinterpret_cast<const uint4*>(src + 2 * i);
            const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&u4);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 uf = __bfloat1622float2(u2[j]);
              const float g0 = bf16_round(acc[i + 2 * j]), g1 = bf16_round(acc[i + 2 * j + 1]);
              const float a0 = bf16_round(silu_contract(g0)), a1 = bf16_round(silu_contract(g1));
              acc[i + 2 * j] = bf16_round(__fmul_rn(a0, uf.x));
              acc[i + 2 * j + 1] = bf16_round(__fmul_rn(a1, uf.y));
            }
          }
          if (S.kind == SEG_SWIGLU_BF16) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(S.out) + (int64_t)row * S.ld + n0;
#pragma unroll
            for (int i = 0; i < 128; i += 8) {
              uint4 w4 = make_uint4(pack_bf16x2(acc[i], acc[i + 1]), pack_bf16x2(acc[i + 2], acc[i + 3]),
                                    pack_bf16x2(acc[i + 4], acc[i + 5]), pack_bf16x2(acc[i + 6], acc[i + 7]));
              *reinterpret_cast<uint4*>(o + i) = w4;
            }
          } else {
          hadamard128_regs(acc);
          float amax = 0.0f;
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            acc[i] = __fmul_rn(acc[i], kHadamardScale);
            amax = fmaxf(amax, fabsf(acc[i]));
          }
          const __half hs = group_scale(amax);
          const float sd = __half2float(hs);
          const int grp = n0 / 128;  // output group (128 columns) index
          S.out_scale[(int64_t)row * (S.n / 128) + grp] = hs;
          uint8_t* o = reinterpret_cast<uint8_t*>(S.out) + (int64_t)row * S.ld + grp * 64;
          const float rcp = sd > 0.0f ? __frcp_rn(sd) : 0.0f;
#pragma unroll
          for (int i = 0; i < 128; i += 32) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t word = 0;
              if (sd > 0.0f) {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  word |= (uint32_t)(quant_code(acc[i + 8 * j + e], sd, rcp) & 0xF) << (4 * e);
              }
              w[j] = word;
            }
            *reinterpret_cast<uint4*>(o + i / 2) = make_uint4(w[0], w[1], w[2], w[3]);
          }
          }
        }
      }
    }
  }

  // ---------------------------------------------------------- teardown
  if (*abort_flag) {
    // let copies and MMAs that were already issued land before the CTA exits
    if (warp == 0 && lane == 0) {
      for (int g = (issued_w > GEMM_STAGES ? issued_w - GEMM_STAGES : 0); g < issued_w; ++g)
        mbar_drain(&full_w[g % GEMM_STAGES], (g / GEMM_STAGES) & 1);
      for (int g = (issued_pa > GEMM_PSTAGES ? issued_pa - GEMM_PSTAGES : 0); g < issued_pa; ++g)
        mbar_drain(&full_pa[g % GEMM_PSTAGES], (g / GEMM_PSTAGES) & 1);
      for (int g = (issued_sc > GEMM_PSTAGES ? issued_sc - GEMM_PSTAGES : 0); g < issued_sc; ++g)
        mbar_drain(&full_sc[g % GEMM_PSTAGES], (g / GEMM_PSTAGES) & 1);
    }
    if (warp == 1 && lane == 0 && issued_mma > 0) {
      const int g = issued_mma - 1;
      mbar_drain(&tmem_full[g & 1], (g >> 1) & 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace k2b
