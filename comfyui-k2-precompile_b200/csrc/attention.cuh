// attention.cuh -- GQA flash attention (forward, non-causal) on tcgen05.
//
// Replaces the Triton Kohaku FA (KohakuKernelRouter/attention.py:31-110):
// kv head = h / (Hq/Hkv) with no K/V replication, softmax scale
// c = log2(e)/sqrt(D) folded into exp2, fp32 online softmax, P rounded to
// bf16 before the PV product, o = acc/l (0 where l == 0), optional gate store
// (gate_kind 1: sigmoid applied here, 2: gate already sigmoided), and a fused
// H128 rotation + group-128 INT4 quantisation of o for the out-projection.
//
// One CTA owns two Q slots that read the same KV head, so every K/V tile
// brought in by TMA feeds both slots' MMAs:
//   * even GQA group (the Krea2 blocks, 48/12): one 128-token Q tile of two Q
//     heads 2p, 2p+1 (grid.y = heads / 2);
//   * odd group (group 1: the text-fusion blocks, 20/20): two consecutive
//     128-token Q tiles of one head (grid.y = heads, p.qpair = 1).
// TMEM (512 columns):
//   S0 [0,128)  S1 [128,256)  O0 [256,384)  O1 [384,512)
// P_t (bf16, 64 packed columns) overwrites S_t after the softmax has read it;
// tcgen05.mma ops of the issuing thread execute in order, so the next S MMA
// into the same columns follows the PV MMA that reads P.
// Roles (384 threads): warp 0 TMA loads, warp 1 TMEM alloc + MMA issue,
// warps 4-7 softmax/epilogue of slot 0, warps 8-11 of slot 1.
// O is rescaled in TMEM only when a row's running max grows by more than
// 2^8 in exp2 units (the max used for P may lag the true max); the final
// o = acc/l is unchanged by that choice up to rounding.
#pragma once
#include "k2b_common.cuh"

namespace k2b {

constexpr int FA_BM = 128;      // Q tokens per tile
constexpr int FA_BN = 128;      // keys per KV tile
constexpr int FA_D = 128;
constexpr int FA_KV_STAGES = 2;
constexpr int FA_THREADS = 384;
constexpr int FA_TILE_BYTES = FA_BM * FA_D * 2;  // 32 KB (two 16 KB 128B-swizzled boxes)
constexpr int FA_OFF_Q = 0;
constexpr int FA_OFF_K = FA_OFF_Q + 2 * FA_TILE_BYTES;
constexpr int FA_OFF_V = FA_OFF_K + FA_KV_STAGES * FA_TILE_BYTES;
constexpr int FA_OFF_BAR = FA_OFF_V + FA_KV_STAGES * FA_TILE_BYTES;
constexpr int FA_NBARS = 1 + 4 * FA_KV_STAGES + 6;
constexpr int FA_SMEM_BYTES = FA_OFF_BAR + FA_NBARS * 8 + 16 + 1024;
constexpr float FA_RESCALE_THRESHOLD = 8.0f;  // log2 units

struct AttnMaps {
  CUtensorMap q, k, v;
};

struct AttnParams {
  int batch, heads, kvheads, lq, lk;
  float c;                          // log2(e)/sqrt(D)
  const __nv_bfloat16* gate;        // [B, lq, heads*D] or null
  int gate_kind;                    // 1: apply sigmoid, 2: pre-sigmoided
  __nv_bfloat16* out;               // [B, lq, heads*D] or null
  uint8_t* oq;                      // [B*lq, heads*D/2] packed, [B*lq, heads*D] e4m3 bytes, or null
  __half* os;                       // [B*lq, heads] fp16 scales
  int oq_bytes;                     // oq holds e4m3 bytes (the block loop's container)
  int qpair;                        // slots = two Q tiles of one head (odd GQA group)
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(FA_THREADS, 1)
    attention_kernel(const __grid_constant__ AttnMaps maps, const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FA_OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + FA_KV_STAGES;
  uint64_t* v_full = k_empty + FA_KV_STAGES;
  uint64_t* v_empty = v_full + FA_KV_STAGES;
  uint64_t* s_full = v_empty + FA_KV_STAGES;  // [2]
  uint64_t* p_full = s_full + 2;              // [2]
  uint64_t* o_full = p_full + 2;              // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + FA_NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const int group = p.heads / p.kvheads;
  // slot t: head h0 + t*hstep, tokens [q0 + t*qstep, +128)
  const int h0 = p.qpair ? blockIdx.y : 2 * blockIdx.y;
  const int hstep = p.qpair ? 0 : 1;
  const int q0 = blockIdx.x * (p.qpair ? 2 * FA_BM : FA_BM);
  const int qstep = p.qpair ? FA_BM : 0;
  const int hk = h0 / group;
  const int nkv = (p.lk + FA_BN - 1) / FA_BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < FA_KV_STAGES; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_full[t], 1);
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

  int issued_k = 0, issued_v = 0, issued_pv = 0;
  bool q_issued = false;
  if (warp == 0) {
    // --------------------------------------------------------- TMA loads
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * FA_TILE_BYTES);
      for (int t = 0; t < 2; ++t)
        for (int hb = 0; hb < 2; ++hb)
          tma_load_4d(smem + FA_OFF_Q + t * FA_TILE_BYTES + hb * (FA_TILE_BYTES / 2), &maps.q, q_full, hb * 64,
                      q0 + t * qstep, h0 + t * hstep, b);
      q_issued = true;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % FA_KV_STAGES;
        const uint32_t ph = (j / FA_KV_STAGES) & 1;
        if (j >= FA_KV_STAGES && !mbar_wait(&k_empty[s], ph ^ 1, abort_flag, ERR_WAIT_LOAD)) break;
        mbar_arrive_expect_tx(&k_full[s], FA_TILE_BYTES);
        for (int hb = 0; hb < 2; ++hb)
          tma_load_4d(smem + FA_OFF_K + s * FA_TILE_BYTES + hb * (FA_TILE_BYTES / 2), &maps.k, &k_full[s], hb * 64,
                      j * FA_BN, hk, b);
        issued_k = j + 1;
        if (j >= FA_KV_STAGES && !mbar_wait(&v_empty[s], ph ^ 1, abort_flag, ERR_WAIT_LOAD)) break;
        mbar_arrive_expect_tx(&v_full[s], FA_TILE_BYTES);
        for (int hb = 0; hb < 2; ++hb)
          tma_load_4d(smem + FA_OFF_V + s * FA_TILE_BYTES + hb * (FA_TILE_BYTES / 2), &maps.v, &v_full[s], hb * 64,
                      j * FA_BN, hk, b);
        issued_v = j + 1;
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc(1, 1, 1, 0, 0, FA_BM, FA_BN);  // Q.K^T, both K-major
      constexpr uint32_t idesc_o = make_idesc(1, 1, 1, 0, 1, FA_BM, FA_D);   // P.V, V MN-major
      auto issue_s = [&](int t, int s) {
        const uint32_t qa = smem_u32(smem + FA_OFF_Q + t * FA_TILE_BYTES);
        const uint32_t ka = smem_u32(smem + FA_OFF_K + s * FA_TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * (FA_TILE_BYTES / 2) + (kk & 3) * 32;
          mma_bf16_ss(tmem + t * 128, umma_desc_sw128(qa + off, 16, 1024), umma_desc_sw128(ka + off, 16, 1024),
                      idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[t]);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, ERR_WAIT_MMA) && mbar_wait(&k_full[0], 0, abort_flag, ERR_WAIT_MMA);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        mma_commit(&k_empty[0]);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % FA_KV_STAGES;
        const uint32_t ph = (j / FA_KV_STAGES) & 1;
        for (int t = 0; t < 2 && ok; ++t) {
          if (!mbar_wait(&p_full[t], j & 1, abort_flag, ERR_WAIT_MMA)) { ok = false; break; }
          if (t == 0 && !mbar_wait(&v_full[s], ph, abort_flag, ERR_WAIT_MMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t va = smem_u32(smem + FA_OFF_V + s * FA_TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            // 16 keys per MMA: 16 rows of 128 B -> 2048 B per step; the two
            // 64-wide d halves are FA_TILE_BYTES/2 apart (LBO).
            mma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8,
                        umma_desc_sw128(va + kk * 2048, FA_TILE_BYTES / 2, 1024), idesc_o,
                        (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&o_full[t]);
          issued_pv = j + 1;
          if (t == 1) mma_commit(&v_empty[s]);
          if (j + 1 < nkv) {
            const int s2 = (j + 1) % FA_KV_STAGES;
            const uint32_t ph2 = ((j + 1) / FA_KV_STAGES) & 1;
            if (t == 0 && !mbar_wait(&k_full[s2], ph2, abort_flag, ERR_WAIT_MMA)) { ok = false; break; }
            tc_fence_after();
            issue_s(t, s2);
            if (t == 1) mma_commit(&k_empty[s2]);
          }
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;  // which slot
    const int q = warp & 3;
    const int r = 32 * q + lane;    // row within the Q tile
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    const uint32_t s_col = t * 128, o_col = 256 + t * 128;
    const float c = p.c;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, abort_flag, ERR_WAIT_SOFTMAX)) { ok = false; break; }
      tc_fence_after();
      // all eight loads in flight before one wait (the first wait::ld covers
      // every load; the others only pin their registers below it)
      float sv[128];
      {
        uint32_t u[8][16];
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) tmem_ld16(lane_base + s_col + 16 * cc, u[cc]);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          tmem_wait_ld_regs(u[cc]);
#pragma unroll
          for (int i = 0; i < 16; ++i) sv[16 * cc + i] = __uint_as_float(u[cc][i]);
        }
      }
      const int valid = p.lk - j * FA_BN;
      if (valid < FA_BN) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= valid) sv[i] = -INFINITY;
      }
      // row max as eight interleaved chains of 3-input max (exact, order-free)
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        m8[k] = sv[k];
#pragma unroll
        for (int jj = 1; jj < 15; jj += 2) m8[k] = fmax3(m8[k], sv[k + 8 * jj], sv[k + 8 * jj + 8]);
        m8[k] = fmaxf(m8[k], sv[k + 120]);
      }
      const float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      float m_use = m_run, alpha = 1.0f;
      bool rescale = false;
      if (j == 0) {
        m_use = mx;
      } else if (__fmul_rn(mx - m_run, c) > FA_RESCALE_THRESHOLD) {
        m_use = mx;
        alpha = fast_exp2(__fmul_rn(m_run - mx, c));
        rescale = true;
      }
      const float mc = __fmul_rn(m_use, c);
      float part[4];  // one partial row sum per 32 columns, summed at the end
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t pk[16];
        part[cc] = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = fast_exp2(__fmaf_rn(sv[32 * cc + 2 * i], c, -mc));
          const float p1 = fast_exp2(__fmaf_rn(sv[32 * cc + 2 * i + 1], c, -mc));
          part[cc] += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        tmem_st16(lane_base + s_col + 16 * cc, pk);
      }
      const float rowsum = (part[0] + part[1]) + (part[2] + part[3]);
      l_run = __fmaf_rn(l_run, alpha, rowsum);
      m_run = m_use;
      // O of this head is stable here: S_t(j) completing implies PV_t(j-1) completed.
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t u[16];
          tmem_ld16(lane_base + o_col + 16 * cc, u);
          tmem_wait_ld_regs(u);
#pragma unroll
          for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(__fmul_rn(__uint_as_float(u[i]), alpha));
          tmem_st16(lane_base + o_col + 16 * cc, u);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    // ------------------------------------------------------ epilogue
    if (ok && mbar_wait(&o_full[t], (nkv - 1) & 1, abort_flag, ERR_WAIT_SOFTMAX)) {
      tc_fence_after();
      const int tok = q0 + t * qstep + r;
      const int h = h0 + t * hstep;
      const float inv_l = l_run > 0.0f ? __frcp_rn(l_run) : 0.0f;
      float o[128];
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint32_t u[16];
        tmem_ld16(lane_base + o_col + 16 * cc, u);
        tmem_wait_ld_regs(u);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[16 * cc + i] = bf16_round(__fmul_rn(__uint_as_float(u[i]), inv_l));
      }
      if (tok < p.lq) {
        const int64_t orow = ((int64_t)b * p.lq + tok);
        if (p.gate) {
          const __nv_bfloat16* g = p.gate + orow * p.heads * FA_D + h * FA_D;
#pragma unroll
          for (int i = 0; i < 128; i += 8) {
            const uint4 g4 = __ldg(reinterpret_cast<const uint4*>(g + i));
            const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g4);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float2 gf = __bfloat1622float2(g2[e]);
              if (p.gate_kind == 1) {
                gf.x = bf16_round(sigmoid_contract(gf.x));
                gf.y = bf16_round(sigmoid_contract(gf.y));
              }
              o[i + 2 * e] = bf16_round(__fmul_rn(o[i + 2 * e], gf.x));
              o[i + 2 * e + 1] = bf16_round(__fmul_rn(o[i + 2 * e + 1], gf.y));
            }
          }
        }
        if (p.out) {
          __nv_bfloat16* dst = p.out + orow * p.heads * FA_D + h * FA_D;
#pragma unroll
          for (int i = 0; i < 128; i += 8) {
            const __nv_bfloat162 a0 = __floats2bfloat162_rn(o[i], o[i + 1]);
            const __nv_bfloat162 a1 = __floats2bfloat162_rn(o[i + 2], o[i + 3]);
            const __nv_bfloat162 a2 = __floats2bfloat162_rn(o[i + 4], o[i + 5]);
            const __nv_bfloat162 a3 = __floats2bfloat162_rn(o[i + 6], o[i + 7]);
            uint4 w4;
            w4.x = *reinterpret_cast<const uint32_t*>(&a0);
            w4.y = *reinterpret_cast<const uint32_t*>(&a1);
            w4.z = *reinterpret_cast<const uint32_t*>(&a2);
            w4.w = *reinterpret_cast<const uint32_t*>(&a3);
            *reinterpret_cast<uint4*>(dst + i) = w4;
          }
        }
        if (p.oq) {
          // H128 rotation + group-128 INT4 of this head's 128 channels
          hadamard128_regs(o);
          float amax = 0.0f;
#pragma unroll
          for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(o[i]));
          const QuantGroup qg = quant_group(amax);
          p.os[orow * p.heads + h] = qg.scale;
          const int per_col = p.oq_bytes ? 1 : 0;  // code bytes per column = 2^per_col / 2
          uint8_t* dq = p.oq + orow * ((p.heads * FA_D) << per_col >> 1) + ((h * 64) << per_col);
#pragma unroll
          for (int i = 0; i < 128; i += 32) {
            uint32_t w[4];
#pragma unroll
            for (int jw = 0; jw < 4; ++jw) {
              uint32_t b[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) b[e] = quant_bits(o[i + 8 * jw + e], qg.c, qg.clamp);
              w[jw] = pack8_codes(b);
            }
            if (p.oq_bytes) {
              uint4 lo, hi;
              unpack_chunk(make_uint4(w[0], w[1], w[2], w[3]), lo, hi);
              *reinterpret_cast<uint4*>(dq + i) = lo;
              *reinterpret_cast<uint4*>(dq + i + 16) = hi;
            } else {
              *reinterpret_cast<uint4*>(dq + i / 2) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown
  if (*abort_flag) {
    if (warp == 0 && lane == 0) {
      if (q_issued) mbar_drain(q_full, 0);
      for (int j = (issued_k > FA_KV_STAGES ? issued_k - FA_KV_STAGES : 0); j < issued_k; ++j)
        mbar_drain(&k_full[j % FA_KV_STAGES], (j / FA_KV_STAGES) & 1);
      for (int j = (issued_v > FA_KV_STAGES ? issued_v - FA_KV_STAGES : 0); j < issued_v; ++j)
        mbar_drain(&v_full[j % FA_KV_STAGES], (j / FA_KV_STAGES) & 1);
    }
    if (warp == 1 && lane == 0 && issued_pv > 0) {
      // the last commit covers every MMA issued before it
      mbar_drain(&o_full[0], (issued_pv - 1) & 1);
      mbar_drain(&o_full[1], (issued_pv - 1) & 1);
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
