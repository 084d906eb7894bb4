// gemm_w4a4.cuh -- group-scaled W4A4 GEMM on tcgen05 kind::f8f6f4 with fused
// epilogues (dequant, per-head QK RMSNorm + RoPE, sigmoid gate, gated
// residual, SwiGLU + INT4 requant of the down-projection input).
//
// Replaces the reference's SM89 mma.sync s4 kernels: qkv_kernel / swiglu_kernel
// / residual_norm_kernel (kernels/joint_projection.cu:68-202), the CUTLASS EVT
// ResidualGemm (kernels/int4_epilogue.cu:18-66) and QKGemm + NormRopeStore
// (kernels/qk_norm_rope.cu:19-133).
//
// Operands: the INT4 codes (-8..7) of both operands are fed to the tensor
// cores as e4m3 bytes, which hold every code exactly; every product is an
// integer of magnitude <= 64 and every partial sum of a 128-wide group an
// integer of magnitude <= 8192, so the fp32 accumulator of a group is the
// exact integer group sum (the int32 accumulator of an s8 MMA, already in
// floating point).  kind::f8f6f4 runs at the int8 rate.
// A (activations) arrives in one of two forms:
//   BYTEA = false: packed INT4 [M, K/2] (the library's activation contract);
//               two unpacker warps turn each 128-wide group into e4m3 bytes
//               in the 128B-swizzled UMMA layout (a byte-permute lookup);
//   BYTEA = true:  e4m3 bytes [M, K] written by the block loop's producers
//               (norm_quant, attention, SwiGLU epilogues); TMA loads them
//               straight into the UMMA layout and the unpackers idle.
// W is prepared once (k2b_prepare_weight) as e4m3 bytes [N, K].
//
// Reference-contract modes (the data the reference's kernel library receives
// through its own symbol names): one fp32 scale per activation row and per
// weight channel, so the accumulator runs over the whole of K and is scaled
// once, p = fp32(fp32(acc * xs[r]) * ws[c]) (kernels/joint_projection.cu:57-59):
//   GM_REF4:  packed INT4 A and packed INT4 W (a checkpoint's ConvRot W4A4
//             weight as it is stored); W is turned into e4m3 in the CTA by the
//             epilogue warps, idle until the last group;
//   GM_REF8:  int8 A and W bytes (kind::i8, int32 accumulator);
//   GM_REFF8: fp8 A and W bytes, e4m3 or e5m2 (fp32 accumulator), scales
//             given per row / channel or as one value (stride 0).
//
// Tile: a CTA pair (cluster of 2 along M) computes 256 rows x 256 columns;
// each CTA owns 128 rows of A and holds half of the W tile (128 of the 256
// columns; for SwiGLU the leader holds the gate rows, the peer the up rows).
// The leader issues tcgen05.mma.cta_group::2 (M = 256, N = 256): the tensor
// cores of both SMs read A from their own CTA and B from both, so each SM
// streams 16 KB of A + 16 KB of W per 128-wide K group instead of 16 + 32
// (a single-CTA M = 128 MMA measured ~740 cycles per group against ~400 for
// the pair).  K is consumed one quantisation group per pipeline stage.
// Roles (640 threads per CTA):
//   warp 0      TMA producers: lane 0 the A group tile (packed 128 x 64 B, or
//               bytes 128 x 128 B 128B-swizzled) and this CTA's half of the W
//               group tile (128 x 128 B, 128B-swizzled); packed A: lane 1 the
//               W scales of all 256 columns, in chunks of 8 (SwiGLU) or 16
//               groups, two chunk buffers (byte A: lane 0 of warp 3)
//   warp 1      TMEM allocator (both CTAs, cta_group::2); leader: single-thread
//               MMA issuer (4 x K=32 MMAs per group); peer: relays "stage
//               ready" (W landed + A unpacked) to the leader
//   warps 2-3   A unpackers (packed A): s4 -> e4m3 into the UMMA layout;
//               byte A: lane 0 of warp 2 issues the A tensor copies (a second
//               issuing thread: one thread's copies complete one at a time) and
//               lane 0 of warp 3 the W scales
//   warps 4-19  epilogue: TMEM lane quadrant = warp % 4, column quarter
//               = (warp-4)/4 (64 columns of one row per thread)
// Stage barrier full_s[s] collects this CTA's W (and byte A) bytes (producer
// expect_tx), its two unpacker arrivals (packed A) and, on the leader, the
// peer's relay.  MMA completion is committed to the same barrier offset in both
// CTAs (multicast commit); the peer's relay and its epilogue warps arrive on
// the leader's barriers remotely.  TMA copies complete on local barriers only,
// so each CTA can drain its own copies.
// TMEM: 2 x 256 fp32 columns, one per group in flight (ping-pong), so the MMA
// of group g+1 overlaps the dequant of group g.  The fp32 group sum lives in
// the epilogue registers (64 per thread); TMEM loads are software-pipelined
// one 16-column chunk ahead.  setmaxnreg gives the TMA/MMA/unpack warpgroup
// 32 registers and the four epilogue warpgroups 112.  For SwiGLU a thread
// owns 32 gate and the same 32 up columns (its 32 output columns), so the
// final SwiGLU + rotation + requant is spread over all 16 epilogue warps.
//
// Dequant contract (oracle: k2o_gemm_w4a4):
//   p = 0;  for g:  u = fp32(acc_g * sA[r,g]);  p = fmaf(u, sW[c,g], p)
// With |acc_g| <= 2^13 (at most 13 significant bits) and an fp16 sA (at most
// 11), acc_g * sA has at most 24 significant bits: u is exact, one fp32
// multiply of the TMEM word (the exact group sum) by sA.  Both steps run on
// packed f32x2 pairs.
#pragma once
#include "k2b_common.cuh"

namespace k2b {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BN = 256;
constexpr int GEMM_STAGES = 4;   // prepared W half + unpacked A
constexpr int GEMM_PSTAGES = 4;  // packed A and W scales
constexpr int GEMM_EPI_WARPS = 16;
constexpr int kGemmBand = 16;    // M pairs (of 256 rows) per band of the tile order
constexpr int GEMM_THREADS = 128 + 32 * GEMM_EPI_WARPS;  // 640
// Registers per thread the kernel is compiled with (65536 / 640 rounded down
// to the allocation granule).  Warpgroup 0 drops to 32 and the epilogue
// warpgroups grow to 112 (128*32 + 512*112 == 640*96); the launcher refuses
// any other allocation.
constexpr int GEMM_LAUNCH_REGS = 96;

constexpr int GEMM_W_BYTES = GEMM_BN / 2 * 128;   // 16 KB: this CTA's half of the W tile
constexpr int GEMM_UA_BYTES = GEMM_BM * 128;      // 16 KB
constexpr int GEMM_PA_BYTES = GEMM_BM * 64;       // 8 KB
// W scales arrive in chunks of up to 16 K groups, two chunk buffers of 16 KB,
// copied by a producer thread of their own.  The SwiGLU kernel (two copies per
// group: gate and up scales) takes chunks of 8 groups: gate/up at 33792 rows
// measured 11.15 ms with 8, 11.24 with 4, 11.38 with 16 and 11.35 with 2 (with
// the epilogue's handoff order as built; an earlier epilogue preferred 4).  The
// other kinds are within noise between 8 and 16 and keep 16.
constexpr int GEMM_SC_MAX_GROUPS = 16;
constexpr int GEMM_SC_BYTES = GEMM_BN * 4 * GEMM_SC_MAX_GROUPS;
constexpr int GEMM_OFF_W = 0;
constexpr int GEMM_OFF_UA = GEMM_OFF_W + GEMM_STAGES * GEMM_W_BYTES;
constexpr int GEMM_OFF_PA = GEMM_OFF_UA + GEMM_STAGES * GEMM_UA_BYTES;
constexpr int GEMM_OFF_SC = GEMM_OFF_PA + GEMM_PSTAGES * GEMM_PA_BYTES;
constexpr int GEMM_OFF_BAR = GEMM_OFF_SC + 2 * GEMM_SC_BYTES;
constexpr int GEMM_NBARS = 2 * GEMM_STAGES + 2 * GEMM_PSTAGES + 2 * 2 + 4 + 2 * GEMM_PSTAGES;
constexpr int GEMM_PW_BYTES = 128 * 64;  // packed W rows of one CTA and group (reference contract)
static_assert(GEMM_PSTAGES * GEMM_PW_BYTES <= 2 * GEMM_SC_BYTES, "packed W stages use the scale-chunk space");
constexpr int GEMM_SMEM_BYTES = GEMM_OFF_BAR + GEMM_NBARS * 8 + 16 + 1024;  // + alignment slack
// The final epilogue exchanges rows through the (then idle) W, unpacked-A and
// packed-A stages: SwiGLU needs two 4 x 128 x 33-float stage buffers and 512
// floats for the group maxima.
constexpr int kSwXch = 4 * 128 * 33;
static_assert(GEMM_OFF_SC >= (2 * kSwXch + 512) * 4 && GEMM_OFF_SC >= 128 * 260 * 4, "exchange space");

enum SegKind : int {
  SEG_BF16 = 0,       // bf16(p)
  SEG_QKNORM = 1,     // per-head RMSNorm + RoPE of bf16(p)
  SEG_SIGMOID = 2,    // bf16(sigmoid(bf16(p)))
  SEG_RESIDUAL = 3,   // bf16(resid + bf16(bf16(p) * gate))
  SEG_SWIGLU = 4,     // SwiGLU of (gate, up) column pairs + H128 + INT4 requant
  SEG_F32 = 5,        // p itself (tests: exact accumulators)
  SEG_SWIGLU_BF16 = 6,// SwiGLU of (gate, up) column pairs, bf16 h
  SEG_F32_SCATTER = 7,// p stored into the owner rank's slot of a peer buffer (tensor-parallel partials)
  SEG_SWIGLU_E4M3 = 8 // SEG_SWIGLU with the INT4 codes stored as e4m3 bytes [M, width] (block-loop container)
};

struct GemmSegment {
  int tiles;             // N tiles of this segment (256 columns; SwiGLU: 128 output columns)
  int kind;              // SegKind
  int n;                 // columns of the segment's prepared weight(s)
  int ld;                // leading dimension (elements) of the output
  void* out;             // output base (bf16 / fp32 / packed u8 / e4m3 bytes)
  const float* wscale;   // prepared W scales, fp32 [G, n]
  const float* wscale2;  // SwiGLU: up-projection scales, fp32 [G, n]
  const float* normw;    // SEG_QKNORM: fp32 [128] ("w+1" form)
  float eps;             // SEG_QKNORM
  __half* out_scale;     // SEG_SWIGLU(_E4M3): fp16 [M, n/128]
  // Optional LoRA bypass delta (graph_ops.py:246-249: value + T(T(x down^T)
  // up^T) * s), applied to T(p) before the segment's epilogue:
  // p' = T(T(p) + T(T(d) * s)), d[r, c] = sum_k lt[r, k] * lup[c, k] (fp32),
  // lt bf16 [M, lr] = T(x down^T), lup bf16 [n, lr], lr % 8 == 0.  SwiGLU:
  // lt/lup for the gate half, lt2/lup2 for the up half.
  const __nv_bfloat16* lt;
  const __nv_bfloat16* lup;
  int lr;
  float ls;
  const __nv_bfloat16* lt2;
  const __nv_bfloat16* lup2;
  int lr2;
  float ls2;
};

enum GemmMode : int {
  GM_PACKED = 0,  // group-128 contract, packed INT4 A
  GM_BYTES = 1,   // group-128 contract, e4m3 byte A
  GM_REF4 = 2,    // reference contract, packed INT4 A and W
  GM_REF8 = 3,    // reference contract, int8 A and W
  GM_REFF8 = 4    // reference contract, fp8 A and W
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
  // SEG_F32_SCATTER: row r goes to rank r / scatter_chunk, whose buffer
  // peer[rank] (fp32 [tp, scatter_chunk, ld], this GPU's or an NVLink peer's)
  // takes it in slot scatter_rank at row r % scatter_chunk
  float* peer[4];
  int scatter_chunk, scatter_rank;
  // reference-contract modes: activation scales xs[r * xs_stride], weight
  // scales seg.wscale[c * ws_stride] (fp32), optional fp32 bias [n], and the
  // fp8 operand formats (GM_REFF8: a | b << 3, 0 e4m3 / 1 e5m2)
  const float* xs;
  int xs_stride, ws_stride;
  const float* bias;
  uint32_t f8fmt;
};

struct WeightMaps {
  CUtensorMap m[4];
};


// Named barrier over the 16 epilogue warps only.
__device__ __forceinline__ void epi_barrier() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * GEMM_EPI_WARPS) : "memory");
}

__device__ __forceinline__ void store_bf16x64(__nv_bfloat16* o, const float (&v)[64]) {
#pragma unroll
  for (int i = 0; i < 64; i += 8) {
    uint4 w4 = make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                          pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
    *reinterpret_cast<uint4*>(o + i) = w4;
  }
}

// LoRA delta of 32 register slots holding consecutive columns c .. c+31 of
// one row: acc = T(T(acc) + T(T(d) * s)), d = trow . up[c + j] in fp32.  The
// factor rows are read with 16-byte loads that are uniform across the warp
// (every lane of a warp covers the same columns), eight slots at a time to
// stay inside the epilogue's register budget.
__device__ __forceinline__ void lora_delta32(float* acc, const __nv_bfloat16* __restrict__ trow,
                                             const __nv_bfloat16* __restrict__ up, int r, float s) {
#pragma unroll
  for (int h = 0; h < 32; h += 8) {
    float d[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] = 0.0f;
    for (int k = 0; k < r; k += 8) {
      const uint4 t4 = __ldg(reinterpret_cast<const uint4*>(trow + k));
      const __nv_bfloat162* t2 = reinterpret_cast<const __nv_bfloat162*>(&t4);
      float2 tf[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) tf[e] = __bfloat1622float2(t2[e]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 u4 = __ldg(reinterpret_cast<const uint4*>(up + (int64_t)(h + j) * r + k));
        const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&u4);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 uf = __bfloat1622float2(u2[e]);
          d[j] = __fmaf_rn(tf[e].x, uf.x, d[j]);
          d[j] = __fmaf_rn(tf[e].y, uf.y, d[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      acc[h + j] = bf16_round(__fadd_rn(bf16_round(acc[h + j]), bf16_round(__fmul_rn(bf16_round(d[j]), s))));
  }
}

// PAIRW: SwiGLU launches (one segment of gate/up column pairs); the column
// mapping of the epilogue threads is then a compile-time choice.  MODE: a
// GemmMode (operand forms and scale contract).  LORA: the variant that
// applies the segments' LoRA deltas (its code stays out of the others'
// register allocation).
template <bool PAIRW, int MODE, bool LORA = false>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_w4a4_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ WeightMaps wmaps,
                     const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kScGroups = PAIRW ? 8 : GEMM_SC_MAX_GROUPS;
  // A arrives as bytes loaded by TMA (else packed INT4 unpacked by warps 2-3)
  constexpr bool BYTEA = MODE == GM_BYTES || MODE == GM_REF8 || MODE == GM_REFF8;
  constexpr bool REF = MODE >= GM_REF4;  // full-K accumulation, per-row / per-channel scales
  constexpr bool PW = MODE == GM_REF4;   // packed W, unpacked by the epilogue warps
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + GEMM_OFF_BAR);
  // full_s[s]: this CTA's W half landed (producer's expect_tx arrival + TMA
  // bytes) and its A unpacked (2 unpacker arrivals); on the leader also the
  // peer's stage (1 arrival relayed by the peer).
  uint64_t* full_s = bars;                          // [STAGES]
  uint64_t* empty_s = full_s + GEMM_STAGES;         // [STAGES] MMAs done with W/A stage (both CTAs)
  uint64_t* full_pa = empty_s + GEMM_STAGES;        // [PSTAGES] TMA packed A landed
  uint64_t* empty_pa = full_pa + GEMM_PSTAGES;      // [PSTAGES] unpackers done
  uint64_t* full_sc = empty_pa + GEMM_PSTAGES;      // [2] W scale chunk landed
  uint64_t* empty_sc = full_sc + 2;                 // [2] epilogue done with a scale chunk
  uint64_t* tmem_full = empty_sc + 2;               // [2] MMAs of a group done (both CTAs)
  uint64_t* tmem_empty = tmem_full + 2;             // [2] leader: buffer drained by both CTAs
  uint64_t* full_pw = tmem_empty + 2;               // [PSTAGES] GM_REF4: packed W landed
  uint64_t* empty_pw = full_pw + GEMM_PSTAGES;      // [PSTAGES] GM_REF4: W unpacked
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + GEMM_NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: leader (issues the pair's MMAs), 1: peer
  const bool leader = rank == 0;
  // Banded tile order: the launch-order index of the CTA pair is remapped so
  // that kGemmBand consecutive M pairs (4096 rows of packed A, ~13 MB) walk
  // every N tile before the next band starts.  A band stays in L2 while the
  // weights stream once per band (launch order alone re-streams all of A for
  // each N tile).  Both CTAs of a pair decode the same (pair, N tile).
  const int pairs_m = (int)(gridDim.x >> 1), ntiles = (int)gridDim.y;
  const int lin = (int)blockIdx.y * pairs_m + (int)(blockIdx.x >> 1);
  const int band0 = lin / (kGemmBand * ntiles) * kGemmBand;
  const int band_pairs = min(kGemmBand, pairs_m - band0);
  const int in_band = lin - band0 * ntiles;
  const int ntile = in_band / band_pairs;
  const int m0 = (2 * (band0 + in_band % band_pairs) + (int)rank) * GEMM_BM;
  // Segment of this N tile.
  int seg = 0, tile = ntile;
  while (seg + 1 < p.nseg && tile >= p.seg[seg].tiles) {
    tile -= p.seg[seg].tiles;
    ++seg;
  }
  const GemmSegment& S = p.seg[seg];
  // SwiGLU tiles pair 128 gate rows (map 0) with the same 128 up rows (map 1).
  constexpr bool pairw = PAIRW;  // the launcher checks S.kind against it
  const int n0 = tile * (pairw ? GEMM_BN / 2 : GEMM_BN);
  // A segment may end half way through its last tile (width a multiple of
  // 128): the weight rows beyond it are zero-filled by TMA, only the valid
  // scales are copied and the epilogue stores no column past the end.
  const int vcols = pairw ? GEMM_BN : min(GEMM_BN, S.n - n0);
  const int G = p.G;

  if (threadIdx.x == 0) {
    for (int i = 0; i < GEMM_STAGES; ++i) {
      // W producer's expect_tx arrival + (byte A) the A producer's expect_tx
      // arrival or (packed A) 2 unpacker arrivals (+ the peer's relay on the
      // leader)
      // (GM_REF4: 2 A unpacker + 16 W unpacker arrivals, no copy into the stage)
      mbar_init(&full_s[i], (PW ? 2 + GEMM_EPI_WARPS : BYTEA ? 2 : 3) + (leader ? 1 : 0));
      mbar_init(&empty_s[i], 1);
    }
    for (int i = 0; i < GEMM_PSTAGES; ++i) {
      mbar_init(&full_pa[i], 1);
      mbar_init(&empty_pa[i], 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full_sc[i], 1);
      mbar_init(&empty_sc[i], GEMM_EPI_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 2 * GEMM_EPI_WARPS);
    }
    for (int i = 0; i < GEMM_PSTAGES; ++i) {
      mbar_init(&full_pw[i], 1);
      mbar_init(&empty_pw[i], GEMM_EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Both CTAs' barriers are initialised before either CTA signals the other.
  cluster_sync_all();
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int issued_w = 0, issued_pa = 0, issued_sc = 0, issued_mma = 0;
  // ------------------------------------------------ W-scale chunk producer
  // Chunk c (groups kScGroups*c ..) goes to buffer c % 2 once the epilogue
  // has released chunk c - 2.  A thread of its own: copies issued by one
  // thread complete one after another, so the scale copies never queue with
  // the W/A copies.  Byte A: lane 0 of warp 3, which has no other work, so
  // every scheduler hosts one single-thread role (warp 0 the W copies, warp 1
  // the MMAs, warp 2 the A copies).  The epilogue warps that share a scheduler
  // with two divergent producer lanes of one warp were measured ~1100 cycles
  // per K group behind the others, and the slowest warp releases the TMEM
  // buffer.  Packed A: lane 1 of warp 0 (warps 2-3 unpack A).
  auto scale_producer = [&]() {
    const int nchunks = (G + kScGroups - 1) / kScGroups;
    for (int chunk = 0; chunk < nchunks; ++chunk) {
      const int cb = chunk & 1;
      if (chunk >= 2 && !mbar_wait(&empty_sc[cb], ((chunk >> 1) & 1) ^ 1, abort_flag, ERR_WAIT_PRODUCER)) break;
      const int g0 = chunk * kScGroups;
      const int ng = min(kScGroups, G - g0);
      mbar_arrive_expect_tx(&full_sc[cb], ng * (pairw ? GEMM_BN : vcols) * 4);
      uint8_t* dst = smem + GEMM_OFF_SC + cb * GEMM_SC_BYTES;
      for (int j = 0; j < ng; ++j) {
        const int64_t off = (int64_t)(g0 + j) * S.n + n0;
        if (pairw) {
          bulk_load(dst + j * GEMM_BN * 4, S.wscale + off, GEMM_BN * 2, &full_sc[cb]);
          bulk_load(dst + j * GEMM_BN * 4 + GEMM_BN * 2, S.wscale2 + off, GEMM_BN * 2, &full_sc[cb]);
        } else {
          bulk_load(dst + j * GEMM_BN * 4, S.wscale + off, (uint32_t)vcols * 4u, &full_sc[cb]);
        }
      }
      issued_sc = chunk + 1;
    }
  };
  if (warp < 4) {
    setmaxnreg_dec32();
    if (warp == 0) {
      // ----------------------------------------------------- TMA producer
      if (lane == 0) {
        const CUtensorMap* wmap = &wmaps.m[pairw ? rank : seg];
        const int wrow = pairw ? n0 : n0 + 128 * (int)rank;
        for (int g = 0; g < G; ++g) {
          const int s = g % GEMM_STAGES, ps = g % GEMM_PSTAGES;
          const uint32_t ph = (g / GEMM_STAGES) & 1, pph = (g / GEMM_PSTAGES) & 1;
          if (PW) {
            // packed W rows of this CTA into the packed-W stage (the epilogue
            // warps unpack them into the stage the MMA reads)
            if (g >= GEMM_PSTAGES && !mbar_wait(&empty_pw[ps], pph ^ 1, abort_flag, ERR_WAIT_PRODUCER)) break;
            mbar_arrive_expect_tx(&full_pw[ps], GEMM_PW_BYTES);
            tma_load_2d(smem + GEMM_OFF_SC + ps * GEMM_PW_BYTES, wmap, &full_pw[ps], g * 64, wrow);
            issued_w = g + 1;
          } else {
            if (g >= GEMM_STAGES && !mbar_wait(&empty_s[s], ph ^ 1, abort_flag, ERR_WAIT_PRODUCER)) break;
            mbar_arrive_expect_tx(&full_s[s], GEMM_W_BYTES);
            // this CTA's 128 of the pair's 256 B columns (SwiGLU: gate | up)
            tma_load_2d(smem + GEMM_OFF_W + s * GEMM_W_BYTES, wmap, &full_s[s], g * 128, wrow);
            issued_w = g + 1;
          }
          if (BYTEA) continue;  // A comes from the A producer (warp 2)
          if (g >= GEMM_PSTAGES && !mbar_wait(&empty_pa[ps], pph ^ 1, abort_flag, ERR_WAIT_PRODUCER)) break;
          mbar_arrive_expect_tx(&full_pa[ps], GEMM_PA_BYTES);
          tma_load_2d(smem + GEMM_OFF_PA + ps * GEMM_PA_BYTES, &amap, &full_pa[ps], g * 64, m0);
          issued_pa = g + 1;
        }
      } else if (lane == 1 && !REF && !BYTEA) {
        scale_producer();
      }
    } else if (warp == 1) {
      // ------------------------------------- MMA issuer (leader) / relay (peer)
      if (lane == 0 && leader) {
        // fp32 accumulators of e4m3 (or fp8 formats of p.f8fmt) operands, or
        // int32 of int8 operands (GM_REF8); both K-major
        const uint32_t idesc = MODE == GM_REF8    ? make_idesc(2, 1, 1, 0, 0, 2 * GEMM_BM, GEMM_BN)
                               : MODE == GM_REFF8 ? make_idesc(1, p.f8fmt & 7, (p.f8fmt >> 3) & 7, 0, 0,
                                                               2 * GEMM_BM, GEMM_BN)
                                                  : make_idesc(1, 0, 0, 0, 0, 2 * GEMM_BM, GEMM_BN);
        for (int g = 0; g < G; ++g) {
          // reference contract: one accumulator over all of K in buffer 0
          const int s = g % GEMM_STAGES, b = REF ? 0 : (g & 1);
          const uint32_t ph = (g / GEMM_STAGES) & 1, bph = (g >> 1) & 1;
          if (!mbar_wait_cluster(&full_s[s], ph, abort_flag, ERR_WAIT_MMA)) {
            if (REF && issued_mma > 0) mma_commit_pair(&tmem_full[0]);  // for the teardown drain
            break;
          }
          if (!REF && g >= 2 && !mbar_wait_cluster(&tmem_empty[b], bph ^ 1, abort_flag, ERR_WAIT_MMA)) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + GEMM_OFF_UA + s * GEMM_UA_BYTES);
          const uint32_t w_base = smem_u32(smem + GEMM_OFF_W + s * GEMM_W_BYTES);
          // one descriptor per operand and group; the K step of 32 bytes is +2 in
          // the descriptor's 16-byte address field (shared addresses stay far below
          // its 256 KB range, so the add never carries out of it)
          const uint64_t ad0 = umma_desc_sw128(a_base, 16, 1024), bd0 = umma_desc_sw128(w_base, 16, 1024);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = ad0 + 2u * k;
            const uint64_t bd = bd0 + 2u * k;
            const uint32_t acc = (k > 0 || (REF && g > 0)) ? 1u : 0u;
            if (MODE == GM_REF8) mma_i8_pair(tmem + b * GEMM_BN, ad, bd, idesc, acc);
            else mma_f8_pair(tmem + b * GEMM_BN, ad, bd, idesc, acc);
          }
          mma_commit_pair(&empty_s[s]);
          if (!REF || g == G - 1) mma_commit_pair(&tmem_full[b]);
          issued_mma = g + 1;
        }
      } else if (lane == 0) {
        // the peer's W half has landed and its A is unpacked: tell the leader
        const uint32_t ready0 = cluster_map(smem_u32(&full_s[0]), 0);
        for (int g = 0; g < G; ++g) {
          const int s = g % GEMM_STAGES;
          const uint32_t ph = (g / GEMM_STAGES) & 1;
          if (!mbar_wait(&full_s[s], ph, abort_flag, ERR_WAIT_MMA)) break;
          mbar_arrive_remote(ready0 + 8u * (uint32_t)s);
        }
      }
    } else if (BYTEA && warp == 3) {
      if (lane == 0 && !REF) scale_producer();
    } else if (BYTEA) {
      // --------------------------------------------- A producer (byte A)
      // A tensor copies go out from a warp of their own: copies issued by one
      // thread complete one after another (~545 cycles each, nearly
      // independent of size), so one thread issuing both the W and the A copy
      // of every group would hold the K-group period above ~1100 cycles.
      if (warp == 2 && lane == 0) {
        for (int g = 0; g < G; ++g) {
          const int s = g % GEMM_STAGES;
          const uint32_t ph = (g / GEMM_STAGES) & 1;
          if (g >= GEMM_STAGES && !mbar_wait(&empty_s[s], ph ^ 1, abort_flag, ERR_WAIT_PRODUCER)) break;
          mbar_arrive_expect_tx(&full_s[s], GEMM_UA_BYTES);
          // e4m3 A rows of this CTA, straight into the UMMA layout
          tma_load_2d(smem + GEMM_OFF_UA + s * GEMM_UA_BYTES, &amap, &full_s[s], g * 128, m0);
          issued_pa = g + 1;
        }
      }
    } else {
      // ----------------------------------------------------- A unpackers
      const int t = threadIdx.x - 64;  // 0..63
      for (int g = 0; g < G; ++g) {
        const int s = g % GEMM_STAGES, ps = g % GEMM_PSTAGES;
        const uint32_t ph = (g / GEMM_STAGES) & 1, pph = (g / GEMM_PSTAGES) & 1;
        if (!mbar_wait(&full_pa[ps], pph, abort_flag, ERR_WAIT_UNPACK)) break;
        if (g >= GEMM_STAGES && !mbar_wait(&empty_s[s], ph ^ 1, abort_flag, ERR_WAIT_UNPACK)) break;
        const uint4* src = reinterpret_cast<const uint4*>(smem + GEMM_OFF_PA + ps * GEMM_PA_BYTES);
        uint8_t* dst = smem + GEMM_OFF_UA + s * GEMM_UA_BYTES;
        // 16-byte packed chunk i = t + 64*it: row i/4 (= t/4 + 16*it), K columns
        // 32*(i%4) .. +31, which land in the row's 16-byte UMMA chunks 2*(i%4)
        // (columns +0..15) and 2*(i%4)+1 (columns +16..31), XOR-swizzled by row
        const int c = t & 3, r0 = t >> 2;  // (r0 + 16*it) & 7 == r0 & 7
        uint8_t* d0 = dst + r0 * 128 + (((2 * c) ^ (r0 & 7)) << 4);
        uint8_t* d1 = dst + r0 * 128 + (((2 * c + 1) ^ (r0 & 7)) << 4);
#pragma unroll
        // two chunks in flight per step: the lookup's temporaries must fit
        // the 32 registers this warpgroup runs with
#pragma unroll
        for (int part = 0; part < 4; ++part) {
          uint4 pk[2];
#pragma unroll
          for (int it = 0; it < 2; ++it) pk[it] = src[t + 64 * (2 * part + it)];
#pragma unroll
          for (int it = 0; it < 2; ++it) {
            uint4 lo, hi;
            unpack_chunk(pk[it], lo, hi);
            *reinterpret_cast<uint4*>(d0 + (2 * part + it) * 16 * 128) = lo;
            *reinterpret_cast<uint4*>(d1 + (2 * part + it) * 16 * 128) = hi;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty_pa[ps]);
          mbar_arrive(&full_s[s]);
        }
      }
    }
  } else {
    // ------------------------------------------------------- epilogue
    setmaxnreg_inc112();
    const int q = warp & 3;
    const int cq = (warp - 4) >> 2;  // column quarter 0..3
    const int rloc = 32 * q + lane;
    const int row = m0 + rloc;
    const bool row_ok = row < p.M;
    const __half* sa_row = p.sa + (int64_t)(row_ok ? row : 0) * G;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    // This thread's TMEM / scale columns: chunks ca, ca+16, ca+kCd, ca+kCd+16
    // land in register slots 0, 16, 32, 48.  SwiGLU: 32 gate columns (ca) and
    // the same 32 up columns (ca + 128); other kinds: 64 consecutive columns.
    constexpr int kCd = pairw ? GEMM_BN / 2 : 32;
    const int ca = pairw ? 32 * cq : 64 * cq;
    const uint32_t tmem_empty_remote = cluster_map(smem_u32(tmem_empty), 0);
    bool ok = true;
    float2 acc2[32];  // register slots (2j, 2j+1)
#pragma unroll
    for (int j = 0; j < 32; ++j) acc2[j] = make_float2(0.0f, 0.0f);
    // TMEM loads are software-pipelined: the load of chunk c+1 (16 columns)
    // is in flight while chunk c is dequantised.  Barriers, scales and the abort
    // flag are addressed with 32-bit shared addresses to leave the registers
    // to the accumulators and the two load buffers.
    const uint32_t s_full_sc = smem_u32(full_sc), s_empty_sc = smem_u32(empty_sc);
    const uint32_t s_tfull = smem_u32(tmem_full), s_tempty = smem_u32(tmem_empty);
    const uint32_t s_abort = smem_u32((const void*)abort_flag);
    const uint32_t s_scales = smem_u32(smem + GEMM_OFF_SC) + 4 * ca;
    // TMEM words are the exact fp32 group sums: u = acc_g * sA (exact), then
    // p = fma(u, sW, p), two columns per packed instruction.
    auto dequant16 = [&](const uint32_t (&v)[16], uint32_t scs, int slot0, float2 sa2) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 sw = lds128(scs + 4 * i);  // scales of this chunk's columns i .. i+3
        const float2 u0 = __fmul2_rn(make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), sa2);
        const float2 u1 = __fmul2_rn(make_float2(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3])), sa2);
        acc2[(slot0 + i) / 2] = __ffma2_rn(u0, make_float2(sw.x, sw.y), acc2[(slot0 + i) / 2]);
        acc2[(slot0 + i) / 2 + 1] = __ffma2_rn(u1, make_float2(sw.z, sw.w), acc2[(slot0 + i) / 2 + 1]);
      }
    };
    float acc[64];
    if constexpr (REF) {
      if constexpr (PW) {
        // Until the last group the epilogue warps unpack this CTA's packed W
        // rows (one 16-byte chunk = 32 codes per thread and group) into the
        // stage the MMA reads, in the A unpackers' layout.
        const int t = threadIdx.x - 128;  // 0..511: row t/4, 32-column piece t%4
        const int c = t & 3, r0 = t >> 2;
        for (int g = 0; g < G && ok; ++g) {
          const int s = g % GEMM_STAGES, ps = g % GEMM_PSTAGES;
          const uint32_t ph = (g / GEMM_STAGES) & 1, pph = (g / GEMM_PSTAGES) & 1;
          if (!mbar_wait_s(smem_u32(&full_pw[ps]), pph, s_abort, ERR_WAIT_EPILOGUE) ||
              (g >= GEMM_STAGES && !mbar_wait_s(smem_u32(&empty_s[s]), ph ^ 1, s_abort, ERR_WAIT_EPILOGUE))) {
            ok = false;
            break;
          }
          const uint4 v = reinterpret_cast<const uint4*>(smem + GEMM_OFF_SC + ps * GEMM_PW_BYTES)[t];
          uint4 lo, hi;
          unpack_chunk(v, lo, hi);
          uint8_t* dst = smem + GEMM_OFF_W + s * GEMM_W_BYTES + r0 * 128;
          *reinterpret_cast<uint4*>(dst + (((2 * c) ^ (r0 & 7)) << 4)) = lo;
          *reinterpret_cast<uint4*>(dst + (((2 * c + 1) ^ (r0 & 7)) << 4)) = hi;
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&empty_pw[ps]);
            mbar_arrive(&full_s[s]);
          }
        }
      }
      // One accumulator over all of K: p = fp32(fp32(acc * xs[r]) * ws[c])
      // (+ bias[c]), the reference's projected() before its rounding to T.
      ok = ok && mbar_wait_s(s_tfull, 0, s_abort, ERR_WAIT_EPILOGUE);
      if (ok) {
        tc_fence_after();
        constexpr int kCd = pairw ? GEMM_BN / 2 : 32;
        const uint32_t tcol = lane_base + ca;
        uint32_t v[4][16];
        tmem_ld16(tcol, v[0]);
        tmem_ld16(tcol + 16, v[1]);
        tmem_ld16(tcol + kCd, v[2]);
        tmem_ld16(tcol + kCd + 16, v[3]);
        tmem_wait_ld_regs(v[0]);
        tmem_wait_ld_regs(v[1]);
        tmem_wait_ld_regs(v[2]);
        tmem_wait_ld_regs(v[3]);
        const float xs = row_ok ? p.xs[(int64_t)row * p.xs_stride] : 0.0f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          // register slot j: chunk j/16 of this thread's columns
          const int cc = (j < 32 ? j : j - 32 + kCd);  // column within the tile, from ca
          const int col = n0 + ca + cc;                // SwiGLU: gate (j < 32) / up (j >= 32) weight row
          const bool up = pairw && j >= 32;
          const int wcol = up ? n0 + ca + (j - 32) : (pairw ? n0 + ca + j : col);
          const float* wsp = up ? S.wscale2 : S.wscale;
          const bool cok = pairw || col < S.n;
          const uint32_t raw = v[j >> 4][j & 15];
          const float a = MODE == GM_REF8 ? __int2float_rn((int)raw) : __uint_as_float(raw);
          float pv = cok ? __fmul_rn(__fmul_rn(a, xs), wsp[(int64_t)wcol * p.ws_stride]) : 0.0f;
          if (p.bias && cok && !pairw) pv = __fadd_rn(pv, p.bias[col]);
          acc[j] = pv;
        }
      }
    } else {
      const uint32_t tcol = lane_base + ca;  // this thread's first column in buffer 0
      uint32_t va[16], vb[16];
      ok = mbar_wait_s(s_full_sc, 0, s_abort, ERR_WAIT_EPILOGUE) && mbar_wait_s(s_tfull, 0, s_abort, ERR_WAIT_EPILOGUE);
      if (ok) {
        tc_fence_after();
        tmem_ld16(tcol, va);
      }
      __half sa_next = sa_row[0];  // activation scales are prefetched one group ahead
      for (int g = 0; g < G && ok; ++g) {
        if (g > 0) {
          // group g's scales (first group of a chunk) and accumulators; every
          // chunk of group g-1 was dequantised before this wait, which ends the
          // MMA -> epilogue -> release chain of the next buffer (traced: doing
          // the last chunk after the wait kept ~630 cycles per group on it)
          const int c = g / kScGroups;
          if (!((g % kScGroups != 0 ||
                 mbar_wait_s(s_full_sc + 8u * (uint32_t)(c & 1), (c >> 1) & 1, s_abort, ERR_WAIT_EPILOGUE)) &&
                mbar_wait_s(s_tfull + 8u * (uint32_t)(g & 1), (g >> 1) & 1, s_abort, ERR_WAIT_EPILOGUE))) {
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_ld16(tcol + (g & 1) * GEMM_BN, va);
        }
        const int b = g & 1, cbuf = (g / kScGroups) & 1;
        const float sa = row_ok ? __half2float(sa_next) : 0.0f;
        if (g + 1 < G) sa_next = sa_row[g + 1];
        const float2 sa2 = make_float2(sa, sa);
        const uint32_t scs = s_scales + cbuf * GEMM_SC_BYTES + (g % kScGroups) * GEMM_BN * 4;
        const uint32_t taddr = tcol + b * GEMM_BN;
        tmem_wait_ld_regs(va);
        tmem_ld16(taddr + 16, vb);
        dequant16(va, scs, 0, sa2);
        tmem_wait_ld_regs(vb);
        tmem_ld16(taddr + kCd, va);
        dequant16(vb, scs + 64, 16, sa2);
        tmem_wait_ld_regs(va);
        tmem_ld16(taddr + kCd + 16, vb);
        dequant16(va, scs + 4 * kCd, 32, sa2);
        tmem_wait_ld_regs(vb);
        // every column of group g is in registers: hand the buffer back to the MMA
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive_s(s_tempty + 8u * (uint32_t)b);
          else mbar_arrive_remote(tmem_empty_remote + 8u * (uint32_t)b);
        }
        dequant16(vb, scs + 4 * kCd + 64, 48, sa2);
        __syncwarp();
        if (lane == 0 && (g % kScGroups == kScGroups - 1 || g == G - 1))
          mbar_arrive_s(s_empty_sc + 8u * (uint32_t)cbuf);
      }
      if (!ok) tmem_wait_ld();  // no TMEM load stays in flight

  #pragma unroll
      for (int j = 0; j < 32; ++j) {
        acc[2 * j] = acc2[j].x;
        acc[2 * j + 1] = acc2[j].y;
      }

    }
    // LoRA bypass deltas (the slots hold consecutive columns: 64 from
    // n0 + 64 cq, or 32 gate + 32 up columns from n0 + 32 cq for SwiGLU)
    if (LORA && ok && row_ok && (S.lt || S.lt2)) {
      const int c0 = n0 + ca;
      if (pairw) {
        if (S.lt) lora_delta32(acc, S.lt + (int64_t)row * S.lr, S.lup + (int64_t)c0 * S.lr, S.lr, S.ls);
        if (S.lt2)
          lora_delta32(acc + 32, S.lt2 + (int64_t)row * S.lr2, S.lup2 + (int64_t)c0 * S.lr2, S.lr2, S.ls2);
      } else if (S.lt && c0 < S.n) {
        lora_delta32(acc, S.lt + (int64_t)row * S.lr, S.lup + (int64_t)c0 * S.lr, S.lr, S.ls);
        lora_delta32(acc + 32, S.lt + (int64_t)row * S.lr, S.lup + (int64_t)(c0 + 32) * S.lr, S.lr, S.ls);
      }
    }
    // ---------------------------------------------------- final epilogue
    // CTA-uniform decision: every epilogue warp reaches this barrier, then all
    // of them see the same abort flag (the pair-exchanging paths have more).
    epi_barrier();
    ok = ok && (*abort_flag == 0);
    // Exchange space: the W stages are idle once every MMA has completed.
    float* xch = reinterpret_cast<float*>(smem + GEMM_OFF_W);
    if (ok) {
      const int col0 = n0 + cq * 64;  // first segment column of this thread (non-SwiGLU kinds)
      const bool col_ok = pairw || col0 < S.n;
      if (S.kind == SEG_F32 || S.kind == SEG_F32_SCATTER) {
        // The tile goes through shared memory so that every warp store covers
        // 512 contiguous bytes of one row: row-per-lane stores would send one
        // 16-byte transaction per lane, which NVLink (the scatter's peer
        // stores) carries far below its bandwidth.  Row stride 260 floats
        // keeps the 16-byte writes of 8 consecutive rows on distinct banks.
        float* trow = xch + rloc * 260 + cq * 64;
#pragma unroll
        for (int i = 0; i < 64; i += 4)
          *reinterpret_cast<float4*>(trow + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
        epi_barrier();
        const int ew = warp - 4;  // epilogue warp 0..15: rows ew, ew + 16, ...
        const int vc = min(GEMM_BN, S.n - n0);  // valid columns of this tile
        for (int rr = ew; rr < GEMM_BM; rr += GEMM_EPI_WARPS) {
          const int grow = m0 + rr;
          if (grow >= p.M) break;
          float* o;
          if (S.kind == SEG_F32) {
            o = reinterpret_cast<float*>(S.out) + (int64_t)grow * S.ld + n0;
          } else {
            const int dest = grow / p.scatter_chunk;
            o = p.peer[dest] +
                ((int64_t)p.scatter_rank * p.scatter_chunk + (grow - dest * p.scatter_chunk)) * S.ld + n0;
          }
          const float* src = xch + rr * 260;
#pragma unroll
          for (int h = 0; h < GEMM_BN; h += 128) {
            const int c = h + 4 * lane;
            if (c < vc) *reinterpret_cast<float4*>(o + c) = *reinterpret_cast<const float4*>(src + c);
          }
        }

      } else if (S.kind == SEG_BF16 || S.kind == SEG_SIGMOID) {
        if (row_ok && col_ok) {
          if (S.kind == SEG_SIGMOID) {
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = sigmoid_contract(bf16_round(acc[i]));
          }
          store_bf16x64(reinterpret_cast<__nv_bfloat16*>(S.out) + (int64_t)row * S.ld + col0, acc);
        }
      } else if (S.kind == SEG_RESIDUAL) {
        if (row_ok && col_ok) {
          const int bidx = row / p.length;
          const __nv_bfloat16* gt = p.gate + (int64_t)bidx * S.n + col0;
          const __nv_bfloat16* rs = p.resid + (int64_t)row * S.ld + col0;
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(S.out) + (int64_t)row * S.ld + col0;
#pragma unroll
          for (int i = 0; i < 64; i += 8) {
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
      } else if (S.kind == SEG_QKNORM) {
        // A head (128 columns) spans the warp pair (cq even: columns 0-63,
        // cq odd: 64-127).  Reduction order of kernels/joint_projection.cu:141-146:
        // lane l of the reference holds columns 4l..4l+3, then a shfl_down tree.
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = bf16_round(acc[i]);
        float part[16];
#pragma unroll
        for (int l = 0; l < 16; ++l) {
          float s2 = 0.0f;
#pragma unroll
          for (int j = 0; j < 4; ++j) s2 = __fmaf_rn(acc[4 * l + j], acc[4 * l + j], s2);
          part[l] = s2;
        }
        float* pbuf = xch + ((cq >> 1) * 128 + rloc) * 17;  // per (head, row): 16 partials + inv
        if (cq & 1) {
#pragma unroll
          for (int l = 0; l < 16; ++l) pbuf[l] = part[l];
        }
        epi_barrier();
        if (!(cq & 1)) {
          // tree step 16: reference lane l (< 16) adds lane l + 16 (the odd warp's partial l)
#pragma unroll
          for (int l = 0; l < 16; ++l) part[l] = __fadd_rn(part[l], pbuf[l]);
#pragma unroll
          for (int off = 8; off; off >>= 1)
#pragma unroll
            for (int l = 0; l < off; ++l) part[l] = __fadd_rn(part[l], part[l + off]);
          pbuf[16] = __frsqrt_rn(__fadd_rn(__fmul_rn(part[0], 0.0078125f), S.eps));
        }
        epi_barrier();
        const float inv = pbuf[16];
        if (row_ok && col_ok) {
          const int token = row % p.length;
          const int hc0 = (cq & 1) * 64;  // column of this thread's first value within the head
          const float* f = p.freqs + (int64_t)token * 256 + 2 * hc0;
          const float* nw = S.normw + hc0;
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(S.out) + (int64_t)row * S.ld + col0;
#pragma unroll
          for (int i = 0; i < 64; i += 8) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const int c = i + j;
              const float a = bf16_round(__fmul_rn(__fmul_rn(acc[c], inv), __fadd_rn(nw[c], 1.0f)));
              const float bb = bf16_round(__fmul_rn(__fmul_rn(acc[c + 1], inv), __fadd_rn(nw[c + 1], 1.0f)));
              const float4 fr = __ldg(reinterpret_cast<const float4*>(f + 2 * c));
              const float o0 = __fmaf_rn(fr.x, a, __fmul_rn(fr.y, bb));
              const float o1 = __fmaf_rn(fr.z, a, __fmul_rn(fr.w, bb));
              w[j / 2] = pack_bf16x2(o0, o1);
            }
            *reinterpret_cast<uint4*>(o + i) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      } else if (pairw) {
        // acc[0..31]: gate, acc[32..63]: up of output columns 32*cq .. +31 of
        // this tile's 128 (SwiGLU rounding of kernels/joint_projection.cu:94-97).
        float hv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float gv = bf16_round(acc[i]);
          const float av = bf16_round(silu_contract(gv));
          hv[i] = bf16_round(__fmul_rn(av, bf16_round(acc[32 + i])));
        }
        if (S.kind == SEG_SWIGLU_BF16) {
          if (row_ok) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(S.out) + (int64_t)row * S.ld + n0 + 32 * cq;
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(o + i) =
                  make_uint4(pack_bf16x2(hv[i], hv[i + 1]), pack_bf16x2(hv[i + 2], hv[i + 3]),
                             pack_bf16x2(hv[i + 4], hv[i + 5]), pack_bf16x2(hv[i + 6], hv[i + 7]));
          }
        } else {
          // H128 of the row's 128 outputs, held 32 per thread by the four
          // column quarters: stages 2, 4, 8, 1, 16 in registers, then 32
          // (partner quarter cq^1) and 64 (cq^2) through shared memory.
#pragma unroll
          for (int st = 0; st < 5; ++st) {
            const int lh = hadamard_stage_bit(st);
            const int h = 1 << lh;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int lo = ((i >> lh) << (lh + 1)) | (i & (h - 1));
              const float x0 = hv[lo], x1 = hv[lo + h];
              hv[lo] = __fadd_rn(x0, x1);
              hv[lo + h] = __fsub_rn(x0, x1);
            }
          }
#pragma unroll
          for (int xs = 0; xs < 2; ++xs) {
            const int bit = 1 << xs;  // partner quarter cq ^ bit: output distance 32 << xs
            float* mine = xch + xs * kSwXch + (cq * 128 + rloc) * 33;
            const float* other = xch + xs * kSwXch + ((cq ^ bit) * 128 + rloc) * 33;
#pragma unroll
            for (int i = 0; i < 32; ++i) mine[i] = hv[i];
            epi_barrier();
            const bool upper = (cq & bit) != 0;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float lo = upper ? other[i] : hv[i];
              const float hi = upper ? hv[i] : other[i];
              hv[i] = upper ? __fsub_rn(lo, hi) : __fadd_rn(lo, hi);
            }
          }
          float amax = 0.0f;
#pragma unroll
          for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(hv[i]));
          float* gmax = xch + 2 * kSwXch + rloc * 4;
          gmax[cq] = amax;
          epi_barrier();
          amax = fmaxf(fmaxf(gmax[0], gmax[1]), fmaxf(gmax[2], gmax[3]));
          const QuantGroup qg = quant_group(amax);
          const int grp = n0 / 128;  // output group (128 columns) index
          if (row_ok) {
            if (cq == 0) S.out_scale[(int64_t)row * (S.n / 128) + grp] = qg.scale;
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t bits8[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) bits8[e] = quant_bits(hv[8 * j + e], qg.c, qg.clamp);
              w[j] = pack8_codes(bits8);
            }
            uint8_t* orow = reinterpret_cast<uint8_t*>(S.out) + (int64_t)row * S.ld;
            if (S.kind == SEG_SWIGLU_E4M3) {
              // the same 32 codes as e4m3 bytes, column order
              uint4 lo, hi;
              unpack_chunk(make_uint4(w[0], w[1], w[2], w[3]), lo, hi);
              *reinterpret_cast<uint4*>(orow + grp * 128 + cq * 32) = lo;
              *reinterpret_cast<uint4*>(orow + grp * 128 + cq * 32 + 16) = hi;
            } else {
              *reinterpret_cast<uint4*>(orow + grp * 64 + cq * 16) = make_uint4(w[0], w[1], w[2], w[3]);
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
      // (a stage's full barrier also waits for unpacker arrivals, so only
      // the transaction bytes are certain: drain with a bounded wait)
      if (!PW)
        for (int g = (issued_w > GEMM_STAGES ? issued_w - GEMM_STAGES : 0); g < issued_w; ++g)
          mbar_drain(&full_s[g % GEMM_STAGES], (g / GEMM_STAGES) & 1);
      for (int g = (issued_pa > GEMM_PSTAGES ? issued_pa - GEMM_PSTAGES : 0); g < issued_pa; ++g)
        mbar_drain(&full_pa[g % GEMM_PSTAGES], (g / GEMM_PSTAGES) & 1);
    }
    if (BYTEA && warp == 2 && lane == 0)
      for (int g = (issued_pa > GEMM_STAGES ? issued_pa - GEMM_STAGES : 0); g < issued_pa; ++g)
        mbar_drain(&full_s[g % GEMM_STAGES], (g / GEMM_STAGES) & 1);
    if (BYTEA ? (warp == 3 && lane == 0) : (warp == 0 && lane == 1))
      for (int c = (issued_sc > 2 ? issued_sc - 2 : 0); c < issued_sc; ++c)
        mbar_drain(&full_sc[c & 1], (c >> 1) & 1);
    if (warp == 1 && lane == 0 && issued_mma > 0) {
      const int g = issued_mma - 1;
      if (REF) mbar_drain(&tmem_full[0], 0);
      else mbar_drain(&tmem_full[g & 1], (g >> 1) & 1);
    }
    if (PW && warp == 0 && lane == 0)
      for (int g = (issued_w > GEMM_PSTAGES ? issued_w - GEMM_PSTAGES : 0); g < issued_w; ++g)
        mbar_drain(&full_pw[g % GEMM_PSTAGES], (g / GEMM_PSTAGES) & 1);
  }
  tc_fence_before();
  __syncthreads();
  // Scatter: the owner rank reads its slots after a stream-ordered barrier
  // that follows this kernel; one system-scope fence per CTA (cumulative over
  // the CTA's stores through the barrier above) publishes them.
  if (p.scatter_chunk > 0 && threadIdx.x == 0) __threadfence_system();
  // The leader's MMAs (which read the peer's shared memory) are complete and
  // no arrival from one CTA to the other is in flight once both get here.
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace k2b
