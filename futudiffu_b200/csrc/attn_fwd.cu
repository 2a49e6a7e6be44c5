// Quantized attention forward (A5/A6) on tcgen05.
//
// Reference semantics: _sage_attn_fwd_int8qk_bf16pv_masked_lse and siblings,
// src/futudiffu/sage_kernels.py:1379-1477 (production), :592-798 (int8
// unmasked), :107-315 (fp8 QK), :1037-1168 (fp8 PV).  Per query row:
//   L[n]  = S[n] * q_desc * k_desc[n]            (log2 domain, sm_scale folded)
//   online softmax over KV tiles: m, l, O with exp2, LSE = m + log2(l),
//   out   = O / l.
//
// CTA = one 128-row Q tile of one (b, h); 10 warps:
//   warps 0-7  softmax: two threads per query row (TMEM lane), 64 keys each.
//              Read S from TMEM, scale, row max (exchanged with the partner
//              thread), exp2, row sum, write P to shared memory; rescale their
//              half of the O row in TMEM when the running max moves.
//   warp 8     TMA producer: Q once, then K (+ per-token K scales) and V
//              tiles of 128 keys into K and V rings (2 stages each for e4m3 V,
//              1 each for bf16 V); a K stage is released when its QK^T is
//              done, a V stage when its PV is done.
//   warp 9     MMA issuer: S = Q K^T (kind::i8 -> s32, or kind::f8f6f4 -> f32)
//              and O += P V (kind::f8f6f4 e4m3, or kind::f16 bf16).
// TMEM: S at columns [0,128), O at [128,256).  Two CTAs fit on one SM (the
// bf16-V variant by keeping one K and one V stage: 102 KiB of shared memory), so
// one CTA's softmax overlaps the other's MMAs; inside a CTA the next S = Q K^T is
// issued as soon as the softmax has pulled S into registers.
//
// Running-max threshold: O is rescaled only when a row max grows by more
// than TAU (log2 units) over the reference max used for exp2, so P <= 2^TAU
// (TAU = 8 for bf16 P, stored as is; TAU = 2 for e4m3 P, encoded as
// P8 = e4m3(p * 448 / 4) and undone in the epilogue).  Results equal the reference online
// softmax up to fp32 rounding (exp2 is shift-exact in bf16 / e4m3 up to
// rounding of the argument).
#include "fd_act.cuh"
#include "fd_host.h"

namespace fd {
namespace attn {

constexpr int BQ = 128;   // query rows per CTA
constexpr int BKV = 128;  // keys per KV tile
constexpr int HD = 128;
// K and V pipeline stages: 2 with e4m3 V (16 KiB per V tile); 1 with bf16 V
// (32 KiB) so that two CTAs still fit on one SM.
constexpr int kv_stages(int pv) { return pv == FD_PV_BF16 ? 1 : 2; }
// Per-token K scale slots: tile i uses slot i % (stages + 2).  The K stage of tile
// i is free once QK^T(i - stages) is done, which was issued after the softmax of
// tile i - stages - 1 released S, i.e. after the softmax of tile i - stages - 2
// (the previous user of the slot) had finished reading its scales.
constexpr int kd_slots(int pv) { return kv_stages(pv) + 2; }
constexpr int NUM_SOFTMAX_WARPS = 8;  // two threads per query row, 64 keys each
constexpr int WARP_TMA = 8, WARP_MMA = 9;
constexpr int NUM_THREADS = 320;
// Rescale threshold (log2 units): bf16 P keeps full relative precision at any
// scale, so a wide threshold (O rescaled rarely) is free; e4m3 P must map
// p <= 2^TAU onto 448, so a narrow one keeps small probabilities normal.
template <int PV>
struct PScale {
  static constexpr float TAU = PV == FD_PV_FP8 ? 2.0f : 8.0f;
  static constexpr float SCALE = PV == FD_PV_FP8 ? 448.0f / 4.0f : 1.0f;
  static constexpr float LOG2_SCALE = PV == FD_PV_FP8 ? 6.8073549220576041f : 0.0f;  // log2(112)
};

FD_DEV float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// max of 64 consecutive values with four independent 3-input chains
FD_DEV float max_reduce64(const float* x) {
  float m0 = max3(x[0], x[1], x[2]), m1 = max3(x[3], x[4], x[5]);
  float m2 = max3(x[6], x[7], x[8]), m3 = max3(x[9], x[10], x[11]);
#pragma unroll
  for (int c = 12; c < 60; c += 8) {
    m0 = max3(m0, x[c], x[c + 1]);
    m1 = max3(m1, x[c + 2], x[c + 3]);
    m2 = max3(m2, x[c + 4], x[c + 5]);
    m3 = max3(m3, x[c + 6], x[c + 7]);
  }
  m0 = max3(m0, x[60], x[61]);
  m1 = max3(m1, x[62], x[63]);
  return fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
}

template <int PV>
struct Smem {
  static constexpr bool PT = PV == FD_PV_FP8_TILE;
  static constexpr int KST = kv_stages(PV);
  static constexpr int KDS = kd_slots(PV);
  static constexpr uint32_t Q_BYTES = BQ * HD;                           // int8/e4m3 codes
  static constexpr uint32_t K_BYTES = BKV * HD;
  static constexpr uint32_t V_BYTES = BKV * HD * (PV == FD_PV_BF16 ? 2 : 1);
  static constexpr uint32_t P_BYTES = BQ * BKV * (PV == FD_PV_BF16 ? 2 : 1);
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + KST * K_BYTES;
  static constexpr uint32_t OFF_P = OFF_V + KST * V_BYTES;
  static constexpr uint32_t OFF_KD = OFF_P + P_BYTES;                    // KDS x 128 f32 (per-token K)
  static constexpr uint32_t OFF_VD = OFF_KD + KDS * 512;                 // 128 f32
  static constexpr uint32_t OFF_VDT = OFF_VD + 512;                      // PT: KST x [2][128] f32 tile V scales
  static constexpr uint32_t OFF_PX = OFF_VDT + (PT ? KST * 1024 : 0);    // PT: [2][2][128] f32 P descale / sum
  static constexpr uint32_t OFF_RED = OFF_PX + (PT ? 2048 : 0);          // row max / sum exchange
  static constexpr uint32_t OFF_BAR = OFF_RED + (2 * 2 * 128 + 2 * 128) * 4;
  static constexpr uint32_t RAW = OFF_BAR + 256 + 1024;                 // + barriers, align slack
  // PT: one CTA per SM (its 512 TMEM columns are the whole TMEM)
  static constexpr uint32_t TOTAL = PT && RAW < 120 * 1024 ? 120 * 1024 : RAW;
};

struct Params {
  const float* q_desc;
  const float* k_desc;
  const float* v_desc;
  const uint8_t* mask;
  int64_t mask_bh_stride;
  __nv_bfloat16* out;
  float* lse;
  int N;
  int n_kv_tiles;
  int nkb64;       // ceil(N/64): mask columns
  int q_gran;
  int64_t q_desc_stride;
  int64_t k_desc_stride;
  int64_t out_heads;  // 0: out is (BH, N, 128); H > 0: out is (BH / H, N, H, 128)
  // Quantised output (qout != nullptr, out_heads = H): each row's 128 head values
  // are one 1 x 128 group of the output linear's input, written as e4m3 codes +
  // an fp32 dequant scale.  Rows n < split go to region 0, rows n >= split to
  // region 1; in region r, sample b's row n sits at row b * rows_r + (n - start_r)
  // with `qstride[r]` code bytes and `sstride[r]` scales per row.
  uint8_t* qout[2];
  float* qscale[2];
  int64_t qstride[2];
  int64_t sstride[2];
  int split;
};

FD_DEV void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

FD_DEV bool tile_valid(const Params& p, int bh, int qb, int j) {
  if (!p.mask) return true;
  const uint8_t* m = p.mask + (int64_t)bh * p.mask_bh_stride + (int64_t)qb * p.nkb64;
  const uint8_t a = m[2 * j];
  const uint8_t b = (2 * j + 1 < p.nkb64) ? m[2 * j + 1] : 0;
  return (a | b) != 0;
}

FD_DEV void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > FD_WAIT_NS) {
      atomicOr(&g_status, FD_STATUS_TIMEOUT);
      return;
    }
  }
}

// Four f32 -> four e4m3 in one word (keys in byte order), RNE with saturation.
FD_DEV uint32_t f32x4_to_e4m3x4(float a, float b, float c, float d) {
  uint32_t r;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n\t"
      "mov.b32 %0, {lo, hi};\n\t}"
      : "=r"(r)
      : "f"(a), "f"(b), "f"(c), "f"(d));
  return r;
}

// INT8 QK^T scores are accumulated on top of the bit pattern of 1.5*2^23
// (S_BIAS_BITS, written into the S columns before every QK^T): |s| <= 128*127*127
// < 2^22, so the s32 accumulator holds exactly the bits of the float 1.5*2^23 + s.
// The softmax then reads scores as floats with no integer conversion: the row
// max is a float max of biased values, and s = biased - 1.5*2^23 exactly.
constexpr uint32_t S_BIAS_BITS = 0x4B400000u;
constexpr float S_BIAS = 12582912.0f;  // 1.5 * 2^23

// Pass 1 over 64 keys (two 32-key chunks): the maximum score.  Per-block K:
// the maximum of the raw scores (still biased for INT8; the 64 keys share one
// factor, applied by the caller); per-token K: max_n(s * k_desc[n]), times
// q_desc by the caller (q_desc > 0).  The row maximum only sets the exp2 offset
// (the lazy-rescale reference), so its last-bit rounding does not reach P.
template <int QK, int KG, bool FULL>
FD_DEV float chunk_max(const uint32_t (&r)[64], int col0, int N, bool half_ok, float qd, const float* kd) {
  float x[64];
#pragma unroll
  for (int e = 0; e < 64; e += 2) {
    x[e] = __uint_as_float(r[e]);
    x[e + 1] = __uint_as_float(r[e + 1]);
    if (KG == FD_GRAN_TOKEN) {
      uint64_t v = pk(x[e], x[e + 1]);
      if (QK == FD_QK_INT8) v = add2(v, pk(-S_BIAS, -S_BIAS));
      unpk(mul2(v, pk(kd[e], kd[e + 1])), x[e], x[e + 1]);
    }
  }
  if (!FULL) {
#pragma unroll
    for (int e = 0; e < 64; ++e)
      if (!(half_ok && col0 + e < N)) x[e] = -INFINITY;
  }
  return max_reduce64(x);
}

// Pass 2 over one 32-key chunk: P = exp2(L + nb) written into the shared-memory
// P tile (128-byte swizzled, K-major) at 32-key group g of the row; returns the
// chunk's sum of P.  nb folds in -(m_ref - log2 SCALE).
template <int QK, int KG, int PV, bool FULL>
FD_DEV float chunk_exp_store(const uint32_t (&r)[32], int col0, int N, bool half_ok, float qd,
                             const float* kd, float c, float nb, uint8_t* sP, int row, int g) {
  float a[32];
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    uint64_t v = pk(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
    if (KG == FD_GRAN_BLOCK) {
      v = fma2(v, pk(c, c), pk(nb, nb));  // nb carries -S_BIAS * c for INT8
    } else {
      // ((s * q_desc) * k_desc) + nb with the last two steps fused.  INT8: the
      // score bias is removed inside the first FMA, (s + B) * q_desc - B * q_desc:
      // the product is exact inside the FMA, so the only added error is the
      // rounding of B * q_desc (about q_desc / 4, against scores of order 10^3 q_desc)
      if (QK == FD_QK_INT8) {
        const float nbq = -S_BIAS * qd;
        v = fma2(fma2(v, pk(qd, qd), pk(nbq, nbq)), pk(kd[e], kd[e + 1]), pk(nb, nb));
      } else {
        v = fma2(mul2(v, pk(qd, qd)), pk(kd[e], kd[e + 1]), pk(nb, nb));
      }
    }
    unpk(v, a[e], a[e + 1]);
    if (!FULL) {
      if (!(half_ok && col0 + e < N)) a[e] = -INFINITY;
      if (!(half_ok && col0 + e + 1 < N)) a[e + 1] = -INFINITY;
    }
  }
  if (PV == FD_PV_FP8) {
    // f32 exp2 (one MUFU op per key; the f16x2 form costs the same MUFU work plus
    // packing), sum in f32 pairs, e4m3 pairs packed four keys per word
    float pv[32];
    uint64_t acc = pk(0.f, 0.f);
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      pv[e] = ex2_approx(a[e]);
      pv[e + 1] = ex2_approx(a[e + 1]);
      acc = add2(acc, pk(pv[e], pv[e + 1]));
    }
    // 32 keys = two 16-byte chunks (2g, 2g+1) of the 128-byte e4m3 P row
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int e = 16 * k + 4 * q;
        w[q] = f32x4_to_e4m3x4(pv[e], pv[e + 1], pv[e + 2], pv[e + 3]);
      }
      *reinterpret_cast<uint4*>(sP + row * 128 + (((2 * g + k) ^ (row & 7)) << 4)) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
    float s0, s1;
    unpk(acc, s0, s1);
    return s0 + s1;
  } else {
    uint64_t acc = pk(0.f, 0.f);
    uint32_t w[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const float p0 = ex2_approx(a[2 * u]), p1 = ex2_approx(a[2 * u + 1]);
      acc = add2(acc, pk(p0, p1));
      w[u] = pack_bf16x2(p0, p1);
    }
    // 32 keys = four 16-byte chunks of the 128-byte bf16 panel row (keys 64h..64h+63)
    const int panel = g >> 1;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int ch = (g & 1) * 4 + k;
      *reinterpret_cast<uint4*>(sP + panel * (BQ * 128) + row * 128 + ((ch ^ (row & 7)) << 4)) =
          make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
    }
    float s0, s1;
    unpk(acc, s0, s1);
    return s0 + s1;
  }
}

// PT mode: chunk_max over 32 keys (the scores as in chunk_max)
template <int QK, int KG, bool FULL>
FD_DEV float chunk_max32(const uint32_t (&r)[32], int col0, int N, bool half_ok, const float* kd) {
  float m = -INFINITY;
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    float x0 = __uint_as_float(r[e]), x1 = __uint_as_float(r[e + 1]);
    if (KG == FD_GRAN_TOKEN) {
      uint64_t v = pk(x0, x1);
      if (QK == FD_QK_INT8) v = add2(v, pk(-S_BIAS, -S_BIAS));
      unpk(mul2(v, pk(kd[e], kd[e + 1])), x0, x1);
    }
    if (!FULL) {
      if (!(half_ok && col0 + e < N)) x0 = -INFINITY;
      if (!(half_ok && col0 + e + 1 < N)) x1 = -INFINITY;
    }
    m = max3(m, x0, x1);
  }
  return m;
}

// PT mode: p = exp2(L + nb) of one 32-key chunk into p[32] (the arithmetic of
// chunk_exp_store, without the store); keys out of range give 0.
template <int QK, int KG, bool FULL>
FD_DEV void chunk_p(const uint32_t (&r)[32], int col0, int N, bool half_ok, float qd, const float* kd, float c,
                    float nb, float (&pout)[32]) {
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    uint64_t v = pk(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
    if (KG == FD_GRAN_BLOCK) {
      v = fma2(v, pk(c, c), pk(nb, nb));
    } else if (QK == FD_QK_INT8) {
      const float nbq = -S_BIAS * qd;
      v = fma2(fma2(v, pk(qd, qd), pk(nbq, nbq)), pk(kd[e], kd[e + 1]), pk(nb, nb));
    } else {
      v = fma2(mul2(v, pk(qd, qd)), pk(kd[e], kd[e + 1]), pk(nb, nb));
    }
    float a0, a1;
    unpk(v, a0, a1);
    if (!FULL) {
      if (!(half_ok && col0 + e < N)) a0 = -INFINITY;
      if (!(half_ok && col0 + e + 1 < N)) a1 = -INFINITY;
    }
    pout[e] = ex2_approx(a0);
    pout[e + 1] = ex2_approx(a1);
  }
}

// QK: FD_QK_INT8 / FD_QK_FP8; KG: k granularity; PV: FD_PV_BF16 / FD_PV_FP8 / FD_PV_FP8_TILE
template <int QK, int KG, int PV>
__global__ void __launch_bounds__(NUM_THREADS, PV == FD_PV_FP8_TILE ? 1 : 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
  using SM = Smem<PV>;
  constexpr int KST = SM::KST, KDS = SM::KDS;
  constexpr uint32_t TMEM_COLS = PV == FD_PV_FP8_TILE ? 512 : 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + SM::OFF_Q;
  uint8_t* sK = smem + SM::OFF_K;
  uint8_t* sV = smem + SM::OFF_V;
  uint8_t* sP = smem + SM::OFF_P;
  float* sKd = reinterpret_cast<float*>(smem + SM::OFF_KD);
  float* sVd = reinterpret_cast<float*>(smem + SM::OFF_VD);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::OFF_BAR);
  uint64_t* bQ = bars + 0;
  uint64_t* bKfull = bars + 1;            // [KST]
  uint64_t* bVfull = bars + 1 + KST;      // [KST]
  uint64_t* bKempty = bars + 1 + 2 * KST; // [KST] QK^T done with the K stage
  uint64_t* bVempty = bars + 1 + 3 * KST; // [KST] PV done with the V stage
  uint64_t* bKdfull = bars + 1 + 4 * KST; // [KDS] per-token K scales of tile i in slot i % KDS
  uint64_t* bSfull = bKdfull + KDS;
  uint64_t* bSfree = bSfull + 1;
  uint64_t* bPfull = bSfull + 2;
  uint64_t* bOready = bSfull + 3;
  uint64_t* bDrain = bSfull + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bSfull + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int qb = blockIdx.x;
  const int bh = blockIdx.y;
  const int q0 = qb * BQ;

  if (threadIdx.x == 0) {
    mbar_init(bQ, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(&bKfull[s], 1);
      mbar_init(&bVfull[s], 1);
      mbar_init(&bKempty[s], 1);
      // PT: the V stage (codes and tile scales) is released by the softmax warps
      // after they have promoted its PV; otherwise by the PV MMAs' commit
      mbar_init(&bVempty[s], PV == FD_PV_FP8_TILE ? NUM_SOFTMAX_WARPS : 1);
    }
    for (int s = 0; s < KDS; ++s) mbar_init(&bKdfull[s], 1);
    mbar_init(bSfull, 1);
    mbar_init(bSfree, NUM_SOFTMAX_WARPS);
    mbar_init(bPfull, NUM_SOFTMAX_WARPS);
    mbar_init(bOready, 1);
    mbar_init(bDrain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // TMEM: S at [0, 128); O at [128, 256), or (PT) the two 64-key halves' PV
  // products at [128, 256) and [256, 384) (O then lives in registers)
  const uint32_t tS = tmem_base, tO = tmem_base + 128;
  const uint32_t tPV1 = tmem_base + 256;

  if (warp == WARP_TMA) {
    // ================================================================ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(bQ, SM::Q_BYTES);
      tma_load_3d(sQ, &tmQ, bQ, 0, q0, bh);
      uint32_t i = 0;
      uint32_t issued = 0, v_issued = 0;  // tiles whose K / V copies were issued
      for (int j = 0; j < p.n_kv_tiles; ++j) {
        if (!tile_valid(p, bh, qb, j)) continue;
        const uint32_t s = i % KST, use = i / KST;
        if (!mbar_wait(&bKempty[s], (use & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bKfull[s], SM::K_BYTES);
        tma_load_3d(sK + s * SM::K_BYTES, &tmK, &bKfull[s], 0, j * BKV, bh);
        if (KG == FD_GRAN_TOKEN) {
          const uint32_t ks = i % KDS;  // free: see kd_slots
          mbar_arrive_expect_tx(&bKdfull[ks], 512);
          bulk_load(sKd + ks * 128, p.k_desc + (int64_t)bh * p.k_desc_stride + (int64_t)j * BKV, 512,
                    &bKdfull[ks]);
        }
        ++i;
        issued = i;
        if (!mbar_wait(&bVempty[s], (use & 1) ^ 1, abort_flag)) break;
        if (PV == FD_PV_FP8_TILE) {
          // codes + the scales of the tile's one or two 64-row halves
          const int nh = (2 * j + 1 < p.nkb64) ? 2 : 1;
          mbar_arrive_expect_tx(&bVfull[s], SM::V_BYTES + nh * 512);
          tma_load_3d(sV + s * SM::V_BYTES, &tmV, &bVfull[s], 0, j * BKV, bh);
          bulk_load(reinterpret_cast<float*>(smem + SM::OFF_VDT) + s * 256,
                    p.v_desc + ((int64_t)bh * p.nkb64 + 2 * j) * HD, nh * 512, &bVfull[s]);
        } else if (PV == FD_PV_FP8) {
          mbar_arrive_expect_tx(&bVfull[s], SM::V_BYTES);
          tma_load_3d(sV + s * SM::V_BYTES, &tmV, &bVfull[s], 0, j * BKV, bh);
        } else {
          mbar_arrive_expect_tx(&bVfull[s], SM::V_BYTES);
          tma_load_3d(sV + s * SM::V_BYTES, &tmV, &bVfull[s], 0, j * BKV, bh);
          tma_load_3d(sV + s * SM::V_BYTES + BKV * 128, &tmV, &bVfull[s], 64, j * BKV, bh);
        }
        v_issued = i;
      }
      // drain: every stage's newest loads must have landed (the last tile's V
      // may not have been issued if its wait gave up)
      drain_wait(bQ, 0);
      for (uint32_t k = 0; k < (uint32_t)KST && k < issued; ++k) {
        const uint32_t last = issued - 1 - k;
        const uint32_t s = last % KST, ph = (last / KST) & 1;
        drain_wait(&bKfull[s], ph);
        if (v_issued > last) drain_wait(&bVfull[s], ph);
      }
      for (uint32_t k = 0; KG == FD_GRAN_TOKEN && k < (uint32_t)KDS && k < issued; ++k) {
        const uint32_t last = issued - 1 - k;
        drain_wait(&bKdfull[last % KDS], (last / KDS) & 1);
      }
    }
  } else if (warp == WARP_MMA) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk =
          QK == FD_QK_INT8 ? make_idesc(/*S32*/ 2, /*S8*/ 1, 1, 0, 0, BQ, BKV)
                           : make_idesc(/*F32*/ 1, /*E4M3*/ 0, 0, 0, 0, BQ, BKV);
      constexpr uint32_t idesc_pv =
          PV != FD_PV_BF16 ? make_idesc(1, /*E4M3*/ 0, 0, /*A K-major*/ 0, /*B MN-major*/ 1, BQ, HD)
                           : make_idesc(1, /*BF16*/ 1, 1, 0, 1, BQ, HD);
      const uint32_t aQ = smem_u32(sQ);
      bool ok = mbar_wait(bQ, 0, abort_flag);
      // list of valid tiles is re-derived here in the same order as the producer
      int jcur = -1;
      auto next_valid = [&](int from) {
        for (int j = from; j < p.n_kv_tiles; ++j)
          if (tile_valid(p, bh, qb, j)) return j;
        return p.n_kv_tiles;
      };
      auto issue_qk = [&](uint32_t i) -> bool {
        const uint32_t s = i % KST, use = i / KST;
        if (!mbar_wait(&bKfull[s], use & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t bK = smem_u32(sK + s * SM::K_BYTES);
#pragma unroll
        for (int k = 0; k < HD / 32; ++k) {
          const uint64_t ad = make_sdesc_sw128(aQ + k * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(bK + k * 32, 16, 1024);
          if (QK == FD_QK_INT8) mma_i8_ss(tS, ad, bd, idesc_qk, 1u);  // onto S_BIAS_BITS
          else mma_f8f6f4_ss(tS, ad, bd, idesc_qk, k > 0);
        }
        tc_commit(&bKempty[s]);  // the K stage is free once these MMAs are done
        tc_commit(bSfull);
        return true;
      };
      uint32_t i = 0;
      jcur = next_valid(0);
      // bSfree phase k completes when the softmax has refilled S for QK^T(k):
      // phase 0 after the initial fill, phase i + 1 once S(i) is in registers.
      if (ok && jcur < p.n_kv_tiles) ok = mbar_wait(bSfree, 0, abort_flag);
      if (ok && jcur < p.n_kv_tiles) {
        tc_fence_after();
        ok = issue_qk(0);
      }
      while (ok && jcur < p.n_kv_tiles) {
        const int jn = next_valid(jcur + 1);
        if (jn < p.n_kv_tiles) {
          if (!mbar_wait(bSfree, (i + 1) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          if (!issue_qk(i + 1)) { ok = false; break; }
        }
        const uint32_t s = i % KST, use = i / KST;
        if (!mbar_wait(bPfull, i & 1, abort_flag)) { ok = false; break; }
        if (!mbar_wait(&bVfull[s], use & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aP = smem_u32(sP);
        const uint32_t bV = smem_u32(sV + s * SM::V_BYTES);
        if (PV == FD_PV_FP8_TILE) {
          // each 64-key half into its own TMEM product (keys [64 h, 64 h + 64) of P
          // and rows [64 h, 64 h + 64) of V), promoted by the softmax warps
#pragma unroll
          for (int k = 0; k < BKV / 32; ++k) {
            const uint64_t ad = make_sdesc_sw128(aP + k * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(bV + k * 32 * 128, 16, 1024);
            mma_f8f6f4_ss(k < 2 ? tO : tPV1, ad, bd, idesc_pv, (k & 1) ? 1u : 0u);
          }
        } else if (PV == FD_PV_FP8) {
#pragma unroll
          for (int k = 0; k < BKV / 32; ++k) {
            const uint64_t ad = make_sdesc_sw128(aP + k * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(bV + k * 32 * 128, 16, 1024);
            mma_f8f6f4_ss(tO, ad, bd, idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
          }
        } else {
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k) {
            const uint64_t ad = make_sdesc_sw128(aP + (k >> 2) * (BQ * 128) + (k & 3) * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(bV + k * 16 * 128, BKV * 128, 1024);
            mma_f16_ss(tO, ad, bd, idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
          }
        }
        if (PV != FD_PV_FP8_TILE) tc_commit(&bVempty[s]);
        tc_commit(bOready);
        ++i;
        jcur = jn;
      }
      tc_commit(bDrain);
      drain_wait(bDrain, 0);
    }
  } else {
    // ================================================================ softmax (warps 0-7)
    // Two threads per query row: warp w owns row (w & 3) * 32 + lane (its TMEM lane
    // quadrant is w & 3) and key columns [64 h, 64 h + 64) of every tile, h = w >> 2.
    // The partners exchange row maxima through shared memory once per tile.
    const int quad = warp & 3, h = warp >> 2;
    const int row = quad * 32 + lane;
    const int qrow = q0 + row;
    const int cb = h * 64;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* red_max = reinterpret_cast<float*>(smem + SM::OFF_RED);  // [parity][half][128]
    float* red_l = red_max + 2 * 2 * 128;                           // [half][128]
    if (PV == FD_PV_FP8 && h == 0) sVd[row] = p.v_desc[(int64_t)bh * HD + row];
    // initial fill of this thread's S columns; the arrival releases QK^T(0)
    if (QK == FD_QK_INT8) {
      tmem_fill32(tS + lane_base + cb, S_BIAS_BITS);
      tmem_fill32(tS + lane_base + cb + 32, S_BIAS_BITS);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bSfree);
    named_bar_sync(1, NUM_SOFTMAX_WARPS * 32);
    const float qd = p.q_gran == FD_GRAN_TOKEN
                         ? p.q_desc[(int64_t)bh * p.q_desc_stride + (qrow < p.N ? qrow : 0)]
                         : p.q_desc[(int64_t)bh * p.q_desc_stride + qb];
    if constexpr (PV == FD_PV_FP8_TILE) {
    // ---------------------------------------------------------------- PT softmax
    // The reference's FP8-PV update, 64 keys at a time (sage_kernels.py:1124-1154):
    // thread h owns the 64-key half h of every 128-key tile, i.e. one reference
    // tile.  Per half: m_new = max(m, rowmax), alpha = exp2(m - m_new),
    // p = exp2(s - m_new), l = alpha l + sum p, P8 = e4m3(p * 448 / amax(p)),
    // o = alpha o + (P8 V8 * amax(p) / 448) * v_desc[tile, d].  O stays in
    // registers: thread h owns output columns [64 h, 64 h + 64).
    float* px = reinterpret_cast<float*>(smem + SM::OFF_PX);  // [0][h][row] P descale, [1][h][row] sum p
    const float* vdt = reinterpret_cast<const float*>(smem + SM::OFF_VDT);
    float o[64];
#pragma unroll
    for (int e = 0; e < 64; ++e) o[e] = 0.f;
    float m_run = -INFINITY, l = 0.f;
    float pa1 = 0.f, pa2 = 0.f, ppd0 = 0.f, ppd1 = 0.f;  // the previous tile's update factors
    bool ph1ok = false;
    uint32_t pstage = 0;
    // o = (o a1 + pv0 pd0 vd0) a2 + pv1 pd1 vd1 with the previous tile's products
    auto promote = [&](uint32_t iprev) -> bool {
      if (!mbar_wait(bOready, iprev & 1, abort_flag)) return false;
      tc_fence_after();
      const float* vd = vdt + pstage * 256 + cb;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t r0[16], r1[16];
        tmem_ld16(tO + lane_base + cb + 16 * cc, r0);
        tmem_ld16(tPV1 + lane_base + cb + 16 * cc, r1);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int c = 16 * cc + e;
          float x = __fmul_rn(o[c], pa1);
          x = __fadd_rn(x, __fmul_rn(__fmul_rn(__uint_as_float(r0[e]), ppd0), vd[c]));
          x = __fmul_rn(x, pa2);
          if (ph1ok) x = __fadd_rn(x, __fmul_rn(__fmul_rn(__uint_as_float(r1[e]), ppd1), vd[128 + c]));
          o[c] = x;
        }
      }
      // the tile's V codes and scales are used: release its V stage
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bVempty[pstage]);
      return true;
    };
    uint32_t i = 0;
    bool ok = true;
    for (int j = 0; j < p.n_kv_tiles && ok; ++j) {
      const int col0 = j * BKV + cb;
      const bool half_ok = col0 < p.N;
      const bool full = col0 + 64 <= p.N;
      if (!mbar_wait(bSfull, i & 1, abort_flag)) { ok = false; break; }
      if (KG == FD_GRAN_TOKEN) {
        if (!mbar_wait(&bKdfull[i % KDS], (i / KDS) & 1, abort_flag)) { ok = false; break; }
      }
      tc_fence_after();
      const float* kd = sKd + (i % KDS) * 128 + cb;
      float c = 0.f;
      if (KG == FD_GRAN_BLOCK) {
        const int kb = 2 * j + h;
        c = (kb < p.nkb64) ? p.k_desc[(int64_t)bh * p.k_desc_stride + kb] * qd : 0.f;
      }
      // ---- row maxima of the two halves
      float mloc = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t r[32];
        tmem_ld32(tS + lane_base + cb + 32 * cc, r);
        tmem_wait_ld();
        mloc = fmaxf(mloc, full ? chunk_max32<QK, KG, true>(r, col0 + 32 * cc, p.N, half_ok, kd + 32 * cc)
                                : chunk_max32<QK, KG, false>(r, col0 + 32 * cc, p.N, half_ok, kd + 32 * cc));
      }
      if (KG == FD_GRAN_BLOCK) {
        if (QK == FD_QK_INT8) mloc -= S_BIAS;
        mloc = mloc == -INFINITY ? -INFINITY : mloc * c;
      } else {
        mloc = mloc == -INFINITY ? -INFINITY : mloc * qd;
      }
      float* rm = red_max + (i & 1) * 256;
      rm[h * 128 + row] = mloc;
      named_bar_sync(2 + quad, 64);
      const float mx0 = h == 0 ? mloc : rm[row], mx1 = h == 1 ? mloc : rm[128 + row];
      const float m1 = fmaxf(m_run, mx0), m2 = fmaxf(m1, mx1);
      const float a1 = m_run == -INFINITY ? 0.f : ex2_approx(m_run - m1);
      const float a2 = m1 == -INFINITY ? 0.f : ex2_approx(m1 - m2);
      const float mh = h == 0 ? m1 : m2;
      // ---- the previous tile's PV (frees P, the PV products and its V stage)
      if (i > 0) {
        if (!promote(i - 1)) { ok = false; break; }
      }
      // ---- p of this half: absmax and sum first, then the e4m3 codes (p recomputed)
      const float nb0 = mh == -INFINITY ? 0.f : -mh;
      const float nb = (KG == FD_GRAN_BLOCK && QK == FD_QK_INT8) ? fmaf(-S_BIAS, c, nb0) : nb0;
      float pam = 0.f, psum = 0.f;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t r[32];
        float pv[32];
        tmem_ld32(tS + lane_base + cb + 32 * cc, r);
        tmem_wait_ld();
        if (full) chunk_p<QK, KG, true>(r, col0 + 32 * cc, p.N, half_ok, qd, kd + 32 * cc, c, nb, pv);
        else chunk_p<QK, KG, false>(r, col0 + 32 * cc, p.N, half_ok, qd, kd + 32 * cc, c, nb, pv);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          pam = fmaxf(pam, pv[e]);
          psum += pv[e];
        }
      }
      const float pinv = div_full(448.0f, fmaxf(pam, 1e-12f));
      const float pd = div_full(pam, 448.0f);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t r[32];
        float pv[32];
        tmem_ld32(tS + lane_base + cb + 32 * cc, r);
        tmem_wait_ld();
        if (QK == FD_QK_INT8) tmem_fill32(tS + lane_base + cb + 32 * cc, S_BIAS_BITS);
        if (cc == 1) {
          if (QK == FD_QK_INT8) tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bSfree);  // the tensor core may overwrite S now
        }
        if (full) chunk_p<QK, KG, true>(r, col0 + 32 * cc, p.N, half_ok, qd, kd + 32 * cc, c, nb, pv);
        else chunk_p<QK, KG, false>(r, col0 + 32 * cc, p.N, half_ok, qd, kd + 32 * cc, c, nb, pv);
        // 32 keys = two 16-byte chunks of the 128-byte e4m3 P row (chunk 4 h + 2 cc + k)
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          uint32_t w[4];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int e = 16 * k + 4 * q4;
            w[q4] = f32x4_to_e4m3x4(__fmul_rn(pv[e], pinv), __fmul_rn(pv[e + 1], pinv),
                                    __fmul_rn(pv[e + 2], pinv), __fmul_rn(pv[e + 3], pinv));
          }
          const int chunk = 4 * h + 2 * cc + k;
          *reinterpret_cast<uint4*>(sP + row * 128 + ((chunk ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      px[h * 128 + row] = pd;
      px[256 + h * 128 + row] = psum;
      named_bar_sync(2 + quad, 64);
      const float pd0 = px[row], pd1 = px[128 + row];
      l = __fadd_rn(__fmul_rn(a2, __fadd_rn(__fmul_rn(a1, l), px[256 + row])), px[384 + row]);
      m_run = m2;
      pa1 = a1;
      pa2 = a2;
      ppd0 = pd0;
      ppd1 = pd1;
      ph1ok = 2 * j + 1 < p.nkb64;
      pstage = i % KST;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bPfull);
      ++i;
    }
    if (ok && i > 0) ok = promote(i - 1);
    // ---- epilogue: out = o / l (bf16), LSE = m + log2(l)
    const bool row_ok = qrow < p.N;
    const float l_div = i > 0 ? l : 0.f;
    if (ok && row_ok && h == 0 && p.lse) p.lse[(int64_t)bh * p.N + qrow] = i > 0 ? m_run + log2f(l) : -INFINITY;
    if (ok && row_ok) {
      __nv_bfloat16* orow = p.out + ((int64_t)bh * p.N + qrow) * HD + cb;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) w[e] = pack_bf16x2(div_full(o[32 * cc + 2 * e], l_div), div_full(o[32 * cc + 2 * e + 1], l_div));
        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        dst[2] = make_uint4(w[8], w[9], w[10], w[11]);
        dst[3] = make_uint4(w[12], w[13], w[14], w[15]);
      }
    }
    } else {
    // l accumulates this thread's share of P in its stored scale (x PScale::SCALE)
    float m_ref = -INFINITY, l = 0.f;
    uint32_t i = 0;
    bool ok = true;
    for (int j = 0; j < p.n_kv_tiles && ok; ++j) {
      if (!tile_valid(p, bh, qb, j)) continue;
      const int col0 = j * BKV + cb;  // first key of this thread's half-tile
      bool my_half_ok = true, other_half_ok = true;
      if (p.mask) {
        const uint8_t* mr = p.mask + (int64_t)bh * p.mask_bh_stride + (int64_t)qb * p.nkb64;
        my_half_ok = (2 * j + h < p.nkb64) && mr[2 * j + h] != 0;
        other_half_ok = (2 * j + (h ^ 1) < p.nkb64) && mr[2 * j + (h ^ 1)] != 0;
      }
      // the whole half-tile is in range and unmasked: the common case, no selects
      const bool full = (col0 + 64 <= p.N) && my_half_ok;
      (void)other_half_ok;
      float c = 0.f;  // per-block K: logit factor of this thread's 64 keys
      if (KG == FD_GRAN_BLOCK) {
        const int kb = 2 * j + h;
        c = (kb < p.nkb64) ? p.k_desc[(int64_t)bh * p.k_desc_stride + kb] * qd : 0.f;
      }
      if (!mbar_wait(bSfull, i & 1, abort_flag)) { ok = false; break; }
      if (KG == FD_GRAN_TOKEN) {
        if (!mbar_wait(&bKdfull[i % KDS], (i / KDS) & 1, abort_flag)) { ok = false; break; }
      }
      tc_fence_after();
      const float* kd = sKd + (i % KDS) * 128 + cb;  // per-token K scales of this thread's keys
      // ---- pass 1: row max over this thread's 64 keys (two 32-key chunks from TMEM)
      float mloc;
      {
        uint32_t r[64];
        tmem_ld64(tS + lane_base + cb, r);
        tmem_wait_ld();
        mloc = full ? chunk_max<QK, KG, true>(r, col0, p.N, my_half_ok, qd, kd)
                    : chunk_max<QK, KG, false>(r, col0, p.N, my_half_ok, qd, kd);
      }
      if (KG == FD_GRAN_BLOCK) {
        if (QK == FD_QK_INT8) mloc -= S_BIAS;  // exact; -inf stays -inf
        mloc = mloc == -INFINITY ? -INFINITY : mloc * c;  // c >= 0
      } else {
        mloc = mloc == -INFINITY ? -INFINITY : mloc * qd;  // q_desc >= 0
      }
      float* rm = red_max + (i & 1) * 256;
      rm[h * 128 + row] = mloc;
      named_bar_sync(2 + quad, 64);
      const float mt = fmaxf(mloc, rm[(h ^ 1) * 128 + row]);
      // both partners see the same mt and m_ref, so they take the same decisions
      const bool need = mt > m_ref + PScale<PV>::TAU;
      const float m_new = need ? mt : m_ref;
      if (__any_sync(0xffffffffu, need)) {
        const float alpha = (m_ref == -INFINITY) ? 0.f : ex2_approx(m_ref - m_new);
        l *= alpha;
        if (i > 0) {
          // PV(i-1) must be complete before O is touched
          if (!mbar_wait(bOready, (i - 1) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          uint32_t r[16];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            tmem_ld16(tO + lane_base + cb + cc * 16, r);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st16(tO + lane_base + cb + cc * 16, r);
          }
          tmem_wait_st();
        }
        m_ref = m_new;
      }
      // exp2 argument: L - (m_ref - log2 SCALE), so ex2 yields P already in its stored scale
      const float nb0 = (m_ref == -INFINITY) ? 0.f : -(m_ref - PScale<PV>::LOG2_SCALE);
      // per-block INT8: fold the score bias into the offset, L + nb0 = b * c + (nb0 - S_BIAS * c)
      const float nb = (KG == FD_GRAN_BLOCK && QK == FD_QK_INT8) ? fmaf(-S_BIAS, c, nb0) : nb0;
      // P buffer is free once PV(i-1) has completed
      if (i > 0) {
        if (!mbar_wait(bOready, (i - 1) & 1, abort_flag)) { ok = false; break; }
      }
      // ---- pass 2: P = exp2(L + nb) into shared memory, row-sum into l
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t r[32];
        tmem_ld32(tS + lane_base + cb + 32 * cc, r);
        tmem_wait_ld();
        if (QK == FD_QK_INT8) tmem_fill32(tS + lane_base + cb + 32 * cc, S_BIAS_BITS);
        if (cc == 1) {
          if (QK == FD_QK_INT8) tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bSfree);  // the tensor core may overwrite S now
        }
        l += full ? chunk_exp_store<QK, KG, PV, true>(r, col0 + 32 * cc, p.N, my_half_ok, qd, kd + 32 * cc, c,
                                                      nb, sP, row, 2 * h + cc)
                  : chunk_exp_store<QK, KG, PV, false>(r, col0 + 32 * cc, p.N, my_half_ok, qd, kd + 32 * cc, c,
                                                       nb, sP, row, 2 * h + cc);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bPfull);
      ++i;
    }
    // ---------------------------------------------------------------- epilogue
    if (ok && i > 0) ok = mbar_wait(bOready, (i - 1) & 1, abort_flag);
    red_l[h * 128 + row] = l;
    named_bar_sync(2 + quad, 64);
    const float l_tot = l + red_l[(h ^ 1) * 128 + row];
    if (ok) tc_fence_after();
    const bool any = i > 0;
    // reference: LSE = m + log2(l) (tl.math.log2 == log2f), out = o / l (Triton f32 divide)
    const float lse_v = any ? m_ref + (log2f(l_tot) - PScale<PV>::LOG2_SCALE) : -INFINITY;
    const float l_div = any ? l_tot : 0.f;  // 0/0 -> NaN for rows that saw no key, as the reference
    const bool row_ok = qrow < p.N;
    if (ok && row_ok && h == 0 && p.lse) p.lse[(int64_t)bh * p.N + qrow] = lse_v;
    // this thread's 64 output values of chunk cc (32 each), O / l, as fp32
    auto load_out = [&](int cc, float (&o)[32]) {
      uint32_t r[32];
      if (any) {
        tmem_ld32(tO + lane_base + cb + cc * 32, r);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = 0u;
      }
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        float v = __uint_as_float(r[e]);
        if (PV == FD_PV_FP8) v *= sVd[cb + cc * 32 + e];  // O and l carry the P scale; V carries v_desc
        o[e] = div_full(v, l_div);
      }
    };
    if (p.qout[0]) {
      // Quantised output: O / l rounded to bf16 (the values the bf16 store would
      // hold), then the 1 x 128 quantiser over the row's 128 head values, which
      // two threads hold: codes and scale equal fp8_act_quant of the bf16 output.
      // Two TMEM passes (amax, then codes) keep the register count down; the
      // partner exchange runs whether or not this thread's waits succeeded.
      const int64_t b = bh / p.out_heads, hh = bh % p.out_heads;
      const int n = row_ok ? qrow : 0;
      const int rg = n < p.split ? 0 : 1;
      const int64_t rows_r = rg == 0 ? p.split : p.N - p.split;
      const int64_t qr = b * rows_r + (rg == 0 ? n : n - p.split);
      float amax = 0.f;
      if (ok) {
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          float o[32];
          load_out(cc, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(round_to_bf16(o[e])));
        }
      }
      red_max[h * 128 + row] = amax;
      named_bar_sync(2 + quad, 64);
      amax = fmaxf(amax, red_max[(h ^ 1) * 128 + row]);
      if (ok) {
        const float qm = quant_mult(amax);
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          float o[32];
          load_out(cc, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = round_to_bf16(o[e]);
          if (row_ok) {
            uint4* dst = reinterpret_cast<uint4*>(p.qout[rg] + qr * p.qstride[rg] + hh * HD + cb + cc * 32);
#pragma unroll
            for (int k = 0; k < 2; ++k)
              dst[k] = make_uint4(quant4(o[16 * k], o[16 * k + 1], o[16 * k + 2], o[16 * k + 3], qm),
                                  quant4(o[16 * k + 4], o[16 * k + 5], o[16 * k + 6], o[16 * k + 7], qm),
                                  quant4(o[16 * k + 8], o[16 * k + 9], o[16 * k + 10], o[16 * k + 11], qm),
                                  quant4(o[16 * k + 12], o[16 * k + 13], o[16 * k + 14], o[16 * k + 15], qm));
          }
        }
        if (row_ok && h == 0) p.qscale[rg][qr * p.sstride[rg] + hh] = dequant_scale(amax);
      }
    } else if (ok) {
      const int64_t orow_idx = p.out_heads == 0
                                   ? (int64_t)bh * p.N + (row_ok ? qrow : 0)
                                   : ((int64_t)(bh / p.out_heads) * p.N + (row_ok ? qrow : 0)) * p.out_heads +
                                         bh % p.out_heads;
      __nv_bfloat16* orow = p.out + orow_idx * HD + cb;
      // tcgen05.ld is warp-collective: every lane loads, only valid rows store
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float o[32];
        load_out(cc, o);
        if (row_ok) {
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) w[e] = pack_bf16x2(o[2 * e], o[2 * e + 1]);
          uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
          dst[2] = make_uint4(w[8], w[9], w[10], w[11]);
          dst[3] = make_uint4(w[12], w[13], w[14], w[15]);
        }
      }
    }
    }  // PV != FD_PV_FP8_TILE
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == WARP_MMA) tmem_dealloc(tmem_base, TMEM_COLS);
}

template <int QK, int KG, int PV>
static int launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const Params& p,
                  int BH, cudaStream_t st) {
  auto kern = attn_fwd_kernel<QK, KG, PV>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<PV>::TOTAL);
    if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "attn smem attribute: %s", cudaGetErrorString(e));
    attr_done = true;
  }
  dim3 grid((unsigned)((p.N + BQ - 1) / BQ), (unsigned)BH);
  kern<<<grid, NUM_THREADS, Smem<PV>::TOTAL, st>>>(tq, tk, tv, p);
  return check_launch("sage_attn_fwd");
}

}  // namespace attn
}  // namespace fd

using namespace fd;

int64_t fd_desc_stride(int64_t N, int gran, int rows_per_block);

struct QuantOut {
  void* codes[2];
  float* scales[2];
  int64_t code_stride[2];
  int64_t scale_stride[2];
  int64_t split;
};

static int sage_attn_fwd_impl(const void* q_codes, const float* q_desc, const void* k_codes,
                                const float* k_desc, const void* v, const float* v_desc,
                                const uint8_t* block_mask, int64_t mask_bh_stride, void* out,
                                float* lse, int64_t BH, int64_t N, int qk_kind, int q_gran,
                                int k_gran, int pv_kind, int64_t out_heads, void* stream,
                                const QuantOut* qo = nullptr) {
  FD_CHECK_ARG(BH > 0 && BH <= 65535 && N > 0 && N < (1ll << 30), "bad shape");
  FD_CHECK_ARG(qk_kind == FD_QK_INT8 || qk_kind == FD_QK_FP8, "bad qk_kind");
  FD_CHECK_ARG(q_gran == FD_GRAN_TOKEN || q_gran == FD_GRAN_BLOCK, "bad q_gran");
  FD_CHECK_ARG(k_gran == FD_GRAN_TOKEN || k_gran == FD_GRAN_BLOCK, "bad k_gran");
  FD_CHECK_ARG(pv_kind == FD_PV_BF16 || pv_kind == FD_PV_FP8 || pv_kind == FD_PV_FP8_TILE, "bad pv_kind");
  FD_CHECK_ARG(pv_kind != FD_PV_FP8_TILE || (q_gran == FD_GRAN_TOKEN && k_gran == FD_GRAN_TOKEN &&
                                             block_mask == nullptr && out_heads == 0 && qo == nullptr && out),
               "FD_PV_FP8_TILE: per-token Q/K, no block mask, (BH, N, 128) output");
  FD_CHECK_ARG(pv_kind != FD_PV_FP8_TILE || aligned16(v_desc), "v_desc must be 16-byte aligned");
  FD_CHECK_ARG(q_codes && q_desc && k_codes && k_desc && v && (out || qo), "null pointer");
  FD_CHECK_ARG(pv_kind == FD_PV_BF16 || v_desc, "v_desc required for fp8 PV");
  FD_CHECK_ARG(aligned16(q_codes) && aligned16(k_codes) && aligned16(v) && (qo || aligned16(out)) &&
                   aligned16(k_desc),
               "q/k/v codes, out and k_desc must be 16-byte aligned");
  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[3] = {128, (uint64_t)N, (uint64_t)BH};
    const uint64_t strides[2] = {128, (uint64_t)N * 128};
    const uint32_t box[3] = {128, 128, 1};
    int rc = encode_tiled(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, q_codes, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, k_codes, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (pv_kind != FD_PV_BF16) {
      rc = encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, v, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
      const uint64_t vstr[2] = {256, (uint64_t)N * 256};
      const uint32_t vbox[3] = {64, 128, 1};
      rc = encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, v, dims, vstr, vbox,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (rc) return rc;
  }
  attn::Params p;
  p.q_desc = q_desc;
  p.k_desc = k_desc;
  p.v_desc = v_desc;
  p.mask = block_mask;
  p.mask_bh_stride = mask_bh_stride;
  p.out = (__nv_bfloat16*)out;
  p.lse = lse;
  p.out_heads = out_heads;
  p.qout[0] = p.qout[1] = nullptr;
  p.qscale[0] = p.qscale[1] = nullptr;
  p.qstride[0] = p.qstride[1] = p.sstride[0] = p.sstride[1] = 0;
  p.split = (int)N;
  if (qo) {
    FD_CHECK_ARG(out_heads > 0 && BH % out_heads == 0, "quantised output needs H dividing BH");
    FD_CHECK_ARG(qo->split >= 1 && qo->split <= N, "split must be in [1, N]");
    for (int r = 0; r < (qo->split < N ? 2 : 1); ++r) {
      FD_CHECK_ARG(qo->codes[r] && qo->scales[r], "null quantised-output pointer");
      FD_CHECK_ARG(aligned16(qo->codes[r]) && qo->code_stride[r] % 16 == 0 &&
                       qo->code_stride[r] >= out_heads * 128 && qo->scale_stride[r] >= out_heads,
                   "codes must be 16-byte aligned with a row stride >= H * 128 (multiple of 16), "
                   "scale row stride >= H");
      p.qout[r] = (uint8_t*)qo->codes[r];
      p.qscale[r] = qo->scales[r];
      p.qstride[r] = qo->code_stride[r];
      p.sstride[r] = qo->scale_stride[r];
    }
    p.split = (int)qo->split;
  }
  p.N = (int)N;
  p.n_kv_tiles = (int)((N + 127) / 128);
  p.nkb64 = (int)((N + 63) / 64);
  p.q_gran = q_gran;
  p.q_desc_stride = fd_desc_stride(N, q_gran, 128);
  p.k_desc_stride = fd_desc_stride(N, k_gran, 64);
  cudaStream_t st = (cudaStream_t)stream;
#define FD_ATTN(QKV, KGV, PVV) return attn::launch<QKV, KGV, PVV>(tq, tk, tv, p, (int)BH, st)
  if (pv_kind == FD_PV_FP8_TILE) {
    if (qk_kind == FD_QK_INT8) FD_ATTN(FD_QK_INT8, FD_GRAN_TOKEN, FD_PV_FP8_TILE);
    else FD_ATTN(FD_QK_FP8, FD_GRAN_TOKEN, FD_PV_FP8_TILE);
  }
  if (qk_kind == FD_QK_INT8) {
    if (k_gran == FD_GRAN_TOKEN) {
      if (pv_kind == FD_PV_FP8) FD_ATTN(FD_QK_INT8, FD_GRAN_TOKEN, FD_PV_FP8);
      else FD_ATTN(FD_QK_INT8, FD_GRAN_TOKEN, FD_PV_BF16);
    } else {
      if (pv_kind == FD_PV_FP8) FD_ATTN(FD_QK_INT8, FD_GRAN_BLOCK, FD_PV_FP8);
      else FD_ATTN(FD_QK_INT8, FD_GRAN_BLOCK, FD_PV_BF16);
    }
  } else {
    if (k_gran == FD_GRAN_TOKEN) {
      if (pv_kind == FD_PV_FP8) FD_ATTN(FD_QK_FP8, FD_GRAN_TOKEN, FD_PV_FP8);
      else FD_ATTN(FD_QK_FP8, FD_GRAN_TOKEN, FD_PV_BF16);
    } else {
      if (pv_kind == FD_PV_FP8) FD_ATTN(FD_QK_FP8, FD_GRAN_BLOCK, FD_PV_FP8);
      else FD_ATTN(FD_QK_FP8, FD_GRAN_BLOCK, FD_PV_BF16);
    }
  }
#undef FD_ATTN
}

extern "C" int fd_sage_attn_fwd(const void* q_codes, const float* q_desc, const void* k_codes,
                                const float* k_desc, const void* v, const float* v_desc,
                                const uint8_t* block_mask, int64_t mask_bh_stride, void* out,
                                float* lse, int64_t BH, int64_t N, int qk_kind, int q_gran,
                                int k_gran, int pv_kind, void* stream) {
  return sage_attn_fwd_impl(q_codes, q_desc, k_codes, k_desc, v, v_desc, block_mask, mask_bh_stride, out,
                            lse, BH, N, qk_kind, q_gran, k_gran, pv_kind, 0, stream);
}

extern "C" int fd_sage_attn_fwd_bnhd(const void* q_codes, const float* q_desc, const void* k_codes,
                                     const float* k_desc, const void* v, const float* v_desc,
                                     const uint8_t* block_mask, int64_t mask_bh_stride, void* out,
                                     float* lse, int64_t BH, int64_t N, int64_t H, int qk_kind,
                                     int q_gran, int k_gran, int pv_kind, void* stream) {
  FD_CHECK_ARG(H > 0 && BH % H == 0, "H must divide BH");
  return sage_attn_fwd_impl(q_codes, q_desc, k_codes, k_desc, v, v_desc, block_mask, mask_bh_stride, out,
                            lse, BH, N, qk_kind, q_gran, k_gran, pv_kind, H, stream);
}

// Attention whose output is written as the e4m3 1 x 128 codes + fp32 scales of the
// output linear's input: row (b, n) of head h is the group [h * 128, h * 128 + 128)
// of output row n.  Rows n < split go to (codes0, scales0), rows n >= split to
// (codes1, scales1) (each region holds its rows of every sample contiguously),
// with the given row strides (code bytes, scales).
extern "C" int fd_sage_attn_fwd_quant_out(const void* q_codes, const float* q_desc, const void* k_codes,
                                          const float* k_desc, const void* v, const float* v_desc,
                                          const uint8_t* block_mask, int64_t mask_bh_stride, float* lse,
                                          int64_t BH, int64_t N, int64_t H, int qk_kind, int q_gran,
                                          int k_gran, int pv_kind, void* codes0, float* scales0,
                                          int64_t code_stride0, int64_t scale_stride0, void* codes1,
                                          float* scales1, int64_t code_stride1, int64_t scale_stride1,
                                          int64_t split, void* stream) {
  QuantOut qo;
  qo.codes[0] = codes0;
  qo.codes[1] = codes1;
  qo.scales[0] = scales0;
  qo.scales[1] = scales1;
  qo.code_stride[0] = code_stride0;
  qo.code_stride[1] = code_stride1;
  qo.scale_stride[0] = scale_stride0;
  qo.scale_stride[1] = scale_stride1;
  qo.split = split;
  FD_CHECK_ARG(H > 0, "H must be positive");
  return sage_attn_fwd_impl(q_codes, q_desc, k_codes, k_desc, v, v_desc, block_mask, mask_bh_stride, nullptr,
                            lse, BH, N, qk_kind, q_gran, k_gran, pv_kind, H, stream, &qo);
}
