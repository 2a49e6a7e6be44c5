// Attention backward (A7): the Delta pre-pass (_sage_attn_d_prepass,
// src/futudiffu/sage_kernels.py:322-349) and, on tcgen05, a dK/dV kernel and a dQ
// kernel, the split of the reference's _sage_attn_bwd_dkdv_int8(_masked) /
// _sage_attn_bwd_dq_int8(_masked) (:805-1015, :1491-1722; fp8 QK :356-567).
//
// Per (query i, key j), exactly as the forward's P:
//   L   = ((S_ij q_desc_i) k_desc_j)  with S = Qc Kc^T on the quantised codes
//   p   = exp2(L - lse_i)             (0 on masked 128 x 64 tiles, keys / queries >= N)
//   dP  = dO V^T,   dS = p (dP - Delta_i)
//   dV  = sum_i bf16(p) dO_i,   dK = sum_i bf16(dS sm_scale) Q_i,
//   dQ  = sm_scale sum_j bf16(dS) Ks_j      (Ks = the smoothed K of the forward)
// fp32 accumulation in TMEM, one bf16 rounding of each gradient at the end.
//
// dK/dV kernel: CTA = one 128-key tile of one (b, h), looping over 64-query steps.
//   resident: Kc (codes) and V (bf16) of the tile
//   per step (4-stage ring): Qc, Q (bf16), dO (bf16) of 64 queries + q_desc /
//   -lse / -Delta of those queries
//   MMA:  S^T  = Kc Qc^T        (M 128 keys, N 64, kind::i8 onto the score bias, or f8f6f4)
//         dP^T = V dO^T         (kind::f16, both K-major)
//         dV  += P^T dO         (A = P^T in TMEM, B = the dO tile read MN-major)
//         dK  += dSs^T Q        (A = dSs^T in TMEM, B = the Q tile read MN-major)
//   S^T / dP^T are double-buffered in TMEM, so the next step's products run on the
//   tensor core while the compute warps turn this step's into P^T and dS^T, which
//   they write back as bf16 pairs over the dP^T columns they have read (the dV / dK
//   products of step i are issued before step i + 2's S^T / dP^T, and tcgen05 MMAs
//   of one thread run in issue order).
//   TMEM: dV [0,128), dK [128,256), S^T(b) [256+128b, +64), dP^T(b) [320+128b, +64);
//   the thread that read dP^T columns [CW c, CW c + CW) (its queries) writes P^T of
//   those queries over the first CW / 2 of them and dSs^T over the next CW / 2.
// dQ kernel: CTA = one 128-query tile, looping over 64-key steps:
//         S = Qc Kc^T, dP = dO V^T (double-buffered), dQ += dS Ks (A = dS in TMEM,
//         B = the Ks tile read MN-major).
//   TMEM: dQ [0,128), S(b) [128+64b, +64), dP(b) [256+64b, +64), dS(b) [384+32b, +32).
// Compute warps 0 .. 7 (TMEM lane quadrant w & 3, CW = 32 of the step's 64 columns
// each), then the TMA producer warp and the MMA issuer warp.  Every wait is bounded (fd_common.cuh).
#include "fd_common.cuh"
#include "fd_host.h"

namespace fd {
namespace attn_bwd {

// Delta[bh, n] = sum_d dO[bh, n, d] * O[bh, n, d]; one warp per row.
__global__ void __launch_bounds__(256) prepass_kernel(const __nv_bfloat16* __restrict__ dout,
                                                     const __nv_bfloat16* __restrict__ out,
                                                     float* __restrict__ delta, int64_t rows) {
  const int lane = lane_id();
  for (int64_t r = (int64_t)blockIdx.x * 8 + warp_id(); r < rows; r += (int64_t)gridDim.x * 8) {
    const uint2 a = *reinterpret_cast<const uint2*>(dout + r * 128 + lane * 4);
    const uint2 b = *reinterpret_cast<const uint2*>(out + r * 128 + lane * 4);
    float s = bf16_bits_to_f32(a.x & 0xFFFF) * bf16_bits_to_f32(b.x & 0xFFFF) +
              bf16_bits_to_f32(a.x >> 16) * bf16_bits_to_f32(b.x >> 16) +
              bf16_bits_to_f32(a.y & 0xFFFF) * bf16_bits_to_f32(b.y & 0xFFFF) +
              bf16_bits_to_f32(a.y >> 16) * bf16_bits_to_f32(b.y >> 16);
    s = warp_sum(s);
    if (lane == 0) delta[r] = s;
  }
}


constexpr int HD = 128;
constexpr int BT = 128;  // rows of the resident tile
constexpr int BS = 64;   // rows per step
constexpr int NST = 4;   // stage ring depth
#ifndef FD_BWD_COMPUTE_WARPS
#define FD_BWD_COMPUTE_WARPS 8
#endif
constexpr int NUM_COMPUTE_WARPS = FD_BWD_COMPUTE_WARPS;  // 8 or 16: two or four per TMEM lane quadrant
constexpr int WARP_TMA = NUM_COMPUTE_WARPS, WARP_MMA = NUM_COMPUTE_WARPS + 1;
constexpr int NUM_THREADS = 32 * (NUM_COMPUTE_WARPS + 2);
constexpr int CW = BS * 4 / NUM_COMPUTE_WARPS;  // step columns per compute warp (32 or 16)
constexpr int EW = HD * 4 / NUM_COMPUTE_WARPS;  // accumulator columns per compute warp in the epilogue
static_assert(CW == 16 || CW == 32, "8 or 16 compute warps");
constexpr uint32_t TMEM_COLS = 512;

// INT8 scores accumulate onto the bits of 1.5 * 2^23 written into the S columns
// before every QK^T (|s| <= 128 * 127 * 127 < 2^22), so the s32 accumulator holds
// the bits of the float 1.5 * 2^23 + s and no integer conversion is needed.
constexpr uint32_t S_BIAS_BITS = 0x4B400000u;
constexpr float S_BIAS = 12582912.0f;

// ----------------------------------------------------------------- layouts
struct SmemKV {  // dK / dV kernel
  static constexpr uint32_t KC_BYTES = BT * HD;          // int8 / e4m3 codes, one 128-byte panel
  static constexpr uint32_t V_BYTES = BT * HD * 2;       // bf16, two 64-column panels
  static constexpr uint32_t QC_BYTES = BS * HD;
  static constexpr uint32_t Q_BYTES = BS * HD * 2;       // two panels of BS x 128 B
  static constexpr uint32_t DO_BYTES = BS * HD * 2;
  static constexpr uint32_t STAGE_BYTES = QC_BYTES + Q_BYTES + DO_BYTES;
  static constexpr uint32_t OFF_KC = 0;
  static constexpr uint32_t OFF_V = OFF_KC + KC_BYTES;
  static constexpr uint32_t OFF_ST = OFF_V + V_BYTES;
  static constexpr uint32_t OFF_VEC = OFF_ST + NST * STAGE_BYTES;  // per stage: qd, nbq, nl, nd [4][64] f32
  static constexpr uint32_t OFF_BAR = OFF_VEC + NST * 1024;
  static constexpr uint32_t TOTAL = OFF_BAR + 256 + 1024;  // + barriers, alignment slack
};
static_assert(SmemKV::OFF_ST % 1024 == 0 && SmemKV::STAGE_BYTES % 1024 == 0,
              "swizzled tiles need 1024-byte alignment");
static_assert(SmemKV::TOTAL <= 232448, "dK/dV shared memory");

struct SmemQ {  // dQ kernel
  static constexpr uint32_t QC_BYTES = BT * HD;
  static constexpr uint32_t DO_BYTES = BT * HD * 2;
  static constexpr uint32_t KC_BYTES = BS * HD;
  static constexpr uint32_t V_BYTES = BS * HD * 2;
  static constexpr uint32_t KS_BYTES = BS * HD * 2;
  static constexpr uint32_t STAGE_BYTES = KC_BYTES + V_BYTES + KS_BYTES;
  static constexpr uint32_t OFF_QC = 0;
  static constexpr uint32_t OFF_DO = OFF_QC + QC_BYTES;
  static constexpr uint32_t OFF_ST = OFF_DO + DO_BYTES;
  static constexpr uint32_t OFF_KD = OFF_ST + NST * STAGE_BYTES;  // per stage 64 f32
  static constexpr uint32_t OFF_BAR = OFF_KD + 1024;
  static constexpr uint32_t TOTAL = OFF_BAR + 256 + 1024;
};
static_assert(SmemQ::OFF_ST % 1024 == 0 && SmemQ::STAGE_BYTES % 1024 == 0, "swizzled tiles need 1024-byte alignment");
static_assert(NST * 256 <= 1024, "dQ key-scale slots");
static_assert(SmemQ::TOTAL <= 232448, "dQ shared memory");

struct Params {
  const float* q_desc;  // (BH, dstride) per-token, zero-padded
  const float* k_desc;
  const float* lse;     // (BH, N)
  const float* delta;   // (BH, N)
  const uint8_t* mask;  // (BH or 1, ceil(N/128), ceil(N/64)) or null
  int64_t mask_bh_stride;
  __nv_bfloat16* g0;    // dK (dkdv) / dQ (dq), (BH, N, 128)
  __nv_bfloat16* g1;    // dV (dkdv)
  int N;
  int nkb64;
  int64_t dstride;
  float sm_scale;
};

FD_DEV bool mask_at(const Params& p, int bh, int qt, int kb) {
  return p.mask[(int64_t)bh * p.mask_bh_stride + (int64_t)qt * p.nkb64 + kb] != 0;
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

// lane 0 waits (bounded); the verdict is broadcast and every lane then takes the
// completed phase itself (acquire), so the whole warp may touch the guarded data
FD_DEV bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  bool ok = lane_id() == 0 ? mbar_wait(bar, parity, abort_flag) : false;
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (ok) mbar_try_wait(bar, parity);
  return ok;
}


// TMEM access of a compute warp's CW step columns
FD_DEV void ld_cols(uint32_t t, uint32_t (&r)[16]) { tmem_ld16(t, r); }
FD_DEV void ld_cols(uint32_t t, uint32_t (&r)[32]) { tmem_ld32(t, r); }
FD_DEV void st_cols(uint32_t t, const uint32_t (&r)[8]) { tmem_st8(t, r); }
FD_DEV void st_cols(uint32_t t, const uint32_t (&r)[16]) { tmem_st16(t, r); }
FD_DEV void fill_cols(uint32_t t) {
  if constexpr (CW == 16) tmem_fill16(t, S_BIAS_BITS);
  else tmem_fill32(t, S_BIAS_BITS);
}
// A-operand columns of the bf16 pairs of step queries [16 k, 16 k + 16): the compute
// warp owning those CW queries wrote P^T over the first CW / 2 of its CW columns
__host__ __device__ constexpr uint32_t pt_col(int k) { return CW * (16 * k / CW) + (16 * k % CW) / 2; }

// EW accumulator columns of this thread's row -> bf16 at dst (scaled by `scale`)
FD_DEV void store_acc(uint32_t taddr, bool any, bool row_ok, float scale, __nv_bfloat16* dst) {
#pragma unroll
  for (int cc = 0; cc < EW / 32; ++cc) {
    uint32_t r[32];
    if (any) {
      tmem_ld32(taddr + 32 * cc, r);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) r[e] = 0u;
    }
    if (row_ok) {
      uint32_t w[16];
#pragma unroll
      for (int e = 0; e < 16; ++e)
        w[e] = pack_bf16x2(__uint_as_float(r[2 * e]) * scale, __uint_as_float(r[2 * e + 1]) * scale);
      uint4* d = reinterpret_cast<uint4*>(dst + 32 * cc);
#pragma unroll
      for (int k = 0; k < 4; ++k) d[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
    }
  }
}

// ========================================================================= dK / dV
// step t covers queries [64 t, 64 t + 64) (128-row query tile t / 2); it is skipped
// when both 64-key halves of the key tile are masked for that query tile
FD_DEV bool kv_step_valid(const Params& p, int bh, int kt, int t) {
  if (!p.mask) return true;
  const int qt = t >> 1;
  const bool a = mask_at(p, bh, qt, 2 * kt);
  const bool b = (2 * kt + 1 < p.nkb64) && mask_at(p, bh, qt, 2 * kt + 1);
  return a || b;
}

template <int QK>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmKc, const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmQc, const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmDO, const Params p) {
  using SM = SmemKV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sKc = smem + SM::OFF_KC;
  uint8_t* sV = smem + SM::OFF_V;
  float* sVec = reinterpret_cast<float*>(smem + SM::OFF_VEC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::OFF_BAR);
  uint64_t* bRes = bars + 0;
  uint64_t* bFull = bars + 1;               // [NST]
  uint64_t* bEmpty = bFull + NST;           // [NST]
  uint64_t* bSdpFull = bEmpty + NST;        // [2]
  uint64_t* bSdpFree = bSdpFull + 2;        // [2]
  uint64_t* bPsFull = bSdpFree + 2;        // [2]
  uint64_t* bAcc = bPsFull + 2;
  uint64_t* bDrain = bAcc + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bDrain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int kt = blockIdx.x, bh = blockIdx.y;
  const int k0 = kt * BT;
  const int nsteps = (p.N + BS - 1) / BS;

  if (threadIdx.x == 0) {
    mbar_init(bRes, 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&bFull[s], 1);
      mbar_init(&bEmpty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bSdpFull[b], 1);
      mbar_init(&bSdpFree[b], NUM_COMPUTE_WARPS);
      mbar_init(&bPsFull[b], NUM_COMPUTE_WARPS);
    }
    mbar_init(bAcc, 1);
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
  const uint32_t tdV = tmem_base, tdK = tmem_base + 128;
  auto tS = [&](uint32_t b) { return tmem_base + 256 + 128 * b; };
  auto tdP = [&](uint32_t b) { return tmem_base + 320 + 128 * b; };

  if (warp == WARP_TMA) {
    // ================================================================ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmKc);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmQc);
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(bRes, SM::KC_BYTES + SM::V_BYTES);
      tma_load_3d(sKc, &tmKc, bRes, 0, k0, bh);
      tma_load_3d(sV, &tmV, bRes, 0, k0, bh);
      tma_load_3d(sV + BT * 128, &tmV, bRes, 64, k0, bh);
    }
    // per-query constants of a step: q_desc, -S_BIAS q_desc (INT8), -lse (-inf past
    // N, which zeroes those columns' P), -Delta; the next step's are loaded into
    // registers while this step waits for its stage, so no global-load latency sits
    // between a free stage and its refill
    auto next_valid = [&](int from) {
      for (int t = from; t < nsteps; ++t)
        if (kv_step_valid(p, bh, kt, t)) return t;
      return nsteps;
    };
    auto load_vec = [&](int t, float (&r)[6]) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int qi = t * BS + lane + 32 * u;
        const bool ok = t < nsteps && qi < p.N;
        r[3 * u] = ok ? p.q_desc[(int64_t)bh * p.dstride + qi] : 0.f;
        r[3 * u + 1] = ok ? -p.lse[(int64_t)bh * p.N + qi] : -INFINITY;
        r[3 * u + 2] = ok ? -p.delta[(int64_t)bh * p.N + qi] : 0.f;
      }
    };
    uint32_t i = 0;
    int t = next_valid(0);
    float cur[6];
    load_vec(t, cur);
    for (; t < nsteps; ++i) {
      const int tn = next_valid(t + 1);
      float nxt[6];
      load_vec(tn, nxt);
      const uint32_t s = i % NST, use = i / NST;
      if (!warp_wait(&bEmpty[s], (use & 1) ^ 1, abort_flag)) break;
      float* v = sVec + s * 256;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int e = lane + 32 * u;
        v[e] = cur[3 * u];
        v[64 + e] = QK == FD_QK_INT8 ? -S_BIAS * cur[3 * u] : 0.f;
        v[128 + e] = cur[3 * u + 1];
        v[192 + e] = cur[3 * u + 2];
      }
      __syncwarp();
      if (lane == 0) {
        uint8_t* st = smem + SM::OFF_ST + s * SM::STAGE_BYTES;
        mbar_arrive_expect_tx(&bFull[s], SM::STAGE_BYTES);
        tma_load_3d(st, &tmQc, &bFull[s], 0, t * BS, bh);
        tma_load_3d(st + SM::QC_BYTES, &tmQ, &bFull[s], 0, t * BS, bh);
        tma_load_3d(st + SM::QC_BYTES + BS * 128, &tmQ, &bFull[s], 64, t * BS, bh);
        tma_load_3d(st + SM::QC_BYTES + SM::Q_BYTES, &tmDO, &bFull[s], 0, t * BS, bh);
        tma_load_3d(st + SM::QC_BYTES + SM::Q_BYTES + BS * 128, &tmDO, &bFull[s], 64, t * BS, bh);
      }
      __syncwarp();
#pragma unroll
      for (int e = 0; e < 6; ++e) cur[e] = nxt[e];
      t = tn;
    }
    if (lane == 0) {
      drain_wait(bRes, 0);
      for (uint32_t k = 0; k < (uint32_t)NST && k < i; ++k) {
        const uint32_t last = i - 1 - k;
        drain_wait(&bFull[last % NST], (last / NST) & 1);
      }
    }
  } else if (warp == WARP_MMA) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = QK == FD_QK_INT8 ? make_idesc(/*S32*/ 2, /*S8*/ 1, 1, 0, 0, BT, BS)
                                                    : make_idesc(/*F32*/ 1, /*E4M3*/ 0, 0, 0, 0, BT, BS);
      constexpr uint32_t idesc_dp = make_idesc(1, /*BF16*/ 1, 1, 0, 0, BT, BS);
      constexpr uint32_t idesc_acc = make_idesc(1, 1, 1, /*A K-major*/ 0, /*B MN-major*/ 1, BT, HD);
      const uint32_t aKc = smem_u32(sKc), aV = smem_u32(sV);
      bool ok = mbar_wait(bRes, 0, abort_flag);
      // the valid steps, in the producer's order
      auto next_valid = [&](int from) {
        for (int t = from; t < nsteps; ++t)
          if (kv_step_valid(p, bh, kt, t)) return t;
        return nsteps;
      };
      auto issue_sdp = [&](uint32_t i) -> bool {
        const uint32_t s = i % NST, b = i & 1;
        if (!mbar_wait(&bFull[s], (i / NST) & 1, abort_flag)) return false;
        if (!mbar_wait(&bSdpFree[b], (i >> 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + SM::OFF_ST + s * SM::STAGE_BYTES);
        const uint32_t bQc = st, bDO = st + SM::QC_BYTES + SM::Q_BYTES;
#pragma unroll
        for (int k = 0; k < HD / 32; ++k) {
          const uint64_t ad = make_sdesc_sw128(aKc + k * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(bQc + k * 32, 16, 1024);
          if (QK == FD_QK_INT8) mma_i8_ss(tS(b), ad, bd, idesc_s, 1u);  // onto S_BIAS_BITS
          else mma_f8f6f4_ss(tS(b), ad, bd, idesc_s, k > 0);
        }
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t ad = make_sdesc_sw128(aV + (k >> 2) * (BT * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(bDO + (k >> 2) * (BS * 128) + (k & 3) * 32, 16, 1024);
          mma_f16_ss(tdP(b), ad, bd, idesc_dp, k > 0);
        }
        tc_commit(&bSdpFull[b]);
        return true;
      };
      auto issue_acc = [&](uint32_t i) -> bool {
        const uint32_t s = i % NST, b = i & 1;
        if (!mbar_wait(&bPsFull[b], (i >> 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + SM::OFF_ST + s * SM::STAGE_BYTES);
        const uint32_t bQ = st + SM::QC_BYTES, bDO = st + SM::QC_BYTES + SM::Q_BYTES;
        // queries [16 k, 16 k + 16): P^T at pt_col(k), dSs^T CW / 2 columns further
#pragma unroll
        for (int k = 0; k < BS / 16; ++k) {
          const uint64_t bd = make_sdesc_sw128(bDO + k * 16 * 128, BS * 128, 1024);
          mma_f16_ts(tdV, tdP(b) + pt_col(k), bd, idesc_acc, (i > 0 || k > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < BS / 16; ++k) {
          const uint64_t bd = make_sdesc_sw128(bQ + k * 16 * 128, BS * 128, 1024);
          mma_f16_ts(tdK, tdP(b) + pt_col(k) + CW / 2, bd, idesc_acc, (i > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&bEmpty[s]);
        return true;
      };
      // order: S/dP(0), S/dP(1), then acc(i), S/dP(i + 2), ...
      int nvalid = 0;
      for (int t = next_valid(0); t < nsteps; t = next_valid(t + 1)) ++nvalid;
      for (int i = 0; ok && i < 2 && i < nvalid; ++i) ok = issue_sdp((uint32_t)i);
      for (int i = 0; ok && i < nvalid; ++i) {
        ok = issue_acc((uint32_t)i);
        if (ok && i + 2 < nvalid) ok = issue_sdp((uint32_t)(i + 2));
      }
      tc_commit(bAcc);
      tc_commit(bDrain);
      drain_wait(bDrain, 0);
    }
  } else {
    // ================================================================ compute warps
    // warp w: TMEM lane quadrant w & 3 (key rows), step columns [CW c, CW c + CW), c = w >> 2
    const int quad = warp & 3, c4 = warp >> 2;
    const int row = quad * 32 + lane;  // key row of the tile
    const int key = k0 + row;
    const bool key_ok = key < p.N;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int cb = CW * c4;  // this warp's CW query columns of the step
    const float kd = key_ok ? p.k_desc[(int64_t)bh * p.dstride + key] : 0.f;
    const int kb = 2 * kt + (row >> 6);
    const float sm = p.sm_scale;
    if (QK == FD_QK_INT8) {
      fill_cols(tS(0) + lane_base + cb);
      fill_cols(tS(1) + lane_base + cb);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&bSdpFree[0]);
      mbar_arrive(&bSdpFree[1]);
    }
    bool ok = true;
    uint32_t i = 0;
    for (int t = 0; t < nsteps; ++t) {
      if (!kv_step_valid(p, bh, kt, t)) continue;
      const uint32_t s = i % NST, b = i & 1;
      if (!mbar_wait(&bSdpFull[b], (i >> 1) & 1, abort_flag)) { ok = false; break; }
      if (!mbar_wait(&bFull[s], (i / NST) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t rs[CW], rd[CW];
      ld_cols(tS(b) + lane_base + cb, rs);
      ld_cols(tdP(b) + lane_base + cb, rd);
      tmem_wait_ld();
      // the score bias for S(i + 2), written now and waited for with the P^T / dSs^T
      // stores below (S(i + 2) is issued after this step's dV / dK products)
      if (QK == FD_QK_INT8) fill_cols(tS(b) + lane_base + cb);
      // rows of a masked 64-key half, and keys past N, contribute nothing
      const bool row_ok = key_ok && (!p.mask || mask_at(p, bh, t >> 1, kb));
      const float* v = sVec + s * 256 + cb;
      uint32_t wp[CW / 2], wd[CW / 2];
#pragma unroll
      for (int e = 0; e < CW; e += 4) {
        const float4 qd4 = *reinterpret_cast<const float4*>(v + e);
        const float4 nq4 = *reinterpret_cast<const float4*>(v + 64 + e);
        const float4 nl4 = *reinterpret_cast<const float4*>(v + 128 + e);
        const float4 nd4 = *reinterpret_cast<const float4*>(v + 192 + e);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = e + 2 * u;
          const uint64_t qd2 = u ? pk(qd4.z, qd4.w) : pk(qd4.x, qd4.y);
          const uint64_t nq2 = u ? pk(nq4.z, nq4.w) : pk(nq4.x, nq4.y);
          const uint64_t nl2 = u ? pk(nl4.z, nl4.w) : pk(nl4.x, nl4.y);
          const uint64_t nd2 = u ? pk(nd4.z, nd4.w) : pk(nd4.x, nd4.y);
          uint64_t x = pk(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1]));
          // L - lse = ((s q_desc) k_desc) - lse; INT8: s q_desc = (s + B) q_desc - B q_desc
          x = QK == FD_QK_INT8 ? fma2(fma2(x, qd2, nq2), pk(kd, kd), nl2) : fma2(mul2(x, qd2), pk(kd, kd), nl2);
          float l0, l1;
          unpk(x, l0, l1);
          const float p0 = row_ok ? ex2_approx(l0) : 0.f, p1 = row_ok ? ex2_approx(l1) : 0.f;
          const uint64_t ds2 =
              mul2(pk(p0, p1), add2(pk(__uint_as_float(rd[c]), __uint_as_float(rd[c + 1])), nd2));
          float d0, d1;
          unpk(mul2(ds2, pk(sm, sm)), d0, d1);
          wp[c >> 1] = pack_bf16x2(p0, p1);
          wd[c >> 1] = pack_bf16x2(d0, d1);
        }
      }
      // P^T and dSs^T over the CW dP^T columns this thread has read: its queries as
      // bf16 pairs, P^T over the first CW / 2 columns, dSs^T over the next CW / 2
      st_cols(tdP(b) + lane_base + cb, wp);
      st_cols(tdP(b) + lane_base + cb + CW / 2, wd);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bSdpFree[b]);
        mbar_arrive(&bPsFull[b]);
      }
      ++i;
    }
    // ---------------------------------------------------------------- epilogue
    if (ok) ok = mbar_wait(bAcc, 0, abort_flag);
    if (ok) {
      tc_fence_after();
      const int64_t orow = ((int64_t)bh * p.N + (key_ok ? key : 0)) * HD + EW * c4;
      store_acc(tdV + lane_base + EW * c4, i > 0, key_ok, 1.f, p.g1 + orow);
      store_acc(tdK + lane_base + EW * c4, i > 0, key_ok, 1.f, p.g0 + orow);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == WARP_MMA) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ========================================================================= dQ
// step j covers keys [64 j, 64 j + 64) = the mask's 64-key block j
template <int QK>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQc, const __grid_constant__ CUtensorMap tmDO,
                  const __grid_constant__ CUtensorMap tmKc, const __grid_constant__ CUtensorMap tmV,
                  const __grid_constant__ CUtensorMap tmKs, const Params p) {
  using SM = SmemQ;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQc = smem + SM::OFF_QC;
  uint8_t* sDO = smem + SM::OFF_DO;
  float* sKd = reinterpret_cast<float*>(smem + SM::OFF_KD);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::OFF_BAR);
  uint64_t* bRes = bars + 0;
  uint64_t* bFull = bars + 1;          // [NST]
  uint64_t* bEmpty = bFull + NST;      // [NST]
  uint64_t* bSdpFull = bEmpty + NST;   // [2]
  uint64_t* bSdpFree = bSdpFull + 2;   // [2]
  uint64_t* bDsFull = bSdpFree + 2;    // [2]
  uint64_t* bAcc = bDsFull + 2;
  uint64_t* bDrain = bAcc + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bDrain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int qt = blockIdx.x, bh = blockIdx.y;
  const int q0 = qt * BT;
  const int nsteps = (p.N + BS - 1) / BS;
  auto step_valid = [&](int j) { return !p.mask || mask_at(p, bh, qt, j); };

  if (threadIdx.x == 0) {
    mbar_init(bRes, 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&bFull[s], 1);
      mbar_init(&bEmpty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bSdpFull[b], 1);
      mbar_init(&bSdpFree[b], NUM_COMPUTE_WARPS);
      mbar_init(&bDsFull[b], NUM_COMPUTE_WARPS);
    }
    mbar_init(bAcc, 1);
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
  const uint32_t tdQ = tmem_base;
  auto tS = [&](uint32_t b) { return tmem_base + 128 + 64 * b; };
  auto tdP = [&](uint32_t b) { return tmem_base + 256 + 64 * b; };
  auto tdS = [&](uint32_t b) { return tmem_base + 384 + 32 * b; };

  if (warp == WARP_TMA) {
    // ================================================================ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQc);
      tma_prefetch_desc(&tmDO);
      tma_prefetch_desc(&tmKc);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmKs);
      mbar_arrive_expect_tx(bRes, SM::QC_BYTES + SM::DO_BYTES);
      tma_load_3d(sQc, &tmQc, bRes, 0, q0, bh);
      tma_load_3d(sDO, &tmDO, bRes, 0, q0, bh);
      tma_load_3d(sDO + BT * 128, &tmDO, bRes, 64, q0, bh);
    }
    // per-key scales of a step, loaded one step ahead (as in the dK / dV producer)
    auto next_valid = [&](int from) {
      for (int j = from; j < nsteps; ++j)
        if (step_valid(j)) return j;
      return nsteps;
    };
    auto load_kd = [&](int j, float (&r)[2]) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int key = j * BS + lane + 32 * u;
        r[u] = (j < nsteps && key < p.N) ? p.k_desc[(int64_t)bh * p.dstride + key] : 0.f;
      }
    };
    uint32_t i = 0;
    int j = next_valid(0);
    float cur[2];
    load_kd(j, cur);
    for (; j < nsteps; ++i) {
      const int jn = next_valid(j + 1);
      float nxt[2];
      load_kd(jn, nxt);
      const uint32_t s = i % NST, use = i / NST;
      if (!warp_wait(&bEmpty[s], (use & 1) ^ 1, abort_flag)) break;
      float* kdv = sKd + s * 64;
      kdv[lane] = cur[0];
      kdv[lane + 32] = cur[1];
      __syncwarp();
      if (lane == 0) {
        uint8_t* st = smem + SM::OFF_ST + s * SM::STAGE_BYTES;
        mbar_arrive_expect_tx(&bFull[s], SM::STAGE_BYTES);
        tma_load_3d(st, &tmKc, &bFull[s], 0, j * BS, bh);
        tma_load_3d(st + SM::KC_BYTES, &tmV, &bFull[s], 0, j * BS, bh);
        tma_load_3d(st + SM::KC_BYTES + BS * 128, &tmV, &bFull[s], 64, j * BS, bh);
        tma_load_3d(st + SM::KC_BYTES + SM::V_BYTES, &tmKs, &bFull[s], 0, j * BS, bh);
        tma_load_3d(st + SM::KC_BYTES + SM::V_BYTES + BS * 128, &tmKs, &bFull[s], 64, j * BS, bh);
      }
      __syncwarp();
      cur[0] = nxt[0];
      cur[1] = nxt[1];
      j = jn;
    }
    if (lane == 0) {
      drain_wait(bRes, 0);
      for (uint32_t k = 0; k < (uint32_t)NST && k < i; ++k) {
        const uint32_t last = i - 1 - k;
        drain_wait(&bFull[last % NST], (last / NST) & 1);
      }
    }
  } else if (warp == WARP_MMA) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = QK == FD_QK_INT8 ? make_idesc(2, 1, 1, 0, 0, BT, BS)
                                                    : make_idesc(1, 0, 0, 0, 0, BT, BS);
      constexpr uint32_t idesc_dp = make_idesc(1, 1, 1, 0, 0, BT, BS);
      constexpr uint32_t idesc_acc = make_idesc(1, 1, 1, 0, 1, BT, HD);
      const uint32_t aQc = smem_u32(sQc), aDO = smem_u32(sDO);
      bool ok = mbar_wait(bRes, 0, abort_flag);
      auto issue_sdp = [&](uint32_t i) -> bool {
        const uint32_t s = i % NST, b = i & 1;
        if (!mbar_wait(&bFull[s], (i / NST) & 1, abort_flag)) return false;
        if (!mbar_wait(&bSdpFree[b], (i >> 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + SM::OFF_ST + s * SM::STAGE_BYTES);
        const uint32_t bKc = st, bV = st + SM::KC_BYTES;
#pragma unroll
        for (int k = 0; k < HD / 32; ++k) {
          const uint64_t ad = make_sdesc_sw128(aQc + k * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(bKc + k * 32, 16, 1024);
          if (QK == FD_QK_INT8) mma_i8_ss(tS(b), ad, bd, idesc_s, 1u);
          else mma_f8f6f4_ss(tS(b), ad, bd, idesc_s, k > 0);
        }
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t ad = make_sdesc_sw128(aDO + (k >> 2) * (BT * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(bV + (k >> 2) * (BS * 128) + (k & 3) * 32, 16, 1024);
          mma_f16_ss(tdP(b), ad, bd, idesc_dp, k > 0);
        }
        tc_commit(&bSdpFull[b]);
        return true;
      };
      auto issue_acc = [&](uint32_t i) -> bool {
        const uint32_t s = i % NST, b = i & 1;
        if (!mbar_wait(&bDsFull[b], (i >> 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + SM::OFF_ST + s * SM::STAGE_BYTES);
        const uint32_t bKs = st + SM::KC_BYTES + SM::V_BYTES;
#pragma unroll
        for (int k = 0; k < BS / 16; ++k) {
          const uint64_t bd = make_sdesc_sw128(bKs + k * 16 * 128, BS * 128, 1024);
          mma_f16_ts(tdQ, tdS(b) + 8 * k, bd, idesc_acc, (i > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&bEmpty[s]);
        return true;
      };
      int nvalid = 0;
      for (int j = 0; j < nsteps; ++j) nvalid += step_valid(j) ? 1 : 0;
      for (int i = 0; ok && i < 2 && i < nvalid; ++i) ok = issue_sdp((uint32_t)i);
      for (int i = 0; ok && i < nvalid; ++i) {
        ok = issue_acc((uint32_t)i);
        if (ok && i + 2 < nvalid) ok = issue_sdp((uint32_t)(i + 2));
      }
      tc_commit(bAcc);
      tc_commit(bDrain);
      drain_wait(bDrain, 0);
    }
  } else {
    // ================================================================ compute warps
    // warp w: TMEM lane quadrant w & 3 (query rows), step columns [CW c, CW c + CW), c = w >> 2
    const int quad = warp & 3, c4 = warp >> 2;
    const int row = quad * 32 + lane;  // query row of the tile
    const int qrow = q0 + row;
    const bool q_ok = qrow < p.N;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int cb = CW * c4;  // this warp's CW key columns of the step
    const float qd = q_ok ? p.q_desc[(int64_t)bh * p.dstride + qrow] : 0.f;
    const float nq = QK == FD_QK_INT8 ? -S_BIAS * qd : 0.f;
    const float nl = q_ok ? -p.lse[(int64_t)bh * p.N + qrow] : -INFINITY;
    const float nd = q_ok ? -p.delta[(int64_t)bh * p.N + qrow] : 0.f;
    if (QK == FD_QK_INT8) {
      fill_cols(tS(0) + lane_base + cb);
      fill_cols(tS(1) + lane_base + cb);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&bSdpFree[0]);
      mbar_arrive(&bSdpFree[1]);
    }
    bool ok = true;
    uint32_t i = 0;
    for (int j = 0; j < nsteps; ++j) {
      if (!step_valid(j)) continue;
      const uint32_t s = i % NST, b = i & 1;
      if (!mbar_wait(&bSdpFull[b], (i >> 1) & 1, abort_flag)) { ok = false; break; }
      if (!mbar_wait(&bFull[s], (i / NST) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t rs[CW], rd[CW];
      ld_cols(tS(b) + lane_base + cb, rs);
      ld_cols(tdP(b) + lane_base + cb, rd);
      tmem_wait_ld();
      // the score bias for S(i + 2) (issued after this step's dQ product), waited for
      // with the dS store below
      if (QK == FD_QK_INT8) fill_cols(tS(b) + lane_base + cb);
      const int key0 = j * BS + cb;  // first key of this thread's columns
      const bool full = key0 + CW <= p.N;
      const float* kdv = sKd + s * 64 + cb;
      uint32_t wd[CW / 2];
#pragma unroll
      for (int e = 0; e < CW; e += 4) {
        const float4 kd4 = *reinterpret_cast<const float4*>(kdv + e);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = e + 2 * u;
          const uint64_t kd2 = u ? pk(kd4.z, kd4.w) : pk(kd4.x, kd4.y);
          uint64_t x = pk(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1]));
          x = QK == FD_QK_INT8 ? fma2(fma2(x, pk(qd, qd), pk(nq, nq)), kd2, pk(nl, nl))
                               : fma2(mul2(x, pk(qd, qd)), kd2, pk(nl, nl));
          float l0, l1;
          unpk(x, l0, l1);
          float p0 = ex2_approx(l0), p1 = ex2_approx(l1);
          if (!full) {
            if (key0 + c >= p.N) p0 = 0.f;
            if (key0 + c + 1 >= p.N) p1 = 0.f;
          }
          float d0, d1;
          unpk(mul2(pk(p0, p1), add2(pk(__uint_as_float(rd[c]), __uint_as_float(rd[c + 1])), pk(nd, nd))), d0,
               d1);
          wd[c >> 1] = pack_bf16x2(d0, d1);
        }
      }
      // dS(b) is free: step i - 2's dQ product read it before S(i) / dP(i) (issued
      // after it) completed
      st_cols(tdS(b) + lane_base + CW / 2 * c4, wd);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bSdpFree[b]);
        mbar_arrive(&bDsFull[b]);
      }
      ++i;
    }
    if (ok) ok = mbar_wait(bAcc, 0, abort_flag);
    if (ok) {
      tc_fence_after();
      const int64_t orow = ((int64_t)bh * p.N + (q_ok ? qrow : 0)) * HD + EW * c4;
      store_acc(tdQ + lane_base + EW * c4, i > 0, q_ok, p.sm_scale, p.g0 + orow);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == WARP_MMA) tmem_dealloc(tmem_base, TMEM_COLS);
}

template <typename K>
static int set_smem(K kern, uint32_t bytes, bool& done) {
  if (done) return FD_OK;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "attn bwd smem attribute: %s", cudaGetErrorString(e));
  done = true;
  return FD_OK;
}

}  // namespace attn_bwd
}  // namespace fd

using namespace fd;

extern "C" int fd_sage_attn_bwd_prepass(const void* dout, const void* out, float* delta, int64_t BH,
                                        int64_t N, void* stream) {
  FD_CHECK_ARG(BH > 0 && N > 0, "bad shape");
  FD_CHECK_ARG(dout && out && delta, "null pointer");
  FD_CHECK_ARG(aligned8(dout) && aligned8(out), "dout and out must be 8-byte aligned");
  const int64_t rows = BH * N;
  int64_t grid = (rows + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (grid > cap) grid = cap;
  attn_bwd::prepass_kernel<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)dout, (const __nv_bfloat16*)out, delta, rows);
  return check_launch("sage_attn_bwd_prepass");
}

// 3-D map over a (BH, N, 128) tensor of 1- or 2-byte elements: box of `rows` rows,
// 128 bytes wide (the whole row for codes, one 64-column panel for bf16).
static int map_rows(CUtensorMap* m, const void* base, bool bf16, int64_t BH, int64_t N, uint32_t rows) {
  const uint64_t es = bf16 ? 2 : 1;
  const uint64_t dims[3] = {128, (uint64_t)N, (uint64_t)BH};
  const uint64_t strides[2] = {128 * es, (uint64_t)N * 128 * es};
  const uint32_t box[3] = {bf16 ? 64u : 128u, rows, 1};
  return encode_tiled(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims,
                      strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

extern "C" int fd_sage_attn_bwd(const void* q, const void* k, const void* v, const void* dout,
                                   const float* lse, const float* delta, const void* q_codes,
                                   const float* q_desc, const void* k_codes, const float* k_desc,
                                   const uint8_t* block_mask, int64_t mask_bh_stride, void* dq, void* dk,
                                   void* dv, int64_t BH, int64_t N, int qk_kind, float sm_scale, void* stream) {
  using namespace attn_bwd;
  FD_CHECK_ARG(BH > 0 && BH <= 65535 && N > 0 && N < (1ll << 30), "bad shape");
  FD_CHECK_ARG(qk_kind == FD_QK_INT8 || qk_kind == FD_QK_FP8, "bad qk_kind");
  FD_CHECK_ARG(q && k && v && dout && lse && delta && q_codes && q_desc && k_codes && k_desc && dq && dk && dv,
               "null pointer");
  FD_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(dout) && aligned16(q_codes) &&
                   aligned16(k_codes) && aligned16(dq) && aligned16(dk) && aligned16(dv),
               "tensors must be 16-byte aligned");
  CUtensorMap mKc128, mV128, mQc64, mQ64, mDO64, mQc128, mDO128, mKc64, mV64, mKs64;
  int rc = 0;
  if (!rc) rc = map_rows(&mKc128, k_codes, false, BH, N, BT);
  if (!rc) rc = map_rows(&mV128, v, true, BH, N, BT);
  if (!rc) rc = map_rows(&mQc64, q_codes, false, BH, N, BS);
  if (!rc) rc = map_rows(&mQ64, q, true, BH, N, BS);
  if (!rc) rc = map_rows(&mDO64, dout, true, BH, N, BS);
  if (!rc) rc = map_rows(&mQc128, q_codes, false, BH, N, BT);
  if (!rc) rc = map_rows(&mDO128, dout, true, BH, N, BT);
  if (!rc) rc = map_rows(&mKc64, k_codes, false, BH, N, BS);
  if (!rc) rc = map_rows(&mV64, v, true, BH, N, BS);
  if (!rc) rc = map_rows(&mKs64, k, true, BH, N, BS);
  if (rc) return rc;
  Params p;
  p.q_desc = q_desc;
  p.k_desc = k_desc;
  p.lse = lse;
  p.delta = delta;
  p.mask = block_mask;
  p.mask_bh_stride = mask_bh_stride;
  p.N = (int)N;
  p.nkb64 = (int)((N + 63) / 64);
  p.dstride = ((N + 127) / 128) * 128;  // per-token descale layout of fd_attn_quant
  p.sm_scale = sm_scale;
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((unsigned)((N + BT - 1) / BT), (unsigned)BH);
  static bool done[4] = {false, false, false, false};
  const bool i8 = qk_kind == FD_QK_INT8;
  auto kkv = i8 ? bwd_dkdv_kernel<FD_QK_INT8> : bwd_dkdv_kernel<FD_QK_FP8>;
  auto kq = i8 ? bwd_dq_kernel<FD_QK_INT8> : bwd_dq_kernel<FD_QK_FP8>;
  if ((rc = set_smem(kkv, SmemKV::TOTAL, done[i8 ? 0 : 1]))) return rc;
  if ((rc = set_smem(kq, SmemQ::TOTAL, done[i8 ? 2 : 3]))) return rc;
  p.g0 = (__nv_bfloat16*)dk;
  p.g1 = (__nv_bfloat16*)dv;
  kkv<<<grid, NUM_THREADS, SmemKV::TOTAL, st>>>(mKc128, mV128, mQc64, mQ64, mDO64, p);
  if ((rc = check_launch("sage_attn_bwd dkdv"))) return rc;
  p.g0 = (__nv_bfloat16*)dq;
  p.g1 = nullptr;
  kq<<<grid, NUM_THREADS, SmemQ::TOTAL, st>>>(mQc128, mDO128, mKc64, mV64, mKs64, p);
  return check_launch("sage_attn_bwd dq");
}
