// tcgen05 FP8 blockwise-scaled GEMM (G2):
//   C[m, n] = sum_kb ( dot128(A8[m, kb], B8[n, kb]) * a_s[m, kb] * b_s[n/128, kb] ) (+ bias[n])
// Reference: fp8_gemm_blockwise_kernel / fp8_addmm_blockwise_kernel,
// src/futudiffu/fp8_kernels.py:125-193, :235-299 (promotion :183, bias :290-292);
// fp8_gemm_v1t (B stored K x N), :1417-1525.
//
// Design (one persistent CTA per SM, warp specialised, 10 warps):
//   warp 0      TMA producer: 128x128 A and B tiles per 128-K slice into a
//               6-stage shared-memory ring (128-byte swizzle, no multicast).
//   warp 1      MMA issuer: 4 x tcgen05.mma.kind::f8f6f4 (M128 N128 K32) per
//               slice into one of 4 TMEM slice buffers (4 x 128 fp32 columns),
//               then tcgen05.commit to free the smem stage and to publish the
//               slice.
//   warps 2..9  promotion / epilogue: each thread owns one output row and 64
//               columns; per slice it tcgen05.ld's its 64 partial sums, frees
//               the TMEM buffer and does acc += partial * (a_s * b_s) in fp32
//               registers (the per-128-K-slice promotion of the reference).
//               At the end of a tile it adds the bias and stores the row.
// The 4-deep TMEM ring lets the tensor core run up to 3 slices ahead of the
// promotion, so MMA and promotion overlap.
//
// Fused epilogues (EPI), each replacing a GEMM + quantiser pair of the
// reference and producing its exact codes and scales:
//   EPI_STORE      C = acc (+ bias) in bf16 / f16 / f32.
//   EPI_QUANT      fp8_gemm_quant (fp8_kernels.py:573-709): the fp32
//                  accumulator quantised 1 x 128 to e4m3 + fp32 dequant scales.
//   EPI_GELU_TANH  GEMM -> bf16 -> GELU(tanh) -> 1 x 128 e4m3 (the MMDiT MLP:
//                  replaces fp8_addmm + fp8_gelu_tanh_quant).
//   EPI_SILU_GATE  the FFN chain head (transformer.py:536-545): B = [w1; w3]
//                  (2 H x K); a CTA computes the w1 tile and then the matching
//                  w3 tile of the same rows, parks w1 as bf16 in shared memory
//                  and emits silu(w1) * w3 quantised 1 x 128 (replaces
//                  fp8_addmm -> bf16 (M, 2H) -> fp8_silu_gate_quant).
// The two threads that hold the halves of a 128-column group exchange their
// maxima through shared memory (named barrier of the quadrant's two warps).
#include "fd_act.cuh"
#include "fd_host.h"

namespace fd {
namespace gemm {

constexpr int BM = 128, BN = 128, BK = 128;
constexpr int NTBUF = 4;
constexpr int NUM_THREADS = 320;
constexpr int EPI_WARPS = 8;
constexpr uint32_t STAGE_BYTES = BM * BK + BN * BK;  // 32 KiB

enum { EPI_STORE = 0, EPI_QUANT = 1, EPI_GELU_TANH = 2, EPI_SILU_GATE = 3 };

template <int EPI>
struct Layout {
  static constexpr int STAGES = EPI == EPI_SILU_GATE ? 5 : 6;
  static constexpr uint32_t OFF_STASH = STAGES * STAGE_BYTES;                  // w1 tile, bf16
  static constexpr uint32_t STASH_BYTES = EPI == EPI_SILU_GATE ? BM * BN * 2 : 0;
  static constexpr uint32_t OFF_RED = OFF_STASH + STASH_BYTES;                 // [2][2][128] f32
  static constexpr uint32_t RED_BYTES = EPI == EPI_STORE ? 0 : 2 * 2 * 128 * 4;
  static constexpr uint32_t OFF_BAR = OFF_RED + RED_BYTES;
  static constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 /*barriers*/ + 1024 /*align*/;
};

struct Params {
  const float* a_s;
  const float* b_s;
  const void* bias;
  void* c;
  float* c_s;      // quantising epilogues: 1 x 128 dequant scales (M, N_out / 128)
  int M, N, K;     // N: columns of the output (for EPI_SILU_GATE: H, B has 2 H rows)
  int ntm, ntn, ntiles;
  int kblocks;
};

template <int CDT>
FD_DEV void store_row64(void* c, int64_t row_off, int n_start, int N, const float (&v)[64]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int n = n_start + j * 8;
    if (n >= N) break;
    if constexpr (CDT == FD_DT_F32) {
      float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(c) + row_off + n);
      p[0] = make_float4(v[8 * j], v[8 * j + 1], v[8 * j + 2], v[8 * j + 3]);
      p[1] = make_float4(v[8 * j + 4], v[8 * j + 5], v[8 * j + 6], v[8 * j + 7]);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if constexpr (CDT == FD_DT_BF16) {
          w[e] = pack_bf16x2(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
        } else {
          __half2 h = __floats2half2_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
          w[e] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(c) + row_off + n) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <int BDT>
FD_DEV float load_bias(const void* bias, int n) {
  if constexpr (BDT == FD_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
  else if constexpr (BDT == FD_DT_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  else return reinterpret_cast<const float*>(bias)[n];
}

// Wait that ignores the abort flag: used only to drain this thread's own
// in-flight asynchronous work before the CTA exits.
FD_DEV void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > FD_WAIT_NS) {
      atomicOr(&g_status, FD_STATUS_TIMEOUT);
      return;
    }
  }
}

// BMODE: 0 -> B stored (N, K) (K-major), b_s (ceil(N/128), K/128)
//        1 -> B stored (K, N) (MN-major, v1t), b_s (K/128, ceil(N/128))
//        2 -> B stored (N, K), per-row scales b_s (N,) applied after the K loop
FD_DEV void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <int BMODE, int CDT, int BDT, int EPI>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const Params p) {
  using LY = Layout<EPI>;
  constexpr int STAGES = LY::STAGES;
  constexpr int NSUB = EPI == EPI_SILU_GATE ? 2 : 1;  // GEMM tiles per output tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * BM * BK;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::OFF_BAR);
  uint64_t* full = bars;                   // [STAGES]
  uint64_t* empty = bars + STAGES;         // [STAGES]
  uint64_t* tfull = bars + 2 * STAGES;     // [NTBUF]
  uint64_t* tempty = tfull + NTBUF;        // [NTBUF]
  uint64_t* drain = tempty + NTBUF;        // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  constexpr int B_MN = BMODE == 1 ? 1 : 0;
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < NTBUF; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      uint32_t issued_mask = 0;  // stages with a load issued
      for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
        const int mb = tile % p.ntm, nbo = tile / p.ntm;
        for (int sub = 0; sub < NSUB && ok; ++sub) {
          const int nb = nbo + sub * p.ntn;  // EPI_SILU_GATE: w3 rows follow the H w1 rows
          for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
            const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
            tma_load_2d(sA + s * (BM * BK), &tmA, &full[s], kb * BK, mb * BM);
            if (B_MN) tma_load_2d(sB + s * (BN * BK), &tmB, &full[s], nb * BN, kb * BK);
            else tma_load_2d(sB + s * (BN * BK), &tmB, &full[s], kb * BK, nb * BN);
            issued_mask |= 1u << s;
          }
        }
      }
      // Drain: the newest load of every stage must have landed before exit.
      for (uint32_t s = 0; s < (uint32_t)STAGES; ++s) {
        if (!(issued_mask & (1u << s))) continue;
        // newest load into stage s was iteration j with j % STAGES == s, j < it
        const uint32_t last = it - 1 - ((it - 1 - s) % STAGES);
        drain_wait(&full[s], (last / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(/*c F32*/ 1, /*E4M3*/ 0, 0, /*a K-major*/ 0, B_MN, BM, BN);
      uint32_t it = 0;
      bool ok = true;
      // GEMM tiles in the producer's order: per output tile, NSUB sub-tiles
      const int ngemm = ((p.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * NSUB;
      for (int g = 0; g < ngemm && ok; ++g) {
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
          const uint32_t tb = it % NTBUF, tph = (it / NTBUF) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&tempty[tb], tph ^ 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * (BM * BK));
          const uint32_t b0 = smem_u32(sB + s * (BN * BK));
          const uint32_t d = tmem_base + tb * BN;
#pragma unroll
          for (int k4 = 0; k4 < BK / 32; ++k4) {
            const uint64_t ad = make_sdesc_sw128(a0 + k4 * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sdesc_sw128(b0 + k4 * 32 * 128, 16, 1024)
                                     : make_sdesc_sw128(b0 + k4 * 32, 16, 1024);
            mma_f8f6f4_ss(d, ad, bd, idesc, k4 > 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          tc_commit(&tfull[tb]);
        }
      }
      tc_commit(drain);
      drain_wait(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ promotion + epilogue
    const int q = warp & 3;             // TMEM lane quadrant this warp may access
    const int h = (warp - 2) >> 2;      // column half: 0 -> cols 0..63, 1 -> 64..127
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int r = q * 32 + lane;        // row within the tile
    const int et = h * 128 + r;         // epilogue thread index 0..255
    uint4* stash = reinterpret_cast<uint4*>(smem + LY::OFF_STASH);  // [8][256] x 16 B
    float* red = reinterpret_cast<float*>(smem + LY::OFF_RED);      // [parity][half][128]
    uint32_t it = 0, nt = 0;
    bool ok = true;
    // A thread whose wait timed out keeps walking the tiles (skipping the work)
    // so its partner is never left at the max-exchange barrier.
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++nt) {
      const int mb = tile % p.ntm, nbo = tile / p.ntm;
      const int m = mb * BM + r;
      const bool row_ok = m < p.M;
      const float* as_row = p.a_s + (int64_t)(row_ok ? m : 0) * p.kblocks;
      for (int sub = 0; sub < NSUB; ++sub) {
        const int nb = nbo + sub * p.ntn;
        float acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = 0.f;
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const uint32_t tb = it % NTBUF, tph = (it / NTBUF) & 1;
          const float bs = BMODE == 1   ? __ldg(p.b_s + (int64_t)kb * (p.ntn * NSUB) + nb)
                           : BMODE == 0 ? __ldg(p.b_s + (int64_t)nb * p.kblocks + kb)
                                        : 1.0f;
          const float sc = (row_ok ? __ldg(as_row + kb) : 0.f) * bs;
          ok = ok && mbar_wait(&tfull[tb], tph, abort_flag);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) continue;
          tc_fence_after();
          uint32_t r0[32], r1[32];
          const uint32_t taddr = tmem_base + lane_base + tb * BN + h * 64;
          tmem_ld32(taddr, r0);
          tmem_ld32(taddr + 32, r1);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[tb]);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            acc[i] = fmaf(__uint_as_float(r0[i]), sc, acc[i]);
            acc[32 + i] = fmaf(__uint_as_float(r1[i]), sc, acc[32 + i]);
          }
        }
        const int n0 = nb * BN + h * 64;  // column of acc[0] in the GEMM output
        if (BMODE == 2) {
          // fp8_gemm_rowwise_kernel: accumulator *= b_s[n] after the K loop (:407-408)
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int n = n0 + i;
            acc[i] *= (n < p.N) ? __ldg(p.b_s + n) : 0.f;
          }
        }
        if (BDT >= 0 && p.bias) {
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int n = n0 + i;
            if (EPI == EPI_SILU_GATE || n < p.N) acc[i] += load_bias<BDT < 0 ? FD_DT_F32 : BDT>(p.bias, n);
          }
        }
        if constexpr (EPI == EPI_STORE) {
          if (ok && row_ok) store_row64<CDT>(p.c, (int64_t)m * p.N, n0, p.N, acc);
        } else {
          if (EPI == EPI_SILU_GATE && sub == 0) {
            // w1 tile: the reference rounds the w1w3 GEMM output to bf16; park it
#pragma unroll
            for (int k = 0; k < 8; ++k)
              stash[k * 256 + et] =
                  make_uint4(pack_bf16x2(acc[8 * k], acc[8 * k + 1]), pack_bf16x2(acc[8 * k + 2], acc[8 * k + 3]),
                             pack_bf16x2(acc[8 * k + 4], acc[8 * k + 5]), pack_bf16x2(acc[8 * k + 6], acc[8 * k + 7]));
            continue;
          }
          if (EPI == EPI_GELU_TANH) {
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = gelu_tanh(round_to_bf16(acc[i]));
          } else if (EPI == EPI_SILU_GATE) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint4 w = stash[k * 256 + et];
              const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                acc[8 * k + 2 * e] = silu_gate(__uint_as_float(ww[e] << 16), round_to_bf16(acc[8 * k + 2 * e]));
                acc[8 * k + 2 * e + 1] =
                    silu_gate(__uint_as_float(ww[e] & 0xFFFF0000u), round_to_bf16(acc[8 * k + 2 * e + 1]));
              }
            }
          }
          // 1 x 128 group = this thread's 64 columns and its partner's
          float amax = 0.f;
#pragma unroll
          for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(acc[i]));
          float* rd = red + (nt & 1) * 256;
          rd[h * 128 + r] = amax;
          named_bar_sync(1 + q, 64);
          amax = fmaxf(amax, rd[(h ^ 1) * 128 + r]);
          if (ok && row_ok) {
            const float qm = quant_mult(amax);
            const int c0 = nbo * BN + h * 64;  // output column of acc[0]
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.c) + (int64_t)m * p.N + c0);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              dst[k] = make_uint4(quant4(acc[16 * k], acc[16 * k + 1], acc[16 * k + 2], acc[16 * k + 3], qm),
                                  quant4(acc[16 * k + 4], acc[16 * k + 5], acc[16 * k + 6], acc[16 * k + 7], qm),
                                  quant4(acc[16 * k + 8], acc[16 * k + 9], acc[16 * k + 10], acc[16 * k + 11], qm),
                                  quant4(acc[16 * k + 12], acc[16 * k + 13], acc[16 * k + 14], acc[16 * k + 15], qm));
            if (h == 0) p.c_s[(int64_t)m * (p.N / BN) + nbo] = dequant_scale(amax);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 512);
}

template <int BMODE, int CDT, int BDT, int EPI = EPI_STORE>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, cudaStream_t st) {
  auto kern = gemm_fp8_kernel<BMODE, CDT, BDT, EPI>;
  constexpr uint32_t smem_bytes = Layout<EPI>::SMEM_BYTES;
  static bool attr_done = false;  // per instantiation
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "gemm smem attribute: %s", cudaGetErrorString(e));
    attr_done = true;
  }
  const int grid = p.ntiles < num_sms() ? p.ntiles : num_sms();
  kern<<<grid, NUM_THREADS, smem_bytes, st>>>(ta, tb, p);
  return check_launch("fp8_gemm_blockwise");
}

template <int EPI>
static int launch_quant(int bdt, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                        cudaStream_t st) {
  if (!p.bias) return launch<0, -1, -1, EPI>(ta, tb, p, st);
  switch (bdt) {
    case FD_DT_BF16: return launch<0, -1, FD_DT_BF16, EPI>(ta, tb, p, st);
    case FD_DT_F16: return launch<0, -1, FD_DT_F16, EPI>(ta, tb, p, st);
    case FD_DT_F32: return launch<0, -1, FD_DT_F32, EPI>(ta, tb, p, st);
    default: return set_error(FD_ERR_ARG, "unsupported bias dtype");
  }
}

template <int BMODE, int CDT>
static int launch_bias(int bdt, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                       cudaStream_t st) {
  if (!p.bias) return launch<BMODE, CDT, -1>(ta, tb, p, st);
  switch (bdt) {
    case FD_DT_BF16: return launch<BMODE, CDT, FD_DT_BF16>(ta, tb, p, st);
    case FD_DT_F16: return launch<BMODE, CDT, FD_DT_F16>(ta, tb, p, st);
    case FD_DT_F32: return launch<BMODE, CDT, FD_DT_F32>(ta, tb, p, st);
    default: return set_error(FD_ERR_ARG, "unsupported bias dtype");
  }
}

template <int BMODE>
static int launch_c(int cdt, int bdt, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                    cudaStream_t st) {
  switch (cdt) {
    case FD_DT_BF16: return launch_bias<BMODE, FD_DT_BF16>(bdt, ta, tb, p, st);
    case FD_DT_F16: return launch_bias<BMODE, FD_DT_F16>(bdt, ta, tb, p, st);
    case FD_DT_F32: return launch_bias<BMODE, FD_DT_F32>(bdt, ta, tb, p, st);
    default: return set_error(FD_ERR_ARG, "unsupported output dtype");
  }
}

}  // namespace gemm
}  // namespace fd

using namespace fd;

extern "C" int fd_fp8_gemm_blockwise(const void* a, const float* a_s, const void* b,
                                     const float* b_s, const void* bias, int bias_dtype, void* c,
                                     int c_dtype, int64_t M, int64_t N, int64_t K, int b_layout,
                                     void* stream) {
  FD_CHECK_ARG(M >= 0 && N > 0 && K > 0, "bad shape");
  FD_CHECK_ARG(K % 128 == 0, "K must be a multiple of 128");
  FD_CHECK_ARG(N % 16 == 0, "N must be a multiple of 16");
  FD_CHECK_ARG(b_layout >= 0 && b_layout <= 2,
               "b_layout must be 0 (N,K), 1 (K,N) or 2 (N,K) with per-row scales");
  FD_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "dimension too large");
  if (M == 0) return FD_OK;
  FD_CHECK_ARG(a && a_s && b && b_s && c, "null pointer");
  FD_CHECK_ARG(aligned16(a) && aligned16(b) && aligned16(c), "a, b, c must be 16-byte aligned");
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {128, 128};
    int rc = encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if (b_layout != 1) {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {128, 128};
    int rc = encode_tiled(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, b, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)N};
    const uint32_t box[2] = {128, 128};
    int rc = encode_tiled(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, b, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  gemm::Params p;
  p.a_s = a_s;
  p.b_s = b_s;
  p.bias = bias;
  p.c = c;
  p.c_s = nullptr;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ntm = (int)((M + 127) / 128);
  p.ntn = (int)((N + 127) / 128);
  p.ntiles = p.ntm * p.ntn;
  p.kblocks = (int)(K / 128);
  cudaStream_t st = (cudaStream_t)stream;
  if (b_layout == 0) return gemm::launch_c<0>(c_dtype, bias_dtype, ta, tb, p, st);
  if (b_layout == 1) return gemm::launch_c<1>(c_dtype, bias_dtype, ta, tb, p, st);
  return gemm::launch_c<2>(c_dtype, bias_dtype, ta, tb, p, st);
}

// GEMM with a quantising epilogue (see the header of this file): act 0 requantises
// the fp32 accumulator (fp8_gemm_quant), 1 applies GELU(tanh) to the bf16 GEMM
// output first, 2 is the SiLU gate with b = [w1; w3] of shape (2 N, K).
extern "C" int fd_fp8_gemm_quant(const void* a, const float* a_s, const void* b, const float* b_s,
                                 const void* bias, int bias_dtype, void* c, float* c_s, int64_t M,
                                 int64_t N, int64_t K, int act, void* stream) {
  FD_CHECK_ARG(M >= 0 && N > 0 && K > 0, "bad shape");
  FD_CHECK_ARG(K % 128 == 0, "K must be a multiple of 128");
  FD_CHECK_ARG(N % 128 == 0, "N must be a multiple of 128 (1 x 128 output groups)");
  FD_CHECK_ARG(act >= FD_ACT_NONE && act <= FD_ACT_SILU_GATE, "bad act");
  const int64_t nb_rows = act == FD_ACT_SILU_GATE ? 2 * N : N;  // rows of b
  FD_CHECK_ARG(M < (1ll << 31) && nb_rows < (1ll << 31) && K < (1ll << 31), "dimension too large");
  if (M == 0) return FD_OK;
  FD_CHECK_ARG(a && a_s && b && b_s && c && c_s, "null pointer");
  FD_CHECK_ARG(aligned16(a) && aligned16(b) && aligned16(c), "a, b, c must be 16-byte aligned");
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {128, 128};
    int rc = encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)nb_rows};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {128, 128};
    int rc = encode_tiled(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, b, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  gemm::Params p;
  p.a_s = a_s;
  p.b_s = b_s;
  p.bias = bias;
  p.c = c;
  p.c_s = c_s;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ntm = (int)((M + 127) / 128);
  p.ntn = (int)(N / 128);
  p.ntiles = p.ntm * p.ntn;
  p.kblocks = (int)(K / 128);
  cudaStream_t st = (cudaStream_t)stream;
  if (act == FD_ACT_NONE) return gemm::launch_quant<gemm::EPI_QUANT>(bias_dtype, ta, tb, p, st);
  if (act == FD_ACT_GELU_TANH) return gemm::launch_quant<gemm::EPI_GELU_TANH>(bias_dtype, ta, tb, p, st);
  return gemm::launch_quant<gemm::EPI_SILU_GATE>(bias_dtype, ta, tb, p, st);
}
