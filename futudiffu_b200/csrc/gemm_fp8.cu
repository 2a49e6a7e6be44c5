// tcgen05 FP8 blockwise-scaled GEMM (G2):
//   C[m, n] = sum_kb ( dot128(A8[m, kb], B8[n, kb]) * a_s[m, kb] * b_s[n/128, kb] ) (+ bias[n])
// Reference: fp8_gemm_blockwise_kernel / fp8_addmm_blockwise_kernel,
// src/futudiffu/fp8_kernels.py:125-193, :235-299 (promotion :183, bias :290-292);
// fp8_gemm_v1t (B stored K x N), :1417-1525.
//
// Design (one persistent CTA per SM, warp specialised, 10 warps):
//   warp 0      TMA producer: a 128 x 128 A tile and a 256 x 128 B tile per
//               128-K slice into a 4-stage shared-memory ring (128-byte
//               swizzle, one plain TMA copy per tile).
//   warp 1      MMA issuer: 4 x tcgen05.mma.kind::f8f6f4 (M128 N256 K32) per
//               slice into one of 2 TMEM slice buffers (2 x 256 fp32 columns),
//               then tcgen05.commit to free the smem stage and to publish the
//               slice.
//   warps 2..9  promotion / epilogue: each thread owns one output row and 128
//               columns (one 1 x 128 output group); per slice it tcgen05.ld's
//               its partial sums, frees the TMEM buffer and does
//               acc += partial * (a_s * b_s) in fp32 registers (the
//               per-128-K-slice promotion of the reference).
// Why N = 256: an M128 N128 K32 MMA reads 8 KiB of operands from shared memory
// in its 64 cycles, the SM's whole shared-memory bandwidth, and the TMA writes
// of the next slice compete for the same bandwidth; at N = 256 each staged
// byte feeds twice the MMA work (48 KiB per 512 MMA cycles instead of 32 KiB
// per 256).  Tiles are visited in groups of GROUP_M row tiles so that the
// tiles running at the same time share their A and B tiles in L2.
//
// Fused epilogues (EPI), each replacing a GEMM + quantiser pair of the
// reference and producing its exact codes and scales:
//   EPI_STORE      C = acc (+ bias) in bf16 / f16 / f32.
//   EPI_QUANT      fp8_gemm_quant (fp8_kernels.py:573-709): the fp32
//                  accumulator quantised 1 x 128 to e4m3 + fp32 dequant scales.
//   EPI_GELU_TANH  GEMM -> bf16 -> GELU(tanh) -> 1 x 128 e4m3 (the MMDiT MLP:
//                  replaces fp8_addmm + the GELU-tanh quantiser).
//   EPI_SILU_GATE  the FFN chain head (src_ii/transformer.py:536-545): B = [w1; w3]
//                  (2 H x K); the B tile holds w1 block nb and w3 block nb, so one
//                  accumulator holds both halves of a gate group; emits
//                  silu(bf16 w1) * bf16 w3 quantised 1 x 128 (replaces
//                  fp8_addmm -> bf16 (M, 2H) -> fp8_silu_gate_quant).
// For EPI_QUANT / EPI_GELU_TANH a thread's 128 columns are one output group; for
// EPI_SILU_GATE the two threads holding the halves of a group exchange their
// maxima through shared memory (named barrier of the quadrant's two warps).
//
// Multi-LoRA (EPI_STORE): the adapter delta sum_j s_j (x A_j^T) B_j^T of the
// reference's MultiLoRALinear (src_ii/multi_lora.py:231-325, lora_kernels.py:55-157)
// enters as extra 64-wide K slices after the FP8 slices: A = the per-token
// scaled mid activations h (M, K_lora) bf16, B = [B_1 | B_2 | ...] (N, K_lora)
// bf16, one tcgen05 kind::f16 MMA group per slice, promoted with scale 1, so
// the delta is added to the fp32 accumulator before the single output rounding.
#include "fd_act.cuh"
#include "fd_p3.cuh"
#include "fd_host.h"

namespace fd {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 128;  // BN: MMA / TMEM columns per tile
constexpr int NTBUF = 2;                       // TMEM slice buffers (2 x 256 columns)
constexpr int EPI_WARPS = 8;                   // promotion warps
constexpr int GROUP_M = 16;                    // row tiles per rasterisation group
constexpr uint32_t A_BYTES = BM * BK;          // 16 KiB
constexpr uint32_t STAGE_BYTES = BM * BK + BN * BK;  // 48 KiB

enum { EPI_STORE = 0, EPI_QUANT = 1, EPI_GELU_TANH = 2, EPI_SILU_GATE = 3, EPI_QKV = 4 };

constexpr uint32_t STG_WARP = 32 * 128;  // output staging per epilogue warp: 32 rows x 128 B

// Per-epilogue configuration.  Every epilogue but GELU-tanh runs on 10 warps:
// warp 0 TMA producer, warp 1 MMA issuer, warps 2-9 promotion + epilogue, with
// a 4-stage operand ring.  GELU-tanh (deferred): its epilogue costs about as
// much issue time per tile as the promotion of all K slices, and on the
// promotion warps it left the tensor core idle for that long, so it runs on
// four more warps instead: the promotion warps (4-11) hand the bf16-rounded
// tile to warps 12-15 through shared memory and go on with the next tile while
// those evaluate GELU(tanh) and requantise.  The 64 KiB tile copy leaves room
// for 3 operand stages.
template <int EPI>
struct Cfg {
  static constexpr bool DEFER = EPI == EPI_GELU_TANH || EPI == EPI_QKV;
  static constexpr int STAGES = DEFER ? 3 : 4;
  static constexpr int THREADS = DEFER ? 512 : 320;
  static constexpr int PROMO_WARP0 = DEFER ? 4 : 2;  // first promotion warp
  static constexpr int GELU_WARP0 = 12;              // deferred GELU warps 12-15
  // non-deferred: TMA-store staging (32 rows x 128 B per promotion warp), whose
  // bytes the SiLU-gate epilogue uses for its [2][2][128] f32 max exchange;
  // deferred: the bf16 tile copy, 128 rows x 256 values (512 B per row)
  static constexpr uint32_t OFF_STG = STAGES * STAGE_BYTES;
  static constexpr uint32_t OFF_RED = OFF_STG;
  static constexpr uint32_t STG_BYTES = DEFER ? BM * BN * 2 : EPI_WARPS * STG_WARP;
  // EPI_QKV: per-(head, virtual warp, column) K sums or V absmax, [2][8][128] f32,
  // and the Q block maxima per (head, virtual warp)
  static constexpr uint32_t OFF_QKV = OFF_STG + STG_BYTES;
  static constexpr uint32_t QKV_BYTES = EPI == EPI_QKV ? 2 * 8 * 128 * 4 + 64 : 0;
  static constexpr uint32_t OFF_BAR = OFF_QKV + QKV_BYTES;
  static constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 /*barriers*/ + 1024 /*align*/;
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

// Register split of the deferred-epilogue kernels, launched with 128 registers
// per thread x 512 threads (the whole register file; ptxas reports 128 for
// these instantiations): warps 0-3 (producer, MMA issuer, two idle) keep 40, the
// eight promotion warps take 168 (their 128 fp32 accumulators), the four
// epilogue warps keep 104 (GELU) or take 136 (EPI_QKV: each lane holds 16 values
// of a row and their rotations): 128 x 40 + 256 x 168 + 128 x 104 = 61440 and 128 x 40 + 256 x 168 +
// 128 x 136 = 65536 registers, within the launch's 65536.
template <int N>
FD_DEV void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
FD_DEV void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Maximum of the eight bf16 values packed in u.
FD_DEV float max8_bf16(const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(bf16_bits_to_f32(w[j] & 0xffffu), bf16_bits_to_f32(w[j] >> 16)));
  return m;
}

// |GELU(tanh)| maximum of the eight bf16 values packed in u (low half first).
FD_DEV float gelu8_absmax(const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    m = fmaxf(m, fmaxf(fabsf(gelu_tanh(bf16_bits_to_f32(w[j] & 0xffffu))), fabsf(gelu_tanh(bf16_bits_to_f32(w[j] >> 16)))));
  return m;
}

// e4m3 codes of GELU(tanh) of the eight bf16 values in u, multiplied by qm.
FD_DEV uint2 gelu8_codes(const uint4& u, float qm) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float g[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    g[2 * j] = bf16_bits_to_f32(w[j] & 0xffffu);
    g[2 * j + 1] = bf16_bits_to_f32(w[j] >> 16);
    gelu_tanh2(g[2 * j], g[2 * j + 1]);
  }
  return make_uint2(quant4(g[0], g[1], g[2], g[3], qm), quant4(g[4], g[5], g[6], g[7], qm));
}

// EPI_QKV: the QKV linear of one stream of a joint attention with P3 (per-head
// Q/K RMSNorm + RoPE) and the attention prologue's first pass in its epilogue
// (the arithmetic of qkv_quant_kernel in attn_prologue.cu, shared through
// fd_p3.cuh): Q as codes + descales, K and V in bf16, per-chunk K column sums and
// V column absmax in the workspace.  GEMM rows are the stream's B x S tokens
// (S a multiple of 128), GEMM columns [Q | K | V] x H heads x 128.
struct QkvEpi {
  const float* qw;      // (128,) Q norm weight
  const float* kw;      // (128,) K norm weight
  const float* freqs;   // (B S, 64, 2, 2) RoPE rotations of the stream's rows
  uint8_t* q_codes;     // (B H, Nj, 128)
  float* q_desc;        // (B H, q_desc_stride)
  __nv_bfloat16* k_out; // (B H, Nj, 128)
  __nv_bfloat16* v_out;
  float* ws_sum;        // (B H, nchunks, 128)
  float* ws_amax;
  int64_t q_desc_stride;
  float eps, sm_scale_log2e;
  int S, H, Nj, s_off, q_gran, qk, nchunks, do_v;
};

struct Params {
  const float* a_s;
  const float* b_s;
  const void* bias;
  void* c;
  float* c_s;      // quantising epilogues: 1 x 128 dequant scales (M, N_out / 128)
  int M, N, K;     // N: columns of the output (for EPI_SILU_GATE: H, B has 2 H rows)
  int ntm, ntn, ntiles;  // ntn: output column tiles (256 wide; 128 wide for EPI_SILU_GATE)
  int kblocks;
  int nbs;         // rows of b_s (BMODE 0: ceil(rows of B / 128)); BMODE 1: its columns
  int lora_slices; // 64-column bf16 LoRA slices after the FP8 slices (EPI_STORE, BMODE 0)
  int64_t ldc;     // row stride of c in elements (N unless the output is a column window)
  int64_t ldcs;    // row stride of c_s in scales (N / 128 likewise)
  QkvEpi qe;       // EPI_QKV only
};

// Tile t -> (row tile, column tile), GROUP_M row tiles at a time so that the
// CTAs running together reuse their A and B tiles from L2.
FD_DEV void tile_coords(const Params& p, int t, int& mb, int& nb) {
  const int per_group = GROUP_M * p.ntn;
  const int g = t / per_group, r = t % per_group;
  const int m0 = g * GROUP_M;
  const int gm = min(GROUP_M, p.ntm - m0);
  mb = m0 + r % gm;
  nb = r / gm;
}

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

template <int CDT>
FD_DEV uint32_t pack2(float a, float b) {
  if constexpr (CDT == FD_DT_BF16) {
    return pack_bf16x2(a, b);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <int BDT>
FD_DEV float load_bias(const void* bias, int n) {
  if constexpr (BDT == FD_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
  else if constexpr (BDT == FD_DT_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  else return reinterpret_cast<const float*>(bias)[n];
}

// bias[n .. n + 8) as floats; bias 16-byte aligned, n a multiple of 8
template <int BDT>
FD_DEV void load_bias8(const void* bias, int n, float (&b)[8]) {
  if constexpr (BDT == FD_DT_F32) {
    const float4 u = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(bias) + n));
    const float4 v = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(bias) + n + 4));
    b[0] = u.x; b[1] = u.y; b[2] = u.z; b[3] = u.w; b[4] = v.x; b[5] = v.y; b[6] = v.z; b[7] = v.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(bias) + n));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (BDT == FD_DT_BF16) {
        b[2 * j] = __uint_as_float(w[j] << 16);
        b[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
      } else {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
        const float2 f = __half22float2(h);
        b[2 * j] = f.x;
        b[2 * j + 1] = f.y;
      }
    }
  }
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

// AND of `pred` over the `nthreads` threads of named barrier `id` (all of them wait).
FD_DEV bool named_bar_and(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

constexpr int QKV_BAR = 6;  // named barrier of the four EPI_QKV epilogue warps

// EPI_QKV epilogue of one 128 x 256 tile (two heads of Q, K or V) by the four
// epilogue warps, from the promotion warps' bf16 copy of the tile (hbuf: row r at
// r * 512, 16-byte chunk c of the row at c ^ (r & 7)).  Every value, sum and code
// equals qkv_quant_kernel's (attn_prologue.cu) bit for bit.  That kernel gives a
// (row, head) to a warp, lane L holding columns 4L .. 4L + 3, and its "virtual
// warp" v in 0..7 takes rows v + 8 i in increasing i.  Here eight lanes share a
// (row, head): lane l of a group plays lanes l, l + 8, l + 16 and l + 24, whose
// partial sums of squares it adds as the xor-16 and xor-8 steps of the warp
// butterfly would ((p0 + p2) + (p1 + p3)); the xor-4 / 2 / 1 steps stay inside the
// group.  Group g of warp w4 is virtual warp 2 w4 + (g & 1) for head g >> 1, so
// each K / V column sum still runs over a virtual warp's rows in increasing order
// and over the eight virtual warps in order.
template <int QK>
FD_DEV void qkv_epilogue_tile(const Params& p, uint8_t* hbuf, float* red, int mb, int nb, int w4, int lane) {
  const QkvEpi& e = p.qe;
  const float qmax = (QK == FD_QK_INT8) ? 127.0f : 448.0f;
  const int D = e.H * 128;
  const int col0 = nb * BN;
  const int part = col0 / D;  // 0 Q, 1 K, 2 V
  const int h0 = (col0 - part * D) / 128;
  const int row0 = mb * BM;
  const int b = row0 / e.S, s0 = row0 - b * e.S;
  const int chunk = (e.s_off + s0) / 128;
  const int grp = lane >> 3, l8 = lane & 7;
  const int vw = 2 * w4 + (grp & 1);  // virtual warp
  const int hh = grp >> 1;            // head of the tile
  const int64_t bh = (int64_t)b * e.H + h0 + hh;
  float* sh_c = red;                  // [2 heads][8 virtual warps][128] K sums or V absmax
  float* sh_q = red + 2048;           // [2 heads][8 virtual warps] Q block maxima
  const int t128 = w4 * 32 + lane;
  // the norm weights (read at use from L1: registers go to the row's values)
  const float4* wp = reinterpret_cast<const float4*>(part == 0 ? e.qw : e.kw);
  float cs[4][4];  // K column sums / V column absmax of the four played lanes
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int k = 0; k < 4; ++k) cs[q][k] = 0.f;
  float bmax = 0.f;
  // smem address of played lane q's four values in row r
  auto haddr = [&](int r, int q) {
    return hbuf + r * 512 + ((((hh * 16) + 4 * q + (l8 >> 1)) ^ (r & 7)) << 4) + ((l8 & 1) << 3);
  };
#pragma unroll 1
  for (int i = 0; i < 16; ++i) {
    const int r = vw + 8 * i;
    const int64_t n = e.s_off + s0 + r;
    const int64_t obase = (bh * e.Nj + n) * 128 + 4 * l8;  // + 32 q: played lane l8 + 8 q
    float4 f[4][2];
    if (part != 2) {
      const float4* fr = reinterpret_cast<const float4*>(e.freqs + (int64_t)(row0 + r) * 256);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        f[q][0] = __ldg(fr + 2 * (l8 + 8 * q));
        f[q][1] = __ldg(fr + 2 * (l8 + 8 * q) + 1);
      }
    }
    uint2 u[4];
    float x[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      u[q] = *reinterpret_cast<const uint2*>(haddr(r, q));
      x[q][0] = bf16_bits_to_f32(u[q].x & 0xFFFF);
      x[q][1] = bf16_bits_to_f32(u[q].x >> 16);
      x[q][2] = bf16_bits_to_f32(u[q].y & 0xFFFF);
      x[q][3] = bf16_bits_to_f32(u[q].y >> 16);
    }
    if (part == 2) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        *reinterpret_cast<uint2*>(e.v_out + obase + 32 * q) = u[q];
#pragma unroll
        for (int k = 0; k < 4; ++k) cs[q][k] = fmaxf(cs[q][k], fabsf(x[q][k]));
      }
      continue;
    }
    float ss = __fadd_rn(__fadd_rn(p3_sumsq4(x[0]), p3_sumsq4(x[2])), __fadd_rn(p3_sumsq4(x[1]), p3_sumsq4(x[3])));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rr = p3_rinv(ss, e.eps);
    float y[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 t = __ldg(wp + l8 + 8 * q);
      const float wq[4] = {t.x, t.y, t.z, t.w};
      p3_rope4(x[q], rr, wq, f[q], y[q]);
#pragma unroll
      for (int k = 0; k < 4; ++k) y[q][k] = round_to_bf16(y[q][k]);
    }
    if (part == 1) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        *reinterpret_cast<uint2*>(e.k_out + obase + 32 * q) =
            make_uint2(pack_bf16x2(y[q][0], y[q][1]), pack_bf16x2(y[q][2], y[q][3]));
#pragma unroll
        for (int k = 0; k < 4; ++k) cs[q][k] += y[q][k];
      }
      continue;
    }
    float qa = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int k = 0; k < 4; ++k) qa = fmaxf(qa, fabsf(y[q][k]));
    if (e.q_gran == FD_GRAN_TOKEN) {
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) qa = fmaxf(qa, __shfl_xor_sync(0xffffffffu, qa, o));
      const float inv = div_full(qmax, fmaxf(qa, 1e-12f));
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint32_t*>(e.q_codes + obase + 32 * q) =
            quant_code<QK>(y[q][0], inv) | (quant_code<QK>(y[q][1], inv) << 8) |
            (quant_code<QK>(y[q][2], inv) << 16) | (quant_code<QK>(y[q][3], inv) << 24);
      if (l8 == 0) e.q_desc[bh * e.q_desc_stride + n] = div_full(qa, qmax) * e.sm_scale_log2e;
    } else {
      bmax = fmaxf(bmax, qa);
#pragma unroll
      for (int q = 0; q < 4; ++q)  // kept until the block's absmax is known
        *reinterpret_cast<uint2*>(haddr(r, q)) = make_uint2(pack_bf16x2(y[q][0], y[q][1]), pack_bf16x2(y[q][2], y[q][3]));
    }
  }
  if (part != 0) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int k = 0; k < 4; ++k) sh_c[(hh * 8 + vw) * 128 + 4 * (l8 + 8 * q) + k] = cs[q][k];
    named_bar_sync(QKV_BAR, 128);
    const int c = t128;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int64_t bh2 = (int64_t)b * e.H + h0 + h2;
      float tsum = 0.f, amax = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float t = sh_c[(h2 * 8 + w) * 128 + c];
        tsum += t;
        amax = fmaxf(amax, t);
      }
      if (part == 1) e.ws_sum[(bh2 * e.nchunks + chunk) * 128 + c] = tsum;
      else if (e.do_v) e.ws_amax[(bh2 * e.nchunks + chunk) * 128 + c] = amax;
    }
    named_bar_sync(QKV_BAR, 128);
  } else if (e.q_gran == FD_GRAN_BLOCK) {
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, o));
    if (l8 == 0) sh_q[hh * 8 + vw] = bmax;
    named_bar_sync(QKV_BAR, 128);
    float mx = sh_q[hh * 8];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, sh_q[hh * 8 + w]);
    if (vw == 0 && l8 == 0) e.q_desc[bh * e.q_desc_stride + chunk] = div_full(mx, qmax) * e.sm_scale_log2e;
    const float inv = div_full(qmax, fmaxf(mx, 1e-12f));
#pragma unroll 2
    for (int i = 0; i < 16; ++i) {
      const int r = vw + 8 * i;
      const int64_t obase = (bh * e.Nj + e.s_off + s0 + r) * 128 + 4 * l8;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint2 u = *reinterpret_cast<const uint2*>(haddr(r, q));
        const float y0 = bf16_bits_to_f32(u.x & 0xFFFF), y1 = bf16_bits_to_f32(u.x >> 16);
        const float y2 = bf16_bits_to_f32(u.y & 0xFFFF), y3 = bf16_bits_to_f32(u.y >> 16);
        *reinterpret_cast<uint32_t*>(e.q_codes + obase + 32 * q) = quant_code<QK>(y0, inv) |
                                                                  (quant_code<QK>(y1, inv) << 8) |
                                                                  (quant_code<QK>(y2, inv) << 16) |
                                                                  (quant_code<QK>(y3, inv) << 24);
      }
    }
    named_bar_sync(QKV_BAR, 128);
  }
}

// GROUPED: two independent problems (p0 with tmA / tmB, p1 with tmLA / tmLB) in one
// persistent launch; tiles [0, p0.ntiles) belong to p0, the rest to p1, so a small
// problem (a 512-row text stream) fills the SMs the large one leaves idle.
// tmC0 / tmC1: the output of p0 / p1 for the epilogues that write through TMA
// (bf16 / f16 stores and the 1 x 128 code epilogues except the SiLU gate).
template <int BMODE, int CDT, int BDT, int EPI, bool LORA, bool GROUPED>
__global__ void __launch_bounds__(Cfg<EPI>::THREADS, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmLA, const __grid_constant__ CUtensorMap tmLB,
                    const __grid_constant__ CUtensorMap tmC0, const __grid_constant__ CUtensorMap tmC1,
                    const Params p0, const Params p1) {
  // the epilogue's rows leave through a shared-memory staging buffer and one TMA
  // store per warp and round, so the promotion warps start the next tile while
  // the stores drain (direct 16-byte stores of 128 rows x 256 columns took
  // thousands of cycles per tile, during which no TMEM buffer was released)
  constexpr bool TMA_OUT = (EPI == EPI_STORE && CDT != FD_DT_F32) || EPI == EPI_QUANT;
  using CF = Cfg<EPI>;
  constexpr int STAGES = CF::STAGES;
  static_assert(!(LORA && GROUPED), "LoRA slices and grouped problems share the second tensor maps");
  const int total_tiles = p0.ntiles + (GROUPED ? p1.ntiles : 0);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // stage s: A tile at s * STAGE_BYTES, B tile (256 rows) right after it
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + CF::OFF_BAR);
  uint64_t* full = bars;                   // [STAGES]
  uint64_t* empty = bars + STAGES;         // [STAGES]
  uint64_t* tfull = bars + 2 * STAGES;     // [NTBUF]
  uint64_t* tempty = tfull + NTBUF;        // [NTBUF]
  uint64_t* drain = tempty + NTBUF;        // [1]
  uint64_t* hfull = drain + 1;             // deferred GELU: tile copy written
  uint64_t* hempty = hfull + 1;            // deferred GELU: tile copy read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(hempty + 1);
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
    mbar_init(hfull, EPI_WARPS * 32);
    mbar_init(hempty, 128);
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
    if constexpr (CF::DEFER) reg_dealloc<40>();
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      uint32_t issued_mask = 0;  // stages with a load issued
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const bool g1 = GROUPED && tile >= p0.ntiles;
        const Params& p = g1 ? p1 : p0;
        const CUtensorMap* mA = g1 ? &tmLA : &tmA;
        const CUtensorMap* mB = g1 ? &tmLB : &tmB;
        int mb, nb;
        tile_coords(p, g1 ? tile - p0.ntiles : tile, mb, nb);
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + s * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(sa, mA, &full[s], kb * BK, mb * BM);
          if (EPI == EPI_SILU_GATE) {
            // B rows [w1 block nb | w3 block nb]: the w3 rows start H rows further
            tma_load_2d(sb, mB, &full[s], kb * BK, nb * 128);
            tma_load_2d(sb + 128 * BK, mB, &full[s], kb * BK, p.N + nb * 128);
          } else if (B_MN) {
            // (K, N) storage: two 128-column panels of the 256-wide tile
            tma_load_2d(sb, mB, &full[s], nb * BN, kb * BK);
            tma_load_2d(sb + 128 * BK, mB, &full[s], nb * BN + 128, kb * BK);
          } else {
            tma_load_2d(sb, mB, &full[s], kb * BK, nb * BN);
          }
          issued_mask |= 1u << s;
        }
        for (int ls = 0; LORA && ls < p.lora_slices && ok; ++ls, ++it) {
          // bf16 LoRA slice: 128 x 64 of h and 256 x 64 of B_cat (128-byte rows, same layout)
          const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(sa, &tmLA, &full[s], ls * 64, mb * BM);
          tma_load_2d(sa + A_BYTES, &tmLB, &full[s], ls * 64, nb * BN);
          issued_mask |= 1u << s;
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
    if constexpr (CF::DEFER) reg_dealloc<40>();
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(/*c F32*/ 1, /*E4M3*/ 0, 0, /*a K-major*/ 0, B_MN, BM, BN);
      constexpr uint32_t idesc_lora = make_idesc(/*c F32*/ 1, /*BF16*/ 1, 1, 0, 0, BM, BN);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const Params& p = (GROUPED && tile >= p0.ntiles) ? p1 : p0;
        const int nslices = p.kblocks + (LORA ? p.lora_slices : 0);
        for (int kb = 0; kb < nslices; ++kb, ++it) {
          const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
          const uint32_t tb = it % NTBUF, tph = (it / NTBUF) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&tempty[tb], tph ^ 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t b0 = a0 + A_BYTES;
          const uint32_t d = tmem_base + tb * BN;
          if (!LORA || kb < p.kblocks) {
#pragma unroll
            for (int k4 = 0; k4 < BK / 32; ++k4) {
              const uint64_t ad = make_sdesc_sw128(a0 + k4 * 32, 16, 1024);
              // MN-major B: 128-column panels 128 x BK bytes apart (LBO), 8 K rows per 1 KiB
              const uint64_t bd = B_MN ? make_sdesc_sw128(b0 + k4 * 32 * 128, 128 * BK, 1024)
                                       : make_sdesc_sw128(b0 + k4 * 32, 16, 1024);
              mma_f8f6f4_ss(d, ad, bd, idesc, k4 > 0 ? 1u : 0u);
            }
          } else {
            // LoRA slice: 64 bf16 columns = 4 x K16, 32 bytes per step as for e4m3 K32
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              const uint64_t ad = make_sdesc_sw128(a0 + k4 * 32, 16, 1024);
              const uint64_t bd = make_sdesc_sw128(b0 + k4 * 32, 16, 1024);
              mma_f16_ss(d, ad, bd, idesc_lora, k4 > 0 ? 1u : 0u);
            }
          }
          tc_commit(&empty[s]);
          tc_commit(&tfull[tb]);
        }
      }
      tc_commit(drain);
      drain_wait(drain, 0);
    }
  } else if (CF::DEFER && warp >= CF::GELU_WARP0) {
    // ------------------------------------------------------------ deferred GELU + requant / QKV prologue
    // Thread t owns row t of the tile: per tile it reads the promotion warps' bf16
    // copy of its row (two 1 x 128 output groups) from shared memory and stores
    // the e4m3 codes of GELU(tanh) and the group scale.  The group absmax needs
    // no GELU per value: GELU(tanh) is increasing above x = -0.75 and |GELU| <=
    // 0.17004 below it, so whenever GELU(max x) > 0.171 it is the absmax (the
    // computed GELU of bf16 inputs keeps that order: neighbouring inputs differ by
    // 2^-8 relative, far above fp32 rounding); otherwise every value is
    // evaluated as before.  The codes then take one GELU per value.
    if constexpr (EPI == EPI_QKV) reg_alloc<136>();
    else reg_dealloc<104>();
    const int t = (warp - CF::GELU_WARP0) * 32 + lane;
    const uint8_t* hrow = smem + CF::OFF_STG + t * 512;
    uint32_t nt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++nt) {
      const bool g1 = GROUPED && tile >= p0.ntiles;
      const Params& p = g1 ? p1 : p0;
      int mb, nb;
      tile_coords(p, g1 ? tile - p0.ntiles : tile, mb, nb);
      ok = ok && mbar_wait(hfull, nt & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if constexpr (EPI == EPI_QKV) {
        // the four warps run the tile together (named barriers): all or none
        ok = named_bar_and(QKV_BAR, 128, ok);
        if (ok) {
          uint8_t* hbuf = smem + CF::OFF_STG;
          float* red = reinterpret_cast<float*>(smem + CF::OFF_QKV);
          if (p.qe.qk == FD_QK_INT8) qkv_epilogue_tile<FD_QK_INT8>(p, hbuf, red, mb, nb, warp - CF::GELU_WARP0, lane);
          else qkv_epilogue_tile<FD_QK_FP8>(p, hbuf, red, mb, nb, warp - CF::GELU_WARP0, lane);
        }
        mbar_arrive(hempty);
        continue;
      }
      const int m = mb * BM + t;
      const bool row_ok = m < p.M;
#pragma unroll 1
      for (int g = 0; g < 2; ++g) {
        const int n0 = nb * BN + g * 128;
        if (!ok || n0 >= p.N) continue;
        float xmax = -INFINITY;
#pragma unroll 4
        for (int j = 0; j < 16; ++j)
          xmax = fmaxf(xmax, max8_bf16(*reinterpret_cast<const uint4*>(hrow + (((g * 16 + j) ^ (t & 7)) << 4))));
        float amax = gelu_tanh(xmax);
        if (!(amax > 0.171f)) {
          amax = 0.f;
#pragma unroll 2
          for (int j = 0; j < 16; ++j)
            amax = fmaxf(amax, gelu8_absmax(*reinterpret_cast<const uint4*>(hrow + (((g * 16 + j) ^ (t & 7)) << 4))));
        }
        const float qm = quant_mult(amax);
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.c) + (int64_t)m * p.ldc + n0);
#pragma unroll 2
        for (int j = 0; j < 16; j += 2) {
          const uint2 lo = gelu8_codes(*reinterpret_cast<const uint4*>(hrow + (((g * 16 + j) ^ (t & 7)) << 4)), qm);
          const uint2 hi = gelu8_codes(*reinterpret_cast<const uint4*>(hrow + (((g * 16 + j + 1) ^ (t & 7)) << 4)), qm);
          if (row_ok) dst[j >> 1] = make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
        if (row_ok) p.c_s[(int64_t)m * p.ldcs + n0 / 128] = dequant_scale(amax);
      }
      mbar_arrive(hempty);
    }
  } else if (CF::DEFER && warp < CF::PROMO_WARP0) {
    // warps 2-3 of the deferred-GELU kernel have no role
    reg_dealloc<40>();
  } else {
    // ------------------------------------------------------------ promotion + epilogue
    // Thread (q, h): row q * 32 + lane; TMEM columns [128 h, 128 h + 128) of the
    // 256-column accumulator (EPI_SILU_GATE: w1 columns [64 h, 64 h + 64) and the
    // matching w3 columns 128 + [64 h, 64 h + 64)).
    if constexpr (CF::DEFER) reg_alloc<168>();
    const int q = warp & 3;             // TMEM lane quadrant this warp may access
    const int h = (warp - CF::PROMO_WARP0) >> 2;  // column half
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int r = q * 32 + lane;        // row within the tile
    float* red = reinterpret_cast<float*>(smem + CF::OFF_RED);  // [parity][half][128]
    uint32_t it = 0, nt = 0;
    bool ok = true;
    // A thread whose wait timed out keeps walking the tiles (skipping the work)
    // so its partner is never left at the max-exchange barrier.
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++nt) {
      const bool g1 = GROUPED && tile >= p0.ntiles;
      const Params& p = g1 ? p1 : p0;
      int mb, nb;
      tile_coords(p, g1 ? tile - p0.ntiles : tile, mb, nb);
      const int m = mb * BM + r;
      const bool row_ok = m < p.M;
      const float* as_row = p.a_s + (int64_t)(row_ok ? m : 0) * p.kblocks;
      // GEMM columns (rows of B) of acc[0..63] and acc[64..127]
      const int n_lo = EPI == EPI_SILU_GATE ? nb * 128 + h * 64 : nb * BN + h * 128;
      const int n_hi = EPI == EPI_SILU_GATE ? p.N + nb * 128 + h * 64 : n_lo + 64;
      const uint32_t col_lo = EPI == EPI_SILU_GATE ? h * 64 : h * 128;
      const uint32_t col_hi = col_lo + (EPI == EPI_SILU_GATE ? 128 : 64);
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.f;
      const int nslices = p.kblocks + (LORA ? p.lora_slices : 0);
      // The slice scales come from global memory; they are loaded two slices
      // ahead so that no load latency sits between "slice ready" and the
      // release of its TMEM buffer (the MMA issuer waits on that release).
      // LoRA slices (the bf16 operands carry their scales) and rows past M use
      // a_s = 1 / 0 as before; columns past the end of B read the last block's
      // scale (they are never stored).
      const int blo = min(n_lo / 128, p.nbs - 1), bhi = min(n_hi / 128, p.nbs - 1);
      auto load_scales = [&](int kb, float& as, float& bl, float& bh) {
        as = 1.0f;
        bl = 1.0f;
        bh = 1.0f;
        if (kb >= p.kblocks) return;
        if (BMODE == 1) {
          bl = __ldg(p.b_s + (int64_t)kb * p.nbs + blo);
          bh = __ldg(p.b_s + (int64_t)kb * p.nbs + bhi);
        } else if (BMODE == 0) {
          bl = __ldg(p.b_s + (int64_t)blo * p.kblocks + kb);
          bh = __ldg(p.b_s + (int64_t)bhi * p.kblocks + kb);
        }
        as = row_ok ? __ldg(as_row + kb) : 0.f;
      };
      float as0, bl0, bh0, as1, bl1, bh1;
      load_scales(0, as0, bl0, bh0);
      load_scales(1, as1, bl1, bh1);
      for (int kb = 0; kb < nslices; ++kb, ++it) {
        const uint32_t tb = it % NTBUF, tph = (it / NTBUF) & 1;
        float as2, bl2, bh2;
        load_scales(kb + 2, as2, bl2, bh2);
        // acc += partial * (a_s * b_s): the reference's (dot * a_s) * b_s rounded
        // as one product of the two scales, as before
        const float sc_lo = as0 * bl0, sc_hi = as0 * bh0;
        as0 = as1; bl0 = bl1; bh0 = bh1;
        as1 = as2; bl1 = bl2; bh1 = bh2;
        ok = ok && mbar_wait(&tfull[tb], tph, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) continue;
        tc_fence_after();
        const uint32_t taddr = tmem_base + lane_base + tb * BN;
        // chunk c + 1 is loaded before chunk c is accumulated; the buffer is
        // released as soon as the last chunk is in registers
        uint32_t r0[16], r1[16];
        tmem_ld16(taddr + col_lo, r0);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t(&cur)[16] = (c & 1) ? r1 : r0;
          uint32_t(&nxt)[16] = (c & 1) ? r0 : r1;
          tmem_wait_ld();
          if (c < 7) {
            tmem_ld16(taddr + (c + 1 < 4 ? col_lo : col_hi) + ((c + 1) & 3) * 16, nxt);
          } else {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[tb]);
          }
          const float sc = c < 4 ? sc_lo : sc_hi;
          const uint64_t sc2 = pk(sc, sc);
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            uint64_t a2 = pk(acc[16 * c + i], acc[16 * c + i + 1]);
            a2 = fma2(pk(__uint_as_float(cur[i]), __uint_as_float(cur[i + 1])), sc2, a2);
            unpk(a2, acc[16 * c + i], acc[16 * c + i + 1]);
          }
        }
      }
      if (BMODE == 2) {
        // fp8_gemm_rowwise_kernel: accumulator *= b_s[n] after the K loop (:407-408)
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          const int n = n_lo + i;
          acc[i] *= (n < p.N) ? __ldg(p.b_s + n) : 0.f;
        }
      }
      if (BDT >= 0 && p.bias) {
        // eight columns per 16-byte load (32 bytes for f32); the scalar path covers
        // a bias that is not 16-byte aligned and the columns of a partial last tile
        constexpr int BT = BDT < 0 ? FD_DT_F32 : BDT;
        const bool vec = (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0;
#pragma unroll
        for (int c8 = 0; c8 < 16; ++c8) {
          const int n = (c8 < 8 ? n_lo : n_hi) + (c8 & 7) * 8;
          float b[8];
          if (vec && (EPI == EPI_SILU_GATE || n + 8 <= p.N)) {
            load_bias8<BT>(p.bias, n, b);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) b[j] = (EPI == EPI_SILU_GATE || n + j < p.N) ? load_bias<BT>(p.bias, n + j) : 0.f;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[8 * c8 + j] += b[j];
        }
      }
      // staging buffer, first output row and output map of this warp
      uint8_t* stg = smem + CF::OFF_STG + (warp - CF::PROMO_WARP0) * STG_WARP;
      const int row0 = mb * BM + q * 32;
      const CUtensorMap* mC = g1 ? &tmC1 : &tmC0;
      if constexpr (CF::DEFER) {
        // the bf16-rounded tile (the GELU input) to the GELU warps: row r, this
        // thread's 128 columns as 16-byte chunks h * 16 + j, chunk index XOR
        // (r & 7) so that the 32 rows of a warp spread over the banks
        const bool free = mbar_wait(hempty, (nt & 1) ^ 1, abort_flag);  // previous copy read
        uint8_t* hrow = smem + CF::OFF_STG + r * 512;
        if (ok && free) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int i = 8 * j;
            *reinterpret_cast<uint4*>(hrow + (((h * 16 + j) ^ (r & 7)) << 4)) =
                make_uint4(pack_bf16x2(acc[i], acc[i + 1]), pack_bf16x2(acc[i + 2], acc[i + 3]),
                           pack_bf16x2(acc[i + 4], acc[i + 5]), pack_bf16x2(acc[i + 6], acc[i + 7]));
          }
        }
        mbar_arrive(hfull);
      } else if constexpr (EPI == EPI_STORE && TMA_OUT) {
        // two rounds of 64 columns: bf16 / f16 rows of 128 B in the 128-byte
        // swizzle the output tensor map expects (granule g of row j at g ^ (j & 7))
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if (lane == 0) bulk_wait_read_all();  // the previous store has read the buffer
          __syncwarp();
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const int i = 64 * j + 8 * g;
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((g ^ (lane & 7)) << 4)) =
                make_uint4(pack2<CDT>(acc[i], acc[i + 1]), pack2<CDT>(acc[i + 2], acc[i + 3]),
                           pack2<CDT>(acc[i + 4], acc[i + 5]), pack2<CDT>(acc[i + 6], acc[i + 7]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          // rows past M and columns past N are clipped by the tensor map
          if (lane == 0 && ok && row0 < p.M && n_lo + 64 * j < p.N) {
            tma_store_2d(stg, mC, n_lo + 64 * j, row0);
            bulk_commit_group();
          }
        }
      } else if constexpr (EPI == EPI_STORE) {
        if (ok && row_ok) {
          store_row64<CDT>(p.c, (int64_t)m * p.ldc, n_lo, p.N, *reinterpret_cast<float(*)[64]>(acc));
          store_row64<CDT>(p.c, (int64_t)m * p.ldc, n_lo + 64, p.N, *reinterpret_cast<float(*)[64]>(acc + 64));
        }
      } else if constexpr (EPI == EPI_SILU_GATE) {
        // the reference rounds the w1w3 GEMM output to bf16 before the gate
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = silu_gate(round_to_bf16(acc[i]), round_to_bf16(acc[64 + i]));
        // 1 x 128 group = this thread's 64 gate columns and its partner's
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(acc[i]));
        float* rd = red + (nt & 1) * 256;
        rd[h * 128 + r] = amax;
        named_bar_sync(1 + q, 64);
        amax = fmaxf(amax, rd[(h ^ 1) * 128 + r]);
        if (ok && row_ok) {
          const float qm = quant_mult(amax);
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.c) + (int64_t)m * p.ldc + nb * 128 + h * 64);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            dst[k] = make_uint4(quant4(acc[16 * k], acc[16 * k + 1], acc[16 * k + 2], acc[16 * k + 3], qm),
                                quant4(acc[16 * k + 4], acc[16 * k + 5], acc[16 * k + 6], acc[16 * k + 7], qm),
                                quant4(acc[16 * k + 8], acc[16 * k + 9], acc[16 * k + 10], acc[16 * k + 11], qm),
                                quant4(acc[16 * k + 12], acc[16 * k + 13], acc[16 * k + 14], acc[16 * k + 15], qm));
          if (h == 0) p.c_s[(int64_t)m * p.ldcs + nb] = dequant_scale(amax);
        }
      } else {
        // EPI_QUANT: this thread's 128 columns are one whole output group, 128 codes per row (128 B, 128-byte swizzle) through the staging buffer
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(acc[i]));
        const float qm = quant_mult(amax);
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<uint4*>(stg + lane * 128 + ((k ^ (lane & 7)) << 4)) =
              make_uint4(quant4(acc[16 * k], acc[16 * k + 1], acc[16 * k + 2], acc[16 * k + 3], qm),
                         quant4(acc[16 * k + 4], acc[16 * k + 5], acc[16 * k + 6], acc[16 * k + 7], qm),
                         quant4(acc[16 * k + 8], acc[16 * k + 9], acc[16 * k + 10], acc[16 * k + 11], qm),
                         quant4(acc[16 * k + 12], acc[16 * k + 13], acc[16 * k + 14], acc[16 * k + 15], qm));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && ok && row0 < p.M && n_lo < p.N) {
          tma_store_2d(stg, mC, n_lo, row0);
          bulk_commit_group();
        }
        if (ok && row_ok && n_lo < p.N) p.c_s[(int64_t)m * p.ldcs + n_lo / 128] = dequant_scale(amax);
      }
    }
    if (TMA_OUT && lane == 0) bulk_wait_all();  // every output store has completed
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 512);
}

template <int BMODE, int CDT, int BDT, int EPI = EPI_STORE, bool LORA = false, bool GROUPED = false>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Params& p,
                  cudaStream_t st, const CUtensorMap* tla = nullptr, const CUtensorMap* tlb = nullptr,
                  const Params* p1 = nullptr, const CUtensorMap* tc1 = nullptr) {
  auto kern = gemm_fp8_kernel<BMODE, CDT, BDT, EPI, LORA, GROUPED>;
  constexpr uint32_t smem_bytes = Cfg<EPI>::SMEM_BYTES;
  static bool attr_done = false;  // per instantiation
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "gemm smem attribute: %s", cudaGetErrorString(e));
    attr_done = true;
  }
  const int total = p.ntiles + (GROUPED ? p1->ntiles : 0);
  const int grid = total < num_sms() ? total : num_sms();
  kern<<<grid, Cfg<EPI>::THREADS, smem_bytes, st>>>(ta, tb, tla ? *tla : ta, tlb ? *tlb : tb, tc, tc1 ? *tc1 : tc, p,
                                              p1 ? *p1 : p);
  return check_launch("fp8_gemm_blockwise");
}

template <int EPI>
static int launch_quant(int bdt, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                        const Params& p, cudaStream_t st) {
  if (!p.bias) return launch<0, -1, -1, EPI>(ta, tb, tc, p, st);
  switch (bdt) {
    case FD_DT_BF16: return launch<0, -1, FD_DT_BF16, EPI>(ta, tb, tc, p, st);
    case FD_DT_F16: return launch<0, -1, FD_DT_F16, EPI>(ta, tb, tc, p, st);
    case FD_DT_F32: return launch<0, -1, FD_DT_F32, EPI>(ta, tb, tc, p, st);
    default: return set_error(FD_ERR_ARG, "unsupported bias dtype");
  }
}

template <int BMODE, int CDT, bool LORA = false>
static int launch_bias(int bdt, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Params& p,
                       cudaStream_t st, const CUtensorMap* tla = nullptr, const CUtensorMap* tlb = nullptr) {
  if (!p.bias) return launch<BMODE, CDT, -1, EPI_STORE, LORA>(ta, tb, tc, p, st, tla, tlb);
  switch (bdt) {
    case FD_DT_BF16: return launch<BMODE, CDT, FD_DT_BF16, EPI_STORE, LORA>(ta, tb, tc, p, st, tla, tlb);
    case FD_DT_F16: return launch<BMODE, CDT, FD_DT_F16, EPI_STORE, LORA>(ta, tb, tc, p, st, tla, tlb);
    case FD_DT_F32: return launch<BMODE, CDT, FD_DT_F32, EPI_STORE, LORA>(ta, tb, tc, p, st, tla, tlb);
    default: return set_error(FD_ERR_ARG, "unsupported bias dtype");
  }
}

template <int BMODE, bool LORA = false>
static int launch_c(int cdt, int bdt, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                    const Params& p, cudaStream_t st, const CUtensorMap* tla = nullptr,
                    const CUtensorMap* tlb = nullptr) {
  switch (cdt) {
    case FD_DT_BF16: return launch_bias<BMODE, FD_DT_BF16, LORA>(bdt, ta, tb, tc, p, st, tla, tlb);
    case FD_DT_F16: return launch_bias<BMODE, FD_DT_F16, LORA>(bdt, ta, tb, tc, p, st, tla, tlb);
    case FD_DT_F32: return launch_bias<BMODE, FD_DT_F32, LORA>(bdt, ta, tb, tc, p, st, tla, tlb);
    default: return set_error(FD_ERR_ARG, "unsupported output dtype");
  }
}

// Output tensor map of the TMA-store epilogues: rows of ldc elements, 32-row
// boxes of 128 bytes (64 bf16 / f16 or 128 e4m3 codes), 128-byte swizzle.
// kind: FD_DT_BF16 / FD_DT_F16 / FD_DT_E4M3; f32 outputs are stored directly
// and get a placeholder map (never read).
static int encode_out(CUtensorMap* m, void* c, int kind, int64_t M, int64_t N, int64_t ldc, const CUtensorMap& dummy) {
  if (kind == FD_DT_F32 || kind < 0) {
    *m = dummy;
    return FD_OK;
  }
  const bool codes = kind == FD_DT_E4M3;
  const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
  const uint64_t strides[1] = {(uint64_t)ldc * (codes ? 1 : 2)};
  const uint32_t box[2] = {codes ? 128u : 64u, 32u};
  return encode_tiled(m,
                      codes ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                            : (kind == FD_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16),
                      2, c, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace gemm

int gemm_status(unsigned int* out, int clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_status, sizeof(*out));
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "fd_get_status (gemm): %s", cudaGetErrorString(e));
  if (clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_status, &z, sizeof(z));
    if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "fd_get_status (gemm): %s", cudaGetErrorString(e));
  }
  return FD_OK;
}

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
    const uint32_t box[2] = {128, 256};
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
  p.lora_slices = 0;
  p.ldc = N;
  p.ldcs = N / 128;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ntm = (int)((M + 127) / 128);
  p.ntn = (int)((N + 255) / 256);
  p.nbs = (int)((N + 127) / 128);
  p.ntiles = p.ntm * p.ntn;
  p.kblocks = (int)(K / 128);
  cudaStream_t st = (cudaStream_t)stream;
  CUtensorMap tc;
  const int rc = gemm::encode_out(&tc, c, c_dtype, M, N, N, ta);
  if (rc) return rc;
  if (b_layout == 0) return gemm::launch_c<0>(c_dtype, bias_dtype, ta, tb, tc, p, st);
  if (b_layout == 1) return gemm::launch_c<1>(c_dtype, bias_dtype, ta, tb, tc, p, st);
  return gemm::launch_c<2>(c_dtype, bias_dtype, ta, tb, tc, p, st);
}

// GEMM with a quantising epilogue (see the header of this file): act 0 requantises
// the fp32 accumulator (fp8_gemm_quant), 1 applies GELU(tanh) to the bf16 GEMM
// output first, 2 is the SiLU gate with b = [w1; w3] of shape (2 N, K).
static int gemm_quant_impl(const void* a, const float* a_s, const void* b, const float* b_s, const void* bias,
                           int bias_dtype, void* c, float* c_s, int64_t M, int64_t N, int64_t K, int act,
                           int64_t ldc, int64_t ldcs, void* stream) {
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
    // SiLU gate: two 128-row boxes (w1 block, w3 block) per B tile
    const uint32_t box[2] = {128, act == FD_ACT_SILU_GATE ? 128u : 256u};
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
  p.ntn = act == FD_ACT_SILU_GATE ? (int)(N / 128) : (int)((N + 255) / 256);
  p.nbs = (int)(nb_rows / 128);
  p.lora_slices = 0;
  p.ldc = ldc;
  p.ldcs = ldcs;
  p.ntiles = p.ntm * p.ntn;
  p.kblocks = (int)(K / 128);
  cudaStream_t st = (cudaStream_t)stream;
  CUtensorMap tc;
  const int rc = gemm::encode_out(&tc, c, act == FD_ACT_SILU_GATE ? -1 : FD_DT_E4M3, M, N, ldc, ta);
  if (rc) return rc;
  if (act == FD_ACT_NONE) return gemm::launch_quant<gemm::EPI_QUANT>(bias_dtype, ta, tb, tc, p, st);
  if (act == FD_ACT_GELU_TANH) return gemm::launch_quant<gemm::EPI_GELU_TANH>(bias_dtype, ta, tb, tc, p, st);
  return gemm::launch_quant<gemm::EPI_SILU_GATE>(bias_dtype, ta, tb, tc, p, st);
}

extern "C" int fd_fp8_gemm_quant(const void* a, const float* a_s, const void* b, const float* b_s,
                                 const void* bias, int bias_dtype, void* c, float* c_s, int64_t M,
                                 int64_t N, int64_t K, int act, void* stream) {
  return gemm_quant_impl(a, a_s, b, b_s, bias, bias_dtype, c, c_s, M, N, K, act, N, N / 128, stream);
}

// fd_fp8_gemm_quant writing into a column window of wider code / scale rows:
// row m of the output starts at c + m * ldc (codes) and c_s + m * ldcs (scales),
// e.g. the second half of the [attention | MLP] input of a fused output linear.
extern "C" int fd_fp8_gemm_quant_ld(const void* a, const float* a_s, const void* b, const float* b_s,
                                    const void* bias, int bias_dtype, void* c, float* c_s, int64_t M,
                                    int64_t N, int64_t K, int act, int64_t ldc, int64_t ldcs, void* stream) {
  FD_CHECK_ARG(ldc >= N && ldc % 16 == 0 && ldcs >= N / 128, "ldc must be >= N and a multiple of 16, ldcs >= N / 128");
  FD_CHECK_ARG(aligned16(c), "c must be 16-byte aligned");
  return gemm_quant_impl(a, a_s, b, b_s, bias, bias_dtype, c, c_s, M, N, K, act, ldc, ldcs, stream);
}

// FP8 block GEMM (b_layout 0) plus the multi-LoRA delta lora_a @ lora_b^T in the same
// accumulator: lora_a (M, lora_k) bf16 = per-token scaled mid activations, lora_b
// (N, lora_k) bf16 = the adapters' B matrices side by side; lora_k a positive
// multiple of 64 (zero-padded).  K may be 0 (delta only: a, a_s, b, b_s unused).
extern "C" int fd_fp8_gemm_blockwise_lora(const void* a, const float* a_s, const void* b,
                                          const float* b_s, const void* bias, int bias_dtype, void* c,
                                          int c_dtype, int64_t M, int64_t N, int64_t K,
                                          const void* lora_a, const void* lora_b, int64_t lora_k,
                                          void* stream) {
  FD_CHECK_ARG(M >= 0 && N > 0 && K >= 0, "bad shape");
  FD_CHECK_ARG(K % 128 == 0, "K must be a multiple of 128");
  FD_CHECK_ARG(N % 16 == 0, "N must be a multiple of 16");
  FD_CHECK_ARG(lora_k > 0 && lora_k % 64 == 0 && lora_k <= 65536, "lora_k must be a positive multiple of 64");
  FD_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "dimension too large");
  if (M == 0) return FD_OK;
  FD_CHECK_ARG(lora_a && lora_b && c, "null pointer");
  FD_CHECK_ARG(K == 0 || (a && a_s && b && b_s), "null FP8 operand");
  FD_CHECK_ARG(aligned16(lora_a) && aligned16(lora_b) && aligned16(c) && (K == 0 || (aligned16(a) && aligned16(b))),
               "operands must be 16-byte aligned");
  CUtensorMap ta, tb, tla, tlb;
  {
    const uint64_t dims[2] = {(uint64_t)lora_k, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)lora_k * 2};
    const uint32_t box[2] = {64, 128};
    int rc = encode_tiled(&tla, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, lora_a, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)lora_k, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)lora_k * 2};
    const uint32_t box[2] = {64, 256};
    int rc = encode_tiled(&tlb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, lora_b, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if (K > 0) {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {128, 128};
    int rc = encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t bdims[2] = {(uint64_t)K, (uint64_t)N};
    const uint32_t bbox[2] = {128, 256};
    rc = encode_tiled(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, b, bdims, strides, bbox,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    ta = tla;  // never read: no FP8 slices
    tb = tlb;
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
  p.ntn = (int)((N + 255) / 256);
  p.nbs = (int)((N + 127) / 128);
  p.ntiles = p.ntm * p.ntn;
  p.kblocks = (int)(K / 128);
  p.lora_slices = (int)(lora_k / 64);
  p.ldc = N;
  p.ldcs = N / 128;
  CUtensorMap tc;
  const int rc = gemm::encode_out(&tc, c, c_dtype, M, N, N, tla);
  if (rc) return rc;
  return gemm::launch_c<0, true>(c_dtype, bias_dtype, ta, tb, tc, p, (cudaStream_t)stream, &tla, &tlb);
}

// ---------------------------------------------------------------------------
// Two problems in one persistent launch (e.g. the text and image streams of a
// double-stream block, same epilogue): act FD_GEMM_STORE_BF16 stores bf16
// (+ bias), FD_ACT_* quantise as fd_fp8_gemm_quant.  B stored (N, K); bias
// FD_DT_BF16 or none.
static int grouped_problem(const fd_gemm_problem& q, int act, CUtensorMap& ta, CUtensorMap& tb, CUtensorMap& tc,
                           gemm::Params& p) {
  const bool quant = act != FD_GEMM_STORE_BF16;
  FD_CHECK_ARG(q.M > 0 && q.N > 0 && q.K > 0 && q.K % 128 == 0, "bad shape");
  FD_CHECK_ARG(quant ? q.N % 128 == 0 : q.N % 16 == 0, "bad N");
  const int64_t nb_rows = act == FD_ACT_SILU_GATE ? 2 * q.N : q.N;
  FD_CHECK_ARG(q.M < (1ll << 31) && nb_rows < (1ll << 31) && q.K < (1ll << 31), "dimension too large");
  FD_CHECK_ARG(q.a && q.a_s && q.b && q.b_s && q.c && (!quant || q.c_s), "null pointer");
  FD_CHECK_ARG(aligned16(q.a) && aligned16(q.b) && aligned16(q.c), "a, b, c must be 16-byte aligned");
  {
    const uint64_t dims[2] = {(uint64_t)q.K, (uint64_t)q.M};
    const uint64_t strides[1] = {(uint64_t)q.K};
    const uint32_t box[2] = {128, 128};
    int rc = encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q.a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)q.K, (uint64_t)nb_rows};
    const uint64_t strides[1] = {(uint64_t)q.K};
    const uint32_t box[2] = {128, act == FD_ACT_SILU_GATE ? 128u : 256u};
    int rc = encode_tiled(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q.b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  p.a_s = q.a_s;
  p.b_s = q.b_s;
  p.bias = q.bias;
  p.c = q.c;
  p.c_s = q.c_s;
  p.M = (int)q.M;
  p.N = (int)q.N;
  p.K = (int)q.K;
  p.ntm = (int)((q.M + 127) / 128);
  p.ntn = act == FD_ACT_SILU_GATE ? (int)(q.N / 128) : (int)((q.N + 255) / 256);
  p.nbs = (int)((nb_rows + 127) / 128);
  p.ntiles = p.ntm * p.ntn;
  p.kblocks = (int)(q.K / 128);
  p.lora_slices = 0;
  p.ldc = q.N;
  p.ldcs = q.N / 128;
  return gemm::encode_out(&tc, q.c, act == FD_GEMM_STORE_BF16 ? FD_DT_BF16 : (act == FD_ACT_SILU_GATE ? -1 : FD_DT_E4M3),
                          q.M, q.N, q.N, ta);
}

extern "C" int fd_fp8_gemm_grouped2(const fd_gemm_problem* q0, const fd_gemm_problem* q1, int bias_dtype, int act,
                                    void* stream) {
  FD_CHECK_ARG(q0 && q1, "null problem");
  FD_CHECK_ARG(act == FD_GEMM_STORE_BF16 || (act >= FD_ACT_NONE && act <= FD_ACT_SILU_GATE), "bad act");
  FD_CHECK_ARG((q0->bias == nullptr) == (q1->bias == nullptr), "both problems or neither take a bias");
  FD_CHECK_ARG(q0->bias == nullptr || bias_dtype == FD_DT_BF16, "grouped GEMM bias must be bf16");
  CUtensorMap ta0, tb0, tc0, ta1, tb1, tc1;
  gemm::Params p0, p1;
  int rc = grouped_problem(*q0, act, ta0, tb0, tc0, p0);
  if (rc) return rc;
  rc = grouped_problem(*q1, act, ta1, tb1, tc1, p1);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool bias = q0->bias != nullptr;
  using namespace gemm;
#define FD_G2(CD, BD, E) return launch<0, CD, BD, E, false, true>(ta0, tb0, tc0, p0, st, &ta1, &tb1, &p1, &tc1)
  if (act == FD_GEMM_STORE_BF16) {
    if (bias) FD_G2(FD_DT_BF16, FD_DT_BF16, EPI_STORE);
    FD_G2(FD_DT_BF16, -1, EPI_STORE);
  }
  if (act == FD_ACT_NONE) {
    if (bias) FD_G2(-1, FD_DT_BF16, EPI_QUANT);
    FD_G2(-1, -1, EPI_QUANT);
  }
  if (act == FD_ACT_GELU_TANH) {
    if (bias) FD_G2(-1, FD_DT_BF16, EPI_GELU_TANH);
    FD_G2(-1, -1, EPI_GELU_TANH);
  }
  if (bias) FD_G2(-1, FD_DT_BF16, EPI_SILU_GATE);
  FD_G2(-1, -1, EPI_SILU_GATE);
#undef FD_G2
}

int64_t fd_desc_stride(int64_t N, int gran, int rows_per_block);  // attn_prologue.cu

// ---------------------------------------------------------------------------
// The QKV linear(s) of a joint attention with P3 and the attention prologue's
// first pass in the GEMM epilogue (EPI_QKV); equals fd_fp8_gemm_blockwise (bf16)
// followed by fd_qkv_postprocess_quant per stream.
static int qkv_problem(const fd_gemm_problem& q, const fd_qkv_stream& st, int64_t B, int64_t H, int64_t N,
                       int qk_kind, int q_gran, int pv_kind, float sm_scale_log2e, void* q_codes, float* q_desc,
                       void* k_out, void* v_out, float* workspace, CUtensorMap& ta, CUtensorMap& tb,
                       gemm::Params& p) {
  FD_CHECK_ARG(q.M == B * st.S && q.N == 3 * H * 128 && q.K > 0 && q.K % 128 == 0, "bad shape");
  FD_CHECK_ARG(st.S > 0 && st.S % 128 == 0 && st.s_off >= 0 && st.s_off % 128 == 0 && st.s_off + st.S <= N,
               "S and s_off must be multiples of 128 inside N");
  FD_CHECK_ARG(q.M < (1ll << 31) && q.K < (1ll << 31), "dimension too large");
  FD_CHECK_ARG(q.a && q.a_s && q.b && q.b_s && st.q_norm && st.k_norm && st.freqs, "null pointer");
  FD_CHECK_ARG(aligned16(q.a) && aligned16(q.b) && aligned16(st.q_norm) && aligned16(st.k_norm) &&
                   aligned16(st.freqs),
               "misaligned pointer");
  {
    const uint64_t dims[2] = {(uint64_t)q.K, (uint64_t)q.M};
    const uint64_t strides[1] = {(uint64_t)q.K};
    const uint32_t box[2] = {128, 128};
    int rc = encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q.a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)q.K, (uint64_t)q.N};
    const uint64_t strides[1] = {(uint64_t)q.K};
    const uint32_t box[2] = {128, 256};
    int rc = encode_tiled(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q.b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  const int nchunks = (int)(N / 128);
  p.a_s = q.a_s;
  p.b_s = q.b_s;
  p.bias = q.bias;
  p.c = nullptr;
  p.c_s = nullptr;
  p.M = (int)q.M;
  p.N = (int)q.N;
  p.K = (int)q.K;
  p.ntm = (int)(q.M / 128);
  p.ntn = (int)(q.N / 256);
  p.nbs = (int)(q.N / 128);
  p.ntiles = p.ntm * p.ntn;
  p.kblocks = (int)(q.K / 128);
  p.lora_slices = 0;
  p.ldc = q.N;
  p.ldcs = 0;
  gemm::QkvEpi& e = p.qe;
  e.qw = st.q_norm;
  e.kw = st.k_norm;
  e.freqs = st.freqs;
  e.q_codes = (uint8_t*)q_codes;
  e.q_desc = q_desc;
  e.k_out = (__nv_bfloat16*)k_out;
  e.v_out = (__nv_bfloat16*)v_out;
  e.ws_sum = workspace;
  e.ws_amax = workspace + B * H * nchunks * 128;
  e.q_desc_stride = fd_desc_stride(N, q_gran, 128);
  e.eps = st.eps;
  e.sm_scale_log2e = sm_scale_log2e;
  e.S = (int)st.S;
  e.H = (int)H;
  e.Nj = (int)N;
  e.s_off = (int)st.s_off;
  e.q_gran = q_gran;
  e.qk = qk_kind;
  e.nchunks = nchunks;
  e.do_v = pv_kind == FD_PV_FP8;
  return FD_OK;
}

extern "C" int fd_fp8_gemm_qkv_quant(const fd_gemm_problem* p0, const fd_qkv_stream* s0, const fd_gemm_problem* p1,
                                     const fd_qkv_stream* s1, int bias_dtype, int64_t B, int64_t H, int64_t N,
                                     int qk_kind, int q_gran, int pv_kind, float sm_scale_log2e, void* q_codes,
                                     float* q_desc, void* k_out, void* v_out, float* workspace, void* stream) {
  FD_CHECK_ARG(p0 && s0 && (p1 == nullptr) == (s1 == nullptr), "a problem needs its stream description");
  FD_CHECK_ARG(B > 0 && H > 0 && H % 2 == 0 && B * H <= 65535, "H must be even (two heads per 256-column tile)");
  FD_CHECK_ARG(N > 0 && N % 128 == 0 && N < (1ll << 30), "N must be a positive multiple of 128");
  FD_CHECK_ARG(qk_kind == FD_QK_INT8 || qk_kind == FD_QK_FP8, "bad qk_kind");
  FD_CHECK_ARG(q_gran == FD_GRAN_TOKEN || q_gran == FD_GRAN_BLOCK, "bad q_gran");
  FD_CHECK_ARG(pv_kind == FD_PV_BF16 || pv_kind == FD_PV_FP8, "bad pv_kind");
  FD_CHECK_ARG(q_codes && q_desc && k_out && v_out && workspace, "null pointer");
  FD_CHECK_ARG(aligned8(k_out) && aligned8(v_out) && (reinterpret_cast<uintptr_t>(q_codes) & 3) == 0,
               "misaligned pointer");
  FD_CHECK_ARG((p0->bias == nullptr || bias_dtype == FD_DT_BF16) && (p1 == nullptr || (p1->bias == nullptr) == (p0->bias == nullptr)),
               "bias must be bf16, on both problems or neither");
  CUtensorMap ta0, tb0, ta1, tb1;
  gemm::Params q0p, q1p;
  int rc = qkv_problem(*p0, *s0, B, H, N, qk_kind, q_gran, pv_kind, sm_scale_log2e, q_codes, q_desc, k_out, v_out,
                       workspace, ta0, tb0, q0p);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  using namespace gemm;
  const bool bias = p0->bias != nullptr;
  if (p1) {
    rc = qkv_problem(*p1, *s1, B, H, N, qk_kind, q_gran, pv_kind, sm_scale_log2e, q_codes, q_desc, k_out, v_out,
                     workspace, ta1, tb1, q1p);
    if (rc) return rc;
    if (bias) return launch<0, -1, FD_DT_BF16, EPI_QKV, false, true>(ta0, tb0, ta0, q0p, st, &ta1, &tb1, &q1p, &ta1);
    return launch<0, -1, -1, EPI_QKV, false, true>(ta0, tb0, ta0, q0p, st, &ta1, &tb1, &q1p, &ta1);
  }
  if (bias) return launch<0, -1, FD_DT_BF16, EPI_QKV>(ta0, tb0, ta0, q0p, st);
  return launch<0, -1, -1, EPI_QKV>(ta0, tb0, ta0, q0p, st);
}
