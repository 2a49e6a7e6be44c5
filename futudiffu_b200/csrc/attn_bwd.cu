// Attention backward (A7): Delta pre-pass and dQ / dK / dV with the same
// quantised P recomputation as the forward.
// Reference: _sage_attn_d_prepass src/futudiffu/sage_kernels.py:322-349;
// _sage_attn_bwd_dkdv_int8(_masked) :805-911, :1491-1605;
// _sage_attn_bwd_dq_int8(_masked) :918-1015, :1617-1722; fp8 :356-567.
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


// ---------------------------------------------------------------------------
// dK / dV and dQ.  CUDA-core fp32 kernels over 64 x 64 tiles (the backward is
// the QAT training path, outside the timed forward configs).  Per tile pair:
//   S  = (Qc . Kc) * q_desc * k_desc            (codes exact, as the forward)
//   P  = exp2(S - lse);  dP = dO . V^T;  dS = P * (dP - delta)
//   dV += bf16(P)^T dO;  dK += bf16(dS * sm_scale)^T Q;  dQ += bf16(dS) K
// with bf16-rounded operands where the reference casts (:896-907, :1007-1010).
constexpr int TB = 64;     // tile rows / cols
constexpr int LD = 129;    // padded row stride (floats) to avoid bank conflicts
constexpr int LDT = 65;
constexpr uint32_t BWD_SMEM = (5 * TB * LD + 2 * TB * LDT + 6 * TB) * 4;

template <int QK>
FD_DEV float code_val(const uint8_t* codes, int64_t i) {
  if constexpr (QK == FD_QK_INT8) return (float)(int8_t)codes[i];
  else {
    __nv_fp8_e4m3 c;
    c.__x = codes[i];
    return float(c);
  }
}

FD_DEV bool pair_valid(const uint8_t* mask, int64_t mstride, int nkb, int bh, int q0, int kblk) {
  if (!mask) return true;
  return mask[(int64_t)bh * mstride + (int64_t)(q0 / 128) * nkb + kblk] != 0;
}

// load a 64 x 128 tile of codes (row r0..r0+63) into smem as float, rows >= N as 0
template <int QK>
FD_DEV void load_codes(float* dst, const uint8_t* src, int64_t base_row, int r0, int N) {
  for (int e = threadIdx.x; e < TB * 128; e += blockDim.x) {
    const int r = e >> 7, d = e & 127;
    dst[r * LD + d] = (r0 + r < N) ? code_val<QK>(src, (base_row + r0 + r) * 128 + d) : 0.f;
  }
}

FD_DEV void load_bf16(float* dst, const __nv_bfloat16* src, int64_t base_row, int r0, int N) {
  for (int e = threadIdx.x; e < TB * 128; e += blockDim.x) {
    const int r = e >> 7, d = e & 127;
    dst[r * LD + d] = (r0 + r < N) ? __bfloat162float(src[(base_row + r0 + r) * 128 + d]) : 0.f;
  }
}

template <int QK>
__global__ void __launch_bounds__(256) dkdv_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ v,
    const __nv_bfloat16* __restrict__ dout, const float* __restrict__ lse,
    const float* __restrict__ delta, const uint8_t* __restrict__ qc, const float* __restrict__ qd,
    const uint8_t* __restrict__ kc, const float* __restrict__ kd, const uint8_t* __restrict__ mask,
    int64_t mstride, __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv, int N,
    int64_t dstride, float sm_scale) {
  extern __shared__ float sm[];
  float* sK = sm;                 // [64][LD] K codes
  float* sV = sK + TB * LD;       // [64][LD] V
  float* sQc = sV + TB * LD;      // [64][LD] Q codes
  float* sQ = sQc + TB * LD;      // [64][LD] Q bf16
  float* sDO = sQ + TB * LD;      // [64][LD] dO
  float* sPt = sDO + TB * LD;     // [64 k][LDT] bf16(P)^T
  float* sDSt = sPt + TB * LDT;   // [64 k][LDT] bf16(dS * sm_scale)^T
  float* sKd = sDSt + TB * LDT;   // [64]
  float* sQd = sKd + TB;          // [64]
  float* sL = sQd + TB;           // [64]
  float* sDl = sL + TB;           // [64]
  const int kblk = blockIdx.x, bh = blockIdx.y;
  const int k0 = kblk * TB;
  const int64_t row0 = (int64_t)bh * N;
  const int t = threadIdx.x;
  const int nkb = (N + 63) / 64;
  load_codes<QK>(sK, kc, row0, k0, N);
  load_bf16(sV, v, row0, k0, N);
  if (t < TB) sKd[t] = (k0 + t < N) ? kd[(int64_t)bh * dstride + k0 + t] : 0.f;
  // S^T / dP^T tile mapping: keys ty*4+i, queries tx*4+j
  const int ty = t >> 4, tx = t & 15;
  // dV / dK mapping: keys (t>>5)*8 + i, d (t&31)*4 + j
  const int ak = (t >> 5) * 8, ad = (t & 31) * 4;
  float accV[8][4], accK[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) accV[i][j] = accK[i][j] = 0.f;

  for (int q0 = 0; q0 < N; q0 += TB) {
    if (!pair_valid(mask, mstride, nkb, bh, q0, kblk)) continue;
    __syncthreads();
    load_codes<QK>(sQc, qc, row0, q0, N);
    load_bf16(sQ, q, row0, q0, N);
    load_bf16(sDO, dout, row0, q0, N);
    if (t < TB) {
      const bool ok = q0 + t < N;
      sQd[t] = ok ? qd[(int64_t)bh * dstride + q0 + t] : 0.f;
      sL[t] = ok ? lse[row0 + q0 + t] : 0.f;
      sDl[t] = ok ? delta[row0 + q0 + t] : 0.f;
    }
    __syncthreads();
    float s[4][4], dp[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = dp[i][j] = 0.f;
    for (int d = 0; d < 128; ++d) {
      float kk[4], vv[4], qq[4], oo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kk[i] = sK[(ty * 4 + i) * LD + d];
        vv[i] = sV[(ty * 4 + i) * LD + d];
        qq[i] = sQc[(tx * 4 + i) * LD + d];
        oo[i] = sDO[(tx * 4 + i) * LD + d];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(kk[i], qq[j], s[i][j]);
          dp[i][j] = fmaf(vv[i], oo[j], dp[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int kr = ty * 4 + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int qr = tx * 4 + j;
        float p = 0.f, ds = 0.f;
        if (k0 + kr < N && q0 + qr < N) {
          const float sc = (s[i][j] * sQd[qr]) * sKd[kr];
          p = ex2_approx(sc - sL[qr]);
          ds = p * (dp[i][j] - sDl[qr]);
        }
        sPt[kr * LDT + qr] = round_to_bf16(p);
        sDSt[kr * LDT + qr] = round_to_bf16(ds * sm_scale);
      }
    }
    __syncthreads();
    for (int qi = 0; qi < TB; ++qi) {
      float o[4], qv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[j] = sDO[qi * LD + ad + j];
        qv[j] = sQ[qi * LD + ad + j];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float pt = sPt[(ak + i) * LDT + qi];
        const float dt = sDSt[(ak + i) * LDT + qi];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          accV[i][j] = fmaf(pt, o[j], accV[i][j]);
          accK[i][j] = fmaf(dt, qv[j], accK[i][j]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int kr = k0 + ak + i;
    if (kr < N) {
      const int64_t o = (row0 + kr) * 128 + ad;
      *reinterpret_cast<uint2*>(dv + o) = make_uint2(pack_bf16x2(accV[i][0], accV[i][1]), pack_bf16x2(accV[i][2], accV[i][3]));
      *reinterpret_cast<uint2*>(dk + o) = make_uint2(pack_bf16x2(accK[i][0], accK[i][1]), pack_bf16x2(accK[i][2], accK[i][3]));
    }
  }
}

template <int QK>
__global__ void __launch_bounds__(256) dq_kernel(
    const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const __nv_bfloat16* __restrict__ dout, const float* __restrict__ lse,
    const float* __restrict__ delta, const uint8_t* __restrict__ qc, const float* __restrict__ qd,
    const uint8_t* __restrict__ kc, const float* __restrict__ kd, const uint8_t* __restrict__ mask,
    int64_t mstride, __nv_bfloat16* __restrict__ dq, int N, int64_t dstride, float sm_scale) {
  extern __shared__ float sm[];
  float* sQc = sm;                // [64 q][LD]
  float* sDO = sQc + TB * LD;     // [64 q][LD]
  float* sKc = sDO + TB * LD;     // [64 k][LD]
  float* sV = sKc + TB * LD;      // [64 k][LD]
  float* sK = sV + TB * LD;       // [64 k][LD] smoothed K bf16
  float* sDS = sK + TB * LD;      // [64 q][LDT] bf16(dS)
  float* sKd = sDS + 2 * TB * LDT;
  float* sQd = sKd + TB;
  float* sL = sQd + TB;
  float* sDl = sL + TB;
  const int qblk = blockIdx.x, bh = blockIdx.y;
  const int q0 = qblk * TB;
  const int64_t row0 = (int64_t)bh * N;
  const int t = threadIdx.x;
  const int nkb = (N + 63) / 64;
  load_codes<QK>(sQc, qc, row0, q0, N);
  load_bf16(sDO, dout, row0, q0, N);
  if (t < TB) {
    const bool ok = q0 + t < N;
    sQd[t] = ok ? qd[(int64_t)bh * dstride + q0 + t] : 0.f;
    sL[t] = ok ? lse[row0 + q0 + t] : 0.f;
    sDl[t] = ok ? delta[row0 + q0 + t] : 0.f;
  }
  const int ty = t >> 4, tx = t & 15;           // S: queries ty*4+i, keys tx*4+j
  const int aq = (t >> 5) * 8, ad = (t & 31) * 4;  // dQ: queries aq+i, d ad+j
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int kb = 0; kb < nkb; ++kb) {
    const int k0 = kb * TB;
    if (!pair_valid(mask, mstride, nkb, bh, q0, kb)) continue;
    __syncthreads();
    load_codes<QK>(sKc, kc, row0, k0, N);
    load_bf16(sV, v, row0, k0, N);
    load_bf16(sK, k, row0, k0, N);
    if (t < TB) sKd[t] = (k0 + t < N) ? kd[(int64_t)bh * dstride + k0 + t] : 0.f;
    __syncthreads();
    float s[4][4], dp[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = dp[i][j] = 0.f;
    for (int d = 0; d < 128; ++d) {
      float qq[4], oo[4], kk[4], vv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        qq[i] = sQc[(ty * 4 + i) * LD + d];
        oo[i] = sDO[(ty * 4 + i) * LD + d];
        kk[i] = sKc[(tx * 4 + i) * LD + d];
        vv[i] = sV[(tx * 4 + i) * LD + d];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qq[i], kk[j], s[i][j]);
          dp[i][j] = fmaf(oo[i], vv[j], dp[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qr = ty * 4 + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kr = tx * 4 + j;
        float ds = 0.f;
        if (k0 + kr < N && q0 + qr < N) {
          const float p = ex2_approx((s[i][j] * sQd[qr]) * sKd[kr] - sL[qr]);
          ds = p * (dp[i][j] - sDl[qr]);
        }
        sDS[qr * LDT + kr] = round_to_bf16(ds);
      }
    }
    __syncthreads();
    for (int ki = 0; ki < TB; ++ki) {
      float kv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = sK[ki * LD + ad + j];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float dsv = sDS[(aq + i) * LDT + ki];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(dsv, kv[j], acc[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int qr = q0 + aq + i;
    if (qr < N) {
      const int64_t o = (row0 + qr) * 128 + ad;
      *reinterpret_cast<uint2*>(dq + o) =
          make_uint2(pack_bf16x2(acc[i][0] * sm_scale, acc[i][1] * sm_scale),
                     pack_bf16x2(acc[i][2] * sm_scale, acc[i][3] * sm_scale));
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core backward, elementwise step.  The products of the backward run as
// batched library GEMMs on a chunk of heads and query rows:
//   S  = Qc Kc^T (codes, exact for INT8), dP = dO V^T          (fp32 out)
// then this kernel, per (query row i, key j) of the chunk:
//   p  = exp2((S_ij q_desc_i) k_desc_j - lse_i), 0 on masked (128 x 64) tiles
//   dS = p (dP_ij - Delta_i)
//   P16 = bf16(p), dSs16 = bf16(dS * sm_scale), dS16 = bf16(dS)
// exactly the per-element arithmetic of the CUDA-core kernels above (and of the
// reference, sage_kernels.py:896-907, :1007-1010); the GEMMs dV = P16^T dO,
// dK = dSs16^T Q, dQ = dS16 Ks (x sm_scale) follow.  Eight keys per thread.
__global__ void __launch_bounds__(256) bwd_elementwise_kernel(
    const float* __restrict__ S, const float* __restrict__ dP, const float* __restrict__ qd,
    const float* __restrict__ kd, const float* __restrict__ lse, const float* __restrict__ delta,
    const uint8_t* __restrict__ mask, int64_t mstride, __nv_bfloat16* __restrict__ P16,
    __nv_bfloat16* __restrict__ dSs16, __nv_bfloat16* __restrict__ dS16, int HC, int R, int r0, int N,
    int64_t dstride, int bh0, float sm_scale) {
  const int nv = N / 8;                       // 8-key vectors per row (N % 8 == 0)
  const int64_t items = (int64_t)HC * R * nv;
  const int nkb = (N + 63) / 64;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items; it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = it / nv;              // chunk row: head hc * R + local row
    const int j0 = (int)(it % nv) * 8;
    const int hc = (int)(row / R);
    const int i = r0 + (int)(row % R);        // query row in the head
    const int bh = bh0 + hc;
    const float q_d = qd[(int64_t)bh * dstride + i];
    const float l = lse[(int64_t)bh * N + i];
    const float dl = delta[(int64_t)bh * N + i];
    const bool valid = !mask || mask[(int64_t)bh * mstride + (int64_t)(i / 128) * nkb + j0 / 64] != 0;
    const float4* s4 = reinterpret_cast<const float4*>(S + row * N + j0);
    const float4* d4 = reinterpret_cast<const float4*>(dP + row * N + j0);
    const float4 sa = s4[0], sb = s4[1], da = d4[0], db = d4[1];
    const float sv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
    const float dv[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
    float p[8], ds[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      p[e] = valid ? ex2_approx((sv[e] * q_d) * kd[(int64_t)bh * dstride + j0 + e] - l) : 0.f;
      ds[e] = p[e] * (dv[e] - dl);
    }
    const int64_t o = row * N + j0;
    *reinterpret_cast<uint4*>(P16 + o) = make_uint4(pack_bf16x2(p[0], p[1]), pack_bf16x2(p[2], p[3]),
                                                    pack_bf16x2(p[4], p[5]), pack_bf16x2(p[6], p[7]));
    *reinterpret_cast<uint4*>(dSs16 + o) =
        make_uint4(pack_bf16x2(ds[0] * sm_scale, ds[1] * sm_scale), pack_bf16x2(ds[2] * sm_scale, ds[3] * sm_scale),
                   pack_bf16x2(ds[4] * sm_scale, ds[5] * sm_scale), pack_bf16x2(ds[6] * sm_scale, ds[7] * sm_scale));
    *reinterpret_cast<uint4*>(dS16 + o) = make_uint4(pack_bf16x2(ds[0], ds[1]), pack_bf16x2(ds[2], ds[3]),
                                                     pack_bf16x2(ds[4], ds[5]), pack_bf16x2(ds[6], ds[7]));
  }
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

extern "C" int fd_sage_attn_bwd(const void* q, const void* k, const void* v, const void* dout,
                                const float* lse, const float* delta, const void* q_codes,
                                const float* q_desc, const void* k_codes, const float* k_desc,
                                const uint8_t* block_mask, int64_t mask_bh_stride, void* dq,
                                void* dk, void* dv, int64_t BH, int64_t N, int qk_kind,
                                float sm_scale, void* stream) {
  FD_CHECK_ARG(BH > 0 && BH <= 65535 && N > 0 && N < (1ll << 30), "bad shape");
  FD_CHECK_ARG(qk_kind == FD_QK_INT8 || qk_kind == FD_QK_FP8, "bad qk_kind");
  FD_CHECK_ARG(q && k && v && dout && lse && delta && q_codes && q_desc && k_codes && k_desc && dq &&
                   dk && dv,
               "null pointer");
  FD_CHECK_ARG(aligned8(dq) && aligned8(dk) && aligned8(dv), "gradients must be 8-byte aligned");
  const int64_t dstride = ((N + 127) / 128) * 128;  // per-token descale layout of fd_attn_quant
  cudaStream_t st = (cudaStream_t)stream;
  static bool attr_done[2] = {false, false};
  const int kind = qk_kind == FD_QK_INT8 ? 0 : 1;
  auto k_dkdv = kind == 0 ? attn_bwd::dkdv_kernel<FD_QK_INT8> : attn_bwd::dkdv_kernel<FD_QK_FP8>;
  auto k_dq = kind == 0 ? attn_bwd::dq_kernel<FD_QK_INT8> : attn_bwd::dq_kernel<FD_QK_FP8>;
  if (!attr_done[kind]) {
    if (cudaFuncSetAttribute(k_dkdv, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_bwd::BWD_SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(k_dq, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_bwd::BWD_SMEM) != cudaSuccess)
      return check_launch("sage_attn_bwd attributes");
    attr_done[kind] = true;
  }
  dim3 grid((unsigned)((N + 63) / 64), (unsigned)BH);
  k_dkdv<<<grid, 256, attn_bwd::BWD_SMEM, st>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)v, (const __nv_bfloat16*)dout, lse, delta,
      (const uint8_t*)q_codes, q_desc, (const uint8_t*)k_codes, k_desc, block_mask, mask_bh_stride,
      (__nv_bfloat16*)dk, (__nv_bfloat16*)dv, (int)N, dstride, sm_scale);
  int rc = check_launch("sage_attn_bwd dkdv");
  if (rc) return rc;
  k_dq<<<grid, 256, attn_bwd::BWD_SMEM, st>>>(
      (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (const __nv_bfloat16*)dout, lse, delta,
      (const uint8_t*)q_codes, q_desc, (const uint8_t*)k_codes, k_desc, block_mask, mask_bh_stride,
      (__nv_bfloat16*)dq, (int)N, dstride, sm_scale);
  return check_launch("sage_attn_bwd dq");
}

// Elementwise step of the tensor-core backward for a chunk of HC heads (bh0 ..
// bh0 + HC - 1) and query rows [r0, r0 + R): S, dP (HC, R, N) fp32 in; P16,
// dSs16, dS16 (HC, R, N) bf16 out.  q_desc / k_desc are the per-token descales
// of fd_attn_quant (row stride round_up(N, 128)); lse, delta (BH, N).  N % 8 == 0.
extern "C" int fd_sage_attn_bwd_elementwise(const float* S, const float* dP, const float* q_desc, const float* k_desc,
                                            const float* lse, const float* delta, const uint8_t* block_mask,
                                            int64_t mask_bh_stride, void* P16, void* dSs16, void* dS16, int64_t HC,
                                            int64_t R, int64_t r0, int64_t N, int64_t bh0, float sm_scale,
                                            void* stream) {
  FD_CHECK_ARG(HC > 0 && R > 0 && N > 0 && N % 8 == 0 && r0 >= 0 && r0 + R <= N && bh0 >= 0, "bad shape");
  FD_CHECK_ARG(N < (1ll << 31) && HC * R * N < (1ll << 40), "chunk too large");
  FD_CHECK_ARG(S && dP && q_desc && k_desc && lse && delta && P16 && dSs16 && dS16, "null pointer");
  FD_CHECK_ARG(aligned16(S) && aligned16(dP) && aligned16(k_desc) && aligned16(P16) && aligned16(dSs16) &&
                   aligned16(dS16),
               "misaligned pointer");
  const int64_t dstride = ((N + 127) / 128) * 128;
  const int64_t items = HC * R * (N / 8);
  int64_t grid = (items + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (grid > cap) grid = cap;
  attn_bwd::bwd_elementwise_kernel<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>(
      S, dP, q_desc, k_desc, lse, delta, block_mask, mask_bh_stride, (__nv_bfloat16*)P16, (__nv_bfloat16*)dSs16,
      (__nv_bfloat16*)dS16, (int)HC, (int)R, (int)r0, (int)N, dstride, (int)bh0, sm_scale);
  return check_launch("sage_attn_bwd_elementwise");
}
