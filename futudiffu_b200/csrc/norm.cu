// Fused RMSNorm prologues of the DiT block:
//   P1 rms_norm_modulate    (src/futudiffu/fused_kernels.py:43-86)
//   P2 rms_norm_gate_residual (src/futudiffu/fused_kernels.py:99-148)
//   P3 qkv_postprocess       (src/futudiffu/fused_kernels.py:270-385)
//   P1 + G1 rms_norm_modulate_quant: P1's bf16 row quantised 1 x 128 to e4m3 in
//      the same pass (the input of the next FP8 GEMM), equal to P1 followed by
//      fp8_act_quant (src/futudiffu/fp8_kernels.py:54-90) code for code.
//
// P1/P2: one warp per token row; the row is held in registers (dim <= 8192,
// 16-byte vectors), so x is read exactly once and the output written once.
// P3: one warp per (token, head): each lane owns two RoPE pairs (4 values)
// of Q and K and 4 values of V.
//
// Arithmetic follows the Triton kernels: fp32 throughout, mean of squares and
// rrms = 1 / sqrt(mean + eps) with Triton's lowerings of `/` (div.full.f32) and
// tl.sqrt (sqrt.approx.f32), products evaluated left to right.
#include "fd_act.cuh"
#include "fd_host.h"
#include "fd_p3.cuh"

namespace fd {

template <int DT>
FD_DEV float load_elem(const void* p, int64_t i) {
  if constexpr (DT == FD_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  else if constexpr (DT == FD_DT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  else return reinterpret_cast<const float*>(p)[i];
}

FD_DEV void unpack_bf16x8(const uint4& u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

FD_DEV uint4 pack_bf16x8(const float (&v)[8]) {
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

// Eight consecutive elements of a DT array as floats; p + i must be 16-byte
// aligned (one 16-byte load for bf16 / f16, two for f32).
template <int DT>
FD_DEV void load8(const void* p, int64_t i, float (&v)[8]) {
  if constexpr (DT == FD_DT_F32) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i));
    const float4 b = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + i));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if constexpr (DT == FD_DT_BF16) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
      } else {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
        v[2 * k] = __low2float(h);
        v[2 * k + 1] = __high2float(h);
      }
    }
  }
}

// n = (x rrms) w for the eight values of one vector, each pair's multiplies as
// packed f32x2 instructions (mul.rn.f32x2 rounds every lane as a scalar
// multiply does, so the products are those of the left-to-right scalar form).
FD_DEV void normed8(const float (&x)[8], float rrms, const float (&w)[8], float (&n)[8]) {
  const uint64_t r = pk(rrms, rrms);
#pragma unroll
  for (int e = 0; e < 8; e += 2) unpk(mul2(mul2(pk(x[e], x[e + 1]), r), pk(w[e], w[e + 1])), n[e], n[e + 1]);
}

// o = n f, pairs packed as in normed8.
FD_DEV void times8(const float (&n)[8], const float (&f)[8], float (&o)[8]) {
#pragma unroll
  for (int e = 0; e < 8; e += 2) unpk(mul2(pk(n[e], n[e + 1]), pk(f[e], f[e + 1])), o[e], o[e + 1]);
}

// Max 8192 / (32 lanes * 8) = 32 vectors per lane.
constexpr int kMaxVecPerLane = 32;

// MODE 0: P1 (modulate), MODE 1: P2 (gate + residual), MODE 2: P1 + 1 x 128 e4m3
// quantisation (out holds the codes, qs the dequant scales).  A 128-column group
// is 16 consecutive 8-column vectors, i.e. one half-warp for a given j.
//
// Grid (B, CTAs per sample): a CTA serves rows of one sample b, so the
// per-column factors -- the norm weight and (1 + scale[b]) or tanh(gate[b]),
// which the reference evaluates per element -- are computed once per CTA into
// shared memory (fp32, dim <= 8192) and read back as 16-byte vectors.
//
// Row ranges (packed multi-image sequences, per-token adaLN): with `ranges`
// set, "sample" b is the row range [ranges[b], ranges[b + 1]) and its factors
// come from parameter row rparam[b] of scale / gate (n_params rows), so a
// packed sequence's per-image modulation is applied without materialising a
// (tokens, dim) tensor.  Ranges or parameter rows out of bounds are skipped.
// Registers: the row (NV 16-byte vectors per lane) dominates; P1 and P2 rows of up
// to 3072 values (NV <= 12) fit three CTAs per SM, wider rows two; P1 + G1 runs two
// (at three its register cap of 85 spilled).
template <int MODE, int WDT, int SDT, int NV>
__global__ void __launch_bounds__(256, (NV <= 12 && MODE != 2 ? 3 : 2)) rms_row_kernel(const __nv_bfloat16* __restrict__ x,
                                                     const void* __restrict__ w,
                                                     const void* __restrict__ sg,
                                                     const __nv_bfloat16* __restrict__ res,
                                                     __nv_bfloat16* __restrict__ out,
                                                     float* __restrict__ qs,
                                                     int64_t rows, int64_t S, int dim, float eps,
                                                     const int* __restrict__ ranges,
                                                     const int* __restrict__ rparam, int64_t n_params) {
  extern __shared__ float4 norm_smem[];
  float* s_w = reinterpret_cast<float*>(norm_smem);  // [dim] weight
  float* s_f = s_w + dim;                             // [dim] 1 + scale  or  tanh(gate)
  const int lane = lane_id();
  const int64_t b = blockIdx.x;
  int64_t prow = b, row0 = b * S, nrows = S;
  if (ranges) {
    prow = rparam[b];
    row0 = ranges[b];
    nrows = (int64_t)ranges[b + 1] - row0;
    if (prow < 0 || prow >= n_params || row0 < 0 || nrows < 0 || row0 + nrows > rows) return;
  }
  if ((int64_t)blockIdx.y * (blockDim.x >> 5) >= nrows) return;  // no row for this CTA
  // Stage the factors: 16-byte loads, at most four per thread (dim <= 8192), all
  // independent, so the CTA pays about one memory latency before its rows.
  const size_t sb = SDT == FD_DT_F32 ? 4 : 2;
  const bool vec_ok =
      ((reinterpret_cast<uintptr_t>(w) | (reinterpret_cast<uintptr_t>(sg) + (size_t)prow * dim * sb)) & 15) == 0;
  if (vec_ok) {
#pragma unroll 4
    for (int c8 = threadIdx.x; c8 < dim / 8; c8 += blockDim.x) {
      float wv[8], sv[8];
      load8<WDT>(w, (int64_t)c8 * 8, wv);
      load8<SDT>(sg, prow * dim + (int64_t)c8 * 8, sv);
      float fv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) fv[e] = MODE == 1 ? tanhf(sv[e]) : 1.0f + sv[e];
      reinterpret_cast<float4*>(s_w)[2 * c8] = make_float4(wv[0], wv[1], wv[2], wv[3]);
      reinterpret_cast<float4*>(s_w)[2 * c8 + 1] = make_float4(wv[4], wv[5], wv[6], wv[7]);
      reinterpret_cast<float4*>(s_f)[2 * c8] = make_float4(fv[0], fv[1], fv[2], fv[3]);
      reinterpret_cast<float4*>(s_f)[2 * c8 + 1] = make_float4(fv[4], fv[5], fv[6], fv[7]);
    }
  } else {
    for (int col = threadIdx.x; col < dim; col += blockDim.x) {
      s_w[col] = load_elem<WDT>(w, col);
      const float sv = load_elem<SDT>(sg, prow * dim + col);
      s_f[col] = MODE == 1 ? tanhf(sv) : 1.0f + sv;
    }
  }
  __syncthreads();
  const int nvec = dim / 8;
  const int64_t wpb = (int64_t)gridDim.y * (blockDim.x >> 5);  // warps serving this sample
  for (int64_t sr = (int64_t)blockIdx.y * (blockDim.x >> 5) + warp_id(); sr < nrows; sr += wpb) {
    const int64_t row = row0 + sr;
    uint4 xr[NV];  // the row, still packed bf16 (half the registers of fp32)
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j);
      if (c < nvec) {
        xr[j] = __ldg(reinterpret_cast<const uint4*>(x + row * dim) + c);
        float t[8];
        unpack_bf16x8(xr[j], t);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += t[e] * t[e];
      }
    }
    ss = warp_sum(ss);
    const float mean_sq = div_full(ss, (float)dim);
    const float rrms = div_full(1.0f, sqrt_approx(mean_sq + eps));
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j);
      if constexpr (MODE == 2) {
        if (32 * j >= nvec) break;  // warp-uniform
        // the unfused pair stores P1's row in bf16 and quantises those values
        float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (c < nvec) {
          const float4* w4 = reinterpret_cast<const float4*>(s_w + c * 8);
          const float4* f4 = reinterpret_cast<const float4*>(s_f + c * 8);
          const float4 wa = w4[0], wb = w4[1], fa = f4[0], fb = f4[1];
          const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
          const float fv[8] = {fa.x, fa.y, fa.z, fa.w, fb.x, fb.y, fb.z, fb.w};
          float xv[8], nv[8], pv[8];
          unpack_bf16x8(xr[j], xv);
          normed8(xv, rrms, wv, nv);
          times8(nv, fv, pv);
          // bf16 rounding two values per cvt, back to f32 as in unpack_bf16x8
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const uint32_t h = pack_bf16x2(pv[e], pv[e + 1]);
            o[e] = __uint_as_float(h << 16);
            o[e + 1] = __uint_as_float(h & 0xFFFF0000u);
          }
        }
        float amax = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(o[e]));
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        if (c < nvec) {
          const float qm = quant_mult(amax);
          uint8_t* codes = reinterpret_cast<uint8_t*>(out);
          *reinterpret_cast<uint2*>(codes + row * dim + c * 8) =
              make_uint2(quant4p(o[0], o[1], o[2], o[3], qm), quant4p(o[4], o[5], o[6], o[7], qm));
          if ((lane & 15) == 0) qs[row * (dim / 128) + c / 16] = dequant_scale(amax);
        }
      } else if (c < nvec) {
        float o[8];
        float r[8];
        if constexpr (MODE == 1)
          unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(res + row * dim) + c), r);
        const float4* w4 = reinterpret_cast<const float4*>(s_w + c * 8);
        const float4* f4 = reinterpret_cast<const float4*>(s_f + c * 8);
        const float4 wa = w4[0], wb = w4[1], fa = f4[0], fb = f4[1];
        const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const float fv[8] = {fa.x, fa.y, fa.z, fa.w, fb.x, fb.y, fb.z, fb.w};
        float xv[8];
        unpack_bf16x8(xr[j], xv);
        if constexpr (MODE == 1) {
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = r[e] + fv[e] * ((xv[e] * rrms) * wv[e]);
        } else {
          float nv[8];
          normed8(xv, rrms, wv, nv);
          times8(nv, fv, o);
        }
        reinterpret_cast<uint4*>(out + row * dim)[c] = pack_bf16x8(o);
      }
    }
  }
}

template <int MODE, int WDT, int SDT>
static void launch_rms(const void* x, const void* w, const void* sg, const void* res, void* out,
                       float* qs, int64_t rows, int64_t S, int dim, float eps, cudaStream_t st,
                       const int* ranges, const int* rparam, int64_t n_ranges, int64_t n_params) {
  const int nvec = dim / 8;
  const int64_t B = ranges ? n_ranges : rows / S;
  // about 8 CTAs (64 warps) per SM in total, spread over the samples (ranges),
  // and no more CTAs than one row per warp needs (ranges: sized by the total row
  // count, since one range may hold most rows).  The per-CTA staging of the
  // factors is one round of 16-byte loads, cheap next to a warp's rows.
  int64_t per_b = ((int64_t)num_sms() * 8 + B - 1) / B;
  const int64_t need = ((ranges ? rows : S) + 7) / 8;
  if (per_b > need) per_b = need;
  if (per_b < 1) per_b = 1;
  const dim3 grid((unsigned)B, (unsigned)per_b);
  const size_t smem = 2 * (size_t)dim * sizeof(float);
#define FD_RMS_LAUNCH(NVV)                                                                  \
  do {                                                                                      \
    auto kern = rms_row_kernel<MODE, WDT, SDT, NVV>;                                        \
    static bool attr_done = false;                                                          \
    if (!attr_done) {                                                                       \
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 8192 * 4); \
      attr_done = true;                                                                     \
    }                                                                                       \
    kern<<<grid, 256, smem, st>>>((const __nv_bfloat16*)x, w, sg, (const __nv_bfloat16*)res, \
                                  (__nv_bfloat16*)out, qs, rows, S, dim, eps, ranges, rparam, \
                                  n_params);                                                \
  } while (0)
  // the row lives in registers: the smallest vector count that holds it
  if (nvec <= 32 * 4) FD_RMS_LAUNCH(4);
  else if (nvec <= 32 * 8) FD_RMS_LAUNCH(8);
  else if (nvec <= 32 * 12) FD_RMS_LAUNCH(12);  // dim 3072
  else if (nvec <= 32 * 16) FD_RMS_LAUNCH(16);
  else if (nvec <= 32 * 20) FD_RMS_LAUNCH(20);  // dim 5120
  else FD_RMS_LAUNCH(32);
#undef FD_RMS_LAUNCH
}

template <int MODE>
static int dispatch_rms(const void* x, const void* w, int wdt, const void* sg, int sdt,
                        const void* res, void* out, int64_t rows, int64_t S, int dim, float eps,
                        cudaStream_t st, float* qs = nullptr, const int* ranges = nullptr,
                        const int* rparam = nullptr, int64_t n_ranges = 0, int64_t n_params = 0) {
#define FD_RMS_ARGS x, w, sg, res, out, qs, rows, S, dim, eps, st, ranges, rparam, n_ranges, n_params
#define FD_RMS_W(WD)                                                                       \
  switch (sdt) {                                                                           \
    case FD_DT_BF16: launch_rms<MODE, WD, FD_DT_BF16>(FD_RMS_ARGS); break;                 \
    case FD_DT_F16: launch_rms<MODE, WD, FD_DT_F16>(FD_RMS_ARGS); break;                   \
    case FD_DT_F32: launch_rms<MODE, WD, FD_DT_F32>(FD_RMS_ARGS); break;                   \
    default: return set_error(FD_ERR_ARG, "unsupported scale/gate dtype");                 \
  }
  switch (wdt) {
    case FD_DT_BF16: FD_RMS_W(FD_DT_BF16); break;
    case FD_DT_F16: FD_RMS_W(FD_DT_F16); break;
    case FD_DT_F32: FD_RMS_W(FD_DT_F32); break;
    default: return set_error(FD_ERR_ARG, "unsupported weight dtype");
  }
#undef FD_RMS_W
#undef FD_RMS_ARGS
  return check_launch(MODE == 0 ? "rms_norm_modulate" : MODE == 1 ? "rms_norm_gate_residual" : "rms_norm_modulate_quant");
}

// ---------------------------------------------------------------- P3
// One warp per (token row, head); lane l owns elements 4l .. 4l+3 (pairs
// 2l and 2l+1) of Q, K and V of that head.
__global__ void __launch_bounds__(256) qkv_post_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                      const float* __restrict__ qw,
                                                      const float* __restrict__ kw,
                                                      const float* __restrict__ freqs,
                                                      __nv_bfloat16* __restrict__ oq,
                                                      __nv_bfloat16* __restrict__ ok,
                                                      __nv_bfloat16* __restrict__ ov,
                                                      int64_t rows, int64_t S, int H, float eps,
                                                      int64_t S_out, int64_t s_off) {
  constexpr int HD = 128;
  const int lane = lane_id();
  const int64_t items = rows * H;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int dim = H * HD;
  const float4 wq = reinterpret_cast<const float4*>(qw)[lane];
  const float4 wk = reinterpret_cast<const float4*>(kw)[lane];
  for (int64_t it = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp_id(); it < items; it += warps) {
    const int64_t row = it / H;
    const int h = (int)(it % H);
    const __nv_bfloat16* base = qkv + row * 3 * dim + h * HD + lane * 4;
    const uint2 uq = *reinterpret_cast<const uint2*>(base);
    const uint2 uk = *reinterpret_cast<const uint2*>(base + dim);
    const uint2 uv = *reinterpret_cast<const uint2*>(base + 2 * dim);
    float q[4] = {bf16_bits_to_f32(uq.x & 0xFFFF), bf16_bits_to_f32(uq.x >> 16),
                  bf16_bits_to_f32(uq.y & 0xFFFF), bf16_bits_to_f32(uq.y >> 16)};
    float k[4] = {bf16_bits_to_f32(uk.x & 0xFFFF), bf16_bits_to_f32(uk.x >> 16),
                  bf16_bits_to_f32(uk.y & 0xFFFF), bf16_bits_to_f32(uk.y >> 16)};
    const float rq = p3_rinv(warp_sum(p3_sumsq4(q)), eps);
    const float rk = p3_rinv(warp_sum(p3_sumsq4(k)), eps);
    const float wqa[4] = {wq.x, wq.y, wq.z, wq.w};
    const float wka[4] = {wk.x, wk.y, wk.z, wk.w};
    float qo[4], ko[4];
    // freqs (rows, 64, 2, 2): pair p at row*256 + p*4: [cos, -sin, sin, cos]
    const float4* fr = reinterpret_cast<const float4*>(freqs + row * 256) + lane * 2;
    p3_rope4(q, rq, wqa, fr, qo);
    p3_rope4(k, rk, wka, fr, ko);
    const int64_t b = row / S, s = row % S;
    const int64_t o = ((b * H + h) * S_out + s_off + s) * HD + lane * 4;
    *reinterpret_cast<uint2*>(oq + o) = make_uint2(pack_bf16x2(qo[0], qo[1]), pack_bf16x2(qo[2], qo[3]));
    *reinterpret_cast<uint2*>(ok + o) = make_uint2(pack_bf16x2(ko[0], ko[1]), pack_bf16x2(ko[2], ko[3]));
    *reinterpret_cast<uint2*>(ov + o) = uv;
  }
}

}  // namespace fd

using namespace fd;

extern "C" int fd_rms_norm_modulate(const void* x, const void* w, int w_dtype, const void* scale,
                                    int scale_dtype, void* out, int64_t B, int64_t S, int64_t dim,
                                    float eps, void* stream) {
  FD_CHECK_ARG(B >= 0 && S >= 0 && dim > 0 && dim % 8 == 0 && dim <= 8192,
               "dim must be a multiple of 8 and at most 8192");
  if (B * S == 0) return FD_OK;
  FD_CHECK_ARG(x && w && scale && out, "null pointer");
  FD_CHECK_ARG(aligned16(x) && aligned16(out), "x and out must be 16-byte aligned");
  return dispatch_rms<0>(x, w, w_dtype, scale, scale_dtype, nullptr, out, B * S, S, (int)dim, eps,
                         (cudaStream_t)stream);
}

extern "C" int fd_rms_norm_modulate_quant(const void* x, const void* w, int w_dtype, const void* scale,
                                          int scale_dtype, void* y, float* y_s, int64_t B, int64_t S,
                                          int64_t dim, float eps, void* stream) {
  FD_CHECK_ARG(B >= 0 && S >= 0 && dim > 0 && dim % 128 == 0 && dim <= 8192,
               "dim must be a multiple of 128 and at most 8192");
  if (B * S == 0) return FD_OK;
  FD_CHECK_ARG(x && w && scale && y && y_s, "null pointer");
  FD_CHECK_ARG(aligned16(x) && aligned16(y), "x and y must be 16-byte aligned");
  return dispatch_rms<2>(x, w, w_dtype, scale, scale_dtype, nullptr, y, B * S, S, (int)dim, eps,
                         (cudaStream_t)stream, y_s);
}

extern "C" int fd_rms_norm_gate_residual(const void* x, const void* w, int w_dtype,
                                         const void* gate, int gate_dtype, const void* residual,
                                         void* out, int64_t B, int64_t S, int64_t dim, float eps,
                                         void* stream) {
  FD_CHECK_ARG(B >= 0 && S >= 0 && dim > 0 && dim % 8 == 0 && dim <= 8192,
               "dim must be a multiple of 8 and at most 8192");
  if (B * S == 0) return FD_OK;
  FD_CHECK_ARG(x && w && gate && residual && out, "null pointer");
  FD_CHECK_ARG(aligned16(x) && aligned16(out) && aligned16(residual),
               "x, residual and out must be 16-byte aligned");
  return dispatch_rms<1>(x, w, w_dtype, gate, gate_dtype, residual, out, B * S, S, (int)dim, eps,
                         (cudaStream_t)stream);
}

// Row-range variants (packed sequences with per-image adaLN): rows
// [range_rows[i], range_rows[i + 1]) use parameter row range_param[i] of
// scale / gate (n_params x dim).  range_rows (n_ranges + 1) and range_param
// (n_ranges) are int32 DEVICE arrays; rows outside every range are not written.
#define FD_RANGE_CHECKS                                                                     \
  FD_CHECK_ARG(rows >= 0 && dim > 0 && dim <= 8192 && n_ranges >= 0 && n_params > 0, "bad shape"); \
  FD_CHECK_ARG(rows < (1ll << 31) && n_ranges < (1ll << 31), "too many rows");             \
  if (rows == 0 || n_ranges == 0) return FD_OK;                                             \
  FD_CHECK_ARG(range_rows && range_param, "null range arrays")

extern "C" int fd_rms_norm_modulate_ranges(const void* x, const void* w, int w_dtype, const void* scale,
                                           int scale_dtype, void* out, int64_t rows, int64_t dim, float eps,
                                           const int32_t* range_rows, const int32_t* range_param,
                                           int64_t n_ranges, int64_t n_params, void* stream) {
  FD_RANGE_CHECKS;
  FD_CHECK_ARG(dim % 8 == 0, "dim must be a multiple of 8");
  FD_CHECK_ARG(x && w && scale && out, "null pointer");
  FD_CHECK_ARG(aligned16(x) && aligned16(out), "x and out must be 16-byte aligned");
  return dispatch_rms<0>(x, w, w_dtype, scale, scale_dtype, nullptr, out, rows, rows, (int)dim, eps,
                         (cudaStream_t)stream, nullptr, range_rows, range_param, n_ranges, n_params);
}

extern "C" int fd_rms_norm_modulate_quant_ranges(const void* x, const void* w, int w_dtype,
                                                 const void* scale, int scale_dtype, void* y, float* y_s,
                                                 int64_t rows, int64_t dim, float eps,
                                                 const int32_t* range_rows, const int32_t* range_param,
                                                 int64_t n_ranges, int64_t n_params, void* stream) {
  FD_RANGE_CHECKS;
  FD_CHECK_ARG(dim % 128 == 0, "dim must be a multiple of 128");
  FD_CHECK_ARG(x && w && scale && y && y_s, "null pointer");
  FD_CHECK_ARG(aligned16(x) && aligned16(y), "x and y must be 16-byte aligned");
  return dispatch_rms<2>(x, w, w_dtype, scale, scale_dtype, nullptr, y, rows, rows, (int)dim, eps,
                         (cudaStream_t)stream, y_s, range_rows, range_param, n_ranges, n_params);
}

extern "C" int fd_rms_norm_gate_residual_ranges(const void* x, const void* w, int w_dtype, const void* gate,
                                                int gate_dtype, const void* residual, void* out, int64_t rows,
                                                int64_t dim, float eps, const int32_t* range_rows,
                                                const int32_t* range_param, int64_t n_ranges,
                                                int64_t n_params, void* stream) {
  FD_RANGE_CHECKS;
  FD_CHECK_ARG(dim % 8 == 0, "dim must be a multiple of 8");
  FD_CHECK_ARG(x && w && gate && residual && out, "null pointer");
  FD_CHECK_ARG(aligned16(x) && aligned16(out) && aligned16(residual),
               "x, residual and out must be 16-byte aligned");
  return dispatch_rms<1>(x, w, w_dtype, gate, gate_dtype, residual, out, rows, rows, (int)dim, eps,
                         (cudaStream_t)stream, nullptr, range_rows, range_param, n_ranges, n_params);
}
#undef FD_RANGE_CHECKS

extern "C" int fd_qkv_postprocess_into(const void* qkv, const float* qw, const float* kw,
                                       const float* freqs, void* oq, void* ok, void* ov, int64_t B,
                                       int64_t S, int64_t H, int64_t hd, float eps, int64_t S_out,
                                       int64_t s_off, void* stream) {
  FD_CHECK_ARG(hd == 128, "head_dim must be 128");
  FD_CHECK_ARG(B >= 0 && S >= 0 && H > 0, "bad shape");
  FD_CHECK_ARG(s_off >= 0 && S_out >= s_off + S, "S_out must hold rows [s_off, s_off + S)");
  if (B * S == 0) return FD_OK;
  FD_CHECK_ARG(qkv && qw && kw && freqs && oq && ok && ov, "null pointer");
  FD_CHECK_ARG(aligned16(qw) && aligned16(kw) && aligned16(freqs) && aligned8(qkv) &&
                   aligned8(oq) && aligned8(ok) && aligned8(ov),
               "misaligned pointer");
  const int64_t items = B * S * H;
  int64_t grid = (items + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (grid > cap) grid = cap;
  qkv_post_kernel<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)qkv, qw, kw, freqs, (__nv_bfloat16*)oq, (__nv_bfloat16*)ok,
      (__nv_bfloat16*)ov, B * S, S, (int)H, eps, S_out, s_off);
  return check_launch("qkv_postprocess");
}

extern "C" int fd_qkv_postprocess(const void* qkv, const float* qw, const float* kw,
                                  const float* freqs, void* oq, void* ok, void* ov, int64_t B,
                                  int64_t S, int64_t H, int64_t hd, float eps, void* stream) {
  return fd_qkv_postprocess_into(qkv, qw, kw, freqs, oq, ok, ov, B, S, H, hd, eps, S, 0, stream);
}
