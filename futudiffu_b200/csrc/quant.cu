// Memory-bound FP8 quantisers: activation quant (1 x 128), weight quant
// (128 x 128), blockwise dequant, SiLU-gate requant, GELU requant.
//
// All of them move 16-byte vectors per thread and reduce each 128-element
// group inside 16 consecutive lanes, so one warp covers two groups per
// iteration and every global access is a fully coalesced 512-byte warp
// transaction.  Grids are sized to a multiple of the SM count and stride
// over the work.
#include "fd_act.cuh"
#include "fd_host.h"

namespace fd {

template <typename T>
FD_DEV void load8(const T* p, float (&v)[8]);

template <>
FD_DEV void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <>
FD_DEV void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <>
FD_DEV void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

FD_DEV uint2 quant8(const float (&v)[8], float qm) {
  return make_uint2(quant4(v[0], v[1], v[2], v[3], qm), quant4(v[4], v[5], v[6], v[7], qm));
}

// max over the 16 lanes of a half-warp
FD_DEV float half_warp_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

FD_DEV float amax8(const float (&v)[8]) {
  float a = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[i]));
  return a;
}

// ---------------------------------------------------------------- G1
// fp8_act_quant_kernel, src/futudiffu/fp8_kernels.py:54-76.
template <typename T>
__global__ void __launch_bounds__(256) act_quant_kernel(const T* __restrict__ x,
                                                       uint8_t* __restrict__ y,
                                                       float* __restrict__ s, int64_t ngroups) {
  const int64_t half_warps = (int64_t)gridDim.x * (blockDim.x >> 4);
  const int sub = threadIdx.x & 15;
  for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 4) + (threadIdx.x >> 4); g < ngroups;
       g += half_warps) {
    float v[8];
    load8<T>(x + g * 128 + sub * 8, v);
    const float amax = half_warp_max(amax8(v));
    const float qm = quant_mult(amax);
    *reinterpret_cast<uint2*>(y + g * 128 + sub * 8) = quant8(v, qm);
    if (sub == 0) s[g] = dequant_scale(amax);
  }
}

// ---------------------------------------------------------------- G6
// quantize_fp8_blockwise, src/futudiffu/fp8.py:352-369: one CTA per
// 128 x 128 tile, two passes over the (L2-resident) tile.  This reference
// path is torch code, so its quotients follow torch's scalar / tensor rule.
template <typename T>
__global__ void __launch_bounds__(256) weight_quant_kernel(const T* __restrict__ w,
                                                          uint8_t* __restrict__ y,
                                                          float* __restrict__ s, int64_t N,
                                                          int64_t K) {
  const int64_t kb = blockIdx.x, nb = blockIdx.y;
  const int64_t kblocks = K / 128;
  __shared__ float red[8];
  // 256 threads: thread t covers row (t / 16) + 16 * i, columns (t % 16) * 8 .. +8
  const int col = (threadIdx.x & 15) * 8;
  float amax = 0.f;
  for (int r = threadIdx.x >> 4; r < 128; r += 16) {
    float v[8];
    load8<T>(w + (nb * 128 + r) * K + kb * 128 + col, v);
    amax = fmaxf(amax, amax8(v));
  }
  amax = warp_max(amax);
  if (lane_id() == 0) red[warp_id()] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  // torch evaluates `448 / t` as t.reciprocal() * 448: two correctly rounded steps
  const float qs = __fmul_rn(__frcp_rn(fmaxf(amax, 1e-12f)), 448.0f);
  for (int r = threadIdx.x >> 4; r < 128; r += 16) {
    float v[8];
    load8<T>(w + (nb * 128 + r) * K + kb * 128 + col, v);
    *reinterpret_cast<uint2*>(y + (nb * 128 + r) * K + kb * 128 + col) = quant8(v, qs);
  }
  if (threadIdx.x == 0) s[nb * kblocks + kb] = __frcp_rn(qs);  // (1.0 / quant_scale).float()
}

// dequantize_fp8_blockwise, src/futudiffu/fp8.py:469-480.
template <typename TO>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ w,
                                                     const float* __restrict__ s,
                                                     TO* __restrict__ out, int64_t N, int64_t K,
                                                     int64_t total8) {
  const int64_t kblocks = K / 128;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total8;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t n = e / K, k = e % K;
    const float sc = s[(n / 128) * kblocks + k / 128];
    const uint2 c = *reinterpret_cast<const uint2*>(w + e);
    const uint32_t cw[2] = {c.x, c.y};
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      __nv_fp8_e4m3 q;
      q.__x = (cw[j / 4] >> ((j % 4) * 8)) & 0xFF;
      f[j] = float(q) * sc;
    }
    if constexpr (sizeof(TO) == 4) {
      float4* o = reinterpret_cast<float4*>(out + e);
      o[0] = make_float4(f[0], f[1], f[2], f[3]);
      o[1] = make_float4(f[4], f[5], f[6], f[7]);
    } else {
      uint4 u;
      uint32_t* uw = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (std::is_same<TO, __nv_bfloat16>::value) {
          uw[j] = pack_bf16x2(f[2 * j], f[2 * j + 1]);
        } else {
          __half2 h = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
          uw[j] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      *reinterpret_cast<uint4*>(out + e) = u;
    }
  }
}

// ---------------------------------------------------------------- G4
// fp8_silu_gate_quant_kernel, src/futudiffu/fp8_kernels.py:843-916.
__global__ void __launch_bounds__(256) silu_gate_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                             uint8_t* __restrict__ y,
                                                             float* __restrict__ s, int64_t M,
                                                             int64_t N) {
  const int64_t gpr = N / 128;  // groups per row
  const int64_t ngroups = M * gpr;
  const int64_t half_warps = (int64_t)gridDim.x * (blockDim.x >> 4);
  const int sub = threadIdx.x & 15;
  for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 4) + (threadIdx.x >> 4); g < ngroups;
       g += half_warps) {
    const int64_t m = g / gpr, nb = g % gpr;
    float w1[8], w3[8], v[8];
    load8<__nv_bfloat16>(x + m * 2 * N + nb * 128 + sub * 8, w1);
    load8<__nv_bfloat16>(x + m * 2 * N + N + nb * 128 + sub * 8, w3);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = silu_gate(w1[i], w3[i]);
    const float amax = half_warp_max(amax8(v));
    const float qm = quant_mult(amax);
    *reinterpret_cast<uint2*>(y + m * N + nb * 128 + sub * 8) = quant8(v, qm);
    if (sub == 0) s[g] = dequant_scale(amax);
  }
}

// GELU (tanh approximation, torch F.gelu(approximate="tanh")) + G1 quantiser.
__global__ void __launch_bounds__(256) gelu_tanh_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                             uint8_t* __restrict__ y,
                                                             float* __restrict__ s,
                                                             int64_t ngroups) {
  const int64_t half_warps = (int64_t)gridDim.x * (blockDim.x >> 4);
  const int sub = threadIdx.x & 15;
  for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 4) + (threadIdx.x >> 4); g < ngroups;
       g += half_warps) {
    float v[8];
    load8<__nv_bfloat16>(x + g * 128 + sub * 8, v);
#pragma unroll
    for (int i = 0; i < 8; i += 2) gelu_tanh2(v[i], v[i + 1]);
    const float amax = half_warp_max(amax8(v));
    const float qm = quant_mult(amax);
    *reinterpret_cast<uint2*>(y + g * 128 + sub * 8) = quant8(v, qm);
    if (sub == 0) s[g] = dequant_scale(amax);
  }
}

// fp8_gelu_kernel, src/futudiffu/fp8_kernels.py:720-786 (erf GELU).
__global__ void __launch_bounds__(256) gelu_requant_kernel(const uint8_t* __restrict__ x,
                                                          const float* __restrict__ sx,
                                                          uint8_t* __restrict__ y,
                                                          float* __restrict__ sy,
                                                          int64_t ngroups) {
  const int64_t half_warps = (int64_t)gridDim.x * (blockDim.x >> 4);
  const int sub = threadIdx.x & 15;
  for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 4) + (threadIdx.x >> 4); g < ngroups;
       g += half_warps) {
    const uint2 c = *reinterpret_cast<const uint2*>(x + g * 128 + sub * 8);
    const uint32_t cw[2] = {c.x, c.y};
    const float sc = sx[g];
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      __nv_fp8_e4m3 q;
      q.__x = (cw[j / 4] >> ((j % 4) * 8)) & 0xFF;
      const float a = float(q) * sc;
      v[j] = a * 0.5f * (1.0f + erff(div_full(a, 1.41421356237f)));
    }
    const float amax = half_warp_max(amax8(v));
    const float qm = quant_mult(amax);
    *reinterpret_cast<uint2*>(y + g * 128 + sub * 8) = quant8(v, qm);
    if (sub == 0) sy[g] = dequant_scale(amax);
  }
}

}  // namespace fd

using namespace fd;

static int grid_for(int64_t work_items, int per_block) {
  int64_t g = (work_items + per_block - 1) / per_block;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

extern "C" int fd_fp8_act_quant(const void* x, int x_dtype, void* y, float* s, int64_t M,
                                int64_t K, int block, void* stream) {
  FD_CHECK_ARG(block == 128, "block_size must be 128");
  FD_CHECK_ARG(M >= 0 && K > 0 && K % 128 == 0, "K must be a positive multiple of 128");
  if (M == 0) return FD_OK;
  FD_CHECK_ARG(x && y && s, "null pointer");
  FD_CHECK_ARG(aligned16(x) && aligned8(y), "x must be 16-byte and y 8-byte aligned");
  const int64_t ng = M * (K / 128);
  const int grid = grid_for(ng, 16);
  cudaStream_t st = (cudaStream_t)stream;
  switch (x_dtype) {
    case FD_DT_BF16:
      act_quant_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, (uint8_t*)y, s, ng);
      break;
    case FD_DT_F16:
      act_quant_kernel<__half><<<grid, 256, 0, st>>>((const __half*)x, (uint8_t*)y, s, ng);
      break;
    case FD_DT_F32:
      act_quant_kernel<float><<<grid, 256, 0, st>>>((const float*)x, (uint8_t*)y, s, ng);
      break;
    default:
      return set_error(FD_ERR_ARG, "unsupported x dtype");
  }
  return check_launch("act_quant");
}

extern "C" int fd_fp8_weight_quant(const void* w, int w_dtype, void* y, float* s, int64_t N,
                                   int64_t K, int block, void* stream) {
  FD_CHECK_ARG(block == 128, "block_size must be 128");
  FD_CHECK_ARG(N > 0 && K > 0 && N % 128 == 0 && K % 128 == 0,
               "both dimensions must be multiples of 128");
  FD_CHECK_ARG(w && y && s, "null pointer");
  FD_CHECK_ARG(aligned16(w) && aligned8(y), "w must be 16-byte and y 8-byte aligned");
  FD_CHECK_ARG(N / 128 <= 65535, "too many row blocks");
  dim3 grid((unsigned)(K / 128), (unsigned)(N / 128));
  cudaStream_t st = (cudaStream_t)stream;
  switch (w_dtype) {
    case FD_DT_BF16:
      weight_quant_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)w, (uint8_t*)y, s, N, K);
      break;
    case FD_DT_F16:
      weight_quant_kernel<__half><<<grid, 256, 0, st>>>((const __half*)w, (uint8_t*)y, s, N, K);
      break;
    case FD_DT_F32:
      weight_quant_kernel<float><<<grid, 256, 0, st>>>((const float*)w, (uint8_t*)y, s, N, K);
      break;
    default:
      return set_error(FD_ERR_ARG, "unsupported weight dtype");
  }
  return check_launch("weight_quant");
}

extern "C" int fd_fp8_dequant_blockwise(const void* w, const float* s, void* out, int out_dtype,
                                        int64_t N, int64_t K, int block, void* stream) {
  FD_CHECK_ARG(block == 128, "block_size must be 128");
  FD_CHECK_ARG(N > 0 && K > 0 && N % 128 == 0 && K % 128 == 0,
               "both dimensions must be multiples of 128");
  FD_CHECK_ARG(w && s && out, "null pointer");
  FD_CHECK_ARG(aligned8(w) && aligned16(out), "w must be 8-byte and out 16-byte aligned");
  const int64_t total8 = N * K / 8;
  const int grid = grid_for(total8, 256);
  cudaStream_t st = (cudaStream_t)stream;
  switch (out_dtype) {
    case FD_DT_BF16:
      dequant_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const uint8_t*)w, s, (__nv_bfloat16*)out, N, K, total8);
      break;
    case FD_DT_F16:
      dequant_kernel<__half><<<grid, 256, 0, st>>>((const uint8_t*)w, s, (__half*)out, N, K, total8);
      break;
    case FD_DT_F32:
      dequant_kernel<float><<<grid, 256, 0, st>>>((const uint8_t*)w, s, (float*)out, N, K, total8);
      break;
    default:
      return set_error(FD_ERR_ARG, "unsupported output dtype");
  }
  return check_launch("dequant");
}

extern "C" int fd_fp8_silu_gate_quant(const void* x, void* y, float* s, int64_t M, int64_t N,
                                      int block, void* stream) {
  FD_CHECK_ARG(block == 128, "block_size must be 128");
  FD_CHECK_ARG(M >= 0 && N > 0 && N % 128 == 0, "N must be a positive multiple of 128");
  if (M == 0) return FD_OK;
  FD_CHECK_ARG(x && y && s, "null pointer");
  FD_CHECK_ARG(aligned16(x) && aligned8(y), "x must be 16-byte and y 8-byte aligned");
  const int grid = grid_for(M * (N / 128), 16);
  silu_gate_quant_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)x,
                                                                 (uint8_t*)y, s, M, N);
  return check_launch("silu_gate_quant");
}

extern "C" int fd_fp8_gelu_tanh_quant(const void* x, void* y, float* s, int64_t M, int64_t N,
                                      int block, void* stream) {
  FD_CHECK_ARG(block == 128, "block_size must be 128");
  FD_CHECK_ARG(M >= 0 && N > 0 && N % 128 == 0, "N must be a positive multiple of 128");
  if (M == 0) return FD_OK;
  FD_CHECK_ARG(x && y && s, "null pointer");
  FD_CHECK_ARG(aligned16(x) && aligned8(y), "x must be 16-byte and y 8-byte aligned");
  const int64_t ng = M * (N / 128);
  gelu_tanh_quant_kernel<<<grid_for(ng, 16), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, (uint8_t*)y, s, ng);
  return check_launch("gelu_tanh_quant");
}

extern "C" int fd_fp8_gelu_requant(const void* x, const float* sx, void* y, float* sy, int64_t M,
                                   int64_t N, int block, void* stream) {
  FD_CHECK_ARG(block == 128, "block_size must be 128");
  FD_CHECK_ARG(M >= 0 && N > 0 && N % 128 == 0, "N must be a positive multiple of 128");
  if (M == 0) return FD_OK;
  FD_CHECK_ARG(x && sx && y && sy, "null pointer");
  FD_CHECK_ARG(aligned8(x) && aligned8(y), "x and y must be 8-byte aligned");
  const int64_t ng = M * (N / 128);
  gelu_requant_kernel<<<grid_for(ng, 16), 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)x, sx, (uint8_t*)y, sy, ng);
  return check_launch("gelu_requant");
}
