// fp8_gelu: dequantise 1 x 128 e4m3 groups, erf GELU, requantise
// (fp8_gelu_kernel, src/futudiffu/fp8_kernels.py:720-786).
//
// This file is compiled with -ftz=true (futudiffu_b200/build.py).  The
// reference's Triton kernels link libdevice with its flush-to-zero variants
// selected (Triton's NVIDIA backend sets the libdevice FTZ reflection by
// default), and erff's FTZ variant differs from the default one in the last
// bits; compiling this one kernel the same way makes its codes and scales equal
// to the reference's.  The other arithmetic here sees no subnormal operands that
// matter: the GELU output of a subnormal input is itself below every 1 x 128
// group's quantisation step.
#include "fd_act.cuh"
#include "fd_host.h"

namespace fd {

// One 128-value group per 16 lanes, 8 values per lane (as the quantisers of quant.cu).
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
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      __nv_fp8_e4m3 q;
      q.__x = (cw[j / 4] >> ((j % 4) * 8)) & 0xFF;
      const float a = float(q) * sc;
      // x * 0.5 * (1 + erf(x / sqrt_2)), evaluated left to right as the reference writes it
      v[j] = __fmul_rn(__fmul_rn(a, 0.5f), __fadd_rn(1.0f, erff(div_full(a, 1.41421356237f))));
      amax = fmaxf(amax, fabsf(v[j]));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float qm = quant_mult(amax);
    *reinterpret_cast<uint2*>(y + g * 128 + sub * 8) =
        make_uint2(quant4(v[0], v[1], v[2], v[3], qm), quant4(v[4], v[5], v[6], v[7], qm));
    if (sub == 0) sy[g] = dequant_scale(amax);
  }
}

}  // namespace fd

using namespace fd;

extern "C" int fd_fp8_gelu_requant(const void* x, const float* sx, void* y, float* sy, int64_t M,
                                   int64_t N, int block, void* stream) {
  FD_CHECK_ARG(block == 128, "block_size must be 128");
  FD_CHECK_ARG(M >= 0 && N > 0 && N % 128 == 0, "N must be a positive multiple of 128");
  if (M == 0) return FD_OK;
  FD_CHECK_ARG(x && sx && y && sy, "null pointer");
  FD_CHECK_ARG(aligned8(x) && aligned8(y), "x and y must be 8-byte aligned");
  const int64_t ng = M * (N / 128);
  int64_t grid = (ng + 15) / 16;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (grid > cap) grid = cap;
  gelu_requant_kernel<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)x, sx, (uint8_t*)y, sy, ng);
  return check_launch("gelu_requant");
}
