// Scalar pieces shared by the standalone quantisers and the fused GEMM
// epilogues, written with explicit rounding (no compiler contraction freedom),
// so a fused epilogue produces exactly the codes and scales of the unfused
// kernel pair it replaces.
#pragma once

#include "fd_common.cuh"

namespace fd {

// G1 quantiser arithmetic, fp8_act_quant_kernel (src/futudiffu/fp8_kernels.py:65-76):
// the reference divides are Triton's f32 `/` (div.full.f32, see fd_common.cuh).
FD_DEV float quant_mult(float amax) { return div_full(448.0f, fmaxf(amax, 1e-12f)); }
FD_DEV float dequant_scale(float amax) { return fmaxf(div_full(amax, 448.0f), 1e-12f); }

// The reference clamps to +-448 before the cast; the saturating cvt would do
// the same, the explicit clamp keeps NaN handling identical as well.
FD_DEV float clamp448(float v) { return fminf(fmaxf(v, -448.0f), 448.0f); }

// Four values -> four e4m3 codes in one word (byte order = value order).
FD_DEV uint32_t quant4(float a, float b, float c, float d, float qm) {
  return f32x2_to_e4m3x2(clamp448(__fmul_rn(a, qm)), clamp448(__fmul_rn(b, qm))) |
         (f32x2_to_e4m3x2(clamp448(__fmul_rn(c, qm)), clamp448(__fmul_rn(d, qm))) << 16);
}

// Triton lowers fp32 tl.exp(x) to ex2.approx.f32(x * log2(e)) (measured: bit
// identical); the same two instructions are used here.
FD_DEV float exp_like_triton(float x) {
  float y;
  asm("{\n\t.reg .f32 t;\n\t"
      "mul.f32 t, %1, 0f3FB8AA3B;\n\t"
      "ex2.approx.f32 %0, t;\n\t}"
      : "=f"(y)
      : "f"(x));
  return y;
}

// SiLU gate of fp8_silu_gate_quant_kernel (src/futudiffu/fp8_kernels.py:877-905):
// (w1 * (1 / (1 + exp(-w1)))) * w3 in fp32.
FD_DEV float silu_gate(float w1, float w3) {
  const float sig = div_full(1.0f, __fadd_rn(1.0f, exp_like_triton(-w1)));
  return __fmul_rn(__fmul_rn(w1, sig), w3);
}

// GELU, tanh approximation (torch F.gelu(approximate="tanh")):
// 0.5 a (1 + tanh(sqrt(2/pi) (a + 0.044715 a^3))).
FD_DEV float gelu_tanh(float a) {
  const float inner = __fmul_rn(0.7978845608028654f, fmaf(__fmul_rn(0.044715f, a), __fmul_rn(a, a), a));
  return __fmul_rn(__fmul_rn(0.5f, a), __fadd_rn(1.0f, tanhf(inner)));
}

}  // namespace fd
