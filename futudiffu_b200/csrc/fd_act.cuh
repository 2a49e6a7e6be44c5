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

// quant4 with each pair's two multiplies in one packed f32x2 instruction
// (mul.rn.f32x2 rounds every lane as __fmul_rn does): the same codes.
FD_DEV uint32_t quant4p(float a, float b, float c, float d, float qm) {
  const uint64_t q = pk(qm, qm);
  float a2, b2, c2, d2;
  unpk(mul2(pk(a, b), q), a2, b2);
  unpk(mul2(pk(c, d), q), c2, d2);
  return f32x2_to_e4m3x2(clamp448(a2), clamp448(b2)) | (f32x2_to_e4m3x2(clamp448(c2), clamp448(d2)) << 16);
}

// GELU, tanh approximation (torch F.gelu(approximate="tanh")):
// 0.5 a (1 + tanh(u)), u = sqrt(2/pi) (a + 0.044715 a^3), evaluated in the
// logistic form of tanh, 0.5 (1 + tanh u) = 1 / (1 + e^(-2u)):
//   GELU(a) = a / (1 + 2^z),  z = -2 log2(e) u = a (K1 + K3 a^2),
// with K1 = -2 sqrt(2/pi) log2(e) and K3 = 0.044715 K1 rounded to f32 once.
// One ex2.approx and one rcp.approx per value (relative error a few f32 ulp; the
// denominator is >= 1, so nothing cancels), about a third of the issue slots of
// an accurate tanhf.  Where 2^z >= 2^26 the factor is flushed to 0: that is
// where 1 + tanh(u) rounds to exactly 0 in f32 (tanh(u) within half an ulp of
// -1), so large negative inputs give -0 as the tanh form does.
constexpr float GELU_K1 = -2.302208198144325f;
constexpr float GELU_K3 = -0.1029432395800235f;

FD_DEV float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

FD_DEV float gelu_factor(float e) { return e < 67108864.0f ? rcp_approx(__fadd_rn(1.0f, e)) : 0.0f; }

FD_DEV float gelu_tanh(float a) {
  const float z = __fmul_rn(a, fmaf(GELU_K3, __fmul_rn(a, a), GELU_K1));
  return __fmul_rn(a, gelu_factor(ex2_approx(z)));
}

// Two values at once on the packed f32x2 pipes; bit for bit gelu_tanh of each
// (fma.rn / mul.rn .f32x2 round every lane as the scalar instructions do).
FD_DEV void gelu_tanh2(float& a0, float& a1) {
  const uint64_t a = pk(a0, a1);
  float z0, z1;
  unpk(mul2(a, fma2(pk(GELU_K3, GELU_K3), mul2(a, a), pk(GELU_K1, GELU_K1))), z0, z1);
  a0 = __fmul_rn(a0, gelu_factor(ex2_approx(z0)));
  a1 = __fmul_rn(a1, gelu_factor(ex2_approx(z1)));
}

}  // namespace fd
