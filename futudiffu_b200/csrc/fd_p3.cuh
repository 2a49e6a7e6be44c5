// P3 and Q/K code arithmetic shared by the kernels that evaluate it: P3 alone
// (norm.cu), P3 fused with the attention prologue (attn_prologue.cu) and the QKV
// linear's GEMM epilogue (gemm_fp8.cu).  Every rounding is explicit, so the three
// agree bit for bit whatever the surrounding code lets the compiler contract.
// Reference: fused_qkv_postprocess (src/futudiffu/fused_kernels.py:270-471):
// per-head RMSNorm of Q and K (eps, weights), then RoPE on consecutive pairs.
#pragma once

#include "fd_common.cuh"

namespace fd {

// This lane's share of a 128-wide head row's sum of squares (lane l holds
// columns 4l .. 4l + 3; warp_sum adds the 32 shares).
FD_DEV float p3_sumsq4(const float (&x)[4]) {
  return __fmaf_rn(x[3], x[3], __fmaf_rn(x[2], x[2], __fmaf_rn(x[1], x[1], __fmul_rn(x[0], x[0]))));
}

// 1 / sqrt(mean square + eps) from the row's sum of squares; the divides and the
// square root as the reference's Triton kernel evaluates them (div.full,
// sqrt.approx).
FD_DEV float p3_rinv(float ss, float eps) { return div_full(1.0f, sqrt_approx(__fadd_rn(div_full(ss, 128.0f), eps))); }

// Normalised and weighted, then rotated: pairs (0, 1) and (2, 3) of the lane's
// four values with f[p] = [cos, -sin, sin, cos] of pair 2l + p.  Not rounded.
FD_DEV void p3_rope4(const float (&x)[4], float r, const float (&w)[4], const float4* f, float (&o)[4]) {
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const float4 c = f[p];
    const float e = __fmul_rn(__fmul_rn(x[2 * p], r), w[2 * p]);
    const float d = __fmul_rn(__fmul_rn(x[2 * p + 1], r), w[2 * p + 1]);
    o[2 * p] = __fmaf_rn(c.x, e, __fmul_rn(c.y, d));
    o[2 * p + 1] = __fmaf_rn(c.z, e, __fmul_rn(c.x, d));
  }
}

// One Q/K code: INT8 truncated toward zero (the reference's .to(tl.int8); |x inv|
// <= 127 by construction) or e4m3 round-to-nearest.
template <int QK>  // FD_QK_INT8 or FD_QK_FP8
FD_DEV uint32_t quant_code(float x, float inv) {
  const float y = __fmul_rn(x, inv);
  if constexpr (QK == FD_QK_INT8) {
    return (uint32_t)(__float2int_rz(y) & 0xFF);
  } else {
    return f32x2_to_e4m3x2(y, 0.f) & 0xFF;
  }
}

}  // namespace fd
