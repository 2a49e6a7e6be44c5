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
  (void)q; (void)k; (void)v; (void)dout; (void)lse; (void)delta; (void)q_codes; (void)q_desc;
  (void)k_codes; (void)k_desc; (void)block_mask; (void)mask_bh_stride; (void)dq; (void)dk;
  (void)dv; (void)BH; (void)N; (void)qk_kind; (void)sm_scale; (void)stream;
  return set_error(FD_ERR_UNSUPPORTED, "fd_sage_attn_bwd: not built yet");
}
