// Attention quantisation prologue (A1..A4): K mean-smoothing, INT8 / e4m3
// quantisation of Q and K (per token or per block) and e4m3 quantisation of V
// (one scale per (bh, d) over the sequence).
//
// Two launches, both deterministic (fixed reduction order, no atomics):
//   1. colstats: per (bh, row chunk) partial column sums of K and column
//      absmax of V -> workspace.
//   2. quant: per (bh, 128-row block): reduce the partials in chunk order,
//      round the K mean to bf16, smooth, quantise, write codes and scales.
//
// Quotients use Triton's f32 divide (div.full.f32) like the reference kernels.
// Reference arithmetic:
//   _smooth_k          src/futudiffu/sage_attention.py:63-71 (bf16 mean, bf16 sub)
//   INT8 Q/K per token src/futudiffu/sage_kernels.py:632-639, :656-663
//   FP8 Q/K per token  src/futudiffu/sage_kernels.py:151-155, :176-179
//   V e4m3 per channel src/futudiffu/sage_kernels.py:1142-1148 (here over the
//                      whole sequence instead of one 64-row tile)
#include <mutex>

#include "fd_common.cuh"
#include "fd_host.h"
#include "fd_p3.cuh"

namespace fd {

constexpr int kChunkRows = 256;  // rows per colstats CTA

// Scratch of fd_attn_quant_noalloc: a fixed device array, so that entry point
// never allocates.  FD_NOALLOC_WS_FLOATS floats (4 MiB) on every GPU that loads
// the library, held until the process exits.
constexpr int64_t kNoAllocWsFloats = FD_NOALLOC_WS_FLOATS;
static __device__ __align__(256) float g_attn_quant_ws[kNoAllocWsFloats];

FD_DEV void unpack8(const uint4& u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// grid (nchunks, BH), 256 threads: thread t -> column group (t & 15) * 8,
// row lane t >> 4 (16 row lanes).
__global__ void __launch_bounds__(256) colstats_kernel(const __nv_bfloat16* __restrict__ k,
                                                      const __nv_bfloat16* __restrict__ v,
                                                      float* __restrict__ ws_sum,
                                                      float* __restrict__ ws_amax, int64_t N,
                                                      int nchunks, int do_k, int do_v) {
  const int chunk = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int cg = threadIdx.x & 15, rl = threadIdx.x >> 4;
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0}, a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int64_t r0 = (int64_t)chunk * kChunkRows;
  const int rows = (int)((N - r0) < kChunkRows ? (N - r0) : kChunkRows);
  // four rows per lane per iteration: eight independent 16-byte loads in flight
  for (int r = rl; r < rows; r += 64) {
    uint4 kv[4], vv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const bool ok = r + 16 * u < rows;
      const int64_t off = (bh * N + r0 + r + 16 * u) * 128 + cg * 8;
      kv[u] = (do_k && ok) ? __ldg(reinterpret_cast<const uint4*>(k + off)) : make_uint4(0, 0, 0, 0);
      vv[u] = (do_v && ok) ? __ldg(reinterpret_cast<const uint4*>(v + off)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float x[8];
      unpack8(kv[u], x);
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] += x[e];
      unpack8(vv[u], x);
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] = fmaxf(a[e], fabsf(x[e]));
    }
  }
  __shared__ float sh_s[16][128];
  __shared__ float sh_a[16][128];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    sh_s[rl][cg * 8 + e] = s[e];
    sh_a[rl][cg * 8 + e] = a[e];
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    const int c = threadIdx.x;
    float ts = 0.f, ta = 0.f;
    for (int i = 0; i < 16; ++i) {
      ts += sh_s[i][c];
      ta = fmaxf(ta, sh_a[i][c]);
    }
    ws_sum[(bh * nchunks + chunk) * 128 + c] = ts;
    ws_amax[(bh * nchunks + chunk) * 128 + c] = ta;
  }
}

// One CTA per head: reduces the per-chunk column partials into the final
// smoothing mean (bf16-rounded, as torch's bf16 mean) and the V inverse scale,
// once per head instead of once per quantisation CTA.  The partials are summed
// in chunk order (loads batched, additions sequential), and the results go to
// chunk 0's slot of the workspace, where quant_kernel reads them.
__global__ void __launch_bounds__(128) colstats_final_kernel(float* __restrict__ ws_sum,
                                                            float* __restrict__ ws_amax, int64_t N,
                                                            int nchunks, int do_k, int do_v,
                                                            float* __restrict__ k_mean,
                                                            float* __restrict__ v_desc) {
  const int64_t bh = blockIdx.x;
  const int c = threadIdx.x;
  const int64_t base = bh * nchunks * 128 + c;
  if (do_k) {
    float tot = 0.f;
    int i = 0;
    for (; i + 8 <= nchunks; i += 8) {
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = ws_sum[base + (int64_t)(i + u) * 128];
#pragma unroll
      for (int u = 0; u < 8; ++u) tot += t[u];
    }
    for (; i < nchunks; ++i) tot += ws_sum[base + (int64_t)i * 128];
    // torch bf16 mean: fp32 accumulate, times 1/N, round to bf16
    const float mean = round_to_bf16(tot * (1.0f / (float)N));
    ws_sum[base] = mean;
    if (k_mean) k_mean[bh * 128 + c] = mean;
  }
  if (do_v) {
    float am = 0.f;
    int i = 0;
    for (; i + 8 <= nchunks; i += 8) {
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = ws_amax[base + (int64_t)(i + u) * 128];
#pragma unroll
      for (int u = 0; u < 8; ++u) am = fmaxf(am, t[u]);
    }
    for (; i < nchunks; ++i) am = fmaxf(am, ws_amax[base + (int64_t)i * 128]);
    ws_amax[base] = div_full(448.0f, fmaxf(am, 1e-12f));
    v_desc[bh * 128 + c] = div_full(am, 448.0f);
  }
}

template <int QK>
FD_DEV uint2 quant_row8(const float (&x)[8], float inv) {
  uint32_t c[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) c[e] = quant_code<QK>(x[e], inv);
  return make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24),
                    c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
}

FD_DEV float amax8(const float (&v)[8]) {
  float a = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[i]));
  return a;
}

FD_DEV float half_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// grid (ceil(N/128), BH, 2 or 3), 256 threads; blockIdx.z selects Q, K or V, so
// the three tensors are quantised by independent CTAs.  Thread t handles column
// group (t & 15) * 8 of rows (t >> 4) + 16 i, i = 0..7, of the 128-row block.
// The 64 values a thread holds between its amax pass and its quantise pass stay
// packed as bf16 (K after smoothing is bf16-rounded too), so three CTAs fit per
// SM and their loads overlap each other's reductions.
template <int QK, bool KV_ONLY>
__global__ void __launch_bounds__(256, KV_ONLY ? 4 : 3) quant_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, int64_t N, int nchunks, int smooth_k, int q_gran,
    int k_gran, int pv_fp8, float sm_scale_log2e, uint8_t* __restrict__ q_codes,
    float* __restrict__ q_desc, uint8_t* __restrict__ k_codes, float* __restrict__ k_desc,
    uint8_t* __restrict__ v_codes, float* __restrict__ v_desc, float* __restrict__ k_mean,
    const float* __restrict__ ws_sum, const float* __restrict__ ws_amax, int64_t q_desc_stride,
    int64_t k_desc_stride, int z0) {
  const int blk = blockIdx.x;
  const int64_t bh = blockIdx.y;
  // 0 Q, 1 K, 2 V; the K / V-only instantiation (the second pass of the fused
  // prologue) carries no Q code
  const int which = KV_ONLY ? (int)blockIdx.z + 1 : (int)blockIdx.z + z0;
  const int cg = threadIdx.x & 15, rl = threadIdx.x >> 4;
  const int64_t r0 = (int64_t)blk * 128;
  const float qmax = (QK == FD_QK_INT8) ? 127.0f : 448.0f;

  __shared__ float sh_mean[128];
  __shared__ float sh_vinv[128];
  __shared__ float sh_red[8];
  __shared__ float sh_red2[2][8];

  if (threadIdx.x < 128 && which != 0) {
    // final per-head statistics from colstats_final_kernel (chunk 0's slot)
    const int c = threadIdx.x;
    sh_mean[c] = (which == 1 && smooth_k) ? ws_sum[bh * nchunks * 128 + c] : 0.f;
    if (which == 2) sh_vinv[c] = ws_amax[bh * nchunks * 128 + c];
  }
  __syncthreads();

  // ---------------- Q
  if (!KV_ONLY && which == 0) {
    uint4 xr[8];
    float rowmax[8];
    float blkmax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = r0 + rl + 16 * i;
      xr[i] = n < N ? __ldg(reinterpret_cast<const uint4*>(q + (bh * N + n) * 128 + cg * 8)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float x[8];
      unpack8(xr[i], x);
      rowmax[i] = half_max(amax8(x));
      blkmax = fmaxf(blkmax, rowmax[i]);
    }
    if (q_gran == FD_GRAN_BLOCK) {
      blkmax = warp_max(blkmax);
      if (lane_id() == 0) sh_red[warp_id()] = blkmax;
      __syncthreads();
      blkmax = sh_red[0];
#pragma unroll
      for (int w = 1; w < 8; ++w) blkmax = fmaxf(blkmax, sh_red[w]);
      if (threadIdx.x == 0)
        q_desc[bh * q_desc_stride + blk] = div_full(blkmax, qmax) * sm_scale_log2e;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = r0 + rl + 16 * i;
      const float am = (q_gran == FD_GRAN_BLOCK) ? blkmax : rowmax[i];
      const float inv = div_full(qmax, fmaxf(am, 1e-12f));
      if (n < N) {
        float x[8];
        unpack8(xr[i], x);
        *reinterpret_cast<uint2*>(q_codes + (bh * N + n) * 128 + cg * 8) = quant_row8<QK>(x, inv);
        if (q_gran == FD_GRAN_TOKEN && cg == 0)
          q_desc[bh * q_desc_stride + n] = div_full(am, qmax) * sm_scale_log2e;
      } else if (q_gran == FD_GRAN_TOKEN && cg == 0 && n < q_desc_stride) {
        q_desc[bh * q_desc_stride + n] = 0.f;
      }
    }
  }

  // ---------------- K (smoothed)
  if (which == 1) {
    uint4 xr[8];
    float rowmax[8];
    float hmax[2] = {0.f, 0.f};  // rows 0..63 / 64..127 of the block
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = r0 + rl + 16 * i;
      xr[i] = n < N ? __ldg(reinterpret_cast<const uint4*>(k + (bh * N + n) * 128 + cg * 8)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = r0 + rl + 16 * i;
      float x[8];
      unpack8(xr[i], x);
      if (n < N) {
        // torch bf16 subtraction: the difference rounded to bf16 (exact in packed form)
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = round_to_bf16(x[e] - sh_mean[cg * 8 + e]);
        xr[i] = make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]),
                           pack_bf16x2(x[6], x[7]));
      }
      rowmax[i] = half_max(amax8(x));
      hmax[i >> 2] = fmaxf(hmax[i >> 2], rowmax[i]);  // row rl+16i < 64 iff i < 4
    }
    if (k_gran == FD_GRAN_BLOCK) {
      hmax[0] = warp_max(hmax[0]);
      hmax[1] = warp_max(hmax[1]);
      if (lane_id() == 0) {
        sh_red2[0][warp_id()] = hmax[0];
        sh_red2[1][warp_id()] = hmax[1];
      }
      __syncthreads();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float m = sh_red2[h][0];
#pragma unroll
        for (int w = 1; w < 8; ++w) m = fmaxf(m, sh_red2[h][w]);
        hmax[h] = m;
      }
      if (threadIdx.x < 2) {
        const int64_t kb = (int64_t)blk * 2 + threadIdx.x;
        if (kb * 64 < N) k_desc[bh * k_desc_stride + kb] = div_full(hmax[threadIdx.x], qmax);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = r0 + rl + 16 * i;
      const float am = (k_gran == FD_GRAN_BLOCK) ? hmax[i >> 2] : rowmax[i];
      const float inv = div_full(qmax, fmaxf(am, 1e-12f));
      if (n < N) {
        float x[8];
        unpack8(xr[i], x);
        *reinterpret_cast<uint2*>(k_codes + (bh * N + n) * 128 + cg * 8) = quant_row8<QK>(x, inv);
        if (k_gran == FD_GRAN_TOKEN && cg == 0) k_desc[bh * k_desc_stride + n] = div_full(am, qmax);
      } else if (k_gran == FD_GRAN_TOKEN && cg == 0 && n < k_desc_stride) {
        k_desc[bh * k_desc_stride + n] = 0.f;
      }
    }
  }

  // ---------------- V (e4m3, per channel)
  if (which == 2) {
    // all eight rows' loads issued before any conversion: 128 bytes in flight per thread
    uint4 xr[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = r0 + rl + 16 * i;
      xr[i] = n < N ? __ldg(reinterpret_cast<const uint4*>(v + (bh * N + n) * 128 + cg * 8)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = r0 + rl + 16 * i;
      if (n < N) {
        float x[8];
        unpack8(xr[i], x);
        uint32_t c[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = fminf(fmaxf(x[2 * e] * sh_vinv[cg * 8 + 2 * e], -448.f), 448.f);
          const float b = fminf(fmaxf(x[2 * e + 1] * sh_vinv[cg * 8 + 2 * e + 1], -448.f), 448.f);
          c[e] = f32x2_to_e4m3x2(a, b);
        }
        *reinterpret_cast<uint2*>(v_codes + (bh * N + n) * 128 + cg * 8) =
            make_uint2(c[0] | (c[1] << 16), c[2] | (c[3] << 16));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Fused P3 + attention prologue, first pass (one launch per stream of a joint
// attention).  CTA = one 128-row block of one head of one sample; warp w takes
// rows w, w + 8, ... of the block, lane l columns 4l .. 4l + 3 of the head.
// Per row: the P3 arithmetic of qkv_post_kernel (per-head RMSNorm of Q and K,
// RoPE, bf16 rounding of the stored values), then
//   Q -> INT8 / e4m3 codes + descale, exactly as quant_kernel would quantise
//        the bf16 Q P3 stores (per token: at once; per 128-row block: after the
//        CTA has the block's absmax);
//   K, V -> stored in bf16 (K still needs the sequence mean, V its column
//        absmax, before they can be quantised), with this block's K column sums
//        and V column absmax written to the workspace slot of its joint chunk.
// Q / K / V rows are rows s_off + s of the joint (B, H, N, 128) layout; the
// caller guarantees s_off % 128 == 0 and that every stream but the last has a
// multiple of 128 rows, so a chunk never spans two launches.
template <int QK>
__global__ void __launch_bounds__(256, 3) qkv_quant_kernel(
    const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ qw, const float* __restrict__ kw,
    const float* __restrict__ freqs, int64_t S, int H, float eps, int64_t N, int64_t s_off, int q_gran,
    float sm_scale_log2e, uint8_t* __restrict__ q_codes, float* __restrict__ q_desc, int64_t q_desc_stride,
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out, float* __restrict__ ws_sum,
    float* __restrict__ ws_amax, int nchunks, int do_v) {
  constexpr int HD = 128;
  const int blk = blockIdx.x, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t bh = b * H + h;
  const int warp = warp_id(), lane = lane_id();
  const int dim = H * HD;
  const float qmax = (QK == FD_QK_INT8) ? 127.0f : 448.0f;
  const int chunk = (int)((s_off + (int64_t)blk * 128) / 128);
  const float4 wq = reinterpret_cast<const float4*>(qw)[lane];
  const float4 wk = reinterpret_cast<const float4*>(kw)[lane];
  const float wqa[4] = {wq.x, wq.y, wq.z, wq.w};
  const float wka[4] = {wk.x, wk.y, wk.z, wk.w};
  __shared__ float sh_k[8][128];
  __shared__ float sh_v[8][128];
  __shared__ float sh_q[8];
  __shared__ uint2 sh_qkeep[128][32];  // per-block Q: the block's bf16 Q rows until its absmax is known
  float ksum[4] = {0.f, 0.f, 0.f, 0.f}, vmax[4] = {0.f, 0.f, 0.f, 0.f};
  float bmax = 0.f;
#pragma unroll 2
  for (int i = 0; i < 16; ++i) {
    const int r = warp + 8 * i;  // row within the block
    const int64_t s = (int64_t)blk * 128 + r;
    const int64_t n = s_off + s;  // joint row
    if (s >= S) {
      if (q_gran == FD_GRAN_TOKEN && lane == 0 && n < q_desc_stride && s_off + S == N)
        q_desc[bh * q_desc_stride + n] = 0.f;
      continue;
    }
    const int64_t row = b * S + s;
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
    float qo[4], ko[4];
    const float4* fr = reinterpret_cast<const float4*>(freqs + row * 256) + lane * 2;
    p3_rope4(q, rq, wqa, fr, qo);
    p3_rope4(k, rk, wka, fr, ko);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      qo[e] = round_to_bf16(qo[e]);
      ko[e] = round_to_bf16(ko[e]);
    }
    const int64_t o = (bh * N + n) * HD + lane * 4;
    *reinterpret_cast<uint2*>(k_out + o) = make_uint2(pack_bf16x2(ko[0], ko[1]), pack_bf16x2(ko[2], ko[3]));
    *reinterpret_cast<uint2*>(v_out + o) = uv;
#pragma unroll
    for (int e = 0; e < 4; ++e) ksum[e] += ko[e];
    if (do_v) {
      const float v[4] = {bf16_bits_to_f32(uv.x & 0xFFFF), bf16_bits_to_f32(uv.x >> 16),
                          bf16_bits_to_f32(uv.y & 0xFFFF), bf16_bits_to_f32(uv.y >> 16)};
#pragma unroll
      for (int e = 0; e < 4; ++e) vmax[e] = fmaxf(vmax[e], fabsf(v[e]));
    }
    const float qa = fmaxf(fmaxf(fabsf(qo[0]), fabsf(qo[1])), fmaxf(fabsf(qo[2]), fabsf(qo[3])));
    if (q_gran == FD_GRAN_TOKEN) {
      const float am = warp_max(qa);
      const float inv = div_full(qmax, fmaxf(am, 1e-12f));
      const uint32_t c = quant_code<QK>(qo[0], inv) | (quant_code<QK>(qo[1], inv) << 8) |
                         (quant_code<QK>(qo[2], inv) << 16) | (quant_code<QK>(qo[3], inv) << 24);
      *reinterpret_cast<uint32_t*>(q_codes + (bh * N + n) * HD + lane * 4) = c;
      if (lane == 0) q_desc[bh * q_desc_stride + n] = div_full(am, qmax) * sm_scale_log2e;
    } else {
      bmax = fmaxf(bmax, qa);
      sh_qkeep[r][lane] = make_uint2(pack_bf16x2(qo[0], qo[1]), pack_bf16x2(qo[2], qo[3]));
    }
  }
  // K column sums and V column absmax of this block -> workspace slot (bh, chunk)
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    sh_k[warp][lane * 4 + e] = ksum[e];
    sh_v[warp][lane * 4 + e] = vmax[e];
  }
  if (q_gran == FD_GRAN_BLOCK) {
    bmax = warp_max(bmax);
    if (lane == 0) sh_q[warp] = bmax;
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    const int c = threadIdx.x;
    float t = 0.f, a = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      t += sh_k[w][c];
      a = fmaxf(a, sh_v[w][c]);
    }
    ws_sum[(bh * nchunks + chunk) * 128 + c] = t;
    if (do_v) ws_amax[(bh * nchunks + chunk) * 128 + c] = a;
  }
  if (q_gran == FD_GRAN_BLOCK) {
    float m = sh_q[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, sh_q[w]);
    if (threadIdx.x == 0) q_desc[bh * q_desc_stride + chunk] = div_full(m, qmax) * sm_scale_log2e;
    const float inv = div_full(qmax, fmaxf(m, 1e-12f));
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int r = warp + 8 * i;
      const int64_t s = (int64_t)blk * 128 + r;
      if (s >= S) continue;
      const uint2 u = sh_qkeep[r][lane];  // written by this same thread
      const float v4[4] = {__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                           __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u)};
      const uint32_t c = quant_code<QK>(v4[0], inv) | (quant_code<QK>(v4[1], inv) << 8) |
                         (quant_code<QK>(v4[2], inv) << 16) | (quant_code<QK>(v4[3], inv) << 24);
      *reinterpret_cast<uint32_t*>(q_codes + (bh * N + s_off + s) * HD + lane * 4) = c;
    }
  }
}

}  // namespace fd

using namespace fd;

static int64_t n_chunks(int64_t N) { return (N + kChunkRows - 1) / kChunkRows; }

extern "C" int64_t fd_attn_quant_workspace_floats(int64_t BH, int64_t N) {
  return 2 * BH * n_chunks(N) * 128;
}

// Internal layouts of the descale arrays (shared with the attention kernel):
//   per-token q/k: (BH, round_up(N, 128)), zero beyond N
//   per-block q:   (BH, ceil(N/128)); per-block k: (BH, ceil(N/64))
int64_t fd_desc_stride(int64_t N, int gran, int rows_per_block) {
  return gran == FD_GRAN_TOKEN ? ((N + 127) / 128) * 128 : (N + rows_per_block - 1) / rows_per_block;
}

extern "C" int fd_attn_quant(const void* q, const void* k, const void* v, int64_t BH, int64_t N,
                             int smooth_k, int qk_kind, int q_gran, int k_gran, int pv_kind,
                             float sm_scale_log2e, void* q_codes, float* q_desc, void* k_codes,
                             float* k_desc, void* v_codes, float* v_desc, float* k_mean,
                             float* workspace, void* stream) {
  FD_CHECK_ARG(BH > 0 && N > 0, "empty input");
  FD_CHECK_ARG(BH <= 65535, "BH too large");
  FD_CHECK_ARG(N < (1ll << 30), "N too large");
  FD_CHECK_ARG(qk_kind == FD_QK_INT8 || qk_kind == FD_QK_FP8, "bad qk_kind");
  FD_CHECK_ARG((q_gran == FD_GRAN_TOKEN || q_gran == FD_GRAN_BLOCK) &&
                   (k_gran == FD_GRAN_TOKEN || k_gran == FD_GRAN_BLOCK),
               "bad granularity");
  FD_CHECK_ARG(pv_kind == FD_PV_BF16 || pv_kind == FD_PV_FP8, "bad pv_kind");
  FD_CHECK_ARG(q && k && q_codes && q_desc && k_codes && k_desc && workspace, "null pointer");
  FD_CHECK_ARG(pv_kind == FD_PV_BF16 || (v && v_codes && v_desc), "null V pointer");
  FD_CHECK_ARG(aligned16(q) && aligned16(k) && (v == nullptr || aligned16(v)) &&
                   aligned8(q_codes) && aligned8(k_codes) &&
                   (v_codes == nullptr || aligned8(v_codes)),
               "misaligned pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int nchunks = (int)n_chunks(N);
  float* ws_sum = workspace;
  float* ws_amax = workspace + BH * nchunks * 128;
  const int pv_fp8 = pv_kind == FD_PV_FP8;
  if (smooth_k || pv_fp8) {
    colstats_kernel<<<dim3(nchunks, (unsigned)BH), 256, 0, st>>>(
        (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, ws_sum, ws_amax, N, nchunks, smooth_k,
        pv_fp8);
    int rc = check_launch("attn_quant colstats");
    if (rc) return rc;
    colstats_final_kernel<<<(unsigned)BH, 128, 0, st>>>(ws_sum, ws_amax, N, nchunks, smooth_k, pv_fp8,
                                                        k_mean, v_desc);
    rc = check_launch("attn_quant colstats final");
    if (rc) return rc;
  }
  const int64_t qs = fd_desc_stride(N, q_gran, 128), ks = fd_desc_stride(N, k_gran, 64);
  dim3 grid((unsigned)((N + 127) / 128), (unsigned)BH, pv_fp8 ? 3u : 2u);
#define FD_Q_LAUNCH(QK)                                                                         \
  quant_kernel<QK, false><<<grid, 256, 0, st>>>(                                                \
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, N, nchunks,   \
      smooth_k, q_gran, k_gran, pv_fp8, sm_scale_log2e, (uint8_t*)q_codes, q_desc,              \
      (uint8_t*)k_codes, k_desc, (uint8_t*)v_codes, v_desc, k_mean, ws_sum, ws_amax, qs, ks, 0)
  if (qk_kind == FD_QK_INT8) FD_Q_LAUNCH(FD_QK_INT8);
  else FD_Q_LAUNCH(FD_QK_FP8);
#undef FD_Q_LAUNCH
  return check_launch("attn_quant");
}

// ---------------------------------------------------------------------------
// V of the reference's FP8-PV kernel (_sage_attn_fwd_fp8qk_fp8pv_lse,
// src/futudiffu/sage_kernels.py:1142-1148): per 64-row tile and column d,
// amax over the tile's rows (rows past N count as 0), codes e4m3(v * (448 /
// max(amax, 1e-12))) and descale amax / 448.  One CTA per (tile, bh), one
// thread per column: every row read is one coalesced 256-byte line.
namespace fd {
__global__ void __launch_bounds__(128) v_tile_quant_kernel(const __nv_bfloat16* __restrict__ v, int64_t N,
                                                          uint8_t* __restrict__ v_codes,
                                                          float* __restrict__ v_desc) {
  const int64_t t = blockIdx.x, bh = blockIdx.y, ntiles = gridDim.x;
  const int c = threadIdx.x;
  const int64_t r0 = t * 64;
  const int rows = (int)min((int64_t)64, N - r0);
  const __nv_bfloat16* src = v + (bh * N + r0) * 128 + c;
  float x[64];
  float am = 0.f;
#pragma unroll
  for (int r = 0; r < 64; ++r) {
    x[r] = r < rows ? __bfloat162float(src[(int64_t)r * 128]) : 0.f;
    am = fmaxf(am, fabsf(x[r]));
  }
  const float inv = div_full(448.0f, fmaxf(am, 1e-12f));
  v_desc[(bh * ntiles + t) * 128 + c] = div_full(am, 448.0f);
  uint8_t* dst = v_codes + (bh * N + r0) * 128 + c;
#pragma unroll
  for (int r = 0; r < 64; ++r)
    if (r < rows) dst[(int64_t)r * 128] = (uint8_t)(f32x2_to_e4m3x2(__fmul_rn(x[r], inv), 0.f) & 0xFF);
}
}  // namespace fd

extern "C" int fd_attn_quant_v_tile(const void* v, int64_t BH, int64_t N, void* v_codes, float* v_desc,
                                    void* stream) {
  FD_CHECK_ARG(BH > 0 && N > 0 && BH <= 65535 && N < (1ll << 30), "bad shape");
  FD_CHECK_ARG(v && v_codes && v_desc, "null pointer");
  const int64_t ntiles = (N + 63) / 64;
  v_tile_quant_kernel<<<dim3((unsigned)ntiles, (unsigned)BH), 128, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)v, N, (uint8_t*)v_codes, v_desc);
  return check_launch("attn_quant_v_tile");
}

// ---------------------------------------------------------------------------
// fd_attn_quant_noalloc: fd_attn_quant with its scratch in g_attn_quant_ws.
//
// For callers that cannot allocate device memory themselves -- hosts that hand
// this library only their input and output buffers (a serving process that
// carves all device memory from one arena planned at start-up, or a foreign
// runtime calling through the C ABI with no allocator of its own), and code
// paths where cudaMalloc's implicit synchronisation is not allowed.
//
// The host cannot use the array's name as a device address, so the address is
// looked up with cudaGetSymbolAddress, with the device current, on the first
// call made in a CUDA context (the device's primary context, as torch and most
// runtimes use, or a context the caller made current), and kept for that
// context; make that first call before any stream capture.  The colstats
// launch writes every scratch element the quantisation launch reads, so
// nothing needs clearing between calls; but all calls in a context share the
// one array, so calls that overlap on the GPU (different streams, or different
// host threads, on one device) race on it.
static std::mutex g_ws_mutex;
struct WsSlot {
  CUcontext ctx;
  float* addr;
};
static WsSlot g_ws_slots[64][4] = {};  // per device: the last four contexts seen
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);  // cuCtxGetCurrent, through the runtime
static CtxGetCurrentFn g_ctx_current = nullptr;

static int noalloc_ws(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "fd_attn_quant_noalloc: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(FD_ERR_ARG, "fd_attn_quant_noalloc: device index %d unsupported", dev);
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  if (!g_ctx_current) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 4000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return set_error(FD_ERR_CUDA, "fd_attn_quant_noalloc: cuCtxGetCurrent unavailable");
    g_ctx_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  CUcontext ctx = nullptr;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS)
    return set_error(FD_ERR_CUDA, "fd_attn_quant_noalloc: cuCtxGetCurrent failed");
  WsSlot* slots = g_ws_slots[dev];
  for (int i = 0; ctx != nullptr && i < 4; ++i) {
    if (slots[i].ctx == ctx && slots[i].addr) {
      *out = slots[i].addr;
      return FD_OK;
    }
  }
  // first call in this context (with no context current yet, the runtime makes
  // the device's primary context current here, and the launches use it too)
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_attn_quant_ws);
  if (e != cudaSuccess || p == nullptr)
    return set_error(FD_ERR_CUDA, "fd_attn_quant_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
  if (ctx == nullptr && (g_ctx_current(&ctx) != CUDA_SUCCESS || ctx == nullptr))
    return set_error(FD_ERR_CUDA, "fd_attn_quant_noalloc: no current CUDA context");
  // newest first; the oldest of four contexts is forgotten (looked up again if it returns)
  for (int i = 3; i > 0; --i) slots[i] = slots[i - 1];
  slots[0] = WsSlot{ctx, static_cast<float*>(p)};
  *out = slots[0].addr;
  return FD_OK;
}

extern "C" int64_t fd_attn_quant_noalloc_max_floats(void) { return kNoAllocWsFloats; }

extern "C" int fd_attn_quant_noalloc(const void* q, const void* k, const void* v, int64_t BH,
                                     int64_t N, int smooth_k, int qk_kind, int q_gran, int k_gran,
                                     int pv_kind, float sm_scale_log2e, void* q_codes,
                                     float* q_desc, void* k_codes, float* k_desc, void* v_codes,
                                     float* v_desc, float* k_mean, void* stream) {
  FD_CHECK_ARG(BH > 0 && N > 0, "empty input");
  FD_CHECK_ARG(BH <= 65535 && N < (1ll << 30), "BH or N too large");
  const int64_t need = fd_attn_quant_workspace_floats(BH, N);
  if (need > kNoAllocWsFloats)
    return set_error(FD_ERR_ARG,
                     "fd_attn_quant_noalloc: BH=%lld, N=%lld needs %lld scratch floats, above the "
                     "built-in maximum of %lld (2 * BH * ceil(N / 256) * 128 must not exceed it); "
                     "use fd_attn_quant with a caller-provided workspace",
                     (long long)BH, (long long)N, (long long)need, (long long)kNoAllocWsFloats);
  float* ws = nullptr;
  const int rc = noalloc_ws(&ws);
  if (rc) return rc;
  return fd_attn_quant(q, k, v, BH, N, smooth_k, qk_kind, q_gran, k_gran, pv_kind, sm_scale_log2e,
                       q_codes, q_desc, k_codes, k_desc, v_codes, v_desc, k_mean, ws, stream);
}

// ---------------------------------------------------------------------------
// Fused P3 + prologue: fd_qkv_postprocess_quant once per stream, then
// fd_attn_quant_kv once.  Workspace: fd_qkv_quant_workspace_floats(BH, N) floats.
extern "C" int64_t fd_qkv_quant_workspace_floats(int64_t BH, int64_t N) { return 2 * BH * ((N + 127) / 128) * 128; }

extern "C" int fd_qkv_postprocess_quant(const void* qkv, const float* qw, const float* kw, const float* freqs,
                                        int64_t B, int64_t S, int64_t H, float eps, int64_t N, int64_t s_off,
                                        int qk_kind, int q_gran, int pv_kind, float sm_scale_log2e,
                                        void* q_codes, float* q_desc, void* k_out, void* v_out,
                                        float* workspace, void* stream) {
  FD_CHECK_ARG(B > 0 && S > 0 && H > 0 && B <= 65535 && H <= 65535, "bad shape");
  FD_CHECK_ARG(s_off >= 0 && s_off % 128 == 0 && s_off + S <= N, "s_off must be a multiple of 128 inside N");
  FD_CHECK_ARG(S % 128 == 0 || s_off + S == N, "only the last stream may end mid-block");
  FD_CHECK_ARG(qk_kind == FD_QK_INT8 || qk_kind == FD_QK_FP8, "bad qk_kind");
  FD_CHECK_ARG(q_gran == FD_GRAN_TOKEN || q_gran == FD_GRAN_BLOCK, "bad q_gran");
  FD_CHECK_ARG(qkv && qw && kw && freqs && q_codes && q_desc && k_out && v_out && workspace, "null pointer");
  FD_CHECK_ARG(aligned8(qkv) && aligned16(qw) && aligned16(kw) && aligned16(freqs) && aligned8(k_out) &&
                   aligned8(v_out) && (reinterpret_cast<uintptr_t>(q_codes) & 3) == 0,
               "misaligned pointer");
  const int nchunks = (int)((N + 127) / 128);
  float* ws_sum = workspace;
  float* ws_amax = workspace + B * H * nchunks * 128;
  const int64_t qs = fd_desc_stride(N, q_gran, 128);
  dim3 grid((unsigned)((S + 127) / 128), (unsigned)H, (unsigned)B);
  cudaStream_t st = (cudaStream_t)stream;
  const int do_v = pv_kind == FD_PV_FP8;
#define FD_QQ(QK)                                                                                         \
  qkv_quant_kernel<QK><<<grid, 256, 0, st>>>((const __nv_bfloat16*)qkv, qw, kw, freqs, S, (int)H, eps, N, \
                                             s_off, q_gran, sm_scale_log2e, (uint8_t*)q_codes, q_desc, qs, \
                                             (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out, ws_sum, ws_amax,  \
                                             nchunks, do_v)
  if (qk_kind == FD_QK_INT8) FD_QQ(FD_QK_INT8);
  else FD_QQ(FD_QK_FP8);
#undef FD_QQ
  return check_launch("qkv_postprocess_quant");
}

extern "C" int fd_attn_quant_kv(const void* k, const void* v, int64_t BH, int64_t N, int smooth_k, int qk_kind,
                                int k_gran, int pv_kind, void* k_codes, float* k_desc, void* v_codes,
                                float* v_desc, float* k_mean, float* workspace, void* stream) {
  FD_CHECK_ARG(BH > 0 && N > 0 && BH <= 65535, "bad shape");
  FD_CHECK_ARG(qk_kind == FD_QK_INT8 || qk_kind == FD_QK_FP8, "bad qk_kind");
  FD_CHECK_ARG(k_gran == FD_GRAN_TOKEN || k_gran == FD_GRAN_BLOCK, "bad granularity");
  FD_CHECK_ARG(pv_kind == FD_PV_BF16 || pv_kind == FD_PV_FP8, "bad pv_kind");
  FD_CHECK_ARG(k && k_codes && k_desc && workspace, "null pointer");
  FD_CHECK_ARG(pv_kind == FD_PV_BF16 || (v && v_codes && v_desc), "null V pointer");
  FD_CHECK_ARG(aligned16(k) && (v == nullptr || aligned16(v)) && aligned8(k_codes) &&
                   (v_codes == nullptr || aligned8(v_codes)),
               "misaligned pointer");
  const int nchunks = (int)((N + 127) / 128);
  float* ws_sum = workspace;
  float* ws_amax = workspace + BH * nchunks * 128;
  const int pv_fp8 = pv_kind == FD_PV_FP8;
  cudaStream_t st = (cudaStream_t)stream;
  if (smooth_k || pv_fp8) {
    colstats_final_kernel<<<(unsigned)BH, 128, 0, st>>>(ws_sum, ws_amax, N, nchunks, smooth_k, pv_fp8, k_mean,
                                                        v_desc);
    const int rc = check_launch("attn_quant_kv final");
    if (rc) return rc;
  }
  const int64_t ks = fd_desc_stride(N, k_gran, 64);
  dim3 grid((unsigned)((N + 127) / 128), (unsigned)BH, pv_fp8 ? 2u : 1u);
#define FD_KV(QK)                                                                                         \
  quant_kernel<QK, true><<<grid, 256, 0, st>>>(nullptr, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, N, \
                                         nchunks, smooth_k, FD_GRAN_TOKEN, k_gran, pv_fp8, 1.0f, nullptr, \
                                         nullptr, (uint8_t*)k_codes, k_desc, (uint8_t*)v_codes, v_desc,   \
                                         k_mean, ws_sum, ws_amax, 0, ks, 1)
  if (qk_kind == FD_QK_INT8) FD_KV(FD_QK_INT8);
  else FD_KV(FD_QK_FP8);
#undef FD_KV
  return check_launch("attn_quant_kv");
}
