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
//   V e4m3 per channel src/futudiffu/sage_kernels.py:1146-1151 (here over the
//                      whole sequence instead of one 64-row tile)
#include <mutex>

#include "fd_common.cuh"
#include "fd_host.h"

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

template <int QK>  // FD_QK_INT8 or FD_QK_FP8
FD_DEV uint32_t quant_code(float x, float inv) {
  const float y = x * inv;
  if constexpr (QK == FD_QK_INT8) {
    // .to(tl.int8) truncates toward zero (|y| <= 127 by construction)
    return (uint32_t)(__float2int_rz(y) & 0xFF);
  } else {
    return f32x2_to_e4m3x2(y, 0.f) & 0xFF;
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
template <int QK>
__global__ void __launch_bounds__(256, 3) quant_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, int64_t N, int nchunks, int smooth_k, int q_gran,
    int k_gran, int pv_fp8, float sm_scale_log2e, uint8_t* __restrict__ q_codes,
    float* __restrict__ q_desc, uint8_t* __restrict__ k_codes, float* __restrict__ k_desc,
    uint8_t* __restrict__ v_codes, float* __restrict__ v_desc, float* __restrict__ k_mean,
    const float* __restrict__ ws_sum, const float* __restrict__ ws_amax, int64_t q_desc_stride,
    int64_t k_desc_stride) {
  const int blk = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int which = blockIdx.z;  // 0 Q, 1 K, 2 V
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
  if (which == 0) {
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
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t n = r0 + rl + 16 * i;
      if (n < N) {
        float x[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(v + (bh * N + n) * 128 + cg * 8)), x);
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
  quant_kernel<QK><<<grid, 256, 0, st>>>(                                                       \
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, N, nchunks,   \
      smooth_k, q_gran, k_gran, pv_fp8, sm_scale_log2e, (uint8_t*)q_codes, q_desc,              \
      (uint8_t*)k_codes, k_desc, (uint8_t*)v_codes, v_desc, k_mean, ws_sum, ws_amax, qs, ks)
  if (qk_kind == FD_QK_INT8) FD_Q_LAUNCH(FD_QK_INT8);
  else FD_Q_LAUNCH(FD_QK_FP8);
#undef FD_Q_LAUNCH
  return check_launch("attn_quant");
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
// looked up once per device with cudaGetSymbolAddress, with that device
// current, on the first call made on it; make that first call before any
// stream capture.  The colstats launch writes every scratch element the
// quantisation launch reads, so nothing needs clearing between calls; but all
// calls share the one array, so calls that overlap on the GPU (different
// streams, or different host threads, on one device) race on it.
static std::mutex g_ws_mutex;
static float* g_ws_addr[64] = {nullptr};

static int noalloc_ws(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "fd_attn_quant_noalloc: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(FD_ERR_ARG, "fd_attn_quant_noalloc: device index %d unsupported", dev);
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  if (!g_ws_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_quant_ws);
    if (e != cudaSuccess || p == nullptr)
      return set_error(FD_ERR_CUDA, "fd_attn_quant_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
    g_ws_addr[dev] = static_cast<float*>(p);
  }
  *out = g_ws_addr[dev];
  return FD_OK;
}

extern "C" int64_t fd_attn_quant_noalloc_max_floats(void) { return kNoAllocWsFloats; }

extern "C" int fd_attn_quant_noalloc(const void* q, const void* k, const void* v, int64_t BH,
                                     int64_t N, int smooth_k, int qk_kind, int q_gran, int k_gran,
                                     int pv_kind, float sm_scale_log2e, void* q_codes,
                                     float* q_desc, void* k_codes, float* k_desc, void* v_codes,
                                     float* v_desc, float* k_mean, void* stream) {
  FD_CHECK_ARG(BH > 0 && N > 0, "empty input");
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
