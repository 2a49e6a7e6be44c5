// TMEM -> register load throughput microbenchmark (tcgen05.ld.sync.aligned.32x32b).
//
// The FP8 block GEMM promotes every 128-K slice of its fp32 accumulator from
// TMEM into registers (acc += partial * scale), which needs 256 B/clk/SM of
// TMEM reads at the full FP8 MMA rate.  This probe measures what tcgen05.ld
// delivers: each CTA (one per SM) allocates all 512 TMEM columns; `warps` warps
// read them (warp w reads its TMEM lane quadrant w & 3 and a column window
// chosen by w >> 2) with `width`-column loads, `per_wait` loads issued before each
// tcgen05.wait::ld, over a 128-column window per warp, `iters` times.  With `fma` set, every loaded value is also
// accumulated into a 128-register row as the GEMM's promotion does
// (acc[i] = fma(v, s, acc[i])).  Each warp records its clock64 cycle count.
//
// Launch: grid = number of SMs, 160 KiB of dynamic shared memory so that one CTA
// holds each SM (its TMEM allocation never waits on another CTA's).
#include "fd_common.cuh"
#include "fd_host.h"

namespace fd {
namespace probe {

constexpr int MAX_WARPS = 12;  // pure-load runs (170 registers a thread: no spills at 128 columns per wait)

template <int W>
FD_DEV void ld_w(uint32_t a, uint32_t* r);
template <>
FD_DEV void ld_w<16>(uint32_t a, uint32_t* r) { tmem_ld16(a, *reinterpret_cast<uint32_t(*)[16]>(r)); }
template <>
FD_DEV void ld_w<32>(uint32_t a, uint32_t* r) { tmem_ld32(a, *reinterpret_cast<uint32_t(*)[32]>(r)); }
template <>
FD_DEV void ld_w<64>(uint32_t a, uint32_t* r) { tmem_ld64(a, *reinterpret_cast<uint32_t(*)[64]>(r)); }

// W columns per load, L loads per wait, FMA: accumulate as the promotion does.
// One round = 128 columns of a row (128 / (W L) waits); `iters` rounds.
template <int W, int L, bool FMA>
__global__ void __launch_bounds__(FMA ? 320 : MAX_WARPS * 32, 1)
    tmem_ld_kernel(int warps, int iters, long long* cycles, float* sink) {
  __shared__ uint32_t slot;
  const int warp = warp_id(), lane = lane_id();
  if (warp == 0) {
    tmem_alloc(&slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t base = slot;
  if (warp < warps) {
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    constexpr int SPAN = W * L;                  // columns per wait
    constexpr int WAITS = SPAN >= 128 ? 1 : 128 / SPAN;
    const uint32_t col0 = (uint32_t)(((warp >> 2) * 128) % 512);  // this warp's 128-column window
    uint32_t r[SPAN];
    float acc[FMA ? 128 : 1];
#pragma unroll
    for (int i = 0; i < (FMA ? 128 : 1); ++i) acc[i] = 0.f;
    float chk = 0.f;
    const float s = 1.0f + 1e-7f * lane;
    __syncwarp();
    const long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int w = 0; w < WAITS; ++w) {
#pragma unroll
        for (int l = 0; l < L; ++l) ld_w<W>(base + lane_base + ((col0 + w * SPAN + l * W) % 512), r + l * W);
        tmem_wait_ld();
        if constexpr (FMA) {
#pragma unroll
          for (int i = 0; i < SPAN; ++i) acc[(w * SPAN + i) & 127] = fmaf(__uint_as_float(r[i]), s, acc[(w * SPAN + i) & 127]);
        } else {
          chk += __uint_as_float(r[0]) + __uint_as_float(r[SPAN - 1]);
        }
      }
    }
    const long long t1 = clock64();
    if (FMA) {
#pragma unroll
      for (int i = 0; i < 128; ++i) chk += acc[i];
    }
    if (lane == 0) cycles[(int64_t)blockIdx.x * MAX_WARPS + warp] = t1 - t0;
    if (chk == 12345.678f) sink[0] = chk;  // keeps the loads' results live
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(base, 512);
}

}  // namespace probe
}  // namespace fd

using namespace fd;

extern "C" int fd_probe_tmem_ld(int width, int per_wait, int warps, int fma, int iters, long long* cycles,
                                float* sink, void* stream) {
  FD_CHECK_ARG(warps >= 1 && warps <= (fma ? 10 : probe::MAX_WARPS) && iters >= 1 && iters <= (1 << 20),
               "bad warps / iters");
  FD_CHECK_ARG(cycles && sink, "null pointer");
  FD_CHECK_ARG(width * per_wait <= 64 || (!fma && width * per_wait <= 128), "too many columns per wait");
  const size_t smem = 160 * 1024;  // one CTA per SM
  cudaStream_t st = (cudaStream_t)stream;
  const int grid = num_sms();
#define FD_PROBE(W, L, F)                                                                                    \
  do {                                                                                                       \
    auto k = probe::tmem_ld_kernel<W, L, F>;                                                                 \
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);         \
    if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "probe smem attribute: %s", cudaGetErrorString(e)); \
    k<<<grid, F ? 320 : probe::MAX_WARPS * 32, smem, st>>>(warps, iters, cycles, sink);                      \
    return check_launch("probe_tmem_ld");                                                                    \
  } while (0)
  const bool f = fma != 0;
  if (width == 16 && per_wait == 1) { if (f) FD_PROBE(16, 1, true); else FD_PROBE(16, 1, false); }
  if (width == 16 && per_wait == 2) { if (f) FD_PROBE(16, 2, true); else FD_PROBE(16, 2, false); }
  if (width == 16 && per_wait == 4) { if (f) FD_PROBE(16, 4, true); else FD_PROBE(16, 4, false); }
  if (width == 32 && per_wait == 1) { if (f) FD_PROBE(32, 1, true); else FD_PROBE(32, 1, false); }
  if (width == 32 && per_wait == 2) { if (f) FD_PROBE(32, 2, true); else FD_PROBE(32, 2, false); }
  if (width == 64 && per_wait == 1) { if (f) FD_PROBE(64, 1, true); else FD_PROBE(64, 1, false); }
  if (width == 32 && per_wait == 4 && !f) FD_PROBE(32, 4, false);
  if (width == 64 && per_wait == 2 && !f) FD_PROBE(64, 2, false);
#undef FD_PROBE
  return set_error(FD_ERR_ARG, "unsupported width / per_wait");
}
