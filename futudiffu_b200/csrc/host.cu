// Host plumbing of the C ABI: error strings, device status word, tensor-map
// encoding through the driver entry point.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "fd_common.cuh"
#include "fd_host.h"

namespace fd {

__device__ unsigned int g_status = 0;

static thread_local char t_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return FD_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error(FD_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dt, (cuuint32_t)rank, const_cast<void*>(base),
                        reinterpret_cast<const cuuint64_t*>(dims),
                        reinterpret_cast<const cuuint64_t*>(strides_bytes),
                        reinterpret_cast<const cuuint32_t*>(box), estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FD_OK;
}

__global__ void div_full_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = div_full(a[i], b[i]);
}

}  // namespace fd

extern "C" int fd_div_full_f32(const float* a, const float* b, float* out, int64_t n, void* stream) {
  FD_CHECK_ARG(n >= 0, "negative size");
  if (n == 0) return FD_OK;
  FD_CHECK_ARG(a && b && out, "null pointer");
  int64_t grid = (n + 255) / 256;
  if (grid > 4096) grid = 4096;
  fd::div_full_kernel<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>(a, b, out, n);
  return fd::check_launch("div_full");
}

extern "C" const char* fd_version(void) { return "futudiffu_b200 0.1 sm_100a"; }

extern "C" const char* fd_last_error(void) { return fd::t_err; }

extern "C" int fd_get_status(unsigned int* out, int clear) {
  if (!out) return fd::set_error(FD_ERR_ARG, "fd_get_status: null pointer");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fd::set_error(FD_ERR_CUDA, "fd_get_status: %s", cudaGetErrorString(e));
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, fd::g_status, sizeof(v));
  if (e != cudaSuccess) return fd::set_error(FD_ERR_CUDA, "fd_get_status: %s", cudaGetErrorString(e));
  if (clear) {
    unsigned int z = 0;
    e = cudaMemcpyToSymbol(fd::g_status, &z, sizeof(z));
    if (e != cudaSuccess) return fd::set_error(FD_ERR_CUDA, "fd_get_status: %s", cudaGetErrorString(e));
  }
  unsigned int g = 0;
  const int rc = fd::gemm_status(&g, clear);
  if (rc) return rc;
  *out = v | g;
  return FD_OK;
}
