// Host-side helpers shared by the C-ABI entry points: error reporting,
// argument checks, SM count, TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fd_b200.h"

namespace fd {

// Records a thread-local message retrievable through fd_last_error().
int set_error(int code, const char* fmt, ...);

// Returns FD_OK, or FD_ERR_CUDA with the message of the last launch error.
int check_launch(const char* what);

// Streaming multiprocessor count of the current device (cached per device).
int num_sms();

// cuTensorMapEncodeTiled obtained through the runtime's driver entry point,
// so the library links no libcuda stub.
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

// Status word of the FP8 GEMM's translation unit (compiled as a whole program,
// see fd_common.cuh): reads it into *out and clears it when `clear` is set.
int gemm_status(unsigned int* out, int clear);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }
inline bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; }

}  // namespace fd

#define FD_CHECK_ARG(cond, msg)                                         \
  do {                                                                  \
    if (!(cond)) return ::fd::set_error(FD_ERR_ARG, "%s: %s", __func__, msg); \
  } while (0)
