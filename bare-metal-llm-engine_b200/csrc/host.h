// host.h -- the host half of the library's shared machinery: the C-ABI error
// convention (status codes plus a thread-local message, mirroring the
// reference's ENGINE_CHECK / CUDA_CHECK / CUDA_CHECK_KERNEL in
// include/engine/check.hpp:36-107), device property caches, the driver entry
// point for TMA tensor-map encoding and the PDL launch helper.  Plain C++ (the
// host-only sources include it directly); common.cuh adds the device half.
#pragma once

#include <cuda.h>  // CUtensorMap and enums only; libcuda is reached via cudaGetDriverEntryPoint
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>

#include "engine_b200.h"  // include/ is on the compiler include path (build.py)

namespace b200 {

// ------------------------------------------------------------------ host side

/// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
/// Records a CUDA runtime error with its name and string, returns ENGINE_ERR_CUDA.
int set_cuda_error(cudaError_t err, const char* what);

/// Post-launch check: launch errors always; with ENGINE_ALWAYS_SYNC_CHECK=1 in the
/// environment it also synchronises the device and surfaces execution faults and
/// device-side wait timeouts (the reference's debug-build CUDA_CHECK_KERNEL).
int check_launch(const char* what);

bool always_sync_check();
int sm_count();            // current device
int max_smem_optin();      // current device, bytes
/// Device error word of the current device (timeouts set bits here).
unsigned int* device_error_word();
/// Wait limit for every bounded device-side spin, in nanoseconds.
unsigned long long wait_limit_ns();

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

/// Programmatic dependent launch is on unless ENGINE_PDL=0.
bool pdl_enabled();

/// Launches `kern` with programmatic stream serialization (PDL): the kernel may
/// start while its predecessor on the stream finishes, runs its set-up, and
/// waits in griddepcontrol.wait before touching any input.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

/// 2-D row-major tensor map: `rows` x `cols` elements of `elem_bytes`, row pitch
/// `ld` elements, box `box_rows` x `box_cols`, 128-byte swizzle.  Cached per
/// (pointer, shape, box); returns false (with the error recorded) on failure.
bool make_tmap_2d(CUtensorMap* out, const void* ptr, CUtensorMapDataType dtype, int elem_bytes,
                  uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                  uint32_t box_cols);

/// 3-D tensor map (dims innermost first, element strides of dims 1 and 2 in
/// elements), box `box` (innermost first), 128-byte swizzle, zero fill out of
/// bounds.  Not cached.  Returns false (with the error recorded) on failure.
bool make_tmap_3d(CUtensorMap* out, const void* ptr, CUtensorMapDataType dtype, int elem_bytes,
                  const uint64_t (&dims)[3], const uint64_t (&strides)[2],
                  const uint32_t (&box)[3]);

}  // namespace b200

#define B200_REQUIRE(cond, msg)                                      \
  do {                                                               \
    if (!(cond)) return ::b200::set_error(ENGINE_ERR_INVALID, (msg)); \
  } while (0)

#define B200_CUDA(call)                                           \
  do {                                                            \
    cudaError_t b200_e_ = (call);                                 \
    if (b200_e_ != cudaSuccess) return ::b200::set_cuda_error(b200_e_, #call); \
  } while (0)

#define B200_ENTRY_BEGIN try {
#define B200_ENTRY_END                                                     \
  }                                                                        \
  catch (const std::exception& e) {                                        \
    return ::b200::set_error(ENGINE_ERR_INTERNAL, e.what());              \
  }                                                                        \
  catch (...) {                                                            \
    return ::b200::set_error(ENGINE_ERR_INTERNAL, "unknown C++ exception"); \
  }
