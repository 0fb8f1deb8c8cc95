// Host-side helpers shared by the C-ABI entry points.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/aios_b200.h"

namespace aiosb {

// Records an error message for aiosb_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
// Turns a failed kernel launch into AIOSB_ERR_LAUNCH.
int check_launch(const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device).
int sm_count();

// Launches `kernel` with programmatic dependent launch enabled, so it may start
// while the previous kernel on the stream drains. Every kernel launched this way
// executes griddepcontrol.wait in every block before it touches memory that an
// earlier kernel writes or reads, and before any early return, so completion
// stays transitive along the stream.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace aiosb

#define AIOSB_REQUIRE(cond, code, ...) \
  do {                                                   \
    if (!(cond)) return ::aiosb::set_error(code, __VA_ARGS__); \
  } while (0)
