// Host-side helpers shared by the C ABI translation units: thread-local error
// text, CUDA error checks, device properties and TMA tensor-map encoding.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/stageml_b200.h"

namespace sb {

// Record an error message for stageml_last_error() and return `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();
const char* last_error_text();

// Count one kernel launch made by this library (reported by stageml_launch_count).
void count_launch();

// Multiprocessor count of the current device (cached per device).
int sm_count();

// Encode a 2-D row-major tensor map: `rows` x `cols` elements of `elem_bytes`
// bytes, row pitch `row_pitch_bytes`, box `box_rows` x `box_cols`, with a
// `swizzle_bytes`-byte swizzle (0, 32, 64 or 128; the box row must then be
// exactly that many bytes).
int make_tmap_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_pitch_bytes, uint32_t box_rows, uint32_t box_cols, int swizzle_bytes);

// Encode a 3-D tensor map: dims {d0 (contiguous), d1, d2} elements, byte strides
// s1 (between consecutive d1 indices) and s2 (d2), box {b0, b1, b2}. The strides
// may overlap (e.g. d2 stepping inside a d1 row): the caller keeps every
// coordinate it loads inside dims so that each address stays in the allocation.
int make_tmap_3d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                 uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                 int swizzle_bytes);

// Programmatic dependent launch (PDL) of the decode-sized layer's kernel chain:
// on by default, STAGEML_PDL=0 turns it off.
bool pdl_enabled();

// Launch `kernel` on `stream`. With `pdl` it is a programmatic dependent launch:
// its CTAs may start while the previous kernel in the stream is still running, so
// the kernel must call pdl_wait() (common.cuh) before it reads anything that
// kernel writes. Without `pdl` it is an ordinary launch.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

}  // namespace sb

#define SB_CUDA_CHECK(expr)                                                                     \
  do {                                                                                          \
    cudaError_t _e = (expr);                                                                    \
    if (_e != cudaSuccess)                                                                      \
      return ::sb::set_error(STAGEML_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                             __FILE__, __LINE__);                                               \
  } while (0)

#define SB_CHECK_ARG(cond, ...)                                    \
  do {                                                             \
    if (!(cond)) return ::sb::set_error(STAGEML_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

#define SB_TRY(expr)            \
  do {                          \
    int _rc = (expr);           \
    if (_rc != STAGEML_OK) return _rc; \
  } while (0)
