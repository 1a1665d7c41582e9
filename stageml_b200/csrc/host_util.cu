// Host-side helpers: thread-local error text, SM count, TMA tensor maps.
#include <atomic>
#include <mutex>
#include <string.h>

#include "host_util.h"

#include <cstdlib>

namespace sb {

static thread_local char g_last_error[1024] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = 0; }

const char* last_error_text() { return g_last_error; }

static std::atomic<unsigned long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace sb

extern "C" unsigned long long stageml_launch_count(void) { return sb::g_launches.load(std::memory_order_relaxed); }

namespace sb {

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("STAGEML_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_pitch_bytes, uint32_t box_rows, uint32_t box_cols, int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(STAGEML_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(STAGEML_ERR_INVALID_ARG, "TMA base address %p is not 16-byte aligned", base);
  if (row_pitch_bytes % 16 != 0)
    return set_error(STAGEML_ERR_INVALID_ARG, "TMA row pitch %llu is not a multiple of 16 bytes",
                     (unsigned long long)row_pitch_bytes);
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 0:
      sw = CU_TENSOR_MAP_SWIZZLE_NONE;
      break;
    case 32:
      sw = CU_TENSOR_MAP_SWIZZLE_32B;
      break;
    case 64:
      sw = CU_TENSOR_MAP_SWIZZLE_64B;
      break;
    case 128:
      sw = CU_TENSOR_MAP_SWIZZLE_128B;
      break;
    default:
      return set_error(STAGEML_ERR_INVALID_ARG, "unsupported TMA swizzle %d", swizzle_bytes);
  }
  if (swizzle_bytes && box_cols * (uint32_t)elem_bytes != (uint32_t)swizzle_bytes)
    return set_error(STAGEML_ERR_INVALID_ARG, "%dB swizzle needs a %d-byte box row", swizzle_bytes, swizzle_bytes);
  if (box_rows == 0 || box_rows > 256 || box_cols == 0 || box_cols > 256)
    return set_error(STAGEML_ERR_INVALID_ARG, "TMA box %ux%u out of range", box_rows, box_cols);
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(STAGEML_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu", (int)r,
                     (unsigned long long)rows, (unsigned long long)cols);
  return STAGEML_OK;
}

int make_tmap_3d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                 uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                 int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(STAGEML_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(STAGEML_ERR_INVALID_ARG, "TMA base address %p is not 16-byte aligned", base);
  if (s1 % 16 != 0 || s2 % 16 != 0)
    return set_error(STAGEML_ERR_INVALID_ARG, "TMA strides %llu, %llu are not multiples of 16 bytes",
                     (unsigned long long)s1, (unsigned long long)s2);
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 0:
      sw = CU_TENSOR_MAP_SWIZZLE_NONE;
      break;
    case 32:
      sw = CU_TENSOR_MAP_SWIZZLE_32B;
      break;
    case 64:
      sw = CU_TENSOR_MAP_SWIZZLE_64B;
      break;
    case 128:
      sw = CU_TENSOR_MAP_SWIZZLE_128B;
      break;
    default:
      return set_error(STAGEML_ERR_INVALID_ARG, "unsupported TMA swizzle %d", swizzle_bytes);
  }
  if (swizzle_bytes && b0 * (uint32_t)elem_bytes != (uint32_t)swizzle_bytes)
    return set_error(STAGEML_ERR_INVALID_ARG, "%dB swizzle needs a %d-byte box row", swizzle_bytes, swizzle_bytes);
  if (b0 == 0 || b0 > 256 || b1 == 0 || b1 > 256 || b2 == 0 || b2 > 256)
    return set_error(STAGEML_ERR_INVALID_ARG, "TMA box %ux%ux%u out of range", b0, b1, b2);
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(out, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(STAGEML_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d) dims=%llu,%llu,%llu", (int)r,
                     (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2);
  return STAGEML_OK;
}

}  // namespace sb
