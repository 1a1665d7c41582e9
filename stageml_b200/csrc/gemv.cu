// Single LoRA linear in fp32 with the [in,out] layout of the config-1 workload
// (benchmarks/triton_lora_equivalence_check.py:11-22):
//   dynamic: y = x W + s (x A) B        folded: y = x W'
// x [M, in] with M <= 16, W [in, out], A [in, r], B [r, out]. Real fp32 FMAs
// (no TF32). HBM-bound on the W read: split-K over (column block, K slice)
// CTAs with float4 loads of W, fp32 partials reduced in a fixed order by a
// second kernel that also applies the rank-r expansion, so results are
// deterministic.
#include <mutex>

#include "common.cuh"
#include "host_util.h"
#include "kernels.h"
#include "stage_timer.h"

namespace sb {
namespace {

constexpr int GV_COLS = 512;   // columns per CTA (128 threads x float4)
constexpr int GV_MAXM = 16;

__global__ void __launch_bounds__(128) gemv_partial_kernel(const float* __restrict__ x, const float* __restrict__ W,
                                                           const float* __restrict__ A, int M, int in_f, int out_f,
                                                           int rank, int slice, float* __restrict__ part,
                                                           float* __restrict__ xa_part) {
  extern __shared__ float xs[];  // [M][slice]
  const int ks = blockIdx.y;
  const int i0 = ks * slice, i1 = min(in_f, i0 + slice);
  const int ni = i1 - i0;
  for (int t = threadIdx.x; t < M * slice; t += blockDim.x) {
    const int m = t / slice, i = t % slice;
    xs[t] = (i < ni) ? x[(int64_t)m * in_f + i0 + i] : 0.f;
  }
  __syncthreads();
  const int c = blockIdx.x * GV_COLS + threadIdx.x * 4;
  if (c < out_f) {
    float acc[GV_MAXM][4];
#pragma unroll
    for (int m = 0; m < GV_MAXM; ++m)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[m][q] = 0.f;
    const bool vec = (c + 4 <= out_f) && (out_f % 4 == 0);
    for (int i = 0; i < ni; ++i) {
      float w[4];
      const float* wr = W + (int64_t)(i0 + i) * out_f + c;
      if (vec) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(wr));
        w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) w[q] = (c + q < out_f) ? wr[q] : 0.f;
      }
#pragma unroll
      for (int m = 0; m < GV_MAXM; ++m)
        if (m < M) {
          const float xv = xs[m * slice + i];
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[m][q] = fmaf(xv, w[q], acc[m][q]);
        }
    }
#pragma unroll
    for (int m = 0; m < GV_MAXM; ++m)
      if (m < M)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (c + q < out_f) part[((int64_t)ks * M + m) * out_f + c + q] = acc[m][q];
  }
  if (A && blockIdx.x == 0) {
    for (int t = threadIdx.x; t < M * rank; t += blockDim.x) {
      const int m = t / rank, j = t % rank;
      float a = 0.f;
      for (int i = 0; i < ni; ++i) a = fmaf(xs[m * slice + i], A[(int64_t)(i0 + i) * rank + j], a);
      xa_part[((int64_t)ks * M + m) * rank + j] = a;
    }
  }
}

__global__ void gemv_reduce_kernel(const float* __restrict__ part, const float* __restrict__ xa_part,
                                   const float* __restrict__ B, float scale, int M, int out_f, int rank, int KS,
                                   float* __restrict__ y) {
  extern __shared__ float xa[];  // [M][rank]
  if (B) {
    for (int t = threadIdx.x; t < M * rank; t += blockDim.x) {
      float a = 0.f;
      for (int ks = 0; ks < KS; ++ks) a += xa_part[(int64_t)ks * M * rank + t];
      xa[t] = a;
    }
  }
  __syncthreads();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= out_f) return;
  for (int m = 0; m < M; ++m) {
    float v = 0.f;
    for (int ks = 0; ks < KS; ++ks) v += part[((int64_t)ks * M + m) * out_f + n];
    if (B) {
      float l = 0.f;
      for (int j = 0; j < rank; ++j) l = fmaf(xa[m * rank + j], B[(int64_t)j * out_f + n], l);
      v = fmaf(scale, l, v);
    }
    y[(int64_t)m * out_f + n] = v;
  }
}

void gemv_plan(int in_f, int out_f, int* KS, int* slice) {
  const int ncb = (out_f + GV_COLS - 1) / GV_COLS;
  int ks = std::max(1, (8 * sm_count() + ncb - 1) / ncb);
  ks = std::min(ks, std::max(1, (in_f + 31) / 32));
  *slice = (in_f + ks - 1) / ks;
  *KS = (in_f + *slice - 1) / *slice;
}

}  // namespace

size_t gemv_f32_workspace(int M, int in_f, int out_f, int rank) {
  int KS, slice;
  gemv_plan(in_f, out_f, &KS, &slice);
  size_t b = (((size_t)KS * M * out_f * 4) + 255) & ~size_t(255);
  b += (((size_t)KS * M * std::max(rank, 1) * 4) + 255) & ~size_t(255);
  return b;
}

int launch_gemv_f32(const float* x, const float* W, const float* A, const float* B, float scale, int M, int in_f,
                    int out_f, int rank, float* y, void* ws, cudaStream_t stream) {
  SB_CHECK_ARG(x && W && y, "lora_gemv_f32: null pointer");
  SB_CHECK_ARG(M >= 1 && M <= GV_MAXM, "lora_gemv_f32: M=%d must be in [1, %d]", M, GV_MAXM);
  SB_CHECK_ARG(in_f >= 1 && out_f >= 1, "lora_gemv_f32: bad sizes");
  SB_CHECK_ARG(!A || (B && rank >= 1 && rank <= 256), "lora_gemv_f32: A needs B and 1 <= rank <= 256");
  SB_CHECK_ARG(ws, "lora_gemv_f32: null workspace");
  SB_CHECK_ARG(reinterpret_cast<uintptr_t>(W) % 16 == 0, "lora_gemv_f32: W must be 16-byte aligned");
  int KS, slice;
  gemv_plan(in_f, out_f, &KS, &slice);
  float* part = static_cast<float*>(ws);
  float* xa_part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) +
                                            ((((size_t)KS * M * out_f * 4) + 255) & ~size_t(255)));
  const size_t smem1 = (size_t)M * slice * 4;
  SB_CHECK_ARG(smem1 <= 200 * 1024, "lora_gemv_f32: K slice too large");
  SB_CUDA_CHECK(cudaFuncSetAttribute(gemv_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1));
  dim3 g1((out_f + GV_COLS - 1) / GV_COLS, KS);
  (gemv_partial_kernel<<<g1, 128, smem1, stream>>>(x, W, A, M, in_f, out_f, A ? rank : 0, slice, part, xa_part), ::sb::count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  const size_t smem2 = (size_t)M * (A ? rank : 1) * 4;
  (gemv_reduce_kernel<<<(out_f + 255) / 256, 256, smem2, stream>>>(part, xa_part, A ? B : nullptr, scale, M, out_f,
                                                                   A ? rank : 0, KS, y), ::sb::count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

}  // namespace sb

// ---------------------------------------------------------------------------
// Allocation-free variant of the fp32 single-LoRA GEMV.
//
// stageml_lora_gemv_f32 keeps its split-K partial sums in a workspace the
// caller allocates. Some callers cannot allocate device memory where they run
// this layer: a plugin reached only through the C ABI with no allocator of its
// own, an inference loop that must never call cudaMalloc/cudaFree (both can
// synchronize the device and stall concurrent work), or a host whose memory
// lives in a fixed, pre-planned arena. For them the partial sums go to the
// array below, which belongs to this library: a file-scope device array of
// kGemvNoAllocScratchBytes bytes, created when the library's code is loaded on
// a GPU and held on every GPU that loads it until the process exits.
namespace sb {
namespace {

constexpr size_t kGemvNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_gemv_noalloc_scratch[kGemvNoAllocScratchBytes];

std::mutex g_scratch_mu;
// Device address of the array per device ordinal, with the driver context it was
// taken in: a caller that makes a different context current on the device (a
// non-primary context, or the primary context recreated after cudaDeviceReset)
// gets the array's address in that context, not a stale one.
struct ScratchAddr {
  void* ctx = nullptr;
  void* addr = nullptr;
};
ScratchAddr g_scratch_addr[64];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The current driver context (null when the driver entry point is unavailable).
void* current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext c = nullptr;
  if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}

// Device address of the scratch array on the current device. Host code cannot
// use the array's name as a device pointer, so the address is queried with the
// device current, once per device and driver context, and cached.
int gemv_noalloc_scratch(void** out) {
  int dev = 0;
  SB_CUDA_CHECK(cudaGetDevice(&dev));
  SB_CHECK_ARG(dev >= 0 && dev < 64, "lora_gemv_f32_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  void* ctx = current_context();
  ScratchAddr& c = g_scratch_addr[dev];
  if (!c.addr || c.ctx != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(STAGEML_ERR_CUDA, "lora_gemv_f32_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                       cudaGetErrorString(e));
    c.addr = p;
    c.ctx = ctx;
  }
  *out = c.addr;
  return STAGEML_OK;
}

}  // namespace
}  // namespace sb

extern "C" int stageml_lora_gemv_f32_noalloc(const float* x, const float* W, const float* A, const float* B,
                                             float scale, int M, int in_features, int out_features, int rank, float* y,
                                             stageml_stream_t stream) {
  using namespace sb;
  clear_error();
  SB_CHECK_ARG(M >= 1 && in_features >= 1 && out_features >= 1, "lora_gemv_f32_noalloc: bad sizes");
  const size_t need = gemv_f32_workspace(M, in_features, out_features, A ? rank : 0);
  if (need > kGemvNoAllocScratchBytes)
    return set_error(STAGEML_ERR_INVALID_ARG,
                     "lora_gemv_f32_noalloc: M=%d in=%d out=%d rank=%d needs %zu bytes of scratch, more than the "
                     "%zu-byte static scratch; call stageml_lora_gemv_f32 with a workspace instead",
                     M, in_features, out_features, rank, need, kGemvNoAllocScratchBytes);
  void* scratch = nullptr;
  SB_TRY(gemv_noalloc_scratch(&scratch));
  // Every partial sum is written before it is read, so nothing in the scratch needs clearing.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  StageScope scope(STAGEML_STAGE_GEMV, st);
  return launch_gemv_f32(x, W, A, B, scale, M, in_features, out_features, rank, y, scratch, st);
}
