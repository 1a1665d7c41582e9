// Single LoRA linear in fp32 with the [in,out] layout of the config-1 workload
// (benchmarks/triton_lora_equivalence_check.py:11-22):
//   dynamic: y = x W + s (x A) B        folded: y = x W'
// x [M, in] with M <= 16, W [in, out], A [in, r], B [r, out]. Real fp32 FMAs
// (no TF32). HBM-bound on the W read (4 B per element): split-K over
// (512-column block, K slice) CTAs of 128 column threads x G row groups; every
// thread issues RPT independent 16-byte streaming loads of W before its FMAs, so
// each SM keeps ~128 KB in flight; the row groups are summed in shared memory in
// a fixed order and one fp32 partial per (K slice, row, column) is written. A
// second kernel (a programmatic dependent launch) adds the partials in slice
// order and applies the rank-r expansion, so results are deterministic.
#include <mutex>

#include "common.cuh"
#include "host_util.h"
#include "kernels.h"
#include "stage_timer.h"

namespace sb {
namespace {

constexpr int GV_COLS = 512;   // columns per CTA (128 threads x float4)
constexpr int GV_MAXM = 16;

// MB: rows of x handled (>= M); G: row groups per CTA; RPT: W rows per thread per pass.
template <int MB, int G, int RPT>
__global__ void __launch_bounds__(128 * G) gemv_partial_kernel(const float* __restrict__ x, const float* __restrict__ W,
                                                               const float* __restrict__ A, int M, int in_f, int out_f,
                                                               int rank, int slice, float* __restrict__ part,
                                                               float* __restrict__ xa_part) {
  extern __shared__ float sm[];  // xs [MB][slice], then the row groups' sums [G][MB][GV_COLS]
  float* xs = sm;
  float* red = sm + MB * slice;
  pdl_trigger();  // the reduce kernel may be scheduled now; it waits for this grid before reading
  const int ks = blockIdx.y;
  const int i0 = ks * slice, i1 = min(in_f, i0 + slice);
  const int ni = i1 - i0;
  for (int t = threadIdx.x; t < MB * slice; t += blockDim.x) {
    const int m = t / slice, i = t % slice;
    xs[t] = (m < M && i < ni) ? x[(int64_t)m * in_f + i0 + i] : 0.f;
  }
  __syncthreads();
  const int ct = threadIdx.x & 127, g = threadIdx.x >> 7;
  const int c = blockIdx.x * GV_COLS + ct * 4;
  const bool vec = (c + 4 <= out_f) && (out_f % 4 == 0);
  float acc[MB][4];
#pragma unroll
  for (int m = 0; m < MB; ++m)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[m][q] = 0.f;
  if (c < out_f) {
    for (int base = g * RPT; base < ni; base += G * RPT) {
      float4 w[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) {  // all loads of the pass in flight before the first FMA
        const int i = base + r;
        const float* wr = W + (int64_t)(i0 + i) * out_f + c;
        if (i < ni && vec) {
          w[r] = __ldcs(reinterpret_cast<const float4*>(wr));
        } else if (i < ni) {
          w[r].x = wr[0];
          w[r].y = c + 1 < out_f ? wr[1] : 0.f;
          w[r].z = c + 2 < out_f ? wr[2] : 0.f;
          w[r].w = c + 3 < out_f ? wr[3] : 0.f;
        } else {
          w[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int i = min(base + r, slice - 1);  // rows past ni carry zero weights
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          const float xv = xs[m * slice + i];
          acc[m][0] = fmaf(xv, w[r].x, acc[m][0]);
          acc[m][1] = fmaf(xv, w[r].y, acc[m][1]);
          acc[m][2] = fmaf(xv, w[r].z, acc[m][2]);
          acc[m][3] = fmaf(xv, w[r].w, acc[m][3]);
        }
      }
    }
  }
  // row groups summed in group order
#pragma unroll
  for (int m = 0; m < MB; ++m)
#pragma unroll
    for (int q = 0; q < 4; ++q) red[((size_t)g * MB + m) * GV_COLS + ct * 4 + q] = acc[m][q];
  __syncthreads();
  for (int t = threadIdx.x; t < MB * GV_COLS; t += blockDim.x) {
    const int m = t / GV_COLS, cc = t % GV_COLS;
    const int col = blockIdx.x * GV_COLS + cc;
    if (m >= M || col >= out_f) continue;
    float v = red[(size_t)m * GV_COLS + cc];
#pragma unroll
    for (int gg = 1; gg < G; ++gg) v += red[((size_t)gg * MB + m) * GV_COLS + cc];
    part[((int64_t)ks * M + m) * out_f + col] = v;
  }
  if (A) {
    // x A over this slice: the column blocks share the rank columns; every thread sums its
    // rows (fixed order), then warps (shuffle tree) and warps in order: deterministic
    const int jpb = (rank + gridDim.x - 1) / gridDim.x;
    const int j0 = blockIdx.x * jpb, nj = max(0, min(rank, j0 + jpb) - j0);
    const int npair = M * nj;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    float* wsum = red;  // [nwarps][16], reused once every thread has read its sums above
    __syncthreads();
    for (int p0 = 0; p0 < npair; p0 += 16) {
      float v[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) v[q] = 0.f;
      for (int i = threadIdx.x; i < ni; i += blockDim.x) {
        const float* arow = A + (int64_t)(i0 + i) * rank;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int pr = p0 + q;
          if (pr < npair) {
            const int m = pr / nj, j = j0 + pr % nj;
            v[q] = fmaf(xs[m * slice + i], __ldg(arow + j), v[q]);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 16; ++q)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v[q] += __shfl_xor_sync(0xffffffffu, v[q], off);
      if (lane == 0)
#pragma unroll
        for (int q = 0; q < 16; ++q) wsum[warp * 16 + q] = v[q];
      __syncthreads();
      if (threadIdx.x < 16 && p0 + (int)threadIdx.x < npair) {
        const int pr = p0 + threadIdx.x;
        const int m = pr / nj, j = j0 + pr % nj;
        float a = 0.f;
        for (int w = 0; w < nwarps; ++w) a += wsum[w * 16 + threadIdx.x];
        xa_part[((int64_t)ks * M + m) * rank + j] = a;
      }
      __syncthreads();
    }
  }
}

__global__ void gemv_reduce_kernel(const float* __restrict__ part, const float* __restrict__ xa_part,
                                   const float* __restrict__ B, float scale, int M, int out_f, int rank, int KS,
                                   float* __restrict__ y) {
  extern __shared__ float xa[];  // [M][rank]
  pdl_wait();  // the partials of the kernel before
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

// K slices: two (column block, slice) items per SM in all (one resident 512-thread CTA per
// SM for two waves), slices at least 32 rows.
void gemv_plan(int in_f, int out_f, int* KS, int* slice) {
  const int ncb = (out_f + GV_COLS - 1) / GV_COLS;
  int ks = std::max(1, (2 * sm_count() + ncb - 1) / ncb);
  ks = std::min(ks, std::max(1, (in_f + 31) / 32));
  *slice = (in_f + ks - 1) / ks;
  *KS = (in_f + *slice - 1) / *slice;
}

template <int MB, int G, int RPT>
int launch_gemv_partial(const float* x, const float* W, const float* A, int M, int in_f, int out_f, int rank,
                        int KS, int slice, float* part, float* xa_part, cudaStream_t stream) {
  const size_t smem = ((size_t)MB * slice + (size_t)G * MB * GV_COLS) * 4;
  SB_CHECK_ARG(smem <= 200 * 1024, "lora_gemv_f32: K slice too large");
  auto kern = gemv_partial_kernel<MB, G, RPT>;
  SB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((out_f + GV_COLS - 1) / GV_COLS, KS);
  (kern<<<grid, 128 * G, smem, stream>>>(x, W, A, M, in_f, out_f, rank, slice, part, xa_part), ::sb::count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
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
  const int rk = A ? rank : 0;
  if (M == 1)
    SB_TRY((launch_gemv_partial<1, 4, 16>(x, W, A, M, in_f, out_f, rk, KS, slice, part, xa_part, stream)));
  else if (M <= 4)
    SB_TRY((launch_gemv_partial<4, 4, 8>(x, W, A, M, in_f, out_f, rk, KS, slice, part, xa_part, stream)));
  else
    SB_TRY((launch_gemv_partial<16, 2, 8>(x, W, A, M, in_f, out_f, rk, KS, slice, part, xa_part, stream)));
  const size_t smem2 = (size_t)M * (A ? rank : 1) * 4;
  SB_CUDA_CHECK(launch_kernel(gemv_reduce_kernel, dim3((out_f + 255) / 256), dim3(256), smem2, stream, pdl_enabled(),
                              part, xa_part, A ? B : nullptr, scale, M, out_f, rk, KS, y));
  ::sb::count_launch();
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
