// Single LoRA linear in fp32 with the [in,out] layout of the config-1 workload
// (benchmarks/triton_lora_equivalence_check.py:11-22):
//   dynamic: y = x W + s (x A) B        folded: y = x W'
// x [M, in] with M <= 16, W [in, out], A [in, r], B [r, out]. Real fp32 FMAs
// (no TF32). HBM-bound on the W read (4 B per element): split-K over
// (512-column block, K slice) CTAs in one resident wave; each CTA streams its
// slice of W through a cp.async ring in shared memory (~144 KB in flight per SM)
// and writes one fp32 partial per (K slice, row, column). A second kernel (a
// programmatic dependent launch) adds the partials in slice order and applies
// the rank-r expansion, so results are deterministic.
#include <mutex>

#include "common.cuh"
#include "host_util.h"
#include "kernels.h"
#include "stage_timer.h"

namespace sb {
namespace {

constexpr int GV_COLS = 512;   // columns per CTA (128 threads x float4)
constexpr int GV_MAXM = 16;

__device__ __forceinline__ void gv_cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void gv_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void gv_cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One resident wave of 128-thread CTAs: CTA (column block, K slice) owns 512 columns (4
// per thread) and a contiguous K slice of `slice` rows, which streams through a 4-stage
// cp.async ring of 8-row stages of W (16 KB each; three in flight, ~144 KB per SM at 3
// CTAs per SM) while every thread accumulates its columns for the MB rows of x in
// registers, rows in order. MB: rows of x handled (>= M).
constexpr int GV_SROWS = 8, GV_STAGES = 4, GV_CTAS_PER_SM = 3;
template <int MB>
__global__ void __launch_bounds__(128) gemv_partial_kernel(const float* __restrict__ x, const float* __restrict__ W,
                                                           const float* __restrict__ A, int M, int in_f, int out_f,
                                                           int rank, int slice, float* __restrict__ part,
                                                           float* __restrict__ xa_part) {
  extern __shared__ __align__(16) float sm[];  // W ring [GV_STAGES][GV_SROWS][GV_COLS], xs [MB][slice], warp sums
  float* ring = sm;
  float* xs = sm + GV_STAGES * GV_SROWS * GV_COLS;
  float* wsum = xs + MB * slice;
  pdl_trigger();  // the reduce kernel may be scheduled now; it waits for this grid before reading
  const int ks = blockIdx.y;
  const int i0 = ks * slice, i1 = min(in_f, i0 + slice);
  const int ni = i1 - i0;
  const int t = threadIdx.x;
  const int c = blockIdx.x * GV_COLS + t * 4;
  const bool vec = (c + 4 <= out_f) && (out_f % 4 == 0);
  const int nst = (ni + GV_SROWS - 1) / GV_SROWS;
  auto issue = [&](int st) {
    if (st < nst && vec) {
      float* dst = ring + (size_t)(st % GV_STAGES) * GV_SROWS * GV_COLS + t * 4;
#pragma unroll
      for (int r = 0; r < GV_SROWS; ++r) {
        const int i = st * GV_SROWS + r;
        const bool v = i < ni;
        gv_cp_async16(smem_u32(dst + r * GV_COLS), v ? (const void*)(W + (int64_t)(i0 + i) * out_f + c) : W, v);
      }
    }
    gv_cp_commit();  // possibly empty: keeps the group count in step
  };
#pragma unroll
  for (int st = 0; st < GV_STAGES - 1; ++st) issue(st);
  for (int e = t; e < MB * slice; e += blockDim.x) {
    const int m = e / slice, i = e % slice;
    xs[e] = (m < M && i < ni) ? x[(int64_t)m * in_f + i0 + i] : 0.f;
  }
  float acc[MB][4];
#pragma unroll
  for (int m = 0; m < MB; ++m)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[m][q] = 0.f;
  __syncthreads();  // xs
  for (int st = 0; st < nst; ++st) {
    gv_cp_wait<GV_STAGES - 2>();  // this thread's copies of stage st have landed (it reads only those)
    issue(st + GV_STAGES - 1);    // refills the slot of stage st - 1, which this thread has finished
    const float* stage = ring + (size_t)(st % GV_STAGES) * GV_SROWS * GV_COLS + t * 4;
#pragma unroll
    for (int r = 0; r < GV_SROWS; ++r) {
      const int i = st * GV_SROWS + r;
      if (i >= ni) break;
      float4 w;
      if (vec) {
        w = *reinterpret_cast<const float4*>(stage + r * GV_COLS);
      } else {  // ragged column tail: direct loads
        const float* wr = W + (int64_t)(i0 + i) * out_f + c;
        w.x = c < out_f ? wr[0] : 0.f;
        w.y = c + 1 < out_f ? wr[1] : 0.f;
        w.z = c + 2 < out_f ? wr[2] : 0.f;
        w.w = c + 3 < out_f ? wr[3] : 0.f;
      }
#pragma unroll
      for (int m = 0; m < MB; ++m) {
        const float xv = xs[m * slice + i];
        acc[m][0] = fmaf(xv, w.x, acc[m][0]);
        acc[m][1] = fmaf(xv, w.y, acc[m][1]);
        acc[m][2] = fmaf(xv, w.z, acc[m][2]);
        acc[m][3] = fmaf(xv, w.w, acc[m][3]);
      }
    }
  }
  gv_cp_wait<0>();
#pragma unroll
  for (int m = 0; m < MB; ++m)
    if (m < M)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (c + q < out_f) part[((int64_t)ks * M + m) * out_f + c + q] = acc[m][q];
  if (A) {
    // x A over this slice: the column blocks share the rank columns; every thread sums its
    // rows (fixed order), then warps (shuffle tree) and warps in order: deterministic
    const int jpb = (rank + gridDim.x - 1) / gridDim.x;
    const int j0 = blockIdx.x * jpb, nj = max(0, min(rank, j0 + jpb) - j0);
    const int npair = M * nj;
    const int warp = t >> 5, lane = t & 31, nwarps = blockDim.x >> 5;
    for (int p0 = 0; p0 < npair; p0 += 16) {
      float v[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) v[q] = 0.f;
      for (int i = t; i < ni; i += blockDim.x) {
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
      if (t < 16 && p0 + t < npair) {
        const int pr = p0 + t;
        const int m = pr / nj, j = j0 + pr % nj;
        float a = 0.f;
        for (int w = 0; w < nwarps; ++w) a += wsum[w * 16 + t];
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

// K slices: one resident wave of GV_CTAS_PER_SM CTAs per SM over (column block, slice)
// items, slices a multiple of the 8-row stage.
void gemv_plan(int in_f, int out_f, int* KS, int* slice) {
  const int ncb = (out_f + GV_COLS - 1) / GV_COLS;
  const int slots = GV_CTAS_PER_SM * sm_count();
  int ks = std::max(1, slots / ncb);
  ks = std::min(ks, std::max(1, (in_f + GV_SROWS - 1) / GV_SROWS));
  *slice = ((in_f + ks - 1) / ks + GV_SROWS - 1) / GV_SROWS * GV_SROWS;
  *KS = (in_f + *slice - 1) / *slice;
}

template <int MB>
int launch_gemv_partial(const float* x, const float* W, const float* A, int M, int in_f, int out_f, int rank,
                        int KS, int slice, float* part, float* xa_part, cudaStream_t stream) {
  const size_t smem = ((size_t)GV_STAGES * GV_SROWS * GV_COLS + (size_t)MB * slice + 4 * 16) * 4;
  SB_CHECK_ARG(smem <= 200 * 1024, "lora_gemv_f32: K slice too large");
  auto kern = gemv_partial_kernel<MB>;
  SB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((out_f + GV_COLS - 1) / GV_COLS, KS);
  (kern<<<grid, 128, smem, stream>>>(x, W, A, M, in_f, out_f, rank, slice, part, xa_part), ::sb::count_launch());
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
    SB_TRY((launch_gemv_partial<1>(x, W, A, M, in_f, out_f, rk, KS, slice, part, xa_part, stream)));
  else if (M <= 4)
    SB_TRY((launch_gemv_partial<4>(x, W, A, M, in_f, out_f, rk, KS, slice, part, xa_part, stream)));
  else
    SB_TRY((launch_gemv_partial<16>(x, W, A, M, in_f, out_f, rk, KS, slice, part, xa_part, stream)));
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
