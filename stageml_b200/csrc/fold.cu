// Stage-0 LoRA fold (R7): W' = W + s * L . R, batched over matrices.
//   layout 0 ([out,in]): L = B [out, r], R = A [r, in]   (W + s * B @ A)
//   layout 1 ([in,out]): L = A [in, r],  R = B [r, out]  (W + s * A @ B)
// Restates materialize_residual_weight (stageml/triton_generator.py:175-191),
// the per-adapter merge of StageMLAdapterBankLinear (stageml/adapter_bank.py:90-94)
// and StageMLCostBasedAdapterCache (stageml/adapter_cache.py:72-81), and the
// einsum("eor,eri->eoi") fold of MaterializedMoELoRALayer (stageml/moe_lora_layers.py:104-110).
//
// The fold streams W once and writes W' once: HBM-bound (4 bytes per 16-bit
// element). The rank-r product costs r FMAs per element, which for r = 16 at
// HBM speed would saturate the fp32 pipes, so the 16-bit path computes it with
// warp-level tensor-core MMAs (m16n8k16, fp32 accumulate) on a 64 x 128 tile
// staged in shared memory, with 16-byte loads and stores of W and W'.
// fp32 (and unaligned shapes) use plain fp32 FMAs, one element per thread.
#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace sb {
namespace {

constexpr int FT_M = 64, FT_N = 128, FT_PAD = 8;

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<bf16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<f16>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2_raw(T lo, T hi) {
  uint32_t r;
  T* h = reinterpret_cast<T*>(&r);
  h[0] = lo;
  h[1] = hi;
  return r;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<bf16>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<f16>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct FoldArgs {
  const void* W;
  const void* A;
  const void* B;
  const float* scale;
  int rows, cols, rank, layout;
  int64_t w_bs, a_bs, b_bs;
  void* out;
};

template <typename T>
__device__ __forceinline__ void fold_operands(const FoldArgs& f, int b, const T** L, const T** R) {
  const T* A = static_cast<const T*>(f.A) + (int64_t)b * f.a_bs;
  const T* B = static_cast<const T*>(f.B) + (int64_t)b * f.b_bs;
  if (f.layout == 0) {
    *L = B;
    *R = A;
  } else {
    *L = A;
    *R = B;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) fold_mma_kernel(const FoldArgs f) {
  __shared__ __align__(16) T tile[FT_M][FT_N + FT_PAD];
  const int b = blockIdx.z;
  const int m0 = blockIdx.y * FT_M, n0 = blockIdx.x * FT_N;
  const T* W = static_cast<const T*>(f.W) + (int64_t)b * f.w_bs;
  T* O = static_cast<T*>(f.out) + (int64_t)b * f.rows * f.cols;
  const T *L, *R;
  fold_operands<T>(f, b, &L, &R);
  const float s = f.scale[b];
  // 1. W tile -> shared (16-byte accesses)
  for (int i = threadIdx.x; i < FT_M * FT_N / 8; i += 256) {
    const int r = i / (FT_N / 8), c8 = (i % (FT_N / 8)) * 8;
    const int gm = m0 + r, gn = n0 + c8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (gm < f.rows && gn < f.cols) v = __ldg(reinterpret_cast<const uint4*>(W + (int64_t)gm * f.cols + gn));
    *reinterpret_cast<uint4*>(&tile[r][c8]) = v;
  }
  __syncthreads();
  // 2. rank-r product on tensor cores, added into the tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int mb = (warp & 3) * 16;   // 4 row blocks of 16
  const int nh = (warp >> 2) * 64;  // 2 column halves of 64
  float acc[8][4];
#pragma unroll
  for (int nb = 0; nb < 8; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[nb][q] = 0.f;
  const T zero = from_f32<T>(0.f);
  for (int k0 = 0; k0 < f.rank; k0 += 16) {
    auto Lv = [&](int m, int j) -> T { return (m < f.rows && j < f.rank) ? L[(int64_t)m * f.rank + j] : zero; };
    const int ml = m0 + mb + g, mh = ml + 8;
    const int ja = k0 + tig * 2, jb = ja + 8;
    const uint32_t a0 = pack2_raw<T>(Lv(ml, ja), Lv(ml, ja + 1));
    const uint32_t a1 = pack2_raw<T>(Lv(mh, ja), Lv(mh, ja + 1));
    const uint32_t a2 = pack2_raw<T>(Lv(ml, jb), Lv(ml, jb + 1));
    const uint32_t a3 = pack2_raw<T>(Lv(mh, jb), Lv(mh, jb + 1));
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const int n = n0 + nh + nb * 8 + g;
      auto Rv = [&](int j) -> T { return (j < f.rank && n < f.cols) ? R[(int64_t)j * f.cols + n] : zero; };
      const uint32_t b0 = pack2_raw<T>(Rv(ja), Rv(ja + 1));
      const uint32_t b1 = pack2_raw<T>(Rv(jb), Rv(jb + 1));
      mma16816<T>(acc[nb], a0, a1, a2, a3, b0, b1);
    }
  }
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
    const int c = nh + nb * 8 + tig * 2;
    const int rl = mb + g, rh = rl + 8;
    uint32_t* pl = reinterpret_cast<uint32_t*>(&tile[rl][c]);
    uint32_t* ph = reinterpret_cast<uint32_t*>(&tile[rh][c]);
    const T* wl = reinterpret_cast<const T*>(pl);
    const T* wh = reinterpret_cast<const T*>(ph);
    const uint32_t nl = pack2<T>(to_f32<T>(wl[0]) + s * acc[nb][0], to_f32<T>(wl[1]) + s * acc[nb][1]);
    const uint32_t nhv = pack2<T>(to_f32<T>(wh[0]) + s * acc[nb][2], to_f32<T>(wh[1]) + s * acc[nb][3]);
    *pl = nl;
    *ph = nhv;
  }
  __syncthreads();
  // 3. tile -> W' (16-byte accesses)
  for (int i = threadIdx.x; i < FT_M * FT_N / 8; i += 256) {
    const int r = i / (FT_N / 8), c8 = (i % (FT_N / 8)) * 8;
    const int gm = m0 + r, gn = n0 + c8;
    if (gm < f.rows && gn < f.cols)
      *reinterpret_cast<uint4*>(O + (int64_t)gm * f.cols + gn) = *reinterpret_cast<const uint4*>(&tile[r][c8]);
  }
}

// One output element per thread, fp32 FMAs in j order.
template <typename T>
__global__ void fold_scalar_kernel(const FoldArgs f) {
  const int b = blockIdx.y;
  const int64_t n_el = (int64_t)f.rows * f.cols;
  const T* W = static_cast<const T*>(f.W) + (int64_t)b * f.w_bs;
  T* O = static_cast<T*>(f.out) + (int64_t)b * n_el;
  const T *L, *R;
  fold_operands<T>(f, b, &L, &R);
  const float s = f.scale[b];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_el; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / f.cols, n = i - m * f.cols;
    float acc = 0.f;
    for (int j = 0; j < f.rank; ++j) acc = fmaf(to_f32<T>(L[m * f.rank + j]), to_f32<T>(R[(int64_t)j * f.cols + n]), acc);
    O[i] = from_f32<T>(to_f32<T>(W[i]) + s * acc);
  }
}

}  // namespace

int launch_lora_fold(const void* W, const void* A, const void* B, const float* scale, int batch, int rows, int cols,
                     int rank, int layout, int64_t w_bs, int64_t a_bs, int64_t b_bs, int dtype, void* out,
                     cudaStream_t stream) {
  SB_CHECK_ARG(W && A && B && scale && out, "lora_fold: null pointer");
  SB_CHECK_ARG(batch >= 0 && rows >= 0 && cols >= 0 && rank >= 1, "lora_fold: bad sizes");
  SB_CHECK_ARG(layout == 0 || layout == 1, "lora_fold: layout must be 0 ([out,in]) or 1 ([in,out])");
  SB_CHECK_ARG(batch <= 65535, "lora_fold: batch too large");
  if (batch == 0 || rows == 0 || cols == 0) return STAGEML_OK;
  FoldArgs f{W, A, B, scale, rows, cols, rank, layout, w_bs, a_bs, b_bs, out};
  const bool aligned16 = (cols % 8 == 0) && (reinterpret_cast<uintptr_t>(W) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(out) % 16 == 0) && (w_bs % 8 == 0);
  if (dtype == STAGEML_F32) {
    const int64_t n_el = (int64_t)rows * cols;
    const unsigned gx = (unsigned)std::min<int64_t>((n_el + 255) / 256, 8 * (int64_t)sm_count());
    (fold_scalar_kernel<float><<<dim3(gx, batch), 256, 0, stream>>>(f), ::sb::count_launch());
  } else if (dtype == STAGEML_BF16 || dtype == STAGEML_F16) {
    if (aligned16 && rank <= 64) {
      dim3 grid((cols + FT_N - 1) / FT_N, (rows + FT_M - 1) / FT_M, batch);
      SB_CHECK_ARG(grid.y <= 65535u, "lora_fold: too many rows");
      if (dtype == STAGEML_BF16)
        (fold_mma_kernel<bf16><<<grid, 256, 0, stream>>>(f), ::sb::count_launch());
      else
        (fold_mma_kernel<f16><<<grid, 256, 0, stream>>>(f), ::sb::count_launch());
    } else {
      const int64_t n_el = (int64_t)rows * cols;
      const unsigned gx = (unsigned)std::min<int64_t>((n_el + 255) / 256, 8 * (int64_t)sm_count());
      if (dtype == STAGEML_BF16)
        (fold_scalar_kernel<bf16><<<dim3(gx, batch), 256, 0, stream>>>(f), ::sb::count_launch());
      else
        (fold_scalar_kernel<f16><<<dim3(gx, batch), 256, 0, stream>>>(f), ::sb::count_launch());
    }
  } else {
    return set_error(STAGEML_ERR_INVALID_ARG, "lora_fold: unsupported dtype %d", dtype);
  }
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

}  // namespace sb
