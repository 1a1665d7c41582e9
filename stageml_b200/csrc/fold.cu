// Stage-0 LoRA fold (R7): W' = W + s * L . R, batched over matrices.
//   layout 0 ([out,in]): L = B [out, r], R = A [r, in]   (W + s * B @ A)
//   layout 1 ([in,out]): L = A [in, r],  R = B [r, out]  (W + s * A @ B)
// Restates materialize_residual_weight (stageml/triton_generator.py:175-191),
// the per-adapter merge of StageMLAdapterBankLinear (stageml/adapter_bank.py:90-94)
// and StageMLCostBasedAdapterCache (stageml/adapter_cache.py:72-81), and the
// einsum("eor,eri->eoi") fold of MaterializedMoELoRALayer (stageml/moe_lora_layers.py:104-110).
//
// The fold streams W once and writes W' once: HBM-bound (4 bytes per 16-bit
// element, 8 per fp32 element). The rank-r product costs r FMAs per element, which
// for r = 16 at HBM speed would saturate the fp32 pipes on 16-bit weights, so the
// 16-bit path computes it with warp-level tensor-core MMAs (m16n8k16, fp32
// accumulate) on a 64 x 128 tile staged in shared memory (cp.async) with its L and R
// slices, with 16-byte accesses of W and W'. fp32 (rank <= 16) keeps each thread's R
// columns in registers and streams W rows through a cp.async ring in shared memory;
// other fp32 and unaligned shapes use plain fp32 FMAs, one element per thread.
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

__device__ __forceinline__ void fold_cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void fold_cp_async8(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(valid ? 8 : 0) : "memory");
}
__device__ __forceinline__ void fold_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void fold_cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
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

// Grid x = (column tile) * batch + matrix: the matrices of one tile run next to each
// other, so a W shared by the batch (w_bs = 0) is read from DRAM once per tile.
// Dynamic shared memory: the W tile [FT_M][FT_N + FT_PAD], L rows [FT_M][rk16 + 8], R columns [rk16][FT_N + 8].
inline size_t fold_mma_smem(int rank, size_t esz) {
  const int rk16 = (rank + 15) & ~15;
  return esz * ((size_t)FT_M * (FT_N + FT_PAD) + (size_t)FT_M * (rk16 + 8) + (size_t)rk16 * (FT_N + 8));
}

template <typename T>
__global__ void __launch_bounds__(256) fold_mma_kernel(const FoldArgs f, int batch) {
  extern __shared__ __align__(16) uint8_t fold_smem[];
  const int rk16 = (f.rank + 15) & ~15;
  auto tile = reinterpret_cast<T(*)[FT_N + FT_PAD]>(fold_smem);
  T* Ls_base = reinterpret_cast<T*>(fold_smem) + FT_M * (FT_N + FT_PAD);
  T* Rs_base = Ls_base + FT_M * (rk16 + 8);
  auto Ls = [&](int r, int j) -> T& { return Ls_base[r * (rk16 + 8) + j]; };
  auto Rs = [&](int j, int c) -> T& { return Rs_base[j * (FT_N + 8) + c]; };
  const int b = blockIdx.x % batch;
  const int m0 = blockIdx.y * FT_M, n0 = (blockIdx.x / batch) * FT_N;
  const T* W = static_cast<const T*>(f.W) + (int64_t)b * f.w_bs;
  T* O = static_cast<T*>(f.out) + (int64_t)b * f.rows * f.cols;
  const T *L, *R;
  fold_operands<T>(f, b, &L, &R);
  const float s = f.scale[b];
  // 1. W tile -> shared by cp.async (16-byte pieces, zero-filled past the edges), in flight
  //    while the L and R tiles are loaded (zero past the rank / the edges)
  for (int i = threadIdx.x; i < FT_M * FT_N / 8; i += 256) {
    const int r = i / (FT_N / 8), c8 = (i % (FT_N / 8)) * 8;
    const int gm = m0 + r, gn = n0 + c8;
    const bool v = gm < f.rows && gn < f.cols;
    fold_cp_async16(smem_u32(&tile[r][c8]), v ? (const void*)(W + (int64_t)gm * f.cols + gn) : f.W, v);
  }
  fold_cp_commit();
  const T zero = from_f32<T>(0.f);
  for (int i = threadIdx.x; i < FT_M * rk16; i += 256) {
    const int r = i / rk16, j = i % rk16;
    Ls(r, j) = (m0 + r < f.rows && j < f.rank) ? L[(int64_t)(m0 + r) * f.rank + j] : zero;
  }
  for (int i = threadIdx.x; i < rk16 * FT_N / 8; i += 256) {
    const int j = i / (FT_N / 8), c8 = (i % (FT_N / 8)) * 8;
    const int gn = n0 + c8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (j < f.rank) {
      if (gn + 8 <= f.cols && (f.cols % 8) == 0)
        v = __ldg(reinterpret_cast<const uint4*>(R + (int64_t)j * f.cols + gn));
      else {
        T* e = reinterpret_cast<T*>(&v);
        for (int q = 0; q < 8; ++q) e[q] = gn + q < f.cols ? R[(int64_t)j * f.cols + gn + q] : zero;
      }
    }
    *reinterpret_cast<uint4*>(&Rs(j, c8)) = v;
  }
  fold_cp_wait<0>();
  __syncthreads();
  // 2. rank-r product on tensor cores (operands from shared memory), added into the tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int mb = (warp & 3) * 16;   // 4 row blocks of 16
  const int nh = (warp >> 2) * 64;  // 2 column halves of 64
  float acc[8][4];
#pragma unroll
  for (int nb = 0; nb < 8; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[nb][q] = 0.f;
  for (int k0 = 0; k0 < rk16; k0 += 16) {
    const int ja = k0 + tig * 2, jb = ja + 8;
    const uint32_t a0 = pack2_raw<T>(Ls(mb + g, ja), Ls(mb + g, ja + 1));
    const uint32_t a1 = pack2_raw<T>(Ls(mb + g + 8, ja), Ls(mb + g + 8, ja + 1));
    const uint32_t a2 = pack2_raw<T>(Ls(mb + g, jb), Ls(mb + g, jb + 1));
    const uint32_t a3 = pack2_raw<T>(Ls(mb + g + 8, jb), Ls(mb + g + 8, jb + 1));
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const int n = nh + nb * 8 + g;
      const uint32_t b0 = pack2_raw<T>(Rs(ja, n), Rs(ja + 1, n));
      const uint32_t b1 = pack2_raw<T>(Rs(jb, n), Rs(jb + 1, n));
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

// fp32, rank <= 16, even cols, 8-byte aligned rows: one resident wave of 128-thread CTAs,
// each folding a contiguous range of rows of one 256-column block. Every thread owns 2
// columns and keeps their rank-r slice of R in registers; the W rows and their L rows
// stream through a 4-stage cp.async ring of 8-row stages (three in flight, ~150 KB per SM
// at 6 CTAs per SM), independent of registers. fp32 FMAs in j order (no TF32); W' stores
// are streaming.
constexpr int FC_COLS = 256, FC_SROWS = 8, FC_STAGES = 4, FC_CTAS_PER_SM = 6;
__global__ void __launch_bounds__(128) fold_f32_ring_kernel(const FoldArgs f, int rows_per_cta) {
  __shared__ __align__(16) float Ws[FC_STAGES][FC_SROWS][FC_COLS];
  __shared__ __align__(16) float Lss[FC_STAGES][FC_SROWS][16];
  const int b = blockIdx.z;
  const float* W = static_cast<const float*>(f.W) + (int64_t)b * f.w_bs;
  float* O = static_cast<float*>(f.out) + (int64_t)b * f.rows * f.cols;
  const float *L, *R;
  fold_operands<float>(f, b, &L, &R);
  const float s = f.scale[b];
  const int t = threadIdx.x;
  const int n = blockIdx.x * FC_COLS + t * 2;
  const bool col_ok = n < f.cols;
  const int m0 = blockIdx.y * rows_per_cta, m_end = min(f.rows, m0 + rows_per_cta);
  if (m0 >= m_end) return;
  const int nst = (m_end - m0 + FC_SROWS - 1) / FC_SROWS;
  auto issue = [&](int st) {
    if (st < nst) {
      const int slot = st % FC_STAGES;
#pragma unroll
      for (int r = 0; r < FC_SROWS; ++r) {
        const int row = m0 + st * FC_SROWS + r;
        const bool v = col_ok && row < m_end;
        fold_cp_async8(smem_u32(&Ws[slot][r][t * 2]), v ? (const void*)(W + (int64_t)row * f.cols + n) : f.W, v);
      }
      {  // the stage's L rows: 8 rows x 16 ranks, one 4-byte piece per thread (zero past the rank)
        const int r = t >> 4, j = t & 15, row = m0 + st * FC_SROWS + r;
        const bool v = row < m_end && j < f.rank;
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(&Lss[slot][r][j])),
                     "l"(v ? (const void*)(L + (int64_t)row * f.rank + j) : f.scale), "r"(v ? 4 : 0)
                     : "memory");
      }
    }
    fold_cp_commit();  // possibly empty: keeps the group count in step
  };
#pragma unroll
  for (int st = 0; st < FC_STAGES - 1; ++st) issue(st);
  float2 rv[16];
#pragma unroll
  for (int j = 0; j < 16; ++j)
    rv[j] = (col_ok && j < f.rank) ? __ldg(reinterpret_cast<const float2*>(R + (int64_t)j * f.cols + n))
                                   : make_float2(0.f, 0.f);
  for (int st = 0; st < nst; ++st) {
    fold_cp_wait<FC_STAGES - 2>();  // stage st has landed (st + 1, st + 2 may still be in flight)
    __syncthreads();                // visible to every thread; every thread is done with stage st - 1
    issue(st + FC_STAGES - 1);      // refills the slot of stage st - 1
    const int slot = st % FC_STAGES;
#pragma unroll
    for (int r = 0; r < FC_SROWS; ++r) {
      const int row = m0 + st * FC_SROWS + r;
      if (row >= m_end || !col_ok) break;
      const float2 w = *reinterpret_cast<const float2*>(&Ws[slot][r][t * 2]);
      const float4* l4 = reinterpret_cast<const float4*>(&Lss[slot][r][0]);  // 4 broadcast 16-byte reads
      float lv[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = l4[q];
        lv[4 * q] = v.x, lv[4 * q + 1] = v.y, lv[4 * q + 2] = v.z, lv[4 * q + 3] = v.w;
      }
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        acc.x = fmaf(lv[j], rv[j].x, acc.x);
        acc.y = fmaf(lv[j], rv[j].y, acc.y);
      }
      __stcs(reinterpret_cast<float2*>(O + (int64_t)row * f.cols + n), make_float2(w.x + s * acc.x, w.y + s * acc.y));
    }
  }
  fold_cp_wait<0>();
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
    const bool vec2 = (cols % 2 == 0) && (reinterpret_cast<uintptr_t>(W) % 8 == 0) &&
                      (reinterpret_cast<uintptr_t>(out) % 8 == 0) && (w_bs % 2 == 0) && rank <= 16;
    if (vec2) {
      // one resident wave: the row ranges of every column block and matrix fill the SMs once
      const int ncb = (cols + FC_COLS - 1) / FC_COLS;
      const int64_t slots = (int64_t)FC_CTAS_PER_SM * sm_count();
      const int nrb = (int)std::max<int64_t>(1, std::min<int64_t>(slots / std::max<int64_t>(1, (int64_t)ncb * batch),
                                                                  (rows + FC_SROWS - 1) / FC_SROWS));
      const int rows_per = ((rows + nrb - 1) / nrb + FC_SROWS - 1) / FC_SROWS * FC_SROWS;
      dim3 grid(ncb, (rows + rows_per - 1) / rows_per, batch);
      SB_CHECK_ARG(grid.y <= 65535u, "lora_fold: too many rows");
      (fold_f32_ring_kernel<<<grid, 128, 0, stream>>>(f, rows_per), ::sb::count_launch());
    } else {
      const int64_t n_el = (int64_t)rows * cols;
      const unsigned gx = (unsigned)std::min<int64_t>((n_el + 255) / 256, 8 * (int64_t)sm_count());
      (fold_scalar_kernel<float><<<dim3(gx, batch), 256, 0, stream>>>(f), ::sb::count_launch());
    }
  } else if (dtype == STAGEML_BF16 || dtype == STAGEML_F16) {
    if (aligned16 && rank <= 64) {
      const int64_t gx = (int64_t)((cols + FT_N - 1) / FT_N) * batch;
      dim3 grid((unsigned)gx, (rows + FT_M - 1) / FT_M, 1);
      SB_CHECK_ARG(grid.y <= 65535u && gx < (int64_t(1) << 31), "lora_fold: too many rows");
      const size_t smem = fold_mma_smem(rank, 2);
      if (dtype == STAGEML_BF16) {
        SB_CUDA_CHECK(cudaFuncSetAttribute(fold_mma_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem));
        (fold_mma_kernel<bf16><<<grid, 256, smem, stream>>>(f, batch), ::sb::count_launch());
      } else {
        SB_CUDA_CHECK(cudaFuncSetAttribute(fold_mma_kernel<f16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem));
        (fold_mma_kernel<f16><<<grid, 256, smem, stream>>>(f, batch), ::sb::count_launch());
      }
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
