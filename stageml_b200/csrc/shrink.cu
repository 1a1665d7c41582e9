// Row gather into the permuted layout (R2) and the LoRA shrink (R4):
//   S[row, :] = scale[tenant(row)] * x[src(row), :] . A[tenant(row), group(row)]^T
// A is [R, K] per (tenant, group) with R = rank (or 2*rank for the packed w1|w3
// factors). This is the (xs @ A[e].t()) half of the LoRA branch in
// RequestExecutor.dynamic_one (benchmarks/multitenant_bta_system_bench.py:409),
// DynamicMoELoRALayer.forward (stageml/moe_lora_layers.py:88) and
// DynamicLoRALinear.forward (stageml/adapter_bank.py:67).
//
// The shrink is a GEMM with a tiny N (R <= 64) whose B operand changes with the
// row's tenant, so it runs on warp-level tensor-core MMAs (m16n8k16, fp32
// accumulate): one warp owns 16 rows and one 512-wide K slice; rows of the same
// tenant (contiguous after the (expert, tenant) sort) share one pass over A.
// K slices write fp32 partials that a second kernel sums in a fixed order and
// scales, so the result is deterministic. The same CTA copies its rows' K slice
// from x into the permuted activation buffer with 16-byte accesses.
#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace sb {
namespace {

struct ShrinkParams {
  const void* src;
  const int32_t* src_row_of;
  void* gather_dst;
  int K;
  const int32_t* num_tiles_dev;
  int64_t static_rows;
  int64_t rows_cap;
  const int32_t* row_tenant;
  const int32_t* tile_group;
  const void* lora_a;
  int64_t a_tenant_stride;
  int64_t a_group_stride;
  int R;
  float* spart;
};

__device__ __forceinline__ int64_t active_rows(const int32_t* num_tiles_dev, int64_t static_rows, int64_t rows_cap) {
  if (!num_tiles_dev) return static_rows;
  const int64_t r = (int64_t)(*num_tiles_dev) * 128;
  return r < rows_cap ? r : rows_cap;
}

template <typename T>
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma_16816<bf16>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma_16816<f16>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// One 32-wide K chunk of the shrink for a warp's 16 rows: each lane holds 8
// consecutive K elements (16 bytes) of rows g and g+8 and of B-row g of every
// 8-column block. The two m16n8k16 MMAs consume those registers as if lane
// (g, tig) held logical k = {2tig, 2tig+1, 2tig+8, 2tig+9}; the same
// logical->physical K permutation is applied to both operands, so the sum over
// K is unchanged while every global load is a full 16-byte vector.
struct ShrinkChunk {
  uint4 xl, xh;
  uint4 b[8];
};

template <typename T>
__device__ __forceinline__ void shrink_load(ShrinkChunk& c, const T* x_lo, const T* x_hi, const T* A, int K, int nbs,
                                            int g, int kk) {
  const bool v = kk < K;
  const uint4 z = make_uint4(0, 0, 0, 0);
  c.xl = (v && x_lo) ? ld16(x_lo + kk) : z;
  c.xh = (v && x_hi) ? ld16(x_hi + kk) : z;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb)
    if (nb < nbs) c.b[nb] = v ? ld16(A + (int64_t)(nb * 8 + g) * K + kk) : z;
}

template <typename T>
__device__ __forceinline__ void shrink_mma(float (&acc)[8][4], const ShrinkChunk& c, int nbs) {
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
    if (nb < nbs) {
      mma_16816<T>(acc[nb], c.xl.x, c.xh.x, c.xl.y, c.xh.y, c.b[nb].x, c.b[nb].y);
      mma_16816<T>(acc[nb], c.xl.z, c.xh.z, c.xl.w, c.xh.w, c.b[nb].z, c.b[nb].w);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(128) gather_shrink_kernel(const ShrinkParams p) {
  const int64_t rows_active = active_rows(p.num_tiles_dev, p.static_rows, p.rows_cap);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.y * 64 + warp * 16;
  if (row0 >= rows_active) return;
  const int K = p.K;
  const int k_begin = blockIdx.x * kShrinkKSlice;
  const int k_end = min(K, k_begin + kShrinkKSlice);
  const T* src = static_cast<const T*>(p.src);

  if (p.gather_dst) {
    T* dstb = static_cast<T*>(p.gather_dst);
#pragma unroll 4
    for (int r = 0; r < 16; ++r) {
      const int64_t row = row0 + r;
      if (row >= rows_active) break;
      const int64_t srow = p.src_row_of ? (int64_t)p.src_row_of[row] : row;
      T* dst = dstb + row * K;
      const T* s = srow >= 0 ? src + srow * K : nullptr;
      for (int c = k_begin + lane * 8; c < k_end; c += 256) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (s) v = ld16(s + c);
        *reinterpret_cast<uint4*>(dst + c) = v;
      }
    }
  }
  if (p.R == 0) return;

  int my_tenant = -1;
  if (lane < 16 && row0 + lane < rows_active) my_tenant = p.row_tenant[row0 + lane];
  unsigned pending = __ballot_sync(0xffffffffu, lane < 16 && my_tenant >= 0) & 0xFFFFu;
  if (!pending) return;
  const int group = p.tile_group ? p.tile_group[row0 / 128] : 0;
  const int g = lane >> 2, tig = lane & 3;
  const int64_t r_lo = row0 + g, r_hi = row0 + g + 8;
  const T* x_lo = nullptr;
  const T* x_hi = nullptr;
  if (r_lo < rows_active) {
    const int64_t s = p.src_row_of ? (int64_t)p.src_row_of[r_lo] : r_lo;
    if (s >= 0) x_lo = src + s * K;
  }
  if (r_hi < rows_active) {
    const int64_t s = p.src_row_of ? (int64_t)p.src_row_of[r_hi] : r_hi;
    if (s >= 0) x_hi = src + s * K;
  }
  const int nbs = p.R / 8;
  const T* lora_a = static_cast<const T*>(p.lora_a);

  while (pending) {
    const int leader = __ffs(pending) - 1;
    const int key = __shfl_sync(0xffffffffu, my_tenant, leader);
    const unsigned sel = __ballot_sync(0xffffffffu, lane < 16 && my_tenant == key) & pending;
    pending &= ~sel;
    const T* A = lora_a + key * p.a_tenant_stride + group * p.a_group_stride;
    float acc[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[nb][q] = 0.f;
    ShrinkChunk cur, nxt;
    shrink_load<T>(cur, x_lo, x_hi, A, K, nbs, g, k_begin + tig * 8);
    for (int k0 = k_begin; k0 < k_end; k0 += 32) {
      const bool more = k0 + 32 < k_end;
      if (more) shrink_load<T>(nxt, x_lo, x_hi, A, K, nbs, g, k0 + 32 + tig * 8);
      shrink_mma<T>(acc, cur, nbs);
      if (more) cur = nxt;
    }
    float* sp = p.spart + (int64_t)blockIdx.x * p.rows_cap * p.R;
    const bool lo_sel = (sel >> g) & 1u, hi_sel = (sel >> (g + 8)) & 1u;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      if (nb < nbs) {
        const int col = nb * 8 + tig * 2;
        if (lo_sel) *reinterpret_cast<float2*>(sp + r_lo * p.R + col) = make_float2(acc[nb][0], acc[nb][1]);
        if (hi_sel) *reinterpret_cast<float2*>(sp + r_hi * p.R + col) = make_float2(acc[nb][2], acc[nb][3]);
      }
    }
  }
}

template <typename T>
__global__ void shrink_reduce_kernel(const float* __restrict__ spart, int KS, int64_t rows_cap, int R,
                                     const int32_t* __restrict__ num_tiles_dev, int64_t static_rows,
                                     const int32_t* __restrict__ row_tenant, const float* __restrict__ scale,
                                     T* __restrict__ s_out) {
  const int64_t rows_active = active_rows(num_tiles_dev, static_rows, rows_cap);
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows_active * R) return;
  const int64_t row = idx / R;
  const int tn = row_tenant[row];
  float v = 0.f;
  if (tn >= 0) {
    for (int ks = 0; ks < KS; ++ks) v += spart[((int64_t)ks * rows_cap + row) * R + (idx - row * R)];
    v *= scale ? scale[tn] : 1.f;
  }
  s_out[idx] = from_f32<T>(v);
}

}  // namespace

int launch_gather_shrink(const ShrinkLaunch& s, cudaStream_t stream) {
  SB_CHECK_ARG(s.src, "shrink: null source");
  SB_CHECK_ARG(s.K > 0 && s.K % 8 == 0, "shrink: K=%d must be a positive multiple of 8", s.K);
  SB_CHECK_ARG(s.R % 8 == 0 && s.R <= 64, "shrink: R=%d must be a multiple of 8 <= 64", s.R);
  SB_CHECK_ARG(s.R == 0 || (s.lora_a && s.spart && s.s_out && s.row_tenant), "shrink: missing LoRA buffers");
  SB_CHECK_ARG(reinterpret_cast<uintptr_t>(s.src) % 16 == 0, "shrink: source must be 16-byte aligned");
  if (!s.gather_dst && s.R == 0) return STAGEML_OK;
  const int KS = shrink_num_slices(s.K);
  const int64_t rows_max = s.num_tiles_dev ? s.rows_cap : s.static_rows;
  if (rows_max == 0) return STAGEML_OK;
  ShrinkParams p;
  p.src = s.src;
  p.src_row_of = s.src_row_of;
  p.gather_dst = s.gather_dst;
  p.K = s.K;
  p.num_tiles_dev = s.num_tiles_dev;
  p.static_rows = s.static_rows;
  p.rows_cap = s.num_tiles_dev ? s.rows_cap : s.static_rows;
  p.row_tenant = s.row_tenant;
  p.tile_group = s.tile_group;
  p.lora_a = s.lora_a;
  p.a_tenant_stride = s.a_tenant_stride;
  p.a_group_stride = s.a_group_stride;
  p.R = s.R;
  p.spart = s.spart;
  dim3 grid(KS, (unsigned)((rows_max + 63) / 64));
  SB_CHECK_ARG(grid.y <= 65535u, "shrink: too many rows for one launch");
  if (s.dtype_bf16)
    (gather_shrink_kernel<bf16><<<grid, 128, 0, stream>>>(p), ::sb::count_launch());
  else
    (gather_shrink_kernel<f16><<<grid, 128, 0, stream>>>(p), ::sb::count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  if (s.R > 0) {
    const int64_t n = rows_max * s.R;
    if (s.dtype_bf16)
      (shrink_reduce_kernel<bf16><<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
           s.spart, KS, p.rows_cap, s.R, s.num_tiles_dev, s.static_rows, s.row_tenant, s.lora_scale,
           static_cast<bf16*>(s.s_out)),
       ::sb::count_launch());
    else
      (shrink_reduce_kernel<f16><<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
           s.spart, KS, p.rows_cap, s.R, s.num_tiles_dev, s.static_rows, s.row_tenant, s.lora_scale,
           static_cast<f16*>(s.s_out)),
       ::sb::count_launch());
    SB_CUDA_CHECK(cudaGetLastError());
  }
  return STAGEML_OK;
}

}  // namespace sb
