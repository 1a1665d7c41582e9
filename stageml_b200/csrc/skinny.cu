// Grouped GEMM for a handful of rows per group (decode-sized batches): at most
// 16 valid rows in every 128-row tile, so the work is streaming the weights.
//
// A work item is 8 output columns of one tile, computed by 1-8 warps that split
// K; each warp streams its K range of the item's 8 weight rows (SwiGLU: 8 gate +
// 8 up rows) with 16-byte loads, eight 32-wide chunks in flight per lane, and
// multiplies by the tile's rows on warp-level tensor cores (m16n8k16, rows past
// the valid count are zeros). The warps per item follow from K only, so a row's
// result does not depend on the rest of the batch. Partial sums meet in shared
// memory; the epilogue adds the
// per-tenant LoRA expand S . B^T (S = the pre-scaled shrink output), then SwiGLU
// or the plain scale / bias / routing weight, and stores 16-bit rows. The same
// computation as the grouped tcgen05 GEMM (grouped_gemm.cu) for the
// per-(slot, expert) body of RequestExecutor.dynamic_one
// (benchmarks/multitenant_bta_system_bench.py:408-413).
#include "common.cuh"
#include "grouped_gemm.cuh"
#include "host_util.h"

namespace sb {
namespace {

constexpr int kSkNB = 8;        // output columns per CTA
constexpr int kSkWarps = 8;
constexpr int kSkUnroll = 8;

struct SkParams {
  const void* a;
  const int32_t* a_row_of;
  int K;
  const void* b;
  int64_t b_rows_total;
  int b_group_rows;
  const int32_t* b_group_map;  // optional row group -> weight group
  int N;
  const int32_t* num_tiles_dev;
  int tiles_cap;
  const int32_t* tile_group;
  const int32_t* group_offsets;
  const int32_t* group_counts;
  int64_t m_rows;
  const int32_t* row_tenant;
  int rank;
  int lora_cols;
  const void* s16;
  const void* lora_b;
  int64_t lb_tenant_stride;
  int64_t lb_group_stride;
  const float* row_scale;
  const void* bias;
  int64_t bias_group_stride;
  int bias_group_mod;
  const float* b_scale;
  void* out;
  int64_t ldo;
  int wait_late;  // PDL launch after a kernel that writes only S: wait before the epilogue (else at the start)
};

template <typename T>
__device__ __forceinline__ void sk_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1);
template <>
__device__ __forceinline__ void sk_mma<bf16>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void sk_mma<f16>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
// Weight stream: read-only, and L2 fetches the surrounding 256 bytes (a warp load
// touches 64 contiguous bytes of each of 8 rows; the next chunks follow right after).
__device__ __forceinline__ uint4 ldg16_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Lane (g, tig) holds 8 consecutive K values (16 bytes) of rows g, g+8 and of
// weight row g; the two MMAs read them as logical k = {2tig, 2tig+1, 2tig+8,
// 2tig+9}, the same permutation on both operands, so the dot products are exact.
template <typename T, int NBLK>
__device__ __forceinline__ void sk_chunk(float (&acc)[NBLK][4], const uint4& xl, const uint4& xh, const uint4 (&w)[NBLK]) {
#pragma unroll
  for (int b = 0; b < NBLK; ++b) {
    sk_mma<T>(acc[b], xl.x, xh.x, xl.y, xh.y, w[b].x, w[b].y);
    sk_mma<T>(acc[b], xl.z, xh.z, xl.w, xh.w, w[b].z, w[b].w);
  }
}

// Item = (tile, 8 output columns), computed by WPI warps that split K; the partial sums of
// an item meet in shared memory and its first warp runs the epilogue from the
// MMA fragment: lane (g, tig) owns rows g, g+8 and columns 2tig, 2tig+1.
// HI: rows 8-15 of a tile may be valid (more than 8 routed rows in all); without it
// the second m16 half of the MMA reads constant zeros and its x rows are never loaded.
template <typename T, bool SWIGLU, int WPI, bool HI>
__global__ void __launch_bounds__(256, 2) skinny_gemm_kernel(const SkParams p, int n_items) {
  constexpr int NBLK = SWIGLU ? 2 : 1;
  constexpr int IPC = kSkWarps / WPI;  // items per CTA
  __shared__ float red[WPI > 1 ? kSkWarps : 1][NBLK][32][4];
  // Weight streaming does not depend on the shrink that precedes this kernel: with
  // wait_late the partial sums are formed while it runs, and only S waits.
  if (!p.wait_late) pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = warp / WPI, part = warp - slot * WPI;
  const int g = lane >> 2, tig = lane & 3;
  const int nblocks = (p.N + kSkNB - 1) / kSkNB;
  const int item = blockIdx.x * IPC + slot;
  const int m = item / nblocks, n0 = (item - m * nblocks) * kSkNB;
  const int ntiles = p.tile_group ? min(*p.num_tiles_dev, p.tiles_cap) : (int)((p.m_rows + 127) / 128);
  int group = 0;
  int64_t valid = 0;
  if (item < n_items && m < ntiles) {
    group = p.tile_group ? p.tile_group[m] : 0;
    valid = p.tile_group ? (int64_t)p.group_counts[group] - ((int64_t)m * 128 - p.group_offsets[group])
                         : p.m_rows - (int64_t)m * 128;
    valid = valid < 0 ? 0 : (valid > 16 ? 16 : valid);
  }
  const int K = p.K;
  const T* A = static_cast<const T*>(p.a);
  const T* W = static_cast<const T*>(p.b);
  const int64_t row0 = (int64_t)m * 128;
  float acc[NBLK][4];
#pragma unroll
  for (int b = 0; b < NBLK; ++b)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[b][j] = 0.f;
  if (valid > 0) {  // warp-uniform
    const int64_t r_lo = row0 + g, r_hi = row0 + g + 8;
    const T* x_lo = g < valid ? A + (p.a_row_of ? (int64_t)p.a_row_of[r_lo] : r_lo) * K : nullptr;
    const T* x_hi = (HI && g + 8 < valid) ? A + (p.a_row_of ? (int64_t)p.a_row_of[r_hi] : r_hi) * K : nullptr;
    const T* wrow[NBLK];
#pragma unroll
    for (int b = 0; b < NBLK; ++b) {
      const int64_t r = (int64_t)weight_group(p.b_group_map, group) * p.b_group_rows + n0 + g + (b ? p.N : 0);
      wrow[b] = (n0 + g < p.N && r < p.b_rows_total) ? W + r * K : nullptr;
    }
    const int kw = ((K + WPI * 32 - 1) / (WPI * 32)) * 32;
    const int kb = part * kw, ke = min(K, kb + kw);
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int k0 = kb; k0 < ke; k0 += 32 * kSkUnroll) {
      uint4 xl[kSkUnroll], xh[kSkUnroll], w[kSkUnroll][NBLK];
#pragma unroll
      for (int u = 0; u < kSkUnroll; ++u) {
        const int kk = k0 + u * 32 + tig * 8;
        const bool v = kk < ke;
        xl[u] = (v && x_lo) ? ldg16(x_lo + kk) : z;
        if constexpr (HI)
          xh[u] = (v && x_hi) ? ldg16(x_hi + kk) : z;
        else
          xh[u] = z;
#pragma unroll
        for (int b = 0; b < NBLK; ++b) w[u][b] = (v && wrow[b]) ? ldg16_stream(wrow[b] + kk) : z;
      }
#pragma unroll
      for (int u = 0; u < kSkUnroll; ++u) sk_chunk<T, NBLK>(acc, xl[u], xh[u], w[u]);
    }
  }
  if (WPI > 1) {
#pragma unroll
    for (int b = 0; b < NBLK; ++b)
#pragma unroll
      for (int j = 0; j < 4; ++j) red[WPI > 1 ? warp : 0][b][lane][j] = acc[b][j];
    __syncthreads();
    if (part == 0) {
#pragma unroll
      for (int q = 1; q < WPI; ++q)
#pragma unroll
        for (int b = 0; b < NBLK; ++b)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[b][j] += red[WPI > 1 ? warp + q : 0][b][lane][j];
    }
  }
  // Every thread waits, so this grid completes only after the kernel before it.
  if (p.wait_late) pdl_wait();
  if (part != 0 || valid == 0) return;
  T* out = static_cast<T*>(p.out);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = g + (j >= 2 ? 8 : 0), c = tig * 2 + (j & 1);
    const int col = n0 + c;
    if (r >= valid || col >= p.N) continue;
    const int64_t row = row0 + r;
    float v0 = acc[0][j];
    float v1 = SWIGLU ? acc[NBLK - 1][j] : 0.f;
    if (p.rank > 0) {
      const int t = p.row_tenant[row];
      if (t >= 0) {
        const T* S = static_cast<const T*>(p.s16) + row * p.lora_cols;
        const T* Bl = static_cast<const T*>(p.lora_b) + t * p.lb_tenant_stride + group * p.lb_group_stride;
        const T* b0 = Bl + (int64_t)col * p.rank;
        float d0 = 0.f, d1 = 0.f;
        for (int q = 0; q < p.rank; ++q) d0 += to_f32<T>(S[q]) * to_f32<T>(b0[q]);
        if (SWIGLU) {
          const T* b1 = Bl + (int64_t)(p.N + col) * p.rank;
          for (int q = 0; q < p.rank; ++q) d1 += to_f32<T>(S[p.rank + q]) * to_f32<T>(b1[q]);
        }
        v0 += d0;
        v1 += d1;
      }
    }
    if (SWIGLU) {
      if (p.b_scale) {
        const float* bs = p.b_scale + (int64_t)weight_group(p.b_group_map, group) * p.b_group_rows;
        v0 *= bs[col];
        v1 *= bs[p.N + col];
      }
      out[row * p.ldo + col] = from_f32<T>(silu_f32(v0) * v1);
    } else {
      if (p.b_scale) v0 *= p.b_scale[(int64_t)weight_group(p.b_group_map, group) * p.b_group_rows + col];
      if (p.bias) {
        const int bg = p.bias_group_mod > 0 ? group % p.bias_group_mod : group;
        v0 += to_f32<T>(static_cast<const T*>(p.bias)[bg * p.bias_group_stride + col]);
      }
      if (p.row_scale) v0 *= p.row_scale[row];
      out[row * p.ldo + col] = from_f32<T>(v0);
    }
  }
}

template <typename T, bool SWIGLU, bool HI>
cudaError_t launch_sk_hi(int wpi, int n_items, const SkParams& p, cudaStream_t stream, bool pdl) {
  const dim3 grid((unsigned)(((int64_t)n_items * wpi + kSkWarps - 1) / kSkWarps)), block(256);
  ::sb::count_launch();
  switch (wpi) {
    case 1:
      return launch_kernel(skinny_gemm_kernel<T, SWIGLU, 1, HI>, grid, block, 0, stream, pdl, p, n_items);
    case 2:
      return launch_kernel(skinny_gemm_kernel<T, SWIGLU, 2, HI>, grid, block, 0, stream, pdl, p, n_items);
    case 4:
      return launch_kernel(skinny_gemm_kernel<T, SWIGLU, 4, HI>, grid, block, 0, stream, pdl, p, n_items);
    default:
      return launch_kernel(skinny_gemm_kernel<T, SWIGLU, 8, HI>, grid, block, 0, stream, pdl, p, n_items);
  }
}

template <typename T, bool SWIGLU>
cudaError_t launch_sk(int wpi, int n_items, bool hi, const SkParams& p, cudaStream_t stream, bool pdl) {
  return hi ? launch_sk_hi<T, SWIGLU, true>(wpi, n_items, p, stream, pdl)
            : launch_sk_hi<T, SWIGLU, false>(wpi, n_items, p, stream, pdl);
}

}  // namespace

int launch_skinny_gemm(const GemmLaunch& g, const int32_t* row_tenant, const int32_t* group_offsets,
                       const int32_t* group_counts, cudaStream_t stream, int64_t max_rows, int pdl_mode) {
  SB_CHECK_ARG(g.a && g.b && g.out, "skinny gemm: null operand");
  SB_CHECK_ARG(!g.b_fp8, "skinny gemm: 16-bit weights only");
  SB_CHECK_ARG(g.K > 0 && g.K % 8 == 0 && g.N > 0, "skinny gemm: K=%d must be a positive multiple of 8", g.K);
  SB_CHECK_ARG(!g.tile_group || (g.num_tiles_dev && group_offsets && group_counts),
               "skinny gemm: grouped rows need the tile count, group offsets and counts");
  SB_CHECK_ARG(g.rank == 0 || (g.s16 && g.lora_b && row_tenant), "skinny gemm: LoRA needs S, B and the row tenants");
  SB_CHECK_ARG((reinterpret_cast<uintptr_t>(g.a) % 16) == 0 && (reinterpret_cast<uintptr_t>(g.b) % 16) == 0,
               "skinny gemm: operands must be 16-byte aligned");
  SkParams p;
  p.a = g.a;
  p.a_row_of = g.a_row_of;
  p.K = g.K;
  p.b = g.b;
  p.b_rows_total = g.b_rows_total;
  p.b_group_rows = g.b_group_rows;
  p.b_group_map = g.b_group_map;
  p.N = g.N;
  p.num_tiles_dev = g.num_tiles_dev;
  p.tiles_cap = g.tiles_cap;
  p.tile_group = g.tile_group;
  p.group_offsets = group_offsets;
  p.group_counts = group_counts;
  p.m_rows = g.m_rows;
  p.row_tenant = row_tenant;
  p.rank = g.rank;
  p.lora_cols = g.swiglu ? 2 * g.rank : g.rank;
  p.s16 = g.s16;
  p.lora_b = g.lora_b;
  p.lb_tenant_stride = g.lora_b_tenant_stride;
  p.lb_group_stride = g.lora_b_group_stride;
  p.row_scale = g.row_scale;
  p.bias = g.bias;
  p.bias_group_stride = g.bias_group_stride;
  p.bias_group_mod = g.bias_group_mod;
  p.b_scale = g.b_scale;
  p.out = g.out;
  p.ldo = g.ldo;
  p.wait_late = pdl_mode == 2;
  const int64_t tiles = g.tile_group ? (int64_t)g.tiles_cap : (g.m_rows + 127) / 128;
  if (tiles == 0) return STAGEML_OK;
  const int64_t items = tiles * ((g.N + kSkNB - 1) / kSkNB);
  SB_CHECK_ARG(items * 8 < (int64_t(1) << 31), "skinny gemm: too many output blocks");
  // Warps per item from K alone (so a row's sums do not depend on the batch): one
  // warp per ~3-6K of K, at most 8.
  int wpi = 1;
  while (wpi < 8 && g.K >= wpi * 2 * 3072) wpi *= 2;
  const bool hi = max_rows > 8;  // a tile holds at most max_rows valid rows
  const bool pdl = pdl_mode != 0;
  cudaError_t e;
  if (g.in_bf16)
    e = g.swiglu ? launch_sk<bf16, true>(wpi, (int)items, hi, p, stream, pdl)
                 : launch_sk<bf16, false>(wpi, (int)items, hi, p, stream, pdl);
  else
    e = g.swiglu ? launch_sk<f16, true>(wpi, (int)items, hi, p, stream, pdl)
                 : launch_sk<f16, false>(wpi, (int)items, hi, p, stream, pdl);
  SB_CUDA_CHECK(e);
  return STAGEML_OK;
}

}  // namespace sb
