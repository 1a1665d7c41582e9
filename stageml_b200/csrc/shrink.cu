// Row gather into the permuted layout (R2) and the LoRA shrink (R4):
//   S[row, :] = scale[tenant(row)] * x[src(row), :] . A[tenant(row), group(row)]^T
// A is [R, K] per (tenant, group) with R = rank (or 2*rank for the packed w1|w3
// factors). This is the (xs @ A[e].t()) half of the LoRA branch in
// RequestExecutor.dynamic_one (benchmarks/multitenant_bta_system_bench.py:409),
// DynamicMoELoRALayer.forward (stageml/moe_lora_layers.py:88) and
// DynamicLoRALinear.forward (stageml/adapter_bank.py:67).
//
// The shrink is a GEMM with a tiny N (R <= 64) whose B operand changes with the
// row's tenant; it is bound by reading x and the touched A slices, so the
// kernel is built for bytes in flight: one warp owns 16 rows and one 512-wide
// K slice, rows of the same tenant (contiguous after the (expert, tenant) sort)
// share one pass over A, and the warp's (pass, 64-wide chunk) items stream
// through a 4-stage cp.async ring in shared memory feeding ldmatrix and
// warp-level tensor-core MMAs (m16n8k16, fp32 accumulate). K slices write fp32
// partials that a second kernel sums in a fixed order and scales, so the result
// is deterministic. The first pass also writes the staged x rows to the
// permuted activation buffer.
#include <cstdlib>
#include <cstring>

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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  // src-size 0 fills the 16 bytes with zeros (rows without a source, K past the end)
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Shared-memory ring of one warp: each stage holds a 64-wide K chunk of the warp's
// 16 rows of x and of the R rows of one tenant's A, rows padded to 144 bytes so
// that the eight 16-byte row segments an ldmatrix reads fall in distinct banks.
constexpr int kShrinkKC = 64;
constexpr int kShrinkPitch = kShrinkKC * 2 + 16;
constexpr int kShrinkStages = 4;
constexpr int kShrinkMaxPasses = 16;

template <int NBS>
struct ShrinkRing {
  static constexpr int R = NBS * 8;
  static constexpr int X_BYTES = 16 * kShrinkPitch;
  static constexpr int STAGE = X_BYTES + R * kShrinkPitch;
  static constexpr int WARP_BYTES = kShrinkStages * STAGE;
  static constexpr int SMEM = 4 * WARP_BYTES + 4 * kShrinkMaxPasses * 8;
};

// One warp: 16 consecutive rows, one 512-wide K slice. The distinct tenants of
// the rows are the warp's passes (rows of one tenant are contiguous after the
// (expert, tenant) sort, so there are few); the (pass, 64-wide chunk) items
// stream through a 4-stage cp.async ring so that about three chunks of x and A
// are in flight per warp. The first pass also copies the staged x rows to the
// permuted activation buffer.
template <typename T, int NBS>
__global__ void __launch_bounds__(128) gather_shrink_kernel(const ShrinkParams p) {
  using Ring = ShrinkRing<NBS>;
  constexpr int R = Ring::R;
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_wait();  // the plan and the source rows may come from the previous kernels
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows_active = active_rows(p.num_tiles_dev, p.static_rows, p.rows_cap);
  const int64_t row0 = (int64_t)blockIdx.y * 64 + warp * 16;
  if (row0 >= rows_active) return;
  const int K = p.K;
  const int k_begin = blockIdx.x * kShrinkKSlice;
  const int k_end = min(K, k_begin + kShrinkKSlice);
  const int nkc = (k_end - k_begin + kShrinkKC - 1) / kShrinkKC;
  const T* src = static_cast<const T*>(p.src);
  uint8_t* ring = smem + warp * Ring::WARP_BYTES;
  int32_t* s_key = reinterpret_cast<int32_t*>(smem + 4 * Ring::WARP_BYTES) + warp * 2 * kShrinkMaxPasses;
  uint32_t* s_sel = reinterpret_cast<uint32_t*>(s_key + kShrinkMaxPasses);

  // passes: distinct tenants of the 16 rows, first-seen order
  int np = 0;
  if (R > 0) {
    const int my_tenant = (lane < 16 && row0 + lane < rows_active) ? p.row_tenant[row0 + lane] : -1;
    unsigned pending = __ballot_sync(0xffffffffu, lane < 16 && my_tenant >= 0) & 0xFFFFu;
    while (pending) {
      const int leader = __ffs(pending) - 1;
      const int key = __shfl_sync(0xffffffffu, my_tenant, leader);
      const unsigned sel = __ballot_sync(0xffffffffu, lane < 16 && my_tenant == key) & pending;
      pending &= ~sel;
      if (lane == 0) {
        s_key[np] = key;
        s_sel[np] = sel;
      }
      ++np;
    }
    __syncwarp();
  }
  const bool gather = p.gather_dst != nullptr;
  const int npass = np > 0 ? np : (gather ? 1 : 0);
  if (npass == 0) return;
  const int total = npass * nkc;
  const int group = p.tile_group ? p.tile_group[row0 / 128] : 0;
  const T* lora_a = static_cast<const T*>(p.lora_a);

  // x pieces of this lane: rows (lane >> 3) + 4q, 16-byte column lane & 7 of the chunk
  const int xc = lane & 7;
  const T* xrow[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t row = row0 + (lane >> 3) + 4 * q;
    int64_t sr = -1;
    if (row < rows_active) sr = p.src_row_of ? (int64_t)p.src_row_of[row] : row;
    xrow[q] = sr >= 0 ? src + sr * K : nullptr;
  }

  auto issue = [&](int i) {
    if (i < total) {
      const int pass = i / nkc, kc = i - pass * nkc;
      const uint32_t st = smem_u32(ring + (i % kShrinkStages) * Ring::STAGE);
      const int kk = k_begin + kc * kShrinkKC + xc * 8;
      const bool kv = kk < k_end;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = (lane >> 3) + 4 * q;
        const bool v = kv && xrow[q] != nullptr;
        cp_async16(st + r * kShrinkPitch + xc * 16, v ? (const void*)(xrow[q] + kk) : p.src, v);
      }
      if (R > 0 && pass < np) {
        const T* A = lora_a + s_key[pass] * p.a_tenant_stride + group * p.a_group_stride;
#pragma unroll
        for (int q = 0; q < R / 4; ++q) {
          const int ar = (lane >> 3) + 4 * q;
          cp_async16(st + Ring::X_BYTES + ar * kShrinkPitch + xc * 16, kv ? (const void*)(A + (int64_t)ar * K + kk) : p.src,
                     kv);
        }
      }
    }
    cp_async_commit();  // possibly empty: keeps the group count in step
  };

  float acc[NBS > 0 ? NBS : 1][4];
  const int g = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int i = 0; i < kShrinkStages - 1; ++i) issue(i);
  for (int i = 0; i < total; ++i) {
    issue(i + kShrinkStages - 1);
    cp_async_wait<kShrinkStages - 1>();
    __syncwarp();
    const int pass = i / nkc, kc = i - pass * nkc;
    const uint8_t* st = ring + (i % kShrinkStages) * Ring::STAGE;
    if (pass == 0 && gather) {
      T* dstb = static_cast<T*>(p.gather_dst);
      const int kk = k_begin + kc * kShrinkKC + xc * 8;
      if (kk < k_end) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int r = (lane >> 3) + 4 * q;
          if (row0 + r < rows_active)
            *reinterpret_cast<uint4*>(dstb + (row0 + r) * K + kk) =
                *reinterpret_cast<const uint4*>(st + r * kShrinkPitch + xc * 16);
        }
      }
    }
    if (NBS > 0 && pass < np) {
      if (kc == 0) {
#pragma unroll
        for (int nb = 0; nb < (NBS > 0 ? NBS : 1); ++nb)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[nb][j] = 0.f;
      }
      const uint32_t xs = smem_u32(st), as = smem_u32(st + Ring::X_BYTES);
      const int mi = lane >> 3, mr = lane & 7;
#pragma unroll
      for (int k16 = 0; k16 < kShrinkKC / 16; ++k16) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(xs + ((mi & 1) * 8 + mr) * kShrinkPitch + (k16 * 16 + (mi >> 1) * 8) * 2, a0, a1, a2, a3);
#pragma unroll
        for (int nb = 0; nb + 1 < NBS; nb += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(as + ((nb + (mi >> 1)) * 8 + mr) * kShrinkPitch + (k16 * 16 + (mi & 1) * 8) * 2, b0, b1, b2, b3);
          mma_16816<T>(acc[nb], a0, a1, a2, a3, b0, b1);
          mma_16816<T>(acc[nb + 1], a0, a1, a2, a3, b2, b3);
        }
        if constexpr ((NBS & 1) != 0) {  // a last single block of 8 output columns
          uint32_t b0, b1;
          ldsm_x2(as + ((NBS - 1) * 8 + mr) * kShrinkPitch + (k16 * 16 + (mi & 1) * 8) * 2, b0, b1);
          mma_16816<T>(acc[NBS - 1], a0, a1, a2, a3, b0, b1);
        }
      }
      if (kc == nkc - 1) {
        const unsigned sel = s_sel[pass];
        float* sp = p.spart + (int64_t)blockIdx.x * p.rows_cap * R;
        const int64_t r_lo = row0 + g, r_hi = row0 + g + 8;
        const bool lo_sel = (sel >> g) & 1u, hi_sel = (sel >> (g + 8)) & 1u;
#pragma unroll
        for (int nb = 0; nb < NBS; ++nb) {
          const int col = nb * 8 + tig * 2;
          if (lo_sel) *reinterpret_cast<float2*>(sp + r_lo * R + col) = make_float2(acc[nb][0], acc[nb][1]);
          if (hi_sel) *reinterpret_cast<float2*>(sp + r_hi * R + col) = make_float2(acc[nb][2], acc[nb][3]);
        }
      }
    }
    __syncwarp();  // the stage is refilled by a later issue
  }
  cp_async_wait<0>();
}

// S[row, c] = scale[tenant] * sum over K slices (fixed order) of the partials; one
// thread per 8 output columns of a row (two 16-byte partial loads per slice, one
// 16-byte store). With row_run (rank 8 on the one-CTA GEMM): each 8-column group of
// S is written as 16 columns, the values in the half given by the parity of the
// row's run index in its tile and zeros in the other, so that one K = 16 expand step
// serves two runs.
template <typename T>
__global__ void shrink_reduce_kernel(const float* __restrict__ spart, int KS, int64_t rows_cap, int R,
                                     const int32_t* __restrict__ num_tiles_dev, int64_t static_rows,
                                     const int32_t* __restrict__ row_tenant, const float* __restrict__ scale,
                                     T* __restrict__ s_out, const int8_t* __restrict__ row_run) {
  pdl_wait();  // the partial sums of the kernel before
  pdl_trigger();
  const int64_t rows_active = active_rows(num_tiles_dev, static_rows, rows_cap);
  const int G_out = (row_run ? 2 * R : R) / 8;  // 8-column output groups per row
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows_active * G_out) return;
  const int64_t row = idx / G_out;
  const int og = (int)(idx - row * G_out);
  int c0 = og * 8;  // first input column
  bool live = true;
  if (row_run) {  // output group og = input group (og / 2) in parity half (og & 1)
    const int run = row_run[row];
    c0 = (og >> 1) * 8;
    live = run >= 0 && ((run & 1) == (og & 1));
  }
  const int tn = row_tenant[row];
  float v[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) v[q] = 0.f;
  if (tn >= 0 && live) {
    const float4* src = reinterpret_cast<const float4*>(spart + row * R + c0);
    const int64_t step = rows_cap * R / 4;  // one K slice, in float4
    for (int ks0 = 0; ks0 < KS; ks0 += 4) {  // four slices' loads in flight, added in slice order
      float4 lo[4], hi[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (ks0 + u < KS) {
          lo[u] = __ldg(src + (ks0 + u) * step);
          hi[u] = __ldg(src + (ks0 + u) * step + 1);
        }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (ks0 + u < KS) {
          v[0] += lo[u].x, v[1] += lo[u].y, v[2] += lo[u].z, v[3] += lo[u].w;
          v[4] += hi[u].x, v[5] += hi[u].y, v[6] += hi[u].z, v[7] += hi[u].w;
        }
    }
    const float sc = scale ? scale[tn] : 1.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] *= sc;
  }
  *reinterpret_cast<uint4*>(s_out + row * (G_out * 8) + og * 8) = pack8<T>(v);
}

// The same sums one output column per thread, for many K slices (each thread's
// slices are a dependent chain, so more threads keep more loads in flight).
template <typename T>
__global__ void shrink_reduce_scalar_kernel(const float* __restrict__ spart, int KS, int64_t rows_cap, int R,
                                            const int32_t* __restrict__ num_tiles_dev, int64_t static_rows,
                                            const int32_t* __restrict__ row_tenant, const float* __restrict__ scale,
                                            T* __restrict__ s_out, const int8_t* __restrict__ row_run) {
  pdl_wait();  // the partial sums of the kernel before
  pdl_trigger();
  const int64_t rows_active = active_rows(num_tiles_dev, static_rows, rows_cap);
  const int R_out = row_run ? 2 * R : R;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows_active * R_out) return;
  const int64_t row = idx / R_out;
  const int oc = (int)(idx - row * R_out);
  int c = oc;
  bool live = true;
  if (row_run) {  // output column oc = group (8 input columns) x 16 + parity x 8 + column
    const int run = row_run[row];
    c = (oc >> 4) * 8 + (oc & 7);
    live = run >= 0 && ((run & 1) == ((oc >> 3) & 1));
  }
  const int tn = row_tenant[row];
  float v = 0.f;
  if (tn >= 0 && live) {
    for (int ks = 0; ks < KS; ++ks) v += spart[((int64_t)ks * rows_cap + row) * R + c];
    v *= scale ? scale[tn] : 1.f;
  }
  s_out[idx] = from_f32<T>(v);
}

// Up to this many K slices a thread takes 8 output columns.
constexpr int kReduceVecMaxSlices = 4;

template <int NBS>
int launch_shrink_variant(bool bf, dim3 grid, const ShrinkParams& p, cudaStream_t stream, bool pdl) {
  constexpr int smem = ShrinkRing<NBS>::SMEM;
  if (bf) {
    SB_CUDA_CHECK(cudaFuncSetAttribute(gather_shrink_kernel<bf16, NBS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    SB_CUDA_CHECK(launch_kernel(gather_shrink_kernel<bf16, NBS>, grid, dim3(128), smem, stream, pdl, p));
  } else {
    SB_CUDA_CHECK(cudaFuncSetAttribute(gather_shrink_kernel<f16, NBS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    SB_CUDA_CHECK(launch_kernel(gather_shrink_kernel<f16, NBS>, grid, dim3(128), smem, stream, pdl, p));
  }
  ::sb::count_launch();
  return STAGEML_OK;
}

// Decode-sized batches: CTA (pair, nb) computes S[row, 8nb .. 8nb+8) for the pair's
// plan row; warp w sums its K range [w kw, (w+1) kw) with 16-byte loads, all of
// them in flight, and the 8 warp sums are added in warp order.
struct PairShrinkParams {
  const void* src;
  const int32_t* src_row_of;
  int K;
  const int32_t* pair_row;
  const int32_t* row_tenant;
  const int32_t* tile_group;
  const void* lora_a;
  int64_t a_tenant_stride;
  int64_t a_group_stride;
  int R;
  const float* lora_scale;
  void* s_out;
};

__device__ __forceinline__ uint4 ldg16_nc(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32<T>(h[i]);
}

template <typename T>
__global__ void __launch_bounds__(256, 1) pair_shrink_kernel(const PairShrinkParams p) {
  constexpr int U = 4;
  __shared__ float red[8][8];
  pdl_wait();  // the plan and the source rows may come from the previous kernels
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = p.pair_row ? p.pair_row[blockIdx.x] : (int)blockIdx.x;  // no map: pair i is row i
  if (row < 0) return;  // dropped pair
  const int tn = p.row_tenant[row];
  T* s_out = static_cast<T*>(p.s_out) + (int64_t)row * p.R + blockIdx.y * 8;
  if (tn < 0) {
    if (threadIdx.x < 8) s_out[threadIdx.x] = from_f32<T>(0.f);
    return;
  }
  const int K = p.K;
  const int group = p.tile_group ? p.tile_group[row / 128] : 0;
  const T* x = static_cast<const T*>(p.src) + (p.src_row_of ? (int64_t)p.src_row_of[row] : (int64_t)row) * K;
  const T* A = static_cast<const T*>(p.lora_a) + tn * p.a_tenant_stride + group * p.a_group_stride +
               (int64_t)(blockIdx.y * 8) * K;
  const int kw = ((K + 63) / 64) * 8;
  const int kb = warp * kw, ke = min(K, kb + kw);
  float acc[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) acc[r] = 0.f;
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int k0 = kb + lane * 8; k0 < ke; k0 += 256 * U) {
    uint4 xv[U], av[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + 256 * u;
      const bool v = k < ke;
      xv[u] = v ? __ldg(reinterpret_cast<const uint4*>(x + k)) : z;
#pragma unroll
      for (int r = 0; r < 8; ++r) av[u][r] = v ? ldg16_nc(A + (int64_t)r * K + k) : z;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float xf[8];
      unpack8<T>(xv[u], xf);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        float af[8];
        unpack8<T>(av[u][r], af);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[r] = fmaf(xf[q], af[q], acc[r]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < 8; ++r) red[warp][r] = acc[r];
  }
  __syncthreads();
  if (threadIdx.x < 8) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) v += red[w][threadIdx.x];
    s_out[threadIdx.x] = from_f32<T>(v * (p.lora_scale ? p.lora_scale[tn] : 1.f));
  }
}

// STAGEML_SHRINK (read once per process): "mma" keeps every shrink on the per-warp
// mma.sync kernel; "tc" (default) runs shrinks of rows already in place with at
// least 16 output columns on the tensor-core kernel; "tc_all" runs every shrink
// there, gathered rows after a gather-only pass. With 8 columns a slot's A rows are
// 1 KB copies, and the per-copy cost of ~14 of them per K block made the
// tensor-core kernel slower than the per-warp one (fine-grained layer's h shrink:
// 0.174 vs 0.123 ms); with 16 it is faster (Mixtral layer's: 0.071 vs 0.075 ms).
enum ShrinkMode { kShrinkWarpMma = 0, kShrinkTcInPlace = 1, kShrinkTcAll = 2 };
int shrink_mode() {
  static const int mode = [] {
    const char* e = getenv("STAGEML_SHRINK");
    if (!e) return (int)kShrinkTcInPlace;
    if (!strcmp(e, "mma")) return (int)kShrinkWarpMma;
    if (!strcmp(e, "tc_all")) return (int)kShrinkTcAll;
    return (int)kShrinkTcInPlace;
  }();
  return mode;
}

}  // namespace

int launch_pair_shrink(const ShrinkLaunch& s, const int32_t* pair_row, int64_t P, cudaStream_t stream, bool pdl) {
  SB_CHECK_ARG(s.src && s.lora_a && s.s_out && s.row_tenant, "pair shrink: missing buffers");
  SB_CHECK_ARG(s.K > 0 && s.K % 8 == 0, "pair shrink: K=%d must be a positive multiple of 8", s.K);
  SB_CHECK_ARG(s.R > 0 && s.R % 8 == 0 && s.R <= 64, "pair shrink: R=%d must be a multiple of 8 up to 64", s.R);
  SB_CHECK_ARG(P >= 0 && P <= 65535, "pair shrink: %lld pairs", (long long)P);
  SB_CHECK_ARG(reinterpret_cast<uintptr_t>(s.src) % 16 == 0 && reinterpret_cast<uintptr_t>(s.lora_a) % 16 == 0,
               "pair shrink: operands must be 16-byte aligned");
  if (P == 0) return STAGEML_OK;
  PairShrinkParams p;
  p.src = s.src;
  p.src_row_of = s.src_row_of;
  p.K = s.K;
  p.pair_row = pair_row;
  p.row_tenant = s.row_tenant;
  p.tile_group = s.tile_group;
  p.lora_a = s.lora_a;
  p.a_tenant_stride = s.a_tenant_stride;
  p.a_group_stride = s.a_group_stride;
  p.R = s.R;
  p.lora_scale = s.lora_scale;
  p.s_out = s.s_out;
  const dim3 grid((unsigned)P, (unsigned)(s.R / 8));
  if (s.dtype_bf16)
    SB_CUDA_CHECK(launch_kernel(pair_shrink_kernel<bf16>, grid, dim3(256), 0, stream, pdl, p));
  else
    SB_CUDA_CHECK(launch_kernel(pair_shrink_kernel<f16>, grid, dim3(256), 0, stream, pdl, p));
  ::sb::count_launch();
  return STAGEML_OK;
}

int launch_gather_shrink(const ShrinkLaunch& s, cudaStream_t stream) {
  SB_CHECK_ARG(s.src, "shrink: null source");
  SB_CHECK_ARG(s.K > 0 && s.K % 8 == 0, "shrink: K=%d must be a positive multiple of 8", s.K);
  SB_CHECK_ARG(s.R == 0 || s.R == 8 || s.R == 16 || s.R == 32 || s.R == 64, "shrink: R=%d must be 0, 8, 16, 32 or 64",
               s.R);
  SB_CHECK_ARG(s.R == 0 || (s.lora_a && s.spart && s.s_out && s.row_tenant), "shrink: missing LoRA buffers");
  SB_CHECK_ARG(reinterpret_cast<uintptr_t>(s.src) % 16 == 0, "shrink: source must be 16-byte aligned");
  if (!s.gather_dst && s.R == 0) return STAGEML_OK;
  const int KS = shrink_num_slices(s.K);
  const int64_t rows_max = s.num_tiles_dev ? s.rows_cap : s.static_rows;
  if (rows_max == 0) return STAGEML_OK;
  // Tensor-core shrink: rows in place, or the gathered rows once the gather wrote them.
  ShrinkLaunch in_place = s;
  bool tc = false;
  if (s.R > 0 && shrink_mode() != kShrinkWarpMma) {
    if (!s.gather_dst) {
      tc = tc_shrink_supported(s) && (s.R >= 16 || shrink_mode() == kShrinkTcAll);
    } else if (shrink_mode() == kShrinkTcAll) {
      in_place.src = s.gather_dst;
      in_place.src_row_of = nullptr;
      in_place.gather_dst = nullptr;
      tc = tc_shrink_supported(in_place);
    }
  }
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
  if (tc) {
    if (s.gather_dst) {  // the gather alone first
      p.R = 0;
      SB_TRY(launch_shrink_variant<0>(s.dtype_bf16, grid, p, stream, s.pdl));
    }
    SB_TRY(launch_tc_shrink(in_place, in_place.src, stream));
  } else {
  switch (s.R / 8) {
    case 0:
      SB_TRY(launch_shrink_variant<0>(s.dtype_bf16, grid, p, stream, s.pdl));
      break;
    case 1:
      SB_TRY(launch_shrink_variant<1>(s.dtype_bf16, grid, p, stream, s.pdl));
      break;
    case 2:
      SB_TRY(launch_shrink_variant<2>(s.dtype_bf16, grid, p, stream, s.pdl));
      break;
    case 4:
      SB_TRY(launch_shrink_variant<4>(s.dtype_bf16, grid, p, stream, s.pdl));
      break;
    case 8:
      SB_TRY(launch_shrink_variant<8>(s.dtype_bf16, grid, p, stream, s.pdl));
      break;
    default:
      return set_error(STAGEML_ERR_INVALID_ARG, "shrink: R=%d must be 0, 8, 16, 32 or 64", s.R);
  }
  }
  SB_CUDA_CHECK(cudaGetLastError());
  if (s.R > 0) {
    SB_CHECK_ARG(!s.row_run || s.R % 8 == 0, "shrink: the run-parity layout needs R a multiple of 8");
    SB_CHECK_ARG(reinterpret_cast<uintptr_t>(s.spart) % 16 == 0 && reinterpret_cast<uintptr_t>(s.s_out) % 16 == 0,
                 "shrink: partials and S must be 16-byte aligned");
    const bool vec = KS <= kReduceVecMaxSlices;
    const int64_t n = rows_max * (s.row_run ? 2 * s.R : s.R) / (vec ? 8 : 1);
    const dim3 rgrid((unsigned)((n + 255) / 256));
    if (s.dtype_bf16)
      SB_CUDA_CHECK(launch_kernel(vec ? shrink_reduce_kernel<bf16> : shrink_reduce_scalar_kernel<bf16>, rgrid,
                                  dim3(256), 0, stream, s.pdl, s.spart, KS, p.rows_cap, s.R, s.num_tiles_dev,
                                  s.static_rows, s.row_tenant, s.lora_scale, static_cast<bf16*>(s.s_out), s.row_run));
    else
      SB_CUDA_CHECK(launch_kernel(vec ? shrink_reduce_kernel<f16> : shrink_reduce_scalar_kernel<f16>, rgrid,
                                  dim3(256), 0, stream, s.pdl, s.spart, KS, p.rows_cap, s.R, s.num_tiles_dev,
                                  s.static_rows, s.row_tenant, s.lora_scale, static_cast<f16*>(s.s_out), s.row_run));
    ::sb::count_launch();
    SB_CUDA_CHECK(cudaGetLastError());
  }
  return STAGEML_OK;
}

}  // namespace sb
