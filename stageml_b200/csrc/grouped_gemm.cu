// Grouped (per-expert / per-weight-group) GEMM on the 5th-generation tensor
// cores: TMA -> 128B-swizzled shared memory -> tcgen05.mma (cta_group::1,
// M=128, N=256, K=16, fp32 accumulators in TMEM) -> tcgen05.ld epilogue.
//
// One persistent CTA per SM, 6 warps:
//   warp 0      TMA producer (one thread), 4-stage ring of 48 KB stages
//   warp 1      TMEM allocator + MMA issuer (one thread)
//   warps 2..5  epilogue: TMEM lane quarter (warp % 4), one accumulator row per thread
// Two 256-column accumulators in TMEM let the epilogue of tile i overlap the
// main loop of tile i+1.
//
// Epilogue (fused, CUDA cores, fp32):
//   LoRA expand: + sum_j S[row, j] * B_lora[tenant(row), group, col, j] (S already scaled)
//   SwiGLU:      h = silu(g) * u over the paired gate / up accumulators
//   plain:       (acc * b_scale[col] + bias[col] + lora) * row_scale[row]
// This is the per-(slot, expert) body of RequestExecutor.dynamic_one
// (benchmarks/multitenant_bta_system_bench.py:408-413) for a whole 128-row tile.
#include "common.cuh"
#include "grouped_gemm.cuh"
#include "host_util.h"

namespace sb {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;            // accumulator columns per tile (SwiGLU: 128 gate + 128 up)
constexpr int BK = 64;             // 64 x 16-bit = one 128 B swizzle row
constexpr int STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;         // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;         // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 2 * BN;                  // double-buffered accumulator
constexpr int NUM_THREADS = 192;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

struct KParams {
  int K;
  int N;
  int b_group_rows;
  int num_n_tiles;
  int swiglu;
  const int32_t* num_tiles_dev;
  int tiles_cap;
  const int32_t* tile_group;
  int64_t m_rows;
  const int32_t* row_tenant;
  const float* row_lora;
  int rank;
  int lora_cols;
  const void* lora_b;
  int64_t lora_b_tenant_stride;
  int64_t lora_b_group_stride;
  const float* row_scale;
  const void* bias;
  int64_t bias_group_stride;
  int bias_group_mod;
  const float* b_scale;
  void* out;
  int64_t ldo;
  int32_t* status;
  unsigned long long timeout_ns;
};

template <typename T>
struct IsBf16 {
  static constexpr int value = 0;
};
template <>
struct IsBf16<bf16> {
  static constexpr int value = 1;
};

template <typename T>
__device__ __forceinline__ void lora_expand16(float (&acc)[16], const float (&s)[32], int r8, const T* bp,
                                              int rank, int ncols_valid) {
  // acc[i] += sum_j s[j] * bp[i*rank + j] for the first ncols_valid columns.
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i < ncols_valid) {
      float sum = 0.f;
#pragma unroll
      for (int j8 = 0; j8 < 4; ++j8) {
        if (j8 < r8) {
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(bp + (int64_t)i * rank + j8 * 8));
          float f[8];
          unpack8<T>(u, f);
#pragma unroll
          for (int q = 0; q < 8; ++q) sum = fmaf(s[j8 * 8 + q], f[q], sum);
        }
      }
      acc[i] += sum;
    }
  }
}

template <typename T>
__device__ __forceinline__ void store16(T* dst, const float (&v)[16], int ncols_valid, bool vec_ok) {
  if (vec_ok && ncols_valid >= 16) {
    float lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      lo[i] = v[i];
      hi[i] = v[8 + i];
    }
    reinterpret_cast<uint4*>(dst)[0] = pack8<T>(lo);
    reinterpret_cast<uint4*>(dst)[1] = pack8<T>(hi);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < ncols_valid) dst[i] = from_f32<T>(v[i]);
  }
}

template <typename T>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const KParams p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars[0..S) full, [S..2S) empty, [2S..2S+2) tmem_full, [2S+2..2S+4) tmem_empty, [2S+4] drain
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t smem_base = smem_u32(smem);
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + 2 + a]); };
  const uint32_t drain_bar = smem_u32(&bars[2 * STAGES + 4]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_base_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  const int num_m_tiles = p.tile_group ? min(*p.num_tiles_dev, p.tiles_cap) : (int)((p.m_rows + BM - 1) / BM);
  const int total_tiles = num_m_tiles * p.num_n_tiles;
  const int num_kb = (p.K + BK - 1) / BK;
  volatile int never_abort = 0;  // the drain waits below ignore the abort flag

  if (threadIdx.x == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    const uint64_t pol_a = l2_policy_evict_last();
    const uint64_t pol_b = l2_policy_evict_normal();
    int last_phase[STAGES];
    for (int s = 0; s < STAGES; ++s) last_phase[s] = -1;
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
      const int m_tile = tile % num_m_tiles;
      const int n_tile = tile / num_m_tiles;
      const int group = p.tile_group ? p.tile_group[m_tile] : 0;
      const int a_row = m_tile * BM;
      int b_row0, b_row1;
      if (p.swiglu) {
        b_row0 = group * p.b_group_rows + n_tile * 128;
        b_row1 = b_row0 + p.N;
      } else {
        b_row0 = group * p.b_group_rows + n_tile * BN;
        b_row1 = b_row0 + 128;
      }
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(empty_bar(s), ph ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        const uint32_t sa = smem_base + s * STAGE_BYTES;
        const uint32_t sbm = sa + A_STAGE_BYTES;
        mbar_arrive_expect_tx(full_bar(s), STAGE_BYTES);
        tma_load_2d(sa, &tm_a, full_bar(s), kb * BK, a_row, pol_a);
        tma_load_2d(sbm, &tm_b, full_bar(s), kb * BK, b_row0, pol_b);
        tma_load_2d(sbm + 128 * BK * 2, &tm_b, full_bar(s), kb * BK, b_row1, pol_b);
        last_phase[s] = (int)ph;
      }
    }
    if (!ok) {
      // Let the copies already in flight land before the CTA exits.
      for (int s = 0; s < STAGES; ++s)
        if (last_phase[s] >= 0)
          mbar_wait(full_bar(s), (uint32_t)last_phase[s], &never_abort, p.status, 1000000000ull, kDevTimeoutDrain);
    }
  } else if (threadIdx.x == 32) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_f16(BM, BN, IsBf16<T>::value);
    uint32_t it = 0;
    int tcount = 0;
    bool ok = true;
    bool issued_any = false;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x, ++tcount) {
      const int acc = tcount & 1;
      const uint32_t aph = (tcount >> 1) & 1;
      if (!mbar_wait(tempty_bar(acc), aph ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(full_bar(s), ph, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_base + s * STAGE_BYTES;
        const uint64_t adesc = smem_desc_sw128(sa);
        const uint64_t bdesc = smem_desc_sw128(sa + A_STAGE_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        tc_commit(empty_bar(s));
        issued_any = true;
      }
      if (!ok) break;
      tc_commit(tfull_bar(acc));
    }
    if (!ok && issued_any) {
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, &never_abort, p.status, 1000000000ull, kDevTimeoutDrain);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const int r8 = p.rank / 8;
    const T* lora_b = reinterpret_cast<const T*>(p.lora_b);
    const T* bias = reinterpret_cast<const T*>(p.bias);
    T* out = reinterpret_cast<T*>(p.out);
    const bool vec_ok = (p.ldo % 8 == 0) && (p.N % 8 == 0);
    int tcount = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++tcount) {
      const int acc = tcount & 1;
      const uint32_t aph = (tcount >> 1) & 1;
      if (!mbar_wait(tfull_bar(acc), aph, abort_flag, p.status, p.timeout_ns, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int m_tile = tile % num_m_tiles;
      const int n_tile = tile / num_m_tiles;
      const int group = p.tile_group ? p.tile_group[m_tile] : 0;
      const int64_t row = (int64_t)m_tile * BM + row_in_tile;
      const bool row_ok = p.tile_group ? true : (row < p.m_rows);
      int tenant = -1;
      if (row_ok && p.row_tenant && p.rank > 0) tenant = p.row_tenant[row];
      float s_a[32], s_b[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        s_a[j] = 0.f;
        s_b[j] = 0.f;
      }
      if (tenant >= 0) {
        const float* sp = p.row_lora + row * p.lora_cols;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < p.rank) {
            s_a[j] = sp[j];
            if (p.swiglu) s_b[j] = sp[p.rank + j];
          }
      }
      const float rscale = (row_ok && p.row_scale) ? p.row_scale[row] : 1.f;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      const T* lb = (tenant >= 0) ? lora_b + tenant * p.lora_b_tenant_stride + group * p.lora_b_group_stride : nullptr;

      if (p.swiglu) {
        const int n0 = n_tile * 128;
        for (int c = 0; c < 128; c += 16) {
          uint32_t rg[16], ru[16];
          tmem_ld_x16(t_row + c, rg);
          tmem_ld_x16(t_row + 128 + c, ru);
          tmem_wait_ld();
          const int col = n0 + c;
          const int nvalid = min(16, p.N - col);
          float g[16], u[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            g[i] = __uint_as_float(rg[i]);
            u[i] = __uint_as_float(ru[i]);
          }
          if (p.b_scale && nvalid > 0) {
            const float* bsg = p.b_scale + (int64_t)group * p.b_group_rows + col;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (i < nvalid) {
                g[i] *= bsg[i];
                u[i] *= bsg[p.N + i];
              }
          }
          if (lb && nvalid > 0) {
            lora_expand16<T>(g, s_a, r8, lb + (int64_t)col * p.rank, p.rank, nvalid);
            lora_expand16<T>(u, s_b, r8, lb + (int64_t)(p.N + col) * p.rank, p.rank, nvalid);
          }
          float h[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) h[i] = silu_f32(g[i]) * u[i];
          if (row_ok && nvalid > 0) store16<T>(out + row * p.ldo + col, h, nvalid, vec_ok);
        }
      } else {
        const int n0 = n_tile * BN;
        for (int c = 0; c < BN; c += 16) {
          uint32_t rv[16];
          tmem_ld_x16(t_row + c, rv);
          tmem_wait_ld();
          const int col = n0 + c;
          const int nvalid = min(16, p.N - col);
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(rv[i]);
          if (nvalid > 0) {
            if (p.b_scale) {
              const float* bs = p.b_scale + (int64_t)group * p.b_group_rows + col;
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (i < nvalid) v[i] *= bs[i];
            }
            if (bias) {
              const int bg = p.bias_group_mod > 0 ? group % p.bias_group_mod : group;
              const T* bp = bias + bg * p.bias_group_stride + col;
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (i < nvalid) v[i] += to_f32<T>(bp[i]);
            }
            if (lb) lora_expand16<T>(v, s_a, r8, lb + (int64_t)col * p.rank, p.rank, nvalid);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] *= rscale;
            if (row_ok) store16<T>(out + row * p.ldo + col, v, nvalid, vec_ok);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace

int launch_grouped_gemm(const GemmLaunch& g, cudaStream_t stream) {
  SB_CHECK_ARG(g.a && g.b && g.out, "grouped gemm: null operand");
  SB_CHECK_ARG(g.K > 0 && g.K % 8 == 0, "grouped gemm: K=%d must be a positive multiple of 8", g.K);
  SB_CHECK_ARG(g.N > 0, "grouped gemm: N must be positive");
  SB_CHECK_ARG(g.rank % 8 == 0 && g.rank <= 32, "grouped gemm: LoRA rank %d must be a multiple of 8 <= 32", g.rank);
  SB_CHECK_ARG(g.rank == 0 || (g.row_lora && g.lora_b), "grouped gemm: LoRA rank > 0 needs S and B");
  SB_CHECK_ARG((reinterpret_cast<uintptr_t>(g.a) % 16) == 0 && (reinterpret_cast<uintptr_t>(g.b) % 16) == 0,
               "grouped gemm: operands must be 16-byte aligned");
  SB_CHECK_ARG(g.b_rows_total < (int64_t(1) << 31) && g.a_rows < (int64_t(1) << 31),
               "grouped gemm: operand rows exceed the TMA coordinate range");
  if (g.rank > 0) SB_CHECK_ARG(reinterpret_cast<uintptr_t>(g.lora_b) % 16 == 0, "grouped gemm: lora_b alignment");

  const CUtensorMapDataType dt = g.in_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tm_a, tm_b;
  SB_TRY(make_tmap_2d(&tm_a, g.a, dt, 2, (uint64_t)g.a_rows, (uint64_t)g.K, (uint64_t)g.K * 2, BM, BK, true));
  SB_TRY(make_tmap_2d(&tm_b, g.b, dt, 2, (uint64_t)g.b_rows_total, (uint64_t)g.K, (uint64_t)g.K * 2, 128, BK, true));

  KParams p;
  p.K = g.K;
  p.N = g.N;
  p.b_group_rows = g.b_group_rows;
  p.swiglu = g.swiglu ? 1 : 0;
  p.num_n_tiles = g.swiglu ? (g.N + 127) / 128 : (g.N + BN - 1) / BN;
  p.num_tiles_dev = g.num_tiles_dev;
  p.tiles_cap = g.tiles_cap;
  p.tile_group = g.tile_group;
  p.m_rows = g.m_rows;
  p.row_tenant = g.row_tenant;
  p.row_lora = g.row_lora;
  p.rank = g.rank;
  p.lora_cols = g.swiglu ? 2 * g.rank : g.rank;
  p.lora_b = g.lora_b;
  p.lora_b_tenant_stride = g.lora_b_tenant_stride;
  p.lora_b_group_stride = g.lora_b_group_stride;
  p.row_scale = g.row_scale;
  p.bias = g.bias;
  p.bias_group_stride = g.bias_group_stride;
  p.bias_group_mod = g.bias_group_mod;
  p.b_scale = g.b_scale;
  p.out = g.out;
  p.ldo = g.ldo;
  p.status = g.status;
  p.timeout_ns = kDefaultWaitNs;

  int64_t tiles_upper = g.tile_group ? (int64_t)g.tiles_cap : (g.m_rows + BM - 1) / BM;
  tiles_upper *= p.num_n_tiles;
  if (tiles_upper == 0) return STAGEML_OK;
  const int grid = (int)std::min<int64_t>(tiles_upper, sm_count());

  if (g.in_bf16) {
    static bool attr_set = false;
    if (!attr_set) {
      SB_CUDA_CHECK(cudaFuncSetAttribute(grouped_gemm_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES));
      attr_set = true;
    }
    (grouped_gemm_kernel<bf16><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tm_a, tm_b, p), ::sb::count_launch());
  } else {
    static bool attr_set = false;
    if (!attr_set) {
      SB_CUDA_CHECK(cudaFuncSetAttribute(grouped_gemm_kernel<f16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES));
      attr_set = true;
    }
    (grouped_gemm_kernel<f16><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tm_a, tm_b, p), ::sb::count_launch());
  }
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

}  // namespace sb
