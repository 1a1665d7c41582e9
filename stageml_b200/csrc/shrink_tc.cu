// LoRA shrink (R4) on the 5th-generation tensor cores for rows that already sit
// in the layout the GEMMs read (the SwiGLU output h of the down projection's LoRA,
// the gathered token rows, or a dense linear's rows in place):
//   S_part[slice, row, :] = x[row, slice] . A[tenant(row), group(tile)][:, slice]^T
// This is the (xs @ A[e].t()) half of the LoRA branch of
// DynamicMoELoRALayer.forward (stageml/moe_lora_layers.py:88) and
// RequestExecutor.dynamic_one (benchmarks/multitenant_bta_system_bench.py:409).
//
// Work item = (128-row tile, 512-wide K slice); a persistent CTA per SM takes a
// contiguous range of items (the K slices of one or a few tiles) with one TMA ring
// running across them:
//   warp 0      producer: x tile (128 x 64, 128B swizzle) + the A rows of every
//               distinct tenant ("slot") of the tile, stacked as the B operand
//   warp 1      TMEM allocator + MMA issuer: one unmasked M=128, N = slots x R
//               tcgen05.mma per K=16 step, so every row meets every slot's A
//   warps 2-5   epilogue: each row keeps the R columns of its own slot
//   warp 6      planner: per tile, the slots (distinct tenants in order of their
//               first row), each row's slot and the tile's weight group, into one of
//               two shared-memory plans, one tile ahead of the others
// The x tile crosses the SM once per item whatever the number of tenants in it
// (the per-warp mma.sync kernel re-streamed it per tenant), and A is fetched once
// per (tile, tenant). Slots beyond 256 / R columns start another unit of the
// same item (x is streamed again). Two 256-column accumulators let the epilogue
// of one unit overlap the next unit's MMAs. The K slices are summed in a fixed
// order by the reduce kernel of shrink.cu, so the result is deterministic.
#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace sb {
namespace {

constexpr int TS_BM = 128;
constexpr int TS_BK = 64;                           // one 128 B swizzle row of 16-bit values
constexpr int TS_KB_PER_SLICE = kShrinkKSlice / TS_BK;
constexpr int TS_STAGES = 4;
constexpr int TS_X_BYTES = TS_BM * TS_BK * 2;       // 16 KB
constexpr int TS_B_BYTES = 256 * TS_BK * 2;         // 32 KB: up to 256 stacked A rows
constexpr int TS_STAGE_BYTES = TS_X_BYTES + TS_B_BYTES;
constexpr int TS_THREADS = 224;
// barriers: full, empty (per stage), tmem_full x2, tmem_empty x2, drain, plan_full x2, plan_empty x2
constexpr int TS_NBARS = 2 * TS_STAGES + 9;
// a tile plan: slot count, weight group, slot -> tenant, row -> slot
struct TilePlan {
  int32_t ns;
  int32_t group;
  int32_t pad[2];
  int32_t slot_tenant[TS_BM];
  int8_t row_slot[TS_BM];
};
constexpr int TS_PLAN_OFF = 256;  // after the barriers
constexpr int TS_TAIL = TS_PLAN_OFF + 2 * (int)sizeof(TilePlan);
constexpr int TS_SMEM = TS_STAGES * TS_STAGE_BYTES + 1024 /*align*/ + 2048 /*barriers, plans*/;
static_assert(TS_KB_PER_SLICE * TS_BK == kShrinkKSlice, "slice = whole K blocks");
static_assert(TS_NBARS * 8 + 16 <= TS_PLAN_OFF && TS_TAIL <= 2048 && sizeof(TilePlan) % 16 == 0, "tail area");
static_assert(TS_SMEM <= 232448, "shared memory per block");

struct TsParams {
  int K;
  int KS;                  // K slices (kShrinkKSlice wide)
  int R;                   // output columns per tenant: 8, 16, 32 or 64
  int G;                   // slots per unit: 256 / R
  const int32_t* num_tiles_dev;
  int64_t static_rows;
  int64_t rows_cap;
  const int32_t* row_tenant;
  const int32_t* tile_group;
  const void* lora_a;      // [a_rows_total, K]
  int64_t a_rows_total;
  int64_t a_tenant_rows;   // A bank strides in rows of K elements
  int64_t a_group_rows;
  float* spart;            // [KS][rows_cap][R]
  int32_t* status;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

// Tenants of rows 4*lane .. 4*lane+3 of a tile (-1 past the active rows).
__device__ __forceinline__ void load_tile_tenants(const TsParams& p, int64_t rows_active, int m_tile, int lane,
                                                  int (&t)[4]) {
  const int64_t r0 = (int64_t)m_tile * TS_BM + 4 * lane;
#pragma unroll
  for (int i = 0; i < 4; ++i) t[i] = (r0 + i < rows_active) ? p.row_tenant[r0 + i] : -1;
}

// Distinct tenants of the tile in order of their first row (warp-wide): slot[i] =
// index of row (4*lane+i)'s tenant among them, -1 for rows without a tenant.
// Lane 0 writes slot -> tenant into `slot_tenant` when given. Returns the count.
__device__ __forceinline__ int tile_slots(const int (&t)[4], int lane, int (&slot)[4], int32_t* slot_tenant) {
  bool pend[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    pend[i] = t[i] >= 0;
    slot[i] = -1;
  }
  int ns = 0;
  while (true) {
    const bool any = pend[0] || pend[1] || pend[2] || pend[3];
    const unsigned m = __ballot_sync(0xffffffffu, any);
    if (!m) break;
    const int leader = __ffs(m) - 1;
    const int mine = pend[0] ? t[0] : pend[1] ? t[1] : pend[2] ? t[2] : t[3];
    const int key = __shfl_sync(0xffffffffu, mine, leader);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (pend[i] && t[i] == key) {
        slot[i] = ns;
        pend[i] = false;
      }
    if (slot_tenant && lane == 0) slot_tenant[ns] = key;
    ++ns;
  }
  return ns;
}

__device__ __forceinline__ int64_t ts_rows_active(const TsParams& p) {
  if (!p.num_tiles_dev) return p.static_rows;
  const int64_t r = (int64_t)(*p.num_tiles_dev) * TS_BM;
  return r < p.rows_cap ? r : p.rows_cap;
}

template <typename T>
struct TsBf16 {
  static constexpr int value = 0;
};
template <>
struct TsBf16<bf16> {
  static constexpr int value = 1;
};

template <typename T>
__global__ void __launch_bounds__(TS_THREADS, 1)
    tc_shrink_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_a,
                     const TsParams p) {
  extern __shared__ uint8_t smem_raw[];
  pdl_wait();  // the rows, the plan and the previous user of the partials come first
  pdl_trigger();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TS_STAGES * TS_STAGE_BYTES);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + TS_NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  TilePlan* plans = reinterpret_cast<TilePlan*>(reinterpret_cast<uint8_t*>(bars) + TS_PLAN_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t smem_base = smem_u32(smem);
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[TS_STAGES + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * TS_STAGES + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * TS_STAGES + 2 + a]); };
  const uint32_t drain_bar = smem_u32(&bars[2 * TS_STAGES + 4]);
  auto pfull_bar = [&](int b) { return smem_u32(&bars[2 * TS_STAGES + 5 + b]); };
  auto pempty_bar = [&](int b) { return smem_u32(&bars[2 * TS_STAGES + 7 + b]); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < TS_STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
      mbar_init(pfull_bar(a), 1);
      mbar_init(pempty_bar(a), 6);  // producer, MMA issuer, 4 epilogue warps
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_base_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  const int64_t rows_active = ts_rows_active(p);
  const int num_tiles = (int)((rows_active + TS_BM - 1) / TS_BM);
  const int total_items = num_tiles * p.KS;
  // this CTA's contiguous item range: the K slices of one or a few tiles
  const int i0 = (int)((int64_t)total_items * blockIdx.x / gridDim.x);
  const int i1 = (int)((int64_t)total_items * (blockIdx.x + 1) / gridDim.x);
  const int num_kb = (p.K + TS_BK - 1) / TS_BK;
  const int R = p.R, G = p.G;
  volatile int never_abort = 0;

  // A consumer's view of the plans: the plan of tile m_tile is the (m_tile - first
  // tile)-th plan; a new tile releases the previous plan and waits for its own.
  auto next_plan = [&](int& pi, bool release, bool& ok) -> const TilePlan* {
    if (release && lane == 0) mbar_arrive(pempty_bar(pi & 1));
    ++pi;
    // every lane waits, so that every lane's later reads of the plan follow the planner's writes
    const bool got = ok && mbar_wait(pfull_bar(pi & 1), (pi >> 1) & 1, abort_flag, p.status, p.timeout_ns,
                                     kDevTimeoutMma);
    if (!__all_sync(0xffffffffu, got)) ok = false;
    return &plans[pi & 1];
  };

  if (warp == 6) {
    // ------------------------------------------------------------ planner
    int pi = 0;
    for (int m_tile = (i0 < i1 ? i0 / p.KS : 0); i0 < i1 && m_tile <= (i1 - 1) / p.KS; ++m_tile, ++pi) {
      const int b = pi & 1;
      // every lane waits: its writes below follow the consumers' reads of the buffer
      const bool got =
          pi < 2 || mbar_wait(pempty_bar(b), ((pi >> 1) & 1) ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma);
      if (!__all_sync(0xffffffffu, got)) break;
      int tn[4], sl[4];
      load_tile_tenants(p, rows_active, m_tile, lane, tn);
      TilePlan* pl = &plans[b];
      const int ns = tile_slots(tn, lane, sl, pl->slot_tenant);
#pragma unroll
      for (int i = 0; i < 4; ++i) pl->row_slot[4 * lane + i] = (int8_t)sl[i];
      if (lane == 0) {
        pl->ns = ns;
        pl->group = p.tile_group ? p.tile_group[m_tile] : 0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(pfull_bar(b));
    }
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_a);
    }
    const uint64_t pol = l2_policy_evict_normal();
    int last_phase[TS_STAGES];
    for (int s = 0; s < TS_STAGES; ++s) last_phase[s] = -1;
    uint32_t it = 0;
    bool ok = true;
    int pi = -1, cur_tile = -1;
    const TilePlan* pl = nullptr;
    for (int item = i0; ok && item < i1; ++item) {
      const int m_tile = item / p.KS, slice = item - m_tile * p.KS;
      if (m_tile != cur_tile) {
        pl = next_plan(pi, cur_tile >= 0, ok);
        cur_tile = m_tile;
        if (!ok) break;
      }
      if (lane == 0) {
        const int ns = pl->ns;
        const int64_t group_rows = (int64_t)pl->group * p.a_group_rows;
        const int kb0 = slice * TS_KB_PER_SLICE, kb1 = min(num_kb, kb0 + TS_KB_PER_SLICE);
        for (int u0 = 0; ok && u0 < ns; u0 += G) {
          const int nsu = min(G, ns - u0);
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % TS_STAGES;
            const uint32_t ph = (it / TS_STAGES) & 1;
            if (!mbar_wait(empty_bar(s), ph ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutProducer)) {
              ok = false;
              break;
            }
            const uint32_t sa = smem_base + s * TS_STAGE_BYTES;
            mbar_arrive_expect_tx(full_bar(s), TS_X_BYTES + nsu * R * TS_BK * 2);
            tma_load_2d(sa, &tm_x, full_bar(s), kb * TS_BK, m_tile * TS_BM, pol);
            for (int j = 0; j < nsu; ++j) {
              const int64_t arow = (int64_t)pl->slot_tenant[u0 + j] * p.a_tenant_rows + group_rows;
              tma_load_2d(sa + TS_X_BYTES + j * R * TS_BK * 2, &tm_a, full_bar(s), kb * TS_BK, (int)arow, pol);
            }
            last_phase[s] = (int)ph;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
    if (lane == 0 && !ok) {
      // let the copies in flight land before the CTA exits
      for (int s = 0; s < TS_STAGES; ++s)
        if (last_phase[s] >= 0)
          mbar_wait(full_bar(s), (uint32_t)last_phase[s], &never_abort, p.status, 1000000000ull, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    uint32_t it = 0;
    int ucount = 0;
    bool ok = true, issued_any = false;
    int pi = -1, cur_tile = -1;
    const TilePlan* pl = nullptr;
    for (int item = i0; ok && item < i1; ++item) {
      const int m_tile = item / p.KS, slice = item - m_tile * p.KS;
      if (m_tile != cur_tile) {
        pl = next_plan(pi, cur_tile >= 0, ok);
        cur_tile = m_tile;
        if (!ok) break;
      }
      if (lane == 0) {
        const int ns = pl->ns;
        const int kb0 = slice * TS_KB_PER_SLICE, kb1 = min(num_kb, kb0 + TS_KB_PER_SLICE);
        for (int u0 = 0; ok && u0 < ns; u0 += G, ++ucount) {
          const int nsu = min(G, ns - u0);
          const int n_cols = ((nsu * R + 15) / 16) * 16;
          const uint32_t idesc = idesc_f16(TS_BM, n_cols, TsBf16<T>::value);
          const int acc = ucount & 1;
          const uint32_t aph = (ucount >> 1) & 1;
          if (!mbar_wait(tempty_bar(acc), aph ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * 256;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % TS_STAGES;
            const uint32_t ph = (it / TS_STAGES) & 1;
            if (!mbar_wait(full_bar(s), ph, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_base + s * TS_STAGE_BYTES;
            const uint64_t adesc = smem_desc_sw128(sa);
            const uint64_t bdesc = smem_desc_sw128(sa + TS_X_BYTES);
#pragma unroll
            for (int k = 0; k < TS_BK / 16; ++k)
              tc_mma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            tc_commit(empty_bar(s));
            issued_any = true;
          }
          if (!ok) break;
          tc_commit(tfull_bar(acc));
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
    if (lane == 0 && !ok && issued_any) {
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, &never_abort, p.status, 1000000000ull, kDevTimeoutDrain);
    }
  } else if (warp >= 2 && warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int ucount = 0;
    bool ok = true;
    int pi = -1, cur_tile = -1;
    const TilePlan* pl = nullptr;
    for (int item = i0; ok && item < i1; ++item) {
      const int m_tile = item / p.KS, slice = item - m_tile * p.KS;
      if (m_tile != cur_tile) {
        pl = next_plan(pi, cur_tile >= 0, ok);
        cur_tile = m_tile;
        if (!ok) break;
      }
      const int ns = pl->ns;
      const int my_slot = pl->row_slot[row_in_tile];
      const int64_t row = (int64_t)m_tile * TS_BM + row_in_tile;
      float* sp = p.spart + ((int64_t)slice * p.rows_cap + row) * R;
      for (int u0 = 0; u0 < ns; u0 += G, ++ucount) {
        const int nsu = min(G, ns - u0);
        const int acc = ucount & 1;
        const uint32_t aph = (ucount >> 1) & 1;
        const bool got = mbar_wait(tfull_bar(acc), aph, abort_flag, p.status, p.timeout_ns, kDevTimeoutEpilogue);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int ls = my_slot - u0;
        bool pend = ls >= 0 && ls < nsu;
        const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * 256;
        // one TMEM read per distinct slot among the warp's 32 rows
        while (true) {
          const unsigned m = __ballot_sync(0xffffffffu, pend);
          if (!m) break;
          const int key = __shfl_sync(0xffffffffu, ls, __ffs(m) - 1);
          const uint32_t tc = t_row + key * R;
          const bool mine = pend && ls == key;
          if (R == 8) {
            uint32_t v[8];
            tmem_ld_x8(tc, v);
            tmem_wait_ld();
            if (mine) {
              reinterpret_cast<float4*>(sp)[0] = make_float4(__uint_as_float(v[0]), __uint_as_float(v[1]),
                                                             __uint_as_float(v[2]), __uint_as_float(v[3]));
              reinterpret_cast<float4*>(sp)[1] = make_float4(__uint_as_float(v[4]), __uint_as_float(v[5]),
                                                             __uint_as_float(v[6]), __uint_as_float(v[7]));
            }
          } else {
            for (int c = 0; c < R; c += 16) {
              uint32_t v[16];
              tmem_ld_x16(tc + c, v);
              tmem_wait_ld();
              if (mine) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  reinterpret_cast<float4*>(sp + c)[q] =
                      make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                  __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
              }
            }
          }
          if (mine) pend = false;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar(acc));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace

bool tc_shrink_supported(const ShrinkLaunch& s) {
  if (!(s.R == 8 || s.R == 16 || s.R == 32 || s.R == 64)) return false;
  if (s.src_row_of || !s.lora_a || !s.spart || !s.row_tenant || s.a_rows_total <= 0) return false;
  if (s.a_tenant_stride % s.K != 0 || s.a_group_stride % s.K != 0) return false;
  if (reinterpret_cast<uintptr_t>(s.src) % 16 != 0 || reinterpret_cast<uintptr_t>(s.lora_a) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(s.spart) % 16 != 0)
    return false;
  return s.K % 8 == 0;
}

int launch_tc_shrink(const ShrinkLaunch& s, const void* rows, cudaStream_t stream) {
  SB_CHECK_ARG(tc_shrink_supported(s), "tc shrink: unsupported arguments");
  const int64_t rows_max = s.num_tiles_dev ? s.rows_cap : s.static_rows;
  if (rows_max == 0) return STAGEML_OK;
  const CUtensorMapDataType dt = s.dtype_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tm_x, tm_a;
  SB_TRY(make_tmap_2d(&tm_x, rows, dt, 2, (uint64_t)rows_max, (uint64_t)s.K, (uint64_t)s.K * 2, TS_BM, TS_BK, 128));
  SB_CHECK_ARG(s.a_rows_total < (int64_t(1) << 31), "tc shrink: LoRA bank exceeds the TMA coordinate range");
  SB_TRY(make_tmap_2d(&tm_a, s.lora_a, dt, 2, (uint64_t)s.a_rows_total, (uint64_t)s.K, (uint64_t)s.K * 2,
                      (uint32_t)s.R, TS_BK, 128));
  TsParams p;
  p.K = s.K;
  p.KS = shrink_num_slices(s.K);
  p.R = s.R;
  p.G = 256 / s.R;
  p.num_tiles_dev = s.num_tiles_dev;
  p.static_rows = s.static_rows;
  p.rows_cap = s.num_tiles_dev ? s.rows_cap : s.static_rows;
  p.row_tenant = s.row_tenant;
  p.tile_group = s.tile_group;
  p.lora_a = s.lora_a;
  p.a_rows_total = s.a_rows_total;
  p.a_tenant_rows = s.a_tenant_stride / s.K;
  p.a_group_rows = s.a_group_stride / s.K;
  p.spart = s.spart;
  p.status = s.status;
  p.timeout_ns = kDefaultWaitNs;
  const int64_t items_upper = ((rows_max + TS_BM - 1) / TS_BM) * p.KS;
  const dim3 grid((unsigned)std::min<int64_t>(items_upper, sm_count()));
  if (s.dtype_bf16) {
    SB_CUDA_CHECK(cudaFuncSetAttribute(tc_shrink_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, TS_SMEM));
    SB_CUDA_CHECK(launch_kernel(tc_shrink_kernel<bf16>, grid, dim3(TS_THREADS), TS_SMEM, stream, s.pdl, tm_x, tm_a, p));
  } else {
    SB_CUDA_CHECK(cudaFuncSetAttribute(tc_shrink_kernel<f16>, cudaFuncAttributeMaxDynamicSharedMemorySize, TS_SMEM));
    SB_CUDA_CHECK(launch_kernel(tc_shrink_kernel<f16>, grid, dim3(TS_THREADS), TS_SMEM, stream, s.pdl, tm_x, tm_a, p));
  }
  ::sb::count_launch();
  return STAGEML_OK;
}

}  // namespace sb
