// Grouped GEMM on CTA pairs: the 256 x 256 tile of a two-CTA cluster computed by
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16, fp32 accumulators in TMEM).
//
// Same computation as grouped_gemm.cu (per-group weights, SwiGLU or plain
// epilogue, per-token-tenant LoRA expand fused as masked MMAs; 16-bit weights —
// e4m3 weights use grouped_gemm.cu), laid out so that each SM moves a third fewer
// bytes per FLOP: every CTA of the pair stages its own 128 rows of A and only
// half of the 256 B rows (SwiGLU: the gate half on the even CTA, the up half
// on the odd one), and the pair MMA issued by the even CTA reads both.
//
// A pair covers two 128-row tiles of the same group (consecutive tiles of a
// padded group segment). A group with an odd tile count ends with a half unit
// (half_units): its one 128-row tile on both CTAs, 64 rows each, computed by the
// M = 128 pair MMA. That MMA's accumulator holds a CTA's 64 rows in two lane
// halves: columns [0, N/2) of row m in TMEM lane m, columns [N/2, N) in lane
// 64 + m, both at TMEM columns [0, N/2). SwiGLU half units therefore order their
// 256 B rows as 64 gate, 64 up (even CTA) and the next 64 gate, 64 up (odd CTA),
// so that each lane holds the gate and up values of the same 64 output columns.
// Without half_units the odd tile forms a pair whose odd half is idle (its rows
// are loaded but never stored).
//
// Per CTA: warp 0 TMA producer, warp 1 TMEM allocator and -- on the even CTA --
// MMA issuer; warps 2..5 epilogue over the CTA's own 128 TMEM lanes. Both CTAs'
// copies complete on the even CTA's stage barrier (cta_group::2 copies), which
// the even CTA arms with both halves' bytes; stage and accumulator releases go
// to both CTAs in one commit. Every wait is bounded. No load is multicast.
#include "common.cuh"
#include "grouped_gemm.cuh"
#include "host_util.h"

#include <mutex>

namespace sb {
namespace {

constexpr int BM = 128;                        // rows per CTA (256 per pair)
constexpr int BN = 256;                        // accumulator columns
constexpr int BK = 64;                         // one 128 B swizzle row of 16-bit values
constexpr int A_BYTES = BM * BK * 2;           // 16 KB
constexpr int B_BYTES = 128 * BK * 2;          // this CTA's half of B: 16 KB
constexpr int MMA_STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int HALF_A_BYTES = 64 * BK * 2;      // half unit: 64 rows of A per CTA (8 KB)
constexpr int HALF_STAGE_BYTES = HALF_A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int LCHUNK = 128 * 32;               // 128 rows x 16 columns, 16-bit (4 KB)
constexpr int LHALF = 64 * 32;                 // 64 rows x 16 columns, 16-bit (2 KB)

constexpr int STAGES = 7;
constexpr int STAGE_BYTES = MMA_STAGE_BYTES;
constexpr int THREADS = 192;
// The MMA issuer reads the row masks of a unit's first kMmaRuns LoRA runs (and the run
// count) from shared memory: it bulk-copies them at the unit's start, so they land while
// the K loop runs instead of costing one global round trip per run in the LoRA phase.
constexpr int kMmaRuns = 32;
constexpr int MMA_RUN_BYTES = kRunHdrInts * 4 + kMmaRuns * kPairRunInts * 4;  // 128 + 1152
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 512 /*barriers*/ + MMA_RUN_BYTES;
static_assert(SMEM_BYTES <= 232448, "shared memory per block");
static_assert((kMmaRuns * kPairRunInts * 4) % 16 == 0, "bulk copy size");
// barrier area (512 B): the barriers, the TMEM address and abort flag (< 160 B), the
// producer's header barrier at byte 160, the MMA issuer's run barrier at byte 168 and
// the producer's 128-byte run header at byte 256; then the MMA issuer's run header
// (128 B) and its runs (kMmaRuns x 36 B) at byte 512
static_assert((2 * STAGES + 5) * 8 + 8 <= 160, "barrier area");

struct PParams {
  int K;
  int N;
  int b_group_rows;
  const int32_t* b_group_map;  // optional row group -> weight group
  int64_t b_rows_total;
  int num_n_tiles;
  int swiglu;
  const int32_t* tile_group;     // null: one group (direct rows)
  int64_t m_rows;                // direct mode: valid rows
  const int32_t* pairs;          // [pairs_cap][4]: m-tile of each half (-1: idle half), group's first pair, its pair count
  const int32_t* num_pairs_dev;
  int pairs_cap;
  // LoRA
  int rank;
  int lchunks;
  int s_bytes;
  int run_bytes;
  int runs_per_block;
  int64_t lb_tenant_rows;
  int64_t lb_group_rows;
  const int32_t* runs;           // [tiles][kMaxRunsPerPair][9], at each pair's first tile
  const int32_t* nruns;          // [tiles][kRunHdrInts] run headers
  // epilogue
  const float* row_scale;
  const void* bias;
  int64_t bias_group_stride;
  int bias_group_mod;
  const float* b_scale;          // per-B-row scale in the epilogue (or null)
  void* out;
  int64_t ldo;
  int32_t* status;
  unsigned long long timeout_ns;
  // side by side with the odd-tile kernel (split_sms > 0)
  const int32_t* split_singles_dev;
  int split_sms;
  int half_units;                // a pair whose second tile is -1 is a half unit (M = 128)
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

// LoRA runs of a pair are stored at its first tile m0.
__device__ __forceinline__ const int32_t* pair_run(const PParams& p, int m0, int r) {
  return p.runs + ((int64_t)m0 * kMaxRunsPerPair + min(r, kMaxRunsPerPair - 1)) * kPairRunInts;
}

__device__ __forceinline__ int num_pairs(const PParams& p) {
  const int n = *p.num_pairs_dev;
  return n < p.pairs_cap ? n : p.pairs_cap;
}

// Work unit u -> (pair, n-tile), group-major: every n-tile of a group's pairs (pairs
// fastest) before the next group, so a weight tile is read by all its row pairs at
// about the same time and only one group's activations need to stay in L2. The units
// of group g are [first_pair(g) * n_tiles, (first_pair(g) + pairs(g)) * n_tiles).
__device__ __forceinline__ void unit_coords(const PParams& p, int u, int& pm, int& n_tile) {
  const int pstar = u / p.num_n_tiles;
  const int first = p.pairs[4 * pstar + 2], cnt = p.pairs[4 * pstar + 3];
  const int local = u - first * p.num_n_tiles;
  n_tile = local / cnt;
  pm = first + (local - n_tile * cnt);
}

template <typename T>
__global__ void __launch_bounds__(THREADS, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                             const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_lb,
                             const __grid_constant__ CUtensorMap tm_a64, const __grid_constant__ CUtensorMap tm_b64,
                             const PParams p) {
  // Every CTA waits before anything else, the ones that leave at once too, so that
  // this grid never completes ahead of the kernel before it.
  pdl_wait();
  pdl_trigger();
  // Beside the odd-tile kernel only the first `nclusters` clusters work; the others
  // leave their SMs to it (both CTAs of a cluster decide alike, before any barrier).
  int nclusters = gridDim.x >> 1;
  if (p.split_sms > 0) {
    const int budget =
        (p.split_sms - split_single_ctas(p.num_pairs_dev, p.split_singles_dev, p.pairs_cap, p.split_sms)) >> 1;
    nclusters = min(nclusters, max(budget, 1));
    if ((int)(blockIdx.x >> 1) >= nclusters) return;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars: [0,S) full (both halves landed; used on the even CTA), [S,2S) empty,
  // [2S,2S+2) tmem_full, [2S+2,2S+4) tmem_empty (even CTA), [2S+4] drain
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  // the producer's copy of the current unit's run header (LoRA), and its barrier
  uint64_t* hdr_bar_p = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(bars) + 160);
  const int32_t* hdr_smem = reinterpret_cast<const int32_t*>(reinterpret_cast<uint8_t*>(bars) + 256);
  // the MMA issuer's copy of the current unit's run header and first kMmaRuns runs, and its barrier
  uint64_t* mrun_bar_p = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(bars) + 168);
  const int32_t* mhdr_smem = reinterpret_cast<const int32_t*>(reinterpret_cast<uint8_t*>(bars) + 512);
  const int32_t* mruns_smem = mhdr_smem + kRunHdrInts;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const uint32_t smem_base = smem_u32(smem);
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + 2 + a]); };
  const uint32_t drain_bar = smem_u32(&bars[2 * STAGES + 4]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);  // the even CTA's expect_tx
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8);  // 4 epilogue warps of each CTA
    }
    mbar_init(drain_bar, 1);
    mbar_init(smem_u32(hdr_bar_p), 1);
    mbar_init(smem_u32(mrun_bar_p), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_base_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  const int npairs = num_pairs(p);
  const int total_units = npairs * p.num_n_tiles;
  const int num_kb = (p.K + BK - 1) / BK;
  volatile int never_abort = 0;

  if (threadIdx.x == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    if (p.half_units) {
      tma_prefetch_desc(&tm_a64);
      tma_prefetch_desc(&tm_b64);
    }
    if (p.rank) {
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_lb);
    }
    const uint64_t pol_a = l2_policy_evict_last();
    const uint64_t pol_b = l2_policy_evict_normal();
    // Both CTAs' copies complete on the even CTA's full barrier, which the even CTA
    // arms with the bytes of both halves (the halves are the same size).
    const uint32_t lead_full0 = mapa_shared(full_bar(0), 0);
    auto arm = [&](int s, uint32_t bytes) {
      if (leader) mbar_arrive_expect_tx(full_bar(s), 2 * bytes);
    };
    auto load = [&](uint32_t dst, const CUtensorMap* tm, int s, int x, int y, uint64_t pol) {
      tma_load_2d_pair(dst, tm, lead_full0 + 8u * (uint32_t)s, x, y, pol);
    };
    int last_phase[STAGES];
    for (int s = 0; s < STAGES; ++s) last_phase[s] = -1;
    uint32_t it = 0, hdr_uses = 0;
    bool ok = true;
    const uint32_t hdr_bar = smem_u32(hdr_bar_p);
    bool hdr_inflight = false;
    for (int u = cluster; ok && u < total_units; u += nclusters) {
      int pm, n_tile;
      unit_coords(p, u, pm, n_tile);
      const int m0 = p.pairs[4 * pm];
      const bool half = p.half_units && p.pairs[4 * pm + 1] < 0;
      const int mine = p.pairs[4 * pm + rank];
      const int m_load = mine >= 0 ? mine : m0;  // an idle half loads defined rows it never stores
      const int group = p.tile_group ? p.tile_group[m0] : 0;
      const int a_row = half ? m0 * BM + 64 * (int)rank : m_load * BM;
      const int n0 = p.swiglu ? n_tile * 128 : n_tile * BN;
      const int b_base = weight_group(p.b_group_map, group) * p.b_group_rows;
      const int b_row = b_base + n0 + (int)rank * (p.swiglu ? p.N : 128);
      if (p.rank) {  // the run header arrives while the K loop's copies are issued
        mbar_arrive_expect_tx(hdr_bar, kRunHdrInts * 4);
        bulk_load_1d(smem_u32(hdr_smem), p.nruns + (int64_t)m0 * kRunHdrInts, kRunHdrInts * 4, hdr_bar);
        hdr_inflight = true;
      }
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait_cluster(empty_bar(s), ph ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        const uint32_t sa = smem_base + s * STAGE_BYTES;
        if (half) {
          // 64 rows of A; SwiGLU B: gate rows [n0 + 64 rank, +64), then the same up rows
          arm(s, HALF_STAGE_BYTES);
          load(sa, &tm_a64, s, kb * BK, a_row, pol_a);
          if (p.swiglu) {
            const int g_row = b_base + n0 + 64 * (int)rank;
            load(sa + A_BYTES, &tm_b64, s, kb * BK, g_row, pol_b);
            load(sa + A_BYTES + B_BYTES / 2, &tm_b64, s, kb * BK, g_row + p.N, pol_b);
          } else {
            load(sa + A_BYTES, &tm_b, s, kb * BK, b_row, pol_b);
          }
        } else {
          arm(s, MMA_STAGE_BYTES);
          load(sa, &tm_a, s, kb * BK, a_row, pol_a);
          load(sa + A_BYTES, &tm_b, s, kb * BK, b_row, pol_b);
        }
        last_phase[s] = (int)ph;
      }
      // LoRA blocks: this CTA's rows of S + its half of the B rows of each tenant run
      int nruns = 0;
      if (p.rank && ok) {
        ok = mbar_wait(hdr_bar, hdr_uses & 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutProducer);
        ++hdr_uses;
        hdr_inflight = !ok;
        nruns = ok ? min(hdr_smem[0], kMaxRunsPerPair) : 0;
      }
      for (int r0 = 0; ok && r0 < nruns; r0 += p.runs_per_block, ++it) {
        const int nr = min(p.runs_per_block, nruns - r0);
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait_cluster(empty_bar(s), ph ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        const uint32_t base = smem_base + s * STAGE_BYTES;
        arm(s, p.s_bytes + nr * p.run_bytes);
        for (int ch = 0; ch < p.lchunks; ++ch) {
          load(base + ch * LCHUNK, &tm_s, s, ch * 16, a_row, pol_a);
          if (p.swiglu) load(base + (p.lchunks + ch) * LCHUNK, &tm_s, s, p.rank + ch * 16, a_row, pol_a);
        }
        for (int jj = 0; jj < nr; ++jj) {
          const int r = r0 + jj;
          const int tenant = r < kRunHdrInts - 1 ? hdr_smem[1 + r] : pair_run(p, m0, r)[0];
          const int brow = (int)(tenant * p.lb_tenant_rows + group * p.lb_group_rows) + n0;
          const uint32_t rb = base + p.s_bytes + jj * p.run_bytes;
          for (int ch = 0; ch < p.lchunks; ++ch) {
            if (p.swiglu) {
              // gate / up MMAs have N = 128: this CTA holds rows [64 * rank, 64 * rank + 64) of each
              load(rb + ch * LHALF, &tm_lb, s, ch * 16, brow + 64 * (int)rank, pol_b);
              load(rb + (p.lchunks + ch) * LHALF, &tm_lb, s, ch * 16, brow + p.N + 64 * (int)rank, pol_b);
            } else {
              load(rb + ch * LCHUNK, &tm_lb, s, ch * 16, brow + 128 * (int)rank, pol_b);
              load(rb + ch * LCHUNK + LHALF, &tm_lb, s, ch * 16, brow + 128 * (int)rank + 64, pol_b);
            }
          }
        }
        last_phase[s] = (int)ph;
      }
    }
    if (!ok) {
      // Let the copies already in flight land before the CTA pair leaves. The odd CTA's
      // copies complete on the even CTA's barrier; it waits a fixed, ample time.
      if (hdr_inflight) mbar_wait(hdr_bar, hdr_uses & 1, &never_abort, p.status, 200000000ull, kDevTimeoutDrain);
      if (leader) {
        for (int s = 0; s < STAGES; ++s)
          if (last_phase[s] >= 0)
            mbar_wait(full_bar(s), (uint32_t)last_phase[s], &never_abort, p.status, 200000000ull, kDevTimeoutDrain);
      } else {
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) {
        }
      }
    }
  } else if (threadIdx.x == 32 && leader) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    const uint32_t idesc = idesc_f16(2 * BM, BN, IsBf16<T>::value);
    const uint32_t idesc_n128 = idesc_f16(2 * BM, 128, IsBf16<T>::value);
    const uint32_t idesc_h = idesc_f16(BM, BN, IsBf16<T>::value);        // half unit: M = 128
    const uint32_t idesc_h_n128 = idesc_f16(BM, 128, IsBf16<T>::value);
    uint32_t it = 0;
    int tcount = 0;
    bool ok = true;
    const uint32_t mrun_bar = smem_u32(mrun_bar_p);
    uint32_t mrun_uses = 0;
    bool mrun_inflight = false;
    for (int u = cluster; ok && u < total_units; u += nclusters, ++tcount) {
      const int acc = tcount & 1;
      const uint32_t aph = (tcount >> 1) & 1;
      int pm, n_tile_unused;
      unit_coords(p, u, pm, n_tile_unused);
      const int m0 = p.pairs[4 * pm];
      const bool half = p.half_units && p.pairs[4 * pm + 1] < 0;
      const uint32_t id_main = half ? idesc_h : idesc;
      if (p.rank) {  // the unit's run header and first runs arrive while the K loop is issued
        fence_proxy_async_smem();  // the previous unit's reads of the buffer come first
        mbar_arrive_expect_tx(mrun_bar, MMA_RUN_BYTES);
        bulk_load_1d(smem_u32(mhdr_smem), p.nruns + (int64_t)m0 * kRunHdrInts, kRunHdrInts * 4, mrun_bar);
        bulk_load_1d(smem_u32(mruns_smem), p.runs + (int64_t)m0 * kMaxRunsPerPair * kPairRunInts,
                     kMmaRuns * kPairRunInts * 4, mrun_bar);
        mrun_inflight = true;
      }
      if (!mbar_wait_cluster(tempty_bar(acc), aph ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait_cluster(full_bar(s), ph, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_base + s * STAGE_BYTES;
        const uint64_t adesc = smem_desc_sw128(sa);
        const uint64_t bdesc = smem_desc_sw128(sa + A_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma_f16_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, id_main, (kb > 0 || k > 0) ? 1u : 0u);
        tc_commit_pair_both(empty_bar(s), 0x3);
      }
      int nruns = 0;
      if (ok && p.rank) {
        ok = mbar_wait(mrun_bar, mrun_uses & 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma);
        mrun_inflight = !ok;
        ++mrun_uses;
        nruns = ok ? min(mhdr_smem[0], kMaxRunsPerPair) : 0;
      }
      for (int r0 = 0; ok && r0 < nruns; r0 += p.runs_per_block, ++it) {
        const int nr = min(p.runs_per_block, nruns - r0);
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait_cluster(full_bar(s), ph, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = smem_base + s * STAGE_BYTES;
        for (int jj = 0; jj < nr; ++jj) {
          const int r = r0 + jj;
          const int32_t* run = r < kMmaRuns ? mruns_smem + r * kPairRunInts : pair_run(p, m0, r);
          // Disable mask per TMEM lane: a pair unit's 256 rows are the lanes of both CTAs;
          // a half unit's row m (of 128) is lanes m % 64 and 64 + m % 64 of CTA m / 64.
          uint32_t dis[8];
          if (half) {
#pragma unroll
            for (int w = 0; w < 8; ++w) dis[w] = ~(uint32_t)run[1 + 2 * (w >> 2) + (w & 1)];
          } else {
#pragma unroll
            for (int w = 0; w < 8; ++w) dis[w] = ~(uint32_t)run[1 + w];
          }
          const uint32_t rb = base + p.s_bytes + jj * p.run_bytes;
          for (int ch = 0; ch < p.lchunks; ++ch) {
            if (p.swiglu) {
              // gate into accumulator columns [0, 128) (half unit: [0, 64) of both lane halves),
              // up into [128, 256) ([64, 128))
              const uint32_t id_n128 = half ? idesc_h_n128 : idesc_n128;
              tc_mma_f16_pair_masked(d_tmem, smem_desc_sw32(base + ch * LCHUNK), smem_desc_sw32(rb + ch * LHALF),
                                     id_n128, 1u, dis);
              tc_mma_f16_pair_masked(d_tmem + (half ? 64 : 128), smem_desc_sw32(base + (p.lchunks + ch) * LCHUNK),
                                     smem_desc_sw32(rb + (p.lchunks + ch) * LHALF), id_n128, 1u, dis);
            } else {
              tc_mma_f16_pair_masked(d_tmem, smem_desc_sw32(base + ch * LCHUNK), smem_desc_sw32(rb + ch * LCHUNK),
                                     id_main, 1u, dis);
            }
          }
        }
        tc_commit_pair_both(empty_bar(s), 0x3);
      }
      if (!ok) break;
      tc_commit_pair_both(tfull_bar(acc), 0x3);
    }
    // The run copy in flight lands before the CTA pair leaves (error paths).
    if (mrun_inflight) mbar_wait(mrun_bar, mrun_uses & 1, &never_abort, p.status, 200000000ull, kDevTimeoutDrain);
    // Every MMA of this CTA pair has completed (and stopped reading either CTA's
    // shared memory) before the final cluster barrier.
    tc_commit_pair(drain_bar);
    mbar_wait(drain_bar, 0, &never_abort, p.status, 1000000000ull, kDevTimeoutDrain);
  } else if (warp >= 2 && warp < 6) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const T* bias = reinterpret_cast<const T*>(p.bias);
    T* out = reinterpret_cast<T*>(p.out);
    const bool vec_ok = (p.ldo % 8 == 0) && (p.N % 8 == 0);
    const uint32_t leader_tempty0 = mapa_shared(tempty_bar(0), 0);
    int tcount = 0;
    for (int u = cluster; u < total_units; u += nclusters, ++tcount) {
      const int acc = tcount & 1;
      const uint32_t aph = (tcount >> 1) & 1;
      if (!mbar_wait_cluster(tfull_bar(acc), aph, abort_flag, p.status, p.timeout_ns, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      int pm, n_tile;
      unit_coords(p, u, pm, n_tile);
      const int m0 = p.pairs[4 * pm];
      const bool half = p.half_units && p.pairs[4 * pm + 1] < 0;
      const int mine = p.pairs[4 * pm + rank];
      const int group = p.tile_group ? p.tile_group[m0] : 0;
      // half unit: this CTA's 64 rows of tile m0; lane quarters 0-1 hold the first half
      // of the unit's columns, quarters 2-3 the second half
      const int64_t row = half ? (int64_t)m0 * BM + 64 * (int)rank + (quarter & 1) * 32 + lane
                               : (int64_t)mine * BM + row_in_tile;
      const int col_half = half ? (quarter >> 1) : 0;
      const bool live = half || mine >= 0;  // uniform over the CTA: tcgen05.ld below is warp-collective
      const bool row_ok = live && (p.tile_group ? true : row < p.m_rows);
      const float rscale = (row_ok && p.row_scale) ? p.row_scale[row] : 1.f;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (p.swiglu) {
        const int n0 = n_tile * 128 + 64 * col_half;
        const int ncols = half ? 64 : 128;  // up values sit ncols columns after the gate values
        for (int c = 0; c < ncols && live; c += 16) {
          uint32_t rg[16], ru[16];
          tmem_ld_x16(t_row + c, rg);
          tmem_ld_x16(t_row + ncols + c, ru);
          tmem_wait_ld();
          const int col = n0 + c;
          const int nvalid = min(16, p.N - col);
          float h[16];
          if (p.b_scale && nvalid > 0) {
            const float* bsg = p.b_scale + (int64_t)weight_group(p.b_group_map, group) * p.b_group_rows + col;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float sg = i < nvalid ? bsg[i] : 0.f, su = i < nvalid ? bsg[p.N + i] : 0.f;
              h[i] = silu_f32(__uint_as_float(rg[i]) * sg) * (__uint_as_float(ru[i]) * su);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) h[i] = silu_f32(__uint_as_float(rg[i])) * __uint_as_float(ru[i]);
          }
          if (row_ok && nvalid > 0) store16<T>(out + row * p.ldo + col, h, nvalid, vec_ok);
        }
      } else {
        const int n0 = n_tile * BN + 128 * col_half;
        const int ncols = half ? 128 : BN;
        for (int c = 0; c < ncols && live; c += 16) {
          uint32_t rv[16];
          tmem_ld_x16(t_row + c, rv);
          tmem_wait_ld();
          const int col = n0 + c;
          const int nvalid = min(16, p.N - col);
          if (nvalid > 0) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(rv[i]);
            if (p.b_scale) {
              const float* bs = p.b_scale + (int64_t)weight_group(p.b_group_map, group) * p.b_group_rows + col;
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
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] *= rscale;
            if (row_ok) store16<T>(out + row * p.ldo + col, v, nvalid, vec_ok);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_tempty0 + 8u * (uint32_t)acc);
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // no MMA, TMEM read or remote arrive of either CTA is still outstanding
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------ pair list and LoRA runs
// Tile t opens a pair when its distance from its group's first tile is even; its
// partner is t + 1 when that tile exists and belongs to the same group. A group's
// trailing odd tile is a single when singles are listed (for the one-CTA kernel),
// else it forms a pair with an idle half (-1).
struct TileRole {
  int start, partner, in_group, group_tiles;
};

__device__ __forceinline__ TileRole tile_role(const int32_t* tile_group, const int32_t* group_offsets, int ntiles,
                                              int t) {
  TileRole r{0, -1, 0, 0};
  if (t >= ntiles) return r;
  if (tile_group) {
    const int g = tile_group[t];
    const int t0 = group_offsets[g] >> 7;
    r.in_group = (t - t0) >> 1;
    r.group_tiles = (group_offsets[g + 1] - group_offsets[g]) >> 7;
    r.start = ((t - t0) & 1) == 0;
    if (r.start && t + 1 < ntiles && tile_group[t + 1] == g) r.partner = t + 1;
  } else {
    r.in_group = t >> 1;
    r.group_tiles = ntiles;
    r.start = (t & 1) == 0;
    if (r.start && t + 1 < ntiles) r.partner = t + 1;
  }
  return r;
}

constexpr int kPlanThreads = 128;
constexpr int kPlanWarps = kPlanThreads / 32;

// Distinct tenants (>= 0) of NQ row quarters of 32 (first-seen order) and the
// rows each one owns, one warp; every quarter's tenant is loaded before the
// first match so the loads overlap. Writes runs[j * ints + 0] = tenant,
// [1 .. NQ] = mask words, and *nruns.
template <int NQ>
__device__ __forceinline__ void quarter_runs(const int32_t* row_tenant, const int64_t (&qrow)[NQ], int64_t row_bound,
                                             int32_t* s_ten, uint32_t (*s_mask)[8], int32_t* runs, int32_t* nruns,
                                             int max_runs) {
  const int lane = threadIdx.x & 31;
  int ten[NQ];
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int64_t row = qrow[q] < 0 ? -1 : qrow[q] + lane;
    ten[q] = (row >= 0 && row < row_bound) ? row_tenant[row] : -1;
  }
  int count = 0;
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int t = ten[q];
    const unsigned peers = __match_any_sync(0xffffffffu, t);
    const bool lead = (t >= 0) && ((peers & ((1u << lane) - 1u)) == 0u);
    int found = -1;
    if (lead)
      for (int j = 0; j < count; ++j)
        if (s_ten[j] == t) {
          found = j;
          break;
        }
    const unsigned is_new = __ballot_sync(0xffffffffu, lead && found < 0);
    if (lead) {
      int idx = found;
      if (found < 0) {
        idx = count + __popc(is_new & ((1u << lane) - 1u));
        if (idx < max_runs) {
          s_ten[idx] = t;
#pragma unroll
          for (int qq = 0; qq < NQ; ++qq) s_mask[idx][qq] = 0u;
        }
      }
      if (idx < max_runs) s_mask[idx][q] = peers;
    }
    count += __popc(is_new);
    __syncwarp();
  }
  count = min(count, max_runs);
  for (int j = lane; j < count; j += 32) {
    int32_t* r = runs + (int64_t)j * (1 + NQ);
    r[0] = s_ten[j];
#pragma unroll
    for (int qq = 0; qq < NQ; ++qq) r[1 + qq] = (int32_t)s_mask[j][qq];
  }
  if (NQ == 8) {  // pair: run header (count, then the first kRunHdrInts - 1 tenants)
    nruns[lane] = lane == 0 ? count : (lane - 1 < count ? s_ten[lane - 1] : -1);
  } else if (lane == 0) {
    *nruns = count;
  }
}

// One launch for the whole plan. Block 0 lists the pairs (and the singles) in tile
// order, each with its group's first pair and pair count (for the unit order), and
// with hpairs the second list in which each trailing odd tile is a half unit.
// Blocks 1.. (with row_tenant): one warp per tile t, which writes the LoRA runs of
// the pair t opens at pruns[t] / pnruns[t] (256 rows, 8 mask words; a half unit's
// words 4-7 are zero), and of the single t at sruns[t] / snruns[t] (128 rows, 4 mask
// words): runs are indexed by the first tile, so no block waits for the lists.
__global__ void __launch_bounds__(kPlanThreads) pair_plan_kernel(
    const int32_t* __restrict__ tile_group, const int32_t* __restrict__ group_offsets,
    const int32_t* __restrict__ num_tiles_dev, int tiles_cap, int64_t static_rows, const int32_t* __restrict__ row_tenant,
    int32_t* __restrict__ pairs, int32_t* __restrict__ num_pairs_out, int32_t* __restrict__ singles,
    int32_t* __restrict__ num_singles_out, int32_t* __restrict__ pruns, int32_t* __restrict__ pnruns,
    int32_t* __restrict__ sruns, int32_t* __restrict__ snruns, int32_t* __restrict__ hpairs,
    int32_t* __restrict__ num_hpairs_out) {
  pdl_wait();  // the permutation plan and the tenants may come from the previous kernels
  pdl_trigger();
  const int ntiles = num_tiles_dev ? min(*num_tiles_dev, tiles_cap) : (int)((static_rows + 127) / 128);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const bool split = singles != nullptr;
  if (blockIdx.x > 0) {
    __shared__ int32_t s_ten[kPlanWarps][kMaxRunsPerPair];
    __shared__ uint32_t s_mask[kPlanWarps][kMaxRunsPerPair][8];
    const int t = (blockIdx.x - 1) * kPlanWarps + w;
    const TileRole r = tile_role(tile_group, group_offsets, ntiles, t);
    if (!r.start) return;
    const int64_t bound = num_tiles_dev ? INT64_MAX : static_rows;
    const bool odd = r.partner < 0;
    if (split && odd && sruns) {
      const int64_t q4[4] = {(int64_t)t * 128, (int64_t)t * 128 + 32, (int64_t)t * 128 + 64, (int64_t)t * 128 + 96};
      quarter_runs<4>(row_tenant, q4, bound, s_ten[w], s_mask[w], sruns + (int64_t)t * kMaxRunsPerTile * 5,
                      snruns + t, kMaxRunsPerTile);
      __syncwarp();  // the warp's staging arrays are reused below
    }
    if (!(split && odd) || hpairs) {
      int64_t q8[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int tile = q < 4 ? t : r.partner;
        q8[q] = tile < 0 ? -1 : (int64_t)tile * 128 + (q & 3) * 32;
      }
      quarter_runs<8>(row_tenant, q8, bound, s_ten[w], s_mask[w],
                      pruns + (int64_t)t * kMaxRunsPerPair * kPairRunInts, pnruns + (int64_t)t * kRunHdrInts,
                      kMaxRunsPerPair);
    }
    return;
  }
  __shared__ int32_t warp_tot[3][kPlanWarps];
  __shared__ int32_t carry[3];
  if (tid < 3) carry[tid] = 0;
  __syncthreads();
  for (int base = 0; base < ntiles; base += kPlanThreads) {
    const int t = base + tid;
    const TileRole r = tile_role(tile_group, group_offsets, ntiles, t);
    const bool as_single = split && r.start && r.partner < 0;
    const bool as_pair = r.start && !as_single;
    const bool as_hpair = hpairs != nullptr && r.start;
    const unsigned bp = __ballot_sync(0xffffffffu, as_pair), bs = __ballot_sync(0xffffffffu, as_single);
    const unsigned bh = __ballot_sync(0xffffffffu, as_hpair);
    if (lane == 0) {
      warp_tot[0][w] = __popc(bp);
      warp_tot[1][w] = __popc(bs);
      warp_tot[2][w] = __popc(bh);
    }
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
    if (as_pair) {
      int before = carry[0] + __popc(bp & lt);
      for (int i = 0; i < w; ++i) before += warp_tot[0][i];
      pairs[4 * before] = t;
      pairs[4 * before + 1] = r.partner;
      pairs[4 * before + 2] = before - r.in_group;  // the group's first pair
      pairs[4 * before + 3] = split ? r.group_tiles >> 1 : (r.group_tiles + 1) >> 1;
    }
    if (as_single) {
      int before = carry[1] + __popc(bs & lt);
      for (int i = 0; i < w; ++i) before += warp_tot[1][i];
      singles[before] = t;
    }
    if (as_hpair) {
      int before = carry[2] + __popc(bh & lt);
      for (int i = 0; i < w; ++i) before += warp_tot[2][i];
      hpairs[4 * before] = t;
      hpairs[4 * before + 1] = r.partner;
      hpairs[4 * before + 2] = before - r.in_group;
      hpairs[4 * before + 3] = (r.group_tiles + 1) >> 1;
    }
    __syncthreads();
    if (tid < 3) {
      int tot = 0;
      for (int i = 0; i < kPlanWarps; ++i) tot += warp_tot[tid][i];
      carry[tid] += tot;
    }
    __syncthreads();
  }
  if (tid == 0) {
    *num_pairs_out = carry[0];
    if (num_singles_out) *num_singles_out = carry[1];
    if (num_hpairs_out) *num_hpairs_out = carry[2];
  }
}

template <typename T>
int launch_pair_kernel(int64_t units_upper, cudaStream_t stream, bool pdl, const CUtensorMap& tm_a,
                       const CUtensorMap& tm_b,
                       const CUtensorMap& tm_s, const CUtensorMap& tm_lb, const CUtensorMap& tm_a64,
                       const CUtensorMap& tm_b64, const PParams& p) {
  auto kern = grouped_gemm_pair_kernel<T>;
  SB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  // Persistent grid: as many CTA pairs as can be resident at once.
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  SB_CUDA_CHECK(cudaGetDevice(&dev));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // the occupancy query below sees the cluster shape only
  int max_clusters = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64) max_clusters = cached[dev];
    if (max_clusters == 0) {
      cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
      if (cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg) != cudaSuccess || max_clusters <= 0) {
        cudaGetLastError();
        max_clusters = sm_count() / 2;
      }
      if (dev >= 0 && dev < 64) cached[dev] = max_clusters;
    }
  }
  const int64_t clusters = std::min<int64_t>(units_upper, max_clusters);
  cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
  cfg.numAttrs = pdl ? 2 : 1;
  SB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tm_a, tm_b, tm_s, tm_lb, tm_a64, tm_b64, p));
  ::sb::count_launch();
  return STAGEML_OK;
}

}  // namespace

size_t pair_runs_ints(int64_t pairs_cap) { return (size_t)pairs_cap * kMaxRunsPerPair * kPairRunInts; }

int launch_pair_plan(const int32_t* tile_group, const int32_t* group_offsets, const int32_t* num_tiles_dev,
                     int tiles_cap, int64_t static_rows, const int32_t* row_tenant, int32_t* pairs,
                     int32_t* num_pairs, int32_t* runs, int32_t* nruns, cudaStream_t stream, int32_t* singles,
                     int32_t* num_singles, int32_t* sruns, int32_t* snruns, int32_t* hpairs,
                     int32_t* num_hpairs, bool pdl) {
  SB_CHECK_ARG(pairs && num_pairs, "pair plan: null output");
  SB_CHECK_ARG(!singles == !num_singles, "pair plan: singles need their count");
  SB_CHECK_ARG(!hpairs == !num_hpairs, "pair plan: the half-unit list needs its count");
  SB_CHECK_ARG(!tile_group || (group_offsets && num_tiles_dev), "pair plan: grouped tiles need offsets and a count");
  SB_CHECK_ARG(!row_tenant || (runs && nruns), "pair plan: LoRA runs need output buffers");
  SB_CHECK_ARG(!sruns == !snruns, "pair plan: single-tile runs need their counts");
  const int64_t tiles = num_tiles_dev ? tiles_cap : (static_rows + 127) / 128;
  const int64_t run_blocks = (row_tenant && tiles > 0) ? (tiles + kPlanWarps - 1) / kPlanWarps : 0;
  SB_CHECK_ARG(run_blocks < 65535 * 1024LL, "pair plan: too many tiles");
  SB_CUDA_CHECK(launch_kernel(pair_plan_kernel, dim3((unsigned)(1 + run_blocks)), dim3(kPlanThreads), 0, stream, pdl,
                              tile_group, group_offsets, num_tiles_dev, tiles_cap, static_rows, row_tenant, pairs,
                              num_pairs, singles, num_singles, row_tenant ? runs : nullptr, nruns,
                              row_tenant ? sruns : nullptr, snruns, hpairs, num_hpairs));
  ::sb::count_launch();
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

int launch_grouped_gemm_pair(const GemmLaunch& g, cudaStream_t stream) {
  SB_CHECK_ARG(g.pairs && g.num_pairs_dev && g.pairs_cap >= 0, "pair gemm: missing pair list");
  SB_CHECK_ARG(!g.b_fp8, "pair gemm: e4m3 weights run on the one-CTA grouped GEMM");
  SB_CHECK_ARG(g.rank == 0 || (g.pair_runs && g.pair_nruns), "pair gemm: LoRA needs the pair runs");

  const CUtensorMapDataType dt = g.in_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tm_a, tm_b, tm_s, tm_lb, tm_a64, tm_b64;
  SB_TRY(make_tmap_2d(&tm_a, g.a, dt, 2, (uint64_t)g.a_rows, (uint64_t)g.K, (uint64_t)g.K * 2, BM, BK, 128));
  SB_TRY(make_tmap_2d(&tm_b, g.b, dt, 2, (uint64_t)g.b_rows_total, (uint64_t)g.K, (uint64_t)g.K * 2, 128, BK, 128));
  if (g.pair_half_units) {
    SB_TRY(make_tmap_2d(&tm_a64, g.a, dt, 2, (uint64_t)g.a_rows, (uint64_t)g.K, (uint64_t)g.K * 2, 64, BK, 128));
    SB_TRY(make_tmap_2d(&tm_b64, g.b, dt, 2, (uint64_t)g.b_rows_total, (uint64_t)g.K, (uint64_t)g.K * 2, 64, BK,
                        128));
  } else {
    tm_a64 = tm_a;  // unused
    tm_b64 = tm_b;
  }
  const int lora_cols = g.swiglu ? 2 * g.rank : g.rank;
  if (g.rank) {
    SB_TRY(make_tmap_2d(&tm_s, g.s16, dt, 2, (uint64_t)g.s_rows, (uint64_t)lora_cols, (uint64_t)lora_cols * 2, 128,
                        16, 32));
    SB_TRY(make_tmap_2d(&tm_lb, g.lora_b, dt, 2, (uint64_t)g.lora_b_rows_total, (uint64_t)g.rank,
                        (uint64_t)g.rank * 2, 64, 16, 32));
  } else {
    tm_s = tm_a;  // unused
    tm_lb = tm_a;
  }

  PParams p;
  p.K = g.K;
  p.N = g.N;
  p.b_group_rows = g.b_group_rows;
  p.b_group_map = g.b_group_map;
  p.b_rows_total = g.b_rows_total;
  p.swiglu = g.swiglu ? 1 : 0;
  p.num_n_tiles = g.swiglu ? (g.N + 127) / 128 : (g.N + BN - 1) / BN;
  p.tile_group = g.tile_group;
  p.m_rows = g.m_rows;
  p.pairs = g.pairs;
  p.num_pairs_dev = g.num_pairs_dev;
  p.pairs_cap = g.pairs_cap;
  p.rank = g.rank;
  p.lchunks = (g.rank + 15) / 16;
  p.s_bytes = (g.swiglu ? 2 : 1) * p.lchunks * LCHUNK;
  p.run_bytes = p.lchunks * LCHUNK;  // this CTA's half: 2 x 64 rows (SwiGLU) or 128 rows per chunk
  p.runs_per_block = g.rank ? (MMA_STAGE_BYTES - p.s_bytes) / p.run_bytes : 1;
  p.lb_tenant_rows = g.rank ? g.lora_b_tenant_stride / g.rank : 0;
  p.lb_group_rows = g.rank ? g.lora_b_group_stride / g.rank : 0;
  p.runs = g.pair_runs;
  p.nruns = g.pair_nruns;
  p.row_scale = g.row_scale;
  p.bias = g.bias;
  p.bias_group_stride = g.bias_group_stride;
  p.bias_group_mod = g.bias_group_mod;
  p.b_scale = g.b_scale;
  p.out = g.out;
  p.ldo = g.ldo;
  p.status = g.status;
  p.timeout_ns = kDefaultWaitNs;
  p.split_singles_dev = g.split_singles_dev;
  p.split_sms = g.split_singles_dev ? g.split_sms : 0;
  p.half_units = g.pair_half_units ? 1 : 0;

  const int64_t units_upper = (int64_t)g.pairs_cap * p.num_n_tiles;
  if (units_upper == 0) return STAGEML_OK;
  return g.in_bf16 ? launch_pair_kernel<bf16>(units_upper, stream, g.pdl, tm_a, tm_b, tm_s, tm_lb, tm_a64, tm_b64, p)
                   : launch_pair_kernel<f16>(units_upper, stream, g.pdl, tm_a, tm_b, tm_s, tm_lb, tm_a64, tm_b64, p);
}

}  // namespace sb
