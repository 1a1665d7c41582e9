// Grouped (per-expert / per-weight-group) GEMM on the 5th-generation tensor
// cores: TMA -> 128B-swizzled shared memory -> tcgen05.mma (cta_group::1,
// M=128, N=256, K=16, fp32 accumulators in TMEM) -> tcgen05.ld epilogue.
//
// One persistent CTA per SM:
//   warp 0      TMA producer (one thread)
//   warp 1      TMEM allocator + MMA issuer (one thread)
//   warps 2..5  epilogue: TMEM lane quarter (warp % 4), one accumulator row per thread
//   warps 6..21 (FP8 weights only) converters: e4m3 -> 16-bit with the
//               per-output-channel scale, written in the MMA's swizzled layout
// Two 256-column accumulators in TMEM let the epilogue of tile i overlap the
// main loop of tile i+1. 16-bit weights: 4 stages of 48 KB (A 16 KB, B 32 KB).
// FP8 weights: a 4-stage TMA ring of 40 KB (A 16 KB, e4m3 B 16 KB; LoRA blocks
// use all 40) and two 32 KB buffers for the converted 16-bit B tiles, so that
// four K blocks of copies stay in flight while the converters fill one buffer
// and the MMAs read the other.
//
// Per-token-tenant LoRA expand is fused on the tensor cores: after a tile's K
// loop, the producer streams "LoRA blocks" through the same ring -- the
// tile's 16-bit shrink output S (32B-swizzled, K = 16 per chunk) and, for each
// distinct tenant of the tile, the matching rows of its B factor -- and the MMA
// thread adds S . B^T into the same TMEM accumulator with the
// disable-output-lane mask set to every row that does not belong to that
// tenant. The epilogue is then only SwiGLU (or bias / routing weight) and the
// 16-bit store. This is the per-(slot, expert) body of
// RequestExecutor.dynamic_one (benchmarks/multitenant_bta_system_bench.py:408-413)
// for a whole 128-row tile, with the LoRA branch of
// DynamicMoELoRALayer.forward (stageml/moe_lora_layers.py:88-89) on every projection.
#include "common.cuh"
#include "grouped_gemm.cuh"
#include "host_util.h"

namespace sb {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;            // accumulator columns per tile (SwiGLU: 128 gate + 128 up)
constexpr int BK = 64;             // 64 x 16-bit = one 128 B swizzle row
constexpr int A_STAGE_BYTES = BM * BK * 2;         // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;         // 32 KB
constexpr int MMA_STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;  // operands the MMA reads (48 KB)
constexpr int RAW_B_BYTES = BN * BK;               // e4m3 B staging (16 KB)
constexpr int TMEM_COLS = 2 * BN;                  // double-buffered accumulator
constexpr int LCHUNK = 128 * 32;                   // one 128-row x 16-column 16-bit LoRA tile (4 KB)
constexpr int CONVERTER_THREADS = 512;
constexpr int CONV_ITEMS = 256 * 4 / CONVERTER_THREADS;  // 16-byte e4m3 chunks per converter thread and K block
static_assert(CONV_ITEMS * CONVERTER_THREADS == 256 * 4, "converter items");

template <bool FP8B>
struct Cfg {
  static constexpr int STAGES = 4;  // TMA ring
  // a TMA stage: A and B (16-bit weights) or A and the e4m3 B (FP8 weights, with 8 KB more so
  // that a LoRA block, which uses a stage whole, holds four tenant runs)
  static constexpr int STAGE_BYTES = FP8B ? A_STAGE_BYTES + RAW_B_BYTES + 8192 : MMA_STAGE_BYTES;
  static constexpr int CONV = FP8B ? 2 : 0;  // converted 16-bit B tiles (FP8 weights)
  static constexpr int THREADS = FP8B ? 192 + CONVERTER_THREADS : 192;
  static constexpr int SMEM_BYTES =
      STAGES * STAGE_BYTES + CONV * B_STAGE_BYTES + 1024 /*align*/ + 2048 /*barriers, run copies*/;
  static constexpr int NBARS = 2 * STAGES + 5 + 2 * CONV + (FP8B ? STAGES : 0);
};
static_assert(Cfg<true>::SMEM_BYTES <= 232448 && Cfg<false>::SMEM_BYTES <= 232448, "shared memory per block");
static_assert(Cfg<true>::NBARS * 8 + 8 <= 192 && Cfg<false>::NBARS * 8 + 8 <= 192, "barrier area");
// The producer and the MMA issuer each bulk-copy the first kHdrRuns runs (tenant + 4
// mask words each) of a unit's tile at the unit's start, so the LoRA phase costs no
// global round trip per run: area after the stages = barriers (< 192 B), the
// producer's copy barrier at byte 192 and the MMA issuer's at byte 200, the
// producer's runs at byte 256, the MMA issuer's at byte 1024.
constexpr int kHdrRuns = 32;
static_assert(256 + kHdrRuns * 5 * 4 <= 1024 && (kHdrRuns * 5 * 4) % 16 == 0, "run header area");

struct KParams {
  int K;
  int N;
  int b_group_rows;
  const int32_t* b_group_map;  // optional row group -> weight group
  int64_t b_rows_total;
  int num_n_tiles;
  int swiglu;
  const int32_t* num_tiles_dev;
  int tiles_cap;
  const int32_t* tile_group;
  const int32_t* tile_list;   // optional: m-tile i is tile_list[i] (LoRA runs indexed by the tile id)
  const int32_t* group_offsets;  // grouped rows without a list: group-major unit order
  int64_t m_rows;
  // LoRA
  int rank;
  int lchunks;         // rank / 16
  int s_bytes;         // S bytes per LoRA block
  int run_bytes;       // B bytes per run
  int runs_per_block;  // LoRA slots (runs, or pairs of runs with pack8) per LoRA block
  int pack8;           // rank 8: two runs per K = 16 step (S in the run-parity layout)
  int64_t lb_tenant_rows;
  int64_t lb_group_rows;
  const int32_t* tile_runs;
  const int32_t* tile_nruns;
  // epilogue
  const float* row_scale;
  const void* bias;
  int64_t bias_group_stride;
  int bias_group_mod;
  const float* b_scale;       // 16-bit weights: per-B-row scale applied in the epilogue (or null)
  const float* b_row_scale;   // FP8 weights: per-B-row dequantisation scale applied by the converters
  void* out;
  int64_t ldo;
  int32_t* status;
  // beside the pair kernel (split_sms > 0): only the odd-tile share of the SMs
  const int32_t* split_pairs_dev;
  const int32_t* split_singles_dev;
  int split_cap;
  int split_sms;
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

// Unit u -> (m-tile position, n-tile). With group offsets (grouped rows, no list) the
// order is group-major: every n-tile of a group's m-tiles (m-tiles fastest) before
// the next group, so a weight tile is read by all of its group's m-tiles at about
// the same time and only one group's activation rows need to stay in L2. The units
// of group g are [first_tile(g) * n_tiles, (first_tile(g) + tiles(g)) * n_tiles).
// Otherwise m-tiles fastest.
__device__ __forceinline__ void unit_mn(const KParams& p, int u, int num_m_tiles, int& m_pos, int& n_tile) {
  if (p.group_offsets) {
    const int g = p.tile_group[u / p.num_n_tiles];
    const int first = p.group_offsets[g] >> 7, cnt = (p.group_offsets[g + 1] >> 7) - first;
    const int local = u - first * p.num_n_tiles;
    n_tile = local / cnt;
    m_pos = first + (local - n_tile * cnt);
  } else {
    m_pos = u % num_m_tiles;
    n_tile = u / num_m_tiles;
  }
}

// K-major operand without swizzle: 8-row core matrices of 16-byte rows, `sbo` bytes
// between 8-row groups and `lbo` bytes between the two 8-column halves of a K = 16 step.
__device__ __forceinline__ uint64_t smem_desc_nosw(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(lbo >> 4) << 16;
  d |= static_cast<uint64_t>(sbo >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100; layout 0 = no swizzle
  return d;
}

// LoRA slots of a tile with n runs: the runs, or (packed rank 8) pairs of runs.
__device__ __forceinline__ int lora_slots(int pack8, int nruns) { return pack8 ? (nruns + 1) / 2 : nruns; }

// LoRA runs of m-tile m_pos are stored at its tile id (tile_list[m_pos] with a list).
__device__ __forceinline__ int run_slot(const KParams& p, int m_pos) { return p.tile_list ? p.tile_list[m_pos] : m_pos; }

__device__ __forceinline__ int tile_lora_runs(const KParams& p, int m_pos) {
  if (p.rank == 0) return 0;
  const int n = p.tile_nruns[run_slot(p, m_pos)];
  return n < kMaxRunsPerTile ? n : kMaxRunsPerTile;
}
// Run r of the tile whose runs are in slot `slot`.
__device__ __forceinline__ const int32_t* tile_run(const KParams& p, int slot, int r) {
  return p.tile_runs + ((int64_t)slot * kMaxRunsPerTile + min(r, kMaxRunsPerTile - 1)) * 5;
}

// 16 e4m3 values (one 16-byte chunk) -> 16 x 16-bit, scaled.
template <typename T>
__device__ __forceinline__ void dequant16(const uint4& q, float s, uint4& lo, uint4& hi) {
  const __nv_fp8x2_storage_t* p2 = reinterpret_cast<const __nv_fp8x2_storage_t*>(&q);
  float f[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(p2[i], __NV_E4M3);
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    f[2 * i] = v.x * s;
    f[2 * i + 1] = v.y * s;
  }
  float a[8], b[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    a[i] = f[i];
    b[i] = f[8 + i];
  }
  lo = pack8<T>(a);
  hi = pack8<T>(b);
}

template <typename T, bool FP8B>
__global__ void __launch_bounds__(Cfg<FP8B>::THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_lb,
                        const KParams p) {
  constexpr int STAGES = Cfg<FP8B>::STAGES;
  constexpr int STAGE_BYTES = Cfg<FP8B>::STAGE_BYTES;
  constexpr int CONV = Cfg<FP8B>::CONV;
  extern __shared__ uint8_t smem_raw[];
  // Every CTA waits before anything else, the ones that leave at once too, so that
  // this grid never completes ahead of the kernel before it.
  pdl_wait();
  pdl_trigger();
  // 1024-byte alignment for the 128B-swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* conv_smem = smem + STAGES * STAGE_BYTES;  // FP8 weights: CONV converted B tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(conv_smem + CONV * B_STAGE_BYTES);
  // bars: [0,S) full (the stage's copies landed), [S,2S) empty, [2S,2S+2) tmem_full,
  // [2S+2,2S+4) tmem_empty, [2S+4] drain; FP8 weights: [2S+5,2S+5+C) conv_full (a
  // converted B tile is ready), [2S+5+C,2S+5+2C) conv_empty (the MMAs are done with it),
  // [2S+5+2C,3S+5+2C) lseen (every converter saw a LoRA block's stage land)
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + Cfg<FP8B>::NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  uint64_t* hdr_bar_p = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(bars) + 192);
  const int32_t* hdr_smem = reinterpret_cast<const int32_t*>(reinterpret_cast<uint8_t*>(bars) + 256);
  uint64_t* mrun_bar_p = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(bars) + 200);
  const int32_t* mruns_smem = reinterpret_cast<const int32_t*>(reinterpret_cast<uint8_t*>(bars) + 1024);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t smem_base = smem_u32(smem);
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + 2 + a]); };
  const uint32_t drain_bar = smem_u32(&bars[2 * STAGES + 4]);
  auto conv_full_bar = [&](int c) { return smem_u32(&bars[2 * STAGES + 5 + c]); };
  auto conv_empty_bar = [&](int c) { return smem_u32(&bars[2 * STAGES + 5 + CONV + c]); };
  // The converters wait on every stage of the ring in order (they are never two phases
  // behind a stage's barrier); a LoRA block's stage is released only after all of them
  // saw it land, so the ring cannot lap them while they skip it.
  auto lseen_bar = [&](int st) { return smem_u32(&bars[2 * STAGES + 5 + 2 * CONV + st]); };
  auto land_bar = [&](int s) { return full_bar(s); };
  const uint32_t conv_base = smem_u32(conv_smem);

  // Beside the pair kernel only the first `nctas` CTAs work; the others leave at once.
  int nctas = gridDim.x;
  if (p.split_sms > 0) {
    nctas = min(nctas, split_single_ctas(p.split_pairs_dev, p.split_singles_dev, p.split_cap, p.split_sms));
    if ((int)blockIdx.x >= nctas) return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int c = 0; c < CONV; ++c) {
      mbar_init(conv_full_bar(c), CONVERTER_THREADS);
      mbar_init(conv_empty_bar(c), 1);
    }
    if (FP8B)
      for (int st = 0; st < STAGES; ++st) mbar_init(lseen_bar(st), CONVERTER_THREADS);
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(drain_bar, 1);
    mbar_init(smem_u32(hdr_bar_p), 1);
    mbar_init(smem_u32(mrun_bar_p), 1);
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

  const int num_m_tiles = (p.tile_group || p.tile_list) ? min(*p.num_tiles_dev, p.tiles_cap)
                                                        : (int)((p.m_rows + BM - 1) / BM);
  const int total_tiles = num_m_tiles * p.num_n_tiles;
  const int num_kb = (p.K + BK - 1) / BK;
  volatile int never_abort = 0;  // the drain waits below ignore the abort flag

  if (threadIdx.x == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    if (p.rank) {
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_lb);
    }
    const uint64_t pol_a = l2_policy_evict_last();
    const uint64_t pol_b = l2_policy_evict_normal();
    int last_phase[STAGES];
    for (int s = 0; s < STAGES; ++s) last_phase[s] = -1;
    uint32_t it = 0, hdr_uses = 0;
    bool ok = true;
    const uint32_t hdr_bar = smem_u32(hdr_bar_p);
    bool hdr_inflight = false;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += nctas) {
      int m_pos, n_tile;
      unit_mn(p, tile, num_m_tiles, m_pos, n_tile);
      const int m_tile = p.tile_list ? p.tile_list[m_pos] : m_pos;
      int nruns = 0;
      if (p.rank) {  // the tile's first runs arrive while the K loop's copies are issued
        mbar_arrive_expect_tx(hdr_bar, kHdrRuns * 5 * 4);
        bulk_load_1d(smem_u32(hdr_smem), p.tile_runs + (int64_t)m_tile * kMaxRunsPerTile * 5, kHdrRuns * 5 * 4,
                     hdr_bar);
        hdr_inflight = true;
        nruns = tile_lora_runs(p, m_pos);  // used after the K loop
      }
      const int group = p.tile_group ? p.tile_group[m_tile] : 0;
      const int a_row = m_tile * BM;
      const int n0 = p.swiglu ? n_tile * 128 : n_tile * BN;
      const int b_row0 = weight_group(p.b_group_map, group) * p.b_group_rows + n0;
      const int b_row1 = p.swiglu ? b_row0 + p.N : b_row0 + 128;
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(empty_bar(s), ph ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        const uint32_t sa = smem_base + s * STAGE_BYTES;
        if (FP8B) {
          const uint32_t sraw = sa + A_STAGE_BYTES;
          mbar_arrive_expect_tx(full_bar(s), A_STAGE_BYTES + RAW_B_BYTES);
          tma_load_2d(sa, &tm_a, full_bar(s), kb * BK, a_row, pol_a);
          tma_load_2d(sraw, &tm_b, full_bar(s), kb * BK, b_row0, pol_b);
          tma_load_2d(sraw + 128 * BK, &tm_b, full_bar(s), kb * BK, b_row1, pol_b);
        } else {
          const uint32_t sbm = sa + A_STAGE_BYTES;
          mbar_arrive_expect_tx(full_bar(s), MMA_STAGE_BYTES);
          tma_load_2d(sa, &tm_a, full_bar(s), kb * BK, a_row, pol_a);
          tma_load_2d(sbm, &tm_b, full_bar(s), kb * BK, b_row0, pol_b);
          tma_load_2d(sbm + 128 * BK * 2, &tm_b, full_bar(s), kb * BK, b_row1, pol_b);
        }
        last_phase[s] = (int)ph;
      }
      // LoRA blocks: S of the tile + B rows of each tenant run
      if (p.rank && ok) {
        ok = mbar_wait(hdr_bar, hdr_uses & 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutProducer);
        ++hdr_uses;
        hdr_inflight = !ok;
      }
      if (!ok) nruns = 0;
      const int nslots = lora_slots(p.pack8, nruns);
      for (int r0 = 0; ok && r0 < nslots; r0 += p.runs_per_block, ++it) {
        const int nr = min(p.runs_per_block, nslots - r0);
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(empty_bar(s), ph ^ 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        const uint32_t base = smem_base + s * STAGE_BYTES;
        const uint32_t bar = land_bar(s);
        mbar_arrive_expect_tx(bar, p.s_bytes + nr * p.run_bytes);
        for (int ch = 0; ch < p.lchunks; ++ch) {
          if (p.swiglu)  // one 3-D box: the gate chunk and, r columns on, the up chunk
            tma_load_3d(base + ch * 2 * LCHUNK, &tm_s, bar, ch * 16, a_row, 0, pol_a);
          else
            tma_load_2d(base + ch * LCHUNK, &tm_s, bar, ch * 16, a_row, pol_a);
        }
        for (int jj = 0; jj < nr && p.pack8; ++jj) {
          // packed rank 8: the 8 B columns of runs 2q and 2q+1 in two 16-byte-row blocks
          // (no swizzle), K columns 0-7 and 8-15 of one K = 16 step
          for (int h = 0; h < 2; ++h) {
            const int r = 2 * (r0 + jj) + h;
            const uint32_t dst = base + p.s_bytes + jj * p.run_bytes + h * (p.run_bytes / 2);
            int brow = 0, x = 8;  // no second run: a box past the 8 columns, all zeros
            if (r < nruns) {
              const int tenant = r < kHdrRuns ? hdr_smem[r * 5] : tile_run(p, m_tile, r)[0];
              brow = (int)(tenant * p.lb_tenant_rows + group * p.lb_group_rows) + n0;
              x = 0;
            }
            if (p.swiglu)
              tma_load_3d(dst, &tm_lb, bar, x, brow, 0, pol_b);
            else
              tma_load_2d(dst, &tm_lb, bar, x, brow, pol_b);
          }
        }
        for (int jj = 0; jj < nr && !p.pack8; ++jj) {
          const int r = r0 + jj;
          const int tenant = r < kHdrRuns ? hdr_smem[r * 5] : tile_run(p, m_tile, r)[0];
          const int brow = (int)(tenant * p.lb_tenant_rows + group * p.lb_group_rows) + n0;
          const uint32_t rb = base + p.s_bytes + jj * p.run_bytes;
          // one box per 16-column chunk: the gate rows and, N rows on, the up rows (3-D), or
          // all 256 rows of the tile
          for (int ch = 0; ch < p.lchunks; ++ch) {
            if (p.swiglu)
              tma_load_3d(rb + ch * 2 * LCHUNK, &tm_lb, bar, ch * 16, brow, 0, pol_b);
            else
              tma_load_2d(rb + ch * 2 * LCHUNK, &tm_lb, bar, ch * 16, brow, pol_b);
          }
        }
        last_phase[s] = (int)ph;
      }
    }
    if (!ok) {
      // Let the copies already in flight land before the CTA exits.
      if (hdr_inflight) mbar_wait(hdr_bar, hdr_uses & 1, &never_abort, p.status, 1000000000ull, kDevTimeoutDrain);
      for (int s = 0; s < STAGES; ++s)
        if (last_phase[s] >= 0)
          mbar_wait(land_bar(s), (uint32_t)last_phase[s], &never_abort, p.status, 1000000000ull, kDevTimeoutDrain);
    }
  } else if (threadIdx.x == 32) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_f16(BM, BN, IsBf16<T>::value);
    const uint32_t idesc_n128 = idesc_f16(BM, 128, IsBf16<T>::value);
    uint32_t it = 0, cv = 0;
    uint32_t lpar = 0;  // FP8 weights: parity bit per stage of its next LoRA use
    int tcount = 0;
    bool ok = true;
    bool issued_any = false;
    const uint32_t mrun_bar = smem_u32(mrun_bar_p);
    uint32_t mrun_uses = 0;
    bool mrun_inflight = false;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += nctas, ++tcount) {
      const int acc = tcount & 1;
      const uint32_t aph = (tcount >> 1) & 1;
      int m_pos, n_tile_unused;
      unit_mn(p, tile, num_m_tiles, m_pos, n_tile_unused);
      const int slot = run_slot(p, m_pos);
      // the tile's run count (used after the K loop) and first kHdrRuns runs, in flight meanwhile
      const int nruns_unit = tile_lora_runs(p, m_pos);
      if (p.rank) {
        fence_proxy_async_smem();  // the previous unit's reads of the buffer come first
        mbar_arrive_expect_tx(mrun_bar, kHdrRuns * 5 * 4);
        bulk_load_1d(smem_u32(mruns_smem), p.tile_runs + (int64_t)slot * kMaxRunsPerTile * 5, kHdrRuns * 5 * 4,
                     mrun_bar);
        mrun_inflight = true;
      }
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
        const int c = FP8B ? (int)(cv % CONV) : 0;
        if (FP8B && !mbar_wait(conv_full_bar(c), (cv / CONV) & 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_base + s * STAGE_BYTES;
        const uint64_t adesc = smem_desc_sw128(sa);
        const uint64_t bdesc = smem_desc_sw128(FP8B ? conv_base + c * B_STAGE_BYTES : sa + A_STAGE_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        tc_commit(empty_bar(s));
        if (FP8B) {
          tc_commit(conv_empty_bar(c));
          ++cv;
        }
        issued_any = true;
      }
      if (ok && p.rank) {
        ok = mbar_wait(mrun_bar, mrun_uses & 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma);
        mrun_inflight = !ok;
        ++mrun_uses;
      }
      const int nruns = ok ? nruns_unit : 0;
      const int nslots = lora_slots(p.pack8, nruns);
      for (int r0 = 0; ok && r0 < nslots; r0 += p.runs_per_block, ++it) {
        const int nr = min(p.runs_per_block, nslots - r0);
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(full_bar(s), ph, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        if (FP8B) {
          if (!mbar_wait(lseen_bar(s), (lpar >> s) & 1u, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          lpar ^= 1u << s;
        }
        tc_fence_after();
        const uint32_t base = smem_base + s * STAGE_BYTES;
        for (int jj = 0; jj < nr && p.pack8; ++jj) {
          // two runs in one K = 16 step: S holds each row's values in the 8 columns of its
          // run's parity, so one MASKED MMA over the rows of both runs adds both products
          const int ra = 2 * (r0 + jj), rb2 = ra + 1;
          const int32_t* run_a = ra < kHdrRuns ? mruns_smem + ra * 5 : tile_run(p, slot, ra);
          uint32_t m0 = (uint32_t)run_a[1], m1 = (uint32_t)run_a[2], m2 = (uint32_t)run_a[3], m3 = (uint32_t)run_a[4];
          if (rb2 < nruns) {
            const int32_t* run_b = rb2 < kHdrRuns ? mruns_smem + rb2 * 5 : tile_run(p, slot, rb2);
            m0 |= (uint32_t)run_b[1];
            m1 |= (uint32_t)run_b[2];
            m2 |= (uint32_t)run_b[3];
            m3 |= (uint32_t)run_b[4];
          }
          const uint32_t rb = base + p.s_bytes + jj * p.run_bytes;
          const uint32_t half = (uint32_t)p.run_bytes / 2;  // run b's block after run a's
          if (p.swiglu) {
            tc_mma_f16_masked(d_tmem, smem_desc_sw32(base), smem_desc_nosw(rb, half, 128), idesc_n128, 1u, ~m0, ~m1,
                              ~m2, ~m3);
            tc_mma_f16_masked(d_tmem + 128, smem_desc_sw32(base + LCHUNK), smem_desc_nosw(rb + half / 2, half, 128),
                              idesc_n128, 1u, ~m0, ~m1, ~m2, ~m3);
          } else {
            tc_mma_f16_masked(d_tmem, smem_desc_sw32(base), smem_desc_nosw(rb, half, 128), idesc, 1u, ~m0, ~m1, ~m2,
                              ~m3);
          }
        }
        for (int jj = 0; jj < nr && !p.pack8; ++jj) {
          const int r = r0 + jj;
          const int32_t* run = r < kHdrRuns ? mruns_smem + r * 5 : tile_run(p, slot, r);
          const uint32_t d0 = ~(uint32_t)run[1], d1 = ~(uint32_t)run[2], d2 = ~(uint32_t)run[3],
                         d3 = ~(uint32_t)run[4];
          const uint32_t rb = base + p.s_bytes + jj * p.run_bytes;
          for (int ch = 0; ch < p.lchunks; ++ch) {
            if (p.swiglu) {
              tc_mma_f16_masked(d_tmem, smem_desc_sw32(base + ch * 2 * LCHUNK), smem_desc_sw32(rb + ch * 2 * LCHUNK),
                                idesc_n128, 1u, d0, d1, d2, d3);
              tc_mma_f16_masked(d_tmem + 128, smem_desc_sw32(base + (2 * ch + 1) * LCHUNK),
                                smem_desc_sw32(rb + (2 * ch + 1) * LCHUNK), idesc_n128, 1u, d0, d1, d2, d3);
            } else {
              tc_mma_f16_masked(d_tmem, smem_desc_sw32(base + ch * LCHUNK), smem_desc_sw32(rb + ch * 2 * LCHUNK),
                                idesc, 1u, d0, d1, d2, d3);
            }
          }
        }
        tc_commit(empty_bar(s));
      }
      if (!ok) break;
      tc_commit(tfull_bar(acc));
    }
    if (mrun_inflight) mbar_wait(mrun_bar, mrun_uses & 1, &never_abort, p.status, 200000000ull, kDevTimeoutDrain);
    if (!ok && issued_any) {
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, &never_abort, p.status, 1000000000ull, kDevTimeoutDrain);
    }
  } else if (warp >= 2 && warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const T* bias = reinterpret_cast<const T*>(p.bias);
    T* out = reinterpret_cast<T*>(p.out);
    const bool vec_ok = (p.ldo % 8 == 0) && (p.N % 8 == 0);
    int tcount = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += nctas, ++tcount) {
      const int acc = tcount & 1;
      const uint32_t aph = (tcount >> 1) & 1;
      if (!mbar_wait(tfull_bar(acc), aph, abort_flag, p.status, p.timeout_ns, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      int m_pos, n_tile;
      unit_mn(p, tile, num_m_tiles, m_pos, n_tile);
      const int m_tile = p.tile_list ? p.tile_list[m_pos] : m_pos;
      const int group = p.tile_group ? p.tile_group[m_tile] : 0;
      const int64_t row = (int64_t)m_tile * BM + row_in_tile;
      const bool row_ok = p.tile_group ? true : (row < p.m_rows);
      const float rscale = (row_ok && p.row_scale) ? p.row_scale[row] : 1.f;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;

      if (p.swiglu) {
        const int n0 = n_tile * 128;
        for (int c = 0; c < 128; c += 16) {
          uint32_t rg[16], ru[16];
          tmem_ld_x16(t_row + c, rg);
          tmem_ld_x16(t_row + 128 + c, ru);
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
        const int n0 = n_tile * BN;
        for (int c = 0; c < BN; c += 16) {
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
      if (lane == 0) mbar_arrive(tempty_bar(acc));
    }
  } else if (FP8B && warp >= 6) {
    // ------------------------------------------------------------ e4m3 -> 16-bit converters
    // Item (r, c): row r of the 256-row B tile, 16-byte chunk c (16 weights) of its 64-byte
    // e4m3 row; written as 16-bit logical chunks 2c, 2c+1 of the 128-byte row, stored at
    // physical chunk (logical ^ (r & 7)) -- the 128B swizzle the MMA descriptor expects.
    const int ct = threadIdx.x - 192;
    uint32_t it = 0, cv = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += nctas) {
      int m_pos, n_tile;
      unit_mn(p, tile, num_m_tiles, m_pos, n_tile);
      const int m_tile = p.tile_list ? p.tile_list[m_pos] : m_pos;
      const int group = p.tile_group ? p.tile_group[m_tile] : 0;
      const int n0 = p.swiglu ? n_tile * 128 : n_tile * BN;
      const int64_t b_row0 = (int64_t)weight_group(p.b_group_map, group) * p.b_group_rows + n0;
      const int64_t b_row1 = p.swiglu ? b_row0 + p.N : b_row0 + 128;
      const int tile_nruns = tile_lora_runs(p, m_pos);  // used after the K loop
      float sc[CONV_ITEMS];
      int rr[CONV_ITEMS], cc[CONV_ITEMS];
#pragma unroll
      for (int q = 0; q < CONV_ITEMS; ++q) {
        const int idx = ct + CONVERTER_THREADS * q;
        rr[q] = idx >> 2;
        cc[q] = idx & 3;
        const int64_t grow = rr[q] < 128 ? b_row0 + rr[q] : b_row1 + (rr[q] - 128);
        sc[q] = grow < p.b_rows_total ? p.b_row_scale[grow] : 0.f;
      }
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb, ++it, ++cv) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const int c = (int)(cv % CONV);
        if (!mbar_wait(full_bar(s), ph, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma) ||
            !mbar_wait(conv_empty_bar(c), ((cv / CONV) & 1) ^ 1, abort_flag, p.status, p.timeout_ns,
                       kDevTimeoutMma)) {
          ok = false;
          break;
        }
        const uint8_t* raw = smem + s * STAGE_BYTES + A_STAGE_BYTES;
        uint8_t* bt = conv_smem + c * B_STAGE_BYTES;
#pragma unroll
        for (int q = 0; q < CONV_ITEMS; ++q) {
          const uint4 qv = *reinterpret_cast<const uint4*>(raw + rr[q] * BK + cc[q] * 16);
          uint4 lo, hi;
          dequant16<T>(qv, sc[q], lo, hi);
          uint8_t* row = bt + rr[q] * 128;
          const int sw = rr[q] & 7;
          *reinterpret_cast<uint4*>(row + (((2 * cc[q]) ^ sw) << 4)) = lo;
          *reinterpret_cast<uint4*>(row + (((2 * cc[q] + 1) ^ sw) << 4)) = hi;
        }
        fence_proxy_async_smem();
        mbar_arrive(conv_full_bar(c));
      }
      // LoRA blocks (16-bit already) go from the TMA ring to the MMAs; the converters only
      // report that they saw each one land
      const int nslots = ok ? lora_slots(p.pack8, tile_nruns) : 0;
      for (int r0 = 0; ok && r0 < nslots; r0 += p.runs_per_block, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(full_bar(s), (it / STAGES) & 1, abort_flag, p.status, p.timeout_ns, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        mbar_arrive(lseen_bar(s));
      }
      if (!ok) break;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// One warp per 128-row tile: distinct tenants (in first-seen order over the
// 4 row quarters) and the 128-bit mask of the rows each one owns.
// The run index a leader lane took in tile_runs_kernel's matching round (found, or a
// new index after the `base` runs known before the round).
__device__ __forceinline__ int idx_or(bool leader, int found, int base, unsigned is_new, int lane) {
  if (!leader) return -1;
  return found >= 0 ? found : base + __popc(is_new & ((1u << lane) - 1u));
}

__global__ void __launch_bounds__(128) tile_runs_kernel(const int32_t* __restrict__ row_tenant,
                                                        const int32_t* __restrict__ num_tiles_dev,
                                                        int64_t static_rows, int tiles_cap, int32_t* __restrict__ runs,
                                                        int32_t* __restrict__ nruns,
                                                        const int32_t* __restrict__ tile_list,
                                                        int8_t* __restrict__ row_run) {
  __shared__ int32_t s_ten[4][kMaxRunsPerTile];
  __shared__ uint32_t s_mask[4][kMaxRunsPerTile][4];
  pdl_wait();  // the plan and the tenants may come from the previous kernels
  pdl_trigger();
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * 4 + w;  // entry of the output (and of tile_list)
  const int ntiles = num_tiles_dev ? min(*num_tiles_dev, tiles_cap) : (int)((static_rows + 127) / 128);
  if (tile >= ntiles) return;
  const int64_t src_tile = tile_list ? tile_list[tile] : tile;
  const int64_t rows_active = tile_list ? (static_rows > 0 ? static_rows : INT64_MAX)
                                        : (num_tiles_dev ? (int64_t)ntiles * 128 : static_rows);
  int count = 0;
  for (int q = 0; q < 4; ++q) {
    const int64_t row = src_tile * 128 + q * 32 + lane;
    const int t = row < rows_active ? row_tenant[row] : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, t);
    const bool leader = (t >= 0) && ((peers & ((1u << lane) - 1u)) == 0u);
    int found = -1;
    if (leader)
      for (int j = 0; j < count; ++j)
        if (s_ten[w][j] == t) {
          found = j;
          break;
        }
    const unsigned is_new = __ballot_sync(0xffffffffu, leader && found < 0);
    if (leader) {
      int idx = found;
      if (found < 0) {
        idx = count + __popc(is_new & ((1u << lane) - 1u));
        s_ten[w][idx] = t;
        for (int qq = 0; qq < 4; ++qq) s_mask[w][idx][qq] = 0u;
      }
      s_mask[w][idx][q] = peers;
    }
    count += __popc(is_new);
    if (row_run) {  // every row learns its run index from its leader
      const int my_idx = __shfl_sync(0xffffffffu, idx_or(leader, found, count - __popc(is_new), is_new, lane),
                                     t >= 0 ? __ffs(peers) - 1 : lane);
      row_run[src_tile * 128 + q * 32 + lane] = (int8_t)(t >= 0 ? my_idx : -1);
    }
    __syncwarp();
  }
  for (int j = lane; j < count; j += 32) {
    int32_t* r = runs + ((int64_t)src_tile * kMaxRunsPerTile + j) * 5;
    r[0] = s_ten[w][j];
    r[1] = (int32_t)s_mask[w][j][0];
    r[2] = (int32_t)s_mask[w][j][1];
    r[3] = (int32_t)s_mask[w][j][2];
    r[4] = (int32_t)s_mask[w][j][3];
  }
  if (lane == 0) nruns[src_tile] = count;
}

template <typename T, bool FP8B>
int launch_gemm_kernel(int grid, cudaStream_t stream, bool pdl, const CUtensorMap& tm_a, const CUtensorMap& tm_b,
                       const CUtensorMap& tm_s, const CUtensorMap& tm_lb, const KParams& p) {
  SB_CUDA_CHECK(cudaFuncSetAttribute(grouped_gemm_kernel<T, FP8B>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Cfg<FP8B>::SMEM_BYTES));
  SB_CUDA_CHECK(launch_kernel(grouped_gemm_kernel<T, FP8B>, dim3(grid), dim3(Cfg<FP8B>::THREADS),
                              Cfg<FP8B>::SMEM_BYTES, stream, pdl, tm_a, tm_b, tm_s, tm_lb, p));
  ::sb::count_launch();
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

}  // namespace

int launch_tile_runs(const int32_t* row_tenant, const int32_t* num_tiles_dev, int64_t static_rows, int tiles_cap,
                     int32_t* runs, int32_t* nruns, cudaStream_t stream, const int32_t* tile_list, bool pdl,
                     int8_t* row_run) {
  SB_CHECK_ARG(row_tenant && runs && nruns, "tile_runs: null pointer");
  SB_CHECK_ARG(!tile_list || num_tiles_dev, "tile_runs: a tile list needs its device count");
  const int64_t tiles = num_tiles_dev ? tiles_cap : (static_rows + 127) / 128;
  if (tiles == 0) return STAGEML_OK;
  SB_CUDA_CHECK(launch_kernel(tile_runs_kernel, dim3((unsigned)((tiles + 3) / 4)), dim3(128), 0, stream, pdl,
                              row_tenant, num_tiles_dev, static_rows, tiles_cap, runs, nruns, tile_list, row_run));
  ::sb::count_launch();
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

int launch_grouped_gemm(const GemmLaunch& g, cudaStream_t stream) {
  SB_CHECK_ARG(g.a && g.b && g.out, "grouped gemm: null operand");
  SB_CHECK_ARG(g.K > 0 && g.K % 8 == 0, "grouped gemm: K=%d must be a positive multiple of 8", g.K);
  SB_CHECK_ARG(!g.b_fp8 || g.K % 16 == 0, "grouped gemm: FP8 weights need K=%d to be a multiple of 16", g.K);
  SB_CHECK_ARG(!g.b_fp8 || g.b_scale, "grouped gemm: FP8 weights need per-row scales");
  SB_CHECK_ARG(g.N > 0, "grouped gemm: N must be positive");
  SB_CHECK_ARG(g.rank == 0 || g.rank == 8 || g.rank == 16 || g.rank == 32,
               "grouped gemm: LoRA rank %d must be 0, 8, 16 or 32", g.rank);
  SB_CHECK_ARG(g.rank == 0 || (g.s16 && g.lora_b && (g.pairs ? (g.pair_runs && g.pair_nruns) : (g.tile_runs && g.tile_nruns)) &&
                               g.s_rows > 0 && g.lora_b_rows_total > 0),
               "grouped gemm: LoRA rank > 0 needs S, B, the tile runs and their sizes");
  SB_CHECK_ARG((reinterpret_cast<uintptr_t>(g.a) % 16) == 0 && (reinterpret_cast<uintptr_t>(g.b) % 16) == 0,
               "grouped gemm: operands must be 16-byte aligned");
  SB_CHECK_ARG(g.b_rows_total < (int64_t(1) << 31) && g.a_rows < (int64_t(1) << 31),
               "grouped gemm: operand rows exceed the TMA coordinate range");
  SB_CHECK_ARG(g.lora_b_rows_total < (int64_t(1) << 31), "grouped gemm: LoRA bank exceeds the TMA coordinate range");
  if (g.pairs) return launch_grouped_gemm_pair(g, stream);

  const CUtensorMapDataType dt = g.in_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tm_a, tm_b, tm_s, tm_lb;
  SB_TRY(make_tmap_2d(&tm_a, g.a, dt, 2, (uint64_t)g.a_rows, (uint64_t)g.K, (uint64_t)g.K * 2, BM, BK, 128));
  if (g.b_fp8)
    SB_TRY(make_tmap_2d(&tm_b, g.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)g.b_rows_total, (uint64_t)g.K,
                        (uint64_t)g.K, 128, BK, 0));
  else
    SB_TRY(make_tmap_2d(&tm_b, g.b, dt, 2, (uint64_t)g.b_rows_total, (uint64_t)g.K, (uint64_t)g.K * 2, 128, BK, 128));
  const int lora_cols = g.swiglu ? 2 * g.rank : g.rank;
  if (g.rank) {
    // rank 8: the 16-wide boxes read past the 8 columns of a rank, which TMA fills with
    // zeros, so the K=16 MMA adds nothing for the other 8 columns of its operands.
    // SwiGLU: one 3-D box per 16-column chunk loads both halves -- S: the gate columns
    // [c, c+16) and, r columns on, the up columns; B: the tile's gate rows and, N rows
    // on, its up rows. The row extents stop where the up half would leave the
    // allocation: d1 = S rows, and B rows - N (every gate row a tile loads lies below).
    if (g.pack8) {
      // S in the run-parity layout: 16 columns per half ([rows][32] SwiGLU, [rows][16]
      // otherwise); B: one run's 8 columns per box, 16-byte rows without swizzle
      SB_CHECK_ARG(g.rank == 8, "grouped gemm: packed LoRA needs rank 8");
      if (g.swiglu) {
        SB_TRY(make_tmap_3d(&tm_s, g.s16, dt, 2, 16, (uint64_t)g.s_rows, 2, 64, 32, 16, 128, 2, 32));
        SB_TRY(make_tmap_3d(&tm_lb, g.lora_b, dt, 2, 8, (uint64_t)(g.lora_b_rows_total - g.N), 2, 16,
                            (uint64_t)g.N * 16, 8, 128, 2, 0));
      } else {
        SB_TRY(make_tmap_2d(&tm_s, g.s16, dt, 2, (uint64_t)g.s_rows, 16, 32, 128, 16, 32));
        SB_TRY(make_tmap_2d(&tm_lb, g.lora_b, dt, 2, (uint64_t)g.lora_b_rows_total, 8, 16, 256, 8, 0));
      }
    } else if (g.swiglu) {
      SB_TRY(make_tmap_3d(&tm_s, g.s16, dt, 2, (uint64_t)g.rank, (uint64_t)g.s_rows, 2, (uint64_t)lora_cols * 2,
                          (uint64_t)g.rank * 2, 16, 128, 2, 32));
      SB_TRY(make_tmap_3d(&tm_lb, g.lora_b, dt, 2, (uint64_t)g.rank, (uint64_t)(g.lora_b_rows_total - g.N), 2,
                          (uint64_t)g.rank * 2, (uint64_t)g.N * g.rank * 2, 16, 128, 2, 32));
    } else {
      SB_TRY(make_tmap_2d(&tm_s, g.s16, dt, 2, (uint64_t)g.s_rows, (uint64_t)lora_cols, (uint64_t)lora_cols * 2, 128,
                          16, 32));
      SB_TRY(make_tmap_2d(&tm_lb, g.lora_b, dt, 2, (uint64_t)g.lora_b_rows_total, (uint64_t)g.rank,
                          (uint64_t)g.rank * 2, 256, 16, 32));
    }
  } else {
    tm_s = tm_a;  // unused
    tm_lb = tm_a;
  }

  KParams p;
  p.K = g.K;
  p.N = g.N;
  p.b_group_rows = g.b_group_rows;
  p.b_group_map = g.b_group_map;
  p.b_rows_total = g.b_rows_total;
  p.swiglu = g.swiglu ? 1 : 0;
  p.num_n_tiles = g.swiglu ? (g.N + 127) / 128 : (g.N + BN - 1) / BN;
  p.num_tiles_dev = g.num_tiles_dev;
  p.tiles_cap = g.tiles_cap;
  p.tile_group = g.tile_group;
  p.tile_list = g.tile_list;
  p.group_offsets = (g.tile_group && !g.tile_list) ? g.group_offsets : nullptr;
  p.m_rows = g.m_rows;
  p.rank = g.rank;
  p.lchunks = (g.rank + 15) / 16;
  p.s_bytes = (g.swiglu ? 2 : 1) * p.lchunks * LCHUNK;
  p.run_bytes = 2 * p.lchunks * LCHUNK;
  // a LoRA block (S and the runs' B rows) fills one TMA stage
  const int lora_block_bytes = g.b_fp8 ? Cfg<true>::STAGE_BYTES : Cfg<false>::STAGE_BYTES;
  p.runs_per_block = g.rank ? (lora_block_bytes - p.s_bytes) / p.run_bytes : 1;
  p.pack8 = g.pack8 ? 1 : 0;
  p.lb_tenant_rows = g.rank ? g.lora_b_tenant_stride / g.rank : 0;
  p.lb_group_rows = g.rank ? g.lora_b_group_stride / g.rank : 0;
  p.tile_runs = g.tile_runs;
  p.tile_nruns = g.tile_nruns;
  p.row_scale = g.row_scale;
  p.bias = g.bias;
  p.bias_group_stride = g.bias_group_stride;
  p.bias_group_mod = g.bias_group_mod;
  p.b_scale = g.b_fp8 ? nullptr : g.b_scale;
  p.b_row_scale = g.b_fp8 ? g.b_scale : nullptr;
  p.out = g.out;
  p.ldo = g.ldo;
  p.status = g.status;
  p.timeout_ns = kDefaultWaitNs;
  p.split_pairs_dev = g.split_pairs_dev;
  p.split_singles_dev = g.split_singles_dev;
  p.split_cap = g.split_cap;
  p.split_sms = (g.split_pairs_dev && g.split_singles_dev) ? g.split_sms : 0;

  int64_t tiles_upper = (g.tile_group || g.tile_list) ? (int64_t)g.tiles_cap : (g.m_rows + BM - 1) / BM;
  tiles_upper *= p.num_n_tiles;
  if (tiles_upper == 0) return STAGEML_OK;
  const int grid = (int)std::min<int64_t>(tiles_upper, sm_count());

  if (g.b_fp8)
    return g.in_bf16 ? launch_gemm_kernel<bf16, true>(grid, stream, g.pdl, tm_a, tm_b, tm_s, tm_lb, p)
                     : launch_gemm_kernel<f16, true>(grid, stream, g.pdl, tm_a, tm_b, tm_s, tm_lb, p);
  return g.in_bf16 ? launch_gemm_kernel<bf16, false>(grid, stream, g.pdl, tm_a, tm_b, tm_s, tm_lb, p)
                   : launch_gemm_kernel<f16, false>(grid, stream, g.pdl, tm_a, tm_b, tm_s, tm_lb, p);
}

}  // namespace sb
