// Host-side launch description of the grouped tcgen05 GEMM (grouped_gemm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sb {

// out[row, n] = epilogue( sum_k A[row, k] * B[group(row) * b_group_rows + n, k]
//                         + lora(row, n) )
//
// A rows are either the padded permuted rows of a MoE plan (tile_group != nullptr:
// 128-row tile m belongs to group tile_group[m], the number of tiles is read from
// num_tiles_dev) or the rows of a plain matrix (tile_group == nullptr: group 0,
// rows >= m_rows are masked).
//
// LoRA expand (rank > 0) runs on the tensor cores into the same accumulator:
// for every tenant run of a tile (tile_runs: tenant + 128-bit row mask),
//   acc[rows of the run, n] += S[row, :] . Bl[tenant, group, n, :]
// with S the pre-scaled shrink output (16-bit, [s_rows, lora_cols]) and Bl the
// LoRA B bank (16-bit, element (tenant, group, n, j) at
// tenant*lora_b_tenant_stride + group*lora_b_group_stride + n*rank + j).
//
// SwiGLU mode: B group = [W1 (N rows); W3 (N rows)], S = [s1 | s3] (2*rank
// columns), Bl rows [0,N) for W1 and [N,2N) for W3; out = silu(g) * u.
// Plain mode: out = (acc * b_scale[col] + bias[col]) * row_scale[row].
// FP8 weights (b_fp8): B holds e4m3 codes and b_scale (required) the per-B-row
// scale; every weight is dequantised to the activation type before the MMA,
// so the epilogue applies no further scale.
struct GemmLaunch {
  const void* a = nullptr;       // [a_rows, K] 16-bit
  int64_t a_rows = 0;
  const int32_t* a_row_of = nullptr;  // skinny GEMM only: output row r reads A row a_row_of[r]
  int K = 0;
  const void* b = nullptr;       // [b_rows_total, K] 16-bit, or e4m3 when b_fp8
  int64_t b_rows_total = 0;
  bool b_fp8 = false;            // e4m3 weights, dequantised in shared memory with b_scale[row]
  int b_group_rows = 0;          // rows of B per group (N or 2N)
  const int32_t* b_group_map = nullptr;  // optional: the weights (and scales) of group g are B group
                                         // b_group_map[g] (several row groups reading one weight group)
  int N = 0;                     // output columns
  bool swiglu = false;
  bool in_bf16 = true;           // false: fp16
  // tiles
  const int32_t* num_tiles_dev = nullptr;
  int tiles_cap = 0;
  const int32_t* tile_group = nullptr;
  const int32_t* tile_list = nullptr;  // one-CTA kernel: process tiles tile_list[0 .. *num_tiles_dev)
  const int32_t* group_offsets = nullptr;  // one-CTA kernel, grouped rows: [groups + 1] padded row offsets
                                           // (group-major unit order; null: m-tile fastest)
  int64_t m_rows = 0;            // direct mode row count
  // LoRA (tensor-core expand)
  int rank = 0;                          // 0, 16 or 32
  const void* s16 = nullptr;             // [s_rows, lora_cols] 16-bit, pre-scaled shrink output
  int64_t s_rows = 0;
  const void* lora_b = nullptr;          // 16-bit bank
  int64_t lora_b_tenant_stride = 0;      // elements
  int64_t lora_b_group_stride = 0;       // elements
  int64_t lora_b_rows_total = 0;         // bank elements / rank
  const int32_t* tile_runs = nullptr;    // [tiles][128][5]: tenant, row-mask words 0..3
  const int32_t* tile_nruns = nullptr;   // [tiles]
  // epilogue
  const float* row_scale = nullptr;      // [rows] or null
  const void* bias = nullptr;            // 16-bit [G, N] or null
  int64_t bias_group_stride = 0;
  int bias_group_mod = 0;                // bias group = group % mod when > 0
  const float* b_scale = nullptr;        // fp32 per B row or null
  void* out = nullptr;                   // [rows, ldo] 16-bit
  int64_t ldo = 0;
  int32_t* status = nullptr;
  // CTA-pair kernel (grouped_gemm_pair.cu), used when `pairs` is set: the pair
  // list and per-pair LoRA runs written by launch_pair_plan.
  const int32_t* pairs = nullptr;        // [pairs_cap][4]
  const int32_t* num_pairs_dev = nullptr;
  int pairs_cap = 0;
  const int32_t* pair_runs = nullptr;    // [tiles][kMaxRunsPerPair][kPairRunInts], at each pair's first tile
  const int32_t* pair_nruns = nullptr;   // [tiles][kRunHdrInts] run headers, at each pair's first tile
  // A pair whose second tile is -1 is a half unit: its one tile on both CTAs (64 rows
  // each, M = 128 MMAs) instead of a pair with an idle half.
  bool pair_half_units = false;
  // rank 8 on the one-CTA kernel: S in the run-parity layout of the shrink reduce
  // (ShrinkLaunch::row_run) and the B rows of two runs in one K = 16 step
  bool pack8 = false;
  // Programmatic dependent launch (the kernels wait for the previous kernel first).
  bool pdl = false;
  // The pair kernel and the odd-tile kernel side by side (split_sms > 0): each
  // reads the pair and odd-tile counts and keeps only its share of the split_sms
  // SMs busy (split_single_ctas); the CTAs past its share exit at once.
  const int32_t* split_pairs_dev = nullptr;
  const int32_t* split_singles_dev = nullptr;
  int split_cap = 0;
  int split_sms = 0;
};

// CTAs of the odd-tile kernel next to the pair kernel on `sms` SMs: its share of
// the work (a pair unit keeps two SMs busy about as long as an odd-tile unit keeps
// one), at least one, leaving the pair kernel an even count of at least two.
__device__ __forceinline__ int split_single_ctas(const int32_t* n_pairs_dev, const int32_t* n_singles_dev, int cap,
                                                 int sms) {
  const int np = min(*n_pairs_dev, cap), ns = min(*n_singles_dev, cap);
  if (ns <= 0) return 0;
  if (np <= 0) return sms;
  const int64_t den = 2LL * np + ns;
  int s = (int)(((int64_t)sms * ns + den / 2) / den);
  s = max(1, min(s, sms - 2));
  if ((sms - s) & 1) s = min(s + 1, sms - 2);
  return s;
}

// Weight group of row group g (identity without a map).
__device__ __forceinline__ int weight_group(const int32_t* map, int g) { return map ? map[g] : g; }

int launch_grouped_gemm(const GemmLaunch& g, cudaStream_t stream);

// Distinct LoRA tenants of every 128-row tile and the rows each one owns:
// runs[(tile*128 + j)*5 + 0] = tenant, [1..4] = row mask words; nruns[tile].
// Rows with tenant < 0 belong to no run. Active rows: 128 * (*num_tiles_dev)
// (capped at tiles_cap tiles) or static_rows when num_tiles_dev is null.
// row_run (optional, [tiles * 128]): each row's run index in its tile, -1 for none.
int launch_tile_runs(const int32_t* row_tenant, const int32_t* num_tiles_dev, int64_t static_rows, int tiles_cap,
                     int32_t* runs, int32_t* nruns, cudaStream_t stream, const int32_t* tile_list = nullptr,
                     bool pdl = false, int8_t* row_run = nullptr);
// With tile_list, entry i covers tile tile_list[i] (i < *num_tiles_dev) and runs / nruns
// are indexed by that tile id; static_rows > 0 then bounds the rows read (direct rows).
constexpr int kMaxRunsPerTile = 128;

// CTA-pair variant of the grouped GEMM: 256-row tiles made of two 128-row tiles
// of the same group, computed by a two-CTA cluster (tcgen05 cta_group::2).
constexpr int kMaxRunsPerPair = 256;
constexpr int kPairRunInts = 9;  // tenant, 8 row-mask words
// Run header of a pair (at its first tile t): nruns[t * kRunHdrInts] = run count,
// [1 + j] = tenant of run j for j < kRunHdrInts - 1 (one 128-byte block the pair
// kernel's producer bulk-copies at the start of each unit).
constexpr int kRunHdrInts = 32;
int launch_grouped_gemm_pair(const GemmLaunch& g, cudaStream_t stream);

// Pair list and per-pair LoRA runs. Grouped rows (tile_group != nullptr): pairs of
// consecutive tiles of the same group, taken from the group's first tile
// (group_offsets[g] / 128), a trailing odd tile paired with -1. Direct rows:
// tiles (2j, 2j+1) of ceil(static_rows / 128). pairs[4p..4p+3] = first tile,
// second tile or -1, first pair of the group, pairs in the group. pairs_cap =
// tiles_cap (grouped) or the direct tile count. With row_tenant set, also writes the
// LoRA runs of every pair at its first tile t: runs[(t*kMaxRunsPerPair + j)*kPairRunInts
// + 0] = tenant, [1..8] = mask words over the pair's 256 rows; nruns[t].
// With `singles`, a group's trailing odd tile is listed there (count in *num_singles)
// instead of forming a pair with an idle half; the one-CTA kernel runs those tiles
// (GemmLaunch::tile_list), and with row_tenant and sruns / snruns their runs are
// written as launch_tile_runs does (at the tile id). With `hpairs`, a second pair
// list in which every trailing odd tile is a pair with second tile -1 (a half unit
// of GemmLaunch::pair_half_units), its runs written at the tile as for a pair.
// One launch.
int launch_pair_plan(const int32_t* tile_group, const int32_t* group_offsets, const int32_t* num_tiles_dev,
                     int tiles_cap, int64_t static_rows, const int32_t* row_tenant, int32_t* pairs,
                     int32_t* num_pairs, int32_t* runs, int32_t* nruns, cudaStream_t stream,
                     int32_t* singles = nullptr, int32_t* num_singles = nullptr, int32_t* sruns = nullptr,
                     int32_t* snruns = nullptr, int32_t* hpairs = nullptr, int32_t* num_hpairs = nullptr,
                     bool pdl = false);
size_t pair_runs_ints(int64_t pairs_cap);

// Weight-streaming variant for at most 16 valid rows per 128-row tile (decode-sized
// batches), skinny.cu: same GemmLaunch semantics (16-bit weights; LoRA from s16 /
// lora_b with the row's tenant), valid rows per tile from the group counts; max_rows
// bounds the valid rows of any tile (at most 8 selects the one-m8-block variant).
// pdl_mode 0: ordinary launch; 1: programmatic dependent launch that waits at the
// start; 2: PDL launch right after a kernel that writes only S (the shrink), which
// streams the weights before it waits -- everything else it reads must come from
// kernels before that one.
int launch_skinny_gemm(const GemmLaunch& g, const int32_t* row_tenant, const int32_t* group_offsets,
                       const int32_t* group_counts, cudaStream_t stream, int64_t max_rows = 16, int pdl_mode = 0);

}  // namespace sb
