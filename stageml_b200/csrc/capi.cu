// extern "C" entry points of libstageml_b200.so (include/stageml_b200.h).
// Each entry validates its arguments on the host, carves its scratch from the
// caller's workspace and launches the kernels of the path on `stream`.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "grouped_gemm.cuh"
#include "host_util.h"
#include "kernels.h"
#include "stage_timer.h"

// Launch `expr` as pipeline stage `stage` (timed when the stage timer is on).
#define SB_STAGE(stage, expr)           \
  do {                                  \
    ::sb::StageScope _scope(stage, st); \
    SB_TRY(expr);                       \
  } while (0)

namespace sb {
namespace {

constexpr int kAbiVersion = 2;  // 2: stageml_moe_args.fold_slot / n_fold

// Bump allocator over the caller's workspace; with base == nullptr it only
// measures (the *_workspace_bytes queries run the same carve).
struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <typename T>
  T* take(size_t n) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
  void* take_bytes(size_t n) { return take<uint8_t>(n); }
};

inline size_t esize(int dtype) {
  switch (dtype) {
    case STAGEML_F32:
    case STAGEML_I32:
      return 4;
    case STAGEML_BF16:
    case STAGEML_F16:
      return 2;
    case STAGEML_E4M3:
      return 1;
    case STAGEML_I64:
      return 8;
    default:
      return 0;
  }
}

inline bool is16(int dtype) { return dtype == STAGEML_BF16 || dtype == STAGEML_F16; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

void carve_plan(Carver& c, int64_t P, int n_groups, stageml_moe_plan* plan) {
  const int64_t rows_cap = stageml_plan_rows_cap(P, n_groups);
  plan->rows_cap = rows_cap;
  plan->row_token = c.take<int32_t>(rows_cap);
  plan->row_tenant = c.take<int32_t>(rows_cap);
  plan->row_weight = c.take<float>(rows_cap);
  plan->row_pair = c.take<int32_t>(rows_cap);
  plan->pair_row = c.take<int32_t>(std::max<int64_t>(P, 1));
  plan->tile_group = c.take<int32_t>(rows_cap / 128);
  plan->group_offsets = c.take<int32_t>(n_groups + 1);
  plan->group_counts = c.take<int32_t>(n_groups);
  plan->num_tiles = c.take<int32_t>(1);
}

// ------------------------------------------------------------------ CTA-pair GEMM plan
// Pairs of 128-row tiles for the CTA-pair grouped GEMM, the groups' trailing odd
// tiles for the one-CTA kernel, and the tenant runs of both, for one row layout
// (shared by every GEMM over those rows).
struct PairPlan {
  int32_t* pairs = nullptr;      // [tiles_cap, 4]
  int32_t* num_pairs = nullptr;  // [1]
  int32_t* pruns = nullptr;      // [tiles_cap, kMaxRunsPerPair, kPairRunInts]
  int32_t* pnruns = nullptr;     // [tiles_cap, kRunHdrInts] run headers
  int32_t* singles = nullptr;    // [tiles_cap]
  int32_t* num_singles = nullptr;
  int32_t* sruns = nullptr;      // [tiles_cap, kMaxRunsPerTile, 5]
  int32_t* snruns = nullptr;
  int32_t* hpairs = nullptr;     // [tiles_cap, 4]: the pairs with each odd tile as a half unit
  int32_t* num_hpairs = nullptr;
  int tiles_cap = 0;
  bool on() const { return pairs != nullptr; }
};

// The grouped GEMMs run on CTA pairs (tcgen05 cta_group::2) unless the
// environment sets STAGEML_GEMM_PAIRS=0 (one CTA per tile), read once per process.
bool gemm_pairs_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("STAGEML_GEMM_PAIRS");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Pairs pay off once the groups average two tiles: with fewer rows most groups are a
// single tile, which the plan would route to the one-CTA kernel anyway.
bool pairs_pay(int64_t rows, int n_groups) { return rows >= 256 * (int64_t)n_groups; }

// With per-token-tenant LoRA, pairs pay off only while the masked expand MMAs stay a
// small share of a pair's work: each tenant run of a 256-row pair costs about one K=16
// step of the pair's main loop (two N=128 masked MMAs over all 256 rows), against
// K/16 steps, and a pair holds about twice the runs of a 128-row tile. Runs per pair,
// rows spread evenly over (group, tenant): 256 / (rows per key) + 1. Measured: the
// Mixtral shape (17 runs per pair, K >= 4096) is even between the two kernels; the
// fine-grained shape (~34 runs, K = 1408) runs 21 % faster on one-CTA tiles.
bool pair_lora_pays(int64_t rows, int n_groups, int n_tenants, int k_min) {
  if (n_tenants <= 0 || rows <= 0 || n_groups <= 0 || k_min <= 0) return true;
  const double rows_per_key = (double)rows / ((double)n_groups * n_tenants);
  const double runs = 256.0 / std::max(rows_per_key, 1.0) + 1.0;
  return runs * 16.0 / k_min < 0.15;
}

void carve_pair_plan(Carver& c, int64_t tiles_cap, bool lora, PairPlan* pp) {
  *pp = PairPlan{};
  if (!gemm_pairs_enabled() || tiles_cap <= 0) return;
  pp->tiles_cap = (int)tiles_cap;
  pp->pairs = c.take<int32_t>((size_t)tiles_cap * 4);
  pp->num_pairs = c.take<int32_t>(1);
  pp->singles = c.take<int32_t>((size_t)tiles_cap);
  pp->num_singles = c.take<int32_t>(1);
  pp->hpairs = c.take<int32_t>((size_t)tiles_cap * 4);
  pp->num_hpairs = c.take<int32_t>(1);
  if (lora) {
    pp->pruns = c.take<int32_t>(pair_runs_ints(tiles_cap));
    pp->pnruns = c.take<int32_t>((size_t)tiles_cap * kRunHdrInts);
    pp->sruns = c.take<int32_t>((size_t)tiles_cap * kMaxRunsPerTile * 5);
    pp->snruns = c.take<int32_t>((size_t)tiles_cap);
  }
}

// Grouped rows (tile_group, group_offsets, num_tiles_dev from a plan) or direct
// rows (static_rows); row_tenant only when the GEMMs carry LoRA.
int build_pair_plan(const PairPlan& pp, const int32_t* tile_group, const int32_t* group_offsets,
                    const int32_t* num_tiles_dev, int64_t static_rows, const int32_t* row_tenant, cudaStream_t st,
                    bool pdl = false) {
  return launch_pair_plan(tile_group, group_offsets, num_tiles_dev, pp.tiles_cap, static_rows,
                          pp.pruns ? row_tenant : nullptr, pp.pairs, pp.num_pairs, pp.pruns, pp.pnruns, st,
                          pp.singles, pp.num_singles, pp.sruns, pp.snruns, pp.hpairs, pp.num_hpairs, pdl);
}

// Per host thread and device: a side stream and two events for running the odd tiles
// of a grouped GEMM next to the CTA-pair kernel.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
int side_stream(SideStream** out) {
  thread_local SideStream per_dev[64];
  int dev = 0;
  SB_CUDA_CHECK(cudaGetDevice(&dev));
  SB_CHECK_ARG(dev >= 0 && dev < 64, "side stream: device %d", dev);
  SideStream& ss = per_dev[dev];
  if (!ss.s) {
    SB_CUDA_CHECK(cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking));
    SB_CUDA_CHECK(cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming));
    SB_CUDA_CHECK(cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming));
  }
  *out = &ss;
  return STAGEML_OK;
}

// How a grouped GEMM on CTA pairs runs the groups' trailing odd tiles: as half units
// of the pair kernel (one tile on both CTAs of a pair, 64 rows each), or on the
// one-CTA kernel beside it. STAGEML_ODD_TILES=half|split (read once per process)
// forces one; by default half units run where each cluster gets many units to even
// out their different lengths (at least kHalfUnitsMinNTiles column tiles).
constexpr int kHalfUnitsMinNTiles = 32;
int odd_tiles_env() {  // 0 auto, 1 half, 2 split
  static const int mode = [] {
    const char* v = std::getenv("STAGEML_ODD_TILES");
    if (!v) return 0;
    if (std::strcmp(v, "half") == 0) return 1;
    if (std::strcmp(v, "split") == 0) return 2;
    return 0;
  }();
  return mode;
}
// Rank 8 on the one-CTA GEMMs packs two tenant runs into each K = 16 expand step
// (S in the run-parity layout, B rows of both runs side by side); STAGEML_PACK_RANK8=0
// (read once per process) keeps one masked step per run. Both give the same bits.
bool pack_rank8_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("STAGEML_PACK_RANK8");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

bool odd_tiles_as_half_units(const GemmLaunch& g) {
  const int mode = odd_tiles_env();
  if (mode != 0) return mode == 1;
  const int n_tiles = g.swiglu ? (g.N + 127) / 128 : (g.N + 255) / 256;
  return n_tiles >= kHalfUnitsMinNTiles;
}

// A grouped GEMM with a pair plan: full tile pairs on the CTA-pair kernel; the
// trailing odd tiles either as half units of the same kernel, or on the one-CTA
// kernel from a side stream launched right after it, so their CTAs take the SMs the
// persistent pair kernel leaves them. Without a plan (or with e4m3 weights): the
// one-CTA kernel over all tiles (g.tile_runs set by the caller). *two_streams tells
// the caller that the side stream ran (the next kernel then takes an ordinary launch).
int run_grouped_gemm(GemmLaunch g, const PairPlan& pp, cudaStream_t st, bool* two_streams = nullptr) {
  if (two_streams) *two_streams = false;
  if (!pp.on() || g.b_fp8) return launch_grouped_gemm(g, st);
  if (odd_tiles_as_half_units(g)) {
    g.pairs = pp.hpairs;
    g.num_pairs_dev = pp.num_hpairs;
    g.pairs_cap = pp.tiles_cap;
    g.pair_runs = pp.pruns;
    g.pair_nruns = pp.pnruns;
    g.pair_half_units = true;
    return launch_grouped_gemm(g, st);
  }
  g.pdl = false;  // two kernels on two streams: ordinary launches
  if (two_streams) *two_streams = true;
  g.split_pairs_dev = pp.num_pairs;
  g.split_singles_dev = pp.num_singles;
  g.split_cap = pp.tiles_cap;
  g.split_sms = 2 * (sm_count() / 2);
  GemmLaunch s1 = g;
  g.pairs = pp.pairs;
  g.num_pairs_dev = pp.num_pairs;
  g.pairs_cap = pp.tiles_cap;
  g.pair_runs = pp.pruns;
  g.pair_nruns = pp.pnruns;
  SideStream* ss = nullptr;
  SB_TRY(side_stream(&ss));
  SB_CUDA_CHECK(cudaEventRecord(ss->fork, st));
  SB_TRY(launch_grouped_gemm(g, st));
  SB_CUDA_CHECK(cudaStreamWaitEvent(ss->s, ss->fork, 0));
  s1.tile_list = pp.singles;
  s1.num_tiles_dev = pp.num_singles;
  s1.tiles_cap = pp.tiles_cap;
  s1.tile_runs = pp.sruns;
  s1.tile_nruns = pp.snruns;
  SB_TRY(launch_grouped_gemm(s1, ss->s));
  SB_CUDA_CHECK(cudaEventRecord(ss->join, ss->s));
  SB_CUDA_CHECK(cudaStreamWaitEvent(st, ss->join, 0));
  return STAGEML_OK;
}

// ------------------------------------------------------------------ MoE layer
struct MoeBuffers {
  stageml_moe_plan plan;
  float* logits = nullptr;
  int32_t* ids = nullptr;
  float* weights = nullptr;
  void* perm_scratch = nullptr;
  void* xp = nullptr;    // [rows_cap, H]; reused for Y [rows_cap, H]
  void* hbuf = nullptr;  // [rows_cap, I]
  float* spart13 = nullptr;
  void* s13 = nullptr;   // [rows_cap, 2r] 16-bit
  float* spart2 = nullptr;
  void* s2 = nullptr;    // [rows_cap, r] 16-bit
  int32_t* runs = nullptr;   // [tiles_cap, 128, 5]
  int32_t* nruns = nullptr;  // [tiles_cap]
  int8_t* row_run = nullptr; // [rows_cap]: each row's run index in its tile (rank 8, one-CTA GEMMs)
  PairPlan pp;                   // CTA-pair GEMM plan (16-bit weights)
  int32_t* status = nullptr;
  size_t bytes = 0;
};

// The grouped GEMMs run on CTA pairs (tcgen05 cta_group::2) unless the
// environment sets STAGEML_GEMM_PAIRS=0 (one CTA per tile), read once per process.
constexpr int64_t kSkinnyMaxPairs = 16;

int moe_validate(const stageml_moe_args* a, bool check_ptrs = true) {
  SB_CHECK_ARG(a, "moe: null args");
  SB_CHECK_ARG(a->T >= 0 && a->H > 0 && a->I > 0 && a->E > 0 && a->k >= 0 && a->n_shared >= 0,
               "moe: bad sizes T=%d H=%d I=%d E=%d k=%d n_shared=%d", a->T, a->H, a->I, a->E, a->k, a->n_shared);
  SB_CHECK_ARG(a->k + a->n_shared >= 1, "moe: need k + n_shared >= 1");
  SB_CHECK_ARG(a->k <= a->E && a->k <= 8, "moe: k=%d must be <= min(E, 8)", a->k);
  SB_CHECK_ARG(a->H % 8 == 0 && a->I % 8 == 0, "moe: H=%d and I=%d must be multiples of 8", a->H, a->I);
  SB_CHECK_ARG(is16(a->act_dtype), "moe: act_dtype must be BF16 or F16");
  SB_CHECK_ARG(a->weight_dtype == a->act_dtype || a->weight_dtype == STAGEML_E4M3,
               "moe: weight_dtype must equal act_dtype or be E4M3");
  if (a->weight_dtype == STAGEML_E4M3) {
    SB_CHECK_ARG(a->H % 16 == 0 && a->I % 16 == 0, "moe: E4M3 weights need H=%d and I=%d to be multiples of 16",
                 a->H, a->I);
    SB_CHECK_ARG(!check_ptrs || a->T == 0 || (a->gate_up_scale && a->down_scale),
                 "moe: E4M3 weights need gate_up_scale and down_scale");
  }
  SB_CHECK_ARG(a->rank == 0 || a->rank == 8 || a->rank == 16 || a->rank == 32,
               "moe: rank=%d must be 0, 8, 16 or 32 (zero-pad other ranks)", a->rank);
  const bool lora13 = a->rank > 0 && a->lora_a13;
  const bool lora2 = a->rank > 0 && a->lora_a2;
  SB_CHECK_ARG(!lora13 || a->lora_b13, "moe: lora_a13 without lora_b13");
  SB_CHECK_ARG(!lora2 || a->lora_b2, "moe: lora_a2 without lora_b2");
  SB_CHECK_ARG(!(lora13 || lora2) || (a->tenant_ids && a->n_tenants > 0 && a->lora_scale),
               "moe: LoRA needs tenant_ids, n_tenants > 0 and lora_scale");
  SB_CHECK_ARG(a->k == 0 || a->topk_ids || a->router_w, "moe: need topk_ids or router_w");
  SB_CHECK_ARG(a->n_fold >= 0 && (a->n_fold == 0 || a->fold_slot), "moe: n_fold=%d needs fold_slot", a->n_fold);
  if (a->fold_slot) {
    SB_CHECK_ARG(a->tenant_ids && a->n_tenants > 0, "moe: fold_slot needs tenant_ids and n_tenants > 0");
    SB_CHECK_ARG(a->weight_dtype != STAGEML_E4M3, "moe: folded weight sets need 16-bit weights, not E4M3");
  }
  if (a->topk_ids) SB_CHECK_ARG(a->ids_dtype == STAGEML_I32 || a->ids_dtype == STAGEML_I64, "moe: ids dtype");
  if (a->T > 0 && check_ptrs) {
    SB_CHECK_ARG(a->x && a->gate_up && a->down && a->out, "moe: null tensor");
    SB_CHECK_ARG(aligned16(a->x) && aligned16(a->gate_up) && aligned16(a->down) && aligned16(a->out),
                 "moe: x, gate_up, down and out must be 16-byte aligned");
    if (lora13) SB_CHECK_ARG(aligned16(a->lora_a13) && aligned16(a->lora_b13), "moe: LoRA w13 alignment");
    if (lora2) SB_CHECK_ARG(aligned16(a->lora_a2) && aligned16(a->lora_b2), "moe: LoRA w2 alignment");
  }
  return STAGEML_OK;
}

// Folded weight groups of a call (0 without a fold map).
inline int moe_n_fold(const stageml_moe_args* a) { return a->fold_slot ? a->n_fold : 0; }

void moe_carve(const stageml_moe_args* a, void* ws, MoeBuffers* b) {
  Carver c(ws);
  const int E_tot = a->E + a->n_shared;
  const int n_fold = moe_n_fold(a);
  const int64_t P = (int64_t)a->T * (a->k + a->n_shared);
  const size_t es = esize(a->act_dtype);
  if (a->plan_out)
    b->plan = *a->plan_out;
  else
    carve_plan(c, P, E_tot + n_fold, &b->plan);
  const int64_t rows_cap = stageml_plan_rows_cap(P, E_tot + n_fold);
  if (!a->topk_ids && a->k > 0) {
    b->logits = c.take<float>((size_t)a->T * a->E);
    b->ids = c.take<int32_t>((size_t)a->T * a->k);
    b->weights = c.take<float>((size_t)a->T * a->k);
  }
  const int64_t nkeys = permute_num_keys(n_fold, a->n_tenants, 0, E_tot);
  b->perm_scratch = c.take_bytes(permute_scratch_bytes(P, nkeys));
  b->xp = c.take_bytes((size_t)rows_cap * a->H * es);
  b->hbuf = c.take_bytes((size_t)rows_cap * a->I * es);
  const int sfac = a->rank == 8 ? 2 : 1;  // rank 8: room for S in the run-parity layout
  if (a->rank > 0 && a->lora_a13) {
    b->spart13 = c.take<float>((size_t)shrink_num_slices(a->H) * rows_cap * 2 * a->rank);
    b->s13 = c.take_bytes((size_t)rows_cap * 2 * a->rank * sfac * es);
  }
  if (a->rank > 0 && a->lora_a2) {
    b->spart2 = c.take<float>((size_t)shrink_num_slices(a->I) * rows_cap * a->rank);
    b->s2 = c.take_bytes((size_t)rows_cap * a->rank * sfac * es);
  }
  const bool lora = a->rank > 0 && (a->lora_a13 || a->lora_a2);
  if (a->weight_dtype != STAGEML_E4M3 && pairs_pay(P, E_tot) &&
      (!lora || pair_lora_pays(P, E_tot, a->n_tenants, std::min(a->H, a->I))))
    carve_pair_plan(c, rows_cap / 128, lora, &b->pp);
  if (!b->pp.on() && lora) {
    b->runs = c.take<int32_t>((size_t)(rows_cap / 128) * kMaxRunsPerTile * 5);
    b->nruns = c.take<int32_t>((size_t)(rows_cap / 128));
    if (a->rank == 8) b->row_run = c.take<int8_t>((size_t)rows_cap);
  }
  b->status = c.take<int32_t>(1);
  b->bytes = c.off;
}

// One expert projection of the MoE layer: decode-sized batches on the skinny GEMM,
// otherwise the grouped GEMM with the layer's pair plan.
int run_moe_gemm(const GemmLaunch& g, const MoeBuffers& b, bool skinny, cudaStream_t st, int64_t max_rows,
                 int pdl_mode = 0, bool* two_streams = nullptr) {
  if (two_streams) *two_streams = false;
  if (skinny)
    return launch_skinny_gemm(g, b.plan.row_tenant, b.plan.group_offsets, b.plan.group_counts, st, max_rows,
                              pdl_mode);
  return run_grouped_gemm(g, b.pp, st, two_streams);
}

// A one-expert top-1 layer (a dense SwiGLU MLP with per-row LoRA tenants, e.g. a
// transformer block's MLP served through this layer) needs no permutation: every
// token is one row of its only expert. Its rows stay in token order -- the shrinks
// read x and h in place, the GEMMs take the rows as one group, the down projection
// applies the routing weight and writes the output rows, and there is no gather or
// combine. Same bits as the permuted path (each GEMM row and each S row is computed
// independently of the others). STAGEML_DIRECT_ROWS=0 (read once per process) keeps
// the permuted path.
bool direct_rows_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("STAGEML_DIRECT_ROWS");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

int moe_forward_direct(const stageml_moe_args* a, const MoeBuffers& b, int32_t* status, bool pdl, cudaStream_t st) {
  const int bf = a->act_dtype == STAGEML_BF16;
  const bool lora13 = a->rank > 0 && a->lora_a13;
  const bool lora2 = a->rank > 0 && a->lora_a2;
  const bool lora = lora13 || lora2;
  const int64_t T = a->T;
  int32_t* row_tenant = b.plan.row_tenant;  // [rows_cap] >= T
  float* row_scale = b.plan.row_weight;
  bool two_streams = false;
  // R1 + R2: one expert, top-1 -- the router's weight is 1 (softmax over one logit);
  // caller ids / weights are validated like the permutation does
  SB_STAGE(STAGEML_STAGE_PERMUTE,
           launch_direct_rows(a->topk_ids, a->ids_dtype, a->topk_ids ? a->topk_weights : nullptr, a->weights_dtype,
                              a->tenant_ids, a->n_tenants, T, row_tenant, row_scale, status, st, pdl));
  if (b.pp.on())
    SB_STAGE(STAGEML_STAGE_PERMUTE,
             build_pair_plan(b.pp, nullptr, nullptr, nullptr, T, lora ? row_tenant : nullptr, st, pdl));
  else if (lora)
    SB_STAGE(STAGEML_STAGE_PERMUTE, launch_tile_runs(row_tenant, nullptr, T, (int)((T + 127) / 128), b.runs, b.nruns,
                                                     st, nullptr, pdl));
  auto shrink = [&](const void* src, int K, const void* A, int R, float* spart, void* s_out) {
    ShrinkLaunch s;
    s.src = src;
    s.K = K;
    s.dtype_bf16 = bf;
    s.static_rows = T;
    s.rows_cap = T;
    s.row_tenant = row_tenant;
    s.lora_a = A;
    s.a_group_stride = (int64_t)R * K;
    s.a_tenant_stride = s.a_group_stride;
    s.a_rows_total = (int64_t)a->n_tenants * R;
    s.R = R;
    s.spart = spart;
    s.s_out = s_out;
    s.lora_scale = a->lora_scale;
    s.status = status;
    s.pdl = pdl && !two_streams;
    return launch_gather_shrink(s, st);
  };
  if (lora13)
    SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, shrink(a->x, a->H, a->lora_a13, 2 * a->rank, b.spart13, b.s13));
  {
    GemmLaunch g;
    g.a = a->x;
    g.a_rows = T;
    g.m_rows = T;
    g.K = a->H;
    g.b = a->gate_up;
    g.b_rows_total = (int64_t)2 * a->I;
    g.b_group_rows = 2 * a->I;
    g.N = a->I;
    g.swiglu = true;
    g.in_bf16 = bf;
    if (lora13) {
      g.s16 = b.s13;
      g.s_rows = T;
      g.rank = a->rank;
      g.lora_b = a->lora_b13;
      g.lora_b_group_stride = (int64_t)2 * a->I * a->rank;
      g.lora_b_tenant_stride = g.lora_b_group_stride;
      g.lora_b_rows_total = (int64_t)a->n_tenants * 2 * a->I;
      g.tile_runs = b.runs;
      g.tile_nruns = b.nruns;
    }
    g.b_scale = a->gate_up_scale;
    g.b_fp8 = a->weight_dtype == STAGEML_E4M3;
    g.out = b.hbuf;
    g.ldo = a->I;
    g.status = status;
    g.pdl = pdl;
    SB_STAGE(STAGEML_STAGE_GEMM_GATE_UP, run_grouped_gemm(g, b.pp, st, &two_streams));
  }
  if (lora2) SB_STAGE(STAGEML_STAGE_SHRINK_H, shrink(b.hbuf, a->I, a->lora_a2, a->rank, b.spart2, b.s2));
  {
    GemmLaunch g;
    g.a = b.hbuf;
    g.a_rows = T;
    g.m_rows = T;
    g.K = a->I;
    g.b = a->down;
    g.b_rows_total = a->H;
    g.b_group_rows = a->H;
    g.N = a->H;
    g.in_bf16 = bf;
    if (lora2) {
      g.s16 = b.s2;
      g.s_rows = T;
      g.rank = a->rank;
      g.lora_b = a->lora_b2;
      g.lora_b_group_stride = (int64_t)a->H * a->rank;
      g.lora_b_tenant_stride = g.lora_b_group_stride;
      g.lora_b_rows_total = (int64_t)a->n_tenants * a->H;
      g.tile_runs = b.runs;
      g.tile_nruns = b.nruns;
    }
    g.row_scale = row_scale;
    g.b_scale = a->down_scale;
    g.b_fp8 = a->weight_dtype == STAGEML_E4M3;
    g.out = a->out;
    g.ldo = a->H;
    g.status = status;
    g.pdl = pdl && (lora2 || !two_streams);
    SB_STAGE(STAGEML_STAGE_GEMM_DOWN, run_grouped_gemm(g, b.pp, st, &two_streams));
  }
  return STAGEML_OK;
}

int moe_forward_impl(const stageml_moe_args* a, void* ws, size_t ws_bytes, cudaStream_t st) {
  SB_TRY(moe_validate(a));
  if (a->T == 0) return STAGEML_OK;
  MoeBuffers b;
  moe_carve(a, nullptr, &b);
  if (!ws || ws_bytes < b.bytes)
    return set_error(STAGEML_ERR_WORKSPACE, "moe: workspace of %zu bytes < required %zu", ws_bytes, b.bytes);
  moe_carve(a, ws, &b);
  const int E_tot = a->E + a->n_shared;
  const int n_fold = moe_n_fold(a);
  const int64_t P = (int64_t)a->T * (a->k + a->n_shared);
  if (a->plan_out)
    SB_CHECK_ARG(a->plan_out->rows_cap >= stageml_plan_rows_cap(P, E_tot + n_fold),
                 "moe: plan_out rows_cap too small");
  int32_t* status = a->status ? a->status : b.status;
  const int bf = a->act_dtype == STAGEML_BF16;
  const bool lora13 = a->rank > 0 && a->lora_a13;
  const bool lora2 = a->rank > 0 && a->lora_a2;
  // Decode-sized batches (at most 16 routed rows in all) stream the weights with the
  // skinny GEMM; larger ones use the tensor-memory GEMM and its tile / pair plan.
  const bool skinny = P <= kSkinnyMaxPairs && a->weight_dtype != STAGEML_E4M3;
  // Their chain of small kernels runs as programmatic dependent launches: each one is
  // scheduled while the previous one finishes, and each skinny GEMM streams its
  // weights while the shrink before it runs.
  const bool pdl = skinny && pdl_enabled();
  // larger batches: programmatic dependent launches between the kernels after the router
  const bool pdl_big = !skinny && pdl_enabled();
  bool two_streams = false;  // the last grouped GEMM ran its odd tiles on the side stream
  // rank 8 on the one-CTA GEMMs: two runs per expand step (the shrinks write S by run parity)
  const bool pack8 = !skinny && b.row_run && pack_rank8_enabled();
  if (!skinny && a->E == 1 && a->n_shared == 0 && a->k == 1 && n_fold == 0 && !a->T_dev && !a->plan_out &&
      direct_rows_enabled())
    return moe_forward_direct(a, b, status, pdl_big, st);

  // R1: routing
  const void* ids = a->topk_ids;
  int ids_dtype = a->ids_dtype;
  const void* wts = a->topk_weights;
  int wts_dtype = a->weights_dtype;
  if (!ids && a->k > 0) {
    SB_STAGE(STAGEML_STAGE_ROUTE, launch_route(a->x, a->act_dtype, a->router_w, a->T, a->H, a->E, a->k,
                                               a->renormalize, b.logits, b.ids, b.weights, st, pdl));
    ids = b.ids;
    ids_dtype = STAGEML_I32;
    wts = b.weights;
    wts_dtype = STAGEML_F32;
  }
  // R2: permutation
  PermuteScratch scr;
  const int64_t nkeys = permute_num_keys(n_fold, a->n_tenants, 0, E_tot);
  permute_carve(b.perm_scratch, P, nkeys, &scr);
  SB_STAGE(STAGEML_STAGE_PERMUTE, launch_permute(ids, ids_dtype, wts, wts_dtype, a->tenant_ids, a->T, a->k,
                                                 a->n_shared, E_tot, a->n_tenants, 0, b.plan, status, scr, st,
                                                 a->T_dev, pdl || pdl_big, a->fold_slot, n_fold));
  const int tiles_cap = (int)(b.plan.rows_cap / 128);
  if (!skinny && b.pp.on()) {
    SB_STAGE(STAGEML_STAGE_PERMUTE, build_pair_plan(b.pp, b.plan.tile_group, b.plan.group_offsets, b.plan.num_tiles,
                                                    0, b.plan.row_tenant, st, pdl_big));
  } else if (!skinny && b.runs) {
    SB_STAGE(STAGEML_STAGE_PERMUTE, launch_tile_runs(b.plan.row_tenant, b.plan.num_tiles, 0, tiles_cap, b.runs,
                                                     b.nruns, st, nullptr, pdl_big, pack8 ? b.row_run : nullptr));
  }
  // gather + R4 shrink of w1|w3 (decode-sized batches: no gather, the skinny GEMM
  // reads the token rows in place, and the per-pair shrink)
  if (!skinny || lora13) {
    ShrinkLaunch s;
    s.src = a->x;
    s.src_row_of = b.plan.row_token;
    s.gather_dst = b.xp;
    s.K = a->H;
    s.dtype_bf16 = bf;
    s.num_tiles_dev = b.plan.num_tiles;
    s.rows_cap = b.plan.rows_cap;
    s.row_tenant = b.plan.row_tenant;
    s.tile_group = b.plan.tile_group;
    s.pdl = pdl_big;
    if (lora13) {
      s.lora_a = a->lora_a13;
      s.a_group_stride = (int64_t)2 * a->rank * a->H;
      s.a_tenant_stride = (int64_t)E_tot * s.a_group_stride;
      s.R = 2 * a->rank;
      s.a_rows_total = (int64_t)a->n_tenants * E_tot * 2 * a->rank;
      s.status = status;
      s.row_run = pack8 ? b.row_run : nullptr;
      s.spart = b.spart13;
      s.s_out = b.s13;
      s.lora_scale = a->lora_scale;
    }
    if (skinny)
      SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, launch_pair_shrink(s, b.plan.pair_row, P, st, pdl));
    else
      SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, launch_gather_shrink(s, st));
  }
  // R3 + R5: gate/up GEMM, LoRA expand, SwiGLU
  {
    GemmLaunch g;
    g.a = skinny ? a->x : b.xp;
    g.a_rows = skinny ? a->T : b.plan.rows_cap;
    g.a_row_of = skinny ? b.plan.row_token : nullptr;
    g.K = a->H;
    g.b = a->gate_up;
    g.b_rows_total = (int64_t)(E_tot + n_fold) * 2 * a->I;
    g.b_group_rows = 2 * a->I;
    g.N = a->I;
    g.swiglu = true;
    g.in_bf16 = bf;
    g.num_tiles_dev = b.plan.num_tiles;
    g.tiles_cap = (int)(b.plan.rows_cap / 128);
    g.tile_group = b.plan.tile_group;
    g.group_offsets = b.plan.group_offsets;
    if (lora13) {
      g.s16 = b.s13;
      g.s_rows = b.plan.rows_cap;
      g.rank = a->rank;
      g.lora_b = a->lora_b13;
      g.lora_b_group_stride = (int64_t)2 * a->I * a->rank;
      g.lora_b_tenant_stride = (int64_t)E_tot * g.lora_b_group_stride;
      g.lora_b_rows_total = (int64_t)a->n_tenants * E_tot * 2 * a->I;
      g.tile_runs = b.runs;
      g.tile_nruns = b.nruns;
      g.pack8 = pack8;
    }
    g.b_scale = a->gate_up_scale;
    g.b_fp8 = a->weight_dtype == STAGEML_E4M3;
    g.out = b.hbuf;
    g.ldo = a->I;
    g.status = status;
    g.pdl = pdl_big;
    SB_STAGE(STAGEML_STAGE_GEMM_GATE_UP,
             run_moe_gemm(g, b, skinny, st, P, pdl ? (lora13 ? 2 : 1) : 0, &two_streams));
  }
  // R4 shrink of h for w2
  if (lora2) {
    ShrinkLaunch s;
    s.src = b.hbuf;
    s.K = a->I;
    s.dtype_bf16 = bf;
    s.num_tiles_dev = b.plan.num_tiles;
    s.rows_cap = b.plan.rows_cap;
    s.row_tenant = b.plan.row_tenant;
    s.tile_group = b.plan.tile_group;
    s.lora_a = a->lora_a2;
    s.a_group_stride = (int64_t)a->rank * a->I;
    s.a_tenant_stride = (int64_t)E_tot * s.a_group_stride;
    s.R = a->rank;
    s.a_rows_total = (int64_t)a->n_tenants * E_tot * a->rank;
    s.status = status;
    s.row_run = pack8 ? b.row_run : nullptr;
    s.pdl = pdl_big && !two_streams;
    s.spart = b.spart2;
    s.s_out = b.s2;
    s.lora_scale = a->lora_scale;
    if (skinny)
      SB_STAGE(STAGEML_STAGE_SHRINK_H, launch_pair_shrink(s, b.plan.pair_row, P, st, pdl));
    else
      SB_STAGE(STAGEML_STAGE_SHRINK_H, launch_gather_shrink(s, st));
  }
  // R3 + R5: down GEMM, LoRA expand, routing weight
  {
    GemmLaunch g;
    g.a = b.hbuf;
    g.a_rows = b.plan.rows_cap;
    g.K = a->I;
    g.b = a->down;
    g.b_rows_total = (int64_t)(a->down_group ? E_tot : E_tot + n_fold) * a->H;
    g.b_group_rows = a->H;
    g.N = a->H;
    g.swiglu = false;
    g.in_bf16 = bf;
    g.num_tiles_dev = b.plan.num_tiles;
    g.tiles_cap = (int)(b.plan.rows_cap / 128);
    g.tile_group = b.plan.tile_group;
    g.group_offsets = b.plan.group_offsets;
    if (lora2) {
      g.s16 = b.s2;
      g.s_rows = b.plan.rows_cap;
      g.rank = a->rank;
      g.lora_b = a->lora_b2;
      g.lora_b_group_stride = (int64_t)a->H * a->rank;
      g.lora_b_tenant_stride = (int64_t)E_tot * g.lora_b_group_stride;
      g.lora_b_rows_total = (int64_t)a->n_tenants * E_tot * a->H;
      g.tile_runs = b.runs;
      g.tile_nruns = b.nruns;
      g.pack8 = pack8;
    }
    g.row_scale = b.plan.row_weight;
    g.b_group_map = a->down_group;
    g.b_scale = a->down_scale;
    g.b_fp8 = a->weight_dtype == STAGEML_E4M3;
    g.out = b.xp;
    g.ldo = a->H;
    g.status = status;
    g.pdl = pdl_big && (lora2 || !two_streams);
    SB_STAGE(STAGEML_STAGE_GEMM_DOWN,
             run_moe_gemm(g, b, skinny, st, P, pdl ? (lora2 ? 2 : 1) : 0, &two_streams));
  }
  // combine
  SB_STAGE(STAGEML_STAGE_COMBINE,
           launch_combine(b.xp, b.plan.pair_row, a->T, a->k + a->n_shared, a->H, bf, a->out, st, a->T_dev,
                          pdl || (pdl_big && !two_streams)));
  return STAGEML_OK;
}

// ------------------------------------------ routed / grouped linear layers
// Buffers shared by stageml_moe_linear and stageml_lora_linear.
struct LinBuffers {
  stageml_moe_plan plan{};
  void* perm = nullptr;
  void* xp = nullptr;     // permuted input rows [rows_cap, K]
  float* spart = nullptr;
  void* s = nullptr;      // 16-bit S [rows, rank]
  void* yp = nullptr;     // permuted output rows [rows_cap, N]
  int32_t* runs = nullptr;
  int32_t* nruns = nullptr;
  PairPlan pp;
  int32_t* tenants = nullptr;  // direct mode: validated row tenants
  int32_t* status = nullptr;
  size_t bytes = 0;
};

// Small batches take the LoRA shrink per row (pair shrink): a 16-row warp of the tiled
// shrink walks the distinct tenants of its rows one after the other, and the rows of a
// small mixed-adapter batch (e.g. 256 rows over 64 Zipf-distributed adapters) span many
// of them.
constexpr int64_t kRowShrinkMaxRows = 512;

// permuted: P pairs over n_groups groups (nkeys from n_tenants / group_by_tenant);
// direct: rows = M, no permutation.
void lin_carve(bool permuted, int64_t P_or_M, int n_groups, int n_tenants, int group_by_tenant, int K, int N, int rank,
               int nkeys_groups, size_t es, void* ws, LinBuffers* b) {
  Carver c(ws);
  int64_t rows;
  if (permuted) {
    carve_plan(c, P_or_M, n_groups, &b->plan);
    rows = b->plan.rows_cap;
    b->perm = c.take_bytes(permute_scratch_bytes(P_or_M, permute_num_keys(0, n_tenants, group_by_tenant, nkeys_groups)));
    b->xp = c.take_bytes((size_t)rows * K * es);
    b->yp = c.take_bytes((size_t)rows * N * es);
  } else {
    rows = P_or_M;
    b->tenants = c.take<int32_t>((size_t)std::max<int64_t>(rows, 1));
  }
  const int64_t tiles = (rows + 127) / 128;
  if (pairs_pay(P_or_M, permuted ? n_groups : 1)) carve_pair_plan(c, tiles, rank > 0, &b->pp);
  if (rank > 0) {
    b->spart = c.take<float>((size_t)shrink_num_slices(K) * rows * rank);
    b->s = c.take_bytes((size_t)rows * rank * es);
    if (!b->pp.on()) {
      b->runs = c.take<int32_t>((size_t)tiles * kMaxRunsPerTile * 5);
      b->nruns = c.take<int32_t>((size_t)tiles);
    }
  }
  b->status = c.take<int32_t>(1);
  b->bytes = c.off;
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" {

const char* stageml_last_error(void) { return last_error_text(); }

int stageml_abi_version(void) { return kAbiVersion; }

size_t stageml_struct_size(int which) {
  switch (which) {
    case 0:
      return sizeof(stageml_moe_plan);
    case 1:
      return sizeof(stageml_moe_args);
    case 2:
      return sizeof(stageml_lora_linear_args);
    case 3:
      return sizeof(stageml_ep_layout);
    case 4:
      return sizeof(stageml_ep_args);
    default:
      return 0;
  }
}

int stageml_route_topk(const void* x, int x_dtype, const float* gate_w, int T, int H, int E, int k, int renormalize,
                       float* logits_out, int32_t* ids_out, float* weights_out, stageml_stream_t stream) {
  clear_error();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SB_CHECK_ARG(logits_out, "route_topk: logits_out is required as scratch ([T, E] fp32)");
  return launch_route(x, x_dtype, gate_w, T, H, E, k, renormalize, logits_out, ids_out, weights_out, st);
}

int stageml_topk_from_logits(const float* logits, int T, int E, int k, int renormalize, int32_t* ids_out,
                             float* weights_out, stageml_stream_t stream) {
  clear_error();
  return launch_topk(logits, T, E, k, renormalize, ids_out, weights_out, static_cast<cudaStream_t>(stream));
}

size_t stageml_permute_workspace_bytes(int T, int k, int n_shared, int n_experts_total, int n_tenants,
                                       int group_by_tenant) {
  const int64_t P = (int64_t)T * (k + n_shared);
  return permute_scratch_bytes(P, permute_num_keys(0, n_tenants, group_by_tenant, n_experts_total));
}

int stageml_permute(const void* ids, int ids_dtype, const void* weights, int weights_dtype, const int32_t* tenant_ids,
                    int T, int k, int n_shared, int n_experts_total, int n_tenants, int group_by_tenant,
                    const stageml_moe_plan* plan, int32_t* status, void* workspace, size_t workspace_bytes,
                    stageml_stream_t stream) {
  clear_error();
  SB_CHECK_ARG(plan, "permute: null plan");
  const size_t need = stageml_permute_workspace_bytes(T, k, n_shared, n_experts_total, n_tenants, group_by_tenant);
  if (!workspace || workspace_bytes < need)
    return set_error(STAGEML_ERR_WORKSPACE, "permute: workspace of %zu bytes < required %zu", workspace_bytes, need);
  PermuteScratch scr;
  const int64_t P = (int64_t)T * (k + n_shared);
  permute_carve(workspace, P, permute_num_keys(0, n_tenants, group_by_tenant, n_experts_total), &scr);
  return launch_permute(ids, ids_dtype, weights, weights_dtype, tenant_ids, T, k, n_shared, n_experts_total, n_tenants,
                        group_by_tenant, *plan, status, scr, static_cast<cudaStream_t>(stream));
}

int stageml_combine_rows(const void* y, const int32_t* pair_row, int T, int kk, int H, int dtype, void* out,
                         stageml_stream_t stream) {
  clear_error();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SB_CHECK_ARG(T >= 0 && kk >= 1 && H > 0, "combine_rows: bad sizes");
  SB_CHECK_ARG(is16(dtype), "combine_rows: dtype must be BF16 or F16");
  if (T == 0) return STAGEML_OK;
  SB_CHECK_ARG(y && pair_row && out, "combine_rows: null pointer");
  SB_CHECK_ARG(aligned16(y) && aligned16(out), "combine_rows: 16-byte alignment");
  SB_STAGE(STAGEML_STAGE_COMBINE, launch_combine(y, pair_row, T, kk, H, dtype == STAGEML_BF16, out, st));
  return STAGEML_OK;
}

size_t stageml_moe_workspace_bytes(const stageml_moe_args* args) {
  if (!args || moe_validate(args, false) != STAGEML_OK) return 0;
  MoeBuffers b;
  moe_carve(args, nullptr, &b);
  return b.bytes;
}

int stageml_moe_forward(const stageml_moe_args* args, void* workspace, size_t workspace_bytes,
                        stageml_stream_t stream) {
  clear_error();
  return moe_forward_impl(args, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

static void residual_args(stageml_moe_args* a, const void* hidden, const void* gate_up, const void* down,
                          const void* topk_weights, int weights_dtype, const void* topk_ids, int ids_dtype, int T,
                          int H, int I, int E, int k, int dtype, void* out, int32_t* status) {
  *a = stageml_moe_args{};
  a->T = T;
  a->H = H;
  a->I = I;
  a->E = E;
  a->k = k;
  a->n_shared = 0;
  a->act_dtype = dtype;
  a->weight_dtype = dtype;
  a->x = hidden;
  a->topk_ids = topk_ids;
  a->ids_dtype = ids_dtype;
  a->topk_weights = topk_weights;
  a->weights_dtype = weights_dtype;
  a->gate_up = gate_up;
  a->down = down;
  a->out = out;
  a->status = status;
}

size_t stageml_residual_moe_workspace_bytes(int T, int H, int I, int E, int k) {
  stageml_moe_args a;
  static const int dummy_ids = 0;
  residual_args(&a, nullptr, nullptr, nullptr, nullptr, STAGEML_F32, &dummy_ids, STAGEML_I64, T, H, I, E, k,
                STAGEML_BF16, nullptr, nullptr);
  if (moe_validate(&a, false) != STAGEML_OK) return 0;
  MoeBuffers b;
  moe_carve(&a, nullptr, &b);
  return b.bytes;
}

int stageml_residual_moe(const void* hidden, const void* gate_up, const void* down, const void* topk_weights,
                         int weights_dtype, const void* topk_ids, int ids_dtype, int T, int H, int I, int E, int k,
                         int dtype, void* out, int32_t* status, void* workspace, size_t workspace_bytes,
                         stageml_stream_t stream) {
  clear_error();
  SB_CHECK_ARG(topk_ids && topk_weights, "residual_moe: topk_ids and topk_weights are required");
  stageml_moe_args a;
  residual_args(&a, hidden, gate_up, down, topk_weights, weights_dtype, topk_ids, ids_dtype, T, H, I, E, k, dtype,
                out, status);
  return moe_forward_impl(&a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t stageml_moe_linear_workspace_bytes(int T, int K, int N, int E, int k, int group_by_tenant, int n_tenants,
                                          int rank) {
  LinBuffers b;
  const int n_groups = group_by_tenant ? n_tenants * E : E;
  lin_carve(true, (int64_t)T * k, n_groups, n_tenants, group_by_tenant, K, N, group_by_tenant ? 0 : rank, E, 2,
            nullptr, &b);
  return b.bytes;
}

int stageml_moe_linear(const void* x, const void* weight, const void* bias, const void* topk_ids, int ids_dtype,
                       const void* topk_weights, int weights_dtype, const int32_t* tenant_ids, int T, int K, int N,
                       int E, int k, int group_by_tenant, int n_tenants, int rank, const void* lora_a,
                       const void* lora_b, const float* lora_scale, int dtype, void* out, int32_t* status,
                       void* workspace, size_t workspace_bytes, stageml_stream_t stream) {
  clear_error();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SB_CHECK_ARG(T >= 0 && K > 0 && N > 0 && E > 0 && k >= 1 && k <= E, "moe_linear: bad sizes");
  SB_CHECK_ARG(K % 8 == 0 && N % 8 == 0, "moe_linear: K=%d and N=%d must be multiples of 8", K, N);
  SB_CHECK_ARG(is16(dtype), "moe_linear: dtype must be BF16 or F16");
  SB_CHECK_ARG(ids_dtype == STAGEML_I32 || ids_dtype == STAGEML_I64, "moe_linear: ids dtype");
  SB_CHECK_ARG(rank == 0 || rank == 8 || rank == 16 || rank == 32, "moe_linear: rank=%d must be 0, 8, 16 or 32", rank);
  const bool lora = rank > 0 && lora_a && !group_by_tenant;
  SB_CHECK_ARG(!lora || (lora_b && lora_scale && tenant_ids && n_tenants > 0), "moe_linear: incomplete LoRA inputs");
  SB_CHECK_ARG(!group_by_tenant || (tenant_ids && n_tenants > 0), "moe_linear: group_by_tenant needs tenant ids");
  if (T == 0) return STAGEML_OK;
  SB_CHECK_ARG(x && weight && topk_ids && out, "moe_linear: null tensor");
  SB_CHECK_ARG(aligned16(x) && aligned16(weight) && aligned16(out), "moe_linear: 16-byte alignment");
  if (lora) SB_CHECK_ARG(aligned16(lora_a) && aligned16(lora_b), "moe_linear: LoRA alignment");
  const int n_groups = group_by_tenant ? n_tenants * E : E;
  const int r = lora ? rank : 0;
  LinBuffers b;
  lin_carve(true, (int64_t)T * k, n_groups, n_tenants, group_by_tenant, K, N, r, E, esize(dtype), nullptr, &b);
  if (!workspace || workspace_bytes < b.bytes)
    return set_error(STAGEML_ERR_WORKSPACE, "moe_linear: workspace of %zu bytes < required %zu", workspace_bytes,
                     b.bytes);
  lin_carve(true, (int64_t)T * k, n_groups, n_tenants, group_by_tenant, K, N, r, E, esize(dtype), workspace, &b);
  int32_t* stat = status ? status : b.status;
  const int bf = dtype == STAGEML_BF16;
  PermuteScratch scr;
  permute_carve(b.perm, (int64_t)T * k, permute_num_keys(0, n_tenants, group_by_tenant, E), &scr);
  SB_STAGE(STAGEML_STAGE_PERMUTE,
           launch_permute(topk_ids, ids_dtype, topk_weights, weights_dtype, tenant_ids, T, k, 0, E,
                          group_by_tenant || lora ? n_tenants : 0, group_by_tenant, b.plan, stat, scr, st));
  const int tiles_cap = (int)(b.plan.rows_cap / 128);
  if (b.pp.on())
    SB_STAGE(STAGEML_STAGE_PERMUTE, build_pair_plan(b.pp, b.plan.tile_group, b.plan.group_offsets, b.plan.num_tiles,
                                                    0, lora ? b.plan.row_tenant : nullptr, st));
  else if (lora)
    SB_STAGE(STAGEML_STAGE_PERMUTE,
             launch_tile_runs(b.plan.row_tenant, b.plan.num_tiles, 0, tiles_cap, b.runs, b.nruns, st));
  ShrinkLaunch sh;
  sh.src = x;
  sh.src_row_of = b.plan.row_token;
  sh.gather_dst = b.xp;
  sh.K = K;
  sh.dtype_bf16 = bf;
  sh.num_tiles_dev = b.plan.num_tiles;
  sh.rows_cap = b.plan.rows_cap;
  sh.row_tenant = b.plan.row_tenant;
  sh.tile_group = b.plan.tile_group;
  if (lora) {
    sh.lora_a = lora_a;
    sh.a_group_stride = (int64_t)rank * K;
    sh.a_tenant_stride = (int64_t)E * sh.a_group_stride;
    sh.R = rank;
    sh.a_rows_total = (int64_t)n_tenants * E * rank;
    sh.status = stat;
    sh.spart = b.spart;
    sh.s_out = b.s;
    sh.lora_scale = lora_scale;
  }
  SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, launch_gather_shrink(sh, st));
  GemmLaunch g;
  g.a = b.xp;
  g.a_rows = b.plan.rows_cap;
  g.K = K;
  g.b = weight;
  g.b_rows_total = (int64_t)n_groups * N;
  g.b_group_rows = N;
  g.N = N;
  g.in_bf16 = bf;
  g.num_tiles_dev = b.plan.num_tiles;
  g.tiles_cap = tiles_cap;
  g.tile_group = b.plan.tile_group;
  if (lora) {
    g.s16 = b.s;
    g.s_rows = b.plan.rows_cap;
    g.rank = rank;
    g.lora_b = lora_b;
    g.lora_b_group_stride = (int64_t)N * rank;
    g.lora_b_tenant_stride = (int64_t)E * g.lora_b_group_stride;
    g.lora_b_rows_total = (int64_t)n_tenants * E * N;
    g.tile_runs = b.runs;
    g.tile_nruns = b.nruns;
  }
  g.bias = bias;
  g.bias_group_stride = N;
  g.bias_group_mod = E;
  g.row_scale = b.plan.row_weight;
  g.out = b.yp;
  g.ldo = N;
  g.status = stat;
  SB_STAGE(STAGEML_STAGE_GEMM, run_grouped_gemm(g, b.pp, st));
  SB_STAGE(STAGEML_STAGE_COMBINE, launch_combine(b.yp, b.plan.pair_row, T, k, N, bf, out, st));
  return STAGEML_OK;
}

int stageml_lora_fold(const void* W, const void* A, const void* B, const float* scale, int batch, int rows, int cols,
                      int rank, int layout, int64_t w_batch_stride, int64_t a_batch_stride, int64_t b_batch_stride,
                      int dtype, void* out, stageml_stream_t stream) {
  clear_error();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SB_STAGE(STAGEML_STAGE_FOLD, launch_lora_fold(W, A, B, scale, batch, rows, cols, rank, layout, w_batch_stride,
                                                a_batch_stride, b_batch_stride, dtype, out, st));
  return STAGEML_OK;
}

static void lora_linear_carve(const stageml_lora_linear_args* a, void* ws, LinBuffers* b) {
  const bool lora = a->rank > 0 && a->lora_a && a->row_tenant;
  const int n_ten = lora ? a->n_tenants : 0;
  lin_carve(a->n_groups > 1, a->M, a->n_groups, n_ten, 0, a->K, a->N, lora ? a->rank : 0, a->n_groups,
            esize(a->dtype) ? esize(a->dtype) : 2, ws, b);
}

size_t stageml_lora_linear_workspace_bytes(const stageml_lora_linear_args* a) {
  if (!a || a->M < 0 || a->n_groups < 1) return 0;
  LinBuffers b;
  lora_linear_carve(a, nullptr, &b);
  return b.bytes;
}

int stageml_lora_linear(const stageml_lora_linear_args* a, void* workspace, size_t workspace_bytes,
                        stageml_stream_t stream) {
  clear_error();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SB_CHECK_ARG(a, "lora_linear: null args");
  SB_CHECK_ARG(a->M >= 0 && a->K > 0 && a->N > 0 && a->n_groups >= 1, "lora_linear: bad sizes");
  SB_CHECK_ARG(a->K % 8 == 0 && a->N % 8 == 0, "lora_linear: K=%d and N=%d must be multiples of 8", a->K, a->N);
  SB_CHECK_ARG(is16(a->dtype), "lora_linear: dtype must be BF16 or F16");
  SB_CHECK_ARG(a->rank == 0 || a->rank == 8 || a->rank == 16 || a->rank == 32,
               "lora_linear: rank=%d must be 0, 8, 16 or 32", a->rank);
  const bool lora = a->rank > 0 && a->lora_a && a->row_tenant;
  SB_CHECK_ARG(!lora || (a->lora_b && a->lora_scale && a->n_tenants > 0), "lora_linear: incomplete LoRA inputs");
  SB_CHECK_ARG(a->n_groups == 1 || a->row_group, "lora_linear: n_groups > 1 needs row_group");
  if (a->M == 0) return STAGEML_OK;
  SB_CHECK_ARG(a->x && a->w_bank && a->y, "lora_linear: null tensor");
  SB_CHECK_ARG(aligned16(a->x) && aligned16(a->w_bank) && aligned16(a->y), "lora_linear: 16-byte alignment");
  if (lora) SB_CHECK_ARG(aligned16(a->lora_a) && aligned16(a->lora_b), "lora_linear: LoRA alignment");
  LinBuffers b;
  lora_linear_carve(a, nullptr, &b);
  if (!workspace || workspace_bytes < b.bytes)
    return set_error(STAGEML_ERR_WORKSPACE, "lora_linear: workspace of %zu bytes < required %zu", workspace_bytes,
                     b.bytes);
  lora_linear_carve(a, workspace, &b);
  int32_t* stat = a->status ? a->status : b.status;
  const int bf = a->dtype == STAGEML_BF16;
  const int n_ten = lora ? a->n_tenants : 0;
  const bool pdl = pdl_enabled();  // programmatic dependent launches along the chain
  GemmLaunch g;
  g.pdl = pdl;
  g.K = a->K;
  g.b = a->w_bank;
  g.b_rows_total = (int64_t)a->n_groups * a->N;
  g.b_group_rows = a->N;
  g.N = a->N;
  g.in_bf16 = bf;
  g.bias = a->bias;
  g.bias_group_stride = 0;
  g.status = stat;
  ShrinkLaunch sh;
  sh.K = a->K;
  sh.dtype_bf16 = bf;
  sh.pdl = pdl;
  if (lora) {
    sh.lora_a = a->lora_a;
    sh.a_tenant_stride = (int64_t)a->rank * a->K;
    sh.a_group_stride = 0;
    sh.R = a->rank;
    sh.a_rows_total = (int64_t)a->n_tenants * a->rank;
    sh.status = stat;
    sh.spart = b.spart;
    sh.s_out = b.s;
    sh.lora_scale = a->lora_scale;
    g.s16 = b.s;
    g.rank = a->rank;
    g.lora_b = a->lora_b;
    g.lora_b_tenant_stride = (int64_t)a->N * a->rank;
    g.lora_b_group_stride = 0;
    g.lora_b_rows_total = (int64_t)a->n_tenants * a->N;
    g.tile_runs = b.runs;
    g.tile_nruns = b.nruns;
  }
  if (a->n_groups == 1) {
    if (lora) {
      SB_STAGE(STAGEML_STAGE_GATHER_SHRINK,
               launch_validate_tenants(a->row_tenant, a->M, n_ten, b.tenants, stat, st, pdl));
      if (!b.pp.on())
        SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, launch_tile_runs(b.tenants, nullptr, a->M, (int)((a->M + 127) / 128),
                                                               b.runs, b.nruns, st, nullptr, pdl));
      sh.src = a->x;
      sh.static_rows = a->M;
      sh.rows_cap = a->M;
      sh.row_tenant = b.tenants;
      if (a->M <= kRowShrinkMaxRows)
        SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, launch_pair_shrink(sh, nullptr, a->M, st, pdl));
      else
        SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, launch_gather_shrink(sh, st));
      g.s_rows = a->M;
    }
    if (b.pp.on())
      SB_STAGE(STAGEML_STAGE_PERMUTE,
               build_pair_plan(b.pp, nullptr, nullptr, nullptr, a->M, lora ? b.tenants : nullptr, st, pdl));
    g.a = a->x;
    g.a_rows = a->M;
    g.m_rows = a->M;
    g.out = a->y;
    g.ldo = a->N;
    SB_STAGE(STAGEML_STAGE_GEMM, run_grouped_gemm(g, b.pp, st));
    return STAGEML_OK;
  }
  PermuteScratch scr;
  permute_carve(b.perm, a->M, permute_num_keys(0, n_ten, 0, a->n_groups), &scr);
  SB_STAGE(STAGEML_STAGE_PERMUTE,
           launch_permute(a->row_group, STAGEML_I32, nullptr, STAGEML_F32, lora ? a->row_tenant : nullptr, a->M, 1, 0,
                          a->n_groups, n_ten, 0, b.plan, stat, scr, st, nullptr, pdl));
  const int tiles_cap = (int)(b.plan.rows_cap / 128);
  if (b.pp.on())
    SB_STAGE(STAGEML_STAGE_PERMUTE, build_pair_plan(b.pp, b.plan.tile_group, b.plan.group_offsets, b.plan.num_tiles,
                                                    0, lora ? b.plan.row_tenant : nullptr, st, pdl));
  else if (lora)
    SB_STAGE(STAGEML_STAGE_PERMUTE, launch_tile_runs(b.plan.row_tenant, b.plan.num_tiles, 0, tiles_cap, b.runs,
                                                     b.nruns, st, nullptr, pdl));
  sh.src = a->x;
  sh.src_row_of = b.plan.row_token;
  sh.gather_dst = b.xp;
  sh.num_tiles_dev = b.plan.num_tiles;
  sh.rows_cap = b.plan.rows_cap;
  sh.row_tenant = b.plan.row_tenant;
  sh.tile_group = b.plan.tile_group;
  if (lora && a->M <= kRowShrinkMaxRows) {
    // gather alone, then the shrink per row (reading the source rows in place)
    ShrinkLaunch gather = sh;
    gather.R = 0;
    gather.lora_a = nullptr;
    SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, launch_gather_shrink(gather, st));
    SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, launch_pair_shrink(sh, b.plan.pair_row, a->M, st, pdl));
  } else {
    SB_STAGE(STAGEML_STAGE_GATHER_SHRINK, launch_gather_shrink(sh, st));
  }
  g.a = b.xp;
  g.a_rows = b.plan.rows_cap;
  g.num_tiles_dev = b.plan.num_tiles;
  g.tiles_cap = tiles_cap;
  g.tile_group = b.plan.tile_group;
  g.s_rows = b.plan.rows_cap;
  g.out = b.yp;
  g.ldo = a->N;
  bool two_streams = false;
  SB_STAGE(STAGEML_STAGE_GEMM, run_grouped_gemm(g, b.pp, st, &two_streams));
  SB_STAGE(STAGEML_STAGE_COMBINE,
           launch_combine(b.yp, b.plan.pair_row, a->M, 1, a->N, bf, a->y, st, nullptr, pdl && !two_streams));
  return STAGEML_OK;
}

size_t stageml_lora_gemv_f32_workspace_bytes(int M, int in_features, int out_features, int rank) {
  if (M < 1 || in_features < 1 || out_features < 1) return 0;
  return gemv_f32_workspace(M, in_features, out_features, rank);
}

int stageml_lora_gemv_f32(const float* x, const float* W, const float* A, const float* B, float scale, int M,
                          int in_features, int out_features, int rank, float* y, void* workspace,
                          size_t workspace_bytes, stageml_stream_t stream) {
  clear_error();
  SB_CHECK_ARG(M >= 1 && in_features >= 1 && out_features >= 1, "lora_gemv_f32: bad sizes");
  const size_t need = gemv_f32_workspace(M, in_features, out_features, rank);
  if (!workspace || workspace_bytes < need)
    return set_error(STAGEML_ERR_WORKSPACE, "lora_gemv_f32: workspace of %zu bytes < required %zu",
                     workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SB_STAGE(STAGEML_STAGE_GEMV,
           launch_gemv_f32(x, W, A, B, scale, M, in_features, out_features, rank, y, workspace, st));
  return STAGEML_OK;
}

int stageml_quantize_e4m3_rows(const void* w, int dtype, int64_t rows, int64_t cols, uint8_t* q_out, float* scale_out,
                               stageml_stream_t stream) {
  clear_error();
  return launch_quantize_e4m3_rows(w, dtype, rows, cols, q_out, scale_out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
