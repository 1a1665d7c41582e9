// Internal launchers shared between the kernel translation units and the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/stageml_b200.h"

namespace sb {

// route.cu
int launch_router_logits(const void* x, int x_dtype, const float* gate_w, int T, int H, int E, float* logits,
                         cudaStream_t stream);
int launch_topk(const float* logits, int T, int E, int k, int renorm, int32_t* ids, float* weights,
                cudaStream_t stream);
// Router logits + top-k; a few tokens (at most 64, gate and 8 rows per CTA in
// shared memory) take one fused kernel, more tokens with E <= 32 another (gate in
// shared memory, two tokens per warp), otherwise launch_router_logits then
// launch_topk. pdl: the fused kernel as a programmatic dependent launch (host_util.h).
int launch_route(const void* x, int x_dtype, const float* gate_w, int T, int H, int E, int k, int renorm,
                 float* logits, int32_t* ids, float* weights, cudaStream_t stream, bool pdl = false);

// permute.cu
struct PermuteScratch {
  uint32_t* sorted;  // [nchunks * 2048]
  int32_t* hist;     // [nkeys * nchunks]
  int32_t* off;      // [nchunks * nkeys] destination offsets
  int32_t* ticket;   // [1] chunks finished (multi-chunk rank kernel); zeroed by launch_permute
};
constexpr int kPermChunk = 2048;
// Sort keys of a permutation: (expert, tenant + 1) or (tenant, expert) keys, plus one per folded weight group.
int64_t permute_num_keys(int n_fold, int n_tenants, int group_by_tenant, int n_experts_total);
size_t permute_scratch_bytes(int64_t num_pairs, int64_t nkeys);
void permute_carve(void* base, int64_t num_pairs, int64_t nkeys, PermuteScratch* out);
int launch_permute(const void* ids, int ids_dtype, const void* weights, int weights_dtype, const int32_t* tenant_ids,
                   int T, int k, int n_shared, int n_experts_total, int n_tenants, int group_by_tenant,
                   const stageml_moe_plan& plan, int32_t* status, const PermuteScratch& scr, cudaStream_t stream,
                   const int32_t* T_dev = nullptr,  // T_dev: optional device count of valid tokens
                   bool pdl = false,                // pdl: single-kernel plans as PDL launches
                   const int32_t* fold_slot = nullptr,  // [n_tenants, E_tot] folded weight group per (tenant,
                   int n_fold = 0);                     // expert) or -1; groups E_tot .. E_tot + n_fold - 1

// shrink.cu: gather rows and/or LoRA shrink partials (split-K), then reduce.
struct ShrinkLaunch {
  const void* src = nullptr;          // [src_rows, K] 16-bit
  const int32_t* src_row_of = nullptr;  // row -> source row (-1 = zero row); null = identity
  void* gather_dst = nullptr;         // [rows_cap, K] or null
  int K = 0;
  int dtype_bf16 = 1;
  const int32_t* num_tiles_dev = nullptr;  // active rows = 128 * (*num_tiles_dev); null -> static_rows
  int64_t static_rows = 0;
  int64_t rows_cap = 0;
  const int32_t* row_tenant = nullptr;
  const int32_t* tile_group = nullptr;  // null -> group 0
  const void* lora_a = nullptr;         // [tenant][group][R][K]
  int64_t a_tenant_stride = 0;
  int64_t a_group_stride = 0;
  int64_t a_rows_total = 0;             // rows of K elements in the whole A bank (0: unknown)
  int R = 0;                            // output columns (multiple of 8, <= 64)
  float* spart = nullptr;               // [KS][rows_cap][R]
  void* s_out = nullptr;                // [rows_cap][R] 16-bit (reduced, scaled): the LoRA-expand MMA operand
  const float* lora_scale = nullptr;    // [n_tenants]
  bool pdl = false;                     // programmatic dependent launches (both kernels wait first)
  int32_t* status = nullptr;            // error word for expired bounded waits (tensor-core shrink)
  // optional [rows_cap]: each row's run index in its 128-row tile (launch_tile_runs);
  // S is then written [rows_cap][2R] in the run-parity layout of the packed rank-8 expand
  const int8_t* row_run = nullptr;
};
constexpr int kShrinkKSlice = 512;
inline int shrink_num_slices(int K) { return (K + kShrinkKSlice - 1) / kShrinkKSlice; }
// Gather and/or shrink. Rows already in the GEMM layout (no gather), and gathered rows
// once they are written (STAGEML_SHRINK), take the tensor-core shrink of shrink_tc.cu;
// the rest the per-warp mma.sync kernel.
int launch_gather_shrink(const ShrinkLaunch& s, cudaStream_t stream);
// shrink_tc.cu: the partials of the shrink of rows `rows` ([rows_cap or static_rows, K],
// the plan's layout) on tcgen05, one persistent CTA per SM; same partial layout as
// the per-warp kernel, reduced by the same kernel.
bool tc_shrink_supported(const ShrinkLaunch& s);
int launch_tc_shrink(const ShrinkLaunch& s, const void* rows, cudaStream_t stream);
// The shrink per row, for decode-sized batches and for small batches whose rows span
// many tenants: pairs p < P (pair_row[p] = their plan row; pair_row null: row p),
// one CTA per (pair, 8 output columns) whose 8 warps split K in a fixed order;
// writes the scaled 16-bit S rows (zeros for rows without a tenant) and reads the
// source rows in place (src_row_of, if given, maps a plan row to its source row).
// pdl: as a programmatic dependent launch that lets the next kernel start at once.
int launch_pair_shrink(const ShrinkLaunch& s, const int32_t* pair_row, int64_t P, cudaStream_t stream,
                       bool pdl = false);

// combine.cu: out[t] = sum_j Y[pair_row[t*kk + j]]
int launch_combine(const void* y, const int32_t* pair_row, int T, int kk, int H, int dtype_bf16, void* out,
                   cudaStream_t stream, const int32_t* T_dev = nullptr,  // rows >= *T_dev left untouched
                   bool pdl = false);
// One-expert top-1 layer in token order: row_tenant[t] = validated tenant, row_scale[t] =
// routing weight (1 without weights), both -1 / 0 with status for an expert id other
// than 0 or a tenant out of range.
int launch_direct_rows(const void* ids, int ids_dtype, const void* weights, int weights_dtype, const int32_t* tenant_ids,
                       int n_tenants, int64_t T, int32_t* row_tenant, float* row_scale, int32_t* status,
                       cudaStream_t stream, bool pdl = false);
// clamp caller tenant ids into [-1, n_tenants) (invalid -> -1 + status)
int launch_validate_tenants(const int32_t* in, int64_t n, int n_tenants, int32_t* out, int32_t* status,
                            cudaStream_t stream, bool pdl = false);

// fold.cu
int launch_lora_fold(const void* W, const void* A, const void* B, const float* scale, int batch, int rows, int cols,
                     int rank, int layout, int64_t w_bs, int64_t a_bs, int64_t b_bs, int dtype, void* out,
                     cudaStream_t stream);

// gemv.cu
size_t gemv_f32_workspace(int M, int in_f, int out_f, int rank);
int launch_gemv_f32(const float* x, const float* W, const float* A, const float* B, float scale, int M, int in_f,
                    int out_f, int rank, float* y, void* ws, cudaStream_t stream);

// fp8.cu
int launch_quantize_e4m3_rows(const void* w, int dtype, int64_t rows, int64_t cols, uint8_t* q, float* scale,
                              cudaStream_t stream);

}  // namespace sb
