/*
 * stageml_b200.h -- C ABI of the B200 (sm_100a) implementation of StageML's
 * request-time multi-tenant MoE-LoRA residual program.
 *
 * Plain C: device pointers, sizes, dtype codes and a CUDA stream handle. No
 * torch types. Every entry point is asynchronous on `stream`, allocates
 * nothing (scratch comes from the caller's `workspace`, sized by the matching
 * *_workspace_bytes query) and returns STAGEML_OK or an error code whose text is
 * available from stageml_last_error() on the calling thread. Argument checks
 * happen on the host before anything is launched; data-dependent faults found
 * on the device (an expert id or tenant id out of range, a bounded wait that
 * expired) are recorded in the caller-supplied device status word instead of
 * trapping, and the offending pair or row is skipped.
 *
 * Reference interfaces replaced (paths inside the uwm-se/stageML project):
 *   csrc/stageml_residual_op.cpp:8-19        residual_moe custom op (skeleton that throws)
 *   stageml/custom_op_registry.py:23-37     _fallback_moe (per-token Python loop)
 *   stageml/moe_lora_layers.py:45-142       DynamicMoELoRALayer / MaterializedMoELoRALayer
 *   stageml/moe_lora_layers.py:178-183      normalize_routing_weights
 *   stageml/adapter_bank.py:42-135          DynamicLoRALinear / StageMLAdapterBankLinear / OnTheFlyMergeLinear
 *   stageml/adapter_cache.py:37-100         StageMLCostBasedAdapterCache
 *   stageml/triton_generator.py:175-191     materialize_residual_weight
 *   benchmarks/multitenant_bta_system_bench.py:379-443   RequestExecutor (SwiGLU expert MLP + LoRA)
 *   benchmarks/real_moe_lora_residual_bench.py:360-386   make_routing (softmax / top-k / renorm)
 *   benchmarks/triton_lora_equivalence_check.py:11-22    single LoRA linear, [in,out] layout
 */
#ifndef STAGEML_B200_H
#define STAGEML_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* stageml_stream_t; /* a cudaStream_t; NULL = legacy default stream */

/* Return codes. */
enum {
  STAGEML_OK = 0,
  STAGEML_ERR_INVALID_ARG = 1, /* shape, dtype, pointer or alignment rejected on the host */
  STAGEML_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed */
  STAGEML_ERR_UNSUPPORTED = 3, /* valid request this build does not implement */
  STAGEML_ERR_WORKSPACE = 4    /* workspace pointer NULL or smaller than the query says */
};

/* Element type codes. */
enum {
  STAGEML_F32 = 0,
  STAGEML_BF16 = 1,
  STAGEML_F16 = 2,
  STAGEML_E4M3 = 3, /* float8 e4m3fn, weights only, with fp32 per-output-channel scales */
  STAGEML_I32 = 4,
  STAGEML_I64 = 5
};

/* Device status words (written to `status` by kernels, 0 = ok). */
enum {
  STAGEML_DEV_OK = 0,
  STAGEML_DEV_TIMEOUT = 101,   /* 101..104: a bounded wait in a pipelined kernel expired */
  STAGEML_DEV_BAD_INDEX = 110, /* an expert / tenant / group id was out of range; that item was skipped */
  STAGEML_DEV_PEER_TIMEOUT = 105 /* expert parallel: another GPU did not signal within the bound */
};

/* Text of the last error reported on this thread ("" if none). */
const char* stageml_last_error(void);
/* ABI version of this library (bumped on any signature or struct change). */
int stageml_abi_version(void);
/* sizeof() of the public structs, so bindings can check their mirrors. 0 = plan, 1 = moe args, 2 = lora linear args. */
size_t stageml_struct_size(int which);

/* Per-stage device timing (benchmark support; no counterpart in the reference,
 * whose timing is CUDA events around whole calls, stageml/benchmark_stats.py:85-113).
 * While enabled on the calling thread, the entry points below record a CUDA
 * event pair around each of their kernel stages on their stream.
 * stageml_stage_timer_read waits for those events, adds the elapsed
 * milliseconds of stage s to ms_out[s] and the number of timed launches to
 * counts_out[s] (s < n), and forgets them. Disabled by default.
 * stageml_stage_timer_select limits the recorded stages to those whose bit is
 * set in `mask` (bit s = stage s; all stages by default), so that a benchmark can
 * time one stage inside its timed calls at the cost of one event pair per call. */
enum {
  STAGEML_STAGE_ROUTE = 0,
  STAGEML_STAGE_PERMUTE = 1,
  STAGEML_STAGE_GATHER_SHRINK = 2, /* row gather + LoRA shrink of the layer input */
  STAGEML_STAGE_GEMM_GATE_UP = 3,  /* grouped gate/up GEMM + LoRA expand + SwiGLU */
  STAGEML_STAGE_SHRINK_H = 4,      /* LoRA shrink of the SwiGLU output */
  STAGEML_STAGE_GEMM_DOWN = 5,     /* grouped down GEMM + LoRA expand + routing weight */
  STAGEML_STAGE_COMBINE = 6,
  STAGEML_STAGE_GEMM = 7,          /* the GEMM of lora_linear / moe_linear */
  STAGEML_STAGE_FOLD = 8,
  STAGEML_STAGE_GEMV = 9,
  STAGEML_NUM_STAGES = 10
};
int stageml_stage_timer_enable(int on);
int stageml_stage_timer_select(unsigned int mask);
int stageml_stage_timer_read(float* ms_out, int32_t* counts_out, int n);
/* Number of kernels this library has launched in the process so far (all threads). */
unsigned long long stageml_launch_count(void);

/* ------------------------------------------------------------------ routing
 * Replaces make_routing (benchmarks/real_moe_lora_residual_bench.py:360-386)
 * followed by normalize_routing_weights (stageml/moe_lora_layers.py:178-183):
 *   logits = float(x) . gate_w^T   (fp32 accumulate)       [T, E]
 *   probs  = softmax(logits)                                [T, E]
 *   ids, weights = top-k(probs), larger first, ties -> lower expert index
 *   if renormalize: weights /= max(sum(weights), 1e-12)
 * x: [T, H] (F32/BF16/F16), gate_w: [E, H] fp32. E <= 256, k <= 8, k <= E.
 * logits_out may be NULL. ids_out int32 [T, k], weights_out fp32 [T, k].
 */
int stageml_route_topk(const void* x, int x_dtype, const float* gate_w, int T, int H, int E, int k,
                       int renormalize, float* logits_out, int32_t* ids_out, float* weights_out,
                       stageml_stream_t stream);

/* The softmax / top-k / renorm half of stageml_route_topk on given fp32 logits [T, E]. */
int stageml_topk_from_logits(const float* logits, int T, int E, int k, int renormalize, int32_t* ids_out,
                             float* weights_out, stageml_stream_t stream);

/* -------------------------------------------------------------- permutation
 * Token -> expert permutation (the grouping that RequestExecutor.dynamic_one
 * does with one torch.nonzero per (slot, expert),
 * benchmarks/multitenant_bta_system_bench.py:401-406).
 *
 * The T*(k+n_shared) pairs (t, j) -- j < k routed slot with expert ids[t, j]
 * and weight w[t, j]; j >= k always-on shared expert E + (j - k) with weight
 * 1 -- are stably sorted by key (expert, tenant) (tenant -1 sorts first), and
 * each expert's segment is padded to a multiple of 128 rows. Pair index
 * p = t*(k+n_shared) + j is the stable tie order. With group_by_tenant != 0
 * the grouping key's expert part is tenant*E_total + expert (one weight group
 * per (adapter, expert), as in MaterializedMoELoRALayer) and rows carry no
 * LoRA tenant.
 */
typedef struct stageml_moe_plan {
  int32_t* row_token;      /* [rows_cap] token of each padded row, -1 = padding */
  int32_t* row_tenant;     /* [rows_cap] LoRA tenant of each row, -1 = none / padding */
  float* row_weight;       /* [rows_cap] routing weight of each row, 0 for padding */
  int32_t* row_pair;       /* [rows_cap] pair index of each row, -1 = padding */
  int32_t* pair_row;       /* [T*(k+n_shared)] padded row of each pair, -1 = dropped (bad id) */
  int32_t* tile_group;     /* [rows_cap/128] weight group (expert) of each 128-row tile */
  int32_t* group_offsets;  /* [n_groups+1] padded row offset of each group's segment */
  int32_t* group_counts;   /* [n_groups] real rows per group */
  int32_t* num_tiles;      /* [1] number of 128-row tiles in use */
  int64_t rows_cap;        /* capacity of the row arrays; >= stageml_plan_rows_cap(...) */
} stageml_moe_plan;

/* Row capacity needed for P pairs spread over n_groups groups (each padded to 128). */
int64_t stageml_plan_rows_cap(int64_t num_pairs, int n_groups);
size_t stageml_permute_workspace_bytes(int T, int k, int n_shared, int n_experts_total, int n_tenants,
                                       int group_by_tenant);
/* ids: [T, k] int32 or int64 (ids_dtype); weights: [T, k] F32/BF16/F16 or NULL (= 1);
 * tenant_ids: [T] int32 or NULL (= -1). n_experts_total includes the n_shared shared experts. */
int stageml_permute(const void* ids, int ids_dtype, const void* weights, int weights_dtype,
                    const int32_t* tenant_ids, int T, int k, int n_shared, int n_experts_total, int n_tenants,
                    int group_by_tenant, const stageml_moe_plan* plan, int32_t* status, void* workspace,
                    size_t workspace_bytes, stageml_stream_t stream);

/* Combine (the index_add_ of RequestExecutor.dynamic_one,
 * benchmarks/multitenant_bta_system_bench.py:413, done once per token):
 * out[t, :] = sum_{j < kk} y[pair_row[t*kk + j], :] in fp32 with one rounding,
 * slots in order; pair_row < 0 is skipped. y / out: [*, H] BF16 or F16, H % 8 == 0. */
int stageml_combine_rows(const void* y, const int32_t* pair_row, int T, int kk, int H, int dtype, void* out,
                         stageml_stream_t stream);

/* ------------------------------------------------------- MoE-LoRA layer
 * The request-time residual program for one MoE FFN layer (R1..R5 + combine):
 *   route (when topk_ids == NULL) -> permute -> gather + LoRA shrink ->
 *   grouped gate/up GEMM with LoRA expand and SwiGLU in the epilogue ->
 *   LoRA shrink of h -> grouped down GEMM with LoRA expand and routing weight
 *   in the epilogue -> combine.
 * For token t: out[t] = sum_j w[t,j] * down_e( silu(g) * u ), e = expert of slot j,
 *   g = x W1_e^T + s_a (x A1[a,e]^T) B1[a,e]^T,   W1_e = gate_up[e, :I]
 *   u = x W3_e^T + s_a (x A3[a,e]^T) B3[a,e]^T,   W3_e = gate_up[e, I:]
 *   down_e(h) = h W2_e^T + s_a (h A2[a,e]^T) B2[a,e]^T,  a = tenant_ids[t]
 * This is RequestExecutor.dynamic_one (benchmarks/multitenant_bta_system_bench.py:398-414,
 * LoRA on w1) with the same LoRA term on w3 and w2 as DynamicMoELoRALayer.forward
 * (stageml/moe_lora_layers.py:85-89); with all LoRA pointers NULL it is exactly
 * _fallback_moe (stageml/custom_op_registry.py:23-37), i.e. the residual_moe op.
 * Tenants with a folded (materialized) gate_up either pass tenant -1 and their own
 * gate_up, as bta_one does (:416-433), or share one call with every other tenant
 * through fold_slot: folded weight sets are stored after the E_tot base experts in
 * gate_up / down, and a pair whose (tenant, expert) has a folded set runs on it
 * (group E_tot + slot) with no dynamic LoRA, in the same permutation and the same
 * GEMM launches as the dynamic pairs (the decision residual_planner.py:48-153
 * makes per (adapter, expert), served without splitting the batch on the host).
 *
 * Layouts (row-major, contiguous):
 *   x [T,H]; gate_up [E_tot + n_fold, 2I, H]; down [E_tot + n_fold, H, I]   (E_tot = E + n_shared;
 *     with down_group, down [E_tot, H, I])
 *   gate_up_scale [E_tot, 2I] / down_scale [E_tot, H] fp32 when weight_dtype == E4M3
 *   fold_slot [n_tenants, E_tot] int32: -1 = dynamic, s in [0, n_fold) = folded set s
 *   lora_a13 [n_tenants, E_tot, 2r, H] rows [0,r) = A1, [r,2r) = A3
 *   lora_b13 [n_tenants, E_tot, 2I, r] rows [0,I) = B1, [I,2I) = B3
 *   lora_a2 [n_tenants, E_tot, r, I]; lora_b2 [n_tenants, E_tot, H, r]
 *   lora_scale [n_tenants] fp32 (alpha / rank)
 * r must be a multiple of 8 and <= 32 (zero-pad A rows / B columns to get there).
 * H and I must be multiples of 8 (16-byte TMA row pitch).
 */
typedef struct stageml_moe_args {
  int T, H, I, E, k, n_shared;
  int act_dtype;         /* BF16 or F16: x, out, LoRA factors */
  int weight_dtype;      /* == act_dtype, or E4M3 */
  const void* x;
  const void* topk_ids;  /* [T,k] int32/int64, or NULL to route with router_w */
  int ids_dtype;
  const void* topk_weights; /* [T,k] F32/BF16/F16 (used as given); ignored when routing here */
  int weights_dtype;
  const float* router_w; /* [E,H] fp32, used when topk_ids == NULL */
  int renormalize;       /* routing here: renormalize the top-k weights */
  const int32_t* tenant_ids; /* [T] or NULL */
  int n_tenants;
  int rank;              /* 0 = no LoRA */
  const void* gate_up;
  const void* down;
  const float* gate_up_scale;
  const float* down_scale;
  const void* lora_a13;  /* NULL = no LoRA on w1/w3 */
  const void* lora_b13;
  const void* lora_a2;   /* NULL = no LoRA on w2 */
  const void* lora_b2;
  const float* lora_scale;
  void* out;             /* [T,H] act_dtype */
  int32_t* status;       /* device status word, may be NULL */
  const stageml_moe_plan* plan_out; /* optional: keep the permutation in caller memory */
  const int32_t* T_dev;  /* optional device int: only tokens [0, *T_dev) are valid (<= T); the rest
                            are skipped and their output rows left untouched. Used when the token
                            count is known only on the device (rows received from other GPUs). */
  const int32_t* fold_slot; /* optional [n_tenants, E_tot]: per (tenant, expert), -1 = base weights plus
                               that tenant's LoRA, s >= 0 = folded weight group E_tot + s, no LoRA.
                               An entry outside [-1, n_fold) drops the pair (STAGEML_DEV_BAD_INDEX).
                               16-bit weights only (not with E4M3). */
  int n_fold;               /* folded weight groups stored after the E_tot base experts (0 = none) */
  const int32_t* down_group; /* optional [E_tot + n_fold], entries in [0, E_tot): weight group g takes its
                                down projection from down[down_group[g]], and down holds only the E_tot base
                                experts (folded sets of adapters with no LoRA on w2 share their base expert's
                                down weights); NULL: down holds all E_tot + n_fold groups */
} stageml_moe_args;

size_t stageml_moe_workspace_bytes(const stageml_moe_args* args);
int stageml_moe_forward(const stageml_moe_args* args, void* workspace, size_t workspace_bytes,
                        stageml_stream_t stream);

/* The 5-argument residual_moe op of csrc/stageml_residual_op.cpp:8-19 with the
 * semantics of _fallback_moe (stageml/custom_op_registry.py:23-37):
 *   out[t] = sum_j w[t,j] * down[e] . (silu(gate_up[e,:I] . x_t) * gate_up[e,I:] . x_t), e = ids[t,j].
 * hidden [T,H] BF16/F16, gate_up [E,2I,H], down [E,H,I] same dtype, topk_weights [T,k]
 * (F32/BF16/F16), topk_ids [T,k] (I32/I64). out [T,H] hidden dtype. */
size_t stageml_residual_moe_workspace_bytes(int T, int H, int I, int E, int k);
int stageml_residual_moe(const void* hidden, const void* gate_up, const void* down, const void* topk_weights,
                         int weights_dtype, const void* topk_ids, int ids_dtype, int T, int H, int I, int E,
                         int k, int dtype, void* out, int32_t* status, void* workspace,
                         size_t workspace_bytes, stageml_stream_t stream);

/* ------------------------------------------- MoE single-linear LoRA layer
 * DynamicMoELoRALayer.forward (stageml/moe_lora_layers.py:63-90):
 *   out[t] = sum_j w[t,j] * (x_t W[e]^T + bias[e] + s_a (x_t A[a,e]^T) B[a,e]^T)
 * and, with lora == NULL and group_by_tenant = 1 on merged weights
 * [n_adapters*E, N, K], MaterializedMoELoRALayer.forward (:117-142).
 * x [T,K]; weight [G, N, K]; bias [E, N] or NULL; lora_a [n_tenants, E, r, K];
 * lora_b [n_tenants, E, N, r]. K, N multiples of 8. */
size_t stageml_moe_linear_workspace_bytes(int T, int K, int N, int E, int k, int group_by_tenant, int n_tenants,
                                          int rank);
int stageml_moe_linear(const void* x, const void* weight, const void* bias, const void* topk_ids, int ids_dtype,
                       const void* topk_weights, int weights_dtype, const int32_t* tenant_ids, int T, int K, int N,
                       int E, int k, int group_by_tenant, int n_tenants, int rank, const void* lora_a,
                       const void* lora_b, const float* lora_scale, int dtype, void* out, int32_t* status,
                       void* workspace, size_t workspace_bytes, stageml_stream_t stream);

/* ---------------------------------------------------- stage-0 LoRA fold
 * W' = W + scale * L . R for `batch` independent matrices (R7):
 *   layout 0 ([out,in], StageML's layout): W [out,in], L = B [out,r], R = A [r,in]
 *     (materialize_residual_weight, stageml/triton_generator.py:175-191;
 *      StageMLAdapterBankLinear.__init__, stageml/adapter_bank.py:90-94;
 *      MaterializedMoELoRALayer.__init__ einsum("eor,eri->eoi"), stageml/moe_lora_layers.py:104-110)
 *   layout 1 ([in,out]): W [in,out], L = A [in,r], R = B [r,out]
 *     (the folded single LoRA x(W + sAB), benchmarks/triton_lora_equivalence_check.py:11-22)
 * Matrix b reads W + b*w_batch_stride, A + b*a_batch_stride, B + b*b_batch_stride
 * (element strides; 0 broadcasts one W over every adapter) and writes
 * out + b*rows*cols. scale[b] per matrix. dtype F32 (fp32 FMA, no TF32), BF16 or F16.
 * out may alias W only when w_batch_stride == rows*cols. */
int stageml_lora_fold(const void* W, const void* A, const void* B, const float* scale, int batch, int rows,
                      int cols, int rank, int layout, int64_t w_batch_stride, int64_t a_batch_stride,
                      int64_t b_batch_stride, int dtype, void* out, stageml_stream_t stream);

/* ------------------------------------------- multi-tenant dense LoRA linear
 * Mixed-adapter batch y = x W_g^T + bias + s_a (x A_a^T) B_a^T per row (R8):
 *   row_group[m] selects the weight (0 = base W, g > 0 = folded W'), row_tenant[m]
 *   selects the dynamic adapter (-1 = none).
 * DynamicLoRALinear.forward (stageml/adapter_bank.py:58-69): all rows group 0 + tenant;
 * StageMLAdapterBankLinear.forward (:101-109): group = adapter + 1, no tenant;
 * StageMLCostBasedAdapterCache.forward (stageml/adapter_cache.py:83-100): cached
 * adapters by group, the others by tenant.
 * x [M,K]; w_bank [n_groups, N, K]; bias [N] or NULL; lora_a [n_tenants, r, K];
 * lora_b [n_tenants, N, r]; lora_scale [n_tenants]. K, N multiples of 8. */
typedef struct stageml_lora_linear_args {
  int M, K, N;
  int dtype;              /* BF16 or F16 */
  const void* x;
  const void* w_bank;
  int n_groups;
  const void* bias;
  const int32_t* row_group;   /* NULL = all rows group 0 */
  const int32_t* row_tenant;  /* NULL = no LoRA */
  int n_tenants;
  int rank;
  const void* lora_a;
  const void* lora_b;
  const float* lora_scale;
  void* y;                /* [M,N] */
  int32_t* status;
} stageml_lora_linear_args;

size_t stageml_lora_linear_workspace_bytes(const stageml_lora_linear_args* args);
int stageml_lora_linear(const stageml_lora_linear_args* args, void* workspace, size_t workspace_bytes,
                        stageml_stream_t stream);

/* ---------------------------------------------- single LoRA linear, fp32
 * Config-1 form with W [in,out] (benchmarks/triton_lora_equivalence_check.py:11-22,
 * stageml/peft_bridge.py:59-63 transposed): y = x W + scale (x A) B, x [M,in],
 * A [in,r], B [r,out]; A == NULL gives the folded form y = x W'. fp32 FMA only.
 * M <= 16. */
size_t stageml_lora_gemv_f32_workspace_bytes(int M, int in_features, int out_features, int rank);
int stageml_lora_gemv_f32(const float* x, const float* W, const float* A, const float* B, float scale, int M,
                          int in_features, int out_features, int rank, float* y, void* workspace,
                          size_t workspace_bytes, stageml_stream_t stream);

/* Allocation-free variant of stageml_lora_gemv_f32 (no counterpart in the
 * reference; it exists for callers of this library that cannot allocate).
 * Same inputs, outputs and results, but no workspace argument: the split-K
 * partial sums go to a 16 MiB scratch array in device global memory that the
 * library itself holds, on every GPU that loads it, until the process exits.
 * Meant for callers that cannot call cudaMalloc where they run this layer:
 * a plugin reached only through this C ABI with no allocator of its own, a
 * serving loop that must never allocate or free device memory (both can
 * synchronize the device), or a host that plans its device memory in a fixed
 * arena. Inputs and the output y are still the caller's memory.
 *  - Shapes whose partial sums exceed the 16 MiB scratch return
 *    STAGEML_ERR_INVALID_ARG (in = out = 4096 fits every M up to 16; very wide
 *    outputs do not, e.g. M = 16 with out > 262,144 columns);
 *    stageml_lora_gemv_f32 with a workspace has no such limit.
 *  - The first call on a device looks up the scratch array's device address
 *    (cudaGetSymbolAddress, with that device current) and caches it together
 *    with the current driver context; a call made under another context of the
 *    device (a non-primary context, or the primary context recreated after
 *    cudaDeviceReset) looks the address up again. Make the first call on each
 *    device before any stream capture, since the lookup may load the module.
 *  - All calls share the one array, which keeps the last call's contents. No
 *    part of it needs to start at zero (each partial is written before it is
 *    read), but two calls whose kernels can overlap on the GPU (different
 *    streams or threads without ordering between them) race on it and give
 *    wrong results: order such calls, e.g. on one stream.
 *  - No allocation of any kind: no cudaMalloc, cudaFree or allocating library
 *    routine is called. */
int stageml_lora_gemv_f32_noalloc(const float* x, const float* W, const float* A, const float* B, float scale, int M,
                                  int in_features, int out_features, int rank, float* y, stageml_stream_t stream);

/* ------------------------------------------------------- FP8 weights (R6)
 * Per-output-channel e4m3 quantization of row-major weights [rows, cols]:
 * scale[r] = max(|w[r,:]|) / 448 (1 when the row is all zero), q = e4m3(w / scale)
 * with round-to-nearest-even and saturation to +-448. Input F32/BF16/F16. */
int stageml_quantize_e4m3_rows(const void* w, int dtype, int64_t rows, int64_t cols, uint8_t* q_out,
                               float* scale_out, stageml_stream_t stream);

/* ------------------------------------------------------- expert parallel over peer memory
 * No counterpart in the reference, which has no distributed code: this is the
 * expert-parallel layout of the MoE-LoRA layer (experts and their adapter-bank
 * slices sharded over `world` GPUs, one process per GPU). Instead of NCCL
 * all-to-alls with host-side split sizes, rows move with plain stores into the
 * other GPUs' memory (CUDA IPC mappings over NVLink / NVSwitch) and epoch flags;
 * the host never waits for counts.
 *
 * Every rank allocates one workspace with stageml_ep_workspace_alloc (layout from
 * stageml_ep_get_layout, identical on all ranks; zero-filled), exchanges the IPC
 * handles out of band (e.g. torch.distributed.all_gather_object), opens the
 * others' with stageml_ep_workspace_open and keeps a device array peers[world]
 * of all workspace bases (its own at index rank). A layer call with a new epoch
 * (1, 2, 3, ... per workspace) is:
 *   stageml_ep_dispatch  route this rank's pairs to the owners of their experts;
 *                        afterwards the receive region holds recv_tokens dense rows
 *                        (x, local expert, tenant, routing weight, source);
 *   (local expert computation on those rows, e.g. stageml_moe_forward with k = 1,
 *    T = world * tokens_cap * k and T_dev = the recv_tokens word)
 *   stageml_ep_return    send each result row back to its source;
 *   stageml_ep_combine   out[t] = sum_j result(t, j) (+ add[t]).
 * All three calls of an epoch go on one stream, and every rank makes them in the
 * same order. Waits on other GPUs are bounded (timeout_ns, default 5 s); on
 * expiry the status word gets STAGEML_DEV_PEER_TIMEOUT. world <= 8. */
typedef struct stageml_ep_layout {
  size_t count_matrix;  /* int32 [world][world]: row s = pairs rank s sends to each rank */
  size_t flags_count, flags_rows, flags_return; /* int32 [world] epoch flags, one per source */
  size_t counters;      /* int32 [4] */
  size_t recv_tokens;   /* int32: rows received in the current epoch */
  size_t recv_expert;   /* int32 [world*tokens_cap*k]: local expert of each received row */
  size_t recv_weight;   /* f32   [..]: routing weight */
  size_t recv_tenant;   /* int32 [..]: tenant (-1 = none) */
  size_t recv_source;   /* int32 [..]: source pair * world + source rank */
  size_t recv_x;        /* 16-bit [world*tokens_cap*k][H] */
  size_t ret_y;         /* 16-bit [tokens_cap*k][H]: result rows, by this rank's pair index */
  size_t total;
} stageml_ep_layout;

typedef struct stageml_ep_args {
  int world, rank;
  int T, k, H, E_loc;     /* this rank's tokens, slots, hidden size, experts per rank */
  int act_dtype;          /* BF16 or F16 */
  int epoch;              /* > 0, one more than the previous call on this workspace */
  int64_t tokens_cap;     /* T <= tokens_cap on every rank (sizes the buffers) */
  uint64_t timeout_ns;    /* 0 = 5 s */
  const uint64_t* peers;  /* device [world]: workspace base of every rank */
  void* self;             /* this rank's workspace */
  const int32_t* topk_ids;    /* [T,k] global expert ids (owner = id / E_loc) */
  const float* topk_weights;  /* [T,k] */
  const int32_t* tenant_ids;  /* [T] or NULL */
  const void* x;              /* [T,H] act_dtype */
  int32_t* pos;               /* [T*k] scratch */
  int32_t* status;            /* device status word or NULL */
} stageml_ep_args;

int stageml_ep_get_layout(int world, int64_t tokens_cap, int k, int H, int act_dtype, stageml_ep_layout* out);
int stageml_ep_workspace_alloc(size_t bytes, void** ptr, void* ipc_handle_64);
int stageml_ep_workspace_free(void* ptr);
int stageml_ep_workspace_open(const void* ipc_handle_64, void** ptr);
int stageml_ep_workspace_close(void* ptr);
int stageml_ep_dispatch(const stageml_ep_args* args, stageml_stream_t stream);
int stageml_ep_return(const stageml_ep_args* args, const void* y_local, stageml_stream_t stream);
int stageml_ep_combine(const stageml_ep_args* args, const void* add, void* out, stageml_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* STAGEML_B200_H */
