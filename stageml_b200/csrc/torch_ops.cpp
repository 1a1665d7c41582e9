// PyTorch custom-op library for the StageML B200 residual path.
//
// Loading this library (torch.ops.load_library, e.g. through the
// STAGEML_CUSTOM_OP_LIB hook of stageml/custom_op_registry.py:40-48) registers
// the `stageml` namespace with the unchanged schema of the reference's
//   residual_moe(Tensor hidden, Tensor gate_up, Tensor down, Tensor topk_weights, Tensor topk_ids) -> Tensor
// (csrc/stageml_residual_op.cpp:17-19) plus the ops of the rest of the path.
// Only the CUDA dispatch key is implemented: a CPU tensor raises "no kernel
// for CPU" instead of silently running a slow fallback. Every op marshals its
// tensors into the C ABI of libstageml_b200.so (include/stageml_b200.h) on the
// current CUDA stream; workspaces come from the caching allocator.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <mutex>
#include <unordered_map>

#include "../../include/stageml_b200.h"

namespace {

using at::Tensor;

int dtype_code(const Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat:
      return STAGEML_F32;
    case at::kBFloat16:
      return STAGEML_BF16;
    case at::kHalf:
      return STAGEML_F16;
    case at::kFloat8_e4m3fn:
      return STAGEML_E4M3;
    case at::kInt:
      return STAGEML_I32;
    case at::kLong:
      return STAGEML_I64;
    default:
      TORCH_CHECK(false, "stageml: unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == STAGEML_OK, "stageml::", what, " failed (code ", rc, "): ", stageml_last_error());
}

void check_cuda(const Tensor& t, const char* name, const Tensor& ref) {
  TORCH_CHECK(t.is_cuda(), "stageml: ", name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == ref.device(), "stageml: ", name, " is on ", t.device(), " but expected ", ref.device());
  TORCH_CHECK(t.is_contiguous(), "stageml: ", name, " must be contiguous");
}

const void* opt_ptr(const c10::optional<Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

Tensor workspace(size_t bytes, const Tensor& ref) {
  return at::empty({(int64_t)std::max<size_t>(bytes, 16)}, ref.options().dtype(at::kByte));
}

// Per-device status word that kernels write data-dependent errors into.
int32_t* status_word(const Tensor& ref) {
  static std::mutex mu;
  static std::unordered_map<int, Tensor> words;
  std::lock_guard<std::mutex> lk(mu);
  const int dev = ref.device().index();
  auto it = words.find(dev);
  if (it == words.end()) {
    it = words.emplace(dev, at::zeros({1}, ref.options().dtype(at::kInt))).first;
  }
  return it->second.data_ptr<int32_t>();
}

stageml_stream_t cur_stream() { return static_cast<stageml_stream_t>(at::cuda::getCurrentCUDAStream().stream()); }

// ------------------------------------------------------------------ ops
Tensor residual_moe(const Tensor& hidden, const Tensor& gate_up, const Tensor& down, const Tensor& topk_weights,
                    const Tensor& topk_ids) {
  TORCH_CHECK(hidden.dim() == 2 && gate_up.dim() == 3 && down.dim() == 3, "residual_moe: bad ranks");
  TORCH_CHECK(topk_ids.dim() == 2 && topk_weights.sizes() == topk_ids.sizes(), "residual_moe: bad top-k shapes");
  const int64_t T = hidden.size(0), H = hidden.size(1), E = gate_up.size(0), I2 = gate_up.size(1);
  TORCH_CHECK(I2 % 2 == 0 && gate_up.size(2) == H && down.size(0) == E && down.size(1) == H && down.size(2) == I2 / 2,
              "residual_moe: gate_up [E,2I,H] / down [E,H,I] do not match hidden [T,H]");
  TORCH_CHECK(topk_ids.size(0) == T, "residual_moe: topk_ids rows != tokens");
  TORCH_CHECK(gate_up.scalar_type() == hidden.scalar_type() && down.scalar_type() == hidden.scalar_type(),
              "residual_moe: gate_up and down must have hidden's dtype");
  for (auto* p : {&hidden, &gate_up, &down, &topk_weights, &topk_ids}) check_cuda(*p, "input", hidden);
  c10::cuda::CUDAGuard guard(hidden.device());
  auto out = at::empty({T, H}, hidden.options());
  const int k = (int)topk_ids.size(1);
  const size_t ws = stageml_residual_moe_workspace_bytes((int)T, (int)H, (int)(I2 / 2), (int)E, k);
  auto w = workspace(ws, hidden);
  check_rc(stageml_residual_moe(hidden.data_ptr(), gate_up.data_ptr(), down.data_ptr(), topk_weights.data_ptr(),
                                dtype_code(topk_weights), topk_ids.data_ptr(), dtype_code(topk_ids), (int)T, (int)H,
                                (int)(I2 / 2), (int)E, k, dtype_code(hidden), out.data_ptr(), status_word(hidden),
                                w.data_ptr(), (size_t)w.numel(), cur_stream()),
           "residual_moe");
  return out;
}

Tensor moe_forward(const Tensor& x, const Tensor& gate_up, const Tensor& down, const c10::optional<Tensor>& topk_weights,
                   const c10::optional<Tensor>& topk_ids, const c10::optional<Tensor>& router_w, int64_t k,
                   int64_t n_shared, bool renormalize, const c10::optional<Tensor>& tenant_ids, int64_t n_tenants,
                   int64_t rank, const c10::optional<Tensor>& lora_a13, const c10::optional<Tensor>& lora_b13,
                   const c10::optional<Tensor>& lora_a2, const c10::optional<Tensor>& lora_b2,
                   const c10::optional<Tensor>& lora_scale, const c10::optional<Tensor>& gate_up_scale,
                   const c10::optional<Tensor>& down_scale, const c10::optional<Tensor>& T_dev,
                   const c10::optional<Tensor>& fold_slot, int64_t n_fold,
                   const c10::optional<Tensor>& down_group) {
  TORCH_CHECK(x.dim() == 2 && gate_up.dim() == 3 && down.dim() == 3, "moe_forward: bad ranks");
  if (T_dev.has_value())
    TORCH_CHECK(T_dev->is_cuda() && T_dev->scalar_type() == at::kInt && T_dev->numel() >= 1,
                "moe_forward: T_dev must be a CUDA int32 tensor");
  TORCH_CHECK(n_fold >= 0 && n_fold < gate_up.size(0), "moe_forward: n_fold out of range");
  if (!fold_slot.has_value()) TORCH_CHECK(n_fold == 0, "moe_forward: n_fold > 0 needs fold_slot");
  // gate_up / down hold the E_tot base experts, then the n_fold folded weight groups
  const int64_t T = x.size(0), H = x.size(1), E_tot = gate_up.size(0) - n_fold, I = gate_up.size(1) / 2;
  const int64_t down_groups = down_group.has_value() ? E_tot : E_tot + n_fold;
  TORCH_CHECK(gate_up.size(2) == H && down.size(0) == down_groups && down.size(1) == H && down.size(2) == I,
              "moe_forward: weight shapes do not match x");
  if (down_group.has_value()) {
    check_cuda(*down_group, "down_group", x);
    TORCH_CHECK(down_group->scalar_type() == at::kInt && down_group->is_contiguous() &&
                    down_group->numel() == E_tot + n_fold,
                "moe_forward: down_group must be contiguous int32 [E_tot + n_fold]");
  }
  if (fold_slot.has_value()) {
    check_cuda(*fold_slot, "fold_slot", x);
    TORCH_CHECK(fold_slot->scalar_type() == at::kInt && fold_slot->is_contiguous() &&
                    fold_slot->numel() == n_tenants * E_tot,
                "moe_forward: fold_slot must be contiguous int32 [n_tenants, E_tot]");
  }
  check_cuda(x, "x", x);
  check_cuda(gate_up, "gate_up", x);
  check_cuda(down, "down", x);
  for (const auto* o : {&topk_weights, &topk_ids, &router_w, &tenant_ids, &lora_a13, &lora_b13, &lora_a2, &lora_b2,
                        &lora_scale, &gate_up_scale, &down_scale})
    if (o->has_value()) check_cuda(**o, "optional input", x);
  if (tenant_ids.has_value())
    TORCH_CHECK(tenant_ids->scalar_type() == at::kInt && tenant_ids->numel() == T,
                "moe_forward: tenant_ids must be int32 [T]");
  if (lora_scale.has_value()) TORCH_CHECK(lora_scale->scalar_type() == at::kFloat, "moe_forward: lora_scale fp32");
  if (router_w.has_value()) TORCH_CHECK(router_w->scalar_type() == at::kFloat, "moe_forward: router_w must be fp32");
  TORCH_CHECK(gate_up.scalar_type() == down.scalar_type(), "moe_forward: gate_up and down must share a dtype");
  if (gate_up.scalar_type() == at::kFloat8_e4m3fn) {
    TORCH_CHECK(gate_up_scale.has_value() && down_scale.has_value(),
                "moe_forward: e4m3 weights need gate_up_scale and down_scale");
    TORCH_CHECK(gate_up_scale->scalar_type() == at::kFloat && gate_up_scale->numel() == E_tot * 2 * I &&
                    gate_up_scale->is_contiguous(),
                "moe_forward: gate_up_scale must be contiguous fp32 [E_tot, 2I]");
    TORCH_CHECK(down_scale->scalar_type() == at::kFloat && down_scale->numel() == E_tot * H &&
                    down_scale->is_contiguous(),
                "moe_forward: down_scale must be contiguous fp32 [E_tot, H]");
  }
  c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty({T, H}, x.options());
  stageml_moe_args a{};
  a.T = (int)T;
  a.H = (int)H;
  a.I = (int)I;
  a.n_shared = (int)n_shared;
  a.E = (int)(E_tot - n_shared);
  a.k = (int)k;
  a.act_dtype = dtype_code(x);
  a.weight_dtype = dtype_code(gate_up);
  a.x = x.data_ptr();
  a.topk_ids = opt_ptr(topk_ids);
  a.ids_dtype = topk_ids.has_value() ? dtype_code(*topk_ids) : STAGEML_I32;
  a.topk_weights = opt_ptr(topk_weights);
  a.weights_dtype = topk_weights.has_value() ? dtype_code(*topk_weights) : STAGEML_F32;
  a.router_w = static_cast<const float*>(opt_ptr(router_w));
  a.renormalize = renormalize ? 1 : 0;
  a.tenant_ids = static_cast<const int32_t*>(opt_ptr(tenant_ids));
  a.n_tenants = (int)n_tenants;
  a.rank = (int)rank;
  a.gate_up = gate_up.data_ptr();
  a.down = down.data_ptr();
  a.gate_up_scale = static_cast<const float*>(opt_ptr(gate_up_scale));
  a.down_scale = static_cast<const float*>(opt_ptr(down_scale));
  a.lora_a13 = opt_ptr(lora_a13);
  a.lora_b13 = opt_ptr(lora_b13);
  a.lora_a2 = opt_ptr(lora_a2);
  a.lora_b2 = opt_ptr(lora_b2);
  a.lora_scale = static_cast<const float*>(opt_ptr(lora_scale));
  a.out = out.data_ptr();
  a.status = status_word(x);
  a.T_dev = static_cast<const int32_t*>(opt_ptr(T_dev));
  a.fold_slot = static_cast<const int32_t*>(opt_ptr(fold_slot));
  a.n_fold = (int)n_fold;
  a.down_group = static_cast<const int32_t*>(opt_ptr(down_group));
  const size_t ws = stageml_moe_workspace_bytes(&a);
  TORCH_CHECK(ws > 0 || T == 0, "moe_forward: invalid arguments: ", stageml_last_error());
  auto w = workspace(ws, x);
  check_rc(stageml_moe_forward(&a, w.data_ptr(), (size_t)w.numel(), cur_stream()), "moe_forward");
  return out;
}

std::tuple<Tensor, Tensor, Tensor> route_topk(const Tensor& x, const Tensor& gate_w, int64_t k, bool renormalize) {
  check_cuda(x, "x", x);
  check_cuda(gate_w, "gate_w", x);
  TORCH_CHECK(gate_w.scalar_type() == at::kFloat && gate_w.dim() == 2 && gate_w.size(1) == x.size(1),
              "route_topk: gate_w must be fp32 [E, H]");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), E = gate_w.size(0);
  auto ids = at::empty({T, k}, x.options().dtype(at::kInt));
  auto w = at::empty({T, k}, x.options().dtype(at::kFloat));
  auto logits = at::empty({T, E}, x.options().dtype(at::kFloat));
  check_rc(stageml_route_topk(x.data_ptr(), dtype_code(x), gate_w.data_ptr<float>(), (int)T, (int)x.size(1), (int)E,
                              (int)k, renormalize ? 1 : 0, logits.data_ptr<float>(), ids.data_ptr<int32_t>(),
                              w.data_ptr<float>(), cur_stream()),
           "route_topk");
  return {ids, w, logits};
}

std::tuple<Tensor, Tensor> topk_from_logits(const Tensor& logits, int64_t k, bool renormalize) {
  check_cuda(logits, "logits", logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2, "topk_from_logits: fp32 [T, E] logits");
  c10::cuda::CUDAGuard guard(logits.device());
  const int64_t T = logits.size(0);
  auto ids = at::empty({T, k}, logits.options().dtype(at::kInt));
  auto w = at::empty({T, k}, logits.options().dtype(at::kFloat));
  check_rc(stageml_topk_from_logits(logits.data_ptr<float>(), (int)T, (int)logits.size(1), (int)k, renormalize ? 1 : 0,
                                    ids.data_ptr<int32_t>(), w.data_ptr<float>(), cur_stream()),
           "topk_from_logits");
  return {ids, w};
}

std::vector<Tensor> permute(const Tensor& ids, const c10::optional<Tensor>& weights,
                            const c10::optional<Tensor>& tenant_ids, int64_t n_experts_total, int64_t n_shared,
                            int64_t n_tenants, bool group_by_tenant) {
  check_cuda(ids, "ids", ids);
  TORCH_CHECK(ids.dim() == 2, "permute: ids must be [T, k]");
  if (weights.has_value()) check_cuda(*weights, "weights", ids);
  if (tenant_ids.has_value()) {
    check_cuda(*tenant_ids, "tenant_ids", ids);
    TORCH_CHECK(tenant_ids->scalar_type() == at::kInt && tenant_ids->numel() == ids.size(0), "permute: tenant_ids");
  }
  c10::cuda::CUDAGuard guard(ids.device());
  const int T = (int)ids.size(0), k = (int)ids.size(1);
  const int64_t P = (int64_t)T * (k + n_shared);
  const int n_groups = group_by_tenant ? (int)(n_tenants * n_experts_total) : (int)n_experts_total;
  const int64_t rows_cap = stageml_plan_rows_cap(P, n_groups);
  auto io = ids.options().dtype(at::kInt);
  Tensor row_token = at::empty({rows_cap}, io), row_tenant = at::empty({rows_cap}, io),
         row_weight = at::empty({rows_cap}, io.dtype(at::kFloat)), row_pair = at::empty({rows_cap}, io),
         pair_row = at::empty({std::max<int64_t>(P, 1)}, io), tile_group = at::empty({rows_cap / 128}, io),
         group_offsets = at::empty({n_groups + 1}, io), group_counts = at::empty({n_groups}, io),
         num_tiles = at::empty({1}, io);
  stageml_moe_plan plan;
  plan.row_token = row_token.data_ptr<int32_t>();
  plan.row_tenant = row_tenant.data_ptr<int32_t>();
  plan.row_weight = row_weight.data_ptr<float>();
  plan.row_pair = row_pair.data_ptr<int32_t>();
  plan.pair_row = pair_row.data_ptr<int32_t>();
  plan.tile_group = tile_group.data_ptr<int32_t>();
  plan.group_offsets = group_offsets.data_ptr<int32_t>();
  plan.group_counts = group_counts.data_ptr<int32_t>();
  plan.num_tiles = num_tiles.data_ptr<int32_t>();
  plan.rows_cap = rows_cap;
  const size_t ws = stageml_permute_workspace_bytes(T, k, (int)n_shared, (int)n_experts_total, (int)n_tenants,
                                                    group_by_tenant ? 1 : 0);
  auto w = workspace(ws, ids);
  check_rc(stageml_permute(ids.data_ptr(), dtype_code(ids), opt_ptr(weights),
                           weights.has_value() ? dtype_code(*weights) : STAGEML_F32,
                           static_cast<const int32_t*>(opt_ptr(tenant_ids)), T, k, (int)n_shared, (int)n_experts_total,
                           (int)n_tenants, group_by_tenant ? 1 : 0, &plan, status_word(ids), w.data_ptr(),
                           (size_t)w.numel(), cur_stream()),
           "permute");
  return {row_token, row_tenant, row_weight, row_pair, pair_row, tile_group, group_offsets, group_counts, num_tiles};
}

// W: [rows, cols] (broadcast over the batch) or [batch, rows, cols]; A/B: [batch, ...] or unbatched.
Tensor lora_fold(const Tensor& W, const Tensor& A, const Tensor& B, const Tensor& scale, int64_t layout) {
  check_cuda(W, "W", W);
  check_cuda(A, "A", W);
  check_cuda(B, "B", W);
  check_cuda(scale, "scale", W);
  TORCH_CHECK(scale.scalar_type() == at::kFloat, "lora_fold: scale must be fp32 [batch]");
  TORCH_CHECK(A.scalar_type() == W.scalar_type() && B.scalar_type() == W.scalar_type(), "lora_fold: dtype mismatch");
  const bool batched = A.dim() == 3;
  TORCH_CHECK((batched && B.dim() == 3) || (!batched && A.dim() == 2 && B.dim() == 2), "lora_fold: A/B ranks");
  const int64_t batch = batched ? A.size(0) : 1;
  TORCH_CHECK(W.dim() == 2 || (W.dim() == 3 && W.size(0) == batch), "lora_fold: W must be [rows, cols] or [batch, ...]");
  const int64_t rows = W.size(-2), cols = W.size(-1);
  const int64_t rank = layout == 0 ? A.size(-2) : A.size(-1);
  if (layout == 0) {
    TORCH_CHECK(A.size(-1) == cols && B.size(-2) == rows && B.size(-1) == rank, "lora_fold: [out,in] shapes");
  } else {
    TORCH_CHECK(A.size(-2) == rows && B.size(-2) == rank && B.size(-1) == cols, "lora_fold: [in,out] shapes");
  }
  TORCH_CHECK(scale.numel() == batch, "lora_fold: one scale per matrix");
  c10::cuda::CUDAGuard guard(W.device());
  auto out = batched ? at::empty({batch, rows, cols}, W.options()) : at::empty({rows, cols}, W.options());
  check_rc(stageml_lora_fold(W.data_ptr(), A.data_ptr(), B.data_ptr(), scale.data_ptr<float>(), (int)batch, (int)rows,
                             (int)cols, (int)rank, (int)layout, W.dim() == 3 ? rows * cols : 0,
                             batched ? A.stride(0) : 0, batched ? B.stride(0) : 0, dtype_code(W), out.data_ptr(),
                             cur_stream()),
           "lora_fold");
  return out;
}

Tensor lora_linear(const Tensor& x, const Tensor& w_bank, const c10::optional<Tensor>& bias,
                   const c10::optional<Tensor>& row_group, const c10::optional<Tensor>& row_tenant, int64_t n_tenants,
                   int64_t rank, const c10::optional<Tensor>& lora_a, const c10::optional<Tensor>& lora_b,
                   const c10::optional<Tensor>& lora_scale) {
  check_cuda(x, "x", x);
  check_cuda(w_bank, "w_bank", x);
  TORCH_CHECK(x.dim() == 2 && w_bank.dim() == 3 && w_bank.size(2) == x.size(1), "lora_linear: shapes");
  TORCH_CHECK(w_bank.scalar_type() == x.scalar_type(), "lora_linear: dtype mismatch");
  for (const auto* o : {&bias, &row_group, &row_tenant, &lora_a, &lora_b, &lora_scale})
    if (o->has_value()) check_cuda(**o, "optional input", x);
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t M = x.size(0), K = x.size(1), N = w_bank.size(1);
  auto y = at::empty({M, N}, x.options());
  stageml_lora_linear_args a{};
  a.M = (int)M;
  a.K = (int)K;
  a.N = (int)N;
  a.dtype = dtype_code(x);
  a.x = x.data_ptr();
  a.w_bank = w_bank.data_ptr();
  a.n_groups = (int)w_bank.size(0);
  a.bias = opt_ptr(bias);
  a.row_group = static_cast<const int32_t*>(opt_ptr(row_group));
  a.row_tenant = static_cast<const int32_t*>(opt_ptr(row_tenant));
  a.n_tenants = (int)n_tenants;
  a.rank = (int)rank;
  a.lora_a = opt_ptr(lora_a);
  a.lora_b = opt_ptr(lora_b);
  a.lora_scale = static_cast<const float*>(opt_ptr(lora_scale));
  a.y = y.data_ptr();
  a.status = status_word(x);
  auto w = workspace(stageml_lora_linear_workspace_bytes(&a), x);
  check_rc(stageml_lora_linear(&a, w.data_ptr(), (size_t)w.numel(), cur_stream()), "lora_linear");
  return y;
}

Tensor moe_linear(const Tensor& x, const Tensor& weight, const c10::optional<Tensor>& bias, const Tensor& topk_ids,
                  const Tensor& topk_weights, const c10::optional<Tensor>& tenant_ids, int64_t n_experts,
                  bool group_by_tenant, int64_t n_tenants, int64_t rank, const c10::optional<Tensor>& lora_a,
                  const c10::optional<Tensor>& lora_b, const c10::optional<Tensor>& lora_scale) {
  check_cuda(x, "x", x);
  check_cuda(weight, "weight", x);
  check_cuda(topk_ids, "topk_ids", x);
  check_cuda(topk_weights, "topk_weights", x);
  for (const auto* o : {&bias, &tenant_ids, &lora_a, &lora_b, &lora_scale})
    if (o->has_value()) check_cuda(**o, "optional input", x);
  TORCH_CHECK(weight.dim() == 3 && weight.size(2) == x.size(1), "moe_linear: weight [G, N, K]");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), K = x.size(1), N = weight.size(1);
  auto out = at::empty({T, N}, x.options());
  const int k = (int)topk_ids.size(1);
  const size_t ws = stageml_moe_linear_workspace_bytes((int)T, (int)K, (int)N, (int)n_experts, k, group_by_tenant ? 1 : 0,
                                                       (int)n_tenants, (int)rank);
  auto w = workspace(ws, x);
  check_rc(stageml_moe_linear(x.data_ptr(), weight.data_ptr(), opt_ptr(bias), topk_ids.data_ptr(), dtype_code(topk_ids),
                              topk_weights.data_ptr(), dtype_code(topk_weights),
                              static_cast<const int32_t*>(opt_ptr(tenant_ids)), (int)T, (int)K, (int)N, (int)n_experts,
                              k, group_by_tenant ? 1 : 0, (int)n_tenants, (int)rank, opt_ptr(lora_a), opt_ptr(lora_b),
                              static_cast<const float*>(opt_ptr(lora_scale)), dtype_code(x), out.data_ptr(),
                              status_word(x), w.data_ptr(), (size_t)w.numel(), cur_stream()),
           "moe_linear");
  return out;
}

Tensor lora_gemv_f32(const Tensor& x, const Tensor& W, const c10::optional<Tensor>& A, const c10::optional<Tensor>& B,
                     double scale) {
  check_cuda(x, "x", x);
  check_cuda(W, "W", x);
  TORCH_CHECK(x.scalar_type() == at::kFloat && W.scalar_type() == at::kFloat, "lora_gemv_f32: fp32 only");
  TORCH_CHECK(x.dim() == 2 && W.dim() == 2 && W.size(0) == x.size(1), "lora_gemv_f32: x [M,in], W [in,out]");
  const int64_t M = x.size(0), in_f = x.size(1), out_f = W.size(1);
  int64_t rank = 0;
  if (A.has_value()) {
    check_cuda(*A, "A", x);
    TORCH_CHECK(B.has_value(), "lora_gemv_f32: A without B");
    check_cuda(*B, "B", x);
    rank = A->size(1);
    TORCH_CHECK(A->size(0) == in_f && B->size(0) == rank && B->size(1) == out_f, "lora_gemv_f32: A [in,r], B [r,out]");
  }
  c10::cuda::CUDAGuard guard(x.device());
  auto y = at::empty({M, out_f}, x.options());
  auto w = workspace(stageml_lora_gemv_f32_workspace_bytes((int)M, (int)in_f, (int)out_f, (int)rank), x);
  check_rc(stageml_lora_gemv_f32(x.data_ptr<float>(), W.data_ptr<float>(),
                                 A.has_value() ? A->data_ptr<float>() : nullptr,
                                 B.has_value() ? B->data_ptr<float>() : nullptr, (float)scale, (int)M, (int)in_f,
                                 (int)out_f, (int)rank, y.data_ptr<float>(), w.data_ptr(), (size_t)w.numel(),
                                 cur_stream()),
           "lora_gemv_f32");
  return y;
}

std::tuple<Tensor, Tensor> quantize_e4m3_rows(const Tensor& w) {
  check_cuda(w, "w", w);
  TORCH_CHECK(w.dim() >= 1, "quantize_e4m3_rows: need at least one dim");
  c10::cuda::CUDAGuard guard(w.device());
  const int64_t cols = w.size(-1), rows = w.numel() / std::max<int64_t>(cols, 1);
  auto q = at::empty(w.sizes(), w.options().dtype(at::kFloat8_e4m3fn));
  auto sizes = w.sizes().vec();
  sizes.pop_back();
  auto s = at::empty(sizes, w.options().dtype(at::kFloat));
  check_rc(stageml_quantize_e4m3_rows(w.data_ptr(), dtype_code(w), rows, cols, static_cast<uint8_t*>(q.data_ptr()),
                                      s.data_ptr<float>(), cur_stream()),
           "quantize_e4m3_rows");
  return {q, s};
}

Tensor combine_rows(const Tensor& y, const Tensor& pair_row, int64_t T, int64_t kk) {
  check_cuda(y, "y", y);
  check_cuda(pair_row, "pair_row", y);
  TORCH_CHECK(y.dim() == 2 && pair_row.scalar_type() == at::kInt && pair_row.numel() >= T * kk,
              "combine_rows: y [rows, H], pair_row int32 [T*kk]");
  c10::cuda::CUDAGuard guard(y.device());
  auto out = at::empty({T, y.size(1)}, y.options());
  check_rc(stageml_combine_rows(y.data_ptr(), pair_row.data_ptr<int32_t>(), (int)T, (int)kk, (int)y.size(1),
                                dtype_code(y), out.data_ptr(), cur_stream()),
           "combine_rows");
  return out;
}

// Returns the device status word (synchronising on it) and clears it.
int64_t take_status(const Tensor& like) {
  c10::cuda::CUDAGuard guard(like.device());
  int32_t* p = status_word(like);
  auto t = at::from_blob(p, {1}, like.options().dtype(at::kInt));
  const int64_t v = t.item<int32_t>();
  t.zero_();
  return v;
}

}  // namespace

TORCH_LIBRARY(stageml, m) {
  m.def("residual_moe(Tensor hidden, Tensor gate_up, Tensor down, Tensor topk_weights, Tensor topk_ids) -> Tensor");
  m.def(
      "moe_forward(Tensor x, Tensor gate_up, Tensor down, Tensor? topk_weights, Tensor? topk_ids, Tensor? router_w, "
      "int k, int n_shared, bool renormalize, Tensor? tenant_ids, int n_tenants, int rank, Tensor? lora_a13, "
      "Tensor? lora_b13, Tensor? lora_a2, Tensor? lora_b2, Tensor? lora_scale, Tensor? gate_up_scale, "
      "Tensor? down_scale, Tensor? T_dev=None, Tensor? fold_slot=None, int n_fold=0, Tensor? down_group=None) "
      "-> Tensor");
  m.def("route_topk(Tensor x, Tensor gate_w, int k, bool renormalize) -> (Tensor, Tensor, Tensor)");
  m.def("topk_from_logits(Tensor logits, int k, bool renormalize) -> (Tensor, Tensor)");
  m.def(
      "permute(Tensor ids, Tensor? weights, Tensor? tenant_ids, int n_experts_total, int n_shared, int n_tenants, "
      "bool group_by_tenant) -> Tensor[]");
  m.def("lora_fold(Tensor W, Tensor A, Tensor B, Tensor scale, int layout) -> Tensor");
  m.def(
      "lora_linear(Tensor x, Tensor w_bank, Tensor? bias, Tensor? row_group, Tensor? row_tenant, int n_tenants, "
      "int rank, Tensor? lora_a, Tensor? lora_b, Tensor? lora_scale) -> Tensor");
  m.def(
      "moe_linear(Tensor x, Tensor weight, Tensor? bias, Tensor topk_ids, Tensor topk_weights, Tensor? tenant_ids, "
      "int n_experts, bool group_by_tenant, int n_tenants, int rank, Tensor? lora_a, Tensor? lora_b, "
      "Tensor? lora_scale) -> Tensor");
  m.def("lora_gemv_f32(Tensor x, Tensor W, Tensor? A, Tensor? B, float scale) -> Tensor");
  m.def("quantize_e4m3_rows(Tensor w) -> (Tensor, Tensor)");
  m.def("combine_rows(Tensor y, Tensor pair_row, int T, int kk) -> Tensor");
  m.def("take_status(Tensor like) -> int");
}

TORCH_LIBRARY_IMPL(stageml, CUDA, m) {
  m.impl("residual_moe", &residual_moe);
  m.impl("moe_forward", &moe_forward);
  m.impl("route_topk", &route_topk);
  m.impl("topk_from_logits", &topk_from_logits);
  m.impl("permute", &permute);
  m.impl("lora_fold", &lora_fold);
  m.impl("lora_linear", &lora_linear);
  m.impl("moe_linear", &moe_linear);
  m.impl("lora_gemv_f32", &lora_gemv_f32);
  m.impl("quantize_e4m3_rows", &quantize_e4m3_rows);
  m.impl("combine_rows", &combine_rows);
  m.impl("take_status", &take_status);
}
