// Host-side launch description of the grouped tcgen05 GEMM (grouped_gemm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sb {

// out[row, n] = epilogue( sum_k A[row, k] * B[group(row) * b_group_rows + n, k] )
//
// A rows are either the padded permuted rows of a MoE plan (tile_group != nullptr:
// 128-row tile m belongs to group tile_group[m], the number of tiles is read from
// num_tiles_dev) or the rows of a plain matrix (tile_group == nullptr: group 0,
// rows >= m_rows are masked).
//
// SwiGLU mode: B group = [W1 (N rows); W3 (N rows)]; out = silu(g) * u with
//   g = acc(W1 rows) + lora(S[:, 0:r], lora_b rows [0,N)),
//   u = acc(W3 rows) + lora(S[:, r:2r], lora_b rows [N,2N)).
// Plain mode: out = (acc * b_scale + bias + lora(S[:, 0:r])) * row_scale.
struct GemmLaunch {
  const void* a = nullptr;       // [a_rows, K] 16-bit
  int64_t a_rows = 0;
  int K = 0;
  const void* b = nullptr;       // [b_rows_total, K] 16-bit
  int64_t b_rows_total = 0;
  int b_group_rows = 0;          // rows of B per group (N or 2N)
  int N = 0;                     // output columns
  bool swiglu = false;
  bool in_bf16 = true;           // false: fp16
  // tiles
  const int32_t* num_tiles_dev = nullptr;
  int tiles_cap = 0;
  const int32_t* tile_group = nullptr;
  int64_t m_rows = 0;            // direct mode row count
  // epilogue inputs
  const int32_t* row_tenant = nullptr;   // [rows] or null
  const float* row_lora = nullptr;       // [rows, lora_cols] pre-scaled shrink output
  int rank = 0;                          // multiple of 8, <= 32; 0 = no LoRA
  const void* lora_b = nullptr;          // 16-bit
  int64_t lora_b_tenant_stride = 0;      // elements
  int64_t lora_b_group_stride = 0;       // elements
  const float* row_scale = nullptr;      // [rows] or null
  const void* bias = nullptr;            // 16-bit [G, N] or null
  int64_t bias_group_stride = 0;
  int bias_group_mod = 0;                // bias group = group % mod when > 0
  const float* b_scale = nullptr;        // fp32 per B row or null
  void* out = nullptr;                   // [rows, ldo] 16-bit
  int64_t ldo = 0;
  int32_t* status = nullptr;
};

int launch_grouped_gemm(const GemmLaunch& g, cudaStream_t stream);

}  // namespace sb
