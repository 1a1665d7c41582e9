// Router (R1): logits = float(x) . G^T in fp32, softmax over experts, top-k,
// optional renormalisation. Restates make_routing
// (benchmarks/real_moe_lora_residual_bench.py:360-386) and
// normalize_routing_weights (stageml/moe_lora_layers.py:178-183) on the GPU.
//
// Logits: one CTA per 32 tokens; x and G are staged through shared memory in
// 64-wide K chunks so each G element is read once per 32 tokens; each thread
// accumulates a (token, expert) register block with fp32 FMAs.
// Top-k: one warp per token, lane j owns experts j, j+32, ...; k rounds of a
// warp arg-max (larger logit first, ties -> lower expert index).
#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace sb {
namespace {

constexpr int RT_TOK = 32;     // tokens per CTA
constexpr int RT_KC = 64;      // K chunk
constexpr int RT_THREADS = 256;

template <typename T>
__global__ void __launch_bounds__(RT_THREADS) router_logits_kernel(const T* __restrict__ x,
                                                                   const float* __restrict__ gw, int T_, int H,
                                                                   int E, float* __restrict__ logits) {
  extern __shared__ float rsm[];
  float* xs = rsm;                      // [RT_TOK][RT_KC + 1]
  float* gs = rsm + RT_TOK * (RT_KC + 1);  // [E][RT_KC + 1]
  const int t0 = blockIdx.x * RT_TOK;
  const int ntok = min(RT_TOK, T_ - t0);
  // Thread block of outputs: token index tt = threadIdx.x % 32, experts e = threadIdx.x/32 + 8*i.
  const int tt = threadIdx.x & 31;
  const int e0 = threadIdx.x >> 5;      // 0..7
  constexpr int MAXE = 256;
  float acc[MAXE / 8];
#pragma unroll
  for (int i = 0; i < MAXE / 8; ++i) acc[i] = 0.f;

  for (int k0 = 0; k0 < H; k0 += RT_KC) {
    const int kc = min(RT_KC, H - k0);
    for (int i = threadIdx.x; i < RT_TOK * RT_KC; i += RT_THREADS) {
      const int r = i / RT_KC, c = i % RT_KC;
      xs[r * (RT_KC + 1) + c] = (r < ntok && c < kc) ? to_f32<T>(x[(int64_t)(t0 + r) * H + k0 + c]) : 0.f;
    }
    for (int i = threadIdx.x; i < E * RT_KC; i += RT_THREADS) {
      const int r = i / RT_KC, c = i % RT_KC;
      gs[r * (RT_KC + 1) + c] = (c < kc) ? gw[(int64_t)r * H + k0 + c] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < MAXE / 8; ++i) {
      const int e = e0 + 8 * i;
      if (e < E) {
        float a = acc[i];
        const float* xr = xs + tt * (RT_KC + 1);
        const float* gr = gs + e * (RT_KC + 1);
#pragma unroll 16
        for (int c = 0; c < RT_KC; ++c) a = fmaf(xr[c], gr[c], a);
        acc[i] = a;
      }
    }
    __syncthreads();
  }
  if (tt < ntok) {
#pragma unroll
    for (int i = 0; i < MAXE / 8; ++i) {
      const int e = e0 + 8 * i;
      if (e < E) logits[(int64_t)(t0 + tt) * E + e] = acc[i];
    }
  }
}

// Gate resident in shared memory (E*H fp32 <= 200 KB): each CTA copies G once,
// then every warp takes whole tokens; lane l accumulates E partial dot products
// over columns 4l + 128i with float4 reads of G and 8-byte reads of x, and the
// warp reduces them with shuffles. E <= 32.
template <typename T, int E_MAX>
__global__ void __launch_bounds__(256) router_logits_smem_kernel(const T* __restrict__ x, const float* __restrict__ gw,
                                                                 int T_, int H, int E, float* __restrict__ logits) {
  extern __shared__ float4 gsm4[];
  float* gsm = reinterpret_cast<float*>(gsm4);
  const int n = E * H;
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
    *reinterpret_cast<float4*>(gsm + i) = __ldg(reinterpret_cast<const float4*>(gw + i));
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int t = blockIdx.x * wpb + warp; t < T_; t += gridDim.x * wpb) {
    const T* xr = x + (int64_t)t * H;
    float acc[E_MAX];
#pragma unroll
    for (int e = 0; e < E_MAX; ++e) acc[e] = 0.f;
    for (int h = lane * 4; h < H; h += 128) {
      float xv[4];
      if (sizeof(T) == 2) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(xr + h));
        const T* hv = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int q = 0; q < 4; ++q) xv[q] = to_f32<T>(hv[q]);
      } else {
        const float4 f = __ldg(reinterpret_cast<const float4*>(xr + h));
        xv[0] = f.x, xv[1] = f.y, xv[2] = f.z, xv[3] = f.w;
      }
#pragma unroll
      for (int e = 0; e < E_MAX; ++e) {
        if (e < E) {
          const float4 gv = *reinterpret_cast<const float4*>(gsm + e * H + h);
          acc[e] = fmaf(xv[0], gv.x, acc[e]);
          acc[e] = fmaf(xv[1], gv.y, acc[e]);
          acc[e] = fmaf(xv[2], gv.z, acc[e]);
          acc[e] = fmaf(xv[3], gv.w, acc[e]);
        }
      }
    }
#pragma unroll
    for (int e = 0; e < E_MAX; ++e) {
      if (e < E) {
        float v = acc[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) logits[(int64_t)t * E + e] = v;
      }
    }
  }
}

// One warp per token.
__global__ void topk_kernel(const float* __restrict__ logits, int T_, int E, int k, int renorm,
                            int32_t* __restrict__ ids, float* __restrict__ weights) {
  const int warps_per_block = blockDim.x >> 5;
  const int t = blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T_) return;
  constexpr int PER = 8;  // E <= 256
  float v[PER];
  const float* lrow = logits + (int64_t)t * E;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    v[i] = (e < E) ? lrow[e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    if (e < E) sum += expf(v[i] - mx);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);

  float sel_w[8];
  int sel_e[8];
  bool taken[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) taken[i] = false;
  for (int r = 0; r < k; ++r) {
    // local best: larger value first, ties -> lower expert index
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !taken[i] && (v[i] > bv || (v[i] == bv && e < be))) {
        bv = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == be) taken[i] = true;
    sel_e[r] = be;
    sel_w[r] = expf(bv - mx) / sum;
  }
  if (lane == 0) {
    float wsum = 0.f;
    for (int r = 0; r < k; ++r) wsum += sel_w[r];
    const float denom = fmaxf(wsum, 1e-12f);
    for (int r = 0; r < k; ++r) {
      ids[(int64_t)t * k + r] = sel_e[r];
      weights[(int64_t)t * k + r] = renorm ? sel_w[r] / denom : sel_w[r];
    }
  }
}

}  // namespace

int launch_topk(const float* logits, int T_, int E, int k, int renorm, int32_t* ids, float* weights,
                cudaStream_t stream) {
  SB_CHECK_ARG(E >= 1 && E <= 256, "top-k: E=%d must be in [1, 256]", E);
  SB_CHECK_ARG(k >= 1 && k <= 8 && k <= E, "top-k: k=%d must be in [1, min(8, E)]", k);
  if (T_ == 0) return STAGEML_OK;
  SB_CHECK_ARG(logits && ids && weights, "top-k: null pointer");
  const int wpb = 8;
  (topk_kernel<<<(T_ + wpb - 1) / wpb, wpb * 32, 0, stream>>>(logits, T_, E, k, renorm, ids, weights), ::sb::count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

int launch_router_logits(const void* x, int x_dtype, const float* gate_w, int T_, int H, int E, float* logits,
                         cudaStream_t stream) {
  SB_CHECK_ARG(E >= 1 && E <= 256, "router: E=%d must be in [1, 256]", E);
  SB_CHECK_ARG(H >= 1, "router: H must be positive");
  if (T_ == 0) return STAGEML_OK;
  SB_CHECK_ARG(x && gate_w && logits, "router: null pointer");
  const size_t gbytes = sizeof(float) * (size_t)E * H;
  const bool aligned = (reinterpret_cast<uintptr_t>(gate_w) % 16 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  if (E <= 32 && H % 4 == 0 && gbytes <= 200 * 1024 && aligned &&
      (x_dtype == STAGEML_BF16 || x_dtype == STAGEML_F16 || x_dtype == STAGEML_F32)) {
    const int grid = std::min<int>(sm_count(), (T_ + 7) / 8);
    auto launch = [&](auto kern, const auto* xp) -> int {
      SB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gbytes));
      (kern<<<grid, 256, gbytes, stream>>>(xp, gate_w, T_, H, E, logits), ::sb::count_launch());
      SB_CUDA_CHECK(cudaGetLastError());
      return STAGEML_OK;
    };
    if (x_dtype == STAGEML_BF16) {
      const bf16* xp = static_cast<const bf16*>(x);
      if (E <= 8) return launch(router_logits_smem_kernel<bf16, 8>, xp);
      if (E <= 16) return launch(router_logits_smem_kernel<bf16, 16>, xp);
      return launch(router_logits_smem_kernel<bf16, 32>, xp);
    }
    if (x_dtype == STAGEML_F16) {
      const f16* xp = static_cast<const f16*>(x);
      if (E <= 8) return launch(router_logits_smem_kernel<f16, 8>, xp);
      if (E <= 16) return launch(router_logits_smem_kernel<f16, 16>, xp);
      return launch(router_logits_smem_kernel<f16, 32>, xp);
    }
    const float* xp = static_cast<const float*>(x);
    if (E <= 8) return launch(router_logits_smem_kernel<float, 8>, xp);
    if (E <= 16) return launch(router_logits_smem_kernel<float, 16>, xp);
    return launch(router_logits_smem_kernel<float, 32>, xp);
  }
  const size_t smem = sizeof(float) * (size_t)(RT_TOK + E) * (RT_KC + 1);
  const int grid = (T_ + RT_TOK - 1) / RT_TOK;
  if (x_dtype == STAGEML_BF16) {
    SB_CUDA_CHECK(cudaFuncSetAttribute(router_logits_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    (router_logits_kernel<bf16><<<grid, RT_THREADS, smem, stream>>>(static_cast<const bf16*>(x), gate_w, T_, H, E,
                                                                    logits), ::sb::count_launch());
  } else if (x_dtype == STAGEML_F16) {
    SB_CUDA_CHECK(cudaFuncSetAttribute(router_logits_kernel<f16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    (router_logits_kernel<f16><<<grid, RT_THREADS, smem, stream>>>(static_cast<const f16*>(x), gate_w, T_, H, E,
                                                                   logits), ::sb::count_launch());
  } else if (x_dtype == STAGEML_F32) {
    SB_CUDA_CHECK(cudaFuncSetAttribute(router_logits_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    (router_logits_kernel<float><<<grid, RT_THREADS, smem, stream>>>(static_cast<const float*>(x), gate_w, T_, H,
                                                                     E, logits), ::sb::count_launch());
  } else {
    return set_error(STAGEML_ERR_INVALID_ARG, "router: unsupported x dtype %d", x_dtype);
  }
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

}  // namespace sb
