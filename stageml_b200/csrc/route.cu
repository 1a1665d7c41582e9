// Router (R1): logits = float(x) . G^T in fp32, softmax over experts, top-k,
// optional renormalisation. Restates make_routing
// (benchmarks/real_moe_lora_residual_bench.py:360-386) and
// normalize_routing_weights (stageml/moe_lora_layers.py:178-183) on the GPU.
//
// Logits: for E <= 32 with the gate fitting shared memory, each CTA keeps G
// resident and warps take whole tokens (a few tokens: one warp per (token,
// expert) reading G from L2, with the same per-lane sum order); more experts with
// bf16 tokens: tensor-core tiles on an exact three-way bf16 split of the fp32 gate;
// otherwise a register-blocked tiled kernel over (32 tokens x 64 experts) tiles.
// Top-k: one warp per token, lane j owns experts j, j+32, ...; k rounds of a
// warp arg-max (larger logit first, ties -> lower expert index).
#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

#include <type_traits>

namespace sb {
namespace {

constexpr int RT_TT = 32;      // tokens per CTA
constexpr int RT_TE = 64;      // experts per CTA
constexpr int RT_KC = 32;      // K chunk
constexpr int RT_PAD = RT_TE + 4;
constexpr int RT_THREADS = 128;

// General case (any E <= 256, gate too large for shared memory): a 32-token x
// 64-expert output tile per CTA; x and G are staged K-major through shared memory
// in 32-wide chunks (16-byte global loads when rows are 16-byte aligned) and each
// thread accumulates a 4 x 4 (token, expert) register block, 16 FMAs per two
// 16-byte shared-memory reads.
// Loader of one K chunk: x 32 tokens x 32 K (8 values per thread), G 64 experts x 32 K
// (16 values per thread), 16-byte global loads when VEC.
template <typename T, bool VEC>
__device__ __forceinline__ void router_chunk_load(const T* __restrict__ x, const float* __restrict__ gw, int T_, int H,
                                                  int E, int t0, int e0, int k0, float (&vx)[8], float (&vg)[2][8]) {
  const int tid = threadIdx.x;
  const int r = tid >> 2, kk = (tid & 3) * 8;
  {
    const int t = t0 + r, k = k0 + kk;
    if (VEC && t < T_ && k + 8 <= H) {
      if (sizeof(T) == 2) {
        unpack8<T>(__ldg(reinterpret_cast<const uint4*>(x + (int64_t)t * H + k)), vx);
      } else {
        const float4 a = __ldg(reinterpret_cast<const float4*>(x + (int64_t)t * H + k));
        const float4 b = __ldg(reinterpret_cast<const float4*>(x + (int64_t)t * H + k + 4));
        vx[0] = a.x, vx[1] = a.y, vx[2] = a.z, vx[3] = a.w, vx[4] = b.x, vx[5] = b.y, vx[6] = b.z, vx[7] = b.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) vx[q] = (t < T_ && k + q < H) ? to_f32<T>(x[(int64_t)t * H + k + q]) : 0.f;
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int e = e0 + r + 32 * h, k = k0 + kk;
    if (VEC && e < E && k + 8 <= H) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(gw + (int64_t)e * H + k));
      const float4 b = __ldg(reinterpret_cast<const float4*>(gw + (int64_t)e * H + k + 4));
      vg[h][0] = a.x, vg[h][1] = a.y, vg[h][2] = a.z, vg[h][3] = a.w;
      vg[h][4] = b.x, vg[h][5] = b.y, vg[h][6] = b.z, vg[h][7] = b.w;
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) vg[h][q] = (e < E && k + q < H) ? gw[(int64_t)e * H + k + q] : 0.f;
    }
  }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(RT_THREADS) router_logits_kernel(const T* __restrict__ x,
                                                                   const float* __restrict__ gw, int T_, int H,
                                                                   int E, float* __restrict__ logits) {
  __shared__ __align__(16) float xs[2][RT_KC][RT_PAD];
  __shared__ __align__(16) float gs[2][RT_KC][RT_PAD];
  const int t0 = blockIdx.x * RT_TT, e0 = blockIdx.y * RT_TE;
  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;  // tokens ty*4.., experts tx*4..
  const int r = tid >> 2, kk = (tid & 3) * 8;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  float vx[8], vg[2][8];
  router_chunk_load<T, VEC>(x, gw, T_, H, E, t0, e0, 0, vx, vg);
  int buf = 0;
  for (int k0 = 0; k0 < H; k0 += RT_KC, buf ^= 1) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      xs[buf][kk + q][r] = vx[q];
      gs[buf][kk + q][r] = vg[0][q];
      gs[buf][kk + q][r + 32] = vg[1][q];
    }
    __syncthreads();
    // the next chunk's loads are in flight while this one is multiplied
    if (k0 + RT_KC < H) router_chunk_load<T, VEC>(x, gw, T_, H, E, t0, e0, k0 + RT_KC, vx, vg);
#pragma unroll 8
    for (int k = 0; k < RT_KC; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(&xs[buf][k][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&gs[buf][k][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= T_) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + tx * 4 + j;
      if (e < E) logits[(int64_t)t * E + e] = acc[i][j];
    }
  }
}

// More than 32 experts with bf16 tokens: the same fp32 dot products on the tensor
// cores. Each fp32 gate value is split exactly into three bf16 parts (g = hi + mid +
// lo: 8 + 8 + 8 significant bits), so x . g = x . hi + x . mid + x . lo with every
// product exact and fp32 accumulation (mma.sync m16n8k16; per 16-wide K step the
// three parts in that order, K steps in order). CTA tile: 64 tokens x 32 experts, 4
// warps of 16 tokens. x and the fp32 gate arrive in 64-wide K chunks through a
// 4-stage cp.async ring (three chunks in flight while one is used); the CTA splits
// each gate chunk into its three bf16 planes in shared memory. A token's sums do
// not depend on the other tokens of the batch.
constexpr int RTC_TT = 64, RTC_TE = 32, RTC_KC = 64, RTC_STAGES = 4;
constexpr int RTC_XP = RTC_KC + 8;  // x row pitch in bf16 (144 B: ldmatrix rows in distinct banks)
constexpr int RTC_RP = RTC_KC + 4;  // raw gate row pitch in fp32 (272 B)
constexpr int RTC_GP = RTC_KC + 8;  // bf16 gate plane row pitch
constexpr int RTC_X_BYTES = RTC_STAGES * RTC_TT * RTC_XP * 2;
constexpr int RTC_R_BYTES = RTC_STAGES * RTC_TE * RTC_RP * 4;
constexpr int RTC_G_BYTES = 3 * RTC_TE * RTC_GP * 2;
constexpr int RTC_SMEM = RTC_X_BYTES + RTC_R_BYTES + RTC_G_BYTES;

__device__ __forceinline__ void rtc_ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void rtc_ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void rtc_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void rtc_cp16(uint32_t dst, const void* src, bool valid) {
  // src-size 0 fills the 16 bytes with zeros (tokens / experts / columns past the end)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}

__global__ void __launch_bounds__(128) router_logits_tc_kernel(const bf16* __restrict__ x, const float* __restrict__ gw,
                                                               int T_, int H, int E, float* __restrict__ logits) {
  extern __shared__ __align__(16) uint8_t rtc_smem[];
  bf16* xs = reinterpret_cast<bf16*>(rtc_smem);                                   // [S][TT][XP]
  float* graw = reinterpret_cast<float*>(rtc_smem + RTC_X_BYTES);                 // [S][TE][RP]
  bf16* gs = reinterpret_cast<bf16*>(rtc_smem + RTC_X_BYTES + RTC_R_BYTES);       // [3][TE][GP]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * RTC_TT, e0 = blockIdx.y * RTC_TE;
  const int nchunks = (H + RTC_KC - 1) / RTC_KC;
  // one chunk: x 64 rows x 64 bf16 (512 16-byte pieces), gate 32 rows x 64 fp32 (512)
  auto issue = [&](int c) {
    if (c < nchunks) {
      const int slot = c % RTC_STAGES, k0 = c * RTC_KC;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = tid + 128 * i, r = idx >> 3, q = (idx & 7) * 8;
        const int t = t0 + r;
        const bool v = t < T_ && k0 + q < H;
        rtc_cp16(smem_u32(xs + ((size_t)slot * RTC_TT + r) * RTC_XP + q), v ? x + (int64_t)t * H + k0 + q : x, v);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = tid + 128 * i, r = idx >> 4, q = (idx & 15) * 4;
        const int e = e0 + r;
        const bool v = e < E && k0 + q < H;
        rtc_cp16(smem_u32(graw + ((size_t)slot * RTC_TE + r) * RTC_RP + q), v ? gw + (int64_t)e * H + k0 + q : gw, v);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");  // empty groups keep the count uniform
  };
  float acc[RTC_TE / 8][4];
#pragma unroll
  for (int nb = 0; nb < RTC_TE / 8; ++nb)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[nb][j] = 0.f;
#pragma unroll
  for (int c = 0; c < RTC_STAGES - 1; ++c) issue(c);
  for (int c = 0; c < nchunks; ++c) {
    const int slot = c % RTC_STAGES;
    asm volatile("cp.async.wait_group %0;" ::"n"(RTC_STAGES - 2) : "memory");
    __syncthreads();  // chunk c landed for every thread; chunk c - 1's MMAs are done
    issue(c + RTC_STAGES - 1);
    // split this chunk's gate values into the three bf16 planes
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + 128 * i, r = idx >> 4, q = (idx & 15) * 4;
      const float4 g4 = *reinterpret_cast<const float4*>(graw + ((size_t)slot * RTC_TE + r) * RTC_RP + q);
      const float g[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bf16 hi = __float2bfloat16_rn(g[j]);
        const float r1 = g[j] - __bfloat162float(hi);
        const bf16 mid = __float2bfloat16_rn(r1);
        const bf16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
        gs[(0 * RTC_TE + r) * RTC_GP + q + j] = hi;
        gs[(1 * RTC_TE + r) * RTC_GP + q + j] = mid;
        gs[(2 * RTC_TE + r) * RTC_GP + q + j] = lo;
      }
    }
    __syncthreads();
    const bf16* xsl = xs + (size_t)slot * RTC_TT * RTC_XP;
#pragma unroll
    for (int k16 = 0; k16 < RTC_KC / 16; ++k16) {
      uint32_t a0, a1, a2, a3;
      rtc_ldsm_x4(smem_u32(xsl + (warp * 16 + (lane & 15)) * RTC_XP + k16 * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
      for (int nb = 0; nb < RTC_TE / 8; ++nb) {
#pragma unroll
        for (int part = 0; part < 3; ++part) {
          uint32_t b0, b1;
          rtc_ldsm_x2(smem_u32(gs + (part * RTC_TE + nb * 8 + (lane & 7)) * RTC_GP + k16 * 16 + ((lane >> 3) & 1) * 8),
                      b0, b1);
          rtc_mma(acc[nb], a0, a1, a2, a3, b0, b1);
        }
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  const int g = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int nb = 0; nb < RTC_TE / 8; ++nb) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = t0 + warp * 16 + g + (j >= 2 ? 8 : 0);
      const int e = e0 + nb * 8 + tig * 2 + (j & 1);
      if (t < T_ && e < E) logits[(int64_t)t * E + e] = acc[nb][j];
    }
  }
}

// Four consecutive values of an x row as fp32 (zeros past the end).
template <typename T>
__device__ __forceinline__ void load_x4(const T* xr, int h, int H, float (&xv)[4]) {
  if (h >= H) {
    xv[0] = xv[1] = xv[2] = xv[3] = 0.f;
  } else if (sizeof(T) == 2) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(xr + h));
    const T* hv = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int q = 0; q < 4; ++q) xv[q] = to_f32<T>(hv[q]);
  } else {
    const float4 f = __ldg(reinterpret_cast<const float4*>(xr + h));
    xv[0] = f.x, xv[1] = f.y, xv[2] = f.z, xv[3] = f.w;
  }
}
constexpr int RT_XU = 8;

// Bulk-copies `a_bytes` from `a` (and `b_bytes` from `b`) into shared memory at
// `dst` (b right after a), all in flight at once; every thread of the CTA returns
// once they landed (false if the bounded wait gave up). Sizes and addresses are
// multiples of 16 bytes.
__device__ __forceinline__ bool stage_to_smem(uint32_t dst, const void* a, uint32_t a_bytes, const void* b,
                                              uint32_t b_bytes, uint64_t* bar, volatile int* abort_flag) {
  constexpr uint32_t kChunk = 16384;
  const uint32_t mb = smem_u32(bar);
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(mb, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(mb, a_bytes + b_bytes);
    for (uint32_t off = 0; off < a_bytes; off += kChunk)
      bulk_load_1d(dst + off, static_cast<const char*>(a) + off, min(kChunk, a_bytes - off), mb);
    for (uint32_t off = 0; off < b_bytes; off += kChunk)
      bulk_load_1d(dst + a_bytes + off, static_cast<const char*>(b) + off, min(kChunk, b_bytes - off), mb);
  }
  return mbar_wait(mb, 0, abort_flag, nullptr, kDefaultWaitNs, 0);
}

// Gate resident in shared memory (E*H fp32 <= 200 KB): each CTA bulk-copies G once,
// then every warp takes whole tokens; lane l accumulates E partial dot products
// over columns 4l + 128i with float4 reads of G and 8-byte reads of x, and the
// warp reduces them with shuffles. E <= 32.
template <typename T, int E_MAX>
__global__ void __launch_bounds__(256) router_logits_smem_kernel(const T* __restrict__ x, const float* __restrict__ gw,
                                                                 int T_, int H, int E, float* __restrict__ logits) {
  extern __shared__ float4 gsm4[];
  float* gsm = reinterpret_cast<float*>(gsm4);
  __shared__ uint64_t bar;
  __shared__ volatile int abort_flag;
  const bool staged = stage_to_smem(smem_u32(gsm), gw, (uint32_t)(sizeof(float) * E * H), nullptr, 0, &bar, &abort_flag);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int t = blockIdx.x * wpb + warp; t < T_; t += gridDim.x * wpb) {
    const T* xr = x + (int64_t)t * H;
    float acc[E_MAX];
#pragma unroll
    for (int e = 0; e < E_MAX; ++e) acc[e] = 0.f;
    // 8 steps of x loaded ahead of their FMAs (the per-lane order of the sums is unchanged)
    for (int h0 = lane * 4; h0 < H; h0 += 128 * RT_XU) {
      float xv[RT_XU][4];
#pragma unroll
      for (int u = 0; u < RT_XU; ++u) load_x4<T>(xr, h0 + 128 * u, H, xv[u]);
#pragma unroll
      for (int u = 0; u < RT_XU; ++u) {
        const int h = h0 + 128 * u;
        if (h < H) {
#pragma unroll
          for (int e = 0; e < E_MAX; ++e) {
            if (e < E) {
              const float4 gv = *reinterpret_cast<const float4*>(gsm + e * H + h);
              acc[e] = fmaf(xv[u][0], gv.x, acc[e]);
              acc[e] = fmaf(xv[u][1], gv.y, acc[e]);
              acc[e] = fmaf(xv[u][2], gv.z, acc[e]);
              acc[e] = fmaf(xv[u][3], gv.w, acc[e]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int e = 0; e < E_MAX; ++e) {
      if (e < E) {
        float v = acc[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) logits[(int64_t)t * E + e] = staged ? v : __int_as_float(0x7fc00000);
      }
    }
  }
}

// Softmax over one token's E logits, top-k (ties -> lower expert index) and the
// optional renormalisation of the k weights; one warp, results written by lane 0.
// PER = logits per lane (E <= 32 * PER); any PER that covers E gives the same bits (the
// extra slots add exact zeros to the sum and never win a round).
template <int PER>
__device__ __forceinline__ void topk_row(const float* lrow, int E, int k, int renorm, int lane,
                                         int32_t* __restrict__ ids_row, float* __restrict__ w_row) {
  float v[PER];
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
      ids_row[r] = sel_e[r];
      w_row[r] = renorm ? sel_w[r] / denom : sel_w[r];
    }
  }
}

// One warp per token.
template <int PER>
__global__ void topk_kernel(const float* __restrict__ logits, int T_, int E, int k, int renorm,
                            int32_t* __restrict__ ids, float* __restrict__ weights) {
  const int warps_per_block = blockDim.x >> 5;
  const int t = blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T_) return;
  topk_row<PER>(logits + (int64_t)t * E, E, k, renorm, lane, ids + (int64_t)t * k, weights + (int64_t)t * k);
}

constexpr int kRouteSmallT = 8;    // tokens per CTA of router_small_kernel
constexpr int kRouteSmallMaxT = 64;

// Up to 8 tokens per CTA: G and the CTA's token rows arrive in shared memory by
// bulk copies, and warp w takes the (token, expert) dot products w, w + 8, ...; each
// lane's sum over columns 4l + 128i and the shuffle reduction are those of
// router_logits_smem_kernel, so both kernels give the same logits for a token.
// The top-k of topk_kernel follows in the same CTA.
template <typename T>
__global__ void __launch_bounds__(256) router_small_kernel(const T* __restrict__ x, const float* __restrict__ gw,
                                                           int T_, int H, int E, int k, int renorm,
                                                           float* __restrict__ logits, int32_t* __restrict__ ids,
                                                           float* __restrict__ weights) {
  extern __shared__ float4 sm4[];
  float* gsm = reinterpret_cast<float*>(sm4);                   // [E, H]
  const T* xsm = reinterpret_cast<const T*>(gsm + (size_t)E * H);  // [T_, H]
  __shared__ uint64_t bar;
  __shared__ volatile int abort_flag;
  __shared__ float lsm[kRouteSmallT * 32];
  pdl_wait();  // x may come from the previous kernel
  pdl_trigger();
  const int t0 = blockIdx.x * kRouteSmallT;
  const int nt = min(kRouteSmallT, T_ - t0);
  const bool staged = stage_to_smem(smem_u32(gsm), gw, (uint32_t)(sizeof(float) * E * H), x + (size_t)t0 * H,
                                    (uint32_t)(sizeof(T) * nt * H), &bar, &abort_flag);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  logits += (int64_t)t0 * E;
  ids += (int64_t)t0 * k;
  weights += (int64_t)t0 * k;
  for (int u = warp; u < nt * E; u += 8) {
    const int t = u / E, e = u - t * E;
    const T* xr = xsm + (size_t)t * H;
    const float* gr = gsm + (size_t)e * H;
    float acc = 0.f;
    for (int h = lane * 4; h < H; h += 128) {
      float xv[4];
      if (sizeof(T) == 2) {
        const uint2 w = *reinterpret_cast<const uint2*>(xr + h);
        const T* hv = reinterpret_cast<const T*>(&w);
#pragma unroll
        for (int q = 0; q < 4; ++q) xv[q] = to_f32<T>(hv[q]);
      } else {
        const float4 f = *reinterpret_cast<const float4*>(xr + h);
        xv[0] = f.x, xv[1] = f.y, xv[2] = f.z, xv[3] = f.w;
      }
      const float4 gv = *reinterpret_cast<const float4*>(gr + h);
      acc = fmaf(xv[0], gv.x, acc);
      acc = fmaf(xv[1], gv.y, acc);
      acc = fmaf(xv[2], gv.z, acc);
      acc = fmaf(xv[3], gv.w, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      const float v = staged ? acc : __int_as_float(0x7fc00000);
      lsm[u] = v;
      logits[(int64_t)t * E + e] = v;
    }
  }
  __syncthreads();
  for (int t = warp; t < nt; t += 8)
    topk_row<1>(lsm + t * E, E, k, renorm, lane, ids + (int64_t)t * k, weights + (int64_t)t * k);
}

// Logits + top-k in one kernel for E <= 32 with the gate resident in shared memory:
// as router_logits_smem_kernel, but each warp takes two tokens at a time (every G
// read from shared memory serves both) and runs topk_row on their logits right
// away. Each token's per-lane sums are those of router_logits_smem_kernel (same
// columns, same order), so the logits are the same bits. The token rows stream
// through registers in steps of 1024 columns, double-buffered: the loads of step
// s + 1 are in flight while step s is summed, and the first step's loads are issued
// before the wait for the staged gate.
template <typename T>
struct XChunk {
  using type = uint2;  // 4 x 16-bit
};
template <>
struct XChunk<float> {
  using type = float4;
};
template <typename T>
__device__ __forceinline__ typename XChunk<T>::type load_chunk(const T* xr, int h, int H) {
  using C = typename XChunk<T>::type;
  if (h >= H) return C{};
  return __ldg(reinterpret_cast<const C*>(xr + h));
}
template <typename T>
__device__ __forceinline__ void chunk_f32(const typename XChunk<T>::type& c, float (&v)[4]) {
  if constexpr (sizeof(T) == 2) {
    const T* hv = reinterpret_cast<const T*>(&c);
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = to_f32<T>(hv[q]);
  } else {
    v[0] = c.x, v[1] = c.y, v[2] = c.z, v[3] = c.w;
  }
}

constexpr int RT_TPW = 2;
template <typename T, int E_MAX>
__global__ void __launch_bounds__(256) router_route_smem_kernel(const T* __restrict__ x, const float* __restrict__ gw,
                                                                int T_, int H, int E, int k, int renorm,
                                                                float* __restrict__ logits, int32_t* __restrict__ ids,
                                                                float* __restrict__ weights) {
  constexpr int XU = 8;  // 4-column chunks per lane and step: 1024 columns per step
  using C = typename XChunk<T>::type;
  extern __shared__ float4 gsm4[];
  float* gsm = reinterpret_cast<float*>(gsm4);
  __shared__ uint64_t bar;
  __shared__ volatile int abort_flag;
  __shared__ float lsm[8][RT_TPW][E_MAX];
  const uint32_t mb = smem_u32(&bar);
  const uint32_t gbytes = (uint32_t)(sizeof(float) * E * H);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(mb, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(mb, gbytes);
    for (uint32_t off = 0; off < gbytes; off += 16384u)
      bulk_load_1d(smem_u32(gsm) + off, reinterpret_cast<const char*>(gw) + off, min(16384u, gbytes - off), mb);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsteps = (H + 128 * XU - 1) / (128 * XU);
  bool gate_waited = false, staged = true;
  for (int t0 = (blockIdx.x * 8 + warp) * RT_TPW; t0 < T_; t0 += gridDim.x * 8 * RT_TPW) {
    const int nt = min(RT_TPW, T_ - t0);
    const T* xr[RT_TPW];
#pragma unroll
    for (int j = 0; j < RT_TPW; ++j) xr[j] = x + (int64_t)(t0 + min(j, nt - 1)) * H;
    float acc[RT_TPW][E_MAX];
#pragma unroll
    for (int j = 0; j < RT_TPW; ++j)
#pragma unroll
      for (int e = 0; e < E_MAX; ++e) acc[j][e] = 0.f;
    C xa[RT_TPW][XU], xb[RT_TPW][XU];
    auto load_step = [&](C (&buf)[RT_TPW][XU], int st) {
#pragma unroll
      for (int j = 0; j < RT_TPW; ++j)
#pragma unroll
        for (int u = 0; u < XU; ++u) buf[j][u] = load_chunk<T>(xr[j], st * 128 * XU + lane * 4 + 128 * u, H);
    };
    auto sum_step = [&](const C (&buf)[RT_TPW][XU], int st) {
#pragma unroll
      for (int u = 0; u < XU; ++u) {
        const int h = st * 128 * XU + lane * 4 + 128 * u;
        if (h < H) {
          float xv[RT_TPW][4];
#pragma unroll
          for (int j = 0; j < RT_TPW; ++j) chunk_f32<T>(buf[j][u], xv[j]);
#pragma unroll
          for (int e = 0; e < E_MAX; ++e) {
            if (e < E) {
              const float4 gv = *reinterpret_cast<const float4*>(gsm + e * H + h);
#pragma unroll
              for (int j = 0; j < RT_TPW; ++j) {
                acc[j][e] = fmaf(xv[j][0], gv.x, acc[j][e]);
                acc[j][e] = fmaf(xv[j][1], gv.y, acc[j][e]);
                acc[j][e] = fmaf(xv[j][2], gv.z, acc[j][e]);
                acc[j][e] = fmaf(xv[j][3], gv.w, acc[j][e]);
              }
            }
          }
        }
      }
    };
    load_step(xa, 0);
    if (!gate_waited) {  // the first step's rows are in flight while the gate lands
      staged = mbar_wait(mb, 0, &abort_flag, nullptr, kDefaultWaitNs, 0);
      gate_waited = true;
    }
    for (int st = 0; st < nsteps; st += 2) {
      if (st + 1 < nsteps) load_step(xb, st + 1);
      sum_step(xa, st);
      if (st + 1 < nsteps) {
        if (st + 2 < nsteps) load_step(xa, st + 2);
        sum_step(xb, st + 1);
      }
    }
#pragma unroll
    for (int j = 0; j < RT_TPW; ++j) {
#pragma unroll
      for (int e = 0; e < E_MAX; ++e) {
        if (e < E && j < nt) {
          float v = acc[j][e];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == 0) {
            const float lv = staged ? v : __int_as_float(0x7fc00000);
            lsm[warp][j][e] = lv;
            logits[(int64_t)(t0 + j) * E + e] = lv;
          }
        }
      }
    }
    __syncwarp();
    for (int j = 0; j < nt; ++j)
      topk_row<1>(&lsm[warp][j][0], E, k, renorm, lane, ids + (int64_t)(t0 + j) * k,
                  weights + (int64_t)(t0 + j) * k);
    __syncwarp();
  }
  if (!gate_waited) mbar_wait(mb, 0, &abort_flag, nullptr, kDefaultWaitNs, 0);  // the copy lands before exit
}

}  // namespace

int launch_topk(const float* logits, int T_, int E, int k, int renorm, int32_t* ids, float* weights,
                cudaStream_t stream) {
  SB_CHECK_ARG(E >= 1 && E <= 256, "top-k: E=%d must be in [1, 256]", E);
  SB_CHECK_ARG(k >= 1 && k <= 8 && k <= E, "top-k: k=%d must be in [1, min(8, E)]", k);
  if (T_ == 0) return STAGEML_OK;
  SB_CHECK_ARG(logits && ids && weights, "top-k: null pointer");
  const int wpb = 8;
  const unsigned grid = (unsigned)((T_ + wpb - 1) / wpb);
  if (E <= 32)
    topk_kernel<1><<<grid, wpb * 32, 0, stream>>>(logits, T_, E, k, renorm, ids, weights);
  else if (E <= 64)
    topk_kernel<2><<<grid, wpb * 32, 0, stream>>>(logits, T_, E, k, renorm, ids, weights);
  else if (E <= 128)
    topk_kernel<4><<<grid, wpb * 32, 0, stream>>>(logits, T_, E, k, renorm, ids, weights);
  else
    topk_kernel<8><<<grid, wpb * 32, 0, stream>>>(logits, T_, E, k, renorm, ids, weights);
  ::sb::count_launch();
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
  const bool vec_dtype = x_dtype == STAGEML_BF16 || x_dtype == STAGEML_F16 || x_dtype == STAGEML_F32;
  if (E <= 32 && H % 4 == 0 && gbytes <= 200 * 1024 && aligned && vec_dtype) {
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
  if (x_dtype == STAGEML_BF16 && H % 32 == 0 && aligned) {
    const dim3 g2((unsigned)((T_ + RTC_TT - 1) / RTC_TT), (unsigned)((E + RTC_TE - 1) / RTC_TE));
    SB_CUDA_CHECK(cudaFuncSetAttribute(router_logits_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RTC_SMEM));
    (router_logits_tc_kernel<<<g2, 128, RTC_SMEM, stream>>>(static_cast<const bf16*>(x), gate_w, T_, H, E, logits),
     ::sb::count_launch());
    SB_CUDA_CHECK(cudaGetLastError());
    return STAGEML_OK;
  }
  const dim3 grid((unsigned)((T_ + RT_TT - 1) / RT_TT), (unsigned)((E + RT_TE - 1) / RT_TE));
  const bool vec = H % 8 == 0 && aligned;
  auto launch = [&](auto kern, const auto* xp) { (kern<<<grid, RT_THREADS, 0, stream>>>(xp, gate_w, T_, H, E, logits), ::sb::count_launch()); };
  if (x_dtype == STAGEML_BF16) {
    const bf16* xp = static_cast<const bf16*>(x);
    vec ? launch(router_logits_kernel<bf16, true>, xp) : launch(router_logits_kernel<bf16, false>, xp);
  } else if (x_dtype == STAGEML_F16) {
    const f16* xp = static_cast<const f16*>(x);
    vec ? launch(router_logits_kernel<f16, true>, xp) : launch(router_logits_kernel<f16, false>, xp);
  } else if (x_dtype == STAGEML_F32) {
    const float* xp = static_cast<const float*>(x);
    vec ? launch(router_logits_kernel<float, true>, xp) : launch(router_logits_kernel<float, false>, xp);
  } else {
    return set_error(STAGEML_ERR_INVALID_ARG, "router: unsupported x dtype %d", x_dtype);
  }
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

int launch_route(const void* x, int x_dtype, const float* gate_w, int T_, int H, int E, int k, int renorm,
                 float* logits, int32_t* ids, float* weights, cudaStream_t stream, bool pdl) {
  SB_CHECK_ARG(E >= 1 && E <= 256, "router: E=%d must be in [1, 256]", E);
  SB_CHECK_ARG(k >= 1 && k <= 8 && k <= E, "top-k: k=%d must be in [1, min(8, E)]", k);
  SB_CHECK_ARG(H >= 1, "router: H must be positive");
  if (T_ == 0) return STAGEML_OK;
  SB_CHECK_ARG(x && gate_w && logits && ids && weights, "router: null pointer");
  const size_t es = x_dtype == STAGEML_F32 ? 4 : 2;
  const size_t gbytes = sizeof(float) * (size_t)E * H, xbytes = es * (size_t)std::min(T_, kRouteSmallT) * H;
  const bool aligned = (reinterpret_cast<uintptr_t>(gate_w) % 16 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  const bool vec_dtype = x_dtype == STAGEML_BF16 || x_dtype == STAGEML_F16 || x_dtype == STAGEML_F32;
  if (T_ <= kRouteSmallMaxT && E <= 32 && H % 4 == 0 && (es * H) % 16 == 0 && gbytes + xbytes <= 220 * 1024 &&
      aligned && vec_dtype) {
    auto launch = [&](auto kern, const auto* xp) -> int {
      SB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(gbytes + xbytes)));
      SB_CUDA_CHECK(launch_kernel(kern, dim3((T_ + kRouteSmallT - 1) / kRouteSmallT), dim3(256), gbytes + xbytes, stream,
                                  pdl, xp, gate_w, T_, H, E, k, renorm, logits, ids, weights));
      ::sb::count_launch();
      return STAGEML_OK;
    };
    if (x_dtype == STAGEML_BF16) return launch(router_small_kernel<bf16>, static_cast<const bf16*>(x));
    if (x_dtype == STAGEML_F16) return launch(router_small_kernel<f16>, static_cast<const f16*>(x));
    return launch(router_small_kernel<float>, static_cast<const float*>(x));
  }
  if (E <= 32 && H % 4 == 0 && gbytes <= 200 * 1024 && aligned && vec_dtype) {
    const int grid = (int)std::min<int64_t>(sm_count(), ((int64_t)T_ + 8 * RT_TPW - 1) / (8 * RT_TPW));
    auto launch = [&](auto kern, const auto* xp) -> int {
      SB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gbytes));
      (kern<<<grid, 256, gbytes, stream>>>(xp, gate_w, T_, H, E, k, renorm, logits, ids, weights), ::sb::count_launch());
      SB_CUDA_CHECK(cudaGetLastError());
      return STAGEML_OK;
    };
    auto pick = [&](const auto* xp) -> int {
      using TT = std::remove_cv_t<std::remove_pointer_t<decltype(xp)>>;
      if (E <= 8) return launch(router_route_smem_kernel<TT, 8>, xp);
      if (E <= 16) return launch(router_route_smem_kernel<TT, 16>, xp);
      return launch(router_route_smem_kernel<TT, 32>, xp);
    };
    if (x_dtype == STAGEML_BF16) return pick(static_cast<const bf16*>(x));
    if (x_dtype == STAGEML_F16) return pick(static_cast<const f16*>(x));
    return pick(static_cast<const float*>(x));
  }
  SB_TRY(launch_router_logits(x, x_dtype, gate_w, T_, H, E, logits, stream));
  return launch_topk(logits, T_, E, k, renorm, ids, weights, stream);
}

}  // namespace sb
