// Token -> expert permutation (R2): a deterministic, stable counting sort of
// the routed (token, slot) pairs by key (expert, tenant), each expert segment
// padded to 128 rows so every 128-row GEMM tile belongs to one expert.
//
// The reference groups rows with one torch.nonzero per (slot, expert) and a
// host sync each (benchmarks/multitenant_bta_system_bench.py:401-406); here the
// whole grouping runs on the device with no host round trip. Up to 1024 keys
// (every MoE-LoRA shape here) one kernel ranks the pairs of each 2048-pair chunk
// by warp matching and its last CTA builds the plan (perm_rank_kernel; a second
// kernel places the pairs beyond 8 chunks). Beyond 1024 keys it is two
// kernels (one when P <= 2048):
//   count   one CTA per 2048-pair chunk: bitonic sort of (key << 11 | index)
//           in shared memory, per-key counts of the chunk -> hist[chunk][key],
//           added to the per-key totals with integer atomics; the last CTA turns
//           the totals into per-group counts, padded group offsets, the tile ->
//           group map and each key's first row
//   scatter one CTA per chunk: destination = the key's first row + the key's
//           pairs in the earlier chunks + rank of the pair inside its key segment
//           of the (already sorted) chunk
// (A single CTA summing the [chunks x keys] counts took 68 µs of the fine-grained
// layer's 105 µs permutation at 8514 keys and 32 chunks.)
// Sorting (key, pair index) makes the order within a key the pair order, so
// the permutation is the stable sort the oracle defines, bit for bit.
//
// Keys: the dynamic groups (experts, or (tenant, expert) with group_by_tenant)
// own tkeys consecutive keys each, one per tenant + 1; with a fold map, a pair
// whose (tenant, expert) has folded weights takes the single key of its folded
// weight group (n_dyn * tkeys + slot), after every dynamic key, and its row
// carries no LoRA tenant.
#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace sb {
namespace {

constexpr uint32_t kSentKey = 0x1FFFFFu;  // 21-bit key field; dropped pairs and empty slots
constexpr int kMaxKeys = 32768;           // keys held in shared memory by the scan kernel

struct PairSrc {
  const void* ids;
  int ids_i64;
  const void* weights;
  int weights_dtype;
  const int32_t* tenant_ids;
  int T, k, kk, E_routed, E_tot, n_tenants, group_by_tenant, tkeys;
  int n_dyn;                // dynamic weight groups (keys [0, n_dyn * tkeys))
  const int32_t* fold_slot; // optional [n_tenants, E_tot]: -1 dynamic, s >= 0 folded weight group n_dyn + s
  int n_fold;
  int64_t P;
  const int32_t* T_dev;  // optional: tokens >= *T_dev are not routed (no error)
};

// Pairs that exist: all P, or those of the first *T_dev tokens.
__device__ __forceinline__ int64_t live_pairs(const PairSrc& a) {
  if (!a.T_dev) return a.P;
  const int64_t n = (int64_t)(*a.T_dev) * a.kk;
  return n < a.P ? (n < 0 ? 0 : n) : a.P;
}

__device__ __forceinline__ int pair_expert(const PairSrc& a, int t, int j, bool* bad) {
  if (j >= a.k) return a.E_routed + (j - a.k);
  const int64_t idx = (int64_t)t * a.k + j;
  const int64_t e = a.ids_i64 ? static_cast<const int64_t*>(a.ids)[idx] : (int64_t) static_cast<const int32_t*>(a.ids)[idx];
  if (e < 0 || e >= a.E_routed) {
    *bad = true;
    return 0;
  }
  return (int)e;
}

__device__ __forceinline__ int pair_tenant(const PairSrc& a, int t, bool* bad) {
  if (!a.tenant_ids) return -1;
  const int tn = a.tenant_ids[t];
  if (tn < -1 || tn >= a.n_tenants) {
    *bad = true;
    return -1;
  }
  return tn;
}

__device__ __forceinline__ float pair_weight(const PairSrc& a, int t, int j) {
  if (j >= a.k || !a.weights) return 1.f;
  const int64_t idx = (int64_t)t * a.k + j;
  if (a.weights_dtype == STAGEML_BF16) return __bfloat162float(static_cast<const bf16*>(a.weights)[idx]);
  if (a.weights_dtype == STAGEML_F16) return __half2float(static_cast<const f16*>(a.weights)[idx]);
  return static_cast<const float*>(a.weights)[idx];
}

// Sort key of pair p, or kSentKey when an id is out of range.
__device__ __forceinline__ uint32_t pair_key(const PairSrc& a, int64_t p, int32_t* status) {
  const int t = (int)(p / a.kk);
  const int j = (int)(p - (int64_t)t * a.kk);
  bool bad = false;
  const int e = pair_expert(a, t, j, &bad);
  const int tn = pair_tenant(a, t, &bad);
  if (a.group_by_tenant && tn < 0) bad = true;
  int slot = -1;
  if (!bad && a.fold_slot && tn >= 0) {
    slot = a.fold_slot[(int64_t)tn * a.E_tot + e];
    if (slot < -1 || slot >= a.n_fold) bad = true;
  }
  if (bad) {
    if (status) atomicCAS(status, 0, (int)kDevBadIndex);
    return kSentKey;
  }
  if (slot >= 0) return (uint32_t)(a.n_dyn * a.tkeys + slot);
  if (a.group_by_tenant) return (uint32_t)(tn * a.E_tot + e);
  return (uint32_t)(e * a.tkeys + (tn + 1));
}

// Keys of weight group g: [first, first + count).
__device__ __forceinline__ int group_first_key(int g, int tkeys, int n_dyn) {
  return g < n_dyn ? g * tkeys : n_dyn * tkeys + (g - n_dyn);
}
__device__ __forceinline__ int group_key_count(int g, int tkeys, int n_dyn) { return g < n_dyn ? tkeys : 1; }

// Sorts s[0..2048) ascending when s[n..2048) already hold the largest value
// (the sentinel): only the first next_pow2(n) entries go through the network.
__device__ __forceinline__ void bitonic_sort_2048(uint32_t* s, int n) {
  // 1024 threads, at most one compare-exchange pair each per stage.
  const int tid = threadIdx.x;
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (tid < (n2 >> 1)) {
        const int i = 2 * tid - (tid & (j - 1));
        const int ixj = i + j;
        const bool up = (i & k) == 0;
        const uint32_t a = s[i], b = s[ixj];
        if ((a > b) == up) {
          s[i] = b;
          s[ixj] = a;
        }
      }
      __syncthreads();
    }
  }
}

// First index in sorted s[0..n) whose key field is >= key.
__device__ __forceinline__ int lower_bound_key(const uint32_t* s, int n, uint32_t key) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((s[mid] >> 11) < key)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// Forward declaration: the last count CTA builds the plan.
__device__ __forceinline__ void plan_groups(int32_t* tot, int tkeys, int n_dyn, int n_groups,
                                            const stageml_moe_plan& plan, int32_t* warp_part);

// One CTA per 2048-pair chunk: sort the chunk's (key, index) words, write its per-key
// counts hist[chunk][key] and add them to the totals tot_g[key] (integer atomics, so
// the sums do not depend on the order). The last CTA to finish turns the totals into
// the plan (per-group counts, padded offsets, tile -> group map) and leaves each key's
// first row in tot_g.
__global__ void __launch_bounds__(1024) perm_count_kernel(PairSrc a, int nkeys, int nch, int n_groups,
                                                           stageml_moe_plan plan, uint32_t* sorted_out,
                                                           int32_t* hist, int32_t* tot_g, int32_t* ticket,
                                                           int32_t* status) {
  __shared__ uint32_t s[kPermChunk];
  __shared__ int32_t warp_part[32];
  __shared__ int s_last;
  extern __shared__ int32_t tot[];  // [nkeys], the last CTA only
  const int64_t base = (int64_t)blockIdx.x * kPermChunk;
  const int64_t live = live_pairs(a);
  for (int i = threadIdx.x; i < kPermChunk; i += 1024) {
    const int64_t p = base + i;
    s[i] = (p < live) ? ((pair_key(a, p, status) << 11) | (uint32_t)i) : 0xFFFFFFFFu;
  }
  __syncthreads();
  const int64_t n_live = live - base;
  bitonic_sort_2048(s, n_live <= 0 ? 0 : (n_live < kPermChunk ? (int)n_live : kPermChunk));
  for (int i = threadIdx.x; i < kPermChunk; i += 1024) {
    const uint32_t v = s[i];
    sorted_out[base + i] = v;
    const uint32_t key = v >> 11;
    if (key == kSentKey) continue;
    if (i == kPermChunk - 1 || (s[i + 1] >> 11) != key) {
      const int n = i - lower_bound_key(s, i + 1, key) + 1;
      hist[(int64_t)blockIdx.x * nkeys + key] = n;
      atomicAdd(tot_g + key, n);
    }
  }
  // Classic last-block pattern: every thread's writes are fenced before the ticket.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    s_last = atomicAdd(ticket, 1) == nch - 1;
    if (s_last) *ticket = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int k = threadIdx.x; k < nkeys; k += 1024) tot[k] = __ldcg(tot_g + k);
  __syncthreads();
  plan_groups(tot, a.tkeys, a.n_dyn, n_groups, plan, warp_part);
  for (int k = threadIdx.x; k < nkeys; k += 1024) tot_g[k] = tot[k];
}

// From the per-key totals tot[nkeys] (in shared memory, 1024 threads): per-group
// counts, padded group offsets, tile -> group map and padding rows of the plan;
// tot is left holding each key's first row.
__device__ __forceinline__ void plan_groups(int32_t* tot, int tkeys, int n_dyn, int n_groups,
                                            const stageml_moe_plan& plan, int32_t* warp_part) {
  const int tid = threadIdx.x;
  const int lane = tid & 31, wid = tid >> 5;
  // 2. per-group real counts (a warp per group); padded sizes parked in group_offsets[g]
  for (int g = wid; g < n_groups; g += 32) {
    const int k0 = group_first_key(g, tkeys, n_dyn), nk = group_key_count(g, tkeys, n_dyn);
    int cnt = 0;
    for (int tk = lane; tk < nk; tk += 32) cnt += tot[k0 + tk];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) {
      plan.group_counts[g] = cnt;
      plan.group_offsets[g] = (cnt + 127) & ~127;
    }
  }
  __syncthreads();
  // 3. exclusive scan of padded sizes (each thread a contiguous run of groups)
  const int per = (n_groups + 1023) / 1024;
  const int g0 = min(tid * per, n_groups), g1 = min(g0 + per, n_groups);
  int local = 0;
  for (int g = g0; g < g1; ++g) local += plan.group_offsets[g];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_part[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    int w = warp_part[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += v;
    }
    warp_part[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  int run = incl - local + (wid > 0 ? warp_part[wid - 1] : 0);
  for (int g = g0; g < g1; ++g) {
    const int sz = plan.group_offsets[g];
    plan.group_offsets[g] = run;
    run += sz;
  }
  if (tid == 1023) {
    plan.group_offsets[n_groups] = run;
    plan.num_tiles[0] = run / 128;
  }
  __syncthreads();
  // 4. key bases (in place in tot), tile -> group, padding rows: one warp per group
  for (int g = wid; g < n_groups; g += 32) {
    const int o = plan.group_offsets[g];
    const int cnt = plan.group_counts[g];
    const int end = o + ((cnt + 127) & ~127);
    for (int t = o / 128 + lane; t < end / 128; t += 32) plan.tile_group[t] = g;
    for (int r = o + cnt + lane; r < end; r += 32) {
      plan.row_token[r] = -1;
      plan.row_tenant[r] = -1;
      plan.row_weight[r] = 0.f;
      plan.row_pair[r] = -1;
    }
    // exclusive scan of the group's key counts in key order: each lane a contiguous run of keys
    const int k0 = group_first_key(g, tkeys, n_dyn), nk = group_key_count(g, tkeys, n_dyn);
    const int per = (nk + 31) / 32;
    const int a0 = min(lane * per, nk), a1 = min(a0 + per, nk);
    int ksum = 0;
    for (int key = k0 + a0; key < k0 + a1; ++key) ksum += tot[key];
    int incl_k = ksum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl_k, d);
      if (lane >= d) incl_k += v;
    }
    int b = o + incl_k - ksum;
    for (int key = k0 + a0; key < k0 + a1; ++key) {
      const int v = tot[key];
      tot[key] = b;
      b += v;
    }
  }
  __syncthreads();
}

// Pair p (sort key `key`) lands in plan row `row`; rows of folded weight groups carry no LoRA tenant.
__device__ __forceinline__ void place_pair(const PairSrc& a, const stageml_moe_plan& plan, int64_t p, int row,
                                           uint32_t key) {
  const int t = (int)(p / a.kk);
  const int j = (int)(p - (int64_t)t * a.kk);
  bool dummy = false;
  const int tn = pair_tenant(a, t, &dummy);
  plan.row_token[row] = t;
  plan.row_tenant[row] = (a.group_by_tenant || key >= (uint32_t)(a.n_dyn * a.tkeys)) ? -1 : tn;
  plan.row_weight[row] = pair_weight(a, t, j);
  plan.row_pair[row] = (int32_t)p;
  plan.pair_row[p] = row;
}

// One CTA per chunk: a key's first pair in this chunk lands at the key's first row
// plus the key's pairs in the chunks before (summed here from hist), the others
// follow it in sorted order.
__global__ void __launch_bounds__(1024) perm_scatter_kernel(PairSrc a, int nkeys, const uint32_t* __restrict__ sorted,
                                                             const int32_t* __restrict__ hist,
                                                             const int32_t* __restrict__ key_first,
                                                             stageml_moe_plan plan) {
  __shared__ uint32_t s[kPermChunk];
  __shared__ int32_t first_row[kPermChunk];  // at the first position of each key
  const int64_t base = (int64_t)blockIdx.x * kPermChunk;
  for (int i = threadIdx.x; i < kPermChunk; i += 1024) s[i] = sorted[base + i];
  __syncthreads();
  for (int i = threadIdx.x; i < kPermChunk; i += 1024) {
    const uint32_t key = s[i] >> 11;
    if (key == kSentKey || (i > 0 && (s[i - 1] >> 11) == key)) continue;
    int b = key_first[key];
#pragma unroll 4
    for (int c = 0; c < (int)blockIdx.x; ++c) b += hist[(int64_t)c * nkeys + key];
    first_row[i] = b;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kPermChunk; i += 1024) {
    const uint32_t v = s[i];
    const int64_t p = base + (v & 2047u);
    if (p >= a.P) continue;
    const uint32_t key = v >> 11;
    if (key == kSentKey) {
      plan.pair_row[p] = -1;
      continue;
    }
    const int start = lower_bound_key(s, i, key);
    place_pair(a, plan, p, first_row[start] + (i - start), key);
  }
}

// P <= 2048 (one chunk): count, scan and scatter in one CTA, the per-key counts
// in shared memory; the same plan as the three kernels.
__global__ void __launch_bounds__(1024) perm_fused_kernel(PairSrc a, int nkeys, int n_groups, stageml_moe_plan plan,
                                                           int32_t* status) {
  extern __shared__ int32_t tot[];  // [nkeys]
  __shared__ uint32_t s[kPermChunk];
  __shared__ int32_t warp_part[32];
  const int64_t live = live_pairs(a);
  for (int key = threadIdx.x; key < nkeys; key += 1024) tot[key] = 0;
  for (int i = threadIdx.x; i < kPermChunk; i += 1024)
    s[i] = (i < live) ? ((pair_key(a, i, status) << 11) | (uint32_t)i) : 0xFFFFFFFFu;
  __syncthreads();
  bitonic_sort_2048(s, live < kPermChunk ? (int)live : kPermChunk);
  for (int i = threadIdx.x; i < kPermChunk; i += 1024) {
    const uint32_t key = s[i] >> 11;
    if (key == kSentKey) continue;
    if (i == kPermChunk - 1 || (s[i + 1] >> 11) != key) tot[key] = i - lower_bound_key(s, i + 1, key) + 1;
  }
  __syncthreads();
  plan_groups(tot, a.tkeys, a.n_dyn, n_groups, plan, warp_part);
  for (int64_t p = live + threadIdx.x; p < a.P; p += 1024) plan.pair_row[p] = -1;  // pairs of tokens past *T_dev
  for (int i = threadIdx.x; i < kPermChunk; i += 1024) {
    const uint32_t v = s[i];
    const int64_t p = v & 2047u;
    if (p >= a.P) continue;
    const uint32_t key = v >> 11;
    if (key == kSentKey) {
      plan.pair_row[p] = -1;
      continue;
    }
    place_pair(a, plan, p, tot[key] + (i - lower_bound_key(s, i, key)), key);
  }
}

// Up to kRankMaxKeys keys: ranks by warp matching instead of a sort. One CTA per
// 2048-pair chunk; warp w owns chunk entries [64 w, 64 w + 64) in two rounds of 32.
// Within a round __match_any_sync finds the lanes of each key, so an entry's rank
// among the chunk's entries of its key is (earlier warps' count of the key) +
// (this warp's count from its earlier round) + (lower lanes of the same key) --
// chunk order, i.e. the stable order. Each entry is written as key << 11 | rank.
// The last CTA to finish (ticket) turns the per-chunk counts into the plan
// (plan_groups) and the per-(chunk, key) first rows; with few chunks it also
// places every pair, else perm_place_kernel does.
constexpr int kRankMaxKeys = 1024;
constexpr int kLastPlacesChunks = 8;

__global__ void __launch_bounds__(1024) perm_rank_kernel(PairSrc a, int nkeys, int n_groups, stageml_moe_plan plan,
                                                          uint32_t* __restrict__ rank_key, int32_t* __restrict__ hist,
                                                          int32_t* __restrict__ off, int32_t* __restrict__ ticket,
                                                          int32_t* status) {
  extern __shared__ int32_t sm[];  // [32][nkeys] per-warp counts (+ [nkeys] totals for one chunk); in the
                                   // last CTA of several: tot[nkeys] + offsets
  __shared__ int32_t warp_part[32];
  __shared__ int s_last;
  pdl_wait();  // ids / weights may come from the previous kernel
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int nch = (int)gridDim.x;
  const int64_t base = (int64_t)blockIdx.x * kPermChunk;
  const int64_t live = live_pairs(a);
  for (int i = tid; i < 32 * nkeys; i += 1024) sm[i] = 0;
  __syncthreads();
  const unsigned below = (1u << lane) - 1u;
  uint32_t key[2];
  int rnk[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t p = base + w * 64 + r * 32 + lane;
    const uint32_t k = p < live ? pair_key(a, p, status) : kSentKey;
    const unsigned peers = __match_any_sync(0xffffffffu, k);
    const int before = k != kSentKey ? sm[w * nkeys + (int)k] : 0;
    __syncwarp();
    if (k != kSentKey && (peers & below) == 0u) sm[w * nkeys + (int)k] = before + __popc(peers);
    __syncwarp();
    key[r] = k;
    rnk[r] = before + __popc(peers & below);
  }
  __syncthreads();
  if (nch == 1) {
    // One chunk: the key totals and the ranks stay on chip; the plan is built and
    // every pair placed here (no global round trip).
    int32_t* tot = sm + 32 * nkeys;  // [nkeys]
    for (int k = tid; k < nkeys; k += 1024) {
      int run = 0;
      for (int ww = 0; ww < 32; ++ww) {
        const int c = sm[ww * nkeys + k];
        sm[ww * nkeys + k] = run;
        run += c;
      }
      tot[k] = run;
    }
    __syncthreads();
    plan_groups(tot, a.tkeys, a.n_dyn, n_groups, plan, warp_part);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int64_t p = w * 64 + r * 32 + lane;
      if (p >= a.P) continue;
      if (key[r] == kSentKey)
        plan.pair_row[p] = -1;
      else
        place_pair(a, plan, p, tot[key[r]] + sm[w * nkeys + (int)key[r]] + rnk[r], key[r]);
    }
    return;
  }
  for (int k = tid; k < nkeys; k += 1024) {  // exclusive prefix over warps, chunk total
    int run = 0;
    for (int ww = 0; ww < 32; ++ww) {
      const int c = sm[ww * nkeys + k];
      sm[ww * nkeys + k] = run;
      run += c;
    }
    hist[(int64_t)blockIdx.x * nkeys + k] = run;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t p = base + w * 64 + r * 32 + lane;
    if (p < a.P)
      rank_key[p] = key[r] == kSentKey ? 0xFFFFFFFFu : ((key[r] << 11) | (uint32_t)(sm[w * nkeys + (int)key[r]] + rnk[r]));
  }
  // Classic last-block pattern: every thread's writes are fenced before the ticket.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int t = nch == 1 ? 0 : atomicAdd(ticket, 1);
    s_last = t == nch - 1;
    if (s_last && nch > 1) *ticket = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  int32_t* tot = sm;  // [nkeys]
  for (int k = tid; k < nkeys; k += 1024) {
    int s = 0;
#pragma unroll 4
    for (int c = 0; c < nch; ++c) s += __ldcg(hist + (int64_t)c * nkeys + k);
    tot[k] = s;
  }
  __syncthreads();
  plan_groups(tot, a.tkeys, a.n_dyn, n_groups, plan, warp_part);
  const bool place_here = nch <= kLastPlacesChunks;
  int32_t* offs = place_here ? sm + nkeys : off;  // [nch][nkeys]
  for (int k = tid; k < nkeys; k += 1024) {
    int b = tot[k];
#pragma unroll 4
    for (int c = 0; c < nch; ++c) {
      const int v = __ldcg(hist + (int64_t)c * nkeys + k);
      offs[(int64_t)c * nkeys + k] = b;
      b += v;
    }
  }
  if (!place_here) return;
  __syncthreads();
  for (int64_t p = tid; p < a.P; p += 1024) {
    const uint32_t v = __ldcg(rank_key + p);
    const uint32_t k = v >> 11;
    if (k == kSentKey) {
      plan.pair_row[p] = -1;
      continue;
    }
    place_pair(a, plan, p, offs[(p / kPermChunk) * nkeys + k] + (int)(v & 2047u), k);
  }
}

__global__ void __launch_bounds__(256) perm_place_kernel(PairSrc a, int nkeys, const uint32_t* __restrict__ rank_key,
                                                          const int32_t* __restrict__ off, stageml_moe_plan plan) {
  const int64_t p = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (p >= a.P) return;
  const uint32_t v = rank_key[p];
  const uint32_t k = v >> 11;
  if (k == kSentKey) {
    plan.pair_row[p] = -1;
    return;
  }
  place_pair(a, plan, p, off[(p / kPermChunk) * nkeys + k] + (int)(v & 2047u), k);
}

}  // namespace

int64_t permute_num_keys(int n_fold, int n_tenants, int group_by_tenant, int n_experts_total) {
  if (group_by_tenant) return (int64_t)n_tenants * n_experts_total + n_fold;
  return (int64_t)n_experts_total * (n_tenants + 1) + n_fold;
}

static int64_t nchunks_of(int64_t P) { return P > 0 ? (P + kPermChunk - 1) / kPermChunk : 1; }

size_t permute_scratch_bytes(int64_t P, int64_t nkeys) {
  const int64_t nch = nchunks_of(P);
  size_t b = 0;
  b += ((size_t)nch * kPermChunk * 4 + 255) & ~size_t(255);
  b += ((size_t)nkeys * nch * 4 + 255) & ~size_t(255);
  b += ((size_t)nkeys * nch * 4 + 255) & ~size_t(255);
  b += 256;  // ticket
  return b;
}

void permute_carve(void* base, int64_t P, int64_t nkeys, PermuteScratch* out) {
  const int64_t nch = nchunks_of(P);
  uint8_t* p = static_cast<uint8_t*>(base);
  out->sorted = reinterpret_cast<uint32_t*>(p);
  p += ((size_t)nch * kPermChunk * 4 + 255) & ~size_t(255);
  out->hist = reinterpret_cast<int32_t*>(p);
  p += ((size_t)nkeys * nch * 4 + 255) & ~size_t(255);
  out->off = reinterpret_cast<int32_t*>(p);
  p += ((size_t)nkeys * nch * 4 + 255) & ~size_t(255);
  out->ticket = reinterpret_cast<int32_t*>(p);
}

int launch_permute(const void* ids, int ids_dtype, const void* weights, int weights_dtype, const int32_t* tenant_ids,
                   int T, int k, int n_shared, int n_experts_total, int n_tenants, int group_by_tenant,
                   const stageml_moe_plan& plan, int32_t* status, const PermuteScratch& scr, cudaStream_t stream,
                   const int32_t* T_dev, bool pdl, const int32_t* fold_slot, int n_fold) {
  SB_CHECK_ARG(T >= 0 && k >= 0 && n_shared >= 0, "permute: negative size");
  SB_CHECK_ARG(k + n_shared >= 1, "permute: need at least one slot per token");
  SB_CHECK_ARG(n_experts_total > n_shared || (k == 0 && n_experts_total == n_shared),
               "permute: n_experts_total=%d must exceed n_shared=%d", n_experts_total, n_shared);
  SB_CHECK_ARG(ids_dtype == STAGEML_I32 || ids_dtype == STAGEML_I64, "permute: ids must be int32 or int64");
  SB_CHECK_ARG(k == 0 || T == 0 || ids, "permute: null ids");
  SB_CHECK_ARG(!weights || weights_dtype == STAGEML_F32 || weights_dtype == STAGEML_BF16 ||
                   weights_dtype == STAGEML_F16,
               "permute: weights must be f32, bf16 or f16");
  SB_CHECK_ARG(n_tenants >= 0, "permute: negative tenant count");
  SB_CHECK_ARG(!group_by_tenant || (tenant_ids && n_tenants > 0), "permute: group_by_tenant needs tenant ids");
  SB_CHECK_ARG(n_fold >= 0 && (n_fold == 0 || fold_slot), "permute: n_fold=%d needs a fold map", n_fold);
  SB_CHECK_ARG(!fold_slot || (!group_by_tenant && tenant_ids && n_tenants > 0),
               "permute: a fold map needs tenant ids and per-expert groups");
  const int64_t P = (int64_t)T * (k + n_shared);
  if (!fold_slot) n_fold = 0;
  const int64_t nkeys = permute_num_keys(n_fold, n_tenants, group_by_tenant, n_experts_total);
  const int n_dyn = group_by_tenant ? n_tenants * n_experts_total : n_experts_total;
  const int n_groups = n_dyn + n_fold;
  SB_CHECK_ARG(nkeys >= 1 && nkeys <= kMaxKeys, "permute: %lld (expert, tenant) keys exceed the limit %d",
               (long long)nkeys, kMaxKeys);
  SB_CHECK_ARG(plan.rows_cap >= stageml_plan_rows_cap(P, n_groups), "permute: plan rows_cap %lld < required %lld",
               (long long)plan.rows_cap, (long long)stageml_plan_rows_cap(P, n_groups));
  SB_CHECK_ARG(plan.row_token && plan.row_tenant && plan.row_weight && plan.row_pair && plan.tile_group &&
                   plan.group_offsets && plan.group_counts && plan.num_tiles && (P == 0 || plan.pair_row),
               "permute: null plan array");
  SB_CHECK_ARG(P < (int64_t(1) << 31), "permute: too many pairs");

  PairSrc a;
  a.ids = ids;
  a.ids_i64 = ids_dtype == STAGEML_I64;
  a.weights = weights;
  a.weights_dtype = weights_dtype;
  a.tenant_ids = tenant_ids;
  a.T = T;
  a.k = k;
  a.kk = k + n_shared;
  a.E_tot = n_experts_total;
  a.E_routed = n_experts_total - n_shared;
  a.n_tenants = n_tenants;
  a.group_by_tenant = group_by_tenant;
  a.tkeys = group_by_tenant ? 1 : n_tenants + 1;
  a.n_dyn = n_dyn;
  a.fold_slot = fold_slot;
  a.n_fold = n_fold;
  a.P = P;
  a.T_dev = T_dev;

  const int64_t nch = nchunks_of(P);
  if (nkeys <= kRankMaxKeys) {
    const size_t smem_r = (size_t)33 * nkeys * 4;
    SB_CHECK_ARG(nch <= 65535, "permute: too many pairs");
    if (nch > 1) SB_CUDA_CHECK(cudaMemsetAsync(scr.ticket, 0, sizeof(int32_t), stream));
    SB_CUDA_CHECK(cudaFuncSetAttribute(perm_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_r));
    SB_CUDA_CHECK(launch_kernel(perm_rank_kernel, dim3((unsigned)nch), dim3(1024), smem_r, stream, pdl && nch == 1, a,
                                (int)nkeys, n_groups, plan, scr.sorted, scr.hist, scr.off, scr.ticket, status));
    ::sb::count_launch();
    if (nch > kLastPlacesChunks) {
      (perm_place_kernel<<<(unsigned)((P + 255) / 256), 256, 0, stream>>>(a, (int)nkeys, scr.sorted, scr.off, plan),
       ::sb::count_launch());
      SB_CUDA_CHECK(cudaGetLastError());
    }
    return STAGEML_OK;
  }
  const size_t smem = (size_t)nkeys * 4;
  if (nch == 1) {
    SB_CUDA_CHECK(cudaFuncSetAttribute(perm_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    (perm_fused_kernel<<<1, 1024, smem, stream>>>(a, (int)nkeys, n_groups, plan, status), ::sb::count_launch());
    SB_CUDA_CHECK(cudaGetLastError());
    return STAGEML_OK;
  }
  // Several chunks: per-chunk counts and the totals (off[0, nkeys)) start at zero; the
  // last count CTA builds the plan and leaves each key's first row in off.
  SB_CHECK_ARG(nch <= 65535, "permute: too many pairs");
  int32_t* key_first = scr.off;
  SB_CUDA_CHECK(cudaMemsetAsync(scr.hist, 0, (size_t)nkeys * nch * 4, stream));
  SB_CUDA_CHECK(cudaMemsetAsync(key_first, 0, (size_t)nkeys * 4, stream));
  SB_CUDA_CHECK(cudaMemsetAsync(scr.ticket, 0, sizeof(int32_t), stream));
  SB_CUDA_CHECK(cudaFuncSetAttribute(perm_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  (perm_count_kernel<<<(unsigned)nch, 1024, smem, stream>>>(a, (int)nkeys, (int)nch, n_groups, plan, scr.sorted,
                                                             scr.hist, key_first, scr.ticket, status),
   ::sb::count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  (perm_scatter_kernel<<<(unsigned)nch, 1024, 0, stream>>>(a, (int)nkeys, scr.sorted, scr.hist, key_first, plan),
   ::sb::count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

}  // namespace sb

extern "C" int64_t stageml_plan_rows_cap(int64_t num_pairs, int n_groups) {
  if (num_pairs <= 0) return 128;
  const int64_t g = n_groups < num_pairs ? n_groups : num_pairs;
  const int64_t r = num_pairs + g * 127;
  return (r + 127) / 128 * 128;
}
