// Expert-parallel dispatch and return over peer memory (NVLink / NVSwitch).
//
// One process per GPU; every rank owns a workspace of identical layout in its
// own HBM, mapped into every other rank through CUDA IPC. A layer call with
// epoch e (monotonic per layer object):
//   1. count  (1 CTA)   positions of this rank's (token, slot) pairs inside each
//                        destination's block, in pair order; this rank's count
//                        row is stored into every rank's count matrix, then each
//                        rank's count flag[rank] is raised to e.
//   2. send   (grid)    waits until every rank's count row arrived, derives this
//                        rank's base offset in each destination's dense receive
//                        buffer, stores x rows and (local expert, tenant, weight,
//                        source) records into the destinations' buffers, then the
//                        last CTA raises each destination's row flag[rank].
//   3. recv   (1 CTA)   waits for every source's row flag; writes the received
//                        row count for the local expert computation.
//   4. return (grid)    stores each output row into its source's return buffer
//                        at the source's own pair index; raises return flags.
//   5. combine (grid)   waits for every return flag; out[t] = sum_j ret[t*k+j]
//                        (+ the shared experts' output).
// Every wait is bounded (error word on expiry, never a trap). Buffer reuse across
// epochs is ordered by the protocol itself: a rank sends epoch e+1 only after its
// epoch-e combine, which needed every destination's epoch-e return, which each
// destination issued after consuming its epoch-e receive buffer. No multicast:
// plain stores to peer memory and release/acquire flags.
#include <cstring>

#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace sb {
namespace {

constexpr int kEpMaxWorld = 8;

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct EpDev {
  int world, rank, T, k, H, E_loc, esz;
  int epoch;
  unsigned long long timeout_ns;
  const uint64_t* peers;  // [world] workspace base of every rank (this rank's included)
  uint8_t* self;
  stageml_ep_layout L;
  const int32_t* ids;     // [T*k] global expert ids
  const float* weights;   // [T*k]
  const int32_t* tenants; // [T] or null
  const void* x;          // [T, H] 16-bit
  int32_t* pos;           // [T*k] position inside the destination block
  int32_t* status;
};

template <typename P>
__device__ __forceinline__ P* at(uint64_t base, size_t off) {
  return reinterpret_cast<P*>(base + off);
}

// Bounded wait until flags[s] >= epoch for every source s.
__device__ bool wait_all(const int* flags, int world, int epoch, unsigned long long timeout_ns, int32_t* status) {
  const unsigned long long t0 = globaltimer_ns();
  for (int s = 0; s < world; ++s) {
    while (ld_acquire_sys(flags + s) < epoch) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        if (status) atomicCAS(status, 0, (int)kDevTimeoutPeer);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

__device__ __forceinline__ int pair_dest(const EpDev& a, int64_t p) {
  const int e = a.ids[p];
  return (e >= 0 && e < a.E_loc * a.world) ? e / a.E_loc : -1;
}

__global__ void __launch_bounds__(1024) ep_count_kernel(const EpDev a) {
  __shared__ int warp_tot[32][kEpMaxWorld];
  __shared__ int carry[kEpMaxWorld];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid < kEpMaxWorld) carry[tid] = 0;
  if (tid == 0) {
    int* ctr = reinterpret_cast<int*>(a.self + a.L.counters);
    ctr[0] = 0;  // send-done counter of this epoch
    ctr[1] = 0;  // return-done counter
  }
  __syncthreads();
  const int64_t P = (int64_t)a.T * a.k;
  for (int64_t base = 0; base < P; base += 1024) {
    const int64_t p = base + tid;
    int d = -1;
    if (p < P) {
      d = pair_dest(a, p);
      if (d < 0 && a.status) atomicCAS(a.status, 0, (int)kDevBadIndex);
    }
    int prefix = 0;
    for (int dd = 0; dd < a.world; ++dd) {
      const unsigned bal = __ballot_sync(0xffffffffu, d == dd);
      if (d == dd) prefix = __popc(bal & ((1u << lane) - 1u));
      if (lane == 0) warp_tot[w][dd] = __popc(bal);
    }
    __syncthreads();
    if (d >= 0) {
      int before = carry[d];
      for (int ww = 0; ww < w; ++ww) before += warp_tot[ww][d];
      a.pos[p] = before + prefix;
    } else if (p < P) {
      a.pos[p] = -1;
    }
    __syncthreads();
    if (tid < a.world) {
      int tot = 0;
      for (int ww = 0; ww < 32; ++ww) tot += warp_tot[ww][tid];
      carry[tid] += tot;
    }
    __syncthreads();
  }
  // this rank's count row into every rank's count matrix, then the count flags
  if (tid < a.world * a.world) {
    const int q = tid / a.world, dd = tid - q * a.world;
    at<int>(a.peers[q], a.L.count_matrix)[a.rank * a.world + dd] = carry[dd];
  }
  __threadfence_system();
  __syncthreads();
  if (tid < a.world) st_release_sys(at<int>(a.peers[tid], a.L.flags_count) + a.rank, a.epoch);
}

__global__ void __launch_bounds__(256) ep_send_kernel(const EpDev a) {
  __shared__ int base[kEpMaxWorld];
  __shared__ int ok;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) {
    const int* flags = reinterpret_cast<const int*>(a.self + a.L.flags_count);
    ok = wait_all(flags, a.world, a.epoch, a.timeout_ns, a.status) ? 1 : 0;
    if (ok) {
      const int* m = reinterpret_cast<const int*>(a.self + a.L.count_matrix);
      for (int d = 0; d < a.world; ++d) {
        int b = 0;
        for (int s = 0; s < a.rank; ++s) b += __ldcg(m + s * a.world + d);
        base[d] = b;
      }
    }
  }
  __syncthreads();
  if (ok) {
    const int64_t P = (int64_t)a.T * a.k;
    const int vec_per_row = a.H * a.esz / 16;
    for (int64_t p = (int64_t)blockIdx.x * 8 + w; p < P; p += (int64_t)gridDim.x * 8) {
      const int d = pair_dest(a, p);
      if (d < 0) continue;
      const int64_t row = base[d] + a.pos[p];
      const int t = (int)(p / a.k);
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.x) + (int64_t)t * a.H * a.esz);
      uint4* dst = at<uint4>(a.peers[d], a.L.recv_x + (size_t)row * a.H * a.esz);
      for (int c = lane; c < vec_per_row; c += 32) dst[c] = __ldg(src + c);
      if (lane == 0) {
        at<int32_t>(a.peers[d], a.L.recv_expert)[row] = a.ids[p] - d * a.E_loc;
        at<float>(a.peers[d], a.L.recv_weight)[row] = a.weights[p];
        at<int32_t>(a.peers[d], a.L.recv_tenant)[row] = a.tenants ? a.tenants[t] : -1;
        at<int32_t>(a.peers[d], a.L.recv_source)[row] = (int32_t)(p * a.world + a.rank);
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    int* ctr = reinterpret_cast<int*>(a.self + a.L.counters);
    if (atomicAdd(ctr, 1) == (int)gridDim.x - 1) {
      __threadfence_system();
      for (int q = 0; q < a.world; ++q) st_release_sys(at<int>(a.peers[q], a.L.flags_rows) + a.rank, a.epoch);
    }
  }
}

__global__ void ep_recv_kernel(const EpDev a) {
  if (threadIdx.x != 0) return;
  const int* flags = reinterpret_cast<const int*>(a.self + a.L.flags_rows);
  int n = 0;
  if (wait_all(flags, a.world, a.epoch, a.timeout_ns, a.status)) {
    const int* m = reinterpret_cast<const int*>(a.self + a.L.count_matrix);
    for (int s = 0; s < a.world; ++s) n += __ldcg(m + s * a.world + a.rank);
  }
  *reinterpret_cast<int32_t*>(a.self + a.L.recv_tokens) = n;
}

__global__ void __launch_bounds__(256) ep_return_kernel(const EpDev a, const void* __restrict__ y) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int n = *reinterpret_cast<const int32_t*>(a.self + a.L.recv_tokens);
  const int32_t* src_of = reinterpret_cast<const int32_t*>(a.self + a.L.recv_source);
  const int vec_per_row = a.H * a.esz / 16;
  for (int64_t i = (int64_t)blockIdx.x * 8 + w; i < n; i += (int64_t)gridDim.x * 8) {
    const int src = src_of[i];
    const int s = src % a.world;
    const int64_t p = src / a.world;
    const uint4* from = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(y) + i * a.H * a.esz);
    uint4* to = at<uint4>(a.peers[s], a.L.ret_y + (size_t)p * a.H * a.esz);
    for (int c = lane; c < vec_per_row; c += 32) to[c] = __ldg(from + c);
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    int* ctr = reinterpret_cast<int*>(a.self + a.L.counters);
    if (atomicAdd(ctr + 1, 1) == (int)gridDim.x - 1) {
      __threadfence_system();
      for (int q = 0; q < a.world; ++q) st_release_sys(at<int>(a.peers[q], a.L.flags_return) + a.rank, a.epoch);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(128) ep_combine_kernel(const EpDev a, const T* __restrict__ add, T* __restrict__ out) {
  __shared__ int ok;
  const int t = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (threadIdx.x == 0) {
    const int* flags = reinterpret_cast<const int*>(a.self + a.L.flags_return);
    ok = wait_all(flags, a.world, a.epoch, a.timeout_ns, a.status) ? 1 : 0;
  }
  __syncthreads();
  if (!ok || c >= a.H) return;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  const T* ret = reinterpret_cast<const T*>(a.self + a.L.ret_y);
  for (int j = 0; j < a.k; ++j) {
    const int64_t p = (int64_t)t * a.k + j;
    if (pair_dest(a, p) < 0) continue;
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(ret + p * a.H + c));  // written by peers: bypass L1
    float f[8];
    unpack8<T>(u, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += f[i];
  }
  if (add) {
    float f[8];
    unpack8<T>(__ldg(reinterpret_cast<const uint4*>(add + (int64_t)t * a.H + c)), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += f[i];
  }
  *reinterpret_cast<uint4*>(out + (int64_t)t * a.H + c) = pack8<T>(acc);
}

int ep_dev(const stageml_ep_args* in, EpDev* a) {
  SB_CHECK_ARG(in, "ep: null args");
  SB_CHECK_ARG(in->world >= 1 && in->world <= kEpMaxWorld, "ep: world=%d must be in [1, %d]", in->world, kEpMaxWorld);
  SB_CHECK_ARG(in->rank >= 0 && in->rank < in->world, "ep: rank %d outside world %d", in->rank, in->world);
  SB_CHECK_ARG(in->T >= 0 && in->T <= in->tokens_cap && in->k >= 1 && in->E_loc >= 1,
               "ep: bad sizes T=%d (cap %lld) k=%d E_loc=%d", in->T, (long long)in->tokens_cap, in->k, in->E_loc);
  SB_CHECK_ARG(in->H > 0 && in->H % 8 == 0, "ep: H=%d must be a positive multiple of 8", in->H);
  SB_CHECK_ARG(in->act_dtype == STAGEML_BF16 || in->act_dtype == STAGEML_F16, "ep: activations must be BF16 or F16");
  SB_CHECK_ARG(in->peers && in->self && in->epoch > 0, "ep: need the peer table, this rank's workspace and epoch > 0");
  SB_CHECK_ARG((int64_t)in->world * in->tokens_cap * in->k < (int64_t(1) << 31) / in->world,
               "ep: pair capacity too large");
  stageml_ep_layout L;
  SB_TRY(stageml_ep_get_layout(in->world, in->tokens_cap, in->k, in->H, in->act_dtype, &L));
  a->world = in->world;
  a->rank = in->rank;
  a->T = in->T;
  a->k = in->k;
  a->H = in->H;
  a->E_loc = in->E_loc;
  a->esz = 2;
  a->epoch = in->epoch;
  a->timeout_ns = in->timeout_ns ? in->timeout_ns : 5000000000ull;
  a->peers = in->peers;
  a->self = static_cast<uint8_t*>(in->self);
  a->L = L;
  a->ids = in->topk_ids;
  a->weights = in->topk_weights;
  a->tenants = in->tenant_ids;
  a->x = in->x;
  a->pos = in->pos;
  a->status = in->status;
  return STAGEML_OK;
}

int ep_grid() { return 2 * sm_count(); }

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" int stageml_ep_get_layout(int world, int64_t tokens_cap, int k, int H, int act_dtype,
                                     stageml_ep_layout* out) {
  clear_error();
  SB_CHECK_ARG(out && world >= 1 && world <= kEpMaxWorld && tokens_cap >= 0 && k >= 1 && H > 0,
               "ep layout: bad arguments");
  SB_CHECK_ARG(act_dtype == STAGEML_BF16 || act_dtype == STAGEML_F16, "ep layout: activations must be BF16 or F16");
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t pairs_cap = (size_t)tokens_cap * k;
  const size_t recv_cap = (size_t)world * pairs_cap;
  size_t o = 0;
  out->count_matrix = o;
  o = al(o + (size_t)world * world * 4);
  out->flags_count = o;
  o = al(o + (size_t)world * 4);
  out->flags_rows = o;
  o = al(o + (size_t)world * 4);
  out->flags_return = o;
  o = al(o + (size_t)world * 4);
  out->counters = o;
  o = al(o + 16);
  out->recv_tokens = o;
  o = al(o + 4);
  out->recv_expert = o;
  o = al(o + recv_cap * 4);
  out->recv_weight = o;
  o = al(o + recv_cap * 4);
  out->recv_tenant = o;
  o = al(o + recv_cap * 4);
  out->recv_source = o;
  o = al(o + recv_cap * 4);
  out->recv_x = o;
  o = al(o + recv_cap * H * 2);
  out->ret_y = o;
  o = al(o + pairs_cap * H * 2);
  out->total = o;
  return STAGEML_OK;
}

extern "C" int stageml_ep_workspace_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  clear_error();
  SB_CHECK_ARG(ptr && ipc_handle && bytes > 0, "ep workspace: bad arguments");
  void* p = nullptr;
  SB_CUDA_CHECK(cudaMalloc(&p, bytes));
  const cudaError_t e1 = cudaMemset(p, 0, bytes);  // all flags start below epoch 1
  cudaIpcMemHandle_t h;
  const cudaError_t e2 = e1 == cudaSuccess ? cudaIpcGetMemHandle(&h, p) : e1;
  if (e2 != cudaSuccess) {
    cudaFree(p);
    return set_error(STAGEML_ERR_CUDA, "ep workspace: %s", cudaGetErrorString(e2));
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return STAGEML_OK;
}

extern "C" int stageml_ep_workspace_free(void* ptr) {
  clear_error();
  if (ptr) SB_CUDA_CHECK(cudaFree(ptr));
  return STAGEML_OK;
}

extern "C" int stageml_ep_workspace_open(const void* ipc_handle, void** ptr) {
  clear_error();
  SB_CHECK_ARG(ipc_handle && ptr, "ep open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  SB_CUDA_CHECK(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return STAGEML_OK;
}

extern "C" int stageml_ep_workspace_close(void* ptr) {
  clear_error();
  if (ptr) SB_CUDA_CHECK(cudaIpcCloseMemHandle(ptr));
  return STAGEML_OK;
}

extern "C" int stageml_ep_dispatch(const stageml_ep_args* in, void* stream) {
  clear_error();
  EpDev a;
  SB_TRY(ep_dev(in, &a));
  SB_CHECK_ARG(in->T == 0 || (in->topk_ids && in->topk_weights && in->x && in->pos),
               "ep dispatch: need ids, weights, x and the position scratch");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  (ep_count_kernel<<<1, 1024, 0, st>>>(a), count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  (ep_send_kernel<<<ep_grid(), 256, 0, st>>>(a), count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  (ep_recv_kernel<<<1, 32, 0, st>>>(a), count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

extern "C" int stageml_ep_return(const stageml_ep_args* in, const void* y_local, void* stream) {
  clear_error();
  EpDev a;
  SB_TRY(ep_dev(in, &a));
  SB_CHECK_ARG(y_local, "ep return: null output rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  (ep_return_kernel<<<ep_grid(), 256, 0, st>>>(a, y_local), count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

extern "C" int stageml_ep_combine(const stageml_ep_args* in, const void* add, void* out, void* stream) {
  clear_error();
  EpDev a;
  SB_TRY(ep_dev(in, &a));
  SB_CHECK_ARG(out || in->T == 0, "ep combine: null output");
  if (in->T == 0) return STAGEML_OK;
  SB_CHECK_ARG(in->T <= 65535, "ep combine: at most 65535 tokens per rank");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((in->H / 8 + 127) / 128), (unsigned)in->T);
  if (in->act_dtype == STAGEML_BF16)
    (ep_combine_kernel<bf16><<<grid, 128, 0, st>>>(a, static_cast<const bf16*>(add), static_cast<bf16*>(out)),
     count_launch());
  else
    (ep_combine_kernel<f16><<<grid, 128, 0, st>>>(a, static_cast<const f16*>(add), static_cast<f16*>(out)),
     count_launch());
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}
