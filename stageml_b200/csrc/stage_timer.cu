// Thread-local stage timer: pooled CUDA events recorded around kernel stages.
#include <vector>

#include "host_util.h"
#include "stage_timer.h"

namespace sb {
namespace {

struct Rec {
  int stage;
  cudaEvent_t a;
  cudaEvent_t b;
};

thread_local bool t_on = false;
thread_local unsigned t_mask = ~0u;  // stages recorded while on (bit s = stage s)
thread_local std::vector<Rec> t_recs;
thread_local std::vector<cudaEvent_t> t_pool;
thread_local int t_open_stage = -1;
thread_local cudaEvent_t t_open_event = nullptr;

cudaEvent_t get_event() {
  if (!t_pool.empty()) {
    cudaEvent_t e = t_pool.back();
    t_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

}  // namespace

bool stage_timer_on(int stage) { return t_on && stage >= 0 && stage < 32 && ((t_mask >> stage) & 1u); }

void stage_timer_record(int stage, cudaStream_t stream, bool begin) {
  cudaEvent_t e = get_event();
  if (!e) return;
  cudaEventRecord(e, stream);
  if (begin) {
    t_open_stage = stage;
    t_open_event = e;
  } else if (t_open_stage == stage && t_open_event) {
    t_recs.push_back({stage, t_open_event, e});
    t_open_stage = -1;
    t_open_event = nullptr;
  } else {
    t_pool.push_back(e);
  }
}

}  // namespace sb

extern "C" int stageml_stage_timer_enable(int on) {
  sb::t_on = on != 0;
  return STAGEML_OK;
}

extern "C" int stageml_stage_timer_select(unsigned int mask) {
  sb::t_mask = mask;
  return STAGEML_OK;
}

extern "C" int stageml_stage_timer_read(float* ms_out, int32_t* counts_out, int n) {
  using namespace sb;
  for (const Rec& r : t_recs) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.b) != cudaSuccess || cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess)
      return set_error(STAGEML_ERR_CUDA, "stage timer: event query failed");
    if (r.stage >= 0 && r.stage < n) {
      if (ms_out) ms_out[r.stage] += ms;
      if (counts_out) counts_out[r.stage] += 1;
    }
    t_pool.push_back(r.a);
    t_pool.push_back(r.b);
  }
  t_recs.clear();
  return STAGEML_OK;
}
