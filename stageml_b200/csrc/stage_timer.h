// Optional per-stage CUDA-event timing of the pipeline entry points.
#pragma once
#include <cuda_runtime.h>

namespace sb {

// True while the calling thread has the timer enabled and `stage` selected.
bool stage_timer_on(int stage);
void stage_timer_record(int stage, cudaStream_t stream, bool begin);

// Records a begin event on construction and an end event on destruction
// (only while the calling thread has the timer enabled for this stage).
struct StageScope {
  int stage;
  cudaStream_t stream;
  bool on;
  StageScope(int s, cudaStream_t st) : stage(s), stream(st), on(stage_timer_on(s)) {
    if (on) stage_timer_record(stage, stream, true);
  }
  ~StageScope() {
    if (on) stage_timer_record(stage, stream, false);
  }
};

}  // namespace sb
