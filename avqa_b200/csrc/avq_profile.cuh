// Optional per-kernel device timing: when enabled (avq_profile_begin), every
// launch wrapped in AVQ_TIMED records a CUDA event pair on its stream; the
// host reads the accumulated durations per kernel after the stream work is
// done (avq_profile_end).  Disabled by default: no events are recorded.
#pragma once

#include <cuda_runtime.h>

namespace avq {

struct ProfileScope {
  const char* name;
  cudaStream_t st;
  cudaEvent_t e0;
  bool on;
  ProfileScope(const char* n, cudaStream_t s);
  ~ProfileScope();
};

}  // namespace avq

#define AVQ_TIMED(name, st) ::avq::ProfileScope _avq_prof_scope_(name, st)
