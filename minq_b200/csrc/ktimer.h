// Optional per-launch CUDA-event timing of one kernel family (diagnostic
// used by the benchmark to measure a kernel's launch durations inside the
// real decode step). Off unless minq_kernel_timer_start() named a family.
#pragma once

#include <cuda_runtime.h>

namespace minq {

enum KFamily { KF_NONE = 0, KF_QMATVEC = 1, KF_F32_MATVEC = 2, KF_ATTENTION = 3 };

// Returns true when launches of `fam` are being timed; then the caller
// brackets its launch with timer_before()/timer_after().
bool timer_active(KFamily fam);
void timer_before(cudaStream_t s);
void timer_after(cudaStream_t s, double bytes);

struct ScopedKTimer {
  bool on;
  cudaStream_t s;
  double bytes;
  ScopedKTimer(KFamily fam, cudaStream_t st, double b) : on(timer_active(fam)), s(st), bytes(b) {
    if (on) timer_before(s);
  }
  ~ScopedKTimer() {
    if (on) timer_after(s, bytes);
  }
};

}  // namespace minq
