// Kernel timing hook shared by every entry point of the library: while
// enabled for one kernel family (lucid_profile_enable), each launch of that
// family is bracketed by a pair of CUDA events on its stream.
#pragma once
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

namespace lb {

// ---- kernel timing hook -----------------------------------------------------
struct Profiler {
  std::mutex mu;
  int kernel = 0;
  std::vector<cudaEvent_t> ev;  // start/stop pairs
  int used = 0;                 // pairs recorded
};
inline Profiler& profiler() {
  static Profiler p;
  return p;
}

// Brackets one launch with events when the hook is enabled for `kernel`.
struct ProfileScope {
  cudaEvent_t stop = nullptr;
  cudaStream_t st;
  ProfileScope(int kernel, cudaStream_t s) : st(s) {
    Profiler& p = profiler();
    std::lock_guard<std::mutex> g(p.mu);
    if (p.kernel != kernel || p.used >= 512) return;
    if ((int)p.ev.size() < 2 * (p.used + 1)) {
      cudaEvent_t a, b;
      if (cudaEventCreate(&a) != cudaSuccess) return;
      if (cudaEventCreate(&b) != cudaSuccess) { cudaEventDestroy(a); return; }
      p.ev.push_back(a);
      p.ev.push_back(b);
    }
    cudaEventRecord(p.ev[2 * p.used], st);
    stop = p.ev[2 * p.used + 1];
    ++p.used;
  }
  ~ProfileScope() {
    if (stop) cudaEventRecord(stop, st);
  }
};

}  // namespace lb
