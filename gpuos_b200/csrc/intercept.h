// intercept.h — scheduler_context's op intercept in C++ (intercept.cpp) and what it shares
// with the CPython binding (pyext.cpp).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "gpuos_b200.h"

namespace gpuos_py {

constexpr int kMaxDev = 64;

// ---- provided by pyext.cpp ----
// The device's runtime (nullptr if none, or while it shuts down).
gpuos_rt* runtime(int dev);
// Calls in flight on a runtime without the GIL; shutdown waits until none is left.
void busy_add(int dev, int delta);

// ---- provided by intercept.cpp ----
struct InterceptStats {
  int64_t scheduled = 0;
  int64_t fallbacks = 0;
  std::vector<std::pair<std::string, int64_t>> scheduled_ops;  // aten op name -> requests
  std::vector<std::pair<std::string, int64_t>> fallback_ops;   // aten op name -> calls left to PyTorch
};

// Route the calling thread's ATen calls through the intercept (counters and the pending set
// start empty).  False with *err set when the dispatcher key is taken by another library.
bool intercept_enable(int64_t size_threshold, std::string* err);
void intercept_disable();
bool intercept_enabled();
InterceptStats intercept_stats();
// The routing table: aten op name -> (kind: 1 binary, 2 unary, 3 parametric unary, 4 reduction,
// 5 top-k; element-wise or reduction op code).
std::vector<std::pair<std::string, std::pair<int, int>>> intercept_routes();
// Forget the storages of pending requests (after a synchronous flush of every device).
void intercept_clear_pending();

// Publish the device's pending requests (gpuos_rt_flush with `flags`, dependency `dep`) and tie
// the intercept's references to the flush ticket in one step, so that no request submitted
// meanwhile has its references tied to a flush that does not carry it.
int intercept_flush(int dev, gpuos_rt* rt, int flags, cudaStream_t dep, uint64_t* seq_out);
// Drop the references of flushes with ticket <= completed (outside every lock).
void intercept_release(int dev, uint64_t completed);
void intercept_release_all(int dev);

}  // namespace gpuos_py
