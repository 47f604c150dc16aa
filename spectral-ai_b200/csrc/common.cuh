// common.cuh — host-side helpers shared by the library's translation units:
// error reporting, CUDA checks, tensor-map creation and device properties.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <string>

#include "../../include/spectral_b200.h"

namespace sb {

// Records the calling thread's last error message and returns `code`.
int fail(int code, const char* fmt, ...);

#define SB_CUDA_TRY(expr)                                                              \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    if (_e != cudaSuccess)                                                             \
      return ::sb::fail(SB_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                   \
                        cudaGetErrorString(_e), __FILE__, __LINE__);                   \
  } while (0)

#define SB_REQUIRE(cond, ...)                                                          \
  do {                                                                                 \
    if (!(cond)) return ::sb::fail(SB_ERR_INVALID, __VA_ARGS__);                       \
  } while (0)

// Number of SMs of the current device (cached per device).
int num_sms();

// 2-D tiled tensor map over a row-major [rows, cols] matrix of `elem_bytes`
// elements with a box of box_cols x box_rows and the given swizzle.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 int elem_bytes, uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                 uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// One-time set-up per device for one call site (kernel attributes, occupancy
// queries): the first caller on a device runs `fn` under the object's lock,
// concurrent first callers wait for it, and later callers only read an
// atomic flag.  `value[dev]` keeps an int that `fn` may store (it is read
// after once() returned SB_OK, which orders it after the store).
struct PerDevice {
  static constexpr int kMaxDevices = 64;
  int value[kMaxDevices] = {};
  template <typename F>
  int once(int dev, F&& fn) {
    if (dev < 0 || dev >= kMaxDevices) return fail(SB_ERR_CUDA, "device ordinal %d out of range", dev);
    if (done_[dev].load(std::memory_order_acquire)) return SB_OK;
    std::lock_guard<std::mutex> g(mu_);
    if (done_[dev].load(std::memory_order_relaxed)) return SB_OK;
    const int rc = fn();
    if (rc == SB_OK) done_[dev].store(true, std::memory_order_release);
    return rc;
  }

 private:
  std::mutex mu_;
  std::atomic<bool> done_[kMaxDevices] = {};
};

// Per-kernel CUDA-event timing (off by default).  A ProfScope records an event
// pair around one launch on its stream; sb_profile_count()/sb_profile_entry()
// resolve them.
bool prof_enabled();
void prof_record(const char* name, cudaEvent_t start, cudaEvent_t stop);
cudaEvent_t prof_event();

struct ProfScope {
  const char* name;
  cudaStream_t stream;
  cudaEvent_t start = nullptr;
  ProfScope(const char* n, cudaStream_t s) : name(n), stream(s) {
    if (prof_enabled()) {
      start = prof_event();
      if (start) cudaEventRecord(start, stream);
    }
  }
  ~ProfScope() {
    if (start) {
      cudaEvent_t stop = prof_event();
      if (stop) {
        cudaEventRecord(stop, stream);
        prof_record(name, start, stop);
      }
    }
  }
};

}  // namespace sb
