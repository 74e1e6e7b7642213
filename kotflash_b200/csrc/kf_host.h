// Host-side helpers shared by the C-ABI translation units: thread-local error
// text, argument checks, and TMA tensor-map encoding through the driver entry
// point (so the library needs no link-time dependency on libcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/kotflash_b200.h"

namespace kf {

int set_error(int code, const char* fmt, ...);

// Returns KF_ERR_CUDA (and records the message) if the last launch failed.
int check_launch(const char* what);

// Encode a 4-D tiled TMA descriptor over a 16-bit [n0,n1,n2,n3] view whose
// innermost dimension (n3) is contiguous.  The box is (box_inner along n3,
// box_rows along n2, 1, 1) with 128-byte swizzle; out-of-range elements read
// as zero.  Returns KF_OK or an error code with the message recorded.
int encode_tmap_4d(CUtensorMap* map, const kf_tensor4* t, int box_inner, int box_rows);

// Encode a 2-D tiled TMA descriptor over a row-major fp32 matrix
// [rows][cols] (cols contiguous) with a (box_cols x box_rows) box and 128-byte
// swizzle (box_cols * 4 must be <= 128).
int encode_tmap_2d_f32(CUtensorMap* map, void* ptr, int64_t rows, int64_t cols, int box_cols,
                       int box_rows);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count_current_device();

// Makes the GPU that owns `ptr` the current device for the guard's lifetime
// and restores the caller's device afterwards, so an entry point launches,
// encodes tensor maps and reads device properties on the tensor's own GPU
// whatever device the calling thread has current (the C-ABI counterpart of
// the reference extension's c10::cuda::CUDAGuard on its cache tensor,
// kotflash/csrc/kv_append_cuda.cu:77).  A pointer the runtime does not know
// (host memory, null) leaves the current device alone.  status() is KF_OK or
// KF_ERR_CUDA with the message recorded.
class DeviceGuard {
 public:
  explicit DeviceGuard(const void* ptr);
  ~DeviceGuard();
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
  int status() const { return rc_; }

 private:
  int prev_ = -1;
  bool switched_ = false;
  int rc_ = 0;
};

}  // namespace kf
