// Host-side plumbing shared by the C-ABI entry points: per-thread error
// messages, a per-device attribute cache, and small launch helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "hp_rms_norm_b200.h"

namespace hprn {

// Records `msg` as this thread's last error and returns `status`.
int fail(int status, const std::string& msg);
// Clears this thread's last error and returns HPRN_OK.
int ok();

// Attributes of one CUDA device, read once per device and cached.
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  int max_threads_per_sm = 0;
  int regs_per_sm = 0;
  size_t smem_per_sm = 0;
  size_t smem_per_block_optin = 0;
  size_t l2_bytes = 0;
};

// Info for the calling thread's current device; returns HPRN_OK or an error
// status (with the message recorded) when the device is not an sm_100 part.
int current_device(const DeviceInfo** out);

inline bool aligned(const void* p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(bytes)) == 0;
}

// Reports a failed launch (cudaGetLastError after the launch) as HPRN_ERR_CUDA.
int check_launch(const char* what);

}  // namespace hprn
