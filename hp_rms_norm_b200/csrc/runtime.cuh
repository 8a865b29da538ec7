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

// CTAs of kernel `fn` that one SM of `dev` holds at once at `threads`
// threads and `smem` bytes of dynamic shared memory
// (cudaOccupancyMaxActiveBlocksPerMultiprocessor), cached per (device,
// kernel, threads, smem); 0 when the query fails.
int resident_ctas_per_sm(const DeviceInfo* dev, const void* fn, int threads, size_t smem);

// How many leading CTAs of a grid of kernel `fn` (at `threads` threads, no
// dynamic shared memory) are resident at launch, i.e. the first wave:
// resident CTAs per SM x SMs.  The kernels prefetch their first rows into L2
// ahead of the programmatic-launch wait in those CTAs only (later CTAs start
// after the preceding grid is done, so a prefetch would only repeat the
// loads' own requests).  0 when the occupancy query fails: no prefetch.
inline int64_t first_wave_ctas(const DeviceInfo* dev, const void* fn, int threads) {
  return static_cast<int64_t>(resident_ctas_per_sm(dev, fn, threads, 0)) * dev->sm_count;
}

inline bool aligned(const void* p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(bytes)) == 0;
}

// Reports a failed launch (cudaGetLastError after the launch) as HPRN_ERR_CUDA.
int check_launch(const char* what);

}  // namespace hprn
