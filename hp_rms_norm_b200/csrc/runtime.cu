// Host-side plumbing for the C ABI: errors, device cache, version.
#include <mutex>
#include <string>

#include "runtime.cuh"

namespace hprn {

namespace {
thread_local std::string t_last_error;

constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::once_flag g_device_once[kMaxDevices];
int g_device_status[kMaxDevices];
std::string g_device_msg[kMaxDevices];

void probe_device(int dev) {
  DeviceInfo& d = g_devices[dev];
  d.device = dev;
  int v = 0;
  cudaError_t e = cudaSuccess;
  auto get = [&](cudaDeviceAttr a, int* out) {
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(out, a, dev);
  };
  get(cudaDevAttrMultiProcessorCount, &d.sm_count);
  get(cudaDevAttrComputeCapabilityMajor, &d.cc_major);
  get(cudaDevAttrComputeCapabilityMinor, &d.cc_minor);
  get(cudaDevAttrMaxThreadsPerMultiProcessor, &d.max_threads_per_sm);
  get(cudaDevAttrMaxRegistersPerMultiprocessor, &d.regs_per_sm);
  get(cudaDevAttrMaxSharedMemoryPerMultiprocessor, &v);
  d.smem_per_sm = static_cast<size_t>(v);
  get(cudaDevAttrMaxSharedMemoryPerBlockOptin, &v);
  d.smem_per_block_optin = static_cast<size_t>(v);
  get(cudaDevAttrL2CacheSize, &v);
  d.l2_bytes = static_cast<size_t>(v);
  if (e != cudaSuccess) {
    g_device_status[dev] = HPRN_ERR_CUDA;
    g_device_msg[dev] = std::string("cudaDeviceGetAttribute failed: ") + cudaGetErrorString(e);
    return;
  }
  // The library ships sm_100a code only, which loads on compute capability 10.0.
  if (d.cc_major != 10 || d.cc_minor != 0) {
    g_device_status[dev] = HPRN_ERR_UNSUPPORTED_DEVICE;
    g_device_msg[dev] = "hp_rms_norm_b200 is built for sm_100a (compute capability 10.0); device " +
                        std::to_string(dev) + " is " + std::to_string(d.cc_major) + "." +
                        std::to_string(d.cc_minor);
    return;
  }
  g_device_status[dev] = HPRN_OK;
}
}  // namespace

int fail(int status, const std::string& msg) {
  t_last_error = msg;
  return status;
}

int ok() {
  t_last_error.clear();
  return HPRN_OK;
}

int current_device(const DeviceInfo** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(HPRN_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(HPRN_ERR_CUDA, "device index out of range");
  std::call_once(g_device_once[dev], probe_device, dev);
  if (g_device_status[dev] != HPRN_OK) return fail(g_device_status[dev], g_device_msg[dev]);
  *out = &g_devices[dev];
  return HPRN_OK;
}

int resident_ctas_per_sm(const DeviceInfo* dev, const void* fn, int threads, size_t smem) {
  struct Entry {
    int device;
    const void* fn;
    int threads;
    size_t smem;
    int ctas;
  };
  // A small per-thread cache in front of the shared table keeps the lock off
  // the launch path after a thread's first call with each kernel shape.
  constexpr int kLocal = 16;
  thread_local Entry local[kLocal] = {};
  const size_t slot = (reinterpret_cast<uintptr_t>(fn) / 16 + static_cast<size_t>(threads) +
                       static_cast<size_t>(dev->device) * 7) % kLocal;
  Entry& l = local[slot];
  if (l.fn == fn && l.device == dev->device && l.threads == threads && l.smem == smem)
    return l.ctas;
  static std::mutex mu;
  static Entry table[1024];
  static int used = 0;
  int ctas = -1;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (table[i].fn == fn && table[i].device == dev->device && table[i].threads == threads &&
          table[i].smem == smem) {
        ctas = table[i].ctas;
        break;
      }
    if (ctas < 0) {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas, fn, threads, smem) != cudaSuccess) {
        cudaGetLastError();  // the query's error is not the caller's
        return 0;
      }
      if (used < 1024) table[used++] = Entry{dev->device, fn, threads, smem, ctas};
    }
  }
  l = Entry{dev->device, fn, threads, smem, ctas};
  return ctas;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(HPRN_ERR_CUDA, std::string(what) + " launch failed: " + cudaGetErrorString(e));
  }
  return ok();
}

}  // namespace hprn

extern "C" {

const char* hprn_last_error(void) { return hprn::t_last_error.c_str(); }

const char* hprn_status_string(int status) {
  switch (status) {
    case HPRN_OK: return "HPRN_OK";
    case HPRN_ERR_INVALID_ARGUMENT: return "HPRN_ERR_INVALID_ARGUMENT";
    case HPRN_ERR_UNSUPPORTED_DTYPE: return "HPRN_ERR_UNSUPPORTED_DTYPE";
    case HPRN_ERR_UNSUPPORTED_DEVICE: return "HPRN_ERR_UNSUPPORTED_DEVICE";
    case HPRN_ERR_CUDA: return "HPRN_ERR_CUDA";
    default: return "HPRN_ERR_UNKNOWN";
  }
}

int hprn_version(void) { return HPRN_VERSION; }

}  // extern "C"
