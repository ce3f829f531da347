// Fixed device scratch for callers that cannot allocate GPU memory.
//
// The bucketed backward sorts head-rows into spatial buckets and needs a
// bucket plan in device memory (msda_bucketed.cu). The regular entry points take
// it from the stream-ordered allocator. Some callers may not allocate at all:
// deployments that plan every byte of device memory before start-up and forbid
// allocation afterwards (automotive and other real-time inference runtimes),
// and plugin hosts that own the device memory and do not let a plugin call the
// CUDA allocator. For them, msda_backward_static_scratch (msda_capi.cpp) runs
// the same backward on the array below instead.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds kStaticScratchBytes of it until the process exits, and all
// calls on a device share it. Host code cannot use the symbol as a device
// pointer (in host code it names a host-side shadow), so the device address is
// looked up once per device with cudaGetSymbolAddress, with that device
// current, and cached.
#include <cuda_runtime.h>

#include <mutex>

#include "msda_kernels.h"

namespace msda {
namespace {

constexpr size_t kStaticScratchBytes = size_t{8} << 20;  // 8 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

}  // namespace

size_t static_scratch_capacity() { return kStaticScratchBytes; }

// Device address of the static scratch on the current device (set up on the
// first call per device).
cudaError_t static_scratch_address(void** out) {
  int device = -1;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_address[device] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (err != cudaSuccess) return err;
    g_scratch_address[device] = ptr;
  }
  *out = g_scratch_address[device];
  return cudaSuccess;
}

}  // namespace msda
