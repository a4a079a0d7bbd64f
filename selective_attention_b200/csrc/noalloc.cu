// noalloc.cu - the SSD forward for callers that cannot allocate device memory.
//
// ssd_scan_fwd needs a workspace of ssd_scan_fwd_workspace_size() bytes that the
// caller allocates. Some callers cannot do that when they run the scan: a host
// whose device memory is fully reserved by another runtime's pool, or a caller
// whose hot path must not block on the device-wide synchronisation an allocation
// can imply. ssd_scan_fwd_noalloc gives them the same kernels with a fixed scratch
// array that is part of this library instead of a caller workspace.
//
// The array is a file-scope __device__ variable: every GPU that loads the library
// holds its SSD_NOALLOC_SCRATCH_BYTES until the process exits. Host code cannot use
// the variable's name as a device address, so its address is resolved with
// cudaGetSymbolAddress once per device, with that device current, on the first call
// on that device (that first call should come before any stream capture; a lookup that
// fails is not remembered, so a later call on that device tries again). All calls
// share the one array and it keeps the last call's contents; nothing in it needs to
// start at zero because every call writes each region before reading it. Calls that
// overlap on the GPU (other streams, other host threads) race on the array.
#include <mutex>

#include "kernels.h"

namespace {

static __device__ __align__(256) unsigned char g_ssd_noalloc_scratch[SSD_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
bool g_resolved[kMaxDevices];
void* g_scratch_addr[kMaxDevices];

// Device address of the scratch array on the current device. Only a successful lookup
// is cached: a lookup that failed (for instance one made while the stream was being
// captured) is tried again on the next call.
cudaError_t scratch_on_current_device(void** addr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_resolved[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ssd_noalloc_scratch);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();  // clear the failed lookup from the thread's last-error state
      return e;
    }
    g_scratch_addr[dev] = p;
    g_resolved[dev] = true;
  }
  *addr = g_scratch_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int ssd_scan_fwd_noalloc(const ssd_params* p, void* stream) {
  if (!p) return SSD_ERR_INVALID_ARGUMENT;
  const size_t need = ssd_scan_fwd_workspace_size(p);
  if (need == 0) return SSD_ERR_INVALID_ARGUMENT;
  if (need > (size_t)SSD_NOALLOC_SCRATCH_BYTES) return SSD_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (scratch_on_current_device(&scratch) != cudaSuccess) return SSD_ERR_CUDA;
  ssd_params q = *p;
  q.workspace = scratch;
  q.workspace_bytes = (size_t)SSD_NOALLOC_SCRATCH_BYTES;
  return ssd_scan_fwd(&q, stream);
}
