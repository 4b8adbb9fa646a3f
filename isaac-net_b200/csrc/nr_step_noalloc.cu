// inb_nr_step_noalloc: the control step for hosts that cannot hand the library a scratch buffer.
//
// Its one scratch, the per-slot fading-gain rows, lives in a fixed array of this translation unit's device image.
// This file holds no kernel, so under CUDA's lazy module loading (the default) its module, and with it the 128 MiB
// array, is loaded on a device only when the first inb_nr_step_noalloc call there resolves the array's address;
// processes that only call inb_nr_step never reserve it.
#include <mutex>

#include "nr_step_entry.cuh"

namespace inb {
// Gain rows of inb_nr_step_noalloc, one array per device the library runs on.  Its contents need no initial value:
// the fading launch of a step writes every row the MAC launch of that step reads.
static __device__ __align__(256) float g_gain_scratch[INB_NOALLOC_GAIN_MAX];
constexpr int kMaxDevices = 64;
static float* g_scratch_addr[kMaxDevices];
static std::mutex g_scratch_mu;

// The device address of g_gain_scratch on the current device (host code cannot use the symbol itself: on the host it
// names a stand-in, not device memory).  Resolved once per device, under a lock.
static int scratch_of_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -8;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gain_scratch) != cudaSuccess || p == nullptr) return -9;
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return 0;
}
}  // namespace inb

extern "C" int inb_nr_step_noalloc(const InbStepArgs* args, void* cuda_stream) {
  if (args == nullptr) return -1;
  if (args->p.E <= 0) return 0;
  long long need = 0;
  const int rc = inb::check_args(*args, &need);
  if (rc != 0) return rc;
  InbStepArgs a = *args;
  if (inb::uses_gain_rows(a.phases)) {   // a radio-only call (phases == 1) touches no gain row
    if (need > (long long)INB_NOALLOC_GAIN_MAX) return -10;
    float* scratch = nullptr;
    const int sr = inb::scratch_of_current_device(&scratch);
    if (sr != 0) return sr;
    a.gain = scratch;
    a.gain_cap = INB_NOALLOC_GAIN_MAX;
  }
  return inb::launch_all(a, (cudaStream_t)cuda_stream, nullptr);
}
