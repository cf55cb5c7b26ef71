// dcn_forward_noalloc: the forward pass for callers that cannot allocate GPU
// memory.  Some hosts run the operator where no allocator may be called: code
// that runs while a stream is being recorded into a graph by a framework that
// forbids allocation there, real-time or embedded runtimes whose memory is fixed
// at start-up, and plugins handed only input and output buffers by a host that
// owns every allocation.  Such callers cannot provide dcn_forward's workspace,
// so this entry point takes its scratch from one fixed array in the library's
// own device memory instead.
//
// The array lives for as long as the library is loaded, on every GPU that uses
// this entry point, and is shared by all calls: calls that overlap on the GPU
// (different streams, or different host threads on one device) race on it and
// must be serialised by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "dcn_b200.h"

namespace {

// Scratch of the forward pass: packed input, packed weight tiles and the
// device status word.  Its size is the limit on problems this entry point takes.
static __device__ __align__(256) unsigned char g_forward_scratch[DCN_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices];  // device address of g_forward_scratch per device

// Device address of the scratch array on the current device.  Host code cannot
// use the array's name as a pointer (it names a host-side stand-in), so the
// address is asked from the runtime once per device, with that device current.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DCN_E_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_forward_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // clear the error so later runtime calls do not report it
      return DCN_E_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return DCN_OK;
}

}  // namespace

extern "C" {

int dcn_forward_noalloc(const dcn_desc* d, const void* input, const void* weight,
                        const void* mask, const void* offset, const void* bias, void* output,
                        void* stream) {
  if (d == nullptr) return DCN_E_NULLPTR;
  const size_t need = dcn_forward_workspace_size(d);
  if (need == 0) return DCN_E_INVALID;
  if (need > (size_t)DCN_NOALLOC_SCRATCH_BYTES) return DCN_E_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != DCN_OK) return rc;
  // dcn_forward clears the status word and overwrites every byte of packed
  // input and weight it reads, so nothing left by an earlier call is used; the
  // reuse flags do not apply to the shared scratch and are ignored.
  dcn_desc dd = *d;
  dd.flags = 0;
  return dcn_forward(&dd, input, weight, mask, offset, bias, output, scratch,
                     (size_t)DCN_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
