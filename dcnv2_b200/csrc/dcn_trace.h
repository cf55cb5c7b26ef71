// Optional per-launch timing of the library's kernels with CUDA events recorded
// on the launch stream (enabled by dcn_trace_enable; off by default, zero cost
// when off).
#pragma once
#include <cuda_runtime.h>

namespace dcn {

enum TraceId {
  TR_PACK_INPUT = 0,
  TR_PACK_WEIGHT_FWD,
  TR_FORWARD,
  TR_PACK_WEIGHT_BWD,
  TR_ZERO_ACCUM,
  TR_BACKWARD_DATA,
  TR_BACKWARD_WEIGHT,
  TR_FINISH_GRAD_INPUT,
  TR_FINISH_GRAD_WEIGHT,
  TR_PACK_GRAD_OUTPUT,
  TR_BACKWARD_SCATTER,
  TR_COUNT
};

bool trace_on();

// Records an event pair around the enclosed launches when tracing is on.
class TraceScope {
 public:
  TraceScope(int id, cudaStream_t s);
  ~TraceScope();

 private:
  int id_;
  cudaStream_t s_;
  void* rec_;
};

}  // namespace dcn
