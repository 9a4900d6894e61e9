// hs_abi_ctx.h — the opaque hs_ctx behind include/headshot_cuda.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>
#include <vector>

#include "../../include/headshot_cuda.h"

// One bracketed kernel launch recorded while profiling is on.
struct hs_prof_rec {
  std::string kernel;
  cudaEvent_t start;
  cudaEvent_t stop;
};

struct hs_ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;       // owned
  cudaStream_t user_stream = nullptr;  // borrowed (hs_ctx_set_stream); may be the legacy stream 0
  bool has_user_stream = false;
  int* d_status = nullptr;             // device status word: first bounded-wait site that timed out
  uint32_t* d_sched = nullptr;         // attention work counter pair (d_status + 2), zero between launches
  unsigned int* d_norm2 = nullptr;     // q'/k' max squared row norms (d_status + 4), zero between launches
  void* scratch = nullptr;             // normalised/rotated K (and 16-bit V for f32 callers)
  size_t scratch_bytes = 0;
  uint32_t wait_timeout_ms = 2000;
  std::atomic<int> cancel{0};
  bool prof_on = false;
  std::vector<hs_prof_rec> prof;     // recorded launches, oldest first
  std::vector<cudaEvent_t> prof_free;  // recycled events
};

namespace hs {
// Brackets one kernel launch with events when profiling is on.
struct ProfScope {
  hs_ctx* ctx;
  cudaStream_t st;
  const char* name;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  ProfScope(hs_ctx* c, cudaStream_t s, const char* n);
  ~ProfScope();
};
}  // namespace hs

namespace hs {
hs_status abi_fail(hs_status s, const std::string& msg);
hs_status abi_cuda_fail(cudaError_t e, const char* what);
cudaStream_t ctx_stream(hs_ctx* ctx);
uint64_t ctx_timeout_ns(hs_ctx* ctx);
hs_status ctx_scratch(hs_ctx* ctx, size_t bytes, void** out);
}  // namespace hs
