// Allocation-free variant of w4a16_moe_forward.
//
// Some callers cannot allocate device memory at the point where they run the
// MoE layer: code that runs under another framework's memory pool or
// allocator hooks (where a stray cudaMalloc would bypass or break the pool's
// accounting), plug-in hosts whose rules forbid allocation on the hot path,
// and early-initialisation or error-handling paths where allocating is unsafe.
// They can still pass inputs and outputs, but not a workspace.  This entry
// point keeps its scratch in a fixed, statically sized device array compiled
// into the library, so a call allocates nothing.
//
// Costs and limits:
//   * every GPU that loads the library holds kNoAllocScratchBytes (16 MiB)
//     of device memory for the array until the process exits;
//   * shapes whose workspace (w4a16_moe_workspace_size) exceeds that are
//     rejected with status 2 and a message; decode-sized batches of the
//     256-expert / 3072 x 1024 layer fit (M*topk up to ~650 slots);
//   * all calls on one device share the array, which keeps the last call's
//     contents: each call clears the counters it needs at zero, and calls
//     that may overlap on the GPU (unordered streams) race on the array and
//     corrupt each other's results;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress; make that first call before any stream capture.
#include <mutex>

#include "../../include/w4a16_moe_b200.h"
#include "launch.cuh"

namespace w4moe {

constexpr int64_t kNoAllocScratchBytes = 16ll << 20;

// Host code must not use this name as a pointer: on the host it only stands
// for the symbol.  Its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};  // device address of g_noalloc_scratch, per device

// Device address of the scratch array on the current device (looked up once
// per device, with that device current).
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess) return err;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace w4moe

using namespace w4moe;

extern "C" {

int64_t w4a16_moe_noalloc_max_workspace(void) { return kNoAllocScratchBytes; }

int w4a16_moe_forward_noalloc(const void* hidden, int64_t M, int64_t H, int64_t hidden_ld,
                              const void* w13_rep, const void* s13_rep, const void* w2_rep,
                              const void* s2_rep, int64_t E, int64_t I, const float* topk_weights,
                              const void* topk_ids, int ids_is_int64, int64_t topk,
                              const int32_t* expert_map, int64_t global_num_experts, void* out,
                              void* stream) {
  const int64_t need = w4a16_moe_workspace_size(M, topk, E, H, I);
  if (need < 0)
    return report_error(1, "w4a16_moe_forward_noalloc: bad sizes (M, topk, E, H, I)");
  if (need > kNoAllocScratchBytes)
    return report_error(2, "w4a16_moe_forward_noalloc: this shape needs a workspace larger than the "
                           "16 MiB static scratch; use w4a16_moe_forward with a caller workspace");
  void* scratch = nullptr;
  cudaError_t err = noalloc_scratch(&scratch);
  if (err != cudaSuccess)
    return report_error(3, "w4a16_moe_forward_noalloc: cudaGetSymbolAddress of the scratch array failed");
  // The array holds whatever the previous call (of any shape) left there:
  // clear the counters this shape expects to find at zero.
  const int64_t zero_bytes = workspace_zero_prefix_bytes(M, topk, E, H, I);
  if (M > 0 && zero_bytes > 0) {
    err = cudaMemsetAsync(scratch, 0, (size_t)zero_bytes, (cudaStream_t)stream);
    if (err != cudaSuccess) return report_error(3, "w4a16_moe_forward_noalloc: clearing the scratch failed");
  }
  return w4a16_moe_forward(hidden, M, H, hidden_ld, w13_rep, s13_rep, w2_rep, s2_rep, E, I,
                           topk_weights, topk_ids, ids_is_int64, topk, expert_map,
                           global_num_experts, out, scratch, kNoAllocScratchBytes, stream);
}

// Error bits of the last w4a16_moe_forward_noalloc call of this shape on the
// current device (bounded device waits that ran out), read from the static
// scratch and then cleared.  Synchronises `stream`.
int w4a16_moe_noalloc_read_status(int64_t M, int64_t topk, int64_t E, int64_t H, int64_t I, int32_t* status_out,
                                  void* stream) {
  if (w4a16_moe_workspace_size(M, topk, E, H, I) < 0)
    return report_error(1, "w4a16_moe_noalloc_read_status: bad sizes (M, topk, E, H, I)");
  void* scratch = nullptr;
  if (noalloc_scratch(&scratch) != cudaSuccess)
    return report_error(3, "w4a16_moe_noalloc_read_status: cudaGetSymbolAddress of the scratch array failed");
  return w4a16_moe_read_status(scratch, M, topk, E, H, I, status_out, stream);
}

}  // extern "C"
