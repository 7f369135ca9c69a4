// Fused router: per token, top-k of the router logits and the softmax of the
// k selected logits (equivalently the full softmax renormalised over the top
// k), producing the topk_ids / topk_weights the MoE layer consumes.
//
// Semantics follow the reference's routing (bench/bench_moe.py:225-231:
// torch.topk(logits, k) -> ids in descending logit order, then
// torch.softmax over the k values, fp32).  Ties go to the lower expert id.
// One warp per token: the logit row is staged in shared memory, k rounds of
// warp-wide argmax select the experts, lane j < k then holds the j-th value.
// The weights are computed in double precision and rounded once to fp32.
#include <math.h>

#include "../../include/w4a16_moe_b200.h"
#include "launch.cuh"

namespace w4moe {

constexpr int kRouterWarps = 8;
constexpr int kRouterMaxE = 1024;
constexpr int kRouterMaxK = 32;

__global__ void __launch_bounds__(kRouterWarps * 32) topk_softmax_kernel(const float* logits, int M, int E,
                                                                         long long ld, int topk, float* weights,
                                                                         int32_t* ids) {
  extern __shared__ float rows[];  // [kRouterWarps][E]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* row = rows + (size_t)warp * E;
  for (int m = blockIdx.x * kRouterWarps + warp; m < M; m += gridDim.x * kRouterWarps) {
    for (int e = lane; e < E; e += 32) row[e] = logits[(size_t)m * ld + e];
    __syncwarp();
    float my_v = -INFINITY;
    int my_i = 0;
    for (int j = 0; j < topk; ++j) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        const float v = row[e];
        if (v > bv || (v == bv && e < bi)) {
          bv = v;
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == j) {
        my_v = bv;
        my_i = bi;
      }
      __syncwarp();
      if (lane == 0) row[bi] = -INFINITY;  // taken
      __syncwarp();
    }
    // softmax over the k selected values (the first is the largest), in
    // double precision and rounded once: within 1 ulp of the exact value
    const float vmax = __shfl_sync(0xffffffffu, my_v, 0);
    const double ex = lane < topk ? exp((double)my_v - (double)vmax) : 0.0;
    double sum = ex;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane < topk) {
      weights[(size_t)m * topk + lane] = (float)(ex / sum);
      ids[(size_t)m * topk + lane] = my_i;
    }
    __syncwarp();
  }
}

}  // namespace w4moe

using namespace w4moe;

extern "C" {

W4A16_API int w4a16_topk_softmax(const float* logits, int64_t M, int64_t E, int64_t logits_ld, int64_t topk,
                                 float* topk_weights, int32_t* topk_ids, void* stream) {
  if (M < 0 || E <= 0 || E > kRouterMaxE || logits_ld < E || topk <= 0 || topk > kRouterMaxK || topk > E)
    return report_error(kInvalidArgument, "w4a16_topk_softmax: need 0 < topk <= min(E, 32), E <= 1024, ld >= E");
  if (M == 0) return kOk;
  if (!logits || !topk_weights || !topk_ids) return report_error(kInvalidArgument, "w4a16_topk_softmax: null pointer");
  const long long blocks = (M + kRouterWarps - 1) / kRouterWarps;
  const int grid = (int)(blocks < 148 * 16 ? blocks : 148 * 16);
  const size_t smem = (size_t)kRouterWarps * E * sizeof(float);
  topk_softmax_kernel<<<grid, kRouterWarps * 32, smem, (cudaStream_t)stream>>>(logits, (int)M, (int)E, logits_ld,
                                                                               (int)topk, topk_weights, topk_ids);
  const cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? kOk : report_error(kCudaError, cudaGetErrorString(err));
}

}  // extern "C"
