// Expert-parallel token exchange: planning, packing and combining the rows a
// rank sends to / receives from the ranks that own the routed experts.
//
// The reference runs one GPU and has no expert parallelism; vLLM's EP contract
// (compressed_tensors_moe_wna16.py apply(): expert_map / global_num_experts)
// is the interface these kernels serve.  Rank r owns the contiguous experts
// [r * E / G, (r + 1) * E / G).  A token is sent once to every rank that owns
// at least one of its top-k experts (not once per slot); the receiving rank
// runs w4a16_moe_forward with its expert_map over the received rows and sends
// back one bf16 row per (token, rank), which the source sums in rank order.
//
//   plan    : per-token destination mask -> per-rank counts / offsets, the
//             rank-major send order (tokens ascending inside a rank) and
//             tok_row[m * G + r] = send row of (m, r) or -1;
//   pack    : gathers hidden rows, top-k ids and weights into the send order;
//   combine : out[m] = bf16(sum over r in order of fp32(back[tok_row[m, r]])),
//             zero rows for tokens routed nowhere.
#include <algorithm>

#include "../../include/w4a16_moe_b200.h"
#include "launch.cuh"

namespace w4moe {

constexpr int kEpPlanThreads = 1024;

__device__ __forceinline__ long long ep_id(const void* ids, int is64, long long i) {
  return is64 ? ((const int64_t*)ids)[i] : (long long)((const int32_t*)ids)[i];
}

// Single CTA: M is the per-rank source batch (thousands of tokens).
__global__ void __launch_bounds__(kEpPlanThreads, 1)
    ep_plan_kernel(const void* ids, int is64, int M, int topk, int E, int G, int32_t* counts, int32_t* offsets,
                   int32_t* send_tok, int32_t* tok_row) {
  __shared__ int warp_tot[33];
  __shared__ int s_base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = E / G;
  if (tid == 0) s_base = 0;
  __syncthreads();
  for (int r = 0; r < G; ++r) {
    for (int m0 = 0; m0 < M; m0 += kEpPlanThreads) {
      const int m = m0 + tid;
      int f = 0;
      if (m < M) {
        for (int t = 0; t < topk; ++t) {
          const long long e = ep_id(ids, is64, (long long)m * topk + t);
          if (e >= 0 && e < E && (int)(e / per) == r) f = 1;
        }
      }
      // block exclusive scan of f
      int incl = f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      if (lane == 31) warp_tot[warp] = incl;
      __syncthreads();
      if (warp == 0) {
        const int w = warp_tot[lane];
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int u = __shfl_up_sync(0xffffffffu, wi, o);
          if (lane >= o) wi += u;
        }
        warp_tot[lane] = wi - w;
        if (lane == 31) warp_tot[32] = wi;
      }
      __syncthreads();
      const int row = s_base + warp_tot[warp] + incl - f;
      if (m < M) {
        tok_row[(size_t)m * G + r] = f ? row : -1;
        if (f) send_tok[row] = m;
      }
      __syncthreads();
      if (tid == 0) s_base += warp_tot[32];
      __syncthreads();
    }
    if (tid == 0) {
      const int end = s_base;
      const int beg = r == 0 ? 0 : offsets[r];
      counts[r] = end - beg;
      offsets[r + 1] = end;
      if (r == 0) offsets[0] = 0;
    }
    __syncthreads();
  }
}

// Send-order gather of hidden rows (16-byte vectors) and of the per-row
// metadata meta[i] = [top-k ids (int32) | top-k weights (fp32 bits)].
__global__ void ep_pack_kernel(const __nv_bfloat16* x, long long x_ld, const void* ids, int is64, const float* w,
                               int topk, int H, const int32_t* offsets, int G, const int32_t* send_tok,
                               __nv_bfloat16* x_send, int32_t* meta) {
  const int n = offsets[G], h8 = H / 8;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < (long long)n * h8; idx += stride) {
    const int i = (int)(idx / h8), c = (int)(idx - (long long)i * h8) * 8;
    const int m = send_tok[i];
    *reinterpret_cast<uint4*>(x_send + (size_t)i * H + c) = *reinterpret_cast<const uint4*>(x + (size_t)m * x_ld + c);
  }
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < (long long)n * topk; idx += stride) {
    const int i = (int)(idx / topk), t = (int)(idx - (long long)i * topk);
    const long long src = (long long)send_tok[i] * topk + t;
    meta[(size_t)i * 2 * topk + t] = (int32_t)ep_id(ids, is64, src);
    meta[(size_t)i * 2 * topk + topk + t] = __float_as_int(w[src]);
  }
}

__global__ void ep_combine_kernel(const __nv_bfloat16* back, const int32_t* tok_row, int M, int G, int H,
                                  __nv_bfloat16* out) {
  const int h8 = H / 8;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < (long long)M * h8;
       idx += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(idx / h8), c = (int)(idx - (long long)m * h8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < G; ++r) {
      const int row = tok_row[(size_t)m * G + r];
      if (row < 0) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(back + (size_t)row * H + c);
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] += __uint_as_float(wv[i] << 16);
        acc[2 * i + 1] += __uint_as_float(wv[i] & 0xFFFF0000u);
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      ow[i] = *reinterpret_cast<uint32_t*>(&b2);
    }
    *reinterpret_cast<uint4*>(out + (size_t)m * H + c) = o;
  }
}


// ---- fixed-capacity dispatch (no host read of the counts) ----
// Every rank sends every rank a block of `cap` rows (cap >= the source batch,
// a token goes to a rank at most once): block r holds, in ascending token
// order, the tokens routed to rank r, then padding rows whose top-k ids are
// -1 (they route nowhere).  A row is [hidden (H bf16) | top-k ids (int32) |
// top-k weights (fp32 bits) | zero pad], row_stride bf16 elements, so one
// all-to-all with equal splits moves rows and routing together.

// Plan over a (token chunk, destination rank) grid: chunk c of kEpPlanThreads
// tokens.  Pass 1 counts the chunk's tokens routed to rank r; pass 2 adds the
// counts of the earlier chunks and scans inside the chunk (ascending tokens).
__device__ __forceinline__ int ep_routed_to(const void* ids, int is64, int m, int M, int topk, int E, int per,
                                            int r) {
  if (m >= M) return 0;
  for (int t = 0; t < topk; ++t) {
    const long long e = ep_id(ids, is64, (long long)m * topk + t);
    if (e >= 0 && e < E && (int)(e / per) == r) return 1;
  }
  return 0;
}

// Block-wide exclusive scan of f (kEpPlanThreads threads); returns the
// exclusive prefix, *total receives the block sum.
__device__ __forceinline__ int ep_block_scan(int f, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = warp_tot[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += u;
    }
    warp_tot[lane] = wi - w;
    if (lane == 31) warp_tot[32] = wi;
  }
  __syncthreads();
  *total = warp_tot[32];
  return warp_tot[warp] + incl - f;
}

__global__ void __launch_bounds__(kEpPlanThreads) ep_plan_fixed_count_kernel(const void* ids, int is64, int M,
                                                                             int topk, int E, int G,
                                                                             int32_t* chunk_counts) {
  __shared__ int warp_tot[33];
  const int c = blockIdx.x, r = blockIdx.y;
  const int f = ep_routed_to(ids, is64, c * kEpPlanThreads + threadIdx.x, M, topk, E, E / G, r);
  int total;
  ep_block_scan(f, warp_tot, &total);
  if (threadIdx.x == 0) chunk_counts[(size_t)r * gridDim.x + c] = total;
}

__global__ void __launch_bounds__(kEpPlanThreads) ep_plan_fixed_scatter_kernel(const void* ids, int is64, int M,
                                                                               int topk, int E, int G, int cap,
                                                                               const int32_t* chunk_counts,
                                                                               int32_t* counts, int32_t* send_tok,
                                                                               int32_t* tok_row) {
  __shared__ int warp_tot[33];
  __shared__ int s_base;
  const int c = blockIdx.x, r = blockIdx.y, nch = gridDim.x;
  if (threadIdx.x < 32) {  // counts of the earlier chunks of rank r
    int b = 0;
    for (int cc = threadIdx.x; cc < c; cc += 32) b += chunk_counts[(size_t)r * nch + cc];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) b += __shfl_xor_sync(0xffffffffu, b, o);
    if (threadIdx.x == 0) s_base = b;
  }
  const int m = c * kEpPlanThreads + threadIdx.x;
  const int f = ep_routed_to(ids, is64, m, M, topk, E, E / G, r);
  int total;
  const int ex = ep_block_scan(f, warp_tot, &total);  // its __syncthreads also publishes s_base
  const int pos = s_base + ex;
  if (m < M) {
    tok_row[(size_t)m * G + r] = f ? r * cap + pos : -1;
    if (f) send_tok[(size_t)r * cap + pos] = m;
  }
  if (c == nch - 1 && threadIdx.x == 0) counts[r] = s_base + total;
}

__global__ void ep_pack_fixed_kernel(const __nv_bfloat16* x, long long x_ld, const void* ids, int is64,
                                     const float* w, int topk, int H, int G, int cap, int rs,
                                     const int32_t* counts, const int32_t* send_tok, __nv_bfloat16* send) {
  const int v_per_row = rs / 8, h8 = H / 8;
  const long long total = (long long)G * cap * v_per_row;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(idx / v_per_row), v = (int)(idx - (long long)i * v_per_row);
    const int r = i / cap, j = i - r * cap;
    const bool valid = j < counts[r];
    uint4* dst = reinterpret_cast<uint4*>(send + (size_t)i * rs) + v;
    if (v < h8) {
      if (valid) *dst = *reinterpret_cast<const uint4*>(x + (size_t)send_tok[i] * x_ld + v * 8);
      continue;
    }
    // routing metadata: 4 int32 words per vector
    const int m = valid ? send_tok[i] : 0;
    uint32_t word[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int k = (v - h8) * 4 + q;
      uint32_t val = 0;
      if (k < topk) val = valid ? (uint32_t)(int32_t)ep_id(ids, is64, (long long)m * topk + k) : 0xFFFFFFFFu;
      else if (k < 2 * topk) val = valid ? (uint32_t)__float_as_int(w[(size_t)m * topk + k - topk]) : 0u;
      word[q] = val;
    }
    *dst = make_uint4(word[0], word[1], word[2], word[3]);
  }
}

static int grid_for(long long work, int threads) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long b = (work + threads - 1) / threads;
  return (int)std::max<long long>(1, std::min<long long>(b, (long long)sms * 8));
}

}  // namespace w4moe

using namespace w4moe;

extern "C" {

W4A16_API int w4a16_ep_plan(const void* topk_ids, int ids_is_int64, int64_t M, int64_t topk, int64_t num_experts,
                            int64_t n_ranks, int32_t* send_counts, int32_t* send_offsets, int32_t* send_tok,
                            int32_t* tok_row, void* stream) {
  if (M < 0 || topk <= 0 || n_ranks <= 0 || num_experts <= 0 || num_experts % n_ranks != 0 || M > (1 << 24))
    return report_error(kInvalidArgument, "w4a16_ep_plan: bad sizes (num_experts must divide evenly over ranks)");
  if ((M > 0 && !topk_ids) || !send_counts || !send_offsets || (M > 0 && (!send_tok || !tok_row)))
    return report_error(kInvalidArgument, "w4a16_ep_plan: null pointer");
  ep_plan_kernel<<<1, kEpPlanThreads, 0, (cudaStream_t)stream>>>(topk_ids, ids_is_int64, (int)M, (int)topk,
                                                                   (int)num_experts, (int)n_ranks, send_counts,
                                                                   send_offsets, send_tok, tok_row);
  const cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? kOk : report_error(kCudaError, cudaGetErrorString(err));
}

W4A16_API int w4a16_ep_pack(const void* hidden, int64_t hidden_ld, const void* topk_ids, int ids_is_int64,
                            const float* topk_weights, int64_t M, int64_t topk, int64_t H, int64_t n_ranks,
                            const int32_t* send_offsets, const int32_t* send_tok, void* x_send, int32_t* meta_send,
                            void* stream) {
  if (M < 0 || topk <= 0 || H <= 0 || H % 8 != 0 || hidden_ld < H || n_ranks <= 0)
    return report_error(kInvalidArgument, "w4a16_ep_pack: bad sizes (H % 8 == 0, hidden_ld >= H)");
  if (M == 0) return kOk;
  if (!hidden || !topk_ids || !topk_weights || !send_offsets || !send_tok || !x_send || !meta_send)
    return report_error(kInvalidArgument, "w4a16_ep_pack: null pointer");
  const long long work = M * n_ranks * (H / 8);
  ep_pack_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)hidden, hidden_ld, topk_ids, ids_is_int64, topk_weights, (int)topk, (int)H, send_offsets,
      (int)n_ranks, send_tok, (__nv_bfloat16*)x_send, meta_send);
  const cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? kOk : report_error(kCudaError, cudaGetErrorString(err));
}


W4A16_API int w4a16_ep_dispatch_fixed(const void* hidden, int64_t hidden_ld, const void* topk_ids, int ids_is_int64,
                                      const float* topk_weights, int64_t M, int64_t topk, int64_t num_experts,
                                      int64_t H, int64_t n_ranks, int64_t capacity, int64_t row_stride,
                                      void* send_rows, int32_t* send_counts, int32_t* send_tok, int32_t* tok_row,
                                      void* stream) {
  if (M < 0 || topk <= 0 || H <= 0 || H % 8 != 0 || hidden_ld < H || n_ranks <= 0 || num_experts <= 0 ||
      num_experts % n_ranks != 0 || capacity < M || capacity > (1 << 24) ||
      row_stride < H + 4 * topk || row_stride % 8 != 0)
    return report_error(kInvalidArgument,
                        "w4a16_ep_dispatch_fixed: bad sizes (H % 8 == 0, capacity >= M, row_stride >= H + 4*topk "
                        "and a multiple of 8, num_experts divisible by n_ranks)");
  if ((M > 0 && (!hidden || !topk_ids || !topk_weights || !tok_row)) || !send_rows || !send_counts || !send_tok)
    return report_error(kInvalidArgument, "w4a16_ep_dispatch_fixed: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int nch = (int)((M + kEpPlanThreads - 1) / kEpPlanThreads);
  if (nch > 0) {
    int32_t* chunk_counts = send_counts + n_ranks;  // scratch tail of the counts buffer
    const dim3 grid(nch, (unsigned)n_ranks);
    ep_plan_fixed_count_kernel<<<grid, kEpPlanThreads, 0, st>>>(topk_ids, ids_is_int64, (int)M, (int)topk,
                                                                 (int)num_experts, (int)n_ranks, chunk_counts);
    ep_plan_fixed_scatter_kernel<<<grid, kEpPlanThreads, 0, st>>>(topk_ids, ids_is_int64, (int)M, (int)topk,
                                                                   (int)num_experts, (int)n_ranks, (int)capacity,
                                                                   chunk_counts, send_counts, send_tok, tok_row);
  } else {
    cudaError_t e0 = cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * n_ranks, st);
    if (e0 != cudaSuccess) return report_error(kCudaError, cudaGetErrorString(e0));
  }
  const long long work = n_ranks * capacity * (row_stride / 8);
  ep_pack_fixed_kernel<<<grid_for(work, 256), 256, 0, st>>>(
      (const __nv_bfloat16*)hidden, hidden_ld, topk_ids, ids_is_int64, topk_weights, (int)topk, (int)H,
      (int)n_ranks, (int)capacity, (int)row_stride, send_counts, send_tok, (__nv_bfloat16*)send_rows);
  const cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? kOk : report_error(kCudaError, cudaGetErrorString(err));
}

W4A16_API int w4a16_ep_combine(const void* back, const int32_t* tok_row, int64_t M, int64_t n_ranks, int64_t H,
                               void* out, void* stream) {
  if (M < 0 || n_ranks <= 0 || H <= 0 || H % 8 != 0)
    return report_error(kInvalidArgument, "w4a16_ep_combine: bad sizes (H % 8 == 0)");
  if (M == 0) return kOk;
  if (!back || !tok_row || !out) return report_error(kInvalidArgument, "w4a16_ep_combine: null pointer");
  ep_combine_kernel<<<grid_for(M * (H / 8), 256), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)back, tok_row, (int)M, (int)n_ranks, (int)H, (__nv_bfloat16*)out);
  const cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? kOk : report_error(kCudaError, cudaGetErrorString(err));
}

}  // extern "C"
