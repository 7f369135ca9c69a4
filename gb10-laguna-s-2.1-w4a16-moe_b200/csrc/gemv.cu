// Small-M grouped GEMM ("decode" path) for both MoE projections.
//
// Work item = (active expert, output row block).  All of the expert's routed
// slots are processed against one streamed pass of its weights, so every
// weight byte leaves HBM once per call.  The 8 warps of a CTA split the
// K dimension (chunk c goes to warp c % 8); weights are decoded straight from
// coalesced 16-byte loads into m16n8k16 A fragments (no shared-memory staging:
// the fragment-major layout in common.cuh makes each lane's 16 bytes exactly
// its four A fragments), activations (<= 8*NG slots per pass) are the B
// operand, and partial sums are reduced across warps in shared memory.
//
//   MODE 0 (w13): rows = gate tile p and up tile p + I/16; epilogue writes
//                 bf16(silu(gate) * up) to inter[slot, I]
//                 (reference: _w4a16_moe_w1_fused_kernel,
//                  kernels/w4a16_moe.py:374-499).
//   MODE 1 (w2):  rows = 32 consecutive hidden rows; epilogue scales by the
//                 router weight, writes fp32 partial[slot, H], and the last of
//                 a token's slots to finish a row block sums that token's
//                 partials in slot order and writes bf16 out[m, H].
//                 Deterministic; replaces _w4a16_moe_w2_kernel + _moe_sum_kernel
//                 (kernels/w4a16_moe.py:502-670).
#include "launch.cuh"

namespace w4moe {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvUnroll = 3;  // chunks in flight per warp

__device__ __forceinline__ uint32_t lo_bcast(uint32_t v) { return __byte_perm(v, 0, 0x1010); }
__device__ __forceinline__ uint32_t hi_bcast(uint32_t v) { return __byte_perm(v, 0, 0x3232); }

__device__ __forceinline__ uint32_t ldg_b32(const __nv_bfloat16* p) {
  return __ldg(reinterpret_cast<const unsigned int*>(p));
}

template <int MODE, int NG>
__global__ void __launch_bounds__(kGemvThreads, 2) moe_gemv_kernel(GemvParams p) {
  __shared__ float red[kGemvWarps][NG][2][128];
  __shared__ int s_slot[8 * NG];
  __shared__ int s_last[8 * NG];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int ipe = p.items_per_expert;
  const int n_items = p.rt.num_active[0] * ipe;

  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int j = item / ipe, qi = item - j * ipe;
    const int e = p.rt.active[j];
    const int T = p.rt.counts[e];
    const int base = p.rt.offsets[e];
    const int rt0 = (MODE == 0) ? qi : 2 * qi;
    const int rt1 = (MODE == 0) ? qi + ipe : 2 * qi + 1;
    const size_t blk0 = ((size_t)e * p.n_rowtiles + rt0) * p.n_chunks;
    const size_t blk1 = ((size_t)e * p.n_rowtiles + rt1) * p.n_chunks;
    const uint4* w0 = p.w + blk0 * 32 + lane;
    const uint4* w1 = p.w + blk1 * 32 + lane;
    const uint2* s0 = p.s + blk0 * 8 + g;
    const uint2* s1 = p.s + blk1 * 8 + g;

    for (int tp = 0; tp < T; tp += 8 * NG) {
      const __nv_bfloat16* xr[NG];
#pragma unroll
      for (int q = 0; q < NG; ++q) {
        const int idx = tp + q * 8 + g;
        xr[q] = nullptr;
        if (idx < T) {
          const int slot = p.rt.sorted[base + idx];
          xr[q] = p.x + (long long)(slot / p.x_row_div) * p.x_ld + 2 * t;
        }
      }
      float acc[NG][2][4];
#pragma unroll
      for (int q = 0; q < NG; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[q][h][i] = 0.f;

      for (int c0 = warp; c0 < p.n_chunks; c0 += kGemvWarps * kGemvUnroll) {
        uint4 wa[kGemvUnroll], wb[kGemvUnroll];
        uint2 sa[kGemvUnroll], sb[kGemvUnroll];
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
          const int c = c0 + u * kGemvWarps;
          if (c < p.n_chunks) {
            wa[u] = ldg_stream(w0 + (size_t)c * 32);
            wb[u] = ldg_stream(w1 + (size_t)c * 32);
            sa[u] = ldg_stream2(s0 + (size_t)c * 8);
            sb[u] = ldg_stream2(s1 + (size_t)c * 8);
          }
        }
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
          const int c = c0 + u * kGemvWarps;
          if (c >= p.n_chunks) break;
          const uint32_t wav[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
          const uint32_t wbv[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const uint32_t sav = (jj < 2) ? sa[u].x : sa[u].y;
            const uint32_t sbv = (jj < 2) ? sb[u].x : sb[u].y;
            uint32_t A0[4], A1[4];
            dequant_word(wav[jj], lo_bcast(sav), hi_bcast(sav), A0);
            dequant_word(wbv[jj], lo_bcast(sbv), hi_bcast(sbv), A1);
            const int koff = c * kChunkK + jj * 16;
#pragma unroll
            for (int q = 0; q < NG; ++q) {
              uint32_t b0 = 0, b1 = 0;
              if (xr[q] != nullptr) {
                b0 = ldg_b32(xr[q] + koff);
                b1 = ldg_b32(xr[q] + koff + 8);
              }
              mma_bf16_16816(acc[q][0], A0, b0, b1);
              mma_bf16_16816(acc[q][1], A1, b0, b1);
            }
          }
        }
      }

      // Cross-warp reduction of the split-K partial tiles.
#pragma unroll
      for (int q = 0; q < NG; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          red[warp][q][h][g * 8 + 2 * t] = acc[q][h][0];
          red[warp][q][h][g * 8 + 2 * t + 1] = acc[q][h][1];
          red[warp][q][h][(g + 8) * 8 + 2 * t] = acc[q][h][2];
          red[warp][q][h][(g + 8) * 8 + 2 * t + 1] = acc[q][h][3];
        }
      if (tid < 8 * NG) s_slot[tid] = (tp + tid < T) ? p.rt.sorted[base + tp + tid] : -1;
      __syncthreads();

      if (MODE == 0) {
        for (int idx = tid; idx < NG * 128; idx += kGemvThreads) {
          const int q = idx >> 7, r = (idx >> 3) & 15, col = idx & 7;
          const int slot = s_slot[q * 8 + col];
          if (slot < 0) continue;
          float gs = 0.f, us = 0.f;
#pragma unroll
          for (int w = 0; w < kGemvWarps; ++w) {
            gs += red[w][q][0][r * 8 + col];
            us += red[w][q][1][r * 8 + col];
          }
          p.inter[(size_t)slot * p.I + qi * 16 + r] = __float2bfloat16(silu_f(gs) * us);
        }
      } else {
        for (int idx = tid; idx < NG * 256; idx += kGemvThreads) {
          const int q = idx >> 8, h = (idx >> 7) & 1, r = (idx >> 3) & 15, col = idx & 7;
          const int slot = s_slot[q * 8 + col];
          if (slot < 0) continue;
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < kGemvWarps; ++w) v += red[w][q][h][r * 8 + col];
          v *= p.topk_w[slot];
          p.partial[(size_t)slot * p.H + qi * 32 + h * 16 + r] = v;
        }
        __threadfence();
        __syncthreads();
        if (tid < 8 * NG) {
          const int slot = s_slot[tid];
          int last = -1;
          if (slot >= 0) {
            const int m = slot / p.topk;
            int* cnt = p.counters + (size_t)m * ipe + qi;
            const int old = atomicAdd(cnt, 1);
            if (old == p.rt.tok_valid[m] - 1) {
              *cnt = 0;  // self-cleaning for the next call
              last = m;
            }
          }
          s_last[tid] = last;
        }
        __syncthreads();
        __threadfence();
        for (int idx = tid; idx < 8 * NG * 32; idx += kGemvThreads) {
          const int col = idx >> 5, r = idx & 31;
          const int m = s_last[col];
          if (m < 0) continue;
          float sum = 0.f;
          for (int tt = 0; tt < p.topk; ++tt) {
            const int slot = m * p.topk + tt;
            if (p.map(slot) < 0) continue;
            sum += __ldcg(p.partial + (size_t)slot * p.H + qi * 32 + r);
          }
          p.out[(size_t)m * p.H + qi * 32 + r] = __float2bfloat16(sum);
        }
      }
      __syncthreads();
    }
  }
}

template <int MODE>
cudaError_t launch_gemv_ng(const GemvParams& p, int ng, int grid, cudaStream_t stream) {
  switch (ng) {
    case 1: moe_gemv_kernel<MODE, 1><<<grid, kGemvThreads, 0, stream>>>(p); break;
    case 2: moe_gemv_kernel<MODE, 2><<<grid, kGemvThreads, 0, stream>>>(p); break;
    default: moe_gemv_kernel<MODE, 4><<<grid, kGemvThreads, 0, stream>>>(p); break;
  }
  return cudaGetLastError();
}

template <int MODE, int NG>
int blocks_per_sm_of() {
  static thread_local int cached_dev = -1, cached = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, moe_gemv_kernel<MODE, NG>, kGemvThreads, 0) !=
            cudaSuccess || n <= 0)
      n = 1;
    cached = n;
    cached_dev = dev;
  }
  return cached;
}

int gemv_blocks_per_sm(int mode, int ng) {
  if (mode == 0) return ng == 1 ? blocks_per_sm_of<0, 1>() : ng == 2 ? blocks_per_sm_of<0, 2>() : blocks_per_sm_of<0, 4>();
  return ng == 1 ? blocks_per_sm_of<1, 1>() : ng == 2 ? blocks_per_sm_of<1, 2>() : blocks_per_sm_of<1, 4>();
}

cudaError_t launch_gemv(const GemvParams& p, int mode, int ng, int grid, cudaStream_t stream) {
  return mode == 0 ? launch_gemv_ng<0>(p, ng, grid, stream)
                   : launch_gemv_ng<1>(p, ng, grid, stream);
}

}  // namespace w4moe
