// Load-time weight transform: vLLM (E, N_out, K/2) uint8 + (E, N_out, K/G) bf16
// -> the fragment-major layout documented in common.cuh.
//
// Replaces kernels/w4a16_moe.py:63-116 of the reference (repack_weights),
// which produced an N-tile-major layout for its Triton kernels; only this
// library's kernels read the result, so the layout is ours to choose.
// Input packing is compressed-tensors / vLLM's: byte j of a row holds element
// 2j in the low nibble and 2j+1 in the high nibble (stored value = q + 8).
// The same kernels also read the checkpoint form directly (vLLM create_weights
// with is_transposed=True): int32 (E, K/8, N_out) with code j of a word at
// bits 4j, scales (E, K/G, N_out) -- so a load path needs no transpose copy.
#include <algorithm>

#include "launch.cuh"

namespace w4moe {

__device__ __forceinline__ uint32_t code_at(const RepackParams& p, int e, int row, int k) {
  if (p.w_i32t != nullptr) {  // checkpoint form: (E, K/8, N_out) int32, code k%8 at bits 4*(k%8)
    const uint32_t word = (uint32_t)p.w_i32t[((size_t)e * (p.K / 8) + (k >> 3)) * p.N_out + row];
    return (word >> (4 * (k & 7))) & 0xFu;
  }
  const uint8_t b = p.w_q[((size_t)e * p.N_out + row) * (p.K / 2) + (k >> 1)];
  return (k & 1) ? (b >> 4) : (b & 0xF);
}

__global__ void repack_weights_kernel(RepackParams p) {
  const int R = p.N_out / kRowTile, C = p.K / kChunkK;
  const size_t total = (size_t)p.E * R * C * 128;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int lj = (int)(idx % 128);
    const size_t blk = idx / 128;
    const int c = (int)(blk % C);
    const int r = (int)((blk / C) % R);
    const int e = (int)(blk / ((size_t)C * R));
    const int lane = lj >> 2, j = lj & 3;
    const int g = lane >> 2, t = lane & 3;
    const int row0 = r * kRowTile + g, row1 = row0 + 8;
    const int k0 = c * kChunkK + j * 16 + 2 * t;
    uint32_t w = 0;
    w |= code_at(p, e, row0, k0) << 0;
    w |= code_at(p, e, row1, k0) << 4;
    w |= code_at(p, e, row0, k0 + 8) << 8;
    w |= code_at(p, e, row1, k0 + 8) << 12;
    w |= code_at(p, e, row0, k0 + 1) << 16;
    w |= code_at(p, e, row1, k0 + 1) << 20;
    w |= code_at(p, e, row0, k0 + 9) << 24;
    w |= code_at(p, e, row1, k0 + 9) << 28;
    p.w_rep[idx] = w;
  }
}

__global__ void repack_scales_kernel(RepackParams p) {
  const int R = p.N_out / kRowTile, C = p.K / kChunkK;
  const int ng = p.K / p.G;
  const size_t total = (size_t)p.E * R * C * kChunkScales;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int i = (int)(idx % kChunkScales);
    const size_t blk = idx / kChunkScales;
    const int c = (int)(blk % C);
    const int r = (int)((blk / C) % R);
    const int e = (int)(blk / ((size_t)C * R));
    const int g = i >> 2, which = i & 3;
    const int row = r * kRowTile + g + (which & 1) * 8;
    const int grp32 = c * 2 + (which >> 1);
    const int src_grp = (grp32 * kGroup) / p.G;
    p.s_rep[idx] = p.scales_t ? p.scales[((size_t)e * ng + src_grp) * p.N_out + row]
                              : p.scales[((size_t)e * p.N_out + row) * ng + src_grp];
  }
}

cudaError_t launch_repack(const RepackParams& p, cudaStream_t stream) {
  const int threads = 256;
  const size_t words = (size_t)p.E * (p.N_out / kRowTile) * (p.K / kChunkK) * 128;
  const int blocks = (int)std::min<size_t>((words + threads - 1) / threads, 148 * 64);
  repack_weights_kernel<<<blocks, threads, 0, stream>>>(p);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  repack_scales_kernel<<<blocks, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace w4moe
