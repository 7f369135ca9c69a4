// moe_align_block_size on the GPU: one CTA, warp-level histogram and scan,
// order-preserving scatter.
//
// Semantics follow kernels/w4a16_moe.py:187-290 of the reference bit for bit:
//   * counts[e]        = number of flat slots (m*topk + t) routed to expert e
//   * offsets          = exclusive cumsum of counts rounded up to block_size
//   * sorted[P]        = for each expert, its slot ids in ascending slot order
//                        (the reference's stable sort, :263-278), then padding;
//                        every unused entry holds n_tok (= M*topk, :230)
//   * expert_ids[P/bs] = owner expert of each block (searchsorted right=True
//                        on offsets[1:], :283-285), -1 past num_post (:286-288)
//   * num_post         = offsets[E] (:261)
//   * P                = roundup(n_tok + E*(bs-1), bs) (:153-157)
//
// Extensions (no reference counterpart): an optional expert_map (global id ->
// local id or -1, the vLLM expert-parallel convention), per-token counts of
// locally routed slots, a compact active-expert list for the GEMM schedulers,
// and zeroing of output rows whose token has no local slot.
#include <algorithm>

#include "launch.cuh"

namespace w4moe {

constexpr int kAlignThreads = 1024;
constexpr int kAlignWarps = kAlignThreads / 32;
constexpr int kAlignGridMinSlots = 8192;   // below: the single-CTA kernel
constexpr int kAlignSlotsPerCta = 2048;

__device__ __forceinline__ int load_expert(const AlignParams& p, int i) { return p.map(i); }

// Block-wide exclusive scan of one int per thread (1024 threads).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_tot[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    warp_tot[lane] = wi - w;  // exclusive warp base
    if (lane == 31) warp_tot[32] = wi;
  }
  __syncthreads();
  int r = warp_tot[warp] + incl - v;
  total = warp_tot[32];
  __syncthreads();
  return r;
}

// First e in [0, E) with off[e+1] > pos (requires pos < off[E]).
__device__ __forceinline__ int owner_of(const int* off, int E, int pos) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (off[mid + 1] > pos) hi = mid; else lo = mid + 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kAlignThreads, 1) moe_align_kernel(AlignParams p) {
  extern __shared__ int smem[];
  int* hist = smem;                                // [32][E]
  int* s_off = hist + kAlignWarps * p.E;           // [E+1]
  int* s_cnt = s_off + p.E + 1;                    // [E]
  __shared__ int warp_tot[33];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E = p.E;

  // Each of the first nseg warps owns one contiguous segment of the flat slot
  // array (few segments for small inputs keep the per-expert scan short).
  const int nseg = max(1, min(kAlignWarps, (p.n_tok + 127) / 128));
  for (int i = tid; i < nseg * E; i += kAlignThreads) hist[i] = 0;
  __syncthreads();

  const int seg = (p.n_tok + nseg - 1) / nseg;
  const int beg = warp < nseg ? min(p.n_tok, warp * seg) : p.n_tok;
  const int end = warp < nseg ? min(p.n_tok, beg + seg) : p.n_tok;
  for (int i = beg + lane; i < end; i += 32) {
    int e = load_expert(p, i);
    if (e >= 0) atomicAdd(&hist[warp * E + e], 1);
  }
  // Per-token local slot counts.
  const int M = p.topk > 0 ? p.n_tok / p.topk : 0;
  if (p.tok_valid != nullptr) {
    for (int m = tid; m < M; m += kAlignThreads) {
      int c = 0;
      for (int t = 0; t < p.topk; ++t) c += load_expert(p, m * p.topk + t) >= 0;
      p.tok_valid[m] = c;
    }
  }
  __syncthreads();

  // Experts are processed in rounds of 1024 (E <= 1024 in practice).
  int carry_pad = 0, carry_act = 0;
  for (int e0 = 0; e0 < E; e0 += kAlignThreads) {
    const int e = e0 + tid;
    int cnt = 0;
    if (e < E) {
      for (int w = 0; w < nseg; ++w) {  // per-segment exclusive prefix
        int h = hist[w * E + e];
        hist[w * E + e] = cnt;
        cnt += h;
      }
    }
    const int padded = (cnt + p.bs - 1) / p.bs * p.bs;
    int tot_pad, tot_act;
    const int ex_pad = block_exclusive_scan(padded, warp_tot, tot_pad);
    const int ex_act = block_exclusive_scan(cnt > 0 ? 1 : 0, warp_tot, tot_act);
    if (e < E) {
      s_off[e] = carry_pad + ex_pad;
      s_cnt[e] = cnt;
      if (p.counts) p.counts[e] = cnt;
      if (p.offsets) p.offsets[e] = carry_pad + ex_pad;
      if (p.active && cnt > 0) p.active[carry_act + ex_act] = e;
    }
    carry_pad += tot_pad;
    carry_act += tot_act;
  }
  if (tid == 0) {
    s_off[E] = carry_pad;
    p.num_post[0] = carry_pad;
    if (p.offsets) p.offsets[E] = carry_pad;
    if (p.num_active) p.num_active[0] = carry_act;
  }
  __syncthreads();
  for (int i = tid; i < nseg * E; i += kAlignThreads) hist[i] += s_off[i % E];
  __syncthreads();

  // Order-preserving scatter: each warp walks its segment 32 slots at a time;
  // lanes with equal expert rank themselves by lane order.
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int i0 = beg; i0 < end; i0 += 32) {
    const int i = i0 + lane;
    const int e = (i < end) ? load_expert(p, i) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int base = 0;
    if (e >= 0) base = hist[warp * E + e];
    __syncwarp();
    if (e >= 0) {
      p.sorted[base + __popc(peers & lt_mask)] = i;
      if ((peers & lt_mask) == 0) hist[warp * E + e] = base + __popc(peers);
    }
    __syncwarp();
  }

  // Padding entries (disjoint from the scatter targets).
  const int num_post = s_off[E];
  for (int pos = tid; pos < p.P; pos += kAlignThreads) {
    bool pad = true;
    if (pos < num_post) {
      const int e = owner_of(s_off, E, pos);
      pad = (pos - s_off[e]) >= s_cnt[e];
    }
    if (pad) p.sorted[pos] = p.n_tok;
  }
  const int nblk = p.P / p.bs;
  for (int b = tid; b < nblk; b += kAlignThreads) {
    const int pos = b * p.bs;
    p.expert_ids[b] = (pos < num_post) ? owner_of(s_off, E, pos) : -1;
  }

  // Tokens with no locally routed slot produce a zero row.
  if (p.zero_rows != nullptr && p.tok_valid != nullptr) {
    __syncthreads();
    for (int m = warp; m < M; m += kAlignWarps) {
      if (p.tok_valid[m] != 0) continue;
      uint4* row = reinterpret_cast<uint4*>(p.zero_rows + (size_t)m * p.H);
      for (int c = lane; c < p.H / 8; c += 32) row[c] = make_uint4(0, 0, 0, 0);
    }
  }
}

// ---------------------------------------------------------------------------
// Multi-CTA variant for large inputs (same outputs, bit for bit).  One
// cooperative launch of C CTAs; CTA c owns a contiguous chunk of the flat slot
// array, split into 32 per-warp segments:
//   1. per-warp expert histograms of the chunk (shared memory), CTA totals to
//      scratch[c][E];
//   2. grid barrier;
//   3. every CTA reads the C x E totals, forms its chunk base per expert and
//      the padded offsets (CTA 0 publishes counts / offsets / active lists);
//   4. order-preserving scatter of the chunk, then padding and block owners
//      grid-strided.
// Slot order inside an expert is the flat slot order, as in the single-CTA
// kernel: chunks, then warps, then lanes are all in ascending slot order.

__global__ void __launch_bounds__(kAlignThreads, 1) moe_align_grid_kernel(AlignParams p) {
  extern __shared__ int smem[];
  const int E = p.E, C = gridDim.x, c = blockIdx.x;
  int* hist = smem;                       // [32][E]
  int* s_off = hist + kAlignWarps * E;    // [E+1] padded offsets
  int* s_cnt = s_off + E + 1;             // [E]
  int* s_base = s_cnt + E;                // [E] this chunk's first rank per expert
  int* tot = s_base + E;                  // [C][E] chunk totals (copied from scratch)
  __shared__ int warp_tot[33];
  __shared__ int s_gen, s_timeout;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = (p.n_tok + C - 1) / C;
  const int cbeg = min(p.n_tok, c * chunk), cend = min(p.n_tok, cbeg + chunk);
  const int seg = (cend - cbeg + kAlignWarps - 1) / kAlignWarps;
  const int beg = min(cend, cbeg + warp * seg), end = min(cend, beg + seg);

  // 1. histograms
  for (int i = tid; i < kAlignWarps * E; i += kAlignThreads) hist[i] = 0;
  if (tid == 0) {
    s_gen = ld_acquire_gpu(p.grid_bar + 1);
    s_timeout = 0;
  }
  __syncthreads();
  for (int i = beg + lane; i < end; i += 32) {
    const int e = load_expert(p, i);
    if (e >= 0) atomicAdd(&hist[warp * E + e], 1);
  }
  const int M = p.topk > 0 ? p.n_tok / p.topk : 0;
  if (p.tok_valid != nullptr) {
    for (int m = c * kAlignThreads + tid; m < M; m += C * kAlignThreads) {
      int v = 0;
      for (int t = 0; t < p.topk; ++t) v += load_expert(p, m * p.topk + t) >= 0;
      p.tok_valid[m] = v;
    }
  }
  __syncthreads();
  for (int e = tid; e < E; e += kAlignThreads) {  // per-warp exclusive prefix, CTA total
    int run = 0;
    for (int w = 0; w < kAlignWarps; ++w) {
      const int h = hist[w * E + e];
      hist[w * E + e] = run;
      run += h;
    }
    p.scratch[c * E + e] = run;
  }

  // 2. grid barrier (arrival counter reset by the last arriver; generation word
  //    only increases, so the barrier needs no cleaning between launches)
  __syncthreads();
  if (p.withhold && c == 0) return;  // test hook: this CTA never arrives
  if (tid == 0) {
    __threadfence();
    const int arrived = atomicAdd(p.grid_bar, 1) + 1;
    if (arrived == C) {
      atomicExch(p.grid_bar, 0);
      __threadfence();
      atomicAdd(p.grid_bar + 1, 1);
    } else {
      const long long t0 = clock64();
      while (ld_acquire_gpu(p.grid_bar + 1) == s_gen) {
        if (clock64() - t0 > p.budget) {
          // the totals are incomplete: report and write no outputs
          atomicOr(p.grid_bar + 2, kAlignErrBarrier);
          if (p.status != nullptr) atomicOr(p.status, kAlignErrBarrier);
          s_timeout = 1;
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
  }
  __syncthreads();
  if (s_timeout) return;

  // 3. chunk totals -> per-expert counts, this chunk's bases, padded offsets
  for (int i = tid; i < C * E; i += kAlignThreads) tot[i] = __ldcg(p.scratch + i);
  __syncthreads();
  int carry_pad = 0, carry_act = 0;
  for (int e0 = 0; e0 < E; e0 += kAlignThreads) {
    const int e = e0 + tid;
    int cnt = 0, before = 0;
    if (e < E) {
      for (int cc = 0; cc < C; ++cc) {
        const int h = tot[cc * E + e];
        before += cc < c ? h : 0;
        cnt += h;
      }
    }
    const int padded = (cnt + p.bs - 1) / p.bs * p.bs;
    int tot_pad, tot_act;
    const int ex_pad = block_exclusive_scan(padded, warp_tot, tot_pad);
    const int ex_act = block_exclusive_scan(cnt > 0 ? 1 : 0, warp_tot, tot_act);
    if (e < E) {
      s_off[e] = carry_pad + ex_pad;
      s_cnt[e] = cnt;
      s_base[e] = carry_pad + ex_pad + before;
      if (c == 0) {
        if (p.counts) p.counts[e] = cnt;
        if (p.offsets) p.offsets[e] = carry_pad + ex_pad;
        if (p.active && cnt > 0) p.active[carry_act + ex_act] = e;
      }
    }
    carry_pad += tot_pad;
    carry_act += tot_act;
  }
  if (tid == 0) {
    s_off[E] = carry_pad;
    if (c == 0) {
      p.num_post[0] = carry_pad;
      if (p.offsets) p.offsets[E] = carry_pad;
      if (p.num_active) p.num_active[0] = carry_act;
    }
  }
  __syncthreads();
  for (int i = tid; i < kAlignWarps * E; i += kAlignThreads) hist[i] += s_base[i % E];
  __syncthreads();

  // 4. scatter (as in the single-CTA kernel), padding, block owners
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int i0 = beg; i0 < end; i0 += 32) {
    const int i = i0 + lane;
    const int e = (i < end) ? load_expert(p, i) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int base = 0;
    if (e >= 0) base = hist[warp * E + e];
    __syncwarp();
    if (e >= 0) {
      p.sorted[base + __popc(peers & lt_mask)] = i;
      if ((peers & lt_mask) == 0) hist[warp * E + e] = base + __popc(peers);
    }
    __syncwarp();
  }
  const int num_post = s_off[E];
  for (int pos = c * kAlignThreads + tid; pos < p.P; pos += C * kAlignThreads) {
    bool pad = true;
    if (pos < num_post) {
      const int e = owner_of(s_off, E, pos);
      pad = (pos - s_off[e]) >= s_cnt[e];
    }
    if (pad) p.sorted[pos] = p.n_tok;
  }
  const int nblk = p.P / p.bs;
  for (int b = c * kAlignThreads + tid; b < nblk; b += C * kAlignThreads) {
    const int pos = b * p.bs;
    p.expert_ids[b] = (pos < num_post) ? owner_of(s_off, E, pos) : -1;
  }
  if (p.zero_rows != nullptr && p.tok_valid != nullptr) {
    // tok_valid of other CTAs' tokens is visible after the grid barrier only
    // for rows written before it; recount locally instead
    for (int m = c * kAlignWarps + warp; m < M; m += C * kAlignWarps) {
      int v = 0;
      for (int t = 0; t < p.topk; ++t) v += load_expert(p, m * p.topk + t) >= 0;
      if (v != 0) continue;
      uint4* row = reinterpret_cast<uint4*>(p.zero_rows + (size_t)m * p.H);
      for (int cc = lane; cc < p.H / 8; cc += 32) row[cc] = make_uint4(0, 0, 0, 0);
    }
  }
}

size_t align_smem_bytes(int E) { return (size_t)(kAlignWarps * E + 2 * E + 1) * sizeof(int); }

cudaError_t launch_align(const AlignParams& p, cudaStream_t stream) {
  const size_t smem = align_smem_bytes(p.E);
  // Per-device opt-in above the 48 KB default (largest size configured so far).
  static thread_local size_t configured[64] = {0};
  if (smem > 48 * 1024) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (configured[dev] < smem) {
      cudaError_t err = cudaFuncSetAttribute(moe_align_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (err != cudaSuccess) return err;
      configured[dev] = smem;
    }
  }
  moe_align_kernel<<<1, kAlignThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

// Largest C whose C x E chunk totals fit in shared memory beside the
// per-warp histograms.
static int align_grid_max_ctas(int E, int sms) {
  const int ints = (227 * 1024 - 256) / 4 - (kAlignWarps * E + 3 * E + 1);
  return std::max(0, std::min(sms, ints / std::max(E, 1)));
}

// CTAs for the multi-CTA variant (0: use the single-CTA kernel).
int align_grid_ctas(int n_tok, int E, int sms) {
  if (n_tok < kAlignGridMinSlots || E > kAlignThreads || sms < 2) return 0;
  const int C = std::min((n_tok + kAlignSlotsPerCta - 1) / kAlignSlotsPerCta, align_grid_max_ctas(E, sms));
  return C >= 2 ? C : 0;
}

// Scratch the multi-CTA variant needs: chunk totals + the 3-word barrier.
size_t align_grid_scratch_ints(int E, int sms) { return (size_t)align_grid_max_ctas(E, sms) * E; }

cudaError_t launch_align_grid(const AlignParams& p_in, int ctas, cudaStream_t stream) {
  AlignParams p = p_in;
  if (p.budget <= 0) p.budget = kAlignBarrierBudget;
  const size_t smem = (size_t)(kAlignWarps * p.E + 3 * p.E + 1 + ctas * p.E) * sizeof(int);
  static thread_local size_t configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (configured[dev] < smem) {
    cudaError_t err = cudaFuncSetAttribute(moe_align_grid_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kAlignThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, moe_align_grid_kernel, p);
}

}  // namespace w4moe
