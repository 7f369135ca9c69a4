// Large-M ("prefill") grouped GEMMs on the 5th-generation tensor cores.
//
// Replaces, for large batches, the reference's _w4a16_moe_w1_fused_kernel,
// _w4a16_moe_w2_kernel and _moe_sum_kernel (kernels/w4a16_moe.py:374-670).
//
// Both projections run the same persistent kernel (one CTA per SM), "swap-AB"
// so that the ragged per-expert token count is the flexible N dimension:
//
//   A (M = 128) = 128 weight rows, dequantised in shared memory:
//       w13 (MODE 0): 64 gate rows + the matching 64 up rows,
//       w2  (MODE 1): 128 hidden rows;
//   B (N <= 256) = the expert's routed token rows (hidden rows for w13,
//       intermediate rows for w2), gathered with cp.async;
//   D = A * B^T, 128 x N fp32 in tensor memory (two 256-column buffers, so
//       the epilogue of one item overlaps the MMAs of the next).
//
// Work item = (active expert, 256-token chunk, weight row tile); items are
// assigned round-robin (CTA b takes b, b+grid, ...).  Per 64-wide k-block:
//   * 8 loader warps: cp.async the packed int4 block (8 row tiles x 512 B +
//     scales) into a staging area and the token rows into the 128-byte-
//     swizzled B tile (rows past the chunk are zero-filled), then decode the
//     staged int4 into the swizzled bf16 A tile ((code - 8) * scale, rounded
//     once to bf16 -- the reference's dequantised value).  Stages ahead: 3.
//   * 1 MMA warp: one thread issues 4 tcgen05.mma (K = 16 each) per k-block
//     and tcgen05.commit frees the stage when they complete.
//   * 4 epilogue warps (one TMEM lane quarter each) read D with tcgen05.ld:
//       MODE 0: bf16(silu(gate) * up) -> intermediate[slot, I] (gate and up
//               rows meet through a small shared-memory exchange);
//       MODE 1: bf16(acc * router weight) -> partial[slot, H].
// A third kernel sums each token's top-k partials in slot order (fp32) and
// writes the bf16 output -- deterministic, like the reference's moe_sum.
//
// Every wait is bounded; after the first timeout a CTA stops waiting (records
// an error bit in the workspace) so the kernel always terminates.
#include <algorithm>

#include "launch.cuh"

namespace w4moe {

constexpr int kPfEpiWarps = 4;                        // warps 0-3: epilogue (TMEM lane quarters)
constexpr int kPfDeqWarps = 8;                        // warps 4-11: int4 -> bf16 A tiles
constexpr int kPfCopyWarps = 4;                       // warps 12-15: async copies
constexpr int kPfDeqFirst = kPfEpiWarps;
constexpr int kPfCopyFirst = kPfDeqFirst + kPfDeqWarps;
constexpr int kPfMmaWarp = kPfCopyFirst + kPfCopyWarps;  // warp 16: tcgen05.mma issue
constexpr int kPfDeq = kPfDeqWarps * 32;
constexpr int kPfCopy = kPfCopyWarps * 32;
constexpr int kPfThreads = (kPfMmaWarp + 1) * 32;
constexpr int kPfStages = 4;
constexpr int kPfMaxTok = 256;                        // tokens per item (MMA N <= 256)
constexpr int kPfAStage = 128 * 128;                  // 128 rows x 64 bf16
constexpr int kPfBStage = kPfMaxTok * 128;            // 256 rows x 64 bf16
constexpr int kPfStaging = 8 * 576;                   // 8 row tiles x (512 B + 64 B scales)
constexpr int kPfStageBytes = kPfAStage + kPfBStage;  // 1024-aligned (staging kept apart)
constexpr int kPfXchgCols = 16;
constexpr int kPfTmemCols = 512;
constexpr long long kPfWaitBudget = 4000000000LL;

constexpr int kPfErrWait = 16;  // error bit in sched[2]

// trace layout [kind][1024] (CTA 0): 0 copies of k issued, 1 dequant saw k
// land, 2 dequant published A(k), 3 MMA saw A(k), 4 MMA committed k
__device__ __forceinline__ void pf_trace(long long* tr, int kind, int k) {
  if (tr != nullptr && blockIdx.x == 0 && k < 1024) tr[kind * 1024 + k] = global_timer_ns();
}

// Arrive on `bar` when all of this thread's earlier cp.async copies have landed
// (the arrival counts toward the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

struct PfItem {
  int e, p, chunk, ntok, n16, base;
};

template <int MODE>
__global__ void __launch_bounds__(kPfThreads, 1) moe_prefill_kernel(PrefillParams p) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  __shared__ uint64_t raw_full[kPfStages], a_full[kPfStages], empty_bar[kPfStages];
  __shared__ uint64_t acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int s_failed, s_nact;

  const int S = p.n_stages;                                    // 3 or 4
  unsigned char* stages = dsm;                                 // S x (A | B), 1024-aligned
  unsigned char* staging = dsm + S * kPfStageBytes;            // S x packed int4 blocks
  int* rowoff = reinterpret_cast<int*>(staging + S * kPfStaging);     // [4 copy warps][256] B-row offsets
  float* xchg = reinterpret_cast<float*>(rowoff + kPfCopyWarps * kPfMaxTok);  // [16 cols][64 rows]
  int* cum = reinterpret_cast<int*>(xchg + kPfXchgCols * 64);  // [E + 1]
  int* s_act = cum + p.E + 1;                                  // [E] active experts
  int* s_cnt = s_act + p.E;                                    // [E] slots per expert
  int* s_off = s_cnt + p.E;                                    // [E] first slot of expert

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tiles = MODE == 0 ? p.I / 64 : p.H / 128;  // weight row tiles per expert
  const int nkb = MODE == 0 ? p.H / 64 : p.I / 64;     // k-blocks per item

  // ---------------- prologue ----------------
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&raw_full[s], 32);      // the lanes of the slot's copy warp
      mbar_init(&a_full[s], kPfDeq / 2);  // one group of 4 dequant warps
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kPfEpiWarps * 32);
    }
    fence_barrier_init();
    s_failed = 0;
  }
  {
    // items of each active expert (ceil(T / 256) chunks x tiles), prefix-summed
    const int na = p.num_active[0];
    for (int e = tid; e < p.E; e += kPfThreads) {
      s_cnt[e] = p.counts[e];
      s_off[e] = p.offsets[e];
    }
    for (int j = tid; j < na; j += kPfThreads) {
      const int e = p.active[j];
      s_act[j] = e;
      cum[j + 1] = (p.counts[e] + kPfMaxTok - 1) / kPfMaxTok * tiles;
    }
    __syncthreads();
    if (warp == 0) {
      int carry = 0;
      for (int j0 = 0; j0 < na; j0 += 32) {
        const int j = j0 + lane;
        int v = j < na ? cum[j + 1] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int u = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v += u;
        }
        if (j < na) cum[j + 1] = carry + v;
        carry += __shfl_sync(0xffffffffu, v, 31);
      }
      if (lane == 0) {
        cum[0] = 0;
        s_nact = na;
      }
    }
  }
  if (warp == 0) tmem_alloc(&tmem_base, kPfTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const int nact = s_nact;
  const int total = cum[nact];
  const int my_items = total > (int)blockIdx.x ? (total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total_k = my_items * nkb;
  const uint32_t tmem = tmem_base;

  auto item_of = [&](int n) {  // n-th item of this CTA
    const int item = blockIdx.x + n * gridDim.x;
    int lo = 0, hi = nact - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cum[mid] <= item) lo = mid; else hi = mid - 1;
    }
    PfItem it;
    it.e = s_act[lo];
    const int r = item - cum[lo];
    it.chunk = r / tiles;
    it.p = r - it.chunk * tiles;
    const int T = s_cnt[it.e];
    it.ntok = min(kPfMaxTok, T - it.chunk * kPfMaxTok);
    it.n16 = (it.ntok + 15) & ~15;
    it.base = s_off[it.e] + it.chunk * kPfMaxTok;
    return it;
  };
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (s_failed) return;
    if (!mbar_wait(bar, parity, kPfWaitBudget)) {
      s_failed = 1;
      atomicOr(p.sched + 2, kPfErrWait);
    }
  };

  if (warp >= kPfCopyFirst && warp < kPfMmaWarp) {
    // ======================= copy warps =======================
    // Copy warp w owns ring slot w: it fills k-blocks k = w, w+S, w+2S, ...
    // (one cp.async commit-free stream per warp; completion is signalled per
    // lane with cp.async.mbarrier.arrive.noinc).  Warps beyond S stay idle.
    const int cw = warp - kPfCopyFirst;
    int* ro = rowoff + cw * kPfMaxTok;  // this warp's B-row offsets of its current item
    int cached_n = -1;
    PfItem it{};
    for (int k = cw; cw < S && k < total_k; k += S) {
      const int n = k / nkb, kb = k - n * nkb;
      if (n != cached_n) {
        it = item_of(n);
        cached_n = n;
        for (int i = lane; i < it.ntok; i += 32)
          ro[i] = (int)((long long)(p.sorted[it.base + i] / p.x_row_div) * p.x_ld);
        __syncwarp();
      }
      const int s = cw, use = k / S;
      if (use > 0) wait(&empty_bar[s], (use - 1) & 1);
      if (lane == 0) pf_trace(p.trace, 5, k);
      unsigned char* bdst = stages + (size_t)s * kPfStageBytes + kPfAStage;
      unsigned char* stg = staging + (size_t)s * kPfStaging;
      // packed weights + scales of the 8 row tiles: 288 16-byte granules
      for (int gi = lane; gi < 8 * 36; gi += 32) {
        const int i = gi / 36, q = gi - i * 36;
        int rt;
        if (MODE == 0) rt = (i < 4) ? it.p * 4 + i : p.I / 16 + it.p * 4 + (i - 4);
        else rt = it.p * 8 + i;
        const size_t blk = ((size_t)it.e * p.n_rowtiles + rt) * p.n_chunks + kb;
        const unsigned char* src = q < 32 ? p.w + blk * 512 + q * 16 : p.s + blk * 64 + (q - 32) * 16;
        cp_async16_zfill(stg + i * 576 + q * 16, src, true);
      }
      if (lane == 0) pf_trace(p.trace, 6, k);
      // token rows (rows in [ntok, n16) keep stale values: they only reach
      // accumulator columns that are never stored)
      const __nv_bfloat16* xk = p.x + kb * 64;
      for (int gi = lane; gi < it.ntok * 8; gi += 32) {
        const int row = gi >> 3, c16 = gi & 7;
        cp_async16_zfill(bdst + swz128(row, c16 * 8), xk + ro[row] + c16 * 8, true);
      }
      cp_async_arrive_noinc(&raw_full[s]);
      if (lane == 0) pf_trace(p.trace, 0, k);
    }
    cp_async_wait_group<0>();
  } else if (warp >= kPfDeqFirst && warp < kPfCopyFirst) {
    // ======================= dequant warps =======================
    // two groups of 4 warps take alternate k-blocks; a thread decodes two of
    // the eight 16-row x 64-k fragment blocks of its k-block
    const int dt = tid - kPfDeqFirst * 32;  // 0..255
    const int grp = dt >> 7, gt = dt & 127;
    const int fl = gt & 31, fg = fl >> 2, ft = fl & 3;
    const int fi0 = gt >> 5;  // fragment blocks fi0 and fi0 + 4
    uint32_t aoff[4][4];      // swizzled offsets for block fi0 (block fi0+4 is +64 rows = +8192 B)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r0 = fi0 * 16 + fg, r1 = r0 + 8, k0 = j * 16 + 2 * ft;
      aoff[j][0] = swz128(r0, k0);
      aoff[j][1] = swz128(r1, k0);
      aoff[j][2] = swz128(r0, k0 + 8);
      aoff[j][3] = swz128(r1, k0 + 8);
    }
    for (int k = grp; k < total_k; k += 2) {
      const int s = k % S;
      wait(&raw_full[s], (k / S) & 1);
      if (gt == 0) pf_trace(p.trace, 1, k);
      unsigned char* st = stages + (size_t)s * kPfStageBytes;
      const unsigned char* stg = staging + (size_t)s * kPfStaging;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int fi = fi0 + 4 * h;
        const uint4 wv = lds128(stg + fi * 576 + fl * 16);
        const uint2 sv = lds64(stg + fi * 576 + 512 + fg * 8);
        const uint32_t sg0 = __byte_perm(sv.x, 0, 0x1010), sg80 = __byte_perm(sv.x, 0, 0x3232);
        const uint32_t sg1 = __byte_perm(sv.y, 0, 0x1010), sg81 = __byte_perm(sv.y, 0, 0x3232);
        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
        unsigned char* sth = st + h * 8192;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          dequant_word(w4[j], j < 2 ? sg0 : sg1, j < 2 ? sg80 : sg81, a);
#pragma unroll
          for (int x = 0; x < 4; ++x) *reinterpret_cast<uint32_t*>(sth + aoff[j][x]) = a[x];
        }
      }
      fence_proxy_async_shared();  // generic smem writes (A, and the cp.async B rows) -> tensor core
      mbar_arrive(&a_full[s]);
      if (gt == 0) pf_trace(p.trace, 2, k);
    }
  } else if (warp == kPfMmaWarp) {
    // ======================= MMA warp =======================
    if (lane == 0) {
      for (int n = 0; n < my_items; ++n) {
        const PfItem it = item_of(n);
        const int b = n & 1, use = n >> 1;
        if (use > 0) wait(&acc_empty[b], (use - 1) & 1);
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * 256);
        const uint32_t idesc = umma_idesc_bf16(128, it.n16);
        for (int kb = 0; kb < nkb; ++kb) {
          const int k = n * nkb + kb, s = k % S;
          wait(&a_full[s], (k / S) & 1);
          pf_trace(p.trace, 3, k);
          tc_fence_after();
          const uint32_t a0 = smem_u32(stages + (size_t)s * kPfStageBytes);
          const uint32_t b0 = a0 + kPfAStage;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16(d, umma_desc_sw128(a0 + ks * 32), umma_desc_sw128(b0 + ks * 32), idesc,
                      (kb > 0 || ks > 0) ? 1u : 0u);
          umma_commit(&empty_bar[s]);
          pf_trace(p.trace, 4, k);
        }
        umma_commit(&acc_full[b]);
      }
    }
    __syncwarp();
  } else {
    // ======================= epilogue warps =======================
    const int r = warp * 32 + lane;  // TMEM lane = weight row within the item
    for (int n = 0; n < my_items; ++n) {
      const PfItem it = item_of(n);
      const int b = n & 1;
      wait(&acc_full[b], (n >> 1) & 1);
      tc_fence_after();
      const int* sl = p.sorted + it.base;  // slot of accumulator column c
      const uint32_t dbase = tmem + (uint32_t)(b * 256) + ((uint32_t)(warp * 32) << 16);
      for (int c0 = 0; c0 < it.n16; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(dbase + c0, v);
        if (MODE == 0) {
#pragma unroll
          for (int h = 0; h < 32; h += kPfXchgCols) {
            if (r >= 64) {
#pragma unroll
              for (int c = 0; c < kPfXchgCols; ++c) xchg[c * 64 + (r - 64)] = __uint_as_float(v[h + c]);
            }
            named_barrier_sync(2, kPfEpiWarps * 32);
            if (r < 64) {
#pragma unroll
              for (int c = 0; c < kPfXchgCols; ++c) {
                if (c0 + h + c >= it.ntok) break;
                const float gv = __uint_as_float(v[h + c]), uv = xchg[c * 64 + r];
                p.inter[(size_t)sl[c0 + h + c] * p.I + it.p * 64 + r] = __float2bfloat16(silu_f(gv) * uv);
              }
            }
            named_barrier_sync(2, kPfEpiWarps * 32);
          }
        } else {
          for (int c = 0; c < 32 && c0 + c < it.ntok; ++c) {
            const int slot = sl[c0 + c];
            p.partial[(size_t)slot * p.H + it.p * 128 + r] =
                __float2bfloat16(__uint_as_float(v[c]) * p.topk_w[slot]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
  }

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kPfTmemCols);
}

// out[m, :] = bf16(sum over t in slot order of partial[m*topk + t, :]) for the
// slots routed to a local expert (0 if none).
__global__ void moe_topk_sum_kernel(const __nv_bfloat16* partial, __nv_bfloat16* out, SlotMap map, int M,
                                    int topk, int H) {
  const int h8 = H / 8;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < (long long)M * h8;
       idx += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(idx / h8), h = (int)(idx - (long long)m * h8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int t = 0; t < topk; ++t) {
      const int slot = m * topk + t;
      if (map(slot) < 0) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(partial + (size_t)slot * H + h);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] += __uint_as_float(w[i] << 16);
        acc[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      ow[i] = *reinterpret_cast<uint32_t*>(&b2);
    }
    *reinterpret_cast<uint4*>(out + (size_t)m * H + h) = o;
  }
}

size_t prefill_smem_bytes(int E, int stages) {
  return (size_t)stages * (kPfStageBytes + kPfStaging) + kPfCopyWarps * kPfMaxTok * 4 + kPfXchgCols * 64 * 4 +
         (4 * E + 1) * 4;
}

// Pipeline depth that fits the opt-in shared memory (static smem is < 512 B).
int prefill_stages(int E, int max_smem_optin) {
  return prefill_smem_bytes(E, kPfStages) + 512 <= (size_t)max_smem_optin ? kPfStages : kPfStages - 1;
}

static cudaError_t prefill_config(int E, int stages) {
  const size_t smem = prefill_smem_bytes(E, stages);
  static thread_local size_t configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (configured[dev] < smem) {
    cudaError_t err = cudaFuncSetAttribute(moe_prefill_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err == cudaSuccess)
      err = cudaFuncSetAttribute(moe_prefill_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    configured[dev] = smem;
  }
  return cudaSuccess;
}

cudaError_t launch_prefill_w13(const PrefillParams& p13, int sms, cudaStream_t stream) {
  cudaError_t err = prefill_config(p13.E, p13.n_stages);
  if (err != cudaSuccess) return err;
  moe_prefill_kernel<0><<<sms, kPfThreads, prefill_smem_bytes(p13.E, p13.n_stages), stream>>>(p13);
  return cudaGetLastError();
}

cudaError_t launch_prefill_w2(const PrefillParams& p2, const SlotMap& map, int M, int topk, int H,
                              __nv_bfloat16* out, int sms, cudaStream_t stream) {
  cudaError_t err = prefill_config(p2.E, p2.n_stages);
  if (err != cudaSuccess) return err;
  moe_prefill_kernel<1><<<sms, kPfThreads, prefill_smem_bytes(p2.E, p2.n_stages), stream>>>(p2);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  const long long work = (long long)M * (H / 8);
  const int blocks = (int)std::min<long long>((work + 255) / 256, (long long)sms * 8);
  moe_topk_sum_kernel<<<blocks > 0 ? blocks : 1, 256, 0, stream>>>(p2.partial, out, map, M, topk, H);
  return cudaGetLastError();
}

}  // namespace w4moe
