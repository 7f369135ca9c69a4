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
//   B (N <= 256) = the expert's routed token rows, read with one 2-D tensor
//       load (TMA) per 64-wide k-block from an expert-sorted copy of the
//       rows (w13: a gather kernel writes the hidden rows in sorted order;
//       w2: the w13 epilogue writes the intermediate in sorted order);
//   D = A * B^T, 128 x N fp32 in tensor memory (two 256-column buffers, so
//       the epilogue of one item overlaps the MMAs of the next).
//
// Work item = (active expert, 256-token chunk, weight row tile); items are
// assigned round-robin (CTA b takes b, b+grid, ...).  Per 64-wide k-block:
//   * loader warps: 3-D tensor loads (TMA) of the packed int4 block (8 row
//     tiles x 512 B + scales) into a staging area and 2-D tensor loads of the
//     token rows into the 128-byte-swizzled B tile (rows past the chunk are
//     zero-filled), then decode the staged int4 into the swizzled bf16 A tile
//     ((code - 8) * scale, rounded once to bf16 -- the reference's
//     dequantised value).
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

#include <cuda.h>

#include "launch.cuh"

namespace w4moe {

constexpr int kPfEpiWarps = 4;                        // warps 0-3: epilogue (TMEM lane quarters)
constexpr int kPfDeqWarps = 8;                        // warps 4-11: int4 -> bf16 A tiles (2 groups)
constexpr int kPfDeqFirst = kPfEpiWarps;
constexpr int kPfWLoadWarp = kPfDeqFirst + kPfDeqWarps;  // warp 12: packed-weight bulk copies
constexpr int kPfBLoadWarp = kPfWLoadWarp + 1;           // warp 13: token-row tensor loads
constexpr int kPfMmaWarp = kPfBLoadWarp + 1;             // warp 14: tcgen05.mma issue
constexpr int kPfDeqGroup = kPfDeqWarps / 2 * 32;        // threads per dequant group
constexpr int kPfThreads = (kPfMmaWarp + 1) * 32;
constexpr int kPfStages = 4;
constexpr int kPfWK = 2;                              // k-blocks per packed-weight stage
constexpr int kPfWStages = 3;                         // packed-weight stages
constexpr int kPfMaxTok = 256;                        // tokens per item (MMA N <= 256)
constexpr int kPfBoxRows = 32;                        // granularity of the token-row tensor loads
constexpr int kPfAStage = 128 * 128;                  // 128 rows x 64 bf16
constexpr int kPfBStage = kPfMaxTok * 128;            // 256 rows x 64 bf16
constexpr int kPfStaging = kPfWK * 8 * 576;           // 8 row tiles x kPfWK x (512 B + 64 B scales)
constexpr int kPfScaleOff = kPfWK * 8 * 512;          // scales after the packed words
constexpr int kPfStageBytes = kPfAStage + kPfBStage;  // 1024-aligned
constexpr int kPfXchgCols = 8;
constexpr int kPfTmemCols = 512;
constexpr long long kPfWaitBudget = 1000000000LL;  // SM clocks (~0.5 s)

constexpr int kPfErrWait = 16;  // error bit in sched[2]

// trace layout [kind][1024] (CTA 0): 0 token rows of k issued, 1 dequant has
// k's weights and a free A slot, 2 dequant published A(k), 3 MMA saw A and B
// of k, 4 MMA committed k, 5 weights of k issued
// Diagnostics builds only: otherwise the helper compiles to nothing (untaken
// trace branches in the pipeline loops cost time).
#ifdef W4A16_DIAGNOSTICS
__device__ __forceinline__ void pf_trace(long long* tr, int kind, int k) {
  if (tr != nullptr && blockIdx.x == 0 && k < 1024) tr[kind * 1024 + k] = global_timer_ns();
}
#else
__device__ __forceinline__ void pf_trace(long long*, int, int) {}
#endif

// Token-row tensor maps with box heights 32, 64, ..., 256 rows: each k-block's
// rows arrive with a single tensor load (the per-load cost is ~45 SM clocks,
// comparable to streaming 3 KB).
struct PfRowMaps {
  CUtensorMap m[kPfMaxTok / kPfBoxRows];
};

struct PfItem {
  int e, p, chunk, ntok, n16, base;
};

template <int MODE>
__global__ void __launch_bounds__(kPfThreads, 1)
    moe_prefill_kernel(const PrefillParams p, const __grid_constant__ PfRowMaps tmb,
                       const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  __shared__ uint64_t a_full[kPfStages], b_full[kPfStages], empty_bar[kPfStages];
  __shared__ uint64_t w_full[kPfWStages], w_empty[kPfWStages];
  __shared__ uint64_t acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int s_failed, s_nact;

  const int S = p.n_stages;                                    // 3 or 4
  unsigned char* stages = dsm;                                 // S x (A | B), 1024-aligned
  unsigned char* wstage = dsm + S * kPfStageBytes;             // kPfWStages x packed int4 blocks
  float* xchg = reinterpret_cast<float*>(wstage + kPfWStages * kPfStaging);  // [16 cols][64 rows]
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
      mbar_init(&a_full[s], kPfDeqGroup);  // one dequant group
      mbar_init(&b_full[s], 1);            // expect_tx of the token-row loads
      mbar_init(&empty_bar[s], 1);         // tcgen05.commit
    }
    for (int s = 0; s < kPfWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 2 * kPfDeqGroup);  // both dequant groups
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

  auto fast_wait = [&](uint64_t* bar, uint32_t parity) {
    if (!mbar_try_wait(bar, parity)) wait(bar, parity);
  };

  if (warp == kPfWLoadWarp) {
    // ====== packed weights: per stage kPfWK k-blocks of 8 row tiles, 4 tensor loads ======
    // (gate/up or hidden row tiles come in two runs of 4; smem order [tile][kb][512 B])
    if (lane == 0) {
      const uint32_t wbase = smem_u32(wstage);
      int ws = 0;
      uint32_t ph = 0;
      bool wrapped = false;
      for (int n = 0; n < my_items; ++n) {
        const PfItem it = item_of(n);
        const int row0 = it.e * p.n_rowtiles + (MODE == 0 ? it.p * 4 : it.p * 8);
        const int row1 = MODE == 0 ? row0 + p.I / 16 : row0 + 4;
        for (int kb = 0; kb < nkb; kb += kPfWK) {
          if (wrapped) fast_wait(&w_empty[ws], ph ^ 1u);
          const uint32_t stg = wbase + (uint32_t)ws * kPfStaging;
          mbar_arrive_expect_tx(&w_full[ws], kPfStaging);
          tma_load_3d_u32(stg, &tmw, 0, kb, row0, &w_full[ws]);
          tma_load_3d_u32(stg + 4 * kPfWK * 512, &tmw, 0, kb, row1, &w_full[ws]);
          tma_load_3d_u32(stg + kPfScaleOff, &tms, 0, kb, row0, &w_full[ws]);
          tma_load_3d_u32(stg + kPfScaleOff + 4 * kPfWK * 64, &tms, 0, kb, row1, &w_full[ws]);
          if (p.trace != nullptr) pf_trace(p.trace, 5, n * nkb + kb);
          if (++ws == kPfWStages) {
            ws = 0;
            ph ^= 1u;
            wrapped = true;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kPfBLoadWarp) {
    // ============ token rows: ceil(ntok / 32) tensor loads of 32 rows x 64 k ============
    // (rows past the item belong to the next expert or are zero-filled; they
    // only reach accumulator columns that are never stored)
    if (lane == 0) {
      const uint32_t bdst0 = smem_u32(stages) + kPfAStage;
      int s = 0;
      uint32_t ph = 0;
      for (int n = 0; n < my_items; ++n) {
        const PfItem it = item_of(n);
        const int nl = (it.ntok + kPfBoxRows - 1) / kPfBoxRows;
        const uint32_t bytes = (uint32_t)nl * kPfBoxRows * 128;
        const CUtensorMap* bm = &tmb.m[nl - 1];  // box of nl * 32 rows: one load per k-block
        for (int kb = 0; kb < nkb; ++kb) {
          if (n > 0 || kb >= S) fast_wait(&empty_bar[s], ph ^ 1u);
          const uint32_t bdst = bdst0 + (uint32_t)s * kPfStageBytes;
          mbar_arrive_expect_tx(&b_full[s], bytes);
          tma_load_2d_u32(bdst, bm, kb * 64, it.base, &b_full[s]);
          if (p.trace != nullptr) pf_trace(p.trace, 0, n * nkb + kb);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp >= kPfDeqFirst && warp < kPfWLoadWarp) {
    // ======================= dequant warps =======================
    // two groups of 4 warps take alternate k-blocks; a thread decodes two of
    // the eight 16-row x 64-k fragment blocks of its k-block
    const int dt = tid - kPfDeqFirst * 32;  // 0..255
    const int grp = dt / kPfDeqGroup, gt = dt % kPfDeqGroup;
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
      const int s = k % S, use = k / S, q = k / kPfWK, ws = q % kPfWStages, sub = k % kPfWK;
      if (use > 0) wait(&empty_bar[s], (use - 1) & 1);
      wait(&w_full[ws], (q / kPfWStages) & 1);
      if (gt == 0) pf_trace(p.trace, 1, k);
      unsigned char* st = stages + (size_t)s * kPfStageBytes;
      const unsigned char* stg = wstage + ws * kPfStaging;
      uint4 wv[2];
      uint2 sv[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int blk = (fi0 + 4 * h) * kPfWK + sub;
        wv[h] = lds128(stg + blk * 512 + fl * 16);
        sv[h] = lds64(stg + kPfScaleOff + blk * 64 + fg * 8);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t sg0 = __byte_perm(sv[h].x, 0, 0x1010), sg80 = __byte_perm(sv[h].x, 0, 0x3232);
        const uint32_t sg1 = __byte_perm(sv[h].y, 0, 0x1010), sg81 = __byte_perm(sv[h].y, 0, 0x3232);
        const uint32_t w4[4] = {wv[h].x, wv[h].y, wv[h].z, wv[h].w};
        unsigned char* sth = st + h * 8192;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          dequant_word(w4[j], j < 2 ? sg0 : sg1, j < 2 ? sg80 : sg81, a);
#pragma unroll
          for (int x = 0; x < 4; ++x) *reinterpret_cast<uint32_t*>(sth + aoff[j][x]) = a[x];
        }
      }
      // The packed-weight staging is released only now, after the loaded words
      // were consumed: arriving right after issuing the shared-memory loads let
      // the next tensor load overwrite the staging under them (a fraction of
      // 16-row A blocks came out nondeterministic at large M).
      mbar_arrive(&w_empty[ws]);
      fence_proxy_async_shared();  // generic smem writes -> tensor-core reads
      mbar_arrive(&a_full[s]);
      if (gt == 0) pf_trace(p.trace, 2, k);
    }
  } else if (warp == kPfMmaWarp) {
    // ======================= MMA warp =======================
    // The issuing thread's instruction stream paces the tensor pipe (a few
    // dozen cycles per issued instruction), so the loop keeps ring positions
    // incrementally and builds descriptors by adding to precomputed bases.
    if (lane == 0) {
      const uint32_t sbase = smem_u32(stages);
      const uint64_t dhi = umma_desc_sw128(sbase) - (uint64_t)((sbase >> 4) & 0x3FFF);
      const uint32_t lo0 = (sbase >> 4) & 0x3FFF;
      int s = 0;
      uint32_t ph = 0, lo = lo0;
      for (int n = 0; n < my_items; ++n) {
        const PfItem it = item_of(n);
        const int b = n & 1;
        if (n >= 2) fast_wait(&acc_empty[b], ((n >> 1) - 1) & 1);
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * 256);
        const uint32_t idesc = umma_idesc_bf16(128, it.n16);
        // k-blocks are consumed in pairs: each readiness check of the issuing
        // thread costs several hundred cycles once MMAs are in flight, so
        // checking two stages at once keeps the tensor pipe fed (nkb is even)
        for (int kb = 0; kb < nkb; kb += 2) {
          int s1 = s + 1;
          uint32_t ph1 = ph, lo1 = lo + (kPfStageBytes >> 4);
          if (s1 == S) {
            s1 = 0;
            ph1 ^= 1u;
            lo1 = lo0;
          }
          fast_wait(&a_full[s], ph);
          fast_wait(&b_full[s], ph);
          fast_wait(&a_full[s1], ph1);
          fast_wait(&b_full[s1], ph1);
          if (p.trace != nullptr) pf_trace(p.trace, 3, n * nkb + kb);
          tc_fence_after();
          const uint64_t da = dhi + lo, db = dhi + lo + (kPfAStage >> 4);
          umma_bf16(d, da, db, idesc, kb > 0 ? 1u : 0u);
          umma_bf16(d, da + 2, db + 2, idesc, 1u);
          umma_bf16(d, da + 4, db + 4, idesc, 1u);
          umma_bf16(d, da + 6, db + 6, idesc, 1u);
          umma_commit(&empty_bar[s]);
          const uint64_t da1 = dhi + lo1, db1 = dhi + lo1 + (kPfAStage >> 4);
          umma_bf16(d, da1, db1, idesc, 1u);
          umma_bf16(d, da1 + 2, db1 + 2, idesc, 1u);
          umma_bf16(d, da1 + 4, db1 + 4, idesc, 1u);
          umma_bf16(d, da1 + 6, db1 + 6, idesc, 1u);
          umma_commit(&empty_bar[s1]);
          s = s1 + 1;
          ph = ph1;
          lo = lo1 + (kPfStageBytes >> 4);
          if (s == S) {
            s = 0;
            ph ^= 1u;
            lo = lo0;
          }
        }
        umma_commit(&acc_full[b]);
        if (p.trace != nullptr) pf_trace(p.trace, 4, n);
      }
    }
    __syncwarp();
  } else {
    // ======================= epilogue warps =======================
    const int r = warp * 32 + lane;  // TMEM lane = weight row within the item
    constexpr int kGroups = kPfMaxTok / 32;
    for (int n = 0; n < my_items; ++n) {
      const PfItem it = item_of(n);
      const int b = n & 1;
      // w2: slots and router weights of the item's columns, loaded while the
      // MMAs still run (one dependent round trip per item, not per column group)
      int sl_r[kGroups];
      float w_r[kGroups];
      if (MODE == 1) {
#pragma unroll
        for (int k = 0; k < kGroups; ++k) {
          const int cl = k * 32 + lane;
          sl_r[k] = cl < it.ntok ? p.sorted[it.base + cl] : 0;
        }
#pragma unroll
        for (int k = 0; k < kGroups; ++k) w_r[k] = k * 32 + lane < it.ntok ? p.topk_w[sl_r[k]] : 0.f;
      }
      wait(&acc_full[b], (n >> 1) & 1);
      tc_fence_after();
      const uint32_t dbase = tmem + (uint32_t)(b * 256) + ((uint32_t)(warp * 32) << 16);
      if (MODE == 1) {
#pragma unroll
        for (int k = 0; k < kGroups; ++k) {
          const int c0 = k * 32;
          if (c0 >= it.n16) break;
          uint32_t v[32];
          tmem_ld32(dbase + c0, v);
          const int ncol = min(32, it.ntok - c0);
          __nv_bfloat16* dst = p.partial + it.p * 128 + r;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int slot = __shfl_sync(0xffffffffu, sl_r[k], c);
            const float wt = __shfl_sync(0xffffffffu, w_r[k], c);
            if (c < ncol) dst[(size_t)slot * p.H] = __float2bfloat16(__uint_as_float(v[c]) * wt);
          }
        }
      }
      for (int c0 = 0; MODE == 0 && c0 < it.n16; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(dbase + c0, v);
        if (MODE == 0) {
          // intermediate rows stay in expert-sorted order (the w2 pass reads
          // them as contiguous tiles)
          __nv_bfloat16* dst = p.inter + (size_t)(it.base + c0) * p.I + it.p * 64 + r;
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
                dst[(size_t)(h + c) * p.I] = __float2bfloat16(silu_f(gv) * uv);
              }
            }
            named_barrier_sync(2, kPfEpiWarps * 32);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
      if (p.trace != nullptr && tid == 0) pf_trace(p.trace, 6, n);
    }
  }

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kPfTmemCols);
}

// xs[pos, :] = x[sorted[pos] / x_row_div, :] for pos < num_post: the w13 token
// rows in expert-sorted order, so the GEMM reads them as contiguous tiles.
__global__ void moe_permute_rows_kernel(const __nv_bfloat16* x, long long x_ld, int x_row_div,
                                        const int32_t* sorted, const int32_t* num_post, int H,
                                        __nv_bfloat16* xs) {
  const int n = num_post[0], h8 = H / 8;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < (long long)n * h8;
       idx += (long long)gridDim.x * blockDim.x) {
    const int pos = (int)(idx / h8), c = (int)(idx - (long long)pos * h8) * 8;
    const int row = sorted[pos] / x_row_div;
    *reinterpret_cast<uint4*>(xs + (size_t)pos * H + c) =
        *reinterpret_cast<const uint4*>(x + (size_t)row * x_ld + c);
  }
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
  return (size_t)stages * kPfStageBytes + kPfWStages * kPfStaging + kPfXchgCols * 64 * 4 + (4 * E + 1) * 4;
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

// cuTensorMapEncodeTiled, resolved through the runtime (no link-time libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// Tensor maps over a row-major bf16 matrix [rows, cols]: boxes of 64 columns
// (128 B) x (32 * (i + 1)) rows, 128-byte swizzled -- the layout of the B tiles.
static cudaError_t rows_tmaps(PfRowMaps* maps, const __nv_bfloat16* base, long long rows, long long cols) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)(rows > 0 ? rows : 1)};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t estr[2] = {1, 1};
  for (int i = 0; i < kPfMaxTok / kPfBoxRows; ++i) {
    const cuuint32_t box[2] = {64, (cuuint32_t)(kPfBoxRows * (i + 1))};
    const CUresult r = fn(&maps->m[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  return cudaSuccess;
}

// Tensor maps over the fragment-major weights (E * n_rowtiles, n_chunks,
// 512 B) and scales (.., 64 B) as u32 elements: boxes of 4 row tiles x kPfWK
// k-blocks, unswizzled.
static cudaError_t weight_tmaps(CUtensorMap* mw, CUtensorMap* ms, const PrefillParams& p) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return cudaErrorNotSupported;
  const cuuint64_t tiles = (cuuint64_t)p.E * p.n_rowtiles, ch = (cuuint64_t)p.n_chunks;
  const cuuint32_t estr[3] = {1, 1, 1};
  const cuuint64_t wd[3] = {128, ch, tiles}, wst[2] = {512, 512 * ch};
  const cuuint32_t wb[3] = {128, kPfWK, 4};
  CUresult r = fn(mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(p.w), wd, wst, wb, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const cuuint64_t sd[3] = {16, ch, tiles}, sst[2] = {64, 64 * ch};
  const cuuint32_t sb[3] = {16, kPfWK, 4};
  r = fn(ms, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(p.s), sd, sst, sb, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_prefill_w13(const PrefillParams& p13, int sms, cudaStream_t stream) {
  cudaError_t err = prefill_config(p13.E, p13.n_stages);
  if (err != cudaSuccess) return err;
  PfRowMaps tm;
  err = rows_tmaps(&tm, p13.xs, p13.n_tok, p13.H);
  if (err != cudaSuccess) return err;
  CUtensorMap tw, ts;
  err = weight_tmaps(&tw, &ts, p13);
  if (err != cudaSuccess) return err;
  const long long work = (long long)p13.n_tok * (p13.H / 8);
  const int blocks = (int)std::min<long long>((work + 255) / 256, (long long)sms * 8);
  moe_permute_rows_kernel<<<blocks > 0 ? blocks : 1, 256, 0, stream>>>(p13.x, p13.x_ld, p13.x_row_div, p13.sorted,
                                                                       p13.num_post, p13.H, p13.xs);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  moe_prefill_kernel<0><<<sms, kPfThreads, prefill_smem_bytes(p13.E, p13.n_stages), stream>>>(p13, tm, tw, ts);
  return cudaGetLastError();
}

cudaError_t launch_prefill_w2(const PrefillParams& p2, const SlotMap& map, int M, int topk, int H,
                              __nv_bfloat16* out, int sms, cudaStream_t stream) {
  cudaError_t err = prefill_config(p2.E, p2.n_stages);
  if (err != cudaSuccess) return err;
  PfRowMaps tm;
  err = rows_tmaps(&tm, p2.inter, p2.n_tok, p2.I);
  if (err != cudaSuccess) return err;
  CUtensorMap tw, ts;
  err = weight_tmaps(&tw, &ts, p2);
  if (err != cudaSuccess) return err;
  moe_prefill_kernel<1><<<sms, kPfThreads, prefill_smem_bytes(p2.E, p2.n_stages), stream>>>(p2, tm, tw, ts);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  const long long work = (long long)M * (H / 8);
  const int blocks = (int)std::min<long long>((work + 255) / 256, (long long)sms * 8);
  moe_topk_sum_kernel<<<blocks > 0 ? blocks : 1, 256, 0, stream>>>(p2.partial, out, map, M, topk, H);
  return cudaGetLastError();
}

}  // namespace w4moe
