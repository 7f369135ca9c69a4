// Fused small-M MoE layer for the fewest-tokens-per-expert regime (at most
// ~1.5 routed slots per active expert, hidden rows <= 72 KB): routing + w13
// (+SiLU*up) + w2 (+ router-weighted top-k sum) in one persistent cooperative
// kernel in which every warp streams its own weights.  An alternative to the
// staged decode kernel (decode.cu), selected with w4a16_set_path(3); on B200
// the re-tuned staged kernel measured at least as fast at every M, so the
// automatic path does not pick this one.
//
// Replaces, in that regime, the reference's moe_align_block_size +
// _w4a16_moe_w1_fused_kernel + _w4a16_moe_w2_kernel + _moe_sum_kernel
// (kernels/w4a16_moe.py:187-290, :374-670).
//
// Structure (no producer warp, no stage ring, no epilogue warps):
//   * the CTA copies the hidden rows [M, H] into shared memory once;
//   * units: w13 (expert, pass of <= 8 tokens, gate/up pair, gate or up half)
//            and w2 (expert, pass, 16-row tile); all w13 units precede all w2
//            units; warp g of the grid takes units g, g + warps, ...;
//   * a w13 warp streams its row tile's fragment-major weight and scale
//     blocks from global memory into registers, 2 x kDdG chunks (64 k each)
//     ahead and refilled kDdG consecutive chunks at a time (DRAM page
//     locality), decodes int4 -> bf16 (code - 8, exact) into m16n8k16 A
//     fragments and multiplies with B fragments read from the staged hidden
//     rows; the bf16 group scales multiply the fp32 partial of each 32-wide
//     group; the gate and up warps of a pair meet in shared memory, the gate
//     warp writes bf16(silu(gate) * up) and bumps the expert's readiness
//     counter;
//   * a w2 warp bulk-copies its whole row tile into its shared buffer (the
//     first one at kernel start, so w2 weights stream during the w13 units),
//     waits (bounded) until the expert's w13 pairs have all published, copies
//     the tokens' intermediate rows next to it, multiplies, scales by the
//     router weight into fp32 partials, and the last unit to finish a (token,
//     32-row block) sums that token's partials in slot order (deterministic).
// Every wait is bounded; counters are self-cleaning.
#include "launch.cuh"

namespace w4moe {

constexpr int kDdWarps = 12;
constexpr int kDdThreads = kDdWarps * 32;
constexpr int kDdNB = 8;       // tokens per pass (one n8 MMA column block)
constexpr int kDdG = 4;        // weight chunks per refill group (2 groups in flight per warp)
constexpr int kDdSplitA = 2;   // w13 pair = gate warp + up warp
constexpr int kDdBRowElems = 1024;  // per-warp staged intermediate (1 row of I = 1024)
constexpr int kDdMaxChB = 16;       // w2 tile k-chunks held in a warp's shared buffer (I <= 1024)
constexpr int kDdWBuf = kDdMaxChB * 576;  // one w2 row tile: packed words + scales
constexpr int kDdMaxXBytes = 72 * 1024;  // hidden rows staged in shared memory
constexpr long long kDdBudget = 2000000000LL;  // SM clocks

// sched[] words shared with the staged decode kernel
constexpr int kDdSchedDone = 1, kDdSchedError = 2;
constexpr int kDdErrReady = 4;

struct DdChunk {
  uint4 w;   // one row tile's fragment words for one 64-k chunk
  uint2 s;   // its group scales
};

// diagnostics (CTA 0, first unit of each warp): tr[warp * 8 + event]; events 0
// unit start, 1 weights of the first chunks landed, 2 compute loop done,
// 3 unit done, 4 ready observed (w2), 6 prologue done (warp 0), 7 kernel start
__device__ __forceinline__ void dd_trace(long long* tr, int warp, int ev) {
  if (tr != nullptr && blockIdx.x == (unsigned)tr[127]) tr[warp * 8 + ev] = global_timer_ns();
}

__device__ __forceinline__ float dd_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float dd_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// acc[4] (C fragment of one row tile) += scale-weighted MMA of one 64-k chunk.
__device__ __forceinline__ void dd_chunk_mma(float (&acc)[4], const uint4& wv, const uint2& sv,
                                             const uint32_t (&b)[8]) {
  uint32_t A0[4], A1[4], A2[4], A3[4];
  unscaled_word(wv.x, A0);
  unscaled_word(wv.y, A1);
  unscaled_word(wv.z, A2);
  unscaled_word(wv.w, A3);
  float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
  mma_bf16_16816_nv(t0, A0, b[0], b[1]);
  mma_bf16_16816_nv(t1, A2, b[4], b[5]);
  mma_bf16_16816_nv(t0, A1, b[2], b[3]);
  mma_bf16_16816_nv(t1, A3, b[6], b[7]);
  const float s0 = dd_lo(sv.x), s08 = dd_hi(sv.x), s1 = dd_lo(sv.y), s18 = dd_hi(sv.y);
  acc[0] = fmaf(s0, t0[0], fmaf(s1, t1[0], acc[0]));
  acc[1] = fmaf(s0, t0[1], fmaf(s1, t1[1], acc[1]));
  acc[2] = fmaf(s08, t0[2], fmaf(s18, t1[2], acc[2]));
  acc[3] = fmaf(s08, t0[3], fmaf(s18, t1[3], acc[3]));
}

// B fragments of one 64-k chunk for this lane's token row (k16 steps 0..3):
// CG = false reads shared memory (staged rows), true reads global through L2.
template <bool CG>
__device__ __forceinline__ void dd_load_b(uint32_t (&b)[8], const __nv_bfloat16* row, int c, int t) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(row + c * 64) + t;
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    if (CG) {
      b[2 * s] = __ldcg(p + s * 8);
      b[2 * s + 1] = __ldcg(p + s * 8 + 4);
    } else {
      b[2 * s] = p[s * 8];
      b[2 * s + 1] = p[s * 8 + 4];
    }
  }
}

__device__ __forceinline__ void dd_load_chunk(DdChunk& ch, const uint8_t* w, const uint8_t* s, size_t blk,
                                              int lane, int g) {
  ch.w = ldg_stream(reinterpret_cast<const uint4*>(w + blk * 512) + lane);
  ch.s = __ldg(reinterpret_cast<const uint2*>(s + blk * 64) + g);
}

// Chunk visited at step c of a tile whose walk starts at chunk `rot`: tiles
// start at different offsets so that the warps streaming neighbouring row
// tiles (24 KB apart) do not hit the same DRAM channels at the same time.
__device__ __forceinline__ int dd_rot(int c, int rot, int n) {
  const int x = c + rot;
  return x >= n ? x - n : x;
}

// acc += the unit's row tile over its n chunks (blocks blk0 + chunk).  Weights
// stay 2 x kDdG chunks ahead, refilled a group of kDdG consecutive chunks at a
// time: back-to-back requests to one 2 KB stretch keep DRAM pages open, which
// doubles what scattered 512-byte requests of many warps achieve.  B fragments
// come from `row` (shared memory or, with CG, global through L2).
__device__ __forceinline__ void dd_load_group(DdChunk (&gr)[kDdG], const uint8_t* w, const uint8_t* s, size_t blk0,
                                              int c, int n, int rot, int lane, int g) {
#pragma unroll
  for (int d = 0; d < kDdG; ++d)
    if (c + d < n) dd_load_chunk(gr[d], w, s, blk0 + dd_rot(c + d, rot, n), lane, g);
}

template <bool CG>
__device__ __forceinline__ void dd_compute_group(float (&acc)[4], const DdChunk (&gr)[kDdG], int c, int n, int rot,
                                                 const __nv_bfloat16* row, int t) {
#pragma unroll
  for (int d = 0; d < kDdG; ++d) {
    if (c + d < n) {
      uint32_t b[8];
      dd_load_b<CG>(b, row, dd_rot(c + d, rot, n), t);
      dd_chunk_mma(acc, gr[d].w, gr[d].s, b);
    }
  }
}

template <bool CG>
__device__ __forceinline__ void dd_stream_tile(float (&acc)[4], const uint8_t* w, const uint8_t* s, size_t blk0,
                                               int n, int rot, const __nv_bfloat16* row, int lane, int g, int t,
                                               DdChunk (&ga)[kDdG], DdChunk (&gb)[kDdG], bool preloaded) {
  if (!preloaded) {
    dd_load_group(ga, w, s, blk0, 0, n, rot, lane, g);
    dd_load_group(gb, w, s, blk0, kDdG, n, rot, lane, g);
  }
  for (int c = 0; c < n; c += 2 * kDdG) {
    dd_compute_group<CG>(acc, ga, c, n, rot, row, t);
    if (c + 2 * kDdG < n) dd_load_group(ga, w, s, blk0, c + 2 * kDdG, n, rot, lane, g);
    dd_compute_group<CG>(acc, gb, c + kDdG, n, rot, row, t);
    if (c + 3 * kDdG < n) dd_load_group(gb, w, s, blk0, c + 3 * kDdG, n, rot, lane, g);
  }
}

__global__ void __launch_bounds__(kDdThreads, 1) moe_decode_direct_kernel(DecodeParams p) {
  extern __shared__ __align__(16) int dd_smem[];
  __shared__ float xchg[kDdWarps / 2][8][32];  // w13 K-half partials (gate 4 + up 4 per lane)
  __shared__ int s_nact, s_nA, s_nB;

  const int E = p.E;
  int* cnt = dd_smem;                 // [E]
  int* off = cnt + E;                 // [E+1]
  int* act = off + E + 1;             // [E]
  int* cur = act + E;                 // [E]
  int* cumP = cur + E;                // [E+1] prefix of passes over active experts
  int* slots = cumP + E + 1;          // [n_tok]
  int* tokcnt = slots + p.n_tok;      // [M]
  unsigned* sok = reinterpret_cast<unsigned*>(tokcnt + p.M);  // [n_tok/32+1]
  int* eid = reinterpret_cast<int*>(sok + p.n_tok / 32 + 1);   // [n_tok] local expert per slot
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(
      dd_smem + ((5 * E + 2 + 2 * p.n_tok + p.M + p.n_tok / 32 + 1 + 3) & ~3));  // [M, H] staged hidden rows

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  if (tid == 0) dd_trace(p.trace, 0, 7);
  __nv_bfloat16* const bbuf = xs + (size_t)p.M * p.H + (size_t)warp * kDdBRowElems;  // this warp's w2 rows
  unsigned char* const wbuf = reinterpret_cast<unsigned char*>(xs + (size_t)p.M * p.H + kDdWarps * kDdBRowElems) +
                              (size_t)warp * kDdWBuf;  // this warp's w2 tile (weights, then scales)
  __shared__ uint64_t wbar[kDdWarps];

  // ---------------- routing tables (every CTA builds its own copy) ----------------
  {  // hidden rows -> shared memory (read by every w13 unit of this CTA)
    const int h8 = p.H / 8;
    for (int i = tid; i < p.M * h8; i += kDdThreads) {
      const int m = i / h8, c = i - m * h8;
      cp_async16_zfill(xs + (size_t)m * p.H + c * 8, p.hidden + (size_t)m * p.hidden_ld + c * 8, true);
    }
    cp_async_commit();
  }
  if (tid < kDdWarps) mbar_init(&wbar[tid], 1);
  fence_barrier_init();
  for (int e = tid; e < E; e += kDdThreads) cnt[e] = 0;
  for (int m = tid; m < p.M; m += kDdThreads) tokcnt[m] = 0;
  for (int w = tid; w <= p.n_tok / 32; w += kDdThreads) sok[w] = 0;
  __syncthreads();
  for (int i = tid; i < p.n_tok; i += kDdThreads) {
    const int e = p.map(i);
    eid[i] = e;
    if (e >= 0) {
      atomicAdd(&cnt[e], 1);
      atomicAdd(&tokcnt[i / p.topk], 1);
      atomicOr(&sok[i >> 5], 1u << (i & 31));
    }
  }
  __syncthreads();
  if (warp == 0) {
    int run = 0, nact = 0, runP = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < E ? cnt[e] : 0;
      const int pc = (c + kDdNB - 1) / kDdNB;
      int inc = c, ia = c > 0, ip = pc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, inc, o);
        const int b = __shfl_up_sync(0xffffffffu, ia, o);
        const int d = __shfl_up_sync(0xffffffffu, ip, o);
        if (lane >= o) {
          inc += a;
          ia += b;
          ip += d;
        }
      }
      if (e < E) {
        off[e] = run + inc - c;
        cur[e] = run + inc - c;
        if (c > 0) {
          act[nact + ia - 1] = e;
          cumP[nact + ia - 1] = runP + ip - pc;
        }
      }
      run += __shfl_sync(0xffffffffu, inc, 31);
      nact += __shfl_sync(0xffffffffu, ia, 31);
      runP += __shfl_sync(0xffffffffu, ip, 31);
    }
    if (lane == 0) {
      off[E] = run;
      cumP[nact] = runP;
      s_nact = nact;
      s_nA = runP * (p.I / 16) * kDdSplitA;
      s_nB = runP * (p.H / 32) * 2;
    }
  }
  __syncthreads();
  if (warp == 0) ordered_slot_scatter(eid, p.n_tok, cur, slots, lane);
  cp_async_wait_group<0>();
  if (p.zero_rows) {  // expert parallelism: tokens with no local slot get a zero row
    for (int m = blockIdx.x * kDdThreads + tid; m < p.M; m += gridDim.x * kDdThreads)
      if (tokcnt[m] == 0)
        for (int h = 0; h < p.H; h += 8)
          *reinterpret_cast<uint4*>(p.out + (size_t)m * p.H + h) = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();

  const int nact = s_nact, nA = s_nA, nB = s_nB;
  if (tid == 0) dd_trace(p.trace, 0, 6);
  long long* const tr = (lane == 0) ? p.trace : nullptr;
  const int PA = p.I / 16;             // gate/up pairs per expert pass
  const int PB = p.H / 32;             // 32-row blocks per expert pass
  const int nrtA = 2 * p.I / 16, nchA = p.H / 64;
  const int nrtB = p.H / 16, nchB = p.I / 64;
  const int nwarps = gridDim.x * kDdWarps;
  const int gw = blockIdx.x * kDdWarps + warp;

  // pass index pi (over all active experts' passes) -> active expert j
  auto expert_of_pass = [&](int pi) {
    int lo = 0, hi = nact - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cumP[mid] <= pi) lo = mid; else hi = mid - 1;
    }
    return lo;
  };

  // w2 unit ub -> first fragment block of its row tile
  auto w2_block = [&](int ub) {
    const int half = ub & 1;
    const int pi = (ub >> 1) / PB, rb = (ub >> 1) - pi * PB;
    const int e = act[expert_of_pass(pi)];
    return ((size_t)e * nrtB + 2 * rb + half) * nchB;
  };
  auto issue_w2 = [&](int ub) {  // whole row tile -> this warp's buffer (lane 0)
    const size_t b0 = w2_block(ub);
    mbar_arrive_expect_tx(&wbar[warp], (uint32_t)nchB * 576);
    bulk_g2s(wbuf, p.w2 + b0 * 512, (uint32_t)nchB * 512, &wbar[warp]);
    bulk_g2s(wbuf + nchB * 512, p.s2 + b0 * 64, (uint32_t)nchB * 64, &wbar[warp]);
  };
  uint32_t wphase = 0;  // w2 tiles this warp has loaded (its barrier's parity)
  // The first w2 unit of this warp (often a second-round unit after a w13
  // unit) is copied at kernel start, so all first-round w2 weights stream
  // concurrently with the w13 units.
  int prefetched = -1;
  {
    int u0 = gw;
    if (u0 < nA) u0 += ((nA - u0 + nwarps - 1) / nwarps) * nwarps;
    if (u0 < nA + nB) {
      prefetched = u0;
      if (lane == 0) issue_w2(u0 - nA);
    }
  }
  for (int u = gw; u < nA + nB; u += nwarps) {
    const bool first = u == gw;
    if (first) dd_trace(tr, warp, 0);
    if (u < nA) {
      // ======================= w13 unit: (pass, pair q, gate or up h) =======================
      const int h = u % kDdSplitA, pu = u / kDdSplitA;
      const int pi = pu / PA, q = pu - pi * PA;
      const int j = expert_of_pass(pi);
      const int e = act[j], pass = pi - cumP[j];
      const int T = cnt[e], base = off[e] + pass * kDdNB;
      const int ntok = min(kDdNB, T - pass * kDdNB);
      const int col = g < ntok ? g : 0;  // this lane's B column (token); extra columns are ignored
      const int slot = slots[base + col];
      const __nv_bfloat16* xrow = xs + (size_t)(slot / p.topk) * p.H;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      DdChunk ga[kDdG], gb[kDdG];
      const int rotA = (int)(((unsigned)(q * 2 + h) * 7u) % (unsigned)nchA);
      dd_stream_tile<false>(acc, p.w13, p.s13, ((size_t)e * nrtA + h * PA + q) * nchA, nchA, rotA, xrow, lane, g,
                            t, ga, gb, false);
      if (first) dd_trace(tr, warp, 2);
      // gate (warp 2k) and up (warp 2k+1) tiles meet in shared memory
      float* xc = &xchg[warp >> 1][0][lane];
      if (h == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) xc[i * 32] = acc[i];
      }
      named_barrier_sync(1 + (warp >> 1), 64);
      if (h == 0) {
        float accg[4], accu[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          accg[i] = acc[i];
          accu[i] = xc[i * 32];
        }
        // rows g, g+8 of pair q; token columns 2t, 2t+1
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int cc = 2 * t + (i & 1), row = q * 16 + g + 8 * (i >> 1);
          if (cc < ntok)
            p.inter[(size_t)slots[base + cc] * p.I + row] = __float2bfloat16(silu_f(accg[i]) * accu[i]);
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.ready + e, 1);
      }
      named_barrier_sync(1 + (warp >> 1), 64);  // xchg free for the next pair
      if (first) dd_trace(tr, warp, 3);
    } else {
      // ======================= w2 unit: (pass, 32-row block rb) =======================
      const int ub = u - nA;
      const int half = ub & 1;  // tile 2rb + half of the 32-row block
      const int pi = (ub >> 1) / PB, rb = (ub >> 1) - pi * PB;
      const int j = expert_of_pass(pi);
      const int e = act[j], pass = pi - cumP[j];
      const int T = cnt[e], base = off[e] + pass * kDdNB;
      const int ntok = min(kDdNB, T - pass * kDdNB);
      const int col = g < ntok ? g : 0;
      const int slot = slots[base + col];
      const __nv_bfloat16* irow = p.inter + (size_t)slot * p.I;
      const size_t b0 = ((size_t)e * nrtB + 2 * rb + half) * nchB;
      float acc0[4] = {0.f, 0.f, 0.f, 0.f};
      // the whole row tile (nchB x 512 B words + nchB x 64 B scales, each
      // contiguous) is bulk-copied into this warp's buffer before the
      // readiness wait, so w2 weights stream while the w13 units still run
      if (lane == 0 && u != prefetched) issue_w2(ub);
      // intermediate rows of expert e are complete once all its pairs of all passes published
      if (lane == 0) {
        const int target = PA * ((T + kDdNB - 1) / kDdNB);
        const long long t0 = clock64();
        while (ld_acquire_gpu(p.ready + e) < target) {
          if (clock64() - t0 > kDdBudget) {
            atomicOr(p.sched + kDdSchedError, kDdErrReady);
            break;
          }
          __nanosleep(64);
        }
      }
      __syncwarp();
      if (first) dd_trace(tr, warp, 4);
      // the unit's intermediate rows into this warp's shared buffer when they fit
      const bool staged = ntok * p.I <= kDdBRowElems;
      const __nv_bfloat16* brow = irow;
      if (staged) {
        const int i8 = p.I / 8;
        for (int i = lane; i < ntok * i8; i += 32) {
          const int cc = i / i8, k8 = i - cc * i8;
          cp_async16_zfill(bbuf + cc * p.I + k8 * 8, p.inter + (size_t)slots[base + cc] * p.I + k8 * 8, true);
        }
        cp_async_commit();
        cp_async_wait_group<0>();
        __syncwarp();
        brow = bbuf + col * p.I;
      }
      if (!mbar_wait(&wbar[warp], wphase & 1u, kDdBudget)) {
        if (lane == 0) atomicOr(p.sched + kDdSchedError, kDdErrReady);
      }
      ++wphase;
      for (int c = 0; c < nchB; ++c) {
        uint32_t b[8];
        if (staged) dd_load_b<false>(b, brow, c, t);
        else dd_load_b<true>(b, irow, c, t);
        const uint4 wv = lds128(wbuf + c * 512 + lane * 16);
        const uint2 sv = lds64(wbuf + nchB * 512 + c * 64 + g * 8);
        dd_chunk_mma(acc0, wv, sv, b);
      }
      __syncwarp();  // buffer reads done before the next tile's copy
      if (first) dd_trace(tr, warp, 2);
      // router-weighted fp32 partials: rows rb*32 + {g, g+8} (+16), token columns 2t, 2t+1
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int cc = 2 * t + (i & 1);
        if (cc < ntok) {
          const int s = slots[base + cc];
          const float wt = p.topk_w[s];
          const int row = rb * 32 + half * 16 + g + 8 * (i >> 1);
          p.partial[(size_t)s * p.H + row] = acc0[i] * wt;
        }
      }
      __threadfence();
      __syncwarp();
      // the last unit to finish (token, row block) sums the token's partials in slot order
      int mine = -1;
      if (lane < ntok) {
        const int m = slots[base + lane] / p.topk;
        int* cptr = p.counters + (size_t)m * PB + rb;
        if (atomicAdd(cptr, 1) == 2 * tokcnt[m] - 1) {  // both 16-row halves of every slot
          *cptr = 0;  // self-cleaning
          mine = m;
        }
      }
      unsigned todo = __ballot_sync(0xffffffffu, mine >= 0);
      if (todo) __threadfence();
      while (todo) {
        const int src = __ffs(todo) - 1;
        todo &= todo - 1;
        const int m = __shfl_sync(0xffffffffu, mine, src);
        const int hr = rb * 32 + lane;
        const float* pp = p.partial + (size_t)m * p.topk * p.H + hr;
        float sum = 0.f;
        for (int tt = 0; tt < p.topk; ++tt) {
          const int s = m * p.topk + tt;
          const float x = __ldcg(pp + (size_t)tt * p.H);
          if ((sok[s >> 5] >> (s & 31)) & 1u) sum += x;
        }
        p.out[(size_t)m * p.H + hr] = __float2bfloat16(sum);
      }
      if (first) dd_trace(tr, warp, 3);
    }
  }

  // ---------------- teardown: the last CTA resets the readiness counters ----------------
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.sched + kDdSchedDone, 1) == (int)gridDim.x - 1) {
      p.sched[kDdSchedDone] = 0;
      for (int e = 0; e < E; ++e) p.ready[e] = 0;
      __threadfence();
    }
  }
}

size_t decode_direct_smem_bytes(const DecodeParams& p) {
  return (size_t)((5 * p.E + 2 + 2 * p.n_tok + p.M + p.n_tok / 32 + 1 + 3) & ~3) * 4 + (size_t)p.M * p.H * 2 +
         (size_t)kDdWarps * kDdBRowElems * 2 + (size_t)kDdWarps * kDdWBuf;
}

// Shapes the kernel supports: pairs split in two K halves of whole 64-k chunks.
bool decode_direct_ok(const DecodeParams& p, int max_smem) {
  return p.NG == 1 && p.M >= p.direct_min_m && (p.H / 64) % kDdSplitA == 0 && p.H % 32 == 0 && p.I % 16 == 0 && p.I / 64 <= kDdMaxChB &&
         (((uintptr_t)p.w2 | (uintptr_t)p.s2) & 15) == 0 &&
         (size_t)p.M * p.H * 2 <= (size_t)kDdMaxXBytes &&
         decode_direct_smem_bytes(p) + sizeof(float) * 8 * 8 * 32 + 1024 <= (size_t)max_smem;
}

cudaError_t launch_decode_direct(const DecodeParams& p, cudaStream_t stream) {
  static thread_local size_t configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const size_t smem = decode_direct_smem_bytes(p);
  if (smem > 48 * 1024 && configured[dev] < smem) {
    cudaError_t err = cudaFuncSetAttribute(moe_decode_direct_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err != cudaSuccess) return err;
    configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kDdThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, moe_decode_direct_kernel, p);
}

}  // namespace w4moe
