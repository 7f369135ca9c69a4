// Expert-sliced fused decode layer for the smallest batches (M <= 4 tokens,
// M*topk <= 64 slots): routing + w13 (+SiLU*up) + w2 (+ router-weighted top-k
// sum) in ONE persistent kernel, one CTA per SM.
//
// Replaces, for those batches, the reference's moe_align_block_size +
// _w4a16_moe_w1_fused_kernel + _w4a16_moe_w2_kernel + _moe_sum_kernel
// (kernels/w4a16_moe.py:187-290, :374-670 in the reference).
//
// Work split (every CTA derives the same schedule from the routing, no
// scheduler state in memory):
//   * w13: the unit is one gate/up row-tile PAIR of one routed expert (16
//     intermediate columns over the full hidden K).  Pair q of the expert-major
//     list (q = active_expert * I/16 + pair) goes to CTA q % G in round q / G,
//     so every CTA works through the experts in ascending order and expert e
//     is complete after round ((e+1) * I/16 - 1) / G.  A pair is finished by
//     one CTA: SiLU(gate)*up is applied locally and written once, then the
//     expert's readiness counter is bumped (no split-K fix-ups).
//   * w2: the unit is one (hidden row tile, expert) block over the full
//     intermediate K.  Units are numbered row-tile-major (r * A + e) and each
//     CTA takes one contiguous range, sized so that w13 + w2 bytes per CTA are
//     equal (CTAs with one pair fewer take six more w2 tiles at 3072x1024).
//     A CTA processes its w2 units expert by expert, interleaved with its w13
//     rounds one round after the expert became ready, so only the last expert
//     is waited for at the end.  The top-k sum of a row tile stays in the CTA
//     (fp32 in shared memory, experts in ascending order); a row tile split
//     between CTAs is finished by the CTA holding its last expert, which adds
//     the other CTAs' fp32 pieces in CTA order (deterministic).
//   * the CTA's schedule is a table of items (a w13 pair, or up to four w2 row
//     tiles of one expert), built once in the prologue.  Each of the 16
//     consumer warps walks every item, taking the 64-wide k-chunks warp,
//     warp + 16, ...: it streams its own weight and scale blocks with cp.async
//     into a private shared-memory ring kSlDepth groups ahead (so at any moment
//     the CTA reads a contiguous stretch of each tile), decodes int4 straight
//     into m16n8k16 A fragments (code - 8 exact in bf16; the bf16 group scale
//     is applied to the fp32 partial of each 32-wide group), and meets the
//     other warps only at the end of an item, in a double-buffered reduction
//     buffer.  Token rows (hidden, intermediate) live in shared memory in a
//     lane-permuted layout (two 16-byte loads give a lane its B fragments for
//     a 64-wide chunk).
//   * one epilogue warp reduces the 16 warps' partials of an item in fixed
//     warp order, applies SiLU*up (w13) or the router weight (w2), publishes.
//   * one loader warp waits (bounded) for each expert's readiness and copies
//     its intermediate rows into shared memory.
//
// All global counters / flags are self-cleaning.  Every wait is bounded
// (clock64 budget); a timeout records an error bit in the workspace status word
// (w4a16_moe_read_status) and aborts the CTA after in-flight copies land.
#include <stdlib.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "launch.cuh"

namespace w4moe {

namespace {

constexpr int kSlConsumers = 16;
constexpr int kSlEpilogue = 16;  // warp index
constexpr int kSlLoader = 17;
constexpr int kSlThreads = 18 * 32;
constexpr int kSlDepth = 4;             // cp.async groups in flight per consumer warp
constexpr int kSlMaxTiles = 4;          // row tiles per w2 item
constexpr long long kSlBudget = 4000000000LL;  // ~2 s of SM clocks
constexpr int kSlMaxA = kSlicedMaxSlots;        // active experts <= slots

// error bits in the workspace status word (sched[2])
constexpr int kSlErrRed = 1 << 10, kSlErrReady = 1 << 11, kSlErrInter = 1 << 12, kSlErrPiece = 1 << 13;

struct SlCtx {
  int A, P, G, c, chA, chB, NR, T2, lag, nrt2;
  int S0, S1;
};

// One item of the CTA's schedule.
struct SlEntry {
  int4 meta;  // y: type (0 = w13 pair, 1 = w2 tiles) | ntile << 4 | ae << 16; z: tile0; w: nch
};

// Round in which the last pair of active expert e is computed.
__host__ __device__ __forceinline__ int sl_ready_round(int e, int P, int G) { return ((e + 1) * P - 1) / G; }

// w2 row tiles [ra, rb] of active expert ae inside the CTA's unit range [S0, S1)
__host__ __device__ __forceinline__ void sl_w2_tiles(int ae, int A, int S0, int S1, int& ra, int& rb) {
  ra = S0 <= ae ? 0 : (S0 - ae + A - 1) / A;
  rb = S1 - 1 < ae ? -1 : (S1 - 1 - ae) / A;
}

__device__ __forceinline__ void sl_record(int32_t* sched, int code) { atomicOr(sched + 2, code); }

// Bounded mbarrier wait that also gives up once the CTA is aborting.
__device__ __forceinline__ bool sl_wait(uint64_t* bar, uint32_t parity, const volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kSlBudget) return false;
  }
}

__device__ __forceinline__ void red_release_add(int32_t* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release(int32_t* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Lane-permuted position of element i of a token row: inside each 64-wide
// chunk, lane t of a quad finds the 16 values of its four k16 steps
// (k = 16j + {2t, 2t+1, 2t+8, 2t+9}, j = 0..3) at [16t, 16t+16).
__device__ __forceinline__ int sl_perm(int i) {
  return (i & ~63) + (((i & 7) >> 1) << 4) + (((i & 63) >> 4) << 2) + (i & 1) + (((i >> 3) & 1) << 1);
}

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// One 16-row x 64-k block: acc[0..3] += scale * (A_block . B) for this lane's
// D fragment (rows g, g+8; columns 2t, 2t+1).
__device__ __forceinline__ void sl_block(float (&acc)[4], const uint4 wv, const uint2 sv, const uint4 q0,
                                         const uint4 q1) {
  uint32_t a[4];
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  unscaled_word(wv.x, a);
  mma_bf16_16816_nv(d0, a, q0.x, q0.y);
  unscaled_word(wv.y, a);
  mma_bf16_16816_nv(d0, a, q0.z, q0.w);
  unscaled_word(wv.z, a);
  mma_bf16_16816_nv(d1, a, q1.x, q1.y);
  unscaled_word(wv.w, a);
  mma_bf16_16816_nv(d1, a, q1.z, q1.w);
  const float s0g = bf_lo(sv.x), s0h = bf_hi(sv.x), s1g = bf_lo(sv.y), s1h = bf_hi(sv.y);
  acc[0] = fmaf(s0g, d0[0], fmaf(s1g, d1[0], acc[0]));
  acc[1] = fmaf(s0g, d0[1], fmaf(s1g, d1[1], acc[1]));
  acc[2] = fmaf(s0h, d0[2], fmaf(s1h, d1[2], acc[2]));
  acc[3] = fmaf(s0h, d0[3], fmaf(s1h, d1[3], acc[3]));
}

__device__ __forceinline__ void sl_trace(long long* tr, int kind, int k) {
  if (tr != nullptr && k < 128) {
    tr[kind * 256 + k] = global_timer_ns();
    tr[kind * 256 + 128 + k] = clock64();
  }
}

}  // namespace

// First w2 unit (row-tile-major numbering r * A + e) of CTA c: contiguous
// ranges sized so that every CTA streams the same weight bytes, counting a
// w13 pair as 2*chA chunk blocks and a w2 tile as chB.  All intermediate
// values stay below 2^31 for the shapes sliced_plan accepts.
__host__ __device__ int sliced_w2_start(int c, int A, int P, int G, int chA, int chB, int nrt2) {
  const int T2 = A * nrt2;
  const int rem = (A * P) % G;
  if (rem == 0) return T2 * c / G;
  const int W2 = T2 * chB, X = 2 * chA * (G - rem);
  if (W2 <= X) return c <= rem ? 0 : T2 * (c - rem) / (G - rem);  // CTAs with the extra pair take no w2
  const int lo = c < rem ? c : rem, hi = c > rem ? c - rem : 0;
  return (lo * (W2 - X) + hi * (W2 - X + 2 * chA * G)) / (G * chB);
}

__global__ void __launch_bounds__(kSlThreads, 1) moe_decode_sliced_kernel(SlicedParams p) {
  __shared__ uint64_t red_full[2], red_empty[2], inter_bar[kSlMaxA], pc_bar;
  __shared__ int s_tok[kSlicedMaxSlots], s_eid[kSlicedMaxSlots], s_first[kSlicedMaxSlots];
  __shared__ float s_wt[kSlicedMaxSlots], s_wt_in[kSlicedMaxSlots];
  __shared__ int s_act[kSlMaxA], s_cnt[kSlMaxA], s_base[kSlMaxA];
  __shared__ int s_w2n[kSlMaxA], s_w2ins[kSlMaxA];
  __shared__ int s_A, s_nst;
  __shared__ int s_pc[kSlicedMaxPieces];
  __shared__ int s_npc;
  __shared__ volatile int s_abort;
  extern __shared__ __align__(128) unsigned char dsm[];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int M = p.M, H = p.H, I = p.I, G = gridDim.x, c = blockIdx.x;
  long long* const tr = (p.trace != nullptr && c == p.trace_cta) ? p.trace : nullptr;

  unsigned char* const xs = dsm + p.off_x;           // [M][H*2 + 16] lane-permuted hidden rows
  unsigned char* const inter_s = dsm + p.off_inter;  // [n_tok][I*2 + 16] lane-permuted intermediate rows
  float* const red = reinterpret_cast<float*>(dsm + p.off_red);    // [2][16 warps][maxT][16][Mp]
  float* const oacc = reinterpret_cast<float*>(dsm + p.off_oacc);  // [nr_cap][M][16]
  float* const pcs = reinterpret_cast<float*>(dsm + p.off_pc);     // [pc_cap][M][16]
  SlEntry* const table = reinterpret_cast<SlEntry*>(dsm + p.off_table);  // [max_stages]
  int* const rscratch = reinterpret_cast<int*>(dsm + p.off_rounds);      // [3][max_rounds + 1]
  unsigned char* const ring = dsm + p.off_ring;                          // [16 warps][kSlDepth][slot_bytes]
  const int xstride = H * 2 + 16, istride = I * 2 + 16;
  const int Mp = p.Mp, maxT = p.maxT;
  const int red_warp = maxT * 16 * Mp;  // floats per warp in one buffer
  const int slot_bytes = p.slot_bytes;

  // ---------------- prologue ----------------
  if (tid == 0) sl_trace(tr, 4, 0);
  if (warp == 0) {
    // Routing for <= 64 slots.  A "column" is one (expert, token) pair: the
    // slots of a token that name the same expert twice share one column whose
    // router weight is their sum (in slot order), so an expert has at most M
    // columns.  Columns are ordered by expert, then token; active experts
    // ascending.
    // Each slot gets the key e * 64 + token (or -1): keys order columns,
    // equal keys share a column, key >> 6 is the expert.
    const int n = p.n_tok;
    int k_l[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h;
      const int e = i < n ? p.map(i) : -1;
      k_l[h] = e >= 0 ? (e << 6) | (i / p.topk) : -1;
      if (i < n) {
        s_eid[i] = k_l[h];
        s_wt_in[i] = p.topk_w[i];
      }
    }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h;
      if (i < n) {
        // bit 0: first slot of its column; bit 1: first slot of its expert
        const int k = k_l[h];
        int same_e = 0, same_col = 0;
#pragma unroll 8
        for (int jj = 0; jj < i; ++jj) {
          const int kj = s_eid[jj];
          same_col |= kj == k;
          same_e |= (kj >> 6) == (k >> 6);
        }
        s_first[i] = k >= 0 ? ((same_col ? 0 : 1) | (same_e ? 0 : 2)) : 0;
      }
    }
    __syncwarp();
    int nact = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h;
      const int k = k_l[h], e = k >> 6;
      const bool mine = i < n && k >= 0 && (s_first[i] & 1);
      int col = 0, below = 0, same = 0, act_below = 0;
      float wsum = 0.f;
#pragma unroll 8
      for (int jj = 0; jj < n; ++jj) {
        const int kj = s_eid[jj];
        const int fj = s_first[jj];
        const int ej = kj >> 6;
        if (fj & 1) {
          col += kj < k;
          below += ej < e;
          same += ej == e;
        }
        act_below += (fj & 2) && ej < e;
        if (kj == k) wsum += s_wt_in[jj];
      }
      if (mine) {
        s_tok[col] = k & 63;
        s_wt[col] = wsum;
        if (s_first[i] & 2) {
          s_act[act_below] = e;
          s_base[act_below] = below;
          s_cnt[act_below] = same;
        }
      }
      nact += __popc(__ballot_sync(0xffffffffu, mine && (s_first[i] & 2)));
    }
    if (lane == 0) {
      s_A = nact;
      sl_trace(tr, 4, 3);
    }
  } else if (warp == kSlLoader) {
    // barriers, initialised lane-parallel
    for (int a = lane; a < kSlMaxA; a += 32) mbar_init(&inter_bar[a], 1);
    if (lane < 2) {
      mbar_init(&red_full[lane], kSlConsumers);
      mbar_init(&red_empty[lane], 1);
    }
    if (lane == 0) {
      mbar_init(&pc_bar, 1);
      s_abort = 0;
    }
    fence_barrier_init();
  } else {
    // hidden rows -> shared memory, lane-permuted (warps 1..16)
    const int h8 = H / 8, nthr = (kSlLoader - 1) * 32, me = tid - 32;
    for (int idx = me; idx < M * h8; idx += nthr) {
      const int m = idx / h8, k8 = idx - m * h8;
      const uint4 v = *reinterpret_cast<const uint4*>(p.hidden + (size_t)m * p.hidden_ld + k8 * 8);
      const int kk0 = k8 * 8, ch = kk0 >> 6, jq = (kk0 & 63) >> 4, hh = (kk0 >> 3) & 1;
      uint32_t* row = reinterpret_cast<uint32_t*>(xs + (size_t)m * xstride);
      const int base = ch * 64 + jq * 4 + 2 * hh;  // element index of pair t = 0
      row[(base + 0) >> 1] = v.x;
      row[(base + 16) >> 1] = v.y;
      row[(base + 32) >> 1] = v.z;
      row[(base + 48) >> 1] = v.w;
    }
  }
  __syncthreads();
  const int A = s_A;
  if (tid == 0) sl_trace(tr, 4, 1);
  if (A == 0) {  // no routed slot on this rank: zero output
    for (int idx = c * kSlThreads + tid; idx < M * H / 8; idx += G * kSlThreads)
      reinterpret_cast<uint4*>(p.out)[idx] = make_uint4(0, 0, 0, 0);
    return;
  }

  SlCtx x;
  x.A = A;
  x.P = I / 16;
  x.G = G;
  x.c = c;
  x.chA = H / 64;
  x.chB = I / 64;
  x.NR = (A * x.P + G - 1) / G;
  x.T2 = p.T2;
  x.lag = p.lag;
  x.nrt2 = H / 16;
  x.S0 = sliced_w2_start(c, A, x.P, G, x.chA, x.chB, x.nrt2);
  x.S1 = sliced_w2_start(c + 1, A, x.P, G, x.chA, x.chB, x.nrt2);
  const int r_lo = x.S1 > x.S0 ? x.S0 / A : 0;
  const int r_hi = x.S1 > x.S0 ? (x.S1 - 1) / A : -1;

  if (warp == kSlEpilogue) {
    // The CTA's item table, built lane-parallel: round j's w13 pair, then the
    // w2 items of the experts inserted after round j (ascending expert), and
    // after the last round the remaining experts.
    int* const rcnt = rscratch;                    // [NR + 1] items per round
    int* const r13 = rscratch + p.max_rounds + 1;  // [NR + 1] w13 items per round
    int* const rstart = r13 + p.max_rounds + 1;    // [NR + 1] first item of each round
    const int NR = x.NR;
    for (int ae = lane; ae < A; ae += 32) {
      int ra, rb;
      sl_w2_tiles(ae, A, x.S0, x.S1, ra, rb);
      const int nt = rb >= ra ? rb - ra + 1 : 0;
      s_w2n[ae] = (nt + x.T2 - 1) / x.T2;
      s_w2ins[ae] = min(NR, sl_ready_round(ae, x.P, G) + x.lag);
    }
    __syncwarp();
    for (int j = lane; j <= NR; j += 32) {
      const int c13 = (j < NR && x.c + j * G < A * x.P) ? 1 : 0;
      int c2 = 0;
      for (int ae = 0; ae < A; ++ae) c2 += s_w2ins[ae] == j ? s_w2n[ae] : 0;
      rcnt[j] = c13 + c2;
      r13[j] = c13;
    }
    __syncwarp();
    if (lane == 0) {
      int run = 0;
      for (int j = 0; j <= NR; ++j) {
        rstart[j] = run;
        run += rcnt[j];
      }
      s_nst = run;
    }
    __syncwarp();
    for (int j = lane; j < NR; j += 32) {
      if (r13[j] == 0) continue;
      const int q = x.c + j * G, ae = q / x.P, pr = q - ae * x.P;
      table[rstart[j]].meta = make_int4(0, 0 | (2 << 4) | (ae << 16), pr, x.chA);
    }
    for (int ae = lane; ae < A; ae += 32) {
      const int j = s_w2ins[ae];
      int pos = rstart[j] + r13[j];
      for (int a2 = 0; a2 < ae; ++a2) pos += s_w2ins[a2] == j ? s_w2n[a2] : 0;
      int ra, rb;
      sl_w2_tiles(ae, A, x.S0, x.S1, ra, rb);
      for (int r = ra; r <= rb; r += x.T2) {
        const int nt = min(x.T2, rb - r + 1);
        table[pos++].meta = make_int4(0, 1 | (nt << 4) | (ae << 16), r, x.chB);
      }
    }
  }
  __syncthreads();
  if (tid == 0) sl_trace(tr, 4, 6);
  const int nitems = s_nst;

  if (warp < kSlConsumers) {
    // ======================= consumer warps =======================
    // Group = one k-chunk of one item (all of its row tiles); this warp's
    // groups are the chunks warp, warp + 16, ... of every item, streamed with
    // cp.async kSlDepth groups ahead into the warp's private ring.
    unsigned char* const wring = ring + (size_t)warp * kSlDepth * slot_bytes;
    const int nrt13 = 2 * x.P;
    int iss_it = 0, iss_ch = warp, iss_n = 0;  // issue cursor; groups issued
    auto issue_next = [&]() {
      while (iss_it < nitems) {
        const int4 m = table[iss_it].meta;
        if (iss_ch < m.w) break;
        ++iss_it;
        iss_ch = warp;
      }
      if (iss_it < nitems) {
        const int4 m = table[iss_it].meta;
        const int type = m.y & 15, nt = (m.y >> 4) & 15, e = s_act[m.y >> 16], ch = iss_ch;
        unsigned char* const dst = wring + (size_t)(iss_n % kSlDepth) * slot_bytes;
#pragma unroll
        for (int tt = 0; tt < kSlMaxTiles; ++tt) {
          if (tt < nt) {
            size_t blk;
            const uint8_t *wsrc, *ssrc;
            if (type == 0) {
              blk = ((size_t)e * nrt13 + (tt == 0 ? 0 : x.P) + m.z) * x.chA + ch;
              wsrc = p.w13;
              ssrc = p.s13;
            } else {
              blk = ((size_t)e * x.nrt2 + m.z + tt) * x.chB + ch;
              wsrc = p.w2;
              ssrc = p.s2;
            }
            cp_async16(dst + tt * 512 + lane * 16, wsrc + blk * 512 + lane * 16);
            if (lane < 8) cp_async8(dst + nt * 512 + tt * 64 + lane * 8, ssrc + blk * 64 + lane * 8);
          }
        }
        ++iss_n;
        iss_ch += kSlConsumers;
      }
      cp_async_commit();
    };
#pragma unroll 1
    for (int k = 0; k < kSlDepth; ++k) issue_next();

    float acc[kSlMaxTiles][4];
#pragma unroll
    for (int tt = 0; tt < kSlMaxTiles; ++tt) acc[tt][0] = acc[tt][1] = acc[tt][2] = acc[tt][3] = 0.f;
    int cons_n = 0;
    bool ok = true;
    for (int it = 0; it < nitems && ok; ++it) {
      const int4 m = table[it].meta;
      const int type = m.y & 15, nt = (m.y >> 4) & 15, ae = m.y >> 16, nch = m.w;
      const int cnt = s_cnt[ae], base = s_base[ae];
      const unsigned char* brow = nullptr;
      if (type == 0) {
        if (g < cnt) brow = xs + (size_t)s_tok[base + g] * xstride;
      } else if (warp < nch) {
        if (!sl_wait(&inter_bar[ae], 0, &s_abort)) {
          if (lane == 0 && !s_abort) sl_record(p.sched, kSlErrInter);
          s_abort = 1;
          ok = false;
          break;
        }
        if (g < cnt) brow = inter_s + (size_t)(base + g) * istride;
      }
      for (int ch = warp; ch < nch; ch += kSlConsumers) {
        cp_async_wait_group<kSlDepth - 1>();
        __syncwarp();
        const unsigned char* const sl = wring + (size_t)(cons_n % kSlDepth) * slot_bytes;
        uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
        if (brow != nullptr) {
          q0 = lds128(brow + (size_t)ch * 128 + t * 32);
          q1 = lds128(brow + (size_t)ch * 128 + t * 32 + 16);
        }
#pragma unroll
        for (int tt = 0; tt < kSlMaxTiles; ++tt) {
          if (tt < nt) {
            const uint4 wv = lds128(sl + tt * 512 + lane * 16);
            const uint2 sv = lds64(sl + nt * 512 + tt * 64 + g * 8);
            sl_block(acc[tt], wv, sv, q0, q1);
          }
        }
        __syncwarp();  // every lane is done with the slot before it is refilled
        ++cons_n;
        issue_next();
      }
      // end of item: partials to the epilogue
      const int b = it & 1;
      if (it >= 2 && !sl_wait(&red_empty[b], ((it >> 1) - 1) & 1, &s_abort)) {
        if (lane == 0 && !s_abort) sl_record(p.sched, kSlErrRed);
        s_abort = 1;
        ok = false;
        break;
      }
      float* rw = red + (size_t)b * kSlConsumers * red_warp + (size_t)warp * red_warp;
      if (2 * t < Mp) {
#pragma unroll
        for (int tt = 0; tt < kSlMaxTiles; ++tt)
          if (tt < nt) {
            *reinterpret_cast<float2*>(rw + (tt * 16 + g) * Mp + 2 * t) = make_float2(acc[tt][0], acc[tt][1]);
            *reinterpret_cast<float2*>(rw + (tt * 16 + g + 8) * Mp + 2 * t) = make_float2(acc[tt][2], acc[tt][3]);
          }
      }
#pragma unroll
      for (int tt = 0; tt < kSlMaxTiles; ++tt) acc[tt][0] = acc[tt][1] = acc[tt][2] = acc[tt][3] = 0.f;
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[b]);
      if (warp == 0 && lane == 0) sl_trace(tr, 1, it);
    }
    cp_async_wait_group<0>();  // nothing in flight into the ring when the warp exits
  } else if (warp == kSlEpilogue) {
    // ======================= epilogue warp =======================
    const int nloc = r_hi >= r_lo ? r_hi - r_lo + 1 : 0;
    for (int idx = lane; idx < nloc * M * 16; idx += 32) oacc[idx] = 0.f;
    __syncwarp();
    // non-final piece: the CTA's last row tile when its range stops before
    // that tile's last expert
    const bool has_np = x.S1 > x.S0 && ((x.S1 - 1) % A) != A - 1;
    const int np_e = has_np ? (x.S1 - 1) % A : -1;
    const int nitems = s_nst;
    bool ok = true;
    for (int gi = 0; gi < nitems; ++gi) {
      const int b = gi & 1;
      if (!sl_wait(&red_full[b], (gi >> 1) & 1, &s_abort)) {
        if (lane == 0 && !s_abort) sl_record(p.sched, kSlErrRed);
        s_abort = 1;
        ok = false;
        break;
      }
      const int4 d = table[gi].meta;
      const int type = d.y & 15;
      const int ntile = (d.y >> 4) & 15, ae = d.y >> 16, tile0 = d.z & 0xFFFF;
      const float* rb = red + (size_t)b * kSlConsumers * red_warp;
      const int cnt = s_cnt[ae], base = s_base[ae];
      if (type == 0) {
        const int tile = lane >> 4, row = lane & 15;
        for (int col = 0; col < cnt; ++col) {
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < kSlConsumers; ++w) v += rb[(size_t)w * red_warp + (tile * 16 + row) * Mp + col];
          const float up = __shfl_sync(0xffffffffu, v, (lane & 15) + 16);
          if (lane < 16) {
            const float h = silu_f(v) * up;
            p.inter[(size_t)(base + col) * I + sl_perm(tile0 * 16 + row)] = __float2bfloat16(h);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_empty[b]);
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_add(p.ready + s_act[ae], 1);
      } else {
        for (int idx = lane; idx < ntile * 16; idx += 32) {
          const int tt = idx >> 4, row = idx & 15;
          float* orow = oacc + (size_t)(tile0 + tt - r_lo) * M * 16 + row;
          for (int col = 0; col < cnt; ++col) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kSlConsumers; ++w) v += rb[(size_t)w * red_warp + (tt * 16 + row) * Mp + col];
            orow[s_tok[base + col] * 16] += s_wt[base + col] * v;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_empty[b]);
        if (has_np && ae == np_e && r_hi >= tile0 && r_hi < tile0 + ntile) {
          const float* src = oacc + (size_t)(r_hi - r_lo) * M * 16;
          for (int idx = lane; idx < M * 16; idx += 32) p.pieces[(size_t)c * M * 16 + idx] = src[idx];
          __threadfence();
          __syncwarp();
          if (lane == 0) st_release(p.pflag + c, 1);
        }
      }
      if (lane == 0) sl_trace(tr, 2, gi);
    }
    // own row tiles and the combined first row tile -> bf16 output
    if (ok) {
      for (int r = r_lo; r <= r_hi; ++r) {
        const bool own = r * A >= x.S0 && r * A + A - 1 <= x.S1 - 1;
        const bool comb = r == r_lo && !own && x.S0 % A != 0 && x.S1 - 1 >= r * A + A - 1;
        if (!own && !comb) continue;
        const float* src = oacc + (size_t)(r - r_lo) * M * 16;
        if (comb && !sl_wait(&pc_bar, 0, &s_abort)) {
          if (lane == 0 && !s_abort) sl_record(p.sched, kSlErrPiece);
          s_abort = 1;
          break;
        }
        const int npc = comb ? s_npc : 0;
        for (int idx = lane; idx < M * 16; idx += 32) {
          float v = 0.f;
          for (int k = 0; k < npc; ++k) v += pcs[(size_t)k * M * 16 + idx];
          v += src[idx];
          const int m = idx >> 4, row = idx & 15;
          p.out[(size_t)m * H + r * 16 + row] = __float2bfloat16(v);
        }
      }
    }
    if (lane == 0) sl_trace(tr, 4, 2);
    if (lane == 0) sl_trace(tr, 4, 2);
  } else if (warp == kSlLoader) {
    // ======================= loader warp =======================
    const bool has_comb = x.S1 > x.S0 && x.S0 % A != 0 && x.S1 - 1 >= r_lo * A + A - 1 &&
                          !(r_lo * A >= x.S0 && r_lo * A + A - 1 <= x.S1 - 1);
    bool ok = true;
    int issued = 0;  // experts whose intermediate copy was issued (bitmask over ae, up to 64)
    unsigned long long issued_mask = 0ull;
    for (int ae = 0; ae < A && ok; ++ae) {
      if (has_comb && ae == A - 1) {
        // fp32 pieces of the first row tile from the preceding CTAs, in CTA order
        if (lane == 0) {
          int n = 0;
          int lst[kSlicedMaxPieces];
          const int tile_start = r_lo * A;
          for (int cc = c - 1; cc >= 0 && n < kSlicedMaxPieces; --cc) {
            const int a0 = sliced_w2_start(cc, A, x.P, G, x.chA, x.chB, x.nrt2);
            const int a1 = sliced_w2_start(cc + 1, A, x.P, G, x.chA, x.chB, x.nrt2);
            if (a1 <= tile_start) break;
            if (a1 > a0) lst[n++] = cc;
          }
          for (int k = 0; k < n; ++k) s_pc[k] = lst[n - 1 - k];
          s_npc = n;
        }
        __syncwarp();
        const int n = s_npc;
        if (lane < n) {
          const int cc = s_pc[lane];
          const long long t0 = clock64();
          while (true) {
            int f;
            asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(f) : "l"(p.pflag + cc) : "memory");
            if (f) break;
            if (clock64() - t0 > kSlBudget || s_abort) {
              if (!s_abort) sl_record(p.sched, kSlErrPiece);
              s_abort = 1;
              break;
            }
            __nanosleep(64);
          }
          if (!s_abort) {
            for (int idx = 0; idx < M * 16; ++idx) pcs[(size_t)lane * M * 16 + idx] = p.pieces[(size_t)cc * M * 16 + idx];
            p.pflag[cc] = 0;  // self-cleaning
          }
        }
        __syncwarp();
        if (s_abort) {
          ok = false;
          break;
        }
        if (lane == 0) mbar_arrive(&pc_bar);
      }
      const int e = s_act[ae];
      if (lane == 0) {
        const long long t0 = clock64();
        int spins = 0;
        while (ld_acquire_gpu(p.ready + e) < x.P) {
          if (s_abort || clock64() - t0 > kSlBudget) {
            if (!s_abort) sl_record(p.sched, kSlErrReady);
            s_abort = 1;
            break;
          }
          if (++spins > 8) __nanosleep(32);
        }
        if (!s_abort) {
          fence_proxy_async_global();
          const int ra = x.S0 <= ae ? 0 : (x.S0 - ae + A - 1) / A;
          const int rb = x.S1 - 1 < ae ? -1 : (x.S1 - 1 - ae) / A;
          if (ra <= rb) {
            const int cnt = s_cnt[ae], base = s_base[ae];
            mbar_arrive_expect_tx(&inter_bar[ae], (uint32_t)(cnt * I * 2));
            for (int n = 0; n < cnt; ++n)
              bulk_g2s(inter_s + (size_t)(base + n) * istride, p.inter + (size_t)(base + n) * I, (uint32_t)(I * 2),
                       &inter_bar[ae]);
            issued_mask |= 1ull << ae;
            ++issued;
          }
        }
        sl_trace(tr, 3, ae);
      }
      __syncwarp();
      if (s_abort) ok = false;
    }
    // every CTA polled every expert's counter: the last one resets it
    if (ok) {
      for (int ae = lane; ae < A; ae += 32) {
        const int e = s_act[ae];
        if (atomicAdd(p.readers + e, 1) == G - 1) {
          p.readers[e] = 0;
          p.ready[e] = 0;
        }
      }
    }
    // intermediate copies still in flight must land before the CTA may exit
    if (lane == 0) {
      for (int ae = 0; ae < A; ++ae)
        if ((issued_mask >> ae) & 1ull) mbar_wait(&inter_bar[ae], 0, kSlBudget);
    }
    (void)issued;
  }
}

namespace {

struct SlPlanKey {
  int n_tok, E, H, I, G;
  bool operator==(const SlPlanKey& o) const {
    return n_tok == o.n_tok && E == o.E && H == o.H && I == o.I && G == o.G;
  }
};
struct SlPlanKeyHash {
  size_t operator()(const SlPlanKey& k) const {
    return ((size_t)k.n_tok * 1315423911u) ^ ((size_t)k.E * 2654435761u) ^ ((size_t)k.H << 20) ^
           ((size_t)k.I << 4) ^ (size_t)k.G;
  }
};
struct SlBounds {
  int nr, pc, items, rounds;
};

// Largest number of w2 row tiles any CTA touches, of pieces any combiner
// adds, of items in any CTA's schedule and of w13 rounds, over every
// possible active-expert count.
SlBounds sliced_bounds(int n_tok, int E, int H, int I, int G, int T2) {
  static std::mutex mu;
  static std::unordered_map<SlPlanKey, SlBounds, SlPlanKeyHash> cache;
  const SlPlanKey key{n_tok, E, H, I, G * 8 + T2};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  SlBounds b{1, 0, 0, 0};
  const int P = I / 16, chA = H / 64, chB = I / 64, nrt2 = H / 16;
  const int amax = n_tok < E ? n_tok : E;
  std::vector<int> S(G + 1);
  for (int A = 1; A <= amax; ++A) {
    for (int cc = 0; cc <= G; ++cc) S[cc] = sliced_w2_start(cc, A, P, G, chA, chB, nrt2);
    b.rounds = std::max(b.rounds, (A * P + G - 1) / G);
    for (int cc = 0; cc < G; ++cc) {
      int n = (A * P - cc + G - 1) / G;
      for (int ae = 0; ae < A; ++ae) {
        int ra, rb;
        sl_w2_tiles(ae, A, S[cc], S[cc + 1], ra, rb);
        if (rb >= ra) n += (rb - ra + 1 + T2 - 1) / T2;
      }
      b.items = std::max(b.items, n);
      if (S[cc + 1] <= S[cc]) continue;
      const int rl = S[cc] / A, rh = (S[cc + 1] - 1) / A;
      b.nr = std::max(b.nr, rh - rl + 1);
      // pieces preceding this CTA's first row tile
      int np = 0;
      for (int c2 = cc - 1; c2 >= 0 && S[c2 + 1] > rl * A; --c2)
        if (S[c2 + 1] > S[c2]) ++np;
      b.pc = std::max(b.pc, np);
    }
  }
  std::lock_guard<std::mutex> lk(mu);
  cache.emplace(key, b);
  return b;
}

}  // namespace

int sliced_plan(SlicedParams& p, int sms, int max_smem) {
  if (p.M < 1 || p.M > kSlicedMaxM || p.n_tok > kSlicedMaxSlots || p.n_tok < 1) return 0;
  if (p.H % 64 || p.I % 64) return 0;
  const int chA = p.H / 64, chB = p.I / 64;
  if (sms > kSlicedMaxGrid) sms = kSlicedMaxGrid;
  // the w2 range arithmetic runs in 32-bit integers
  const long long amax = std::min<long long>(p.n_tok, p.E);
  if (amax * (p.H / 16) * chB * (long long)sms * 2 + 2LL * chA * sms * sms >= (1LL << 31)) return 0;
  if (amax * (p.I / 16) >= (1LL << 15)) return 0;
  p.grid = sms;
  p.Mp = p.M <= 2 ? 2 : 4;
  p.lag = 1;
  auto up = [](int v) { return (v + 127) / 128 * 128; };
  const int static_smem = 6144;  // barriers + routing tables (static shared memory of the kernel)
  // the largest w2 item (row tiles per item) whose consumer rings still fit
  bool fits = false;
  for (p.T2 = kSlMaxTiles; p.T2 >= 1 && !fits; p.T2 >>= 1) {
#ifdef W4A16_DIAGNOSTICS
    if (const char* e = getenv("W4A16_SLICED_T2"))
      if (p.T2 > atoi(e)) continue;
#endif
    p.maxT = std::max(2, p.T2);
    p.slot_bytes = up(p.maxT * 576);
    const SlBounds b = sliced_bounds(p.n_tok, p.E, p.H, p.I, p.grid, p.T2);
    if (b.pc > kSlicedMaxPieces) return 0;
    p.nr_cap = b.nr;
    p.max_stages = b.items;
    p.max_rounds = b.rounds;
    int off = 0;
    p.off_x = off;
    off += up(p.M * (p.H * 2 + 16));
    p.off_inter = off;
    off += up(p.n_tok * (p.I * 2 + 16));
    p.off_red = off;
    off += up(2 * kSlConsumers * p.maxT * 16 * p.Mp * 4);
    p.off_oacc = off;
    off += up(p.nr_cap * p.M * 16 * 4);
    p.off_pc = off;
    off += up(std::max(1, b.pc) * p.M * 16 * 4);
    p.off_table = off;
    off += up(std::max(1, p.max_stages) * (int)sizeof(SlEntry));
    p.off_rounds = off;
    off += up(3 * (p.max_rounds + 1) * 4);
    p.off_ring = off;
    p.n_slots = kSlDepth;
    p.ring_bytes = kSlConsumers * kSlDepth * p.slot_bytes;
    p.smem_bytes = off + p.ring_bytes;
    if (p.smem_bytes + static_smem <= max_smem) {
      fits = true;
      break;
    }
  }
  if (!fits) return 0;
#ifdef W4A16_DIAGNOSTICS
  if (const char* e = getenv("W4A16_SLICED_LAG")) p.lag = atoi(e);
#endif
  return 1;
}

cudaError_t launch_sliced(const SlicedParams& p, cudaStream_t stream) {
  static thread_local int configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (configured[dev] < p.smem_bytes) {
    cudaError_t err =
        cudaFuncSetAttribute(moe_decode_sliced_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem_bytes);
    if (err != cudaSuccess) return err;
    configured[dev] = p.smem_bytes;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kSlThreads);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, moe_decode_sliced_kernel, p);
}

}  // namespace w4moe
