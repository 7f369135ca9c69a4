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
//   * one producer warp streams every stage (w13 pair parts, w2 tile groups)
//     with cp.async.bulk into a byte-granular shared-memory ring, in schedule
//     order; w2 weights therefore stream while w13 is still computing.
//   * 16 consumer warps decode int4 from the ring straight into m16n8k16 A
//     fragments (code - 8 exact in bf16; the bf16 group scale is applied to the
//     fp32 partial of each 32-wide group); token rows (hidden, intermediate)
//     live in shared memory in a lane-permuted layout (two 16-byte loads give a
//     lane its B fragments for a 64-wide chunk).
//   * one epilogue warp reduces the 16 consumer warps' partials in fixed warp
//     order, applies SiLU*up (w13) or the router weight (w2), publishes.
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
constexpr int kSlProducer = 16;  // warp index
constexpr int kSlEpilogue = 17;
constexpr int kSlLoader = 18;
constexpr int kSlThreads = 19 * 32;
constexpr int kSlNSB = 32;              // stage barrier slots (== warp width: lane k tracks slot k)
constexpr int kSlMaxTiles = 4;          // row tiles per stage
constexpr int kSlChunks = 16;           // k-chunks per w13 stage
constexpr long long kSlBudget = 4000000000LL;  // ~2 s of SM clocks
constexpr int kSlMaxA = kSlicedMaxSlots;        // active experts <= slots

// error bits in the workspace status word (sched[2])
constexpr int kSlErrFull = 1 << 8, kSlErrEmpty = 1 << 9, kSlErrRed = 1 << 10, kSlErrReady = 1 << 11,
              kSlErrInter = 1 << 12, kSlErrPiece = 1 << 13;

struct SlCtx {
  int A, P, G, c, chA, chB, nparts, NR, T2, lag, nrt2;
  int S0, S1;
};

// One pipeline stage of the CTA's schedule: its descriptor (consumers read it
// from s_desc) and up to four global source ranges (producer only).
struct SlEntry {
  int4 meta;              // x: type | ntile << 4 | gend << 8 | ae << 16; y: tile0 | c0 << 16; z: nch; w: bytes
  const uint8_t* src[4];  // w13: gate w, up w, gate s, up s; w2: weights, scales
};

// Round in which the last pair of active expert e is computed.
__host__ __device__ __forceinline__ int sl_ready_round(int e, int P, int G) { return ((e + 1) * P - 1) / G; }

// w2 row tiles [ra, rb] of active expert ae inside the CTA's unit range [S0, S1)
__host__ __device__ __forceinline__ void sl_w2_tiles(int ae, int A, long long S0, long long S1, int& ra, int& rb) {
  ra = S0 <= ae ? 0 : (int)((S0 - ae + A - 1) / A);
  rb = S1 - 1 < ae ? -1 : (int)((S1 - 1 - ae) / A);
}

__device__ __forceinline__ void sl_record(int32_t* sched, int code) { atomicOr(sched + 2, code); }

// Bounded mbarrier wait that also gives up once the CTA is aborting.  Between
// checks the warp is parked by try_wait's suspend hint (or by nanosleep when
// sleep_ns > 0).
__device__ __forceinline__ bool sl_wait(uint64_t* bar, uint32_t parity, const volatile int* abort_flag,
                                        int sleep_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (sleep_ns > 0) {
      __nanosleep(sleep_ns);
      if (mbar_try_wait(bar, parity)) return true;
    } else if (mbar_try_wait_sleep(bar, parity, 2000u)) {
      return true;
    }
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
// w13 pair as 2*chA chunk blocks and a w2 tile as chB.
__host__ __device__ long long sliced_w2_start(int c, int A, int P, int G, int chA, int chB, int nrt2) {
  const long long T2 = (long long)A * nrt2;
  const long long pairs = (long long)A * P;
  const long long rem = pairs % G;
  if (rem == 0) return T2 * c / G;
  const long long W2 = T2 * chB, X = 2LL * chA * (G - rem);
  if (W2 <= X) return c <= rem ? 0 : T2 * (c - rem) / (G - rem);  // CTAs with the extra pair take no w2
  const long long lo = c < rem ? c : rem, hi = c > rem ? c - rem : 0;
  return (lo * (W2 - X) + hi * (W2 - X + 2LL * chA * G)) / ((long long)G * chB);
}

__global__ void __launch_bounds__(kSlThreads, 1) moe_decode_sliced_kernel(SlicedParams p) {
  __shared__ uint64_t full_bar[kSlNSB], empty_bar[kSlNSB];
  __shared__ uint64_t red_full[2], red_empty[2], inter_bar[kSlMaxA], pc_bar;
  __shared__ int s_tok[kSlicedMaxSlots], s_eid[kSlicedMaxSlots], s_first[kSlicedMaxSlots];
  __shared__ float s_wt[kSlicedMaxSlots], s_wt_in[kSlicedMaxSlots];
  __shared__ int s_act[kSlMaxA], s_cnt[kSlMaxA], s_base[kSlMaxA];
  __shared__ int s_w2n[kSlMaxA], s_w2ins[kSlMaxA];
  __shared__ int s_A, s_nst;
  __shared__ int s_pc[kSlicedMaxPieces];
  __shared__ int s_npc;
  __shared__ volatile int s_abort;
  __shared__ int4 s_desc[kSlNSB], s_gdesc[2];
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
  SlEntry* const table = reinterpret_cast<SlEntry*>(dsm + p.off_table);  // [max_stages + 1]
  int* const rscratch = reinterpret_cast<int*>(dsm + p.off_rounds);      // [3][max_rounds + 1]
  unsigned char* const ring = dsm + p.off_ring;                          // [n_slots][slot_bytes]
  const int xstride = H * 2 + 16, istride = I * 2 + 16;
  const int Mp = p.Mp, maxT = p.maxT;
  const int red_warp = maxT * 16 * Mp;  // floats per warp in one buffer
  const int nslots = p.n_slots, slot_bytes = p.slot_bytes;

  // ---------------- prologue ----------------
  if (tid == 0) sl_trace(tr, 4, 0);
  if (warp == 0) {
    // Routing for <= 64 slots.  A "column" is one (expert, token) pair: the
    // slots of a token that name the same expert twice share one column whose
    // router weight is their sum (in slot order), so an expert has at most M
    // columns.  Columns are ordered by expert, then token; active experts
    // ascending.
    const int n = p.n_tok;
    int e_l[2], m_l[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h;
      e_l[h] = i < n ? p.map(i) : -1;
      m_l[h] = i / p.topk;
      if (i < n) {
        s_eid[i] = e_l[h];
        s_wt_in[i] = p.topk_w[i];
      }
    }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h;
      if (i < n) {
        // bit 0: first slot of its (expert, token) column; bit 1: of its expert
        int same_e = 0, same_col = 0;
#pragma unroll 8
        for (int jj = 0; jj < i; ++jj) {
          const int ej = s_eid[jj];
          same_e |= ej == e_l[h];
          same_col |= (ej == e_l[h]) & (jj / p.topk == m_l[h]);
        }
        s_first[i] = e_l[h] >= 0 ? ((same_col ? 0 : 1) | (same_e ? 0 : 2)) : 0;
      }
    }
    __syncwarp();
    int nact = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h;
      const int e = e_l[h];
      const bool mine = i < n && e >= 0 && (s_first[i] & 1);
      int below = 0, same_before = 0, same = 0, act_below = 0;
      float wsum = 0.f;
#pragma unroll 8
      for (int jj = 0; jj < n; ++jj) {
        const int ej = s_eid[jj];
        const int fj = s_first[jj];
        const bool valid = ej >= 0;
        const bool col1 = valid && (fj & 1);
        below += col1 && ej < e;
        same += col1 && ej == e;
        same_before += col1 && ej == e && jj < i;
        act_below += valid && ej < e && (fj & 2);
        if (valid && ej == e && jj / p.topk == m_l[h]) wsum += s_wt_in[jj];
      }
      if (mine) {
        const int col = below + same_before;
        s_tok[col] = m_l[h];
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
    for (int s = lane; s < kSlNSB; s += 32) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kSlConsumers);
    }
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
    // hidden rows -> shared memory, lane-permuted (warps 1..17)
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
  x.nparts = (x.chA + kSlChunks - 1) / kSlChunks;
  x.NR = (A * x.P + G - 1) / G;
  x.T2 = p.T2;
  x.lag = p.lag;
  x.nrt2 = H / 16;
  x.S0 = (int)sliced_w2_start(c, A, x.P, G, x.chA, x.chB, x.nrt2);
  x.S1 = (int)sliced_w2_start(c + 1, A, x.P, G, x.chA, x.chB, x.nrt2);
  const int r_lo = x.S1 > x.S0 ? x.S0 / A : 0;
  const int r_hi = x.S1 > x.S0 ? (x.S1 - 1) / A : -1;

  if (warp < kSlConsumers) {
    // ======================= consumer warps =======================
    float acc[kSlMaxTiles][4];
#pragma unroll
    for (int tt = 0; tt < kSlMaxTiles; ++tt) acc[tt][0] = acc[tt][1] = acc[tt][2] = acc[tt][3] = 0.f;
    int si = 0, gi = 0;
    for (;;) {
      const int slot = si % nslots;
      if (!sl_wait(&full_bar[slot], (si / nslots) & 1, &s_abort, p.wait_ns)) {
        if (lane == 0 && !s_abort) sl_record(p.sched, kSlErrFull);
        s_abort = 1;
        break;
      }
      if (warp == 0 && lane == 0) sl_trace(tr, 5, si);
      const int4 d = s_desc[slot];
      const int type = d.y & 15;
      const int ntile = (d.y >> 4) & 15, gend = (d.y >> 8) & 1, ae = d.y >> 16;
      const int tile0 = d.z & 0xFFFF, c0 = d.z >> 16, nch = d.w;
      if (type != 2) {
        const int cnt = s_cnt[ae], base = s_base[ae];
        const unsigned char* brow = nullptr;
        if (type == 0) {
          if (g < cnt) brow = xs + (size_t)s_tok[base + g] * xstride;
        } else {
          if (!(p.diag & 4) && !sl_wait(&inter_bar[ae], 0, &s_abort)) {
            if (lane == 0 && !s_abort) sl_record(p.sched, kSlErrInter);
            s_abort = 1;
            break;
          }
          if (g < cnt) brow = inter_s + (size_t)(base + g) * istride;
        }
        const unsigned char* wb = ring + (size_t)slot * slot_bytes;
        const int nblk = ntile * nch;
        const unsigned char* sb = wb + (size_t)nblk * 512;
        uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
        if (p.diag & 1) {
          // diagnostics: pipeline only, no math
        } else if ((nch & 15) == 0) {
          for (int ch = warp; ch < nch; ch += kSlConsumers) {
            if (brow != nullptr) {
              q0 = lds128(brow + (size_t)(c0 + ch) * 128 + t * 32);
              q1 = lds128(brow + (size_t)(c0 + ch) * 128 + t * 32 + 16);
            }
#pragma unroll
            for (int tt = 0; tt < kSlMaxTiles; ++tt) {
              if (tt < ntile) {
                const int i = tt * nch + ch;
                const uint4 wv = lds128(wb + (size_t)i * 512 + lane * 16);
                const uint2 sv = lds64(sb + (size_t)i * 64 + g * 8);
                sl_block(acc[tt], wv, sv, q0, q1);
              }
            }
          }
        } else {
          int bch = -1;
          for (int i = warp; i < nblk; i += kSlConsumers) {
            const int tile = i / nch, ch = i - tile * nch;
            if (ch != bch) {
              if (brow != nullptr) {
                q0 = lds128(brow + (size_t)(c0 + ch) * 128 + t * 32);
                q1 = lds128(brow + (size_t)(c0 + ch) * 128 + t * 32 + 16);
              }
              bch = ch;
            }
            const uint4 wv = lds128(wb + (size_t)i * 512 + lane * 16);
            const uint2 sv = lds64(sb + (size_t)i * 64 + g * 8);
            float pd[4] = {0.f, 0.f, 0.f, 0.f};
            sl_block(pd, wv, sv, q0, q1);
#pragma unroll
            for (int tt = 0; tt < kSlMaxTiles; ++tt)
              if (tt == tile) {
                acc[tt][0] += pd[0];
                acc[tt][1] += pd[1];
                acc[tt][2] += pd[2];
                acc[tt][3] += pd[3];
              }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[slot]);
        if (warp == 0 && lane == 0) sl_trace(tr, 1, si);
        (void)tile0;
      }
      if (type == 2 || gend) {
        const int b = gi & 1;
        if (gi >= 2 && !sl_wait(&red_empty[b], ((gi >> 1) - 1) & 1, &s_abort)) {
          if (lane == 0 && !s_abort) sl_record(p.sched, kSlErrRed);
          s_abort = 1;
          break;
        }
        if (type != 2) {
          float* rw = red + (size_t)b * kSlConsumers * red_warp + (size_t)warp * red_warp;
          if (2 * t < Mp) {
#pragma unroll
            for (int tt = 0; tt < kSlMaxTiles; ++tt)
              if (tt < ntile) {
                *reinterpret_cast<float2*>(rw + (tt * 16 + g) * Mp + 2 * t) = make_float2(acc[tt][0], acc[tt][1]);
                *reinterpret_cast<float2*>(rw + (tt * 16 + g + 8) * Mp + 2 * t) =
                    make_float2(acc[tt][2], acc[tt][3]);
              }
          }
#pragma unroll
          for (int tt = 0; tt < kSlMaxTiles; ++tt) acc[tt][0] = acc[tt][1] = acc[tt][2] = acc[tt][3] = 0.f;
        }
        if (warp == 0 && lane == 0) s_gdesc[b] = d;
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_full[b]);
        ++gi;
        if (type == 2) break;
      }
      ++si;
    }
  } else if (warp == kSlProducer) {
    // ======================= producer warp =======================
    // Builds the CTA's stage table once (lane-parallel), then streams it:
    // stage s uses ring slot and barrier s % n_slots.  Order: round j's w13
    // pair stages, then the w2 stages of the experts inserted after round j
    // (ascending expert), and after the last round the remaining experts.
    int* const rcnt = rscratch;                    // [NR + 1] stages per round
    int* const r13 = rscratch + p.max_rounds + 1;  // [NR + 1] w13 stages per round
    int* const rstart = r13 + p.max_rounds + 1;    // [NR + 1] first stage of each round
    const int nrt13 = 2 * x.P, NR = x.NR;
    for (int ae = lane; ae < A; ae += 32) {
      int ra, rb;
      sl_w2_tiles(ae, A, x.S0, x.S1, ra, rb);
      const int nt = rb >= ra ? rb - ra + 1 : 0;
      s_w2n[ae] = (nt + x.T2 - 1) / x.T2;
      s_w2ins[ae] = min(NR, sl_ready_round(ae, x.P, G) + x.lag);
    }
    __syncwarp();
    for (int j = lane; j <= NR; j += 32) {
      const int c13 = (j < NR && x.c + j * G < A * x.P) ? x.nparts : 0;
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
    const int nst = s_nst;
    for (int j = lane; j < NR; j += 32) {
      if (r13[j] == 0) continue;
      const int q = x.c + j * G, ae = q / x.P, pr = q - ae * x.P, e = s_act[ae];
      for (int k = 0; k < x.nparts; ++k) {
        const int c0 = k * kSlChunks, nch = min(kSlChunks, x.chA - c0);
        const size_t bg = ((size_t)e * nrt13 + pr) * x.chA + c0;
        const size_t bu = ((size_t)e * nrt13 + x.P + pr) * x.chA + c0;
        SlEntry en;
        en.meta = make_int4(2 * nch * 576, 0 | (2 << 4) | ((k == x.nparts - 1) << 8) | (ae << 16), pr | (c0 << 16), nch);
        en.src[0] = p.w13 + bg * 512;
        en.src[1] = p.w13 + bu * 512;
        en.src[2] = p.s13 + bg * 64;
        en.src[3] = p.s13 + bu * 64;
        table[rstart[j] + k] = en;
      }
    }
    for (int ae = lane; ae < A; ae += 32) {
      const int j = s_w2ins[ae];
      int pos = rstart[j] + r13[j];
      for (int a2 = 0; a2 < ae; ++a2) pos += s_w2ins[a2] == j ? s_w2n[a2] : 0;
      int ra, rb;
      sl_w2_tiles(ae, A, x.S0, x.S1, ra, rb);
      const int e = s_act[ae];
      for (int r = ra; r <= rb; r += x.T2) {
        const int nt = min(x.T2, rb - r + 1);
        const size_t b0 = ((size_t)e * x.nrt2 + r) * x.chB;
        SlEntry en;
        en.meta = make_int4(nt * x.chB * 576, 1 | (nt << 4) | (1 << 8) | (ae << 16), r, x.chB);
        en.src[0] = p.w2 + b0 * 512;
        en.src[1] = p.s2 + b0 * 64;
        en.src[2] = nullptr;
        en.src[3] = nullptr;
        table[pos++] = en;
      }
    }
    __syncwarp();
    if (lane == 0) sl_trace(tr, 4, 6);
    const uint64_t pol = l2_evict_first_policy();
    bool ok = true;
    int s = 0;
    for (; s <= nst; ++s) {
      const int slot = s % nslots;
      if (s >= nslots && !sl_wait(&empty_bar[slot], ((s / nslots) - 1) & 1, &s_abort)) {
        if (lane == 0 && !s_abort) sl_record(p.sched, kSlErrEmpty);
        s_abort = 1;
        ok = false;
        break;
      }
      if (s == nst) {  // end mark
        if (lane == 0) {
          s_desc[slot] = make_int4(0, 2, 0, 0);
          mbar_arrive(&full_bar[slot]);
        }
        break;
      }
      const int4 meta = table[s].meta;
      if (lane == 0) {
        s_desc[slot] = meta;
        mbar_arrive_expect_tx(&full_bar[slot], (uint32_t)meta.x);
      }
      __syncwarp();
      const int type = meta.y & 15, nt = (meta.y >> 4) & 15, nch = meta.w;
      unsigned char* const dst = ring + (size_t)slot * slot_bytes;
      if (lane < (type == 0 ? 4 : 2)) {
        uint32_t off, sz;
        if (type == 0) {
          const uint32_t wb = (uint32_t)nch * 512, sb = (uint32_t)nch * 64;
          off = lane < 2 ? lane * wb : 2 * wb + (lane - 2) * sb;
          sz = lane < 2 ? wb : sb;
        } else {
          const uint32_t wb = (uint32_t)(nt * nch) * 512;
          off = lane == 0 ? 0u : wb;
          sz = lane == 0 ? wb : (uint32_t)(nt * nch) * 64;
        }
        bulk_g2s_hint(dst + off, table[s].src[lane], sz, &full_bar[slot], pol);
      }
      if (lane == 0) sl_trace(tr, 0, s);
    }
    // copies still in flight must land before the CTA may exit (the slot
    // that took the end mark held a stage that was already consumed)
    const int issued = s < nst ? s : nst;
    const int first = ok ? max(0, issued - nslots + 1) : max(0, issued - nslots);
    for (int k = first; k < issued; ++k) mbar_wait(&full_bar[k % nslots], (k / nslots) & 1, kSlBudget);
  } else if (warp == kSlEpilogue) {
    // ======================= epilogue warp =======================
    const int nloc = r_hi >= r_lo ? r_hi - r_lo + 1 : 0;
    for (int idx = lane; idx < nloc * M * 16; idx += 32) oacc[idx] = 0.f;
    __syncwarp();
    // non-final piece: the CTA's last row tile when its range stops before
    // that tile's last expert
    const bool has_np = x.S1 > x.S0 && ((x.S1 - 1) % A) != A - 1;
    const int np_e = has_np ? (x.S1 - 1) % A : -1;
    int gi = 0;
    bool ok = true;
    for (;;) {
      const int b = gi & 1;
      if (!sl_wait(&red_full[b], (gi >> 1) & 1, &s_abort)) {
        if (lane == 0 && !s_abort) sl_record(p.sched, kSlErrRed);
        s_abort = 1;
        ok = false;
        break;
      }
      const int4 d = s_gdesc[b];
      const int type = d.y & 15;
      if (type == 2) break;
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
      ++gi;
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
          const long long tile_start = (long long)r_lo * A;
          for (int cc = c - 1; cc >= 0 && n < kSlicedMaxPieces; --cc) {
            const long long a0 = sliced_w2_start(cc, A, x.P, G, x.chA, x.chB, x.nrt2);
            const long long a1 = sliced_w2_start(cc + 1, A, x.P, G, x.chA, x.chB, x.nrt2);
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
  int nr, pc, stages, rounds;
};

// Largest number of w2 row tiles any CTA touches, of pieces any combiner
// adds, of stages in any CTA's schedule and of w13 rounds, over every
// possible active-expert count.
SlBounds sliced_bounds(int n_tok, int E, int H, int I, int G, int T2) {
  static std::mutex mu;
  static std::unordered_map<SlPlanKey, SlBounds, SlPlanKeyHash> cache;
  const SlPlanKey key{n_tok, E, H, I, G};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  SlBounds b{1, 0, 0, 0};
  const int P = I / 16, chA = H / 64, chB = I / 64, nrt2 = H / 16;
  const int nparts = (chA + kSlChunks - 1) / kSlChunks;
  const int amax = n_tok < E ? n_tok : E;
  std::vector<long long> S(G + 1);
  for (int A = 1; A <= amax; ++A) {
    for (int cc = 0; cc <= G; ++cc) S[cc] = sliced_w2_start(cc, A, P, G, chA, chB, nrt2);
    b.rounds = std::max(b.rounds, (A * P + G - 1) / G);
    for (int cc = 0; cc < G; ++cc) {
      int nst = nparts * ((A * P - cc + G - 1) / G);
      for (int ae = 0; ae < A; ++ae) {
        int ra, rb;
        sl_w2_tiles(ae, A, S[cc], S[cc + 1], ra, rb);
        if (rb >= ra) nst += (rb - ra + 1 + T2 - 1) / T2;
      }
      b.stages = std::max(b.stages, nst);
      if (S[cc + 1] <= S[cc]) continue;
      const long long rl = S[cc] / A, rh = (S[cc + 1] - 1) / A;
      b.nr = std::max<int>(b.nr, (int)(rh - rl + 1));
      // pieces preceding this CTA's first row tile
      int n = 0;
      for (int c2 = cc - 1; c2 >= 0 && S[c2 + 1] > rl * A; --c2)
        if (S[c2 + 1] > S[c2]) ++n;
      b.pc = std::max(b.pc, n);
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
  if (chB > 64 || p.H / 16 > 65535) return 0;
  if (sms > kSlicedMaxGrid) sms = kSlicedMaxGrid;
  p.grid = sms;
  p.Mp = p.M <= 2 ? 2 : 4;
  // ring slots fit one w13 stage (gate + up, <= 16 chunks) or T2 w2 row tiles
  const int w13_stage = 2 * std::min(kSlChunks, chA) * 576;
  p.T2 = std::max(1, std::min(kSlMaxTiles, w13_stage / (chB * 576)));
  p.lag = 1;
#ifdef W4A16_DIAGNOSTICS
  if (const char* e = getenv("W4A16_SLICED_LAG")) p.lag = atoi(e);
  if (const char* e = getenv("W4A16_SLICED_T2")) p.T2 = std::max(1, std::min(p.T2, atoi(e)));
#endif
  p.maxT = std::max(2, p.T2);
  p.slot_bytes = (std::max(w13_stage, p.T2 * chB * 576) + 127) / 128 * 128;
  const SlBounds b = sliced_bounds(p.n_tok, p.E, p.H, p.I, p.grid, p.T2);
  if (b.pc > kSlicedMaxPieces) return 0;
  p.nr_cap = b.nr;
  p.max_stages = b.stages;
  p.max_rounds = b.rounds;
  auto up = [](int v) { return (v + 127) / 128 * 128; };
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
  off += up((p.max_stages + 1) * (int)sizeof(SlEntry));
  p.off_rounds = off;
  off += up(3 * (p.max_rounds + 1) * 4);
  p.off_ring = off;
  const int static_smem = 6144;  // barriers + routing tables (static shared memory of the kernel)
  p.n_slots = std::min(kSlNSB, (max_smem - off - static_smem) / p.slot_bytes);
  if (p.n_slots < 3) return 0;
  p.ring_bytes = p.n_slots * p.slot_bytes;
  p.smem_bytes = off + p.ring_bytes;
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
