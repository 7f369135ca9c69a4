// Fused small-M ("decode") MoE layer: routing + w13 (+SiLU*up) + w2 (+ router-
// weighted top-k sum) in ONE persistent, warp-specialised kernel.
//
// Replaces, for M*topk <= kDecodeMaxSlots, the reference's moe_align_block_size
// + _w4a16_moe_w1_fused_kernel + _w4a16_moe_w2_kernel + _moe_sum_kernel
// (kernels/w4a16_moe.py:187-290, :374-670).
//
// Structure (one CTA per SM; cooperative launch, so every CTA is resident):
//   * prologue: every CTA builds the routing tables in shared memory from the
//     raw top-k ids (histogram, scan, per-expert slot lists) and sizes its
//     pipeline stages from the largest per-expert slot count.
//   * work items, assigned round-robin (CTA b takes items b, b+grid, ...):
//       phase A  (active expert j, RP gate/up row-tile pairs)  -> w13
//       phase B  (active expert j, R2 hidden row tiles)        -> w2
//     all phase-A items precede all phase-B items.  An item's K range is cut
//     into parts that fit one pipeline stage; an expert with more slots than
//     one pass holds (8*NG) is done in passes.
//   * 2 producer warps, each owning one ring slot (both walk the same stage
//     sequence; one stage's issue overlaps the other's): per stage,
//     cp.async.bulk of the item's weight and scale
//     blocks (contiguous per row tile in the fragment-major layout) and of the
//     pass's activation rows (hidden rows in phase A, intermediate rows in
//     phase B) into a shared-memory ring; completion via mbarrier tx-count.
//     Phase-B activation copies wait (bounded) until every phase-A item pass
//     of the same expert has published its intermediate rows; the weight
//     copies of that stage are issued before the wait.  The producers share
//     their SM sub-partitions with busy consumer warps, so stages are large
//     (few per-stage instruction chains).
//   * 16 consumer warps: a warp covers Rw row tiles of the item for its share
//     of the stage's k-chunks, so each activation fragment (ldmatrix) feeds Rw
//     tiles.  Weights are decoded from smem straight into m16n8k16 A
//     fragments; fp32 accumulation in registers.
//       NG == 1: A = bf16(code - 8) (exact); the bf16 group scale multiplies
//                the fp32 partial of each 32-wide group.
//       NG > 1:  A = bf16((code - 8) * scale), the reference's dequantised
//                value, shared by all token groups.
//     At the end of an item pass each warp deposits its accumulators into one
//     of n_red reduction buffers and moves on.
//   * epilogue warps (one per reduction buffer) reduce in fixed warp order
//     (deterministic);
//       A: write bf16(silu(gate) * up) rows, then bump ready[e];
//       B: scale by the router weight and write fp32 partials; then either the
//          last of a token's slots to finish a row block sums that token's
//          partials in slot order (small M), or a grid-wide tail pass does.
//   * all global counters are self-cleaning (the last CTA resets them).
//
// Every wait is bounded (clock64 budget); a timeout records an error bit in
// the workspace (w4a16_moe_read_status) and the waiting warp stops.
#include <stdlib.h>

#include "launch.cuh"

namespace w4moe {

constexpr int kDecConsumers = 16;
constexpr int kDecProducerWarp = kDecConsumers;  // first of kDecProducers producer warps
constexpr int kDecProducers = 2;                  // producer p refills the ring slots s with s % 2 == p
constexpr int kDecEpiWarps = 4;  // epilogue warp k owns reduction buffer k (k < n_red)
constexpr int kDecThreads = (kDecConsumers + kDecProducers + kDecEpiWarps) * 32;
constexpr int kDecMaxStages = 8;
constexpr long long kWaitBudget = 4000000000LL;  // ~2 s of SM clocks

// sched[] words in the workspace
constexpr int kSchedDone = 1, kSchedError = 2, kSchedBDone = 3;

enum DecodeError : int {
  kErrFullWait = 1,
  kErrEmptyWait = 2,
  kErrReadyWait = 4,
  kErrRedWait = 8,
};

// Per-stage descriptor written by the producer: everything the consumer warps
// need, so that they do no integer division per stage.
struct __align__(16) StageInfo {
  int item;  // -1 = end of work
  int pass;
  int part;
  int last;  // last part of the item pass
  int nc;    // k-chunks in the stage
  int R;     // row tiles of the item
  int lgw;   // log2(consumer warps per tile group)
  int rows;  // activation rows (slots) of the pass
};

struct Geometry {
  int ncA, ncB;   // chunks per stage in phase A / B
  int rows_res;   // activation rows reserved per stage
  int n_stages, stage_bytes;
};

// Row tiles per consumer warp: keeps Rw * NG * 4 accumulators <= 16.
__host__ __device__ constexpr int rows_per_warp(int NG) { return NG == 4 ? 1 : 2; }

// Pipeline timestamps (diagnostics builds only: without W4A16_DIAGNOSTICS the
// helpers compile to nothing, since even untaken trace branches in the hot
// loops measurably slowed the kernel).  Layout: [kind][512] for CTA 0 (0
// producer stage issued, 1 consumer warp 0 stage landed, 2 consumer warp 0
// stage done, 3/4 epilogue 0 start/end, 5 kernel start / prologue end /
// teardown), then per-CTA milestones [cta][32] (0 start, 1 prologue end, 4
// producer done, 6 consumer warp 0 done, 9 end).
#ifdef W4A16_DIAGNOSTICS
__device__ __forceinline__ void trace_ev(long long* tr, int kind, int k) {
  if (tr != nullptr && blockIdx.x == 0 && k < 512) tr[kind * 512 + k] = global_timer_ns();
}
__device__ __forceinline__ void trace_cta(long long* tr, int k) {
  if (tr != nullptr) tr[6 * 512 + blockIdx.x * 32 + k] = global_timer_ns();
}
#else
__device__ __forceinline__ void trace_ev(long long*, int, int) {}
__device__ __forceinline__ void trace_cta(long long*, int) {}
#endif

__device__ __forceinline__ void record_error(int* sched, int code) { atomicOr(sched + kSchedError, code); }

__device__ __forceinline__ float bf16_lo_f32(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi_f32(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

struct ItemView {
  bool phB;
  int q;     // row-block index within the expert
  int e;     // local expert
  int T;     // slots routed to e
  int base;  // start of e's slots in the per-CTA slot list
};

// Shared-memory offset of this lane's ldmatrix row address within a stage's
// activation rows (row stride bstride = 16 mod 128, so the eight rows of one
// 8x8 matrix fall in distinct 16-byte bank groups).  Lanes whose row is not
// reserved (row >= nrows) read row 0 at a rotated 16-byte column: those
// columns of the product are never used, and distinct addresses keep the
// load conflict-free.
__device__ __forceinline__ int brow_off(int lane, int nrows, int bstride) {
  const int r = lane & 7, j = lane >> 3;
  return r < nrows ? r * bstride + j * 16 : ((j + r) & 7) * 16;
}

__host__ __device__ __forceinline__ int stage_bytes_for(int R, int nc, int rows) {
  return R * nc * 576 + rows * (nc * 128 + 16);
}

// Largest divisor nc of nchunks with stage bytes <= cap (0 if none).
__host__ __device__ __forceinline__ int pick_nc(int nchunks, int R, int rows, int cap) {
  int best = 0;
  for (int nc = 1; nc <= nchunks; ++nc)
    if (nchunks % nc == 0 && stage_bytes_for(R, nc, rows) <= cap) best = nc;
  return best;
}

template <int NG>
__global__ void __launch_bounds__(kDecThreads, 1) moe_decode_fused_kernel(DecodeParams p) {
  constexpr int NB = 8 * NG;
  constexpr int RW = rows_per_warp(NG);
  constexpr int kRedFloats = kDecConsumers * RW * NG * 128;  // one reduction buffer
  __shared__ uint64_t full_bar[kDecMaxStages], empty_bar[kDecMaxStages];
  __shared__ uint64_t red_full[kDecEpiWarps], red_empty[kDecEpiWarps];
  __shared__ StageInfo sinfo[kDecMaxStages];
  __shared__ StageInfo rinfo[kDecEpiWarps];
  __shared__ int s_nact;
  __shared__ int s_wtot[32], s_wact[32], s_wmax[32];
  __shared__ int s_last;
  __shared__ Geometry s_geo;
  extern __shared__ __align__(128) unsigned char dsm[];

  const int E = p.E;
  int* cnt = reinterpret_cast<int*>(dsm);  // [E]
  int* off = cnt + E;                      // [E+1]
  int* act = off + E + 1;                  // [E]
  int* cur = act + E;                      // [E]
  int* slots = cur + E;                    // [n_tok]
  int* tokcnt = slots + p.n_tok;           // [M] locally routed slots per token
  unsigned* sok = reinterpret_cast<unsigned*>(tokcnt + p.M);  // [n_tok/32+1] slot-is-local bits
  int* eid = reinterpret_cast<int*>(sok + p.n_tok / 32 + 1);   // [n_tok] local expert per slot
  float* red = reinterpret_cast<float*>(dsm + p.red_offset);  // [n_red][tile][warp slot][NG][128]
  unsigned char* ring = dsm + p.ring_offset;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_red = p.n_red;

  // ---------------- prologue: barriers + routing tables ----------------
  // The first top-k id of each thread is loaded before anything else, so its
  // global-memory latency overlaps the barrier set-up.
  const int my_e = tid < p.n_tok ? p.map(tid) : -1;
  if (tid == 0) {
    trace_ev(p.trace, 5, 0);
    trace_cta(p.trace, 0);
  }
  if (tid < kDecMaxStages) {
    mbar_init(&full_bar[tid], 1);
    mbar_init(&empty_bar[tid], kDecConsumers);
    fence_barrier_init();
  } else if (tid >= 32 && tid < 32 + kDecEpiWarps) {
    mbar_init(&red_full[tid - 32], kDecConsumers);
    mbar_init(&red_empty[tid - 32], 1);
    fence_barrier_init();
  }
  for (int e = tid; e < E; e += kDecThreads) cnt[e] = 0;
  for (int m = tid; m < p.M; m += kDecThreads) tokcnt[m] = 0;
  for (int w = tid; w <= p.n_tok / 32; w += kDecThreads) sok[w] = 0;
  __syncthreads();
  for (int i = tid; i < p.n_tok; i += kDecThreads) {
    const int e = i == tid ? my_e : p.map(i);
    eid[i] = e;
    if (e >= 0) {
      atomicAdd(&cnt[e], 1);
      atomicAdd(&tokcnt[i / p.topk], 1);
      atomicOr(&sok[i >> 5], 1u << (i & 31));
    }
  }
  __syncthreads();
  // Exclusive scans of the counts and of (count > 0), and the largest count,
  // by all warps: warp w scans experts [32w, 32w + 32) (pass 1), then adds the
  // totals of the warps before it (pass 2).
  constexpr int kWarps = kDecThreads / 32;
  const int nEw = (E + 31) / 32;  // <= 32 (E <= 1024)
  const unsigned lanes_le = 0xffffffffu >> (31 - lane);
  for (int w = warp; w < nEw; w += kWarps) {
    const int e = w * 32 + lane;
    const int c = e < E ? cnt[e] : 0;
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += a;
    }
    const unsigned actm = __ballot_sync(0xffffffffu, c > 0);
    if (e < E) {
      off[e] = inc - c;                                   // local exclusive offset
      cur[e] = c > 0 ? __popc(actm & lanes_le) - 1 : -1;  // local active rank
    }
    const int mx = (int)__reduce_max_sync(0xffffffffu, (unsigned)c);
    if (lane == 31) {
      s_wtot[w] = inc;
      s_wact[w] = __popc(actm);
      s_wmax[w] = mx;
    }
  }
  __syncthreads();
  for (int w = warp; w < nEw; w += kWarps) {
    const int e = w * 32 + lane;
    const int tot = lane < w ? s_wtot[lane] : 0, na = lane < w ? s_wact[lane] : 0;
    const int base = (int)__reduce_add_sync(0xffffffffu, (unsigned)tot);
    const int abase = (int)__reduce_add_sync(0xffffffffu, (unsigned)na);
    if (e < E) {
      const int o = off[e] + base;
      off[e] = o;
      if (cur[e] >= 0) act[abase + cur[e]] = e;
      cur[e] = o;
    }
    if (w == 0) {
      const int t = lane < nEw ? s_wtot[lane] : 0, a = lane < nEw ? s_wact[lane] : 0;
      const int m = lane < nEw ? s_wmax[lane] : 0;
      const int run = (int)__reduce_add_sync(0xffffffffu, (unsigned)t);
      const int nact = (int)__reduce_add_sync(0xffffffffu, (unsigned)a);
      const int mxall = (int)__reduce_max_sync(0xffffffffu, (unsigned)m);
      if (lane == 0) {
        off[E] = run;
        s_nact = nact;
        // stage geometry for this many reserved activation rows, precomputed
        // on the host (decode_plan) for every row count 1..NB
        const int rr = max(1, min(NB, mxall));
        Geometry gm;
        gm.rows_res = rr;
        gm.ncA = p.geo[rr][0];
        gm.ncB = p.geo[rr][1];
        gm.stage_bytes = p.geo[rr][2];
        gm.n_stages = p.geo[rr][3];
        s_geo = gm;
      }
    }
  }
  __syncthreads();
  if (warp == 0) ordered_slot_scatter(eid, p.n_tok, cur, slots, lane);
  // Expert-parallel: tokens with no local slot get a zero row.
  if (p.zero_rows) {
    for (int m = blockIdx.x * kDecThreads + tid; m < p.M; m += gridDim.x * kDecThreads)
      if (tokcnt[m] == 0)
        for (int h = 0; h < p.H; h += 8)
          *reinterpret_cast<uint4*>(p.out + (size_t)m * p.H + h) = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  if (tid == 0) {
    trace_ev(p.trace, 5, 1);
    trace_cta(p.trace, 1);
  }

  const Geometry geo = s_geo;
  const int nact = s_nact;
  const int PA = (p.I / 16) / p.RP;  // phase-A items per expert
  const int PB = (p.H / 16) / p.R2;  // phase-B items per expert
  const int nA = nact * PA;
  const int total = nA + nact * PB;
  const int chA = p.H / 64, chB = p.I / 64;
  const int partsA = chA / geo.ncA, partsB = chB / geo.ncB;
  const int S = geo.n_stages;

  auto view = [&](int item) {
    ItemView v;
    v.phB = item >= nA;
    const int it = v.phB ? item - nA : item;
    const int per = v.phB ? PB : PA;
    const int j = it / per;
    v.q = it - j * per;
    v.e = act[j];
    v.T = cnt[v.e];
    v.base = off[v.e];
    return v;
  };

  if (warp >= kDecProducerWarp && warp < kDecProducerWarp + kDecProducers) {
    // ======================= producer warps =======================
    // Both walk the same stage sequence; producer pid issues the stages whose
    // ring slot s has s % kDecProducers == pid, so one stage's copy issue,
    // readiness check and item switch overlap the other's.  Ownership is by
    // slot, not by stage: a slot is always refilled by the same producer, in
    // order, so its parity wait for the previous use of the slot can never
    // see a phase two uses old (stages dealt round robin to more producers
    // than slots aliased that wait and corrupted the barriers).
    const int pid = warp - kDecProducerWarp;
    const uint64_t pol = l2_evict_first_policy();
    int stage = 0;
    uint32_t uses = 0;  // stages issued so far (barrier parities)
    bool abort = false;
    for (int item = blockIdx.x; !abort; item += gridDim.x) {
      const bool done = item >= total;
      ItemView v{};
      if (!done) v = view(item);
      const int passes = done ? 1 : (v.T + NB - 1) / NB;
      const int parts = done ? 1 : (v.phB ? partsB : partsA);
      const int nc = v.phB ? geo.ncB : geo.ncA;
      const int R = v.phB ? p.R2 : 2 * p.RP;
      const int nchunks = v.phB ? chB : chA;
      const int nrt = v.phB ? p.H / 16 : 2 * p.I / 16;
      const uint8_t* wsrc = v.phB ? p.w2 : p.w13;
      const uint8_t* ssrc = v.phB ? p.s2 : p.s13;
      const uint32_t wbytes = (uint32_t)nc * 512, sbytes = (uint32_t)nc * 64, bbytes = (uint32_t)nc * 128;
      const int bstride = nc * 128 + 16;
      bool ready_checked = !v.phB;
      for (int pass = 0; pass < passes && !abort; ++pass) {
        const int rows = done ? 0 : min(NB, v.T - pass * NB);
        for (int part = 0; part < parts; ++part) {
          if (stage % kDecProducers != pid) {  // another producer's slot
            ++uses;
            stage = (stage + 1 == S) ? 0 : stage + 1;
            if (done) break;
            continue;
          }
          if (uses >= (uint32_t)S && !mbar_wait(&empty_bar[stage], ((uses / S) - 1) & 1, kWaitBudget)) {
            if (lane == 0) record_error(p.sched, kErrEmptyWait);
            abort = true;
            break;
          }
          unsigned char* buf = ring + (size_t)stage * geo.stage_bytes;
          if (lane == 0) {
            sinfo[stage] = StageInfo{done ? -1 : item, pass, part, part == parts - 1, nc, R,
                                     31 - __clz(kDecConsumers / (R / RW)), rows};
            const uint32_t tx = done ? 0u : (uint32_t)R * (wbytes + sbytes) + (uint32_t)rows * bbytes;
            if (tx) mbar_arrive_expect_tx(&full_bar[stage], tx);
            else mbar_arrive(&full_bar[stage]);
          }
          __syncwarp();
          if (!done) {
            const int c0 = part * nc;
            for (int cpy = lane; cpy < 2 * R; cpy += 32) {
              const int r = cpy % R;
              int rt;
              if (v.phB) rt = v.q * R + r;
              else rt = (r < p.RP) ? v.q * p.RP + r : p.I / 16 + v.q * p.RP + (r - p.RP);
              const size_t blk = ((size_t)v.e * nrt + rt) * nchunks + c0;
              if (cpy < R)
                bulk_g2s_hint(buf + (size_t)r * wbytes, wsrc + blk * 512, wbytes, &full_bar[stage], pol);
              else
                bulk_g2s_hint(buf + (size_t)R * wbytes + (size_t)r * sbytes, ssrc + blk * 64, sbytes,
                              &full_bar[stage], pol);
            }
            if (!ready_checked) {
              // expert e's intermediate rows are complete once all of its
              // phase-A item passes have published
              if (lane == 0) {
                const int target = PA * passes;
                const long long t0 = clock64();
                while (ld_acquire_gpu(p.ready + v.e) < target) {
                  if (clock64() - t0 > p.ready_budget) {
                    record_error(p.sched, kErrReadyWait);
                    break;
                  }
                  __nanosleep(32);
                }
              }
              __syncwarp();
              fence_proxy_async_global();
              ready_checked = true;
            }
            unsigned char* bdst = buf + (size_t)R * (wbytes + sbytes);
            for (int rr = lane; rr < rows; rr += 32) {
              const int slot = slots[v.base + pass * NB + rr];
              const __nv_bfloat16* src = v.phB ? p.inter + (size_t)slot * p.I + c0 * 64
                                               : p.hidden + (size_t)(slot / p.topk) * p.hidden_ld + c0 * 64;
              bulk_g2s(bdst + (size_t)rr * bstride, src, bbytes, &full_bar[stage]);
            }
          }
          if (lane == 0) trace_ev(p.trace, 0, (int)uses);
          ++uses;
          stage = (stage + 1 == S) ? 0 : stage + 1;
          if (done) break;
        }
        if (done) break;
      }
      if (done) break;
    }
    if (lane == 0) trace_cta(p.trace, 4);
  } else if (warp < kDecConsumers) {
    // ======================= consumer warps =======================
    const int g = lane >> 2, t = lane & 3;
    int stage = 0, rb = 0;
    uint32_t uses = 0, ruses = 0;  // stages consumed; item passes handed off
    float acc[RW][NG][4];
    while (true) {
      if (!mbar_wait(&full_bar[stage], (uses / S) & 1, kWaitBudget)) {
        if (lane == 0) record_error(p.sched, kErrFullWait);
        break;
      }
      if (warp == 0 && lane == 0) trace_ev(p.trace, 1, (int)uses);
      const StageInfo si = sinfo[stage];
      if (si.item < 0) {
        // tell every epilogue warp there is nothing more
        for (int k = 0; k < n_red; ++k) {
          const uint32_t ru = ruses / n_red;  // earlier uses of buffer rb
          if (ru > 0 && !mbar_wait(&red_empty[rb], (ru - 1) & 1, kWaitBudget)) {
            if (lane == 0) record_error(p.sched, kErrRedWait);
            break;
          }
          if (warp == 0 && lane == 0) rinfo[rb] = StageInfo{-1, 0, 0, 0, 0, 0, 0, 0};
          __syncwarp();
          if (lane == 0) mbar_arrive(&red_full[rb]);
          ++ruses;
          rb = (rb + 1 == n_red) ? 0 : rb + 1;
        }
        if (warp == 0 && lane == 0) trace_cta(p.trace, 6);
        break;
      }
      const int nc = si.nc, R = si.R;
      const int wpg = 1 << si.lgw;  // warps per tile group
      const int tg = warp >> si.lgw, cw = warp & (wpg - 1);
      if (si.part == 0) {
#pragma unroll
        for (int i = 0; i < RW; ++i)
#pragma unroll
          for (int a = 0; a < NG; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) acc[i][a][b] = 0.f;
      }
      const unsigned char* buf = ring + (size_t)stage * geo.stage_bytes;
      const unsigned char* wt = buf + (size_t)(tg * RW) * nc * 512 + lane * 16;
      const unsigned char* sc = buf + (size_t)R * nc * 512 + (size_t)(tg * RW) * nc * 64 + g * 8;
      const unsigned char* bs = buf + (size_t)R * nc * 576;
      const int bstride = nc * 128 + 16;
      const int rows = si.rows;
      for (int c = cw; c < nc; c += wpg) {
        if constexpr (NG == 1) {
          const unsigned char* brow = bs + brow_off(lane, geo.rows_res, bstride) + c * 128;
          uint32_t b0[4], b1[4];
          ldmatrix_x4(b0, brow);
          ldmatrix_x4(b1, brow + 64);
#pragma unroll
          for (int i = 0; i < RW; ++i) {
            const uint4 wv = lds128(wt + (size_t)(i * nc + c) * 512);
            const uint2 sv = lds64(sc + (size_t)(i * nc + c) * 64);
            uint32_t A0[4], A1[4], A2[4], A3[4];
            unscaled_word(wv.x, A0);
            unscaled_word(wv.y, A1);
            unscaled_word(wv.z, A2);
            unscaled_word(wv.w, A3);
            float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
            mma_bf16_16816_nv(t0, A0, b0[0], b0[1]);
            mma_bf16_16816_nv(t1, A2, b1[0], b1[1]);
            mma_bf16_16816_nv(t0, A1, b0[2], b0[3]);
            mma_bf16_16816_nv(t1, A3, b1[2], b1[3]);
            const float s0 = bf16_lo_f32(sv.x), s08 = bf16_hi_f32(sv.x);
            const float s1 = bf16_lo_f32(sv.y), s18 = bf16_hi_f32(sv.y);
            acc[i][0][0] = fmaf(s0, t0[0], fmaf(s1, t1[0], acc[i][0][0]));
            acc[i][0][1] = fmaf(s0, t0[1], fmaf(s1, t1[1], acc[i][0][1]));
            acc[i][0][2] = fmaf(s08, t0[2], fmaf(s18, t1[2], acc[i][0][2]));
            acc[i][0][3] = fmaf(s08, t0[3], fmaf(s18, t1[3], acc[i][0][3]));
          }
        } else {
          uint32_t A[RW][4][4];
#pragma unroll
          for (int i = 0; i < RW; ++i) {
            const uint4 wv = lds128(wt + (size_t)(i * nc + c) * 512);
            const uint2 sv = lds64(sc + (size_t)(i * nc + c) * 64);
            const uint32_t sg0 = __byte_perm(sv.x, 0, 0x1010), sg80 = __byte_perm(sv.x, 0, 0x3232);
            const uint32_t sg1 = __byte_perm(sv.y, 0, 0x1010), sg81 = __byte_perm(sv.y, 0, 0x3232);
            dequant_word(wv.x, sg0, sg80, A[i][0]);
            dequant_word(wv.y, sg0, sg80, A[i][1]);
            dequant_word(wv.z, sg1, sg81, A[i][2]);
            dequant_word(wv.w, sg1, sg81, A[i][3]);
          }
#pragma unroll
          for (int qq = 0; qq < NG; ++qq) {
            if (qq * 8 >= rows) break;
            const unsigned char* brow = bs + brow_off(lane, geo.rows_res - qq * 8, bstride) + qq * 8 * bstride + c * 128;
            uint32_t b0[4], b1[4];
            ldmatrix_x4(b0, brow);
            ldmatrix_x4(b1, brow + 64);
#pragma unroll
            for (int i = 0; i < RW; ++i) {
              mma_bf16_16816_nv(acc[i][qq], A[i][0], b0[0], b0[1]);
              mma_bf16_16816_nv(acc[i][qq], A[i][1], b0[2], b0[3]);
              mma_bf16_16816_nv(acc[i][qq], A[i][2], b1[0], b1[1]);
              mma_bf16_16816_nv(acc[i][qq], A[i][3], b1[2], b1[3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[stage]);
      if (warp == 0 && lane == 0) trace_ev(p.trace, 2, (int)uses);
      ++uses;
      stage = (stage + 1 == S) ? 0 : stage + 1;
      if (!si.last) continue;

      // end of an item pass: hand the accumulators to an epilogue warp
      const uint32_t ru = ruses / n_red;
      if (ru > 0 && !mbar_wait(&red_empty[rb], (ru - 1) & 1, kWaitBudget)) {
        if (lane == 0) record_error(p.sched, kErrRedWait);
        break;
      }
      float* rbase = red + (size_t)rb * kRedFloats;
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        float* my = rbase + ((size_t)((tg * RW + i) * wpg + cw) * NG) * 128;
#pragma unroll
        for (int qq = 0; qq < NG; ++qq) {
          *reinterpret_cast<float2*>(my + qq * 128 + g * 8 + 2 * t) = make_float2(acc[i][qq][0], acc[i][qq][1]);
          *reinterpret_cast<float2*>(my + qq * 128 + (g + 8) * 8 + 2 * t) =
              make_float2(acc[i][qq][2], acc[i][qq][3]);
        }
      }
      if (warp == 0 && lane == 0) rinfo[rb] = si;
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[rb]);
      ++ruses;
      rb = (rb + 1 == n_red) ? 0 : rb + 1;
    }
  } else if (warp - kDecConsumers - kDecProducers < n_red) {
    // ======================= epilogue warps =======================
    const int rb = warp - kDecConsumers - kDecProducers;  // this warp's reduction buffer
    const float* rbuf = red + (size_t)rb * kRedFloats;
    uint32_t ru = 0;
    while (true) {
      if (!mbar_wait(&red_full[rb], ru & 1, kWaitBudget)) {
        if (lane == 0) record_error(p.sched, kErrRedWait);
        break;
      }
      const StageInfo si = rinfo[rb];
      if (si.item < 0) break;
      if (rb == 0 && lane == 0) trace_ev(p.trace, 3, (int)ru);
      const ItemView v = view(si.item);
      const int rows = min(NB, v.T - si.pass * NB);
      const int* sl = slots + v.base + si.pass * NB;
      const int R = v.phB ? p.R2 : 2 * p.RP;
      const int wpg = kDecConsumers / (R / RW);  // warp slots per tile
      // sum over the wpg warp partials of (tile, qq), elements 4*e4 .. 4*e4+3
      auto tile_sum4 = [&](int tile, int qq, int e4) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < wpg; ++w) {
          const float4 x =
              *reinterpret_cast<const float4*>(rbuf + ((size_t)(tile * wpg + w) * NG + qq) * 128 + e4 * 4);
          s.x += x.x;
          s.y += x.y;
          s.z += x.z;
          s.w += x.w;
        }
        return s;
      };
      if (!v.phB) {
        const int RP = p.RP;
        for (int idx = lane; idx < RP * NG * 32; idx += 32) {
          const int i = idx / (NG * 32), rem = idx - i * (NG * 32);
          const int qq = rem >> 5, e4 = rem & 31;  // row e4/2, columns (e4&1)*4 .. +3
          const float4 gs = tile_sum4(i, qq, e4), us = tile_sum4(RP + i, qq, e4);
          const int row = e4 >> 1, col0 = (e4 & 1) * 4;
          const float gv[4] = {gs.x, gs.y, gs.z, gs.w}, uv[4] = {us.x, us.y, us.z, us.w};
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int colidx = qq * 8 + col0 + cc;
            if (colidx < rows)
              p.inter[(size_t)sl[colidx] * p.I + (v.q * RP + i) * 16 + row] =
                  __float2bfloat16(silu_f(gv[cc]) * uv[cc]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_empty[rb]);  // buffer no longer read
        __threadfence();
        __syncwarp();
        if (lane == 0 && !(p.withhold && blockIdx.x == 0)) atomicAdd(p.ready + v.e, 1);
      } else {
        const int R2 = p.R2, span = R2 * 16;
        for (int idx = lane; idx < R2 * NG * 32; idx += 32) {
          const int rr = idx / (NG * 32), rem = idx - rr * (NG * 32);
          const int qq = rem >> 5, e4 = rem & 31;
          const float4 s4 = tile_sum4(rr, qq, e4);
          const int row = e4 >> 1, col0 = (e4 & 1) * 4;
          const float sv4[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int colidx = qq * 8 + col0 + cc;
            if (colidx < rows) {
              const int slot = sl[colidx];
              p.partial[(size_t)slot * p.H + v.q * span + rr * 16 + row] = sv4[cc] * p.topk_w[slot];
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_empty[rb]);  // buffer no longer read
        __threadfence();
        __syncwarp();
        if (p.tail_reduce) {
          if (lane == 0) atomicAdd(p.sched + kSchedBDone, 1);
        } else {
          // the last arriver per (token, row block) sums the token's partials
          for (int c0 = 0; c0 < rows; c0 += 32) {
            int mine = -1;
            if (c0 + lane < rows) {
              const int m = sl[c0 + lane] / p.topk;
              int* cptr = p.counters + (size_t)m * PB + v.q;
              if (atomicAdd(cptr, 1) == tokcnt[m] - 1) {
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
              for (int hr = lane; hr < span; hr += 32) {
                const float* pp = p.partial + (size_t)m * p.topk * p.H + v.q * span + hr;
                float sum = 0.f;
                for (int t0 = 0; t0 < p.topk; t0 += 16) {
                  // all loads of a batch in flight before the ordered sum
                  float xs[16];
#pragma unroll
                  for (int i = 0; i < 16; ++i) xs[i] = t0 + i < p.topk ? __ldcg(pp + (size_t)(t0 + i) * p.H) : 0.f;
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                    const int slot = m * p.topk + t0 + i;
                    if (t0 + i < p.topk && ((sok[slot >> 5] >> (slot & 31)) & 1u)) sum += xs[i];
                  }
                }
                p.out[(size_t)m * p.H + v.q * span + hr] = __float2bfloat16(sum);
              }
            }
          }
        }
      }
      if (rb == 0 && lane == 0) trace_ev(p.trace, 4, (int)ru);
      ++ru;
    }
  }

  // ---------------- tail: grid-wide top-k sum of the partials ----------------
  // (larger M) once every phase-B item pass of every CTA has stored its
  // partials, out[m, :] = sum over t in slot order of partial[m*topk+t, :].
  __syncthreads();
  if (p.tail_reduce) {
    if (tid == 0) {
      int target = 0;
      for (int jj = 0; jj < nact; ++jj) target += PB * ((cnt[act[jj]] + NB - 1) / NB);
      const long long t0 = clock64();
      while (ld_acquire_gpu(p.sched + kSchedBDone) < target) {
        if (clock64() - t0 > kWaitBudget) {
          record_error(p.sched, kErrReadyWait);
          break;
        }
        __nanosleep(64);
      }
    }
    __syncthreads();
    const int h4 = p.H / 4;
    const int n4 = p.M * h4;
    for (int idx = blockIdx.x * kDecThreads + tid; idx < n4; idx += gridDim.x * kDecThreads) {
      const int m = idx / h4, h = (idx - m * h4) * 4;
      if (tokcnt[m] == 0) continue;
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
      const float* pp = p.partial + (size_t)m * p.topk * p.H + h;
#pragma unroll 4
      for (int tt = 0; tt < p.topk; ++tt) {
        const int slot = m * p.topk + tt;
        const float4 x = __ldcg(reinterpret_cast<const float4*>(pp + (size_t)tt * p.H));
        if ((sok[slot >> 5] >> (slot & 31)) & 1u) {
          sum.x += x.x;
          sum.y += x.y;
          sum.z += x.z;
          sum.w += x.w;
        }
      }
      __nv_bfloat162 lo = __floats2bfloat162_rn(sum.x, sum.y), hi = __floats2bfloat162_rn(sum.z, sum.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&lo);
      pk.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(p.out + (size_t)m * p.H + h) = pk;
    }
  }

  // ---------------- teardown: the last CTA resets the global counters ----------------
  __syncthreads();
  if (tid == 0) {
    trace_ev(p.trace, 5, 2);
    trace_cta(p.trace, 9);
    __threadfence();
    s_last = atomicAdd(p.sched + kSchedDone, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    for (int e = tid; e < E; e += kDecThreads) p.ready[e] = 0;
    if (tid == 0) {
      p.sched[kSchedDone] = 0;
      p.sched[kSchedBDone] = 0;
    }
    __threadfence();
  }
}

int decode_plan(DecodeParams& p, int sms, int max_smem) {
  const int n_tok = p.n_tok;
  if (n_tok > kDecodeMaxSlots || p.E > 1024) return 0;
  const int max_active = n_tok < p.E ? n_tok : p.E;
  const double avg = (double)n_tok / (double)(max_active > 0 ? max_active : 1);
  const int NG = avg <= 1.5 ? 1 : (avg <= 6.0 ? 2 : 4);
  const int M = p.M;
  // item sizes (row tiles per w13 / w2 item), measured on B200 at E=256
  // top-10 3072x1024: larger items amortise per-item handoffs until too few
  // items remain to balance over the SMs
  // (with two producer warps: one gate/up pair per w13 item up to M=8, w2
  // items of 4 row tiles at M=1 and 9..16, 8 otherwise)
  int RP = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  int R2 = (M == 1 || (M > 8 && M <= 16)) ? 4 : 8;
#ifdef W4A16_DIAGNOSTICS
  if (const char* e = getenv("W4A16_DECODE_RP")) RP = atoi(e);
  if (const char* e = getenv("W4A16_DECODE_R2")) R2 = atoi(e);
#endif
  while (RP > 1 && (p.I / 16) % RP) RP >>= 1;
  while (R2 > 2 && (p.H / 16) % R2) R2 >>= 1;
  if ((p.H / 16) % R2 || (p.I / 16) % RP) return 0;
  const int RW = rows_per_warp(NG);
  if ((2 * RP) % RW || R2 % RW) return 0;
  p.NG = NG;
  p.RP = RP;
  p.R2 = R2;
  // grid-wide top-k sum after all w2 items (measured faster than the
  // per-(token, row block) last-arriver sum at every M on B200)
  p.tail_reduce = 1;
  p.ready_budget = kWaitBudget;
  p.withhold = 0;
#ifdef W4A16_DIAGNOSTICS
  if (const char* e = getenv("W4A16_DECODE_TAIL")) p.tail_reduce = atoi(e);
#endif
  const int route_bytes = (4 * p.E + 1 + 2 * n_tok + M + n_tok / 32 + 1) * 4;
  p.red_offset = (route_bytes + 127) / 128 * 128;
  const int red_buf = kDecConsumers * RW * NG * 128 * 4;
  p.n_red = 65536 / red_buf;
  if (p.n_red > kDecEpiWarps) p.n_red = kDecEpiWarps;
  if (p.n_red < 2) p.n_red = 2;
  p.ring_offset = p.red_offset + p.n_red * red_buf;
  p.ring_bytes = (max_smem - p.ring_offset - 1024) / 128 * 128;  // room for static smem
  // the smallest stage (one chunk, all 8*NG rows) must fit three times
  const int minA = 2 * RP * 576 + 8 * NG * (128 + 16), minB = R2 * 576 + 8 * NG * (128 + 16);
  if (p.ring_bytes < 3 * (minA > minB ? minA : minB)) return 0;
  p.smem_bytes = p.ring_offset + p.ring_bytes;
  p.grid = sms;
  // two large stages: measured best at every M (more, smaller stages cost
  // more per-stage handshakes than they hide latency)
  if (p.ring_div <= 0) p.ring_div = 2;
#ifdef W4A16_DIAGNOSTICS
  if (const char* e = getenv("W4A16_DECODE_RING_DIV")) p.ring_div = atoi(e) > 0 ? atoi(e) : p.ring_div;
#endif
  // stage geometry per reserved row count: the largest stages that still fit
  // ring_div of them in the ring
  const int cap = p.ring_bytes / p.ring_div / 128 * 128;
  for (int rr = 1; rr <= 8 * NG && rr < kDecGeoRows; ++rr) {
    const int ncA = pick_nc(p.H / 64, 2 * RP, rr, cap), ncB = pick_nc(p.I / 64, R2, rr, cap);
    if (ncA == 0 || ncB == 0) return 0;
    const int sb = ((stage_bytes_for(2 * RP, ncA, rr) > stage_bytes_for(R2, ncB, rr) ? stage_bytes_for(2 * RP, ncA, rr)
                                                                                       : stage_bytes_for(R2, ncB, rr)) +
                    127) / 128 * 128;
    p.geo[rr][0] = ncA;
    p.geo[rr][1] = ncB;
    p.geo[rr][2] = sb;
    p.geo[rr][3] = p.ring_bytes / sb < kDecMaxStages ? p.ring_bytes / sb : kDecMaxStages;
  }
  return 1;
}

cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream) {
  // per (device, NG instantiation): largest dynamic smem size opted in so far
  static thread_local int configured[64][3] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  auto launch = [&](auto kern, int slot) -> cudaError_t {
    if (configured[dev][slot] < p.smem_bytes) {
      cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem_bytes);
      if (err != cudaSuccess) return err;
      configured[dev][slot] = p.smem_bytes;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
  };
  switch (p.NG) {
    case 1: return launch(moe_decode_fused_kernel<1>, 0);
    case 2: return launch(moe_decode_fused_kernel<2>, 1);
    default: return launch(moe_decode_fused_kernel<4>, 2);
  }
}

}  // namespace w4moe
