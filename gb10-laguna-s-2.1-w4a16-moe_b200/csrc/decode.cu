// Fused small-M ("decode") MoE layer: routing + w13 (+SiLU*up) + w2 (+ router-
// weighted top-k sum) in ONE persistent, warp-specialised kernel.
//
// Replaces, for M*topk <= kDecodeMaxSlots, the reference's moe_align_block_size
// + _w4a16_moe_w1_fused_kernel + _w4a16_moe_w2_kernel + _moe_sum_kernel
// (kernels/w4a16_moe.py:187-290, :374-670).
//
// Structure (one CTA per SM, 9 warps):
//   * prologue: every CTA builds the routing tables in shared memory from the
//     raw top-k ids (histogram, scan, per-expert slot lists); no align launch.
//   * work items, claimed dynamically from a global counter:
//       phase A  (active expert j, RP gate/up row-tile pairs)  -> w13
//       phase B  (active expert j, R2 hidden row tiles)        -> w2
//     every item's K range is cut into parts that fit one pipeline stage, and
//     an expert with more slots than one pass holds (8*NG) is done in passes.
//   * producer warp: for each stage, cp.async.bulk of the item's weight and
//     scale blocks (contiguous per row tile in the fragment-major layout) and
//     of the pass's activation rows (hidden rows in phase A, intermediate rows
//     in phase B) into a shared-memory ring; completion via mbarrier tx-count.
//     Phase-B activation copies wait (bounded) until all phase-A items of the
//     same expert have published their intermediate rows; the weight copies of
//     that stage are issued before the wait, so HBM streaming never pauses at
//     the w13 -> w2 boundary.
//   * 8 consumer warps: decode int4 words from smem straight into m16n8k16 A
//     fragments (scale folded in, bf16-exact like the reference's dequant),
//     B fragments via ldmatrix, fp32 accumulation in registers; warps sharing
//     a row tile reduce through smem at the end of an item pass.
//   * epilogues: A writes bf16(silu(gate)*up) rows to the intermediate buffer
//     and bumps ready[e]; B scales by the router weight, writes fp32 partials,
//     and the last of a token's slots to finish a row block sums that token's
//     partials in slot order (deterministic) and writes the bf16 output.
//   * all global counters are self-cleaning (the last CTA resets them).
#include "launch.cuh"

namespace w4moe {

constexpr int kDecConsumers = 8;
constexpr int kDecThreads = (kDecConsumers + 1) * 32;
constexpr int kDecMaxStages = 8;
constexpr long long kWaitBudget = 4000000000LL;  // ~2 s of SM clocks

// sched[] words in the workspace
constexpr int kSchedNext = 0, kSchedDone = 1, kSchedError = 2;

enum DecodeError : int {
  kErrFullWait = 1,
  kErrEmptyWait = 2,
  kErrReadyWait = 4,
};

struct StageInfo {
  int item;  // -1 = end of work
  int pass;
  int part;
  int pad;
};

__device__ __forceinline__ void record_error(int* sched, int code) { atomicOr(sched + kSchedError, code); }

template <int NG>
__global__ void __launch_bounds__(kDecThreads, 1) moe_decode_fused_kernel(DecodeParams p) {
  constexpr int NB = 8 * NG;
  __shared__ uint64_t full_bar[kDecMaxStages], empty_bar[kDecMaxStages];
  __shared__ StageInfo sinfo[kDecMaxStages];
  __shared__ int s_nact;
  __shared__ int s_last[NB];
  extern __shared__ __align__(128) unsigned char dsm[];

  const int E = p.E;
  int* cnt = reinterpret_cast<int*>(dsm);  // [E]
  int* off = cnt + E;                      // [E+1]
  int* act = off + E + 1;                  // [E]
  int* cur = act + E;                      // [E]
  int* slots = cur + E;                    // [n_tok]
  float* red = reinterpret_cast<float*>(dsm + p.red_offset);  // [8][NG][128]
  unsigned char* ring = dsm + p.ring_offset;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // ---------------- prologue: barriers + routing tables ----------------
  if (tid == 0) {
    for (int s = 0; s < p.n_stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kDecConsumers);
    }
    fence_barrier_init();
  }
  for (int e = tid; e < E; e += kDecThreads) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < p.n_tok; i += kDecThreads) {
    const int e = p.map(i);
    if (e >= 0) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan of counts and of (count > 0)
    int run = 0, nact = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < E ? cnt[e] : 0;
      int inc = c, ia = c > 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, inc, o);
        const int b = __shfl_up_sync(0xffffffffu, ia, o);
        if (lane >= o) { inc += a; ia += b; }
      }
      if (e < E) {
        off[e] = run + inc - c;
        cur[e] = run + inc - c;
        if (c > 0) act[nact + ia - 1] = e;
      }
      run += __shfl_sync(0xffffffffu, inc, 31);
      nact += __shfl_sync(0xffffffffu, ia, 31);
    }
    if (lane == 0) {
      off[E] = run;
      s_nact = nact;
    }
  }
  __syncthreads();
  for (int i = tid; i < p.n_tok; i += kDecThreads) {
    const int e = p.map(i);
    if (e >= 0) slots[atomicAdd(&cur[e], 1)] = i;
  }
  // Expert-parallel: tokens with no local slot get a zero row.
  if (p.zero_rows) {
    for (int m = blockIdx.x * kDecThreads + tid; m < p.M; m += gridDim.x * kDecThreads) {
      int c = 0;
      for (int t = 0; t < p.topk; ++t) c += p.map(m * p.topk + t) >= 0;
      if (c == 0)
        for (int h = 0; h < p.H; h += 8)
          *reinterpret_cast<uint4*>(p.out + (size_t)m * p.H + h) = make_uint4(0, 0, 0, 0);
    }
  }
  __syncthreads();

  const int nact = s_nact;
  const int PA = (p.I / 16) / p.RP;  // phase-A items per expert
  const int PB = (p.H / 16) / p.R2;  // phase-B items per expert
  const int nA = nact * PA;
  const int total = nA + nact * PB;
  const int chA = p.H / 64, chB = p.I / 64;
  const int partsA = chA / p.ncA, partsB = chB / p.ncB;

  if (warp == kDecConsumers) {
    // ======================= producer warp =======================
    const uint64_t pol = l2_evict_first_policy();
    int stage = 0;
    uint32_t uses = 0;  // total stages issued (for barrier parities)
    bool abort = false;
    while (!abort) {
      int item = 0;
      if (lane == 0) item = atomicAdd(p.sched + kSchedNext, 1);
      item = __shfl_sync(0xffffffffu, item, 0);
      const bool done = item >= total;
      const bool phB = item >= nA;
      const int it = phB ? item - nA : item;
      const int per = phB ? PB : PA;
      const int j = done ? 0 : it / per, q = done ? 0 : it - (it / per) * per;
      const int e = done ? 0 : act[j];
      const int T = done ? 0 : cnt[e];
      const int base = done ? 0 : off[e];
      const int passes = done ? 1 : (T + NB - 1) / NB;
      const int parts = done ? 1 : (phB ? partsB : partsA);
      const int nc = phB ? p.ncB : p.ncA;
      const int R = phB ? p.R2 : 2 * p.RP;
      const int nchunks = phB ? chB : chA;
      const int nrt = phB ? p.H / 16 : 2 * p.I / 16;
      const uint8_t* wsrc = phB ? p.w2 : p.w13;
      const uint8_t* ssrc = phB ? p.s2 : p.s13;
      bool ready_checked = !phB;
      for (int pass = 0; pass < passes && !abort; ++pass) {
        for (int part = 0; part < parts; ++part) {
          if (uses >= (uint32_t)p.n_stages) {
            const uint32_t par = ((uses / p.n_stages) - 1) & 1;
            if (!mbar_wait(&empty_bar[stage], par, kWaitBudget)) {
              if (lane == 0) record_error(p.sched, kErrEmptyWait);
              abort = true;
              break;
            }
          }
          unsigned char* buf = ring + (size_t)stage * p.stage_bytes;
          const int rows = done ? 0 : min(NB, T - pass * NB);
          const uint32_t wbytes = (uint32_t)nc * 512, sbytes = (uint32_t)nc * 64, bbytes = (uint32_t)nc * 128;
          if (lane == 0) {
            sinfo[stage] = StageInfo{done ? -1 : item, pass, part, 0};
            const uint32_t tx = done ? 0u : (uint32_t)R * (wbytes + sbytes) + (uint32_t)rows * bbytes;
            if (tx) mbar_arrive_expect_tx(&full_bar[stage], tx);
            else mbar_arrive(&full_bar[stage]);
          }
          __syncwarp();
          if (!done) {
            const int c0 = part * nc;
            // weights + scales of every row tile of the item
            for (int cpy = lane; cpy < 2 * R; cpy += 32) {
              const int r = cpy % R;
              int rt;
              if (phB) rt = q * R + r;
              else rt = (r < p.RP) ? q * p.RP + r : p.I / 16 + q * p.RP + (r - p.RP);
              const size_t blk = ((size_t)e * nrt + rt) * nchunks + c0;
              if (cpy < R) bulk_g2s_hint(buf + (size_t)r * wbytes, wsrc + blk * 512, wbytes, &full_bar[stage], pol);
              else bulk_g2s_hint(buf + (size_t)R * wbytes + (size_t)r * sbytes, ssrc + blk * 64, sbytes,
                                 &full_bar[stage], pol);
            }
            if (!ready_checked) {
              // intermediate rows of expert e are complete once all of its
              // phase-A item passes have published
              if (lane == 0) {
                const int target = PA * passes;
                const long long t0 = clock64();
                while (ld_acquire_gpu(p.ready + e) < target) {
                  if (clock64() - t0 > kWaitBudget) {
                    record_error(p.sched, kErrReadyWait);
                    break;
                  }
                  __nanosleep(64);
                }
              }
              __syncwarp();
              fence_proxy_async_global();
              ready_checked = true;
            }
            unsigned char* bdst = buf + (size_t)R * (wbytes + sbytes);
            const int bstride = nc * 128 + 16;
            for (int rr = lane; rr < rows; rr += 32) {
              const int slot = slots[base + pass * NB + rr];
              const __nv_bfloat16* src =
                  phB ? p.inter + (size_t)slot * p.I + c0 * 64
                      : p.hidden + (size_t)(slot / p.topk) * p.hidden_ld + c0 * 64;
              bulk_g2s(bdst + (size_t)rr * bstride, src, bbytes, &full_bar[stage]);
            }
          }
          ++uses;
          stage = (stage + 1 == p.n_stages) ? 0 : stage + 1;
          if (done) break;
        }
        if (done) break;
      }
      if (done) break;
    }
  } else {
    // ======================= consumer warps =======================
    const int g = lane >> 2, t = lane & 3;
    int stage = 0;
    uint32_t uses = 0;
    float acc[NG][4];
    while (true) {
      if (!mbar_wait(&full_bar[stage], (uses / p.n_stages) & 1, kWaitBudget)) {
        if (lane == 0) record_error(p.sched, kErrFullWait);
        break;
      }
      const StageInfo si = sinfo[stage];
      if (si.item < 0) break;
      const bool phB = si.item >= nA;
      const int it = phB ? si.item - nA : si.item;
      const int per = phB ? PB : PA;
      const int j = it / per, q = it - j * per;
      const int e = act[j];
      const int T = cnt[e];
      const int base = off[e];
      const int parts = phB ? partsB : partsA;
      const int nc = phB ? p.ncB : p.ncA;
      const int R = phB ? p.R2 : 2 * p.RP;
      const int wpt = kDecConsumers / R;  // warps per row tile
      const int r = warp / wpt, cw = warp - (warp / wpt) * wpt;
      if (si.part == 0) {
#pragma unroll
        for (int a = 0; a < NG; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
      }
      const unsigned char* buf = ring + (size_t)stage * p.stage_bytes;
      const unsigned char* wt = buf + (size_t)r * nc * 512;
      const unsigned char* sc = buf + (size_t)R * nc * 512 + (size_t)r * nc * 64;
      const unsigned char* bs = buf + (size_t)R * nc * 576;
      const int bstride = nc * 128 + 16;
      const int rows = min(NB, T - si.pass * NB);
      for (int c = cw; c < nc; c += wpt) {
        const uint4 wv = lds128(wt + (size_t)c * 512 + lane * 16);
        const uint2 sv = lds64(sc + (size_t)c * 64 + g * 8);
        uint32_t A[4][4];
        const uint32_t sg0 = __byte_perm(sv.x, 0, 0x1010), sg80 = __byte_perm(sv.x, 0, 0x3232);
        const uint32_t sg1 = __byte_perm(sv.y, 0, 0x1010), sg81 = __byte_perm(sv.y, 0, 0x3232);
        dequant_word(wv.x, sg0, sg80, A[0]);
        dequant_word(wv.y, sg0, sg80, A[1]);
        dequant_word(wv.z, sg1, sg81, A[2]);
        dequant_word(wv.w, sg1, sg81, A[3]);
#pragma unroll
        for (int qq = 0; qq < NG; ++qq) {
          if (qq * 8 >= rows) break;
          const unsigned char* brow = bs + (size_t)(qq * 8 + (lane & 7)) * bstride + c * 128 + (lane >> 3) * 16;
          uint32_t b[4];
          ldmatrix_x4(b, brow);
          mma_bf16_16816(acc[qq], A[0], b[0], b[1]);
          mma_bf16_16816(acc[qq], A[1], b[2], b[3]);
          ldmatrix_x4(b, brow + 64);
          mma_bf16_16816(acc[qq], A[2], b[0], b[1]);
          mma_bf16_16816(acc[qq], A[3], b[2], b[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[stage]);
      ++uses;
      stage = (stage + 1 == p.n_stages) ? 0 : stage + 1;

      if (si.part != parts - 1) continue;

      // ---------------- end of an item pass: reduce + epilogue ----------------
      float* my = red + (size_t)warp * NG * 128;
#pragma unroll
      for (int qq = 0; qq < NG; ++qq) {
        my[qq * 128 + g * 8 + 2 * t] = acc[qq][0];
        my[qq * 128 + g * 8 + 2 * t + 1] = acc[qq][1];
        my[qq * 128 + (g + 8) * 8 + 2 * t] = acc[qq][2];
        my[qq * 128 + (g + 8) * 8 + 2 * t + 1] = acc[qq][3];
      }
      named_barrier_sync(1, kDecConsumers * 32);
      const int ctid = tid;  // 0..255
      if (!phB) {
        const int RP = p.RP;
        for (int idx = ctid; idx < RP * NG * 128; idx += kDecConsumers * 32) {
          const int i = idx / (NG * 128), rem = idx - i * (NG * 128);
          const int qq = rem >> 7, row = (rem >> 3) & 15, col = rem & 7;
          const int colidx = qq * 8 + col;
          if (colidx >= rows) continue;
          float gs = 0.f, us = 0.f;
          for (int w = 0; w < wpt; ++w) {
            gs += red[((size_t)(i * wpt + w) * NG + qq) * 128 + row * 8 + col];
            us += red[((size_t)((RP + i) * wpt + w) * NG + qq) * 128 + row * 8 + col];
          }
          const int slot = slots[base + si.pass * NB + colidx];
          p.inter[(size_t)slot * p.I + (q * RP + i) * 16 + row] = __float2bfloat16(silu_f(gs) * us);
        }
        __threadfence();
        named_barrier_sync(1, kDecConsumers * 32);
        if (ctid == 0) atomicAdd(p.ready + e, 1);
      } else {
        const int R2 = p.R2;
        for (int idx = ctid; idx < R2 * NG * 128; idx += kDecConsumers * 32) {
          const int rr = idx / (NG * 128), rem = idx - rr * (NG * 128);
          const int qq = rem >> 7, row = (rem >> 3) & 15, col = rem & 7;
          const int colidx = qq * 8 + col;
          if (colidx >= rows) continue;
          float v = 0.f;
          for (int w = 0; w < wpt; ++w) v += red[((size_t)(rr * wpt + w) * NG + qq) * 128 + row * 8 + col];
          const int slot = slots[base + si.pass * NB + colidx];
          p.partial[(size_t)slot * p.H + (q * R2 + rr) * 16 + row] = v * p.topk_w[slot];
        }
        __threadfence();
        named_barrier_sync(1, kDecConsumers * 32);
        if (ctid < NB) {
          int last = -1;
          if (ctid < rows) {
            const int slot = slots[base + si.pass * NB + ctid];
            const int m = slot / p.topk;
            int valid = 0;
            for (int tt = 0; tt < p.topk; ++tt) valid += p.map(m * p.topk + tt) >= 0;
            int* c = p.counters + (size_t)m * PB + q;
            if (atomicAdd(c, 1) == valid - 1) {
              *c = 0;  // self-cleaning
              last = m;
            }
          }
          s_last[ctid] = last;
        }
        named_barrier_sync(1, kDecConsumers * 32);
        __threadfence();
        const int span = R2 * 16;
        for (int idx = ctid; idx < NB * span; idx += kDecConsumers * 32) {
          const int col = idx / span, hr = idx - col * span;
          const int m = s_last[col];
          if (m < 0) continue;
          float sum = 0.f;
          for (int tt = 0; tt < p.topk; ++tt) {
            const int slot = m * p.topk + tt;
            if (p.map(slot) < 0) continue;
            sum += __ldcg(p.partial + (size_t)slot * p.H + q * span + hr);
          }
          p.out[(size_t)m * p.H + q * span + hr] = __float2bfloat16(sum);
        }
      }
      named_barrier_sync(1, kDecConsumers * 32);
    }
  }

  // ---------------- teardown: last CTA resets the global counters ----------------
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.sched + kSchedDone, 1) == (int)gridDim.x - 1) {
      p.sched[kSchedNext] = 0;
      p.sched[kSchedDone] = 0;
      for (int e = 0; e < E; ++e) p.ready[e] = 0;
      __threadfence();
    }
  }
}

static int pick_divisor_chunks(int nchunks, int R, int NB, int slot_bytes) {
  int best = 0;
  for (int nc = 1; nc <= nchunks; ++nc) {
    if (nchunks % nc) continue;
    const long long bytes = (long long)R * nc * 576 + (long long)NB * (nc * 128 + 16);
    if (bytes <= slot_bytes) best = nc;
  }
  return best;
}

int decode_plan(DecodeParams& p, int sms, int max_smem) {
  const int n_tok = p.n_tok;
  if (n_tok > kDecodeMaxSlots || p.E > 1024) return 0;
  const int max_active = n_tok < p.E ? n_tok : p.E;
  const double avg = (double)n_tok / (double)(max_active > 0 ? max_active : 1);
  const int NG = avg <= 2.0 ? 1 : (avg <= 8.0 ? 2 : 4);
  const int NB = 8 * NG;
  const int M = p.M;
  int RP = M <= 16 ? 1 : (M <= 64 ? 2 : 4);
  int R2 = M <= 16 ? 2 : (M <= 64 ? 4 : 8);
  while (RP > 1 && (p.I / 16) % RP) RP >>= 1;
  while (R2 > 2 && (p.H / 16) % R2) R2 >>= 1;
  if ((p.H / 16) % R2) return 0;
  p.NG = NG;
  p.RP = RP;
  p.R2 = R2;
  const int route_bytes = (4 * p.E + 1 + n_tok) * 4;
  p.red_offset = (route_bytes + 127) / 128 * 128;
  const int red_bytes = kDecConsumers * NG * 128 * 4;
  p.ring_offset = p.red_offset + (red_bytes + 127) / 128 * 128;
  const int avail = max_smem - p.ring_offset - 1024;  // static smem + slack
  int stages = 6;
  int slot = 0;
  for (; stages >= 3; --stages) {
    slot = (avail / stages) / 128 * 128;
    p.ncA = pick_divisor_chunks(p.H / 64, 2 * RP, NB, slot);
    p.ncB = pick_divisor_chunks(p.I / 64, R2, NB, slot);
    if (p.ncA > 0 && p.ncB > 0) break;
  }
  if (stages < 3) return 0;
  p.n_stages = stages;
  p.stage_bytes = slot;
  p.smem_bytes = p.ring_offset + stages * slot;
  p.grid = sms;
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
    kern<<<p.grid, kDecThreads, p.smem_bytes, stream>>>(p);
    return cudaGetLastError();
  };
  switch (p.NG) {
    case 1: return launch(moe_decode_fused_kernel<1>, 0);
    case 2: return launch(moe_decode_fused_kernel<2>, 1);
    default: return launch(moe_decode_fused_kernel<4>, 2);
  }
}

}  // namespace w4moe
