// Stream-K fused decode for the smallest batches (M <= 4 tokens, M*topk <= 64
// slots): routing + w13 (+SiLU*up) + w2 (+ router-weighted top-k sum) in one
// cooperative launch (two CTAs of 16 warps per SM).
//
// Replaces, for those batches, the reference's moe_align_block_size +
// _w4a16_moe_w1_fused_kernel + _w4a16_moe_w2_kernel + _moe_sum_kernel
// (kernels/w4a16_moe.py:187-290, :374-670 in the reference).
//
// Both phases split their work at WARP granularity, stream-K style: the units
// of a projection (w13: one 64-wide k-chunk of a gate/up row-tile pair of one
// routed expert; w2: one k-chunk of one (hidden row tile, expert)) are
// numbered so that consecutive units are consecutive in memory, and warp w of
// the W warps of the grid takes the contiguous range [U*w/W, U*(w+1)/W).
// Every warp streams its own weight blocks with 16-byte loads (two chunks in
// flight), decodes int4 straight into m16n8k16 A fragments and accumulates in
// registers; no warp waits for another while it streams.  A warp's range
// covers at most two accumulation groups (w13: a pair, w2: a hidden row tile);
// at the end of a group it stores an fp32 piece, and the last of the group's
// warps to arrive (atomic counter) adds the pieces in warp order -- a
// deterministic sum -- and finishes the group:
//   w13: bf16(SiLU(gate) * up) -> intermediate rows (lane-permuted layout),
//        then one more completed pair on a global counter;
//   w2 : sum over experts of router weight * y (MMA columns are tokens) ->
//        bf16 output rows.
// A warp starts its w2 range by loading its first weight block, then waits
// (bounded) until every pair of the call is complete.
//
// Counters are self-cleaning (the last arriver resets its group's counter;
// the last row tile of the call resets the phase counters).
#include <algorithm>

#include "launch.cuh"

namespace w4moe {

namespace {

constexpr int kSpWarps = 16;
constexpr int kSpThreads = kSpWarps * 32;
constexpr int kSpMaxCols = kSplitMaxSlots;  // columns (expert, token pairs) and active experts
constexpr long long kSpBudget = 4000000000LL;  // ~2 s of SM clocks
constexpr int kSpErrReady = 1 << 14;           // status bit: the w2 phase gave up waiting for w13

// Routing tables of one call (shared memory in every CTA).
struct SpRoute {
  int A;                       // active experts
  int act[kSpMaxCols];         // local expert id of active expert ae
  int cnt[kSpMaxCols];         // columns (tokens) of ae
  int base[kSpMaxCols];        // first column of ae (intermediate row)
  int col_tok[kSpMaxCols];     // token of column
  float col_w[kSpMaxCols];     // router weight of column (duplicate slots summed in slot order)
  int tok_col[kSpMaxCols][4];  // column of (ae, token) or -1
};

// Scratch of the CTA-wide routing.
struct SpRouteScratch {
  int key[kSpMaxCols];  // e * 64 + token, or -1
  float wt[kSpMaxCols];
  int dup_col[kSpMaxCols], dup_e[kSpMaxCols];  // an earlier slot has the same column / expert
  int col[kSpMaxCols], below[kSpMaxCols], same[kSpMaxCols], act_below[kSpMaxCols];
};

// Routing for <= 64 slots by the whole CTA (slot pairs spread over the
// threads, integer shared-memory counts, so the result does not depend on
// thread timing).  A column is one (expert, token) pair; columns are ordered
// by expert then token; active experts ascending.  A token naming an expert
// twice gets one column whose router weight is the sum of its slots' weights
// in slot order.  Ends with __syncthreads.
__device__ void sp_route(const SplitParams& p, SpRoute& rt, SpRouteScratch& sc) {
  const int tid = threadIdx.x, nthr = blockDim.x, n = p.n_tok;
  if (tid < kSpMaxCols) {
    int k = -1;
    if (tid < n) {
      const int e = p.map(tid);
      k = e >= 0 ? (e << 6) | (tid / p.topk) : -1;
      sc.wt[tid] = p.topk_w[tid];
    }
    sc.key[tid] = k;
    sc.dup_col[tid] = sc.dup_e[tid] = 0;
    sc.col[tid] = sc.below[tid] = sc.same[tid] = sc.act_below[tid] = 0;
#pragma unroll
    for (int m = 0; m < 4; ++m) rt.tok_col[tid][m] = -1;
  }
  __syncthreads();
  for (int pi = tid; pi < n * n; pi += nthr) {
    const int i = pi / n, j = pi - i * n;
    const int ki = sc.key[i], kj = sc.key[j];
    if (j < i && ki >= 0 && kj >= 0) {
      if (kj == ki) sc.dup_col[i] = 1;
      if ((kj >> 6) == (ki >> 6)) sc.dup_e[i] = 1;
    }
  }
  __syncthreads();
  for (int pi = tid; pi < n * n; pi += nthr) {
    const int i = pi / n, j = pi - i * n;
    const int ki = sc.key[i], kj = sc.key[j];
    if (ki < 0 || kj < 0) continue;
    const int ei = ki >> 6, ej = kj >> 6;
    if (!sc.dup_col[j]) {
      if (kj < ki) atomicAdd(&sc.col[i], 1);
      if (ej < ei) atomicAdd(&sc.below[i], 1);
      if (ej == ei) atomicAdd(&sc.same[i], 1);
    }
    if (!sc.dup_e[j] && ej < ei) atomicAdd(&sc.act_below[i], 1);
  }
  __syncthreads();
  if (tid < n) {
    const int k = sc.key[tid];
    if (k >= 0 && !sc.dup_col[tid]) {
      float wsum = 0.f;
      for (int j = tid; j < n; ++j)
        if (sc.key[j] == k) wsum += sc.wt[j];  // duplicates follow their first slot
      const int col = sc.col[tid], ab = sc.act_below[tid];
      rt.col_tok[col] = k & 63;
      rt.col_w[col] = wsum;
      rt.tok_col[ab][k & 63] = col;
      if (!sc.dup_e[tid]) {
        rt.act[ab] = k >> 6;
        rt.base[ab] = sc.below[tid];
        rt.cnt[ab] = sc.same[tid];
      }
    }
  }
  if (tid < 32) {
    int na = 0;
    for (int i = tid; i < n; i += 32) na += sc.key[i] >= 0 && !sc.dup_e[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) na += __shfl_xor_sync(0xffffffffu, na, o);
    if (tid == 0) rt.A = na;
  }
  __syncthreads();
}

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// acc[0..3] += scale * (A_block . B) for one 16-row x 64-k block.
__device__ __forceinline__ void sp_block(float (&acc)[4], const uint4 wv, const uint2 sv, const uint4 q0,
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

__device__ __forceinline__ void red_release_add(int32_t* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int sp_perm(int i) {
  return (i & ~63) + (((i & 7) >> 1) << 4) + (((i & 63) >> 4) << 2) + (i & 1) + (((i >> 3) & 1) << 1);
}

// First unit of warp w when U units are split over W warps (U * W < 2^31).
__device__ __forceinline__ int sp_start(int U, int w, int W) { return (int)((unsigned)(U * w) / (unsigned)W); }
// Warp whose (non-empty) range holds unit u.
__device__ __forceinline__ int sp_owner(int U, int u, int W) {
  int w = (int)((unsigned)(u * W) / (unsigned)U);
  while (w + 1 < W && sp_start(U, w + 1, W) <= u) ++w;
  while (w > 0 && sp_start(U, w, W) > u) --w;
  return w;
}
// Warps with a non-empty range in [w_lo, w_hi].
__device__ __forceinline__ int sp_nonempty(int U, int w_lo, int w_hi, int W) {
  int n = 0;
  for (int w = w_lo; w <= w_hi; ++w) n += sp_start(U, w + 1, W) > sp_start(U, w, W);
  return n;
}

// Sum of a group's pieces in warp order (warps w_lo..w_hi whose range is not
// empty; a warp's piece slot is 0 if the group is its first): loads are issued
// eight at a time before they are added, in order.
template <class Addr>
__device__ __forceinline__ float sp_sum_pieces(int U, int W, int w_lo, int w_hi, int grp_units, int grp, Addr addr) {
  float v = 0.f;
  for (int ww0 = w_lo; ww0 <= w_hi; ww0 += 8) {
    float x[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int ww = ww0 + k;
      x[k] = 0.f;
      if (ww <= w_hi) {
        const int s0 = sp_start(U, ww, W);
        if (sp_start(U, ww + 1, W) > s0) x[k] = __ldcg(addr(ww, s0 / grp_units == grp ? 0 : 1));
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) v += x[k];
  }
  return v;
}

// Hidden rows -> shared memory, lane-permuted (two 16-byte loads give a lane
// the B fragments of one 64-wide chunk).
__device__ void sp_load_rows(const __nv_bfloat16* src, long long ld, int rows, int K, unsigned char* dst,
                             int stride, int tid0, int nthr) {
  const int k8n = K / 8;
  for (int idx = threadIdx.x - tid0; idx < rows * k8n; idx += nthr) {
    const int m = idx / k8n, k8 = idx - m * k8n;
    const uint4 v = *reinterpret_cast<const uint4*>(src + (size_t)m * ld + k8 * 8);
    const int kk0 = k8 * 8, ch = kk0 >> 6, jq = (kk0 & 63) >> 4, hh = (kk0 >> 3) & 1;
    uint32_t* row = reinterpret_cast<uint32_t*>(dst + (size_t)m * stride);
    const int base = ch * 64 + jq * 4 + 2 * hh;
    row[(base + 0) >> 1] = v.x;
    row[(base + 16) >> 1] = v.y;
    row[(base + 32) >> 1] = v.z;
    row[(base + 48) >> 1] = v.w;
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// w13: unit u = (pair q = ae * P + pr, chunk c), u = q * chA + c.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void sp_w13(const SplitParams& p, const SpRoute& rt, const unsigned char* xs,
                                       long long* tr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int H = p.H, I = p.I, chA = H / 64, P = I / 16;
  const int xstride = H * 2 + 16;
  const int A = rt.A;
  const int U = A * P * chA;
  const int W = gridDim.x * kSpWarps, w = blockIdx.x * kSpWarps + warp;
  const int u0 = sp_start(U, w, W), u1 = sp_start(U, w + 1, W);
  if (u0 >= u1) return;
  const int nrt = 2 * P;
  const int Mp = p.Mp, piece_f = 2 * 16 * Mp;  // floats per piece
  const uint4* wg = reinterpret_cast<const uint4*>(p.w13);
  const uint2* sg = reinterpret_cast<const uint2*>(p.s13);
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  int slot = 0;
  auto finish = [&](int q) {
    float* pc = p.pieces13 + ((size_t)w * 2 + slot) * piece_f;
    if (2 * t < Mp) {
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        *reinterpret_cast<float2*>(pc + (tt * 16 + g) * Mp + 2 * t) = make_float2(acc[tt][0], acc[tt][1]);
        *reinterpret_cast<float2*>(pc + (tt * 16 + g + 8) * Mp + 2 * t) = make_float2(acc[tt][2], acc[tt][3]);
      }
    }
    __threadfence();
    __syncwarp();
    const int w_lo = sp_owner(U, q * chA, W), w_hi = sp_owner(U, q * chA + chA - 1, W);
    int last = 0;
    if (lane == 0) last = atomicAdd(p.cnt13 + q, 1) == sp_nonempty(U, w_lo, w_hi, W) - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence();
      const int ae = q / P, pr = q - ae * P, cnt = rt.cnt[ae], base = rt.base[ae];
      const int tile = lane >> 4, row = lane & 15;  // lane = tile * 16 + row
      for (int col = 0; col < cnt; ++col) {
        const float v = sp_sum_pieces(U, W, w_lo, w_hi, chA, q, [&](int ww, int sl) {
          return p.pieces13 + ((size_t)ww * 2 + sl) * piece_f + (tile * 16 + row) * Mp + col;
        });
        const float up = __shfl_sync(0xffffffffu, v, (lane & 15) + 16);
        if (lane < 16)
          p.inter[(size_t)(base + col) * I + sp_perm(pr * 16 + row)] = __float2bfloat16(silu_f(v) * up);
      }
      if (lane == 0) p.cnt13[q] = 0;  // self-cleaning
      __threadfence();
      __syncwarp();
      if (lane == 0) red_release_add(p.done13, 1);  // one more pair of intermediate columns complete
    }
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) acc[tt][0] = acc[tt][1] = acc[tt][2] = acc[tt][3] = 0.f;
    ++slot;
  };
  // groups (pairs) of this warp's range; inner loop over k-chunks with
  // pointer increments, two chunks in flight
  for (int u = u0; u < u1;) {
    const int q = u / chA, cb = u - q * chA, ce = min(chA, u1 - q * chA);
    const int ae = q / P, pr = q - ae * P, e = rt.act[ae];
    const size_t bg = ((size_t)e * nrt + pr) * chA, bu = ((size_t)e * nrt + P + pr) * chA;
    const uint4 *pg = wg + bg * 32 + lane, *pu = wg + bu * 32 + lane;
    const uint2 *qg = sg + bg * 8 + g, *qu = sg + bu * 8 + g;
    const int cnt = rt.cnt[ae], base = rt.base[ae];
    const unsigned char* brow = g < cnt ? xs + (size_t)rt.col_tok[base + g] * xstride + t * 32 : nullptr;
    uint4 wA0, wA1, wB0, wB1;
    uint2 sA0, sA1, sB0, sB1;
    wA0 = ldg_stream(pg + cb * 32);
    sA0 = ldg_stream2(qg + cb * 8);
    wA1 = ldg_stream(pu + cb * 32);
    sA1 = ldg_stream2(qu + cb * 8);
    if (cb + 1 < ce) {
      wB0 = ldg_stream(pg + (cb + 1) * 32);
      sB0 = ldg_stream2(qg + (cb + 1) * 8);
      wB1 = ldg_stream(pu + (cb + 1) * 32);
      sB1 = ldg_stream2(qu + (cb + 1) * 8);
    }
    for (int c = cb; c < ce; c += 2) {
      {
        uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
        if (brow) {
          q0 = lds128(brow + (size_t)c * 128);
          q1 = lds128(brow + (size_t)c * 128 + 16);
        }
        sp_block(acc[0], wA0, sA0, q0, q1);
        sp_block(acc[1], wA1, sA1, q0, q1);
        if (c + 2 < ce) {
          wA0 = ldg_stream(pg + (c + 2) * 32);
          sA0 = ldg_stream2(qg + (c + 2) * 8);
          wA1 = ldg_stream(pu + (c + 2) * 32);
          sA1 = ldg_stream2(qu + (c + 2) * 8);
        }
      }
      if (c + 1 < ce) {
        uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
        if (brow) {
          q0 = lds128(brow + (size_t)(c + 1) * 128);
          q1 = lds128(brow + (size_t)(c + 1) * 128 + 16);
        }
        sp_block(acc[0], wB0, sB0, q0, q1);
        sp_block(acc[1], wB1, sB1, q0, q1);
        if (c + 3 < ce) {
          wB0 = ldg_stream(pg + (c + 3) * 32);
          sB0 = ldg_stream2(qg + (c + 3) * 8);
          wB1 = ldg_stream(pu + (c + 3) * 32);
          sB1 = ldg_stream2(qu + (c + 3) * 8);
        }
      }
    }
    if (tr != nullptr && lane == 0 && warp == 0) tr[2 + (u == u0 ? 0 : 1)] = global_timer_ns();
    finish(q);
    if (tr != nullptr && lane == 0 && warp == 0) tr[4 + (u == u0 ? 0 : 1)] = global_timer_ns();
    u = q * chA + ce;
  }
}

// ---------------------------------------------------------------------------
// w2: unit u = (row tile r, active expert ae, chunk c), u = (r * A + ae) * chB + c.
// Columns of the MMA are tokens (0..M-1).
// ---------------------------------------------------------------------------
// Bounded wait of the whole CTA until `target` w13 pairs are complete; false
// (and a status bit) if the budget ran out.  Every thread of the CTA calls it.
__device__ __forceinline__ bool sp_wait_w13(const SplitParams& p, int target) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    const long long t0 = clock64();
    while (ld_acquire_gpu(p.done13) < target) {
      if (clock64() - t0 > kSpBudget) {
        atomicOr(p.sched + 2, kSpErrReady);
        ok = 0;
        break;
      }
      __nanosleep(256);
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

__device__ __forceinline__ void sp_w2(const SplitParams& p, const SpRoute& rt, long long* tr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int H = p.H, I = p.I, M = p.M, chB = I / 64, nrt = H / 16;
  const int A = rt.A;
  const int U = nrt * A * chB, per_tile = A * chB;
  const int W = gridDim.x * kSpWarps, w = blockIdx.x * kSpWarps + warp;
  const int u0 = sp_start(U, w, W), u1 = sp_start(U, w + 1, W);
  if (u0 >= u1) {
    sp_wait_w13(p, A * (I / 16));  // the CTA barrier needs every warp
    return;
  }
  const int Mp = p.Mp, piece_f = 16 * Mp;
  const uint4* wg = reinterpret_cast<const uint4*>(p.w2);
  const uint2* sg = reinterpret_cast<const uint2*>(p.s2);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};   // current (row tile, expert) over its chunks
  float out4[4] = {0.f, 0.f, 0.f, 0.f};  // current row tile, columns = tokens
  int slot = 0;
  auto fold_expert = [&](int fae) {  // out += router weight (per token column) * acc
    const int m0 = 2 * t, m1 = 2 * t + 1;
    const int c0 = m0 < M ? rt.tok_col[fae][m0] : -1, c1 = m1 < M ? rt.tok_col[fae][m1] : -1;
    const float w0 = c0 >= 0 ? rt.col_w[c0] : 0.f, w1 = c1 >= 0 ? rt.col_w[c1] : 0.f;
    out4[0] = fmaf(w0, acc[0], out4[0]);
    out4[1] = fmaf(w1, acc[1], out4[1]);
    out4[2] = fmaf(w0, acc[2], out4[2]);
    out4[3] = fmaf(w1, acc[3], out4[3]);
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
  };
  auto finish = [&](int fr) {
    float* pc = p.pieces2 + ((size_t)w * 2 + slot) * piece_f;
    if (2 * t < Mp) {
      *reinterpret_cast<float2*>(pc + g * Mp + 2 * t) = make_float2(out4[0], out4[1]);
      *reinterpret_cast<float2*>(pc + (g + 8) * Mp + 2 * t) = make_float2(out4[2], out4[3]);
    }
    __threadfence();
    __syncwarp();
    const int w_lo = sp_owner(U, fr * per_tile, W), w_hi = sp_owner(U, fr * per_tile + per_tile - 1, W);
    int last = 0;
    if (lane == 0) last = atomicAdd(p.cnt2 + fr, 1) == sp_nonempty(U, w_lo, w_hi, W) - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence();
      for (int idx = lane; idx < 16 * M; idx += 32) {
        const int row = idx / M, m = idx - row * M;
        const float v = sp_sum_pieces(U, W, w_lo, w_hi, per_tile, fr, [&](int ww, int sl) {
          return p.pieces2 + ((size_t)ww * 2 + sl) * piece_f + row * Mp + m;
        });
        p.out[(size_t)m * H + fr * 16 + row] = __float2bfloat16(v);
      }
      if (lane == 0) p.cnt2[fr] = 0;  // self-cleaning
      __threadfence();
      __syncwarp();
      // the last row tile of the call resets the phase counters
      if (lane == 0 && atomicAdd(p.done2, 1) == nrt - 1) {
        *p.done13 = 0;
        *p.done2 = 0;
      }
    }
    out4[0] = out4[1] = out4[2] = out4[3] = 0.f;
    ++slot;
  };
  // first weight block of the range before waiting for w13
  const int rq0 = u0 / chB, c00 = u0 - rq0 * chB, r0 = rq0 / A, ae0 = rq0 - r0 * A;
  uint4 wA = ldg_stream(wg + (((size_t)rt.act[ae0] * nrt + r0) * chB + c00) * 32 + lane);
  uint2 sA = ldg_stream2(sg + (((size_t)rt.act[ae0] * nrt + r0) * chB + c00) * 8 + g);
  // every w13 pair must be complete before the intermediate is read: one
  // thread per CTA polls (bounded), the CTA's warps meet at a barrier
  if (!sp_wait_w13(p, A * (I / 16))) return;
  if (tr != nullptr && threadIdx.x == 0) tr[2] = global_timer_ns();
  int cur_r = r0;
  bool first = true;
  for (int u = u0; u < u1;) {
    const int rq = u / chB, cb = u - rq * chB, ce = min(chB, u1 - rq * chB);
    const int r = rq / A, ae = rq - r * A;
    if (r != cur_r) {
      finish(cur_r);
      cur_r = r;
    }
    const size_t b0 = ((size_t)rt.act[ae] * nrt + r) * chB;
    const uint4* pw = wg + b0 * 32 + lane;
    const uint2* ps = sg + b0 * 8 + g;
    const int col = g < M ? rt.tok_col[ae][g] : -1;
    const uint4* br = col >= 0 ? reinterpret_cast<const uint4*>(p.inter + (size_t)col * I) + 2 * t : nullptr;
    uint4 wB;
    uint2 sB;
    if (!first) {
      wA = ldg_stream(pw + cb * 32);
      sA = ldg_stream2(ps + cb * 8);
    }
    first = false;
    if (cb + 1 < ce) {
      wB = ldg_stream(pw + (cb + 1) * 32);
      sB = ldg_stream2(ps + (cb + 1) * 8);
    }
    for (int c = cb; c < ce; c += 2) {
      {
        uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
        if (br) {
          q0 = __ldcg(br + c * 8);
          q1 = __ldcg(br + c * 8 + 1);
        }
        sp_block(acc, wA, sA, q0, q1);
        if (c + 2 < ce) {
          wA = ldg_stream(pw + (c + 2) * 32);
          sA = ldg_stream2(ps + (c + 2) * 8);
        }
      }
      if (c + 1 < ce) {
        uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
        if (br) {
          q0 = __ldcg(br + (c + 1) * 8);
          q1 = __ldcg(br + (c + 1) * 8 + 1);
        }
        sp_block(acc, wB, sB, q0, q1);
        if (c + 3 < ce) {
          wB = ldg_stream(pw + (c + 3) * 32);
          sB = ldg_stream2(ps + (c + 3) * 8);
        }
      }
    }
    fold_expert(ae);
    u = rq * chB + ce;
  }
  if (tr != nullptr && threadIdx.x == 0) tr[3] = global_timer_ns();
  finish(cur_r);
  if (tr != nullptr && threadIdx.x == 0) tr[4] = global_timer_ns();
}

// One cooperative launch: routing, the w13 phase, then the w2 phase (which
// starts once every pair's intermediate columns are published).
__global__ void __launch_bounds__(kSpThreads, 2) moe_split_kernel(SplitParams p) {
  __shared__ SpRoute rt;
  __shared__ SpRouteScratch sc;
  extern __shared__ __align__(16) unsigned char xs[];  // [M][H*2 + 16]
  long long* const tr = (p.trace != nullptr && blockIdx.x == 0) ? p.trace : nullptr;
  if (tr != nullptr && threadIdx.x == 0) tr[0] = global_timer_ns();
  sp_load_rows(p.hidden, p.hidden_ld, p.M, p.H, xs, p.H * 2 + 16, 0, kSpThreads);
  sp_route(p, rt, sc);
  if (tr != nullptr && threadIdx.x == 0) tr[1] = global_timer_ns();
  if (rt.A == 0) {  // nothing routed here: zero output
    for (int idx = blockIdx.x * kSpThreads + threadIdx.x; idx < p.M * p.H / 8; idx += gridDim.x * kSpThreads)
      reinterpret_cast<uint4*>(p.out)[idx] = make_uint4(0, 0, 0, 0);
    return;
  }
  sp_w13(p, rt, xs, tr);
  if (tr != nullptr && threadIdx.x == 0) tr[6] = global_timer_ns();
  if (p.trace != nullptr) {  // diagnostics: w13 end of every CTA (all of its warps)
    __syncthreads();
    if (threadIdx.x == 0) p.trace[16 + blockIdx.x] = global_timer_ns();
  }
  sp_w2(p, rt, tr != nullptr ? tr + 8 : nullptr);
}

int split_plan(SplitParams& p, int sms) {
  if (p.M < 1 || p.M > kSplitMaxM || p.n_tok < 1 || p.n_tok > kSplitMaxSlots) return 0;
  if (p.H % 64 || p.I % 64) return 0;
  p.grid = std::min(2 * sms, kSplitMaxGrid);
  p.Mp = p.M <= 2 ? 2 : 4;
  p.smem13 = p.M * (p.H * 2 + 16);
  if (p.smem13 > 48 * 1024) return 0;
  // a warp's range must span at most two accumulation groups
  const long long amax = std::min(p.n_tok, p.E);
  const long long W = (long long)p.grid * kSpWarps;
  const long long U13 = amax * (p.I / 16) * (p.H / 64), U2 = amax * (p.H / 16) * (p.I / 64);
  if ((U13 + W - 1) / W > p.H / 64) return 0;
  if (U13 * W >= (1LL << 31) || U2 * W >= (1LL << 31)) return 0;  // 32-bit range arithmetic
  return 1;
}

cudaError_t launch_split(const SplitParams& p, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kSpThreads);
  cfg.dynamicSmemBytes = p.smem13;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // phases wait on other CTAs: all must be resident
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, moe_split_kernel, p);
}

}  // namespace w4moe
