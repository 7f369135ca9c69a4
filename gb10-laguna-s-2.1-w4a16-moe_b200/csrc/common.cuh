// Shared definitions for the B200 W4A16 grouped-MoE library.
//
// Repacked weight layout ("fragment-major"), produced by repack.cu and read by
// every GEMM kernel in this library:
//
//   w_rep  (E, N_out/16, K/64, 512)  uint8
//   s_rep  (E, N_out/16, K/64, 32)   bf16
//
// One (expert, row-tile of 16 output rows, k-chunk of 64) block of weights is
// 512 contiguous bytes = 32 lanes x 16 bytes.  Lane l (g = l>>2, t = l&3) owns
// four 32-bit words, one per 16-wide k step j (k0 = chunk*64 + j*16).  Word j
// holds eight 4-bit codes (stored value q+8 in [0,15]) at nibble positions:
//
//   n0 = W[g  ][k0+2t  ]   n4 = W[g  ][k0+2t+1]
//   n1 = W[g+8][k0+2t  ]   n5 = W[g+8][k0+2t+1]
//   n2 = W[g  ][k0+2t+8]   n6 = W[g  ][k0+2t+9]
//   n3 = W[g+8][k0+2t+8]   n7 = W[g+8][k0+2t+9]
//
// so that (w >> 4i) & 0x000F000F yields, for i = 0..3, exactly the bf16 pairs
// a warp-level m16n8k16 A fragment wants (a0a1, a2a3, a4a5, a6a7).  The same
// block is decoded by the tensor-core prefill kernel into its smem tiles.
//
// Scales: per (expert, row-tile, chunk) 32 bf16; quad g holds
//   [4g+0] = s(g, grp0)  [4g+1] = s(g+8, grp0)  [4g+2] = s(g, grp1)  [4g+3] = s(g+8, grp1)
// where grp0/grp1 are the two 32-wide groups of the chunk.  Group sizes that
// are multiples of 32 are stored by replicating each scale (exact).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace w4moe {

constexpr int kRowTile = 16;
constexpr int kChunkK = 64;
constexpr int kChunkBytes = 512;   // packed weight bytes per (rowtile, chunk)
constexpr int kChunkScales = 32;   // bf16 scales per (rowtile, chunk)
constexpr int kGroup = 32;         // storage group size

// Status codes returned by every C-ABI entry point.
enum Status : int {
  kOk = 0,
  kInvalidArgument = 1,
  kUnsupported = 2,
  kCudaError = 3,
};

// (a & b) | c in one LOP3.
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Decode one fragment word into four bf16x2 registers holding (q-8)*s,
// rounded once to bf16 (the same value a dequantise-then-bf16 reference
// produces).  The nibble is OR-ed into the mantissa of 128.0 (0x4300), which
// makes the bf16 value 128+code exactly; subtracting 136 leaves code-8.
// sg / sg8: the bf16 scale for rows g and g+8, broadcast to both halves.
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t sg, uint32_t sg8,
                                             uint32_t (&a)[4]) {
  const uint32_t kMask = 0x000F000Fu;
  const uint32_t kMagic = 0x43004300u;   // bf16 {128, 128}
  const uint32_t kBias = 0x43084308u;    // bf16 {136, 136}
  a[0] = bf16x2_mul(bf16x2_sub(and_or(w, kMask, kMagic), kBias), sg);
  a[1] = bf16x2_mul(bf16x2_sub(and_or(w >> 4, kMask, kMagic), kBias), sg8);
  a[2] = bf16x2_mul(bf16x2_sub(and_or(w >> 8, kMask, kMagic), kBias), sg);
  a[3] = bf16x2_mul(bf16x2_sub(and_or(w >> 12, kMask, kMagic), kBias), sg8);
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint2 ldg_stream2(const uint2* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

// ---- shared-memory pipeline primitives (mbarrier + bulk async copy) ----

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the warp sleeps in hardware until the
// phase completes or ~hint_ns elapse, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: false after ~`budget` SM clocks (the caller records an error).
// Spins with plain try_wait for ~20 us of SM clocks (phase completion is
// seen immediately), then sleeps with a suspend hint between checks.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long budget) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    const long long dt = clock64() - t0;
    if (dt > budget) return false;
    if (dt > 40000 && mbar_try_wait_sleep(bar, parity, 20000u)) return true;
  }
  return true;
}

// Same MMA without `volatile`: a pure function of its register operands, so
// the compiler may interleave independent accumulation chains.
__device__ __forceinline__ void mma_bf16_16816_nv(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                  uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (code - 8) in bf16 for the four A-fragment registers of one word (exact).
__device__ __forceinline__ void unscaled_word(uint32_t w, uint32_t (&a)[4]) {
  const uint32_t kMask = 0x000F000Fu, kMagic = 0x43004300u, kBias = 0x43084308u;
  a[0] = bf16x2_sub(and_or(w, kMask, kMagic), kBias);
  a[1] = bf16x2_sub(and_or(w >> 4, kMask, kMagic), kBias);
  a[2] = bf16x2_sub(and_or(w >> 8, kMask, kMagic), kBias);
  a[3] = bf16x2_sub(and_or(w >> 12, kMask, kMagic), kBias);
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 (5th-gen tensor core, accumulators in TMEM) ----

// Byte offset of bf16 element (r, k) inside a [rows x 64] K-major operand
// block in the canonical 128-byte-swizzled layout (8-row x 128 B atoms, the
// 16-byte chunk index XOR-ed with the row within the atom).
__device__ __forceinline__ uint32_t swz128(int r, int k) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((k * 2) >> 4) ^ (r & 7)) << 4) + ((k * 2) & 15));
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (the atom base must be 1024-byte aligned).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset
  d |= (uint64_t)1 << 46;            // descriptor version
  d |= (uint64_t)2 << 61;            // 128-byte swizzle
  return d;
}

// Instruction descriptor of kind::f16: bf16 A/B, fp32 D, both K-major.
__device__ __forceinline__ uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrive (once) on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.  The load and its
// wait are one asm statement: the destination registers are valid only after
// tcgen05.wait::ld, and with two statements the compiler may read or copy
// them in between.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ long long global_timer_ns() {
  long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Global -> shared bulk copy (16-byte aligned, size % 16 == 0) completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// tma_load_2d with the destination given as a shared-memory address.
__device__ __forceinline__ void tma_load_2d_u32(uint32_t dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_u32(uint32_t dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled tensor load (TMA) of box {x .. x+box0, y .. y+box1} into shared
// memory, completing on `bar`.  x * element size must be a multiple of 16 B;
// rows past the tensor's extent are zero-filled (and still counted in bytes).
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ uint2 lds64(const void* p) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }

// Maps a flat slot (m*topk + t) to the local expert it is routed to, or -1.
// ids are int32 or int64; expert_map (nullable) is the vLLM expert-parallel
// table from global expert id to local id (-1 = not on this rank).
struct SlotMap {
  const void* ids;
  int ids_is_64;
  const int32_t* expert_map;
  int global_E;
  int E;  // local experts

  __device__ __forceinline__ int operator()(int slot) const {
    long long v = ids_is_64 ? (long long)((const int64_t*)ids)[slot]
                            : (long long)((const int32_t*)ids)[slot];
    if (expert_map != nullptr) {
      if (v < 0 || v >= global_E) return -1;
      v = expert_map[v];
    }
    return (v >= 0 && v < E) ? (int)v : -1;
  }
};

// Per-expert slot lists in ascending slot order, identical in every CTA that
// builds them (an atomic scatter would order slots differently per CTA, and
// CTAs that split one expert's slots into passes must agree on the split).
// One warp; eid[i] = local expert of slot i or -1; cur[e] = first position of
// expert e (advanced past its slots on return).
__device__ __forceinline__ void ordered_slot_scatter(const int* eid, int n_tok, int* cur, int* slots, int lane) {
  const unsigned lt = (1u << lane) - 1u;
  for (int i0 = 0; i0 < n_tok; i0 += 32) {
    const int i = i0 + lane;
    const int e = i < n_tok ? eid[i] : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int leader = __ffs(peers) - 1;
    int base = (e >= 0 && lane == leader) ? cur[e] : 0;
    base = __shfl_sync(0xffffffffu, base, leader);
    if (e >= 0) slots[base + __popc(peers & lt)] = i;
    __syncwarp();
    if (e >= 0 && lane == leader) cur[e] = base + __popc(peers);
    __syncwarp();
  }
}

// Routing arrays derived once per forward by the align kernel and consumed by
// the GEMM kernels.  All live in the caller-provided workspace.
struct RouteView {
  const int32_t* sorted;      // [P] slot ids grouped by expert, padded per expert
  const int32_t* offsets;     // [E+1] padded start of each expert in `sorted`
  const int32_t* counts;      // [E] valid slots per expert
  const int32_t* active;      // [E] compact list of experts with count > 0
  const int32_t* num_active;  // [1]
  const int32_t* tok_valid;   // [M] locally routed slots per token
};

}  // namespace w4moe
