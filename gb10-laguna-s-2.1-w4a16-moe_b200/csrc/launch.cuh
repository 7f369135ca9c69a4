// Parameter blocks and host launchers of every kernel in this library.
#pragma once

#include "common.cuh"

namespace w4moe {

// ---- align.cu ----
struct AlignParams {
  SlotMap map;              // ids (+ optional expert_map) -> local expert
  int n_tok;
  int topk;
  int E;                    // (local) experts
  int bs;
  int P;
  int32_t* sorted;          // [P]
  int32_t* expert_ids;      // [P/bs]
  int32_t* num_post;        // [1]
  // optional outputs (nullable)
  int32_t* counts;          // [E]
  int32_t* offsets;         // [E+1]
  int32_t* active;          // [E]
  int32_t* num_active;      // [1]
  int32_t* tok_valid;       // [n_tok/topk]
  __nv_bfloat16* zero_rows; // [M, H] rows zeroed where tok_valid == 0
  int H;
  // multi-CTA variant only
  int32_t* scratch;         // [C * E] chunk totals
  int32_t* grid_bar;        // [3] zero-initialised: arrivals, generation, error word
  int32_t* status;          // nullable: a barrier timeout is also OR-ed in here
  long long budget;         // grid-barrier wait limit in SM clocks
  int withhold;             // test hook: CTA 0 does not arrive at the barrier
};
constexpr long long kAlignBarrierBudget = 2000000000LL;  // SM clocks (~1 s)
constexpr int kAlignErrBarrier = 1 << 16;  // status bit: align grid barrier timed out
cudaError_t launch_align(const AlignParams& p, cudaStream_t stream);
int align_grid_ctas(int n_tok, int E, int sms);
size_t align_grid_scratch_ints(int E, int sms);
cudaError_t launch_align_grid(const AlignParams& p, int ctas, cudaStream_t stream);

// ---- repack.cu ----
struct RepackParams {
  const uint8_t* w_q;       // (E, N_out, K/2)
  const uint16_t* scales;   // (E, N_out, K/G) bf16 bits
  int E, N_out, K, G;
  uint32_t* w_rep;          // (E, N_out/16, K/64, 128) words
  uint16_t* s_rep;          // (E, N_out/16, K/64, 32)
  const int32_t* w_i32t;    // checkpoint form (E, K/8, N_out) int32 instead of w_q (nullable)
  int scales_t;             // scales given as (E, K/G, N_out)
};
cudaError_t launch_repack(const RepackParams& p, cudaStream_t stream);

// ---- gemv.cu ----
struct GemvParams {
  const uint4* w;            // fragment-major weights of this projection
  const uint2* s;            // scale quads
  int n_rowtiles;            // N_out / 16
  int n_chunks;              // K / 64
  const __nv_bfloat16* x;    // B operand rows
  long long x_ld;            // row stride in elements
  int x_row_div;             // row of slot = slot / x_row_div
  RouteView rt;
  int topk;
  int items_per_expert;
  // MODE 0 epilogue
  __nv_bfloat16* inter;
  int I;
  // MODE 1 epilogue
  float* partial;
  int H;
  const float* topk_w;       // [n_tok]
  int32_t* counters;         // [M * items_per_expert], zero between calls
  __nv_bfloat16* out;        // [M, H]
  SlotMap map;
};
cudaError_t launch_gemv(const GemvParams& p, int mode, int ng, int grid, cudaStream_t stream);
int gemv_blocks_per_sm(int mode, int ng);

// ---- decode.cu (fused persistent small-M layer) ----
constexpr int kDecodeMaxSlots = 4096;  // M*topk handled by the fused kernel
constexpr int kDecGeoRows = 33;        // stage geometry table rows (reserved activation rows 1..32)

struct DecodeParams {
  const uint8_t* w13;        // fragment-major w13 (gate rows [0,I), up rows [I,2I))
  const uint8_t* s13;
  const uint8_t* w2;         // fragment-major w2
  const uint8_t* s2;
  const __nv_bfloat16* hidden;
  long long hidden_ld;
  SlotMap map;
  int n_tok, topk, M, E, H, I;
  const float* topk_w;       // [n_tok]
  __nv_bfloat16* inter;      // [n_tok, I] bf16(silu(gate)*up)
  float* partial;            // [n_tok, H] router-weighted fp32 partials
  __nv_bfloat16* out;        // [M, H]
  int32_t* counters;         // [M, H/16/R2] per-token arrival counters (zero between calls)
  int32_t* ready;            // [E] published phase-A item passes per expert (zero between calls)
  int32_t* sched;            // [4] next item, finished CTAs, error bits
  int zero_rows;             // write zero rows for tokens with no local slot
  int tail_reduce;           // 1: grid-wide top-k sum after all w2 items; 0: per-token last arriver
  long long ready_budget;    // SM clocks a w2 item waits for its expert's intermediate (set by decode_plan)
  int withhold;              // test hook: CTA 0 publishes no w13 readiness (the waits then run out)
  long long* trace;          // optional event timestamps of CTA 0 (diagnostics; nullptr normally)
  // plan (decode_plan); the stage geometry is derived per CTA on the device
  int NG, RP, R2, n_red, red_offset, ring_offset, ring_bytes, smem_bytes, grid;
  int ring_div;              // stages are sized to ring_bytes / ring_div
  int geo[kDecGeoRows][4];   // per reserved row count: ncA, ncB, stage bytes, stages
};
int decode_plan(DecodeParams& p, int sms, int max_smem);

// ---- prefill.cu (tcgen05 grouped GEMMs for large M) ----
struct PrefillParams {
  const uint8_t* w;          // fragment-major weights of this projection
  const uint8_t* s;          // scales
  int n_rowtiles, n_chunks;  // N_out / 16, K / 64
  const __nv_bfloat16* x;    // w13: hidden states (gathered into xs in sorted order)
  long long x_ld;
  int x_row_div;             // row of slot = slot / x_row_div
  __nv_bfloat16* xs;         // w13: [n_tok, H] token rows in expert-sorted order
  int n_tok;                 // M * topk (rows of xs / inter)
  const int32_t* num_post;   // valid sorted positions
  const int32_t* sorted;     // exact expert-sorted slot list (align, block size 1)
  const int32_t* offsets;
  const int32_t* counts;
  const int32_t* active;
  const int32_t* num_active;
  int E, topk, I, H;
  __nv_bfloat16* inter;      // w13 output [n_tok, I], rows in expert-sorted order
  __nv_bfloat16* partial;    // w2 output [n_tok, H] (router-weighted)
  const float* topk_w;
  int32_t* sched;            // error bits in sched[2]
  int n_stages;              // pipeline depth (prefill_stages)
  long long* trace;          // optional event timestamps of CTA 0 (diagnostics; nullptr normally)
};
int prefill_stages(int E, int max_smem_optin);
cudaError_t launch_prefill_w13(const PrefillParams& p13, int sms, cudaStream_t stream);
cudaError_t launch_prefill_w2(const PrefillParams& p2, const SlotMap& map, int M, int topk, int H,
                              __nv_bfloat16* out, int sms, cudaStream_t stream);

// ---- capi.cu internals shared with other entry points ----
int64_t workspace_zero_prefix_bytes(int64_t M, int64_t topk, int64_t E, int64_t H, int64_t I);
int report_error(int code, const char* msg);
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream);

}  // namespace w4moe
